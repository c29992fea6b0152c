// tcgen05 / TMEM tensor-core GEMM for the prefill path (sm_100a).
//
//   C[z][m, n] = sum_k A[z][m, k] * B[z][n, k]        (bf16 in, fp32 accumulate)
//
// Both operands are K-major ("TN"): the rows of A are tokens (or queries), the rows of
// B are weight rows (or keys / value columns), exactly how every contraction of the
// prefill forward is laid out in memory (model.py:195-250 einsums over hidden / head
// dims).  One CTA computes one BM x BN tile:
//
//   warp 0 lane 0   producer: TMA tiled loads (cp.async.bulk.tensor, 128-byte swizzle,
//                   one destination CTA) of A [BM x 64] and B [BN x 64] per k-block into a
//                   STAGES-deep shared-memory ring, full/empty mbarriers;
//   warp 1          allocates BN TMEM columns; lane 0 issues tcgen05.mma (M=128,
//                   N=BN, K=16, kind::f16, bf16 -> fp32) four per k-block from shared
//                   memory descriptors, tcgen05.commit frees each stage and finally
//                   signals the accumulator;
//   warps 2-5       epilogue: tcgen05.ld of their 32-lane TMEM quadrant (one row per
//                   thread), optional bf16 rounding, masked stores to C.
//
// Batched launches (grid.z) give each z its own row/column offsets into A, B and C
// (attention heads, the two MLP projections, expert groups).  Optional B as a 3-D
// tensor (k-inner, n, slab): K runs over slabs, e.g. the dense-MoE down projection
// sum over (expert, f) of act[t, e, f] * down[e, h, f] (model.py:250) as ONE GEMM.
// Optional causal / sliding band: score tiles with no valid (query, key) pair are not
// computed, and the probability x value product runs only over the key blocks some
// query of the tile can see.
//
// Every mbarrier wait is bounded by %globaltimer; a timeout sets a bit in *status and
// the CTA drains and releases its TMEM before returning.
#pragma once

#include <cuda.h>

#include "g4_common.cuh"

namespace g4 {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle row of bf16
constexpr int kGemmThreads = 192;
constexpr int kGemmAStage = kGemmBM * kGemmBK * 2;  // 16 KB

struct GemmArgs {
  int M, N, K;           // per batch entry; K in elements (multiple of 64 for 2-D B)
  void* C;
  long long ldc;         // elements
  int c_f32;             // 1: fp32 output, 0: bf16 (round to nearest even)
  // batch entry z: coordinate offsets (elements / rows) of its A, B and C
  int za_row, za_col;    // A: row += z * za_row, col += z * za_col
  int zb_div;            // B entry = z / zb_div (query heads sharing one KV head)
  int zb_row, zb_col;    // B: row += (z / zb_div) * zb_row, col += (z / zb_div) * zb_col
  long long zc_row, zc_col;
  int b_kpe;             // > 0: B is 3-D (k, n, slab), k-blocks per slab (ceil(slab K / 64))
  int a_slab;            // with b_kpe: A columns per slab (the slab's K; a multiple of 8)
  int band;              // 0 none; 1 scores (rows = queries, cols = keys); 2 P.V (K = keys)
  int q_pos0, key_pos0;  // absolute positions of row 0 / of column or K index 0
  int window;            // sliding window (0: causal only)
  int a_row0, a_col0;    // constant coordinate offsets of A and B (e.g. the first key row)
  int b_row0, b_col0;
  int ksplit;            // > 1: split-K; grid.z = Z * ksplit, split s writes its fp32 partial
  long long split_stride;  //   sum to C + s * split_stride (elements; C is fp32 then)
  const int* z_rows;     // grouped GEMM: entry z owns A / C rows [z_rows[z], z_rows[z+1]) and
                         //   its M is their count (za_row / zc_row then unused); else null
  int nz;                // batch entries (the persistent kernel walks n_tiles x m_tiles x nz x ksplit)
  int* status;           // error bits (bounded waits)
};

struct GemmParams {
  CUtensorMap ta;  // 64-byte aligned (first member)
  CUtensorMap tb;
  GemmArgs a;
};

__host__ __device__ __forceinline__ int gemm_stages(int bn) { return bn >= 256 ? 4 : 6; }
__host__ __device__ __forceinline__ int gemm_smem_bytes(int bn) {
  return gemm_stages(bn) * (kGemmAStage + bn * kGemmBK * 2) + 1024 /*align*/ + 256 /*barriers*/;
}

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major tile with 128-byte rows, 128-byte
// swizzle (the layout the TMA load wrote): 8-row groups 1024 bytes apart (SBO), the
// leading offset unused for swizzled K-major layouts (1), version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                // LBO (16 bytes)
  d |= (uint64_t)(1024 >> 4) << 32;      // SBO
  d |= (uint64_t)1 << 46;                // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                // SWIZZLE_128B
  return d;
}

// Instruction descriptor of kind::f16: bf16 A and B (K-major), fp32 accumulator, M x N.
__host__ __device__ __forceinline__ uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4)                 // D format F32
         | (1u << 7)               // A format BF16
         | (1u << 10)              // B format BF16
         | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Bounded wait; gives up (status bit) after kLocalTimeoutNs or once *abort is set.
__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity, int* status, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort) return false;
    if (globaltimer_ns() - t0 > kLocalTimeoutNs) {
      if (status) atomicOr(status, G4_STATUS_MBAR_TIMEOUT);
      *abort = 1;
      return false;
    }
  }
  return true;
}

// The k-block range [kb0, kb1) of tile (m0, n0), and whether the tile is computed at all.
__device__ __forceinline__ bool gemm_tile_range(const GemmArgs& a, int M, int m0, int n0, int bn, int& kb0,
                                                int& kb1) {
  const int nkb = (a.K + kGemmBK - 1) / kGemmBK;
  kb0 = 0;
  kb1 = nkb;
  if (a.band == 1) {  // scores: row q sees keys (q - window, q]
    const int qlo = a.q_pos0 + m0, qhi = a.q_pos0 + min(m0 + kGemmBM, M) - 1;
    const int klo = a.key_pos0 + n0, khi = a.key_pos0 + min(n0 + bn, a.N) - 1;
    if (klo > qhi) return false;
    if (a.window > 0 && khi <= qlo - a.window) return false;
  } else if (a.band == 2) {  // P.V: K index j is the key at key_pos0 + j
    const int qlo = a.q_pos0 + m0, qhi = a.q_pos0 + min(m0 + kGemmBM, M) - 1;
    int jlo = (a.window > 0 ? qlo - a.window + 1 : 0) - a.key_pos0;
    int jhi = qhi - a.key_pos0 + 1;
    jlo = max(jlo, 0);
    jhi = min(jhi, a.K);
    kb0 = jlo / kGemmBK;
    kb1 = (jhi + kGemmBK - 1) / kGemmBK;
  }
  return true;
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_kernel(const __grid_constant__ GemmParams P) {
  constexpr int STAGES = BN >= 256 ? 4 : 6;
  constexpr int BSTAGE = BN * kGemmBK * 2;
  constexpr uint32_t STAGE_TX = kGemmAStage + BSTAGE;
  extern __shared__ unsigned char gemm_smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sa = smem;                              // [STAGES][BM x 64] bf16, swizzled
  unsigned char* sb = smem + STAGES * kGemmAStage;       // [STAGES][BN x 64]
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + STAGES * BSTAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* accum = empty + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* issued = abort + 1;    // k-blocks the producer loaded
  volatile int* consumed = abort + 2;  // k-blocks the MMA lane waited for

  const GemmArgs& a = P.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kGemmBM, n0 = blockIdx.x * BN;
  const int ks = a.ksplit > 1 ? a.ksplit : 1;
  const int z = blockIdx.z / ks, split = blockIdx.z % ks;
  int M = a.M, arow_base = a.a_row0 + z * a.za_row;
  long long crow_base = (long long)z * a.zc_row;
  if (a.z_rows) {  // grouped: this entry's rows
    const int r0 = __ldg(a.z_rows + z), r1 = __ldg(a.z_rows + z + 1);
    M = r1 - r0;
    arow_base = a.a_row0 + r0;
    crow_base = r0;
  }
  if (m0 >= M) return;  // uniform over the CTA
  int kb0, kb1;
  if (!gemm_tile_range(a, M, m0, n0, BN, kb0, kb1)) return;
  if (ks > 1) {  // this split's share of the k-blocks (an empty share writes zeros)
    const int per = (kb1 - kb0 + ks - 1) / ks;
    const int s0 = kb0 + split * per;
    kb1 = min(kb1, s0 + per);
    kb0 = min(s0, kb1);
  }
  const bool has_k = kb1 > kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort = 0;
    *issued = 0;
    *consumed = 0;
    mbar_init_fence();
    tma_prefetch_desc(&P.ta);
    tma_prefetch_desc(&P.tb);
  }
  if (warp == 1) {  // TMEM: BN fp32 columns x 128 lanes
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && has_k) {
      const int arow = arow_base + m0, acol0 = a.a_col0 + z * a.za_col;
      const int zb = z / a.zb_div;
      const int brow = a.b_row0 + zb * a.zb_row + n0, bcol0 = a.b_col0 + zb * a.zb_col;
      for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !gemm_wait(&empty[s], ((i / STAGES) - 1) & 1, a.status, abort)) break;
        mbar_arrive_expect_tx(&full[s], STAGE_TX);
        if (a.b_kpe > 0) {  // K = (slab, k within the slab): A columns slab * a_slab + k
          const int slab = kb / a.b_kpe, kin = (kb % a.b_kpe) * kGemmBK;
          tma_load_2d(sa + s * kGemmAStage, &P.ta, acol0 + slab * a.a_slab + kin, arow, &full[s]);
          tma_load_3d(sb + s * BSTAGE, &P.tb, kin, brow, slab, &full[s]);
        } else {
          tma_load_2d(sa + s * kGemmAStage, &P.ta, acol0 + kb * kGemmBK, arow, &full[s]);
          tma_load_2d(sb + s * BSTAGE, &P.tb, bcol0 + kb * kGemmBK, brow, &full[s]);
        }
        *issued = i + 1;
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && has_k) {
      const uint32_t idesc = umma_idesc_bf16(kGemmBM, BN);
      bool ok = true;
      for (int kb = kb0, i = 0; kb < kb1; ++kb, ++i) {
        const int s = i % STAGES;
        if (!gemm_wait(&full[s], (i / STAGES) & 1, a.status, abort)) {
          ok = false;
          break;
        }
        *consumed = i + 1;
        tc_fence_after();
        const uint32_t a_addr = smem_addr(sa + s * kGemmAStage), b_addr = smem_addr(sb + s * BSTAGE);
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk)  // K=16 per instruction: 32 bytes along the row
          umma_bf16(tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), idesc,
                    (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
      (void)ok;
      umma_commit(accum);  // completes when every issued MMA has (also after a failure)
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row = m0 + q * 32 + lane;
    int ready = 1;  // warp-uniform: lane 0 waits, the warp follows its verdict
    if (has_k && lane == 0) ready = gemm_wait(accum, 0, a.status, abort) ? 1 : 0;
    ready = __shfl_sync(0xffffffffu, ready, 0);
    tc_fence_after();
    const bool row_ok = row < M;
    const long long crow = crow_base + row;
    const long long ccol0 = (long long)z * a.zc_col + n0;
    const bool out_f32 = a.c_f32 || ks > 1;
    void* cbase = ks > 1 ? static_cast<void*>(static_cast<float*>(a.C) + split * a.split_stride) : a.C;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
      uint32_t r[32];
      if (has_k && ready) {
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) r[i] = 0u;  // an empty K range contributes zero
      }
      if (!row_ok || n0 + c0 >= a.N || !ready) continue;
      const int ncols = min(32, a.N - (n0 + c0));
      if (out_f32) {
        float* dst = reinterpret_cast<float*>(cbase) + crow * a.ldc + ccol0 + c0;
        if (ncols == 32 && (((uintptr_t)dst) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<uint4*>(dst + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
        } else {
          for (int i = 0; i < ncols; ++i) dst[i] = __uint_as_float(r[i]);
        }
      } else {
        bf16_t* dst = reinterpret_cast<bf16_t*>(cbase) + crow * a.ldc + ccol0 + c0;
        if (ncols == 32 && (((uintptr_t)dst) & 15) == 0) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 u;
            u.x = (uint32_t)f2bf(__uint_as_float(r[i])) | ((uint32_t)f2bf(__uint_as_float(r[i + 1])) << 16);
            u.y = (uint32_t)f2bf(__uint_as_float(r[i + 2])) | ((uint32_t)f2bf(__uint_as_float(r[i + 3])) << 16);
            u.z = (uint32_t)f2bf(__uint_as_float(r[i + 4])) | ((uint32_t)f2bf(__uint_as_float(r[i + 5])) << 16);
            u.w = (uint32_t)f2bf(__uint_as_float(r[i + 6])) | ((uint32_t)f2bf(__uint_as_float(r[i + 7])) << 16);
            *reinterpret_cast<uint4*>(dst + i) = u;
          }
        } else {
          for (int i = 0; i < ncols; ++i) dst[i] = f2bf(__uint_as_float(r[i]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) {
    // a wait gave up: let every TMA load still in flight land before the CTA exits
    for (int i = *consumed; i < *issued; ++i) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && globaltimer_ns() - t0 < kLocalTimeoutNs) {
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
  }
}

// ------------------------------------------------------------------ persistent variant
// Tile t of the launch (n fastest, then m, then batch entry z and split s) and whether it
// is computed; every role walks the same sequence and skips the same tiles.
struct GemmTile {
  int n0, m0, z, split, M, kb0, kb1;
  int arow_base;
  long long crow_base;
};

template <int BN>
__device__ __forceinline__ bool gemm_tile(const GemmArgs& a, int t, int n_tn, int n_tm, int ks, GemmTile& T) {
  T.n0 = (t % n_tn) * BN;
  const int r = t / n_tn;
  T.m0 = (r % n_tm) * kGemmBM;
  const int zs = r / n_tm;
  T.z = zs / ks;
  T.split = zs % ks;
  T.M = a.M;
  T.arow_base = a.a_row0 + T.z * a.za_row;
  T.crow_base = (long long)T.z * a.zc_row;
  if (a.z_rows) {
    const int r0 = __ldg(a.z_rows + T.z), r1 = __ldg(a.z_rows + T.z + 1);
    T.M = r1 - r0;
    T.arow_base = a.a_row0 + r0;
    T.crow_base = r0;
  }
  if (T.m0 >= T.M) return false;
  if (!gemm_tile_range(a, T.M, T.m0, T.n0, BN, T.kb0, T.kb1)) return false;
  if (ks > 1) {
    const int per = (T.kb1 - T.kb0 + ks - 1) / ks;
    const int s0 = T.kb0 + T.split * per;
    T.kb1 = min(T.kb1, s0 + per);
    T.kb0 = min(s0, T.kb1);
  }
  return true;
}

// One persistent CTA per SM walks tiles blockIdx.x, blockIdx.x + gridDim.x, ...  The TMA
// ring runs across tile boundaries, and TMEM holds TWO accumulators (2 x BN columns): the
// MMA lane fills one while the epilogue warps drain the other, so the epilogue of a tile
// overlaps the main loop of the next (acc_full / acc_empty mbarriers per buffer).
template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_persistent_kernel(const __grid_constant__ GemmParams P) {
  constexpr int STAGES = BN >= 256 ? 4 : 6;
  constexpr int BSTAGE = BN * kGemmBK * 2;
  constexpr uint32_t STAGE_TX = kGemmAStage + BSTAGE;
  extern __shared__ unsigned char gemm_smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sa = smem;
  unsigned char* sb = smem + STAGES * kGemmAStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + STAGES * BSTAGE);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* issued = abort + 1;
  volatile int* consumed = abort + 2;

  const GemmArgs& a = P.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ks = a.ksplit > 1 ? a.ksplit : 1;
  const int n_tn = (a.N + BN - 1) / BN, n_tm = (a.M + kGemmBM - 1) / kGemmBM;
  const int ntiles = n_tn * n_tm * (a.nz > 0 ? a.nz : 1) * ks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    *abort = 0;
    *issued = 0;
    *consumed = 0;
    mbar_init_fence();
    tma_prefetch_desc(&P.ta);
    tma_prefetch_desc(&P.tb);
  }
  if (warp == 1) {  // TMEM: two BN-column fp32 accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                 "r"(2 * BN)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int i = 0;  // k-blocks issued by this CTA (ring position)
      for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
        GemmTile T;
        if (!gemm_tile<BN>(a, t, n_tn, n_tm, ks, T)) continue;
        const int acol0 = a.a_col0 + T.z * a.za_col;
        const int zb = T.z / a.zb_div;
        const int brow = a.b_row0 + zb * a.zb_row + T.n0, bcol0 = a.b_col0 + zb * a.zb_col;
        const int arow = T.arow_base + T.m0;
        for (int kb = T.kb0; kb < T.kb1; ++kb, ++i) {
          const int s = i % STAGES;
          if (i >= STAGES && !gemm_wait(&empty[s], ((i / STAGES) - 1) & 1, a.status, abort)) break;
          mbar_arrive_expect_tx(&full[s], STAGE_TX);
          if (a.b_kpe > 0) {
            const int slab = kb / a.b_kpe, kin = (kb % a.b_kpe) * kGemmBK;
            tma_load_2d(sa + s * kGemmAStage, &P.ta, acol0 + slab * a.a_slab + kin, arow, &full[s]);
            tma_load_3d(sb + s * BSTAGE, &P.tb, kin, brow, slab, &full[s]);
          } else {
            tma_load_2d(sa + s * kGemmAStage, &P.ta, acol0 + kb * kGemmBK, arow, &full[s]);
            tma_load_2d(sb + s * BSTAGE, &P.tb, bcol0 + kb * kGemmBK, brow, &full[s]);
          }
          *issued = i + 1;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16(kGemmBM, BN);
      int i = 0, it = 0;  // k-blocks consumed, tiles accumulated
      for (int t = blockIdx.x; t < ntiles && !*abort; t += gridDim.x) {
        GemmTile T;
        if (!gemm_tile<BN>(a, t, n_tn, n_tm, ks, T)) continue;
        const int b = it & 1, use = it >> 1;
        ++it;
        if (use > 0 && !gemm_wait(&acc_empty[b], (use - 1) & 1, a.status, abort)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(b * BN);
        bool ok = true;
        for (int kb = T.kb0; kb < T.kb1; ++kb, ++i) {
          const int s = i % STAGES;
          if (!gemm_wait(&full[s], (i / STAGES) & 1, a.status, abort)) {
            ok = false;
            break;
          }
          *consumed = i + 1;
          tc_fence_after();
          const uint32_t a_addr = smem_addr(sa + s * kGemmAStage), b_addr = smem_addr(sb + s * BSTAGE);
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk)
            umma_bf16(acc, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), idesc,
                      (kb > T.kb0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);  // this tile's MMAs (or none) are complete
        if (!ok) break;
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      GemmTile T;
      if (!gemm_tile<BN>(a, t, n_tn, n_tm, ks, T)) continue;
      const int b = it & 1, use = it >> 1;
      ++it;
      const bool has_k = T.kb1 > T.kb0;
      int ready = 1;
      if (lane == 0) ready = gemm_wait(&acc_full[b], use & 1, a.status, abort) ? 1 : 0;
      ready = __shfl_sync(0xffffffffu, ready, 0);
      if (!ready) break;
      tc_fence_after();
      const int row = T.m0 + q * 32 + lane;
      const bool row_ok = row < T.M;
      const long long crow = T.crow_base + row;
      const long long ccol0 = (long long)T.z * a.zc_col + T.n0;
      const bool out_f32 = a.c_f32 || ks > 1;
      void* cbase = ks > 1 ? static_cast<void*>(static_cast<float*>(a.C) + T.split * a.split_stride) : a.C;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        if (has_k) {
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * BN + c0), r);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        }
        if (!row_ok || T.n0 + c0 >= a.N) continue;
        const int ncols = min(32, a.N - (T.n0 + c0));
        if (out_f32) {
          float* dst = reinterpret_cast<float*>(cbase) + crow * a.ldc + ccol0 + c0;
          if (ncols == 32 && (((uintptr_t)dst) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              *reinterpret_cast<uint4*>(dst + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
          } else {
            for (int i = 0; i < ncols; ++i) dst[i] = __uint_as_float(r[i]);
          }
        } else {
          bf16_t* dst = reinterpret_cast<bf16_t*>(cbase) + crow * a.ldc + ccol0 + c0;
          if (ncols == 32 && (((uintptr_t)dst) & 15) == 0) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 u;
              u.x = (uint32_t)f2bf(__uint_as_float(r[i])) | ((uint32_t)f2bf(__uint_as_float(r[i + 1])) << 16);
              u.y = (uint32_t)f2bf(__uint_as_float(r[i + 2])) | ((uint32_t)f2bf(__uint_as_float(r[i + 3])) << 16);
              u.z = (uint32_t)f2bf(__uint_as_float(r[i + 4])) | ((uint32_t)f2bf(__uint_as_float(r[i + 5])) << 16);
              u.w = (uint32_t)f2bf(__uint_as_float(r[i + 6])) | ((uint32_t)f2bf(__uint_as_float(r[i + 7])) << 16);
              *reinterpret_cast<uint4*>(dst + i) = u;
            }
          } else {
            for (int i = 0; i < ncols; ++i) dst[i] = f2bf(__uint_as_float(r[i]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // this warp's quadrant of buffer b is read
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && *abort) {
    for (int i = *consumed; i < *issued; ++i) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && globaltimer_ns() - t0 < kLocalTimeoutNs) {
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN) : "memory");
  }
}

}  // namespace g4
