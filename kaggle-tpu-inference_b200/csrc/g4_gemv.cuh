// Weight-streaming GEMV engine for the batch-1 decode step (sm_100a).
//
// Every matrix product of the decode step is y = W x with a bf16 weight W that is
// read exactly once per token, so the step is HBM-bound: the engine's job is to keep
// HBM busy from the first to the last byte of every kernel and to spend as little
// fixed time per kernel as possible.
//
//  * One CTA per SM (grid = #SMs).  Warp 8 is a producer: one lane streams the CTA's
//    share of the weights into a ring of kStages shared-memory stages with TMA bulk
//    copies (cp.async.bulk, L2 evict-first), each stage guarded by a full/empty
//    mbarrier pair.  Warps 0-7 consume: a warp takes a whole staged row and dots it
//    with the input vector, which each lane keeps in registers (the chunks it always
//    touches), so the only shared-memory traffic of the dot products is the weights
//    themselves; then a fused epilogue (rounding, GELU gating, router/argmax staging,
//    peer stores).
//  * Prologue data movement is bulk copies too: before griddepcontrol.wait the
//    producer copies the kernel's constant vectors (norm weights) into a shared
//    staging area and issues the first weight stages (weights never depend on the
//    previous kernel); right after the wait it copies the activation vectors.  The
//    consumers then run short loops over shared memory -- no long unrolled code, no
//    chains of dependent global loads at kernel start.
//  * Work split: the CTA's byte range of the concatenated segments (byte-balanced, so
//    mixed segments such as router rows + MLP gate/up rows stay balanced); a tile is
//    up to a stage's worth of consecutive units of one segment.
//
// Operators derive from OpBase and add:
//   __device__ bool seg_dependent(int s) const;   // addresses need prior results
//   __device__ void load_dependent(Smem&) const;  // producer lane, after pdl_wait
//   __device__ void issue(int s,int u0,int n,unsigned char* stage,uint64_t* bar,
//                         uint64_t pol,const Smem&) const;   // producer: bulk copies
//   __device__ int xmode(int s) const;            // see gemv_kernel
//   __device__ bool prologue(Smem&) const;        // consumers (calls pdl_wait)
//   __device__ const float* xvec(int s,int j,const Smem&) const;   // fp32 input
//   __device__ void epilogue(int s,int u0,int n,const Res& res,Smem&,bool ok) const;
//   __device__ void finish(Smem&, bool ok) const; // consumers, after all tiles
#pragma once

#include "g4_common.cuh"

namespace g4 {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads + 32;
constexpr int kStages = 4;
constexpr int kStageBytes = 22528;  // 4 rows of 2816 bf16; 4 stages ~ 88 KB in flight
constexpr int kMaxTileRows = 256;
constexpr int kMaxSeg = 3;
constexpr int kMaxCopies = 6;
constexpr int kBarConsumers = 1;  // named barrier id used by the consumer warps
constexpr int kSmemDead = 63;     // Smem::ints slot: CTA gave up after a timed-out wait

struct SegDesc {
  int units;  // number of work units
  int nsub;   // sub-rows per unit (1 plain, 2 gate/up pair, top-k for MoE down)
  int K;      // elements per sub-row (dot length), multiple of 8
  int group;  // tiles never straddle a multiple of `group` units (0 = no constraint)
};

// One bulk copy of the prologue: `bytes` (multiple of 16) from global `src` to the
// shared staging area at byte offset `dst` (multiple of 16).
struct Copy {
  const void* src;
  int dst;
  int bytes;
};

// Fields every operator carries (filled on the host when the step is planned).
struct OpBase {
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];  // bytes of the two fp32 input vectors in shared memory
  int stgbytes;   // bytes of the staging area (constant + activation vectors)
  int ncc, nac;   // constant copies (before griddepcontrol.wait) / activation copies
  int trace_id;   // launch id for the optional timeline tracer (-DG4_TRACE)
  Copy cc[kMaxCopies];
  Copy ac[kMaxCopies];
};

__host__ __device__ inline int seg_unit_bytes(const SegDesc& s) { return s.nsub * s.K * 2; }

__host__ __device__ inline int seg_max_units(const SegDesc& s) {
  int by_bytes = kStageBytes / seg_unit_bytes(s);
  int by_rows = kMaxTileRows / s.nsub;
  int m = by_bytes < by_rows ? by_bytes : by_rows;
  return m < 1 ? 1 : m;
}

// Shared-memory context handed to the Op callbacks.
struct Smem {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* pbar;    // [2]: constants copied, activations copied
  float* res;        // [kStages][kMaxTileRows]
  float* red;        // [64] block-reduction scratch
  int* ints;         // [64] small shared ints (expert ids, flags, argmax indices)
  float* flts;       // [64] small shared floats (routing weights, argmax values)
  unsigned char* x0; // input vector 0 (fp32)
  unsigned char* x1; // input vector 1 (fp32)
  unsigned char* stg;  // staging area of the prologue copies
  unsigned char* stages;
};

struct SmemSizes {
  int x0, x1, stg;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

// Layout: [bars][res][red][ints][flts][x0][x1][stg][stages]
__host__ __device__ inline int gemv_smem_bytes(SmemSizes z) {
  int off = (2 * kStages + 2) * 8;
  off = align_up(off, 16);
  off += kStages * kMaxTileRows * 4;
  off += 256 * 3;
  off = align_up(off, 128);
  off += align_up(z.x0, 128) + align_up(z.x1, 128) + align_up(z.stg, 128);
  off = align_up(off, 1024);
  off += kStages * kStageBytes;
  return off + 1024;  // slack for base alignment
}

__device__ inline Smem carve_smem(unsigned char* raw, SmemSizes z) {
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  Smem s;
  int off = 0;
  s.full = reinterpret_cast<uint64_t*>(base + off);
  s.empty = s.full + kStages;
  s.pbar = s.empty + kStages;
  off += (2 * kStages + 2) * 8;
  off = align_up(off, 16);
  s.res = reinterpret_cast<float*>(base + off);
  off += kStages * kMaxTileRows * 4;
  s.red = reinterpret_cast<float*>(base + off);
  off += 256;
  s.ints = reinterpret_cast<int*>(base + off);
  off += 256;
  s.flts = reinterpret_cast<float*>(base + off);
  off += 256;
  off = align_up(off, 128);
  s.x0 = base + off;
  off += align_up(z.x0, 128);
  s.x1 = base + off;
  off += align_up(z.x1, 128);
  s.stg = base + off;
  off += align_up(z.stg, 128);
  off = align_up(off, 1024);
  s.stages = base + off;
  return s;
}

// Units of segment `s` owned by CTA `cta`: those whose first byte lies in the CTA's
// slice of the concatenated byte space of all segments.
__device__ inline void cta_unit_range(const SegDesc* seg, int nseg, int s, int cta, int ncta,
                                      int& ub, int& ue) {
  long long total = 0, cum = 0;
  for (int i = 0; i < nseg; ++i) {
    long long b = (long long)seg[i].units * seg_unit_bytes(seg[i]);
    if (i < s) cum += b;
    total += b;
  }
  const long long b0 = total * cta / ncta, b1 = total * (cta + 1) / ncta;
  const long long w = seg_unit_bytes(seg[s]);
  auto first_unit_at = [&](long long b) -> int {
    long long rel = b - cum;
    if (rel <= 0) return 0;
    long long u = (rel + w - 1) / w;
    return u > seg[s].units ? seg[s].units : (int)u;
  };
  ub = first_unit_at(b0);
  ue = first_unit_at(b1);
}

__device__ inline int tile_units(const SegDesc& sd, int u, int ue) {
  int n = seg_max_units(sd);
  if (ue - u < n) n = ue - u;
  if (sd.group > 0) {
    int gend = (u / sd.group + 1) * sd.group;
    if (gend - u < n) n = gend - u;
  }
  return n;
}

// Producer lane: issue a list of prologue copies completing on `bar` (arrives once,
// with the total byte count, even when the list is empty).
__device__ inline void issue_copies(const Copy* cp, int n, unsigned char* stg, uint64_t* bar) {
  uint32_t bytes = 0;
  for (int i = 0; i < n; ++i) bytes += (uint32_t)cp[i].bytes;
  mbar_arrive_expect_tx(bar, bytes);
  for (int i = 0; i < n; ++i) {
    // prologue vectors are re-read by every CTA: keep the default L2 policy
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(stg + cp[i].dst)),
        "l"(cp[i].src), "r"((uint32_t)cp[i].bytes), "r"(smem_addr(bar))
        : "memory");
  }
}

// Consumers: wait until the prologue copies of phase `which` (0 constants, 1
// activations) have landed.
__device__ inline bool wait_copies(Smem& sm, int which, int* status) {
  return mbar_wait(&sm.pbar[which], 0, status);
}

// Per-tile results (one fp32 dot product per staged row), indexed by row.
struct Res {
  const float* p;
  __device__ __forceinline__ float operator[](int r) const { return p[r]; }
};

// 8-element dot product of a bf16 chunk with 8 fp32 values held in registers.
__device__ __forceinline__ float dot8r(const uint4 w, const float* x, float acc) {
  acc = fmaf(bf_lo(w.x), x[0], acc);
  acc = fmaf(bf_hi(w.x), x[1], acc);
  acc = fmaf(bf_lo(w.y), x[2], acc);
  acc = fmaf(bf_hi(w.y), x[3], acc);
  acc = fmaf(bf_lo(w.z), x[4], acc);
  acc = fmaf(bf_hi(w.z), x[5], acc);
  acc = fmaf(bf_lo(w.w), x[6], acc);
  acc = fmaf(bf_hi(w.w), x[7], acc);
  return acc;
}

// Input-vector chunks of one lane: chunk c = lane + 32 i, i < CPLM (CPLM = max chunks
// per lane of the kernel).  The weights are the only shared-memory traffic of the dot
// products; the input vector never leaves registers.
template <int CPLM>
struct XRegs {
  float v[CPLM][8];
  __device__ __forceinline__ void load(const float* x, int C) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < CPLM; ++i) {
      const int c = lane + 32 * i;
      if (c < C) {
        const float4 a = reinterpret_cast<const float4*>(x)[2 * c];
        const float4 b = reinterpret_cast<const float4*>(x)[2 * c + 1];
        v[i][0] = a.x; v[i][1] = a.y; v[i][2] = a.z; v[i][3] = a.w;
        v[i][4] = b.x; v[i][5] = b.y; v[i][6] = b.z; v[i][7] = b.w;
      }
    }
  }
  // Warp-wide dot product of one staged row (C chunks) with the registers.
  __device__ __forceinline__ float dot_row(const uint4* w, int C) const {
    const int lane = threadIdx.x & 31;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < CPLM; ++i) {
      const int c = lane + 32 * i;
      if (c < C) {
        if (i & 1) a1 = dot8r(w[c], v[i], a1);
        else a0 = dot8r(w[c], v[i], a0);
      }
    }
    return warp_sum(a0 + a1);
  }
};

// Chunks per lane needed by a segment.
__host__ __device__ inline int seg_cpl(const SegDesc& s) { return ((s.K >> 3) + 31) / 32; }

// xmode of a segment (Op::xmode(s)): 0 = one input vector for every sub-row (warps
// take whole rows); 1 = sub-row j has its own input vector (top-k expert slices of
// the MoE down projection): warp w owns sub-row j = w % nsub and its vector stays in
// registers for the whole kernel (nsub must divide the consumer warp count).
template <class Op, int CPLM>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ Op op) {
  extern __shared__ unsigned char g4_dyn_smem[];
  Smem sm = carve_smem(g4_dyn_smem, SmemSizes{op.xbytes[0], op.xbytes[1], op.stgbytes});
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = op.ctrl + G4_CTRL_STATUS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsumerWarps);
    }
    mbar_init(&sm.pbar[0], 1);
    mbar_init(&sm.pbar[1], 1);
    mbar_init_fence();
  }
  __syncthreads();
  pdl_trigger();
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 0);

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      issue_copies(op.cc, op.ncc, sm.stg, &sm.pbar[0]);  // constants: before the wait
      bool waited = false, dep_loaded = false;
      int t = 0;
      for (int s = 0; s < op.nseg; ++s) {
        int ub, ue;
        cta_unit_range(op.seg, op.nseg, s, blockIdx.x, gridDim.x, ub, ue);
        if (ub >= ue) continue;
        if (op.seg_dependent(s) && !dep_loaded) {
          if (!waited) {
            pdl_wait();
            G4_TRACE_EV(op.trace_id, 2);
            waited = true;
            issue_copies(op.ac, op.nac, sm.stg, &sm.pbar[1]);
          }
          op.load_dependent(sm);
          dep_loaded = true;
        }
        for (int u = ub; u < ue; ++t) {
          const int n = tile_units(op.seg[s], u, ue);
          const int st = t % kStages;
          if (t >= kStages) {
            if (!waited) {  // the first stages are in flight: now wait, then activations
              pdl_wait();
              G4_TRACE_EV(op.trace_id, 2);
              waited = true;
              issue_copies(op.ac, op.nac, sm.stg, &sm.pbar[1]);
            }
            if (!mbar_wait(&sm.empty[st], ((t / kStages) - 1) & 1, status)) return;
          }
          mbar_arrive_expect_tx(&sm.full[st], (uint32_t)(n * seg_unit_bytes(op.seg[s])));
          op.issue(s, u, n, sm.stages + (size_t)st * kStageBytes, &sm.full[st], pol, sm);
          if (t == 0) G4_TRACE_EV(op.trace_id, 1);
          u += n;
        }
      }
      if (!waited) {
        pdl_wait();
        G4_TRACE_EV(op.trace_id, 2);
        issue_copies(op.ac, op.nac, sm.stg, &sm.pbar[1]);
      }
      G4_TRACE_EV(op.trace_id, 7);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // Every consumer thread executes the same sequence of named barriers whatever
  // happens, so a timed-out wait (which marks the CTA dead) can never strand a warp
  // at a barrier: after it, the remaining tiles are skipped without waiting.
  volatile int* dead = sm.ints + kSmemDead;
  if (threadIdx.x == 0) *dead = 0;
  named_bar(kBarConsumers, kConsumerThreads);
  bool ok = op.prologue(sm);  // griddepcontrol.wait, staged vectors, vector math
  named_bar(kBarConsumers, kConsumerThreads);
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 3);
  XRegs<CPLM> xr;
  int t = 0;
  for (int s = 0; s < op.nseg; ++s) {
    int ub, ue;
    cta_unit_range(op.seg, op.nseg, s, blockIdx.x, gridDim.x, ub, ue);
    if (ub >= ue) continue;
    const SegDesc sd = op.seg[s];
    const int C = sd.K >> 3;
    const int xm = op.xmode(s);
    const int sub = xm ? warp % sd.nsub : 0;
    xr.load(op.xvec(s, sub, sm), C);
    for (int u = ub; u < ue; ++t) {
      const int n = tile_units(sd, u, ue);
      const int st = t % kStages;
      bool live = (*dead == 0);
      if (live && !mbar_wait(&sm.full[st], (t / kStages) & 1, status)) {
        *dead = 1;
        live = false;
      }
      if (t == 0 && threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 4);
      float* res = sm.res + st * kMaxTileRows;
      if (ok && live) {
        const unsigned char* stage = sm.stages + (size_t)st * kStageBytes;
        const int rowbytes = sd.K * 2;
        if (xm == 0) {
          for (int r = warp; r < n * sd.nsub; r += kConsumerWarps) {  // warp-uniform
            const float v = xr.dot_row(reinterpret_cast<const uint4*>(stage + (size_t)r * rowbytes), C);
            if (lane == 0) res[r] = v;
          }
        } else {
          const int step = kConsumerWarps / sd.nsub;
          for (int uu = warp / sd.nsub; uu < n; uu += step) {  // warp-uniform
            const int r = sub * n + uu;
            const float v = xr.dot_row(reinterpret_cast<const uint4*>(stage + (size_t)r * rowbytes), C);
            if (lane == 0) res[r] = v;
          }
        }
      }
      __syncwarp();
      if (lane == 0 && live) mbar_arrive(&sm.empty[st]);
      named_bar(kBarConsumers, kConsumerThreads);
      op.epilogue(s, u, n, Res{res}, sm, ok && (*dead == 0));
      u += n;
    }
  }
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 5);
  op.finish(sm, ok && (*dead == 0));
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 6);
}

}  // namespace g4
