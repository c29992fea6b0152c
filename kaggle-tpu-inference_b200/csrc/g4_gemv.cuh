// Weight-streaming GEMV engine for the batch-1 decode step (sm_100a).
//
// Every matrix product of the decode step is y = W x with a bf16 weight W that is
// read exactly once per token, so the step is HBM-bound: the engine's job is to keep
// HBM busy from the first to the last byte of every kernel.
//
//  * One CTA per SM (grid = #SMs).  Warp 8 is a producer: one lane streams the CTA's
//    share of the weights into a ring of kStages shared-memory stages with TMA bulk
//    copies (cp.async.bulk, L2 evict-first), each stage guarded by a full/empty
//    mbarrier pair.  Warps 0-7 consume: segmented dot products of the staged rows
//    against the input vector(s) held in shared memory, fp32 accumulation, then a
//    fused epilogue (rounding, GELU gating, router/argmax staging, peer stores).
//  * Programmatic dependent launch: the producer issues the first stages BEFORE
//    griddepcontrol.wait (weights never depend on the previous kernel), so the
//    weight stream of kernel N+1 starts while kernel N drains.  No global memory is
//    written and no mutable global memory is read before the wait.
//  * Work split: the CTA's byte range of the concatenated segments (byte-balanced, so
//    mixed segments such as router rows + MLP gate/up rows stay balanced); a tile is
//    up to a stage's worth of consecutive units of one segment.
//
// An "Op" supplies the segments and the fused prologue / epilogue:
//   struct Op {
//     int nseg; SegDesc seg[kMaxSeg];
//     int xbytes[2];                                    // shared-memory input vectors
//     __device__ bool seg_dependent(int s) const;       // addresses need prior results
//     __device__ void load_dependent(Smem&) const;      // producer, after pdl_wait
//     __device__ void issue(int s,int u0,int n,char* stage,uint64_t* bar,uint64_t pol,
//                           const Smem&) const;         // producer lane: bulk copies
//     __device__ bool prologue(Smem&) const;            // consumers, after pdl_wait
//     __device__ const bf16_t* xvec(int s,int j,const Smem&) const;
//     __device__ void epilogue(int s,int u0,int n,const float* res,Smem&,bool ok) const;
//     __device__ void finish(Smem&, bool ok) const;     // consumers, after all tiles
//   };
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
constexpr int kBarConsumers = 1;  // named barrier id used by the consumer warps
constexpr int kSmemDead = 63;     // Smem::ints slot: CTA gave up after a timed-out wait

struct SegDesc {
  int units;  // number of work units
  int nsub;   // sub-rows per unit (1 plain, 2 gate/up pair, top-k for MoE down)
  int K;      // elements per sub-row (dot length), multiple of 8
  int group;  // tiles never straddle a multiple of `group` units (0 = no constraint)
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
  float* res;        // [kStages][kMaxTileRows]
  float* red;        // [64] block-reduction scratch
  int* ints;         // [64] small shared ints (expert ids, flags, argmax indices)
  float* flts;       // [64] small shared floats (routing weights, argmax values)
  unsigned char* x0; // input vector 0
  unsigned char* x1; // input vector 1
  unsigned char* stages;
};

struct SmemSizes {
  int x0, x1;
};

__host__ __device__ inline int align_up(int v, int a) { return (v + a - 1) / a * a; }

// Layout: [bars 2*kStages*8][res][red 256B][ints 256B][flts 256B][x0][x1][stages]
__host__ __device__ inline int gemv_smem_bytes(SmemSizes z) {
  int off = 2 * kStages * 8;
  off += kStages * kMaxTileRows * 4;
  off += 256 * 3;
  off = align_up(off, 128);
  off += align_up(z.x0, 128) + align_up(z.x1, 128);
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
  off += 2 * kStages * 8;
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

// Segmented dot products of `nrows` staged rows (row r at stage + r*K*2 bytes) with the
// input vector chosen per sub-row: sub-row j of the tile's n units is rows [j*n, j*n+n).
template <class Op>
__device__ inline void consume_tile(const Op& op, int s, int n, const unsigned char* stage,
                                    float* res, const Smem& sm) {
  const SegDesc& sd = op.seg[s];
  const int nrows = n * sd.nsub;
  const int C = sd.K >> 3;  // 16-byte chunks per row
  const int L = C >= 32 ? 32 : (C >= 16 ? 16 : (C >= 8 ? 8 : 4));
  const int P = 32 / L;  // rows per warp pass
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = lane / L, li = lane % L;
  const int rowbytes = sd.K * 2;
  for (int r0 = warp * P; r0 < nrows; r0 += kConsumerWarps * P) {
    const int r = r0 + gi;
    float acc = 0.f;
    if (r < nrows) {
      const uint4* w = reinterpret_cast<const uint4*>(stage + (size_t)r * rowbytes);
      const uint4* x = reinterpret_cast<const uint4*>(op.xvec(s, r / n, sm));
#pragma unroll 4
      for (int c = li; c < C; c += L) acc = dot8(w[c], x[c], acc);
    }
    acc = group_sum(acc, L);
    if (li == 0 && r < nrows) res[r] = acc;
  }
}

template <class Op>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ Op op) {
  extern __shared__ unsigned char g4_dyn_smem[];
  Smem sm = carve_smem(g4_dyn_smem, SmemSizes{op.xbytes[0], op.xbytes[1]});
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* status = op.ctrl + G4_CTRL_STATUS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsumerWarps);
    }
    mbar_init_fence();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      bool waited = false;
      int t = 0;
      for (int s = 0; s < op.nseg; ++s) {
        int ub, ue;
        cta_unit_range(op.seg, op.nseg, s, blockIdx.x, gridDim.x, ub, ue);
        if (ub >= ue) continue;
        if (op.seg_dependent(s) && !waited) {
          pdl_wait();
          waited = true;
          op.load_dependent(sm);
        }
        for (int u = ub; u < ue; ++t) {
          const int n = tile_units(op.seg[s], u, ue);
          const int st = t % kStages;
          if (t >= kStages && !mbar_wait(&sm.empty[st], ((t / kStages) - 1) & 1, status)) return;
          mbar_arrive_expect_tx(&sm.full[st], (uint32_t)(n * seg_unit_bytes(op.seg[s])));
          op.issue(s, u, n, sm.stages + (size_t)st * kStageBytes, &sm.full[st], pol, sm);
          u += n;
        }
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  // Every consumer thread executes the same sequence of named barriers whatever
  // happens, so a timed-out wait (which marks the CTA dead) can never strand a warp
  // at a barrier: after it, the remaining tiles are skipped without waiting.
  pdl_wait();
  volatile int* dead = sm.ints + kSmemDead;
  if (threadIdx.x == 0) *dead = 0;
  named_bar(kBarConsumers, kConsumerThreads);
  bool ok = op.prologue(sm);
  named_bar(kBarConsumers, kConsumerThreads);
  int t = 0;
  for (int s = 0; s < op.nseg; ++s) {
    int ub, ue;
    cta_unit_range(op.seg, op.nseg, s, blockIdx.x, gridDim.x, ub, ue);
    for (int u = ub; u < ue; ++t) {
      const int n = tile_units(op.seg[s], u, ue);
      const int st = t % kStages;
      bool live = (*dead == 0);
      if (live && !mbar_wait(&sm.full[st], (t / kStages) & 1, status)) {
        *dead = 1;
        live = false;
      }
      float* res = sm.res + st * kMaxTileRows;
      if (ok && live) consume_tile(op, s, n, sm.stages + (size_t)st * kStageBytes, res, sm);
      __syncwarp();
      if (lane == 0 && live) mbar_arrive(&sm.empty[st]);
      named_bar(kBarConsumers, kConsumerThreads);
      op.epilogue(s, u, n, res, sm, ok && (*dead == 0));
      u += n;
    }
  }
  op.finish(sm, ok && (*dead == 0));
}

}  // namespace g4
