// Weight-streaming GEMV engine for the batch-1 decode step (sm_100a).
//
// Every matrix product of the decode step is y = W x with a bf16 weight W that is
// read exactly once per token, so the step is HBM-bound: the engine's job is to keep
// HBM busy from the first to the last byte of the step.
//
//  * One CTA per SM (grid = #SMs).  Warp 8 is a producer: one lane streams the CTA's
//    share of the weights into a ring of shared-memory stages with TMA bulk copies
//    (cp.async.bulk, L2 evict-first), each stage guarded by a full/empty mbarrier
//    pair.  Warps 0-7 consume: a warp takes a whole staged row and dots it with the
//    input vector, which each lane keeps in registers (the chunks it always touches),
//    so the only shared-memory traffic of the dot products is the weights themselves;
//    then a fused epilogue (rounding, GELU gating, router/argmax staging, peer stores).
//  * Prologue vectors (norm weights, the previous op's outputs) are staged in shared
//    memory before the operator's prologue runs; the consumers then run short loops
//    over shared memory -- no chains of dependent global loads at op start.
//  * Work split: the CTA's byte range of the concatenated segments (byte-balanced, so
//    mixed segments such as router rows + MLP gate/up rows stay balanced); a tile is
//    up to a stage's worth of consecutive units of one segment.
//  * Two drivers share the producer/consumer pieces below: gemv_kernel runs one
//    operator per launch (PDL-chained); the persistent step kernel (g4_step.cuh) runs
//    the whole decode step in one launch with one ring across all operators.
//
// Operators derive from OpBase and add:
//   __device__ bool seg_dependent(int s) const;   // addresses need prior results
//   __device__ void load_dependent(Smem&) const;  // producer lane, once they exist
//   __device__ void issue(int s,int u0,int n,unsigned char* stage,uint64_t* bar,
//                         uint64_t pol,const Smem&) const;   // producer: bulk copies
//   __device__ bool prologue(Smem&) const;        // consumers, staged vectors present
//   __device__ void epilogue(int s,int u0,int n,const Res& res,Smem&,bool ok) const;
//   __device__ void finish(Smem&, bool ok) const; // consumers, after all tiles
#pragma once

#include "g4_common.cuh"

namespace g4 {

constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kGemvThreads = kConsumerThreads + 32;
constexpr int kStages = 3;          // ring depth of the per-op kernels
constexpr int kMaxStages = 16;      // ring depth limit (persistent step kernel)
constexpr int kStageBytes = 45056;  // 8 rows of 2816 bf16: one row per consumer warp
constexpr int kMaxTileRows = 256;
constexpr int kResBufs = 2;         // per-tile result buffers (alternating)
constexpr int kMaxSeg = 3;
constexpr int kMaxCopies = 6;
constexpr int kBarConsumers = 1;  // named barrier id used by the consumer warps
constexpr int kMaxSmemBytes = 232448;  // 227 KB opt-in shared memory per CTA
constexpr int kOpCopyBytes = 640;      // shared copy of the current operator (step kernel)
// Smem::ints slots used by the engine (operators use 0..39)
constexpr int kSmemExp = 0;        // [0,16) expert ids (producer copy)
constexpr int kSmemSeq = 40;      // launch sequence number (persistent step kernel)
constexpr int kSmemIssued = 41;   // tiles issued by the producer lane so far
constexpr int kSmemProdExit = 42; // producer lane has issued its last copy
constexpr int kSmemRangesGiven = 43;  // 1: the CTA's unit ranges come from a host table
constexpr int kSmemDead = 63;     // CTA gave up after a timed-out wait

struct SegDesc {
  int units;  // number of work units
  int nsub;   // sub-rows per unit (1 plain, 2 gate/up pair, top-k for MoE down)
  int K;      // elements per sub-row (dot length), multiple of 8
  int group;  // tiles never straddle a multiple of `group` units (0 = no constraint)
  int weight; // cost factor of a unit's bytes in the CTA partition (0 or 1: bytes)
};

// One bulk copy of the prologue: `bytes` (multiple of 16) from global `src` to the
// shared staging area at byte offset `dst` (multiple of 16).
struct Copy {
  const void* src;
  int dst;
  int bytes;
};

// Fields every operator carries (filled on the host when the step is planned).
// Input vector of segment s: the bf16 vector x<xsel[s]> in shared memory; with
// xsub[s] > 0 (the MoE down projection) sub-row j has its own vector at x0 + j*xsub[s]
// floats and warp w owns sub-row j = w % nsub, its vector in registers for the whole
// segment (nsub must divide the consumer warp count).
struct alignas(16) OpBase {  // 16-byte multiple: plans are moved with bulk copies
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xsel[kMaxSeg];
  int xsub[kMaxSeg];
  int xbytes[2];  // bytes of the two bf16 input vectors in shared memory
  int stgbytes;   // bytes of the staging area (constant + activation vectors)
  int ncc, nac;   // constant copies / activation copies
  int trace_id;   // launch id for the optional timeline tracer (-DG4_TRACE)
  Copy cc[kMaxCopies];
  Copy ac[kMaxCopies];
};

__host__ __device__ __forceinline__ int seg_unit_bytes(const SegDesc& s) { return s.nsub * s.K * 2; }
// Partition cost of one unit: its bytes times the segment's weight.
__host__ __device__ __forceinline__ long long seg_unit_cost(const SegDesc& s) {
  return (long long)seg_unit_bytes(s) * (s.weight > 1 ? s.weight : 1);
}

__host__ __device__ __forceinline__ int seg_max_units(const SegDesc& s) {
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
  float* res;        // [kResBufs][kMaxTileRows]
  float* red;        // [64] block-reduction scratch
  int* ints;         // [64] small shared ints (expert ids, flags, argmax indices)
  float* flts;       // [64] small shared floats (routing weights, argmax values)
  unsigned char* opc;  // [kOpCopyBytes] the current operator's plan (step kernel consumers)
  unsigned char* popc; // [2][kOpCopyBytes] plans of the producer lane (step kernel)
  unsigned char* x0; // input vector 0 (bf16); also the start of the auxiliary area
  unsigned char* x1; // input vector 1 (bf16)
  unsigned char* stg;  // staging area of the prologue copies
  unsigned char* stages;
};

struct SmemSizes {
  int x0, x1, stg;
};

__host__ __device__ __forceinline__ int align_up(int v, int a) { return (v + a - 1) / a * a; }

__host__ __device__ __forceinline__ int smem_head_bytes(int stages) {
  int off = (2 * stages + 2) * 8;
  off = align_up(off, 16);
  off += kResBufs * kMaxTileRows * 4;
  off += 256 * 3;
  off = align_up(off, 16);
  off += 3 * kOpCopyBytes;
  return align_up(off, 128);
}

// Bytes of the auxiliary area [x0][x1][stg].
__host__ __device__ __forceinline__ int smem_aux_bytes(SmemSizes z) {
  return align_up(z.x0, 128) + align_up(z.x1, 128) + align_up(z.stg, 128);
}

// Layout: [bars][res][red][ints][flts][opc][popc][aux: x0 x1 stg][stages]; `aux` >= smem_aux_bytes
__host__ __device__ __forceinline__ int gemv_smem_bytes(int aux, int stages) {
  int off = smem_head_bytes(stages) + aux;
  off = align_up(off, 1024);
  off += stages * kStageBytes;
  return off + 1024;  // slack for base alignment
}

__device__ __forceinline__ Smem carve_smem(unsigned char* raw, SmemSizes z, int aux, int stages) {
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  Smem s;
  int off = 0;
  s.full = reinterpret_cast<uint64_t*>(base + off);
  s.empty = s.full + stages;
  s.pbar = s.empty + stages;
  off += (2 * stages + 2) * 8;
  off = align_up(off, 16);
  s.res = reinterpret_cast<float*>(base + off);
  off += kResBufs * kMaxTileRows * 4;
  s.red = reinterpret_cast<float*>(base + off);
  off += 256;
  s.ints = reinterpret_cast<int*>(base + off);
  off += 256;
  s.flts = reinterpret_cast<float*>(base + off);
  off += 256;
  off = align_up(off, 16);
  s.opc = base + off;
  off += kOpCopyBytes;
  s.popc = base + off;
  off += 2 * kOpCopyBytes;
  off = align_up(off, 128);
  s.x0 = base + off;
  s.x1 = s.x0 + align_up(z.x0, 128);
  s.stg = s.x1 + align_up(z.x1, 128);
  off += aux;
  off = align_up(off, 1024);
  s.stages = base + off;
  return s;
}

// Units of segment `s` owned by CTA `cta`: those whose first byte lies in the CTA's
// slice of the concatenated cost space of all segments (bytes x segment weight).
__host__ __device__ __forceinline__ void cta_unit_range(const SegDesc* seg, int nseg, int s, int cta, int ncta,
                                                        int& ub, int& ue) {
  long long total = 0, cum = 0;
  for (int i = 0; i < nseg; ++i) {
    long long b = (long long)seg[i].units * seg_unit_cost(seg[i]);
    if (i < s) cum += b;
    total += b;
  }
  const long long b0 = total * cta / ncta, b1 = total * (cta + 1) / ncta;
  const long long w = seg_unit_cost(seg[s]);
  auto first_unit_at = [&](long long b) -> int {
    long long rel = b - cum;
    if (rel <= 0) return 0;
    long long u = (rel + w - 1) / w;
    return u > seg[s].units ? seg[s].units : (int)u;
  };
  ub = first_unit_at(b0);
  ue = first_unit_at(b1);
}

__device__ __forceinline__ int tile_units(const SegDesc& sd, int u, int ue) {
  int n = seg_max_units(sd);
  if (ue - u < n) n = ue - u;
  if (sd.group > 0) {
    int gend = (u / sd.group + 1) * sd.group;
    if (gend - u < n) n = gend - u;
  }
  return n;
}

// Issue a list of prologue copies completing on `bar` (arrives once, with the total
// byte count, even when the list is empty).
__device__ __forceinline__ void issue_copies(const Copy* cp, int n, unsigned char* stg, uint64_t* bar) {
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
__device__ __forceinline__ bool wait_copies(Smem& sm, int which, uint32_t parity, int* status) {
  return mbar_wait(&sm.pbar[which], parity, status);
}

// Producer lane: fill the next stage with tile (s, u0, n) of `op`.  Returns false
// (after setting the CTA dead flag) when the stage never became free.
template <class Op>
__device__ __forceinline__ bool produce_tile(const Op& op, int s, int u0, int n, Smem& sm, RingPos& rp,
                                             int stages, uint64_t pol, int* status) {
  volatile int* dead = sm.ints + kSmemDead;
  if (rp.wrapped) {
    // bounded wait for the consumers to release the stage; leave early if they died
    if (!mbar_try_wait(&sm.empty[rp.st], rp.ph ^ 1u)) {
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&sm.empty[rp.st], rp.ph ^ 1u)) {
        if (*dead) return false;
        if (globaltimer_ns() - t0 > kLocalTimeoutNs) {
          atomicOr(status, G4_STATUS_MBAR_TIMEOUT);
          *dead = 1;
          return false;
        }
      }
    }
  }
  mbar_arrive_expect_tx(&sm.full[rp.st], (uint32_t)(n * seg_unit_bytes(op.seg[s])));
  unsigned char* stage = sm.stages + (size_t)rp.st * kStageBytes;
  uint64_t* bar = &sm.full[rp.st];
  op.copies(s, u0, n, sm.ints + kSmemExp, [&](const void* src, uint32_t bytes, uint32_t off) {
    bulk_g2s(stage + off, src, bytes, bar, pol);
  });
  rp.next(stages);
  reinterpret_cast<volatile int*>(sm.ints)[kSmemIssued] = rp.tiles;
  return true;
}

// Producer lane: mark the end of issuing (normal or abandoned).
__device__ __forceinline__ void producer_exit(Smem& sm) {
  __threadfence_block();
  reinterpret_cast<volatile int*>(sm.ints)[kSmemProdExit] = 1;
}

// Consumer thread 0 before the CTA exits after a failure: wait (bounded) for the
// producer to stop issuing, then for every issued stage past `rp` (the first tile
// thread 0 did not see complete), so that no bulk copy is still writing into this
// CTA's shared memory at exit.
__device__ __forceinline__ void drain_ring(Smem& sm, RingPos rp, int stages) {
  volatile int* v = reinterpret_cast<volatile int*>(sm.ints);
  const uint64_t t0 = globaltimer_ns();
  while (!v[kSmemProdExit] && globaltimer_ns() - t0 < kLocalTimeoutNs) __nanosleep(256);
  __threadfence_block();
  const int issued = v[kSmemIssued];
  while (rp.tiles < issued) {
    const uint64_t t1 = globaltimer_ns();
    while (!mbar_try_wait(&sm.full[rp.st], rp.ph) && globaltimer_ns() - t1 < kLocalTimeoutNs) {
    }
    rp.next(stages);
  }
}

// Per-tile results (one fp32 dot product per staged row), indexed by row.
struct Res {
  const float* p;
  __device__ __forceinline__ float operator[](int r) const { return p[r]; }
};

// 8-element dot product of a bf16 weight chunk with 8 bf16 input values packed in
// 4 words; products and sums in fp32 (the products of two bf16 values are exact).
__device__ __forceinline__ float dot8p(const uint4 w, const uint4 x, float acc) {
  acc = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
  acc = fmaf(bf_hi(w.x), bf_hi(x.x), acc);
  acc = fmaf(bf_lo(w.y), bf_lo(x.y), acc);
  acc = fmaf(bf_hi(w.y), bf_hi(x.y), acc);
  acc = fmaf(bf_lo(w.z), bf_lo(x.z), acc);
  acc = fmaf(bf_hi(w.z), bf_hi(x.z), acc);
  acc = fmaf(bf_lo(w.w), bf_lo(x.w), acc);
  acc = fmaf(bf_hi(w.w), bf_hi(x.w), acc);
  return acc;
}

// Input-vector chunks of one lane: chunk c = lane + 32 i, i < CPLM (CPLM = max chunks
// per lane of the kernel).  The weights are the only shared-memory traffic of the dot
// products; the input vector never leaves registers.  Every input vector of the step
// holds bf16 values (bf16 in shared memory too), so a lane keeps them packed, two per
// register: 4 registers per chunk.
template <int CPLM>
struct XRegs {
  uint4 v[CPLM];
  // x: the bf16 input vector in shared memory; chunk c is 8 consecutive elements.
  __device__ __forceinline__ void load(const bf16_t* x, int C) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int i = 0; i < CPLM; ++i) {
      const int c = lane + 32 * i;
      v[i] = c < C ? reinterpret_cast<const uint4*>(x)[c] : make_uint4(0u, 0u, 0u, 0u);
    }
  }
  // Warp-wide dot product of one staged row with the registers, NC iterations of 32
  // chunks: every iteration but the last covers whole warps of chunks, the last is
  // guarded unless FULL (C == 32 NC).  A compile-time trip count keeps the body free
  // of per-lane guards (a runtime bound on every unrolled iteration costs ~2.5x).
  template <int NC, bool FULL>
  __device__ __forceinline__ float dot_row_n(const uint4* w, int C) const {
    const int lane = threadIdx.x & 31;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (FULL || i < NC - 1 || c < C) {
        if (i & 1) a1 = dot8p(w[c], v[i], a1);
        else a0 = dot8p(w[c], v[i], a0);
      }
    }
    return warp_sum(a0 + a1);
  }
  // Four rows at once (row k at w + k * stride chunks), for short rows: the loads and
  // accumulators of all four are in flight together, and one transposing reduction
  // (6 shuffles instead of 4 x 5) leaves row k's sum on lane 8 k.
  template <int NC, bool FULL>
  __device__ __forceinline__ float dot_rows4_n(const uint4* w, int stride, int C) const {
    const int lane = threadIdx.x & 31;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int c = lane + 32 * i;
      if (FULL || i < NC - 1 || c < C) {
        uint4 wk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) wk[k] = w[k * stride + c];
#pragma unroll
        for (int k = 0; k < 4; ++k) a[k] = dot8p(wk[k], v[i], a[k]);
      }
    }
    const bool hi16 = (lane & 16) != 0, hi8 = (lane & 8) != 0;
    float k0 = hi16 ? a[2] : a[0], k1 = hi16 ? a[3] : a[1];
    const float s0 = hi16 ? a[0] : a[2], s1 = hi16 ? a[1] : a[3];
    k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
    k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
    float kk = hi8 ? k1 : k0;
    kk += __shfl_xor_sync(0xffffffffu, hi8 ? k0 : k1, 8);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) kk += __shfl_xor_sync(0xffffffffu, kk, o);
    return kk;  // lane 8 k: row k (k = 2 * bit4 + bit3 of the lane)
  }
  // Rows of at most 4 x 32 chunks: dispatch on the trip count (0.f for longer rows).
  __device__ __forceinline__ float dot_rows4(const uint4* w, int stride, int C) const {
    const int nc = (C + 31) >> 5;
    const bool full = (C & 31) == 0;
    switch (nc) {
#define G4_DOT4_CASE(N)                                                                   \
  case N:                                                                                 \
    if (N <= CPLM) {                                                                      \
      constexpr int M = N <= CPLM ? N : 1;                                                \
      return full ? dot_rows4_n<M, true>(w, stride, C) : dot_rows4_n<M, false>(w, stride, C); \
    }                                                                                     \
    break;
      G4_DOT4_CASE(1) G4_DOT4_CASE(2) G4_DOT4_CASE(3) G4_DOT4_CASE(4)
#undef G4_DOT4_CASE
      default: break;
    }
    return 0.f;
  }
  // C chunks (C <= 32 CPLM): dispatch on the trip count.
  __device__ __forceinline__ float dot_row(const uint4* w, int C) const {
    const int nc = (C + 31) >> 5;
    const bool full = (C & 31) == 0;
    switch (nc) {
#define G4_DOT_CASE(N)                                                      \
  case N:                                                                   \
    if (N <= CPLM) {                                                        \
      constexpr int M = N <= CPLM ? N : 1;                                  \
      return full ? dot_row_n<M, true>(w, C) : dot_row_n<M, false>(w, C);   \
    }                                                                       \
    break;
      G4_DOT_CASE(1) G4_DOT_CASE(2) G4_DOT_CASE(3) G4_DOT_CASE(4) G4_DOT_CASE(5) G4_DOT_CASE(6)
      G4_DOT_CASE(7) G4_DOT_CASE(8) G4_DOT_CASE(9) G4_DOT_CASE(10) G4_DOT_CASE(11) G4_DOT_CASE(12)
      G4_DOT_CASE(13) G4_DOT_CASE(14) G4_DOT_CASE(15) G4_DOT_CASE(16)
#undef G4_DOT_CASE
      default: break;
    }
    return 0.f;
  }
};

// Chunks per lane needed by a segment.
__host__ __device__ __forceinline__ int seg_cpl(const SegDesc& s) { return ((s.K >> 3) + 31) / 32; }

// Consumers: every tile of the operator `ob` owned by this CTA, in ring order.  With
// one vector for every sub-row (xsub == 0) row r goes to warp kConsumerWarps-1-r (mod
// the warp count): with fewer rows than warps, warp 0 -- whose thread 0 also waits at
// the grid barriers of the step kernel -- has no row.  After each tile's barrier,
// epi(s, u0, n, res, ok, t) runs on every consumer thread (the operator's epilogue; t is
// the thread's row index in it, >= n on threads without a row).
// Every consumer thread executes the same sequence of named barriers whatever happens,
// so a timed-out wait (which marks the CTA dead) can never strand a warp at a barrier:
// after it, the remaining tiles are skipped without waiting.
// `wp` advances only over the tiles this thread saw complete (the drain starts there).
// Hooks (all consumer threads call them, in this order per tile):
//   h.before_wait(rp)  -- before the wait for the tile at rp (step kernel: make sure
//                         it has been issued)
//   h.release(st)      -- lane 0 of each warp, after its dot products (per-op kernel:
//                         arrive on the stage's empty barrier)
//   h.after_bar(rp)    -- after the barrier that ends the tile's dot products, before
//                         the epilogue (step kernel: refill the freed stage)
struct NoHooks {
  __device__ __forceinline__ void before_wait(const RingPos&) {}
  __device__ __forceinline__ void release(Smem&, int) {}
  __device__ __forceinline__ void after_bar(const RingPos&) {}
};
struct EmptyBarrierHooks {
  __device__ __forceinline__ void before_wait(const RingPos&) {}
  __device__ __forceinline__ void release(Smem& sm, int st) { mbar_arrive(&sm.empty[st]); }
  __device__ __forceinline__ void after_bar(const RingPos&) {}
};

// The input vector lives here, in the one place the loop is instantiated: a register
// array shared by several inlined copies stays in local memory instead.
// `ranges` (step kernel): this CTA's precomputed [ub, ue) per segment (int2[kMaxSeg]),
// or null to compute them here.
template <int CPLM, class Hooks, class Epi>
__device__ __forceinline__ void consume_segments(const OpBase& ob, Smem& sm, RingPos& rp, RingPos& wp,
                                                 int stages, bool ok, int* status, Hooks& h, Epi&& epi,
                                                 const int2* ranges = nullptr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  XRegs<CPLM> xr;
  volatile int* dead = sm.ints + kSmemDead;
  bool first = true;
  const int nseg = ob.nseg;
  for (int s = 0; s < nseg; ++s) {
    int ub, ue;
    if (ranges) {
      ub = ranges[s].x;
      ue = ranges[s].y;
    } else {
      cta_unit_range(ob.seg, nseg, s, blockIdx.x, gridDim.x, ub, ue);
    }
    if (ub >= ue) continue;
    const SegDesc sd = ob.seg[s];
    const int C = sd.K >> 3;
    const int xsub = ob.xsub[s];
    const int sub = xsub ? warp % sd.nsub : 0;
    const bf16_t* xv = reinterpret_cast<const bf16_t*>(ob.xsel[s] ? sm.x1 : sm.x0) + sub * xsub;
    xr.load(xv, C);
    for (int u = ub; u < ue;) {
      const int n = tile_units(sd, u, ue);
      const int st = rp.st;
      h.before_wait(rp);
      bool live = (*dead == 0);
      if (live && !mbar_wait(&sm.full[st], rp.ph, status)) {
        *dead = 1;
        live = false;
      }
      if (live) wp.next(stages);
      if (first && threadIdx.x == 0) G4_TRACE_EV(ob.trace_id, 4);
      first = false;
      float* res = sm.res + (rp.tiles & (kResBufs - 1)) * kMaxTileRows;
      if (ok && live) {
        const unsigned char* stage = sm.stages + (size_t)st * kStageBytes;
        const int rowbytes = sd.K * 2;
        if (xsub == 0) {
          for (int r = kConsumerWarps - 1 - warp; r < n * sd.nsub; r += kConsumerWarps) {  // warp-uniform
            const float v = xr.dot_row(reinterpret_cast<const uint4*>(stage + (size_t)r * rowbytes), C);
            if (lane == 0) res[r] = v;
          }
        } else {
          const int step = kConsumerWarps / sd.nsub;
          int uu = warp / sd.nsub;
          if (step == 1 && C <= 128) {  // short rows, consecutive for this warp: 4 at a time
            for (; uu + 3 < n; uu += 4) {  // warp-uniform
              const int r = sub * n + uu;
              const float v = xr.dot_rows4(reinterpret_cast<const uint4*>(stage + (size_t)r * rowbytes), C, C);
              if ((lane & 7) == 0) res[r + (lane >> 3)] = v;
            }
          }
          for (; uu < n; uu += step) {  // warp-uniform
            const int r = sub * n + uu;
            const float v = xr.dot_row(reinterpret_cast<const uint4*>(stage + (size_t)r * rowbytes), C);
            if (lane == 0) res[r] = v;
          }
        }
      }
      __syncwarp();
      if (lane == 0 && live) h.release(sm, st);
      named_bar(kBarConsumers, kConsumerThreads);
      h.after_bar(rp);
      // epilogue row index of this thread: tiles of at most 32 units run their per-unit
      // work on one warp -- warp 0 when some warps had no row, else a warp that rotates
      // with the tile, so that no warp adds the epilogue to its dot products every tile
      int et = threadIdx.x;
      if (n <= 32) {
        const int ew = n * sd.nsub < kConsumerWarps ? 0 : (rp.tiles & (kConsumerWarps - 1));
        et = warp == ew ? lane : kConsumerThreads;
      }
      epi(s, u, n, Res{res}, ok && (*dead == 0), et);
      u += n;
      rp.next(stages);
    }
  }
}

// Weight-streaming kernel of one operator (the per-op launch mode of the decode step).
template <class Op, int CPLM>
__global__ void __launch_bounds__(kGemvThreads, 1) gemv_kernel(const __grid_constant__ Op op) {
  extern __shared__ unsigned char g4_dyn_smem[];
  const SmemSizes z{op.xbytes[0], op.xbytes[1], op.stgbytes};
  Smem sm = carve_smem(g4_dyn_smem, z, smem_aux_bytes(z), kStages);
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
    sm.ints[kSmemDead] = 0;
    sm.ints[kSmemIssued] = 0;
    sm.ints[kSmemProdExit] = 0;
    sm.ints[kSmemRangesGiven] = 0;
  }
  __syncthreads();
  pdl_trigger();
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 0);

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    // Constants and the first kStages weight tiles go out before griddepcontrol.wait
    // (weights never depend on the previous kernel); the activation copies right after.
    if (lane == 0) {
      const uint64_t pol = l2_evict_first_policy();
      issue_copies(op.cc, op.ncc, sm.stg, &sm.pbar[0]);
      bool waited = false, dep_loaded = false, alive = true;
      RingPos rp;
      for (int s = 0; s < op.nseg && alive; ++s) {
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
        for (int u = ub; u < ue && alive;) {
          const int n = tile_units(op.seg[s], u, ue);
          if (rp.wrapped && !waited) {
            pdl_wait();
            G4_TRACE_EV(op.trace_id, 2);
            waited = true;
            issue_copies(op.ac, op.nac, sm.stg, &sm.pbar[1]);
          }
          alive = produce_tile(op, s, u, n, sm, rp, kStages, pol, status);
          if (rp.tiles == 1) G4_TRACE_EV(op.trace_id, 1);
          u += n;
        }
      }
      if (!waited) {
        pdl_wait();
        G4_TRACE_EV(op.trace_id, 2);
        issue_copies(op.ac, op.nac, sm.stg, &sm.pbar[1]);
      }
      producer_exit(sm);
      G4_TRACE_EV(op.trace_id, 7);
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  pdl_wait();
  bool ok = wait_copies(sm, 0, 0, status);
  ok = wait_copies(sm, 1, 0, status) && ok;
  ok = op.prologue(sm) && ok;  // staged vectors, vector math
  named_bar(kBarConsumers, kConsumerThreads);
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 3);
  RingPos rp, wp;
  EmptyBarrierHooks hooks;
  consume_segments<CPLM>(op, sm, rp, wp, kStages, ok, status, hooks,
                         [&](int s, int u0, int n, const Res& r, bool eok, int t) { op.epilogue(s, u0, n, r, sm, eok, t); });
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 5);
  op.finish(sm, ok && (sm.ints[kSmemDead] == 0));
  if (threadIdx.x == 0) G4_TRACE_EV(op.trace_id, 6);
  named_bar(kBarConsumers, kConsumerThreads);
  if (threadIdx.x == 0 && sm.ints[kSmemDead]) drain_ring(sm, wp, kStages);
}

}  // namespace g4
