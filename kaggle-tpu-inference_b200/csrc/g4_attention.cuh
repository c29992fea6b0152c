// Split-KV decode attention for one query token (reference: gemma4_tpu/model.py:195-213).
//
// Work items are (KV head hk, split sp), n_kv x nsplit of them.  The live key span of
// KV head h -- (pos-window, pos] for sliding layers, [0, pos] for full layers, instead of
// the reference's masked pass over the whole max_len cache (masked entries contribute
// exp(-1e30 - max) = 0 there, so skipping them is exact) -- is cut into n_active <=
// nsplit slices of at least kAttnMinKeys keys; items past n_active do nothing.
//
// Keys stream through a ring of shared-memory stages.  A producer lane issues TMA tiled
// loads of KPS keys of K and of V per stage (2-D tensor maps over the cache viewed as
// [max_len, n_kv*d], 128-byte swizzle, boxes of 64 elements x KPS rows, L2 evict-first:
// the cache is read once per token); a full / empty mbarrier pair guards each stage.  The
// persistent step kernel feeds its one ring with these tiles too: layer l's attention
// tiles are issued right after layer l's qkv weights, so they stream in under the qkv
// phase.  The standalone kernel has a ring of its own (kAttnStages deep).
//
// Per item, the 8 consumer warps (two groups of 4; group g takes stages g, g+2, ...,
// keeps its own online-softmax state and releases the other group's stages once they
// have landed; the two states are combined at the end of the item):
//   1. q_norm RMSNorm + RoPE of the g query heads (bf16 rounding points of model.py:198
//      and 70-78); the item whose slice holds `pos` also normalises, RoPEs and writes k
//      (and v = rms(v_raw), or rms(k_raw) for k==v layers) into the cache
//      (model.py:200-206) and keeps both in shared memory;
//   2. per stage, on the tensor cores (mma.sync m16n8k16, bf16 in, fp32 accumulate):
//        S^T [KPS keys x 8 heads] = K . Q^T: warp w of a group contracts its own 16-dim
//          groups (w, w+4, ...) and leaves the partial in shared memory; after one group
//          barrier every warp adds the partials in warp order (the same bits in every
//          warp), rounds
//          the scores to bf16 as the reference einsum does, and updates the online
//          softmax (running max m, mass l);
//        O^T [16 dims x 8 heads] += V^T . P^T for the warp's own dim groups, with
//          P = exp(s - m) rounded to bf16.  The reference rounds the normalised
//          probabilities to bf16 before P.V; here the normalisation 1/l is applied once
//          at the end, in fp32.
//      The summed scores land in each thread exactly as its P^T operand fragment (keys
//      2c, 2c+1, 2c+8, 2c+9 of head lane/4), so no transposes are needed.  The cache row
//      at `pos` is never read from the stage: the ldmatrix row address of that key
//      points at the shared copy of the new key / value, and keys past the slice point
//      at a zero row (the stage holds stale or zero-filled rows there).
//   3. (m, l, O) of the item go to the partial buffer; the last CTA of each group of 8
//      splits (atomic counter) folds the group's partials in split order with
//      max-rescaling, and the last group of head h folds the group partials in group
//      order and rounds the context to bf16 (4-element vector loads, 4 to 16 partials in
//      flight per thread).
// Every sum has a fixed order: results are bitwise reproducible, and the step kernel
// and the standalone kernel (same items, same stages) compute identical bits.
#pragma once

#include <cuda.h>

#include "g4_common.cuh"

namespace g4 {

constexpr int kAttnThreads = 256;                      // consumer threads (8 warps)
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnKernelThreads = kAttnThreads + 32;  // + the producer warp (standalone kernel)
constexpr int kAttnStages = 4;                         // ring depth of the standalone kernel
constexpr int kAttnGroups = 2;                         // warp groups taking alternate stages
constexpr int kAttnGroupWarps = kAttnWarps / kAttnGroups;
constexpr int kBarAttnGroup = 3;                       // named barriers 3, 4: one per warp group
constexpr int kAttnMaxChunk = 1024;  // keys per item the host's split aims to stay under
constexpr int kAttnMinKeys = 32;     // keys per item before another split is used
constexpr int kAttnMaxG = 8;         // query heads per KV head: one 8-column MMA tile
constexpr int kAttnMaxD = 512;
constexpr int kAttnMaxSplit = 256;

struct AttnArgs {
  CUtensorMap tmk;         // cache_k as [max_len, n_kv*d] bf16, box 64 x attn_kps(d), 128-byte swizzle
  CUtensorMap tmv;         // cache_v, the same
  const bf16_t* qkv;       // q [n_kv*g*d] | k [n_kv*d] | v [n_kv*d] (v absent if k_eq_v)
  const bf16_t* q_norm;    // [d]
  const bf16_t* k_norm;    // [d]
  bf16_t* cache_k;         // [max_len, n_kv, d]
  bf16_t* cache_v;         // [max_len, n_kv, d]
  const float* inv_freq;   // [d/2]
  bf16_t* ctx;             // [n_kv*g*d]
  float* part;             // attn_part_floats(n_kv, nsplit, g, d): split and group partials
  int* counters;           // attn_counter_ints(n_kv, nsplit), zero at rest
  int* ctrl;               // control block (POS, STATUS)
  int pos_fixed;           // >= 0 overrides ctrl[POS]
  int n_kv, g, d, nsplit, window, k_eq_v, max_len;
  float eps;
  int trace_id;            // launch id for the optional timeline tracer (-DG4_TRACE)
};

// Merge of the split partials: up to kAttnMergeOne live splits, the last CTA of a head folds
// them all (one counter round trip); beyond, the last CTA of each group of kAttnMergeGroup
// splits folds the group's partials into a group partial, and the last such CTA of a head
// folds the group partials into the context.
constexpr int kAttnMergeGroup = 8;
constexpr int kAttnMergeOne = 16;
__host__ __device__ __forceinline__ int attn_groups(int nsplit) {
  return (nsplit + kAttnMergeGroup - 1) / kAttnMergeGroup;
}
// Floats of a layer's partial buffer: split partials O [n_kv][nsplit][g][d], their (m, l)
// [n_kv][nsplit][g][2], then the same two blocks for the group partials [n_kv][groups].
__host__ __device__ __forceinline__ size_t attn_part_floats(int n_kv, int nsplit, int g, int d) {
  return (size_t)n_kv * (size_t)(nsplit + attn_groups(nsplit)) * g * (d + 2);
}
// Ints of a layer's counters (zero at rest): one per head, then one per (head, group).
__host__ __device__ __forceinline__ int attn_counter_ints(int n_kv, int nsplit) {
  return n_kv * (1 + attn_groups(nsplit));
}

// Keys per stage (a multiple of 16), bytes of a stage (K boxes then V boxes, d/64 of
// each, KPS rows of 128 bytes per box) and the head stride of the score partials.
__host__ __device__ __forceinline__ int attn_kps(int d) { return d > 256 ? 16 : 32; }
__host__ __device__ __forceinline__ int attn_stage_bytes(int d) { return 4 * d * attn_kps(d); }
__host__ __device__ __forceinline__ int attn_hs(int d) { return attn_kps(d) + 8; }

// Scratch of one item (byte offsets from a 16-byte aligned base): the normalised query
// heads q [8][d] bf16 (rows past g zero), the new key and value [d] bf16 each, a 16-byte
// zero row, the RoPE table [d] fp32 (cos | sin), the score partials
// [2 groups][2][4 warps][8 heads][hs] fp32 (double-buffered by the group's stages; at the
// end of an item the same area carries group 1's state to group 0) and a flag word.
struct AttnSmem {
  int q, kn, vn, zero, rope, part, flag, bytes;
};
__host__ __device__ __forceinline__ AttnSmem attn_smem_layout(int d) {
  AttnSmem s;
  s.q = 0;
  s.kn = s.q + 8 * d * 2;
  s.vn = s.kn + d * 2;
  s.zero = s.vn + d * 2;
  s.rope = s.zero + 16;
  s.part = s.rope + d * 4;
  const int spart = 2 * kAttnWarps * 8 * attn_hs(d) * 4, xchg = 32 * d + 128;
  s.flag = s.part + (spart > xchg ? spart : xchg);
  s.bytes = s.flag + 64;
  return s;
}
__host__ __device__ __forceinline__ int attn_smem_bytes(int g, int d) {
  (void)g;
  return attn_smem_layout(d).bytes;
}
// Standalone kernel: alignment slack, the ring, the scratch, 2 x kAttnStages mbarriers
// and 4 ints (dead flag, stages issued, producer done).
__host__ __device__ __forceinline__ int attn_kernel_smem_bytes(int d) {
  return 1024 + kAttnStages * attn_stage_bytes(d) + ((attn_smem_layout(d).bytes + 15) & ~15) +
         2 * kAttnStages * 8 + 16;
}

// A ring of stages guarded by full (one producer arrival + bytes) / empty (one arrival
// per consumer warp) mbarriers.
struct AttnRing {
  uint64_t* full;
  uint64_t* empty;
  unsigned char* stages;
  int stride;  // bytes from one stage to the next (a multiple of 1024)
  int n;       // stages
};

// Keys [k0, k1) of split `sp` when the query sits at `pos`, and the number of splits
// that hold keys; false when split sp holds none.  Producer and consumers both use it.
__host__ __device__ __forceinline__ bool attn_span(int pos, int window, int nsplit, int sp, int& k0, int& k1,
                                                   int& n_active) {
  const int start = window > 0 ? (pos - window + 1 > 0 ? pos - window + 1 : 0) : 0;
  const int nlive = pos - start + 1;
  int chunk = (nlive + nsplit - 1) / nsplit;
  chunk = (chunk + kAttnMinKeys - 1) / kAttnMinKeys * kAttnMinKeys;  // whole 32-key stages
  n_active = (nlive + chunk - 1) / chunk;
  if (sp >= n_active) return false;
  k0 = start + sp * chunk;
  k1 = pos + 1 < k0 + chunk ? pos + 1 : k0 + chunk;
  return true;
}

__device__ __forceinline__ int attn_pos(const AttnArgs* a) {
  return a->pos_fixed >= 0 ? a->pos_fixed : ldcg_i(a->ctrl + G4_CTRL_POS);
}

// ------------------------------------------------------------------ warp-level MMA pieces
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}
// d += a . b for one m16n8k16 tile (A row-major 16x16, B column-major 16x8, bf16 in,
// fp32 accumulate).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Two fp32 values -> bf16x2 (round to nearest even), `lo` in the low half.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// 2-D TMA tile load into this CTA's shared memory with an L2 cache policy.
__device__ __forceinline__ void attn_tma_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_addr(dst)),
      "l"(map), "r"(smem_addr(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}

// Bounded wait for a stage to be released; sets *dead and a status bit on timeout (or
// returns at once when the consumers already died).
__device__ __forceinline__ bool ring_wait_free(uint64_t* empty, uint32_t parity, volatile int* dead, int* status) {
  if (mbar_try_wait(empty, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(empty, parity)) {
    if (*dead) return false;
    if (globaltimer_ns() - t0 > kLocalTimeoutNs) {
      atomicOr(status, G4_STATUS_MBAR_TIMEOUT);
      *dead = 1;
      return false;
    }
  }
  return true;
}

// Producer lane: the stages of this CTA's items (it0, it0 + step, ...) into `ring`, in
// the order the consumers take them.  `a` lives in global or kernel-parameter memory
// (the TMA reads its tensor maps there).  `issued` (optional) tracks the stages issued
// for a drain after a failure.  Returns false after setting *dead when a stage never
// became free.
__device__ __forceinline__ bool attn_produce(const AttnArgs* a, int it0, int step, const AttnRing& ring, RingPos& rp,
                                             volatile int* dead, int* status, int* issued) {
  const int d = a->d, nsplit = a->nsplit, kps = attn_kps(d), nbox = d >> 6;
  const int pos = attn_pos(a);
  if (pos < 0 || pos >= a->max_len) return true;  // the consumers skip the layer and report it
  const uint64_t pol = l2_evict_first_policy();
  const uint32_t bytes = (uint32_t)attn_stage_bytes(d);
  const int items = a->n_kv * nsplit;
  for (int it = it0; it < items; it += step) {
    int k0, k1, na;
    if (!attn_span(pos, a->window, nsplit, it % nsplit, k0, k1, na)) continue;
    const int x0 = (it / nsplit) * d;
    for (int ks = k0; ks < k1; ks += kps) {
      if (rp.wrapped && !ring_wait_free(&ring.empty[rp.st], rp.ph ^ 1u, dead, status)) return false;
      uint64_t* bar = &ring.full[rp.st];
      mbar_arrive_expect_tx(bar, bytes);
      unsigned char* stage = ring.stages + (size_t)rp.st * ring.stride;
      for (int j = 0; j < nbox; ++j) {
        attn_tma_load(stage + j * kps * 128, &a->tmk, x0 + 64 * j, ks, bar, pol);
        attn_tma_load(stage + (nbox + j) * kps * 128, &a->tmv, x0 + 64 * j, ks, bar, pol);
      }
      rp.next(ring.n);
      if (issued) *reinterpret_cast<volatile int*>(issued) = rp.tiles;
    }
  }
  return true;
}

// Fold n partials in order -- O rows [G][D] at po + s * G * D, (m, l) [G][2] at
// pml + s * G * 2 -- with max-rescaling: each thread takes 4-element chunks
// i = tid + 256 k of the [G][D] context and, SB partials at a time (their loads in flight
// together), keeps a running max-rescaled sum.  `ctx` non-null: writes the normalised
// context, rounded to bf16, there; else the folded partial to out_o / out_ml.  All
// kAttnThreads threads.
template <int D, int G>
__device__ __forceinline__ void attn_fold(const float* po, const float* pml, int n, bf16_t* ctx, float* out_o,
                                          float* out_ml) {
  constexpr int NC = G * D / 4;                                  // chunks per head set
  constexpr int NE = (NC + kAttnThreads - 1) / kAttnThreads;     // chunks per thread
  constexpr int SB = NE >= 4 ? 4 : 16 / NE;                      // partials per batch
  const float4* ho = reinterpret_cast<const float4*>(po);
  const float2* hml = reinterpret_cast<const float2*>(pml);
  float M[NE], L[NE];
  float4 O[NE];
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    M[k] = -INFINITY;
    L[k] = 0.f;
    O[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll 1
  for (int s0 = 0; s0 < n; s0 += SB) {
    float2 mlv[NE][SB];
    float4 av[NE][SB];
#pragma unroll
    for (int k = 0; k < NE; ++k) {
      const int i = threadIdx.x + kAttnThreads * k;
      const int h = (4 * i) / D;
#pragma unroll
      for (int q = 0; q < SB; ++q) {
        mlv[k][q] = make_float2(-INFINITY, 0.f);
        av[k][q] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < NC && s0 + q < n) {
          mlv[k][q] = __ldcg(hml + (size_t)(s0 + q) * G + h);
          av[k][q] = __ldcg(ho + (size_t)(s0 + q) * NC + i);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < NE; ++k) {
      float mb = M[k];
#pragma unroll
      for (int q = 0; q < SB; ++q) mb = fmaxf(mb, mlv[k][q].x);
      const float cf = M[k] == -INFINITY ? 0.f : expf(M[k] - mb);
      L[k] *= cf;
      O[k].x *= cf;
      O[k].y *= cf;
      O[k].z *= cf;
      O[k].w *= cf;
#pragma unroll
      for (int q = 0; q < SB; ++q) {
        const float f = mlv[k][q].x == -INFINITY ? 0.f : expf(mlv[k][q].x - mb);
        L[k] = fmaf(mlv[k][q].y, f, L[k]);
        O[k].x = fmaf(av[k][q].x, f, O[k].x);
        O[k].y = fmaf(av[k][q].y, f, O[k].y);
        O[k].z = fmaf(av[k][q].z, f, O[k].z);
        O[k].w = fmaf(av[k][q].w, f, O[k].w);
      }
      M[k] = mb;
    }
  }
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    const int i = threadIdx.x + kAttnThreads * k;
    if (i < NC) {
      const int h = (4 * i) / D, e = (4 * i) % D;
      if (ctx) {
        uint2 w;
        w.x = pack_bf16x2(O[k].x / L[k], O[k].y / L[k]);
        w.y = pack_bf16x2(O[k].z / L[k], O[k].w / L[k]);
        *reinterpret_cast<uint2*>(ctx + (size_t)h * D + e) = w;
      } else {
        reinterpret_cast<float4*>(out_o)[i] = O[k];
        if (e == 0) reinterpret_cast<float2*>(out_ml)[h] = make_float2(M[k], L[k]);
      }
    }
  }
}

// One work item (KV head hk, split sp) of decode attention, run by the kAttnThreads
// threads 0..kAttnThreads-1 of the block with named barrier `bar` among them and
// `smem` (attn_smem_bytes(G, D), 16-byte aligned) as scratch; its stages come from
// `ring` at `rp` (`wp` advances over the stages seen complete, for a drain after a
// failure).  Every exit is taken by all of these threads together.  D = head dim (a
// multiple of 64), G = query heads per KV head on this rank.
template <int D, int G>
__device__ __forceinline__ void attn_item(const AttnArgs& a, int hk, int sp, unsigned char* smem, int bar,
                                          const AttnRing& ring, RingPos& rp, RingPos& wp, volatile int* dead,
                                          int* status) {
  constexpr int PER = D / 32;                 // elements per lane of one head vector
  constexpr int KPS = D > 256 ? 16 : 32;      // keys per stage
  constexpr int NMT = KPS / 16;               // 16-key MMA tiles per stage
  constexpr int NDG = D / 16;                 // 16-dim groups
  constexpr int WPG = kAttnGroupWarps;        // warps per group
  constexpr int NPW = NDG < WPG ? NDG : WPG;  // warps of a group owning dim groups
  constexpr int GPW = (NDG + WPG - 1) / WPG;  // dim groups per warp
  constexpr int NBOX = D / 64;
  constexpr int HS = KPS + 8;
  static_assert(D % 64 == 0 && D <= kAttnMaxD && G >= 1 && G <= kAttnMaxG, "attention shape");
  static_assert(D / 2 <= kAttnThreads, "one RoPE frequency per thread");
  const AttnSmem lay = attn_smem_layout(D);
  bf16_t* q_s = reinterpret_cast<bf16_t*>(smem + lay.q);    // [8][D]
  bf16_t* kn_s = reinterpret_cast<bf16_t*>(smem + lay.kn);  // [D] new key
  bf16_t* vn_s = reinterpret_cast<bf16_t*>(smem + lay.vn);  // [D] new value
  float* rope_s = reinterpret_cast<float*>(smem + lay.rope);  // [D/2] cos | [D/2] sin
  float* spart = reinterpret_cast<float*>(smem + lay.part);   // [2][warps][8][HS]
  int* flag = reinterpret_cast<int*>(smem + lay.flag);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g8 = lane >> 2, c4 = lane & 3;  // fragment row / column pair of this lane
  // norm weights of this lane
  float wq[PER], wk[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    wq[i] = bf2f(a.q_norm[e]);
    wk[i] = bf2f(a.k_norm[e]);
  }
  const float fr = (int)threadIdx.x < D / 2 ? a.inv_freq[threadIdx.x] : 0.f;
  // this warp's first vector of step 1 (q head `warp`, or the raw k / v) does not depend
  // on the position: its loads go out now, with the position's
  const bf16_t* qraw = a.qkv;
  const bf16_t* kraw = a.qkv + (size_t)a.n_kv * G * D;
  const bf16_t* vraw = a.k_eq_v ? kraw : kraw + (size_t)a.n_kv * D;
  const bf16_t* src0 = warp < G ? qraw + ((size_t)hk * G + warp) * D
                                : (warp == G ? kraw + (size_t)hk * D : vraw + (size_t)hk * D);
  float pre[PER];
  if (warp < G + 2) {
#pragma unroll
    for (int i = 0; i < PER; ++i) pre[i] = bf2f(ldcg_bf(src0 + lane + 32 * i));
  }
  const int pos = attn_pos(&a);
  if (pos < 0 || pos >= a.max_len) {  // never index the cache out of bounds
    if (threadIdx.x == 0 && hk == 0 && sp == 0) atomicOr(a.ctrl + G4_CTRL_STATUS, G4_STATUS_POS_OVERFLOW);
    return;
  }
  int k0, k1, n_active;
  if (!attn_span(pos, a.window, a.nsplit, sp, k0, k1, n_active)) return;
  const size_t row_stride = (size_t)a.n_kv * D;

  // ---- 1. RoPE table of this position (cos / sin of pos * inv_freq, rounded to bf16
  // as the reference does, model.py:76-78): one sincosf per thread, shared by every
  // vector below.  Then the q heads (and the new k/v if this split holds pos): one
  // warp per vector.
  if ((int)threadIdx.x < D / 2) {
    float sn, cs;
    sincosf((float)pos * fr, &sn, &cs);
    rope_s[threadIdx.x] = rbf(cs);
    rope_s[D / 2 + threadIdx.x] = rbf(sn);
  }
  for (int i = threadIdx.x; i < (8 - G) * D; i += kAttnThreads) q_s[G * D + i] = 0;  // padding heads
  if (threadIdx.x < 4) reinterpret_cast<uint32_t*>(smem + lay.zero)[threadIdx.x] = 0u;
  named_bar(bar, kAttnThreads);
  const bool has_new = (pos >= k0 && pos < k1);
  const int nvec = G + (has_new ? 2 : 0);
  for (int vi = warp; vi < nvec; vi += kAttnWarps) {  // warp-uniform
    const bf16_t* src = vi < G ? qraw + ((size_t)hk * G + vi) * D
                               : (vi == G ? kraw + (size_t)hk * D : vraw + (size_t)hk * D);
    const bool rope = vi <= G;
    float v[PER];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      v[i] = vi == warp ? pre[i] : bf2f(ldcg_bf(src + lane + 32 * i));  // first vector: loaded at entry
      ss += v[i] * v[i];
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / (float)D + a.eps);
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      float o = v[i] * r;
      if (vi < G) o = o * wq[i];
      else if (vi == G) o = o * wk[i];
      v[i] = rbf(o);
    }
    if (rope) {  // rotate-half RoPE in bf16 arithmetic (model.py:70-78)
      float out[PER];
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int f = (lane + 32 * i) % (D / 2);
        const float cs = rope_s[f], sn = rope_s[D / 2 + f];
        const float rot = i < PER / 2 ? -v[i + PER / 2] : v[i - PER / 2];
        out[i] = rbf(rbf(v[i] * cs) + rbf(rot * sn));
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) v[i] = out[i];
    }
    if (vi < G) {
#pragma unroll
      for (int i = 0; i < PER; ++i) q_s[vi * D + lane + 32 * i] = f2bf(v[i]);
    } else {
      bf16_t* dst = (vi == G ? a.cache_k : a.cache_v) + (size_t)pos * row_stride + (size_t)hk * D;
      bf16_t* cpy = vi == G ? kn_s : vn_s;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const bf16_t b = f2bf(v[i]);
        dst[lane + 32 * i] = b;
        cpy[lane + 32 * i] = b;
      }
    }
  }
  named_bar(bar, kAttnThreads);
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 3);

  // ---- 2. the stages of this item (group grp computes stages grp, grp + 2, ...)
  const int grp = warp / WPG, wig = warp % WPG;
  // Q^T operand fragments of this warp's dim groups (column = head lane/4)
  uint32_t qb[GPW][2];
  float o[GPW][4];
#pragma unroll
  for (int i = 0; i < GPW; ++i) {
    const int t = wig + WPG * i;
    qb[i][0] = qb[i][1] = 0u;
    if (t < NDG) {
      qb[i][0] = *reinterpret_cast<const uint32_t*>(q_s + g8 * D + 16 * t + 2 * c4);
      qb[i][1] = *reinterpret_cast<const uint32_t*>(q_s + g8 * D + 16 * t + 2 * c4 + 8);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;  // head g8 (l: this lane's keys only)
  const uint32_t zero_sa = smem_addr(smem + lay.zero);
  const uint32_t kn_sa = smem_addr(kn_s), vn_sa = smem_addr(vn_s);
  const int r8 = lane & 7, mi = lane >> 3;  // ldmatrix: row within an 8x8 matrix, matrix index
  const int nst = (k1 - k0 + KPS - 1) / KPS;
#pragma unroll 1
  for (int s = 0; s < nst; ++s) {
    const int kbase = k0 + s * KPS;
    const int st = rp.st;
    bool live = (*dead == 0);
    if (live && !mbar_wait(&ring.full[st], rp.ph, status)) {
      *dead = 1;
      live = false;
    }
    live = __all_sync(0xffffffffu, live);  // warp-uniform: the shuffles below need the whole warp
    if (live) wp.next(ring.n);
    if ((s & 1) == grp) {  // group-uniform
      const uint32_t stage_sa = smem_addr(ring.stages + (size_t)st * ring.stride);
      float* part_s = spart + (grp * 2 + ((s >> 1) & 1)) * WPG * 8 * HS;
      if (live && wig < NPW) {  // S^T partial over this warp's dim groups
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
          const int kr = 16 * mt + r8 + (mi & 1) * 8;  // A rows = keys; matrices (rows, dims) 00 10 01 11
          const int key = kbase + kr;
#pragma unroll
          for (int i = 0; i < GPW; ++i) {
            const int t = wig + WPG * i;
            if (t < NDG) {
              const int q = 2 * t + (mi >> 1);  // 16-byte chunk of the row
              uint32_t addr = stage_sa + (q >> 3) * (KPS * 128) + kr * 128 + (((q & 7) ^ r8) << 4);
              if (key == pos) addr = kn_sa + q * 16;
              else if (key >= k1) addr = zero_sa;
              uint32_t af[4];
              ldsm_x4(addr, af);
              mma_16816(acc, af, qb[i][0], qb[i][1]);
            }
          }
          float* w_s = part_s + wig * 8 * HS;
          w_s[(2 * c4) * HS + 16 * mt + g8] = acc[0];
          w_s[(2 * c4 + 1) * HS + 16 * mt + g8] = acc[1];
          w_s[(2 * c4) * HS + 16 * mt + g8 + 8] = acc[2];
          w_s[(2 * c4 + 1) * HS + 16 * mt + g8 + 8] = acc[3];
        }
      }
      if (grp == 0) named_bar(kBarAttnGroup, WPG * 32);  // compile-time ids
      else named_bar(kBarAttnGroup + 1, WPG * 32);
      if (live) {
        // scores of head g8 at keys 16 mt + 2c, 2c+1, 2c+8, 2c+9: warp partials in order
        float sv[NMT][4];
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt)
#pragma unroll
          for (int e = 0; e < 4; ++e) sv[mt][e] = 0.f;
#pragma unroll
        for (int w = 0; w < NPW; ++w) {
          const float* hrow = part_s + (w * 8 + g8) * HS;
#pragma unroll
          for (int mt = 0; mt < NMT; ++mt) {
            const float2 lo = *reinterpret_cast<const float2*>(hrow + 16 * mt + 2 * c4);
            const float2 hi = *reinterpret_cast<const float2*>(hrow + 16 * mt + 2 * c4 + 8);
            sv[mt][0] += lo.x;
            sv[mt][1] += lo.y;
            sv[mt][2] += hi.x;
            sv[mt][3] += hi.y;
          }
        }
        float mx = m_run;
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kbase + 16 * mt + 2 * c4 + (e & 1) + (e >> 1) * 8;
            sv[mt][e] = key < k1 ? rbf(sv[mt][e]) : -INFINITY;
            mx = fmaxf(mx, sv[mt][e]);
          }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float corr = mx == -INFINITY ? 1.f : expf(m_run - mx);
        m_run = mx;
        uint32_t pb[NMT][2];
        float psum = 0.f;
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) {
          float p[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            p[e] = sv[mt][e] == -INFINITY ? 0.f : expf(sv[mt][e] - mx);
            psum += p[e];
          }
          pb[mt][0] = pack_bf16x2(p[0], p[1]);
          pb[mt][1] = pack_bf16x2(p[2], p[3]);
        }
        l_run = l_run * corr + psum;
        // rescale O^T: this lane's columns are heads 2c and 2c+1, held by lanes 8c and 8c+4
        const float ca = __shfl_sync(0xffffffffu, corr, 8 * c4);
        const float cb = __shfl_sync(0xffffffffu, corr, 8 * c4 + 4);
#pragma unroll
        for (int i = 0; i < GPW; ++i) {
          o[i][0] *= ca;
          o[i][1] *= cb;
          o[i][2] *= ca;
          o[i][3] *= cb;
        }
#pragma unroll
        for (int mt = 0; mt < NMT; ++mt) {
          const int kr = 16 * mt + r8 + (mi >> 1) * 8;  // A = V^T: matrices (dims, keys) 00 10 01 11
          const int key = kbase + kr;
#pragma unroll
          for (int i = 0; i < GPW; ++i) {
            const int t = wig + WPG * i;
            if (t < NDG) {
              const int q = 2 * t + (mi & 1);
              uint32_t addr = stage_sa + (NBOX + (q >> 3)) * (KPS * 128) + kr * 128 + (((q & 7) ^ r8) << 4);
              if (key == pos) addr = vn_sa + q * 16;
              else if (key >= k1) addr = zero_sa;
              uint32_t af[4];
              ldsm_x4_t(addr, af);
              mma_16816(o[i], af, pb[mt][0], pb[mt][1]);
            }
          }
        }
      }
    }
    // the other group's stage is released once it has landed (its wait above), so no
    // warp can count toward a later fill of the stage
    __syncwarp();
    if (lane == 0 && live) mbar_arrive(&ring.empty[st]);
    rp.next(ring.n);
  }
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 4);

  // ---- 3. the two groups' states combined in group 0 (fixed order), then the item's
  // partials -- O [G][D] in the O block (16-byte aligned rows for the merge's vector
  // loads), (m, l) [G][2] in the block after it -- and the last active CTA of this KV
  // head merges them.  The acq_rel counter update (after the block barrier) publishes
  // this CTA's partials and, for the last CTA, acquires every other CTA's.
  float lt = l_run + __shfl_xor_sync(0xffffffffu, l_run, 1);
  lt = lt + __shfl_xor_sync(0xffffffffu, lt, 2);  // the same bits in the four lanes of a head
  named_bar(bar, kAttnThreads);  // both groups are past their last reads of the partials
  float4* xo = reinterpret_cast<float4*>(spart);                  // [WPG][GPW][32] group 1's O
  float2* xml = reinterpret_cast<float2*>(spart + WPG * GPW * 32 * 4);  // [2 groups][8 heads] (m, l)
  if (wig == 0 && c4 == 0) xml[grp * 8 + g8] = make_float2(m_run, lt);
  if (grp == 1) {
#pragma unroll
    for (int i = 0; i < GPW; ++i) xo[(wig * GPW + i) * 32 + lane] = make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
  }
  named_bar(bar, kAttnThreads);
  const size_t n_items = (size_t)a.n_kv * a.nsplit;
  if (grp == 0) {
    // per head: M = max(m0, m1), factors exp(m - M) (0 for a group without keys; group 0
    // always holds the item's first stage)
    auto fac = [](float m, float M) { return m == -INFINITY ? 0.f : expf(m - M); };
    const float2 a0 = xml[2 * c4], a1 = xml[8 + 2 * c4], b0 = xml[2 * c4 + 1], b1 = xml[8 + 2 * c4 + 1];
    const float Ma = fmaxf(a0.x, a1.x), Mb = fmaxf(b0.x, b1.x);
    const float fa0 = fac(a0.x, Ma), fa1 = fac(a1.x, Ma), fb0 = fac(b0.x, Mb), fb1 = fac(b1.x, Mb);
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      const float4 q = xo[(wig * GPW + i) * 32 + lane];
      o[i][0] = o[i][0] * fa0 + q.x * fa1;
      o[i][1] = o[i][1] * fb0 + q.y * fb1;
      o[i][2] = o[i][2] * fa0 + q.z * fa1;
      o[i][3] = o[i][3] * fb0 + q.w * fb1;
    }
    float* part_o = a.part + ((size_t)hk * a.nsplit + sp) * G * D;
    float* part_ml = a.part + n_items * G * D + ((size_t)hk * a.nsplit + sp) * G * 2;
    if (wig == 0 && c4 == 0 && g8 < G) {
      const float2 h0 = xml[g8], h1 = xml[8 + g8];
      const float M = fmaxf(h0.x, h1.x);
      part_ml[g8 * 2] = M;
      part_ml[g8 * 2 + 1] = h0.y * fac(h0.x, M) + h1.y * fac(h1.x, M);
    }
#pragma unroll
    for (int i = 0; i < GPW; ++i) {
      const int t = wig + WPG * i;
      if (t < NDG) {
        const int dd = 16 * t + g8;
        if (2 * c4 < G) {
          part_o[(2 * c4) * D + dd] = o[i][0];
          part_o[(2 * c4) * D + dd + 8] = o[i][2];
        }
        if (2 * c4 + 1 < G) {
          part_o[(2 * c4 + 1) * D + dd] = o[i][1];
          part_o[(2 * c4 + 1) * D + dd + 8] = o[i][3];
        }
      }
    }
  }
  named_bar(bar, kAttnThreads);
  // level 1: the last CTA of this split's group folds the group's partials
  const bool one = n_active <= kAttnMergeOne;                                // one level
  const int ngs = attn_groups(a.nsplit);                                     // group slots per head
  const int ngr = one ? 1 : (n_active + kAttnMergeGroup - 1) / kAttnMergeGroup;  // live groups
  const int gi = one ? 0 : sp / kAttnMergeGroup;
  const int gsize = one ? n_active : min(kAttnMergeGroup, n_active - gi * kAttnMergeGroup);
  int* cnt_top = a.counters + hk;
  int* cnt_grp = one ? cnt_top : a.counters + a.n_kv + hk * ngs + gi;
  if (threadIdx.x == 0) {
    const int old = atomic_add_acq_rel_gpu(cnt_grp, 1);
    *flag = (old == gsize - 1);
  }
  named_bar(bar, kAttnThreads);
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 5);
  const bool merge = *flag != 0;
  named_bar(bar, kAttnThreads);  // every thread has read the flag before it is reused
  if (!merge) return;
  const size_t gbase = n_items * G * (D + 2);  // group partials after the split partials
  float* gpo = a.part + gbase + (size_t)hk * ngs * G * D;
  float* gpml = a.part + gbase + (size_t)a.n_kv * ngs * G * D + (size_t)hk * ngs * G * 2;
  const size_t s0 = (size_t)hk * a.nsplit + (size_t)gi * kAttnMergeGroup;
  bf16_t* ctx_h = a.ctx + (size_t)hk * G * D;
  if (ngr == 1) {  // one level: the fold is the context
    attn_fold<D, G>(a.part + s0 * G * D, a.part + n_items * G * D + s0 * G * 2, gsize, ctx_h, nullptr, nullptr);
    if (threadIdx.x == 0) {
      atomicExch(cnt_grp, 0);
      G4_TRACE_EV(a.trace_id, 6);
    }
    named_bar(bar, kAttnThreads);  // shared scratch free for the caller's next use
    return;
  }
  attn_fold<D, G>(a.part + s0 * G * D, a.part + n_items * G * D + s0 * G * 2, gsize, nullptr,
                  gpo + (size_t)gi * G * D, gpml + (size_t)gi * G * 2);
  // level 2: the last group of this head folds the group partials (acq_rel counter after
  // the block barrier: publishes this group partial, acquires the others)
  named_bar(bar, kAttnThreads);
  if (threadIdx.x == 0) {
    atomicExch(cnt_grp, 0);
    const int old = atomic_add_acq_rel_gpu(cnt_top, 1);
    *flag = (old == ngr - 1);
  }
  named_bar(bar, kAttnThreads);
  const bool merge2 = *flag != 0;
  named_bar(bar, kAttnThreads);
  if (!merge2) return;
  attn_fold<D, G>(gpo, gpml, ngr, ctx_h, nullptr, nullptr);
  if (threadIdx.x == 0) {
    atomicExch(cnt_top, 0);
    G4_TRACE_EV(a.trace_id, 6);
  }
  named_bar(bar, kAttnThreads);  // shared scratch free for the caller's next use
}

// Consumer thread 0 after a failure: wait (bounded) for the producer to stop issuing,
// then for every issued stage past `wp`, so that no TMA load still writes into this
// CTA's shared memory when it exits.  ints: [1] stages issued, [2] producer done.
__device__ __forceinline__ void attn_drain(const AttnRing& ring, RingPos wp, int* ints) {
  volatile int* v = ints;
  const uint64_t t0 = globaltimer_ns();
  while (!v[2] && globaltimer_ns() - t0 < kLocalTimeoutNs) __nanosleep(256);
  __threadfence_block();
  const int issued = v[1];
  while (wp.tiles < issued) {
    const uint64_t t1 = globaltimer_ns();
    while (!mbar_try_wait(&ring.full[wp.st], wp.ph) && globaltimer_ns() - t1 < kLocalTimeoutNs) {
    }
    wp.next(ring.n);
  }
}

// One item per CTA (standalone launches): item `it` of the items (0, step) of args `a`;
// warps 0-7 consume, warp 8 lane 0 produces the stages into a ring of its own.
template <int D, int G>
__device__ __forceinline__ void attn_cta(const AttnArgs& a, int it, int step) {
  extern __shared__ unsigned char attn_smem_raw[];
  constexpr int SB = 4 * D * (D > 256 ? 16 : 32);
  static_assert(SB % 1024 == 0, "stages stay 1024-byte aligned (128-byte swizzle)");
  unsigned char* base =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(attn_smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* scratch = base + kAttnStages * SB;
  uint64_t* full = reinterpret_cast<uint64_t*>(scratch + ((attn_smem_layout(D).bytes + 15) & ~15));
  uint64_t* empty = full + kAttnStages;
  int* ints = reinterpret_cast<int*>(empty + kAttnStages);  // dead, stages issued, producer done
  int* status = a.ctrl + G4_CTRL_STATUS;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kAttnStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kAttnWarps);
    }
    ints[0] = ints[1] = ints[2] = 0;
    mbar_init_fence();
  }
  __syncthreads();
  pdl_trigger();
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 0);
  pdl_wait();  // the position, the cache rows and qkv come from earlier kernels
  const AttnRing ring{full, empty, base, SB, kAttnStages};
  volatile int* dead = ints;
  if (threadIdx.x >= kAttnThreads) {
    if (threadIdx.x == kAttnThreads) {
      RingPos rp;
      attn_produce(&a, it, step, ring, rp, dead, status, ints + 1);
      __threadfence_block();
      reinterpret_cast<volatile int*>(ints)[2] = 1;
    }
    return;
  }
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 2);
  RingPos rp, wp;
  attn_item<D, G>(a, it / a.nsplit, it % a.nsplit, scratch, 1, ring, rp, wp, dead, status);
  if (threadIdx.x == 0 && *dead) attn_drain(ring, wp, ints);
}

// Standalone launch: grid = n_kv x nsplit, one item per CTA.
template <int D, int G>
__global__ void __launch_bounds__(kAttnKernelThreads, 1) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  attn_cta<D, G>(a, blockIdx.x, gridDim.x);
}

// Batched launch (several sequences' caches, one layer): grid = sequences x items, CTA b
// takes item b % items of sequence b / items, whose args (tensor maps included) live in
// the device array `args`.
template <int D, int G>
__global__ void __launch_bounds__(kAttnKernelThreads, 1) attn_decode_batch_kernel(const AttnArgs* __restrict__ args,
                                                                                   int items) {
  attn_cta<D, G>(args[blockIdx.x / items], blockIdx.x % items, items);
}

}  // namespace g4
