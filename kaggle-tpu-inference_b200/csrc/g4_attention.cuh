// Split-KV decode attention for one query token (reference: gemma4_tpu/model.py:195-213).
//
// Grid = n_kv (local KV heads) x nsplit.  The live key span of KV head h --
// (pos-window, pos] for sliding layers, [0, pos] for full layers, instead of the
// reference's masked pass over the whole max_len cache (masked entries contribute
// exp(-1e30 - max) = 0 there, so skipping them is exact) -- is cut into
// n_active <= nsplit slices of at least kAttnMinKeys keys; CTAs past n_active exit
// at once.  Per active CTA:
//   1. q_norm RMSNorm + RoPE of the g query heads of KV head h (bf16 rounding points
//      of model.py:198 / 70-78); the CTA whose slice holds `pos` also normalises,
//      RoPEs and writes k (and v = rms(v_raw), or rms(k_raw) for k==v layers) into
//      the cache (model.py:200-206).
//   2. every group of LK lanes owns a strided set of keys and runs an online softmax
//      over them: scores s = bf16(q.k) (scale 1.0, rounded like the reference einsum),
//      running max / mass, and acc += exp(s - m) v in fp32 registers; K and V of a
//      batch of keys are loaded together.
//   3. the lane groups are merged in a fixed order (butterfly within a warp, then warp
//      by warp through shared memory) into (m, l, acc[g][d]), which goes to the
//      partial buffer; the last CTA of head h (atomic counter) merges the n_active
//      partials in split order with max-rescaling and rounds the context to bf16.
//      Every sum has a fixed order: results are bitwise reproducible.
// Difference from the reference: it rounds the normalised probabilities to bf16
// before P.V; here P.V uses fp32 weights and the context is rounded once -- closer
// to exact arithmetic, within the tolerance the parity tests state.
#pragma once

#include "g4_common.cuh"

namespace g4 {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxChunk = 1024;  // keys per CTA
constexpr int kAttnMinKeys = 32;     // keys per CTA before another split is used
constexpr int kAttnMaxG = 8;         // query heads per KV head handled by one CTA
constexpr int kAttnMaxD = 512;
constexpr int kAttnMaxSplit = 256;

struct AttnArgs {
  const bf16_t* qkv;       // q [n_kv*g*d] | k [n_kv*d] | v [n_kv*d] (v absent if k_eq_v)
  const bf16_t* q_norm;    // [d]
  const bf16_t* k_norm;    // [d]
  bf16_t* cache_k;         // [max_len, n_kv, d]
  bf16_t* cache_v;         // [max_len, n_kv, d]
  const float* inv_freq;   // [d/2]
  bf16_t* ctx;             // [n_kv*g*d]
  float* part;             // [n_kv, nsplit, g, d+2] (m, l, acc[d])
  int* counters;           // [n_kv], zero at rest
  int* ctrl;               // control block (POS, STATUS)
  int pos_fixed;           // >= 0 overrides ctrl[POS]
  int n_kv, g, d, nsplit, window, k_eq_v, max_len;
  float eps;
  int trace_id;            // launch id for the optional timeline tracer (-DG4_TRACE)
};

// Heads per pass (at most 4) and whether the warps' partial sums are merged through
// per-warp shared-memory slots (one barrier) rather than warp by warp (a barrier each):
// when the slots take at most 32 KB.
__host__ __device__ __forceinline__ int attn_heads_per_pass(int g) { return g > 4 ? 4 : g; }
__host__ __device__ __forceinline__ bool attn_slot_merge(int g, int d) { return attn_heads_per_pass(g) * d <= 1024; }

__host__ __device__ __forceinline__ int attn_smem_bytes(int g, int d) {
  // acc [g][d] + lane-group stats [64][g] x 2 + misc + the normalised query heads
  // q_s [g][d] (bf16) + the new key and value kn_s / vn_s [d] (bf16) + the RoPE
  // table [d] (fp32 cos | sin) + the merge slots [warps][heads per pass][d] (fp32)
  return g * d * 4 + 2 * 64 * g * 4 + 2 * kAttnMaxG * 4 + 64 + g * d * 2 + 2 * d * 2 + d * 4 +
         (attn_slot_merge(g, d) ? kAttnWarps * attn_heads_per_pass(g) * d * 4 : 0);
}

// One work item (KV head hk, split sp) of decode attention, run by the kAttnThreads
// threads 0..kAttnThreads-1 of the block with named barrier `bar` among them and
// `smem` (attn_smem_bytes(G, D), 16-byte aligned) as scratch.  Every exit is taken by
// all of these threads together.  D = head dim, G = query heads per KV head on this
// rank; every loop has a compile-time trip count.
template <int D, int G>
__device__ __forceinline__ void attn_item(const AttnArgs& a, int hk, int sp, unsigned char* smem, int bar) {
  constexpr int PER = D / 32;                 // elements per lane of one head vector
  constexpr int LK = D / 8 < 32 ? D / 8 : 32; // lanes per key
  constexpr int KPW = 32 / LK;                // lane groups per warp
  constexpr int CPL = (D / 8) / LK;           // 16-byte chunks per lane of a key row
  constexpr int NGRP = kAttnWarps * KPW;      // lane groups per CTA
  constexpr int KB = 4;                       // keys per lane group in flight
  // heads kept in registers at once: at most 4, so that the item fits the step
  // kernel's register budget next to everything else (more heads = one more pass
  // over the keys, which then come from L2)
  constexpr int HG = G > 4 ? 4 : G;
  float* acc_s = reinterpret_cast<float*>(smem);                     // [G][D]
  float* gm = acc_s + G * D;                                         // [NGRP][G]
  float* gl = gm + 64 * G;                                           // [NGRP][G]
  float* ml = gl + 64 * G;                                           // M[G], L[G]
  int* flag = reinterpret_cast<int*>(ml + 2 * kAttnMaxG);
  bf16_t* q_s = reinterpret_cast<bf16_t*>(flag + 16);                // [G][D]
  bf16_t* kn_s = q_s + G * D;                                        // [D] new key
  bf16_t* vn_s = kn_s + D;                                           // [D] new value
  float* rope_s = reinterpret_cast<float*>(vn_s + D);                // [D/2] cos | [D/2] sin
  float* mslot = rope_s + D;                                         // [warps][HG][D] (slot merge)
  constexpr bool kSlotMerge = HG * D <= 1024;
  static_assert(kSlotMerge == (HG * D <= 1024), "same rule as attn_slot_merge");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
  const int pos = a.pos_fixed >= 0 ? a.pos_fixed : ldcg_i(a.ctrl + G4_CTRL_POS);
  if (pos < 0 || pos >= a.max_len) {  // never index the cache out of bounds
    if (threadIdx.x == 0 && hk == 0 && sp == 0) atomicOr(a.ctrl + G4_CTRL_STATUS, G4_STATUS_POS_OVERFLOW);
    return;
  }
  const int start = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int nlive = pos - start + 1;
  int chunk = (nlive + a.nsplit - 1) / a.nsplit;
  if (chunk < kAttnMinKeys) chunk = kAttnMinKeys;
  const int n_active = (nlive + chunk - 1) / chunk;
  if (sp >= n_active) return;
  const int k0 = start + sp * chunk;
  const int k1 = min(pos + 1, k0 + chunk);
  int n = k1 - k0;
  if (n > kAttnMaxChunk) {  // host sizes nsplit so this cannot happen; stay in bounds
    if (threadIdx.x == 0) atomicOr(a.ctrl + G4_CTRL_STATUS, G4_STATUS_MBAR_TIMEOUT);
    n = kAttnMaxChunk;
  }
  const size_t row_stride = (size_t)a.n_kv * D;

  // ---- 0. with all heads in one pass and registers to spare (G <= 4, G * CPL <= 4),
  // the first KB keys of every lane group go in flight now, under step 1: the cached
  // rows do not depend on it (only key `pos`, written below, does; it is patched from
  // shared memory before use)
  constexpr bool kEarly = G <= 4 && G * CPL <= 4;
  const int gi_lane = lane / LK, li = lane % LK;
  const int grp = warp * KPW + gi_lane;
  const bf16_t* kbase = a.cache_k + (size_t)hk * D;
  const bf16_t* vbase = a.cache_v + (size_t)hk * D;
  const int jstart = warp * KPW;  // warp-uniform
  uint4 kr[KB][CPL], vr[KB][CPL];
  auto load_keys = [&](int jw) {
#pragma unroll
    for (int m = 0; m < KB; ++m) {
      const int j = jw + gi_lane + m * NGRP;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        if (j < n) {
          kr[m][c] = ldcg_u4(kbase + (size_t)(k0 + j) * row_stride + (li + c * LK) * 8);
          vr[m][c] = ldcg_u4(vbase + (size_t)(k0 + j) * row_stride + (li + c * LK) * 8);
        } else {
          kr[m][c] = make_uint4(0, 0, 0, 0);
          vr[m][c] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  };
  if (kEarly) load_keys(jstart);

  // ---- 1. RoPE table of this position (cos / sin of pos * inv_freq, rounded to bf16
  // as the reference does, model.py:76-78): one sincosf per thread, shared by every
  // vector below.  Then the q heads (and the new k/v if this split holds pos): one
  // warp per vector.
  static_assert(D / 2 <= kAttnThreads, "one RoPE frequency per thread");
  if ((int)threadIdx.x < D / 2) {
    float sn, cs;
    sincosf((float)pos * fr, &sn, &cs);
    rope_s[threadIdx.x] = rbf(cs);
    rope_s[D / 2 + threadIdx.x] = rbf(sn);
  }
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
  for (int i = threadIdx.x; i < G * D; i += kAttnThreads) acc_s[i] = 0.f;
  __threadfence_block();
  named_bar(bar, kAttnThreads);
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 3);

  // ---- 2. online softmax per lane group over its keys
  const int jnew = has_new ? pos - k0 : -1;  // index of the new key in this slice
#pragma unroll 1
  for (int h0 = 0; h0 < G; h0 += HG) {
    uint4 qr[HG][CPL];
#pragma unroll
    for (int h = 0; h < HG; ++h)
#pragma unroll
      for (int c = 0; c < CPL; ++c) qr[h][c] = reinterpret_cast<const uint4*>(q_s + (h0 + h) * D)[li + c * LK];
    float m_run[HG], l_run[HG], acc[HG][CPL * 8];
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      m_run[h] = -INFINITY;
      l_run[h] = 0.f;
#pragma unroll
      for (int e = 0; e < CPL * 8; ++e) acc[h][e] = 0.f;
    }
    // The loop bound is warp-uniform (jw depends on the warp only): every lane of a
    // warp runs the same iterations, so the shuffles in group_sum always see a full
    // warp.  Lane group gi_lane takes keys jw + gi_lane + m*NGRP.
#pragma unroll 1
    for (int jw = jstart; jw < n; jw += NGRP * KB) {
      if (!kEarly || jw != jstart || h0 != 0) load_keys(jw);  // else already in flight
      const int j0 = jw + gi_lane;
#pragma unroll
      for (int m = 0; m < KB; ++m) {
        if (j0 + m * NGRP == jnew) {
#pragma unroll
          for (int c = 0; c < CPL; ++c) {
            kr[m][c] = reinterpret_cast<const uint4*>(kn_s)[li + c * LK];
            vr[m][c] = reinterpret_cast<const uint4*>(vn_s)[li + c * LK];
          }
        }
      }
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        float sc[KB];
        float mx = m_run[h];
#pragma unroll
        for (int m = 0; m < KB; ++m) {
          float s = 0.f;
#pragma unroll
          for (int c = 0; c < CPL; ++c) s = dot8(kr[m][c], qr[h][c], s);
          s = rbf(group_sum(s, LK));
          sc[m] = (j0 + m * NGRP < n) ? s : -INFINITY;
          mx = fmaxf(mx, sc[m]);
        }
        const float corr = mx == -INFINITY ? 1.f : expf(m_run[h] - mx);
        m_run[h] = mx;
        l_run[h] *= corr;
#pragma unroll
        for (int e = 0; e < CPL * 8; ++e) acc[h][e] *= corr;
#pragma unroll
        for (int m = 0; m < KB; ++m) {
          const float p = sc[m] == -INFINITY ? 0.f : expf(sc[m] - mx);
          l_run[h] += p;
#pragma unroll
          for (int c = 0; c < CPL; ++c) {
            const uint4 v = vr[m][c];
            float* o = &acc[h][c * 8];
            o[0] = fmaf(p, bf_lo(v.x), o[0]);
            o[1] = fmaf(p, bf_hi(v.x), o[1]);
            o[2] = fmaf(p, bf_lo(v.y), o[2]);
            o[3] = fmaf(p, bf_hi(v.y), o[3]);
            o[4] = fmaf(p, bf_lo(v.z), o[4]);
            o[5] = fmaf(p, bf_hi(v.z), o[5]);
            o[6] = fmaf(p, bf_lo(v.w), o[6]);
            o[7] = fmaf(p, bf_hi(v.w), o[7]);
          }
        }
      }
    }
    // ---- 3. merge lane groups: CTA max, then rescaled shared-memory sums
    if (li == 0) {
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        gm[grp * G + h0 + h] = m_run[h];
        gl[grp * G + h0 + h] = l_run[h];
      }
    }
    named_bar(bar, kAttnThreads);
    if (threadIdx.x < HG) {
      const int h = h0 + threadIdx.x;
      float M = -INFINITY;
      for (int q = 0; q < NGRP; ++q) M = fmaxf(M, gm[q * G + h]);
      float L = 0.f;
      for (int q = 0; q < NGRP; ++q) {
        const float mq = gm[q * G + h];
        L += mq == -INFINITY ? 0.f : gl[q * G + h] * expf(mq - M);
      }
      ml[h] = M;
      ml[kAttnMaxG + h] = L;
    }
    named_bar(bar, kAttnThreads);
    // rescale to the CTA max, sum the KPW lane groups of a warp with a butterfly (every
    // lane ends with the same bits), then add the warps into acc_s in warp order: a
    // fixed summation order, so results do not depend on scheduling
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      const float f = m_run[h] == -INFINITY ? 0.f : expf(m_run[h] - ml[h0 + h]);
#pragma unroll
      for (int e = 0; e < CPL * 8; ++e) acc[h][e] *= f;
    }
#pragma unroll
    for (int o = LK; o < 32; o <<= 1)
#pragma unroll
      for (int h = 0; h < HG; ++h)
#pragma unroll
        for (int e = 0; e < CPL * 8; ++e) acc[h][e] += __shfl_xor_sync(0xffffffffu, acc[h][e], o);
    if (kSlotMerge) {
      // every warp stores its sums in its own slot; then each thread adds the slots of
      // its elements in warp order, from 0 -- the same additions, in the same order, as
      // the warp-by-warp loop below, with one barrier instead of one per warp
      if (gi_lane == 0) {
#pragma unroll
        for (int h = 0; h < HG; ++h)
#pragma unroll
          for (int c = 0; c < CPL; ++c) {
            float4* dst = reinterpret_cast<float4*>(mslot + (warp * HG + h) * D + (li + c * LK) * 8);
            dst[0] = make_float4(acc[h][c * 8 + 0], acc[h][c * 8 + 1], acc[h][c * 8 + 2], acc[h][c * 8 + 3]);
            dst[1] = make_float4(acc[h][c * 8 + 4], acc[h][c * 8 + 5], acc[h][c * 8 + 6], acc[h][c * 8 + 7]);
          }
      }
      named_bar(bar, kAttnThreads);
      for (int i = threadIdx.x; i < HG * D; i += kAttnThreads) {
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < kAttnWarps; ++q) v += mslot[q * HG * D + i];
        acc_s[h0 * D + i] = v;
      }
      named_bar(bar, kAttnThreads);
    } else {
#pragma unroll 1
      for (int q = 0; q < kAttnWarps; ++q) {
        if (warp == q && gi_lane == 0) {
#pragma unroll
          for (int h = 0; h < HG; ++h)
#pragma unroll
            for (int e = 0; e < CPL * 8; ++e) acc_s[(h0 + h) * D + (li + (e / 8) * LK) * 8 + (e & 7)] += acc[h][e];
        }
        named_bar(bar, kAttnThreads);
      }
    }
  }

  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 4);
  // ---- 4. partials, then the last active CTA of this KV head merges them.  The
  // acq_rel counter update (after the block barrier) publishes this CTA's partials
  // and, for the last CTA, acquires every other CTA's.
  float* pbase = a.part + ((size_t)hk * a.nsplit + sp) * G * (D + 2);
  for (int i = threadIdx.x; i < G * (D + 2); i += kAttnThreads) {
    const int h = i / (D + 2), e = i % (D + 2);
    pbase[i] = e == 0 ? ml[h] : (e == 1 ? ml[kAttnMaxG + h] : acc_s[h * D + e - 2]);
  }
  named_bar(bar, kAttnThreads);
  if (threadIdx.x == 0) {
    const int old = atomic_add_acq_rel_gpu(a.counters + hk, 1);
    *flag = (old == n_active - 1);
  }
  named_bar(bar, kAttnThreads);
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 5);
  const bool merge = *flag != 0;
  named_bar(bar, kAttnThreads);  // every thread has read the flag before it is reused
  if (!merge) return;
  // One pass over the partials: each thread takes elements i = tid + 256 k of the
  // [G][D] context and, SB splits at a time (all their loads in flight together),
  // folds (m, l, acc) into a running max-rescaled sum in split order.
  constexpr int NE = (G * D + kAttnThreads - 1) / kAttnThreads;
  constexpr int SB = NE <= 2 ? 16 : (NE >= 32 ? 1 : 32 / NE);  // <= 96 values in flight
  const float* hbase = a.part + (size_t)hk * a.nsplit * G * (D + 2);
  float M[NE], L[NE], O[NE];
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    M[k] = -INFINITY;
    L[k] = 0.f;
    O[k] = 0.f;
  }
#pragma unroll 1
  for (int s0 = 0; s0 < n_active; s0 += SB) {
    float mv[NE][SB], lv[NE][SB], av[NE][SB];
#pragma unroll
    for (int k = 0; k < NE; ++k) {
      const int i = threadIdx.x + kAttnThreads * k;
      const int h = i / D, e = i % D;
#pragma unroll
      for (int q = 0; q < SB; ++q) {
        mv[k][q] = -INFINITY;
        lv[k][q] = 0.f;
        av[k][q] = 0.f;
        if (i < G * D && s0 + q < n_active) {
          const float* p = hbase + ((size_t)(s0 + q) * G + h) * (D + 2);
          mv[k][q] = ldcg_f(p);
          lv[k][q] = ldcg_f(p + 1);
          av[k][q] = ldcg_f(p + 2 + e);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < NE; ++k) {
      float mb = M[k];
#pragma unroll
      for (int q = 0; q < SB; ++q) mb = fmaxf(mb, mv[k][q]);
      const float cf = M[k] == -INFINITY ? 0.f : expf(M[k] - mb);
      L[k] *= cf;
      O[k] *= cf;
#pragma unroll
      for (int q = 0; q < SB; ++q) {
        const float f = mv[k][q] == -INFINITY ? 0.f : expf(mv[k][q] - mb);
        L[k] = fmaf(lv[k][q], f, L[k]);
        O[k] = fmaf(av[k][q], f, O[k]);
      }
      M[k] = mb;
    }
  }
#pragma unroll
  for (int k = 0; k < NE; ++k) {
    const int i = threadIdx.x + kAttnThreads * k;
    if (i < G * D) a.ctx[((size_t)hk * G + i / D) * D + i % D] = f2bf(O[k] / L[k]);
  }
  if (threadIdx.x == 0) {
    atomicExch(a.counters + hk, 0);
    G4_TRACE_EV(a.trace_id, 6);
  }
  named_bar(bar, kAttnThreads);  // shared scratch free for the caller's next use
}

// Standalone launch: grid = n_kv x nsplit, one item per CTA.
template <int D, int G>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(16) unsigned char attn_smem[];
  pdl_trigger();
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 0);
  pdl_wait();
  if (threadIdx.x == 0) G4_TRACE_EV(a.trace_id, 2);
  attn_item<D, G>(a, blockIdx.x / a.nsplit, blockIdx.x % a.nsplit, attn_smem, 1);
}

}  // namespace g4
