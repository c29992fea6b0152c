// Split-KV decode attention for one query token (reference: gemma4_tpu/model.py:195-213).
//
// Grid = n_kv (local KV heads) x nsplit.  CTA (h, s) owns a contiguous slice of the
// live key span of KV head h -- (pos-window, pos] for sliding layers, [0, pos] for
// full layers -- instead of the reference's masked pass over the whole max_len
// cache (the masked entries contribute exp(-1e30 - max) = 0 there, so skipping
// them is exact).  Per CTA:
//   1. q_norm RMSNorm + RoPE of the g query heads of KV head h (bf16 rounding points
//      of model.py:198 / 70-78); the CTA whose slice holds `pos` also normalises,
//      RoPEs and writes k (and v = rms(v_raw), or rms(k_raw) for k==v layers) into
//      the cache (model.py:200-206).
//   2. scores s = bf16(q.k) (scale 1.0, rounded to bf16 like the reference einsum)
//      for all g heads, held in shared memory; local max m and sum l per head.
//   3. acc = sum_j exp(s_j - m) v_j in fp32 (registers, then a shared-memory reduce).
//   4. (m, l, acc) to the partial buffer; the last CTA of head h (atomic counter)
//      merges the nsplit partials with the usual max-rescaling, divides by the total
//      mass and rounds the context to bf16.
// Difference from the reference: it rounds the normalised probabilities to bf16
// before P.V; here P.V uses fp32 unnormalised weights and the context is rounded
// once -- closer to exact arithmetic, within the tolerance the parity tests state.
#pragma once

#include "g4_common.cuh"

namespace g4 {

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxChunk = 1024;  // keys per CTA
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
};

__host__ __device__ inline int attn_smem_bytes(int g, int d) {
  // scores [g][kAttnMaxChunk] + acc [g][d] + merge scales [g][kAttnMaxSplit] + misc
  return g * kAttnMaxChunk * 4 + g * d * 4 + g * kAttnMaxSplit * 4 + 2 * kAttnMaxG * 4 + 64;
}

// Normalise (optionally with weight w) and optionally RoPE one vector of d elements
// held as lane-strided registers v[i] = x[lane + 32 i]; results rounded to bf16.
__device__ inline void warp_norm_rope(float* v, int d, const bf16_t* w, bool rope, int pos,
                                      const float* inv_freq, float eps) {
  const int lane = threadIdx.x & 31;
  const int per = d / 32;
  float ss = 0.f;
  for (int i = 0; i < per; ++i) ss += v[i] * v[i];
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)d + eps);
  for (int i = 0; i < per; ++i) {
    float o = v[i] * r;
    if (w) o = o * bf2f(w[lane + 32 * i]);
    v[i] = rbf(o);
  }
  if (!rope) return;
  const int half = per / 2;  // element lane+32i pairs with lane+32(i±half)
  float out[kAttnMaxD / 32];
  for (int i = 0; i < per; ++i) {
    const int e = lane + 32 * i;
    const int fi = e < d / 2 ? e : e - d / 2;
    const float ang = (float)pos * inv_freq[fi];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float rot = i < half ? -v[i + half] : v[i - half];
    out[i] = rbf(rbf(v[i] * rbf(cs)) + rbf(rot * rbf(sn)));
  }
  for (int i = 0; i < per; ++i) v[i] = out[i];
}

// CPL = 16-byte chunks of a head vector per lane: 1 for d <= 256, 2 for d = 512.
template <int CPL>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const __grid_constant__ AttnArgs a) {
  extern __shared__ __align__(16) unsigned char attn_smem[];
  float* sc = reinterpret_cast<float*>(attn_smem);                 // [g][kAttnMaxChunk]
  float* acc_s = sc + a.g * kAttnMaxChunk;                          // [g][d]
  float* scale_s = acc_s + a.g * a.d;                               // [g][kAttnMaxSplit]
  float* ml = scale_s + a.g * kAttnMaxSplit;                        // m[g], l[g]
  int* flag = reinterpret_cast<int*>(ml + 2 * kAttnMaxG);
  __shared__ __align__(16) bf16_t q_s[kAttnMaxG * kAttnMaxD];

  pdl_trigger();
  pdl_wait();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.x / a.nsplit, sp = blockIdx.x % a.nsplit;
  const int d = a.d, g = a.g, per = d / 32;
  const int pos = a.pos_fixed >= 0 ? a.pos_fixed : ldcg_i(a.ctrl + G4_CTRL_POS);
  const int start = a.window > 0 ? max(0, pos - a.window + 1) : 0;
  const int nlive = pos - start + 1;
  const int chunk = (nlive + a.nsplit - 1) / a.nsplit;
  const int k0 = start + sp * chunk;
  const int k1 = min(pos + 1, k0 + chunk);
  int n = max(0, k1 - k0);
  if (n > kAttnMaxChunk) {  // host sizes nsplit so this cannot happen; never overrun smem
    if (threadIdx.x == 0) atomicOr(a.ctrl + G4_CTRL_STATUS, G4_STATUS_MBAR_TIMEOUT);
    n = kAttnMaxChunk;
  }
  const size_t row_stride = (size_t)a.n_kv * d;
  const bf16_t* qraw = a.qkv;
  const bf16_t* kraw = a.qkv + (size_t)a.n_kv * g * d;
  const bf16_t* vraw = a.k_eq_v ? kraw : kraw + (size_t)a.n_kv * d;

  // ---- 1. q heads (and the new k/v if this split holds pos)
  const bool has_new = (pos >= k0 && pos < k1);
  const int nvec = g + (has_new ? 2 : 0);
  for (int vi = warp; vi < nvec; vi += kAttnWarps) {
    float v[kAttnMaxD / 32];
    const bf16_t* src;
    const bf16_t* w;
    bool rope;
    if (vi < g) {
      src = qraw + ((size_t)hk * g + vi) * d;
      w = a.q_norm;
      rope = true;
    } else if (vi == g) {
      src = kraw + (size_t)hk * d;
      w = a.k_norm;
      rope = true;
    } else {
      src = vraw + (size_t)hk * d;
      w = nullptr;
      rope = false;
    }
    for (int i = 0; i < per; ++i) v[i] = bf2f(ldcg_bf(src + lane + 32 * i));
    warp_norm_rope(v, d, w, rope, pos, a.inv_freq, a.eps);
    if (vi < g) {
      for (int i = 0; i < per; ++i) q_s[vi * d + lane + 32 * i] = f2bf(v[i]);
    } else {
      bf16_t* dst = (vi == g ? a.cache_k : a.cache_v) + (size_t)pos * row_stride + (size_t)hk * d;
      for (int i = 0; i < per; ++i) dst[lane + 32 * i] = f2bf(v[i]);
    }
  }
  for (int i = threadIdx.x; i < g * d; i += kAttnThreads) acc_s[i] = 0.f;
  __threadfence_block();
  __syncthreads();

  // ---- 2. scores
  const int LK = min(32, d / 8);   // lanes per key
  const int KPW = 32 / LK;         // keys per warp pass
  const int gi_lane = lane / LK, li = lane % LK;
  uint4 qr[kAttnMaxG][CPL];
#pragma unroll
  for (int h = 0; h < kAttnMaxG; ++h)
#pragma unroll
    for (int c = 0; c < CPL; ++c)
      if (h < g) qr[h][c] = reinterpret_cast<const uint4*>(q_s + h * d)[li + c * LK];
  const bf16_t* kbase = a.cache_k + (size_t)hk * d;
  for (int j0 = warp * KPW; j0 < n; j0 += kAttnWarps * KPW * 4) {
    uint4 kr[4][CPL];
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int j = j0 + m * kAttnWarps * KPW + gi_lane;
#pragma unroll
      for (int c = 0; c < CPL; ++c)
        if (j < n) kr[m][c] = ldcg_u4(kbase + (size_t)(k0 + j) * row_stride + (li + c * LK) * 8);
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int j = j0 + m * kAttnWarps * KPW + gi_lane;
#pragma unroll
      for (int h = 0; h < kAttnMaxG; ++h) {
        if (h >= g) break;
        float s = 0.f;
        if (j < n) {
#pragma unroll
          for (int c = 0; c < CPL; ++c) s = dot8(kr[m][c], qr[h][c], s);
        }
        s = group_sum(s, LK);
        if (li == 0 && j < n) sc[h * kAttnMaxChunk + j] = rbf(s);
      }
    }
  }
  __syncthreads();

  // ---- softmax statistics per head (one warp per head)
  for (int h = warp; h < g; h += kAttnWarps) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[h * kAttnMaxChunk + j]);
    m = warp_max(m);
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float p = expf(sc[h * kAttnMaxChunk + j] - m);
      sc[h * kAttnMaxChunk + j] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      ml[h] = m;
      ml[kAttnMaxG + h] = l;
    }
  }
  __syncthreads();

  // ---- 3. P.V, heads in groups so the accumulators stay in registers
  const bf16_t* vbase = a.cache_v + (size_t)hk * d;
  constexpr int HG = CPL == 1 ? kAttnMaxG : kAttnMaxG / 2;
  for (int h0 = 0; h0 < g; h0 += HG) {
    float acc[HG][CPL * 8];
#pragma unroll
    for (int h = 0; h < HG; ++h)
#pragma unroll
      for (int e = 0; e < CPL * 8; ++e) acc[h][e] = 0.f;
    for (int j0 = warp * KPW; j0 < n; j0 += kAttnWarps * KPW * 4) {
      uint4 vr[4][CPL];
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int j = j0 + m * kAttnWarps * KPW + gi_lane;
#pragma unroll
        for (int c = 0; c < CPL; ++c)
          if (j < n) vr[m][c] = ldcg_u4(vbase + (size_t)(k0 + j) * row_stride + (li + c * LK) * 8);
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int j = j0 + m * kAttnWarps * KPW + gi_lane;
        if (j >= n) continue;
#pragma unroll
        for (int h = 0; h < HG; ++h) {
          if (h0 + h >= g) break;
          const float p = sc[(h0 + h) * kAttnMaxChunk + j];
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
    // reduce over the key groups of the warp, then over warps (shared atomics)
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      if (h0 + h >= g) break;
#pragma unroll
      for (int e = 0; e < CPL * 8; ++e) {
        float v = acc[h][e];
        for (int o = LK; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (gi_lane == 0) {
          const int c = e / 8;
          atomicAdd(&acc_s[(h0 + h) * d + (li + c * LK) * 8 + (e & 7)], v);
        }
      }
    }
  }
  __syncthreads();

  // ---- 4. partials, then the last CTA of this KV head merges them
  float* pbase = a.part + ((size_t)hk * a.nsplit + sp) * g * (d + 2);
  for (int i = threadIdx.x; i < g * (d + 2); i += kAttnThreads) {
    const int h = i / (d + 2), e = i % (d + 2);
    float v;
    if (e == 0) v = n > 0 ? ml[h] : -INFINITY;
    else if (e == 1) v = n > 0 ? ml[kAttnMaxG + h] : 0.f;
    else v = acc_s[h * d + e - 2];
    pbase[i] = v;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomic_add_acq_rel_gpu(a.counters + hk, 1);
    *flag = (old == a.nsplit - 1);
  }
  __syncthreads();
  if (!*flag) return;
  __threadfence();
  const float* hbase = a.part + (size_t)hk * a.nsplit * g * (d + 2);
  for (int h = warp; h < g; h += kAttnWarps) {
    float M = -INFINITY;
    for (int s = lane; s < a.nsplit; s += 32) {
      const float* p = hbase + ((size_t)s * g + h) * (d + 2);
      if (ldcg_f(p + 1) > 0.f) M = fmaxf(M, ldcg_f(p));
    }
    M = warp_max(M);
    float L = 0.f;
    for (int s = lane; s < a.nsplit; s += 32) {
      const float* p = hbase + ((size_t)s * g + h) * (d + 2);
      const float l = ldcg_f(p + 1);
      const float f = l > 0.f ? expf(ldcg_f(p) - M) : 0.f;
      scale_s[h * kAttnMaxSplit + s] = f;
      L += l * f;
    }
    L = warp_sum(L);
    if (lane == 0) ml[h] = L;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < g * d; i += kAttnThreads) {
    const int h = i / d, e = i % d;
    float o = 0.f;
    for (int s = 0; s < a.nsplit; ++s) {
      const float f = scale_s[h * kAttnMaxSplit + s];
      if (f != 0.f) o = fmaf(ldcg_f(hbase + ((size_t)s * g + h) * (d + 2) + 2 + e), f, o);
    }
    a.ctx[((size_t)hk * g + h) * d + e] = f2bf(o / ml[h]);
  }
  if (threadIdx.x == 0) atomicExch(a.counters + hk, 0);
}

}  // namespace g4
