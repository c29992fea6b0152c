// Prompt prefill on the tensor cores: the reference's jitted prefill step
// (gemma4_tpu/engine.py:57-69), i.e. model.forward over the prompt with dense_moe=True and
// last_index = prompt_len - 1 (model.py:333-386), then the first token's sample.
//
// The prompt runs in chunks of up to `chunk` tokens through all layers (a chunk attends to
// the cache rows of every earlier chunk, so the result does not depend on the chunking).
// Every contraction is one tcgen05 GEMM (g4_gemm.cuh); the vector work between them --
// RMSNorms, RoPE, cache writes, the masked softmax, GELU gating, router softmax / top-k,
// the MLP || MoE combine -- is a row-parallel kernel here, with the reference's rounding
// points (every einsum output rounded to bf16 after fp32 accumulation, fp32 norms and
// softmax, bf16 probabilities, bf16 elementwise products):
//
//   x = embed[tok] * bf16(sqrt(H))                                   model.py:356-357
//   per layer:  xn = rms(x)*w_in; qkv = xn Wqkv^T                     :299, :197-199
//               q = rope(rms(q)*q_norm) ; k -> cache, v = rms(v) -> cache   :198-206
//               S_h = q_h K^T (bf16), band mask, fp32 softmax -> P_h (bf16)  :208-211
//               ctx_h = P_h V ; o = ctx Wo^T                          :212-213
//               x += rms(o)*w_pa ; MLP: down(gelu(gate)*up)           :300-310, :218-221
//               router: softmax, top-k, renorm, x per_expert_scale    :224-232
//               dense MoE: act[t,e,f] = gelu(g)*u*w[t,e] over ALL experts (w = 0 off
//               the top-k) ; out = sum_{e,f} act * down  (ONE GEMM, 3-D B)   :241-250
//               x = (x + rms(rms(mlp)*pf1 + rms(moe)*pf2)*pf) * layer_scalar  :312-322
//   last row:   rms(x)*norm ; logits = x E^T (bf16) ; softcap ; argmax / sample  :373-385
//
// Tensor-parallel prefill (world > 1) is not built: g4_prefill returns G4_ERR_SHAPE and
// the caller consumes the prompt with decode steps instead.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>

#include "g4_gemm.cuh"
#include "g4_internal.h"

namespace {

constexpr int kRowThreads = 256;
constexpr int kMaxRowElems = kMaxHidden / kRowThreads;  // per-thread elements of a hidden row

// ------------------------------------------------------------------ row helpers
// Sum of v over the block (kRowThreads threads), fixed order, identical on every thread.
__device__ __forceinline__ float row_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();  // earlier users of red are done
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kRowThreads / 32; ++i) s += red[i];
  return s;
}

// Elements h = threadIdx.x + 256 i of a bf16 row into registers (0 beyond n).
__device__ __forceinline__ void load_row(const bf16_t* src, int n, float (&v)[kMaxRowElems]) {
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    v[i] = h < n ? bf2f(src[h]) : 0.f;
  }
}

// 1 / sqrt(mean(v^2) + eps) of a register row (model.py:42-47, fp32).
__device__ __forceinline__ float row_rms(const float (&v)[kMaxRowElems], int n, float eps, float* red) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) ss += v[i] * v[i];
  return 1.0f / sqrtf(row_sum(ss, red) / (float)n + eps);
}

// ------------------------------------------------------------------ kernels
// x[t] = bf16(embed[token] * scale) for the chunk's tokens (model.py:356-357).
__global__ void pf_embed(const int* tokens, const bf16_t* embed, bf16_t* x, int H, int V, float scale, int* ctrl) {
  const int t = blockIdx.x;
  int tok = tokens[t];
  if (tok < 0 || tok >= V) {
    if (threadIdx.x == 0) atomicOr(ctrl + G4_CTRL_STATUS, G4_STATUS_BAD_TOKEN);
    tok = 0;
  }
  for (int h = threadIdx.x; h < H; h += blockDim.x)
    x[(size_t)t * H + h] = f2bf(bf2f(embed[(size_t)tok * H + h]) * scale);
}

// out[t] = bf16(rms(x[t]) * w)
__global__ void pf_rmsnorm(const bf16_t* x, const bf16_t* w, bf16_t* out, int H, float eps) {
  __shared__ float red[32];
  const size_t row = (size_t)blockIdx.x * H;
  float v[kMaxRowElems];
  load_row(x + row, H, v);
  const float r = row_rms(v, H, eps, red);
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    if (h < H) out[row + h] = f2bf((v[i] * r) * bf2f(w[h]));
  }
}

// q heads: rope(bf16(rms(q) * q_norm)) -> q buffer [T, nq * d]; k: the same with k_norm
// -> cache_k[pos]; v: bf16(rms(v_raw)) (k_raw on k==v layers) -> cache_v[pos]
// (model.py:197-206).  One warp per (token, vector); D / 32 elements per lane.
template <int D>
__global__ void pf_qk_rope(const bf16_t* qkv, int rows, bf16_t* qbuf, const bf16_t* q_norm, const bf16_t* k_norm,
                           bf16_t* cache_k, bf16_t* cache_v, const float* inv_freq, int nq, int n_kv, int k_eq_v,
                           int pos0, int M, float eps) {
  constexpr int PER = D / 32;
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int nvec = nq + 2 * n_kv;
  if (gw >= M * nvec) return;
  const int t = gw / nvec, vi = gw % nvec;
  const int pos = pos0 + t;
  const bf16_t* row = qkv + (size_t)t * rows;
  const bf16_t* src;
  int kind;  // 0 q, 1 k, 2 v
  if (vi < nq) {
    src = row + (size_t)vi * D;
    kind = 0;
  } else if (vi < nq + n_kv) {
    src = row + (size_t)nq * D + (size_t)(vi - nq) * D;
    kind = 1;
  } else {
    const int h = vi - nq - n_kv;
    src = k_eq_v ? row + (size_t)nq * D + (size_t)h * D : row + (size_t)(nq + n_kv) * D + (size_t)h * D;
    kind = 2;
  }
  float v[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    v[i] = bf2f(src[lane + 32 * i]);
    ss += v[i] * v[i];
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    float o = v[i] * r;
    if (kind == 0) o = o * bf2f(q_norm[lane + 32 * i]);
    else if (kind == 1) o = o * bf2f(k_norm[lane + 32 * i]);
    v[i] = rbf(o);
  }
  if (kind < 2) {  // rotate-half RoPE with bf16-rounded cos / sin (model.py:64-78)
    float out[PER];
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int f = (lane + 32 * i) % (D / 2);
      float sn, cs;
      sincosf((float)pos * inv_freq[f], &sn, &cs);
      const float rot = i < PER / 2 ? -v[i + PER / 2] : v[i - PER / 2];
      out[i] = rbf(rbf(v[i] * rbf(cs)) + rbf(rot * rbf(sn)));
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) v[i] = out[i];
  }
  bf16_t* dst;
  if (kind == 0) dst = qbuf + (size_t)t * nq * D + (size_t)vi * D;
  else if (kind == 1) dst = cache_k + ((size_t)pos * n_kv + (vi - nq)) * D;
  else dst = cache_v + ((size_t)pos * n_kv + (vi - nq - n_kv)) * D;
#pragma unroll
  for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = f2bf(v[i]);
}

// Vt[h][j][key - lo] = cache_v[key][h][j] for keys [lo, lo + span): V transposed so that
// the P.V product reads it K-major.  32 x 32 tiles through shared memory.
__global__ void pf_vtrans(const bf16_t* cache_v, bf16_t* vt, int lo, int span, int n_kv, int d, int ld) {
  __shared__ bf16_t tile[32][34];
  const int h = blockIdx.z;
  const int k0 = blockIdx.x * 32, j0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int key = k0 + r, j = j0 + threadIdx.x;
    tile[r][threadIdx.x] = key < span ? cache_v[((size_t)(lo + key) * n_kv + h) * d + j] : (bf16_t)0;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int j = j0 + r, key = k0 + threadIdx.x;
    if (key < span) vt[((size_t)h * d + j) * ld + key] = tile[threadIdx.x][r];
  }
}

// Masked softmax of one score row in place (model.py:209-211): keys at key_pos0 + j valid
// for query q = q_pos0 + m when key <= q and (window == 0 or key > q - window); fp32 softmax
// of the bf16 scores over the valid keys (a masked key's exp(-1e30 - max) is exactly 0),
// probabilities rounded to bf16; every column the P.V product reads for this row's tile
// ([j0, j1), the same band arithmetic as gemm_tile_range) gets a value, zero if masked.
__global__ void pf_softmax(bf16_t* sp, int M, int ld, int span, int q_pos0, int key_pos0, int window) {
  __shared__ float red[32];
  const int h = blockIdx.x / M, m = blockIdx.x % M;
  bf16_t* row = sp + ((size_t)h * M + m) * ld;
  const int q = q_pos0 + m;
  const int m0 = (m / kGemmBM) * kGemmBM;
  const int qlo = q_pos0 + m0, qhi = q_pos0 + min(m0 + kGemmBM, M) - 1;
  const int jlo = max((window > 0 ? qlo - window + 1 : 0) - key_pos0, 0);
  const int jhi = min(qhi - key_pos0 + 1, span);
  const int j0 = (jlo / kGemmBK) * kGemmBK, j1 = min((jhi + kGemmBK - 1) / kGemmBK * kGemmBK, span);
  const int vlo = max((window > 0 ? q - window + 1 : 0) - key_pos0, 0), vhi = min(q - key_pos0 + 1, span);
  float mx = -INFINITY;
  for (int j = vlo + threadIdx.x; j < vhi; j += blockDim.x) mx = fmaxf(mx, bf2f(row[j]));
  mx = warp_max(mx);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = -INFINITY;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) mx = fmaxf(mx, red[i]);
  float s = 0.f;
  for (int j = vlo + threadIdx.x; j < vhi; j += blockDim.x) s += expf(bf2f(row[j]) - mx);
  s = row_sum(s, red);
  for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
    const float p = (j >= vlo && j < vhi) ? expf(bf2f(row[j]) - mx) / s : 0.f;
    row[j] = f2bf(p);
  }
}

// After attention (model.py:300-316, one row per CTA): x = x + rms(o) * w_pa (the residual,
// in place); mlp_in = rms(x) * w_pff; h2 = rms(x) * w_pff2 (the MoE input); router input
// rin = rms(h2) * router.scale * bf16(H^-1/2), each product rounded to bf16 (:225-226).
__global__ void pf_post_attn(const bf16_t* o, bf16_t* x, const bf16_t* w_pa, const bf16_t* w_pff,
                             const bf16_t* w_pff2, const bf16_t* rscale, bf16_t* mlp_in, bf16_t* h2, bf16_t* rin,
                             int H, float eps, float hinv) {
  __shared__ float red[32];
  const size_t row = (size_t)blockIdx.x * H;
  float v[kMaxRowElems], t[kMaxRowElems];
  load_row(o + row, H, v);
  const float r = row_rms(v, H, eps, red);
  load_row(x + row, H, t);
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    t[i] = h < H ? rbf(t[i] + rbf((v[i] * r) * bf2f(w_pa[h]))) : 0.f;
    if (h < H) x[row + h] = f2bf(t[i]);
  }
  const float r2 = row_rms(t, H, eps, red);
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    if (h < H) {
      mlp_in[row + h] = f2bf((t[i] * r2) * bf2f(w_pff[h]));
      v[i] = rbf((t[i] * r2) * bf2f(w_pff2[h]));
      h2[row + h] = f2bf(v[i]);
    } else {
      v[i] = 0.f;
    }
  }
  const float r3 = row_rms(v, H, eps, red);
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    if (h < H) rin[row + h] = f2bf(rbf(rbf(v[i] * r3) * bf2f(rscale[h])) * hinv);
  }
}

// act = bf16(bf16(gelu(gate)) * up) (model.py:221)
__global__ void pf_gelu_mul(const bf16_t* gate, const bf16_t* up, bf16_t* act, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    act[i] = f2bf(rbf(gelu_tanh(bf2f(gate[i]))) * bf2f(up[i]));
}

// Router of one token (model.py:227-232): fp32 softmax of the bf16 logits, top-k by
// probability (ties to the lower expert), renormalised, times per_expert_scale -> the
// dense per-expert weight row (0 off the top-k, the one-hot einsum of :243-245).
// Expert e on thread e; sums in expert / rank order (the decode router's arithmetic).
__global__ void pf_router(const bf16_t* logits, const bf16_t* pes, float* wfull, int E, int K) {
  __shared__ float pv[256];
  __shared__ float top_p[kMaxTopK];
  const int t = threadIdx.x;
  const bf16_t* lrow = logits + (size_t)blockIdx.x * E;
  const float l = t < E ? bf2f(lrow[t]) : -INFINITY;
  if (t < E) pv[t] = l;
  __syncthreads();
  float mx = -INFINITY;
  for (int j = 0; j < E; ++j) mx = fmaxf(mx, pv[j]);
  const float ex = t < E ? expf(l - mx) : 0.f;
  __syncthreads();
  if (t < E) pv[t] = ex;
  __syncthreads();
  float sum = 0.f;
  for (int j = 0; j < E; ++j) sum += pv[j];
  const float p = ex / sum;
  __syncthreads();
  if (t < E) pv[t] = p;
  __syncthreads();
  int rank = 0;
  for (int j = 0; j < E; ++j) {
    const float q = pv[j];
    rank += (q > p || (q == p && j < t)) ? 1 : 0;
  }
  const bool sel = t < E && rank < K;
  if (sel) top_p[rank] = p;
  __syncthreads();
  if (t < E) {
    float w = 0.f;
    if (sel) {
      float wsum = 0.f;
      for (int k = 0; k < K; ++k) wsum += top_p[k];
      w = (p / wsum) * bf2f(pes[t]);
    }
    wfull[(size_t)blockIdx.x * E + t] = w;
  }
}

// Dense-MoE activation (model.py:246-248): act[t, e, f] = bf16(bf16(bf16(gelu(g)) * u) *
// bf16(w[t, e])) with g, u = gu[t, e, 0 / 1, f]; zero for experts off the top-k.
__global__ void pf_moe_act(const bf16_t* gu, const float* wfull, bf16_t* act, int M, int E, int F) {
  const size_t n = (size_t)M * E * F;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / ((size_t)E * F);
    const int e = (int)((i / F) % E), f = (int)(i % F);
    const float w = wfull[t * E + e];
    const bf16_t* g = gu + t * (size_t)E * 2 * F + (size_t)e * 2 * F;
    act[i] = w == 0.f ? (bf16_t)0 : f2bf(rbf(rbf(rbf(gelu_tanh(bf2f(g[f]))) * bf2f(g[F + f])) * rbf(w)));
  }
}

// ---- routed MoE: the dense einsums of model.py:241-250 restricted to the (token, expert)
// pairs with a nonzero routing weight.  An expert off a token's top-k has weight 0, so its
// activation is exactly 0 and its products add exactly 0 to the dense sum: computing only
// the routed pairs gives the dense result, up to the fp32 summation order of the down
// projection (per expert, then the experts in increasing order).
// Rows of the grouped buffers: expert e owns rows [z_rows[e], z_rows[e+1]), its tokens in
// increasing order (a stable counting sort, independent of scheduling).

// counts[e] = number of tokens routed to expert e (one CTA per expert).
__global__ void pf_route_count(const float* wfull, int M, int E, int* counts) {
  __shared__ float red[32];
  const int e = blockIdx.x;
  int c = 0;
  for (int t = threadIdx.x; t < M; t += blockDim.x) c += wfull[(size_t)t * E + e] != 0.f ? 1 : 0;
  const float s = row_sum((float)c, red);
  if (threadIdx.x == 0) counts[e] = (int)s;
}

// z_rows = exclusive prefix of counts (z_rows[E] = routed pairs).
__global__ void pf_route_scan(const int* counts, int E, int* z_rows) {
  if (threadIdx.x != 0) return;
  int acc = 0;
  for (int e = 0; e < E; ++e) {
    z_rows[e] = acc;
    acc += counts[e];
  }
  z_rows[E] = acc;
}

// Row of every routed (token, expert) pair: tokens of expert e in increasing order from
// z_rows[e]; rowmap[t][e] = that row or -1 (one CTA per expert, ordered block scan).
__global__ void pf_route_assign(const float* wfull, int M, int E, const int* z_rows, int* gather_tok,
                                float* gather_w, int* rowmap) {
  __shared__ int wcount[kRowThreads / 32];
  const int e = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int base = z_rows[e];
  for (int t0 = 0; t0 < M; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    const float wv = t < M ? wfull[(size_t)t * E + e] : 0.f;
    const bool member = wv != 0.f;
    const unsigned bal = __ballot_sync(0xffffffffu, member);
    if (lane == 0) wcount[warp] = __popc(bal);
    __syncthreads();
    int before = 0, total = 0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) {
      if (i < warp) before += wcount[i];
      total += wcount[i];
    }
    if (t < M) {
      if (member) {
        const int r = base + before + __popc(bal & ((1u << lane) - 1u));
        gather_tok[r] = t;
        gather_w[r] = wv;
        rowmap[(size_t)t * E + e] = r;
      } else {
        rowmap[(size_t)t * E + e] = -1;
      }
    }
    base += total;
    __syncthreads();  // wcount is rewritten by the next chunk
  }
}

// hg[r] = h2[gather_tok[r]] for the routed rows (one CTA per possible row).
__global__ void pf_gather_rows(const bf16_t* h2, const int* gather_tok, const int* z_rows, int E, int H, bf16_t* hg) {
  const int r = blockIdx.x;
  if (r >= z_rows[E]) return;
  const uint4* src = reinterpret_cast<const uint4*>(h2 + (size_t)gather_tok[r] * H);
  uint4* dst = reinterpret_cast<uint4*>(hg + (size_t)r * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) dst[i] = src[i];
}

// act[r, f] = bf16(bf16(bf16(gelu(g)) * u) * bf16(w_r)) of the routed rows (model.py:246-248).
__global__ void pf_routed_act(const bf16_t* gug, const float* gather_w, const int* z_rows, int E, int F,
                              bf16_t* act) {
  const size_t n = (size_t)z_rows[E] * F;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / F;
    const int f = (int)(i % F);
    const bf16_t* g = gug + r * 2 * F;
    act[i] = f2bf(rbf(rbf(rbf(gelu_tanh(bf2f(g[f]))) * bf2f(g[F + f])) * rbf(gather_w[r])));
  }
}

// moe[t] = bf16(sum over t's experts in increasing order of the fp32 down outputs).
__global__ void pf_routed_combine(const float* outg, const int* rowmap, int E, int H, bf16_t* moe,
                                  float* f32_out = nullptr, int ld = 0) {
  // launched with blockDim.x >= E (<= 1024): thread e reads expert e's row index, and the
  // token's routed rows are compacted in expert order (warp ballots, prefix over warps)
  __shared__ int rows[kMaxTopK * 2];
  __shared__ int wcount[32];
  __shared__ int nrows;
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = (int)threadIdx.x < E ? rowmap[(size_t)t * E + threadIdx.x] : -1;
  const unsigned b = __ballot_sync(0xffffffffu, r >= 0);
  if (lane == 0) wcount[warp] = __popc(b);
  __syncthreads();
  if (r >= 0) {
    int pos = __popc(b & ((1u << lane) - 1u));
    for (int w = 0; w < warp; ++w) pos += wcount[w];
    if (pos < kMaxTopK * 2) rows[pos] = r;
  }
  if (threadIdx.x == 0) {
    int n = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) n += wcount[w];
    nrows = min(n, kMaxTopK * 2);
  }
  __syncthreads();
  // columns split over gridDim.y blocks (short prompts: more blocks than tokens)
  for (int h = blockIdx.y * blockDim.x + threadIdx.x; h < H; h += gridDim.y * blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < nrows; ++i) acc += outg[(size_t)rows[i] * H + h];
    if (f32_out) f32_out[(size_t)t * ld + h] = acc;  // a rank's partial (tensor parallel)
    else moe[(size_t)t * H + h] = f2bf(acc);
  }
}

// ------------------------------------------------------------------ tensor-parallel exchange
// Every rank's communicator buffer ends with kMaxWorld 128-byte flag blocks (block src holds
// rank src's phase-1 flag at byte 0 and its phase-2 flag at byte 64: src has finished phase
// p of exchange `seq` when that flag >= seq) and two parity slots of kPfXRows x 2H fp32.
// A rank writes its partial into its OWN slot (earlier kernels of the stream); then
//   phase 1 (pf_xsum_rs, a reduce-scatter): it raises its phase-1 flag on every rank, waits
//     (bounded) for every rank's, and sums its share of the rows -- rows [q M / W, (q+1) M / W)
//     for rank q -- over all ranks' slots in rank order (peer loads over NVLink), writing
//     the fp32 sums back over those rows of its own slot;
//   phase 2 (pf_xsum_ag, an all-gather): it raises its phase-2 flag, waits for every rank's,
//     and reads each share's sums from its owner's slot, rounding them to bf16.
// Every rank gets the same bits, the sum order of a single all-ranks pass, and each rank
// moves ~2 (W-1)/W slots over NVLink instead of W-1.  Only the owner writes a share's rows,
// and no other rank reads them before the owner's phase-2 flag.  A slot is rewritten two
// exchanges later: by then every rank has passed the phase-1 wait of the exchange between,
// which its peers enter only after their phase-2 reads.
struct PfX {
  char* base[kMaxWorld];  // communicator buffer of every rank, mapped here
  size_t off;             // byte offset of the exchange region
  size_t slot_floats;     // floats per parity slot
  int rank, world;
};
__host__ __device__ __forceinline__ float* pfx_slot(const PfX& x, int r, int parity) {
  return reinterpret_cast<float*>(x.base[r] + x.off + (size_t)kMaxWorld * 128) + (size_t)parity * x.slot_floats;
}
__device__ __forceinline__ int* pfx_flag(const PfX& x, int r, int src, int phase) {
  return reinterpret_cast<int*>(x.base[r] + x.off + (size_t)src * 128 + (size_t)phase * 64);
}
// CTA 0 raises this rank's flag of `phase` on every rank; thread 0 of every CTA waits for
// all ranks'.
__device__ __forceinline__ bool pfx_arrive_wait(const PfX& x, int seq, int phase, int* ctrl) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < x.world; ++p) st_release_sys(pfx_flag(x, p, x.rank, phase), seq);
    }
    const int tmo = ldcg_i(ctrl + G4_CTRL_TIMEOUT_US);
    bool good = true;
    for (int src = 0; src < x.world && good; ++src)
      good = wait_flag_geq(pfx_flag(x, x.rank, src, phase), seq, tmo, ctrl + G4_CTRL_STATUS);
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}
__host__ __device__ __forceinline__ int pfx_share_row(int q, int rows, int world) {
  return (int)((long long)q * rows / world);
}
// Phase 1: this rank's share of the rows ([rows, cols] fp32 slots) summed over the ranks.
__global__ void pf_xsum_rs(PfX x, int seq, int parity, int rows, int cols, int* ctrl) {
  if (!pfx_arrive_wait(x, seq, 0, ctrl)) return;
  const size_t i0 = (size_t)pfx_share_row(x.rank, rows, x.world) * cols / 4;
  const size_t i1 = (size_t)pfx_share_row(x.rank + 1, rows, x.world) * cols / 4;
  float4* own = reinterpret_cast<float4*>(pfx_slot(x, x.rank, parity));
  for (size_t i = i0 + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < i1; i += (size_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int src = 0; src < x.world; ++src) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(pfx_slot(x, src, parity)) + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    own[i] = s;
  }
}
// Phase 2: out0 / out1 [rows, H] = bf16 of the summed columns [0, H) / [H, 2H), each row
// read from the slot of the rank whose share it is.
__global__ void pf_xsum_ag(PfX x, int seq, int parity, int rows, int cols, int H, bf16_t* out0, bf16_t* out1,
                           int* ctrl) {
  if (!pfx_arrive_wait(x, seq, 1, ctrl)) return;
  const size_t n4 = (size_t)rows * cols / 4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = (4 * i) / cols, c = (4 * i) % cols;
    int q = (int)((long long)r * x.world / rows);  // the share holding row r
    while (q + 1 < x.world && pfx_share_row(q + 1, rows, x.world) <= (int)r) ++q;
    while (q > 0 && pfx_share_row(q, rows, x.world) > (int)r) --q;
    const float4 s = __ldcg(reinterpret_cast<const float4*>(pfx_slot(x, q, parity)) + i);
    bf16_t* dst = c < (size_t)H ? out0 + r * H + c : out1 + r * H + (c - H);
    uint2 w;
    w.x = (uint32_t)f2bf(s.x) | ((uint32_t)f2bf(s.y) << 16);
    w.y = (uint32_t)f2bf(s.z) | ((uint32_t)f2bf(s.w) << 16);
    *reinterpret_cast<uint2*>(dst) = w;
  }
}
// Two ranks: one pass (phase-1 flags only) in which each rank sums every row of both slots
// -- the same bytes over NVLink as the two phases, one wait fewer.
__global__ void pf_xsum_pair(PfX x, int seq, int parity, int rows, int cols, int H, bf16_t* out0, bf16_t* out1,
                             int* ctrl) {
  if (!pfx_arrive_wait(x, seq, 0, ctrl)) return;
  const size_t n4 = (size_t)rows * cols / 4;
  const float4* s0 = reinterpret_cast<const float4*>(pfx_slot(x, 0, parity));
  const float4* s1 = reinterpret_cast<const float4*>(pfx_slot(x, 1, parity));
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 a = __ldcg(s0 + i), b = __ldcg(s1 + i);
    // 0 + a + b: the order of the two-phase sum
    const float4 s = make_float4((0.f + a.x) + b.x, (0.f + a.y) + b.y, (0.f + a.z) + b.z, (0.f + a.w) + b.w);
    const size_t r = (4 * i) / cols, c = (4 * i) % cols;
    bf16_t* dst = c < (size_t)H ? out0 + r * H + c : out1 + r * H + (c - H);
    uint2 w;
    w.x = (uint32_t)f2bf(s.x) | ((uint32_t)f2bf(s.y) << 16);
    w.y = (uint32_t)f2bf(s.z) | ((uint32_t)f2bf(s.w) << 16);
    *reinterpret_cast<uint2*>(dst) = w;
  }
}
// The exchange of one [rows, cols] partial into out0 / out1: one pass at two ranks, else
// phase 1 then phase 2.
static int pf_xsum(const PfX& x, int seq, int parity, int rows, int cols, int H, bf16_t* out0, bf16_t* out1,
                   int* ctrl, int grid, cudaStream_t st) {
  if (x.world == 2) {
    pf_xsum_pair<<<std::max(1, grid), 256, 0, st>>>(x, seq, parity, rows, cols, H, out0, out1, ctrl);
  } else {
    pf_xsum_rs<<<std::max(1, grid / x.world), 256, 0, st>>>(x, seq, parity, rows, cols, ctrl);
    pf_xsum_ag<<<std::max(1, grid), 256, 0, st>>>(x, seq, parity, rows, cols, H, out0, out1, ctrl);
  }
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  return G4_OK;
}
// The prompt's first token: the best (value, index) pair over the ranks' vocab slices
// (ties: lower index), then the position and the step counter, as a decode step leaves them.
__global__ void pf_xargmax(PfX x, int seq, int parity, int* tok_out, int out_index, int* tokens_host, int* ctrl,
                           int n) {
  if (!pfx_arrive_wait(x, seq, 0, ctrl)) return;
  if (threadIdx.x != 0) return;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int src = 0; src < x.world; ++src) {
    const float* pr = pfx_slot(x, src, parity);
    const float v = __ldcg(pr);
    const int idx = __float_as_int(__ldcg(pr + 1));
    if (v > best || (v == best && idx < bidx)) {
      best = v;
      bidx = idx;
    }
  }
  const int token = bidx == 0x7fffffff ? 0 : bidx;
  tok_out[out_index] = token;
  if (tokens_host) tokens_host[out_index] = token;
  ctrl[G4_CTRL_POS] = n;
  ctrl[G4_CTRL_STEP] = ldcg_i(ctrl + G4_CTRL_STEP) + 1;  // the sampler's and later steps' exchange uses
}

// Layer output (model.py:312-322, one row per CTA): h1 = rms(mlp)*pf1, h2 = rms(moe)*pf2,
// h = rms(h1 + h2)*pf, x = (resid + h) * layer_scalar.
__global__ void pf_combine(const bf16_t* mlp, const bf16_t* moe, bf16_t* x, const bf16_t* pf1, const bf16_t* pf2,
                           const bf16_t* pf, const bf16_t* scalar, int H, float eps) {
  __shared__ float red[32];
  const size_t row = (size_t)blockIdx.x * H;
  float a[kMaxRowElems], b[kMaxRowElems];
  load_row(mlp + row, H, a);
  load_row(moe + row, H, b);
  const float r1 = row_rms(a, H, eps, red), r2 = row_rms(b, H, eps, red);
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    a[i] = h < H ? rbf(rbf((a[i] * r1) * bf2f(pf1[h])) + rbf((b[i] * r2) * bf2f(pf2[h]))) : 0.f;
  }
  const float r3 = row_rms(a, H, eps, red);
  const float sc = bf2f(scalar[0]);
#pragma unroll
  for (int i = 0; i < kMaxRowElems; ++i) {
    const int h = threadIdx.x + kRowThreads * i;
    if (h < H) x[row + h] = f2bf(rbf(rbf(bf2f(x[row + h]) + rbf((a[i] * r3) * bf2f(pf[h]))) * sc));
  }
}

// LM-head epilogue of a row (model.py:381-385 + the greedy branch of :414-424):
// softcapped fp32 logits of this rank's vocab slice, first index of the maximum ->
// tok_out[out_index]; control POS = n.  One CTA per row: row r reads lg + r * V, writes
// logits + r * V, tok_out[out_index + r] and ctrl + r * ctrl_stride (n + r * n_stride).
__global__ void pf_lm_epilogue(const bf16_t* lg, float* logits, int V, int vbegin, float softcap, int* tok_out,
                               int out_index, int* tokens_host, int* ctrl, int n, int ctrl_stride = 0,
                               int n_stride = 0, float* xpair = nullptr) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int row = blockIdx.x;
  lg += (size_t)row * V;
  logits += (size_t)row * V;
  ctrl += (size_t)row * ctrl_stride;
  out_index += row;
  if (n >= 0) n += row * n_stride;
  float best = -INFINITY;
  int bidx = 0x7fffffff;
  for (int u = threadIdx.x; u < V; u += blockDim.x) {
    float v = bf2f(lg[u]);
    if (softcap > 0.f) v = tanhf(v / softcap) * softcap;
    logits[u] = v;
    if (v > best) {  // increasing u per thread: ties keep the lower index
      best = v;
      bidx = u;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bidx, o);
    if (ov > best || (ov == best && oi < bidx)) {
      best = ov;
      bidx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = bidx;
  }
  __syncthreads();
  if (threadIdx.x != 0) return;
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
    if (bv[w] > best || (bv[w] == best && bi[w] < bidx)) {
      best = bv[w];
      bidx = bi[w];
    }
  const int token = bidx == 0x7fffffff ? 0 : vbegin + bidx;
  if (xpair) {  // tensor parallel: this rank's best of its vocab slice, for pf_xargmax
    xpair[0] = best;
    xpair[1] = __int_as_float(token);
    return;
  }
  tok_out[out_index] = token;
  if (tokens_host) tokens_host[out_index] = token;
  ctrl[G4_CTRL_POS] = n >= 0 ? n : ctrl[G4_CTRL_POS] + 1;  // n < 0: a decode step advances
}

// ------------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// A K-major bf16 matrix [rows, inner] (row stride `ld` elements) read in boxes of 64
// elements x box_rows rows with 128-byte swizzle; out-of-range elements read as zero.
int make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (ld * 2) % 16)
    return fail(G4_ERR_ARG, "tensor map: base or row stride not 16-byte aligned");
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kGemmBK, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled (2-D) failed: %d", (int)r);
  return G4_OK;
}

// A bf16 tensor [slabs, rows, inner] read in boxes of 64 x box_rows x 1.
int make_map_3d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t slabs, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (inner * 2) % 16)
    return fail(G4_ERR_ARG, "tensor map: base or row stride not 16-byte aligned");
  const cuuint64_t dims[3] = {inner, rows, slabs};
  const cuuint64_t strides[2] = {inner * 2, inner * rows * 2};
  const cuuint32_t box[3] = {(cuuint32_t)kGemmBK, box_rows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(G4_ERR_CUDA, "cuTensorMapEncodeTiled (3-D) failed: %d", (int)r);
  return G4_OK;
}

// ------------------------------------------------------------------ GEMM launches
struct Operand {
  const void* p;
  uint64_t inner, rows, ld;  // 2-D [rows, inner], row stride ld (elements)
  uint64_t slabs = 0;        // > 0: 3-D [slabs, rows, inner], dense
};

int gemm_prepare(int bn) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, bool> done;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done[{dev, bn}]) return G4_OK;
  const void* ks[2] = {bn == 256 ? reinterpret_cast<const void*>(gemm_kernel<256>)
                                 : reinterpret_cast<const void*>(gemm_kernel<128>),
                       bn == 256 ? reinterpret_cast<const void*>(gemm_persistent_kernel<256>)
                                 : reinterpret_cast<const void*>(gemm_persistent_kernel<128>)};
  for (const void* k : ks)
    G4_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes(bn)),
            G4_ERR_LAUNCH);
  done[{dev, bn}] = true;
  return G4_OK;
}

// The persistent GEMM (one CTA per SM, double-buffered TMEM accumulators) is the default;
// G4_GEMM_TILES=1 launches one CTA per output tile instead (kept for A/B measurement).
bool gemm_tiles_mode() {
  static const bool v = [] {
    const char* e = getenv("G4_GEMM_TILES");
    return e && e[0] == '1';
  }();
  return v;
}

// out[m, n] = sum over the splits of part[s][m][n] (fixed order), as fp32 or bf16.
__global__ void pf_split_reduce(const float* part, int S, int M, int N, void* out, long long ldc, int out_f32) {
  const size_t n = (size_t)M * N;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < S; ++s) acc += part[(size_t)s * n + i];
    const size_t r = i / N, c = i % N;
    if (out_f32) static_cast<float*>(out)[r * ldc + c] = acc;
    else static_cast<bf16_t*>(out)[r * ldc + c] = f2bf(acc);
  }
}

// Split-K scratch: fp32 partial sums of GEMMs whose tiles alone cannot fill the GPU
// (few output tiles: short prompts, narrow outputs).  Set by the prefill for its calls.
struct SplitBuf {
  float* p = nullptr;
  size_t elems = 0;
};

// C[z] (M x N) = A[z] (M x K) . B[z] (N x K)^T; `g` carries the shape, output and offsets.
// A plain (un-batched, un-banded) GEMM with fewer output tiles than SMs is split along K
// into fp32 partials in `sb` and summed by pf_split_reduce.
int gemm(const Operand& A, const Operand& B, GemmArgs g, int Z, cudaStream_t st, SplitBuf sb = SplitBuf{}) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0 || Z <= 0) return G4_OK;
  if (!g.zb_div) g.zb_div = 1;
  // 128-wide tiles for narrow outputs only (measured: the batched decode's routed-expert
  // GEMMs ran slower with them, 11.9 vs 11.4 ms per step, despite the finer tile count)
  const int bn = g.N <= 128 ? 128 : 256;
  int rc = gemm_prepare(bn);
  if (rc) return rc;
  int nsm = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const long long tiles = (long long)((g.N + bn - 1) / bn) * ((g.M + kGemmBM - 1) / kGemmBM) * Z;
  const int nkb = g.b_kpe > 0 ? g.K / kGemmBK : (g.K + kGemmBK - 1) / kGemmBK;
  int S = 1;
  if (sb.p && Z == 1 && !g.band && !g.z_rows && tiles < nsm && g.ldc == g.N) {
    S = (int)std::min<long long>((2LL * nsm + tiles - 1) / tiles, nkb / 2);
    S = (int)std::min<long long>(S, (long long)(sb.elems / ((size_t)g.M * g.N)));
  }
  void* out = g.C;
  const int out_f32 = g.c_f32;
  if (S >= 2) {
    g.ksplit = S;
    g.split_stride = (long long)g.M * g.N;
    g.C = sb.p;
  } else {
    S = 1;
  }
  GemmParams P;
  memset(&P, 0, sizeof(P));
  if ((rc = make_map_2d(&P.ta, A.p, A.inner, A.rows, A.ld, kGemmBM))) return rc;
  if (B.slabs) rc = make_map_3d(&P.tb, B.p, B.inner, B.rows, B.slabs, bn);
  else rc = make_map_2d(&P.tb, B.p, B.inner, B.rows, B.ld, bn);
  if (rc) return rc;
  g.nz = Z;
  P.a = g;
  if (gemm_tiles_mode()) {
    const dim3 grid((g.N + bn - 1) / bn, (g.M + kGemmBM - 1) / kGemmBM, Z * S);
    if (bn == 256)
      gemm_kernel<256><<<grid, kGemmThreads, gemm_smem_bytes(256), st>>>(P);
    else
      gemm_kernel<128><<<grid, kGemmThreads, gemm_smem_bytes(128), st>>>(P);
  } else {
    const long long all = (long long)((g.N + bn - 1) / bn) * ((g.M + kGemmBM - 1) / kGemmBM) * Z * S;
    const dim3 grid((unsigned)std::min<long long>(all, nsm));
    if (bn == 256)
      gemm_persistent_kernel<256><<<grid, kGemmThreads, gemm_smem_bytes(256), st>>>(P);
    else
      gemm_persistent_kernel<128><<<grid, kGemmThreads, gemm_smem_bytes(128), st>>>(P);
  }
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  if (S > 1) {
    const size_t n = (size_t)g.M * g.N;
    pf_split_reduce<<<(unsigned)std::min<size_t>(4096, (n + 255) / 256), 256, 0, st>>>(sb.p, S, g.M, g.N, out,
                                                                                       g.ldc, out_f32);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  }
  return G4_OK;
}

GemmArgs plain(int M, int N, int K, void* C, long long ldc, int* status) {
  GemmArgs g{};
  g.M = M;
  g.N = N;
  g.K = K;
  g.C = C;
  g.ldc = ldc;
  g.zb_div = 1;
  g.status = status;
  return g;
}

size_t up256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

// ------------------------------------------------------------------ workspace
struct PrefillWs {
  int chunk = 0, ks = 0;  // tokens per chunk; padded key capacity (row stride of scores)
  char* base = nullptr;
  bf16_t *x, *xn, *qkv, *q, *sp, *vt, *ctx, *o, *mlp_in, *h2, *rin, *gate, *up, *act, *mlp_out, *rlog, *gu, *mact,
      *moe_out, *xf, *lmlog;
  float* wfull;
  float* split;  // split-K partial sums
  size_t split_elems;
  // routed MoE: per-expert row ranges, the routed rows' token / weight, token x expert row map
  int *counts, *z_rows, *gather_tok, *rowmap;
  float *gather_w, *outg;
  bf16_t *hg, *gug, *actg;
};

constexpr size_t kSplitElems = (size_t)16 << 20;  // 64 MB of fp32 split-K partials

void g4_prefill_release(g4_model* m) {
  if (!m || !m->prefill) return;
  if (m->prefill->base) cudaFree(m->prefill->base);
  delete m->prefill;
  m->prefill = nullptr;
}

static int prefill_workspace(g4_model* m, int chunk) {
  if (m->prefill && m->prefill->chunk >= chunk) return G4_OK;
  g4_prefill_release(m);
  const int H = m->H, E = m->E, F = m->F_local, I = m->I_local;
  size_t rmax = 0, qmax = 0, nqmax = 0, vtmax = 0;
  for (const LayerDev& l : m->L) {
    rmax = std::max(rmax, (size_t)(l.rows_q + l.rows_k + l.rows_v));
    qmax = std::max(qmax, (size_t)l.rows_q);
    nqmax = std::max(nqmax, (size_t)(l.n_kv * l.g));
    vtmax = std::max(vtmax, (size_t)l.n_kv * l.d);
  }
  const size_t ks = ((size_t)m->max_len + 63) / 64 * 64;
  const size_t C = chunk;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += up256(bytes);
    return o;
  };
  const size_t o_x = take(C * H * 2), o_xn = take(C * H * 2), o_qkv = take(C * rmax * 2), o_q = take(C * qmax * 2),
               o_sp = take(nqmax * C * ks * 2), o_vt = take(vtmax * ks * 2), o_ctx = take(C * qmax * 2),
               o_o = take(C * H * 2), o_mi = take(C * H * 2), o_h2 = take(C * H * 2), o_rin = take(C * H * 2),
               o_g = take(C * I * 2), o_u = take(C * I * 2), o_a = take(C * I * 2), o_mo = take(C * H * 2),
               o_rl = take(C * E * 2), o_wf = take(C * E * 4), o_gu = take(C * (size_t)E * 2 * F * 2),
               o_ma = take(C * (size_t)E * F * 2), o_moe = take(C * H * 2), o_xf = take((size_t)H * 2),
               o_lm = take((size_t)m->V_local * 2), o_split = take(kSplitElems * 4);
  const size_t CK = C * (size_t)m->topk;
  const size_t o_cnt = take((size_t)E * 4), o_zr = take((size_t)(E + 1) * 4), o_gt = take(CK * 4),
               o_rm = take(C * (size_t)E * 4), o_gw = take(CK * 4), o_og = take(CK * H * 4), o_hg = take(CK * H * 2),
               o_gug = take(CK * 2 * F * 2), o_ag = take(CK * F * 2);
  PrefillWs* w = new PrefillWs();
  if (cudaMalloc(&w->base, off) != cudaSuccess) {
    delete w;
    return fail(G4_ERR_NOMEM, "prefill workspace cudaMalloc(%zu) failed", off);
  }
  char* b = w->base;
  w->chunk = chunk;
  w->ks = (int)ks;
  w->x = (bf16_t*)(b + o_x);
  w->xn = (bf16_t*)(b + o_xn);
  w->qkv = (bf16_t*)(b + o_qkv);
  w->q = (bf16_t*)(b + o_q);
  w->sp = (bf16_t*)(b + o_sp);
  w->vt = (bf16_t*)(b + o_vt);
  w->ctx = (bf16_t*)(b + o_ctx);
  w->o = (bf16_t*)(b + o_o);
  w->mlp_in = (bf16_t*)(b + o_mi);
  w->h2 = (bf16_t*)(b + o_h2);
  w->rin = (bf16_t*)(b + o_rin);
  w->gate = (bf16_t*)(b + o_g);
  w->up = (bf16_t*)(b + o_u);
  w->act = (bf16_t*)(b + o_a);
  w->mlp_out = (bf16_t*)(b + o_mo);
  w->rlog = (bf16_t*)(b + o_rl);
  w->wfull = (float*)(b + o_wf);
  w->gu = (bf16_t*)(b + o_gu);
  w->mact = (bf16_t*)(b + o_ma);
  w->moe_out = (bf16_t*)(b + o_moe);
  w->xf = (bf16_t*)(b + o_xf);
  w->lmlog = (bf16_t*)(b + o_lm);
  w->split = (float*)(b + o_split);
  w->split_elems = kSplitElems;
  w->counts = (int*)(b + o_cnt);
  w->z_rows = (int*)(b + o_zr);
  w->gather_tok = (int*)(b + o_gt);
  w->rowmap = (int*)(b + o_rm);
  w->gather_w = (float*)(b + o_gw);
  w->outg = (float*)(b + o_og);
  w->hg = (bf16_t*)(b + o_hg);
  w->gug = (bf16_t*)(b + o_gug);
  w->actg = (bf16_t*)(b + o_ag);
  m->prefill = w;
  return G4_OK;
}

static int launch_qk_rope(const LayerDev& l, const bf16_t* qkv, bf16_t* q, bf16_t* ck, bf16_t* cv, const float* inv,
                          int pos0, int M, float eps, cudaStream_t st) {
  const int nq = l.n_kv * l.g, rows = l.rows_q + l.rows_k + l.rows_v;
  const long long warps = (long long)M * (nq + 2 * l.n_kv);
  const dim3 grid((unsigned)((warps + 7) / 8));
#define G4_QK(D)                                                                                          \
  pf_qk_rope<D><<<grid, 256, 0, st>>>(qkv, rows, q, l.q_norm, l.k_norm, ck, cv, inv, nq, l.n_kv, l.k_eq_v, \
                                      pos0, M, eps)
  switch (l.d) {
    case 64: G4_QK(64); break;
    case 128: G4_QK(128); break;
    case 256: G4_QK(256); break;
    case 512: G4_QK(512); break;
    default: return fail(G4_ERR_SHAPE, "prefill: head_dim %d", l.d);
  }
#undef G4_QK
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  return G4_OK;
}

// Routed MoE of the chunk's M tokens (see pf_route_count): routing tables, the gathered
// MoE inputs, one grouped GEMM per projection (entry e = expert e: its rows, its weights),
// the activation, and the per-token sum of the routed experts' outputs.
// `f32_out` (tensor parallel): the per-token sums go there as this rank's fp32 partial
// (row stride `ld`) instead of to moe_out.
static int routed_moe(g4_model* m, const LayerDev& l, int M, int* status, cudaStream_t st,
                      float* f32_out = nullptr, int ld = 0) {
  PrefillWs& w = *m->prefill;
  const int H = m->H, E = m->E, F = m->F_local, MK = M * m->topk;
  int rc;
  pf_route_count<<<E, kRowThreads, 0, st>>>(w.wfull, M, E, w.counts);
  pf_route_scan<<<1, 32, 0, st>>>(w.counts, E, w.z_rows);
  pf_route_assign<<<E, kRowThreads, 0, st>>>(w.wfull, M, E, w.z_rows, w.gather_tok, w.gather_w, w.rowmap);
  pf_gather_rows<<<MK, 128, 0, st>>>(w.h2, w.gather_tok, w.z_rows, E, H, w.hg);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  {  // gate|up of every routed row: entry e reads expert e's [2F, H] rows
    GemmArgs g = plain(M, 2 * F, H, w.gug, 2 * F, status);
    g.zb_row = 2 * F;
    g.z_rows = w.z_rows;
    if ((rc = gemm({w.hg, (uint64_t)H, (uint64_t)MK, (uint64_t)H},
                   {l.exp_gu, (uint64_t)H, (uint64_t)E * 2 * F, (uint64_t)H}, g, E, st)))
      return rc;
  }
  pf_routed_act<<<std::min(8192, (MK * F + 255) / 256), 256, 0, st>>>(w.gug, w.gather_w, w.z_rows, E, F, w.actg);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  {  // down of every routed row (fp32): entry e reads expert e's [H, F] rows
    GemmArgs g = plain(M, H, F, w.outg, H, status);
    g.c_f32 = 1;
    g.zb_row = H;
    g.z_rows = w.z_rows;
    if ((rc = gemm({w.actg, (uint64_t)F, (uint64_t)MK, (uint64_t)F},
                   {l.exp_down, (uint64_t)F, (uint64_t)E * H, (uint64_t)F}, g, E, st)))
      return rc;
  }
  if (E > 256) return fail(G4_ERR_SHAPE, "prefill: %d experts (at most 256)", E);
  pf_routed_combine<<<dim3(M, M < 512 ? (H + 255) / 256 : 1), 256, 0, st>>>(w.outg, w.rowmap, E, H, w.moe_out,
                                                                           f32_out, ld);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  return G4_OK;
}

// Where a prefill reads its tokens and writes its caches and first token: the model's own
// sequence, or one sequence of the batched decoder.
struct PfTarget {
  const int* tokens;                   // prompt tokens [n]
  bf16_t* const* ck;                   // per layer: K / V cache [cache_len, kv, d]
  bf16_t* const* cv;
  int cache_len;
  int* tok_out;                        // the first generated token goes to tok_out[out_index]
  int out_index;
  int* tok_host;                       // optional mapped host mirror of tok_out
  int* ctrl;                           // control block (POS = n, STATUS)
  float* logits;                       // fp32 softcapped logits of the last position
};

// One chunk of `M` prompt tokens at positions [c0, c0 + M) through every layer; `dense`
// runs the MoE over all experts (the reference's prefill as written), else routed.
static int prefill_chunk(g4_model* m, int c0, int M, bool last, int n_total, bool dense, cudaStream_t st,
                         const PfTarget& tg) {
  PrefillWs& w = *m->prefill;
  const SplitBuf sb{w.split, w.split_elems};
  const g4_config& c = m->cfg;
  const int H = m->H, E = m->E, F = m->F_local, I = m->I_local, K = m->topk;
  const float eps = c.rms_norm_eps;
  int* status = tg.ctrl + G4_CTRL_STATUS;
  int rc;
  // tensor parallel: the two all-reduces of every layer and the LM head's argmax go through
  // the communicators' prefill exchange (this rank's partial into its own slot)
  const bool tp = m->world > 1;
  PfX px{};
  if (tp) {
    for (int p = 0; p < kMaxWorld; ++p) px.base[p] = m->comm->peer[p];
    px.off = g4_comm_pf_offset(m->comm->hidden);
    px.slot_floats = (size_t)kPfXRows * 2 * m->comm->hidden;
    px.rank = m->rank;
    px.world = m->world;
  }
  auto xnext = [&](int& seq, int& par) {
    seq = ++m->comm->pf_seq;
    par = seq & 1;
  };
  const int xgrid = std::min(4 * m->nsm, (int)(((size_t)M * 2 * H / 4 + 255) / 256));
  pf_embed<<<M, 256, 0, st>>>(tg.tokens + c0, m->embed, w.x, H, c.vocab_size,
                              g4_host_bf16_round(std::sqrt((float)H)), tg.ctrl);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  const float hinv = g4_host_bf16_round(std::pow((float)H, -0.5f));
  for (size_t li = 0; li < m->L.size(); ++li) {
    const LayerDev& l = m->L[li];
    const AttnArgs& aa = m->k2[li];
    const int nq = l.n_kv * l.g, d = l.d, R = l.rows_q + l.rows_k + l.rows_v;
    // ---- attention (model.py:195-213)
    pf_rmsnorm<<<M, kRowThreads, 0, st>>>(w.x, l.n_in, w.xn, H, eps);
    if ((rc = gemm({w.xn, (uint64_t)H, (uint64_t)M, (uint64_t)H}, {l.qkv, (uint64_t)H, (uint64_t)R, (uint64_t)H},
                   plain(M, R, H, w.qkv, R, status), 1, st, sb)))
      return rc;
    if ((rc = launch_qk_rope(l, w.qkv, w.q, tg.ck[li], tg.cv[li], aa.inv_freq, c0, M, eps, st))) return rc;
    const int window = l.full ? 0 : c.sliding_window;
    const int lo = window > 0 ? std::max(0, c0 - window + 1) : 0, span = c0 + M - lo;
    {  // scores S_h = q_h . K^T, one z per query head (its KV head: z / g)
      GemmArgs g = plain(M, span, d, w.sp, w.ks, status);
      g.za_col = d;
      g.zb_div = l.g;
      g.zb_col = d;
      g.b_row0 = lo;
      g.zc_row = M;
      g.band = 1;
      g.q_pos0 = c0;
      g.key_pos0 = lo;
      g.window = window;
      if ((rc = gemm({w.q, (uint64_t)nq * d, (uint64_t)M, (uint64_t)nq * d},
                     {tg.ck[li], (uint64_t)l.n_kv * d, (uint64_t)tg.cache_len, (uint64_t)l.n_kv * d}, g, nq,
                     st)))
        return rc;
    }
    pf_softmax<<<nq * M, 256, 0, st>>>(w.sp, M, w.ks, span, c0, lo, window);
    pf_vtrans<<<dim3((span + 31) / 32, d / 32, l.n_kv), dim3(32, 8), 0, st>>>(tg.cv[li], w.vt, lo, span, l.n_kv, d,
                                                                              w.ks);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
    {  // ctx_h = P_h . V (V^T rows per KV head)
      GemmArgs g = plain(M, d, span, w.ctx, (long long)nq * d, status);
      g.za_row = M;
      g.zb_div = l.g;
      g.zb_row = d;
      g.zc_col = d;
      g.band = 2;
      g.q_pos0 = c0;
      g.key_pos0 = lo;
      g.window = window;
      if ((rc = gemm({w.sp, (uint64_t)span, (uint64_t)nq * M, (uint64_t)w.ks},
                     {w.vt, (uint64_t)span, (uint64_t)l.n_kv * d, (uint64_t)w.ks}, g, nq, st)))
        return rc;
    }
    if (!tp) {
      if ((rc = gemm({w.ctx, (uint64_t)nq * d, (uint64_t)M, (uint64_t)nq * d},
                     {l.o, (uint64_t)nq * d, (uint64_t)H, (uint64_t)nq * d}, plain(M, H, nq * d, w.o, H, status), 1,
                     st, sb)))
        return rc;
    } else {  // this rank's heads' o_proj partial (fp32), summed over the ranks into w.o
      int seq, par;
      xnext(seq, par);
      GemmArgs g = plain(M, H, nq * d, pfx_slot(px, px.rank, par), H, status);
      g.c_f32 = 1;
      if ((rc = gemm({w.ctx, (uint64_t)nq * d, (uint64_t)M, (uint64_t)nq * d},
                     {l.o, (uint64_t)nq * d, (uint64_t)H, (uint64_t)nq * d}, g, 1, st, sb)))
        return rc;
      if ((rc = pf_xsum(px, seq, par, M, H, H, w.o, nullptr, tg.ctrl, xgrid / 2, st))) return rc;
    }
    pf_post_attn<<<M, kRowThreads, 0, st>>>(w.o, w.x, l.n_post_attn, l.n_pre_ff, l.n_pre_ff2, l.router_scale,
                                             w.mlp_in, w.h2, w.rin, H, eps, hinv);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
    // ---- dense MLP (model.py:218-221)
    if ((rc = gemm({w.mlp_in, (uint64_t)H, (uint64_t)M, (uint64_t)H}, {l.gate, (uint64_t)H, (uint64_t)I, (uint64_t)H},
                   plain(M, I, H, w.gate, I, status), 1, st, sb)))
      return rc;
    if ((rc = gemm({w.mlp_in, (uint64_t)H, (uint64_t)M, (uint64_t)H}, {l.up, (uint64_t)H, (uint64_t)I, (uint64_t)H},
                   plain(M, I, H, w.up, I, status), 1, st, sb)))
      return rc;
    pf_gelu_mul<<<std::min(4096, (M * I + 255) / 256), 256, 0, st>>>(w.gate, w.up, w.act, (size_t)M * I);
    // tensor parallel: this rank's MLP partial and (below) MoE partial share one exchange
    int fseq = 0, fpar = 0;
    float* fslot = nullptr;
    if (tp) {
      xnext(fseq, fpar);
      fslot = pfx_slot(px, px.rank, fpar);
    }
    {
      GemmArgs g = plain(M, H, I, tp ? static_cast<void*>(fslot) : static_cast<void*>(w.mlp_out), tp ? 2 * H : H,
                         status);
      g.c_f32 = tp ? 1 : 0;
      if ((rc = gemm({w.act, (uint64_t)I, (uint64_t)M, (uint64_t)I}, {l.down, (uint64_t)I, (uint64_t)H, (uint64_t)I},
                     g, 1, st, sb)))
        return rc;
    }
    // ---- router + dense MoE over all experts (model.py:224-250)
    if ((rc = gemm({w.rin, (uint64_t)H, (uint64_t)M, (uint64_t)H}, {l.router, (uint64_t)H, (uint64_t)E, (uint64_t)H},
                   plain(M, E, H, w.rlog, E, status), 1, st, sb)))
      return rc;
    pf_router<<<M, 256, 0, st>>>(w.rlog, l.pes, w.wfull, E, K);
    if (!dense) {  // the same sum over the routed (token, expert) pairs only
      if ((rc = routed_moe(m, l, M, status, st, fslot ? fslot + H : nullptr, 2 * H))) return rc;
    } else if ((rc = gemm({w.h2, (uint64_t)H, (uint64_t)M, (uint64_t)H},
                          {l.exp_gu, (uint64_t)H, (uint64_t)E * 2 * F, (uint64_t)H},
                          plain(M, E * 2 * F, H, w.gu, (long long)E * 2 * F, status), 1, st, sb))) {
      return rc;
    }
    if (dense) {
      pf_moe_act<<<std::min(8192, (int)(((size_t)M * E * F + 255) / 256)), 256, 0, st>>>(w.gu, w.wfull, w.mact, M,
                                                                                         E, F);
      G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
    }
    if (dense) {  // sum over (expert, f) in one GEMM: B = down [E, H, F] as 3-D (f, h, e)
      const int kpe = (F + kGemmBK - 1) / kGemmBK;
      GemmArgs g = plain(M, H, E * kpe * kGemmBK, w.moe_out, H, status);
      g.b_kpe = kpe;
      g.a_slab = F;
      Operand B{l.exp_down, (uint64_t)F, (uint64_t)H, (uint64_t)F};
      B.slabs = E;
      if ((rc = gemm({w.mact, (uint64_t)E * F, (uint64_t)M, (uint64_t)E * F}, B, g, 1, st, sb))) return rc;
    }
    if (tp) {
      if ((rc = pf_xsum(px, fseq, fpar, M, 2 * H, H, w.mlp_out, w.moe_out, tg.ctrl, xgrid, st))) return rc;
    }
    pf_combine<<<M, kRowThreads, 0, st>>>(w.mlp_out, w.moe_out, w.x, l.n_post_ff1, l.n_post_ff2, l.n_post_ff,
                                           l.scalar, H, eps);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  }
  if (last && tp) {  // tensor parallel: the LM head's argmax over every rank's vocab slice
    pf_rmsnorm<<<1, kRowThreads, 0, st>>>(w.x + (size_t)(M - 1) * H, m->final_norm, w.xf, H, eps);
    if ((rc = gemm({w.xf, (uint64_t)H, 1, (uint64_t)H},
                   {m->embed + (size_t)m->vbegin * H, (uint64_t)H, (uint64_t)m->V_local, (uint64_t)H},
                   plain(1, m->V_local, H, w.lmlog, m->V_local, status), 1, st, sb)))
      return rc;
    int seq, par;
    xnext(seq, par);
    pf_lm_epilogue<<<1, 1024, 0, st>>>(w.lmlog, tg.logits, m->V_local, m->vbegin, c.final_logit_softcapping,
                                       tg.tok_out, tg.out_index, tg.tok_host, tg.ctrl, n_total, 0, 0,
                                       pfx_slot(px, px.rank, par));
    pf_xargmax<<<1, 32, 0, st>>>(px, seq, par, tg.tok_out, tg.out_index, tg.tok_host, tg.ctrl, n_total);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
    return G4_OK;
  }
  if (last) {  // final norm, LM head of the last prompt position (last_index, model.py:372-385)
    pf_rmsnorm<<<1, kRowThreads, 0, st>>>(w.x + (size_t)(M - 1) * H, m->final_norm, w.xf, H, eps);
    if ((rc = gemm({w.xf, (uint64_t)H, 1, (uint64_t)H},
                   {m->embed + (size_t)m->vbegin * H, (uint64_t)H, (uint64_t)m->V_local, (uint64_t)H},
                   plain(1, m->V_local, H, w.lmlog, m->V_local, status), 1, st, sb)))
      return rc;
    pf_lm_epilogue<<<1, 1024, 0, st>>>(w.lmlog, tg.logits, m->V_local, m->vbegin, c.final_logit_softcapping,
                                       tg.tok_out, tg.out_index, tg.tok_host, tg.ctrl, n_total);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  }
  return G4_OK;
}

// The model's own sequence as a prefill target.
static PfTarget model_target(g4_model* m, std::vector<bf16_t*>& ck, std::vector<bf16_t*>& cv, int n) {
  ck.clear();
  cv.clear();
  for (const LayerDev& l : m->L) {
    ck.push_back(l.cache_k);
    cv.push_back(l.cache_v);
  }
  PfTarget t{};
  t.tokens = m->tokens_in;
  t.ck = ck.data();
  t.cv = cv.data();
  t.cache_len = m->max_len;
  t.tok_out = m->tokens_out;
  t.out_index = n;
  t.tok_host = m->lm.tokens_host;
  t.ctrl = m->ctrl;
  t.logits = m->logits;
  return t;
}

int g4_make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                   uint32_t box_rows) {
  return make_map_2d(map, base, inner, rows, ld, box_rows);
}

extern "C" int g4_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M,
                            int N, int K, int c_f32, int* status, void* stream) {
  if (!A || !B || !C) return fail(G4_ERR_ARG, "g4_gemm_bf16: null pointer");
  if (M < 1 || N < 1 || K < 1 || lda < K || ldb < K || ldc < N)
    return fail(G4_ERR_ARG, "g4_gemm_bf16: bad shape %d x %d x %d", M, N, K);
  GemmArgs g = plain(M, N, K, C, ldc, status);
  g.c_f32 = c_f32 ? 1 : 0;
  return gemm({A, (uint64_t)K, (uint64_t)M, (uint64_t)lda}, {B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb}, g, 1,
              static_cast<cudaStream_t>(stream));
}

extern "C" int g4_prefill(g4_model* m, int n_tokens, int chunk, int flags, void* stream) {
  if (!m) return fail(G4_ERR_ARG, "g4_prefill: null model");
  if (flags & ~G4_PREFILL_DENSE_MOE) return fail(G4_ERR_ARG, "g4_prefill: unknown flags 0x%x", flags);
  if (!m->finalized) return fail(G4_ERR_STATE, "g4_prefill before g4_model_finalize");
  if (m->world > 1 && (flags & G4_PREFILL_DENSE_MOE))
    return fail(G4_ERR_ARG, "g4_prefill: the dense all-expert MoE runs at world 1 (routed pairs under tensor parallelism)");
  if (m->world > 1 && (!m->comm || !m->comm->open))
    return fail(G4_ERR_STATE, "g4_prefill: world %d needs an open communicator", m->world);
  if (m->world > 1 && m->comm->hidden < m->H)
    return fail(G4_ERR_SHAPE, "g4_prefill: communicator hidden %d < model hidden %d", m->comm->hidden, m->H);
  if (n_tokens < 1 || n_tokens > m->max_len)
    return fail(G4_ERR_ARG, "g4_prefill: %d tokens outside [1, %d]", n_tokens, m->max_len);
  if (chunk <= 0) chunk = 4096;
  if (m->world > 1) chunk = std::min(chunk, kPfXRows);  // the exchange slots' rows
  chunk = std::min(chunk, n_tokens);
  chunk = (chunk + kGemmBM - 1) / kGemmBM * kGemmBM;
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  int rc = prefill_workspace(m, chunk);
  if (rc) return rc;
  if ((rc = g4_prepare_sampler(m))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<bf16_t*> ck, cv;
  const PfTarget tg = model_target(m, ck, cv, n_tokens);
  for (int c0 = 0; c0 < n_tokens; c0 += chunk) {
    const int M = std::min(chunk, n_tokens - c0);
    if ((rc = prefill_chunk(m, c0, M, c0 + M == n_tokens, n_tokens, (flags & G4_PREFILL_DENSE_MOE) != 0, st, tg)))
      return rc;
  }
  return g4_launch_sampler(m, st);  // temperature > 0: replaces the greedy first token
}

// ------------------------------------------------------------------ batched decode
// B sequences decoded together (benchmark config 5's batch-8 decode; the reference's
// forward takes [B, T] inputs, model.py:333-386, and its cache has a batch axis,
// model.py:174-185).  Each sequence has its own KV cache [ctx, kv, d] per layer and its
// own control block (position, status); one step runs every projection as a tensor-core
// GEMM with M = B (split-K: the step is weight-streaming bound), the routed MoE as grouped
// GEMMs over the B x top-k pairs (each selected expert's weights read once for all the
// sequences that picked it), and attention per sequence with the decode attention kernel.
struct BatchWs {
  int B = 0, ctx = 0;
  char* mem = nullptr;
  std::vector<bf16_t*> ck, cv;  // per layer: sequence 0's cache; sequence b at + b * ctx * kv * d
  int* ctrl = nullptr;          // [B][G4_CTRL_WORDS]
  int* tokens = nullptr;        // [B] next input token of each sequence
  float* logits = nullptr;      // [B, V_local] fp32 softcapped logits of the last step
  bf16_t* xf = nullptr;         // [B, H]
  bf16_t* lmlog = nullptr;      // [B, V_local]
  std::vector<CUtensorMap> mk, mv;  // [layer * B + b]: attention tensor maps of each cache
  // attention of all sequences in one launch per layer: the sequences' args in device
  // memory (rebuilt when the prefill workspace they point into moves), splits sized for
  // the whole batch, and each sequence's own partials and merge counters
  AttnArgs* dargs = nullptr;       // [layer][B]
  const bf16_t* dargs_qkv = nullptr;  // the workspace's qkv and ctx rows dargs point at
  const bf16_t* dargs_ctx = nullptr;
  std::vector<int> nsplit;         // per layer
  float* part = nullptr;           // [B][part_floats]
  int* cnt = nullptr;              // [B][cnt_ints], zero at rest
  size_t part_floats = 0;
  int cnt_ints = 0;
};

void g4_batch_release(g4_model* m) {
  if (!m || !m->batch) return;
  if (m->batch->mem) cudaFree(m->batch->mem);
  delete m->batch;
  m->batch = nullptr;
}

static void batch_caches(const g4_model* m, int seq, std::vector<bf16_t*>& ck, std::vector<bf16_t*>& cv);

extern "C" int g4_batch_reserve(g4_model* m, int batch, int ctx_len) {
  if (!m || !m->finalized) return fail(G4_ERR_STATE, "g4_batch_reserve: model not finalized");
  if (m->world != 1) return fail(G4_ERR_SHAPE, "g4_batch_reserve: batched decode runs at world 1");
  if (batch < 1 || batch > 64 || ctx_len < 1 || ctx_len > m->max_len)
    return fail(G4_ERR_ARG, "g4_batch_reserve: batch %d (1..64), context %d (1..%d)", batch, ctx_len, m->max_len);
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  g4_batch_release(m);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += up256(bytes);
    return o;
  };
  std::vector<size_t> ok, ov;
  for (const LayerDev& l : m->L) {
    const size_t per = (size_t)batch * ctx_len * l.n_kv * l.d * 2;
    ok.push_back(take(per));
    ov.push_back(take(per));
  }
  const size_t o_ctrl = take((size_t)batch * G4_CTRL_WORDS * 4), o_tok = take((size_t)batch * 4),
               o_lg = take((size_t)batch * m->V_local * 4), o_xf = take((size_t)batch * m->H * 2),
               o_lm = take((size_t)batch * m->V_local * 2);
  // batched attention: one item per SM over all sequences' heads
  std::vector<int> nsplit;
  size_t part_floats = 0;
  int cnt_ints = 0;
  for (const LayerDev& l : m->L) {
    const int max_live = l.full ? ctx_len : std::min(ctx_len, m->cfg.sliding_window);
    const int ns = g4_pick_nsplit(l.n_kv, max_live, std::max(1, m->nsm / batch));
    nsplit.push_back(ns);
    part_floats = std::max(part_floats, attn_part_floats(l.n_kv, ns, l.g, l.d));
    cnt_ints = std::max(cnt_ints, attn_counter_ints(l.n_kv, ns));
  }
  part_floats = (part_floats + 63) / 64 * 64;
  cnt_ints = (cnt_ints + 63) / 64 * 64;
  const size_t o_part = take((size_t)batch * part_floats * 4), o_cnt = take((size_t)batch * cnt_ints * 4),
               o_args = take(m->L.size() * (size_t)batch * sizeof(AttnArgs));
  BatchWs* w = new BatchWs();
  if (cudaMalloc(&w->mem, off) != cudaSuccess) {
    delete w;
    return fail(G4_ERR_NOMEM, "g4_batch_reserve: cudaMalloc(%zu) failed", off);
  }
  G4_CUDA(cudaMemset(w->mem, 0, off), G4_ERR_CUDA);
  w->B = batch;
  w->ctx = ctx_len;
  for (size_t i = 0; i < m->L.size(); ++i) {
    w->ck.push_back(reinterpret_cast<bf16_t*>(w->mem + ok[i]));
    w->cv.push_back(reinterpret_cast<bf16_t*>(w->mem + ov[i]));
  }
  w->ctrl = reinterpret_cast<int*>(w->mem + o_ctrl);
  w->tokens = reinterpret_cast<int*>(w->mem + o_tok);
  w->logits = reinterpret_cast<float*>(w->mem + o_lg);
  w->xf = reinterpret_cast<bf16_t*>(w->mem + o_xf);
  w->lmlog = reinterpret_cast<bf16_t*>(w->mem + o_lm);
  w->nsplit = nsplit;
  w->part_floats = part_floats;
  w->cnt_ints = cnt_ints;
  w->part = reinterpret_cast<float*>(w->mem + o_part);
  w->cnt = reinterpret_cast<int*>(w->mem + o_cnt);
  w->dargs = reinterpret_cast<AttnArgs*>(w->mem + o_args);
  std::vector<int> ctrl((size_t)batch * G4_CTRL_WORDS, 0);
  for (int b = 0; b < batch; ++b) ctrl[(size_t)b * G4_CTRL_WORDS + G4_CTRL_TIMEOUT_US] = 2000000;
  G4_CUDA(cudaMemcpy(w->ctrl, ctrl.data(), ctrl.size() * 4, cudaMemcpyHostToDevice), G4_ERR_CUDA);
  m->batch = w;
  // tensor maps of every sequence's caches, once (the step launches copy them)
  w->mk.resize(m->L.size() * batch);
  w->mv.resize(m->L.size() * batch);
  std::vector<bf16_t*> ck, cv;
  for (int b = 0; b < batch; ++b) {
    batch_caches(m, b, ck, cv);
    for (size_t li = 0; li < m->L.size(); ++li) {
      AttnArgs a = m->k2[li];
      a.cache_k = ck[li];
      a.cache_v = cv[li];
      a.max_len = ctx_len;
      if (int rc = g4_attention_maps(a)) {
        g4_batch_release(m);
        return rc;
      }
      w->mk[li * batch + b] = a.tmk;
      w->mv[li * batch + b] = a.tmv;
    }
  }
  return G4_OK;
}

// Sequence `seq`'s cache pointers.
static void batch_caches(const g4_model* m, int seq, std::vector<bf16_t*>& ck, std::vector<bf16_t*>& cv) {
  const BatchWs& w = *m->batch;
  ck.clear();
  cv.clear();
  for (size_t i = 0; i < m->L.size(); ++i) {
    const size_t per = (size_t)w.ctx * m->L[i].n_kv * m->L[i].d;
    ck.push_back(w.ck[i] + (size_t)seq * per);
    cv.push_back(w.cv[i] + (size_t)seq * per);
  }
}

extern "C" int g4_batch_prefill(g4_model* m, int seq, int n_tokens, int* token_out, void* stream) {
  if (!m || !m->batch) return fail(G4_ERR_STATE, "g4_batch_prefill before g4_batch_reserve");
  BatchWs& bw = *m->batch;
  if (seq < 0 || seq >= bw.B || n_tokens < 1 || n_tokens >= bw.ctx)
    return fail(G4_ERR_ARG, "g4_batch_prefill: sequence %d of %d, %d tokens (context %d)", seq, bw.B, n_tokens, bw.ctx);
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  const int chunk = std::min(4096, (n_tokens + kGemmBM - 1) / kGemmBM * kGemmBM);
  int rc = prefill_workspace(m, std::max(chunk, m->prefill ? m->prefill->chunk : 0));
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<bf16_t*> ck, cv;
  batch_caches(m, seq, ck, cv);
  PfTarget tg{};
  tg.tokens = m->tokens_in;  // the prompt, as for g4_prefill
  tg.ck = ck.data();
  tg.cv = cv.data();
  tg.cache_len = bw.ctx;
  tg.tok_out = bw.tokens;
  tg.out_index = seq;
  tg.ctrl = bw.ctrl + (size_t)seq * G4_CTRL_WORDS;
  tg.logits = bw.logits + (size_t)seq * m->V_local;
  for (int c0 = 0; c0 < n_tokens; c0 += chunk) {
    const int M = std::min(chunk, n_tokens - c0);
    if ((rc = prefill_chunk(m, c0, M, c0 + M == n_tokens, n_tokens, false, st, tg))) return rc;
  }
  if (token_out) G4_CUDA(cudaMemcpyAsync(token_out, bw.tokens + seq, 4, cudaMemcpyDeviceToDevice, st), G4_ERR_CUDA);
  return G4_OK;
}

extern "C" int g4_batch_step(g4_model* m, int* tokens_out, float* logits_out, void* stream) {
  if (!m || !m->batch) return fail(G4_ERR_STATE, "g4_batch_step before g4_batch_reserve");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  BatchWs& bw = *m->batch;
  const int B = bw.B;
  int rc = prefill_workspace(m, std::max(kGemmBM, m->prefill ? m->prefill->chunk : 0));
  if (rc) return rc;
  PrefillWs& w = *m->prefill;
  const SplitBuf sb{w.split, w.split_elems};
  const g4_config& c = m->cfg;
  const int H = m->H, E = m->E, I = m->I_local, K = m->topk;
  const float eps = c.rms_norm_eps;
  int* status = bw.ctrl + G4_CTRL_STATUS;  // sequence 0's status word collects GEMM timeouts
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  pf_embed<<<B, 256, 0, st>>>(bw.tokens, m->embed, w.x, H, c.vocab_size, g4_host_bf16_round(std::sqrt((float)H)),
                              bw.ctrl);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  const float hinv = g4_host_bf16_round(std::pow((float)H, -0.5f));
  if (bw.dargs_qkv != w.qkv || bw.dargs_ctx != w.ctx) {  // the args point into the workspace
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    G4_CUDA(cudaStreamIsCapturing(st, &cs), G4_ERR_CUDA);
    if (cs != cudaStreamCaptureStatusNone)
      return fail(G4_ERR_STATE, "g4_batch_step: capture a step only after an eager step since the last prefill");
    std::vector<bf16_t*> ck, cv;
    std::vector<AttnArgs> host(m->L.size() * (size_t)B);
    for (int b = 0; b < B; ++b) {
      batch_caches(m, b, ck, cv);
      for (size_t li = 0; li < m->L.size(); ++li) {
        const LayerDev& l = m->L[li];
        AttnArgs a = m->k2[li];
        a.qkv = w.qkv + (size_t)b * (l.rows_q + l.rows_k + l.rows_v);
        a.cache_k = ck[li];
        a.cache_v = cv[li];
        a.ctx = w.ctx + (size_t)b * l.n_kv * l.g * l.d;
        a.ctrl = bw.ctrl + (size_t)b * G4_CTRL_WORDS;
        a.part = bw.part + (size_t)b * bw.part_floats;
        a.counters = bw.cnt + (size_t)b * bw.cnt_ints;
        a.nsplit = bw.nsplit[li];
        a.pos_fixed = -1;
        a.max_len = bw.ctx;
        a.trace_id = -1;
        a.tmk = bw.mk[li * B + b];
        a.tmv = bw.mv[li * B + b];
        host[li * B + b] = a;
      }
    }
    G4_CUDA(cudaMemcpy(bw.dargs, host.data(), host.size() * sizeof(AttnArgs), cudaMemcpyHostToDevice), G4_ERR_CUDA);
    bw.dargs_qkv = w.qkv;
    bw.dargs_ctx = w.ctx;
  }
  for (size_t li = 0; li < m->L.size(); ++li) {
    const LayerDev& l = m->L[li];
    const int nq = l.n_kv * l.g, d = l.d, R = l.rows_q + l.rows_k + l.rows_v;
    pf_rmsnorm<<<B, kRowThreads, 0, st>>>(w.x, l.n_in, w.xn, H, eps);
    if ((rc = gemm({w.xn, (uint64_t)H, (uint64_t)B, (uint64_t)H}, {l.qkv, (uint64_t)H, (uint64_t)R, (uint64_t)H},
                   plain(B, R, H, w.qkv, R, status), 1, st, sb)))
      return rc;
    // q/k norm, RoPE, cache write and attention of every sequence: one launch
    if ((rc = g4_launch_attention_batch(bw.dargs + li * B, d, l.g, B, l.n_kv * bw.nsplit[li], st))) return rc;
    if ((rc = gemm({w.ctx, (uint64_t)nq * d, (uint64_t)B, (uint64_t)nq * d},
                   {l.o, (uint64_t)nq * d, (uint64_t)H, (uint64_t)nq * d}, plain(B, H, nq * d, w.o, H, status), 1,
                   st, sb)))
      return rc;
    pf_post_attn<<<B, kRowThreads, 0, st>>>(w.o, w.x, l.n_post_attn, l.n_pre_ff, l.n_pre_ff2, l.router_scale,
                                             w.mlp_in, w.h2, w.rin, H, eps, hinv);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
    if ((rc = gemm({w.mlp_in, (uint64_t)H, (uint64_t)B, (uint64_t)H}, {l.gate, (uint64_t)H, (uint64_t)I, (uint64_t)H},
                   plain(B, I, H, w.gate, I, status), 1, st, sb)) ||
        (rc = gemm({w.mlp_in, (uint64_t)H, (uint64_t)B, (uint64_t)H}, {l.up, (uint64_t)H, (uint64_t)I, (uint64_t)H},
                   plain(B, I, H, w.up, I, status), 1, st, sb)))
      return rc;
    pf_gelu_mul<<<std::min(4096, (B * I + 255) / 256), 256, 0, st>>>(w.gate, w.up, w.act, (size_t)B * I);
    if ((rc = gemm({w.act, (uint64_t)I, (uint64_t)B, (uint64_t)I}, {l.down, (uint64_t)I, (uint64_t)H, (uint64_t)I},
                   plain(B, H, I, w.mlp_out, H, status), 1, st, sb)) ||
        (rc = gemm({w.rin, (uint64_t)H, (uint64_t)B, (uint64_t)H}, {l.router, (uint64_t)H, (uint64_t)E, (uint64_t)H},
                   plain(B, E, H, w.rlog, E, status), 1, st, sb)))
      return rc;
    pf_router<<<B, 256, 0, st>>>(w.rlog, l.pes, w.wfull, E, K);
    if ((rc = routed_moe(m, l, B, status, st))) return rc;
    pf_combine<<<B, kRowThreads, 0, st>>>(w.mlp_out, w.moe_out, w.x, l.n_post_ff1, l.n_post_ff2, l.n_post_ff,
                                           l.scalar, H, eps);
    G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  }
  pf_rmsnorm<<<B, kRowThreads, 0, st>>>(w.x, m->final_norm, bw.xf, H, eps);
  if ((rc = gemm({bw.xf, (uint64_t)H, (uint64_t)B, (uint64_t)H},
                 {m->embed + (size_t)m->vbegin * H, (uint64_t)H, (uint64_t)m->V_local, (uint64_t)H},
                 plain(B, m->V_local, H, bw.lmlog, m->V_local, status), 1, st, sb)))
    return rc;
  // every row: softcapped logits, argmax -> the sequence's next token, position + 1
  pf_lm_epilogue<<<B, 1024, 0, st>>>(bw.lmlog, bw.logits, m->V_local, m->vbegin, c.final_logit_softcapping, bw.tokens,
                                     0, nullptr, bw.ctrl, -1, G4_CTRL_WORDS, 0);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  if (tokens_out) G4_CUDA(cudaMemcpyAsync(tokens_out, bw.tokens, (size_t)B * 4, cudaMemcpyDeviceToDevice, st), G4_ERR_CUDA);
  if (logits_out)
    G4_CUDA(cudaMemcpyAsync(logits_out, bw.logits, (size_t)B * m->V_local * 4, cudaMemcpyDeviceToDevice, st),
            G4_ERR_CUDA);
  return G4_OK;
}

extern "C" int g4_batch_status(g4_model* m, void* stream, int* status_out) {
  if (!m || !m->batch) return fail(G4_ERR_STATE, "g4_batch_status before g4_batch_reserve");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  G4_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), G4_ERR_CUDA);
  std::vector<int> ctrl((size_t)m->batch->B * G4_CTRL_WORDS);
  G4_CUDA(cudaMemcpy(ctrl.data(), m->batch->ctrl, ctrl.size() * 4, cudaMemcpyDeviceToHost), G4_ERR_CUDA);
  int st = 0;
  for (int b = 0; b < m->batch->B; ++b) st |= ctrl[(size_t)b * G4_CTRL_WORDS + G4_CTRL_STATUS];
  if (status_out) *status_out = st;
  if (st) return fail(G4_ERR_TIMEOUT, "batched decode status word 0x%x", st);
  return G4_OK;
}
