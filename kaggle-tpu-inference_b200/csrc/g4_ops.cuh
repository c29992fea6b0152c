// Fused decode-step operators for the weight-streaming engine (g4_gemv.cuh).
//
// One transformer layer of the reference (gemma4_tpu/model.py:297-322) runs as six
// kernels; the vector-wide work between two matrix products (RMSNorms, residual adds,
// router input scaling, the MLP||MoE combine, the layer scalar) is recomputed by
// every CTA in the prologue of the kernel that consumes it, from the L2-resident
// outputs of the previous kernel, so no kernel exists only to normalise a vector:
//
//   K1 QkvOp        [x_l = combine(layer l-1) | embed]  rms(x)*input_layernorm -> q|k|v
//   K2 attention    (g4_attention.cuh) q/k norm, RoPE, cache write, split-KV attention
//   K3 OProjOp      ctx -> o_proj                         (all-reduce site 0: push)
//   K4 RouterMlpOp  post-attn norm + residual; pre-ff norms; router GEMV + top-k (last
//                   CTA); dense MLP gate|up -> gelu(g)*u
//   K5 MoeUpOp      dense MLP down; selected experts' gate|up -> gelu(g)*u*w
//   K6 MoeDownOp    selected experts' down, per-expert bf16 sums (all-reduce site 1:
//                   push MLP and MoE partials together)
//   LM LmHeadOp     combine(last layer), final norm, tied lm_head shard, softcap,
//                   argmax (last CTA; argmax exchange across ranks) -> next token
//
// Rounding follows the reference's bf16 graph: every einsum output is rounded to bf16
// after fp32 accumulation, norms run in fp32 and round once, elementwise products of
// bf16 operands round after each product.  With world > 1 the row-parallel partial
// sums are exchanged in fp32 and reduced in rank order (identical on every rank)
// before the single bf16 rounding.
#pragma once

#include "g4_gemv.cuh"

namespace g4 {

constexpr int kMaxPer = 16;        // hidden elements per consumer thread (H <= 4096)
constexpr int kBarReduce = 2;      // named barrier id for prologue block reductions
constexpr int kSites = 3;          // exchange sites: attention out, FFN out, argmax
constexpr int kSiteAttn = 0, kSiteFfn = 1, kSiteArgmax = 2;
constexpr int kXFlagBytes = kSites * 2 * kMaxWorld * 128;
// Smem::ints slots
constexpr int kSmemExp = 0;        // [0,16) expert ids (producer copy)
constexpr int kSmemRouterDone = 32;
constexpr int kSmemLast = 33;
constexpr int kSmemOk = 34;
constexpr int kSmemWriteLogits = 35;

// Scratch counters (int[kNumCounters] in device memory, zero at rest).
constexpr int kCntRouter = 0, kCntLm = 1, kCntSigAttn = 2, kCntSigFfn = 3;
constexpr int kNumCounters = 32;

struct Common {
  int* ctrl;
  int* counters;
  char* xbase[kMaxWorld];  // exchange buffer of every rank, mapped in this process
  int rank, world;
  int xpayload;            // floats per exchange slot
  int H;
  int layer, nlayers;
  float eps;
};

// ------------------------------------------------------------------ exchange
__device__ inline int* xflag(const Common& c, int peer, int site, int parity, int src) {
  return reinterpret_cast<int*>(c.xbase[peer] + ((site * 2 + parity) * kMaxWorld + src) * 128);
}
__device__ inline float* xslot(const Common& c, int peer, int site, int parity, int src) {
  return reinterpret_cast<float*>(c.xbase[peer] + kXFlagBytes) +
         (size_t)((site * 2 + parity) * kMaxWorld + src) * c.xpayload;
}
__device__ inline int read_step(const Common& c) { return ldcg_i(c.ctrl + G4_CTRL_STEP); }
__device__ inline int site_use(const Common& c, int site, int layer) {
  return site == kSiteArgmax ? read_step(c) : read_step(c) * c.nlayers + layer;
}

// All consumer threads: make this CTA's peer stores visible, then the last CTA of the
// grid publishes flag value use+1 to every rank.
__device__ inline void xchg_signal(const Common& c, int site, int use, int counter_id) {
  __threadfence_system();
  named_bar(kBarReduce, kConsumerThreads);
  if (threadIdx.x == 0) {
    int* cnt = c.counters + counter_id;
    int old = atomic_add_acq_rel_gpu(cnt, 1);
    if (old == (int)gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < c.world; ++p) st_release_sys(xflag(c, p, site, use & 1, c.rank), use + 1);
      atomicExch(cnt, 0);
    }
  }
}

// Thread 0 waits for every rank's flag of (site, use); result broadcast to consumers.
__device__ inline bool xchg_wait(const Common& c, int site, int use, Smem& sm) {
  if (threadIdx.x == 0) {
    int ok = 1;
    const int tmo = ldcg_i(c.ctrl + G4_CTRL_TIMEOUT_US);
    for (int src = 0; src < c.world && ok; ++src)
      ok = wait_flag_geq(xflag(c, c.rank, site, use & 1, src), use + 1, tmo,
                         c.ctrl + G4_CTRL_STATUS);
    sm.ints[kSmemOk] = ok;
  }
  named_bar(kBarReduce, kConsumerThreads);
  return sm.ints[kSmemOk] != 0;
}

// ------------------------------------------------------------------ vector helpers
// Consumer thread t owns hidden elements h = t + 256*i.
#define G4_FOR_H(c, i, h)                                      \
  _Pragma("unroll") for (int i = 0; i < kMaxPer; ++i)          \
    for (int h = (int)threadIdx.x + i * kConsumerThreads; h < (c).H && i < kMaxPer; h = (c).H)

__device__ inline float rms_scale(float ss, int n, float eps) {
  return 1.0f / sqrtf(ss / (float)n + eps);
}

// Output of layer `tail` from the previous kernels (model.py:312-322):
//   h1 = rms(mlp)*pf1, h2 = rms(moe)*pf2, h = rms(h1+h2)*pf, x = (resmid + h)*scalar.
struct Tail {
  const bf16_t* resmid;  // residual after attention (bf16 [H])
  const float* mlp;      // world==1: dense-MLP down output (fp32 [H])
  const bf16_t* moe;     // world==1: MoE output, per-expert bf16 sums (bf16 [H])
  const bf16_t *pf1, *pf2, *pf, *scalar;
  int layer;
};

__device__ inline bool layer_output(const Common& c, const Tail& t, float* x, Smem& sm) {
  float m[kMaxPer], mo[kMaxPer];
  bool ok = true;
  if (c.world == 1) {
    G4_FOR_H(c, i, h) {
      m[i] = rbf(ldcg_f(t.mlp + h));
      mo[i] = bf2f(ldcg_bf(t.moe + h));
    }
  } else {
    const int use = site_use(c, kSiteFfn, t.layer);
    ok = xchg_wait(c, kSiteFfn, use, sm);
    G4_FOR_H(c, i, h) {
      float a = 0.f, b = 0.f;
      for (int src = 0; src < c.world; ++src) {
        const float* sl = xslot(c, c.rank, kSiteFfn, use & 1, src);
        a += ldcg_f(sl + h);
        b += ldcg_f(sl + c.H + h);
      }
      m[i] = rbf(a);
      mo[i] = rbf(b);
    }
  }
  float s1 = 0.f, s2 = 0.f;
  G4_FOR_H(c, i, h) {
    s1 += m[i] * m[i];
    s2 += mo[i] * mo[i];
  }
  const float r1 = rms_scale(block_sum(s1, sm.red, kConsumerThreads, kBarReduce), c.H, c.eps);
  const float r2 = rms_scale(block_sum(s2, sm.red + 32, kConsumerThreads, kBarReduce), c.H, c.eps);
  float s3 = 0.f;
  G4_FOR_H(c, i, h) {
    const float h1 = rbf((m[i] * r1) * bf2f(t.pf1[h]));
    const float h2 = rbf((mo[i] * r2) * bf2f(t.pf2[h]));
    m[i] = rbf(h1 + h2);
    s3 += m[i] * m[i];
  }
  const float r3 = rms_scale(block_sum(s3, sm.red, kConsumerThreads, kBarReduce), c.H, c.eps);
  const float sc = bf2f(t.scalar[0]);
  G4_FOR_H(c, i, h) {
    const float hn = rbf((m[i] * r3) * bf2f(t.pf[h]));
    const float xv = rbf(bf2f(ldcg_bf(t.resmid + h)) + hn);
    x[i] = rbf(xv * sc);
  }
  return ok;
}

// rms(x) * w rounded to bf16, stored as the bf16 input vector `dst` (smem).
__device__ inline void norm_to_smem(const Common& c, const float* x, const bf16_t* w,
                                    bf16_t* dst, Smem& sm) {
  float s = 0.f;
  G4_FOR_H(c, i, h) s += x[i] * x[i];
  const float r = rms_scale(block_sum(s, sm.red, kConsumerThreads, kBarReduce), c.H, c.eps);
  G4_FOR_H(c, i, h) dst[h] = f2bf((x[i] * r) * bf2f(w[h]));
}

// ================================================================== K1: q|k|v
struct QkvOp {
  Common c;
  int* ctrl;  // == c.ctrl (the engine reads op.ctrl)
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];
  const bf16_t* w;     // [rows, H]: q rows, k rows, v rows of this rank
  const bf16_t* w_in;  // input_layernorm
  bf16_t* out;         // q|k|v projections (bf16 [rows])
  bf16_t* xres;        // layer input x (bf16 [H]), written by CTA 0
  // layer 0: token embedding
  const bf16_t* embed;  // replicated [V, H]
  const int* tokens_in;
  const int* tokens_out;
  int vocab;
  float embed_scale;  // bf16(sqrt(H)) as float
  Tail tail;          // layer > 0

  __device__ bool seg_dependent(int) const { return false; }
  __device__ void load_dependent(Smem&) const {}
  __device__ void issue(int, int u0, int n, unsigned char* stage, uint64_t* bar, uint64_t pol,
                        const Smem&) const {
    bulk_g2s(stage, w + (size_t)u0 * c.H, (uint32_t)(n * c.H * 2), bar, pol);
  }
  __device__ const bf16_t* xvec(int, int, const Smem& sm) const {
    return reinterpret_cast<const bf16_t*>(sm.x0);
  }
  __device__ bool prologue(Smem& sm) const {
    float x[kMaxPer];
    bool ok = true;
    if (c.layer == 0) {
      const int pos = ldcg_i(ctrl + G4_CTRL_POS);
      const int forced = ldcg_i(ctrl + G4_CTRL_FORCED_LEN);
      int tok = pos < forced ? ldcg_i(tokens_in + pos) : ldcg_i(tokens_out + pos);
      if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(ctrl + G4_CTRL_STATUS, G4_STATUS_BAD_TOKEN);
        tok = 0;
      }
      const bf16_t* row = embed + (size_t)tok * c.H;
      G4_FOR_H(c, i, h) x[i] = rbf(bf2f(row[h]) * embed_scale);
    } else {
      ok = layer_output(c, tail, x, sm);
    }
    if (blockIdx.x == 0) G4_FOR_H(c, i, h) xres[h] = f2bf(x[i]);
    norm_to_smem(c, x, w_in, reinterpret_cast<bf16_t*>(sm.x0), sm);
    return ok;
  }
  __device__ void epilogue(int, int u0, int n, const float* res, Smem&, bool ok) const {
    if (ok && (int)threadIdx.x < n) out[u0 + threadIdx.x] = f2bf(res[threadIdx.x]);
  }
  __device__ void finish(Smem&, bool) const {}
};

// ================================================================== K3: o_proj
struct OProjOp {
  Common c;
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];
  const bf16_t* w;    // [H, Kc]
  const bf16_t* ctx;  // attention context (bf16 [Kc])
  float* out;         // world==1: o_proj output (fp32 [H])
  int Kc;

  __device__ bool seg_dependent(int) const { return false; }
  __device__ void load_dependent(Smem&) const {}
  __device__ void issue(int, int u0, int n, unsigned char* stage, uint64_t* bar, uint64_t pol,
                        const Smem&) const {
    bulk_g2s(stage, w + (size_t)u0 * Kc, (uint32_t)(n * Kc * 2), bar, pol);
  }
  __device__ const bf16_t* xvec(int, int, const Smem& sm) const {
    return reinterpret_cast<const bf16_t*>(sm.x0);
  }
  __device__ bool prologue(Smem& sm) const {
    const uint4* src = reinterpret_cast<const uint4*>(ctx);
    uint4* dst = reinterpret_cast<uint4*>(sm.x0);
    for (int i = threadIdx.x; i < Kc / 8; i += kConsumerThreads) dst[i] = ldcg_u4(src + i);
    return true;
  }
  __device__ void epilogue(int, int u0, int n, const float* res, Smem& sm, bool ok) const {
    if (!ok || (int)threadIdx.x >= n) return;
    const int u = u0 + threadIdx.x;
    const float v = res[threadIdx.x];
    if (c.world == 1) {
      out[u] = v;
    } else {
      const int use = site_use(c, kSiteAttn, c.layer);
      for (int p = 0; p < c.world; ++p) xslot(c, p, kSiteAttn, use & 1, c.rank)[u] = v;
    }
  }
  __device__ void finish(Smem&, bool) const {
    if (c.world > 1) xchg_signal(c, kSiteAttn, site_use(c, kSiteAttn, c.layer), kCntSigAttn);
  }
};

// ================================================================== K4: router + MLP gate|up
struct RouterMlpOp {
  Common c;
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];
  const float* o_in;     // world==1: o_proj output (fp32 [H])
  const bf16_t* xres;    // layer input
  const bf16_t *n_post_attn, *n_pre_ff, *n_pre_ff2, *router_scale;
  bf16_t* resmid;        // out: residual after attention (CTA 0)
  bf16_t* h2;            // out: MoE input (CTA 0)
  const bf16_t* router_w;  // [E, H]
  const bf16_t* pes;       // per_expert_scale [E]
  const bf16_t* gate;      // [I_local, H]
  const bf16_t* up;        // [I_local, H]
  float* router_logits;    // scratch [E]
  int* top_idx;            // out [K]
  float* top_w;            // out [K]
  bf16_t* mlp_act;         // out [I_local]
  int E, topk;
  float hinv;              // bf16(H^-0.5) as float

  __device__ bool seg_dependent(int) const { return false; }
  __device__ void load_dependent(Smem&) const {}
  __device__ void issue(int s, int u0, int n, unsigned char* stage, uint64_t* bar, uint64_t pol,
                        const Smem&) const {
    const uint32_t bytes = (uint32_t)(n * c.H * 2);
    if (s == 0) {
      bulk_g2s(stage, router_w + (size_t)u0 * c.H, bytes, bar, pol);
    } else {
      bulk_g2s(stage, gate + (size_t)u0 * c.H, bytes, bar, pol);
      bulk_g2s(stage + bytes, up + (size_t)u0 * c.H, bytes, bar, pol);
    }
  }
  __device__ const bf16_t* xvec(int s, int, const Smem& sm) const {
    return reinterpret_cast<const bf16_t*>(s == 0 ? sm.x0 : sm.x1);
  }
  __device__ bool prologue(Smem& sm) const {
    float o[kMaxPer];
    bool ok = true;
    if (c.world == 1) {
      G4_FOR_H(c, i, h) o[i] = rbf(ldcg_f(o_in + h));
    } else {
      const int use = site_use(c, kSiteAttn, c.layer);
      ok = xchg_wait(c, kSiteAttn, use, sm);
      G4_FOR_H(c, i, h) {
        float a = 0.f;
        for (int src = 0; src < c.world; ++src) a += ldcg_f(xslot(c, c.rank, kSiteAttn, use & 1, src) + h);
        o[i] = rbf(a);
      }
    }
    // x = residual + rms(attn)*post_attention_layernorm      (model.py:303-304)
    float s = 0.f;
    G4_FOR_H(c, i, h) s += o[i] * o[i];
    float r = rms_scale(block_sum(s, sm.red, kConsumerThreads, kBarReduce), c.H, c.eps);
    s = 0.f;
    G4_FOR_H(c, i, h) {
      const float a = rbf((o[i] * r) * bf2f(n_post_attn[h]));
      o[i] = rbf(bf2f(ldcg_bf(xres + h)) + a);
      s += o[i] * o[i];
    }
    if (blockIdx.x == 0) G4_FOR_H(c, i, h) resmid[h] = f2bf(o[i]);
    // MLP input (model.py:310) and MoE input (model.py:315)
    r = rms_scale(block_sum(s, sm.red, kConsumerThreads, kBarReduce), c.H, c.eps);
    bf16_t* xm = reinterpret_cast<bf16_t*>(sm.x1);
    float s2 = 0.f;
    G4_FOR_H(c, i, h) {
      xm[h] = f2bf((o[i] * r) * bf2f(n_pre_ff[h]));
      const float v = rbf((o[i] * r) * bf2f(n_pre_ff2[h]));
      if (blockIdx.x == 0) h2[h] = f2bf(v);
      o[i] = v;
      s2 += v * v;
    }
    // router input: rms(h2) * scale * H^-1/2                 (model.py:225-226)
    r = rms_scale(block_sum(s2, sm.red, kConsumerThreads, kBarReduce), c.H, c.eps);
    bf16_t* xr = reinterpret_cast<bf16_t*>(sm.x0);
    G4_FOR_H(c, i, h) {
      const float v = rbf(rbf(rbf(o[i] * r) * bf2f(router_scale[h])) * hinv);
      xr[h] = f2bf(v);
    }
    if (threadIdx.x == 0) sm.ints[kSmemRouterDone] = 0;
    return ok;
  }
  __device__ void epilogue(int s, int u0, int n, const float* res, Smem& sm, bool ok) const {
    const int t = threadIdx.x;
    if (s == 0) {
      if (ok && t < n) router_logits[u0 + t] = rbf(res[t]);
      if (t == 0) sm.ints[kSmemRouterDone] += n;
    } else if (ok && t < n) {
      const float g = rbf(res[t]), u = rbf(res[n + t]);
      mlp_act[u0 + t] = f2bf(rbf(gelu_tanh(g)) * u);
    }
  }
  __device__ void finish(Smem& sm, bool) const {
    // The CTA that completes the router's E logits selects the top-k (model.py:227-232).
    __threadfence();
    named_bar(kBarReduce, kConsumerThreads);
    if (threadIdx.x == 0) {
      int last = 0;
      const int mine = sm.ints[kSmemRouterDone];
      if (mine > 0) {
        int old = atomic_add_acq_rel_gpu(c.counters + kCntRouter, mine);
        last = (old + mine == E);
        if (last) atomicExch(c.counters + kCntRouter, 0);
      }
      sm.ints[kSmemLast] = last;
    }
    named_bar(kBarReduce, kConsumerThreads);
    if (!sm.ints[kSmemLast] || threadIdx.x >= 32) return;
    __threadfence();
    const int lane = threadIdx.x;
    float mx = -INFINITY;
    for (int e = lane; e < E; e += 32) mx = fmaxf(mx, ldcg_f(router_logits + e));
    mx = warp_max(mx);
    float sum = 0.f;
    for (int e = lane; e < E; e += 32) sum += expf(ldcg_f(router_logits + e) - mx);
    sum = warp_sum(sum);
    // probabilities live in sm.flts[0..E) is too small for E=128: recompute per pass
    float wsum = 0.f;
    int chosen[kMaxTopK];
    float chosen_p[kMaxTopK];
    for (int k = 0; k < topk; ++k) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int e = lane; e < E; e += 32) {
        bool taken = false;
        for (int q = 0; q < k; ++q) taken |= (chosen[q] == e);
        if (taken) continue;
        const float p = expf(ldcg_f(router_logits + e) - mx) / sum;
        if (p > bv || (p == bv && e < bi)) {
          bv = p;
          bi = e;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      chosen[k] = bi;
      chosen_p[k] = bv;
      wsum += bv;
    }
    if (lane == 0) {
      for (int k = 0; k < topk; ++k) {
        top_idx[k] = chosen[k];
        top_w[k] = (chosen_p[k] / wsum) * bf2f(pes[chosen[k]]);
      }
    }
  }
};

// ================================================================== K5: MLP down + expert gate|up
struct MoeUpOp {
  Common c;
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];
  const bf16_t* h2;        // MoE input [H]
  const bf16_t* mlp_act;   // [I_local]
  const int* top_idx;      // [K]
  const float* top_w;      // [K]
  const bf16_t* mlp_down;  // [H, I_local]
  const bf16_t* gate_up;   // [E, 2, F, H]
  float* mlp_out;          // out: fp32 [H]
  bf16_t* moe_act;         // out: [K, F]
  int I, F, topk;

  __device__ bool seg_dependent(int s) const { return s == 1; }
  __device__ void load_dependent(Smem& sm) const {
    for (int k = 0; k < topk; ++k) sm.ints[kSmemExp + k] = ldcg_i(top_idx + k);
  }
  __device__ void issue(int s, int u0, int n, unsigned char* stage, uint64_t* bar, uint64_t pol,
                        const Smem& sm) const {
    if (s == 0) {
      bulk_g2s(stage, mlp_down + (size_t)u0 * I, (uint32_t)(n * I * 2), bar, pol);
    } else {
      const int k = u0 / F, f0 = u0 % F;
      const size_t e = (size_t)sm.ints[kSmemExp + k];
      const uint32_t bytes = (uint32_t)(n * c.H * 2);
      bulk_g2s(stage, gate_up + ((e * 2 + 0) * F + f0) * c.H, bytes, bar, pol);
      bulk_g2s(stage + bytes, gate_up + ((e * 2 + 1) * F + f0) * c.H, bytes, bar, pol);
    }
  }
  __device__ const bf16_t* xvec(int s, int, const Smem& sm) const {
    return reinterpret_cast<const bf16_t*>(s == 0 ? sm.x1 : sm.x0);
  }
  __device__ bool prologue(Smem& sm) const {
    uint4* d0 = reinterpret_cast<uint4*>(sm.x0);
    uint4* d1 = reinterpret_cast<uint4*>(sm.x1);
    for (int i = threadIdx.x; i < c.H / 8; i += kConsumerThreads)
      d0[i] = ldcg_u4(reinterpret_cast<const uint4*>(h2) + i);
    for (int i = threadIdx.x; i < I / 8; i += kConsumerThreads)
      d1[i] = ldcg_u4(reinterpret_cast<const uint4*>(mlp_act) + i);
    if ((int)threadIdx.x < topk) sm.flts[threadIdx.x] = ldcg_f(top_w + threadIdx.x);
    return true;
  }
  __device__ void epilogue(int s, int u0, int n, const float* res, Smem& sm, bool ok) const {
    const int t = threadIdx.x;
    if (!ok || t >= n) return;
    if (s == 0) {
      mlp_out[u0 + t] = res[t];
    } else {
      const int u = u0 + t, k = u / F;
      const float g = rbf(res[t]), up = rbf(res[n + t]);
      // gelu(g) * u * w, left to right in bf16 (model.py:271)
      moe_act[u] = f2bf(rbf(rbf(gelu_tanh(g)) * up) * rbf(sm.flts[k]));
    }
  }
  __device__ void finish(Smem&, bool) const {}
};

// ================================================================== K6: expert down
struct MoeDownOp {
  Common c;
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];
  const bf16_t* moe_act;  // [K, F]
  const int* top_idx;
  const bf16_t* down;     // [E, H, F]
  const float* mlp_out;   // world>1: this rank's MLP partial, sent with the MoE partial
  bf16_t* moe_out;        // world==1: bf16 [H]
  int F, topk;

  __device__ bool seg_dependent(int) const { return true; }
  __device__ void load_dependent(Smem& sm) const {
    for (int k = 0; k < topk; ++k) sm.ints[kSmemExp + k] = ldcg_i(top_idx + k);
  }
  __device__ void issue(int, int u0, int n, unsigned char* stage, uint64_t* bar, uint64_t pol,
                        const Smem& sm) const {
    const uint32_t bytes = (uint32_t)(n * F * 2);
    for (int k = 0; k < topk; ++k) {
      const size_t e = (size_t)sm.ints[kSmemExp + k];
      bulk_g2s(stage + (size_t)k * bytes, down + (e * c.H + u0) * F, bytes, bar, pol);
    }
  }
  __device__ const bf16_t* xvec(int, int j, const Smem& sm) const {
    return reinterpret_cast<const bf16_t*>(sm.x0) + j * F;
  }
  __device__ bool prologue(Smem& sm) const {
    uint4* d0 = reinterpret_cast<uint4*>(sm.x0);
    for (int i = threadIdx.x; i < topk * F / 8; i += kConsumerThreads)
      d0[i] = ldcg_u4(reinterpret_cast<const uint4*>(moe_act) + i);
    return true;
  }
  __device__ void epilogue(int, int u0, int n, const float* res, Smem&, bool ok) const {
    const int t = threadIdx.x;
    if (!ok || t >= n) return;
    const int u = u0 + t;
    if (c.world == 1) {
      // per-expert outputs rounded to bf16 and summed in bf16, k = 0..K-1 (model.py:289-293)
      float acc = rbf(res[t]);
      for (int k = 1; k < topk; ++k) acc = rbf(acc + rbf(res[k * n + t]));
      moe_out[u] = f2bf(acc);
    } else {
      float sacc = 0.f;
      for (int k = 0; k < topk; ++k) sacc += res[k * n + t];
      const float mv = ldcg_f(mlp_out + u);
      const int use = site_use(c, kSiteFfn, c.layer);
      for (int p = 0; p < c.world; ++p) {
        float* sl = xslot(c, p, kSiteFfn, use & 1, c.rank);
        sl[u] = mv;
        sl[c.H + u] = sacc;
      }
    }
  }
  __device__ void finish(Smem&, bool) const {
    if (c.world > 1) xchg_signal(c, kSiteFfn, site_use(c, kSiteFfn, c.layer), kCntSigFfn);
  }
};

// ================================================================== LM head + argmax
struct LmHeadOp {
  Common c;
  int* ctrl;
  int nseg;
  SegDesc seg[kMaxSeg];
  int xbytes[2];
  Tail tail;
  const bf16_t* final_norm;
  const bf16_t* embed;  // replicated [V, H]; this rank reads rows [vbegin, vbegin+V_local)
  int vbegin;
  float* logits;        // [V_local] fp32 (written when control[WRITE_LOGITS] != 0)
  float* cand_v;        // scratch [gridDim]
  int* cand_i;          // scratch [gridDim]
  int* tokens_out;      // [max_len + 1]
  int* tokens_host;     // optional mapped pinned host mirror of tokens_out
  float softcap;        // <= 0: none

  __device__ bool seg_dependent(int) const { return false; }
  __device__ void load_dependent(Smem&) const {}
  __device__ void issue(int, int u0, int n, unsigned char* stage, uint64_t* bar, uint64_t pol,
                        const Smem&) const {
    bulk_g2s(stage, embed + (size_t)(vbegin + u0) * c.H, (uint32_t)(n * c.H * 2), bar, pol);
  }
  __device__ const bf16_t* xvec(int, int, const Smem& sm) const {
    return reinterpret_cast<const bf16_t*>(sm.x0);
  }
  __device__ bool prologue(Smem& sm) const {
    float x[kMaxPer];
    bool ok = layer_output(c, tail, x, sm);
    norm_to_smem(c, x, final_norm, reinterpret_cast<bf16_t*>(sm.x0), sm);
    float* bv = reinterpret_cast<float*>(sm.x1);
    int* bi = reinterpret_cast<int*>(sm.x1) + kConsumerThreads;
    bv[threadIdx.x] = -INFINITY;
    bi[threadIdx.x] = 0x7fffffff;
    sm.ints[kSmemWriteLogits] = ldcg_i(ctrl + G4_CTRL_WRITE_LOGITS);
    named_bar(kBarReduce, kConsumerThreads);
    return ok;
  }
  __device__ void epilogue(int, int u0, int n, const float* res, Smem& sm, bool ok) const {
    const int t = threadIdx.x;
    if (!ok || t >= n) return;
    const int u = u0 + t;
    float v = rbf(res[t]);  // einsum output is bf16 (model.py:381-382)
    if (softcap > 0.f) v = tanhf(v / softcap) * softcap;
    if (sm.ints[kSmemWriteLogits]) logits[u] = v;
    float* bv = reinterpret_cast<float*>(sm.x1);
    int* bi = reinterpret_cast<int*>(sm.x1) + kConsumerThreads;
    if (v > bv[t]) {  // units arrive in increasing order: ties keep the lower index
      bv[t] = v;
      bi[t] = u;
    }
  }
  __device__ void finish(Smem& sm, bool ok) const {
    float* bv = reinterpret_cast<float*>(sm.x1);
    int* bi = reinterpret_cast<int*>(sm.x1) + kConsumerThreads;
    named_bar(kBarReduce, kConsumerThreads);
    if (threadIdx.x < 32) {
      float v = -INFINITY;
      int ix = 0x7fffffff;
      for (int i = threadIdx.x; i < kConsumerThreads; i += 32) {
        if (bv[i] > v || (bv[i] == v && bi[i] < ix)) {
          v = bv[i];
          ix = bi[i];
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, ix, o);
        if (ov > v || (ov == v && oi < ix)) {
          v = ov;
          ix = oi;
        }
      }
      if (threadIdx.x == 0) {
        cand_v[blockIdx.x] = v;
        cand_i[blockIdx.x] = ix;
        __threadfence();
        int old = atomic_add_acq_rel_gpu(c.counters + kCntLm, 1);
        sm.ints[kSmemLast] = (old == (int)gridDim.x - 1);
      }
    }
    named_bar(kBarReduce, kConsumerThreads);
    if (!sm.ints[kSmemLast] || threadIdx.x != 0) return;
    // last CTA: reduce the per-CTA candidates in CTA order (deterministic)
    __threadfence();
    atomicExch(c.counters + kCntLm, 0);
    float v = -INFINITY;
    int ix = 0x7fffffff;
    for (int b = 0; b < (int)gridDim.x; ++b) {
      const float cv = ldcg_f(cand_v + b);
      const int ci = ldcg_i(cand_i + b);
      if (cv > v || (cv == v && ci < ix)) {
        v = cv;
        ix = ci;
      }
    }
    int token = ix == 0x7fffffff ? 0 : vbegin + ix;
    if (c.world > 1) {
      const int use = site_use(c, kSiteArgmax, 0);
      for (int p = 0; p < c.world; ++p) {
        float* sl = xslot(c, p, kSiteArgmax, use & 1, c.rank);
        sl[0] = v;
        reinterpret_cast<int*>(sl)[1] = token;
      }
      __threadfence_system();
      for (int p = 0; p < c.world; ++p) st_release_sys(xflag(c, p, kSiteArgmax, use & 1, c.rank), use + 1);
      const int tmo = ldcg_i(ctrl + G4_CTRL_TIMEOUT_US);
      float gv = -INFINITY;
      int gi = 0x7fffffff;
      for (int src = 0; src < c.world; ++src) {
        if (!wait_flag_geq(xflag(c, c.rank, kSiteArgmax, use & 1, src), use + 1, tmo,
                           ctrl + G4_CTRL_STATUS))
          break;
        const float* sl = xslot(c, c.rank, kSiteArgmax, use & 1, src);
        const float sv = ldcg_f(sl);
        const int si = ldcg_i(reinterpret_cast<const int*>(sl) + 1);
        if (sv > gv || (sv == gv && si < gi)) {
          gv = sv;
          gi = si;
        }
      }
      token = gi == 0x7fffffff ? 0 : gi;
    }
    const int pos = ldcg_i(ctrl + G4_CTRL_POS);
    tokens_out[pos + 1] = token;
    if (tokens_host) tokens_host[pos + 1] = token;
    ctrl[G4_CTRL_POS] = pos + 1;
    ctrl[G4_CTRL_STEP] = ldcg_i(ctrl + G4_CTRL_STEP) + 1;
    (void)ok;
  }
};

}  // namespace g4
