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
// Prologue vectors (norm weights; the previous kernel's outputs at world 1) arrive in
// the shared staging area by bulk copies (OpBase::cc / ac, offsets planned on the
// host) before prologue() runs; the vector math runs as short loops over shared memory,
// thread t owning the elements h = t, t+256, ...  Input vectors of the matrix products are fp32 in shared
// memory (values exactly bf16) and move to registers in the engine.
//
// Rounding follows the reference's bf16 graph: every einsum output is rounded to bf16
// after fp32 accumulation, norms run in fp32 and round once, elementwise products of
// bf16 operands round after each product.  With world > 1 the row-parallel partial
// sums are exchanged in fp32 and reduced in rank order (identical on every rank)
// before the single bf16 rounding.
#pragma once

#include "g4_gemv.cuh"

namespace g4 {

constexpr int kMaxHidden = 4096;
constexpr int kBarReduce = 2;      // named barrier id for prologue block reductions
constexpr int kSites = 4;          // exchange sites: attention out, FFN out, argmax, sampling
constexpr int kSiteAttn = 0, kSiteFfn = 1, kSiteArgmax = 2, kSiteSample = 3;
constexpr int kXFlagBytes = kSites * 2 * kMaxWorld * 128;
// Smem::ints slots
constexpr int kSmemRouterEnd = 32;  // end of this CTA's router units (0: none)
constexpr int kSmemRouterMine = 36; // number of this CTA's router units
constexpr int kSmemTopk = 37;       // step kernel: this CTA selects the top-k after its arrival
constexpr int kSmemLast = 33;
constexpr int kSmemOk = 34;
constexpr int kSmemWriteLogits = 35;

// Scratch counters (int[kNumCounters] in device memory, zero at rest).
constexpr int kCntRouter = 0, kCntLm = 1;
constexpr int kNumCounters = 32;

struct Common {
  int* counters;
  char* xbase[kMaxWorld];  // exchange buffer of every rank, mapped in this process
  int rank, world;
  int xpayload;            // floats per exchange slot
  int H;
  int layer, nlayers;
  float eps;
};

// ------------------------------------------------------------------ exchange
__device__ __forceinline__ int* xflag(const Common& c, int peer, int site, int parity, int src) {
  return reinterpret_cast<int*>(c.xbase[peer] + ((site * 2 + parity) * kMaxWorld + src) * 128);
}
__device__ __forceinline__ float* xslot(const Common& c, int peer, int site, int parity, int src) {
  return reinterpret_cast<float*>(c.xbase[peer] + kXFlagBytes) +
         (size_t)((site * 2 + parity) * kMaxWorld + src) * c.xpayload;
}
// LL words (attention-out and FFN-out sites): one 64-bit word per value, the fp32 bits in
// the low half and the tag use + 1 in the high half, written with one 64-bit store (a
// single-copy atomic access), so a reader that sees the tag sees the value: no fence, no
// arrival counter, no flag round trip.  A slot's tags only grow (use is monotonic while
// the communicator serves its model), so a word of an earlier use never matches.
__device__ __forceinline__ unsigned long long* xll(const Common& c, int peer, int site, int parity, int src) {
  return reinterpret_cast<unsigned long long*>(xslot(c, peer, site, parity, src));
}
__device__ __forceinline__ void ll_put(unsigned long long* p, float v, uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// The values of 8 consecutive LL words (64 bytes) once all 8 tags equal `tag`.  Bounded:
// gives up after the control block's timeout (setting PEER_TIMEOUT) or as soon as another
// thread has recorded one.  Returns false when it gave up.
__device__ __forceinline__ bool ll_try8(const unsigned long long* p, uint32_t tag, float* out) {
  bool r = true;
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // two words per 16-byte load; only the values stay live
    uint32_t v0, t0, v1, t1;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v0), "=r"(t0), "=r"(v1), "=r"(t1)
                 : "l"(p + 2 * i)
                 : "memory");
    out[2 * i] = __uint_as_float(v0);
    out[2 * i + 1] = __uint_as_float(v1);
    r = r && t0 == tag && t1 == tag;
  }
  return r;
}
__device__ __forceinline__ bool ll_get8(const unsigned long long* p, uint32_t tag, float* out, int* ctrl) {
  if (ll_try8(p, tag, out)) return true;
  const int tmo = ldcg_i(ctrl + G4_CTRL_TIMEOUT_US);
  const uint64_t limit = static_cast<uint64_t>(tmo > 0 ? tmo : 1000000) * 1000ull;
  const uint64_t t0 = globaltimer_ns();
  int n = 0;
  while (!ll_try8(p, tag, out)) {
    if ((++n & 63) == 0) {
      if (ldcg_i(ctrl + G4_CTRL_STATUS) & G4_STATUS_PEER_TIMEOUT) return false;
      if (globaltimer_ns() - t0 > limit) {
        atomicOr(ctrl + G4_CTRL_STATUS, G4_STATUS_PEER_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}
// AND of a predicate over the consumer threads (one named barrier, id kBarReduce).
__device__ __forceinline__ bool consumers_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(kBarReduce), "r"(kConsumerThreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ int site_use(const int* ctrl, const Common& c, int site, int layer) {
  const int step = ldcg_i(ctrl + G4_CTRL_STEP);
  return site == kSiteArgmax ? step : step * c.nlayers + layer;
}

// ------------------------------------------------------------------ staged vectors
__device__ __forceinline__ const bf16_t* sbf(const Smem& sm, int off) {
  return reinterpret_cast<const bf16_t*>(sm.stg + off);
}
__device__ __forceinline__ float* sf(const Smem& sm, int off) {
  return reinterpret_cast<float*>(sm.stg + off);
}
__device__ __forceinline__ float rms_scale(float ss, int n, float eps) {
  return 1.0f / sqrtf(ss / (float)n + eps);
}
// Prologue vectors of length H live in registers in 8-element chunks: thread t owns
// chunks q = t + 256 j (elements 8q .. 8q+7), j < kChunks; H is a multiple of 8.
constexpr int kChunks = kMaxHidden / 8 / kConsumerThreads;
constexpr int kPerThread = kChunks * 8;
typedef float Vec[kChunks][8];

__device__ __forceinline__ bool chunk_live(int j, int H) {
  return (int)(threadIdx.x + j * kConsumerThreads) * 8 < H;
}
__device__ __forceinline__ int chunk_of(int j) { return threadIdx.x + j * kConsumerThreads; }

__device__ __forceinline__ void unpack8(const uint4 u, float* o) {
  o[0] = bf_lo(u.x); o[1] = bf_hi(u.x); o[2] = bf_lo(u.y); o[3] = bf_hi(u.y);
  o[4] = bf_lo(u.z); o[5] = bf_hi(u.z); o[6] = bf_lo(u.w); o[7] = bf_hi(u.w);
}
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  u.x = (uint32_t)f2bf(f[0]) | ((uint32_t)f2bf(f[1]) << 16);
  u.y = (uint32_t)f2bf(f[2]) | ((uint32_t)f2bf(f[3]) << 16);
  u.z = (uint32_t)f2bf(f[4]) | ((uint32_t)f2bf(f[5]) << 16);
  u.w = (uint32_t)f2bf(f[6]) | ((uint32_t)f2bf(f[7]) << 16);
  return u;
}
// bf16 vector (shared or global, generic loads) -> chunks; dead chunks are zero
__device__ __forceinline__ void load_bf16(const bf16_t* src, int H, Vec& o) {
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    uint4 u = make_uint4(0u, 0u, 0u, 0u);
    if (chunk_live(j, H)) u = reinterpret_cast<const uint4*>(src)[chunk_of(j)];
    unpack8(u, o[j]);
  }
}
// fp32 vector in shared memory -> chunks
__device__ __forceinline__ void load_f32(const float* src, int H, Vec& o) {
#pragma unroll
  for (int j = 0; j < kChunks; ++j) {
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (chunk_live(j, H)) {
      a = reinterpret_cast<const float4*>(src)[2 * chunk_of(j)];
      b = reinterpret_cast<const float4*>(src)[2 * chunk_of(j) + 1];
    }
    o[j][0] = a.x; o[j][1] = a.y; o[j][2] = a.z; o[j][3] = a.w;
    o[j][4] = b.x; o[j][5] = b.y; o[j][6] = b.z; o[j][7] = b.w;
  }
}
// chunks (bf16 values) -> bf16 vector
__device__ __forceinline__ void store_bf16(bf16_t* dst, int H, const Vec& v) {
#pragma unroll
  for (int j = 0; j < kChunks; ++j)
    if (chunk_live(j, H)) reinterpret_cast<uint4*>(dst)[chunk_of(j)] = pack8(v[j]);
}

// Block sum over the consumer threads with ONE barrier: warp partials go to slot
// `slot` of Smem::red (8 slots of 8 floats; a prologue gives each reduction its own
// slot, and the barriers between prologues order the reuse).  Fixed summation order,
// identical on every thread.
__device__ __forceinline__ float bsum1(float v, Smem& sm, int slot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) sm.red[slot * kConsumerWarps + warp] = v;
  named_bar(kBarReduce, kConsumerThreads);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) s += sm.red[slot * kConsumerWarps + i];
  return s;
}
// Two independent sums in one barrier (slots `slot` and `slot + 1`).
__device__ __forceinline__ float2 bsum2(float a, float b, Smem& sm, int slot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  if (lane == 0) {
    sm.red[slot * kConsumerWarps + warp] = a;
    sm.red[(slot + 1) * kConsumerWarps + warp] = b;
  }
  named_bar(kBarReduce, kConsumerThreads);
  float sa = 0.f, sb = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) {
    sa += sm.red[slot * kConsumerWarps + i];
    sb += sm.red[(slot + 1) * kConsumerWarps + i];
  }
  return make_float2(sa, sb);
}

// Output of layer `tail` from the previous kernels (model.py:312-322):
//   h1 = rms(mlp)*pf1, h2 = rms(moe)*pf2, h = rms(h1+h2)*pf, x = (resmid + h)*scalar.
// Staged inputs: pf1/pf2/pf (bf16 constants); world 1: mlp (fp32), moe and resmid
// (bf16).  Result x (bf16 values) in registers (uses reduction slots 0-2).
struct Tail {
  const bf16_t* resmid;  // residual after attention (bf16 [H])
  const bf16_t* scalar;  // layer_scalar [1]
  int layer;
  int o_pf1, o_pf2, o_pf;   // staged constants
  int o_mlp, o_moe, o_res;  // staged activations (world 1)
};

__device__ __forceinline__ bool layer_output(int* ctrl, const Common& c, const Tail& t, Smem& sm, Vec& x,
                                             int trace_id) {
  const int H = c.H;
  bool ok = true;
  // the layer scalar is a global load: issued first, it lands under the reductions
  // (the barriers inside them are compiler fences, so it would not move up by itself)
  const bf16_t scb = t.scalar[0];
  Vec a, b;
  float s1 = 0.f, s2 = 0.f;
  if (c.world == 1) {
    load_f32(sf(sm, t.o_mlp), H, a);
    load_bf16(sbf(sm, t.o_moe), H, b);
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) a[j][e] = rbf(a[j][e]);
  } else {
    // every rank's MLP and MoE partials, summed in rank order (LL words, polled per chunk)
    const int use = site_use(ctrl, c, kSiteFfn, t.layer);
    const uint32_t tag = (uint32_t)use + 1u;
    bool got = true;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
#pragma unroll
      for (int e = 0; e < 8; ++e) a[j][e] = b[j][e] = 0.f;
      if (chunk_live(j, H)) {
        for (int src = 0; src < c.world; ++src) {
          const unsigned long long* sl = xll(c, c.rank, kSiteFfn, use & 1, src);
          float va[8], vb[8];
          got = ll_get8(sl + 8 * chunk_of(j), tag, va, ctrl) && got;
          got = ll_get8(sl + H + 8 * chunk_of(j), tag, vb, ctrl) && got;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            a[j][e] += va[e];
            b[j][e] += vb[e];
          }
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          a[j][e] = rbf(a[j][e]);
          b[j][e] = rbf(b[j][e]);
        }
      }
    }
    ok = consumers_and(got);
    if (threadIdx.x == 0) G4_TRACE_EV(trace_id, 7);  // peer partials in (timeline: exchange wait)
  }
#pragma unroll
  for (int j = 0; j < kChunks; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      s1 += a[j][e] * a[j][e];
      s2 += b[j][e] * b[j][e];
    }
  const float2 ss = bsum2(s1, s2, sm, 0);
  const float r1 = rms_scale(ss.x, H, c.eps), r2 = rms_scale(ss.y, H, c.eps);
  Vec w1, w2;
  load_bf16(sbf(sm, t.o_pf1), H, w1);
  load_bf16(sbf(sm, t.o_pf2), H, w2);
  float s3 = 0.f;
#pragma unroll
  for (int j = 0; j < kChunks; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      a[j][e] = rbf(rbf((a[j][e] * r1) * w1[j][e]) + rbf((b[j][e] * r2) * w2[j][e]));
      s3 += a[j][e] * a[j][e];
    }
  const float r3 = rms_scale(bsum1(s3, sm, 2), H, c.eps);
  const float sc = bf2f(scb);
  load_bf16(sbf(sm, t.o_pf), H, w1);
  load_bf16(sbf(sm, t.o_res), H, w2);
#pragma unroll
  for (int j = 0; j < kChunks; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) x[j][e] = rbf(rbf(w2[j][e] + rbf((a[j][e] * r3) * w1[j][e])) * sc);
  return ok;
}

// dst = bf16(rms(x) * w) for x in registers, bf16 weight w (smem); slot `slot`.
__device__ __forceinline__ void norm_into(const Common& c, const Vec& x, const bf16_t* w, bf16_t* dst,
                                          Smem& sm, int slot) {
  const int H = c.H;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kChunks; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) s += x[j][e] * x[j][e];
  const float r = rms_scale(bsum1(s, sm, slot), H, c.eps);
  Vec wv, y;
  load_bf16(w, H, wv);
#pragma unroll
  for (int j = 0; j < kChunks; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) y[j][e] = (x[j][e] * r) * wv[j][e];
  store_bf16(dst, H, y);
}

// Copy a staged bf16 vector of n elements (n % 8 == 0) into an input vector.
__device__ __forceinline__ void copy_vec(const bf16_t* src, int n, unsigned char* dst) {
  for (int i = threadIdx.x; i < n / 8; i += kConsumerThreads)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
}

// ================================================================== K1: q|k|v
struct QkvOp : OpBase {
  Common c;
  const bf16_t* w;     // [rows, H]: q rows, k rows, v rows of this rank
  bf16_t* out;         // q|k|v projections (bf16 [rows])
  bf16_t* xres;        // layer input x (bf16 [H]), written by CTA 0
  int o_win;
  // layer 0: token embedding
  const bf16_t* embed;  // replicated [V, H]
  const int* tokens_in;
  const int* tokens_out;
  int vocab;
  int max_len;
  float embed_scale;  // bf16(sqrt(H)) as float
  Tail tail;          // layer > 0

  __device__ __forceinline__ bool seg_dependent(int) const { return false; }
  __device__ __forceinline__ void load_dependent(Smem&) const {}
  template <class Fn>
  __device__ __forceinline__ void copies(int, int u0, int n, const int*, Fn&& f) const {
    f(w + (size_t)u0 * c.H, (uint32_t)(n * c.H * 2), 0u);
  }
  __device__ __forceinline__ bool prologue(Smem& sm) const {
    bool ok = true;
    Vec x;
    const int H = c.H;
    if (c.layer == 0) {
      int pos = ldcg_i(ctrl + G4_CTRL_POS);
      if (pos < 0 || pos >= max_len) pos = 0;  // flagged by the attention / lm_head kernels
      const int forced = ldcg_i(ctrl + G4_CTRL_FORCED_LEN);
      int tok = pos < forced ? ldcg_i(tokens_in + pos) : ldcg_i(tokens_out + pos);
      if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(ctrl + G4_CTRL_STATUS, G4_STATUS_BAD_TOKEN);
        tok = 0;
      }
      load_bf16(embed + (size_t)tok * H, H, x);
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) x[j][e] = rbf(x[j][e] * embed_scale);
    } else {
      ok = layer_output(ctrl, c, tail, sm, x, trace_id);
    }
    if (blockIdx.x == 0) store_bf16(xres, H, x);
    norm_into(c, x, sbf(sm, o_win), reinterpret_cast<bf16_t*>(sm.x0), sm, 3);
    return ok;
  }
  __device__ __forceinline__ void epilogue(int, int u0, int n, const Res& res, Smem&, bool ok, int t) const {
    if (ok && t < n) out[u0 + t] = f2bf(res[t]);
  }
  __device__ __forceinline__ void finish(Smem&, bool) const {}
};

// ================================================================== K3: o_proj
struct OProjOp : OpBase {
  Common c;
  const bf16_t* w;  // [H, Kc]
  float* out;       // world==1: o_proj output (fp32 [H])
  int Kc;
  int o_ctx;        // staged ctx (bf16 [Kc])

  __device__ __forceinline__ bool seg_dependent(int) const { return false; }
  __device__ __forceinline__ void load_dependent(Smem&) const {}
  template <class Fn>
  __device__ __forceinline__ void copies(int, int u0, int n, const int*, Fn&& f) const {
    const int ns = seg[0].nsub;
    if (ns == 1) {
      f(w + (size_t)u0 * Kc, (uint32_t)(n * Kc * 2), 0u);
      return;
    }
    // rows split into ns sub-rows (each with its slice of the context): the stage holds
    // sub-row j of every row of the tile after the tile's sub-rows j - 1
    const int ks = Kc / ns;
    for (int r = 0; r < n; ++r)
      for (int j = 0; j < ns; ++j)
        f(w + (size_t)(u0 + r) * Kc + (size_t)j * ks, (uint32_t)(ks * 2), (uint32_t)((j * n + r) * ks * 2));
  }
  __device__ __forceinline__ bool prologue(Smem& sm) const {
    copy_vec(sbf(sm, o_ctx), Kc, sm.x0);
    return true;
  }
  __device__ __forceinline__ void epilogue(int, int u0, int n, const Res& res, Smem&, bool ok, int t) const {
    if (!ok || t >= n) return;
    const int u = u0 + t;
    float v = res[t];
    for (int j = 1; j < seg[0].nsub; ++j) v += res[j * n + t];  // sub-rows in order
    if (c.world == 1) {
      out[u] = v;
    } else {
      const int use = site_use(ctrl, c, kSiteAttn, c.layer);
      for (int p = 0; p < c.world; ++p) ll_put(xll(c, p, kSiteAttn, use & 1, c.rank) + u, v, (uint32_t)use + 1u);
    }
  }
  __device__ __forceinline__ void finish(Smem&, bool) const {}
};

// ================================================================== K4: router + MLP gate|up
// Staging bytes the top-k selection uses as scratch (router_done): E <= 256
// probabilities + kMaxTopK selected ones.
constexpr int kRouterScratchBytes = (kConsumerThreads + kMaxTopK) * 4;
struct RouterMlpOp : OpBase {
  Common c;
  const bf16_t* xres;      // layer input (world > 1 path reads it directly)
  bf16_t* resmid;          // out: residual after attention (CTA 0)
  bf16_t* h2;              // out: MoE input (CTA 0)
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
  int o_wpa, o_wff, o_wff2, o_wrs;  // staged constants
  int o_o, o_x;                     // staged activations: o_proj out (fp32), x (bf16)
  int block_mode;                   // 1: the input is already the MoE input (g4_moe_block)
  const bf16_t* block_x;
  int* ready;                       // step kernel: router flag of this layer (else null)

  __device__ __forceinline__ bool seg_dependent(int) const { return false; }
  __device__ __forceinline__ void load_dependent(Smem&) const {}
  template <class Fn>
  __device__ __forceinline__ void copies(int s, int u0, int n, const int*, Fn&& f) const {
    const uint32_t bytes = (uint32_t)(n * c.H * 2);
    if (s == 0) {
      f(router_w + (size_t)u0 * c.H, bytes, 0u);
    } else {
      f(gate + (size_t)u0 * c.H, bytes, 0u);
      f(up + (size_t)u0 * c.H, bytes, bytes);
    }
  }
  __device__ __forceinline__ bool prologue(Smem& sm) const {
    bool ok = true;
    const int H = c.H, tid = threadIdx.x;
    Vec hv;  // MoE input (model.py:315); the router input derives from it
    if (!block_mode) {
      // attention output (summed over ranks), then x = residual + rms(attn)*post_attn
      Vec t;
      if (c.world == 1) {
        load_f32(sf(sm, o_o), H, t);
      } else {
        // every rank's o_proj partial, summed in rank order (LL words, polled per chunk)
        const int use = site_use(ctrl, c, kSiteAttn, c.layer);
        const uint32_t tag = (uint32_t)use + 1u;
        bool got = true;
#pragma unroll
        for (int j = 0; j < kChunks; ++j) {
#pragma unroll
          for (int e = 0; e < 8; ++e) t[j][e] = 0.f;
          if (chunk_live(j, H))
            for (int src = 0; src < c.world; ++src) {
              float v[8];
              got = ll_get8(xll(c, c.rank, kSiteAttn, use & 1, src) + 8 * chunk_of(j), tag, v, ctrl) && got;
#pragma unroll
              for (int e = 0; e < 8; ++e) t[j][e] += v[e];
            }
        }
        ok = consumers_and(got) && ok;
        if (threadIdx.x == 0) G4_TRACE_EV(trace_id, 7);  // peer partials in (timeline: exchange wait)
      }
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          t[j][e] = rbf(t[j][e]);
          s += t[j][e] * t[j][e];
        }
      const float r = rms_scale(bsum1(s, sm, 0), H, c.eps);
      Vec w, xin;
      load_bf16(sbf(sm, o_wpa), H, w);
      load_bf16(sbf(sm, o_x), H, xin);
      float s2 = 0.f;
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          t[j][e] = rbf(xin[j][e] + rbf((t[j][e] * r) * w[j][e]));  // model.py:303-304
          s2 += t[j][e] * t[j][e];
        }
      if (blockIdx.x == 0) store_bf16(resmid, H, t);
      // MLP input (model.py:310) and MoE input (model.py:315)
      const float r2 = rms_scale(bsum1(s2, sm, 1), H, c.eps);
      Vec w2, xm;
      load_bf16(sbf(sm, o_wff), H, w);
      load_bf16(sbf(sm, o_wff2), H, w2);
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xm[j][e] = (t[j][e] * r2) * w[j][e];
          hv[j][e] = rbf((t[j][e] * r2) * w2[j][e]);
        }
      store_bf16(reinterpret_cast<bf16_t*>(sm.x1), H, xm);
    } else {
#pragma unroll
      for (int j = 0; j < kChunks; ++j) {
        uint4 u = make_uint4(0u, 0u, 0u, 0u);
        if (chunk_live(j, H)) u = __ldcg(reinterpret_cast<const uint4*>(block_x) + chunk_of(j));
        unpack8(u, hv[j]);
      }
    }
    if (blockIdx.x == 0) store_bf16(h2, H, hv);
    // router input: rms(h2) * scale * H^-1/2                 (model.py:225-226)
    float s3 = 0.f;
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) s3 += hv[j][e] * hv[j][e];
    const float r3 = rms_scale(bsum1(s3, sm, 2), H, c.eps);
    Vec ws, xr;
    load_bf16(sbf(sm, o_wrs), H, ws);
#pragma unroll
    for (int j = 0; j < kChunks; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) xr[j][e] = rbf(rbf(hv[j][e] * r3) * ws[j][e]) * hinv;
    store_bf16(reinterpret_cast<bf16_t*>(sm.x0), H, xr);
    if (tid == 0 && !sm.ints[kSmemRangesGiven]) {  // else the step kernel set them
      int ub, ue;
      cta_unit_range(seg, nseg, 0, blockIdx.x, gridDim.x, ub, ue);
      sm.ints[kSmemRouterEnd] = ub < ue ? ue : 0;
      sm.ints[kSmemRouterMine] = ue - ub;
    }
    return ok;
  }
  __device__ __forceinline__ void epilogue(int s, int u0, int n, const Res& res, Smem& sm, bool ok, int t) const {
    if (s == 0) {
      if (ok && t < n) router_logits[u0 + t] = rbf(res[t]);
      // right after this CTA's last router tile (identical test on every thread):
      // count its rows in; the CTA completing all E logits selects the top-k -- here in
      // the per-op kernel, after its grid-barrier arrival in the step kernel (whose
      // expert tiles wait for the router flag, not for the barrier)
      if (u0 + n == sm.ints[kSmemRouterEnd] && router_count(sm.ints[kSmemRouterMine], sm)) {
        if (sm.ints[kSmemRangesGiven]) {  // the step kernel (the per-op kernel sets 0)
          if (threadIdx.x == 0) sm.ints[kSmemTopk] = 1;  // read after the phase's closing barrier
        } else {
          router_topk(sm, reinterpret_cast<float*>(sm.stg));
        }
      }
    } else if (ok && t < n) {
      const float g = rbf(res[t]), u = rbf(res[n + t]);
      mlp_act[u0 + t] = f2bf(rbf(gelu_tanh(g)) * u);
    }
  }
  __device__ __forceinline__ void finish(Smem&, bool) const {}
  // The CTA that completes the router's E logits selects the top-k (model.py:227-232):
  // router_count, then router_topk.
  // Ordering: the acq_rel counter update after the block barrier publishes this CTA's
  // logits and, on the last CTA, acquires the others'; the flag store after the block
  // barrier releases top_idx / top_w.
  // The selection runs on every consumer thread of that CTA (expert e on thread e,
  // E <= kConsumerThreads), with the staging area -- free once the prologue has run --
  // as scratch: softmax max and sum by scans in expert order (identical on every
  // thread), then each probability's rank among all E (ties -> lower expert index,
  // like a stable top-k), the top-k weights summed in rank order.
  // Count this CTA's router rows in; true (on every consumer thread) on the CTA that
  // completes all E logits.
  __device__ __forceinline__ bool router_count(int mine, Smem& sm) const {
    named_bar(kBarReduce, kConsumerThreads);
    if (threadIdx.x == 0) {
      int last = 0;
      if (mine > 0) {
        int old = atomic_add_acq_rel_gpu(c.counters + kCntRouter, mine);
        last = (old + mine == E);
        if (last) atomicExch(c.counters + kCntRouter, 0);
      }
      sm.ints[kSmemLast] = last;
    }
    named_bar(kBarReduce, kConsumerThreads);
    const bool last = sm.ints[kSmemLast] != 0;
    named_bar(kBarReduce, kConsumerThreads);  // the flag slot is reused by later code
    return last;
  }
  // Softmax and top-k over the E logits (all consumer threads of the counting CTA), with
  // `scratch` (>= kConsumerThreads + kMaxTopK floats of shared memory), then the flag.
  __device__ __forceinline__ void router_topk(Smem& sm, float* scratch) const {
    const int t = threadIdx.x;
    const float scale = t < E ? bf2f(pes[t]) : 0.f;
    float* pv = scratch;                   // [E]
    float* top_p = pv + kConsumerThreads;  // [topk] selected probabilities, rank order
    float l = -INFINITY;
    if (t < E) {
      l = ldcg_f(router_logits + t);
      pv[t] = l;
    }
    named_bar(kBarReduce, kConsumerThreads);
    float mx = -INFINITY;
    for (int j = 0; j < E; ++j) mx = fmaxf(mx, pv[j]);
    const float ex = t < E ? expf(l - mx) : 0.f;
    named_bar(kBarReduce, kConsumerThreads);
    if (t < E) pv[t] = ex;
    named_bar(kBarReduce, kConsumerThreads);
    float sum = 0.f;
    for (int j = 0; j < E; ++j) sum += pv[j];
    const float p = ex / sum;
    named_bar(kBarReduce, kConsumerThreads);
    if (t < E) pv[t] = p;
    named_bar(kBarReduce, kConsumerThreads);
    int rank = 0;
    for (int j = 0; j < E; ++j) {
      const float q = pv[j];
      rank += (q > p || (q == p && j < t)) ? 1 : 0;
    }
    const bool sel = t < E && rank < topk;
    if (sel) top_p[rank] = p;
    named_bar(kBarReduce, kConsumerThreads);
    if (sel) {
      float wsum = 0.f;
      for (int k = 0; k < topk; ++k) wsum += top_p[k];
      top_idx[rank] = t;
      top_w[rank] = (p / wsum) * scale;
    }
    named_bar(kBarReduce, kConsumerThreads);
    if (t == 0 && ready)  // the step kernel's producers wait for this flag
      st_release_gpu(ready, sm.ints[kSmemSeq] + 1);
  }
};

// ================================================================== K5: MLP down + expert gate|up
__device__ __forceinline__ void load_expert_ids(const int* top_idx, int topk, Smem& sm) {
  int e[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) e[k] = k < topk ? ldcg_i(top_idx + k) : 0;  // all in flight
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k)
    if (k < topk) sm.ints[kSmemExp + k] = e[k];
}

struct MoeUpOp : OpBase {
  Common c;
  const int* top_idx;      // [K]
  const float* top_w;      // [K]
  const bf16_t* mlp_down;  // [H, I_local]
  const bf16_t* gate_up;   // [E, 2, F, H]
  float* mlp_out;          // out: fp32 [H]
  bf16_t* moe_act;         // out: [K, F]
  int I, F, topk;
  int o_h2, o_act;         // staged activations (bf16)

  __device__ __forceinline__ bool seg_dependent(int s) const { return s == 1; }
  __device__ __forceinline__ void load_dependent(Smem& sm) const { load_expert_ids(top_idx, topk, sm); }
  template <class Fn>
  __device__ __forceinline__ void copies(int s, int u0, int n, const int* ids, Fn&& f) const {
    if (s == 0) {
      f(mlp_down + (size_t)u0 * I, (uint32_t)(n * I * 2), 0u);
    } else {
      const int k = u0 / F, f0 = u0 % F;
      const size_t e = (size_t)ids[k];
      const uint32_t bytes = (uint32_t)(n * c.H * 2);
      f(gate_up + ((e * 2 + 0) * F + f0) * c.H, bytes, 0u);
      f(gate_up + ((e * 2 + 1) * F + f0) * c.H, bytes, bytes);
    }
  }
  __device__ __forceinline__ bool prologue(Smem& sm) const {
    copy_vec(sbf(sm, o_h2), c.H, sm.x0);
    copy_vec(sbf(sm, o_act), I, sm.x1);
    return true;
  }
  __device__ __forceinline__ void epilogue(int s, int u0, int n, const Res& res, Smem& sm, bool ok, int t) const {
    if (!ok || t >= n) return;
    if (s == 0) {
      mlp_out[u0 + t] = res[t];
    } else {
      const int u = u0 + t, k = u / F;
      const float g = rbf(res[t]), up = rbf(res[n + t]);
      // the routing weight: read here, behind this expert's tiles, which the producer
      // issued only after it saw the router flag (the step kernel selects the top-k after
      // the phase barrier; the mbarrier wait orders this load after that flag)
      const float w = ldcg_f(top_w + k);
      // gelu(g) * u * w, left to right in bf16 (model.py:271)
      moe_act[u] = f2bf(rbf(rbf(gelu_tanh(g)) * up) * rbf(w));
    }
  }
  __device__ __forceinline__ void finish(Smem&, bool) const {}
};

// ================================================================== K6: expert down
struct MoeDownOp : OpBase {
  Common c;
  const int* top_idx;
  const bf16_t* down;     // [E, H, F]
  const float* mlp_out;   // world>1: this rank's MLP partial, sent with the MoE partial
  bf16_t* moe_out;        // world==1: bf16 [H]
  int F, topk;
  int o_act;              // staged expert activations (bf16 [K, F])

  __device__ __forceinline__ bool seg_dependent(int) const { return true; }
  __device__ __forceinline__ void load_dependent(Smem& sm) const { load_expert_ids(top_idx, topk, sm); }
  template <class Fn>
  __device__ __forceinline__ void copies(int, int u0, int n, const int* ids, Fn&& f) const {
    const uint32_t bytes = (uint32_t)(n * F * 2);
    for (int k = 0; k < topk; ++k) {
      const size_t e = (size_t)ids[k];
      f(down + (e * c.H + u0) * F, bytes, (uint32_t)k * bytes);
    }
  }
  __device__ __forceinline__ bool prologue(Smem& sm) const {
    copy_vec(sbf(sm, o_act), topk * F, sm.x0);
    return true;
  }
  __device__ __forceinline__ void epilogue(int, int u0, int n, const Res& res, Smem&, bool ok, int t) const {
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
      const int use = site_use(ctrl, c, kSiteFfn, c.layer);
      const uint32_t tag = (uint32_t)use + 1u;
      for (int p = 0; p < c.world; ++p) {
        unsigned long long* sl = xll(c, p, kSiteFfn, use & 1, c.rank);
        ll_put(sl + u, mv, tag);
        ll_put(sl + c.H + u, sacc, tag);
      }
    }
  }
  __device__ __forceinline__ void finish(Smem&, bool) const {}
};

// ================================================================== LM head + argmax
struct LmHeadOp : OpBase {
  Common c;
  Tail tail;
  int o_wn;              // staged final norm weight
  const bf16_t* embed;   // replicated [V, H]; this rank reads rows [vbegin, vbegin+V_local)
  int vbegin;
  float* logits;         // [V_local] fp32 (written when control[WRITE_LOGITS] != 0)
  float* cand_v;         // scratch [gridDim]
  int* cand_i;           // scratch [gridDim]
  int* tokens_out;       // [max_len + 1]
  int* tokens_host;      // optional mapped pinned host mirror of tokens_out
  int max_len;
  float softcap;         // <= 0: none

  __device__ __forceinline__ bool seg_dependent(int) const { return false; }
  __device__ __forceinline__ void load_dependent(Smem&) const {}
  template <class Fn>
  __device__ __forceinline__ void copies(int, int u0, int n, const int*, Fn&& f) const {
    f(embed + (size_t)(vbegin + u0) * c.H, (uint32_t)(n * c.H * 2), 0u);
  }
  __device__ __forceinline__ bool prologue(Smem& sm) const {
    Vec x;
    const bool ok = layer_output(ctrl, c, tail, sm, x, trace_id);
    norm_into(c, x, sbf(sm, o_wn), reinterpret_cast<bf16_t*>(sm.x0), sm, 3);
    float* bv = reinterpret_cast<float*>(sm.x1);
    int* bi = reinterpret_cast<int*>(sm.x1) + kConsumerThreads;
    bv[threadIdx.x] = -INFINITY;
    bi[threadIdx.x] = 0x7fffffff;
    // the sampler (temperature > 0) reads the logits this step writes
    sm.ints[kSmemWriteLogits] = ldcg_i(ctrl + G4_CTRL_WRITE_LOGITS) != 0 ||
                                __int_as_float(ldcg_i(ctrl + G4_CTRL_TEMPERATURE)) > 0.f;
    named_bar(kBarReduce, kConsumerThreads);
    return ok;
  }
  __device__ __forceinline__ void epilogue(int, int u0, int n, const Res& res, Smem& sm, bool ok, int t) const {
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
  __device__ __forceinline__ void finish(Smem& sm, bool ok) const {
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
    if (!sm.ints[kSmemLast] || threadIdx.x >= 32) return;
    // last CTA: one warp reduces the per-CTA candidates (max value, then lowest index)
    __threadfence();
    float v = -INFINITY;
    int ix = 0x7fffffff;
    for (int b = threadIdx.x; b < (int)gridDim.x; b += 32) {
      const float cv = ldcg_f(cand_v + b);
      const int ci = ldcg_i(cand_i + b);
      if (cv > v || (cv == v && ci < ix)) {
        v = cv;
        ix = ci;
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
    if (threadIdx.x != 0) return;
    atomicExch(c.counters + kCntLm, 0);
    int token = ix == 0x7fffffff ? 0 : vbegin + ix;
    if (c.world > 1) {
      const int use = site_use(ctrl, c, kSiteArgmax, 0);
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
    if (pos < 0 || pos >= max_len) {  // the step consumed no valid position
      atomicOr(ctrl + G4_CTRL_STATUS, G4_STATUS_POS_OVERFLOW);
      return;
    }
    tokens_out[pos + 1] = token;
    if (tokens_host) tokens_host[pos + 1] = token;
    ctrl[G4_CTRL_POS] = pos + 1;
    ctrl[G4_CTRL_STEP] = ldcg_i(ctrl + G4_CTRL_STEP) + 1;
    (void)ok;
  }
};

}  // namespace g4
