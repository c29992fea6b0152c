// Device-side stochastic sampling of the next token (reference: gemma4_tpu/model.py:414-424,
// keyed per position as engine.py:66 / :80 do).
//
// Runs after the decode step, whose LM head has written this rank's fp32 softcapped logits
// (its vocab slice) and the greedy token.  With temperature > 0 it replaces that token by
// a sample of
//     top_k(logits / t, K) -> softmax -> keep while (cumsum - p) < top_p -> renormalise
// and leaves greedy decoding (temperature <= 0) untouched, like the reference's
// `where(temperature <= 0, greedy, sampled)`.
//
//  1. grid = ceil(V_local / kSampleChunk) CTAs: each sorts its chunk of logits / t
//     (bitonic sort in shared memory, descending value, ascending index on ties -- the
//     order of a stable top-k) and writes its first K (value, vocab index) candidates;
//  2. the last CTA (acq_rel counter) merges all candidates the same way; with world > 1
//     each rank's K best go to every peer through the exchange buffer and every rank
//     merges all world x K in rank order, so every rank selects the same token;
//  3. one warp computes the softmax, the top-p mask (cumulative sum in rank order) and
//     the renormalised probabilities, and draws u in [0, 1) from a counter-based
//     generator: Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers:
//     as easy as 1, 2, 3", SC 2011) keyed by the 64-bit seed, counter = (position, 0,
//     0, 0) where position is 0 for the token that ends the prompt (the reference folds
//     0 into the key for the prefill sample) and the consumed position for decode steps.
//     The token is the first k whose cumulative renormalised probability exceeds u
//     (inverse CDF).  The distribution equals the reference's categorical draw; the
//     random stream differs from JAX's threefry (parity is distribution-level).
#pragma once

#include "g4_ops.cuh"

namespace g4 {

constexpr int kSampleThreads = 256;
constexpr int kSampleChunk = 4096;  // logits sorted per CTA
constexpr int kSampleMaxK = 128;
constexpr int kSampleMaxCtas = 128; // => V_local <= 128 * 4096 = 524288
constexpr int kCntSample = 4;       // counter slot (Common::counters)

struct SampleArgs {
  const float* logits;  // [V_local] fp32 softcapped logits of this rank's vocab slice
  int V_local, vbegin, max_len;
  int* ctrl;
  int* tokens_out;      // [max_len + 1]
  int* tokens_host;     // optional mapped host mirror
  float* cand_v;        // [gridDim * kSampleMaxK]
  int* cand_i;
  Common c;             // counters, exchange buffer (world > 1)
};

__host__ __device__ __forceinline__ int sample_smem_bytes() {
  return kSampleChunk * 8 > kSampleMaxCtas * kSampleMaxK * 8 ? kSampleChunk * 8 : kSampleMaxCtas * kSampleMaxK * 8;
}

// (value desc, index asc): a goes before b
__device__ __forceinline__ bool sample_before(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// In-place bitonic sort of n (power of two) pairs in shared memory, first = best.
__device__ __forceinline__ void bitonic_sort(float* v, int* ix, int n) {
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < n / 2; t += blockDim.x) {
        const int lo = 2 * t - (t & (stride - 1));  // index with bit `stride` clear
        const int hi = lo + stride;
        const bool desc_block = (lo & size) == 0;   // this run sorts best-first
        const bool swap = desc_block ? sample_before(v[hi], ix[hi], v[lo], ix[lo])
                                     : sample_before(v[lo], ix[lo], v[hi], ix[hi]);
        if (swap) {
          const float tv = v[lo];
          v[lo] = v[hi];
          v[hi] = tv;
          const int ti = ix[lo];
          ix[lo] = ix[hi];
          ix[hi] = ti;
        }
      }
      __syncthreads();
    }
  }
}

__device__ __forceinline__ uint32_t mulhi32(uint32_t a, uint32_t b) { return __umulhi(a, b); }

// Philox-4x32 with 10 rounds (Salmon et al. 2011): multipliers 0xD2511F53 / 0xCD9E8D57,
// key schedule increments 0x9E3779B9 / 0xBB67AE85.
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t ctr[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    const uint32_t a = ctr[0], b = ctr[2];
    const uint64_t p0 = (uint64_t)0xD2511F53u * a, p1 = (uint64_t)0xCD9E8D57u * b;
    const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    const uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    ctr[0] = hi1 ^ ctr[1] ^ k0;
    ctr[1] = lo1;
    ctr[2] = hi0 ^ ctr[3] ^ k1;
    ctr[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Uniform in [0, 1): the top 24 bits of the first Philox output word.
__host__ __device__ __forceinline__ float sample_uniform(uint64_t seed, uint32_t position) {
  uint32_t c[4] = {position, 0u, 0u, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(c[0] >> 8) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float ctrl_float(const int* ctrl, int word) { return __int_as_float(ldcg_i(ctrl + word)); }

// (internal linkage: every translation unit that includes this header launches its own copy)
static __global__ void __launch_bounds__(kSampleThreads) sample_kernel(const __grid_constant__ SampleArgs a) {
  extern __shared__ __align__(16) unsigned char sample_smem[];
  pdl_wait();
  const float temp = ctrl_float(a.ctrl, G4_CTRL_TEMPERATURE);
  const int pos = ldcg_i(a.ctrl + G4_CTRL_POS) - 1;  // position the step consumed
  const int forced = ldcg_i(a.ctrl + G4_CTRL_FORCED_LEN);
  // greedy, a prompt position whose output is not used, or a step that wrote nothing
  if (!(temp > 0.f) || pos < forced - 1 || pos < 0 || pos >= a.max_len) return;
  int K = ldcg_i(a.ctrl + G4_CTRL_TOP_K);
  if (K < 1) K = 1;
  if (K > kSampleMaxK) K = kSampleMaxK;
  float* sv = reinterpret_cast<float*>(sample_smem);
  int* si = reinterpret_cast<int*>(sample_smem + kSampleChunk * 4);
  const int base = blockIdx.x * kSampleChunk;
  for (int i = threadIdx.x; i < kSampleChunk; i += blockDim.x) {
    const int u = base + i;
    sv[i] = u < a.V_local ? ldcg_f(a.logits + u) / temp : -INFINITY;
    si[i] = u < a.V_local ? a.vbegin + u : 0x7fffffff;
  }
  __syncthreads();
  bitonic_sort(sv, si, kSampleChunk);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    a.cand_v[blockIdx.x * kSampleMaxK + k] = sv[k];
    a.cand_i[blockIdx.x * kSampleMaxK + k] = si[k];
  }
  __threadfence();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) {
    const int old = atomic_add_acq_rel_gpu(a.c.counters + kCntSample, 1);
    last = old == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (!last) return;
  // ---- merge the CTAs' candidates (this rank's best K)
  int n = 1;
  while (n < (int)gridDim.x * K) n <<= 1;
  float* mv = reinterpret_cast<float*>(sample_smem);
  int* mi = reinterpret_cast<int*>(sample_smem + n * 4);  // (re-carved for the world merge)
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int b = i / K, k = i % K;
    const bool live = i < (int)gridDim.x * K;
    mv[i] = live ? ldcg_f(a.cand_v + b * kSampleMaxK + k) : -INFINITY;
    mi[i] = live ? ldcg_i(a.cand_i + b * kSampleMaxK + k) : 0x7fffffff;
  }
  __syncthreads();
  bitonic_sort(mv, mi, n);
  if (threadIdx.x == 0) atomicExch(a.c.counters + kCntSample, 0);
  __shared__ int ok;
  if (a.c.world > 1) {
    // every rank's K best to every peer (slot of this rank), then all world x K merged
    const int use = ldcg_i(a.ctrl + G4_CTRL_STEP);
    for (int p = 0; p < a.c.world; ++p) {
      float* sl = xslot(a.c, p, kSiteSample, use & 1, a.c.rank);
      for (int k = threadIdx.x; k < K; k += blockDim.x) {
        sl[2 * k] = mv[k];
        reinterpret_cast<int*>(sl)[2 * k + 1] = mi[k];
      }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
      for (int p = 0; p < a.c.world; ++p) st_release_sys(xflag(a.c, p, kSiteSample, use & 1, a.c.rank), use + 1);
      int good = 1;
      const int tmo = ldcg_i(a.ctrl + G4_CTRL_TIMEOUT_US);
      for (int src = 0; src < a.c.world && good; ++src)
        good = wait_flag_geq(xflag(a.c, a.c.rank, kSiteSample, use & 1, src), use + 1, tmo,
                             a.ctrl + G4_CTRL_STATUS);
      ok = good;
    }
    __syncthreads();
    if (!ok) return;  // the greedy token stays; the status bit reports the timeout
    n = 1;
    while (n < a.c.world * K) n <<= 1;
    // re-carve the value / index arrays for the new length (this rank's K best already
    // sit in the exchange slots, so the old arrays are no longer read)
    mv = reinterpret_cast<float*>(sample_smem);
    mi = reinterpret_cast<int*>(sample_smem + n * 4);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int src = i / K, k = i % K;
      const bool live = i < a.c.world * K;
      const float* sl = xslot(a.c, a.c.rank, kSiteSample, use & 1, live ? src : 0);
      mv[i] = live ? ldcg_f(sl + 2 * k) : -INFINITY;
      mi[i] = live ? ldcg_i(reinterpret_cast<const int*>(sl) + 2 * k + 1) : 0x7fffffff;
    }
    __syncthreads();
    bitonic_sort(mv, mi, n);
  }
  // ---- softmax over the K best, top-p mask, renormalise, inverse-CDF draw (one thread:
  // K <= 128 sequential steps, a fixed order)
  if (threadIdx.x != 0) return;
  const float top_p = ctrl_float(a.ctrl, G4_CTRL_TOP_P);
  const float mx = mv[0];
  float sum = 0.f;
  for (int k = 0; k < K; ++k) sum += expf(mv[k] - mx);
  float csum = 0.f, kept = 0.f;
  int nkeep = 0;
  for (int k = 0; k < K; ++k) {
    const float p = expf(mv[k] - mx) / sum;
    csum += p;
    if (csum - p < top_p) {  // model.py:421
      kept += p;
      nkeep = k + 1;
    } else {
      break;  // probabilities are in decreasing order: the cumulative test fails from here on
    }
  }
  if (nkeep == 0) nkeep = 1;
  const uint32_t position = pos == forced - 1 ? 0u : (uint32_t)pos;
  const uint64_t seed = (uint64_t)(uint32_t)ldcg_i(a.ctrl + G4_CTRL_SEED_LO) |
                        ((uint64_t)(uint32_t)ldcg_i(a.ctrl + G4_CTRL_SEED_HI) << 32);
  const float u = sample_uniform(seed, position) * kept;  // inverse CDF on the kept mass
  float acc = 0.f;
  int token = mi[nkeep - 1];
  for (int k = 0; k < nkeep; ++k) {
    acc += expf(mv[k] - mx) / sum;
    if (u < acc) {
      token = mi[k];
      break;
    }
  }
  a.tokens_out[pos + 1] = token;
  if (a.tokens_host) a.tokens_host[pos + 1] = token;
}

}  // namespace g4
