// Internal declarations shared by the translation units of libg4b200 (not installed;
// the public interface is include/g4b200.h): the model and communicator objects, the
// error helper and launch helpers.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <string>
#include <vector>

#include "g4_attention.cuh"
#include "g4_ops.cuh"
#include "g4_sample.cuh"
#include "g4_step.cuh"

using namespace g4;

// ------------------------------------------------------------------ errors
// Sets the calling thread's last-error message (g4_last_error) and returns `code`.
int g4_fail(int code, const char* fmt, ...);
#define fail g4_fail

#define G4_CUDA(call, code)                                                              \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(code, "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                  __LINE__);                                                             \
  } while (0)

// ------------------------------------------------------------------ communicator
struct g4_comm {
  int device = 0, rank = 0, world = 1, hidden = 0;
  size_t bytes = 0;
  char* local = nullptr;
  char* peer[kMaxWorld] = {};
  bool mapped[kMaxWorld] = {};
  bool open = false;
  int pf_seq = 0;  // tensor-parallel prefill exchanges done (the same count on every rank)
};

// Tensor-parallel prefill exchange: the end of every communicator buffer holds kMaxWorld
// arrival flags (128 bytes apart) and two parity slots of kPfXRows x 2 * hidden fp32.
constexpr int kPfXRows = 4096;  // prompt rows per chunk under tensor parallelism
size_t g4_comm_pf_offset(int hidden);  // byte offset of that region (g4_runtime.cu)

// ------------------------------------------------------------------ launch helper
template <class Kernel, class... Args>
inline cudaError_t launch_pdl(Kernel k, dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

struct PrefillWs;  // g4_prefill.cu
struct BatchWs;    // g4_prefill.cu

// ------------------------------------------------------------------ model
struct LayerDev {
  bool full = false;
  int d = 0, n_kv = 0, g = 0, rows_q = 0, rows_k = 0, rows_v = 0, k_eq_v = 0, nsplit = 1;
  bf16_t *qkv = nullptr, *o = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
  bf16_t *router = nullptr, *router_scale = nullptr, *pes = nullptr, *exp_gu = nullptr,
         *exp_down = nullptr;
  bf16_t *n_in = nullptr, *n_post_attn = nullptr, *n_pre_ff = nullptr, *n_post_ff = nullptr,
         *n_pre_ff2 = nullptr, *n_post_ff1 = nullptr, *n_post_ff2 = nullptr;
  bf16_t *q_norm = nullptr, *k_norm = nullptr, *scalar = nullptr;
  bf16_t *cache_k = nullptr, *cache_v = nullptr;
};

struct g4_model {
  g4_config cfg{};
  std::vector<unsigned char> is_full;
  int rank = 0, world = 1, max_len = 0, device = 0, nsm = 148;
  int H = 0, I_local = 0, F_local = 0, V_local = 0, vbegin = 0, E = 0, topk = 0;
  std::vector<LayerDev> L;
  bf16_t *embed = nullptr, *final_norm = nullptr;
  int *ctrl = nullptr, *tokens_in = nullptr, *tokens_out = nullptr;
  float* logits = nullptr;
  g4_comm* comm = nullptr;
  g4_comm* own_comm = nullptr;  // world == 1 without an attached communicator
  // library scratch
  char* scratch = nullptr;
  bf16_t *xres, *resmid, *h2, *qkv_raw, *ctx, *mlp_act, *moe_act, *moe_out;
  float *o_out, *mlp_out, *router_logits, *top_w, *attn_part, *cand_v, *samp_v;
  int *top_idx, *attn_cnt, *cand_i, *counters, *samp_i;
  bool finalized = false;
  // plans
  std::vector<QkvOp> k1;
  std::vector<AttnArgs> k2;
  std::vector<OProjOp> k3;
  std::vector<RouterMlpOp> k4;
  std::vector<MoeUpOp> k5;
  std::vector<MoeDownOp> k6;
  LmHeadOp lm{};
  SampleArgs sampler{};  // temperature > 0: replaces the greedy token after the LM head
  int sample_ctas = 0;
  // persistent step kernel
  int engine = G4_ENGINE_STEP_KERNEL;
  StepProgram prog{};
  int step_cplm = 0;
  const void* step_kernel = nullptr;
  char* prog_mem = nullptr;  // device copies of the operator plans
  bool prog_dirty = true;    // host plans changed since the last upload
  int* sync = nullptr;       // kNumSyncWords (library scratch)
  float* rope_tab = nullptr;
  int* tokens_host = nullptr;  // mapped pinned mirror of tokens_out (g4_model_host_tokens)
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t gexec = nullptr;
  PrefillWs* prefill = nullptr;  // prefill workspace (g4_prefill), allocated on first use
  BatchWs* batch = nullptr;      // batched decoder (g4_batch_reserve)
};

// Launch the sampler after a step's (or the prefill's) LM head (g4_runtime.cu).
int g4_launch_sampler(const g4_model* m, cudaStream_t st);
int g4_prepare_sampler(const g4_model* m);
// Free the prefill workspace (g4_prefill.cu).
void g4_prefill_release(g4_model* m);
// Free the batched decoder's caches and buffers (g4_prefill.cu).
void g4_batch_release(g4_model* m);
// Launch one decode-attention item grid (g4_runtime.cu).
int g4_launch_attention(const AttnArgs& a, cudaStream_t st);
// One decode-attention launch over several sequences: grid = seqs x items, the sequences'
// args in the device array `dargs` (g4_runtime.cu).
int g4_launch_attention_batch(const AttnArgs* dargs, int d, int g, int seqs, int items, cudaStream_t st);
// Splits per KV head of a decode-attention layer for `nsm` SMs (g4_runtime.cu).
int g4_pick_nsplit(int n_kv, int max_live, int nsm);
// Encode a.tmk / a.tmv from a.cache_k / a.cache_v, n_kv, d and max_len (g4_runtime.cu).
int g4_attention_maps(AttnArgs& a);
// A K-major bf16 matrix [rows, inner] (row stride `ld` elements) as a TMA tensor map with
// boxes of 64 elements x box_rows rows, 128-byte swizzle (g4_prefill.cu).
int g4_make_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t ld,
                   uint32_t box_rows);
// model.py:54-61: fp64 inverse frequencies of the rotated pairs, zero (NoPE) tail.
void g4_rope_inv_freq(int d, double theta, double partial, float* out);
float g4_host_bf16_round(float f);
