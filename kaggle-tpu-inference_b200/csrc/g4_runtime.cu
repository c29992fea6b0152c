// Host runtime of g4b200: communicator, model plan, step launcher, graph capture and
// the C ABI declared in include/g4b200.h.
//
// A decode step runs in one of two engines over the same operator plans:
//   G4_ENGINE_STEP_KERNEL (default): one persistent cooperative launch per token
//     (g4_step.cuh) with a single weight ring across all operators;
//   G4_ENGINE_OP_KERNELS: 6 kernels per layer + 1 (embedding fused into layer 0's
//     first kernel, the argmax into the lm_head kernel), chained with programmatic
//     dependent launches.
// Either step is captured once into a CUDA graph and replayed per token.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "g4_internal.h"

// ------------------------------------------------------------------ errors
static thread_local std::string g_last_error;

int g4_fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

extern "C" const char* g4_version(void) { return "g4b200 0.1 sm_100a"; }

extern "C" const char* g4_strerror(int code) {
  switch (code) {
    case G4_OK: return "ok";
    case G4_ERR_ARG: return "invalid argument";
    case G4_ERR_SHAPE: return "unsupported shape";
    case G4_ERR_LAUNCH: return "kernel launch failed";
    case G4_ERR_TIMEOUT: return "bounded device wait timed out";
    case G4_ERR_STATE: return "invalid call order";
    case G4_ERR_NOMEM: return "device allocation failed";
    case G4_ERR_CUDA: return "CUDA error";
    default: return "unknown error";
  }
}

extern "C" const char* g4_last_error(void) { return g_last_error.c_str(); }

// Flags, then [site][parity][source rank] slots of 4 * hidden floats (the FFN-out site
// carries 2 * hidden LL words of 8 bytes), then the tensor-parallel prefill exchange:
// kMaxWorld flags of 128 bytes and two parity slots of kPfXRows x 2 * hidden fp32.
size_t g4_comm_pf_offset(int hidden) {
  return (size_t)kXFlagBytes + (size_t)kSites * 2 * kMaxWorld * (4 * (size_t)hidden) * 4;
}
static size_t comm_bytes(int hidden) {
  return g4_comm_pf_offset(hidden) + (size_t)kMaxWorld * 128 + 2 * (size_t)kPfXRows * 2 * hidden * 4;
}

extern "C" int g4_comm_create(int device, int rank, int world, int hidden, g4_comm** out) {
  if (!out || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || hidden <= 0)
    return fail(G4_ERR_ARG, "g4_comm_create: bad rank/world/hidden (%d/%d/%d)", rank, world, hidden);
  G4_CUDA(cudaSetDevice(device), G4_ERR_CUDA);
  g4_comm* c = new g4_comm();
  c->device = device;
  c->rank = rank;
  c->world = world;
  c->hidden = hidden;
  c->bytes = comm_bytes(hidden);
  if (cudaMalloc(&c->local, c->bytes) != cudaSuccess) {
    delete c;
    return fail(G4_ERR_NOMEM, "g4_comm_create: cudaMalloc(%zu) failed", comm_bytes(hidden));
  }
  cudaMemset(c->local, 0, c->bytes);
  cudaDeviceSynchronize();
  c->peer[rank] = c->local;
  c->open = (world == 1);
  *out = c;
  return G4_OK;
}

extern "C" int g4_comm_get_handle(const g4_comm* c, void* handle_out) {
  if (!c || !handle_out) return fail(G4_ERR_ARG, "g4_comm_get_handle: null argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
  G4_CUDA(cudaSetDevice(c->device), G4_ERR_CUDA);
  cudaIpcMemHandle_t h;
  G4_CUDA(cudaIpcGetMemHandle(&h, c->local), G4_ERR_CUDA);
  memcpy(handle_out, &h, 64);
  return G4_OK;
}

extern "C" int g4_comm_open(g4_comm* c, const void* handles) {
  if (!c || (!handles && c->world > 1)) return fail(G4_ERR_ARG, "g4_comm_open: null argument");
  G4_CUDA(cudaSetDevice(c->device), G4_ERR_CUDA);
  for (int p = 0; p < c->world; ++p) {
    if (p == c->rank || c->mapped[p]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char*>(handles) + 64 * p, 64);
    void* ptr = nullptr;
    G4_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), G4_ERR_CUDA);
    c->peer[p] = static_cast<char*>(ptr);
    c->mapped[p] = true;
  }
  c->open = true;
  return G4_OK;
}

extern "C" int g4_comm_open_local(g4_comm* const* comms, int n) {
  if (!comms || n < 1 || n > kMaxWorld) return fail(G4_ERR_ARG, "g4_comm_open_local: bad communicator list");
  for (int r = 0; r < n; ++r) {
    const g4_comm* c = comms[r];
    if (!c || c->world != n || c->rank != r || c->hidden != comms[0]->hidden)
      return fail(G4_ERR_ARG, "g4_comm_open_local: communicator %d is not rank %d of world %d", r, r, n);
    for (int q = 0; q < r; ++q)
      if (comms[q]->device == c->device)
        return fail(G4_ERR_ARG, "g4_comm_open_local: ranks %d and %d share device %d", q, r, c->device);
  }
  for (int r = 0; r < n; ++r) {
    g4_comm* c = comms[r];
    G4_CUDA(cudaSetDevice(c->device), G4_ERR_CUDA);
    for (int p = 0; p < n; ++p) {
      if (p == r) continue;
      int can = 0;
      G4_CUDA(cudaDeviceCanAccessPeer(&can, c->device, comms[p]->device), G4_ERR_CUDA);
      if (!can) return fail(G4_ERR_CUDA, "device %d cannot access device %d", c->device, comms[p]->device);
      const cudaError_t e = cudaDeviceEnablePeerAccess(comms[p]->device, 0);
      if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();  // clear the sticky-free error
      else if (e != cudaSuccess)
        return fail(G4_ERR_CUDA, "cudaDeviceEnablePeerAccess(%d -> %d): %s", c->device, comms[p]->device,
                    cudaGetErrorString(e));
      c->peer[p] = comms[p]->local;  // same process: the peer's own allocation, no IPC mapping
    }
    c->open = true;
  }
  return G4_OK;
}

extern "C" int g4_comm_destroy(g4_comm* c) {
  if (!c) return G4_OK;
  cudaSetDevice(c->device);
  for (int p = 0; p < c->world; ++p)
    if (c->mapped[p]) cudaIpcCloseMemHandle(c->peer[p]);
  if (c->local) cudaFree(c->local);
  delete c;
  return G4_OK;
}

template <class Op, int CPLM>
static int prepare_kernel(int smem) {
  static std::mutex mu;
  static std::map<int, int> done;  // device -> max smem configured
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev] >= smem) return G4_OK;
  G4_CUDA(cudaFuncSetAttribute(gemv_kernel<Op, CPLM>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
          G4_ERR_LAUNCH);
  done[dev] = smem;
  return G4_OK;
}

// Register bucket (max input chunks per lane) of an operator's launch.
template <class Op>
static int op_cplm(const Op& op) {
  int m = 1;
  for (int s = 0; s < op.nseg; ++s)
    if (op.seg[s].units > 0 && seg_cpl(op.seg[s]) > m) m = seg_cpl(op.seg[s]);
  return m <= 4 ? 4 : (m <= 8 ? 8 : (m <= 12 ? 12 : (m <= 16 ? 16 : 0)));
}

// The attention kernel instantiation for (head dim, query heads per KV head).
typedef void (*AttnKernel)(AttnArgs);
template <int D>
static AttnKernel attn_kernel_for_g(int g) {
  switch (g) {
    case 1: return attn_decode_kernel<D, 1>;
    case 2: return attn_decode_kernel<D, 2>;
    case 4: return attn_decode_kernel<D, 4>;
    case 8: return attn_decode_kernel<D, 8>;
    default: return nullptr;
  }
}
static AttnKernel attn_kernel_for(int d, int g) {
  switch (d) {
    case 64: return attn_kernel_for_g<64>(g);
    case 128: return attn_kernel_for_g<128>(g);
    case 256: return attn_kernel_for_g<256>(g);
    case 512: return attn_kernel_for_g<512>(g);
    default: return nullptr;
  }
}

static int prepare_attention(int d, int g) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> done;
  int dev = 0;
  cudaGetDevice(&dev);
  AttnKernel k = attn_kernel_for(d, g);
  if (!k) return fail(G4_ERR_SHAPE, "attention: head_dim %d with %d query heads per KV head", d, g);
  const int smem = attn_kernel_smem_bytes(d);
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{dev, d * 16 + g}];
  if (have >= smem) return G4_OK;
  G4_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), G4_ERR_LAUNCH);
  have = smem;
  return G4_OK;
}

template <class Op, int CPLM>
static int launch_gemv_t(const Op& op, int grid, cudaStream_t st) {
  const int smem = gemv_smem_bytes(smem_aux_bytes(SmemSizes{op.xbytes[0], op.xbytes[1], op.stgbytes}), kStages);
  int rc = prepare_kernel<Op, CPLM>(smem);
  if (rc) return rc;
  cudaError_t e = launch_pdl(gemv_kernel<Op, CPLM>, dim3(grid), dim3(kGemvThreads), smem, st, op);
  if (e != cudaSuccess) return fail(G4_ERR_LAUNCH, "gemv launch: %s", cudaGetErrorString(e));
  return G4_OK;
}

template <class Op>
static int launch_gemv(const Op& op, int grid, cudaStream_t st) {
  switch (op_cplm(op)) {
    case 4: return launch_gemv_t<Op, 4>(op, grid, st);
    case 8: return launch_gemv_t<Op, 8>(op, grid, st);
    case 12: return launch_gemv_t<Op, 12>(op, grid, st);
    case 16: return launch_gemv_t<Op, 16>(op, grid, st);
    default: return fail(G4_ERR_SHAPE, "a matrix row is longer than 4096 elements on this rank");
  }
}

static int launch_attention(const AttnArgs& a, cudaStream_t st) {
  int rc = prepare_attention(a.d, a.g);
  if (rc) return rc;
  cudaError_t e = launch_pdl(attn_kernel_for(a.d, a.g), dim3(a.n_kv * a.nsplit), dim3(kAttnKernelThreads),
                             attn_kernel_smem_bytes(a.d), st, a);
  if (e != cudaSuccess) return fail(G4_ERR_LAUNCH, "attention launch: %s", cudaGetErrorString(e));
  return G4_OK;
}
int g4_launch_attention(const AttnArgs& a, cudaStream_t st) { return launch_attention(a, st); }

// The batched attention kernel for (head dim, query heads per KV head).
typedef void (*AttnBatchKernel)(const AttnArgs*, int);
template <int D>
static AttnBatchKernel attn_batch_kernel_for_g(int g) {
  switch (g) {
    case 1: return attn_decode_batch_kernel<D, 1>;
    case 2: return attn_decode_batch_kernel<D, 2>;
    case 4: return attn_decode_batch_kernel<D, 4>;
    case 8: return attn_decode_batch_kernel<D, 8>;
    default: return nullptr;
  }
}
static AttnBatchKernel attn_batch_kernel_for(int d, int g) {
  switch (d) {
    case 64: return attn_batch_kernel_for_g<64>(g);
    case 128: return attn_batch_kernel_for_g<128>(g);
    case 256: return attn_batch_kernel_for_g<256>(g);
    case 512: return attn_batch_kernel_for_g<512>(g);
    default: return nullptr;
  }
}

int g4_launch_attention_batch(const AttnArgs* dargs, int d, int g, int seqs, int items, cudaStream_t st) {
  AttnBatchKernel k = attn_batch_kernel_for(d, g);
  if (!k) return fail(G4_ERR_SHAPE, "batched attention: head_dim %d with %d query heads per KV head", d, g);
  const int smem = attn_kernel_smem_bytes(d);
  {
    static std::mutex mu;
    static std::map<std::pair<int, int>, int> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    int& have = done[{dev, d * 16 + g}];
    if (have < smem) {
      G4_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), G4_ERR_LAUNCH);
      have = smem;
    }
  }
  cudaError_t e = launch_pdl(k, dim3(seqs * items), dim3(kAttnKernelThreads), smem, st, dargs, items);
  if (e != cudaSuccess) return fail(G4_ERR_LAUNCH, "batched attention launch: %s", cudaGetErrorString(e));
  return G4_OK;
}

// The TMA tensor maps of a.cache_k / a.cache_v: [max_len, n_kv * d] bf16, boxes of 64
// elements x attn_kps(d) rows, 128-byte swizzle (the attention kernels' stage layout).
int g4_attention_maps(AttnArgs& a) {
  const uint64_t w = (uint64_t)a.n_kv * a.d;
  int rc = g4_make_map_2d(&a.tmk, a.cache_k, w, (uint64_t)a.max_len, w, (uint32_t)attn_kps(a.d));
  if (!rc) rc = g4_make_map_2d(&a.tmv, a.cache_v, w, (uint64_t)a.max_len, w, (uint32_t)attn_kps(a.d));
  return rc;
}

void g4_rope_inv_freq(int d, double theta, double partial, float* out) {
  // model.py:54-61: fp64 inverse frequencies for the rotated pairs, zero (NoPE) tail
  const int nrot = (int)(partial * d / 2);
  for (int i = 0; i < d / 2; ++i)
    out[i] = i < nrot ? (float)(1.0 / std::pow(theta, (double)(2 * i) / (double)d)) : 0.0f;
}

float g4_host_bf16_round(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  u &= 0xffff0000u;
  float r;
  memcpy(&r, &u, 4);
  return r;
}

// Partition weight of a router row (see the router+MLP operator's plan): with
// `per_tile` router rows per ring tile, the router takes R = ceil(E / per_tile) CTAs
// and a weight w gives each of them one tile when per_tile * row * w equals the MLP
// bytes per remaining CTA.
static int router_row_weight(int E, int I_local, int H, int nsm) {
  const long long row = 2LL * H;
  const int per_tile = (int)(kStageBytes / row);
  if (per_tile < 1) return 1;
  const int R = (E + per_tile - 1) / per_tile;
  if (R >= nsm) return 1;
  const double mlp_per_cta = (double)I_local * 2 * row / (nsm - R);
  const int w = (int)(mlp_per_cta / ((double)per_tile * row) + 0.5);
  return w < 1 ? 1 : w;
}

// Splits per KV head: one item per SM over all heads, each a whole number of 32-key
// stages (the device rounds its slice the same way), at most kAttnMaxChunk keys each.
// Sub-rows of an o_proj row of `k` elements: the fewest (1, 2 or 4) of at most 4,096
// elements each, a multiple of 8 each; 0 when none fits.
static int o_proj_subrows(int k) {
  for (int ns = 1; ns <= 4; ns *= 2)
    if (k % ns == 0 && k / ns <= 4096 && (k / ns) % 8 == 0) return ns;
  return 0;
}

static int pick_nsplit(int n_kv, int max_live, int nsm) {
  int need = (max_live + kAttnMaxChunk - 1) / kAttnMaxChunk;
  int want = nsm / n_kv;
  int ns = want > need ? want : need;
  if (ns < 1) ns = 1;
  if (ns > kAttnMaxSplit) ns = kAttnMaxSplit;
  int chunk = (max_live + ns - 1) / ns;
  chunk = (chunk + kAttnMinKeys - 1) / kAttnMinKeys * kAttnMinKeys;
  return (max_live + chunk - 1) / chunk;
}
int g4_pick_nsplit(int n_kv, int max_live, int nsm) { return pick_nsplit(n_kv, max_live, nsm); }

static bool valid_cfg(const g4_config* c) {
  return c && c->hidden_size > 0 && c->num_hidden_layers > 0 && c->num_attention_heads > 0 &&
         c->head_dim > 0 && c->global_head_dim > 0 && c->num_key_value_heads > 0 &&
         c->num_global_key_value_heads > 0 && c->intermediate_size > 0 &&
         c->moe_intermediate_size > 0 && c->num_experts > 0 && c->top_k_experts > 0 &&
         c->vocab_size > 0;
}

extern "C" int g4_model_create(const g4_config* cfg, const unsigned char* layer_is_full, int rank,
                               int world, int max_len, int device, g4_model** out) {
  if (!out || !valid_cfg(cfg) || !layer_is_full)
    return fail(G4_ERR_ARG, "g4_model_create: null or invalid config");
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || max_len < 1)
    return fail(G4_ERR_ARG, "g4_model_create: bad rank/world/max_len");
  const g4_config& c = *cfg;
  const int G = world;
  if (!c.enable_moe_block) return fail(G4_ERR_SHAPE, "only MoE (enable_moe_block) models are supported");
  if (c.hidden_size % 8 != 0) return fail(G4_ERR_SHAPE, "hidden_size must be a multiple of 8");
  if (c.hidden_size > kMaxHidden) return fail(G4_ERR_SHAPE, "hidden_size > 4096");
  if (c.intermediate_size % (8 * G) || c.moe_intermediate_size % (8 * G) || c.vocab_size % G)
    return fail(G4_ERR_SHAPE, "intermediate / moe_intermediate / vocab not divisible by 8*world");
  if (c.top_k_experts > kMaxTopK || c.top_k_experts > c.num_experts || c.num_experts > 256 ||
      kConsumerWarps % c.top_k_experts)
    return fail(G4_ERR_SHAPE, "top_k_experts must divide %d; num_experts <= 256", kConsumerWarps);
  G4_CUDA(cudaSetDevice(device), G4_ERR_CUDA);
  g4_model* m = new g4_model();
  m->cfg = c;
  m->is_full.assign(layer_is_full, layer_is_full + c.num_hidden_layers);
  m->rank = rank;
  m->world = world;
  m->max_len = max_len;
  m->device = device;
  cudaDeviceGetAttribute(&m->nsm, cudaDevAttrMultiProcessorCount, device);
  m->H = c.hidden_size;
  m->I_local = c.intermediate_size / G;
  m->F_local = c.moe_intermediate_size / G;
  m->V_local = c.vocab_size / G;
  m->vbegin = rank * m->V_local;
  m->E = c.num_experts;
  m->topk = c.top_k_experts;
  m->L.resize(c.num_hidden_layers);
  for (int i = 0; i < c.num_hidden_layers; ++i) {
    LayerDev& l = m->L[i];
    l.full = m->is_full[i] != 0;
    l.k_eq_v = (c.attention_k_eq_v && l.full) ? 1 : 0;
    l.d = l.full ? c.global_head_dim : c.head_dim;
    const int kv = l.k_eq_v ? c.num_global_key_value_heads : c.num_key_value_heads;
    const int gfull = c.num_attention_heads / kv;
    if (c.num_attention_heads % kv) { delete m; return fail(G4_ERR_SHAPE, "heads %% kv_heads"); }
    if (!l.full) {  // sliding: shard KV heads (model.py:141-145)
      if (kv % G) { delete m; return fail(G4_ERR_SHAPE, "layer %d: kv heads %d %% world %d", i, kv, G); }
      l.n_kv = kv / G;
      l.g = gfull;
    } else {        // full: replicate KV, shard query groups (model.py:146-150)
      if (gfull % G) { delete m; return fail(G4_ERR_SHAPE, "layer %d: groups %d %% world %d", i, gfull, G); }
      l.n_kv = kv;
      l.g = gfull / G;
    }
    if (l.g > kAttnMaxG || (l.g & (l.g - 1)) || (l.d != 64 && l.d != 128 && l.d != 256 && l.d != 512)) {
      delete m;
      return fail(G4_ERR_SHAPE, "layer %d: head_dim %d / group %d unsupported", i, l.d, l.g);
    }
    l.rows_q = l.n_kv * l.g * l.d;
    l.rows_k = l.n_kv * l.d;
    l.rows_v = l.k_eq_v ? 0 : l.n_kv * l.d;
    const int max_live = l.full ? max_len : (c.sliding_window < max_len ? c.sliding_window : max_len);
    l.nsplit = pick_nsplit(l.n_kv, max_live, m->nsm);
    if ((max_live + l.nsplit - 1) / l.nsplit > kAttnMaxChunk) {
      delete m;
      return fail(G4_ERR_SHAPE, "layer %d: context %d too long for the split-KV limits", i, max_len);
    }
  }
  for (const LayerDev& l : m->L)
    if (!o_proj_subrows(l.rows_q) || c.hidden_size > 4096 || m->I_local > 4096) {
      delete m;
      return fail(G4_ERR_SHAPE, "a matrix row is longer than the decode engine takes on this rank "
                                "(o_proj of %d heads x %d at world %d)", l.n_kv * l.g, l.d, world);
    }
  *out = m;
  return G4_OK;
}

static size_t expect_bytes(const g4_model* m, const std::string& name, int* layer, std::string* field) {
  const g4_config& c = m->cfg;
  const size_t H = m->H;
  *layer = -1;
  if (name == "embed") return (size_t)c.vocab_size * H * 2;
  if (name == "norm") return H * 2;
  if (name == "control") return G4_CTRL_WORDS * 4;
  if (name == "tokens_in") return (size_t)m->max_len * 4;
  if (name == "tokens_out") return (size_t)(m->max_len + 1) * 4;
  if (name == "logits") return (size_t)m->V_local * 4;
  int li = -1, n = 0;
  if (sscanf(name.c_str(), "layers.%d.%n", &li, &n) != 1 || n <= 0) return 0;
  if (li < 0 || li >= (int)m->L.size()) return 0;
  *layer = li;
  *field = name.substr(n);
  const LayerDev& l = m->L[li];
  const std::string& f = *field;
  if (f == "qkv") return (size_t)(l.rows_q + l.rows_k + l.rows_v) * H * 2;
  if (f == "o_proj") return H * l.rows_q * 2;
  if (f == "mlp.gate_proj" || f == "mlp.up_proj" || f == "mlp.down_proj") return (size_t)m->I_local * H * 2;
  if (f == "router.proj") return (size_t)m->E * H * 2;
  if (f == "router.per_expert_scale") return (size_t)m->E * 2;
  if (f == "experts.gate_up_proj") return (size_t)m->E * 2 * m->F_local * H * 2;
  if (f == "experts.down_proj") return (size_t)m->E * H * m->F_local * 2;
  if (f == "q_norm" || f == "k_norm") return (size_t)l.d * 2;
  if (f == "layer_scalar") return 2;
  if (f == "cache_k" || f == "cache_v") return (size_t)m->max_len * l.n_kv * l.d * 2;
  if (f == "input_layernorm" || f == "post_attention_layernorm" || f == "pre_feedforward_layernorm" ||
      f == "post_feedforward_layernorm" || f == "pre_feedforward_layernorm_2" ||
      f == "post_feedforward_layernorm_1" || f == "post_feedforward_layernorm_2" || f == "router.scale")
    return H * 2;
  return 0;
}

extern "C" int g4_model_set_tensor(g4_model* m, const char* cname, void* ptr, long long nbytes) {
  if (!m || !cname || !ptr) return fail(G4_ERR_ARG, "g4_model_set_tensor: null argument");
  if (m->finalized) return fail(G4_ERR_STATE, "g4_model_set_tensor after finalize");
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return fail(G4_ERR_ARG, "%s: pointer not 16-byte aligned", cname);
  std::string name(cname), field;
  int li = -1;
  const size_t want = expect_bytes(m, name, &li, &field);
  if (want == 0) return fail(G4_ERR_ARG, "unknown tensor name '%s'", cname);
  if ((size_t)nbytes != want)
    return fail(G4_ERR_SHAPE, "%s: %lld bytes, expected %zu", cname, nbytes, want);
  auto* b = static_cast<bf16_t*>(ptr);
  if (li < 0) {
    if (name == "embed") m->embed = b;
    else if (name == "norm") m->final_norm = b;
    else if (name == "control") m->ctrl = static_cast<int*>(ptr);
    else if (name == "tokens_in") m->tokens_in = static_cast<int*>(ptr);
    else if (name == "tokens_out") m->tokens_out = static_cast<int*>(ptr);
    else if (name == "logits") m->logits = static_cast<float*>(ptr);
    return G4_OK;
  }
  LayerDev& l = m->L[li];
  const std::string& f = field;
  if (f == "qkv") l.qkv = b;
  else if (f == "o_proj") l.o = b;
  else if (f == "mlp.gate_proj") l.gate = b;
  else if (f == "mlp.up_proj") l.up = b;
  else if (f == "mlp.down_proj") l.down = b;
  else if (f == "router.proj") l.router = b;
  else if (f == "router.scale") l.router_scale = b;
  else if (f == "router.per_expert_scale") l.pes = b;
  else if (f == "experts.gate_up_proj") l.exp_gu = b;
  else if (f == "experts.down_proj") l.exp_down = b;
  else if (f == "input_layernorm") l.n_in = b;
  else if (f == "post_attention_layernorm") l.n_post_attn = b;
  else if (f == "pre_feedforward_layernorm") l.n_pre_ff = b;
  else if (f == "post_feedforward_layernorm") l.n_post_ff = b;
  else if (f == "pre_feedforward_layernorm_2") l.n_pre_ff2 = b;
  else if (f == "post_feedforward_layernorm_1") l.n_post_ff1 = b;
  else if (f == "post_feedforward_layernorm_2") l.n_post_ff2 = b;
  else if (f == "q_norm") l.q_norm = b;
  else if (f == "k_norm") l.k_norm = b;
  else if (f == "layer_scalar") l.scalar = b;
  else if (f == "cache_k") l.cache_k = b;
  else if (f == "cache_v") l.cache_v = b;
  return G4_OK;
}

extern "C" int g4_model_set_comm(g4_model* m, g4_comm* c) {
  if (!m || !c) return fail(G4_ERR_ARG, "g4_model_set_comm: null argument");
  if (c->world != m->world || c->rank != m->rank || c->hidden != m->H)
    return fail(G4_ERR_ARG, "communicator rank/world/hidden do not match the model");
  if (!c->open) return fail(G4_ERR_STATE, "communicator not opened (g4_comm_open)");
  m->comm = c;
  return G4_OK;
}

static Common make_common(const g4_model* m, int layer) {
  Common c{};
  c.counters = m->counters;
  for (int p = 0; p < kMaxWorld; ++p) c.xbase[p] = m->comm ? m->comm->peer[p] : nullptr;
  c.rank = m->rank;
  c.world = m->world;
  c.xpayload = 4 * m->H;  // floats per slot (2 * H LL words)
  c.H = m->H;
  c.layer = layer;
  c.nlayers = (int)m->L.size();
  c.eps = m->cfg.rms_norm_eps;
  return c;
}

// Host planning of an operator's shared staging area and prologue bulk copies.
struct Stager {
  OpBase* op;
  int off = 0;
  explicit Stager(OpBase* o) : op(o) { op->ncc = op->nac = 0; }
  int space(int bytes) {
    const int o = off;
    off += align_up(bytes, 128);
    op->stgbytes = off;
    return o;
  }
  int constant(const void* src, int bytes) {
    const int o = space(bytes);
    op->cc[op->ncc++] = Copy{src, o, bytes};
    return o;
  }
  int activation(const void* src, int bytes) {
    const int o = space(bytes);
    op->ac[op->nac++] = Copy{src, o, bytes};
    return o;
  }
};

// Staged inputs of "layer `layer` output" (model.py:312-322) for the next kernel.
static Tail plan_tail(const g4_model* m, int layer, Stager& sg) {
  const LayerDev& l = m->L[layer];
  const int H = m->H;
  Tail t{};
  t.resmid = m->resmid;
  t.scalar = l.scalar;
  t.layer = layer;
  t.o_pf1 = sg.constant(l.n_post_ff1, H * 2);
  t.o_pf2 = sg.constant(l.n_post_ff2, H * 2);
  t.o_pf = sg.constant(l.n_post_ff, H * 2);
  if (m->world == 1) {
    t.o_mlp = sg.activation(m->mlp_out, H * 4);
    t.o_moe = sg.activation(m->moe_out, H * 2);
  }
  t.o_res = sg.activation(m->resmid, H * 2);
  return t;
}

static const StepVariant* find_step_variant(const g4_model* m);

// Register bucket of a launch whose longest matrix row needs `chunks_per_lane`.
static int cplm_bucket(int m) { return m <= 4 ? 4 : (m <= 8 ? 8 : (m <= 12 ? 12 : (m <= 16 ? 16 : 0))); }

template <class Op>
static void step_sizes(const Op& op, SmemSizes& z, int& cpl) {
  z.x0 = std::max(z.x0, op.xbytes[0]);
  z.x1 = std::max(z.x1, op.xbytes[1]);
  z.stg = std::max(z.stg, op.stgbytes);
  for (int s = 0; s < op.nseg; ++s)
    if (op.seg[s].units > 0) cpl = std::max(cpl, seg_cpl(op.seg[s]));
}

// Shared-memory plan of the persistent step kernel: the auxiliary area holds the
// largest operator's vectors and staging (or the attention scratch); the ring gets
// every remaining byte (kMaxStages at most).  Device copies of the plans are made by
// upload_step_program.
static int plan_step_program(g4_model* m) {
  const int nl = (int)m->L.size();
  if (nl > kNumSyncWords - kSyncRouter) return fail(G4_ERR_SHAPE, "too many layers for the step kernel");
  SmemSizes z{0, 0, 0};
  int cpl = 1;
  for (int i = 0; i < nl; ++i) {
    step_sizes(m->k1[i], z, cpl);
    step_sizes(m->k3[i], z, cpl);
    step_sizes(m->k4[i], z, cpl);
    step_sizes(m->k5[i], z, cpl);
    step_sizes(m->k6[i], z, cpl);
  }
  step_sizes(m->lm, z, cpl);
  int aux = smem_aux_bytes(z);
  for (const LayerDev& l : m->L) aux = std::max(aux, align_up(attn_smem_bytes(l.g, l.d), 128));
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, m->device);
  const int limit = std::min(kMaxSmemBytes, optin > 0 ? optin : kMaxSmemBytes);
  int stages = kMaxStages;
  while (stages >= 3 && gemv_smem_bytes(aux, stages) + step_range_bytes(nl) > limit) --stages;
  if (stages < 3) return fail(G4_ERR_SHAPE, "step kernel: %d bytes of vectors leave no room for the ring", aux);
  m->step_cplm = cplm_bucket(cpl);
  if (!m->step_cplm) return fail(G4_ERR_SHAPE, "a matrix row is longer than 4096 elements on this rank");
  // default engine: the step kernel when a variant for these shapes is compiled in
  m->engine = find_step_variant(m) ? G4_ENGINE_STEP_KERNEL : G4_ENGINE_OP_KERNELS;
  StepProgram& p = m->prog;
  p = StepProgram{};
  p.sync = m->sync;
  p.ctrl = m->ctrl;
  p.nlayers = nl;
  p.stages = stages;
  p.z = z;
  p.aux = aux;
  const size_t range_bytes = (size_t)m->nsm * step_range_bytes(nl);
  const size_t bytes = (sizeof(QkvOp) + sizeof(AttnArgs) + sizeof(OProjOp) + sizeof(RouterMlpOp) +
                        sizeof(MoeUpOp) + sizeof(MoeDownOp) + 6 * 256) * (size_t)nl +
                       sizeof(LmHeadOp) + 256 + range_bytes + 256;
  if (cudaMalloc(&m->prog_mem, bytes) != cudaSuccess) return fail(G4_ERR_NOMEM, "step program");
  m->prog_dirty = true;
  return G4_OK;
}

// Copy the host plans into the program's device arrays (after any host-side change,
// e.g. g4_model_host_tokens, and before the step kernel's first launch or capture).
static int upload_step_program(g4_model* m) {
  if (!m->prog_dirty) return G4_OK;
  const size_t nl = m->L.size();
  char* d = m->prog_mem;
  size_t off = 0;
  auto put = [&](const void* src, size_t bytes) -> char* {
    char* dst = d + off;
    off += (bytes + 255) / 256 * 256;
    cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    return dst;
  };
  StepProgram& p = m->prog;
  p.k1 = reinterpret_cast<const QkvOp*>(put(m->k1.data(), nl * sizeof(QkvOp)));
  p.k2 = reinterpret_cast<const AttnArgs*>(put(m->k2.data(), nl * sizeof(AttnArgs)));
  p.k3 = reinterpret_cast<const OProjOp*>(put(m->k3.data(), nl * sizeof(OProjOp)));
  p.k4 = reinterpret_cast<const RouterMlpOp*>(put(m->k4.data(), nl * sizeof(RouterMlpOp)));
  p.k5 = reinterpret_cast<const MoeUpOp*>(put(m->k5.data(), nl * sizeof(MoeUpOp)));
  p.k6 = reinterpret_cast<const MoeDownOp*>(put(m->k6.data(), nl * sizeof(MoeDownOp)));
  p.lm = reinterpret_cast<const LmHeadOp*>(put(&m->lm, sizeof(LmHeadOp)));
  // unit ranges of every matrix-product phase for every CTA ([CTA][phase][kRangeSlots])
  {
    const int nops = step_nops((int)nl);
    std::vector<int2> tab((size_t)m->nsm * nops * kRangeSlots, make_int2(0, 0));
    for (int i = 0; i < nops; ++i) {
      const int l = i / 5, r = i - 5 * l;
      const OpBase* op = i == nops - 1 ? static_cast<const OpBase*>(&m->lm)
                         : r == 0      ? static_cast<const OpBase*>(&m->k1[l])
                         : r == 1      ? static_cast<const OpBase*>(&m->k3[l])
                         : r == 2      ? static_cast<const OpBase*>(&m->k4[l])
                         : r == 3      ? static_cast<const OpBase*>(&m->k5[l])
                                       : static_cast<const OpBase*>(&m->k6[l]);
      // MLP-down + experts-up: every CTA takes its share of EACH segment, so it streams
      // dense MLP-down rows (which need no routing) while the router's top-k is selected
      // after the phase barrier, then its expert rows; elsewhere the CTA's slice of the
      // byte-weighted concatenation.  Results do not depend on the split (each row is one
      // warp's dot product), so the per-op kernels' own split gives the same bits.
      const bool per_segment = (i != nops - 1 && r == 3);
      for (int cta = 0; cta < m->nsm; ++cta)
        for (int sg = 0; sg < op->nseg; ++sg) {
          int ub, ue;
          if (per_segment) {
            const long long u = op->seg[sg].units;
            ub = (int)(u * cta / m->nsm);
            ue = (int)(u * (cta + 1) / m->nsm);
          } else {
            cta_unit_range(op->seg, op->nseg, sg, cta, m->nsm, ub, ue);
          }
          tab[((size_t)cta * nops + i) * kRangeSlots + sg] = make_int2(ub, ue);
        }
    }
    p.ranges = reinterpret_cast<const int2*>(put(tab.data(), tab.size() * sizeof(int2)));
  }
  G4_CUDA(cudaDeviceSynchronize(), G4_ERR_CUDA);
  m->prog_dirty = false;
  return G4_OK;
}

// ------------------------------------------------------------------ step variants
static std::vector<StepVariant>& step_variants() {
  static std::vector<StepVariant> v;  // filled by static initialisers of g4_step_*.cu
  return v;
}
void g4::register_step_variant(const StepVariant& v) { step_variants().push_back(v); }

// Attention shape of the sliding / full layers on this rank (a model without one kind
// uses the other's).
static void attn_shapes(const g4_model* m, int& ds, int& gs, int& df, int& gf) {
  ds = gs = df = gf = 0;
  for (const LayerDev& l : m->L) {
    if (l.full) { df = l.d; gf = l.g; }
    else { ds = l.d; gs = l.g; }
  }
  if (!ds) { ds = df; gs = gf; }
  if (!df) { df = ds; gf = gs; }
}

// The compiled step-kernel variant for this model (smallest register bucket that
// holds its longest row), or null.
static const StepVariant* find_step_variant(const g4_model* m) {
  int ds, gs, df, gf;
  attn_shapes(m, ds, gs, df, gf);
  for (const LayerDev& l : m->L)
    if ((l.full ? (l.d != df || l.g != gf) : (l.d != ds || l.g != gs))) return nullptr;
  const StepVariant* best = nullptr;
  for (const StepVariant& v : step_variants())
    if (v.ds == ds && v.gs == gs && v.df == df && v.gf == gf && v.cplm >= m->step_cplm &&
        (!best || v.cplm < best->cplm))
      best = &v;
  return best;
}

// Kernel attributes and the residency check of the cooperative launch.
static int prepare_step(g4_model* m) {
  const StepVariant* v = find_step_variant(m);
  if (!v) return fail(G4_ERR_SHAPE, "no step-kernel variant for this model's shapes");
  const int smem = step_smem_bytes(m->prog);
  cudaFuncAttributes fa{};
  G4_CUDA(cudaFuncGetAttributes(&fa, v->kernel), G4_ERR_LAUNCH);
  if (fa.numRegs != kStepLaunchRegs)  // the setmaxnreg split is sized for this count
    return fail(G4_ERR_LAUNCH, "step kernel built with %d registers per thread, expected %d", fa.numRegs,
                kStepLaunchRegs);
  G4_CUDA(cudaFuncSetAttribute(v->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), G4_ERR_LAUNCH);
  int per_sm = 0;
  G4_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, v->kernel, kStepThreads, smem),
          G4_ERR_LAUNCH);
  if (per_sm < 1) return fail(G4_ERR_LAUNCH, "step kernel does not fit on an SM (%d bytes)", smem);
  m->step_kernel = v->kernel;
  return upload_step_program(m);
}

static int launch_step(g4_model* m, cudaStream_t st) {
  if (!m->step_kernel) return fail(G4_ERR_STATE, "step kernel not prepared");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->nsm);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = step_smem_bytes(m->prog);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: grid barriers are safe
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&m->prog};
  cudaError_t e = cudaLaunchKernelExC(&cfg, m->step_kernel, args);
  if (e != cudaSuccess) return fail(G4_ERR_LAUNCH, "step kernel launch: %s", cudaGetErrorString(e));
  return G4_OK;
}

extern "C" int g4_model_finalize(g4_model* m) {
  if (!m) return fail(G4_ERR_ARG, "g4_model_finalize: null model");
  if (m->finalized) return G4_OK;
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  if (!m->embed || !m->final_norm || !m->ctrl || !m->tokens_in || !m->tokens_out || !m->logits)
    return fail(G4_ERR_STATE, "missing embed/norm/control/tokens_in/tokens_out/logits");
  for (size_t i = 0; i < m->L.size(); ++i) {
    const LayerDev& l = m->L[i];
    const void* req[] = {l.qkv, l.o, l.gate, l.up, l.down, l.router, l.router_scale, l.pes,
                         l.exp_gu, l.exp_down, l.n_in, l.n_post_attn, l.n_pre_ff, l.n_post_ff,
                         l.n_pre_ff2, l.n_post_ff1, l.n_post_ff2, l.q_norm, l.k_norm, l.scalar,
                         l.cache_k, l.cache_v};
    for (const void* p : req)
      if (!p) return fail(G4_ERR_STATE, "layer %zu: missing tensor", i);
  }
  if (m->world > 1 && !m->comm) return fail(G4_ERR_STATE, "world > 1 needs g4_model_set_comm");
  if (!m->comm) {
    int rc = g4_comm_create(m->device, 0, 1, m->H, &m->own_comm);
    if (rc) return rc;
    m->comm = m->own_comm;
  }
  // ---- scratch (one allocation, carved)
  const int H = m->H;
  size_t max_rows = 0, max_ctx = 0, max_part = 0, max_nkv = 0;  // max_nkv: attention counter ints
  for (const LayerDev& l : m->L) {
    max_rows = std::max(max_rows, (size_t)(l.rows_q + l.rows_k + l.rows_v));
    max_ctx = std::max(max_ctx, (size_t)l.rows_q);
    max_part = std::max(max_part, attn_part_floats(l.n_kv, l.nsplit, l.g, l.d));
    max_nkv = std::max(max_nkv, (size_t)attn_counter_ints(l.n_kv, l.nsplit));
  }
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) / 256 * 256;
    return o;
  };
  const size_t o_xres = take(H * 2), o_resmid = take(H * 2), o_h2 = take(H * 2);
  const size_t o_qkv = take(max_rows * 2), o_ctx = take(max_ctx * 2);
  const size_t o_mlpact = take((size_t)m->I_local * 2), o_moeact = take((size_t)m->topk * m->F_local * 2);
  const size_t o_moeout = take(H * 2), o_oout = take(H * 4), o_mlpout = take(H * 4);
  const size_t o_rl = take((size_t)m->E * 4), o_tw = take(kMaxTopK * 4), o_ti = take(kMaxTopK * 4);
  const size_t o_part = take(max_part * 4), o_acnt = take(max_nkv * 4);
  const size_t o_cv = take((size_t)m->nsm * 4), o_ci = take((size_t)m->nsm * 4);
  const size_t o_cnt = take(kNumCounters * 4);
  const size_t o_sync = take(kNumSyncWords * 4);
  const size_t o_sv = take((size_t)kSampleMaxCtas * kSampleMaxK * 4), o_si = take((size_t)kSampleMaxCtas * kSampleMaxK * 4);
  if (cudaMalloc(&m->scratch, off) != cudaSuccess)
    return fail(G4_ERR_NOMEM, "scratch cudaMalloc(%zu) failed", off);
  cudaMemset(m->scratch, 0, off);
  char* s = m->scratch;
  m->xres = (bf16_t*)(s + o_xres);
  m->resmid = (bf16_t*)(s + o_resmid);
  m->h2 = (bf16_t*)(s + o_h2);
  m->qkv_raw = (bf16_t*)(s + o_qkv);
  m->ctx = (bf16_t*)(s + o_ctx);
  m->mlp_act = (bf16_t*)(s + o_mlpact);
  m->moe_act = (bf16_t*)(s + o_moeact);
  m->moe_out = (bf16_t*)(s + o_moeout);
  m->o_out = (float*)(s + o_oout);
  m->mlp_out = (float*)(s + o_mlpout);
  m->router_logits = (float*)(s + o_rl);
  m->top_w = (float*)(s + o_tw);
  m->top_idx = (int*)(s + o_ti);
  m->attn_part = (float*)(s + o_part);
  m->attn_cnt = (int*)(s + o_acnt);
  m->cand_v = (float*)(s + o_cv);
  m->cand_i = (int*)(s + o_ci);
  m->counters = (int*)(s + o_cnt);
  m->sync = (int*)(s + o_sync);
  m->samp_v = (float*)(s + o_sv);
  m->samp_i = (int*)(s + o_si);

  // ---- plans
  const g4_config& c = m->cfg;
  const int nl = (int)m->L.size();
  const float hinv = g4_host_bf16_round(std::pow((float)H, -0.5f));
  m->k1.resize(nl);
  m->k2.resize(nl);
  m->k3.resize(nl);
  m->k4.resize(nl);
  m->k5.resize(nl);
  m->k6.resize(nl);
  for (int i = 0; i < nl; ++i) {
    const LayerDev& l = m->L[i];
    const Common cm = make_common(m, i);
    QkvOp& a = m->k1[i];
    a = QkvOp{};
    a.c = cm;
    a.ctrl = m->ctrl;
    a.nseg = 1;
    a.trace_id = i * 8 + 0;
    a.seg[0] = SegDesc{l.rows_q + l.rows_k + l.rows_v, 1, H, 0};
    a.xbytes[0] = H * 2;
    a.xbytes[1] = 0;
    {
      Stager sg(&a);
      a.o_win = sg.constant(l.n_in, H * 2);
      if (i > 0) a.tail = plan_tail(m, i - 1, sg);
    }
    a.w = l.qkv;
    a.out = m->qkv_raw;
    a.xres = m->xres;
    a.embed = m->embed;
    a.tokens_in = m->tokens_in;
    a.tokens_out = m->tokens_out;
    a.vocab = c.vocab_size;
    a.max_len = m->max_len;
    a.embed_scale = g4_host_bf16_round(std::sqrt((float)H));

    AttnArgs& t = m->k2[i];
    t = AttnArgs{};
    t.qkv = m->qkv_raw;
    t.q_norm = l.q_norm;
    t.k_norm = l.k_norm;
    t.cache_k = l.cache_k;
    t.cache_v = l.cache_v;
    t.inv_freq = nullptr;  // set below (per layer type table)
    t.ctx = m->ctx;
    t.part = m->attn_part;
    t.counters = m->attn_cnt;
    t.ctrl = m->ctrl;
    t.pos_fixed = -1;
    t.n_kv = l.n_kv;
    t.g = l.g;
    t.d = l.d;
    t.nsplit = l.nsplit;
    t.window = l.full ? 0 : c.sliding_window;
    t.k_eq_v = l.k_eq_v;
    t.max_len = m->max_len;
    t.eps = c.rms_norm_eps;
    t.trace_id = i * 8 + 1;
    if (int rc = g4_attention_maps(t)) return rc;

    OProjOp& o = m->k3[i];
    o = OProjOp{};
    o.c = cm;
    o.ctrl = m->ctrl;
    o.nseg = 1;
    o.trace_id = i * 8 + 2;
    // a row longer than the engine's 4,096-element dot (d 512 x 16 query heads at world
    // 1) runs as nsub sub-rows, each dotted with its slice of the context, summed in order
    const int onsub = o_proj_subrows(l.rows_q);
    o.seg[0] = SegDesc{H, onsub, l.rows_q / onsub, 0};
    o.xsub[0] = onsub > 1 ? l.rows_q / onsub : 0;
    o.xbytes[0] = l.rows_q * 2;
    {
      Stager sg(&o);
      o.o_ctx = sg.activation(m->ctx, l.rows_q * 2);
    }
    o.w = l.o;
    o.out = m->o_out;
    o.Kc = l.rows_q;

    RouterMlpOp& r = m->k4[i];
    r = RouterMlpOp{};
    r.c = cm;
    r.ctrl = m->ctrl;
    r.nseg = 2;
    r.trace_id = i * 8 + 3;
    // The CTA completing the router logits also runs the top-k selection, and the
    // experts' weights wait for it: router rows get CTAs of their own, one tile of
    // rows each, by weighing a router row so that one tile of them costs what an MLP
    // CTA streams (the MLP rows then spread over the other CTAs).
    r.seg[0] = SegDesc{m->E, 1, H, 0, router_row_weight(m->E, m->I_local, H, m->nsm)};
    r.seg[1] = SegDesc{m->I_local, 2, H, 0};
    r.xsel[1] = 1;  // router rows: x0 (router input); MLP gate|up: x1 (MLP input)
    r.xbytes[0] = H * 2;
    r.xbytes[1] = H * 2;
    {
      Stager sg(&r);
      r.o_wpa = sg.constant(l.n_post_attn, H * 2);
      r.o_wff = sg.constant(l.n_pre_ff, H * 2);
      r.o_wff2 = sg.constant(l.n_pre_ff2, H * 2);
      r.o_wrs = sg.constant(l.router_scale, H * 2);
      if (m->world == 1) r.o_o = sg.activation(m->o_out, H * 4);
      r.o_x = sg.activation(m->xres, H * 2);
    }
    r.stgbytes = std::max(r.stgbytes, kRouterScratchBytes);  // top-k scratch
    r.xres = m->xres;
    r.resmid = m->resmid;
    r.h2 = m->h2;
    r.router_w = l.router;
    r.pes = l.pes;
    r.gate = l.gate;
    r.up = l.up;
    r.router_logits = m->router_logits;
    r.top_idx = m->top_idx;
    r.top_w = m->top_w;
    r.mlp_act = m->mlp_act;
    r.E = m->E;
    r.topk = m->topk;
    r.hinv = hinv;
    r.ready = m->sync + kSyncRouter + i;

    MoeUpOp& u = m->k5[i];
    u = MoeUpOp{};
    u.c = cm;
    u.ctrl = m->ctrl;
    u.nseg = 2;
    u.trace_id = i * 8 + 4;
    // dense MLP-down rows cost 6/5 of an expert row's bytes in the partition: their tiles
    // (10 rows of 4224 B for config 4) give two warps two rows each, so those CTAs
    // stream slower per byte (measured ~27 vs ~33 KB/us)
    u.seg[0] = SegDesc{H, 1, m->I_local, 0, 6};
    u.seg[1] = SegDesc{m->topk * m->F_local, 2, H, m->F_local, 5};
    u.xsel[0] = 1;  // MLP down: x1 (activation); experts gate|up: x0 (MoE input)
    u.xbytes[0] = H * 2;
    u.xbytes[1] = m->I_local * 2;
    {
      Stager sg(&u);
      u.o_h2 = sg.activation(m->h2, H * 2);
      u.o_act = sg.activation(m->mlp_act, m->I_local * 2);
    }
    u.top_idx = m->top_idx;
    u.top_w = m->top_w;
    u.mlp_down = l.down;
    u.gate_up = l.exp_gu;
    u.mlp_out = m->mlp_out;
    u.moe_act = m->moe_act;
    u.I = m->I_local;
    u.F = m->F_local;
    u.topk = m->topk;

    MoeDownOp& dn = m->k6[i];
    dn = MoeDownOp{};
    dn.c = cm;
    dn.ctrl = m->ctrl;
    dn.nseg = 1;
    dn.trace_id = i * 8 + 5;
    dn.seg[0] = SegDesc{H, m->topk, m->F_local, 0};
    dn.xsub[0] = m->F_local;  // expert slot j: activation j at x0 + j*F
    dn.xbytes[0] = m->topk * m->F_local * 2;
    {
      Stager sg(&dn);
      dn.o_act = sg.activation(m->moe_act, m->topk * m->F_local * 2);
    }
    dn.top_idx = m->top_idx;
    dn.down = l.exp_down;
    dn.mlp_out = m->mlp_out;
    dn.moe_out = m->moe_out;
    dn.F = m->F_local;
    dn.topk = m->topk;
  }
  {
    LmHeadOp& lm = m->lm;
    lm = LmHeadOp{};
    lm.c = make_common(m, nl - 1);
    lm.ctrl = m->ctrl;
    lm.nseg = 1;
    lm.trace_id = nl * 8;
    lm.seg[0] = SegDesc{m->V_local, 1, H, 0};
    lm.xbytes[0] = H * 2;
    lm.xbytes[1] = kConsumerThreads * 8;
    {
      Stager sg(&lm);
      lm.o_wn = sg.constant(m->final_norm, H * 2);
      lm.tail = plan_tail(m, nl - 1, sg);
    }
    lm.embed = m->embed;
    lm.vbegin = m->vbegin;
    lm.logits = m->logits;
    lm.cand_v = m->cand_v;
    lm.cand_i = m->cand_i;
    lm.tokens_out = m->tokens_out;
    lm.max_len = m->max_len;
    lm.softcap = c.final_logit_softcapping;
  }
  {
    SampleArgs& sa = m->sampler;
    sa = SampleArgs{};
    sa.logits = m->logits;
    sa.V_local = m->V_local;
    sa.vbegin = m->vbegin;
    sa.max_len = m->max_len;
    sa.ctrl = m->ctrl;
    sa.tokens_out = m->tokens_out;
    sa.cand_v = m->samp_v;
    sa.cand_i = m->samp_i;
    sa.c = make_common(m, nl - 1);
    m->sample_ctas = (m->V_local + kSampleChunk - 1) / kSampleChunk;
    if (m->sample_ctas > kSampleMaxCtas) return fail(G4_ERR_SHAPE, "vocab slice too large for the sampler");
  }
  // RoPE tables live in a small device buffer shared by all layers of a type.
  {
    const int dsl = c.head_dim, dfu = c.global_head_dim;
    std::vector<float> tab(dsl / 2 + dfu / 2);
    g4_rope_inv_freq(dsl, c.rope_theta_sliding, 1.0, tab.data());
    g4_rope_inv_freq(dfu, c.rope_theta_full, c.rope_partial_rotary_factor_full, tab.data() + dsl / 2);
    float* dev = nullptr;
    if (cudaMalloc(&dev, tab.size() * 4) != cudaSuccess) return fail(G4_ERR_NOMEM, "rope table");
    cudaMemcpy(dev, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice);
    m->rope_tab = dev;
    for (int i = 0; i < nl; ++i) m->k2[i].inv_freq = m->L[i].full ? dev + dsl / 2 : dev;
  }
  int rc = plan_step_program(m);
  if (rc) return rc;
  G4_CUDA(cudaDeviceSynchronize(), G4_ERR_CUDA);
  m->finalized = true;
  return G4_OK;
}

// Dynamic shared memory of the sampler: one sorted chunk, or the merge of every CTA's
// candidates (K <= kSampleMaxK each), whichever is larger.
static int sample_smem(const g4_model* m) {
  int n = 1;
  while (n < m->sample_ctas * kSampleMaxK) n <<= 1;
  return std::max(kSampleChunk * 8, n * 8);
}

int g4_prepare_sampler(const g4_model* m) {
  G4_CUDA(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, sample_smem(m)),
          G4_ERR_LAUNCH);
  return G4_OK;
}

int g4_launch_sampler(const g4_model* m, cudaStream_t st) {
  cudaError_t e = launch_pdl(sample_kernel, dim3(m->sample_ctas), dim3(kSampleThreads), sample_smem(m), st,
                             m->sampler);
  if (e != cudaSuccess) return fail(G4_ERR_LAUNCH, "sampler launch: %s", cudaGetErrorString(e));
  return G4_OK;
}

template <class Op>
static int prepare_op(const Op& op) {
  const int smem = gemv_smem_bytes(smem_aux_bytes(SmemSizes{op.xbytes[0], op.xbytes[1], op.stgbytes}), kStages);
  switch (op_cplm(op)) {
    case 4: return prepare_kernel<Op, 4>(smem);
    case 8: return prepare_kernel<Op, 8>(smem);
    case 12: return prepare_kernel<Op, 12>(smem);
    case 16: return prepare_kernel<Op, 16>(smem);
    default: return fail(G4_ERR_SHAPE, "a matrix row is longer than 4096 elements on this rank");
  }
}

static int prepare_all(g4_model* m) {
  int rc;
  if ((rc = g4_prepare_sampler(m))) return rc;
  if (m->engine == G4_ENGINE_STEP_KERNEL) return prepare_step(m);
  for (size_t i = 0; i < m->L.size(); ++i) {
    if ((rc = prepare_op(m->k1[i])) || (rc = prepare_op(m->k3[i])) || (rc = prepare_op(m->k4[i])) ||
        (rc = prepare_op(m->k5[i])) || (rc = prepare_op(m->k6[i])))
      return rc;
    if ((rc = prepare_attention(m->k2[i].d, m->k2[i].g))) return rc;
  }
  return prepare_op(m->lm);
}

static int enqueue_step(g4_model* m, cudaStream_t st) {
  int rc;
  if (m->engine == G4_ENGINE_STEP_KERNEL) {
    if ((rc = launch_step(m, st))) return rc;
    return g4_launch_sampler(m, st);
  }
  const int nl = (int)m->L.size();
  for (int i = 0; i < nl; ++i) {
    if ((rc = launch_gemv(m->k1[i], m->nsm, st))) return rc;
    if ((rc = launch_attention(m->k2[i], st))) return rc;
    if ((rc = launch_gemv(m->k3[i], m->nsm, st))) return rc;
    if ((rc = launch_gemv(m->k4[i], m->nsm, st))) return rc;
    if ((rc = launch_gemv(m->k5[i], m->nsm, st))) return rc;
    if ((rc = launch_gemv(m->k6[i], m->nsm, st))) return rc;
  }
  if ((rc = launch_gemv(m->lm, m->nsm, st))) return rc;
  return g4_launch_sampler(m, st);
}

extern "C" int g4_model_host_tokens(g4_model* m, int** host_ptr) {
  if (!m || !host_ptr) return fail(G4_ERR_ARG, "g4_model_host_tokens: null argument");
  if (!m->finalized) return fail(G4_ERR_STATE, "g4_model_host_tokens before finalize");
  if (m->gexec) return fail(G4_ERR_STATE, "g4_model_host_tokens after graph capture");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  if (!m->tokens_host) {
    G4_CUDA(cudaHostAlloc(&m->tokens_host, (size_t)(m->max_len + 1) * 4, cudaHostAllocMapped),
            G4_ERR_NOMEM);
    memset(m->tokens_host, 0xff, (size_t)(m->max_len + 1) * 4);
    int* dptr = nullptr;
    G4_CUDA(cudaHostGetDevicePointer((void**)&dptr, m->tokens_host, 0), G4_ERR_CUDA);
    m->lm.tokens_host = dptr;
    m->sampler.tokens_host = dptr;
    m->prog_dirty = true;
  }
  *host_ptr = m->tokens_host;
  return G4_OK;
}

// Per-kernel-class timing: `steps` decode steps launched directly (not from the graph)
// with a CUDA event recorded between consecutive kernels on `stream`; ms_out[c] gets
// the summed duration of class c = 0 qkv, 1 attention, 2 o_proj, 3 router+MLP up,
// 4 MLP down+experts up, 5 experts down, 6 lm_head+argmax.  The events serialise the
// kernels (no programmatic overlap), so per-class times are upper bounds of their
// share inside the graph.
extern "C" int g4_model_profile(g4_model* m, void* stream, int steps, float* ms_out, int nclass) {
  if (!m || !ms_out || nclass < 7 || steps < 1) return fail(G4_ERR_ARG, "g4_model_profile: bad argument");
  if (!m->finalized) return fail(G4_ERR_STATE, "g4_model_profile before finalize");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = prepare_all(m);
  if (rc) return rc;
  // One step of per-operator launches with an event after each, captured into a graph
  // (on a private stream: the caller's may be the legacy default stream) and replayed:
  // the class times are device time between the events, with no host launch gaps.
  const int nl = (int)m->L.size();
  const int per_step = 6 * nl + 1;
  std::vector<cudaEvent_t> ev((size_t)per_step + 1);
  for (auto& e : ev) G4_CUDA(cudaEventCreate(&e), G4_ERR_CUDA);
  cudaStream_t cap = nullptr;
  cudaGraph_t g = nullptr;
  cudaGraphExec_t gx = nullptr;
  if (cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking) != cudaSuccess) {
    rc = fail(G4_ERR_CUDA, "g4_model_profile: stream create failed");
  } else if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    rc = fail(G4_ERR_LAUNCH, "g4_model_profile: begin capture failed");
  } else {
    // an event record node (a plain record inside a capture only orders streams)
    auto mark = [cap](cudaEvent_t e) { cudaEventRecordWithFlags(e, cap, cudaEventRecordExternal); };
    size_t k = 0;
    mark(ev[k++]);
    for (int i = 0; i < nl && !rc; ++i) {
      if (!rc) rc = launch_gemv(m->k1[i], m->nsm, cap);
      mark(ev[k++]);
      if (!rc) rc = launch_attention(m->k2[i], cap);
      mark(ev[k++]);
      if (!rc) rc = launch_gemv(m->k3[i], m->nsm, cap);
      mark(ev[k++]);
      if (!rc) rc = launch_gemv(m->k4[i], m->nsm, cap);
      mark(ev[k++]);
      if (!rc) rc = launch_gemv(m->k5[i], m->nsm, cap);
      mark(ev[k++]);
      if (!rc) rc = launch_gemv(m->k6[i], m->nsm, cap);
      mark(ev[k++]);
    }
    if (!rc) rc = launch_gemv(m->lm, m->nsm, cap);
    mark(ev[k++]);
    const cudaError_t e = cudaStreamEndCapture(cap, &g);
    if (!rc && e != cudaSuccess) rc = fail(G4_ERR_LAUNCH, "g4_model_profile: capture: %s", cudaGetErrorString(e));
    if (!rc && cudaGraphInstantiate(&gx, g, 0) != cudaSuccess)
      rc = fail(G4_ERR_LAUNCH, "g4_model_profile: graph instantiate failed");
  }
  for (int c = 0; c < nclass; ++c) ms_out[c] = 0.f;
  for (int s = 0; s < steps && !rc; ++s) {
    if (cudaGraphLaunch(gx, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
      rc = fail(G4_ERR_LAUNCH, "g4_model_profile: replay failed");
      break;
    }
    for (int j = 1; j <= per_step; ++j) {
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, ev[j - 1], ev[j]) != cudaSuccess) {
        rc = fail(G4_ERR_CUDA, "g4_model_profile: event timing unavailable");
        break;
      }
      const int in_step = j - 1;
      ms_out[in_step == per_step - 1 ? 6 : in_step % 6] += ms;
    }
  }
  if (gx) cudaGraphExecDestroy(gx);
  if (g) cudaGraphDestroy(g);
  if (cap) cudaStreamDestroy(cap);
  for (auto& e : ev) cudaEventDestroy(e);
  return rc;
}

extern "C" int g4_trace_read(void* host_dst, long long bytes) {
#ifdef G4_TRACE
  const long long need = (long long)sizeof(unsigned long long) * kTraceLaunches * kTraceCtas * kTraceEvents;
  if (!host_dst || bytes < need) return fail(G4_ERR_ARG, "g4_trace_read: need %lld bytes", need);
  G4_CUDA(cudaDeviceSynchronize(), G4_ERR_CUDA);
  G4_CUDA(cudaMemcpyFromSymbol(host_dst, g4_trace_buf, need), G4_ERR_CUDA);
  // every step-kernel variant is its own device module with its own buffer: merge
  // (per slot, the latest stamp)
  unsigned long long* dst = static_cast<unsigned long long*>(host_dst);
  std::vector<unsigned long long> tmp((size_t)need / 8);
  for (const StepVariant& v : step_variants()) {
    if (v.trace_read(tmp.data(), need) != 0) continue;
    for (size_t i = 0; i < tmp.size(); ++i) dst[i] = std::max(dst[i], tmp[i]);
  }
  return G4_OK;
#else
  (void)host_dst;
  (void)bytes;
  return fail(G4_ERR_STATE, "library built without -DG4_TRACE");
#endif
}

extern "C" int g4_model_kernel_count(const g4_model* m) {
  if (!m) return 0;
  // + the sampler, which returns at once unless control[TEMPERATURE] > 0
  return m->engine == G4_ENGINE_STEP_KERNEL ? 2 : 6 * (int)m->L.size() + 2;
}

extern "C" int g4_model_set_engine(g4_model* m, int engine) {
  if (!m) return fail(G4_ERR_ARG, "g4_model_set_engine: null model");
  if (engine != G4_ENGINE_STEP_KERNEL && engine != G4_ENGINE_OP_KERNELS)
    return fail(G4_ERR_ARG, "g4_model_set_engine: unknown engine %d", engine);
  if (m->gexec) return fail(G4_ERR_STATE, "g4_model_set_engine after g4_graph_capture");
  if (engine == G4_ENGINE_STEP_KERNEL && m->finalized && !find_step_variant(m))
    return fail(G4_ERR_SHAPE, "no step-kernel variant for this model's shapes");
  m->engine = engine;
  return G4_OK;
}

extern "C" int g4_step(g4_model* m, void* stream) {
  if (!m) return fail(G4_ERR_ARG, "g4_step: null model");
  if (!m->finalized) return fail(G4_ERR_STATE, "g4_step before g4_model_finalize");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  int rc = prepare_all(m);
  if (rc) return rc;
  return enqueue_step(m, static_cast<cudaStream_t>(stream));
}

extern "C" int g4_graph_capture(g4_model* m, void* stream) {
  if (!m) return fail(G4_ERR_ARG, "g4_graph_capture: null model");
  if (!m->finalized) return fail(G4_ERR_STATE, "g4_graph_capture before g4_model_finalize");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  (void)stream;  // the graph is launched on the caller's stream by g4_graph_launch
  if (m->gexec) {
    cudaGraphExecDestroy(m->gexec);
    m->gexec = nullptr;
  }
  if (m->graph) {
    cudaGraphDestroy(m->graph);
    m->graph = nullptr;
  }
  // kernel attributes are set outside of the capture
  int rc;
  if ((rc = prepare_all(m))) return rc;
  // Capture on a private stream: the caller's stream may be the legacy default stream,
  // which cannot be captured; capturing executes nothing, and the graph is launched
  // on the caller's stream by g4_graph_launch.
  cudaStream_t cap = nullptr;
  G4_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking), G4_ERR_CUDA);
  cudaError_t e0 = cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal);
  if (e0 != cudaSuccess) {
    cudaStreamDestroy(cap);
    return fail(G4_ERR_LAUNCH, "cudaStreamBeginCapture: %s", cudaGetErrorString(e0));
  }
  rc = enqueue_step(m, cap);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(cap, &g);
  cudaStreamDestroy(cap);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return fail(G4_ERR_LAUNCH, "EndCapture: %s", cudaGetErrorString(e));
  m->graph = g;
  G4_CUDA(cudaGraphInstantiate(&m->gexec, g, 0), G4_ERR_LAUNCH);
  return G4_OK;
}

extern "C" int g4_graph_launch(g4_model* m, void* stream, int count) {
  if (!m || !m->gexec) return fail(G4_ERR_STATE, "g4_graph_launch without a captured graph");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  for (int i = 0; i < count; ++i)
    G4_CUDA(cudaGraphLaunch(m->gexec, static_cast<cudaStream_t>(stream)), G4_ERR_LAUNCH);
  return G4_OK;
}

extern "C" int g4_model_status(g4_model* m, void* stream, int* status_out) {
  if (!m || !m->ctrl) return fail(G4_ERR_ARG, "g4_model_status: no model/control block");
  G4_CUDA(cudaSetDevice(m->device), G4_ERR_CUDA);
  G4_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), G4_ERR_CUDA);
  int st = 0;
  G4_CUDA(cudaMemcpy(&st, m->ctrl + G4_CTRL_STATUS, 4, cudaMemcpyDeviceToHost), G4_ERR_CUDA);
  if (status_out) *status_out = st;
  if (st) {
    // A step that gave up may leave grid-barrier arrivals, router flags and "last
    // CTA" counters mid-count; the kernels do not start while STATUS is set, so the
    // library's words are cleared here, before the caller clears STATUS.
    if (m->finalized) {
      cudaMemset(m->counters, 0, kNumCounters * 4);
      size_t nkv = 0;
      for (const LayerDev& l : m->L) nkv = std::max(nkv, (size_t)l.n_kv);
      cudaMemset(m->attn_cnt, 0, nkv * 4);
      cudaMemset(m->sync, 0, kNumSyncWords * 4);
      cudaDeviceSynchronize();
    }
    return fail(G4_ERR_TIMEOUT, "device status word 0x%x", st);
  }
  return G4_OK;
}

extern "C" int g4_model_destroy(g4_model* m) {
  if (!m) return G4_OK;
  cudaSetDevice(m->device);
  if (m->gexec) cudaGraphExecDestroy(m->gexec);
  if (m->graph) cudaGraphDestroy(m->graph);
  g4_prefill_release(m);
  g4_batch_release(m);
  if (m->rope_tab) cudaFree(m->rope_tab);
  if (m->prog_mem) cudaFree(m->prog_mem);
  if (m->tokens_host) cudaFreeHost(m->tokens_host);
  if (m->scratch) cudaFree(m->scratch);
  if (m->own_comm) g4_comm_destroy(m->own_comm);
  delete m;
  return G4_OK;
}

// ------------------------------------------------------------------ block entry points
namespace {
struct BlockScratch {
  char* base = nullptr;
  size_t bytes = 0;
};
std::mutex g_block_mu;
std::map<int, BlockScratch> g_block_scratch;

// Per-device scratch shared by the block entry points (grown on demand, kept).  Its
// head has a fixed layout so the zero-at-rest counters never move between calls of
// different shapes: [attention counters | MoE counters | attention control | RoPE
// table | variable-size area].
constexpr size_t kBlockAttnCounters = 0;     // int[kBlockAttnCounterInts] (attn_counter_ints)
constexpr int kBlockMaxKv = 64;
constexpr int kBlockAttnCounterInts = 256;
constexpr size_t kBlockMoeCounters = 1024;   // int[kNumCounters]
constexpr size_t kBlockCtrl = 1280;          // int[G4_CTRL_WORDS] (attention block only)
constexpr size_t kBlockInvFreq = 2048;       // float[kAttnMaxD / 2]
constexpr size_t kBlockPartOffset = 4096;    // attention partials / MoE staging
static_assert(kBlockMoeCounters >= kBlockAttnCounters + kBlockAttnCounterInts * 4 &&
                  kBlockCtrl >= kBlockMoeCounters + kNumCounters * 4 &&
                  kBlockInvFreq >= kBlockCtrl + G4_CTRL_WORDS * 4 &&
                  kBlockPartOffset >= kBlockInvFreq + kAttnMaxD / 2 * 4,
              "block scratch head layout");

char* block_scratch(size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_block_mu);
  BlockScratch& b = g_block_scratch[dev];
  if (b.bytes < bytes) {
    if (b.base) {
      cudaDeviceSynchronize();
      cudaFree(b.base);
    }
    b.base = nullptr;
    b.bytes = 0;
    if (cudaMalloc(&b.base, bytes) != cudaSuccess) return nullptr;
    cudaMemset(b.base, 0, bytes);
    cudaDeviceSynchronize();
    b.bytes = bytes;
  }
  return b.base;
}
}  // namespace

struct RopeTable {
  float v[kAttnMaxD / 2];
  int n;
};
__global__ void rope_table_kernel(const __grid_constant__ RopeTable p, float* dst) {
  for (int i = threadIdx.x; i < p.n; i += blockDim.x) dst[i] = p.v[i];
}

extern "C" int g4_attention_decode(const void* qkv_raw, const void* q_norm, const void* k_norm,
                                   void* cache_k, void* cache_v, int max_len, int n_q_heads,
                                   int n_kv_heads, int head_dim, int k_eq_v, int pos, int window,
                                   float theta, float partial_rotary, float eps, void* ctx,
                                   void* stream) {
  if (!qkv_raw || !q_norm || !k_norm || !cache_k || !cache_v || !ctx)
    return fail(G4_ERR_ARG, "g4_attention_decode: null pointer");
  if (n_kv_heads <= 0 || n_q_heads % n_kv_heads || !attn_kernel_for(head_dim, n_q_heads / n_kv_heads))
    return fail(G4_ERR_SHAPE, "g4_attention_decode: heads %d/%d dim %d unsupported", n_q_heads,
                n_kv_heads, head_dim);
  if (pos < 0 || pos >= max_len) return fail(G4_ERR_ARG, "g4_attention_decode: pos %d out of [0,%d)", pos, max_len);
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int g = n_q_heads / n_kv_heads;
  const int max_live = window > 0 ? std::min(window, max_len) : max_len;
  const int nsplit = pick_nsplit(n_kv_heads, max_live, nsm);
  if ((max_live + nsplit - 1) / nsplit > kAttnMaxChunk) return fail(G4_ERR_SHAPE, "context too long");
  if (n_kv_heads > kBlockMaxKv || attn_counter_ints(n_kv_heads, nsplit) > kBlockAttnCounterInts)
    return fail(G4_ERR_SHAPE, "g4_attention_decode: %d KV heads x %d splits exceed the counters", n_kv_heads, nsplit);
  const size_t part = attn_part_floats(n_kv_heads, nsplit, g, head_dim) * 4;
  char* s = block_scratch(kBlockPartOffset + part);
  if (!s) return fail(G4_ERR_NOMEM, "g4_attention_decode: scratch allocation failed");
  AttnArgs a{};
  a.qkv = static_cast<const bf16_t*>(qkv_raw);
  a.q_norm = static_cast<const bf16_t*>(q_norm);
  a.k_norm = static_cast<const bf16_t*>(k_norm);
  a.cache_k = static_cast<bf16_t*>(cache_k);
  a.cache_v = static_cast<bf16_t*>(cache_v);
  a.ctx = static_cast<bf16_t*>(ctx);
  a.counters = reinterpret_cast<int*>(s + kBlockAttnCounters);
  a.ctrl = reinterpret_cast<int*>(s + kBlockCtrl);
  float* inv = reinterpret_cast<float*>(s + kBlockInvFreq);
  a.part = reinterpret_cast<float*>(s + kBlockPartOffset);
  // the RoPE table travels by value as a kernel parameter (no host copy, no stream sync)
  RopeTable tab;
  tab.n = head_dim / 2;
  g4_rope_inv_freq(head_dim, theta, partial_rotary, tab.v);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rope_table_kernel<<<1, 256, 0, st>>>(tab, inv);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  a.inv_freq = inv;
  a.pos_fixed = pos;
  a.n_kv = n_kv_heads;
  a.g = g;
  a.d = head_dim;
  a.nsplit = nsplit;
  a.window = window;
  a.k_eq_v = k_eq_v;
  a.max_len = max_len;
  a.eps = eps;
  a.trace_id = -1;
  if (int rc = g4_attention_maps(a)) return rc;
  return launch_attention(a, st);
}

// The all-reduce consumers' bounded poll (ll_get8) on a local slot nobody writes: every
// lane waits for 8 words tagged 1 (the slot holds zeros), gives up after the control
// block's timeout and records PEER_TIMEOUT.
__global__ void selftest_peer_wait_kernel(const unsigned long long* slot, int* ctrl) {
  float v[8];
  (void)ll_get8(slot + 8 * threadIdx.x, 1u, v, ctrl);
}

extern "C" int g4_selftest_peer_timeout(int timeout_us, int* status_out) {
  if (timeout_us <= 0 || timeout_us > 10000000 || !status_out)
    return fail(G4_ERR_ARG, "g4_selftest_peer_timeout: timeout %d us (1..10^7), status pointer", timeout_us);
  char* s = block_scratch(kBlockPartOffset + 32 * 8 * 8);
  if (!s) return fail(G4_ERR_NOMEM, "g4_selftest_peer_timeout: scratch allocation failed");
  int* ctrl = reinterpret_cast<int*>(s + kBlockCtrl);
  int words[G4_CTRL_WORDS] = {};
  words[G4_CTRL_TIMEOUT_US] = timeout_us;
  G4_CUDA(cudaMemcpy(ctrl, words, sizeof(words), cudaMemcpyHostToDevice), G4_ERR_CUDA);
  G4_CUDA(cudaMemset(s + kBlockPartOffset, 0, 32 * 8 * 8), G4_ERR_CUDA);
  selftest_peer_wait_kernel<<<1, 32>>>(reinterpret_cast<const unsigned long long*>(s + kBlockPartOffset), ctrl);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  G4_CUDA(cudaDeviceSynchronize(), G4_ERR_CUDA);
  G4_CUDA(cudaMemcpy(words, ctrl, sizeof(words), cudaMemcpyDeviceToHost), G4_ERR_CUDA);
  *status_out = words[G4_CTRL_STATUS];
  int zero[G4_CTRL_WORDS] = {};
  G4_CUDA(cudaMemcpy(ctrl, zero, sizeof(zero), cudaMemcpyHostToDevice), G4_ERR_CUDA);
  if (!(words[G4_CTRL_STATUS] & G4_STATUS_PEER_TIMEOUT))
    return fail(G4_ERR_TIMEOUT, "g4_selftest_peer_timeout: the wait did not report a timeout (status 0x%x)",
                words[G4_CTRL_STATUS]);
  return G4_OK;
}

// A standalone MoE block reuses the layer kernels K4 (router only, block mode), K5
// (experts gate|up only) and K6 (down + fused all-reduce push), plus a small reduce
// kernel for world > 1 that plays the role of the next layer's prologue.
__global__ void moe_block_reduce_kernel(Common c, int* ctrl, bf16_t* out) {
  pdl_wait();
  const int use = site_use(ctrl, c, kSiteFfn, c.layer);
  const uint32_t tag = (uint32_t)use + 1u;
  // every rank's MoE partial (LL words, 8 per poll), summed in rank order
  for (int q = threadIdx.x; q < c.H / 8; q += blockDim.x) {
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    bool got = true;
    for (int src = 0; src < c.world && got; ++src) {
      float v[8];
      got = ll_get8(xll(c, c.rank, kSiteFfn, use & 1, src) + c.H + 8 * q, tag, v, ctrl);
      for (int e = 0; e < 8; ++e) s[e] += v[e];
    }
    if (got)
      for (int e = 0; e < 8; ++e) out[8 * q + e] = f2bf(s[e]);
  }
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(ctrl + G4_CTRL_STEP, 1);  // single block: no reader left
}

extern "C" int g4_moe_block(const g4_config* cfg, int rank, int world, g4_comm* comm, const void* x,
                            const void* router_proj, const void* router_scale,
                            const void* per_expert_scale, const void* gate_up, const void* down,
                            void* out, int* top_idx, float* top_w, int* control, void* stream) {
  if (!valid_cfg(cfg) || !x || !router_proj || !router_scale || !per_expert_scale || !gate_up ||
      !down || !out || !control)
    return fail(G4_ERR_ARG, "g4_moe_block: null argument");
  for (const void* p : {x, static_cast<const void*>(out), router_proj, router_scale, gate_up, down})
    if (reinterpret_cast<uintptr_t>(p) % 16)  // read by 16-byte TMA bulk copies
      return fail(G4_ERR_ARG, "g4_moe_block: x, out, router_proj, router_scale, gate_up and down "
                              "must be 16-byte aligned");
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return fail(G4_ERR_ARG, "g4_moe_block: bad rank/world");
  if (world > 1 && (!comm || !comm->open || comm->world != world || comm->rank != rank))
    return fail(G4_ERR_ARG, "g4_moe_block: world > 1 needs an opened communicator");
  const int H = cfg->hidden_size, E = cfg->num_experts, K = cfg->top_k_experts;
  if (cfg->moe_intermediate_size % (8 * world) || H % 8 || H > kMaxHidden || K > kMaxTopK ||
      E > 256 || K > E || kConsumerWarps % K)
    return fail(G4_ERR_SHAPE, "g4_moe_block: unsupported shape");
  const int F = cfg->moe_intermediate_size / world;
  int dev = 0, nsm = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  // scratch: h2[H] bf16, router logits[E], top (idx,w), act[K*F], mlp placeholder[H]
  size_t off = kBlockPartOffset;
  auto take = [&](size_t b) {
    size_t o = off;
    off += (b + 255) / 256 * 256;
    return o;
  };
  const size_t o_h2 = take((size_t)H * 2), o_rl = take((size_t)E * 4), o_ti = take(kMaxTopK * 4),
               o_tw = take(kMaxTopK * 4), o_act = take((size_t)K * F * 2), o_mlp = take((size_t)H * 4),
               o_z = take(256);
  char* s = block_scratch(off);
  if (!s) return fail(G4_ERR_NOMEM, "g4_moe_block: scratch allocation failed");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Common c{};
  c.counters = reinterpret_cast<int*>(s + kBlockMoeCounters);
  // world 1 never touches an exchange buffer: no communicator is needed
  for (int p = 0; p < kMaxWorld; ++p) c.xbase[p] = world > 1 ? comm->peer[p] : nullptr;
  c.rank = rank;
  c.world = world;
  c.xpayload = 4 * H;  // floats per slot (2 * H LL words)
  c.H = H;
  c.layer = 0;
  c.nlayers = 1;
  c.eps = cfg->rms_norm_eps;
  int* tidx = top_idx ? top_idx : reinterpret_cast<int*>(s + o_ti);
  float* tw = top_w ? top_w : reinterpret_cast<float*>(s + o_tw);

  RouterMlpOp r{};
  r.trace_id = -1;
  r.c = c;
  r.ctrl = control;
  r.nseg = 1;
  r.seg[0] = SegDesc{E, 1, H, 0};
  r.xbytes[0] = H * 2;
  r.xbytes[1] = 0;
  {
    Stager sg(&r);
    r.o_wrs = sg.constant(router_scale, H * 2);
  }
  r.stgbytes = std::max(r.stgbytes, kRouterScratchBytes);  // top-k scratch
  r.block_mode = 1;
  r.block_x = static_cast<const bf16_t*>(x);
  r.h2 = reinterpret_cast<bf16_t*>(s + o_h2);
  r.router_w = static_cast<const bf16_t*>(router_proj);
  r.pes = static_cast<const bf16_t*>(per_expert_scale);
  r.router_logits = reinterpret_cast<float*>(s + o_rl);
  r.top_idx = tidx;
  r.top_w = tw;
  r.E = E;
  r.topk = K;
  r.hinv = g4_host_bf16_round(std::pow((float)H, -0.5f));

  MoeUpOp u{};
  u.trace_id = -1;
  u.c = c;
  u.ctrl = control;
  u.nseg = 2;
  u.seg[0] = SegDesc{0, 1, 8, 0};
  u.seg[1] = SegDesc{K * F, 2, H, F};
  u.xsel[0] = 1;
  u.xbytes[0] = H * 2;
  u.xbytes[1] = 16;
  {
    Stager sg(&u);
    u.o_h2 = sg.activation(r.h2, H * 2);
    u.o_act = sg.activation(s + o_z, 16);  // segment 0 is empty: one zero chunk
  }
  u.top_idx = tidx;
  u.top_w = tw;
  u.mlp_down = static_cast<const bf16_t*>(down);
  u.gate_up = static_cast<const bf16_t*>(gate_up);
  u.mlp_out = reinterpret_cast<float*>(s + o_mlp);
  u.moe_act = reinterpret_cast<bf16_t*>(s + o_act);
  u.I = 8;
  u.F = F;
  u.topk = K;

  MoeDownOp dn{};
  dn.trace_id = -1;
  dn.c = c;
  dn.ctrl = control;
  dn.nseg = 1;
  dn.seg[0] = SegDesc{H, K, F, 0};
  dn.xsub[0] = F;
  dn.xbytes[0] = K * F * 2;
  {
    Stager sg(&dn);
    dn.o_act = sg.activation(u.moe_act, K * F * 2);
  }
  dn.top_idx = tidx;
  dn.down = static_cast<const bf16_t*>(down);
  dn.mlp_out = u.mlp_out;
  dn.moe_out = static_cast<bf16_t*>(out);
  dn.F = F;
  dn.topk = K;

  int rc = G4_OK;
  if (world > 1) cudaMemsetAsync(u.mlp_out, 0, (size_t)H * 4, st);
  if (!rc) rc = launch_gemv(r, nsm, st);
  if (!rc) rc = launch_gemv(u, nsm, st);
  if (!rc) rc = launch_gemv(dn, nsm, st);
  if (!rc && world > 1) {
    cudaError_t e = launch_pdl(moe_block_reduce_kernel, dim3(1), dim3(512), 0, st, c, control,
                               static_cast<bf16_t*>(out));
    if (e != cudaSuccess) rc = fail(G4_ERR_LAUNCH, "reduce launch: %s", cudaGetErrorString(e));
  }
  return rc;
}

// ------------------------------------------------------------------ allocation-free attention
// Some callers cannot allocate device memory when they call into the library: servers
// that reserve their whole memory budget at start-up and must not grow afterwards, hosts
// whose own caching allocator owns the device and forbids allocations behind its back,
// and latency-critical loops that cannot take the device-wide synchronisation a
// cudaMalloc/cudaFree may imply.  g4_attention_decode allocates its scratch (split-KV
// partials and merge counters) on first use; g4_attention_decode_noalloc computes exactly
// the same thing but keeps that scratch in the fixed device array below, which the
// library carries in every GPU it is loaded on until the process exits.
//
// Layout of the array (byte offsets): merge counters, one int per KV head, zero between
// calls; the attention control block (its status word is cleared per call and not read
// back: kernel-side status bits are not reported by this entry point); the RoPE inverse
// frequencies; the split-KV partials.
constexpr size_t kNoAllocScratchBytes = (size_t)4 << 20;  // 4 MiB per device
constexpr size_t kNoAllocCounters = 0;                     // int[kBlockMaxKv]
constexpr size_t kNoAllocCtrl = 256;                       // int[G4_CTRL_WORDS]
constexpr size_t kNoAllocInvFreq = 1024;                   // float[kAttnMaxD / 2]
constexpr size_t kNoAllocPartOffset = 2048;                // partials to the end
static_assert(kNoAllocCtrl >= kNoAllocCounters + kBlockMaxKv * 4 &&
                  kNoAllocInvFreq >= kNoAllocCtrl + G4_CTRL_WORDS * 4 &&
                  kNoAllocPartOffset >= kNoAllocInvFreq + kAttnMaxD / 2 * 4,
              "allocation-free scratch regions overlap");
static __device__ __align__(256) unsigned char g4_noalloc_scratch[kNoAllocScratchBytes];

// Per-call reset of the shared array, with the RoPE table passed by value as a kernel
// parameter (copied at launch): no host buffer has to outlive the call.
struct NoAllocSetup {
  float inv_freq[kAttnMaxD / 2];
  int n_inv;
};
__global__ void noalloc_setup_kernel(const __grid_constant__ NoAllocSetup p, unsigned char* s) {
  int* counters = reinterpret_cast<int*>(s + kNoAllocCounters);
  int* ctrl = reinterpret_cast<int*>(s + kNoAllocCtrl);
  float* inv = reinterpret_cast<float*>(s + kNoAllocInvFreq);
  const int t = threadIdx.x;
  if (t < kBlockMaxKv) counters[t] = 0;
  if (t < G4_CTRL_WORDS) ctrl[t] = 0;
  for (int i = t; i < p.n_inv; i += blockDim.x) inv[i] = p.inv_freq[i];
}

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
unsigned char* g_noalloc_ptr[kNoAllocMaxDevices];  // device address of the array, per device

// The array's name is only a host-side stand-in in host code: its device address must be
// looked up on each device, with that device current, before a kernel can be given it.
int noalloc_scratch(int dev, unsigned char** out) {
  if (dev < 0 || dev >= kNoAllocMaxDevices) return fail(G4_ERR_ARG, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g4_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return fail(G4_ERR_CUDA, "cudaGetSymbolAddress(g4_noalloc_scratch): %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return G4_OK;
}
}  // namespace

extern "C" int g4_attention_decode_noalloc(const void* qkv_raw, const void* q_norm,
                                           const void* k_norm, void* cache_k, void* cache_v,
                                           int max_len, int n_q_heads, int n_kv_heads,
                                           int head_dim, int k_eq_v, int pos, int window,
                                           float theta, float partial_rotary, float eps,
                                           void* ctx, void* stream) {
  if (!qkv_raw || !q_norm || !k_norm || !cache_k || !cache_v || !ctx)
    return fail(G4_ERR_ARG, "g4_attention_decode_noalloc: null pointer");
  if (n_kv_heads <= 0 || n_kv_heads > kBlockMaxKv || n_q_heads % n_kv_heads ||
      !attn_kernel_for(head_dim, n_q_heads / n_kv_heads))
    return fail(G4_ERR_SHAPE, "g4_attention_decode_noalloc: heads %d/%d dim %d unsupported",
                n_q_heads, n_kv_heads, head_dim);
  if (pos < 0 || pos >= max_len)
    return fail(G4_ERR_ARG, "g4_attention_decode_noalloc: pos %d out of [0,%d)", pos, max_len);
  int dev = 0, nsm = 148;
  G4_CUDA(cudaGetDevice(&dev), G4_ERR_CUDA);
  cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int g = n_q_heads / n_kv_heads;
  const int max_live = window > 0 ? std::min(window, max_len) : max_len;
  const int nsplit = pick_nsplit(n_kv_heads, max_live, nsm);
  if ((max_live + nsplit - 1) / nsplit > kAttnMaxChunk) return fail(G4_ERR_SHAPE, "context too long");
  const size_t part = attn_part_floats(n_kv_heads, nsplit, g, head_dim) * 4;
  if (attn_counter_ints(n_kv_heads, nsplit) > kBlockMaxKv)
    return fail(G4_ERR_SHAPE,
                "g4_attention_decode_noalloc: %d KV heads x %d splits need %d counters, the fixed "
                "scratch holds %d (use g4_attention_decode)",
                n_kv_heads, nsplit, attn_counter_ints(n_kv_heads, nsplit), kBlockMaxKv);
  if (part > kNoAllocScratchBytes - kNoAllocPartOffset)
    return fail(G4_ERR_SHAPE,
                "g4_attention_decode_noalloc: needs %zu bytes of split-KV partials, the fixed "
                "scratch holds %zu (use g4_attention_decode)",
                part, kNoAllocScratchBytes - kNoAllocPartOffset);
  unsigned char* s = nullptr;
  int rc = noalloc_scratch(dev, &s);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's contents: the counters and the status word are
  // zeroed and this call's RoPE table written, by one small kernel on the same stream.
  NoAllocSetup setup;
  setup.n_inv = head_dim / 2;
  g4_rope_inv_freq(head_dim, theta, partial_rotary, setup.inv_freq);
  noalloc_setup_kernel<<<1, 256, 0, st>>>(setup, s);
  G4_CUDA(cudaGetLastError(), G4_ERR_LAUNCH);
  AttnArgs a{};
  a.qkv = static_cast<const bf16_t*>(qkv_raw);
  a.q_norm = static_cast<const bf16_t*>(q_norm);
  a.k_norm = static_cast<const bf16_t*>(k_norm);
  a.cache_k = static_cast<bf16_t*>(cache_k);
  a.cache_v = static_cast<bf16_t*>(cache_v);
  a.ctx = static_cast<bf16_t*>(ctx);
  a.counters = reinterpret_cast<int*>(s + kNoAllocCounters);
  a.ctrl = reinterpret_cast<int*>(s + kNoAllocCtrl);
  a.inv_freq = reinterpret_cast<const float*>(s + kNoAllocInvFreq);
  a.part = reinterpret_cast<float*>(s + kNoAllocPartOffset);
  a.pos_fixed = pos;
  a.n_kv = n_kv_heads;
  a.g = g;
  a.d = head_dim;
  a.nsplit = nsplit;
  a.window = window;
  a.k_eq_v = k_eq_v;
  a.max_len = max_len;
  a.eps = eps;
  a.trace_id = -1;
  if ((rc = g4_attention_maps(a))) return rc;
  return launch_attention(a, st);
}
