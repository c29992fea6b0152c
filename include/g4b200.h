/*
 * g4b200 -- C ABI of the B200 (sm_100a) Gemma-4 26B-A4B tensor-parallel decode path.
 *
 * The reference (YLiu95/kaggle-tpu-inference) is pure Python/JAX: its device boundary
 * is the jitted step function, not a foreign-function interface.  The entry points
 * below replace, one for one, the pieces of that boundary:
 *
 *   g4_model_* + g4_step / g4_graph_*  <- the jitted decode step fn and the prefill
 *                                         step body (gemma4_tpu/engine.py:57-83),
 *                                         i.e. model.forward (gemma4_tpu/model.py:333-386)
 *                                         followed by greedy `sample` (model.py:414-424)
 *   g4_model_set_tensor                <- jax.device_put(NamedSharding) of one parameter
 *                                         shard (gemma4_tpu/weights.py:70-83, 131-133)
 *   g4_comm_*                          <- the implicit GSPMD collectives over the 1-D
 *                                         "tp" mesh (model.py:159-161, 303, 310, 316, 381)
 *   g4_moe_block                       <- model.py:224-294 (_router + slice-mode _moe)
 *                                         followed by the all-reduce at model.py:316
 *   g4_attention_decode                <- model.py:195-213 (_attention up to ctx, decode)
 *
 * Conventions: every pointer argument is a device pointer unless documented as host;
 * tensors are dense row-major bf16 (uint16 storage) unless stated; every entry point
 * returns G4_OK (0) or a negative G4_ERR_* code and never aborts the process.
 * g4_last_error() returns a thread-local message describing the last failure.
 * The library never frees memory it did not allocate.
 */
#ifndef G4B200_H_
#define G4B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define G4_OK 0
#define G4_ERR_ARG (-1)     /* bad pointer / argument                               */
#define G4_ERR_SHAPE (-2)   /* shape not supported (divisibility, limits)           */
#define G4_ERR_LAUNCH (-3)  /* kernel launch or graph operation failed              */
#define G4_ERR_TIMEOUT (-4) /* a bounded device wait gave up (see status word)      */
#define G4_ERR_STATE (-5)   /* call order violated (e.g. step before finalize)      */
#define G4_ERR_NOMEM (-6)   /* device allocation failed                             */
#define G4_ERR_CUDA (-7)    /* other CUDA runtime error                             */

/* Bits of the device status word (control block word G4_CTRL_STATUS). */
#define G4_STATUS_PEER_TIMEOUT 0x1  /* a cross-GPU flag never arrived                */
#define G4_STATUS_MBAR_TIMEOUT 0x2  /* a local TMA/mbarrier wait never completed     */
#define G4_STATUS_BAD_TOKEN 0x4     /* an input token id was outside [0, vocab)      */
#define G4_STATUS_POS_OVERFLOW 0x8  /* a step ran at pos >= max_len (nothing written)  */

/* Control block: int32[G4_CTRL_WORDS] in device memory, owned by the caller. */
#define G4_CTRL_POS 0          /* position consumed by the next step                */
#define G4_CTRL_STEP 1         /* completed steps (exchange epoch; never reset)     */
#define G4_CTRL_FORCED_LEN 2   /* positions < this take their token from tokens_in  */
#define G4_CTRL_STATUS 3       /* G4_STATUS_* bits, sticky until the host clears    */
#define G4_CTRL_TIMEOUT_US 4   /* bound of every cross-GPU wait, microseconds       */
#define G4_CTRL_WRITE_LOGITS 5 /* nonzero: each step stores its fp32 logits shard   */
/* Sampling (model.py:414-424): with TEMPERATURE > 0 (fp32 bits) each step replaces the
 * greedy token by a draw from top_k(logits / t, TOP_K) -> softmax -> top-p (TOP_P, fp32
 * bits) -> renormalised, with a Philox-4x32-10 uniform keyed by SEED_HI:SEED_LO and the
 * position (0 for the step that consumes the last forced token, as the reference folds
 * 0 into the prefill key; the consumed position for later steps).  TOP_K <= 128. */
#define G4_CTRL_TEMPERATURE 6
#define G4_CTRL_TOP_P 7
#define G4_CTRL_TOP_K 8
#define G4_CTRL_SEED_LO 9
#define G4_CTRL_SEED_HI 10
#define G4_CTRL_WORDS 16

/* Model hyper-parameters; mirrors TextConfig (gemma4_tpu/config.py:11-49). */
typedef struct g4_config {
  int hidden_size;
  int num_hidden_layers;
  int num_attention_heads;
  int head_dim;
  int global_head_dim;
  int num_key_value_heads;
  int num_global_key_value_heads;
  int intermediate_size;
  int moe_intermediate_size;
  int num_experts;
  int top_k_experts;
  int sliding_window;
  int vocab_size;
  int attention_k_eq_v;
  int enable_moe_block;
  float rms_norm_eps;
  float final_logit_softcapping; /* <= 0 disables the softcap */
  float rope_theta_sliding;
  float rope_theta_full;
  float rope_partial_rotary_factor_full;
} g4_config;

typedef struct g4_model g4_model;
typedef struct g4_comm g4_comm;

const char* g4_version(void);
const char* g4_strerror(int code);
const char* g4_last_error(void);

/* ---------------------------------------------------------------- communicator
 * One per rank (process or device).  Allocates this rank's exchange buffer (flags +
 * double-buffered payload slots) on `device`.  For world > 1 the ranks swap the
 * 64-byte IPC handles from g4_comm_get_handle (any host transport) and pass all of
 * them, in rank order, to g4_comm_open, which maps every peer buffer for direct
 * NVLink stores.  Replaces the implicit GSPMD collectives (model.py:303, 310, 316,
 * 381-382).  The exchange flags count the steps of the control block they serve
 * (control[STEP] is the epoch): a communicator serves one model, or one caller's
 * control block for g4_moe_block; a new model needs a new communicator. */
int g4_comm_create(int device, int rank, int world, int hidden_size, g4_comm** out);
int g4_comm_get_handle(const g4_comm* comm, void* handle_out /* 64 bytes, host */);
int g4_comm_open(g4_comm* comm, const void* handles /* world*64 bytes, host */);
/* g4_comm_open_local: the same for `n` ranks owned by ONE process, one device each (the
 * reference's single-process engine over every device, model.py:159-161 make_mesh):
 * comms[r] is rank r's communicator (created with world = n on its own device); peer
 * access is enabled between the devices and every rank addresses the others' exchange
 * buffers directly (no IPC handles).  The ranks' steps must then be launched so that they
 * run concurrently (one stream per device; each device's graph launched in turn). */
int g4_comm_open_local(g4_comm* const* comms, int n);
int g4_comm_destroy(g4_comm* comm);

/* ---------------------------------------------------------------- model
 * g4_model_create: layer_is_full (host, num_hidden_layers bytes) marks full-attention
 *   layers (config.py layer_types).  rank/world select the tensor-parallel shard.
 * g4_model_set_tensor: registers one device tensor by name; the name set, shapes and
 *   per-rank packing are listed in the package's weights module (pack_rank_shard)
 *   and follow param_specs (model.py:120-156).  nbytes is checked against the
 *   expected size.  Buffers: "control" (int32[G4_CTRL_WORDS]), "tokens_in"
 *   (int32[max_len]), "tokens_out" (int32[max_len+1]), "logits" (fp32[vocab/world]).
 * g4_model_finalize: validates the tensor set, allocates the library's scratch
 *   (attention partials, router/argmax staging) and builds the launch plans.
 * g4_step: enqueues one decode step on `stream` (cudaStream_t): consumes the token at
 *   position control[POS] (tokens_in[pos] while pos < control[FORCED_LEN], else
 *   tokens_out[pos]), writes tokens_out[pos+1] = argmax of the softcapped logits,
 *   advances POS and STEP.  Equivalent to engine.py:71-83 with temperature 0.
 * g4_graph_capture / g4_graph_launch: capture one step into a CUDA graph (with
 *   programmatic dependent launches between the kernels) and replay it.
 * g4_model_status: synchronises `stream` and returns the device status word;
 *   returns G4_ERR_TIMEOUT if any G4_STATUS_* bit is set. */
int g4_model_create(const g4_config* cfg, const unsigned char* layer_is_full, int rank,
                    int world, int max_len, int device, g4_model** out);
int g4_model_set_tensor(g4_model* model, const char* name, void* ptr, long long nbytes);
int g4_model_set_comm(g4_model* model, g4_comm* comm);
int g4_model_finalize(g4_model* model);
int g4_step(g4_model* model, void* stream);
int g4_graph_capture(g4_model* model, void* stream);
int g4_graph_launch(g4_model* model, void* stream, int count);
int g4_model_status(g4_model* model, void* stream, int* status_out);
int g4_model_kernel_count(const g4_model* model); /* kernels launched per step */
/* Decode-step engine (no reference counterpart: the reference's step is one XLA
 * program).  G4_ENGINE_STEP_KERNEL (default): one persistent cooperative kernel per
 * token, one CTA per SM, grid barriers between the operators and one weight ring
 * across the whole step.  G4_ENGINE_OP_KERNELS: 6 kernels per layer + 1, chained by
 * programmatic dependent launch (per-kernel profiling, g4_model_profile).  Both give
 * bit-identical results.  Call before g4_graph_capture (G4_ERR_STATE after).  With the
 * step kernel, a set timeout bit (G4_STATUS_PEER_TIMEOUT / G4_STATUS_MBAR_TIMEOUT)
 * makes every later step a no-op until the host clears it; g4_model_status, on
 * finding any bit set, also clears the library's barrier and counter words so that
 * the next step after the host clears STATUS starts clean. */
#define G4_ENGINE_STEP_KERNEL 0
#define G4_ENGINE_OP_KERNELS 1
int g4_model_set_engine(g4_model* model, int engine);
/* g4_prefill: the prompt tokens_in[0, n_tokens) through the whole model on the tensor
 * cores -- the reference's jitted prefill step (engine.py:57-69: model.forward with
 * dense_moe=True and last_index = n_tokens - 1, model.py:333-386) -- in chunks of at most
 * `chunk` tokens (0: 4096; rounded up to a multiple of 128; a chunk attends to the cache
 * rows of all earlier chunks).  Writes K/V cache rows [0, n_tokens) of every layer, the
 * fp32 logits of position n_tokens - 1 ("logits"), tokens_out[n_tokens] (greedy, or the
 * sample when control[TEMPERATURE] > 0) and sets control[POS] = n_tokens, so the next
 * g4_step continues the sequence.  The caller sets control[FORCED_LEN] = n_tokens (the
 * prompt).  Allocates a workspace on first use (grown for a larger chunk; freed by
 * g4_model_destroy).  world > 1 (tensor parallel, the reference's sharded prefill over
 * its mesh, model.py:84-156): every rank makes the same call on its own stream; each
 * layer's o_proj and MLP + MoE outputs are this rank's fp32 partials, summed over the
 * ranks in rank order through the open communicator (bounded waits: a peer that never
 * arrives sets G4_STATUS_PEER_TIMEOUT), and the first token is the argmax over every
 * rank's vocab slice; chunks are capped at 4096 rows; G4_PREFILL_DENSE_MOE is rejected
 * (G4_ERR_ARG) and a closed communicator is G4_ERR_STATE.
 * flags: 0 computes the MoE over the routed (token, expert) pairs only, as grouped GEMMs:
 * an expert off a token's top-k has routing weight 0 in the reference's dense einsum
 * (model.py:241-250), so its terms are exactly zero and the result is the dense one up to
 * the fp32 summation order; G4_PREFILL_DENSE_MOE runs the dense all-expert computation as
 * written (all 128 experts per token, 16x the MoE FLOPs at top-8). */
#define G4_PREFILL_DENSE_MOE 0x1
int g4_prefill(g4_model* model, int n_tokens, int chunk, int flags, void* stream);
/* Batched decode: `batch` sequences decoded together (the forward over a [B, 1] token batch
 * with a per-sequence cache, model.py:333-386 / 174-185; benchmark config 5's batch-8
 * decode).  World 1, greedy.
 * g4_batch_reserve: allocates a KV cache of ctx_len positions per sequence and layer and
 *   the per-sequence control blocks (replaces any earlier reservation).
 * g4_batch_prefill: sequence `seq`'s prompt, tokens_in[0, n_tokens), through g4_prefill's
 *   tensor-core path into its cache; its first generated token goes to the sequence's
 *   next-input slot (and to *token_out, device, if not NULL); its position becomes n.
 * g4_batch_step: one token of every sequence: each projection as a tensor-core GEMM of the
 *   B rows, the routed MoE over the B x top-k pairs, attention per sequence over its own
 *   cache; writes every sequence's argmax as its next input (and to tokens_out[B] /
 *   logits_out[B, vocab], device, if not NULL) and advances the positions.
 * g4_batch_status: synchronises and ORs the sequences' status words (G4_ERR_TIMEOUT if set). */
int g4_batch_reserve(g4_model* model, int batch, int ctx_len);
int g4_batch_prefill(g4_model* model, int seq, int n_tokens, int* token_out, void* stream);
int g4_batch_step(g4_model* model, int* tokens_out, float* logits_out, void* stream);
int g4_batch_status(g4_model* model, void* stream, int* status_out);
/* g4_gemm_bf16: C[M, N] = A[M, K] . B[N, K]^T on the tensor cores (tcgen05, TMEM accumulator,
 * TMA-fed), bf16 operands with row strides lda / ldb (elements, multiples of 8; 16-byte
 * aligned bases), fp32 accumulation, C in fp32 (c_f32 != 0) or rounded to bf16, row stride
 * ldc.  The GEMM every prefill contraction runs on (the jnp.einsum calls of model.py
 * inside the jitted prefill step, engine.py:57-69).  status: optional int* (device) that
 * receives G4_STATUS_MBAR_TIMEOUT if a bounded wait gives up. */
int g4_gemm_bf16(const void* A, long long lda, const void* B, long long ldb, void* C, long long ldc, int M, int N,
                 int K, int c_f32, int* status, void* stream);
/* Mapped pinned host mirror (int32[max_len+1]) of tokens_out, written by each step's
 * last kernel; lets the host read token i after step i's event without a copy that
 * would queue behind later steps (engine.py:196-200 lookahead read).  Call after
 * finalize and before g4_graph_capture.  The library owns and frees it. */
int g4_model_host_tokens(g4_model* model, int** host_ptr);
/* Per-kernel-class timing of `steps` directly-launched steps with CUDA events between
 * kernels; ms_out[0..6] = qkv, attention, o_proj, router+MLP up, MLP down+experts up,
 * experts down, lm_head+argmax (summed over steps).  Measurement only. */
int g4_model_profile(g4_model* model, void* stream, int steps, float* ms_out, int nclass);
/* Timeline tracer (only in a build with -DG4_TRACE, else G4_ERR_STATE): copies the
 * device buffer of %globaltimer stamps, uint64[512 launches][4 sample CTAs][8 events]
 * (launch id = 8*layer + kernel, lm_head = 8*num_layers), to host memory. */
int g4_trace_read(void* host_dst, long long bytes);
int g4_model_destroy(g4_model* model);

/* ---------------------------------------------------------------- blocks
 * g4_moe_block: one token through router + top-k experts (slice decode mode) on this
 * rank's moe_intermediate shard, with the all-reduce of the [H] output fused into the
 * down-projection kernel (comm may be NULL when world == 1).
 *   x            bf16[H]            MoE input (already pre_feedforward_layernorm_2-normed)
 *   router_proj  bf16[E,H], router_scale bf16[H], per_expert_scale bf16[E]
 *   gate_up      bf16[E,2,F/world,H] (this rank's F slice), down bf16[E,H,F/world]
 *   out          bf16[H]            summed expert output (identical on every rank)
 *   top_idx      int32[K], top_w fp32[K]  (outputs, may be NULL)
 *   scratch_ctl  int32[G4_CTRL_WORDS] control block (STEP used as the exchange epoch)
 * x, out, router_proj, router_scale, gate_up and down must be 16-byte aligned
 * (G4_ERR_ARG otherwise). */
int g4_moe_block(const g4_config* cfg, int rank, int world, g4_comm* comm,
                 const void* x, const void* router_proj, const void* router_scale,
                 const void* per_expert_scale, const void* gate_up, const void* down,
                 void* out, int* top_idx, float* top_w, int* control, void* stream);

/* g4_attention_decode: one query token of one attention layer.
 *   qkv_raw   bf16[(nq + nk + nv) * d]: projections of the normed input, q heads
 *             first (kv-major: head = kv*g + j), then k heads, then v heads (nv = 0
 *             for k==v layers, which reuse k_raw as v_raw)
 *   q_norm, k_norm bf16[d]; cache_k/cache_v bf16[max_len, kv, d] (batch row 0)
 *   pos (host int) position of the token; window (0 = full attention)
 *   theta/partial: RoPE parameters; ctx bf16[nq*d] output.
 * Writes k/v for `pos` into the caches (model.py:205-206) and attends over the live
 * span only: (pos-window, pos] for sliding layers, [0, pos] for full layers. */
int g4_attention_decode(const void* qkv_raw, const void* q_norm, const void* k_norm,
                        void* cache_k, void* cache_v, int max_len, int n_q_heads,
                        int n_kv_heads, int head_dim, int k_eq_v, int pos, int window,
                        float theta, float partial_rotary, float eps, void* ctx,
                        void* stream);

/* g4_attention_decode_noalloc: the same computation and arguments as
 * g4_attention_decode, for callers that must not allocate device memory during the call
 * -- servers that reserve their whole memory budget at start-up, hosts whose own caching
 * allocator owns the GPU, loops that cannot take an allocation's synchronisation.  No
 * counterpart in the reference (its JAX runtime owns all device memory).  Scratch lives
 * in a fixed 4 MiB device array built into the library (kept on every GPU the library is
 * loaded on until exit); shapes whose split-KV partials exceed it fail with
 * G4_ERR_SHAPE.  It calls no cudaMalloc/cudaFree: each call enqueues one small set-up
 * kernel (zeroes the merge counters and status word, writes the RoPE table, passed by
 * value) and the attention kernel on `stream`.  The first call on a device looks the
 * array's address up (cudaGetSymbolAddress) with that device current.  Every call shares
 * the one array: calls that overlap
 * on the GPU (different streams, no ordering) race.  Kernel-side status bits are not
 * reported (the return code covers argument checks and launches only). */
int g4_attention_decode_noalloc(const void* qkv_raw, const void* q_norm, const void* k_norm,
                                void* cache_k, void* cache_v, int max_len, int n_q_heads,
                                int n_kv_heads, int head_dim, int k_eq_v, int pos, int window,
                                float theta, float partial_rotary, float eps, void* ctx,
                                void* stream);

/* g4_selftest_peer_timeout: failure-detection check of the bounded cross-GPU wait, on one
   GPU (the current device), touching no peer memory.  Runs the all-reduce consumers' poll
   of tagged exchange words (the wait of every decode step at world > 1) on a zeroed local
   exchange slot that no producer writes, with a timeout of `timeout_us`; the wait gives
   up, sets G4_STATUS_PEER_TIMEOUT in a control block and the kernel returns.  Synchronises
   and writes that control block's status word to *status_out.  Returns G4_OK when the
   wait ran out as designed (the status bit set), G4_ERR_TIMEOUT otherwise.  No reference
   counterpart (the reference has no device-side waits). */
int g4_selftest_peer_timeout(int timeout_us, int* status_out);

#ifdef __cplusplus
}
#endif
#endif /* G4B200_H_ */
