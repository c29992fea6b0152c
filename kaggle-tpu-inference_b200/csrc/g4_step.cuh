// Persistent decode-step kernel: the whole forward step of one token
// (gemma4_tpu/model.py:333-386, driven by engine.py:57-83) in ONE launch.
//
// The per-op launch mode pays, at every one of the 6 L + 1 kernel boundaries, a
// drained weight ring, a cold parameter fetch and the prologue's dependency chain
// while HBM idles.  Here one CTA per SM (cooperative launch, so every CTA is
// resident) runs the operator program
//
//   for l in layers: QKV, ATTENTION, O_PROJ, ROUTER+MLP, MLP_DOWN+EXPERTS_UP, EXPERTS_DOWN
//   LM_HEAD
//
// with a grid barrier between consecutive operators, and ONE ring of weight stages
// per CTA that runs across the whole program: the producer lane walks the CTA's tiles
// of every operator in program order, so while the consumers wait at a barrier, run
// a prologue or compute attention, the ring already holds the next operator's
// weights.  Weight addresses never depend on activations except the expert tiles,
// for which the producer waits on the layer's router flag.  The CTA that completes the
// router logits arrives at the grid barrier first and then selects the top-k and
// publishes the flag, so the next operator starts on its dense MLP-down rows while the
// selection runs and the expert weights stream in behind it.
//
// Warp specialisation with register reallocation: 12 warps, launched at 168
// registers per thread.  The 4 warps of the producer warpgroup drop to 56
// (setmaxnreg.dec; lane 0 of warp 8 issues the TMA bulk copies, L2 evict-first), the
// 8 consumer warps rise to 224 (setmaxnreg.inc): 8*32*224 + 4*32*56 = 64512 =
// 384*168, so the increase is always satisfiable.  The host launches only a build
// whose kernel uses exactly 168 registers per thread.
//
// Synchronisation (all waits bounded by %globaltimer; a timed-out wait sets a status
// bit, and every CTA gives up at its next wait once a timeout bit is set):
//   * grid barrier: a monotonic arrival counter; operator p starts when it reaches
//     p * gridDim.  The CTA whose arrival completes the final count resets it and
//     advances the launch sequence number, so the next launch starts from zero.
//   * router flags: flag[l] = seq + 1 once the top-k of layer l is in memory.
//   * prologue vectors: norm-weight constants by bulk copy, issued by thread 0 right
//     after the previous operator (before the barrier wait); the previous operator's
//     outputs by the consumer threads with L2 loads after it.
// The per-op launch mode and this kernel share the operators (g4_ops.cuh), the tile
// loop (g4_gemv.cuh) and the attention items (g4_attention.cuh), and every sum has a
// fixed order, so both compute bit-identical results.
#pragma once

#include "g4_attention.cuh"
#include "g4_ops.cuh"

namespace g4 {

constexpr int kStepThreads = kConsumerThreads + 128;  // 2 consumer warpgroups + 1 producer warpgroup
constexpr int kStepLaunchRegs = 168;     // registers per thread at launch (65536 / 384, rounded)
constexpr int kStepConsumerRegs = 224;   // after setmaxnreg.inc
constexpr int kStepProducerRegs = 56;    // after setmaxnreg.dec
static_assert(kConsumerThreads * kStepConsumerRegs + 128 * kStepProducerRegs <= kStepThreads * kStepLaunchRegs,
              "register reallocation exceeds the launch allocation");

// Device words of the step kernel (one int array in scratch, zero at rest).
constexpr int kSyncBarrier = 0;   // grid barrier arrivals of the current launch
constexpr int kSyncSeq = 1;       // launches completed
constexpr int kSyncRouter = 32;   // [layers] router flags
constexpr int kNumSyncWords = kSyncRouter + 256;

struct StepProgram {
  const QkvOp* k1;
  const AttnArgs* k2;
  const OProjOp* k3;
  const RouterMlpOp* k4;
  const MoeUpOp* k5;
  const MoeDownOp* k6;
  const LmHeadOp* lm;
  int* sync;       // kNumSyncWords ints
  int* ctrl;
  const int2* ranges;  // [CTA][matrix-product phase][4] unit ranges per segment
  int nlayers;
  int stages;      // ring depth
  SmemSizes z;     // x0 / x1 / staging sizes (maximum over the operators)
  int aux;         // bytes of the auxiliary area (>= smem_aux_bytes(z), attention scratch)
};

constexpr int kRangeSlots = 4;  // int2 per phase in the range table (kMaxSeg used)

__host__ __device__ __forceinline__ int step_nops(int nlayers) { return 5 * nlayers + 1; }
// The CTA's range table follows the ring in shared memory.
__host__ __device__ __forceinline__ int step_range_bytes(int nlayers) {
  return step_nops(nlayers) * kRangeSlots * 8;
}
__host__ __device__ __forceinline__ int step_smem_bytes(const StepProgram& p) {
  return gemv_smem_bytes(p.aux, p.stages) + step_range_bytes(p.nlayers);
}

// Named barrier that also ANDs a predicate over the consumer threads: a decision
// every consumer thread takes identically.
__device__ __forceinline__ bool consumers_all(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(kBarConsumers), "r"(kConsumerThreads)
      : "memory");
  return r != 0;
}

constexpr int kStatusTimeouts = G4_STATUS_PEER_TIMEOUT | G4_STATUS_MBAR_TIMEOUT;

// Spin until `pred(value)` holds for *p (acquire), bounded; gives up early when a
// timeout bit is already set anywhere.  Returns false after setting a status bit.
template <class Pred>
__device__ __forceinline__ bool spin_until(const int* p, Pred pred, int* status, int timeout_us) {
  if (pred(ld_acquire_gpu(p))) return true;
  const uint64_t limit = static_cast<uint64_t>(timeout_us > 0 ? timeout_us : 2000000) * 1000ull;
  const uint64_t t0 = globaltimer_ns();
  int n = 0;
  while (!pred(ld_acquire_gpu(p))) {
    if ((++n & 63) == 0) {
      if (ldcg_i(status) & kStatusTimeouts) return false;
      if (globaltimer_ns() - t0 > limit) {
        atomicOr(status, G4_STATUS_MBAR_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Consumer-thread copy of the activation vectors of an operator into the staging
// area (L2 loads: the data was written by other CTAs of this launch).  All loads of a
// thread are in flight before its first store.
__device__ __forceinline__ void stage_activations(const Copy* cp, int n, unsigned char* stg) {
  constexpr int U = 8;
  int pre[kMaxCopies + 1];
  pre[0] = 0;
#pragma unroll
  for (int i = 0; i < kMaxCopies; ++i) pre[i + 1] = pre[i] + (i < n ? cp[i].bytes / 16 : 0);
  const int total = pre[kMaxCopies];
  for (int base = threadIdx.x; base < total; base += kConsumerThreads * U) {
    uint4 v[U];
    int dst[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int g = base + u * kConsumerThreads;
      dst[u] = -1;
      if (g < total) {
        int c = 0;
#pragma unroll
        for (int i = 1; i < kMaxCopies; ++i) c += (g >= pre[i]) ? 1 : 0;
        const int k = g - pre[c];
        v[u] = ldcg_u4(reinterpret_cast<const unsigned char*>(cp[c].src) + (size_t)k * 16);
        dst[u] = cp[c].dst + k * 16;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (dst[u] >= 0) *reinterpret_cast<uint4*>(stg + dst[u]) = v[u];
  }
}

// Program order: phase p is layer p / 6, kind p % 6 (0 qkv, 1 attention, 2 o_proj,
// 3 router+MLP, 4 MLP down+experts up, 5 experts down); phase 6 L is the LM head.
template <class F>
__device__ __forceinline__ void with_gemv_op(const StepProgram& P, int p, F&& f) {
  const int l = p / 6, k = p - 6 * l;
  if (l == P.nlayers) f(*P.lm);
  else if (k == 0) f(P.k1[l]);
  else if (k == 2) f(P.k3[l]);
  else if (k == 3) f(P.k4[l]);
  else if (k == 4) f(P.k5[l]);
  else if (k == 5) f(P.k6[l]);
}

// This CTA's unit-range table in shared memory (after the ring).
__device__ __forceinline__ const int2* step_ranges(const StepProgram& P, const Smem& sm) {
  return reinterpret_cast<const int2*>(sm.stages + (size_t)P.stages * kStageBytes);
}

// The program's matrix-product phases in order (attention phases carry no tiles):
// index i -> (layer, kind).
__device__ __forceinline__ void gemv_phase_of(int i, int nlayers, int& l, int& kind) {
  if (i == 5 * nlayers) {
    l = nlayers;
    kind = 6;  // LM head
    return;
  }
  l = i / 5;
  const int r = i - 5 * l;
  kind = r == 0 ? 0 : r + 1;  // 0 qkv, 2 o_proj, 3 router+MLP, 4 MLP down+experts up, 5 experts down
}

// Producer lane: every weight tile of one operator owned by this CTA.
template <class Op>
__device__ __forceinline__ bool produce_op(const Op& op, int layer, const StepProgram& P, Smem& sm, RingPos& rp,
                                           uint64_t pol, int seq, const int2* rng, int& ids_layer) {
  int* status = P.ctrl + G4_CTRL_STATUS;
  bool dep_loaded = false;
  for (int s = 0; s < op.nseg; ++s) {
    int ub, ue;
    ub = rng[s].x;
    ue = rng[s].y;
    if (ub >= ue) continue;
    if (op.seg_dependent(s) && !dep_loaded) {
      if (ids_layer != layer) {  // experts-down reuses the ids experts-up loaded
        const int want = seq + 1;
        if (!spin_until(P.sync + kSyncRouter + layer, [want](int v) { return v == want; }, status,
                        ldcg_i(P.ctrl + G4_CTRL_TIMEOUT_US))) {
          sm.ints[kSmemDead] = 1;
          return false;
        }
        op.load_dependent(sm);
        ids_layer = layer;
      }
      dep_loaded = true;
    }
    for (int u = ub; u < ue;) {
      const int n = tile_units(op.seg[s], u, ue);
      if (!produce_tile(op, s, u, n, sm, rp, P.stages, pol, status)) return false;
      u += n;
    }
  }
  return true;
}

__device__ __forceinline__ const OpBase* producer_op(const StepProgram& P, int l, int kind) {
  switch (kind) {
    case 0: return &P.k1[l];
    case 2: return &P.k3[l];
    case 3: return &P.k4[l];
    case 4: return &P.k5[l];
    case 5: return &P.k6[l];
    default: return P.lm;
  }
}

__device__ __forceinline__ int producer_op_bytes(int kind) {
  switch (kind) {
    case 0: return (int)sizeof(QkvOp);
    case 2: return (int)sizeof(OProjOp);
    case 3: return (int)sizeof(RouterMlpOp);
    case 4: return (int)sizeof(MoeUpOp);
    case 5: return (int)sizeof(MoeDownOp);
    default: return (int)sizeof(LmHeadOp);
  }
}

// Producer lane: bulk-copy the plan of matrix-product phase i into its slot (i & 1);
// completion on Smem::pbar[1], phase i.
__device__ __forceinline__ void fetch_plan(const StepProgram& P, Smem& sm, int i) {
  int l, kind;
  gemv_phase_of(i, P.nlayers, l, kind);
  const uint32_t bytes = (uint32_t)producer_op_bytes(kind);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's old plan was read
  mbar_arrive_expect_tx(&sm.pbar[1], bytes);
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(sm.popc + (i & 1) * kOpCopyBytes)),
      "l"(producer_op(P, l, kind)), "r"(bytes), "r"(smem_addr(&sm.pbar[1]))
      : "memory");
}

// Not inlined (its own register budget after setmaxnreg.dec); Smem by value, so the
// consumers' copy never has its address taken.  The plan of the next operator is
// fetched into the other shared slot while the current one streams, so the first
// tile of an operator never waits for its plan.
static __device__ __noinline__ void produce_step(const StepProgram& P, Smem sm, int seq) {
  const uint64_t pol = l2_evict_first_policy();
  int* status = P.ctrl + G4_CTRL_STATUS;
  RingPos rp;
  const int nops = 5 * P.nlayers + 1;
  fetch_plan(P, sm, 0);
  int ids_layer = -1;  // layer whose expert ids are in Smem::ints[kSmemExp..]
  bool ok = true;
  for (int i = 0; i < nops && ok; ++i) {
    if (!mbar_wait(&sm.pbar[1], i & 1, status)) {
      sm.ints[kSmemDead] = 1;
      break;
    }
    if (i + 1 < nops) fetch_plan(P, sm, i + 1);
    int l, kind;
    gemv_phase_of(i, P.nlayers, l, kind);
    const unsigned char* slot = sm.popc + (i & 1) * kOpCopyBytes;
    const int2* rng = step_ranges(P, sm) + i * kRangeSlots;
    switch (kind) {
      case 0:
        ok = produce_op(*reinterpret_cast<const QkvOp*>(slot), l, P, sm, rp, pol, seq, rng, ids_layer);
        // layer l's attention stages follow its qkv weights in the ring (the cache rows
        // do not depend on qkv; the one row qkv produces is patched by the consumers)
        if (ok) {
          const AttnRing ring{sm.full, sm.empty, sm.stages, kStageBytes, P.stages};
          ok = attn_produce(P.k2 + l, blockIdx.x, gridDim.x, ring, rp, sm.ints + kSmemDead, status,
                            sm.ints + kSmemIssued);
        }
        break;
      case 2: ok = produce_op(*reinterpret_cast<const OProjOp*>(slot), l, P, sm, rp, pol, seq, rng, ids_layer); break;
      case 3: ok = produce_op(*reinterpret_cast<const RouterMlpOp*>(slot), l, P, sm, rp, pol, seq, rng, ids_layer); break;
      case 4: ok = produce_op(*reinterpret_cast<const MoeUpOp*>(slot), l, P, sm, rp, pol, seq, rng, ids_layer); break;
      case 5: ok = produce_op(*reinterpret_cast<const MoeDownOp*>(slot), l, P, sm, rp, pol, seq, rng, ids_layer); break;
      default: ok = produce_op(*reinterpret_cast<const LmHeadOp*>(slot), l < P.nlayers ? l : P.nlayers - 1, P, sm, rp, pol, seq, rng, ids_layer); break;
    }
  }
  producer_exit(sm);
}

using StepHooks = EmptyBarrierHooks;

// Per-CTA state of the consumer side.
struct PhaseState {
  int phase = 0;      // operator index in the program
  bool live = true;   // identical on every consumer thread
  RingPos rp, wp;     // ring position (all tiles) / tiles seen complete
};

// Start of operator ps.phase: wait for every CTA to finish the previous operator (the
// operator's constants are waited for later, by wait_constants, just before use).
__device__ __forceinline__ void phase_begin(const StepProgram& P, Smem& sm, PhaseState& ps, int trace_id) {
  int* status = P.ctrl + G4_CTRL_STATUS;
  bool ok = sm.ints[kSmemDead] == 0;
  if (threadIdx.x == 0 && ok) {
    if (ps.phase > 0) {  // acquire: the other CTAs' outputs of the previous operator
      const int target = ps.phase * (int)gridDim.x;
      ok = spin_until(P.sync + kSyncBarrier, [target](int v) { return v >= target; }, status,
                      ldcg_i(P.ctrl + G4_CTRL_TIMEOUT_US));
    }
    if (!ok) sm.ints[kSmemDead] = 1;
    G4_TRACE_EV(trace_id, 0);
  }
  ps.live = consumers_all(ok && sm.ints[kSmemDead] == 0);
}

// This operator's constant copies (issued at the end of the previous operator) have
// landed; thread 0 waits, the caller's next barrier publishes the result.
__device__ __forceinline__ void wait_constants(const StepProgram& P, Smem& sm, PhaseState& ps) {
  if (threadIdx.x == 0 && sm.ints[kSmemDead] == 0 &&
      !mbar_wait(&sm.pbar[0], ps.phase & 1, P.ctrl + G4_CTRL_STATUS))
    sm.ints[kSmemDead] = 1;
}

// End of operator ps.phase: all of this CTA's stores done -> arrive -> issue the next
// operator's constant copies (the staging area is free; an empty list still
// completes the barrier phase the next operator waits for).
__device__ __forceinline__ void phase_end(const StepProgram& P, Smem& sm, PhaseState& ps, const OpBase* next) {
  named_bar(kBarConsumers, kConsumerThreads);
  if (threadIdx.x == 0) {
    // release: this CTA's stores (ordered before by the barrier above) become
    // visible before the arrival; the arrival goes first, the copies are local
    red_release_gpu_add(P.sync + kSyncBarrier, 1);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic accesses -> async writes
    if (next) issue_copies(next->cc, next->ncc, sm.stg, &sm.pbar[0]);
    else issue_copies(nullptr, 0, sm.stg, &sm.pbar[0]);
  }
  ++ps.phase;
}

// Operator kinds of the program (phase p: layer p / 6, kind p % 6; phase 6 L: LM head).
constexpr int kKindQkv = 0, kKindAttn = 1, kKindOProj = 2, kKindRouterMlp = 3, kKindMoeUp = 4,
              kKindMoeDown = 5, kKindLm = 6;

// The matrix-product operator of (layer, kind), or null for attention.
__device__ __forceinline__ const OpBase* op_base(const StepProgram& P, int l, int kind) {
  switch (kind) {
    case kKindQkv: return &P.k1[l];
    case kKindOProj: return &P.k3[l];
    case kKindRouterMlp: return &P.k4[l];
    case kKindMoeUp: return &P.k5[l];
    case kKindMoeDown: return &P.k6[l];
    case kKindLm: return P.lm;
    default: return nullptr;
  }
}

__device__ __forceinline__ int op_bytes(int kind) {
  switch (kind) {
    case kKindQkv: return (int)sizeof(QkvOp);
    case kKindOProj: return (int)sizeof(OProjOp);
    case kKindRouterMlp: return (int)sizeof(RouterMlpOp);
    case kKindMoeUp: return (int)sizeof(MoeUpOp);
    case kKindMoeDown: return (int)sizeof(MoeDownOp);
    default: return (int)sizeof(LmHeadOp);
  }
}
static_assert(sizeof(QkvOp) <= kOpCopyBytes && sizeof(OProjOp) <= kOpCopyBytes &&
                  sizeof(RouterMlpOp) <= kOpCopyBytes && sizeof(MoeUpOp) <= kOpCopyBytes &&
                  sizeof(MoeDownOp) <= kOpCopyBytes && sizeof(LmHeadOp) <= kOpCopyBytes,
              "operator plan larger than its shared-memory copy");
static_assert(sizeof(QkvOp) % 16 == 0 && sizeof(OProjOp) % 16 == 0 && sizeof(RouterMlpOp) % 16 == 0 &&
                  sizeof(MoeUpOp) % 16 == 0 && sizeof(MoeDownOp) % 16 == 0 && sizeof(LmHeadOp) % 16 == 0,
              "plans are moved in 16-byte units");

// Consumer side of one matrix-product operator up to (not including) its arrival.
// One tile loop serves every operator (only the epilogue, a switch on the kind,
// differs): one hot loop in the instruction cache and one register allocation.  The
// operator's plan is copied into shared memory first: every later read of a plan
// field (per tile, in the epilogue) is a shared-memory load rather than a global load
// that cannot be hoisted past the epilogue's global stores.
template <int CPLM>
__device__ __forceinline__ void gemv_phase_body(const StepProgram& P, int l, int kind, Smem& sm,
                                                PhaseState& ps, StepHooks& h) {
  int* status = P.ctrl + G4_CTRL_STATUS;
  {
    const uint2* src = reinterpret_cast<const uint2*>(op_base(P, l, kind));
    const int words = op_bytes(kind) / 8;
    if ((int)threadIdx.x < words) reinterpret_cast<uint2*>(sm.opc)[threadIdx.x] = __ldg(src + threadIdx.x);
  }
  phase_begin(P, sm, ps, op_base(P, l, kind)->trace_id);  // its barrier publishes the copy
  const OpBase& ob = *reinterpret_cast<const OpBase*>(sm.opc);
  bool ok = ps.live;
  if (ps.live) {
    stage_activations(ob.ac, ob.nac, sm.stg);
    if (threadIdx.x == 0) G4_TRACE_EV(ob.trace_id, 1);
    wait_constants(P, sm, ps);
    if (kind == kKindRouterMlp && threadIdx.x == 0) {
      const int2 r0 = step_ranges(P, sm)[(l * 5 + 2) * kRangeSlots];
      sm.ints[kSmemRouterEnd] = r0.x < r0.y ? r0.y : 0;
      sm.ints[kSmemRouterMine] = r0.y - r0.x;
    }
    named_bar(kBarConsumers, kConsumerThreads);
    if (threadIdx.x == 0) G4_TRACE_EV(ob.trace_id, 2);
    switch (kind) {
      case kKindQkv: ok = reinterpret_cast<const QkvOp*>(sm.opc)->prologue(sm); break;
      case kKindOProj: ok = reinterpret_cast<const OProjOp*>(sm.opc)->prologue(sm); break;
      case kKindRouterMlp: ok = reinterpret_cast<const RouterMlpOp*>(sm.opc)->prologue(sm); break;
      case kKindMoeUp: ok = reinterpret_cast<const MoeUpOp*>(sm.opc)->prologue(sm); break;
      case kKindMoeDown: ok = reinterpret_cast<const MoeDownOp*>(sm.opc)->prologue(sm); break;
      default: ok = reinterpret_cast<const LmHeadOp*>(sm.opc)->prologue(sm); break;
    }
    named_bar(kBarConsumers, kConsumerThreads);
    if (threadIdx.x == 0) G4_TRACE_EV(ob.trace_id, 3);
  }
  // The tile loop runs even when this CTA is dead: it then only advances the ring
  // position (no waits), keeping the consumer threads in step.
  const int gi = kind == kKindLm ? 5 * P.nlayers : l * 5 + (kind == kKindQkv ? 0 : kind - 1);
  const int2* rng = step_ranges(P, sm) + gi * kRangeSlots;
  consume_segments<CPLM>(ob, sm, ps.rp, ps.wp, P.stages, ok && ps.live, status, h,
                         [&](int s, int u0, int n, const Res& r, bool eok, int t) {
                           switch (kind) {
                             case kKindQkv: reinterpret_cast<const QkvOp*>(sm.opc)->epilogue(s, u0, n, r, sm, eok, t); break;
                             case kKindOProj: reinterpret_cast<const OProjOp*>(sm.opc)->epilogue(s, u0, n, r, sm, eok, t); break;
                             case kKindRouterMlp: reinterpret_cast<const RouterMlpOp*>(sm.opc)->epilogue(s, u0, n, r, sm, eok, t); break;
                             case kKindMoeUp: reinterpret_cast<const MoeUpOp*>(sm.opc)->epilogue(s, u0, n, r, sm, eok, t); break;
                             case kKindMoeDown: reinterpret_cast<const MoeDownOp*>(sm.opc)->epilogue(s, u0, n, r, sm, eok, t); break;
                             default: reinterpret_cast<const LmHeadOp*>(sm.opc)->epilogue(s, u0, n, r, sm, eok, t); break;
                           }
                         },
                         rng);
  if (threadIdx.x == 0) G4_TRACE_EV(ob.trace_id, 5);
  if (consumers_all(ps.live)) {
    const bool fok = ok && sm.ints[kSmemDead] == 0;
    switch (kind) {
      case kKindQkv: reinterpret_cast<const QkvOp*>(sm.opc)->finish(sm, fok); break;
      case kKindOProj: reinterpret_cast<const OProjOp*>(sm.opc)->finish(sm, fok); break;
      case kKindRouterMlp: reinterpret_cast<const RouterMlpOp*>(sm.opc)->finish(sm, fok); break;
      case kKindMoeUp: reinterpret_cast<const MoeUpOp*>(sm.opc)->finish(sm, fok); break;
      case kKindMoeDown: reinterpret_cast<const MoeDownOp*>(sm.opc)->finish(sm, fok); break;
      default: reinterpret_cast<const LmHeadOp*>(sm.opc)->finish(sm, fok); break;
    }
  }
  if (threadIdx.x == 0) G4_TRACE_EV(ob.trace_id, 6);
}

// Attention items of this CTA for one layer; their key stages come through the ring.
template <int D, int G>
__device__ __forceinline__ void attn_items(const AttnArgs& a, unsigned char* scratch, Smem& sm, PhaseState& ps,
                                           int stages, int* status) {
  const AttnRing ring{sm.full, sm.empty, sm.stages, kStageBytes, stages};
  const int items = a.n_kv * a.nsplit;
  for (int it = blockIdx.x; it < items; it += gridDim.x)
    attn_item<D, G>(a, it / a.nsplit, it % a.nsplit, scratch, kBarConsumers, ring, ps.rp, ps.wp,
                    sm.ints + kSmemDead, status);
}

// Wait (bounded) for every issued tile thread 0 did not see complete, so that no
// bulk copy still writes into this CTA's shared memory when it exits after a failure.
__device__ __forceinline__ void drain_issued(Smem& sm, RingPos rp, int issued, int stages) {
  while (rp.tiles < issued) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(&sm.full[rp.st], rp.ph) && globaltimer_ns() - t0 < kLocalTimeoutNs) {
    }
    rp.next(stages);
  }
}

// CPLM: input-vector chunks per lane of the longest row; (DS, GS) / (DF, GF): head dim
// and query heads per KV head of the sliding / full attention layers on this rank.
template <int CPLM, int DS, int GS, int DF, int GF>
__global__ void __launch_bounds__(kStepThreads, 1) step_kernel(const __grid_constant__ StepProgram P) {
  extern __shared__ unsigned char g4_dyn_smem[];
  Smem sm = carve_smem(g4_dyn_smem, P.z, P.aux, P.stages);
  int* status = P.ctrl + G4_CTRL_STATUS;

  if (threadIdx.x == 0) {
    for (int i = 0; i < P.stages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsumerWarps);
    }
    sm.ints[kSmemIssued] = 0;
    sm.ints[kSmemProdExit] = 0;
    sm.ints[kSmemRangesGiven] = 1;
    sm.ints[kSmemTopk] = 0;
    mbar_init(&sm.pbar[0], 1);
    mbar_init(&sm.pbar[1], 1);
    mbar_init_fence();
    // a step never starts on top of an unhandled timeout (barrier arrivals, flags and
    // counters may be mid-count): the host clears the status and the library's words
    // first.  BAD_TOKEN / POS_OVERFLOW leave the step's synchronisation intact.
    sm.ints[kSmemDead] = (ldcg_i(status) & kStatusTimeouts) != 0;
    sm.ints[kSmemSeq] = ldcg_i(P.sync + kSyncSeq);
  }
  {  // this CTA's unit ranges (host table) into shared memory, after the ring
    const int n16 = step_range_bytes(P.nlayers) / 16;
    const uint4* src = reinterpret_cast<const uint4*>(P.ranges) + (size_t)blockIdx.x * n16;
    uint4* dst = reinterpret_cast<uint4*>(sm.stages + (size_t)P.stages * kStageBytes);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = __ldg(src + i);
  }
  __syncthreads();
  if (sm.ints[kSmemDead]) return;  // read after the barrier: identical on every thread
  const int seq = sm.ints[kSmemSeq];

  // warp-uniform split: warps 8-11 (one warpgroup) produce, warps 0-7 consume
  if (threadIdx.x >= kConsumerThreads) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kStepProducerRegs) : "memory");
    if (threadIdx.x == kConsumerThreads) produce_step(P, sm, seq);
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kStepConsumerRegs) : "memory");
  PhaseState ps;
  StepHooks h;
  if (threadIdx.x == 0) issue_copies(P.k1[0].cc, P.k1[0].ncc, sm.stg, &sm.pbar[0]);
  // One loop over the program (the LM head is its last phase): every operator's tile
  // loop is the same inlined code.  The next operator's constants are copied at the end
  // of each phase; the LM head's arrival is the final one of the launch.
  const int L = P.nlayers;
  for (int p = 0; p <= 6 * L; ++p) {
    const int l = p / 6, k = p == 6 * L ? kKindLm : p - 6 * l;
    if (k == kKindAttn) {
      phase_begin(P, sm, ps, P.k2[l].trace_id);
      wait_constants(P, sm, ps);  // an empty list: completes at once (keeps the parity)
      if (ps.live) {  // the auxiliary area is free during attention
        const AttnArgs& a = P.k2[l];
        if (a.d == DS && a.g == GS) attn_items<DS, GS>(a, sm.x0, sm, ps, P.stages, status);
        else if (a.d == DF && a.g == GF) attn_items<DF, GF>(a, sm.x0, sm, ps, P.stages, status);
      }
    } else {
      gemv_phase_body<CPLM>(P, l, k, sm, ps, h);
    }
    if (p < 6 * L)
      phase_end(P, sm, ps, op_base(P, (p + 1) / 6, (p + 1) == 6 * L ? kKindLm : (p + 1) % 6));
    if (k == kKindRouterMlp && sm.ints[kSmemTopk]) {
      // this CTA completed the router logits: it selects the top-k after its arrival, so
      // the next phase's barrier does not wait for the selection (its expert tiles wait for
      // the router flag); the per-tile result buffers are free until that phase's tiles
      named_bar(kBarConsumers, kConsumerThreads);  // every thread has read the slot
      if (threadIdx.x == 0) sm.ints[kSmemTopk] = 0;
      if (ps.live) reinterpret_cast<const RouterMlpOp*>(sm.opc)->router_topk(sm, sm.res);
    }
  }
  named_bar(kBarConsumers, kConsumerThreads);
  if (threadIdx.x == 0) {
    __threadfence();
    const int total = (ps.phase + 1) * (int)gridDim.x;
    const int old = atomicAdd(P.sync + kSyncBarrier, 1);
    if (old == total - 1) {  // every CTA has passed its last wait: reset for the next launch
      atomicExch(P.sync + kSyncBarrier, 0);
      atomicAdd(P.sync + kSyncSeq, 1);
    }
    if (sm.ints[kSmemDead]) drain_ring(sm, ps.wp, P.stages);
  }
}

// ------------------------------------------------------------------ variants
// Each instantiation of step_kernel lives in its own translation unit
// (g4_step_*.cu, compiled in parallel) and registers itself with the runtime.
struct StepVariant {
  int cplm, ds, gs, df, gf;
  const void* kernel;
  int (*trace_read)(void* dst, long long bytes);  // this module's timeline buffer
};
void register_step_variant(const StepVariant& v);  // g4_runtime.cu

}  // namespace g4

#ifdef G4_TRACE
#define G4_STEP_TRACE_READER                                                              \
  static int g4_step_trace_read(void* dst, long long bytes) {                             \
    const long long need = (long long)sizeof(g4::g4_trace_buf);                           \
    if (bytes < need) return -1;                                                          \
    return cudaMemcpyFromSymbol(dst, g4::g4_trace_buf, need) == cudaSuccess ? 0 : -1;     \
  }
#else
#define G4_STEP_TRACE_READER \
  static int g4_step_trace_read(void*, long long) { return -1; }
#endif

// One variant per translation unit.
#define G4_STEP_VARIANT(C, DS, GS, DF, GF)                                                \
  namespace {                                                                             \
  G4_STEP_TRACE_READER                                                                    \
  struct StepVariantRegistration {                                                        \
    StepVariantRegistration() {                                                           \
      g4::register_step_variant(g4::StepVariant{                                          \
          C, DS, GS, DF, GF, reinterpret_cast<const void*>(&g4::step_kernel<C, DS, GS, DF, GF>), \
          &g4_step_trace_read});                                                          \
    }                                                                                     \
  } g4_step_variant_registration;                                                         \
  }
