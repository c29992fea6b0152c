// Device-side building blocks shared by every g4b200 kernel (sm_100a only).
//
//  * bf16 <-> fp32 conversions with explicit round-to-nearest-even, so every point
//    where the reference rounds an fp32 value to bf16 is reproduced bit for bit;
//  * mbarrier + cp.async.bulk (TMA bulk copy) wrappers for the weight-streaming
//    pipelines, with an L2 evict-first policy (weights are read once per token);
//  * programmatic dependent launch (griddepcontrol) wrappers;
//  * bounded waits: every spin on an mbarrier or on a peer flag gives up after a
//    %globaltimer deadline, records a status bit and lets the kernel return.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/g4b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "g4b200 kernels target sm_100a (B200) only"
#endif

namespace g4 {

typedef uint16_t bf16_t;  // raw bf16 storage

constexpr int kMaxWorld = 8;
constexpr int kMaxTopK = 16;
constexpr uint64_t kLocalTimeoutNs = 2000000000ull;  // 2 s for local TMA completions

// ------------------------------------------------------------------ bf16 helpers
__host__ __device__ __forceinline__ float bf2f(bf16_t v) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(static_cast<uint32_t>(v) << 16);
#else
  uint32_t u = static_cast<uint32_t>(v) << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// fp32 -> bf16, round to nearest even (NaN kept quiet).
__device__ __forceinline__ bf16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

// Round an fp32 value to the nearest bf16 and return it as fp32.
__device__ __forceinline__ float rbf(float f) { return bf2f(f2bf(f)); }

// Unpack a 32-bit word holding two bf16 values (low element first in memory).
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// 8-element bf16 dot product of two 16-byte chunks, accumulated into `acc`.
__device__ __forceinline__ float dot8(const uint4 w, const uint4 x, float acc) {
  acc = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
  acc = fmaf(bf_hi(w.x), bf_hi(x.x), acc);
  acc = fmaf(bf_lo(w.y), bf_lo(x.y), acc);
  acc = fmaf(bf_hi(w.y), bf_hi(x.y), acc);
  acc = fmaf(bf_lo(w.z), bf_lo(x.z), acc);
  acc = fmaf(bf_hi(w.z), bf_hi(x.z), acc);
  acc = fmaf(bf_lo(w.w), bf_lo(x.w), acc);
  acc = fmaf(bf_hi(w.w), bf_hi(x.w), acc);
  return acc;
}

// tanh-approximate GELU in fp32 (jax.nn.gelu(approximate=True) formula).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f;  // sqrt(2/pi)
  float cdf = 0.5f * (1.0f + tanhf(k0 * (x + 0.044715f * x * x * x)));
  return x * cdf;
}

// ------------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over groups of `width` consecutive lanes (width a power of two <= 32).
__device__ __forceinline__ float group_sum(float v, int width) {
  for (int o = width >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy and the other threads.
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for phase `parity` of `bar`; gives up after kLocalTimeoutNs and sets `status`.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kLocalTimeoutNs) {
      if (status) atomicOr(status, G4_STATUS_MBAR_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 1-D TMA bulk copy global -> shared; completion is signalled on `bar` as tx bytes.
// dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Programmatic dependent launch: wait for the previous kernel's memory / allow the
// next kernel to be scheduled.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Named barrier among `nthreads` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// System-scope acquire/release accessors for cross-GPU flags.
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

// GPU-scope acquire/release accessors for flags between CTAs of one launch.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// L2-coherent loads for data produced by other kernels or other GPUs (bypass L1).
__device__ __forceinline__ float ldcg_f(const float* p) { return __ldcg(p); }
__device__ __forceinline__ int ldcg_i(const int* p) { return __ldcg(p); }
__device__ __forceinline__ bf16_t ldcg_bf(const bf16_t* p) {
  return __ldcg(reinterpret_cast<const unsigned short*>(p));
}
__device__ __forceinline__ uint4 ldcg_u4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}

// Wait until *flag >= target (flag written by a peer with st.release.sys).
// Gives up after timeout_us microseconds, setting G4_STATUS_PEER_TIMEOUT in *status.
__device__ __forceinline__ bool wait_flag_geq(const int* flag, int target, int timeout_us,
                                              int* status) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t limit = static_cast<uint64_t>(timeout_us > 0 ? timeout_us : 1000000) * 1000ull;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(flag) < target) {
    if (globaltimer_ns() - t0 > limit) {
      atomicOr(status, G4_STATUS_PEER_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

// ------------------------------------------------------------------ timeline tracing
// Built only with -DG4_TRACE (libg4b200_trace.so): %globaltimer stamps of selected
// events for the first kTraceCtas CTAs of every launch whose trace id is in
// [0, kTraceLaunches); read back with g4_trace_read.
constexpr int kTraceLaunches = 512, kTraceCtas = 160, kTraceEvents = 8;
#ifdef G4_TRACE
// one buffer per device module (each translation unit of the library is its own module)
static __device__ unsigned long long g4_trace_buf[kTraceLaunches][kTraceCtas][kTraceEvents];
__device__ __forceinline__ int trace_cta_slot() {
  return (int)blockIdx.x < kTraceCtas ? (int)blockIdx.x : -1;
}
#define G4_TRACE_EV(id, ev)                                                         \
  do {                                                                              \
    const int s_ = ::g4::trace_cta_slot();                                          \
    if (s_ >= 0 && (id) >= 0 && (id) < ::g4::kTraceLaunches)                        \
      ::g4::g4_trace_buf[(id)][s_][(ev)] = ::g4::globaltimer_ns();                  \
  } while (0)
#else
#define G4_TRACE_EV(id, ev) \
  do {                      \
  } while (0)
#endif

// ------------------------------------------------------------------ block reductions
// Sum of `v` over the first `nthreads` threads of the block (a multiple of 32), using
// `red` (>= 32 floats of shared memory) and named barrier `bar_id`.
__device__ __forceinline__ float block_sum(float v, float* red, int nthreads, int bar_id) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = nthreads >> 5;
  v = warp_sum(v);
  named_bar(bar_id, nthreads);  // previous users of `red` are done
  if (lane == 0) red[warp] = v;
  named_bar(bar_id, nthreads);
  float s = 0.f;
  for (int i = 0; i < nw; ++i) s += red[i];  // fixed order: identical on every thread
  return s;
}

// ------------------------------------------------------------------ stage rings
// Position in a ring of shared-memory stages (full / empty mbarrier per stage),
// advanced identically by the producer lane and the consumers of a CTA.
struct RingPos {
  int st = 0;         // stage index
  uint32_t ph = 0;    // parity of the stage's current fill
  bool wrapped = false;  // the ring has been filled once (the producer waits for `empty`)
  int tiles = 0;      // tiles passed so far
  __device__ __forceinline__ void next(int stages) {
    ++tiles;
    if (++st == stages) {
      st = 0;
      ph ^= 1u;
      wrapped = true;
    }
  }
};

}  // namespace g4
