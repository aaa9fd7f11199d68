// Shared device helpers for the sm_100a decode kernels: element conversion,
// warp reductions, TMA bulk copies (cp.async.bulk) tracked by mbarriers,
// programmatic dependent launch (griddepcontrol), acquire/release atomics and
// bounded waits that record a status instead of hanging.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mie.h"

namespace mie {

constexpr int kWarp = 32;
// Every bounded wait gives up after this many nanoseconds (%globaltimer).
constexpr unsigned long long kWaitLimitNs = 200ull * 1000ull * 1000ull;  // 200 ms

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static constexpr int kPerVec = 4;  // elements per 16-byte vector
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  return dtype == MIE_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i])
                           : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  if (dtype == MIE_BF16)
    static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(p)[i] = v;
}

// dot of one 16-byte vector of weights with fp32 values xs[0..kPerVec); the
// last argument only selects the element type.
__device__ __forceinline__ float dot_vec(const uint4 w, const float* __restrict__ xs, float acc,
                                         const float*) {
  // fp32: 4 elements
  acc = fmaf(__uint_as_float(w.x), xs[0], acc);
  acc = fmaf(__uint_as_float(w.y), xs[1], acc);
  acc = fmaf(__uint_as_float(w.z), xs[2], acc);
  acc = fmaf(__uint_as_float(w.w), xs[3], acc);
  return acc;
}
__device__ __forceinline__ float dot_vec(const uint4 w, const float* __restrict__ xs, float acc,
                                         const __nv_bfloat16*) {
  // bf16: 8 elements; bf16 -> fp32 is a 16-bit shift of the bit pattern
  acc = fmaf(__uint_as_float(w.x << 16), xs[0], acc);
  acc = fmaf(__uint_as_float(w.x & 0xffff0000u), xs[1], acc);
  acc = fmaf(__uint_as_float(w.y << 16), xs[2], acc);
  acc = fmaf(__uint_as_float(w.y & 0xffff0000u), xs[3], acc);
  acc = fmaf(__uint_as_float(w.z << 16), xs[4], acc);
  acc = fmaf(__uint_as_float(w.z & 0xffff0000u), xs[5], acc);
  acc = fmaf(__uint_as_float(w.w << 16), xs[6], acc);
  acc = fmaf(__uint_as_float(w.w & 0xffff0000u), xs[7], acc);
  return acc;
}

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
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
// Block-wide sum with a fixed reduction order (deterministic across CTAs).
// `red` needs blockDim.x/32 floats of shared memory.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];
  return t;
}
__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int i = 0; i < nw; ++i) t = fmaxf(t, red[i]);
  return t;
}

// ---------------------------------------------------------------------------
// time, status
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void set_status(int32_t* status, int code) {
  if (status) atomicCAS(reinterpret_cast<int*>(status), 0, code);
}
__device__ __forceinline__ bool skip_requested(const int32_t* skip) {
  if (!skip) return false;
  return *reinterpret_cast<const volatile int32_t*>(skip) != 0;
}

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------
// Block until the preceding grid in the stream completed and its memory is
// visible.  A no-op when the kernel was launched without the PDL attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid in the stream to start launching.  The per-op kernels
// call this only after their own pdl_wait (and after any grid-wide barrier),
// so at most one dependent grid is ever resident ahead of a running one.  The
// persistent step calls it first thing: its CTAs fill an SM each, so the next
// step's CTAs only take SMs this grid has left.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// global-memory atomics with explicit ordering
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u64(uint64_t* p, uint64_t v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Grid-wide barrier for a grid whose CTAs are all co-resident (grid <= SMs, one
// CTA per SM fits), on a 64-bit counter that only grows: each launch adds
// exactly gridDim.x arrivals, and every launch sharing the counter uses the
// same grid size.  grid_sync_target (thread 0, any time before this CTA
// arrives, e.g. before the PDL wait) gives the value the counter holds once all
// CTAs of this launch arrived: fewer than gridDim.x arrivals of this launch can
// precede the read, so rounding down to a multiple of gridDim.x finds the
// launch's base.  Arrival is one fire-and-forget release add; waiting polls with
// acquire loads.  Bounded: a CTA that waits longer than kWaitLimitNs records
// MIE_ERR_TIMEOUT and returns false (the counter is then no longer aligned and
// must be zeroed by the host before the next launch).
__device__ __forceinline__ uint64_t grid_sync_target(const uint64_t* ctr, uint32_t nblocks) {
  return (ld_relaxed_u64(ctr) / nblocks + 1) * nblocks;
}
__device__ __forceinline__ bool grid_sync(uint64_t* ctr, uint64_t target, int32_t* status) {
  __shared__ int ok_s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    red_release_add_u64(ctr, 1ull);
    if (ld_acquire_u64(ctr) < target) {
      const unsigned long long t0 = global_ns();
      while (ld_acquire_u64(ctr) < target) {
        if (global_ns() - t0 > kWaitLimitNs) {
          ok = 0;
          set_status(status, MIE_ERR_TIMEOUT);
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  return ok_s != 0;
}

// ---------------------------------------------------------------------------
// shared-memory mbarriers + TMA bulk copies (global -> shared)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Make initialised mbarriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Order prior generic-proxy shared-memory accesses before later async-proxy
// writes into the same buffer (slot reuse).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Transaction bytes the current phase also waits for, without an arrival.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// One arrival on an mbarrier (no transaction bytes).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for an mbarrier phase.  Returns false (and records a timeout)
// if the phase did not complete within limit_ns.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* status,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > limit_ns) {
      set_status(status, MIE_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}
// cp.async.bulk global -> shared, completion counted on `bar` in bytes.
// dst and src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Same with an L2 evict-first policy: streamed-once weights should not push
// activations and the KV cache out of L2.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// L2 policy for data reread every decode step and small enough to stay in L2
// (the LM head): kept in preference to streamed data.
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bulk prefetch of [src, src + bytes) into L2 (no completion to wait for);
// src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Largest chunk one bulk copy moves here (bytes); larger ranges are split.
constexpr uint32_t kBulkMax = 1u << 16;

}  // namespace mie
