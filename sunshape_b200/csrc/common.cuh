// Shared device helpers for the sm_100a SunShape kernels: element loads and
// conversions, mbarrier waits with an iteration cap, and the 1-D bulk-copy
// (TMA engine) primitives used to stream index / value tiles into shared memory.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/sunshape_b200.h"

namespace sunshape {

constexpr float kLog2e = 1.4426950408889634f;

// --------------------------------------------------------------------------
// element conversion
// --------------------------------------------------------------------------
__device__ __forceinline__ float load_as_float(const void* base, int64_t i, int dtype) {
  if (dtype == SUNSHAPE_F32) return reinterpret_cast<const float*>(base)[i];
  if (dtype == SUNSHAPE_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return __half2float(reinterpret_cast<const __half*>(base)[i]);
}

// Round an fp32 value to the given 16-bit dtype and back (the reference scales
// the query in its own dtype before upcasting, vllm_attn_backend.py:235-236).
__device__ __forceinline__ float round_to_dtype(float x, int dtype) {
  if (dtype == SUNSHAPE_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (dtype == SUNSHAPE_F16) return __half2float(__float2half_rn(x));
  return x;
}

__device__ __forceinline__ void store_from_float(void* base, int64_t i, int dtype, float v) {
  if (dtype == SUNSHAPE_F32) reinterpret_cast<float*>(base)[i] = v;
  else if (dtype == SUNSHAPE_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
}

// exp2 on the SFU (ex2.approx, relative error ~2^-22).  Inputs are <= 0 here.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Softmax weight e^d (d <= 0).  The fp32-value path uses the accurate expf so its outputs stay within
// the fp32 parity bound at large logits; the 16-bit paths use ex2.approx (their P is rounded to
// 16 bits anyway).
template <bool PRECISE>
__device__ __forceinline__ float softmax_weight(float d) {
  if constexpr (PRECISE) return expf(d);
  else return fast_exp2(d * kLog2e);
}

// --------------------------------------------------------------------------
// mbarrier + bulk copy (cp.async.bulk, the TMA engine's 1-D mode)
// --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Device error word: first writer wins; the host reads it after the call.
__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Bounded wait.  Gives up after kWaitLimitNs of wall time, records `code` in
// the error word and returns false; callers then carry on with the protocol
// (the results are flagged as invalid) so the kernel always terminates.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - t0 > kWaitLimitNs) {
      record_error(err, code);
      return false;
    }
  }
}

// Global -> shared bulk copy completing on an mbarrier (transaction bytes).
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled TMA load (cp.async.bulk.tensor) of box (x, y) of the tensor map into shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of a 16-byte aligned global range (size a multiple of 16)
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// order this thread's generic-proxy shared-memory writes before later async-proxy (TMA) writes
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace sunshape
