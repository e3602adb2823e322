// Decode attention without any device allocation.
//
// Some hosts cannot hand this library a workspace or let it call cudaMalloc: plugin hosts whose
// device memory is owned by another allocator, engines that reserve all GPU memory up front and
// forbid allocation on the decode path, and thin foreign-language bindings with no access to a
// CUDA allocator.  For them sunshape_decode_attention_noalloc runs the same fused decode kernel
// with its scratch (error word, per-head tickets, per-CTA partial slots) in a fixed-size array
// compiled into this library.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/sunshape_b200.h"

namespace sunshape {
int set_last_error(int code, const char* msg);   // defined in capi.cu
}

namespace {

// Built-in decode scratch: SUNSHAPE_NOALLOC_SCRATCH_BYTES on every GPU that loads the library,
// held until the process exits.  Host code must not pass this name to a kernel: on the host it
// only stands in for the device array; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_decode_scratch[SUNSHAPE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 128;
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Resolve (once per device, with that device current) the device address of the array.  The address
// is cached for the life of the process: after cudaDeviceReset the module is reloaded at a possibly
// different address, so a process that resets a device must not call the entry point again.
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return sunshape::set_last_error(SUNSHAPE_E_CUDA, (std::string("cudaGetDevice: ") + cudaGetErrorString(e)).c_str());
  if (dev < 0 || dev >= kMaxDevices) return sunshape::set_last_error(SUNSHAPE_E_UNSUPPORTED, "device ordinal too large.");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || p == nullptr)
      return sunshape::set_last_error(
          SUNSHAPE_E_CUDA, (std::string("cudaGetSymbolAddress(decode scratch): ") + cudaGetErrorString(e)).c_str());
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return SUNSHAPE_OK;
}

int round_up(int64_t x, int64_t a) { return (int)((x + a - 1) / a * a); }

}  // namespace

extern "C" int sunshape_decode_attention_noalloc(
    const sunshape_codec_t* codec, const sunshape_kv_t* kv, const void* query, int32_t query_dtype, int32_t batch,
    int32_t q_heads, int32_t kv_heads, int32_t query_len, const void* mask, int32_t mask_dtype, int64_t mask_sb,
    int64_t mask_sh, int64_t mask_sq, float scale, void* out, int32_t out_dtype, float* partials, void* stream) {
  if (!kv) return sunshape::set_last_error(SUNSHAPE_E_INVALID, "KV descriptor is NULL.");
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || query_len <= 0 || q_heads % kv_heads != 0)
    return sunshape::set_last_error(SUNSHAPE_E_INVALID, "batch must be >= 0, heads / query_len positive, q_heads a "
                                                        "multiple of kv_heads.");
  if (batch == 0)   // nothing to decode: the regular entry point validates the rest and returns OK
    return sunshape_decode_attention(codec, kv, query, query_dtype, batch, q_heads, kv_heads, query_len, mask,
                                     mask_dtype, mask_sb, mask_sh, mask_sq, scale, out, out_dtype, partials, nullptr,
                                     0, stream);
  const int32_t n_heads = batch * kv_heads;
  // the smallest workspace the decode accepts (per-head LUTs then live in each CTA's shared memory); when
  // the array also holds the LUT area, the decode uses it on its own
  const int64_t need = sunshape_decode_workspace_min_bytes(n_heads, kv->seq_len, (q_heads / kv_heads) * query_len,
                                                           kv->value_dim);
  if (need > (int64_t)SUNSHAPE_NOALLOC_SCRATCH_BYTES)
    return sunshape::set_last_error(
        SUNSHAPE_E_WORKSPACE,
        ("this decode needs " + std::to_string(need) + " bytes of scratch, more than the " +
         std::to_string((long long)SUNSHAPE_NOALLOC_SCRATCH_BYTES) +
         "-byte built-in array of sunshape_decode_attention_noalloc; use sunshape_decode_attention with a "
         "caller-provided workspace")
            .c_str());
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  // the error word and the per-head tickets must start at zero (the array keeps the last call's contents)
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const cudaError_t e = cudaMemsetAsync(scratch, 0, 256 + round_up((int64_t)n_heads * 4, 256), st);
  if (e != cudaSuccess)
    return sunshape::set_last_error(SUNSHAPE_E_CUDA, (std::string("clearing decode scratch: ") + cudaGetErrorString(e)).c_str());
  return sunshape_decode_attention(codec, kv, query, query_dtype, batch, q_heads, kv_heads, query_len, mask, mask_dtype,
                                   mask_sb, mask_sh, mask_sq, scale, out, out_dtype, partials, scratch,
                                   (int64_t)SUNSHAPE_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int sunshape_decode_attention_noalloc_error(int32_t* code) {
  if (!code) return sunshape::set_last_error(SUNSHAPE_E_INVALID, "code pointer is NULL.");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(code, g_decode_scratch, sizeof(int32_t), 0, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess)
    return sunshape::set_last_error(SUNSHAPE_E_CUDA,
                                    (std::string("reading the decode scratch error word: ") + cudaGetErrorString(e)).c_str());
  return SUNSHAPE_OK;
}
