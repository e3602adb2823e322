// Arguments of the key encode kernels (encode.cuh: CUDA cores; encode_tc.cu: tcgen05).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace sunshape {

constexpr int kEncRows = 128;

struct EncodeParams {
  const void* keys;
  int keys_dtype;
  int64_t key_hs, key_ts;   // head / token strides (elements)
  int n_tokens, kv_heads;
  const float* cb;
  int n_cb;
  const int64_t* perm;
  const uint8_t* heavy_mask;
  int nb, bd, C, D;
  void* idx_out;
  int index_dtype;
  void* heavy_out;
  int heavy_dtype;
  int64_t out_hs;           // output head stride (tokens)
  int* err;                 // device error word for bounded waits (may be null)
};

// tensor-core (tcgen05) encode, encode_tc.cu
bool encode_tc_supported(const EncodeParams& p);
// returns 0 when launched, -1 when this shape must use encode_kernel instead
int launch_encode_tc(const EncodeParams& p, int n_heads, int n_heavy, cudaStream_t st);
// read (and optionally clear) the encode kernels' device error word; returns a cudaError_t
int encode_error_word(int* code, bool clear);

}  // namespace sunshape
