// SunShape key encode (ProfilePerm + per-block nearest codeword) and dequantize.
//
// encode_kernel: a CTA takes 128 key rows of one head, stages them permuted in
// shared memory (coalesced row reads, scattered through the inverse permutation),
// then walks the blocks: each block's codebook (C x bd fp32) and the codeword
// norms |c|^2 are staged in shared memory and every thread scans all C codewords
// for its key with  d(c) = |c|^2 - 2 k.c  (the |k|^2 term is common to all
// codewords), keeping the FIRST minimum like torch.argmin (codec.py:376-377).
// SunShape-Mixed heavy blocks are copied densely instead and keep index 0
// (codec.py:367-374).
#pragma once

#include "common.cuh"
#include "encode_params.cuh"

namespace sunshape {



template <int BD>
__global__ void __launch_bounds__(kEncRows) encode_kernel(const __grid_constant__ EncodeParams p) {
  extern __shared__ __align__(16) float esm[];
  const int D = p.D, C = p.C;
  const int ldk = D + 1;
  float* keys_s = esm;                          // [128][D+1]
  float* cb_s = keys_s + kEncRows * ldk;        // [C][BD]
  float* cn_s = cb_s + C * BD;                  // [C]
  int* inv_s = reinterpret_cast<int*>(cn_s + C);  // [D]
  int8_t* hslot_s = reinterpret_cast<int8_t*>(inv_s + D);  // [nb]

  const int tid = threadIdx.x;
  const int64_t hh = blockIdx.y;
  const int row0 = blockIdx.x * kEncRows;
  const int nrows = min(kEncRows, p.n_tokens - row0);

  for (int i = tid; i < D; i += kEncRows) inv_s[(int)p.perm[i]] = i;
  if (tid == 0) {
    int n = 0;
    for (int b = 0; b < p.nb; ++b) {
      const bool h = p.heavy_mask != nullptr && p.heavy_mask[b] != 0;
      hslot_s[b] = h ? (int8_t)n++ : (int8_t)-1;
    }
  }
  __syncthreads();
  int n_heavy = 0;
  for (int b = 0; b < p.nb; ++b) n_heavy += hslot_s[b] >= 0;

  // stage the permuted key rows: keys_s[r][inv[d]] = key[r][d]
  for (int r = 0; r < nrows; ++r) {
    const int64_t base = hh * p.key_hs + (int64_t)(row0 + r) * p.key_ts;
    for (int d = tid; d < D; d += kEncRows)
      keys_s[r * ldk + inv_s[d]] = load_as_float(p.keys, base + d, p.keys_dtype);
  }

  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const float* cb = p.cb + (int64_t)cbh * p.nb * C * BD;
  const int64_t orow = hh * p.out_hs + row0 + tid;

  for (int b = 0; b < p.nb; ++b) {
    __syncthreads();   // keys staged / previous block's codebook no longer read
    if (hslot_s[b] >= 0) {
      if (tid < nrows) {
        const int64_t o = (orow * n_heavy + hslot_s[b]) * BD;
#pragma unroll
        for (int d = 0; d < BD; ++d)
          store_from_float(p.heavy_out, o + d, p.heavy_dtype, keys_s[tid * ldk + b * BD + d]);
        if (p.index_dtype == SUNSHAPE_U8) reinterpret_cast<uint8_t*>(p.idx_out)[orow * p.nb + b] = 0;
        else if (p.index_dtype == SUNSHAPE_I16) reinterpret_cast<int16_t*>(p.idx_out)[orow * p.nb + b] = 0;
        else reinterpret_cast<int32_t*>(p.idx_out)[orow * p.nb + b] = 0;
      }
      continue;
    }
    const float* cbb = cb + (int64_t)b * C * BD;
    for (int e = tid; e < C * BD; e += kEncRows) cb_s[e] = __ldg(cbb + e);
    __syncthreads();
    for (int c = tid; c < C; c += kEncRows) {
      float n2 = 0.f;
#pragma unroll
      for (int d = 0; d < BD; ++d) n2 = fmaf(cb_s[c * BD + d], cb_s[c * BD + d], n2);
      cn_s[c] = n2;
    }
    __syncthreads();
    if (tid < nrows) {
      float x[BD];
#pragma unroll
      for (int d = 0; d < BD; ++d) x[d] = keys_s[tid * ldk + b * BD + d];
      float best = __int_as_float(0x7f800000);
      int besti = 0;
#pragma unroll 4
      for (int c = 0; c < C; ++c) {
        float dot = 0.f;
#pragma unroll
        for (int d = 0; d < BD; ++d) dot = fmaf(x[d], cb_s[c * BD + d], dot);
        const float dist = fmaf(-2.f, dot, cn_s[c]);
        if (dist < best) { best = dist; besti = c; }
      }
      if (p.index_dtype == SUNSHAPE_U8) reinterpret_cast<uint8_t*>(p.idx_out)[orow * p.nb + b] = (uint8_t)besti;
      else if (p.index_dtype == SUNSHAPE_I16) reinterpret_cast<int16_t*>(p.idx_out)[orow * p.nb + b] = (int16_t)besti;
      else reinterpret_cast<int32_t*>(p.idx_out)[orow * p.nb + b] = besti;
    }
  }
}

struct DequantParams {
  const void* idx;
  int index_dtype;
  const void* heavy;
  int heavy_dtype;
  int64_t head_stride;
  int T, kv_heads;
  const float* cb;
  int n_cb;
  const int64_t* perm;
  const uint8_t* heavy_mask;
  int nb, bd, C, D;
  float* out;
};

// out[hh][t][d] = k_hat_perm[inv_perm[d]]  (codec.py:387-398 then _inverse_transform :254-256)
// i.e. out[hh][t][perm[d']] = centroid / passthrough value at permuted position d'.
__global__ void dequant_kernel(const __grid_constant__ DequantParams p) {
  const int64_t hh = blockIdx.y;
  const int64_t n = (int64_t)p.T * p.D;
  int n_heavy = 0;
  if (p.heavy_mask)
    for (int b = 0; b < p.nb; ++b) n_heavy += p.heavy_mask[b] != 0;
  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const float* cb = p.cb + (int64_t)cbh * p.nb * p.C * p.bd;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(e / p.D), dp = (int)(e - (int64_t)t * p.D);
    const int b = dp / p.bd, w = dp - b * p.bd;
    const int64_t row = hh * p.head_stride + t;
    float v;
    if (p.heavy_mask && p.heavy_mask[b]) {
      int slot = 0;
      for (int bb = 0; bb < b; ++bb) slot += p.heavy_mask[bb] != 0;
      v = load_as_float(p.heavy, (row * n_heavy + slot) * p.bd + w, p.heavy_dtype);
    } else {
      int c;
      if (p.index_dtype == SUNSHAPE_U8) c = reinterpret_cast<const uint8_t*>(p.idx)[row * p.nb + b];
      else if (p.index_dtype == SUNSHAPE_I16) c = reinterpret_cast<const int16_t*>(p.idx)[row * p.nb + b];
      else c = reinterpret_cast<const int32_t*>(p.idx)[row * p.nb + b];
      v = cb[((int64_t)b * p.C + c) * p.bd + w];
    }
    p.out[(hh * p.T + t) * p.D + p.perm[dp]] = v;
  }
}

}  // namespace sunshape
