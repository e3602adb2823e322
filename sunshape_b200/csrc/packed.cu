// Scores against bit-packed and wide codeword indices.
//
// The fused decode kernels read one uint8 index per block.  Two other storage formats exist:
//
//   * bit-packed indices for codebooks of 2, 4 or 16 codewords (1, 2 or 4 bits per block): the
//     format of the reference's packed-index kernel (triton_kernels.py:213-292) with uint8 elements --
//     row t is ceil(n_blocks * bits / 8) bytes, block b sits in byte b / (8 / bits) at bit offset
//     (b % (8 / bits)) * bits;
//   * int16 / int32 indices for codebooks above 256 codewords (codec.py:78-83).
//
// lut_scores_kernel serves both: every CTA builds the per-row LUT  lut[b][c][g] = q_b . C_b[c]
// (triton_kernels.py:381-408) for its rows in shared memory, then each thread scores one token as
// sum_b lut[b][idx[t, b]][g] (triton_kernels.py:134-204), unpacking the indices on the fly.
// pack_indices_kernel produces the packed format from uint8 indices.
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"

namespace sunshape {
int set_last_error(int code, const char* msg);   // defined in capi.cu

namespace {

constexpr int kScoreThreads = 256;
constexpr int kMaxRows = 16;

struct ScoreParams {
  const float* cb;          // [n_cb, nb, C, bd]
  int n_cb, kv_heads;
  const int64_t* perm;
  const void* q;            // [n_heads, rows, D]
  int q_dtype;
  const uint8_t* idx;       // [n_heads, head_stride, row_bytes]
  int index_kind;           // 1, 2, 4 = packed bits; 16 = int16; 32 = int32; 8 = uint8
  int64_t row_bytes, head_stride;
  int T, rows, nb, bd, C, D;
  float* out;               // [n_heads, rows, T]
};

__device__ __forceinline__ int index_at(const uint8_t* row, int b, int kind) {
  switch (kind) {
    case 8: return row[b];
    case 16: return (int)reinterpret_cast<const uint16_t*>(row)[b];
    case 32: return reinterpret_cast<const int32_t*>(row)[b];
    default: {
      const int per = 8 / kind;
      return (row[b / per] >> ((b % per) * kind)) & ((1 << kind) - 1);
    }
  }
}

__global__ void __launch_bounds__(kScoreThreads) lut_scores_kernel(const __grid_constant__ ScoreParams p) {
  extern __shared__ float lut_s[];                    // [nb][C][rows]
  __shared__ float q_s[kMaxRows * 256];
  const int64_t hh = blockIdx.y;
  const int tid = threadIdx.x;
  for (int e = tid; e < p.rows * p.D; e += kScoreThreads) {
    const int g = e / p.D, d = e - g * p.D;
    q_s[e] = load_as_float(p.q, (hh * p.rows + g) * p.D + (int)__ldg(p.perm + d), p.q_dtype);
  }
  __syncthreads();
  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const float* cb = p.cb + (int64_t)cbh * p.nb * p.C * p.bd;
  for (int e = tid; e < p.nb * p.C; e += kScoreThreads) {
    const int b = e / p.C;
    const float* cr = cb + (int64_t)e * p.bd;
    for (int g = 0; g < p.rows; ++g) {
      float a = 0.f;
      for (int d = 0; d < p.bd; ++d) a = fmaf(q_s[g * p.D + b * p.bd + d], __ldg(cr + d), a);
      lut_s[(int64_t)e * p.rows + g] = a;
    }
  }
  __syncthreads();
  const int t = blockIdx.x * kScoreThreads + tid;
  if (t >= p.T) return;
  const uint8_t* row = p.idx + (hh * p.head_stride + t) * p.row_bytes;
  float acc[kMaxRows];
#pragma unroll
  for (int g = 0; g < kMaxRows; ++g) acc[g] = 0.f;
  for (int b = 0; b < p.nb; ++b) {
    const float* ent = lut_s + ((int64_t)b * p.C + index_at(row, b, p.index_kind)) * p.rows;
#pragma unroll
    for (int g = 0; g < kMaxRows; ++g)
      if (g < p.rows) acc[g] += ent[g];
  }
#pragma unroll
  for (int g = 0; g < kMaxRows; ++g)
    if (g < p.rows) p.out[(hh * p.rows + g) * (int64_t)p.T + t] = acc[g];
}

__global__ void pack_indices_kernel(const uint8_t* __restrict__ idx, int64_t n_rows, int nb, int bits, int row_bytes,
                                    uint8_t* __restrict__ out) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;   // one output byte
  if (e >= n_rows * row_bytes) return;
  const int64_t r = e / row_bytes;
  const int j = (int)(e - r * row_bytes);
  const int per = 8 / bits;
  unsigned v = 0;
  for (int k = 0; k < per; ++k) {
    const int b = j * per + k;
    if (b < nb) v |= (unsigned)(idx[r * nb + b] & ((1 << bits) - 1)) << (k * bits);
  }
  out[e] = (uint8_t)v;
}

int index_row_bytes(int kind, int nb) {
  if (kind == 8) return nb;
  if (kind == 16) return 2 * nb;
  if (kind == 32) return 4 * nb;
  return (nb * kind + 7) / 8;
}

}  // namespace
}  // namespace sunshape

using namespace sunshape;

extern "C" int64_t sunshape_index_row_bytes(int32_t index_bits, int32_t n_blocks) {
  if (!(index_bits == 1 || index_bits == 2 || index_bits == 4 || index_bits == 8 || index_bits == 16 ||
        index_bits == 32) || n_blocks <= 0)
    return 0;
  return index_row_bytes(index_bits, n_blocks);
}

extern "C" int sunshape_pack_indices(const uint8_t* indices, int64_t n_rows, int32_t n_blocks, int32_t bits,
                                     uint8_t* packed, void* stream) {
  if (!indices || !packed) return set_last_error(SUNSHAPE_E_INVALID, "indices / packed pointer is NULL.");
  if (!(bits == 1 || bits == 2 || bits == 4)) return set_last_error(SUNSHAPE_E_INVALID, "bits must be 1, 2 or 4.");
  if (n_rows < 0 || n_blocks <= 0) return set_last_error(SUNSHAPE_E_INVALID, "bad pack sizes.");
  const int rb = index_row_bytes(bits, n_blocks);
  const int64_t n = n_rows * rb;
  if (n == 0) return SUNSHAPE_OK;
  pack_indices_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      indices, n_rows, n_blocks, bits, rb, packed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_last_error(SUNSHAPE_E_CUDA, (std::string("pack launch: ") + cudaGetErrorString(e)).c_str());
  return SUNSHAPE_OK;
}

extern "C" int sunshape_attention_scores_packed(const sunshape_codec_t* codec, const void* indices, int32_t index_bits,
                                                int32_t seq_len, int64_t head_stride, const void* query,
                                                int32_t query_dtype, int32_t n_heads, int32_t kv_heads, int32_t rows,
                                                float* scores_out, void* stream) {
  if (!codec || !codec->centroids || !codec->permutation)
    return set_last_error(SUNSHAPE_E_INVALID, "codec descriptor / buffers are NULL.");
  if (!indices || !query || !scores_out) return set_last_error(SUNSHAPE_E_INVALID, "indices / query / out is NULL.");
  if (codec->block_dim <= 0 || codec->head_dim % codec->block_dim)
    return set_last_error(SUNSHAPE_E_INVALID, "head_dim must be divisible by block_dim");
  if (codec->head_dim > 256) return set_last_error(SUNSHAPE_E_UNSUPPORTED, "head_dim > 256 is not supported.");
  if (codec->heavy_mask && codec->n_heavy > 0)
    return set_last_error(SUNSHAPE_E_UNSUPPORTED, "packed / wide index scores do not take SunShape-Mixed heavy blocks.");
  const int64_t rb = sunshape_index_row_bytes(index_bits, codec->head_dim / codec->block_dim);
  if (!rb) return set_last_error(SUNSHAPE_E_INVALID, "index_bits must be 1, 2, 4, 8, 16 or 32.");
  if (index_bits <= 8 && codec->n_centroids > (1 << index_bits))
    return set_last_error(SUNSHAPE_E_INVALID, "n_centroids does not fit in index_bits.");
  if (rows <= 0 || rows > kMaxRows) return set_last_error(SUNSHAPE_E_UNSUPPORTED, "rows per head must be in [1, 16].");
  if (seq_len < 0 || head_stride < seq_len || n_heads < 0 || kv_heads <= 0)
    return set_last_error(SUNSHAPE_E_INVALID, "bad sizes.");
  if ((index_bits == 16 && (reinterpret_cast<uintptr_t>(indices) & 1)) ||
      (index_bits == 32 && (reinterpret_cast<uintptr_t>(indices) & 3)))
    return set_last_error(SUNSHAPE_E_INVALID, "wide index buffer is misaligned.");
  ScoreParams p{};
  p.cb = codec->centroids; p.n_cb = codec->n_cb; p.kv_heads = kv_heads; p.perm = codec->permutation;
  p.q = query; p.q_dtype = query_dtype; p.idx = reinterpret_cast<const uint8_t*>(indices);
  p.index_kind = index_bits; p.row_bytes = rb; p.head_stride = head_stride; p.T = seq_len; p.rows = rows;
  p.D = codec->head_dim; p.bd = codec->block_dim; p.nb = p.D / p.bd; p.C = codec->n_centroids; p.out = scores_out;
  const int64_t smem = (int64_t)p.nb * p.C * rows * 4;
  if (smem > 200 * 1024)
    return set_last_error(SUNSHAPE_E_UNSUPPORTED, "the LUT (n_blocks x n_centroids x rows fp32) exceeds shared memory; "
                                                  "call with fewer rows per head.");
  if (n_heads == 0 || seq_len == 0) return SUNSHAPE_OK;
  cudaFuncSetAttribute(lut_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((seq_len + kScoreThreads - 1) / kScoreThreads, n_heads);
  lut_scores_kernel<<<grid, kScoreThreads, (size_t)smem, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_last_error(SUNSHAPE_E_CUDA, (std::string("packed scores launch: ") + cudaGetErrorString(e)).c_str());
  return SUNSHAPE_OK;
}
