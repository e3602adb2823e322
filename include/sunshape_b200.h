/*
 * sunshape_b200 -- C ABI of the B200 (sm_100a) SunShape quantized-key decode path.
 *
 * Every pointer argument is a DEVICE pointer unless stated otherwise; buffers
 * are owned by the caller; every call is asynchronous on the given CUDA stream
 * (a cudaStream_t passed as void*, NULL = legacy default stream) and returns
 * SUNSHAPE_OK (0) or a negative SUNSHAPE_E_* code.  On error,
 * sunshape_last_error() returns a thread-local message in the style of the
 * reference's "fast path unavailable" reasons.  There is no CPU fallback: an
 * unsupported input is an error, never a silent slow path.
 *
 * Reference interfaces replaced (paths inside gauravsaini/sunshape):
 *   sunshape_encode            <- SunShapeBlockCodec.quantize         sunshape/codec.py:362-385
 *                                 quantize_key_states (per-head loop) sunshape/vllm_attn_backend.py:101-123
 *   sunshape_dequantize        <- SunShapeBlockCodec.dequantize       sunshape/codec.py:387-398
 *   sunshape_attention_scores  <- sunshape_attention_scores           sunshape/triton_kernels.py:570-609
 *                                 (+ _precompute_query_centroid_dots  :381-408,
 *                                  _sunshape_precomputed_scores_kernel :134-204)
 *   sunshape_decode_attention  <- _apply_quantized_attention          sunshape/vllm_attn_backend.py:216-253
 *                                 (called by SunShapeAttentionImpl.forward :271-305)
 *   sunshape_merge_partials    <- no counterpart: the reference has no KV-sequence split;
 *                                 this merges per-shard (max, sum, acc) partials.
 */
#ifndef SUNSHAPE_B200_H
#define SUNSHAPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SUNSHAPE_ABI_VERSION 1

/* status codes */
#define SUNSHAPE_OK 0
#define SUNSHAPE_E_INVALID (-1)      /* bad argument (shape, pointer, alignment) */
#define SUNSHAPE_E_UNSUPPORTED (-2)  /* valid input outside what the kernels cover */
#define SUNSHAPE_E_CUDA (-3)         /* CUDA runtime error (launch, device)        */
#define SUNSHAPE_E_WORKSPACE (-4)    /* workspace missing or too small             */

/* element types */
#define SUNSHAPE_F32 0
#define SUNSHAPE_BF16 1
#define SUNSHAPE_F16 2
#define SUNSHAPE_U8 3
#define SUNSHAPE_I16 4
#define SUNSHAPE_I32 5

/* One layer's codec (the buffers of SunShapeBlockCodec, codec.py:230-245, E = I).
 * centroids holds n_cb codebooks; KV head h (h = flat_head % kv_heads) uses
 * codebook (n_cb == 1 ? 0 : h % n_cb), so n_cb = 1 is the reference layout
 * (one codec per layer) and n_cb = kv_heads gives per-KV-head codebooks. */
typedef struct sunshape_codec {
  const float* centroids;      /* [n_cb, n_blocks, n_centroids, block_dim] fp32            */
  const int64_t* permutation;  /* [head_dim] ProfilePerm: permuted[d'] = x[permutation[d']] */
  const uint8_t* heavy_mask;   /* [n_blocks] 1 = SunShape-Mixed dense block, or NULL        */
  int32_t n_cb;
  int32_t head_dim;
  int32_t block_dim;
  int32_t n_centroids;
  int32_t n_heavy;             /* number of nonzero heavy_mask entries (0 without a mask)  */
  const float* centroid_norm_max; /* [n_cb] max_{b,c} |centroids[cb,b,c,:]| (optional, NULL =
                                     computed on the device when a kernel needs it)            */
} sunshape_codec_t;

/* Quantized KV storage of n_heads (= batch * kv_heads) heads, head-major.
 * Row (head, token) of each array starts at ((head * head_stride) + token) rows. */
typedef struct sunshape_kv {
  const void* indices;     /* [n_heads, head_stride, n_blocks] codeword indices         */
  int32_t index_dtype;     /* SUNSHAPE_U8 (decode/scores); U8/I16/I32 for dequantize     */
  const void* heavy;       /* [n_heads, head_stride, n_heavy, block_dim] dense blocks, or NULL */
  int32_t heavy_dtype;     /* SUNSHAPE_BF16 or SUNSHAPE_F32                             */
  const void* value;       /* [n_heads, head_stride, value_dim], or NULL (scores only)   */
  int32_t value_dtype;     /* F32 / BF16 / F16                                          */
  int32_t value_dim;
  int32_t seq_len;         /* tokens used per head                                      */
  int64_t head_stride;     /* tokens between consecutive heads (>= seq_len)             */
} sunshape_kv_t;

int sunshape_abi_version(void);
const char* sunshape_last_error(void);

/* Encode keys: ProfilePerm, then per block the nearest codeword (first index on
 * ties), or a dense copy of SunShape-Mixed heavy blocks.
 * keys: row (head, token) at keys + head*key_head_stride + token*key_token_stride (elements).
 * indices_out: [n_heads, out_head_stride, n_blocks] of index_dtype (U8/I16/I32).
 * heavy_out: [n_heads, out_head_stride, n_heavy, block_dim] of heavy_dtype, or NULL. */
int sunshape_encode(const sunshape_codec_t* codec, const void* keys, int32_t keys_dtype,
                    int32_t n_heads, int32_t kv_heads, int32_t n_tokens,
                    int64_t key_head_stride, int64_t key_token_stride,
                    void* indices_out, int32_t index_dtype,
                    void* heavy_out, int32_t heavy_dtype, int64_t out_head_stride,
                    void* stream);

/* First device-side error code recorded by an encode kernel on the current device since the last
 * clear (0 = none; 121 = a tensor-core completion wait gave up, the indices of that launch are
 * invalid).  Waits for the device's queued work (cudaMemcpyFromSymbol); clear != 0 resets the word.
 * No counterpart in the reference (its encode runs on the host). */
int sunshape_encode_error(int32_t* code, int32_t clear);

/* Dequantize into the model basis: out [n_heads, seq_len, head_dim] fp32. */
int sunshape_dequantize(const sunshape_codec_t* codec, const sunshape_kv_t* kv,
                        int32_t n_heads, int32_t kv_heads, float* out, void* stream);

/* Raw scores <query, k_hat> per KV head: query [n_heads, rows, head_dim] (model basis),
 * scores_out [n_heads, rows, seq_len] fp32.  rows <= 16.  No mask, no softmax.
 * scale: multiplies the query in its own dtype first; NaN = no scaling. */
int sunshape_attention_scores(const sunshape_codec_t* codec, const sunshape_kv_t* kv,
                              const void* query, int32_t query_dtype,
                              int32_t n_heads, int32_t kv_heads, int32_t rows, float scale,
                              float* scores_out, void* stream);

/* Workspace bytes for sunshape_decode_attention on the current device.
 * The workspace must be zero-filled before its first use; every call leaves its
 * counters at zero again, so one workspace serves any number of calls issued in
 * stream order (calls that overlap on the GPU need separate workspaces). */
int64_t sunshape_decode_workspace_bytes(int32_t n_heads, int32_t seq_len, int32_t rows,
                                        int32_t value_dim, int32_t n_blocks);

/* Smallest workspace sunshape_decode_attention accepts for these sizes: the per-head LUTs are then
 * built inside each CTA's shared memory instead of by a separate LUT kernel into the workspace.
 * (sunshape_decode_workspace_bytes is the size that enables the LUT kernel; anything in between
 * behaves like the minimum.)  No counterpart in the reference (it allocates per call). */
int64_t sunshape_decode_workspace_min_bytes(int32_t n_heads, int32_t seq_len, int32_t rows,
                                            int32_t value_dim);

/* Fused quantized-key decode attention (LUT build + LUT-gather scores + online
 * softmax . V, split over the KV sequence inside the GPU).
 * query [batch, q_heads, query_len, head_dim]; the rows of KV head (b, h) are the
 * G*query_len query rows of its group (G = q_heads / kv_heads), row r = g*query_len + l.
 * mask: additive, element (b, hq, l, t) at mask + b*mask_sb + hq*mask_sh + l*mask_sq + t
 *       (strides in elements, 0 = broadcast), F32/BF16/F16, or NULL.
 * out: [batch, q_heads, query_len, value_dim] of out_dtype, or NULL.
 * partials: [batch*q_heads*query_len, 2 + value_dim] fp32 (m, l, acc[value_dim]) of the
 *       unnormalised softmax over this call's tokens, or NULL (for cross-GPU merges). */
int sunshape_decode_attention(const sunshape_codec_t* codec, const sunshape_kv_t* kv,
                              const void* query, int32_t query_dtype,
                              int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t query_len,
                              const void* mask, int32_t mask_dtype,
                              int64_t mask_sb, int64_t mask_sh, int64_t mask_sq,
                              float scale, void* out, int32_t out_dtype, float* partials,
                              void* workspace, int64_t workspace_bytes, void* stream);

/* ---- KV-sequence split across GPUs, exchange over peer memory (no reference counterpart: the
 * reference has no distributed code).  Each rank holds one exchange buffer, allocated with
 * sunshape_peer_alloc and mapped into every other rank's process with sunshape_peer_open (CUDA
 * IPC); sunshape_peer_buffer_bytes gives its size. */
typedef struct sunshape_peer_group {
  int32_t rank;
  int32_t world;          /* 2 .. 8 */
  void* buffers[8];       /* buffers[r] = rank r's exchange buffer as mapped in this process */
} sunshape_peer_group_t;

int64_t sunshape_peer_buffer_bytes(int32_t world, int64_t rows, int32_t value_dim, int32_t n_heads);
/* cudaMalloc + zero-fill a buffer on the current device; *ipc_handle receives 64 bytes (host). */
int sunshape_peer_alloc(int64_t bytes, void** dev_ptr, void* ipc_handle);
/* Map another process's buffer (from its 64-byte handle) into this process. */
int sunshape_peer_open(const void* ipc_handle, void** dev_ptr);
int sunshape_peer_close(void* dev_ptr);
int sunshape_peer_free(void* dev_ptr);

/* sunshape_decode_attention over this rank's KV shard (tokens [start_r, end_r) of every head),
 * producing the full output on every rank: the decode kernel stores each head's rank-local
 * (m, l, acc) rows into every rank's exchange buffer over NVLink and bumps that rank's per-head
 * arrival counter; a merge kernel waits (bounded) for all ranks' rows of each head and writes
 * out [batch, q_heads, query_len, value_dim].  All ranks must make the same sequence of calls.
 * Requires G * query_len <= 16 rows per KV head and 16-bit values.  Errors land in the workspace
 * error word: 104 = the merge gave up waiting for a peer (that call's rows are NaN); the timeout
 * also poisons this rank's exchange buffer, after which every call records 106 and writes NaN rows
 * until the buffers are freed and a new group is set up. */
int sunshape_decode_attention_peers(const sunshape_codec_t* codec, const sunshape_kv_t* kv,
                                    const void* query, int32_t query_dtype,
                                    int32_t batch, int32_t q_heads, int32_t kv_heads, int32_t query_len,
                                    const void* mask, int32_t mask_dtype,
                                    int64_t mask_sb, int64_t mask_sh, int64_t mask_sq,
                                    float scale, void* out, int32_t out_dtype,
                                    const sunshape_peer_group_t* group,
                                    void* workspace, int64_t workspace_bytes, void* stream);

/* ---- Bit-packed and wide codeword indices.
 * Packed format (the reference's packed-index kernel, triton_kernels.py:213-292, with uint8
 * elements): row t holds ceil(n_blocks * bits / 8) bytes; block b is in byte b / (8 / bits) at bit
 * offset (b % (8 / bits)) * bits.  sunshape_index_row_bytes gives the row size for index_bits 1, 2, 4
 * (packed), 8 (uint8), 16 (int16) or 32 (int32).
 * sunshape_pack_indices: uint8 indices [n_rows, n_blocks] -> packed rows (bits 1, 2 or 4).
 * sunshape_attention_scores_packed: scores [n_heads, rows, seq_len] fp32 of query [n_heads, rows,
 * head_dim] (model basis) against indices [n_heads, head_stride, row_bytes] of that format
 * (replaces _sunshape_packed_scores_kernel, triton_kernels.py:213-292, and serves the int16 indices
 * of codebooks above 256 codewords, codec.py:78-83).  rows <= 16; no heavy blocks. */
int64_t sunshape_index_row_bytes(int32_t index_bits, int32_t n_blocks);
int sunshape_pack_indices(const uint8_t* indices, int64_t n_rows, int32_t n_blocks, int32_t bits, uint8_t* packed,
                          void* stream);
int sunshape_attention_scores_packed(const sunshape_codec_t* codec, const void* indices, int32_t index_bits,
                                     int32_t seq_len, int64_t head_stride, const void* query, int32_t query_dtype,
                                     int32_t n_heads, int32_t kv_heads, int32_t rows, float* scores_out,
                                     void* stream);

/* ---- Cross-GPU merge of per-rank partials over NVLink peer memory (no reference counterpart).
 * Each rank allocates one buffer of sunshape_exchange_buffer_bytes(world, rows, value_dim) with
 * sunshape_peer_alloc and maps every other rank's with sunshape_peer_open.  sunshape_exchange_merge
 * takes this rank's partials [rows, 2 + value_dim] fp32 (as written by sunshape_decode_attention),
 * pushes them into every rank's buffer with 16-byte peer stores, waits (bounded, 2 s) for every
 * rank's rows and writes the merged output out [rows, value_dim] of out_dtype -- one kernel, no
 * library collective.  All ranks must make the same sequence of calls; the call count lives in the
 * buffers.  sunshape_exchange_error reads this rank's buffer error word (105 = a wait gave up; that
 * call's output rows are NaN). */
int64_t sunshape_exchange_buffer_bytes(int32_t world, int64_t rows, int32_t value_dim);
int sunshape_exchange_merge(const float* partials, int64_t rows, int32_t value_dim,
                            const sunshape_peer_group_t* group, void* out, int32_t out_dtype, void* stream);
int sunshape_exchange_error(const void* own_buffer, int32_t world, int64_t rows, int32_t value_dim,
                            int32_t* code);

/* Size of the scratch array built into the library for sunshape_decode_attention_noalloc. */
#define SUNSHAPE_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)

/* sunshape_decode_attention without a workspace and without any device allocation.
 * No counterpart in the reference: it exists for callers that cannot allocate device memory or
 * pass a workspace -- plugin hosts whose GPU memory belongs to another allocator, engines that
 * reserve all device memory up front and forbid allocation while decoding, and bindings with no
 * CUDA allocator of their own.  Arguments and results are those of sunshape_decode_attention;
 * the scratch is a fixed array of SUNSHAPE_NOALLOC_SCRATCH_BYTES compiled into the library (each
 * GPU that loads it keeps that much until the process exits).  Decodes whose minimum workspace
 * (sunshape_decode_workspace_min_bytes) exceeds it are rejected with SUNSHAPE_E_WORKSPACE; when
 * the array is also large enough for the per-head LUT area (sunshape_decode_workspace_bytes) the
 * decode uses it.  batch == 0 returns SUNSHAPE_OK without touching the device.
 * The first call on a device looks up the array's device address (with that device current), so
 * make that first call before any stream capture; the address is kept for the life of the process
 * (do not call again after a cudaDeviceReset).  Every call clears the parts of the array that
 * must start at zero, on the given stream; all calls share the one array, so calls that can
 * overlap on the GPU (different streams, or different host threads) race and must be serialised
 * by the caller. */
int sunshape_decode_attention_noalloc(const sunshape_codec_t* codec, const sunshape_kv_t* kv,
                                      const void* query, int32_t query_dtype,
                                      int32_t batch, int32_t q_heads, int32_t kv_heads,
                                      int32_t query_len, const void* mask, int32_t mask_dtype,
                                      int64_t mask_sb, int64_t mask_sh, int64_t mask_sq,
                                      float scale, void* out, int32_t out_dtype, float* partials,
                                      void* stream);

/* Device-side error code of the last sunshape_decode_attention_noalloc call on the current device
 * (0 = none; 101 / 102 = a bounded pipeline wait gave up and that call's output is invalid).  It
 * lives at the start of the built-in array and stays readable until the next call clears it.
 * Waits for the device's queued work (cudaMemcpyFromSymbol); allocates nothing. */
int sunshape_decode_attention_noalloc_error(int32_t* code);

/* Merge n_parts partial sets [n_parts, rows, 2 + value_dim] (as written by
 * sunshape_decode_attention) into out [rows, value_dim] of out_dtype:
 * M = max m_p, L = sum l_p e^(m_p - M), out = sum acc_p e^(m_p - M) / L. */
int sunshape_merge_partials(const float* partials, int32_t n_parts, int64_t rows, int32_t value_dim,
                            void* out, int32_t out_dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SUNSHAPE_B200_H */
