// Fused SunShape quantized-key decode attention for sm_100a.
//
// One persistent CTA per SM walks a contiguous range of 64-token tiles of the
// flattened (KV head, token) space, so the work is balanced to within one tile
// whatever the batch / head / context mix.  Per CTA:
//
//   * one producer warp streams each tile's uint8 index rows, SunShape-Mixed
//     heavy rows and value rows HBM -> shared memory with cp.async.bulk (the TMA
//     engine's 1-D mode) into a ring of stages guarded by mbarriers;
//   * 12 consumer warps build the per-query LUT  lut[b][c][g] = q_b . C_b[c]
//     (the reference's _precompute_query_centroid_dots, triton_kernels.py:381-408)
//     in shared memory whenever the tile range enters a new KV head, then score
//     each token as  sum_b lut[b][idx[t,b]][g]  (triton_kernels.py:134-204):
//     8 lanes per token, lane j owns blocks j, j+8, ... and the LUT is laid out
//     so those 8 lanes hit 8 distinct 16-byte bank groups (conflict-free 128-bit
//     gathers); block sums are combined with a warp-shuffle reduce-scatter that
//     leaves each lane holding the full score of its own query row;
//   * heavy (SunShape-Mixed) blocks are dotted densely against the permuted query;
//   * the scores feed an online softmax . V (vllm_attn_backend.py:241-252) with
//     fp32 accumulators (packed FFMA2), one running (max, sum, acc) per warp;
//   * at the end of each KV head segment the warps' partials are merged in shared
//     memory; if several CTAs share a head, each stores its partial in the
//     workspace and the last one to finish (atomic ticket) merges them
//     (log-sum-exp), so one launch produces the final output.
#pragma once

#include "common.cuh"

namespace sunshape {

constexpr int kWarps = 12;                       // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;      // + one producer warp
constexpr int kConsumerThreads = kWarps * 32;
constexpr int kTileTokens = 64;
constexpr int kWarpTokens = 16;
constexpr int kWarpsPerTile = kTileTokens / kWarpTokens;  // 4
constexpr int kTileGroups = kWarps / kWarpsPerTile;       // 3 tiles in flight across warps
constexpr int kMaxStages = 8;
constexpr int kBarConsumers = 1;                 // named barrier id for consumer-only sync
constexpr int kSmemLimit = 232448;               // 227 KiB opt-in per CTA on sm_100

// error codes written to the workspace error word
// Functions off the consumers' per-tile path (segment ends, LUT builds, the producer loop) stay out of
// line so the hot loop's code is small: instruction fetch is the decode kernel's top stall, and on B200
// outlining them took the c5 step at T 16384 from 74.6 to 70.3 us (full T: 383.4 to 381.0 us).
// SUNSHAPE_INLINE_COLD=1 builds inline them again.
#if defined(SUNSHAPE_INLINE_COLD) && SUNSHAPE_INLINE_COLD
#define SUNSHAPE_COLD __device__
#else
#define SUNSHAPE_COLD __device__ __noinline__
#endif
constexpr int kErrWaitFull = 101;
constexpr int kErrWaitEmpty = 102;

struct DecodeParams {
  // value tiles for the tensor-core kernel: 2-D map over [rows, value_dim], box 64 x 64, 128B swizzle
  CUtensorMap tmap_v;
  // query rows: row r of flat head hh lives at q + (hh * R + r) * D
  const void* q;
  int q_dtype;
  int R;        // rows per KV head (G * query_len)
  int r0;       // first row handled by this launch
  int Rc;       // rows handled by this launch (<= GP)
  int L;        // query_len
  int G;        // q_heads / kv_heads
  int q_heads;
  int kv_heads;
  // codec
  const float* cb;
  const float* cb_norm_max;   // [n_cb] or nullptr
  int n_cb;
  const int64_t* perm;
  const uint8_t* heavy_mask;
  int nb, bd, C, D;
  int nbh;      // ceil(nb / 8)
  // KV storage
  const uint8_t* idx;
  const void* heavy;
  int heavy_dtype;
  const void* v;
  int T;
  int64_t head_stride;
  int n_heads;
  // mask
  const void* mask;
  int mask_dtype;
  int64_t msb, msh, msq;
  // scaling
  float scale;
  int has_scale;
  // outputs
  void* out;
  int out_dtype;
  float* partials;
  float* scores_out;
  // workspace
  int lut_bytes;               // shared-memory LUT bytes of the tensor-core kernel
  int merge_smem_bytes;        // bytes of the LUT/staging region usable by finish_segment
  uint8_t* lut_global;         // per-head LUTs [n_heads][lut_bytes] built by lut_kernel, or null
  float* lut_scale_global;     // [n_heads] inverse LUT scale (fp16 LUT) or 1
  float* slots;
  int* counters;
  int* err;
  // cross-GPU exchange over peer memory (xworld > 0): the final per-head partial rows go to every
  // rank's receive buffer [2 parities][xworld][x_rows][DV + 2], then the rank's arrival counter
  // [2][n_heads] is bumped; the step counter's parity selects the buffer
  int xworld, xrank;
  int64_t x_rows;
  float* xrecv[8];
  unsigned int* xarrive[8];
  const unsigned int* xstep;
  unsigned long long* trace;  // per-CTA marks (trace builds only)
  // partition
  int tph;            // tiles per head
  int64_t total_tiles;
  int max_seg;
  int seg_gap;        // virtual tiles charged per head boundary by the partition
  // shared memory carve-up (bytes)
  int stages;
  int prefetch_ahead;   // tiles streamed into L2 beyond the ring (tensor-core kernel)
  int stage_bytes;
  int off_stage_idx;
  int off_stage_heavy;
  int off_perm, off_hslot, off_q, off_p, off_lut, off_stage;
};

// Partition of the flattened (head, tile) space over the persistent CTAs.  Finishing a head in the
// middle of a CTA's range costs that CTA time (merging the head's partials, loading the next head's
// LUT), so the split is made over a virtual sequence in which every head boundary counts as seg_gap
// extra tiles: CTAs whose range crosses a boundary get correspondingly fewer real tiles.  seg_gap = 0
// is the plain equal split.
__device__ __forceinline__ int64_t virtual_tiles(const DecodeParams& p) {
  return p.total_tiles + (p.total_tiles / p.tph - 1) * p.seg_gap;
}
// first real tile of CTA c (c = grid gives total_tiles)
__device__ __forceinline__ int64_t tile_start(const DecodeParams& p, int64_t c, int64_t grid) {
  const int64_t v = c * virtual_tiles(p) / grid;
  const int64_t span = p.tph + p.seg_gap;
  const int64_t h = v / span;
  return h * p.tph + min(v - h * span, (int64_t)p.tph);
}
// the CTA whose tile range contains real tile f
__device__ __forceinline__ int64_t tile_owner(const DecodeParams& p, int64_t f, int64_t grid) {
  const int64_t vf = f + (f / p.tph) * p.seg_gap;
  return ((vf + 1) * grid - 1) / virtual_tiles(p);
}

// rows held by lane j (0..7 within its token group) after the reduce-scatter
template <int GP>
struct RowMap {
  static constexpr int RPL = GP >= 8 ? GP / 8 : 1;
  __device__ __forceinline__ static int row(int j, int x) {
    if (GP == 4) return j >> 1;
    if (GP == 8) return j;
    return 2 * j + x;
  }
  // lane writes shared values for its row (GP==4 duplicates rows across lane pairs)
  __device__ __forceinline__ static bool owner(int j) { return GP == 4 ? ((j & 1) == 0) : true; }
};

// Reduce-scatter GP partial sums across the 8 lanes of a token group.
template <int GP>
__device__ __forceinline__ void reduce_scatter(const float (&part)[GP], float (&res)[RowMap<GP>::RPL], int j) {
  constexpr int H1 = GP / 2;
  float r1[H1];
  const bool hi = (j >> 2) & 1;
#pragma unroll
  for (int i = 0; i < H1; ++i) {
    const float send = hi ? part[i] : part[H1 + i];
    const float keep = hi ? part[H1 + i] : part[i];
    r1[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  constexpr int H2 = H1 / 2;
  float r2[H2];
  const bool mid = (j >> 1) & 1;
#pragma unroll
  for (int i = 0; i < H2; ++i) {
    const float send = mid ? r1[i] : r1[H2 + i];
    const float keep = mid ? r1[H2 + i] : r1[i];
    r2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  if constexpr (GP == 4) {
    res[0] = r2[0] + __shfl_xor_sync(0xffffffffu, r2[0], 1);
  } else {
    constexpr int H3 = H2 / 2;
    const bool lo = j & 1;
#pragma unroll
    for (int i = 0; i < H3; ++i) {
      const float send = lo ? r2[i] : r2[H3 + i];
      const float keep = lo ? r2[H3 + i] : r2[i];
      res[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
    }
  }
}

template <typename VT, int DPL>
__device__ __forceinline__ void load_value_row(const VT* src, float (&vf)[DPL]) {
  if constexpr (sizeof(VT) == 4) {
#pragma unroll
    for (int k = 0; k < DPL; k += 4) {
      const float4 x = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + k);
      vf[k] = x.x; vf[k + 1] = x.y; vf[k + 2] = x.z; vf[k + 3] = x.w;
    }
  } else if constexpr (std::is_same<VT, __nv_bfloat16>::value) {
    static_assert(DPL % 2 == 0, "DPL");
    const uint32_t* w = reinterpret_cast<const uint32_t*>(src);
    uint32_t u[DPL / 2];
    if constexpr (DPL == 2) {
      u[0] = w[0];
    } else if constexpr (DPL == 4) {
      const uint2 x = *reinterpret_cast<const uint2*>(w);
      u[0] = x.x; u[1] = x.y;
    } else {
#pragma unroll
      for (int k = 0; k < DPL / 2; k += 4) {
        const uint4 x = *reinterpret_cast<const uint4*>(w + k);
        u[k] = x.x; u[k + 1] = x.y; u[k + 2] = x.z; u[k + 3] = x.w;
      }
    }
#pragma unroll
    for (int k = 0; k < DPL / 2; ++k) {
      vf[2 * k] = __uint_as_float(u[k] << 16);
      vf[2 * k + 1] = __uint_as_float(u[k] & 0xffff0000u);
    }
  } else {
    const __half2* h = reinterpret_cast<const __half2*>(src);
#pragma unroll
    for (int k = 0; k < DPL / 2; ++k) {
      const float2 f = __half22float2(h[k]);
      vf[2 * k] = f.x; vf[2 * k + 1] = f.y;
    }
  }
}

// q_s[g][d'] = q[row g of head hh][perm[d']] (scaled in the query dtype), zero for absent rows.
// Loads are issued 8 per thread before any store so their latencies overlap.
template <int GP, int NTHREADS>
__device__ __forceinline__ void load_query_rows(const DecodeParams& p, int64_t hh, const int* perm_s, float* q_s,
                                                int ctid) {
  const int tot = GP * p.D;
  for (int b0 = ctid; b0 < tot; b0 += NTHREADS * 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int e = b0 + u * NTHREADS;
      const int g = e / p.D, dp = e - g * p.D;
      float x = 0.f;
      if (e < tot && g < p.Rc) {
        x = load_as_float(p.q, (hh * p.R + p.r0 + g) * p.D + perm_s[dp], p.q_dtype);
        if (p.has_scale) x = round_to_dtype(x * p.scale, p.q_dtype);
      }
      v[u] = x;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u)
      if (b0 + u * NTHREADS < tot) q_s[b0 + u * NTHREADS] = v[u];
  }
}

// Build the LUT (and the permuted, scaled query rows) for flat head hh.
template <int GP, int NTHREADS>
__device__ void build_lut_t(const DecodeParams& p, int64_t hh, const int* perm_s, const int8_t* hslot_s,
                            float* q_s, uint8_t* lut, int ctid) {
  constexpr int NH = GP / 4;
  named_barrier(kBarConsumers, NTHREADS);
  load_query_rows<GP, NTHREADS>(p, hh, perm_s, q_s, ctid);
  named_barrier(kBarConsumers, NTHREADS);
  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const float* cb = p.cb + (int64_t)cbh * p.nb * p.C * p.bd;
  const int total = p.nbh * 8 * p.C;
  for (int e = ctid; e < total; e += NTHREADS) {
    const int blo = e & 7, rest = e >> 3;
    const int k = rest / p.C, c = rest - k * p.C;
    const int b = blo + 8 * k;
    float vals[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) vals[g] = 0.f;
    if (b < p.nb && hslot_s[b] < 0) {
      const float* cr = cb + ((int64_t)b * p.C + c) * p.bd;
      const float* qb = q_s + b * p.bd;
      for (int d = 0; d < p.bd; ++d) {
        const float x = __ldg(cr + d);
#pragma unroll
        for (int g = 0; g < GP; ++g) vals[g] = fmaf(qb[g * p.D + d], x, vals[g]);
      }
    }
#pragma unroll
    for (int h = 0; h < NH; ++h) {
      float4* dst = reinterpret_cast<float4*>(lut + ((((int64_t)k * NH + h) * p.C + c) * 8 + blo) * 16);
      *dst = make_float4(vals[4 * h], vals[4 * h + 1], vals[4 * h + 2], vals[4 * h + 3]);
    }
  }
  named_barrier(kBarConsumers, NTHREADS);
}

// Producer warp: stream tiles [tb, te) into the stage ring.
template <typename VT, bool SCORES_ONLY, int DV>
__device__ void produce(const DecodeParams& p, int64_t tb, int64_t te, uint64_t* full, uint64_t* empty,
                        uint8_t* stage0, int n_heavy, int lane) {
  const int S = p.stages;
  const int64_t hrow = (int64_t)n_heavy * p.bd * (p.heavy_dtype == SUNSHAPE_F32 ? 4 : 2);
  for (int64_t i = 0; i < te - tb; ++i) {
    const int s = (int)(i % S);
    if (i >= S) mbar_wait(&empty[s], (uint32_t)(((i / S) - 1) & 1), p.err, kErrWaitEmpty);
    const int64_t f = tb + i;
    const int64_t hh = f / p.tph;
    const int t0 = (int)(f - hh * p.tph) * kTileTokens;
    const int ntok = min(kTileTokens, p.T - t0);
    const int64_t row0 = hh * p.head_stride + t0;
    uint8_t* st = stage0 + (int64_t)s * p.stage_bytes;

    // index rows: possibly unaligned -> 16B-aligned bulk body + byte tail
    const uint8_t* isrc = p.idx + row0 * p.nb;
    const int64_t ilen = (int64_t)ntok * p.nb;
    const uintptr_t ia0 = reinterpret_cast<uintptr_t>(isrc) & ~uintptr_t(15);
    const uintptr_t ia1 = (reinterpret_cast<uintptr_t>(isrc) + ilen) & ~uintptr_t(15);
    const uint32_t ibulk = ia1 > ia0 ? (uint32_t)(ia1 - ia0) : 0u;
    {
      const uintptr_t tail0 = max(ia1, reinterpret_cast<uintptr_t>(isrc));
      const int ntail = (int)(reinterpret_cast<uintptr_t>(isrc) + ilen - tail0);
      if (lane < ntail)
        st[p.off_stage_idx + (tail0 - ia0) + lane] = *reinterpret_cast<const uint8_t*>(tail0 + lane);
    }
    uint32_t hbulk = 0;
    uintptr_t ha0 = 0;
    if (n_heavy > 0) {
      const uint8_t* hsrc = reinterpret_cast<const uint8_t*>(p.heavy) + row0 * hrow;
      const int64_t hlen = (int64_t)ntok * hrow;
      ha0 = reinterpret_cast<uintptr_t>(hsrc) & ~uintptr_t(15);
      const uintptr_t ha1 = (reinterpret_cast<uintptr_t>(hsrc) + hlen) & ~uintptr_t(15);
      hbulk = ha1 > ha0 ? (uint32_t)(ha1 - ha0) : 0u;
      const uintptr_t tail0 = max(ha1, reinterpret_cast<uintptr_t>(hsrc));
      const int ntail = (int)(reinterpret_cast<uintptr_t>(hsrc) + hlen - tail0);
      if (lane < ntail)
        st[p.off_stage_heavy + (tail0 - ha0) + lane] = *reinterpret_cast<const uint8_t*>(tail0 + lane);
    }
    const uint32_t vbytes = SCORES_ONLY ? 0u : (uint32_t)ntok * DV * (uint32_t)sizeof(VT);
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(&full[s], vbytes + ibulk + hbulk);
      if (vbytes) bulk_g2s(st, reinterpret_cast<const VT*>(p.v) + row0 * DV, vbytes, &full[s]);
      if (ibulk) bulk_g2s(st + p.off_stage_idx, reinterpret_cast<const void*>(ia0), ibulk, &full[s]);
      if (hbulk) bulk_g2s(st + p.off_stage_heavy, reinterpret_cast<const void*>(ha0), hbulk, &full[s]);
    }
    __syncwarp();
  }
}

// End of a KV-head segment: `stg` holds NW per-warp partials [NW][GP][DV + 2] (m, l, acc).
// Merge them; if this CTA is the head's only contributor write the result, else store
// the CTA partial in the workspace slot and let the last contributor (atomic ticket)
// merge all slots of the head.
// Final (m, l, acc) of output row `orow` (column d): to the output / partial buffers, and in
// cross-GPU mode to every rank's receive buffer (NVLink peer stores).
template <int DV>
__device__ __forceinline__ void emit_row(const DecodeParams& p, int64_t orow, int d, float M, float Lsum, float A,
                                         unsigned parity) {
  const float NEG_INF = -__int_as_float(0x7f800000);
  if (p.out) store_from_float(p.out, orow * DV + d, p.out_dtype, M == NEG_INF ? __int_as_float(0x7fc00000) : A / Lsum);
  if (p.partials) {
    float* pr = p.partials + orow * (int64_t)(DV + 2);
    pr[2 + d] = A;
    if (d == 0) { pr[0] = M; pr[1] = Lsum; }
  }
  for (int r = 0; r < p.xworld; ++r) {
    float* dst = p.xrecv[r] + ((int64_t)(parity * p.xworld + p.xrank) * p.x_rows + orow) * (DV + 2);
    dst[2 + d] = A;
    if (d == 0) { dst[0] = M; dst[1] = Lsum; }
  }
}

// Four consecutive output columns d0..d0+3 of one merged row (d0 % 4 == 0): vector stores where the
// destination is aligned (bf16/f16 outputs 8 bytes, fp32 16 bytes, partial rows 8 bytes), else scalar.
template <int DV>
__device__ __forceinline__ void emit_row4(const DecodeParams& p, int64_t orow, int d0, float M, float Lsum,
                                          const float (&a)[4], unsigned parity) {
  const float NEG_INF = -__int_as_float(0x7f800000);
  if (p.out) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = M == NEG_INF ? __int_as_float(0x7fc00000) : a[j] / Lsum;
    const int64_t i0 = orow * DV + d0;
    const uintptr_t addr = reinterpret_cast<uintptr_t>(p.out);
    if (p.out_dtype == SUNSHAPE_F32 && (addr & 15) == 0) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + i0) = make_float4(v[0], v[1], v[2], v[3]);
    } else if (p.out_dtype == SUNSHAPE_BF16 && (addr & 7) == 0) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
      *reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(p.out) + i0) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    } else if (p.out_dtype == SUNSHAPE_F16 && (addr & 7) == 0) {
      const __half2 lo = __floats2half2_rn(v[0], v[1]), hi = __floats2half2_rn(v[2], v[3]);
      *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.out) + i0) =
          make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) store_from_float(p.out, i0 + j, p.out_dtype, v[j]);
    }
  }
  auto put_row = [&](float* pr) {   // [m, l, acc...] row of DV + 2 floats
    if ((reinterpret_cast<uintptr_t>(pr) & 7) == 0) {
      reinterpret_cast<float2*>(pr + 2 + d0)[0] = make_float2(a[0], a[1]);
      reinterpret_cast<float2*>(pr + 2 + d0)[1] = make_float2(a[2], a[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) pr[2 + d0 + j] = a[j];
    }
    if (d0 == 0) { pr[0] = M; pr[1] = Lsum; }
  };
  if (p.partials) put_row(p.partials + orow * (int64_t)(DV + 2));
  for (int r = 0; r < p.xworld; ++r)
    put_row(p.xrecv[r] + ((int64_t)(parity * p.xworld + p.xrank) * p.x_rows + orow) * (DV + 2));
}

__device__ __forceinline__ int ld_relaxed_gpu(const int* a) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(a));
  return v;
}

// After every thread emitted its rows of head hh: make the peer stores visible system-wide, then
// count this rank's arrival for hh on every rank.
__device__ __forceinline__ void signal_peers(const DecodeParams& p, int64_t hh, unsigned parity, int ctid, int nt) {
  if (p.xworld == 0) return;
  __threadfence_system();
  named_barrier(kBarConsumers, nt);
  if (ctid == 0)
    for (int r = 0; r < p.xworld; ++r) atomicAdd_system(p.xarrive[r] + (int64_t)parity * p.n_heads + hh, 1u);
}

#ifdef SUNSHAPE_TRACE
#define SUNSHAPE_FMARK(k) do { if (ctid == 0 && p.trace) p.trace[blockIdx.x * 32 + (k)] = global_ns(); } while (0)
#else
#define SUNSHAPE_FMARK(k) ((void)0)
#endif
// End of one (head, CTA) segment.  stg holds NW per-warp partial rows [m, l, acc[DV]] per query row.
// They are merged (log-sum-exp, fixed warp order) into this CTA's partial for head hh, which is
//   * emitted directly when this CTA holds the whole head (sole);
//   * otherwise combined with the other CTAs' partials of hh: the contributor that finds all others
//     already counted (ticket == contributors - 1, read before it writes anything, then a fence)
//     merges right away from shared memory and the others' slots; every other contributor writes
//     its slot, fences and takes a ticket, and the one that draws the last ticket merges.
// Shared memory after the staging rows: merge weights [NW][GP], row maxima [GP], row sums [GP], then the
// contributors' slot offsets and (when they fit) the gathered slots.  Sums run in the same order as a
// scalar merge (warps, then contributors in CTA order), so results do not depend on the vector width.
template <int GP, int DV, int NW, bool PRECISE = false>
SUNSHAPE_COLD void finish_segment(const DecodeParams& p, const float* stg, int64_t hh, int64_t tb, int64_t grid,
                               int ctid, int* flag_s) {
  constexpr int ROWF = DV + 2;
  constexpr int NT = NW * 32;
  constexpr int DV4 = DV / 4;
  static_assert(DV % 4 == 0, "value_dim");
  const float NEG_INF = -__int_as_float(0x7f800000);
  const int64_t c_first = tile_owner(p, hh * p.tph, grid);
  const int64_t c_last = tile_owner(p, (hh + 1) * p.tph - 1, grid);
  const bool sole = c_first == c_last;
  const int n_contrib = (int)(c_last - c_first + 1);
  const int seg_local = (int)(hh - tb / p.tph);
  float* slot = p.slots + ((int64_t)blockIdx.x * p.max_seg + seg_local) * GP * ROWF;
  const unsigned parity = p.xworld ? (*reinterpret_cast<const volatile unsigned int*>(p.xstep) & 1u) : 0u;
  float* const stgw = const_cast<float*>(stg);
  float* wgt = stgw + NW * GP * ROWF;   // [NW][GP]
  float* Ms = wgt + NW * GP;             // [GP]
  float* Ls = Ms + GP;                   // [GP]
  int64_t* offs = reinterpret_cast<int64_t*>(Ls + GP + 2);
  float* gath = reinterpret_cast<float*>(offs + n_contrib);
  const int slot_f = p.Rc * ROWF;
  const bool fits = (int64_t)(reinterpret_cast<uint8_t*>(gath + (int64_t)n_contrib * slot_f) -
                              reinterpret_cast<const uint8_t*>(stg)) <= p.merge_smem_bytes;
  const int k_self = (int)(blockIdx.x - c_first);

  // ---- per-row maxima and warp weights (one thread per row); the early ticket check of a split head
  // (issued first so its latency overlaps the weights; the fence below orders the slot reads after it)
  const int ticket_now = (ctid == 0 && !sole && fits) ? ld_relaxed_gpu(p.counters + hh) : -1;
  if (ctid < p.Rc) {
    const int r = ctid;
    float M = NEG_INF;
    for (int w = 0; w < NW; ++w) M = fmaxf(M, stg[(w * GP + r) * ROWF]);
    float L = 0.f;
    for (int w = 0; w < NW; ++w) {
      const float* src = stg + (w * GP + r) * ROWF;
      const float wt = M == NEG_INF ? 0.f : softmax_weight<PRECISE>(src[0] - M);
      wgt[w * GP + r] = wt;
      L = fmaf(src[1], wt, L);
    }
    Ms[r] = M;
    Ls[r] = L;
  }
  if (ctid == 0) {
    const bool last = ticket_now == n_contrib - 1;
    if (last) __threadfence();
    flag_s[3] = last ? 1 : 0;
  }
  named_barrier(kBarConsumers, NT);
  const bool last_now = flag_s[3] != 0;

  // ---- this CTA's partial: 4 columns per thread
  for (int e = ctid; e < p.Rc * DV4; e += NT) {
    const int r = e / DV4, d0 = (e - r * DV4) * 4;
    float a[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < NW; ++w) {
      const float wt = wgt[w * GP + r];
      const float2* src = reinterpret_cast<const float2*>(stg + (w * GP + r) * ROWF + 2 + d0);
      const float2 x0 = src[0], x1 = src[1];
      a[0] = fmaf(x0.x, wt, a[0]); a[1] = fmaf(x0.y, wt, a[1]);
      a[2] = fmaf(x1.x, wt, a[2]); a[3] = fmaf(x1.y, wt, a[3]);
    }
    const float M = Ms[r], L = Ls[r];
    if (sole) {
      emit_row4<DV>(p, hh * p.R + p.r0 + r, d0, M, L, a, parity);
    } else {
      float* dst = last_now ? gath + (int64_t)k_self * slot_f + r * ROWF : slot + r * ROWF;
      reinterpret_cast<float2*>(dst + 2 + d0)[0] = make_float2(a[0], a[1]);
      reinterpret_cast<float2*>(dst + 2 + d0)[1] = make_float2(a[2], a[3]);
      if (d0 == 0) { dst[0] = M; dst[1] = L; }
    }
  }
  SUNSHAPE_FMARK(8);
  if (sole) {
    signal_peers(p, hh, parity, ctid, NT);
    return;
  }
  if (!last_now) {
    __threadfence();
    SUNSHAPE_FMARK(9);
    named_barrier(kBarConsumers, NT);
    if (ctid == 0) {
      const int prev = atomicAdd(&p.counters[hh], 1);
      flag_s[0] = prev == n_contrib - 1;
    }
    named_barrier(kBarConsumers, NT);
    SUNSHAPE_FMARK(10);
    if (!flag_s[0]) return;
  }
  __threadfence();
  // float offsets of the contributing CTAs' slots for this head
  for (int k = ctid; k < n_contrib; k += NT) {
    const int64_t c = c_first + k;
    const int sl = (int)(hh - tile_start(p, c, grid) / p.tph);
    offs[k] = (c * p.max_seg + sl) * GP * ROWF;
  }
  named_barrier(kBarConsumers, NT);
  SUNSHAPE_FMARK(12);
  if (fits) {
    // gather the slots into shared memory in one batch of independent 8-byte loads (the slots were
    // written by other SMs and may sit in HBM), skipping this CTA's own partial when it is already there
    const int slot_h = slot_f / 2;
    const int tot = n_contrib * slot_h;
    for (int b0 = ctid; b0 < tot; b0 += NT * 8) {
      float2 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = b0 + u * NT;
        const int k = min(idx / slot_h, n_contrib - 1);
        v[u] = (idx < tot && !(last_now && k == k_self))
                   ? __ldcg(reinterpret_cast<const float2*>(p.slots + offs[k]) + (idx - k * slot_h))
                   : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int idx = b0 + u * NT;
        const int k = min(idx / slot_h, n_contrib - 1);
        if (idx < tot && !(last_now && k == k_self)) reinterpret_cast<float2*>(gath)[idx] = v[u];
      }
    }
    named_barrier(kBarConsumers, NT);
    SUNSHAPE_FMARK(22);
    // contributor weights per row (the staging rows are no longer needed: reuse them)
    float* w2 = stgw;                       // [n_contrib][GP]
    float* M2 = w2 + n_contrib * GP;        // [GP]
    float* L2 = M2 + GP;                    // [GP]
    if (ctid < p.Rc) {
      const int r = ctid;
      float M = NEG_INF;
      for (int k = 0; k < n_contrib; ++k) M = fmaxf(M, gath[k * slot_f + r * ROWF]);
      float L = 0.f;
      for (int k = 0; k < n_contrib; ++k) {
        const float* src = gath + k * slot_f + r * ROWF;
        const float wt = M == NEG_INF ? 0.f : softmax_weight<PRECISE>(src[0] - M);   // empty slot -> 0
        w2[k * GP + r] = wt;
        L = fmaf(src[1], wt, L);
      }
      M2[r] = M;
      L2[r] = L;
    }
    named_barrier(kBarConsumers, NT);
    for (int e = ctid; e < p.Rc * DV4; e += NT) {
      const int r = e / DV4, d0 = (e - r * DV4) * 4;
      float a[4] = {0.f, 0.f, 0.f, 0.f};
      for (int k = 0; k < n_contrib; ++k) {
        const float wt = w2[k * GP + r];
        const float2* src = reinterpret_cast<const float2*>(gath + k * slot_f + r * ROWF + 2 + d0);
        const float2 x0 = src[0], x1 = src[1];
        a[0] = fmaf(x0.x, wt, a[0]); a[1] = fmaf(x0.y, wt, a[1]);
        a[2] = fmaf(x1.x, wt, a[2]); a[3] = fmaf(x1.y, wt, a[3]);
      }
      emit_row4<DV>(p, hh * p.R + p.r0 + r, d0, M2[r], L2[r], a, parity);
    }
  } else {
    // many contributors (long sequences over few heads): reduce straight from the slots
    const float* base = p.slots;
#pragma unroll 1
    for (int e = ctid; e < p.Rc * DV; e += NT) {
      const int r = e / DV, d = e - r * DV;
      float M = NEG_INF;
      for (int k = 0; k < n_contrib; ++k) M = fmaxf(M, __ldcg(base + offs[k] + r * ROWF));
      float Lsum = 0.f, A = 0.f;
      if (M != NEG_INF) {
        for (int k = 0; k < n_contrib; ++k) {
          const float* src = base + offs[k] + r * ROWF;
          const float sc = softmax_weight<PRECISE>(__ldcg(src) - M);
          Lsum = fmaf(__ldcg(src + 1), sc, Lsum);
          A = fmaf(__ldcg(src + 2 + d), sc, A);
        }
      }
      emit_row<DV>(p, hh * p.R + p.r0 + r, d, M, Lsum, A, parity);
    }
  }
  signal_peers(p, hh, parity, ctid, NT);
  named_barrier(kBarConsumers, NT);
  SUNSHAPE_FMARK(13);
  if (ctid == 0) atomicExch(&p.counters[hh], 0);
  SUNSHAPE_FMARK(11);
}

template <int GP, int DV, typename VT, bool SCORES_ONLY>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RPL = RowMap<GP>::RPL;
  constexpr int NH = GP / 4;
  constexpr int DPL = DV / 32;
  static_assert(DPL % 2 == 0, "value row per lane must be even");

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  int* flag_s = reinterpret_cast<int*>(smem + 128);
  int* perm_s = reinterpret_cast<int*>(smem + p.off_perm);
  int8_t* hslot_s = reinterpret_cast<int8_t*>(smem + p.off_hslot);
  float* q_s = reinterpret_cast<float*>(smem + p.off_q);
  float* pbuf = reinterpret_cast<float*>(smem + p.off_p);
  uint8_t* lut = smem + p.off_lut;
  uint8_t* stage0 = smem + p.off_stage;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t grid = gridDim.x;
  const int64_t tb = tile_start(p, blockIdx.x, grid);
  const int64_t te = tile_start(p, blockIdx.x + 1, grid);

  if (tid == 0) {
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarpsPerTile);
    }
    fence_mbar_init();
    uint32_t bits = 0;
    int n = 0;
    for (int b = 0; b < p.nb; ++b) {
      const bool h = p.heavy_mask != nullptr && p.heavy_mask[b] != 0;
      hslot_s[b] = h ? (int8_t)n : (int8_t)-1;
      if (h) { bits |= 1u << b; ++n; }
    }
    flag_s[1] = (int)bits;
    flag_s[2] = n;
  }
  for (int i = tid; i < p.D; i += kThreads) perm_s[i] = (int)p.perm[i];
  __syncthreads();
  const uint32_t heavy_bits = (uint32_t)flag_s[1];
  const int n_heavy = flag_s[2];
  if (te <= tb) return;

  if (warp == kWarps) {
    produce<VT, SCORES_ONLY, DV>(p, tb, te, full, empty, stage0, n_heavy, lane);
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int ctid = tid;
  const int tg = warp / kWarpsPerTile, sub = warp % kWarpsPerTile;
  const int j = lane & 7, tsub = lane >> 3;
  float* pw = pbuf + warp * (kWarpTokens + 1) * GP;
  const int hsize = p.heavy_dtype == SUNSHAPE_F32 ? 4 : 2;
  const int64_t hrow = (int64_t)n_heavy * p.bd * hsize;
  const float NEG_INF = -__int_as_float(0x7f800000);

  int64_t f = tb;
  while (f < te) {
    const int64_t hh = f / p.tph;
    const int64_t fend = min(te, (hh + 1) * p.tph);
    const int i0 = (int)(f - tb), i1 = (int)(fend - tb);
    build_lut_t<GP, kConsumerThreads>(p, hh, perm_s, hslot_s, q_s, lut, ctid);

    float m_run[RPL], l_run[RPL];
    float2 acc[GP][DPL / 2];
#pragma unroll
    for (int x = 0; x < RPL; ++x) { m_run[x] = NEG_INF; l_run[x] = 0.f; }
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
      for (int k = 0; k < DPL / 2; ++k) acc[g][k] = make_float2(0.f, 0.f);

    const int64_t b_idx = hh / p.kv_heads;
    const int kvh = (int)(hh % p.kv_heads);

    for (int i = i0 + ((tg - i0 % kTileGroups) + kTileGroups) % kTileGroups; i < i1; i += kTileGroups) {
      const int s = i % p.stages;
      mbar_wait(&full[s], (uint32_t)((i / p.stages) & 1), p.err, kErrWaitFull);
      const int64_t ft = tb + i;
      const int t0 = (int)(ft - hh * p.tph) * kTileTokens;
      const int ntok = min(kTileTokens, p.T - t0);
      const int64_t row0 = hh * p.head_stride + t0;
      const uint8_t* st = stage0 + (int64_t)s * p.stage_bytes;
      const uint8_t* itile = st + p.off_stage_idx + (reinterpret_cast<uintptr_t>(p.idx + row0 * p.nb) & 15);
      const uint8_t* htile = st + p.off_stage_heavy;
      if (n_heavy > 0)
        htile += reinterpret_cast<uintptr_t>(reinterpret_cast<const uint8_t*>(p.heavy) + row0 * hrow) & 15;
      const VT* vtile = reinterpret_cast<const VT*>(st);
      const int my0 = sub * kWarpTokens;
      const int nmine = max(0, min(kWarpTokens, ntok - my0));

      if (nmine > 0) {
        float sc[4][RPL];
#pragma unroll
        for (int qd = 0; qd < 4; ++qd) {
          const int tl = qd * 4 + tsub;   // token within this warp's 16
          const bool valid = tl < nmine;
          const int t = my0 + tl;         // token within tile
          float part[GP];
#pragma unroll
          for (int g = 0; g < GP; ++g) part[g] = 0.f;
          if (valid) {
            const uint8_t* irow = itile + t * p.nb;
#pragma unroll 4
            for (int k = 0; k < 4; ++k) {
              if (k >= p.nbh) break;
              const int b = j + 8 * k;
              if (b >= p.nb) break;
              if ((heavy_bits >> b) & 1u) {
                const uint8_t* hv = htile + ((int64_t)t * n_heavy + hslot_s[b]) * p.bd * hsize;
                const float* qb = q_s + b * p.bd;
                for (int d = 0; d < p.bd; ++d) {
                  const float x = hsize == 4 ? reinterpret_cast<const float*>(hv)[d]
                                             : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(hv)[d]);
#pragma unroll
                  for (int g = 0; g < GP; ++g) part[g] = fmaf(qb[g * p.D + d], x, part[g]);
                }
              } else {
                const int c = irow[b];
                const float4* e = reinterpret_cast<const float4*>(lut + ((((int64_t)k * NH) * p.C + c) * 8 + j) * 16);
#pragma unroll
                for (int h = 0; h < NH; ++h) {
                  const float4 v = e[(int64_t)h * p.C * 8];
                  part[4 * h] += v.x; part[4 * h + 1] += v.y; part[4 * h + 2] += v.z; part[4 * h + 3] += v.w;
                }
              }
            }
          }
          float res[RPL];
          reduce_scatter<GP>(part, res, j);
#pragma unroll
          for (int x = 0; x < RPL; ++x) {
            const int g = RowMap<GP>::row(j, x);
            float sv = valid ? res[x] : NEG_INF;
            if (valid && p.mask != nullptr && g < p.Rc) {
              const int r = p.r0 + g;
              const int gq = r / p.L, ql = r - gq * p.L;
              const int64_t hq = (int64_t)kvh * p.G + gq;
              sv += load_as_float(p.mask, b_idx * p.msb + hq * p.msh + ql * p.msq + (t0 + t), p.mask_dtype);
            }
            sc[qd][x] = sv;
            if constexpr (SCORES_ONLY) {
              if (valid && g < p.Rc && RowMap<GP>::owner(j))
                p.scores_out[(hh * p.R + p.r0 + g) * (int64_t)p.T + t0 + t] = sv;
            }
          }
        }

        if constexpr (!SCORES_ONLY) {
          // ---- online softmax over this warp's 16 tokens
          float alpha_mine[RPL];
#pragma unroll
          for (int x = 0; x < RPL; ++x) {
            const int g = RowMap<GP>::row(j, x);
            float mx = fmaxf(fmaxf(sc[0][x], sc[1][x]), fmaxf(sc[2][x], sc[3][x]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(m_run[x], mx);
            float alpha = 1.f, pr[4];
            if (mnew == NEG_INF) {
              pr[0] = pr[1] = pr[2] = pr[3] = 0.f;
            } else {
              alpha = softmax_weight<sizeof(VT) == 4>(m_run[x] - mnew);
#pragma unroll
              for (int qd = 0; qd < 4; ++qd) pr[qd] = softmax_weight<sizeof(VT) == 4>(sc[qd][x] - mnew);
            }
            l_run[x] = l_run[x] * alpha + ((pr[0] + pr[1]) + (pr[2] + pr[3]));
            m_run[x] = mnew;
            alpha_mine[x] = alpha;
            if (RowMap<GP>::owner(j)) {
#pragma unroll
              for (int qd = 0; qd < 4; ++qd) pw[(qd * 4 + tsub) * GP + g] = pr[qd];
              if (tsub == 0) pw[kWarpTokens * GP + g] = alpha;
            }
          }
          __syncwarp();
          bool rescale = false;
#pragma unroll
          for (int x = 0; x < RPL; ++x) rescale |= alpha_mine[x] != 1.f;
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
            for (int g = 0; g < GP; ++g) {
              const float a = pw[kWarpTokens * GP + g];
#pragma unroll
              for (int k = 0; k < DPL / 2; ++k) { acc[g][k].x *= a; acc[g][k].y *= a; }
            }
          }
          // ---- P . V on this warp's tokens; lane owns value columns [lane*DPL, lane*DPL + DPL)
          const VT* vrow = vtile + (int64_t)my0 * DV + lane * DPL;
#pragma unroll 2
          for (int tt = 0; tt < nmine; ++tt) {
            float vf[DPL];
            load_value_row<VT, DPL>(vrow + (int64_t)tt * DV, vf);
            float pg[GP];
#pragma unroll
            for (int g4 = 0; g4 < GP; g4 += 4) {
              const float4 x = *reinterpret_cast<const float4*>(pw + tt * GP + g4);
              pg[g4] = x.x; pg[g4 + 1] = x.y; pg[g4 + 2] = x.z; pg[g4 + 3] = x.w;
            }
#pragma unroll
            for (int g = 0; g < GP; ++g) {
              const float2 pp = make_float2(pg[g], pg[g]);
#pragma unroll
              for (int k = 0; k < DPL / 2; ++k)
                acc[g][k] = __ffma2_rn(pp, make_float2(vf[2 * k], vf[2 * k + 1]), acc[g][k]);
            }
          }
          __syncwarp();
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }

    if constexpr (!SCORES_ONLY) {
      // ---------------- segment end: merge warps, then CTAs sharing this head
      float l_tot[RPL];
#pragma unroll
      for (int x = 0; x < RPL; ++x) {
        float l = l_run[x];
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_tot[x] = l;
      }
      named_barrier(kBarConsumers, kConsumerThreads);   // all LUT reads done: reuse it as staging
      constexpr int ROWF = DV + 2;
      float* stg = reinterpret_cast<float*>(lut);
      float* mine = stg + warp * GP * ROWF;
      if (tsub == 0 && RowMap<GP>::owner(j)) {
#pragma unroll
        for (int x = 0; x < RPL; ++x) {
          const int g = RowMap<GP>::row(j, x);
          mine[g * ROWF] = m_run[x];
          mine[g * ROWF + 1] = l_tot[x];
        }
      }
#pragma unroll
      for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int k = 0; k < DPL / 2; ++k)
          *reinterpret_cast<float2*>(mine + g * ROWF + 2 + lane * DPL + 2 * k) = acc[g][k];
      named_barrier(kBarConsumers, kConsumerThreads);

      finish_segment<GP, DV, kWarps, sizeof(VT) == 4>(p, stg, hh, tb, grid, ctid, flag_s);
    }
    f = fend;
  }
}

// Host-side launch description (filled by the C ABI, consumed by the launchers
// that are instantiated in the decode_*.cu translation units).
struct DecodeLaunch {
  DecodeParams prm;
  int smem;
  long long grid;
};

template <int GP, int DV, typename VT, bool SO>
void launch_decode_t(const DecodeLaunch& l, cudaStream_t st) {
  auto k = decode_kernel<GP, DV, VT, SO>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, l.smem);
  k<<<(unsigned)l.grid, kThreads, l.smem, st>>>(l.prm);
}


// Instantiated in decode_f32.cu / decode_bf16.cu / decode_f16.cu / decode_scores.cu.
extern template void launch_decode_t<4, 64, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 128, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 256, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 64, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 128, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 256, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 64, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 128, float, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 64, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 128, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 256, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 64, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 128, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 256, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 64, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 128, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<4, 64, float, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<8, 64, float, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_t<16, 64, float, true>(const DecodeLaunch&, cudaStream_t);

}  // namespace sunshape
