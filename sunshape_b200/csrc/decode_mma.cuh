// Fused SunShape decode attention for 16-bit values: LUT-gather scores on CUDA
// cores, softmax . V on the tensor cores.
//
// Same persistent split and segment protocol as decode_kernel (decode.cuh); the
// consumer work per token is reorganised:
//
//   * value tiles arrive by TMA tensor copies (cp.async.bulk.tensor, 64 tokens x
//     64 columns per box, 128-byte swizzle), index / heavy rows by 1-D bulk copies;
//     the producer also keeps a few tiles beyond the shared-memory ring streaming
//     into L2 (cp.async.bulk.prefetch) so HBM stays busy while consumers hold stages;
//   * one lane scores one token against all G query rows of its KV head.  At
//     step k of its block loop, lane l gathers block 8*kh + ((kl + l) & 7): the 8
//     lanes of every shared-memory phase read 8 different blocks, and the LUT keeps
//     block b's 16-byte entries in bank group b & 7, so the 128-bit gathers are
//     conflict-free and no cross-lane reduction is needed;
//   * online softmax with a lazy rescale: the running max only moves when a score
//     exceeds it by more than kLazyTau (rare after the first tile), so most tiles
//     need no shuffles and no accumulator rescale;
//   * P (bf16/f16, as the reference casts probabilities to the value dtype before
//     P @ V, vllm_attn_backend.py:251-252) goes to a token-major shared tile and
//     acc^T[dv][g] += V^T[dv][t] P^T[t][g] runs as m16n8k16 MMAs with fp32
//     accumulators, A fragments loaded straight from the swizzled value tile.
#pragma once

#include <algorithm>

#include "decode.cuh"

namespace sunshape {

constexpr int kWarpsM = 8;                       // consumer warps
constexpr int kProducersM = 2;                   // producer warps, interleaving tiles
constexpr int kThreadsM = (kWarpsM + kProducersM) * 32;
constexpr int kConsumerThreadsM = kWarpsM * 32;
constexpr int kWarpsPerTileM = kTileTokens / 32; // 2
constexpr int kTileGroupsM = kWarpsM / kWarpsPerTileM;
constexpr float kLazyTau = 8.0f;                 // p = exp(s - m) <= e^8 between rescales
constexpr int kVBoxBytes = 64 * 128;             // one TMA box: 64 tokens x 64 columns x 2 B
constexpr int kLutC = 256;                       // LUT rows per (block group, half): fixed 256-codeword stride
constexpr int kPrefetchAhead = 0;                // tiles prefetched into L2 beyond the ring (measured: off is fastest)

// Opt-in cycle accounting (built only with -DSUNSHAPE_TRACE): per-CTA counters summed into
// the 64-bit words at workspace offset 64: [0] producer total, [1] producer waiting on empty
// stages, [2] consumer total (sum over warps), [3] consumer waiting on full stages,
// [4] consumer LUT builds, [5] consumer segment ends, [6] producer issuing copies.
#ifdef SUNSHAPE_TRACE
// grid-wide spans of the side kernels: words 148*32 + k of the trace area; even k = earliest start
// (stored complemented so atomicMax keeps the minimum), odd k = latest end
#define SUNSHAPE_SPAN_START(k) do { if (threadIdx.x == 0 && p.trace) atomicMax(p.trace + 148 * 32 + (k), ~(unsigned long long)global_ns()); } while (0)
#define SUNSHAPE_SPAN_END(k) do { if (threadIdx.x == 0 && p.trace) atomicMax(p.trace + 148 * 32 + (k), (unsigned long long)global_ns()); } while (0)
#define SUNSHAPE_LUTMARK(k) do { if (threadIdx.x == 0 && p.trace) p.trace[148 * 32 + 64 + (blockIdx.y * gridDim.x + blockIdx.x) * 4 + (k)] = global_ns(); } while (0)
#define SUNSHAPE_TRACE_ADD(slot, v) atomicAdd(reinterpret_cast<unsigned long long*>(reinterpret_cast<uint8_t*>(p.err) + 64) + (slot), (unsigned long long)(v))
#define SUNSHAPE_CLK() clock64()
// per-CTA wall-clock marks (ns) in the trace area at the end of the workspace: [cta][0] start, [1] first tile landed,
// [2] last tile consumed, [3] consumers done, [4 + 2k] segment k LUT ready, [5 + 2k] segment k merged
#define SUNSHAPE_MARK(k) (p.trace[blockIdx.x * 32 + (k)] = global_ns())
#else
#define SUNSHAPE_MARK(k) ((void)0)
#define SUNSHAPE_SPAN_START(k) ((void)0)
#define SUNSHAPE_SPAN_END(k) ((void)0)
#define SUNSHAPE_LUTMARK(k) ((void)0)
#define SUNSHAPE_TRACE_ADD(slot, v) ((void)0)
#define SUNSHAPE_CLK() 0ll
#endif

// Unroll factor of the per-token block-group loop of the score.  1 (the default) keeps the consumers'
// hot loop small: ncu showed "no instruction" (instruction fetch) as the top stall of this kernel, and
// on B200 the rolled loop measured 384.9 against 387.8 us per c5 step, 74.9 against 77.0 us at T 16384,
// and raised c3 (32 blocks) from 0.76 to 0.79 and c4 from 0.90 to 0.93 of the HBM roofline.
#ifndef SUNSHAPE_KK_UNROLL
#define SUNSHAPE_KK_UNROLL 1
#endif
constexpr int kKkUnroll = SUNSHAPE_KK_UNROLL;

template <typename VT>
struct MmaOp;

template <>
struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void mma(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint16_t bits(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
};

template <>
struct MmaOp<__half> {
  __device__ __forceinline__ static void mma(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint16_t bits(float x) { return __half_as_ushort(__float2half_rn(x)); }
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

__device__ __forceinline__ float warp_max(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// P tile of one warp: 32 token rows x (8 * NT) query rows, 16-bit, token-major.  With two
// 16-byte chunks per row (NT == 2) the chunk index is XOR-swizzled with bit 2 of the row so
// the transposed ldmatrix reads of 8 consecutive rows hit 8 different bank groups.
template <int NT>
__device__ __forceinline__ uint32_t p_chunk_offset(int row, int chunk) {
  if constexpr (NT == 1) return (uint32_t)row * 16u;
  else return (uint32_t)row * 32u + (uint32_t)((chunk ^ ((row >> 2) & 1)) << 4);
}

// LUT rows of one block for this thread: q block held in registers, codebook rows loaded
// eight at a time so their L2 latencies overlap; stores land in bank group b & 7.
// Store one LUT entry (GP query rows of block b, codeword c): fp32 in GP/4 16-byte chunks,
// or (L16) fp16 scaled by `scale` in GP/8 16-byte chunks -- for GP == 4 an 8-byte half of a
// 16-byte slot shared by block groups kh = 2j and 2j + 1 (dst_base already points at the half).
template <int GP, bool L16>
__device__ __forceinline__ void store_lut_entry(uint8_t* dst_base, int c, const float (&v)[GP], float scale) {
  if constexpr (L16 && GP == 4) {
    const uint32_t w0 = (uint32_t)__half_as_ushort(__float2half_rn(v[0] * scale)) |
                        ((uint32_t)__half_as_ushort(__float2half_rn(v[1] * scale)) << 16);
    const uint32_t w1 = (uint32_t)__half_as_ushort(__float2half_rn(v[2] * scale)) |
                        ((uint32_t)__half_as_ushort(__float2half_rn(v[3] * scale)) << 16);
    *reinterpret_cast<uint2*>(dst_base + (int64_t)c * 128) = make_uint2(w0, w1);
  } else if constexpr (L16) {
#pragma unroll
    for (int h = 0; h < GP / 8; ++h) {
      uint32_t w[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        w[k] = (uint32_t)__half_as_ushort(__float2half_rn(v[8 * h + 2 * k] * scale)) |
               ((uint32_t)__half_as_ushort(__float2half_rn(v[8 * h + 2 * k + 1] * scale)) << 16);
      *reinterpret_cast<uint4*>(dst_base + ((int64_t)h * kLutC + c) * 128) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  } else {
#pragma unroll
    for (int h = 0; h < GP / 4; ++h)
      *reinterpret_cast<float4*>(dst_base + ((int64_t)h * kLutC + c) * 128) =
          make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
  }
}

template <int GP, int BD, bool L16>
__device__ __forceinline__ void lut_rows_reg(const DecodeParams& p, const float* qblk, const float* cbb, bool active,
                                             uint8_t* dst_base, int c0, float scale, int c_hi) {
  float q[GP][BD];
#pragma unroll
  for (int g = 0; g < GP; ++g)
#pragma unroll
    for (int d = 0; d < BD; ++d) q[g][d] = active ? qblk[g * p.D + d] : 0.f;
  constexpr int U = 8;   // codeword rows in flight per thread
  for (int cb4 = c0; cb4 < c_hi; cb4 += 32 * U) {
    float x[U][BD];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = cb4 + 32 * u;
      const bool ok = active && c < c_hi;
#pragma unroll
      for (int d4 = 0; d4 < BD; d4 += 4) {   // codebook rows are 16-byte aligned (BD = 4 or 8)
        const float4 v = ok ? __ldg(reinterpret_cast<const float4*>(cbb + (int64_t)c * BD + d4))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
        x[u][d4] = v.x; x[u][d4 + 1] = v.y; x[u][d4 + 2] = v.z; x[u][d4 + 3] = v.w;
      }
    }
#pragma unroll 1   // cold code (runs once per LUT): keep it small for the instruction cache
    for (int u = 0; u < U; ++u) {
      const int c = cb4 + 32 * u;
      if (c >= c_hi) break;
      float v[GP];
#pragma unroll
      for (int g = 0; g < GP; ++g) {
        float a = 0.f;
#pragma unroll
        for (int d = 0; d < BD; ++d) a = fmaf(q[g][d], x[u][d], a);
        v[g] = a;
      }
      store_lut_entry<GP, L16>(dst_base, c, v, scale);
    }
  }
}

// LUT of flat head hh for the tensor-core kernel: 16-byte entry (b, h, c) at
// ((kh * NH + h) * 256 + c) * 128 + (b & 7) * 16 with kh = b / 8, holding q rows 4h..4h+3.
// Heavy and padding blocks get zero rows (their stored index is 0).
// With L16 the entries are stored as fp16 times a power-of-two scale chosen from the bound
// |q_b . c| <= max_b |q_b| * max_{b,c} |c|, so no entry can overflow; the score is the fp32 sum
// of the entries times 1 / scale (exact).  The scale is left in *scale_s.
template <int GP, bool L16>
SUNSHAPE_COLD void build_lut_m(const DecodeParams& p, int64_t hh, const int* perm_s, const int8_t* hslot_s,
                            float* q_s, uint8_t* lut, int ctid, float* scale_s, int kh_lo = 0, int kh_hi = 1 << 20,
                            int c_lo = 0, int c_hi = 1 << 20) {
  c_hi = min(c_hi, p.C);
  kh_hi = min(kh_hi, p.nbh);
  constexpr int NH = L16 ? (GP >= 8 ? GP / 8 : 1) : GP / 4;
  named_barrier(kBarConsumers, kConsumerThreadsM);
  if (L16 && ctid == 0) { scale_s[1] = 0.f; scale_s[2] = 0.f; }
  load_query_rows<GP, kConsumerThreadsM>(p, hh, perm_s, q_s, ctid);
  named_barrier(kBarConsumers, kConsumerThreadsM);
  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const float* cb = p.cb + (int64_t)cbh * p.nb * p.C * p.bd;
  const int blo = ctid & 7, c0 = ctid >> 3;   // 8 bank groups x 32 codeword lanes
#ifdef SUNSHAPE_TRACE
  if (ctid == 0 && p.trace) p.trace[blockIdx.x * 32 + 19] = global_ns();
#endif
  float scale = 1.f;
  if constexpr (L16) {
    float qn = 0.f, cn = 0.f;
    for (int e = ctid; e < GP * p.nb; e += kConsumerThreadsM) {
      const int g = e / p.nb, b = e - g * p.nb;
      float a = 0.f;
      for (int d = 0; d < p.bd; ++d) a = fmaf(q_s[g * p.D + b * p.bd + d], q_s[g * p.D + b * p.bd + d], a);
      qn = fmaxf(qn, a);
    }
    if (p.cb_norm_max != nullptr) {
      const float m = __ldg(p.cb_norm_max + cbh);
      cn = m * m;
    } else {
      for (int e = ctid; e < p.nb * p.C; e += kConsumerThreadsM) {
        const int b = e / p.C;
        if (hslot_s[b] >= 0) continue;
        const float* r = cb + (int64_t)e * p.bd;
        float a = 0.f;
        for (int d = 0; d < p.bd; ++d) a = fmaf(__ldg(r + d), __ldg(r + d), a);
        cn = fmaxf(cn, a);
      }
    }
    qn = warp_max(qn);
    cn = warp_max(cn);
    if ((ctid & 31) == 0) {
      atomicMax(reinterpret_cast<int*>(scale_s + 1), __float_as_int(qn));
      atomicMax(reinterpret_cast<int*>(scale_s + 2), __float_as_int(cn));
    }
    named_barrier(kBarConsumers, kConsumerThreadsM);
    const float bound = sqrtf(scale_s[1]) * sqrtf(scale_s[2]) * 1.001f;
    scale = bound > 0.f ? exp2f(fminf(100.f, floorf(log2f(32768.f / bound)))) : 1.f;
    if (ctid == 0) scale_s[0] = 1.f / scale;
  }
#ifdef SUNSHAPE_TRACE
  if (ctid == 0 && p.trace) p.trace[blockIdx.x * 32 + 20] = global_ns();
#endif
  for (int kh = kh_lo; kh < kh_hi; ++kh) {
    const int b = blo + 8 * kh;
    const bool active = b < p.nb && hslot_s[b] < 0;
    const float* qblk = q_s + (active ? b : 0) * p.bd;
    const float* cbb = cb + (int64_t)(active ? b : 0) * p.C * p.bd;
    uint8_t* dst = (L16 && GP == 4) ? lut + (int64_t)(kh >> 1) * kLutC * 128 + blo * 16 + (kh & 1) * 8
                                    : lut + (int64_t)kh * NH * kLutC * 128 + blo * 16;
    if (p.bd == 8) {
      lut_rows_reg<GP, 8, L16>(p, qblk, cbb, active, dst, c_lo + c0, scale, c_hi);
    } else if (p.bd == 4) {
      lut_rows_reg<GP, 4, L16>(p, qblk, cbb, active, dst, c_lo + c0, scale, c_hi);
    } else {
      for (int c = c_lo + c0; c < c_hi; c += 32) {
        float v[GP];
#pragma unroll
        for (int g = 0; g < GP; ++g) v[g] = 0.f;
        if (active)
          for (int d = 0; d < p.bd; ++d) {
            const float x = __ldg(cbb + (int64_t)c * p.bd + d);
#pragma unroll
            for (int g = 0; g < GP; ++g) v[g] = fmaf(qblk[g * p.D + d], x, v[g]);
          }
        store_lut_entry<GP, L16>(dst, c, v, scale);
      }
    }
  }
  named_barrier(kBarConsumers, kConsumerThreadsM);
}

// Per-head LUTs for one decode launch, in exactly the shared-memory layout the decode kernel
// uses, written to the workspace.  Organised codebook-major: one CTA per (KV head h, block b, group
// of hpc sequences) holds codebook block b of h's codebook (thread = codeword, its row in registers)
// and the query rows of every head (s, h) of the group, and writes the 16-byte LUT entries of all
// those heads.  A launch is kv_heads x 8*nbh x ceil(batch / hpc) CTAs -- a few hundred -- instead of
// one CTA per (head, block).  The grid runs while the decode kernel's producers saturate HBM, when
// every dependent memory round trip costs microseconds, so all global loads (permutation, codebook
// row, query rows) are issued together in one round; the ProfilePerm gather happens in shared
// memory.  The decode kernel is launched as a programmatic dependent of this grid: its producer
// warps start streaming values right away and only its consumers wait (griddepcontrol.wait) before
// copying their first LUT.
// Sequences per LUT CTA: enough CTAs to fill the GPU about once (8 per SM), at most 64 and at most
// 32 KB of query rows in shared memory.
inline int lut_heads_per_cta(int gp, int D, int items, int batch, int n_sms) {
  const int cap = std::max(1, std::min(64, 8192 / (gp * D)));
  const int want = (int)(((int64_t)items * batch) / ((int64_t)n_sms * 8));
  return std::max(1, std::min(cap, want));
}

template <int GP, bool L16>
__global__ void __launch_bounds__(256) lut_cbm_kernel(const __grid_constant__ DecodeParams p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  SUNSHAPE_SPAN_START(0);
  SUNSHAPE_LUTMARK(0);
  extern __shared__ float lut_q_s[];                    // [hpc][GP][D] query rows, scaled, unpermuted
  __shared__ int perm_s[256];
  __shared__ float scale_s[64];
  __shared__ unsigned qn_s[64];
  __shared__ float cn_s;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int D = p.D, bd = p.bd;
  const int batch = p.n_heads / p.kv_heads;
  const int hpc = (batch + gridDim.y - 1) / gridDim.y;   // sequences per CTA, set by the launch
  const int kvh = blockIdx.x / (p.nbh * 8);
  const int b = blockIdx.x - kvh * (p.nbh * 8);    // block (padding blocks >= nb get zero entries)
  const int s0 = blockIdx.y * hpc;
  const int nh = min(hpc, batch - s0);
  const bool active = b < p.nb && (p.heavy_mask == nullptr || p.heavy_mask[b] == 0);
  const int cbh = p.n_cb == 1 ? 0 : kvh % p.n_cb;
  // ---- one round of independent global loads: permutation, this thread's codeword row, query rows
  for (int i = tid; i < D; i += 256) perm_s[i] = (int)__ldg(p.perm + i);
  if (tid < 64) qn_s[tid] = 0u;
  float cw[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) cw[d] = 0.f;
  const int c = tid;
  if (active && c < p.C) {
    const float* cr = p.cb + (((int64_t)cbh * p.nb + b) * p.C + c) * bd;
    if (bd == 8) {
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(cr)), v1 = __ldg(reinterpret_cast<const float4*>(cr) + 1);
      cw[0] = v0.x; cw[1] = v0.y; cw[2] = v0.z; cw[3] = v0.w; cw[4] = v1.x; cw[5] = v1.y; cw[6] = v1.z; cw[7] = v1.w;
    } else if (bd == 4) {
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(cr));
      cw[0] = v0.x; cw[1] = v0.y; cw[2] = v0.z; cw[3] = v0.w;
    } else {
      for (int d = 0; d < bd; ++d) cw[d] = __ldg(cr + d);
    }
  }
  {
    // query rows of the group: 16-byte vector loads, all issued before the first use (one round trip)
    const int rowv = D / 8;                        // 8-element chunks per row
    const int totv = hpc * GP * rowv;
    const int es = p.q_dtype == SUNSHAPE_F32 ? 4 : 2;
    constexpr int kMaxV = 8;                       // chunks per thread: hpc * GP * D <= 8192 elements
    uint4 raw[kMaxV][2];
#pragma unroll
    for (int u = 0; u < kMaxV; ++u) {
      const int e = tid + u * 256;
      const int j = e / (GP * rowv), r = e - j * GP * rowv, g = r / rowv, ch = r - g * rowv;
      raw[u][0] = raw[u][1] = make_uint4(0u, 0u, 0u, 0u);
      if (e < totv && j < nh && g < p.Rc) {
        const int64_t hh = (int64_t)(s0 + j) * p.kv_heads + kvh;
        const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(p.q) +
                                                          ((hh * p.R + p.r0 + g) * D + ch * 8) * es);
        raw[u][0] = __ldg(src);
        if (es == 4) raw[u][1] = __ldg(src + 1);
      }
    }
#pragma unroll
    for (int u = 0; u < kMaxV; ++u) {
      const int e = tid + u * 256;
      if (e >= totv) break;
      float x[8];
      if (es == 4) {
        const uint32_t w[8] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w,
                               raw[u][1].x, raw[u][1].y, raw[u][1].z, raw[u][1].w};
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = __uint_as_float(w[i]);
      } else {
        const uint32_t w[4] = {raw[u][0].x, raw[u][0].y, raw[u][0].z, raw[u][0].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (p.q_dtype == SUNSHAPE_BF16) {
            x[2 * i] = __uint_as_float(w[i] << 16);
            x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
          } else {
            x[2 * i] = __half2float(__ushort_as_half((unsigned short)(w[i] & 0xffffu)));
            x[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(w[i] >> 16)));
          }
        }
      }
      if (p.has_scale) {
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = round_to_dtype(x[i] * p.scale, p.q_dtype);
      }
      float4* dst = reinterpret_cast<float4*>(lut_q_s + (int64_t)e * 8);
      dst[0] = make_float4(x[0], x[1], x[2], x[3]);
      dst[1] = make_float4(x[4], x[5], x[6], x[7]);
    }
  }
  if (L16 && p.cb_norm_max == nullptr) {   // fallback bound (C ABI callers without norms): bd * max c_i^2
    float cn = 0.f;
    const float* cbf = p.cb + (int64_t)cbh * p.nb * p.C * bd;
    for (int e = tid; e < p.nb * p.C * bd; e += 256) cn = fmaxf(cn, cbf[e] * cbf[e] * bd);
    cn = warp_max(cn);
    if (tid == 0) cn_s = 0.f;
    __syncthreads();
    if (lane == 0) atomicMax(reinterpret_cast<int*>(&cn_s), __float_as_int(cn));
  }
  __syncthreads();
  SUNSHAPE_LUTMARK(1);
  if constexpr (L16) {
    // fp16 entries are scaled by a power of two from the bound |q_b . c| <= max_b |q_b| * max |c|
    // (max over the head's rows and blocks), so no entry can overflow: one thread per (head, row, block)
    for (int e = tid; e < nh * GP * p.nb; e += 256) {
      const int j = e / (GP * p.nb), r = e - j * GP * p.nb, g = r / p.nb, bb = r - g * p.nb;
      const float* qr = lut_q_s + ((int64_t)j * GP + g) * D;
      float a = 0.f;
      for (int d = 0; d < bd; ++d) {
        const float x = qr[perm_s[bb * bd + d]];
        a = fmaf(x, x, a);
      }
      atomicMax(&qn_s[j], __float_as_uint(a));   // non-negative floats order like their bits
    }
    __syncthreads();
    if (tid < nh) {
      const int j = tid;
      float cn;
      if (p.cb_norm_max != nullptr) {
        const float m = __ldg(p.cb_norm_max + cbh);
        cn = m * m;
      } else {
        cn = cn_s;
      }
      const float bound = sqrtf(__uint_as_float(qn_s[j])) * sqrtf(cn) * 1.001f;
      const float scale = bound > 0.f ? exp2f(fminf(100.f, floorf(log2f(32768.f / bound)))) : 1.f;
      scale_s[j] = scale;
      if (b == 0) p.lut_scale_global[(int64_t)(s0 + j) * p.kv_heads + kvh] = 1.f / scale;
    }
    __syncthreads();
  } else {
    if (b == 0 && tid < nh) p.lut_scale_global[(int64_t)(s0 + tid) * p.kv_heads + kvh] = 1.f;
  }
  SUNSHAPE_LUTMARK(2);
  if (c >= p.C) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  const int kh = b >> 3, blo = b & 7;
  constexpr int NH = L16 ? (GP >= 8 ? GP / 8 : 1) : GP / 4;
  int pb[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) pb[d] = (active && d < bd) ? perm_s[b * bd + d] : 0;
  for (int j = 0; j < nh; ++j) {
    float v[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) {
      const float* qr = lut_q_s + ((int64_t)j * GP + g) * D;
      float a = 0.f;
      if (bd == 8) {
#pragma unroll
        for (int d = 0; d < 8; ++d) a = fmaf(qr[pb[d]], cw[d], a);
      } else if (bd == 4) {
#pragma unroll
        for (int d = 0; d < 4; ++d) a = fmaf(qr[pb[d]], cw[d], a);
      } else {
#pragma unroll
        for (int d = 0; d < 16; ++d)
          if (d < bd) a = fmaf(qr[pb[d]], cw[d], a);
      }
      v[g] = a;
    }
    const int64_t hh = (int64_t)(s0 + j) * p.kv_heads + kvh;
    uint8_t* base = p.lut_global + hh * (int64_t)p.lut_bytes;
    uint8_t* dst = (L16 && GP == 4) ? base + (int64_t)(kh >> 1) * kLutC * 128 + blo * 16 + (kh & 1) * 8
                                    : base + (int64_t)kh * NH * kLutC * 128 + blo * 16;
    store_lut_entry<GP, L16>(dst, c, v, L16 ? scale_s[j] : 1.f);
  }
  SUNSHAPE_SPAN_END(1);
  SUNSHAPE_LUTMARK(3);
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Launch of a LUT grid as a programmatic dependent of the preceding kernel in the stream.  When that is
// the previous step's decode_mma_kernel, its CTAs trigger (griddepcontrol.launch_dependents) once their
// last global-LUT copy has landed, so this grid can overwrite the LUT tables on SMs the decode has
// already released while its tail merges run.  The LUT kernels end with griddepcontrol.wait: they
// complete only after the preceding grid, which keeps the next decode's consumers (who wait for this
// grid) off the workspace and the outputs that the previous decode is still finishing.
template <typename... Args>
void launch_pdl(void (*kernel)(Args...), dim3 grid, int threads, size_t smem, cudaStream_t st,
                const DecodeParams& prm) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, prm);
}

template <int GP, bool L16>
void launch_lut_head_block_t(const DecodeParams& prm, int n_heads, cudaStream_t st);
// LUT build strategy: one CTA per (head, block) while that grid fits the GPU in a few waves; beyond
// that (many heads) the codebook-major grid, which loads each codebook block once per group of
// sequences.  (Measured on B200: head/block is faster at 64-128 heads x 16 blocks, codebook-major
// at 512 heads x 16 blocks.)
template <int GP, bool L16>
void launch_lut_t(const DecodeParams& prm, int n_heads, int n_sms, cudaStream_t st) {
  if ((int64_t)n_heads * prm.nbh * 8 <= (int64_t)n_sms * 32) {
    launch_lut_head_block_t<GP, L16>(prm, n_heads, st);
    return;
  }
  const int batch = n_heads / prm.kv_heads;
  const int items = prm.kv_heads * prm.nbh * 8;
  const int hpc = lut_heads_per_cta(GP, prm.D, items, batch, n_sms);
  const int groups = (batch + hpc - 1) / hpc;
  const int hpc_eff = (batch + groups - 1) / groups;   // what the kernel derives from gridDim.y
  const size_t smem = (size_t)hpc_eff * GP * prm.D * sizeof(float);
  launch_pdl(lut_cbm_kernel<GP, L16>, dim3(items, groups), 256, smem, st, prm);
}

// Per-head LUTs for one decode launch, in exactly the shared-memory layout the decode kernel
// uses, written to the workspace: one CTA per (KV head, block), one thread per codeword, so the
// whole GPU builds all LUTs in a couple of memory round trips.  The decode kernel is launched as
// a programmatic dependent of this grid: its producer warps start streaming values right away and
// only its consumers wait (griddepcontrol.wait) before copying their first LUT.
template <int GP, bool L16>
__global__ void __launch_bounds__(256) lut_kernel(const __grid_constant__ DecodeParams p) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  SUNSHAPE_SPAN_START(0);
  SUNSHAPE_LUTMARK(0);
  __shared__ float q_s[GP * 256];   // this head's query rows, scaled, in model channel order
  __shared__ int perm_s[256];
  __shared__ float red[2];
  const int tid = threadIdx.x;
  const int64_t hh = blockIdx.x;
  const int b = blockIdx.y;                       // block (0 .. 8 * nbh - 1; padding blocks get zeros)
  const int D = p.D, bd = p.bd;
  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const int c = tid;
  // ---- one round of independent global loads (each dependent round trip costs ~1 us on a loaded GPU):
  // this thread's codebook row, the norm bound, the heavy flag, the permutation and the raw query rows;
  // the ProfilePerm gather then happens in shared memory
  float cw[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) cw[d] = 0.f;
  const bool in_cb = b < p.nb && c < p.C;
  if (in_cb) {
    const float* cr = p.cb + (((int64_t)cbh * p.nb + b) * p.C + c) * bd;
    if (bd == 8) {
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(cr)), v1 = __ldg(reinterpret_cast<const float4*>(cr) + 1);
      cw[0] = v0.x; cw[1] = v0.y; cw[2] = v0.z; cw[3] = v0.w; cw[4] = v1.x; cw[5] = v1.y; cw[6] = v1.z; cw[7] = v1.w;
    } else if (bd == 4) {
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(cr));
      cw[0] = v0.x; cw[1] = v0.y; cw[2] = v0.z; cw[3] = v0.w;
    } else if (bd == 2) {
      const float2 v0 = __ldg(reinterpret_cast<const float2*>(cr));
      cw[0] = v0.x; cw[1] = v0.y;
    } else {
#pragma unroll
      for (int d = 0; d < 16; ++d)
        if (d < bd) cw[d] = __ldg(cr + d);
    }
  }
  const float cnm = (L16 && p.cb_norm_max != nullptr) ? __ldg(p.cb_norm_max + cbh) : 0.f;
  const bool heavy = b < p.nb && p.heavy_mask != nullptr && p.heavy_mask[b] != 0;
  const int pv = tid < D ? (int)__ldg(p.perm + tid) : 0;
  float qv[GP];
#pragma unroll
  for (int u = 0; u < GP; ++u) {   // GP * D <= GP * 256 elements, GP per thread
    const int e = tid + u * 256;
    const int g = e / D, ch = e - g * D;
    qv[u] = (e < GP * D && g < p.Rc) ? load_as_float(p.q, (hh * p.R + p.r0 + g) * D + ch, p.q_dtype) : 0.f;
  }
#pragma unroll
  for (int u = 0; u < GP; ++u) {
    const int e = tid + u * 256;
    if (e < GP * D) q_s[e] = p.has_scale ? round_to_dtype(qv[u] * p.scale, p.q_dtype) : qv[u];
  }
  if (tid < D) perm_s[tid] = pv;
  if (tid == 0) { red[0] = 0.f; red[1] = 1.f; }
  __syncthreads();
  SUNSHAPE_LUTMARK(1);
  float scale = 1.f;
  if constexpr (L16) {
    float qn = 0.f;
    for (int e = tid; e < GP * p.nb; e += 256) {
      const int g = e / p.nb, bb = e - g * p.nb;
      float a = 0.f;
      for (int d = 0; d < bd; ++d) {
        const float x = q_s[g * D + perm_s[bb * bd + d]];
        a = fmaf(x, x, a);
      }
      qn = fmaxf(qn, a);
    }
    qn = warp_max(qn);
    if ((tid & 31) == 0) atomicMax(reinterpret_cast<int*>(&red[0]), __float_as_int(qn));
    __syncthreads();
    float cn;
    if (p.cb_norm_max != nullptr) {
      cn = cnm * cnm;
    } else {   // fallback bound: scan this head's codebook (slow path, C ABI callers without norms)
      cn = 0.f;
      const float* cbf = p.cb + (int64_t)cbh * p.nb * p.C * bd;
      for (int e = tid; e < p.nb * p.C * bd; e += 256) cn = fmaxf(cn, cbf[e] * cbf[e] * bd);
      cn = warp_max(cn);
      if ((tid & 31) == 0) atomicMax(reinterpret_cast<int*>(&red[1]), __float_as_int(cn));
      __syncthreads();
      cn = red[1];
    }
    const float bound = sqrtf(red[0]) * sqrtf(cn) * 1.001f;
    scale = bound > 0.f ? exp2f(fminf(100.f, floorf(log2f(32768.f / bound)))) : 1.f;
    if (b == 0 && tid == 0) p.lut_scale_global[hh] = 1.f / scale;
  } else {
    if (b == 0 && tid == 0) p.lut_scale_global[hh] = 1.f;
  }
  if (c >= p.C) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    return;
  }
  float v[GP];
#pragma unroll
  for (int g = 0; g < GP; ++g) v[g] = 0.f;
  if (in_cb && !heavy) {
#pragma unroll
    for (int d = 0; d < 16; ++d) {
      if (d >= bd) break;
      const int ch = perm_s[b * bd + d];
#pragma unroll
      for (int g = 0; g < GP; ++g) v[g] = fmaf(q_s[g * D + ch], cw[d], v[g]);
    }
  }
  const int kh = b >> 3, blo = b & 7;
  constexpr int NH = L16 ? (GP >= 8 ? GP / 8 : 1) : GP / 4;
  uint8_t* base = p.lut_global + hh * (int64_t)p.lut_bytes;
  uint8_t* dst = (L16 && GP == 4) ? base + (int64_t)(kh >> 1) * kLutC * 128 + blo * 16 + (kh & 1) * 8
                                  : base + (int64_t)kh * NH * kLutC * 128 + blo * 16;
  store_lut_entry<GP, L16>(dst, c, v, scale);
  SUNSHAPE_SPAN_END(1);
  SUNSHAPE_LUTMARK(2);
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <int GP, bool L16>
void launch_lut_head_block_t(const DecodeParams& prm, int n_heads, cudaStream_t st) {
  launch_pdl(lut_kernel<GP, L16>, dim3(n_heads, prm.nbh * 8), 256, 0, st, prm);
}

// Producer warp of the tensor-core kernel: TMA tensor boxes for values, bulk
// copies (+ byte tails) for index and heavy rows, L2 prefetch ahead of the ring.
template <int DV>
SUNSHAPE_COLD void produce_mma(const DecodeParams& p, int64_t tb, int64_t te, uint64_t* full, uint64_t* empty,
                            uint8_t* stage0, int n_heavy, int lane, int pid) {
  const int S = p.stages;
  const int64_t hrow = (int64_t)n_heavy * p.bd * (p.heavy_dtype == SUNSHAPE_F32 ? 4 : 2);
  constexpr int NBOX = DV / 64;
  const int64_t n_tiles = te - tb;
  const int ahead = p.prefetch_ahead;
  // this warp issues tiles pid, pid + kProducersM, ...; cursors advance incrementally
  // (no 64-bit divisions on the issue path)
  int64_t hh = (tb + pid) / p.tph;
  int t0 = (int)(tb + pid - hh * p.tph) * kTileTokens;
  int64_t ph_h = hh;   // prefetch cursor
  int ph_t0 = t0;
  int64_t n_pref = 0;
  auto prefetch_next = [&]() {
    if (n_pref >= n_tiles) return;
    if (lane == 0) {
      const int ntok = min(kTileTokens, p.T - ph_t0);
      const int64_t row0 = ph_h * p.head_stride + ph_t0;
      prefetch_l2(reinterpret_cast<const uint8_t*>(p.v) + row0 * DV * 2, (uint32_t)ntok * DV * 2);
      const uintptr_t a0 = (reinterpret_cast<uintptr_t>(p.idx + row0 * p.nb) + 15) & ~uintptr_t(15);
      const uintptr_t a1 = reinterpret_cast<uintptr_t>(p.idx + (row0 + ntok) * p.nb) & ~uintptr_t(15);
      if (a1 > a0) prefetch_l2(reinterpret_cast<const void*>(a0), (uint32_t)(a1 - a0));
    }
    ++n_pref;
    ph_t0 += kTileTokens;
    if (ph_t0 >= p.T) { ph_t0 = 0; ++ph_h; }
  };
  if (ahead > 0 && pid == 0)
    while (n_pref < S + ahead && n_pref < n_tiles) prefetch_next();
  int s = pid % S;
  uint32_t phase = (uint32_t)((pid / S) & 1);
  const long long tp0 = SUNSHAPE_CLK();
  long long twait = 0, tissue = 0;
  for (int64_t i = pid; i < n_tiles; i += kProducersM) {
    if (i >= S) {
      const long long tw = SUNSHAPE_CLK();
      mbar_wait(&empty[s], phase ^ 1u, p.err, kErrWaitEmpty);
      twait += SUNSHAPE_CLK() - tw;
      if (ahead > 0 && pid == 0) {
        prefetch_next();
        prefetch_next();
      }
    }
    const int ntok = min(kTileTokens, p.T - t0);
    const int64_t row0 = hh * p.head_stride + t0;
    uint8_t* st = stage0 + (int64_t)s * p.stage_bytes;

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
    __syncwarp();
    if (lane == 0) {
      const long long ti = SUNSHAPE_CLK();
#ifdef SUNSHAPE_EXP_BULKV
      mbar_arrive_expect_tx(&full[s], ntok * DV * 2 + ibulk + hbulk);
      bulk_g2s(st, reinterpret_cast<const uint8_t*>(p.v) + row0 * DV * 2, ntok * DV * 2, &full[s]);
#else
      mbar_arrive_expect_tx(&full[s], NBOX * kVBoxBytes + ibulk + hbulk);
#pragma unroll
      for (int bx = 0; bx < NBOX; ++bx) tma_load_2d(st + bx * kVBoxBytes, &p.tmap_v, bx * 64, (int)row0, &full[s]);
#endif
      if (ibulk) bulk_g2s(st + p.off_stage_idx, reinterpret_cast<const void*>(ia0), ibulk, &full[s]);
      if (hbulk) bulk_g2s(st + p.off_stage_heavy, reinterpret_cast<const void*>(ha0), hbulk, &full[s]);
      tissue += SUNSHAPE_CLK() - ti;
    }
    __syncwarp();
    t0 += kProducersM * kTileTokens;
    while (t0 >= p.tph * kTileTokens) { t0 -= p.tph * kTileTokens; ++hh; }
    s += kProducersM;
    while (s >= S) { s -= S; phase ^= 1u; }
  }
  if (lane == 0) {
    SUNSHAPE_TRACE_ADD(0, SUNSHAPE_CLK() - tp0);
    SUNSHAPE_TRACE_ADD(1, twait);
    SUNSHAPE_TRACE_ADD(6, tissue);
  }
}

template <int GP, int DV, typename VT, bool L16>
__global__ void __launch_bounds__(kThreadsM, 1) decode_mma_kernel(const __grid_constant__ DecodeParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128B-swizzled TMA boxes need 1024-byte aligned destinations: align the carve-up base
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int NH = L16 ? (GP >= 8 ? GP / 8 : 1) : GP / 4;   // 16-byte LUT chunks per (block, codeword)
  constexpr int NT = (GP + 7) / 8;    // MMA n-tiles (8 query rows each)
  constexpr int MT = DV / 16;         // MMA m-tiles (16 value columns each)
  using Op = MmaOp<VT>;

  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kMaxStages;
  int* flag_s = reinterpret_cast<int*>(smem + 128);
  float* scale_s = reinterpret_cast<float*>(smem + 192);   // LUT scale (inverse), norm bounds
  uint64_t* lut_bar = reinterpret_cast<uint64_t*>(smem + 232);   // LUT bulk copy completion
  int* perm_s = reinterpret_cast<int*>(smem + p.off_perm);
  int8_t* hslot_s = reinterpret_cast<int8_t*>(smem + p.off_hslot);
  int8_t* hlist_s = hslot_s + 64;                 // heavy block ids in slot order
  float* q_s = reinterpret_cast<float*>(smem + p.off_q);
  uint8_t* pbuf = smem + p.off_p;
  uint8_t* lut = smem + p.off_lut;
  uint8_t* stage0 = smem + p.off_stage;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t grid = gridDim.x;
  const int64_t tb = tile_start(p, blockIdx.x, grid);
  const int64_t te = tile_start(p, blockIdx.x + 1, grid);

  if (tid == 0) {
    SUNSHAPE_MARK(0);
#ifdef SUNSHAPE_TRACE
    {
      unsigned smid;
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
      p.trace[blockIdx.x * 32 + 30] = smid;
    }
#endif
    for (int s = 0; s < p.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kWarpsPerTileM);
    }
    mbar_init(lut_bar, 1);
    fence_mbar_init();
    int n = 0;
    for (int b = 0; b < p.nb; ++b) {
      const bool h = p.heavy_mask != nullptr && p.heavy_mask[b] != 0;
      hslot_s[b] = h ? (int8_t)n : (int8_t)-1;
      if (h) hlist_s[n++] = (int8_t)b;
    }
    flag_s[2] = n;
  }
  for (int i = tid; i < p.D; i += kThreadsM) perm_s[i] = (int)p.perm[i];
  __syncthreads();
  const int n_heavy = flag_s[2];

  if (warp >= kWarpsM) {
    if (te <= tb) return;
    produce_mma<DV>(p, tb, te, full, empty, stage0, n_heavy, lane, warp - kWarpsM);
    return;
  }

  // ------------------------------------------------------------------ consumers
  const int ctid = tid;
  const int tg = warp / kWarpsPerTileM, half = warp % kWarpsPerTileM;
  uint8_t* pw = pbuf + warp * (NT * 512 + 64);      // [32 tokens][8*NT rows] 16-bit P tile
  float* alpha_s = reinterpret_cast<float*>(pw + NT * 512);
  const uint32_t pw_u32 = smem_u32(pw);
  const int hsize = p.heavy_dtype == SUNSHAPE_F32 ? 4 : 2;
  const int64_t hrow = (int64_t)n_heavy * p.bd * hsize;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const bool fast_idx = (p.nb & 7) == 0;
  const int gid = lane >> 2, tig = lane & 3;

  if (te <= tb) return;
  // LUTs come from the preceding lut_kernel grid (programmatic dependent launch)
  if (p.lut_global != nullptr) asm volatile("griddepcontrol.wait;" ::: "memory");
  const long long tc0 = SUNSHAPE_CLK();
  long long t_wait = 0, t_lut = 0, t_end = 0;
  uint32_t lut_phase_bit = 0;
  int64_t f = tb;
  while (f < te) {
    const int64_t hh = f / p.tph;
    const int64_t fend = min(te, (hh + 1) * p.tph);
    const int i0 = (int)(f - tb), i1 = (int)(fend - tb);
    const long long tl = SUNSHAPE_CLK();
    float inv_scale = 1.f;
    if (p.lut_global != nullptr) {
      // the LUT region also served as staging for the last segment's partials: order those generic
      // writes before the async-proxy copy, then bulk-copy this head's LUT from the workspace
      fence_proxy_async_smem();
      named_barrier(kBarConsumers, kConsumerThreadsM);
      if (ctid == 0) {
        mbar_arrive_expect_tx(lut_bar, (uint32_t)p.lut_bytes);
        const uint8_t* src = p.lut_global + hh * (int64_t)p.lut_bytes;
        for (int off = 0; off < p.lut_bytes; off += 32768)
          bulk_g2s(lut + off, src + off, (uint32_t)min(32768, p.lut_bytes - off), lut_bar);
      }
      if (n_heavy > 0)   // permuted, scaled query rows for the dense heavy-block dot products
        load_query_rows<GP, kConsumerThreadsM>(p, hh, perm_s, q_s, ctid);
      mbar_wait(lut_bar, lut_phase_bit, p.err, kErrWaitFull);
      lut_phase_bit ^= 1u;
      if (L16) inv_scale = __ldcg(p.lut_scale_global + hh);
      named_barrier(kBarConsumers, kConsumerThreadsM);
    } else {
      build_lut_m<GP, L16>(p, hh, perm_s, hslot_s, q_s, lut, ctid, scale_s);
      if (L16) inv_scale = scale_s[0];
    }
    // this CTA reads no more global LUT tables: the next LUT grid may start overwriting them
    if (fend >= te) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#ifdef SUNSHAPE_TRACE
    if (ctid == 0 && f - tb < 2 * p.tph && (hh - tb / p.tph) < 2) SUNSHAPE_MARK(4 + 2 * (int)(hh - tb / p.tph));
#endif
    t_lut += SUNSHAPE_CLK() - tl;

    float m_run[GP], l_run[GP];
    float acc[MT][NT][4];
#pragma unroll
    for (int g = 0; g < GP; ++g) { m_run[g] = NEG_INF; l_run[g] = 0.f; }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[mt][nt][c] = 0.f;

    const int64_t b_idx = hh / p.kv_heads;
    const int kvh = (int)(hh % p.kv_heads);

    const int ifirst = i0 + ((tg - i0 % kTileGroupsM) + kTileGroupsM) % kTileGroupsM;
    int s = ifirst % p.stages;
    uint32_t phase = (uint32_t)((ifirst / p.stages) & 1);
    const int64_t seg_tile0 = hh * p.tph;
    for (int i = ifirst; i < i1; i += kTileGroupsM) {
      const long long tw = SUNSHAPE_CLK();
      mbar_wait(&full[s], phase, p.err, kErrWaitFull);
      t_wait += SUNSHAPE_CLK() - tw;
#ifdef SUNSHAPE_TRACE
      if (i == 0 && lane == 0) SUNSHAPE_MARK(1);
      if (i == (int)(te - tb) - 1 && lane == 0) SUNSHAPE_MARK(2);
#endif
      const int t0 = (int)(tb + i - seg_tile0) * kTileTokens;
      const int ntok = min(kTileTokens, p.T - t0);
      const int64_t row0 = hh * p.head_stride + t0;
      uint8_t* st = stage0 + (int64_t)s * p.stage_bytes;
      const uint8_t* itile = st + p.off_stage_idx + (reinterpret_cast<uintptr_t>(p.idx + row0 * p.nb) & 15);
      const uint8_t* htile = st + p.off_stage_heavy;
      if (n_heavy > 0)
        htile += reinterpret_cast<uintptr_t>(reinterpret_cast<const uint8_t*>(p.heavy) + row0 * hrow) & 15;
      const int tok0 = half * 32;
      const int t = tok0 + lane;
      const bool valid = t < ntok;

      if (tok0 < ntok) {
        // tail tile: rows past the sequence may hold stale cache data -> zero them (p is 0 there)
        if (ntok < tok0 + 32) {
          for (int e = lane; e < (tok0 + 32 - ntok) * (DV / 8); e += 32) {
            const int rr = ntok + e / (DV / 8), ch = e % (DV / 8);
            *reinterpret_cast<uint4*>(st + (ch >> 3) * kVBoxBytes + rr * 128 + ((ch & 7) << 4)) =
                make_uint4(0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
          __syncwarp();
        }
        // ---- scores: lane t against all GP rows
        float2 part[GP / 2];
#pragma unroll
        for (int g = 0; g < GP / 2; ++g) part[g] = make_float2(0.f, 0.f);
        if (valid) {
          const uint8_t* irow = itile + t * p.nb;
          const int rot = lane & 7;
          // GP == 4 fp16 LUT: lanes 8-15 of each 16-lane phase walk each block-group pair in the
          // opposite order, so the two 8-byte halves of a slot are read by different lanes
          const int kswap = (L16 && GP == 4) ? ((lane >> 3) & 1) : 0;
#pragma unroll kKkUnroll
          for (int kk = 0; kk < 8; ++kk) {   // block groups of 8 (up to 64 blocks)
            if (kk >= p.nbh) break;
            const int kh = kk ^ kswap;
            uint64_t w;
            if (fast_idx) {
              w = *reinterpret_cast<const uint64_t*>(irow + 8 * kh);
            } else {
              w = 0;
              for (int q = 0; q < 8; ++q) {
                const int b = 8 * kh + q;
                if (b < p.nb) w |= (uint64_t)irow[b] << (8 * q);
              }
            }
            // rotate so byte kl of w holds block 8*kh + ((kl + lane) & 7)
            const uint64_t wr = rot ? ((w >> (8 * rot)) | (w << (64 - 8 * rot))) : w;
            const uint32_t lo = (uint32_t)wr, hi = (uint32_t)(wr >> 32);
            const uint8_t* kbase = (L16 && GP == 4) ? lut + (kh >> 1) * kLutC * 128 + (kh & 1) * 8
                                                    : lut + kh * NH * kLutC * 128;
#pragma unroll
            for (int kl = 0; kl < 8; ++kl) {
              const uint32_t c = ((kl < 4 ? lo : hi) >> (8 * (kl & 3))) & 0xffu;
              const uint8_t* e = kbase + c * 128u + (uint32_t)(((kl + lane) & 7) << 4);
              if constexpr (L16 && GP == 4) {
                const uint2 r = *reinterpret_cast<const uint2*>(e);
                asm("add.f32.f16 %0, %1, %2;" : "=f"(part[0].x) : "h"((unsigned short)(r.x & 0xffffu)), "f"(part[0].x));
                asm("add.f32.f16 %0, %1, %2;" : "=f"(part[0].y) : "h"((unsigned short)(r.x >> 16)), "f"(part[0].y));
                asm("add.f32.f16 %0, %1, %2;" : "=f"(part[1].x) : "h"((unsigned short)(r.y & 0xffffu)), "f"(part[1].x));
                asm("add.f32.f16 %0, %1, %2;" : "=f"(part[1].y) : "h"((unsigned short)(r.y >> 16)), "f"(part[1].y));
                continue;
              }
#pragma unroll
              for (int h = 0; h < NH; ++h) {
                if constexpr (L16) {
                  const uint4 r = *reinterpret_cast<const uint4*>(e + h * kLutC * 128);
                  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    float2& a = part[4 * h + k];
                    asm("add.f32.f16 %0, %1, %2;" : "=f"(a.x) : "h"((unsigned short)(w[k] & 0xffffu)), "f"(a.x));
                    asm("add.f32.f16 %0, %1, %2;" : "=f"(a.y) : "h"((unsigned short)(w[k] >> 16)), "f"(a.y));
                  }
                } else {
                  const float4 v = *reinterpret_cast<const float4*>(e + h * kLutC * 128);
                  part[2 * h] = __fadd2_rn(part[2 * h], make_float2(v.x, v.y));
                  part[2 * h + 1] = __fadd2_rn(part[2 * h + 1], make_float2(v.z, v.w));
                }
              }
            }
          }
          if constexpr (L16) {
#pragma unroll
            for (int g = 0; g < GP / 2; ++g) { part[g].x *= inv_scale; part[g].y *= inv_scale; }
          }
          // SunShape-Mixed heavy blocks: dense dot of the stored block with the permuted query
          if (n_heavy > 0 && p.bd == 8 && hsize == 2 && (reinterpret_cast<uintptr_t>(htile) & 15) == 0) {
            // bf16 blocks of 8: one 16-byte load of the stored block, query rows as float4 pairs
            for (int hs = 0; hs < n_heavy; ++hs) {
              const int b = hlist_s[hs];
              const uint4 raw = *reinterpret_cast<const uint4*>(htile + ((int64_t)t * n_heavy + hs) * 16);
              const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
              float x[8];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                x[2 * k] = __uint_as_float(rw[k] << 16);
                x[2 * k + 1] = __uint_as_float(rw[k] & 0xffff0000u);
              }
              const float* qb = q_s + b * 8;
#pragma unroll
              for (int g = 0; g < GP; ++g) {
                const float4 q0 = *reinterpret_cast<const float4*>(qb + g * p.D);
                const float4 q1 = *reinterpret_cast<const float4*>(qb + g * p.D + 4);
                float a = (g & 1) ? part[g >> 1].y : part[g >> 1].x;
                a = fmaf(q0.x, x[0], a); a = fmaf(q0.y, x[1], a); a = fmaf(q0.z, x[2], a); a = fmaf(q0.w, x[3], a);
                a = fmaf(q1.x, x[4], a); a = fmaf(q1.y, x[5], a); a = fmaf(q1.z, x[6], a); a = fmaf(q1.w, x[7], a);
                if (g & 1) part[g >> 1].y = a; else part[g >> 1].x = a;
              }
            }
          } else
          for (int hs = 0; hs < n_heavy; ++hs) {
            const int b = hlist_s[hs];
            const uint8_t* hv = htile + ((int64_t)t * n_heavy + hs) * p.bd * hsize;
            const float* qb = q_s + b * p.bd;
            for (int d = 0; d < p.bd; ++d) {
              const float x = hsize == 4 ? reinterpret_cast<const float*>(hv)[d]
                                         : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(hv)[d]);
#pragma unroll
              for (int g = 0; g < GP / 2; ++g) {
                part[g].x = fmaf(qb[(2 * g) * p.D + d], x, part[g].x);
                part[g].y = fmaf(qb[(2 * g + 1) * p.D + d], x, part[g].y);
              }
            }
          }
        }
        float sc[GP];
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          float v = valid ? ((g & 1) ? part[g >> 1].y : part[g >> 1].x) : NEG_INF;
          if (valid && p.mask != nullptr && g < p.Rc) {
            const int r = p.r0 + g;
            const int gq = r / p.L, ql = r - gq * p.L;
            const int64_t hq = (int64_t)kvh * p.G + gq;
            v += load_as_float(p.mask, b_idx * p.msb + hq * p.msh + ql * p.msq + (t0 + t), p.mask_dtype);
          }
          sc[g] = v;
        }
        // ---- online softmax with lazy rescale
        bool need = false;
#pragma unroll
        for (int g = 0; g < GP; ++g) need |= sc[g] > m_run[g] + kLazyTau;
        if (__any_sync(0xffffffffu, need)) {
#pragma unroll
          for (int g = 0; g < GP; ++g) {
            const float mn = fmaxf(m_run[g], warp_max(sc[g]));
            const float a = (mn == NEG_INF) ? 1.f : fast_exp2((m_run[g] - mn) * kLog2e);
            m_run[g] = mn;
            l_run[g] *= a;
            if (lane == 0) alpha_s[g] = a;
          }
          __syncwarp();
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int g0 = nt * 8 + 2 * tig;
            const float a0 = g0 < GP ? alpha_s[g0] : 1.f, a1 = g0 + 1 < GP ? alpha_s[g0 + 1] : 1.f;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              acc[mt][nt][0] *= a0; acc[mt][nt][1] *= a1; acc[mt][nt][2] *= a0; acc[mt][nt][3] *= a1;
            }
          }
        }
        uint32_t pk[NT * 4];   // this token's P row, packed 16-bit pairs
#pragma unroll
        for (int g2 = 0; g2 < NT * 4; ++g2) pk[g2] = 0u;
#pragma unroll
        for (int g = 0; g < GP; ++g) {
          const float pr = (m_run[g] == NEG_INF) ? 0.f : fast_exp2((sc[g] - m_run[g]) * kLog2e);
          l_run[g] += pr;
          pk[g >> 1] |= (uint32_t)Op::bits(pr) << (16 * (g & 1));
        }
#pragma unroll
        for (int ch = 0; ch < NT; ++ch)
          *reinterpret_cast<uint4*>(pw + p_chunk_offset<NT>(lane, ch)) =
              make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
        __syncwarp();
        // ---- acc^T[dv][g] += V^T[dv][t] . P^T[t][g] over this warp's 32 tokens
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
          // B fragments (P^T, k = token, n = query row) from the token-major P tile via transposed ldmatrix
          uint32_t bfrag[NT][2];
          {
            const int prow = ks * 16 + (lane & 15);
            if constexpr (NT == 1) {
              ldsm_x2_trans(bfrag[0], pw_u32 + p_chunk_offset<1>(prow, 0));
            } else {
              uint32_t r4[4];
              ldsm_x4_trans(r4, pw_u32 + p_chunk_offset<2>(prow, lane >> 4));
              bfrag[0][0] = r4[0]; bfrag[0][1] = r4[1]; bfrag[1][0] = r4[2]; bfrag[1][1] = r4[3];
            }
          }
          const int mi = lane >> 3;
          const int trow = tok0 + ks * 16 + ((mi >> 1) << 3) + (lane & 7);   // token row of the V tile
          const uint32_t vrow = smem_u32(st) + (uint32_t)trow * 128u;
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const int dv = mt * 16 + ((mi & 1) << 3);
            const int ch = (dv & 63) >> 3;
            uint32_t afrag[4];
            ldsm_x4_trans(afrag, vrow + (uint32_t)(dv >> 6) * kVBoxBytes + (uint32_t)((ch ^ (trow & 7)) << 4));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Op::mma(acc[mt][nt], afrag, bfrag[nt]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      s += kTileGroupsM;
      while (s >= p.stages) { s -= p.stages; phase ^= 1u; }
    }

    // ---------------- segment end: per-warp partials -> staging -> merge
    const long long te0 = SUNSHAPE_CLK();
    float l_tot[GP];
#pragma unroll
    for (int g = 0; g < GP; ++g) l_tot[g] = warp_sum(l_run[g]);
    named_barrier(kBarConsumers, kConsumerThreadsM);   // LUT reads done: reuse it as staging
    constexpr int ROWF = DV + 2;
    float* stg = reinterpret_cast<float*>(lut);
    float* mine = stg + warp * GP * ROWF;
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < GP; ++g) { mine[g * ROWF] = m_run[g]; mine[g * ROWF + 1] = l_tot[g]; }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int g0 = nt * 8 + 2 * tig, dv0 = mt * 16 + gid;
        if (g0 < GP) {
          mine[g0 * ROWF + 2 + dv0] = acc[mt][nt][0];
          mine[g0 * ROWF + 2 + dv0 + 8] = acc[mt][nt][2];
        }
        if (g0 + 1 < GP) {
          mine[(g0 + 1) * ROWF + 2 + dv0] = acc[mt][nt][1];
          mine[(g0 + 1) * ROWF + 2 + dv0 + 8] = acc[mt][nt][3];
        }
      }
    named_barrier(kBarConsumers, kConsumerThreadsM);
    finish_segment<GP, DV, kWarpsM>(p, stg, hh, tb, grid, ctid, flag_s);
    t_end += SUNSHAPE_CLK() - te0;
#ifdef SUNSHAPE_TRACE
    if (ctid == 0 && (hh - tb / p.tph) < 2) SUNSHAPE_MARK(5 + 2 * (int)(hh - tb / p.tph));
#endif
    f = fend;
  }
#ifdef SUNSHAPE_TRACE
  named_barrier(kBarConsumers, kConsumerThreadsM);
  if (ctid == 0) SUNSHAPE_MARK(3);
#endif
  if (lane == 0) {
    SUNSHAPE_TRACE_ADD(2, SUNSHAPE_CLK() - tc0);
    SUNSHAPE_TRACE_ADD(3, t_wait);
    SUNSHAPE_TRACE_ADD(4, t_lut);
    SUNSHAPE_TRACE_ADD(5, t_end);
  }
}

template <int GP, int DV, typename VT, bool L16>
void launch_decode_mma_t(const DecodeLaunch& l, cudaStream_t st) {
  auto k = decode_mma_kernel<GP, DV, VT, L16>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, l.smem);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (l.prm.lut_global == nullptr) {
    k<<<(unsigned)l.grid, kThreadsM, l.smem, st>>>(l.prm);
  } else {
    // programmatic dependent launch after lut_kernel: this grid may start while the LUTs are being
    // built; its consumers wait for them with griddepcontrol.wait
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)l.grid);
    cfg.blockDim = dim3(kThreadsM);
    cfg.dynamicSmemBytes = (size_t)l.smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, k, l.prm);
  }
}


// Instantiated in decode_mma_bf16.cu / decode_mma_f16.cu.
extern template void launch_decode_mma_t<4, 64, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 64, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 128, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 128, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 256, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 256, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 64, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 64, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 128, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 128, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 256, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 256, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 64, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 64, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 128, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 128, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 256, __nv_bfloat16, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 256, __nv_bfloat16, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 64, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 128, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<4, 256, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 64, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 128, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<8, 256, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 64, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 64, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 128, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 128, __half, true>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 256, __half, false>(const DecodeLaunch&, cudaStream_t);
extern template void launch_decode_mma_t<16, 256, __half, true>(const DecodeLaunch&, cudaStream_t);

}  // namespace sunshape
