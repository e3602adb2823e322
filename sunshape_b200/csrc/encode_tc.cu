// SunShape key encode on the 5th-generation tensor cores (tcgen05, kind::tf32).
//
// Per (128-key tile, block b) the squared distances to all C codewords are one
// 128 x C x K GEMM (K = 8, 16, 24 for block_dim 2, 4, 8) whose fp32 accumulator
// lives in tensor memory:
//
//   A row r  (key)      = [ x(bd),      x(bd),      1, 1, 1,             0 ... ]
//   B row c  (codeword) = [ -2 c_hi(bd), -2 c_lo(bd), n_hi, n_mid, n_lo, 0 ... ]
//   D[r][c]             = |c|^2 - 2 x.c            (the |x|^2 term is common)
//
// x is a bf16/f16 key value, exactly representable in tf32.  c = c_hi + c_lo and
// |c|^2 = n_hi + n_mid + n_lo are split into tf32 parts (round-to-nearest for the
// high parts, the remainders exact in fp32), so the products are exact and D
// carries ~2^-22 relative error: near fp32, which the index parity rule needs
// (codec.py:376-377 takes torch.argmin of torch.cdist in fp32).
//
// The operands are written by the CTA's threads into 128B-swizzled K-major
// shared-memory tiles (the ProfilePerm gather and the tf32 split happen on the
// way, which a TMA box cannot express); one elected thread issues K / 8
// tcgen05.mma (K = 8 each) and commits to an mbarrier; each thread then reads its
// key's row of D from tensor memory (tcgen05.ld 32x32b) and keeps the FIRST
// minimum, as torch.argmin does.  Heavy (SunShape-Mixed) blocks are copied and
// keep index 0 (codec.py:367-374).  Two or three CTAs share an SM, so one CTA's
// operand build and argmin overlap another's MMA.
#include "common.cuh"
#include "encode_params.cuh"

namespace sunshape {

// Error word of the encode kernels on this device (first writer wins; read and cleared by
// sunshape_encode_error).  sunshape_encode has no workspace, so the word is library-global.
__device__ int g_encode_error;

namespace {

constexpr int kTcRows = 128;          // keys per CTA = MMA M = TMEM lanes
constexpr int kRowBytes = 128;        // one swizzle row: 32 tf32 words (K = 24 used)
constexpr int kSmemPerSm = 233472;    // 228 KiB of shared memory per SM
constexpr int kSmemReservedPerCta = 1024;
constexpr int kTcSmemLimit = 232448;   // 227 KiB opt-in per CTA

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t y;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(y) : "f"(x));
  return y;
}

// byte offset of 16-byte chunk j of row r in a 128B-swizzled K-major tile (8-row atoms of 1024 B)
__device__ __forceinline__ uint32_t sw128(int r, int j) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * kRowBytes + ((j ^ (r & 7)) << 4));
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// shared-memory matrix descriptor: K-major, 128B swizzle, 8-row groups 1024 B apart
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// instruction descriptor: kind::tf32, fp32 accumulator, A and B K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t idesc_tf32(int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcRows >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane, waited for before return
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// completes every earlier tcgen05.ld of this thread; the registers are tied so no use moves above it
__device__ __forceinline__ void tc_wait_ld(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15])
               :
               : "memory");
}

// orders uses of v after an earlier tcgen05.wait::ld (no instruction emitted)
__device__ __forceinline__ void tc_tie(uint32_t (&v)[16]) {
  asm volatile(""
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]),
                 "+r"(v[15])
               :
               : "memory");
}

__device__ __forceinline__ void argmin16(const uint32_t (&v)[16], int c0, float& best, int& besti) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float dist = __uint_as_float(v[j]);
    if (dist < best) { best = dist; besti = c0 + j; }
  }
}

struct TcLayout {
  int a, b, keys, inv, hslot, idx, bar, tslot, total;   // byte offsets from the 1024-aligned base
  int key_pitch;                                        // bytes per staged key row
};

__host__ __device__ inline TcLayout tc_layout(int D, int C, int nb) {
  TcLayout l;
  l.a = 0;
  l.b = kTcRows * kRowBytes;
  l.keys = l.b + C * kRowBytes;
  l.key_pitch = (D + 8) * 2;                          // 16-byte chunks, 8 consecutive rows hit 8 bank groups
  l.inv = l.keys + kTcRows * l.key_pitch;
  l.hslot = l.inv + D * 4;
  l.idx = l.hslot + ((nb + 15) / 16) * 16;
  l.bar = l.idx + ((kTcRows * nb + 15) / 16) * 16;
  l.tslot = l.bar + 8;
  l.total = l.tslot + 8;
  return l;
}

// Operand row of block_dim BD: words [0, BD) and [BD, 2 BD) pair the key with c_hi and c_lo, words
// [2 BD, 2 BD + 3) carry the codeword norm, the rest up to KW (a multiple of the MMA K = 8) are zero.
template <int BD>
struct TcShape {
  static constexpr int KW = (2 * BD + 3 + 7) / 8 * 8;   // 8, 16, 24 words for BD = 2, 4, 8
  static constexpr int NCH = KW / 4;                   // 16-byte chunks per operand row
  static constexpr int NMMA = KW / 8;                  // tcgen05.mma per block
};

template <int BD>
__global__ void __launch_bounds__(kTcRows) encode_tc_kernel(const __grid_constant__ EncodeParams p, int tmem_cols) {
  using S = TcShape<BD>;
  extern __shared__ uint8_t tc_smem_raw[];
  const uint32_t raw = smem_u32(tc_smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = tc_smem_raw + (base - raw);
  const int D = p.D, C = p.C, nb = p.nb;
  const TcLayout L = tc_layout(D, C, nb);
  const uint32_t sA = base + L.a, sB = base + L.b;
  uint8_t* keys_s = sm + L.keys;
  int* inv_s = reinterpret_cast<int*>(sm + L.inv);
  int8_t* hslot_s = reinterpret_cast<int8_t*>(sm + L.hslot);
  uint8_t* idx_s = sm + L.idx;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.bar);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + L.tslot);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int64_t hh = blockIdx.y;
  const int row0 = blockIdx.x * kTcRows;
  const int nrows = min(kTcRows, p.n_tokens - row0);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
    int n = 0;
    for (int b = 0; b < nb; ++b) {
      const bool h = p.heavy_mask != nullptr && p.heavy_mask[b] != 0;
      hslot_s[b] = h ? (int8_t)n++ : (int8_t)-1;
    }
  }
  for (int i = tid; i < D; i += kTcRows) inv_s[(int)p.perm[i]] = i;
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
  int n_heavy = 0;
  for (int b = 0; b < nb; ++b) n_heavy += hslot_s[b] >= 0;

  // stage the tile's keys permuted (16-bit payload as is): keys_s[r][inv[d]] = key[r][d]
  {
    const uint16_t* keys = reinterpret_cast<const uint16_t*>(p.keys);
    const int cpr = D >> 3;                               // 16-byte chunks per key row
    for (int e = tid; e < kTcRows * cpr; e += kTcRows) {
      const int r = e / cpr, d0 = (e - r * cpr) << 3;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (r < nrows)
        v = __ldg(reinterpret_cast<const uint4*>(keys + hh * p.key_hs + (int64_t)(row0 + r) * p.key_ts + d0));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      uint16_t* dst = reinterpret_cast<uint16_t*>(keys_s + r * L.key_pitch);
#pragma unroll
      for (int i = 0; i < 8; ++i) dst[inv_s[d0 + i]] = (uint16_t)(w[i >> 1] >> ((i & 1) * 16));
    }
  }
  __syncthreads();

  const int cbh = p.n_cb == 1 ? 0 : (int)((hh % p.kv_heads) % p.n_cb);
  const float* cb = p.cb + (int64_t)cbh * nb * C * BD;
  const bool bf16 = p.keys_dtype == SUNSHAPE_BF16;
  const uint32_t idesc = idesc_tf32(C);
  const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
  uint32_t phase = 0;

  for (int b = 0; b < nb; ++b) {
    const uint32_t* kp = reinterpret_cast<const uint32_t*>(keys_s + tid * L.key_pitch + b * BD * 2);
    float x[BD];
#pragma unroll
    for (int i = 0; i < BD; ++i) {
      const uint16_t h = (uint16_t)(kp[i >> 1] >> ((i & 1) * 16));
      x[i] = bf16 ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
    }
    if (hslot_s[b] >= 0) {   // SunShape-Mixed: stored densely, index 0
      if (tid < nrows) {
        const int64_t o = ((hh * p.out_hs + row0 + tid) * n_heavy + hslot_s[b]) * BD;
#pragma unroll
        for (int d = 0; d < BD; ++d) store_from_float(p.heavy_out, o + d, p.heavy_dtype, x[d]);
      }
      idx_s[tid * nb + b] = 0;
      continue;
    }
    // B: this thread's codewords c = tid, tid + 128, ...
    const float* cbb = cb + (int64_t)b * C * BD;
    for (int c = tid; c < C; c += kTcRows) {
      uint32_t w[S::KW];
      float n2 = 0.f;
#pragma unroll
      for (int d = 0; d < BD; ++d) {
        const float cv = __ldg(cbb + c * BD + d);
        n2 = fmaf(cv, cv, n2);
        const uint32_t hi = tf32_rna(cv);
        w[d] = __float_as_uint(-2.f * __uint_as_float(hi));
        w[BD + d] = __float_as_uint(-2.f * (cv - __uint_as_float(hi)));
      }
      const uint32_t nh = tf32_rna(n2);
      const float r1 = n2 - __uint_as_float(nh);
      const uint32_t nm = tf32_rna(r1);
      w[2 * BD] = nh;
      w[2 * BD + 1] = nm;
      w[2 * BD + 2] = __float_as_uint(r1 - __uint_as_float(nm));
#pragma unroll
      for (int k = 2 * BD + 3; k < S::KW; ++k) w[k] = 0u;
#pragma unroll
      for (int j = 0; j < S::NCH; ++j) sts128(sB + sw128(c, j), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    }
    // A: this thread's key, block b, twice (against c_hi and c_lo), then the norm's multipliers
    {
      uint32_t w[S::KW];
#pragma unroll
      for (int d = 0; d < BD; ++d) w[d] = w[BD + d] = __float_as_uint(x[d]);
#pragma unroll
      for (int k = 2 * BD; k < S::KW; ++k) w[k] = k < 2 * BD + 3 ? __float_as_uint(1.0f) : 0u;
#pragma unroll
      for (int j = 0; j < S::NCH; ++j) sts128(sA + sw128(tid, j), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
    }
    fence_proxy_async_smem();   // generic-proxy operand writes -> tensor core (async proxy)
    tc_fence_before();          // the previous block's tcgen05.ld are complete (waited) before the barrier
    __syncthreads();
    if (tid == 0) {
      tc_fence_after();
      const uint64_t ad = smem_desc_sw128(sA), bdsc = smem_desc_sw128(sB);
#pragma unroll
      for (int k = 0; k < S::NMMA; ++k)   // K = 8 tf32 = 32 bytes per MMA: advance 2 descriptor units
        tc_mma_tf32(tmem, ad + 2 * k, bdsc + 2 * k, idesc, k > 0);
      tc_commit(bar);
    }
    mbar_wait(bar, phase, p.err ? p.err : &g_encode_error, 121);
    phase ^= 1u;
    tc_fence_after();

    // argmin over this key's TMEM row, first minimum; up to 64 columns in flight per wait
    float best = __int_as_float(0x7f800000);
    int besti = 0;
    for (int c0 = 0; c0 < C; c0 += 64) {
      uint32_t v0[16], v1[16], v2[16], v3[16];
      const int nq = min(4, (C - c0) >> 4);   // warp-uniform
      tc_ld16(lane_base + (uint32_t)c0, v0);
      if (nq > 1) tc_ld16(lane_base + (uint32_t)(c0 + 16), v1);
      if (nq > 2) tc_ld16(lane_base + (uint32_t)(c0 + 32), v2);
      if (nq > 3) tc_ld16(lane_base + (uint32_t)(c0 + 48), v3);
      tc_wait_ld(v0);
      tc_tie(v1);
      tc_tie(v2);
      tc_tie(v3);
      argmin16(v0, c0, best, besti);
      if (nq > 1) argmin16(v1, c0 + 16, best, besti);
      if (nq > 2) argmin16(v2, c0 + 32, best, besti);
      if (nq > 3) argmin16(v3, c0 + 48, best, besti);
    }
    idx_s[tid * nb + b] = (uint8_t)besti;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tmem_cols) : "memory");
  }
  // the tile's indices are one contiguous run of nrows * nb entries
  const int64_t o0 = (hh * p.out_hs + row0) * nb;
  for (int e = tid; e < nrows * nb; e += kTcRows) {
    const int v = idx_s[e];
    if (p.index_dtype == SUNSHAPE_U8) reinterpret_cast<uint8_t*>(p.idx_out)[o0 + e] = (uint8_t)v;
    else if (p.index_dtype == SUNSHAPE_I16) reinterpret_cast<int16_t*>(p.idx_out)[o0 + e] = (int16_t)v;
    else reinterpret_cast<int32_t*>(p.idx_out)[o0 + e] = v;
  }
}

}  // namespace

// The tensor-core encode takes 16-bit keys with 16-byte aligned rows, block_dim 2, 4 or 8 and
// C a multiple of 16 up to 256 (one MMA N); everything else uses encode_kernel.
bool encode_tc_supported(const EncodeParams& p) {
  const bool k16 = p.keys_dtype == SUNSHAPE_BF16 || p.keys_dtype == SUNSHAPE_F16;
  return k16 && (p.bd == 2 || p.bd == 4 || p.bd == 8) && p.C % 16 == 0 && p.C >= 16 && p.C <= 256 && p.D % 8 == 0 &&
         (reinterpret_cast<uintptr_t>(p.keys) & 15) == 0 && (p.key_ts * 2) % 16 == 0 && (p.key_hs * 2) % 16 == 0 &&
         (reinterpret_cast<uintptr_t>(p.cb) & 15) == 0 && tc_layout(p.D, p.C, p.nb).total + 1024 <= kTcSmemLimit;
}

int launch_encode_tc(const EncodeParams& p, int n_heads, cudaStream_t st) {
  int cols = 32;
  while (cols < p.C) cols <<= 1;
  int smem = tc_layout(p.D, p.C, p.nb).total + 1024;   // + alignment slack for the 1024-byte swizzle atoms
  // CTAs resident per SM must not ask for more than the SM's 512 TMEM columns
  const int max_ctas = 512 / cols;
  if (kSmemPerSm / (smem + kSmemReservedPerCta) > max_ctas) smem = kSmemPerSm / (max_ctas + 1) - kSmemReservedPerCta + 16;
  dim3 grid((p.n_tokens + kTcRows - 1) / kTcRows, n_heads);
  switch (p.bd) {
    case 2:
      cudaFuncSetAttribute(encode_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      encode_tc_kernel<2><<<grid, kTcRows, smem, st>>>(p, cols);
      break;
    case 4:
      cudaFuncSetAttribute(encode_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      encode_tc_kernel<4><<<grid, kTcRows, smem, st>>>(p, cols);
      break;
    default:
      cudaFuncSetAttribute(encode_tc_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      encode_tc_kernel<8><<<grid, kTcRows, smem, st>>>(p, cols);
      break;
  }
  return 0;
}

int encode_error_word(int* code, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_encode_error, sizeof(int), 0, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && *code != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_encode_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice);
  }
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace sunshape
