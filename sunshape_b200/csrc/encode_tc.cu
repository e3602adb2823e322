// SunShape key encode on the 5th-generation tensor cores (tcgen05, kind::tf32), warp-specialised.
//
// For a tile of 128 keys and a codebook block b the squared distances to the codewords are one
// 128 x N x K GEMM whose fp32 accumulator lives in tensor memory (TMEM):
//
//   fp32 keys:   A row r = [ x_hi(bd), x_hi(bd), x_lo(bd), 1, 1, 1, 0 ... ]
//                B row c = [ b_hi(bd), b_lo(bd), b_hi(bd), n_hi, n_mid, n_lo, 0 ... ]
//   16-bit keys: A row r = [ x(bd), x(bd), 1, 1, 1, 0 ... ]
//                B row c = [ b_hi(bd), b_lo(bd), n_hi, n_mid, n_lo, 0 ... ]
//   D[r][c] = x . b + |c|^2 = |c|^2 - 2 x.c            (b = -2 c; the |x|^2 term is common to a row)
//
// Every operand value is split into tf32 parts (round-to-nearest; the remainders are exact in fp32),
// so the products are exact and D carries ~2^-22 relative error ("3xTF32" for fp32 keys; 16-bit keys
// are exact in tf32): near fp32, which the index parity rule needs (codec.py:376-377 takes
// torch.argmin of torch.cdist in fp32).  The first minimum of each row is the codeword index
// (torch.argmin's first index on ties).
//
// One persistent CTA per SM walks tiles (head, 128 keys) and, per tile, steps (light block b,
// codeword slab h) of N = 128 or 256 codewords:
//
//   * key tiles arrive by TMA tensor copies (3-D map [heads, tokens, head_dim], 128-byte swizzle,
//     rows past the sequence zero-filled), double-buffered so tile i+1 lands while tile i computes;
//   * the raw fp32 codebook rows of each step arrive by 1-D bulk copies into a ring several steps
//     ahead (the codebook stays L2-resident; its tf32 split costs a few instructions per row);
//   * builder warps (4) gather the ProfilePerm'd block of their key (A row) and split one or two
//     codeword rows (B rows) into double-buffered, swizzled, K-major shared-memory operands; one
//     elected builder issues the K/8 tcgen05.mma into one of two TMEM accumulators and commits;
//   * argmin warps (4, one TMEM lane quarter each) take the previous step's accumulator row with
//     tcgen05.ld, reduce it with 3-input min over groups of 16 columns, recover the first index of
//     the minimum from the winning group, and release the accumulator -- so the MMA of step s+1
//     overlaps the argmin of step s;
//   * SunShape-Mixed heavy blocks are copied from the staged keys and keep index 0
//     (codec.py:367-374); each tile's indices leave as one contiguous run.
//
// Every wait is bounded; the first timeout records error 121 in the encode error word and turns
// every later wait of the CTA into a no-op, so a protocol fault ends the kernel in microseconds.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "encode_params.cuh"

namespace sunshape {

// Error word of the encode kernels on this device (first writer wins; read and cleared by
// sunshape_encode_error).  sunshape_encode has no workspace, so the word is library-global.
__device__ int g_encode_error;

#ifdef SUNSHAPE_TRACE
// opt-in cycle accounting of the encode pipeline (trace builds only): [0] builder total, [1] builder
// waiting for operand buffers, [2] waiting for keys, [3] waiting for codebook rows, [4] MMA issuer
// waiting for TMEM, [5] argmin total, [6] argmin waiting for MMAs
__device__ unsigned long long g_enc_trace[16];
#define ENC_T0(v) const long long v = clock64()
#define ENC_ADD(k, v) atomicAdd(&g_enc_trace[k], (unsigned long long)(clock64() - (v)))
#else
#define ENC_T0(v) ((void)0)
#define ENC_ADD(k, v) ((void)0)
#endif

namespace {

constexpr int kTcRows = 128;          // keys per tile = MMA M = TMEM lanes
constexpr int kTcThreads = 288;       // warps 0-7: workers (argmin + operands), 8: issuer
constexpr int kWorkers = 256;
constexpr int kTcSmemLimit = 232448;  // 227 KiB opt-in per CTA
constexpr int kCbRing = 6;            // codebook steps in flight
constexpr int kBarArgmin = 1, kBarArgminLo = 2;
constexpr int kErrEncodeWait = 121;

__device__ __forceinline__ uint32_t tf32_rna(float x) {
  uint32_t y;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Operand rows of KW tf32 words: 16 words = 64-byte rows (64B swizzle, 512-byte 8-row atoms) or
// 32 words = 128-byte rows (128B swizzle, 1024-byte atoms).  Byte offset of 16-byte chunk j of row r.
template <int KW>
__device__ __forceinline__ uint32_t op_off(int r, int j) {
  if constexpr (KW == 16) return (uint32_t)((r >> 3) * 512 + (r & 7) * 64 + ((j ^ ((r >> 1) & 3)) << 4));
  else return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((j ^ (r & 7)) << 4));
}

// shared-memory matrix descriptor, K-major, swizzled: start address, SBO = one 8-row atom,
// descriptor version 1 (bit 46), layout type 4 (64B swizzle) or 2 (128B swizzle) in bits 61-63
template <int KW>
__device__ __forceinline__ uint64_t op_desc(uint32_t addr) {
  constexpr uint64_t atom = KW == 16 ? 512 : 1024;
  constexpr uint64_t layout = KW == 16 ? 4 : 2;
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((atom >> 4) << 32) | ((uint64_t)1 << 46) |
         (layout << 61);
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

#define SUNSHAPE_TCLD32(taddr, v)                                                                              \
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, " \
               "%13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "\
               "[%32];"                                                                                        \
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), \
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),      \
                 "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]),    \
                 "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]),    \
                 "=r"(v[29]), "=r"(v[30]), "=r"(v[31])                                                          \
               : "r"(taddr))

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// completes every earlier tcgen05.ld of this thread; the registers are tied so no use moves above it
template <int N>
__device__ __forceinline__ void tc_wait_ld(uint32_t (&v)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(v[i]) : : "memory");
}

__device__ __forceinline__ float min16(const uint32_t* v) {
  const float a0 = min3f(__uint_as_float(v[0]), __uint_as_float(v[1]), __uint_as_float(v[2]));
  const float a1 = min3f(__uint_as_float(v[3]), __uint_as_float(v[4]), __uint_as_float(v[5]));
  const float a2 = min3f(__uint_as_float(v[6]), __uint_as_float(v[7]), __uint_as_float(v[8]));
  const float a3 = min3f(__uint_as_float(v[9]), __uint_as_float(v[10]), __uint_as_float(v[11]));
  const float a4 = min3f(__uint_as_float(v[12]), __uint_as_float(v[13]), __uint_as_float(v[14]));
  return fminf(min3f(a0, a1, a2), min3f(a3, a4, __uint_as_float(v[15])));
}

// Bounded wait that gives up at once when the CTA has already aborted; the first timeout records
// the error and raises the CTA's abort flag.
__device__ __forceinline__ void enc_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_s) {
  if (mbar_try_wait(bar, parity)) return;
  const uint64_t t0 = global_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return;
    if (*abort_s) return;
    if (global_ns() - t0 > kWaitLimitNs) {
      record_error(err, kErrEncodeWait);
      *abort_s = 1;
      return;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace

// Launch-time plan of the tensor-core encode (host side fills it, the kernel reads it).
struct EncTcParams {
  CUtensorMap keys_map;   // [heads, tokens, D] keys, box (128 B / element size, 128 rows, 1), 128B swizzle
  EncodeParams p;
  int nstep;              // codewords per MMA step (N): C or C / 2
  int n_slabs;            // C / nstep
  int n_light;            // light (codebook) blocks
  int n_heavy;
  int tiles_per_head;
  int64_t n_tiles;
  // shared-memory carve-up (bytes from the 1024-aligned base)
  int off_keys, key_bytes, off_a, a_bytes, off_b, b_bytes, off_cb, cb_bytes, off_idx, idx_bytes, off_misc;
  int smem;
  int cb_ring;            // codebook steps in flight (<= kCbRing)
  int debug;              // trace builds: 1 = skip the argmin arithmetic, 2 = skip the operand stores
};

namespace {

template <int BD, bool F32K>
struct EncShape {
  static constexpr int KW = (F32K ? 3 * BD + 3 : 2 * BD + 3) <= 16 ? 16 : 32;   // tf32 words per operand row
  static constexpr int NCH = KW / 4;                                           // 16-byte chunks per row
  static constexpr int ROWB = KW * 4;
};

// staged key element (row r, model channel ch) in the TMA's 128B-swizzled boxes of 128 rows x 128 B
template <bool F32K>
__device__ __forceinline__ float key_at(const uint8_t* keys, int r, int ch, bool bf16) {
  if constexpr (F32K) {
    const int box = ch >> 5, w = ch & 31;
    return *reinterpret_cast<const float*>(keys + box * 16384 + r * 128 + ((((w >> 2) ^ (r & 7)) << 4) | ((w & 3) << 2)));
  } else {
    const int box = ch >> 6, w = ch & 63;
    const uint16_t h =
        *reinterpret_cast<const uint16_t*>(keys + box * 16384 + r * 128 + ((((w >> 3) ^ (r & 7)) << 4) | ((w & 7) << 1)));
    return bf16 ? __uint_as_float((uint32_t)h << 16) : __half2float(__ushort_as_half(h));
  }
}


// Operand rows of one step: the A row of key `r` (worker threads of the lower column half) and the B
// row of codeword `row` of the step's slab (one per worker thread), split into tf32 parts.
template <int BD, bool F32K>
__device__ __forceinline__ void build_a_row(uint32_t a0, int r, const uint8_t* keys, const int* perm_s, int b,
                                            bool bf16) {
  using S = EncShape<BD, F32K>;
  uint32_t w[S::KW];
#pragma unroll
  for (int d = 0; d < BD; ++d) {
    const float x = key_at<F32K>(keys, r, perm_s[b * BD + d], bf16);
    if constexpr (F32K) {
      const uint32_t xh = tf32_rna(x);
      w[d] = w[BD + d] = xh;
      w[2 * BD + d] = tf32_rna(x - __uint_as_float(xh));
    } else {
      w[d] = w[BD + d] = __float_as_uint(x);
    }
  }
  constexpr int k1 = F32K ? 3 * BD : 2 * BD;
#pragma unroll
  for (int k = k1; k < S::KW; ++k) w[k] = k < k1 + 3 ? __float_as_uint(1.0f) : 0u;
#pragma unroll
  for (int j = 0; j < S::NCH; ++j) sts128(a0 + op_off<S::KW>(r, j), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

template <int BD, bool F32K>
__device__ __forceinline__ void build_b_row(uint32_t b0, int row, const float* cbrow) {
  using S = EncShape<BD, F32K>;
  float cw[BD];
  if constexpr (BD >= 4) {
#pragma unroll
    for (int d4 = 0; d4 < BD; d4 += 4) {
      const float4 v = *reinterpret_cast<const float4*>(cbrow + row * BD + d4);
      cw[d4] = v.x; cw[d4 + 1] = v.y; cw[d4 + 2] = v.z; cw[d4 + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int d = 0; d < BD; ++d) cw[d] = cbrow[row * BD + d];
  }
  uint32_t w[S::KW];
  float n2 = 0.f;
#pragma unroll
  for (int d = 0; d < BD; ++d) {
    n2 = fmaf(cw[d], cw[d], n2);
    const float bv = -2.f * cw[d];
    const uint32_t hi = tf32_rna(bv);
    w[d] = hi;
    w[BD + d] = tf32_rna(bv - __uint_as_float(hi));
    if constexpr (F32K) w[2 * BD + d] = hi;
  }
  constexpr int k1 = F32K ? 3 * BD : 2 * BD;
  const uint32_t nh = tf32_rna(n2);
  const float r1 = n2 - __uint_as_float(nh);
  const uint32_t nm = tf32_rna(r1);
  w[k1] = nh;
  w[k1 + 1] = nm;
  w[k1 + 2] = tf32_rna(r1 - __uint_as_float(nm));
#pragma unroll
  for (int k = k1 + 3; k < S::KW; ++k) w[k] = 0u;
#pragma unroll
  for (int j = 0; j < S::NCH; ++j) sts128(b0 + op_off<S::KW>(row, j), w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
}

// Walks this CTA's steps in order: tile (local index ti), light block li, codeword slab h.
struct StepCursor {
  int64_t ti = 0;
  int li = 0, h = 0;
  int64_t hh = 0;   // head of tile ti
  int row0 = 0;     // first key row of tile ti
  int cbh = 0;      // codebook of that head
  __device__ void load_tile(const EncTcParams& P) {
    const int64_t tg = blockIdx.x + ti * gridDim.x;
    hh = tg / P.tiles_per_head;
    row0 = (int)(tg - hh * P.tiles_per_head) * kTcRows;
    cbh = P.p.n_cb == 1 ? 0 : (int)((hh % P.p.kv_heads) % P.p.n_cb);
  }
  __device__ bool last_of_tile(const EncTcParams& P) const { return li == P.n_light - 1 && h == P.n_slabs - 1; }
  __device__ bool first_of_tile() const { return li == 0 && h == 0; }
  __device__ void advance(const EncTcParams& P, int64_t my_tiles) {
    if (++h == P.n_slabs) {
      h = 0;
      if (++li == P.n_light) {
        li = 0;
        if (++ti < my_tiles) load_tile(P);
      }
    }
  }
};

template <int BD, bool F32K, int N>
__global__ void __launch_bounds__(kTcThreads, 1) encode_tc_kernel(const __grid_constant__ EncTcParams P) {
  using S = EncShape<BD, F32K>;
  constexpr int CW = N / 2;   // columns per worker warp
  const EncodeParams& p = P.p;
  extern __shared__ uint8_t tc_smem_raw[];
  const uint32_t raw = smem_u32(tc_smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* sm = tc_smem_raw + (base - raw);
  uint8_t* keys_s = sm + P.off_keys;
  const uint32_t sA = base + P.off_a, sB = base + P.off_b;
  float* cb_s = reinterpret_cast<float*>(sm + P.off_cb);
  uint8_t* idx_s = sm + P.off_idx;
  uint8_t* misc = sm + P.off_misc;
  uint64_t* keybar = reinterpret_cast<uint64_t*>(misc);          // [2] key tile landed
  uint64_t* mma_bar = keybar + 2;                                // [2] MMA of the step done
  uint64_t* tmem_empty = keybar + 4;                             // [2] workers done with the accumulator
  uint64_t* ops_full = keybar + 6;                               // [2] workers done writing the operands
  uint64_t* cb_full = keybar + 12;                               // [kCbRing] codebook rows landed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(keybar + 12 + kCbRing);
  volatile int* abort_s = reinterpret_cast<volatile int*>(tslot + 1);
  int* perm_s = reinterpret_cast<int*>(tslot + 4);               // [D]
  int8_t* light_s = reinterpret_cast<int8_t*>(perm_s + p.D);     // [n_light] light block ids
  int8_t* heavy_s = light_s + 64;                                // [n_heavy] heavy block ids
  float2* xchg = reinterpret_cast<float2*>(misc + 2048);         // [2][128] (min, index) of the upper half

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = p.nb;
  int* err = p.err ? p.err : &g_encode_error;
  const int64_t my_tiles = P.n_tiles > blockIdx.x ? (P.n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int64_t G = my_tiles * P.n_light * P.n_slabs;    // steps of this CTA
  constexpr int kTmemCols = 2 * N <= 256 ? 256 : 512;
  constexpr int kCbStepFloats = N * BD;

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&keybar[i], 1);
      mbar_init(&mma_bar[i], 1);
      mbar_init(&tmem_empty[i], 8);
      mbar_init(&ops_full[i], 8);
    }
    for (int i = 0; i < kCbRing; ++i) mbar_init(&cb_full[i], 1);
    *abort_s = 0;
    int nl = 0, nh = 0;
    for (int b = 0; b < nb; ++b) {
      if (p.heavy_mask != nullptr && p.heavy_mask[b] != 0) heavy_s[nh++] = (int8_t)b;
      else light_s[nl++] = (int8_t)b;
    }
    fence_mbar_init();
  }
  for (int i = tid; i < p.D; i += kTcThreads) perm_s[i] = (int)p.perm[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tslot);
  const bool bf16 = p.keys_dtype == SUNSHAPE_BF16;
  constexpr int kEs = F32K ? 4 : 2, kPerBox = 128 / kEs;

  if (warp == 8) {
    // ---------------------------------------------------------------- issuer: TMA copies and MMAs
    if (lane == 0 && G > 0) {
      auto load_keys = [&](int64_t ti, int slot) {
        StepCursor t;
        t.ti = ti;
        t.load_tile(P);
        mbar_arrive_expect_tx(&keybar[slot], (uint32_t)P.key_bytes);
        for (int x = 0; x < p.D; x += kPerBox)
          tma_load_3d(keys_s + slot * P.key_bytes + (x / kPerBox) * 16384, &P.keys_map, x, t.row0, (int)t.hh,
                      &keybar[slot]);
      };
      auto load_cb = [&](const StepCursor& c, int64_t g) {
        const int slot = (int)(g % P.cb_ring);
        mbar_arrive_expect_tx(&cb_full[slot], (uint32_t)(kCbStepFloats * 4));
        bulk_g2s(cb_s + slot * kCbStepFloats,
                 p.cb + (((int64_t)c.cbh * nb + light_s[c.li]) * p.C + (int64_t)c.h * N) * BD,
                 (uint32_t)(kCbStepFloats * 4), &cb_full[slot]);
      };
      for (int64_t ti = 0; ti < 2 && ti < my_tiles; ++ti) load_keys(ti, (int)ti);
      StepCursor pc;                 // codebook prefetch cursor, kCbRing steps ahead of the MMAs
      pc.load_tile(P);
      int64_t gp = 0;
      for (; gp < P.cb_ring && gp < G; ++gp) {
        load_cb(pc, gp);
        pc.advance(P, my_tiles);
      }
      StepCursor c;
      c.load_tile(P);
      constexpr uint32_t id = idesc_tf32(N);
      for (int64_t g = 0; g < G; ++g) {
        const int buf = (int)(g & 1);
        enc_wait(&ops_full[buf], (uint32_t)((g >> 1) & 1), err, abort_s);   // operands of step g written
        // the workers are done with this step's codebook rows and, after its last step, with the tile's keys
        if (gp < G) {
          load_cb(pc, gp);
          pc.advance(P, my_tiles);
          ++gp;
        }
        if (c.last_of_tile(P) && c.ti + 2 < my_tiles) load_keys(c.ti + 2, (int)(c.ti & 1));
        if (g >= 2) enc_wait(&tmem_empty[buf], (uint32_t)(((g - 2) >> 1) & 1), err, abort_s);
        tc_fence_after();
        const uint64_t ad = op_desc<S::KW>(sA + buf * P.a_bytes), bdsc = op_desc<S::KW>(sB + buf * P.b_bytes);
#pragma unroll
        for (int k = 0; k < S::KW / 8; ++k)   // K = 8 tf32 = 32 bytes per MMA: advance 2 descriptor units
          tc_mma_tf32(tmem + (uint32_t)(buf * N), ad + 2 * k, bdsc + 2 * k, id, k > 0);
        tc_commit(&mma_bar[buf]);
        c.advance(P, my_tiles);
      }
    }
  } else {
    // ---------------------------------------------------------------- workers
    // warp w: TMEM lanes 32 (w % 4) .. +31 (its keys) over the column half qt = w / 4, then a share of
    // the operands of the step two ahead: A row t (half 0), B row(s) tid (+ 256), heavy copies (half 1)
    const int t = tid & 127;
    const int qt = warp >> 2;
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    // builds the operands of step gb (cursor bc) into buffer gb & 1 and signals the issuer
    auto build = [&](int64_t gb, const StepCursor& bc) {
      const int bbuf = (int)(gb & 1);
      const uint8_t* keys = keys_s + (bc.ti & 1) * P.key_bytes;
      if (bc.first_of_tile()) {
        ENC_T0(tk);
        enc_wait(&keybar[bc.ti & 1], (uint32_t)((bc.ti >> 1) & 1), err, abort_s);
        if (tid == 0) ENC_ADD(2, tk);
        // SunShape-Mixed: heavy blocks of this key are stored densely (index 0 is set with the argmin)
        if (qt == 1 && P.n_heavy > 0 && bc.row0 + t < p.n_tokens) {
          for (int s = 0; s < P.n_heavy; ++s) {
            const int hb = heavy_s[s];
            const int64_t o = ((bc.hh * p.out_hs + bc.row0 + t) * P.n_heavy + s) * BD;
#pragma unroll
            for (int d = 0; d < BD; ++d)
              store_from_float(p.heavy_out, o + d, p.heavy_dtype, key_at<F32K>(keys, t, perm_s[hb * BD + d], bf16));
          }
        }
      }
#ifdef SUNSHAPE_TRACE
      const bool skip_ops = P.debug & 2;
#else
      constexpr bool skip_ops = false;
#endif
      ENC_T0(ta);
      if (qt == 0 && !skip_ops) build_a_row<BD, F32K>(sA + bbuf * P.a_bytes, t, keys, perm_s, light_s[bc.li], bf16);
      if (tid == 0) ENC_ADD(10, ta);
      {
        ENC_T0(tc);
        enc_wait(&cb_full[gb % P.cb_ring], (uint32_t)((gb / P.cb_ring) & 1), err, abort_s);
        if (tid == 0) ENC_ADD(3, tc);
      }
      ENC_T0(tbb);
      if (!skip_ops)
        for (int row = tid; row < N; row += kWorkers)
          build_b_row<BD, F32K>(sB + bbuf * P.b_bytes, row, cb_s + (gb % P.cb_ring) * kCbStepFloats);
      if (tid == 0) ENC_ADD(11, tbb);
      ENC_T0(tf);
      fence_proxy_async_smem();   // generic-proxy operand writes -> tensor core (async proxy)
      if (tid == 0) ENC_ADD(12, tf);
      __syncwarp();
      if (lane == 0) mbar_arrive(&ops_full[bbuf]);
    };
    StepCursor c, bc;
    c.load_tile(P);
    bc.load_tile(P);
    for (int64_t gb = 0; gb < 2 && gb < G; ++gb) {   // operands of the first two steps
      build(gb, bc);
      bc.advance(P, my_tiles);
    }
    float best = 0.f;
    int besti = 0;
    // half 0: merge step gs's two half minima (the first minimum wins ties), fold the slab into the
    // block's running minimum and, after a tile's last step, write the tile's indices out
    auto combine = [&](int64_t gs, const StepCursor& cs, float mm, int cc) {
      {
        const float2 o = xchg[(gs & 1) * 128 + t];
        if (o.x < mm) { mm = o.x; cc = __float_as_int(o.y); }
      }
      uint8_t* sidx = idx_s + (cs.ti & 1) * P.idx_bytes;
      if (cs.h == 0 || mm < best) { best = mm; besti = cc; }
      if (cs.h == P.n_slabs - 1) sidx[t * nb + light_s[cs.li]] = (uint8_t)besti;
      if (cs.last_of_tile(P)) {
        // tile complete: its indices leave as one contiguous run of nrows * nb entries
        named_barrier(kBarArgminLo, 128);
        const int nrows = min(kTcRows, p.n_tokens - cs.row0);
        const int64_t o0 = (cs.hh * p.out_hs + cs.row0) * nb;
        for (int e = t; e < nrows * nb; e += 128) {
          const int vv = sidx[e];
          if (p.index_dtype == SUNSHAPE_U8) reinterpret_cast<uint8_t*>(p.idx_out)[o0 + e] = (uint8_t)vv;
          else if (p.index_dtype == SUNSHAPE_I16) reinterpret_cast<int16_t*>(p.idx_out)[o0 + e] = (int16_t)vv;
          else reinterpret_cast<int32_t*>(p.idx_out)[o0 + e] = vv;
        }
      }
    };
    ENC_T0(ta0);
    for (int64_t g = 0; g < G; ++g) {
      const int buf = (int)(g & 1);
      uint8_t* tidx = idx_s + (c.ti & 1) * P.idx_bytes;
      if (qt == 0 && c.first_of_tile())
        for (int s = 0; s < P.n_heavy; ++s) tidx[t * nb + heavy_s[s]] = 0;
      {
        ENC_T0(tw);
        enc_wait(&mma_bar[buf], (uint32_t)((g >> 1) & 1), err, abort_s);
        if (tid == 0) ENC_ADD(6, tw);
      }
      tc_fence_after();
      // first minimum over this warp's N/4 columns, loaded with one wait.  tcgen05.ld addresses are
      // warp-uniform, so the winning group cannot be re-read per lane: each group of 16 is reduced with
      // 3-input min, and a group that lowers the running minimum is kept in registers (selects) for the
      // first-index search.
      const uint32_t col0 = lane_base + (uint32_t)(buf * N + qt * CW);
      ENC_T0(tl);
      uint32_t v[CW];
      if constexpr (CW >= 32) {
#pragma unroll
        for (int q = 0; q < CW; q += 32) SUNSHAPE_TCLD32(col0 + (uint32_t)q, (v + q));
      } else {
        tc_ld16(col0, *reinterpret_cast<uint32_t(*)[16]>(v));
      }
      tc_wait_ld(v);
      if (tid == 0) ENC_ADD(7, tl);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tmem_empty[buf]);   // the accumulator is in registers: MMA g+2 may start
#ifdef SUNSHAPE_TRACE
      if (P.debug & 1) {
        const int ci = (int)v[0] & 255;
        if (qt == 0) tidx[t * nb + light_s[c.li]] = (uint8_t)ci;
        if (g + 2 < G) { build(g + 2, bc); bc.advance(P, my_tiles); }
        c.advance(P, my_tiles);
        continue;
      }
#endif
      // tcgen05.ld addresses are warp-uniform, so the winning group cannot be re-read per lane: each group
      // of 16 is reduced with 3-input min, and a group that lowers the running minimum is kept in
      // registers (selects) for the first-index search.
      float m = __int_as_float(0x7f800000);
      int mg = 0;
      uint32_t bv[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) bv[k] = 0x7f800000u;
#pragma unroll
      for (int i = 0; i < CW / 16; ++i) {
        const float gm = min16(v + 16 * i);
        const bool lower = gm < m;
        m = lower ? gm : m;
        mg = lower ? i : mg;
#pragma unroll
        for (int k = 0; k < 16; ++k) bv[k] = lower ? v[16 * i + k] : bv[k];
      }
      int j = 0;
#pragma unroll
      for (int k = 15; k >= 0; --k)
        if (__uint_as_float(bv[k]) == m) j = k;
      const int ci = c.h * N + qt * CW + mg * 16 + j;
      // the lower half keeps the first minimum: the upper half's only if strictly smaller
      if (qt == 1) xchg[(g & 1) * 128 + t] = make_float2(m, __int_as_float(ci));
      named_barrier(kBarArgmin, kWorkers);
      if (qt == 0) combine(g, c, m, ci);
      // MMA g is done, so its operand buffer takes step g + 2
      if (g + 2 < G) {
        ENC_T0(tbld);
        build(g + 2, bc);
        if (tid == 0) ENC_ADD(9, tbld);
        bc.advance(P, my_tiles);
      }
      c.advance(P, my_tiles);
    }
    if (tid == 0) ENC_ADD(5, ta0);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 enc_tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q{};
    void* f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }
  return fn;
}

int round_up_i(int x, int a) { return (x + a - 1) / a * a; }

// Shared-memory plan for codeword slabs of n columns; false if it does not fit.
bool plan_tc(EncTcParams& P, int n) {
  const EncodeParams& p = P.p;
  const bool f32k = p.keys_dtype == SUNSHAPE_F32;
  const int kw = (f32k ? 3 * p.bd + 3 : 2 * p.bd + 3) <= 16 ? 16 : 32;
  P.nstep = n;
  P.n_slabs = p.C / n;
  P.key_bytes = kTcRows * p.D * (f32k ? 4 : 2);
  P.a_bytes = kTcRows * kw * 4;
  P.b_bytes = n * kw * 4;
  P.cb_ring = kCbRing;
  P.cb_bytes = kCbRing * n * p.bd * 4;
  P.idx_bytes = round_up_i(kTcRows * p.nb, 16);
  P.off_keys = 0;
  P.off_a = P.off_keys + 2 * P.key_bytes;
  P.off_b = P.off_a + 2 * P.a_bytes;
  P.off_cb = P.off_b + 2 * P.b_bytes;
  P.off_idx = P.off_cb + P.cb_bytes;
  P.off_misc = round_up_i(P.off_idx + 2 * P.idx_bytes, 16);
  const int misc = 2048 + 2 * 128 * 8;   // barriers, tmem slot, permutation, block lists | exchange
  P.smem = P.off_misc + misc + 1024;   // + alignment slack for the 1024-byte operand atoms
  // a shallower codebook ring when the rest does not leave room for six steps
  while (P.smem > kTcSmemLimit && P.cb_ring > 3) {
    const int save = n * p.bd * 4;
    --P.cb_ring;
    P.cb_bytes -= save;
    P.off_idx -= save;
    P.off_misc -= save;
    P.smem -= save;
  }
  return P.smem <= kTcSmemLimit;
}

}  // namespace

// The tensor-core encode takes fp32 or 16-bit keys whose rows and head strides are 16-byte multiples
// (TMA), block_dim 2, 4 or 8, n_centroids 64, 128 or 256, at least one codebook block,
// and head_dim a multiple of the 128-byte TMA box; everything else uses encode_kernel.
bool encode_tc_supported(const EncodeParams& p) {
  const int es = p.keys_dtype == SUNSHAPE_F32 ? 4 : 2;
  if (!(p.keys_dtype == SUNSHAPE_F32 || p.keys_dtype == SUNSHAPE_BF16 || p.keys_dtype == SUNSHAPE_F16)) return false;
  if (!(p.bd == 2 || p.bd == 4 || p.bd == 8) || !(p.C == 64 || p.C == 128 || p.C == 256)) return false;
  if (p.nb > 64) return false;
  if ((p.D * es) % 128 != 0 || p.D > 256) return false;
  if ((reinterpret_cast<uintptr_t>(p.keys) & 15) || (p.key_ts * es) % 16 || (p.key_hs * es) % 16) return false;
  if (p.key_ts < p.D) return false;
  if ((reinterpret_cast<uintptr_t>(p.cb) & 15)) return false;
  EncTcParams P{};
  P.p = p;
  return plan_tc(P, p.C) || (p.C % 128 == 0 && plan_tc(P, p.C / 2));
}

int launch_encode_tc(const EncodeParams& p, int n_heads, int n_heavy, cudaStream_t st) {
  EncTcParams P{};
  P.p = p;
  if (!plan_tc(P, p.C) && !(p.C % 128 == 0 && plan_tc(P, p.C / 2))) return -1;
  P.n_heavy = n_heavy;
  P.n_light = p.nb - n_heavy;
#ifdef SUNSHAPE_TRACE
  if (const char* dbg = getenv("SUNSHAPE_ENC_DEBUG")) P.debug = atoi(dbg);
#endif
  if (P.n_light <= 0 || P.n_light > 64 || n_heavy > 64) return -1;
  P.tiles_per_head = (p.n_tokens + kTcRows - 1) / kTcRows;
  P.n_tiles = (int64_t)n_heads * P.tiles_per_head;
  const bool f32k = p.keys_dtype == SUNSHAPE_F32;
  const int es = f32k ? 4 : 2;
  auto enc = enc_tensor_map_encoder();
  if (!enc) return -1;
  const cuuint64_t dims[3] = {(cuuint64_t)p.D, (cuuint64_t)p.n_tokens, (cuuint64_t)n_heads};
  const cuuint64_t strides[2] = {(cuuint64_t)(p.key_ts * es),
                                 (cuuint64_t)(n_heads > 1 ? p.key_hs * es : (int64_t)p.n_tokens * p.key_ts * es)};
  const cuuint32_t box[3] = {(cuuint32_t)(128 / es), (cuuint32_t)kTcRows, 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = f32k ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                      : (p.keys_dtype == SUNSHAPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  if (enc(&P.keys_map, dt, 3, const_cast<void*>(p.keys), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return -1;
  int dev = 0, n_sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned grid = (unsigned)std::min<int64_t>(P.n_tiles, n_sms);
  // more than half an SM's shared memory keeps one CTA per SM, so the 256/512-column TMEM allocation
  // never waits for another CTA
  const int smem = std::max(P.smem, 120 * 1024);
#define SUNSHAPE_TC_CASE(BDV, F32V, NV)                                                         \
  {                                                                                            \
    auto k = encode_tc_kernel<BDV, F32V, NV>;                                                  \
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);                \
    k<<<grid, kTcThreads, smem, st>>>(P);                                                      \
  }
#define SUNSHAPE_TC_N(BDV, F32V)                                                                \
  {                                                                                            \
    if (P.nstep == 256) SUNSHAPE_TC_CASE(BDV, F32V, 256)                                       \
    else if (P.nstep == 128) SUNSHAPE_TC_CASE(BDV, F32V, 128)                                  \
    else SUNSHAPE_TC_CASE(BDV, F32V, 64)                                                       \
  }
  if (f32k) {
    if (p.bd == 2) SUNSHAPE_TC_N(2, true) else if (p.bd == 4) SUNSHAPE_TC_N(4, true) else SUNSHAPE_TC_N(8, true)
  } else {
    if (p.bd == 2) SUNSHAPE_TC_N(2, false) else if (p.bd == 4) SUNSHAPE_TC_N(4, false) else SUNSHAPE_TC_N(8, false)
  }
#undef SUNSHAPE_TC_N
#undef SUNSHAPE_TC_CASE
  return 0;
}

#ifdef SUNSHAPE_TRACE
extern "C" int sunshape_debug_encode_trace(unsigned long long* out, int clear) {
  cudaMemcpyFromSymbol(out, g_enc_trace, sizeof(g_enc_trace));
  if (clear) {
    unsigned long long z[16] = {};
    cudaMemcpyToSymbol(g_enc_trace, z, sizeof(z));
  }
  return 0;
}
#endif

int encode_error_word(int* code, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(code, g_encode_error, sizeof(int), 0, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && clear && *code != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_encode_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice);
  }
  return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace sunshape
