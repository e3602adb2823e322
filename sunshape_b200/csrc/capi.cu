// extern "C" boundary of libsunshape_b200.so: argument validation with
// reference-style reason strings, template dispatch and launch configuration.
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <string>

#include <cudaTypedefs.h>

#include "decode.cuh"
#include "decode_mma.cuh"
#include "encode.cuh"

namespace sunshape {
// Cross-shard merge of (m, l, acc) partial sets: one CTA per row.
__global__ void merge_partials_kernel(const float* __restrict__ parts, int n_parts, int64_t rows, int dv,
                                      void* out, int out_dtype) {
  const int64_t r = blockIdx.x;
  const float NEG_INF = -__int_as_float(0x7f800000);
  for (int d = threadIdx.x; d < dv; d += blockDim.x) {
    float M = NEG_INF;
    for (int k = 0; k < n_parts; ++k) M = fmaxf(M, parts[(k * rows + r) * (dv + 2)]);
    float Lsum = 0.f, A = 0.f;
    if (M != NEG_INF) {
      for (int k = 0; k < n_parts; ++k) {
        const float* src = parts + (k * rows + r) * (dv + 2);
        if (src[0] == NEG_INF) continue;
        const float sc = expf(src[0] - M);
        Lsum = fmaf(src[1], sc, Lsum);
        A = fmaf(src[2 + d], sc, A);
      }
    }
    store_from_float(out, r * dv + d, out_dtype, M == NEG_INF ? __int_as_float(0x7fc00000) : A / Lsum);
  }
}

// Peer exchange buffer layout (bytes): [recv: 2 x world x rows x (DV + 2) fp32 | arrive: 2 x n_heads
// u32 | step u32, done u32], each part 256-byte aligned.
struct PeerLayout { int64_t recv, arrive, step, total; };
inline PeerLayout peer_layout(int world, int64_t rows, int dv, int n_heads) {
  PeerLayout l;
  l.recv = 0;
  l.arrive = ((int64_t)2 * world * rows * (dv + 2) * 4 + 255) / 256 * 256;
  l.step = l.arrive + ((int64_t)2 * n_heads * 4 + 255) / 256 * 256;
  l.total = l.step + 256;
  return l;
}

// Cross-GPU merge: one CTA per KV head waits (bounded) until every rank's rows of the head have
// arrived in this rank's exchange buffer, merges them in rank order and writes the output; the
// last CTA advances the step counter (its parity selects the buffer half of the next call).
// A wait that gives up (error 104) leaves the arrival counts out of step with the peers: a slow
// rank's late arrivals would land in a half that is reused two calls later and be merged as if
// current.  So a timeout also sets a sticky poison word (step + 2); while it is set every later
// call records error 106 and writes NaN rows instead of merging, until the exchange buffers are
// freed and allocated again (a new peer group).
__global__ void xmerge_kernel(float* recv, unsigned int* arrive, unsigned int* step, unsigned int* done, int world,
                              int64_t rows, int R, int dv, int n_heads, void* out, int out_dtype, int* err) {
  __shared__ unsigned parity_s;
  const int64_t hh = blockIdx.x;
  const float NEG_INF = -__int_as_float(0x7f800000);
  __shared__ int bad_s;
  volatile unsigned int* poison = step + 2;
  if (threadIdx.x == 0) {
    const unsigned parity = *reinterpret_cast<volatile unsigned int*>(step) & 1u;
    parity_s = parity;
    bad_s = 0;
    if (*poison != 0u) {
      record_error(err, 106);
      bad_s = 1;
    } else {
      unsigned int* a = arrive + (int64_t)parity * n_heads + hh;
      const uint64_t t0 = global_ns();
      while (true) {
        unsigned int v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
        if ((int)v >= world) break;
        if (global_ns() - t0 > kWaitLimitNs) {
          record_error(err, 104);
          *poison = 1u;
          __threadfence();
          bad_s = 1;
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  const unsigned parity = parity_s;
  const bool bad = bad_s != 0;
  for (int e = threadIdx.x; e < R * dv; e += blockDim.x) {
    const int r = e / dv, d = e - r * dv;
    const int64_t orow = hh * R + r;
    float M = NEG_INF;
    for (int k = 0; k < world; ++k)
      M = fmaxf(M, __ldcv(recv + ((int64_t)(parity * world + k) * rows + orow) * (dv + 2)));
    float Lsum = 0.f, A = 0.f;
    if (M != NEG_INF) {
      for (int k = 0; k < world; ++k) {
        const float* src = recv + ((int64_t)(parity * world + k) * rows + orow) * (dv + 2);
        const float sc = fast_exp2((__ldcv(src) - M) * kLog2e);
        Lsum = fmaf(__ldcv(src + 1), sc, Lsum);
        A = fmaf(__ldcv(src + 2 + d), sc, A);
      }
    }
    store_from_float(out, orow * dv + d, out_dtype, (bad || M == NEG_INF) ? __int_as_float(0x7fc00000) : A / Lsum);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    arrive[(int64_t)parity * n_heads + hh] = 0u;   // reused two calls later
    __threadfence();
    if (atomicAdd(done, 1u) == (unsigned)gridDim.x - 1) {
      *done = 0u;
      __threadfence();
      atomicAdd(step, 1u);
    }
  }
}

}  // namespace sunshape

using namespace sunshape;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SUNSHAPE_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return SUNSHAPE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int dtype_size(int dt) {
  switch (dt) {
    case SUNSHAPE_F32: case SUNSHAPE_I32: return 4;
    case SUNSHAPE_BF16: case SUNSHAPE_F16: case SUNSHAPE_I16: return 2;
    case SUNSHAPE_U8: return 1;
    default: return 0;
  }
}

bool is_float_dtype(int dt) { return dt == SUNSHAPE_F32 || dt == SUNSHAPE_BF16 || dt == SUNSHAPE_F16; }

int check_codec(const sunshape_codec_t* c) {
  if (!c) return fail(SUNSHAPE_E_INVALID, "codec descriptor is NULL.");
  if (!c->centroids || !c->permutation) return fail(SUNSHAPE_E_INVALID, "codec centroids / permutation pointer is NULL.");
  if (c->block_dim <= 0 || c->head_dim <= 0 || c->head_dim % c->block_dim != 0)
    return fail(SUNSHAPE_E_INVALID, "head_dim must be divisible by block_dim");
  if (c->n_centroids <= 0) return fail(SUNSHAPE_E_INVALID, "n_centroids must be positive.");
  if (c->n_cb <= 0) return fail(SUNSHAPE_E_INVALID, "n_cb (number of codebooks) must be positive.");
  if (c->head_dim > 256) return fail(SUNSHAPE_E_UNSUPPORTED, "head_dim > 256 is not supported by the B200 kernels.");
  if (c->n_heavy < 0 || c->n_heavy > c->head_dim / c->block_dim || (c->n_heavy > 0 && !c->heavy_mask))
    return fail(SUNSHAPE_E_INVALID, "n_heavy must count the nonzero heavy_mask entries.");
  return SUNSHAPE_OK;
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int round_up(int x, int a) { return (x + a - 1) / a * a; }

struct DecodePlan {
  bool lut16 = false;   // tensor-core kernel: fp16 (scaled) LUT entries
  int gp = 0;           // padded rows per launch (4, 8 or 16)
  int chunk_rows = 0;   // rows per launch
  int stages = 0;
  int smem = 0;
  DecodeParams prm{};
  int64_t grid = 0;
  int64_t ws_bytes = 0;
};

int pick_gp(int rows) { return rows <= 4 ? 4 : (rows <= 8 ? 8 : 16); }

// Lay out shared memory and the split for one launch configuration.
// Returns false if it cannot fit.

// Virtual tiles charged per head boundary by the CTA partition (see tile_start in decode.cuh):
// SUNSHAPE_SEG_GAP overrides the default, capped at one head's tiles.
constexpr int kSegGapDefault = 16;   // measured on B200: c5 at T 16384 79.3 -> 76.2 us, T 131072 370.0 -> 368.5 us
int seg_gap_tiles(int64_t tph) {
  static const int env = [] {
    const char* e = std::getenv("SUNSHAPE_SEG_GAP");
    return e ? std::max(0, std::atoi(e)) : -1;
  }();
  return (int)std::min<int64_t>(env >= 0 ? env : kSegGapDefault, tph);
}
// Most heads one CTA's range can touch under that partition (sizes the per-CTA partial slots).
int64_t max_segments(int64_t n_heads, int64_t tph, int64_t grid) {
  const int64_t v = n_heads * tph + (n_heads - 1) * seg_gap_tiles(tph);
  const int64_t per_cta = (v + grid - 1) / grid;   // real tiles of one CTA are at most its virtual span
  return (per_cta + tph - 1) / tph + 1;
}

bool plan_decode(DecodePlan& pl, int nb, int C, int D, int dv, int vsize, int n_heavy_max, int bd,
                 int hsize, bool scores_only, int n_heads, int T, int rows, std::string& why) {
  int gp = pick_gp(rows);
  const int nbh = (nb + 7) / 8;
  if (nbh > 4) {
    why = "n_blocks > 32 is not supported by the fused LUT kernel (LUT would not fit in shared memory).";
    return false;
  }
  for (;;) {
    const int lut_bytes = nbh * 8 * C * gp * 4;
    // staging for the warp partials + the contributing-slot table of the cross-CTA merge
    const int stg_bytes = scores_only ? 0 : kWarps * gp * (dv + 2) * 4 + (kWarps + 2) * gp * 4 + 16 + 8 * num_sms();
    const int region = round_up(std::max(lut_bytes, stg_bytes), 128);
    const int off_perm = 256;
    const int off_hslot = off_perm + round_up(D * 4, 16);
    const int off_q = round_up(off_hslot + 64, 16);
    const int off_p = round_up(off_q + gp * D * 4, 16);
    const int off_lut = round_up(off_p + kWarps * (kWarpTokens + 1) * gp * 4, 128);
    const int off_stage = off_lut + region;
    const int vpart = scores_only ? 0 : round_up(kTileTokens * dv * vsize, 128);
    const int ipart = round_up(kTileTokens * nb + 32, 128);
    const int hpart = n_heavy_max > 0 ? round_up(kTileTokens * n_heavy_max * bd * hsize + 32, 128) : 0;
    const int stage_bytes = vpart + ipart + hpart;
    // multiple of the consumer tile groups: each stage is drained by one group in tile order
    const int stages = std::min(kMaxStages, (kSmemLimit - off_stage) / stage_bytes) / kTileGroups * kTileGroups;
    const bool regs_ok = scores_only || gp * (dv / 32) <= 64;
    if (stages >= kTileGroups && regs_ok) {
      pl.gp = gp;
      pl.chunk_rows = std::min(rows, gp);
      pl.stages = stages;
      pl.smem = off_stage + stages * stage_bytes;
      DecodeParams& p = pl.prm;
      p.stages = stages;
      p.stage_bytes = stage_bytes;
      p.off_stage_idx = vpart;
      p.off_stage_heavy = vpart + ipart;
      p.off_perm = off_perm;
      p.off_hslot = off_hslot;
      p.off_q = off_q;
      p.off_p = off_p;
      p.off_lut = off_lut;
      p.off_stage = off_stage;
      p.merge_smem_bytes = region;
      const int tph = (T + kTileTokens - 1) / kTileTokens;
      const int64_t total = (int64_t)n_heads * tph;
      pl.grid = std::min<int64_t>(num_sms(), total);
      p.tph = tph;
      p.total_tiles = total;
      p.seg_gap = seg_gap_tiles(tph);
      p.max_seg = (int)max_segments(n_heads, tph, pl.grid);
      const int64_t slots = pl.grid * p.max_seg * gp * (int64_t)(dv + 2) * 4;
      pl.ws_bytes = 256 + round_up(n_heads * 4, 256) + slots;
      return true;
    }
    if (gp == 4) break;
    gp /= 2;
  }
  why = "decode configuration does not fit in shared memory / registers (n_blocks, n_centroids, rows).";
  return false;
}

// Workspace of the decode kernels: [error word | per-head tickets |
// per-CTA partial slots | per-head LUTs | per-head LUT scales]; the LUT area is empty when the
// LUTs are built inside each CTA instead.
struct MmaWsOffsets { int64_t counters, slots, luts, scales, total; };
constexpr int64_t kGlobalLutMaxBytes = 48ll << 20;   // per-head LUTs (built by lut_kernel) kept in the workspace up to 48 MiB
MmaWsOffsets mma_workspace_offsets(int64_t n_heads, int64_t grid, int64_t max_seg, int64_t gp, int64_t dv,
                                   int64_t lut_bytes) {
  MmaWsOffsets o;
  o.counters = 256;
  o.slots = o.counters + (n_heads * 4 + 255) / 256 * 256;
  o.luts = o.slots + (grid * max_seg * gp * (dv + 2) * 4 + 255) / 256 * 256;
  o.scales = o.luts + n_heads * lut_bytes;
  o.total = o.scales + (n_heads * 4 + 255) / 256 * 256;
#ifdef SUNSHAPE_TRACE
  o.total += 4096 * 256;   // per-CTA trace marks
#endif
  return o;
}
int64_t mma_workspace_bytes(int64_t n_heads, int64_t grid, int64_t max_seg, int64_t gp, int64_t dv,
                            int64_t lut_bytes) {
  return mma_workspace_offsets(n_heads, grid, max_seg, gp, dv, lut_bytes).total;
}

// Shared-memory carve-up and split for the tensor-core kernel (16-bit values).
bool plan_decode_mma(DecodePlan& pl, int nb, int D, int dv, int n_heavy, int bd, int hsize, int n_heads, int T,
                     int rows, std::string& why) {
  const int nbh = (nb + 7) / 8;
  if (nbh > 8) {
    why = "n_blocks > 64 is not supported by the fused LUT kernel (LUT would not fit in shared memory).";
    return false;
  }
  if (dv != 64 && dv != 128 && dv != 256) {
    why = "value_dim must be 64, 128 or 256 for the fused decode kernel.";
    return false;
  }
  for (int gp = pick_gp(rows);; gp /= 2) {
   // fp32 LUT entries first; a half-size fp16 LUT when fp32 would leave fewer than 6 stages
   // (GP = 4 packs two block groups per 16-byte slot, so it needs an even number of groups)
   const bool l16_ok = gp >= 8 || (nbh % 2 == 0);
   for (int l16 = 0; l16 < (l16_ok ? 2 : 1); ++l16) {
    const int nt = (gp + 7) / 8;
    const int lut_bytes = nbh * 8 * kLutC * gp * (l16 ? 2 : 4);
    const int stg_bytes = kWarpsM * gp * (dv + 2) * 4 + (kWarpsM + 2) * gp * 4 + 16 + 8 * num_sms();
    const int region = round_up(std::max(lut_bytes, stg_bytes), 128);
    const int off_perm = 256;
    const int off_hslot = off_perm + round_up(D * 4, 16);
    const int off_q = round_up(off_hslot + 128, 16);
    const int off_p = round_up(off_q + gp * D * 4, 16);
    const int off_lut = round_up(off_p + kWarpsM * (nt * 512 + 64), 128);
    const int off_stage = round_up(off_lut + region, 1024);
    const int vpart = (dv / 64) * kVBoxBytes;
    const int ipart = round_up(kTileTokens * nb + 32, 128);
    const int hpart = n_heavy > 0 ? round_up(kTileTokens * n_heavy * bd * hsize + 32, 128) : 0;
    const int stage_bytes = round_up(vpart + ipart + hpart, 1024);
    // Stage count is a multiple of the consumer tile groups (and of the producer count), so
    // every stage is filled by one producer warp and drained by one tile group, both in tile
    // order: a phase-parity wait can then never match an older phase of the same stage.
    const int stages = std::min(kMaxStages, (kSmemLimit - 1024 - off_stage) / stage_bytes) / kTileGroupsM *
                       kTileGroupsM;
    const bool last = l16 == 1 || !l16_ok;
    // SUNSHAPE_LUT_FP32=1 keeps fp32 LUT entries whenever they fit at all (for precision comparisons)
    const char* f32env = std::getenv("SUNSHAPE_LUT_FP32");
    const bool force_f32 = f32env && std::atoi(f32env) != 0 && l16 == 0;
    if (stages >= 8 || ((last || force_f32) && stages >= kTileGroupsM)) {
      pl.lut16 = l16 == 1;
      pl.gp = gp;
      pl.chunk_rows = std::min(rows, gp);
      pl.stages = stages;
      pl.smem = off_stage + stages * stage_bytes + 1024;
      DecodeParams& p = pl.prm;
      p.stages = stages;
      const char* pf = std::getenv("SUNSHAPE_L2_PREFETCH");
      p.prefetch_ahead = pf ? std::max(0, std::atoi(pf)) : kPrefetchAhead;
      p.stage_bytes = stage_bytes;
      p.off_stage_idx = vpart;
      p.off_stage_heavy = vpart + ipart;
      p.off_perm = off_perm;
      p.off_hslot = off_hslot;
      p.off_q = off_q;
      p.off_p = off_p;
      p.off_lut = off_lut;
      p.off_stage = off_stage;
      const int tph = (T + kTileTokens - 1) / kTileTokens;
      const int64_t total = (int64_t)n_heads * tph;
      pl.grid = std::min<int64_t>(num_sms(), total);
      p.tph = tph;
      p.total_tiles = total;
      p.seg_gap = seg_gap_tiles(tph);
      p.max_seg = (int)max_segments(n_heads, tph, pl.grid);
      p.lut_bytes = lut_bytes;
      p.merge_smem_bytes = off_stage - off_lut;
      pl.ws_bytes = mma_workspace_bytes(n_heads, pl.grid, p.max_seg, gp, dv, 0);
      return true;
    }
   }
    if (gp == 4) break;
  }
  why = "decode configuration does not fit in shared memory (n_blocks, rows).";
  return false;
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// 2-D view [rows, dv] of the 16-bit values, boxes of 64 tokens x 64 columns, 128-byte swizzle.
int make_value_map(CUtensorMap* map, const void* v, int dtype, int dv, int64_t rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(SUNSHAPE_E_CUDA, "cuTensorMapEncodeTiled is unavailable from the CUDA driver.");
  const cuuint64_t dims[2] = {(cuuint64_t)dv, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)dv * 2};
  const cuuint32_t box[2] = {64, 64};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, dtype == SUNSHAPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(v), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SUNSHAPE_E_CUDA, "cuTensorMapEncodeTiled failed for the value tensor.");
  return SUNSHAPE_OK;
}

template <int GP, int DV, typename VT>
void run_mma(const DecodePlan& pl, cudaStream_t st) {
  DecodeLaunch l{pl.prm, pl.smem, pl.grid};
  if (pl.lut16) launch_decode_mma_t<GP, DV, VT, true>(l, st);
  else launch_decode_mma_t<GP, DV, VT, false>(l, st);
}

int launch_lut(const DecodeParams& p, int gp, bool lut16, int n_heads, cudaStream_t st) {
  const int ns = num_sms();
  switch (gp * 2 + (lut16 ? 1 : 0)) {
    case 8: launch_lut_t<4, false>(p, n_heads, ns, st); break;
    case 9: launch_lut_t<4, true>(p, n_heads, ns, st); break;
    case 16: launch_lut_t<8, false>(p, n_heads, ns, st); break;
    case 17: launch_lut_t<8, true>(p, n_heads, ns, st); break;
    case 32: launch_lut_t<16, false>(p, n_heads, ns, st); break;
    default: launch_lut_t<16, true>(p, n_heads, ns, st); break;
  }
  return SUNSHAPE_OK;
}

int launch_decode_mma(const DecodePlan& pl, int dv, int vdt, cudaStream_t st) {
#define SUNSHAPE_MMA_CASE(GPV, DVV)                                              \
  if (pl.gp == GPV && dv == DVV) {                                              \
    if (vdt == SUNSHAPE_BF16) run_mma<GPV, DVV, __nv_bfloat16>(pl, st);        \
    else run_mma<GPV, DVV, __half>(pl, st);                                     \
    return SUNSHAPE_OK;                                                          \
  }
  SUNSHAPE_MMA_CASE(4, 64) SUNSHAPE_MMA_CASE(4, 128) SUNSHAPE_MMA_CASE(4, 256)
  SUNSHAPE_MMA_CASE(8, 64) SUNSHAPE_MMA_CASE(8, 128) SUNSHAPE_MMA_CASE(8, 256)
  SUNSHAPE_MMA_CASE(16, 64) SUNSHAPE_MMA_CASE(16, 128) SUNSHAPE_MMA_CASE(16, 256)
#undef SUNSHAPE_MMA_CASE
  return fail(SUNSHAPE_E_UNSUPPORTED, "no tensor-core decode kernel for this (rows, value_dim).");
}

template <int GP, int DV, typename VT, bool SO>
void run(const DecodePlan& pl, cudaStream_t st) {
  DecodeLaunch l{pl.prm, pl.smem, pl.grid};
  launch_decode_t<GP, DV, VT, SO>(l, st);
}

template <int GP, bool SO>
int launch_decode_dv(const DecodePlan& pl, int dv, int vdt, cudaStream_t st) {
  if constexpr (SO) {
    run<GP, 64, float, true>(pl, st);
    return SUNSHAPE_OK;
  } else {
#define SUNSHAPE_DV_CASE(DVV)                                                      \
  if constexpr (GP * DVV / 32 <= 64) {                                             \
    if (dv == DVV) {                                                               \
      if (vdt == SUNSHAPE_F32) run<GP, DVV, float, false>(pl, st);                 \
      else if (vdt == SUNSHAPE_BF16) run<GP, DVV, __nv_bfloat16, false>(pl, st);   \
      else run<GP, DVV, __half, false>(pl, st);                                    \
      return SUNSHAPE_OK;                                                          \
    }                                                                              \
  }
  SUNSHAPE_DV_CASE(64)
  SUNSHAPE_DV_CASE(128)
  SUNSHAPE_DV_CASE(256)
#undef SUNSHAPE_DV_CASE
  }
  return fail(SUNSHAPE_E_UNSUPPORTED, "value_dim must be 64, 128 or 256 for the fused decode kernel.");
}

template <bool SO>
int launch_decode(const DecodePlan& pl, int dv, int vdt, cudaStream_t st) {
  switch (pl.gp) {
    case 4: return launch_decode_dv<4, SO>(pl, dv, vdt, st);
    case 8: return launch_decode_dv<8, SO>(pl, dv, vdt, st);
    default: return launch_decode_dv<16, SO>(pl, dv, vdt, st);
  }
}

int check_kv(const sunshape_kv_t* kv, const sunshape_codec_t* c, bool need_value) {
  if (!kv) return fail(SUNSHAPE_E_INVALID, "KV descriptor is NULL.");
  if (!kv->indices) return fail(SUNSHAPE_E_INVALID, "Quantized key must expose an indices buffer.");
  if (kv->seq_len < 0) return fail(SUNSHAPE_E_INVALID, "seq_len must be >= 0.");
  if (kv->head_stride < kv->seq_len) return fail(SUNSHAPE_E_INVALID, "head_stride must be >= seq_len.");
  if (need_value) {
    if (!kv->value) return fail(SUNSHAPE_E_INVALID, "value buffer is NULL.");
    if (!is_float_dtype(kv->value_dtype)) return fail(SUNSHAPE_E_INVALID, "value dtype must be F32, BF16 or F16.");
    if (!aligned16(kv->value)) return fail(SUNSHAPE_E_INVALID, "value buffer must be 16-byte aligned.");
  }
  if (!aligned16(kv->indices)) return fail(SUNSHAPE_E_INVALID, "indices buffer must be 16-byte aligned.");
  if (c->heavy_mask && kv->heavy) {
    if (kv->heavy_dtype != SUNSHAPE_BF16 && kv->heavy_dtype != SUNSHAPE_F32)
      return fail(SUNSHAPE_E_INVALID, "heavy (passthrough) dtype must be BF16 or F32.");
    if (!aligned16(kv->heavy)) return fail(SUNSHAPE_E_INVALID, "heavy buffer must be 16-byte aligned.");
  }
  return SUNSHAPE_OK;
}

}  // namespace

namespace sunshape {
// lets other translation units of the library report errors through sunshape_last_error()
int set_last_error(int code, const char* msg) { return fail(code, msg); }
}  // namespace sunshape

extern "C" {

int sunshape_abi_version(void) { return SUNSHAPE_ABI_VERSION; }

const char* sunshape_last_error(void) { return g_last_error.c_str(); }

int sunshape_encode(const sunshape_codec_t* codec, const void* keys, int32_t keys_dtype, int32_t n_heads,
                    int32_t kv_heads, int32_t n_tokens, int64_t key_head_stride, int64_t key_token_stride,
                    void* indices_out, int32_t index_dtype, void* heavy_out, int32_t heavy_dtype,
                    int64_t out_head_stride, void* stream) {
  if (int rc = check_codec(codec)) return rc;
  if (!keys || !indices_out) return fail(SUNSHAPE_E_INVALID, "keys / indices_out pointer is NULL.");
  if (!is_float_dtype(keys_dtype)) return fail(SUNSHAPE_E_INVALID, "keys dtype must be F32, BF16 or F16.");
  if (index_dtype != SUNSHAPE_U8 && index_dtype != SUNSHAPE_I16 && index_dtype != SUNSHAPE_I32)
    return fail(SUNSHAPE_E_INVALID, "index dtype must be U8, I16 or I32.");
  const int C = codec->n_centroids;
  if ((index_dtype == SUNSHAPE_U8 && C > 256) || (index_dtype == SUNSHAPE_I16 && C > 65535))
    return fail(SUNSHAPE_E_INVALID, "index dtype is too narrow for n_centroids (codec.py:78-83 rule).");
  if (n_heads < 0 || n_tokens < 0 || kv_heads <= 0) return fail(SUNSHAPE_E_INVALID, "negative size.");
  if (out_head_stride < n_tokens) return fail(SUNSHAPE_E_INVALID, "out_head_stride must be >= n_tokens.");
  if (codec->heavy_mask && !heavy_out)
    return fail(SUNSHAPE_E_INVALID, "heavy_out is required when the codec has a heavy-block mask.");
  if (heavy_out && heavy_dtype != SUNSHAPE_BF16 && heavy_dtype != SUNSHAPE_F32)
    return fail(SUNSHAPE_E_INVALID, "heavy dtype must be BF16 or F32.");
  if (n_heads == 0 || n_tokens == 0) return SUNSHAPE_OK;
  const int D = codec->head_dim, bd = codec->block_dim;
  EncodeParams p{};
  p.keys = keys; p.keys_dtype = keys_dtype; p.key_hs = key_head_stride; p.key_ts = key_token_stride;
  p.n_tokens = n_tokens; p.kv_heads = kv_heads;
  p.cb = codec->centroids; p.n_cb = codec->n_cb; p.perm = codec->permutation; p.heavy_mask = codec->heavy_mask;
  p.nb = D / bd; p.bd = bd; p.C = C; p.D = D;
  p.idx_out = indices_out; p.index_dtype = index_dtype; p.heavy_out = heavy_out; p.heavy_dtype = heavy_dtype;
  p.out_hs = out_head_stride;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // SUNSHAPE_ENCODE=cuda_cores forces the CUDA-core kernel (a cross-check of the tensor-core one)
  const char* path = getenv("SUNSHAPE_ENCODE");
  const bool force_cc = path && strcmp(path, "cuda_cores") == 0;
  if (!force_cc && encode_tc_supported(p) &&
      launch_encode_tc(p, n_heads, codec->heavy_mask ? codec->n_heavy : 0, st) == 0)
    return cuda_status("encode (tensor cores) launch");
  if (path && strcmp(path, "tensor_cores") == 0)
    return fail(SUNSHAPE_E_UNSUPPORTED, "SUNSHAPE_ENCODE=tensor_cores: needs fp32/bf16/f16 keys with 16-byte multiple "
                                        "row and head strides, head_dim * element size a multiple of 128 bytes, "
                                        "block_dim 2, 4 or 8, at most 64 blocks and n_centroids a multiple of 64 up "
                                        "to 256.");
  const int smem = (kEncRows * (D + 1) + C * bd + C + D) * 4 + 64;
  if (smem > kSmemLimit) return fail(SUNSHAPE_E_UNSUPPORTED, "encode: codebook too large for shared memory.");
  dim3 grid((n_tokens + kEncRows - 1) / kEncRows, n_heads);
#define SUNSHAPE_ENC_CASE(B)                                                         \
  case B: {                                                                          \
    cudaFuncSetAttribute(encode_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
    encode_kernel<B><<<grid, kEncRows, smem, st>>>(p);                               \
    break;                                                                           \
  }
  switch (bd) {
    SUNSHAPE_ENC_CASE(1)
    SUNSHAPE_ENC_CASE(2)
    SUNSHAPE_ENC_CASE(4)
    SUNSHAPE_ENC_CASE(8)
    SUNSHAPE_ENC_CASE(16)
    default: return fail(SUNSHAPE_E_UNSUPPORTED, "encode supports block_dim 1, 2, 4, 8 or 16.");
  }
#undef SUNSHAPE_ENC_CASE
  return cuda_status("encode launch");
}

int sunshape_encode_error(int32_t* code, int32_t clear) {
  if (!code) return fail(SUNSHAPE_E_INVALID, "code pointer is NULL.");
  const int e = encode_error_word(code, clear != 0);
  if (e) return fail(SUNSHAPE_E_CUDA, std::string("reading the encode error word: ") +
                                          cudaGetErrorString(static_cast<cudaError_t>(e)));
  return SUNSHAPE_OK;
}

int sunshape_dequantize(const sunshape_codec_t* codec, const sunshape_kv_t* kv, int32_t n_heads, int32_t kv_heads,
                        float* out, void* stream) {
  if (int rc = check_codec(codec)) return rc;
  if (int rc = check_kv(kv, codec, false)) return rc;
  if (!out) return fail(SUNSHAPE_E_INVALID, "out pointer is NULL.");
  if (codec->heavy_mask && !kv->heavy)
    return fail(SUNSHAPE_E_INVALID, "Mixed-precision quantized keys are missing passthrough values.");
  if (n_heads == 0 || kv->seq_len == 0) return SUNSHAPE_OK;
  DequantParams p{};
  p.idx = kv->indices; p.index_dtype = kv->index_dtype; p.heavy = kv->heavy; p.heavy_dtype = kv->heavy_dtype;
  p.head_stride = kv->head_stride; p.T = kv->seq_len; p.kv_heads = kv_heads;
  p.cb = codec->centroids; p.n_cb = codec->n_cb; p.perm = codec->permutation; p.heavy_mask = codec->heavy_mask;
  p.D = codec->head_dim; p.bd = codec->block_dim; p.nb = p.D / p.bd; p.C = codec->n_centroids; p.out = out;
  const int64_t n = (int64_t)kv->seq_len * p.D;
  dim3 grid((unsigned)std::min<int64_t>((n + 255) / 256, 4096), n_heads);
  dequant_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cuda_status("dequantize launch");
}

static int fill_common(DecodeParams& p, const sunshape_codec_t* codec, const sunshape_kv_t* kv, int n_heads,
                       int kv_heads) {
  p.cb = codec->centroids; p.n_cb = codec->n_cb; p.perm = codec->permutation; p.heavy_mask = codec->heavy_mask;
  p.cb_norm_max = codec->centroid_norm_max;
  p.D = codec->head_dim; p.bd = codec->block_dim; p.nb = p.D / p.bd; p.C = codec->n_centroids;
  p.nbh = (p.nb + 7) / 8;
  p.idx = reinterpret_cast<const uint8_t*>(kv->indices);
  p.heavy = kv->heavy; p.heavy_dtype = kv->heavy ? kv->heavy_dtype : SUNSHAPE_BF16;
  p.v = kv->value; p.T = kv->seq_len; p.head_stride = kv->head_stride; p.n_heads = n_heads;
  p.kv_heads = kv_heads;
  return SUNSHAPE_OK;
}

static int check_decode_codec(const sunshape_codec_t* codec, const sunshape_kv_t* kv) {
  if (kv->index_dtype != SUNSHAPE_U8)
    return fail(SUNSHAPE_E_UNSUPPORTED, "the fused LUT kernels need uint8 indices (n_centroids <= 256).");
  if (codec->n_centroids > 256) return fail(SUNSHAPE_E_UNSUPPORTED, "n_centroids > 256 is not supported by the LUT kernels.");
  if (codec->heavy_mask && !kv->heavy)
    return fail(SUNSHAPE_E_INVALID, "Mixed-precision quantized keys are missing passthrough values.");
  return SUNSHAPE_OK;
}

int sunshape_attention_scores(const sunshape_codec_t* codec, const sunshape_kv_t* kv, const void* query,
                              int32_t query_dtype, int32_t n_heads, int32_t kv_heads, int32_t rows, float scale,
                              float* scores_out, void* stream) {
  if (int rc = check_codec(codec)) return rc;
  if (int rc = check_kv(kv, codec, false)) return rc;
  if (int rc = check_decode_codec(codec, kv)) return rc;
  if (!query || !scores_out) return fail(SUNSHAPE_E_INVALID, "query / scores_out pointer is NULL.");
  if (!is_float_dtype(query_dtype)) return fail(SUNSHAPE_E_INVALID, "query dtype must be F32, BF16 or F16.");
  if (rows <= 0 || rows > 16) return fail(SUNSHAPE_E_UNSUPPORTED, "scores: rows per head must be in [1, 16].");
  if (n_heads == 0 || kv->seq_len == 0) return SUNSHAPE_OK;
  DecodePlan pl;
  std::string why;
  const int nb = codec->head_dim / codec->block_dim;
  const int hsz = kv->heavy_dtype == SUNSHAPE_F32 ? 4 : 2;
  if (!plan_decode(pl, nb, codec->n_centroids, codec->head_dim, 64, 2, codec->heavy_mask ? codec->n_heavy : 0,
                   codec->block_dim, hsz, true, n_heads, kv->seq_len, rows, why))
    return fail(SUNSHAPE_E_UNSUPPORTED, why);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int r0 = 0; r0 < rows; r0 += pl.chunk_rows) {
    DecodeParams p = pl.prm;
    fill_common(p, codec, kv, n_heads, kv_heads);
    p.q = query; p.q_dtype = query_dtype; p.R = rows; p.r0 = r0; p.Rc = std::min(pl.chunk_rows, rows - r0);
    p.L = 1; p.G = rows; p.q_heads = kv_heads * rows;
    p.scale = scale; p.has_scale = std::isnan(scale) ? 0 : 1;
    p.scores_out = scores_out;
    DecodePlan pc = pl;
    pc.prm = p;
    if (int rc = launch_decode<true>(pc, 64, SUNSHAPE_F32, st)) return rc;
  }
  return cuda_status("scores launch");
}

int64_t sunshape_decode_workspace_bytes(int32_t n_heads, int32_t seq_len, int32_t rows, int32_t value_dim,
                                        int32_t n_blocks) {
  if (n_heads <= 0 || seq_len <= 0 || rows <= 0) return 256;
  // the slot area depends only on the grid, the split and (gp, value_dim): use the largest gp
  const int gp = pick_gp(rows);
  const int tph = (seq_len + kTileTokens - 1) / kTileTokens;
  const int64_t total = (int64_t)n_heads * tph;
  const int64_t grid = std::min<int64_t>(num_sms(), total);
  const int64_t max_seg = max_segments(n_heads, tph, grid);
  // per-head LUT area: fp32 entries with a fixed 256-row stride (upper bound), within the policy cap
  const int64_t lut_bytes = (int64_t)((std::max(n_blocks, 1) + 7) / 8) * 8 * kLutC * gp * 4;
  return mma_workspace_bytes(n_heads, grid, max_seg, gp, value_dim,
                             (int64_t)n_heads * lut_bytes <= kGlobalLutMaxBytes ? lut_bytes : 0);
}

int64_t sunshape_decode_workspace_min_bytes(int32_t n_heads, int32_t seq_len, int32_t rows, int32_t value_dim) {
  if (n_heads <= 0 || seq_len <= 0 || rows <= 0) return 256;
  const int gp = pick_gp(rows);
  const int tph = (seq_len + kTileTokens - 1) / kTileTokens;
  const int64_t total = (int64_t)n_heads * tph;
  const int64_t grid = std::min<int64_t>(num_sms(), total);
  const int64_t max_seg = max_segments(n_heads, tph, grid);
  return mma_workspace_bytes(n_heads, grid, max_seg, gp, value_dim, 0);
}

static int decode_impl(const sunshape_codec_t* codec, const sunshape_kv_t* kv, const void* query,
                       int32_t query_dtype, int32_t batch, int32_t q_heads, int32_t kv_heads,
                       int32_t query_len, const void* mask, int32_t mask_dtype, int64_t mask_sb,
                       int64_t mask_sh, int64_t mask_sq, float scale, void* out, int32_t out_dtype,
                       float* partials, void* workspace, int64_t workspace_bytes, void* stream,
                       const sunshape_peer_group_t* group);

int sunshape_decode_attention(const sunshape_codec_t* codec, const sunshape_kv_t* kv, const void* query,
                              int32_t query_dtype, int32_t batch, int32_t q_heads, int32_t kv_heads,
                              int32_t query_len, const void* mask, int32_t mask_dtype, int64_t mask_sb,
                              int64_t mask_sh, int64_t mask_sq, float scale, void* out, int32_t out_dtype,
                              float* partials, void* workspace, int64_t workspace_bytes, void* stream) {
  return decode_impl(codec, kv, query, query_dtype, batch, q_heads, kv_heads, query_len, mask, mask_dtype, mask_sb,
                     mask_sh, mask_sq, scale, out, out_dtype, partials, workspace, workspace_bytes, stream, nullptr);
}

int sunshape_decode_attention_peers(const sunshape_codec_t* codec, const sunshape_kv_t* kv, const void* query,
                                    int32_t query_dtype, int32_t batch, int32_t q_heads, int32_t kv_heads,
                                    int32_t query_len, const void* mask, int32_t mask_dtype, int64_t mask_sb,
                                    int64_t mask_sh, int64_t mask_sq, float scale, void* out, int32_t out_dtype,
                                    const sunshape_peer_group_t* group, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
  if (!group) return fail(SUNSHAPE_E_INVALID, "peer group is NULL.");
  if (group->world < 2 || group->world > 8 || group->rank < 0 || group->rank >= group->world)
    return fail(SUNSHAPE_E_INVALID, "peer group: world must be 2..8 and 0 <= rank < world.");
  for (int r = 0; r < group->world; ++r)
    if (!group->buffers[r]) return fail(SUNSHAPE_E_INVALID, "peer group: missing exchange buffer.");
  if (!out) return fail(SUNSHAPE_E_INVALID, "out pointer is NULL.");
  if (!kv || kv->value_dtype == SUNSHAPE_F32)
    return fail(SUNSHAPE_E_UNSUPPORTED, "the peer exchange path needs 16-bit values.");
  if (q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || (q_heads / kv_heads) * query_len > 16)
    return fail(SUNSHAPE_E_UNSUPPORTED, "the peer exchange path needs G * query_len <= 16.");
  return decode_impl(codec, kv, query, query_dtype, batch, q_heads, kv_heads, query_len, mask, mask_dtype, mask_sb,
                     mask_sh, mask_sq, scale, out, out_dtype, nullptr, workspace, workspace_bytes, stream, group);
}

int64_t sunshape_peer_buffer_bytes(int32_t world, int64_t rows, int32_t value_dim, int32_t n_heads) {
  return peer_layout(world, rows, value_dim, n_heads).total;
}

static int decode_impl(const sunshape_codec_t* codec, const sunshape_kv_t* kv, const void* query,
                       int32_t query_dtype, int32_t batch, int32_t q_heads, int32_t kv_heads,
                       int32_t query_len, const void* mask, int32_t mask_dtype, int64_t mask_sb,
                       int64_t mask_sh, int64_t mask_sq, float scale, void* out, int32_t out_dtype,
                       float* partials, void* workspace, int64_t workspace_bytes, void* stream,
                       const sunshape_peer_group_t* group) {
  if (int rc = check_codec(codec)) return rc;
  if (int rc = check_kv(kv, codec, true)) return rc;
  if (int rc = check_decode_codec(codec, kv)) return rc;
  if (!query) return fail(SUNSHAPE_E_INVALID, "query pointer is NULL.");
  if (!is_float_dtype(query_dtype)) return fail(SUNSHAPE_E_INVALID, "query dtype must be F32, BF16 or F16.");
  if (batch < 0 || q_heads <= 0 || kv_heads <= 0 || query_len <= 0)
    return fail(SUNSHAPE_E_INVALID, "batch / heads / query_len must be positive.");
  if (q_heads % kv_heads != 0) return fail(SUNSHAPE_E_INVALID, "Query head count must be divisible by kv-head count.");
  if (!out && !partials) return fail(SUNSHAPE_E_INVALID, "one of out / partials must be given.");
  if (out && !is_float_dtype(out_dtype)) return fail(SUNSHAPE_E_INVALID, "out dtype must be F32, BF16 or F16.");
  if (mask && !is_float_dtype(mask_dtype)) return fail(SUNSHAPE_E_INVALID, "mask dtype must be F32, BF16 or F16.");
  if (kv->seq_len == 0) return fail(SUNSHAPE_E_INVALID, "seq_len must be positive for decode attention.");
  if (batch == 0) return SUNSHAPE_OK;
  const int G = q_heads / kv_heads;
  const int R = G * query_len;
  const int n_heads = batch * kv_heads;
  const int nb = codec->head_dim / codec->block_dim;
  const int dv = kv->value_dim;
  DecodePlan pl;
  std::string why;
  const int hsz = kv->heavy_dtype == SUNSHAPE_F32 ? 4 : 2;
  const int n_heavy = codec->heavy_mask ? codec->n_heavy : 0;
  const bool use_mma = kv->value_dtype != SUNSHAPE_F32;   // 16-bit values: tensor-core kernel
  const bool ok = use_mma ? plan_decode_mma(pl, nb, codec->head_dim, dv, n_heavy, codec->block_dim, hsz, n_heads,
                                            kv->seq_len, R, why)
                          : plan_decode(pl, nb, codec->n_centroids, codec->head_dim, dv, dtype_size(kv->value_dtype),
                                        n_heavy, codec->block_dim, hsz, false, n_heads, kv->seq_len, R, why);
  if (!ok) return fail(SUNSHAPE_E_UNSUPPORTED, why);
  if (group && pl.chunk_rows < R)
    return fail(SUNSHAPE_E_UNSUPPORTED, "the peer exchange path needs all query rows of a KV head in one launch.");
  if (use_mma) {
    const int64_t rows_total = (int64_t)(n_heads - 1) * kv->head_stride + kv->seq_len;
    if (int rc = make_value_map(&pl.prm.tmap_v, kv->value, kv->value_dtype, dv, rows_total)) return rc;
  }
  if (!workspace) return fail(SUNSHAPE_E_WORKSPACE, "decode workspace is NULL.");
  if (workspace_bytes < pl.ws_bytes) return fail(SUNSHAPE_E_WORKSPACE, "decode workspace is too small.");
  if (!aligned16(workspace)) return fail(SUNSHAPE_E_WORKSPACE, "decode workspace must be 16-byte aligned.");
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  for (int r0 = 0; r0 < R; r0 += pl.chunk_rows) {
    DecodeParams p = pl.prm;
    fill_common(p, codec, kv, n_heads, kv_heads);
    p.q = query; p.q_dtype = query_dtype; p.R = R; p.r0 = r0; p.Rc = std::min(pl.chunk_rows, R - r0);
    p.L = query_len; p.G = G; p.q_heads = q_heads;
    p.mask = mask; p.mask_dtype = mask_dtype; p.msb = mask_sb; p.msh = mask_sh; p.msq = mask_sq;
    p.scale = scale; p.has_scale = std::isnan(scale) ? 0 : 1;
    p.out = out; p.out_dtype = out_dtype; p.partials = partials;
    if (group) {   // rank-local results go to the exchange buffers; xmerge_kernel writes out
      const PeerLayout lay = peer_layout(group->world, (int64_t)n_heads * R, dv, n_heads);
      p.out = nullptr;
      p.xworld = group->world;
      p.xrank = group->rank;
      p.x_rows = (int64_t)n_heads * R;
      for (int r = 0; r < group->world; ++r) {
        p.xrecv[r] = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(group->buffers[r]) + lay.recv);
        p.xarrive[r] = reinterpret_cast<unsigned int*>(reinterpret_cast<uint8_t*>(group->buffers[r]) + lay.arrive);
      }
      p.xstep = reinterpret_cast<const unsigned int*>(reinterpret_cast<uint8_t*>(group->buffers[group->rank]) +
                                                      lay.step);
    }
    p.err = reinterpret_cast<int*>(ws);
    p.counters = reinterpret_cast<int*>(ws + 256);
    p.slots = reinterpret_cast<float*>(ws + 256 + round_up(n_heads * 4, 256));
    if (use_mma) {
      // per-head LUTs built GPU-wide at kernel start when they fit the workspace policy
      const int64_t lut_ws =
          (codec->block_dim <= 16 && codec->head_dim % 8 == 0 && aligned16(query) &&
           kGlobalLutMaxBytes >= (int64_t)n_heads * p.lut_bytes) ? p.lut_bytes : 0;
      const MmaWsOffsets o = mma_workspace_offsets(n_heads, pl.grid, p.max_seg, pl.gp, dv, lut_ws);
      p.slots = reinterpret_cast<float*>(ws + o.slots);
#ifdef SUNSHAPE_TRACE
      p.trace = reinterpret_cast<unsigned long long*>(ws + (workspace_bytes - 4096 * 256) / 256 * 256);
#endif
      if (lut_ws && workspace_bytes >= o.total) {
        p.lut_global = ws + o.luts;
        p.lut_scale_global = reinterpret_cast<float*>(ws + o.scales);
        if (int rc = launch_lut(p, pl.gp, pl.lut16, n_heads, st)) return rc;
      }
#ifdef SUNSHAPE_TRACE
      p.trace = reinterpret_cast<unsigned long long*>(ws + (workspace_bytes - 4096 * 256) / 256 * 256);
#endif
    }
    DecodePlan pc = pl;
    pc.prm = p;
    if (int rc = use_mma ? launch_decode_mma(pc, dv, kv->value_dtype, st)
                         : launch_decode<false>(pc, dv, kv->value_dtype, st))
      return rc;
    if (group) {
      const PeerLayout lay = peer_layout(group->world, (int64_t)n_heads * R, dv, n_heads);
      uint8_t* own = reinterpret_cast<uint8_t*>(group->buffers[group->rank]);
      unsigned int* stp = reinterpret_cast<unsigned int*>(own + lay.step);
      xmerge_kernel<<<n_heads, 128, 0, st>>>(reinterpret_cast<float*>(own + lay.recv),
                                              reinterpret_cast<unsigned int*>(own + lay.arrive), stp, stp + 1,
                                              group->world, (int64_t)n_heads * R, R, dv, n_heads, out, out_dtype,
                                              p.err);
    }
  }
  return cuda_status("decode launch");
}

int sunshape_merge_partials(const float* partials, int32_t n_parts, int64_t rows, int32_t value_dim, void* out,
                            int32_t out_dtype, void* stream) {
  if (!partials || !out) return fail(SUNSHAPE_E_INVALID, "partials / out pointer is NULL.");
  if (n_parts <= 0 || rows < 0 || value_dim <= 0) return fail(SUNSHAPE_E_INVALID, "bad merge sizes.");
  if (!is_float_dtype(out_dtype)) return fail(SUNSHAPE_E_INVALID, "out dtype must be F32, BF16 or F16.");
  if (rows == 0) return SUNSHAPE_OK;
  merge_partials_kernel<<<(unsigned)rows, std::min(256, round_up(value_dim, 32)), 0,
                          reinterpret_cast<cudaStream_t>(stream)>>>(partials, n_parts, rows, value_dim, out,
                                                                    out_dtype);
  return cuda_status("merge launch");
}

}  // extern "C"
