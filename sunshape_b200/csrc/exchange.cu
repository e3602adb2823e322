// Cross-GPU merge of the KV-sequence split in one kernel over NVLink peer memory.
//
// Every rank holds an exchange buffer mapped into every other rank's process (CUDA IPC, see
// peer.cu).  After a rank's decode kernel has written its (m, l, acc) partial rows, one launch of
// exchange_merge_kernel per rank:
//
//   1. pushes slice i of the local partial rows (kRowsPerCta rows per CTA) into every rank's buffer
//      with 16-byte stores over NVLink, then publishes "slice i of rank r is in" by storing the call
//      number into a per-(rank, slice) flag of every rank's buffer (release at system scope);
//   2. waits (bounded) until all ranks' slice i has landed in its own buffer and merges the rows in
//      fixed rank order:  M = max m_r,  L = sum l_r e^(m_r - M),  out = sum acc_r e^(m_r - M) / L.
//
// Each CTA pushes before it waits, so the lowest-numbered waiting CTA of every rank always has its
// data: the exchange cannot deadlock however the grids are scheduled.  The call number lives in the
// buffer (the last CTA to finish advances it), so every call issues the same launch; receive areas
// and flags alternate between two halves by its parity, so a rank that finished call k can start
// call k+1 while a slower rank still merges call k.  No NCCL, no TMA, no multicast: plain peer
// stores and system-scope flag operations.
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"

namespace sunshape {
int set_last_error(int code, const char* msg);   // defined in capi.cu

namespace {

constexpr int kRowsPerCta = 4;
constexpr int kErrExchangeWait = 105;

// Buffer layout (bytes): recv [2][world][rows][row_f] fp32 | flags [2][world][slices] u32 |
// step u32, done u32, error i32.  row_f = dv + 2 rounded up to a multiple of 4 (16-byte rows).
struct XLayout {
  int64_t recv, flags, ctl, total;
  int row_f, slices;
};
__host__ __device__ inline XLayout x_layout(int world, int64_t rows, int dv) {
  XLayout l;
  l.row_f = (dv + 2 + 3) / 4 * 4;
  l.slices = (int)((rows + kRowsPerCta - 1) / kRowsPerCta);
  l.recv = 0;
  l.flags = ((int64_t)2 * world * rows * l.row_f * 4 + 255) / 256 * 256;
  l.ctl = l.flags + ((int64_t)2 * world * l.slices * 4 + 255) / 256 * 256;
  l.total = l.ctl + 256;
  return l;
}

struct XParams {
  const float* partials;      // [rows][dv + 2] this rank's (m, l, acc)
  int64_t rows;
  int dv, world, rank;
  uint8_t* bufs[8];           // every rank's exchange buffer, as mapped in this process
  void* out;                  // [rows][dv]
  int out_dtype;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(128) exchange_merge_kernel(const __grid_constant__ XParams x) {
  const XLayout L = x_layout(x.world, x.rows, x.dv);
  uint8_t* own = x.bufs[x.rank];
  unsigned* ctl = reinterpret_cast<unsigned*>(own + L.ctl);   // [0] step, [1] done, [2] error
  __shared__ unsigned epoch_s;
  __shared__ int ok_s;
  if (threadIdx.x == 0) {
    epoch_s = *reinterpret_cast<volatile unsigned*>(ctl) + 1u;   // this call's number
    ok_s = 1;
  }
  __syncthreads();
  const unsigned epoch = epoch_s, par = epoch & 1u;
  const int slice = blockIdx.x;
  const int64_t r0 = (int64_t)slice * kRowsPerCta;
  const int nr = (int)(x.rows - r0 < kRowsPerCta ? x.rows - r0 : kRowsPerCta);
  const int src_f = x.dv + 2, row_f = L.row_f;
  const int vec_per_row = row_f / 4;

  // 1. push this slice to every rank (16-byte stores; a row's padding floats carry zeros)
  for (int e = threadIdx.x; e < nr * vec_per_row; e += blockDim.x) {
    const int r = e / vec_per_row, q = e - r * vec_per_row;
    const float* src = x.partials + (r0 + r) * src_f + 4 * q;
    float4 v;
    v.x = 4 * q + 0 < src_f ? src[0] : 0.f;
    v.y = 4 * q + 1 < src_f ? src[1] : 0.f;
    v.z = 4 * q + 2 < src_f ? src[2] : 0.f;
    v.w = 4 * q + 3 < src_f ? src[3] : 0.f;
    for (int k = 0; k < x.world; ++k) {
      const int dst_rank = (x.rank + k) % x.world;
      float4* dst = reinterpret_cast<float4*>(x.bufs[dst_rank] + L.recv) +
                    (((int64_t)par * x.world + x.rank) * x.rows + r0 + r) * vec_per_row + q;
      *dst = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < x.world) {
    unsigned* f = reinterpret_cast<unsigned*>(x.bufs[threadIdx.x] + L.flags) +
                  ((int64_t)par * x.world + x.rank) * L.slices + slice;
    st_release_sys(f, epoch);
  }
  // 2. wait until every rank's slice landed here (bounded), then merge in rank order
  if (threadIdx.x < x.world) {
    const unsigned* f = reinterpret_cast<const unsigned*>(own + L.flags) +
                        ((int64_t)par * x.world + threadIdx.x) * L.slices + slice;
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys(f) != epoch) {
      if (global_ns() - t0 > kWaitLimitNs) {
        atomicCAS(reinterpret_cast<int*>(ctl + 2), 0, kErrExchangeWait);
        ok_s = 0;
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  const float NEG_INF = -__int_as_float(0x7f800000);
  const float* recv = reinterpret_cast<const float*>(own + L.recv);
  for (int e = threadIdx.x; e < nr * x.dv; e += blockDim.x) {
    const int r = e / x.dv, d = e - r * x.dv;
    const int64_t row = r0 + r;
    float M = NEG_INF;
    for (int k = 0; k < x.world; ++k)
      M = fmaxf(M, __ldcv(recv + (((int64_t)par * x.world + k) * x.rows + row) * row_f));
    float Lsum = 0.f, A = 0.f;
    if (M != NEG_INF) {
      for (int k = 0; k < x.world; ++k) {
        const float* s = recv + (((int64_t)par * x.world + k) * x.rows + row) * row_f;
        const float sc = fast_exp2((__ldcv(s) - M) * kLog2e);   // empty shard (m = -inf) -> 0
        Lsum = fmaf(__ldcv(s + 1), sc, Lsum);
        A = fmaf(__ldcv(s + 2 + d), sc, A);
      }
    }
    store_from_float(x.out, row * x.dv + d, x.out_dtype,
                     (M == NEG_INF || !ok_s) ? __int_as_float(0x7fc00000) : A / Lsum);
  }
  // the last CTA advances the call number
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ctl + 1, 1u) == gridDim.x - 1) {
      ctl[1] = 0u;
      __threadfence();
      atomicAdd(ctl, 1u);
    }
  }
}

}  // namespace
}  // namespace sunshape

using namespace sunshape;

extern "C" int64_t sunshape_exchange_buffer_bytes(int32_t world, int64_t rows, int32_t value_dim) {
  if (world <= 0 || rows < 0 || value_dim <= 0) return 0;
  return x_layout(world, rows, value_dim).total;
}

extern "C" int sunshape_exchange_merge(const float* partials, int64_t rows, int32_t value_dim,
                                       const sunshape_peer_group_t* group, void* out, int32_t out_dtype,
                                       void* stream) {
  if (!partials || !out || !group) return set_last_error(SUNSHAPE_E_INVALID, "partials / out / group is NULL.");
  if (group->world < 1 || group->world > 8 || group->rank < 0 || group->rank >= group->world)
    return set_last_error(SUNSHAPE_E_INVALID, "peer group: world must be 1..8 and 0 <= rank < world.");
  if (rows < 0 || value_dim <= 0) return set_last_error(SUNSHAPE_E_INVALID, "bad exchange sizes.");
  if (out_dtype != SUNSHAPE_F32 && out_dtype != SUNSHAPE_BF16 && out_dtype != SUNSHAPE_F16)
    return set_last_error(SUNSHAPE_E_INVALID, "out dtype must be F32, BF16 or F16.");
  XParams x{};
  for (int r = 0; r < group->world; ++r) {
    if (!group->buffers[r]) return set_last_error(SUNSHAPE_E_INVALID, "peer group: missing exchange buffer.");
    if (reinterpret_cast<uintptr_t>(group->buffers[r]) & 255)
      return set_last_error(SUNSHAPE_E_INVALID, "exchange buffers must be 256-byte aligned.");
    x.bufs[r] = reinterpret_cast<uint8_t*>(group->buffers[r]);
  }
  if (rows == 0) return SUNSHAPE_OK;
  x.partials = partials;
  x.rows = rows;
  x.dv = value_dim;
  x.world = group->world;
  x.rank = group->rank;
  x.out = out;
  x.out_dtype = out_dtype;
  const XLayout L = x_layout(x.world, rows, value_dim);
  exchange_merge_kernel<<<L.slices, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_last_error(SUNSHAPE_E_CUDA, (std::string("exchange launch: ") + cudaGetErrorString(e)).c_str());
  return SUNSHAPE_OK;
}

extern "C" int sunshape_exchange_error(const void* own_buffer, int32_t world, int64_t rows, int32_t value_dim,
                                       int32_t* code) {
  if (!own_buffer || !code) return set_last_error(SUNSHAPE_E_INVALID, "buffer / code is NULL.");
  const XLayout L = x_layout(world, rows, value_dim);
  const cudaError_t e = cudaMemcpy(code, reinterpret_cast<const uint8_t*>(own_buffer) + L.ctl + 8, sizeof(int32_t),
                                   cudaMemcpyDeviceToHost);
  if (e != cudaSuccess)
    return set_last_error(SUNSHAPE_E_CUDA, (std::string("exchange error word: ") + cudaGetErrorString(e)).c_str());
  return SUNSHAPE_OK;
}
