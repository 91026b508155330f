// gemv_f32.cu -- fp32 GEMV y = W x, W fp32 [d][n] row-major (sm_100a).
//
// The reference's `matmul` launcher (include/model.h:61,
// src/model_cuda_v2_shared.cu:10-25) is the only fp32 GEMV of its forward
// passes: the tied-embedding classifier (:418, :564), 128256 x 2048 fp32 --
// 1.05 GB read per token, more than all the int8 layers together.  The
// reference runs one thread per row, so one load instruction of a warp
// touches 32 rows 8 KB apart.  Here a warp owns a row: each load instruction
// reads 512 contiguous bytes (float4 per lane) with the L1-bypassing
// streaming load, eight of them in flight per lane, and x sits in shared
// memory.  Warps stride over rows; a warp's per-lane products accumulate in
// column order and the butterfly sum finishes the row (not the reference's
// sequential order: results agree within fp32 rounding, max-abs-rel 1e-5).
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {
namespace {

constexpr int kF32Warps = 8;         // warps per CTA
constexpr int kF32InFlight = 8;      // float4 loads per lane before the FMAs
constexpr int kF32CtasPerSm = 4;
constexpr int kF32MaxSmemCols = 48 * 1024 / 4;  // x in static-size dynamic smem

__device__ __forceinline__ float4 ldg_stream_f4(const float4* p) {
  const uint4 u = ldg_stream_u4(p);
  return make_float4(__uint_as_float(u.x), __uint_as_float(u.y), __uint_as_float(u.z), __uint_as_float(u.w));
}

// Fast path: n % 4 == 0, 16-byte aligned w and x, n <= kF32MaxSmemCols.
__global__ void __launch_bounds__(kF32Warps * 32) gemv_f32_kernel(float* __restrict__ y,
                                                                  const float* __restrict__ x,
                                                                  const float* __restrict__ w, int n, int d) {
  extern __shared__ float4 xs4[];
  const int n4 = n >> 2;
  griddep_wait();  // x may be the previous kernel's output
  for (int i = threadIdx.x; i < n4; i += blockDim.x) xs4[i] = reinterpret_cast<const float4*>(x)[i];
  __syncthreads();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * kF32Warps;
  for (int r = blockIdx.x * kF32Warps + (threadIdx.x >> 5); r < d; r += stride) {
    const float4* wr = reinterpret_cast<const float4*>(w + static_cast<size_t>(r) * n);
    float acc = 0.f;
    for (int c0 = 0; c0 < n4; c0 += 32 * kF32InFlight) {
      float4 v[kF32InFlight];
#pragma unroll
      for (int k = 0; k < kF32InFlight; ++k) {
        const int c = c0 + lane + 32 * k;
        v[k] = c < n4 ? ldg_stream_f4(wr + c) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int k = 0; k < kF32InFlight; ++k) {
        const int c = c0 + lane + 32 * k;
        if (c < n4) {
          const float4 xv = xs4[c];
          acc = fmaf(v[k].x, xv.x, acc);
          acc = fmaf(v[k].y, xv.y, acc);
          acc = fmaf(v[k].z, xv.z, acc);
          acc = fmaf(v[k].w, xv.w, acc);
        }
      }
    }
    acc = warp_sum(acc);
    if (lane == 0) y[r] = acc;
  }
}

// Any n and alignment: a warp per row, scalar loads.
__global__ void __launch_bounds__(kF32Warps * 32) gemv_f32_generic_kernel(float* __restrict__ y,
                                                                          const float* __restrict__ x,
                                                                          const float* __restrict__ w, int n,
                                                                          int d) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int stride = gridDim.x * kF32Warps;
  for (int r = blockIdx.x * kF32Warps + (threadIdx.x >> 5); r < d; r += stride) {
    const float* wr = w + static_cast<size_t>(r) * n;
    float acc = 0.f;
    for (int c = lane; c < n; c += 32) acc = fmaf(__ldg(wr + c), __ldg(x + c), acc);
    acc = warp_sum(acc);
    if (lane == 0) y[r] = acc;
  }
}

}  // namespace
}  // namespace mli

using namespace mli;

extern "C" int mli_gemv_f32(float* y, const float* x, const float* w, int n, int d, void* stream) {
  if (!y || !x || !w || n <= 0 || d <= 0) return set_status(MLI_ERR_INVALID_ARG);
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const long long warps_needed = (static_cast<long long>(d) + kF32Warps - 1) / kF32Warps;
  const int grid = static_cast<int>(warps_needed < static_cast<long long>(dev.sm_count) * kF32CtasPerSm
                                        ? warps_needed
                                        : static_cast<long long>(dev.sm_count) * kF32CtasPerSm);
  const bool fast = n % 4 == 0 && n <= kF32MaxSmemCols && aligned(w, 16) && aligned(x, 16);
  if (fast)
    return check_cuda(launch(gemv_f32_kernel, dim3(grid), dim3(kF32Warps * 32), static_cast<size_t>(n) * 4, st,
                             true, y, x, w, n, d));
  return check_cuda(launch(gemv_f32_generic_kernel, dim3(grid), dim3(kF32Warps * 32), 0, st, true, y, x, w, n,
                           d));
}
