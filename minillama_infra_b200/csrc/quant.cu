// quant.cu -- activation and weight quantisers for the INT8 group-64 path.
//
//  * Activations (per token, dynamic): bit-identical to the reference's
//    quantize_activation_kernel (src/model_cuda_v2_shared.cu:429-455).
//    One CTA per token; max|x| is exact in any reduction order.
//  * Weights (per row, per group, offline): bit-identical to
//    scripts/quantize_int8_group.py:55-71.  One warp per group.
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

constexpr int kQuantThreads = 512;

__global__ void __launch_bounds__(kQuantThreads)
    quantize_rows_kernel(int8_t* xq, float* xs, const float* x, int n) {
  __shared__ float red[kQuantThreads / 32];
  griddep_wait();
  const size_t row = blockIdx.x;
  const float* xr = x + row * n;
  int8_t* qr = xq + row * n;
  float m = 0.f;
  for (int i = threadIdx.x; i < n; i += kQuantThreads) m = fmaxf(m, fabsf(xr[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = red[0];
#pragma unroll
  for (int w = 1; w < kQuantThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  float scale = amax / 127.0f;
  if (scale < 1e-8f) scale = 1e-8f;
  if (threadIdx.x == 0) xs[row] = scale;
  const float inv = 1.0f / scale;
  griddep_launch_dependents();
  for (int i = threadIdx.x; i < n; i += kQuantThreads)
    qr[i] = static_cast<int8_t>(max(-127, min(127, __float2int_rn(xr[i] * inv))));
}

__global__ void __launch_bounds__(256)
    quantize_weights_kernel(int8_t* q, float* s, const float* w, long long rows,
                            long long cols, int gs) {
  const long long ng = cols / gs;
  const long long total = rows * ng;
  const int lane = threadIdx.x & 31;
  for (long long gid = (blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x) >> 5;
       gid < total; gid += (static_cast<long long>(gridDim.x) * blockDim.x) >> 5) {
    const long long r = gid / ng;
    const long long g = gid - r * ng;
    const float* src = w + r * cols + g * gs;
    int8_t* dst = q + r * cols + g * gs;
    float amax = 0.f;
    for (int j = lane; j < gs; j += 32) amax = fmaxf(amax, fabsf(src[j]));
    amax = warp_max(amax);
    if (amax == 0.f) amax = 1e-9f;
    const float scale = __fdiv_rn(amax, 127.0f);
    if (lane == 0) s[gid] = scale;
    for (int j = lane; j < gs; j += 32) {
      float v = rintf(__fdiv_rn(src[j], scale));
      v = fminf(fmaxf(v, -127.f), 127.f);
      dst[j] = static_cast<int8_t>(v);
    }
  }
}

int launch_quantize_rows(int8_t* xq, float* xs, const float* x, int m, int n,
                         cudaStream_t stream) {
  return check_cuda(launch(quantize_rows_kernel, dim3(static_cast<unsigned>(m)),
                           dim3(kQuantThreads), 0, stream, true, xq, xs, x, n));
}

}  // namespace mli

using namespace mli;

extern "C" {

int mli_quantize_activation(int8_t* xq, float* xs, const float* x, int n,
                            void* stream) {
  if (!xq || !xs || !x || n <= 0) return set_status(MLI_ERR_INVALID_ARG);
  return launch_quantize_rows(xq, xs, x, 1, n, static_cast<cudaStream_t>(stream));
}

int mli_quantize_activation_rows(int8_t* xq, float* xs, const float* x, int m,
                                 int n, void* stream) {
  if (!xq || !xs || !x || n <= 0 || m <= 0) return set_status(MLI_ERR_INVALID_ARG);
  return launch_quantize_rows(xq, xs, x, m, n, static_cast<cudaStream_t>(stream));
}

int mli_quantize_weights(int8_t* w_q, float* w_s, const float* w, int rows,
                         int cols, int group_size, void* stream) {
  if (!w_q || !w_s || !w || rows <= 0 || cols <= 0 || group_size <= 0 ||
      cols % group_size != 0)
    return set_status(MLI_ERR_INVALID_ARG);
  const long long groups = static_cast<long long>(rows) * (cols / group_size);
  long long blocks = (groups * 32 + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  return check_cuda(launch(quantize_weights_kernel, dim3(static_cast<unsigned>(blocks)),
                           dim3(256), 0, static_cast<cudaStream_t>(stream), false, w_q,
                           w_s, w, static_cast<long long>(rows),
                           static_cast<long long>(cols), group_size));
}

}  // extern "C"
