// gemm_w8a8.cu -- W8A8 group-64 linear op for a batch of m decode tokens.
//
// Y[t][r] = sum_g ((float)I[t][r][g] * w_s[r][g]) * xs[t], I the exact int32
// dot of group g of row r with token t's int8 activation.  The batch extends
// the reference's matmul_dp4a (src/model_cuda_v2_shared.cu:465-501) from one
// token to m; the reference itself decodes one token at a time.
//
// This file holds the CUDA-core path: the batch-1 GEMV's warp/slice layout
// with T tokens' int8 activations resident in registers, so every weight byte
// fetched from HBM feeds T dp4a.  Each token's row is reduced with the same
// butterfly as the batch-1 kernel, so a token's result does not depend on m.
// The tcgen05 tensor-core path for m >= 16 lives in gemm_tc.cu.
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

namespace {
constexpr int kThreadsB = 256;
constexpr int kWarpsB = 8;
constexpr int kSmemHeaderB = 128;
}  // namespace

struct BatchArgs {
  float* y;
  const int8_t* xq;
  const float* xs;
  const int8_t* w;
  const float* s;
  int m, n, d;
  int t0;  // first token of this pass
  int S, wps, rpw, R, n_tiles;
};

template <int T>
__global__ void __launch_bounds__(kThreadsB, 1)
    gemm_w8a8_cuda_core_kernel(const BatchArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  int8_t* xqs = reinterpret_cast<int8_t*>(smem + kSmemHeaderB);
  float* part = reinterpret_cast<float*>(xqs + static_cast<size_t>(T) * a.n);  // [R][T][S]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sl = warp % a.S, wj = warp / a.S;
  const bool warp_on = wj < a.wps;
  const int g0 = sl * 32 + (lane >> 2) * 4;
  const bool lane_on = warp_on && g0 < (a.n >> 6);
  const int col0 = g0 * 64 + (lane & 3) * 16;
  const int G = a.n >> 6;

  griddep_wait();
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(bar, static_cast<uint32_t>(T * a.n));
    bulk_copy_g2s(xqs, a.xq + static_cast<size_t>(a.t0) * a.n,
                  static_cast<uint32_t>(T * a.n), bar);
  }
  __syncthreads();
  const bool ok = mbar_wait_bounded(bar, 0, kWaitLimitNs);
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) {
      record_device_error(kDevStageTimeout);
      mbar_wait_bounded(bar, 0, kWaitLimitNs);
    }
    return;
  }
  griddep_launch_dependents();

  uint4 xv[T][4];
  float xsc[T];
#pragma unroll
  for (int t = 0; t < T; ++t) {
    xsc[t] = a.xs[a.t0 + t];
#pragma unroll
    for (int k = 0; k < 4; ++k)
      xv[t][k] = lane_on ? *reinterpret_cast<const uint4*>(xqs + t * a.n + col0 + 64 * k)
                         : make_uint4(0, 0, 0, 0);
  }

  const int my_tiles =
      (a.n_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1;
  for (int tt = 0; tt < my_tiles; ++tt) {
    const int row0 = (static_cast<int>(blockIdx.x) + tt * static_cast<int>(gridDim.x)) * a.R;
    for (int i = 0; i < a.rpw; ++i) {
      const int row = row0 + wj + i * a.wps;
      if (!warp_on || row >= a.d) continue;
      uint4 w[4] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0),
                    make_uint4(0, 0, 0, 0)};
      float ws = 0.f;
      if (lane_on) {
        const int8_t* p = a.w + static_cast<size_t>(row) * a.n + col0;
        w[0] = ldg_stream_u4(p);
        w[1] = ldg_stream_u4(p + 64);
        w[2] = ldg_stream_u4(p + 128);
        w[3] = ldg_stream_u4(p + 192);
        ws = ldg_f1(a.s + static_cast<size_t>(row) * G + g0 + (lane & 3));
      }
#pragma unroll
      for (int t = 0; t < T; ++t) {
        int pk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          int acc = __dp4a(static_cast<int>(w[k].x), static_cast<int>(xv[t][k].x), 0);
          acc = __dp4a(static_cast<int>(w[k].y), static_cast<int>(xv[t][k].y), acc);
          acc = __dp4a(static_cast<int>(w[k].z), static_cast<int>(xv[t][k].z), acc);
          pk[k] = __dp4a(static_cast<int>(w[k].w), static_cast<int>(xv[t][k].w), acc);
        }
        // quad reduce-scatter (see gemv_g64.cu): lane q keeps group q's dot
        const int q = lane & 3;
        const bool b0 = q & 1;
        int ka = b0 ? pk[1] : pk[0], sa = b0 ? pk[0] : pk[1];
        int kb = b0 ? pk[3] : pk[2], sb = b0 ? pk[2] : pk[3];
        ka += __shfl_xor_sync(0xffffffffu, sa, 1);
        kb += __shfl_xor_sync(0xffffffffu, sb, 1);
        const bool b1 = q & 2;
        int I = b1 ? kb : ka;
        I += __shfl_xor_sync(0xffffffffu, b1 ? ka : kb, 2);
        float term = lane_on ? (static_cast<float>(I) * ws) * xsc[t] : 0.f;
        term = warp_sum(term);
        if (lane == 0) {
          if (a.S == 1)
            a.y[static_cast<size_t>(a.t0 + t) * a.d + row] = term;
          else
            part[((wj + i * a.wps) * T + t) * a.S + sl] = term;
        }
      }
    }
    if (a.S > 1) {
      __syncthreads();
      for (int e = threadIdx.x; e < a.R * T; e += kThreadsB) {
        const int r = e / T, t = e - r * T;
        const int row = row0 + r;
        if (row < a.d) {
          float v = part[e * a.S];
          for (int s = 1; s < a.S; ++s) v += part[e * a.S + s];
          a.y[static_cast<size_t>(a.t0 + t) * a.d + row] = v;
        }
      }
      __syncthreads();
    }
  }
}

namespace {

template <int T>
int launch_pass(BatchArgs a, cudaStream_t stream, const DeviceInfo& dev) {
  a.S = (a.n + 2047) / 2048;
  a.wps = kWarpsB / a.S;
  const int grid_cap = dev.sm_count;
  const long long warps_cap = static_cast<long long>(grid_cap) * a.wps;
  int rpw = static_cast<int>((a.d + warps_cap - 1) / warps_cap);
  if (rpw < 1) rpw = 1;
  if (rpw > 32) rpw = 32;
  a.rpw = rpw;
  a.R = a.wps * rpw;
  a.n_tiles = (a.d + a.R - 1) / a.R;
  const int grid = a.n_tiles < grid_cap ? a.n_tiles : grid_cap;
  const size_t smem = kSmemHeaderB + static_cast<size_t>(T) * a.n +
                      (a.S > 1 ? static_cast<size_t>(a.R) * T * a.S * 4 : 0);
  if (smem > static_cast<size_t>(dev.smem_optin_per_cta)) return set_status(MLI_ERR_UNSUPPORTED);
  cudaError_t err = cudaSuccess;
  err = ensure_dynamic_smem(reinterpret_cast<const void*>(gemm_w8a8_cuda_core_kernel<T>), smem);
  if (err == cudaSuccess)
    err = launch(gemm_w8a8_cuda_core_kernel<T>, dim3(grid), dim3(kThreadsB), smem, stream, true, a);
  return check_cuda(err);
}

}  // namespace

// CUDA-core batched W8A8: n % 256 == 0, n <= 16384, 16-byte aligned xq / w_q.
int gemm_w8a8_cuda_core(float* y, const int8_t* xq, const float* xs, const int8_t* w_q,
                        const float* w_s, int m, int n, int d, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  BatchArgs a = {};
  a.y = y; a.xq = xq; a.xs = xs; a.w = w_q; a.s = w_s; a.m = m; a.n = n; a.d = d;
  int t0 = 0;
  while (t0 < m) {
    const int left = m - t0;
    a.t0 = t0;
    int rc;
    if (left >= 8) { rc = launch_pass<8>(a, stream, dev); t0 += 8; }
    else if (left >= 4) { rc = launch_pass<4>(a, stream, dev); t0 += 4; }
    else if (left >= 2) { rc = launch_pass<2>(a, stream, dev); t0 += 2; }
    else { rc = launch_pass<1>(a, stream, dev); t0 += 1; }
    if (rc != MLI_OK) return rc;
  }
  return set_status(MLI_OK);
}

size_t gemm_tc_workspace_bytes(int m, int n, int d, int sm_count);
int gemm_w8a8_tc(float* y, const int8_t* xq, const float* xs, const int8_t* w_q, const float* w_s,
                 int m, int n, int d, void* workspace, size_t workspace_bytes, cudaStream_t stream);

}  // namespace mli

using namespace mli;

extern "C" {

size_t mli_gemm_w8a8_workspace_bytes(int m, int n, int d) {
  if (m <= 0 || n <= 0 || d <= 0) return 0;
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return 0;
  return gemm_tc_workspace_bytes(m, n, d, dev.sm_count);
}

int mli_gemm_w8a8(float* y, const int8_t* xq, const float* xs, const int8_t* w_q,
                  const float* w_s, int m, int n, int d, int group_size, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (!y || !xq || !xs || !w_q || !w_s || m <= 0 || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (group_size == 64 && m >= 16) {
    const int rc = gemm_w8a8_tc(y, xq, xs, w_q, w_s, m, n, d, workspace, workspace_bytes, st);
    if (rc != MLI_ERR_UNSUPPORTED) return rc;
  }
  if (group_size == 64 && n % 256 == 0 && n <= 16384 && aligned(xq, 16) && aligned(w_q, 16) &&
      aligned(w_s, 4))
    return gemm_w8a8_cuda_core(y, xq, xs, w_q, w_s, m, n, d, st);
  // Any other shape: one generic W8A8 GEMV per token.
  for (int t = 0; t < m; ++t) {
    const int rc = mli_gemv_w8a8(y + static_cast<size_t>(t) * d, xq + static_cast<size_t>(t) * n,
                                 xs + t, w_q, w_s, n, d, group_size, stream);
    if (rc != MLI_OK) return rc;
  }
  return set_status(MLI_OK);
}

/* The CUDA-core batched path alone (any m), for comparisons with the
 * tensor-core path. */
int mli_gemm_w8a8_cuda_core(float* y, const int8_t* xq, const float* xs, const int8_t* w_q,
                            const float* w_s, int m, int n, int d, int group_size, void* stream) {
  if (!y || !xq || !xs || !w_q || !w_s || m <= 0 || n <= 0 || d <= 0 || group_size != 64 ||
      n % 256 != 0 || n > 16384 || !aligned(xq, 16) || !aligned(w_q, 16))
    return set_status(MLI_ERR_INVALID_ARG);
  return gemm_w8a8_cuda_core(y, xq, xs, w_q, w_s, m, n, d, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
