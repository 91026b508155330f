// rowshard.cu -- row-sharded classifier support: peer buffers over CUDA IPC,
// device argmax, and the bounded wait that completes a sharded GEMV step.
//
// A row-sharded step on every rank is two launches on that rank's stream
// (or one, mli_gemv_rowshard_argmax, which does both):
//   1. mli_gemv_rowshard: the streaming GEMV over this rank's rows, storing
//      each output row, tagged with the step, straight into every rank's
//      logits words over NVLink, and each CTA's (max, first index) as one
//      tagged partial word into every rank's block;
//   2. mli_rowshard_wait_argmax: polls (bounded) every rank's partial words
//      of this step until their tags arrive, reduces them to the argmax and
//      advances the step counter (which also flips the half the next step
//      writes, so a slow rank still reading this step's half is never
//      overwritten).  No fence and no counter is needed: each word says by
//      itself whether it belongs to this step.
// The argmax replaces the reference's device-to-host copy of the logits and
// host argmax (src/main_cuda.cpp:96-98, src/model_cuda_v2_shared.cu:571-575)
// with the same first-maximum rule.
#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

constexpr int kArgmaxThreads = 1024;
constexpr int kWaitThreads = 256;

// Grid the row-sharded streaming GEMV uses for `rows` rows (gemv_g64.cu).
int rowshard_grid(int form, int n, int rows);

// Block-wide argmax of x[0..n) (every thread of a 1024-thread CTA calls it);
// returns the index on every thread.  Each thread scans its elements in
// increasing index order with a strict `>`, so its candidate is its first
// maximum; candidates then combine with argmax_combine (the reference's
// first-maximum rule).  Loads bypass L1:
// the values may have just been written by other GPUs.
__device__ __forceinline__ int block_argmax(const float* x, int n) {
  __shared__ float red_v[kArgmaxThreads / 32];
  __shared__ int red_i[kArgmaxThreads / 32];
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    // kUnroll independent 16-byte loads in flight per thread.
    constexpr int kUnroll = 8;
    const int n4 = n >> 2;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int base = 0; base < n4; base += kUnroll * kArgmaxThreads) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = base + u * kArgmaxThreads + threadIdx.x;
        v[u] = i < n4 ? __ldcg(x4 + i) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i = 4 * (base + u * kArgmaxThreads + threadIdx.x);
        if (v[u].x > bv) { bv = v[u].x; bi = i; }
        if (v[u].y > bv) { bv = v[u].y; bi = i + 1; }
        if (v[u].z > bv) { bv = v[u].z; bi = i + 2; }
        if (v[u].w > bv) { bv = v[u].w; bi = i + 3; }
      }
    }
    for (int i = 4 * n4 + threadIdx.x; i < n; i += kArgmaxThreads)
      if (__ldcg(x + i) > bv) { bv = __ldcg(x + i); bi = i; }
  } else {
    for (int i = threadIdx.x; i < n; i += kArgmaxThreads) {
      const float v = __ldcg(x + i);
      if (v > bv) { bv = v; bi = i; }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    argmax_combine(bv, bi, ov, oi);
  }
  if ((threadIdx.x & 31) == 0) {
    red_v[threadIdx.x >> 5] = bv;
    red_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  bv = red_v[0];
  bi = red_i[0];
#pragma unroll
  for (int w = 1; w < kArgmaxThreads / 32; ++w) argmax_combine(bv, bi, red_v[w], red_i[w]);
  __syncthreads();
  // The reference starts from x[0]: if it is NaN nothing ever compares
  // greater and the answer is 0; so it is when no element beat -inf.
  if (bi == 0x7fffffff || x[0] != x[0]) bi = 0;
  return bi;
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_kernel(const float* x, int n, long long* out) {
  griddep_wait();
  griddep_launch_dependents();  // the next GEMV may start streaming its weights now
  const int idx = block_argmax(x, n);
  if (threadIdx.x == 0) *out = idx;
}

struct WaitArgs {
  const unsigned long long* logits;  // this rank's logits words [2][d_total] (partials follow)
  unsigned* step;                    // this rank's step counter
  long long* out;
  int world, d_total;
  unsigned long long timeout_ns;
  int shard_ctas[kMaxPeers];         // CTAs (partial words) each rank writes per step
};

__global__ void __launch_bounds__(kWaitThreads) rowshard_wait_argmax_kernel(const WaitArgs a) {
  __shared__ float red_v[kWaitThreads / 32];
  __shared__ int red_i[kWaitThreads / 32];
  __shared__ int s_int;
  griddep_wait();
  // Let the next kernel launch and stream its weights during the wait; it
  // reads *step only after this kernel completes (its own griddepcontrol.wait).
  griddep_launch_dependents();
  const unsigned s = *a.step;
  const long long best = rowshard_poll_argmax<kWaitThreads>(a.logits, a.d_total, s & 1u, rowshard_tag(s), a.world,
                                                            a.shard_ctas, a.timeout_ns, red_v, red_i, &s_int);
  if (threadIdx.x == 0) {
    if (best < 0) record_device_error(kDevPeerTimeout);
    *a.out = best;
    if (best >= 0) *a.step = s + 1;
  }
}

}  // namespace mli

using namespace mli;

extern "C" {

int mli_peer_alloc(size_t bytes, void** ptr, unsigned char* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return set_status(MLI_ERR_INVALID_ARG);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    return check_cuda(e);
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return set_status(MLI_OK);
}

int mli_peer_open(const unsigned char* ipc_handle, void** ptr) {
  if (!ptr || !ipc_handle) return set_status(MLI_ERR_INVALID_ARG);
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int mli_peer_close(void* ptr) {
  if (!ptr) return set_status(MLI_ERR_INVALID_ARG);
  return check_cuda(cudaIpcCloseMemHandle(ptr));
}

int mli_peer_free(void* ptr) {
  if (!ptr) return set_status(MLI_ERR_INVALID_ARG);
  return check_cuda(cudaFree(ptr));
}

int mli_argmax(const float* x, int n, long long* out, void* stream) {
  if (!x || !out || n <= 0) return set_status(MLI_ERR_INVALID_ARG);
  return check_cuda(launch(argmax_kernel, dim3(1), dim3(kArgmaxThreads), 0,
                           static_cast<cudaStream_t>(stream), true, x, n, out));
}

int mli_rowshard_wait_argmax(int form, int n, const unsigned long long* logits, unsigned* step,
                             const int* shard_rows, int world, int d_total, long long* out,
                             int timeout_us, void* stream) {
  if (!logits || !step || !shard_rows || !out || world <= 0 || world > kMaxPeers ||
      d_total <= 0 || timeout_us <= 0 || n <= 0 || (form != 0 && form != 2))
    return set_status(MLI_ERR_INVALID_ARG);
  if (d_total >= kMaxRowshardRows) return set_status(MLI_ERR_UNSUPPORTED);
  WaitArgs a = {};
  a.logits = logits;
  a.step = step;
  a.out = out;
  a.world = world;
  a.d_total = d_total;
  a.timeout_ns = static_cast<unsigned long long>(timeout_us) * 1000ull;
  long long total = 0;
  for (int r = 0; r < world; ++r) {
    if (shard_rows[r] < 0) return set_status(MLI_ERR_INVALID_ARG);
    a.shard_ctas[r] = rowshard_grid(form, n, shard_rows[r]);
    if (a.shard_ctas[r] < 0 || a.shard_ctas[r] > kMaxRankCtas) return set_status(MLI_ERR_UNSUPPORTED);
    total += shard_rows[r];
  }
  if (total != d_total) return set_status(MLI_ERR_INVALID_ARG);
  return check_cuda(launch(rowshard_wait_argmax_kernel, dim3(1), dim3(kWaitThreads), 0,
                           static_cast<cudaStream_t>(stream), true, a));
}

size_t mli_rowshard_block_bytes(int d_total) {
  return d_total > 0 ? rowshard_block_bytes(d_total) : 0;
}

}  // extern "C"
