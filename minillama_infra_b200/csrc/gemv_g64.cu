// gemv_g64.cu -- batch-1 INT8 group-64 GEMV for B200 (sm_100a).
//
// Two forms of the reference's linear op (src/model_cuda_v2_shared.cu):
//   W8A32  y[r] = sum_c (q[r][c] * s[r][c/64]) * x[c]        (:36-62)
//   W8A8   y[r] = sum_g ((float)I[r][g] * s[r][g]) * xs     (:465-501)
//          I[r][g] = exact int32 dot of group g of row r with the int8 x.
//
// Design (HBM-bound: ~1 byte of weight per 2 flops):
//  * Every warp owns one "slice" of 2048 columns (32 groups).  Lane l covers
//    the 16-byte quarter (l & 3) of the four consecutive groups
//    4*(l >> 2) .. +3 of its slice, so one row costs each lane four 16-byte
//    streaming loads (64 bytes apart) plus one load of its scales.  Every
//    32-byte sector a warp touches is fully used.
//  * The activation slice a lane needs never changes from row to row, so it
//    lives in registers for the whole kernel: the CTA stages x once into
//    shared memory with one bulk (TMA-engine) copy, each warp then loads its
//    slice into registers.  Rows stream through a two-deep register pipeline.
//  * W8A32 converts int8 -> fp32 exactly with a byte-permute under a 2^23
//    exponent and packed fp32x2 subtract / FMA (two values per instruction).
//  * W8A8 does four dp4a per 16 bytes, a 3-shuffle quad reduce-scatter that
//    leaves each lane with one whole group's int32 dot, then the reference's
//    per-group fp32 term ((float)I * ws) * xs.  The fused variant quantises x
//    in every CTA's prologue, bit-identical to quantize_activation.
//  * Rows with more than one slice (n > 2048: split-K) are combined through
//    shared memory in slice order.  The arithmetic of one row depends only on
//    n: never on d, the tile, the grid or the GPU count, so a row-sharded
//    classifier returns bit-identical logits on any number of GPUs.
//  * Programmatic dependent launch: the first row's weights are requested
//    before griddepcontrol.wait, so a chain of GEMVs keeps HBM busy across
//    kernel boundaries.
#include <utility>

#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

constexpr int kGroup = 64;
constexpr int kSliceCols = 2048;
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSlices = 8;
constexpr int kMaxCols = kSliceCols * kMaxSlices;  // fast-path limit on n
constexpr int kSmemHeader = 128;                   // mbarrier + reduction scratch

struct GemvArgs {
  float* y;
  const float* x;     // fp32 activation (W8A32, fused W8A8)
  const int8_t* xq;   // int8 activation (W8A8)
  const float* xs;    // activation scale (W8A8)
  int8_t* xq_out;     // fused W8A8: optional copy of the quantised x
  float* xs_out;      //             and of its scale
  const int8_t* w;
  const float* s;
  int n, d;
  int S;        // slices per row = ceil(n / 2048)
  int wps;      // warps per slice = 8 / S
  int rpw;      // rows per warp per tile
  int R;        // rows per tile = wps * rpw
  int n_tiles;  // ceil(d / R)
};

// Work split of one CTA: which warp handles which slice / rows.
struct WarpRole {
  int sl, wj;
  bool warp_on, lane_on;
  int g0;    // first of the lane's four groups (row-relative group index)
  int col0;  // first column of the lane's chunk 0
  __device__ WarpRole(const GemvArgs& a) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    sl = warp % a.S;
    wj = warp / a.S;
    warp_on = wj < a.wps;
    g0 = sl * 32 + (lane >> 2) * 4;
    lane_on = warp_on && g0 < (a.n >> 6);
    col0 = g0 * kGroup + (lane & 3) * 16;
  }
};

__device__ __forceinline__ int my_tile_count(const GemvArgs& a) {
  return blockIdx.x < static_cast<unsigned>(a.n_tiles)
             ? (a.n_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
             : 0;
}

// Row handled by this warp at flattened position idx (tile-major).
__device__ __forceinline__ int row_at(const GemvArgs& a, int wj, int idx) {
  const int t = idx / a.rpw;
  const int i = idx - t * a.rpw;
  return (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * a.R + wj + i * a.wps;
}

// Stage `bytes` from global into shared memory with one bulk copy.  Returns
// false (on every thread) if the copy did not land within the wait limit.
__device__ __forceinline__ bool stage_to_smem(void* dst, const void* src,
                                              uint32_t bytes, uint64_t* bar) {
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
    mbar_arrive_expect_tx(bar, bytes);
    bulk_copy_g2s(dst, src, bytes, bar);
  }
  __syncthreads();
  const bool ok = mbar_wait_bounded(bar, 0, kWaitLimitNs);
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) {
      record_device_error(kDevStageTimeout);
      mbar_wait_bounded(bar, 0, kWaitLimitNs);  // let an in-flight copy drain
    }
    return false;
  }
  return true;
}

// Combine the per-slice partial sums of one tile in slice order.
__device__ __forceinline__ void combine_slices(const GemvArgs& a,
                                               const float* part, int row0) {
  for (int r = threadIdx.x; r < a.R; r += kThreads) {
    const int row = row0 + r;
    if (row < a.d) {
      float v = part[r * a.S];
      for (int s = 1; s < a.S; ++s) v += part[r * a.S + s];
      a.y[row] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// W8A32
// ---------------------------------------------------------------------------
struct RowW8A32 {
  uint4 w[4];
  float4 s;
};

__device__ __forceinline__ void load_row_w8a32(const GemvArgs& a,
                                               const WarpRole& role, int row,
                                               RowW8A32& r) {
  if (role.lane_on && row < a.d) {
    const int8_t* p = a.w + static_cast<size_t>(row) * a.n + role.col0;
    r.w[0] = ldg_stream_u4(p);
    r.w[1] = ldg_stream_u4(p + 64);
    r.w[2] = ldg_stream_u4(p + 128);
    r.w[3] = ldg_stream_u4(p + 192);
    r.s = ldg_f4(a.s + static_cast<size_t>(row) * (a.n >> 6) + role.g0);
  } else {
    r.w[0] = r.w[1] = r.w[2] = r.w[3] = make_uint4(0, 0, 0, 0);
    r.s = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Dot of one lane's 64 weights with its register-resident activations.
// Per 16-byte chunk: sum_j w_j x_j in two interleaved fp32 lanes, then one
// FMA with the group scale.
__device__ __forceinline__ float dot_w8a32(const RowW8A32& r,
                                           const float2 (&xr)[4][8]) {
  const float2 m = make_float2(-kI8Magic, -kI8Magic);
  const float sv[4] = {r.s.x, r.s.y, r.s.z, r.s.w};
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t u0 = r.w[k].x ^ 0x80808080u;
    const uint32_t u1 = r.w[k].y ^ 0x80808080u;
    const uint32_t u2 = r.w[k].z ^ 0x80808080u;
    const uint32_t u3 = r.w[k].w ^ 0x80808080u;
    float2 p = mul2(add2(biased_pair<0>(u0), m), xr[k][0]);
    p = fma2(add2(biased_pair<1>(u0), m), xr[k][1], p);
    p = fma2(add2(biased_pair<0>(u1), m), xr[k][2], p);
    p = fma2(add2(biased_pair<1>(u1), m), xr[k][3], p);
    p = fma2(add2(biased_pair<0>(u2), m), xr[k][4], p);
    p = fma2(add2(biased_pair<1>(u2), m), xr[k][5], p);
    p = fma2(add2(biased_pair<0>(u3), m), xr[k][6], p);
    p = fma2(add2(biased_pair<1>(u3), m), xr[k][7], p);
    acc = fmaf(p.x + p.y, sv[k], acc);
  }
  return acc;
}

__global__ void __launch_bounds__(kThreads, 2)
    gemv_w8a32_g64_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  float* xsm = reinterpret_cast<float*>(smem + kSmemHeader);
  float* part = xsm + a.n;  // [R][S] slice partials (S > 1)

  const WarpRole role(a);
  const int lane = threadIdx.x & 31;
  const int my_tiles = my_tile_count(a);
  const int total = my_tiles * a.rpw;

  // Weights do not depend on the previous kernel: request the first row now.
  RowW8A32 cur;
  load_row_w8a32(a, role, total > 0 && role.warp_on ? row_at(a, role.wj, 0) : a.d, cur);

  griddep_wait();
  if (!stage_to_smem(xsm, a.x, static_cast<uint32_t>(a.n) * 4u, bar)) return;
  griddep_launch_dependents();

  float2 xr[4][8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (role.lane_on) v = *reinterpret_cast<const float4*>(xsm + role.col0 + 64 * k + 4 * p);
      xr[k][2 * p] = make_float2(v.x, v.y);
      xr[k][2 * p + 1] = make_float2(v.z, v.w);
    }
  }

  int idx = 0;
  for (int t = 0; t < my_tiles; ++t) {
    const int row0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * a.R;
    for (int i = 0; i < a.rpw; ++i, ++idx) {
      const int row = row0 + role.wj + i * a.wps;
      RowW8A32 nxt;
      load_row_w8a32(a, role, (idx + 1 < total && role.warp_on) ? row_at(a, role.wj, idx + 1) : a.d, nxt);
      if (role.warp_on && row < a.d) {
        float acc = role.lane_on ? dot_w8a32(cur, xr) : 0.f;
        acc = warp_sum(acc);
        if (lane == 0) {
          if (a.S == 1) a.y[row] = acc;
          else part[(role.wj + i * a.wps) * a.S + role.sl] = acc;
        }
      }
      cur = nxt;
    }
    if (a.S > 1) {
      __syncthreads();
      combine_slices(a, part, row0);
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// W8A8 (dp4a)
// ---------------------------------------------------------------------------
struct RowW8A8 {
  uint4 w[4];
  float s;
};

__device__ __forceinline__ void load_row_w8a8(const GemvArgs& a,
                                              const WarpRole& role, int row,
                                              RowW8A8& r) {
  if (role.lane_on && row < a.d) {
    const int8_t* p = a.w + static_cast<size_t>(row) * a.n + role.col0;
    r.w[0] = ldg_stream_u4(p);
    r.w[1] = ldg_stream_u4(p + 64);
    r.w[2] = ldg_stream_u4(p + 128);
    r.w[3] = ldg_stream_u4(p + 192);
    r.s = ldg_f1(a.s + static_cast<size_t>(row) * (a.n >> 6) + role.g0 + (threadIdx.x & 3));
  } else {
    r.w[0] = r.w[1] = r.w[2] = r.w[3] = make_uint4(0, 0, 0, 0);
    r.s = 0.f;
  }
}

__device__ __forceinline__ int dp4a_chunk(const uint4 w, const uint4 x) {
  int acc = __dp4a(static_cast<int>(w.x), static_cast<int>(x.x), 0);
  acc = __dp4a(static_cast<int>(w.y), static_cast<int>(x.y), acc);
  acc = __dp4a(static_cast<int>(w.z), static_cast<int>(x.z), acc);
  acc = __dp4a(static_cast<int>(w.w), static_cast<int>(x.w), acc);
  return acc;
}

// Lane q of each quad holds int32 partials p[k] (its 16 columns of group k);
// afterwards it holds group q's full 64-column dot.  Integer sums: exact.
__device__ __forceinline__ int quad_reduce_scatter(int p0, int p1, int p2, int p3) {
  const int q = threadIdx.x & 3;
  const bool b0 = q & 1;
  int keep_a = b0 ? p1 : p0, send_a = b0 ? p0 : p1;
  int keep_b = b0 ? p3 : p2, send_b = b0 ? p2 : p3;
  keep_a += __shfl_xor_sync(0xffffffffu, send_a, 1);
  keep_b += __shfl_xor_sync(0xffffffffu, send_b, 1);
  const bool b1 = q & 2;
  int keep = b1 ? keep_b : keep_a, send = b1 ? keep_a : keep_b;
  keep += __shfl_xor_sync(0xffffffffu, send, 2);
  return keep;
}

// Per-token quantisation of the staged fp32 x into shared int8, bit-identical
// to quantize_activation_kernel (src/model_cuda_v2_shared.cu:429-455).
// Returns the activation scale.
__device__ __forceinline__ float quantize_staged(const float* xf, int8_t* xq, int n,
                                 float* red) {
  float m = 0.f;
  for (int i = threadIdx.x; i < n; i += kThreads) m = fmaxf(m, fabsf(xf[i]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) amax = fmaxf(amax, red[w]);
  float scale = amax / 127.0f;
  if (scale < 1e-8f) scale = 1e-8f;
  const float inv = 1.0f / scale;
  for (int i = threadIdx.x * 4; i < n; i += kThreads * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xf + i);
    const int q0 = max(-127, min(127, __float2int_rn(v.x * inv)));
    const int q1 = max(-127, min(127, __float2int_rn(v.y * inv)));
    const int q2 = max(-127, min(127, __float2int_rn(v.z * inv)));
    const int q3 = max(-127, min(127, __float2int_rn(v.w * inv)));
    const uint32_t packed = (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) |
                            (static_cast<uint32_t>(q3 & 0xff) << 24);
    *reinterpret_cast<uint32_t*>(xq + i) = packed;
  }
  return scale;
}

template <bool kFused>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_w8a8_g64_kernel(const GemvArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
  float* red = reinterpret_cast<float*>(smem + 16);
  float* xf = reinterpret_cast<float*>(smem + kSmemHeader);
  int8_t* xqs = reinterpret_cast<int8_t*>(smem + kSmemHeader) + (kFused ? 4 * a.n : 0);
  float* part = reinterpret_cast<float*>(xqs + a.n);

  const WarpRole role(a);
  const int lane = threadIdx.x & 31;
  const int my_tiles = my_tile_count(a);
  const int total = my_tiles * a.rpw;

  RowW8A8 cur;
  load_row_w8a8(a, role, total > 0 && role.warp_on ? row_at(a, role.wj, 0) : a.d, cur);

  griddep_wait();
  float xscale;
  if (kFused) {
    if (!stage_to_smem(xf, a.x, static_cast<uint32_t>(a.n) * 4u, bar)) return;
    xscale = quantize_staged(xf, xqs, a.n, red);
    __syncthreads();
    if (blockIdx.x == 0) {
      if (a.xq_out != nullptr) {
        if ((reinterpret_cast<uintptr_t>(a.xq_out) & 15) == 0) {
          for (int i = threadIdx.x * 16; i < a.n; i += kThreads * 16)
            *reinterpret_cast<uint4*>(a.xq_out + i) = *reinterpret_cast<const uint4*>(xqs + i);
        } else {
          for (int i = threadIdx.x; i < a.n; i += kThreads) a.xq_out[i] = xqs[i];
        }
      }
      if (a.xs_out != nullptr && threadIdx.x == 0) *a.xs_out = xscale;
    }
  } else {
    if (!stage_to_smem(xqs, a.xq, static_cast<uint32_t>(a.n), bar)) return;
    xscale = *a.xs;
  }
  griddep_launch_dependents();

  uint4 xv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    xv[k] = role.lane_on ? *reinterpret_cast<const uint4*>(xqs + role.col0 + 64 * k)
                         : make_uint4(0, 0, 0, 0);

  int idx = 0;
  for (int t = 0; t < my_tiles; ++t) {
    const int row0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * a.R;
    for (int i = 0; i < a.rpw; ++i, ++idx) {
      const int row = row0 + role.wj + i * a.wps;
      RowW8A8 nxt;
      load_row_w8a8(a, role, (idx + 1 < total && role.warp_on) ? row_at(a, role.wj, idx + 1) : a.d, nxt);
      if (role.warp_on && row < a.d) {
        const int I = quad_reduce_scatter(dp4a_chunk(cur.w[0], xv[0]), dp4a_chunk(cur.w[1], xv[1]),
                                          dp4a_chunk(cur.w[2], xv[2]), dp4a_chunk(cur.w[3], xv[3]));
        float term = role.lane_on ? (static_cast<float>(I) * cur.s) * xscale : 0.f;
        term = warp_sum(term);
        if (lane == 0) {
          if (a.S == 1) a.y[row] = term;
          else part[(role.wj + i * a.wps) * a.S + role.sl] = term;
        }
      }
      cur = nxt;
    }
    if (a.S > 1) {
      __syncthreads();
      combine_slices(a, part, row0);
      __syncthreads();
    }
  }
}

// ---------------------------------------------------------------------------
// Generic kernels: any group size, any n, any alignment.  One warp per row,
// byte loads; the reference's semantics (columns past (n / gs) * gs are
// ignored, as its groups_per_row = n / group_size truncates).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    gemv_w8a32_generic_kernel(float* y, const float* x, const int8_t* w,
                              const float* s, int n, int d, int gs) {
  griddep_wait();
  const int row = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= d) return;
  const int ng = n / gs;
  const int8_t* wr = w + static_cast<size_t>(row) * n;
  const float* sr = s + static_cast<size_t>(row) * ng;
  float acc = 0.f;
  for (int g = 0; g < ng; ++g) {
    float part = 0.f;
    for (int j = lane; j < gs; j += 32)
      part = fmaf(static_cast<float>(wr[g * gs + j]), x[g * gs + j], part);
    acc = fmaf(part, sr[g], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) y[row] = acc;
}

__global__ void __launch_bounds__(256)
    gemv_w8a8_generic_kernel(float* y, const int8_t* xq, const float* xs,
                             const int8_t* w, const float* s, int n, int d,
                             int gs) {
  griddep_wait();
  const int row = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= d) return;
  const int ng = n / gs;
  const int8_t* wr = w + static_cast<size_t>(row) * n;
  const float* sr = s + static_cast<size_t>(row) * ng;
  const float xscale = *xs;
  float acc = 0.f;
  for (int g = 0; g < ng; ++g) {
    int part = 0;
    for (int j = lane; j < gs; j += 32)
      part += static_cast<int>(wr[g * gs + j]) * static_cast<int>(xq[g * gs + j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    acc += (static_cast<float>(part) * sr[g]) * xscale;
  }
  if (lane == 0) y[row] = acc;
}

__global__ void __launch_bounds__(256)
    group_dots_kernel(int32_t* out, const int8_t* xq, const int8_t* w, int n,
                      int d, int gs) {
  const int ng = n / gs;
  const size_t total = static_cast<size_t>(d) * ng;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t row = i / ng;
    const int g = static_cast<int>(i - row * ng);
    const int8_t* wr = w + row * n + static_cast<size_t>(g) * gs;
    const int8_t* xr = xq + static_cast<size_t>(g) * gs;
    int acc = 0;
    for (int j = 0; j < gs; ++j) acc += static_cast<int>(wr[j]) * static_cast<int>(xr[j]);
    out[i] = acc;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

enum class Form { kW8A32, kW8A8, kW8A8Fused };

size_t smem_bytes(Form f, int n, int R, int S) {
  size_t stage = 0;
  switch (f) {
    case Form::kW8A32: stage = 4u * n; break;
    case Form::kW8A8: stage = n; break;
    case Form::kW8A8Fused: stage = 5u * n; break;
  }
  const size_t part = (S > 1) ? static_cast<size_t>(R) * S * 4u : 0;
  return kSmemHeader + ((stage + 15) & ~size_t(15)) + part;
}

// Tiles sized so that one wave of resident CTAs covers the matrix.
GemvArgs plan(Form f, const DeviceInfo& dev, int n, int d, size_t* smem_out,
              int* grid_out) {
  GemvArgs a = {};
  a.n = n;
  a.d = d;
  a.S = (n + kSliceCols - 1) / kSliceCols;
  a.wps = kWarps / a.S;
  const size_t smem0 = smem_bytes(f, n, 0, 1);
  int ctas_per_sm = 2;
  while (ctas_per_sm > 1 && static_cast<size_t>(ctas_per_sm) * (smem0 + 1024 + 8192) >
                                static_cast<size_t>(dev.smem_per_sm))
    --ctas_per_sm;
  const int grid_cap = dev.sm_count * ctas_per_sm;
  const long long warps_cap = static_cast<long long>(grid_cap) * a.wps;
  int rpw = static_cast<int>((d + warps_cap - 1) / warps_cap);
  if (rpw < 1) rpw = 1;
  if (rpw > 64) rpw = 64;
  a.rpw = rpw;
  a.R = a.wps * rpw;
  a.n_tiles = (d + a.R - 1) / a.R;
  *grid_out = a.n_tiles < grid_cap ? a.n_tiles : grid_cap;
  *smem_out = smem_bytes(f, n, a.R, a.S);
  return a;
}

bool fast_path_ok(int n, int group_size) {
  return group_size == kGroup && n % 256 == 0 && n <= kMaxCols;
}

template <typename K>
cudaError_t ensure_smem_attr(K kernel, size_t smem) {
  return ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
}

int launch_fast(Form f, GemvArgs args, cudaStream_t stream) {
  cudaError_t err = cudaSuccess;
  const DeviceInfo& dev = current_device(&err);
  if (err != cudaSuccess) return set_status(MLI_ERR_CUDA, err);
  size_t smem = 0;
  int grid = 0;
  GemvArgs p = plan(f, dev, args.n, args.d, &smem, &grid);
  p.y = args.y;
  p.x = args.x;
  p.xq = args.xq;
  p.xs = args.xs;
  p.xq_out = args.xq_out;
  p.xs_out = args.xs_out;
  p.w = args.w;
  p.s = args.s;
  if (smem > static_cast<size_t>(dev.smem_optin_per_cta)) return set_status(MLI_ERR_UNSUPPORTED);
  switch (f) {
    case Form::kW8A32:
      err = ensure_smem_attr(gemv_w8a32_g64_kernel, smem);
      if (err == cudaSuccess)
        err = launch(gemv_w8a32_g64_kernel, dim3(grid), dim3(kThreads), smem, stream, true, p);
      break;
    case Form::kW8A8:
      err = ensure_smem_attr(gemv_w8a8_g64_kernel<false>, smem);
      if (err == cudaSuccess)
        err = launch(gemv_w8a8_g64_kernel<false>, dim3(grid), dim3(kThreads), smem, stream, true, p);
      break;
    case Form::kW8A8Fused:
      err = ensure_smem_attr(gemv_w8a8_g64_kernel<true>, smem);
      if (err == cudaSuccess)
        err = launch(gemv_w8a8_g64_kernel<true>, dim3(grid), dim3(kThreads), smem, stream, true, p);
      break;
  }
  return check_cuda(err);
}

dim3 warp_per_row_grid(int d) { return dim3(static_cast<unsigned>((d + 7) / 8)); }

}  // namespace

// Launches the quantiser of one token (quant.cu).
int launch_quantize_rows(int8_t* xq, float* xs, const float* x, int m, int n,
                         cudaStream_t stream);

}  // namespace mli

using namespace mli;

extern "C" {

int mli_gemv_w8a32(float* y, const float* x, const int8_t* w_q, const float* w_s,
                   int n, int d, int group_size, void* stream) {
  if (!y || !x || !w_q || !w_s || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fast_path_ok(n, group_size) && aligned(x, 16) && aligned(w_q, 16) && aligned(w_s, 16)) {
    GemvArgs a = {};
    a.y = y; a.x = x; a.w = w_q; a.s = w_s; a.n = n; a.d = d;
    return launch_fast(Form::kW8A32, a, st);
  }
  return check_cuda(launch(gemv_w8a32_generic_kernel, warp_per_row_grid(d), dim3(256), 0, st,
                           true, y, x, w_q, w_s, n, d, group_size));
}

int mli_gemv_w8a8(float* y, const int8_t* xq, const float* xs, const int8_t* w_q,
                  const float* w_s, int n, int d, int group_size, void* stream) {
  if (!y || !xq || !xs || !w_q || !w_s || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fast_path_ok(n, group_size) && aligned(xq, 16) && aligned(w_q, 16) && aligned(w_s, 4)) {
    GemvArgs a = {};
    a.y = y; a.xq = xq; a.xs = xs; a.w = w_q; a.s = w_s; a.n = n; a.d = d;
    return launch_fast(Form::kW8A8, a, st);
  }
  return check_cuda(launch(gemv_w8a8_generic_kernel, warp_per_row_grid(d), dim3(256), 0, st,
                           true, y, xq, xs, w_q, w_s, n, d, group_size));
}

int mli_gemv_w8a8_fused(float* y, int8_t* xq_out, float* xs_out, const float* x,
                        const int8_t* w_q, const float* w_s, int n, int d,
                        int group_size, void* stream) {
  if (!y || !x || !w_q || !w_s || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  if ((xq_out == nullptr) != (xs_out == nullptr)) return set_status(MLI_ERR_INVALID_ARG);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fast_path_ok(n, group_size) && aligned(x, 16) && aligned(w_q, 16) && aligned(w_s, 4)) {
    GemvArgs a = {};
    a.y = y; a.x = x; a.xq_out = xq_out; a.xs_out = xs_out; a.w = w_q; a.s = w_s;
    a.n = n; a.d = d;
    return launch_fast(Form::kW8A8Fused, a, st);
  }
  // Unfused fallback for shapes outside the fast path: needs caller buffers.
  if (xq_out == nullptr) return set_status(MLI_ERR_UNSUPPORTED);
  int rc = launch_quantize_rows(xq_out, xs_out, x, 1, n, st);
  if (rc != MLI_OK) return rc;
  return mli_gemv_w8a8(y, xq_out, xs_out, w_q, w_s, n, d, group_size, stream);
}

int mli_debug_group_dots(int32_t* out, const int8_t* xq, const int8_t* w_q, int n,
                         int d, int group_size, void* stream) {
  if (!out || !xq || !w_q || n <= 0 || d <= 0 || group_size <= 0)
    return set_status(MLI_ERR_INVALID_ARG);
  const size_t total = static_cast<size_t>(d) * (n / group_size);
  const unsigned blocks = static_cast<unsigned>((total + 255) / 256 < 65535 ? (total + 255) / 256 : 65535);
  return check_cuda(launch(group_dots_kernel, dim3(blocks > 0 ? blocks : 1), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), false, out, xq, w_q, n, d,
                           group_size));
}

}  // extern "C"
