// gemv_rows.cuh -- the per-row arithmetic of the batch-1 INT8 group-64 GEMV,
// shared by the single-GEMV streaming kernel (gemv_g64.cu) and the chained
// kernel (gemv_chain.cu), so that both give bit-identical rows.
//
//  * Activation prologues: the fp32 activation as four int8 digit planes
//    (W8A32) or quantised per token (fused W8A8), written once per CTA into
//    shared memory.
//  * Row kernels: one warp computes RB consecutive rows of one slice of a
//    stage held in shared memory.
#pragma once

#include "mli_common.cuh"

namespace mli {

constexpr int kGroup = 64;
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;

enum class Form : int { kW8A32 = 0, kW8A8 = 1, kW8A8Fused = 2 };

// 16-byte chunks per lane per row slice: a slice is 512 * K columns (8 * K
// groups).  W8A32 keeps its fp32 slice of x in 2 * 16 registers per lane,
// W8A8 its int8 slice in 4 * 4.
__host__ __device__ constexpr int chunks_per_lane(Form f) { return f == Form::kW8A32 ? 2 : 4; }
__host__ __device__ constexpr int slice_cols(Form f) { return 512 * chunks_per_lane(f); }
// Rows each consumer warp takes per stage (reduced together, see
// warp_sum_rows): enough independent work per pass to hide latency with only
// eight consumer warps per SM.
__host__ __device__ constexpr int rows_per_warp(Form f) { return f == Form::kW8A32 ? 4 : 2; }

// Activation loads.  kL2: bypass L1 (ld.global.cg), for activations that
// other SMs of the same kernel wrote and published through an acquire.
template <bool kL2>
__device__ __forceinline__ float4 load_x4(const float* p) {
  if constexpr (kL2) return __ldcg(reinterpret_cast<const float4*>(p));
  else return *reinterpret_cast<const float4*>(p);
}

// ---------------------------------------------------------------------------
// Activation prologues (consumer threads, once per CTA)
// ---------------------------------------------------------------------------
// W8A32 represents each 64-column group of the fp32 activation exactly enough
// for fp32 parity as four signed 7-bit int8 "digit planes" under a per-group
// power of two:  x~ = 2^-E (d1 + d2 2^-7 + d3 2^-14 + d4 2^-21),
// with E chosen so that max|x_g| * 2^E lies in [32, 64).  Every digit is in
// [-64, 64] and |x - x~| <= 2^-27 max|x_g| (well below the fp32 rounding of
// the dot product itself).  A weight chunk then costs 16 dp4a of exact int32
// partials P1..P4, combined as Q = 128 P1 + P2 and R = 128 P3 + P4 (both
// below 2^24, so exact in fp32):  sum_j w_j x~_j = 2^-(E+7) (Q + 2^-14 R).
//
// rint(u) for |u| <= 64 is (u + 1.5*2^23) - 1.5*2^23 (ties to even), and the
// low byte of the bits of u + 1.5*2^23 is the digit's two's-complement byte.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

// Digit bytes of one value; `u` is the value already scaled by 2^E.
__device__ __forceinline__ void digits4(float u, uint32_t (&t)[4]) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float r = u + kRoundMagic;
    t[p] = __float_as_uint(r);
    if (p < 3) u = (u - (r - kRoundMagic)) * 128.0f;
  }
}

// Digit planes and group factor of the four columns c..c+3 of x held by this
// lane (v; zero and not stored when !valid).  The 16 lanes of a half-warp
// hold one whole 64-column group; all 32 lanes of the warp take part.
__device__ __forceinline__ void digit_quad(const float4 v, bool valid, int c, int n,
                                           int8_t* planes, float* fac, int lane) {
  float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int off = 1; off < 16; off <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  const int e = static_cast<int>(__float_as_uint(m) >> 23);  // biased exponent of max|x_g|
  float scale_up, factor;
  if (e >= 13 && e <= 254) {
    scale_up = __uint_as_float(static_cast<uint32_t>(259 - e) << 23);  // 2^E, E = 132 - e
    factor = __uint_as_float(static_cast<uint32_t>(e - 12) << 23);    // 2^-(E + 7)
  } else if (e == 255) {  // inf / nan in the group: propagate
    scale_up = 0.f;
    factor = __uint_as_float(0x7fc00000u);
  } else {  // max|x_g| < 2^-114: the group contributes nothing measurable
    scale_up = 0.f;
    factor = 0.f;
  }
  uint32_t t0[4], t1[4], t2[4], t3[4];
  digits4(v.x * scale_up, t0);
  digits4(v.y * scale_up, t1);
  digits4(v.z * scale_up, t2);
  digits4(v.w * scale_up, t3);
  if (valid) {
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t lo = __byte_perm(t0[p], t1[p], 0x0040);
      const uint32_t hi = __byte_perm(t2[p], t3[p], 0x0040);
      *reinterpret_cast<uint32_t*>(planes + p * n + c) = __byte_perm(lo, hi, 0x5410);
    }
    if ((lane & 15) == 0) fac[c >> 6] = factor;
  }
}

// Writes the digit planes [4][n] int8 and the per-group factors 2^-(E+7)
// [n/64] of x into shared memory.  Thread t handles columns 4t + 1024j, so
// each half-warp holds one whole 64-column group.
template <bool kL2 = false>
__device__ __forceinline__ void x_digits_prologue(const float* x, int n, int8_t* planes,
                                                  float* fac) {
  const int lane = threadIdx.x & 31;
  for (int c0 = 0; c0 < n; c0 += 4 * kConsumerThreads) {
    const int c = c0 + 4 * threadIdx.x;
    const bool valid = c < n;
    const float4 v = valid ? load_x4<kL2>(x + c) : make_float4(0.f, 0.f, 0.f, 0.f);
    digit_quad(v, valid, c, n, planes, fac, lane);
  }
}

// Activation scale of the reference's quantiser from max|x|
// (src/model_cuda_v2_shared.cu:445-448).
__device__ __forceinline__ float act_scale(float amax) {
  float scale = amax / 127.0f;
  if (scale < 1e-8f) scale = 1e-8f;
  return scale;
}

// Four int8 codes clamp(rint(v * inv), +-127), packed little-endian.
__device__ __forceinline__ uint32_t quant_quad(const float4 v, float inv) {
  const int q0 = max(-127, min(127, __float2int_rn(v.x * inv)));
  const int q1 = max(-127, min(127, __float2int_rn(v.y * inv)));
  const int q2 = max(-127, min(127, __float2int_rn(v.z * inv)));
  const int q3 = max(-127, min(127, __float2int_rn(v.w * inv)));
  return (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) |
         (static_cast<uint32_t>(q3 & 0xff) << 24);
}

// Fused W8A8: quantises x into shared int8 [n], bit-identical to
// quantize_activation_kernel (src/model_cuda_v2_shared.cu:429-455).
// Returns the activation scale.
template <bool kL2 = false>
__device__ __forceinline__ float x_quant_prologue(const float* x, int n, int8_t* xq, float* red) {
  float m = 0.f;
  for (int c = 4 * threadIdx.x; c < n; c += 4 * kConsumerThreads) {
    const float4 v = load_x4<kL2>(x + c);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float amax = red[0];
#pragma unroll
  for (int w = 1; w < kConsumerWarps; ++w) amax = fmaxf(amax, red[w]);
  const float scale = act_scale(amax);
  const float inv = 1.0f / scale;
  for (int c = 4 * threadIdx.x; c < n; c += 4 * kConsumerThreads)
    *reinterpret_cast<uint32_t*>(xq + c) = quant_quad(load_x4<kL2>(x + c), inv);
  return scale;
}

// ---------------------------------------------------------------------------
// Consumer row kernels (one warp, one slice of RB consecutive rows)
// ---------------------------------------------------------------------------
__device__ __forceinline__ int dp4a_chunk(const uint4 w, const uint4 x) {
  int acc = __dp4a(static_cast<int>(w.x), static_cast<int>(x.x), 0);
  acc = __dp4a(static_cast<int>(w.y), static_cast<int>(x.y), acc);
  acc = __dp4a(static_cast<int>(w.z), static_cast<int>(x.z), acc);
  acc = __dp4a(static_cast<int>(w.w), static_cast<int>(x.w), acc);
  return acc;
}

// Per-lane W8A32 partials of RB consecutive rows (row stride n bytes in the
// stage, scale-row stride G floats).  Per 16-byte chunk k (group lane/4 + 8k):
// four digit-plane dots, combined exactly into Q, R, then one rounding into
// fp32 and one FMA with the group scale; chunks in order k = 0, 1.
template <int RB>
__device__ __forceinline__ void rows_w8a32(const int8_t* wr, const float* sr, int n, int G,
                                           int nvalid, const uint4 (&xd)[2][4],
                                           const float (&fac)[2], unsigned vmask, int lane,
                                           float (&out)[RB]) {
  uint4 w[RB][2];
  float sc[RB][2];
#pragma unroll
  for (int r = 0; r < RB; ++r) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const bool v = r < nvalid && ((vmask >> k) & 1u);
      w[r][k] = v ? *reinterpret_cast<const uint4*>(wr + r * n + 16 * (lane + 32 * k))
                  : make_uint4(0, 0, 0, 0);
      sc[r][k] = v ? sr[r * G + (lane >> 2) + 8 * k] : 0.f;
    }
  }
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int q = dp4a_chunk(w[r][k], xd[k][0]) * 128 + dp4a_chunk(w[r][k], xd[k][1]);
      const int rr = dp4a_chunk(w[r][k], xd[k][2]) * 128 + dp4a_chunk(w[r][k], xd[k][3]);
      const float v = fmaf(static_cast<float>(rr), 0x1p-14f, static_cast<float>(q));
      acc = fmaf(v * fac[k], sc[r][k], acc);
    }
    out[r] = acc;
  }
}

// Lane q of each quad holds int32 partials p[k] of group (lane/4 + 8k);
// afterwards it holds the quad's total of p[q].  Integer sums: exact.
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

// Per-lane W8A8 terms of RB consecutive rows: lane q of each quad ends with
// group (lane/4 + 8q)'s exact int32 dot and forms ((float)I * ws) * xs.
template <int RB>
__device__ __forceinline__ void rows_w8a8(const int8_t* wr, const float* sr, int n, int G,
                                          int nvalid, const uint4 (&xv)[4], unsigned vmask,
                                          int lane, float xscale, float (&out)[RB]) {
  uint4 w[RB][4];
#pragma unroll
  for (int r = 0; r < RB; ++r)
#pragma unroll
    for (int k = 0; k < 4; ++k)
      w[r][k] = (r < nvalid && ((vmask >> k) & 1u))
                    ? *reinterpret_cast<const uint4*>(wr + r * n + 16 * (lane + 32 * k))
                    : make_uint4(0, 0, 0, 0);
  const int q = lane & 3;
  const bool gvalid = (vmask >> q) & 1u;  // group lane/4 + 8q exists
#pragma unroll
  for (int r = 0; r < RB; ++r) {
    const int I = quad_reduce_scatter(dp4a_chunk(w[r][0], xv[0]), dp4a_chunk(w[r][1], xv[1]),
                                      dp4a_chunk(w[r][2], xv[2]), dp4a_chunk(w[r][3], xv[3]));
    const bool v = gvalid && r < nvalid;
    const float ws = v ? sr[r * G + (lane >> 2) + 8 * q] : 0.f;
    out[r] = v ? (static_cast<float>(I) * ws) * xscale : 0.f;
  }
}

}  // namespace mli
