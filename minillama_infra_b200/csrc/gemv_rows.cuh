// gemv_rows.cuh -- the per-row arithmetic of the batch-1 INT8 group-64 GEMV,
// shared by the single-GEMV streaming kernel (gemv_g64.cu) and the chained
// kernel (gemv_chain.cu), so that both give bit-identical rows.
//
//  * Activation prologues: the fp32 activation as two int16 planes of 7-bit
//    digit pairs (W8A32) or quantised per token (fused W8A8), written once per
//    CTA into shared memory.
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
// for fp32 parity as four signed 7-bit digits under a per-group power of two:
//   x~ = 2^-E (d1 + d2 2^-7 + d3 2^-14 + d4 2^-21),
// with E chosen so that max|x_g| * 2^E lies in [32, 64).  Every digit is in
// [-64, 64] and |x - x~| <= 2^-27 max|x_g| (well below the fp32 rounding of
// the dot product itself).  The digits are kept in pairs, as two signed 14-bit
// planes C1 = 128 d1 + d2 and C2 = 128 d3 + d4 (int16, |C| <= 8256): a weight
// chunk of 16 columns costs 16 dp2a (int16 x int8 pairs) of exact int32 sums
//   Q = sum w C1 = 128 P1 + P2,  R = sum w C2 = 128 P3 + P4
// (P the four digit-plane dots; both below 2^24, so exact in fp32):
//   sum_j w_j x~_j = 2^-(E+7) (Q + 2^-14 R).
// With u = x 2^E: C1 = rint(128 u) and C2 = rint((128 u - C1) 2^14), ties to
// even -- the same integers as the four digits taken one at a time (each
// digit's remainder is exact, and adding 128 d1, an even integer, leaves a
// tie's rounding unchanged).
//
// rint(s) for |s| < 2^22 is (s + 1.5*2^23) - 1.5*2^23 (ties to even), and the
// bits of s + 1.5*2^23 minus those of 1.5*2^23 are rint(s) as an integer.
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

// The two 14-bit digit pairs of one value; `u` is the value already scaled
// by 2^E.
__device__ __forceinline__ void digit_pairs(float u, int& c1, int& c2) {
  const float s = u * 128.0f;
  const float r = s + kRoundMagic;
  c1 = __float_as_int(r) - __float_as_int(kRoundMagic);
  const float t = (s - (r - kRoundMagic)) * 16384.0f;
  c2 = __float_as_int(t + kRoundMagic) - __float_as_int(kRoundMagic);
}

// Two int16 (low halves of a, b) as one word: a in the low half.
__device__ __forceinline__ uint32_t pack16(int a, int b) {
  return __byte_perm(static_cast<uint32_t>(a), static_cast<uint32_t>(b), 0x5410);
}

// Shared-memory digit planes: [2][n] int16 (C1 then C2), then the group
// factors.  A lane's 16 columns cc .. cc+15 (cc a multiple of 16) as
// xd[0..1] = C1 of columns cc..cc+7, cc+8..cc+15 and xd[2..3] = C2 likewise.
__device__ __forceinline__ void load_digit_chunk(const int8_t* planes, int n, int cc, uint4 (&xd)[4]) {
  const uint4* p1 = reinterpret_cast<const uint4*>(planes + 2 * cc);
  const uint4* p2 = reinterpret_cast<const uint4*>(planes + 2 * n + 2 * cc);
  xd[0] = p1[0];
  xd[1] = p1[1];
  xd[2] = p2[0];
  xd[3] = p2[1];
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
  int a1, a2, b1, b2, c1, c2, d1, d2;
  digit_pairs(v.x * scale_up, a1, a2);
  digit_pairs(v.y * scale_up, b1, b2);
  digit_pairs(v.z * scale_up, c1, c2);
  digit_pairs(v.w * scale_up, d1, d2);
  if (valid) {
    *reinterpret_cast<uint2*>(planes + 2 * c) = make_uint2(pack16(a1, b1), pack16(c1, d1));
    *reinterpret_cast<uint2*>(planes + 2 * n + 2 * c) = make_uint2(pack16(a2, b2), pack16(c2, d2));
    if ((lane & 15) == 0) fac[c >> 6] = factor;
  }
}

// Writes the digit planes [2][n] int16 and the per-group factors 2^-(E+7)
// [n/64] of x into shared memory (4n bytes, then the factors).  Thread t
// handles columns 4t + 1024j, so each half-warp holds one whole 64-column
// group.
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
// Sum over the 16 columns of a weight chunk of w * C, C the int16 digit pairs
// of columns 0..7 (lo) and 8..15 (hi).
__device__ __forceinline__ int dp2a_chunk(const uint4 w, const uint4 lo, const uint4 hi) {
  int acc = __dp2a_lo(static_cast<int>(lo.x), static_cast<int>(w.x), 0);
  acc = __dp2a_hi(static_cast<int>(lo.y), static_cast<int>(w.x), acc);
  acc = __dp2a_lo(static_cast<int>(lo.z), static_cast<int>(w.y), acc);
  acc = __dp2a_hi(static_cast<int>(lo.w), static_cast<int>(w.y), acc);
  acc = __dp2a_lo(static_cast<int>(hi.x), static_cast<int>(w.z), acc);
  acc = __dp2a_hi(static_cast<int>(hi.y), static_cast<int>(w.z), acc);
  acc = __dp2a_lo(static_cast<int>(hi.z), static_cast<int>(w.w), acc);
  acc = __dp2a_hi(static_cast<int>(hi.w), static_cast<int>(w.w), acc);
  return acc;
}

__device__ __forceinline__ int dp4a_chunk(const uint4 w, const uint4 x) {
  int acc = __dp4a(static_cast<int>(w.x), static_cast<int>(x.x), 0);
  acc = __dp4a(static_cast<int>(w.y), static_cast<int>(x.y), acc);
  acc = __dp4a(static_cast<int>(w.z), static_cast<int>(x.z), acc);
  acc = __dp4a(static_cast<int>(w.w), static_cast<int>(x.w), acc);
  return acc;
}

// Per-lane W8A32 partials of RB consecutive rows (row stride n bytes in the
// stage, scale-row stride G floats).  Per 16-byte chunk k (group lane/4 + 8k):
// the two digit-pair dots Q, R (exact int32), then one rounding into fp32
// and one FMA with the group scale; chunks in order k = 0, 1.
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
      const int q = dp2a_chunk(w[r][k], xd[k][0], xd[k][1]);
      const int rr = dp2a_chunk(w[r][k], xd[k][2], xd[k][3]);
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
