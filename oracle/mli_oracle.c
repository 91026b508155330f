/*
 * mli_oracle.c -- CPU restatement of MiniLlama-Infra's INT8 group-64 linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library under minillama_infra_b200/.  Only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg load it; the product path never calls it.
 *
 * Every function restates one reference routine, in the reference's own
 * arithmetic order, so that its outputs are bit-identical to the reference:
 *
 *   oracle_quantize_weights   scripts/quantize_int8_group.py:55-71
 *   oracle_quantize_activation src/model_cuda_v2_shared.cu:429-455
 *   oracle_gemv_w8a32         src/model_cuda_v2_shared.cu:36-62 (+ warpReduceSum :30-34)
 *   oracle_gemv_w8a8          src/model_cuda_v2_shared.cu:465-501
 *   oracle_matmul_f32         src/model_cuda_v2_shared.cu:10-19 (fp32 classifier)
 *   oracle_rmsnorm_chain      src/model_cuda_v2_shared.cu:74-89 in the chained prologue's order
 *   oracle_group_dots         the exact int32 group partials of :483-494
 *   oracle_dequant_matvec     float32 dequant-then-matvec (CPU baseline, OpenMP)
 *   oracle_gemv_*_f64         fp64 recomputes used as tolerance anchors
 *
 * Build with -ffp-contract=off: every fused multiply-add the reference's nvcc
 * build emits is spelled out with fmaf() here, and nothing else may fuse.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float absf_(float v) { return v < 0.0f ? -v : v; }

/* scripts/quantize_int8_group.py:55-64.  Per row, per group of `gs` columns:
 *   amax = max|w| (fp32), amax == 0 -> float32(1e-9)            (:58-59)
 *   scale = amax / 127.0  (fp32 division; numpy keeps float32)  (:60)
 *   q = clip(round_half_even(w / scale), -127, 127)             (:63-64)
 * Output layout (:67-71): scales [rows][cols/gs] fp32, int8 [rows][cols]. */
int oracle_quantize_weights(int8_t* q, float* s, const float* w, long rows,
                            long cols, int gs) {
  if (gs <= 0 || cols % gs != 0) return 1;
  long ng = cols / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < rows; ++r) {
    for (long g = 0; g < ng; ++g) {
      const float* src = w + r * cols + g * gs;
      float amax = 0.0f;
      for (int j = 0; j < gs; ++j) {
        float a = absf_(src[j]);
        if (a > amax) amax = a;
      }
      if (amax == 0.0f) amax = 1e-9f;
      float scale = amax / 127.0f;
      s[r * ng + g] = scale;
      for (int j = 0; j < gs; ++j) {
        float v = nearbyintf(src[j] / scale); /* round-half-even (fenv default) */
        if (v > 127.0f) v = 127.0f;
        if (v < -127.0f) v = -127.0f;
        q[r * cols + g * gs + j] = (int8_t)v;
      }
    }
  }
  return 0;
}

/* src/model_cuda_v2_shared.cu:429-455 (one token of n values):
 *   amax = max|x| (exact; the float-bits atomicMax of :441-442 is an exact max
 *   for non-negative floats), scale = amax / 127.0f, clamp to >= 1e-8f,
 *   inv = 1.0f / scale, q = clamp(__float2int_rn(x * inv), -127, 127). */
void oracle_quantize_activation(int8_t* xq, float* xs, const float* x, long n) {
  float amax = 0.0f;
  for (long i = 0; i < n; ++i) amax = fmaxf(amax, absf_(x[i]));
  float scale = amax / 127.0f;
  if (scale < 1e-8f) scale = 1e-8f;
  *xs = scale;
  float inv = 1.0f / scale;
  for (long i = 0; i < n; ++i) {
    float v = x[i] * inv;
    long r = lrintf(v); /* __float2int_rn: round to nearest, ties to even */
    if (r > 127) r = 127;
    if (r < -127) r = -127;
    xq[i] = (int8_t)r;
  }
}

void oracle_quantize_activation_rows(int8_t* xq, float* xs, const float* x,
                                     long m, long n) {
#pragma omp parallel for schedule(static)
  for (long t = 0; t < m; ++t)
    oracle_quantize_activation(xq + t * n, xs + t, x + t * n, n);
}

/* src/model_cuda_v2_shared.cu:36-62.  One warp per row; lane l accumulates
 *   val = fma((float)q * scale, x[col], val)   for j = l, l+32 inside each group
 * (the reference's nvcc build contracts `val += wf * x` into one FFMA and keeps
 * `(float)q * scale` as its own multiply), then warpReduceSum (:30-34), a
 * shfl_down tree over offsets 16, 8, 4, 2, 1 whose result lane 0 stores. */
static float w8a32_row(const int8_t* wr, const float* sr, const float* x, long n,
                       int gs) {
  float lane[32];
  long ng = n / gs;
  for (int l = 0; l < 32; ++l) {
    float val = 0.0f;
    for (long g = 0; g < ng; ++g) {
      float scale = sr[g];
      for (long j = l; j < gs; j += 32) {
        long col = g * gs + j;
        float wf = (float)wr[col] * scale;
        val = fmaf(wf, x[col], val);
      }
    }
    lane[l] = val;
  }
  for (int off = 16; off > 0; off >>= 1)
    for (int l = 0; l < off; ++l) lane[l] = lane[l] + lane[l + off];
  return lane[0];
}

void oracle_gemv_w8a32(float* y, const float* x, const int8_t* w,
                       const float* s, long n, long d, int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) y[r] = w8a32_row(w + r * n, s + r * ng, x, n, gs);
}

/* Exact int32 dot of one group (the value :483-494 reduces to lane 0). */
static int32_t group_dot(const int8_t* wg, const int8_t* xg, int gs) {
  int32_t acc = 0;
  for (int j = 0; j < gs; ++j) acc += (int32_t)wg[j] * (int32_t)xg[j];
  return acc;
}

void oracle_group_dots(int32_t* out, const int8_t* xq, const int8_t* w, long n,
                       long d, int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r)
    for (long g = 0; g < ng; ++g)
      out[r * ng + g] = group_dot(w + r * n + g * gs, xq + g * gs, gs);
}

/* src/model_cuda_v2_shared.cu:465-501.  Per row, sequentially over groups:
 *   fp32_acc += (float)group_acc * w_scale * x_scale
 * evaluated left to right, with the final add contracted into an FFMA:
 *   acc = fma((float)I * ws, xs, acc). */
void oracle_gemv_w8a8(float* y, const int8_t* xq, const float* xs,
                      const int8_t* w, const float* s, long n, long d, int gs) {
  long ng = n / gs;
  float x_scale = *xs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    float acc = 0.0f;
    for (long g = 0; g < ng; ++g) {
      int32_t I = group_dot(w + r * n + g * gs, xq + g * gs, gs);
      float t = (float)I * s[r * ng + g];
      acc = fmaf(t, x_scale, acc);
    }
    y[r] = acc;
  }
}

/* Batched W8A8: token t uses xq[t][:], xs[t]; y is [m][d] token-major. */
void oracle_gemm_w8a8(float* y, const int8_t* xq, const float* xs,
                      const int8_t* w, const float* s, long m, long n, long d,
                      int gs) {
  for (long t = 0; t < m; ++t)
    oracle_gemv_w8a8(y + t * d, xq + t * n, xs + t, w, s, n, d, gs);
}

/* fp64 recomputes (tolerance anchors).  W8A32: sum of (q*s)*x in double.
 * W8A8: sum_g I_g * ws * xs in double from the exact int32 partials. */
void oracle_gemv_w8a32_f64(double* y, const float* x, const int8_t* w,
                           const float* s, long n, long d, int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    double acc = 0.0;
    for (long c = 0; c < n; ++c)
      acc += (double)w[r * n + c] * (double)s[r * ng + c / gs] * (double)x[c];
    y[r] = acc;
  }
}

void oracle_gemv_w8a8_f64(double* y, const int8_t* xq, const float* xs,
                          const int8_t* w, const float* s, long n, long d,
                          int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    double acc = 0.0;
    for (long g = 0; g < ng; ++g)
      acc += (double)group_dot(w + r * n + g * gs, xq + g * gs, gs) *
             (double)s[r * ng + g];
    y[r] = acc * (double)*xs;
  }
}

/* RMSNorm as the chained GEMV's prologue computes it (the reference's
 * rmsnorm_kernel, src/model_cuda_v2_shared.cu:74-89, whose own sum order is an
 * atomicAdd race): 256 threads, thread t holding columns 1024 j + 4 t .. + 3
 * (j < 8), each summing its squares with fmaf in that order; a warp
 * butterfly over lane offsets 16, 8, 4, 2, 1; the 8 warp sums added in warp
 * order; ss = 1 / sqrtf(sum / n + 1e-5); out = w * (ss * x).  n <= 8192. */
void oracle_rmsnorm_chain(float* out, const float* x, const float* w, long n) {
  float warp_tot[8];
  for (int wp = 0; wp < 8; ++wp) {
    float lane[32];
    for (int l = 0; l < 32; ++l) {
      const long t = wp * 32 + l;
      float ssq = 0.0f;
      for (long j = 0; j < 8; ++j)
        for (long e = 0; e < 4; ++e) {
          const long c = 1024 * j + 4 * t + e;
          const float v = c < n ? x[c] : 0.0f;
          ssq = fmaf(v, v, ssq);
        }
      lane[l] = ssq;
    }
    for (int off = 16; off > 0; off >>= 1) {
      float nxt[32];
      for (int l = 0; l < 32; ++l) nxt[l] = lane[l] + lane[l ^ off];
      memcpy(lane, nxt, sizeof(lane));
    }
    warp_tot[wp] = lane[0];
  }
  float sum = warp_tot[0];
  for (int wp = 1; wp < 8; ++wp) sum += warp_tot[wp];
  const float ss = 1.0f / sqrtf(sum / (float)n + 1e-5f);
  for (long c = 0; c < n; ++c) out[c] = w[c] * (ss * x[c]);
}

/* src/model_cuda_v2_shared.cu:10-19: one thread per row, sequentially over
 * the columns, `val += w * x` contracted into an FFMA by nvcc. */
void oracle_matmul_f32(float* y, const float* x, const float* w, long n, long d) {
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    float val = 0.0f;
    for (long j = 0; j < n; ++j) val = fmaf(w[r * n + j], x[j], val);
    y[r] = val;
  }
}

void oracle_matmul_f64(double* y, const float* x, const float* w, long n, long d) {
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    double val = 0.0;
    for (long j = 0; j < n; ++j) val += (double)w[r * n + j] * (double)x[j];
    y[r] = val;
  }
}

/* Batched fp64 recompute for m tokens (y [m][d] token-major): token t's row r
 * is sum_g I_t[r][g] * ws[r][g], times xs[t], in double from the exact int32
 * partials -- the same value oracle_gemv_w8a8_f64 gives for that token.  One
 * weight row is read once for all tokens (OpenMP over rows), so the full
 * Llama-3.2-3B shapes at m = 256 finish in about a second. */
void oracle_gemm_w8a8_f64(double* y, const int8_t* xq, const float* xs,
                          const int8_t* w, const float* s, long m, long n,
                          long d, int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(dynamic, 8)
  for (long r = 0; r < d; ++r) {
    const int8_t* wr = w + r * n;
    const float* sr = s + r * ng;
    for (long t = 0; t < m; ++t) {
      const int8_t* xt = xq + t * n;
      double acc = 0.0;
      for (long g = 0; g < ng; ++g)
        acc += (double)group_dot(wr + g * gs, xt + g * gs, gs) * (double)sr[g];
      y[t * d + r] = acc * (double)xs[t];
    }
  }
}

/* Exact int64 sums of the int32 group dots weighted by integer scales:
 * y[t][r] = sum_g I_t[r][g] * k[r][g].  With k one-hot per row this reads one
 * group dot per row; the GPU parity tests use it to check the production
 * kernels' group dots bit for bit. */
void oracle_group_dot_sums(int64_t* y, const int8_t* xq, const int8_t* w,
                           const int32_t* k, long m, long n, long d, int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r)
    for (long t = 0; t < m; ++t) {
      int64_t acc = 0;
      for (long g = 0; g < ng; ++g)
        acc += (int64_t)group_dot(w + r * n + g * gs, xq + t * n + g * gs, gs) *
               (int64_t)k[r * ng + g];
      y[t * d + r] = acc;
    }
}

/* CPU baseline: float32 dequant-then-matvec of the same quantised data,
 * OpenMP over rows, the plain loop a host implementation would write. */
void oracle_dequant_matvec(float* y, const float* x, const int8_t* w,
                           const float* s, long n, long d, int gs) {
  long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    const int8_t* wr = w + r * n;
    const float* sr = s + r * ng;
    float acc = 0.0f;
    for (long g = 0; g < ng; ++g) {
      float part = 0.0f;
      for (int j = 0; j < gs; ++j) part += (float)wr[g * gs + j] * x[g * gs + j];
      acc += part * sr[g];
    }
    y[r] = acc;
  }
}

int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int t) {
#ifdef _OPENMP
  if (t > 0) omp_set_num_threads(t);
#else
  (void)t;
#endif
}
