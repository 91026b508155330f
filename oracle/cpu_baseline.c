/*
 * cpu_baseline.c -- the CPU baseline of the INT8 group-64 GEMV path.
 *
 * TEST AND MEASUREMENT INFRASTRUCTURE ONLY: bench.py times it beside the GPU
 * kernels; the product library never calls it.
 *
 * A host implementation of MiniLlama-Infra's W8A32 GEMV
 * (src/model_cuda_v2_shared.cu:36-62): float32 dequant-then-matvec over the
 * same int8 weights and per-(row, 64-column group) fp32 scales, written the
 * way an optimised host library would -- OpenMP over rows, the group's
 * int8 x fp32 products vectorised (`omp simd` reduction, so the compiler may
 * reorder the sum within a group), the group's sum scaled once.  It is
 * compiled with -O3 -march=native on the host that runs it (the CPU of the
 * GPU host may differ from the build machine's), so it is not bit-identical to
 * the reference's order; the oracle in mli_oracle.c is the checker.
 */
#include <stdint.h>
#ifdef _OPENMP
#include <omp.h>
#endif

void cpu_dequant_matvec(float* y, const float* x, const int8_t* w,
                        const float* s, long n, long d, int gs) {
  const long ng = n / gs;
#pragma omp parallel for schedule(static)
  for (long r = 0; r < d; ++r) {
    const int8_t* wr = w + r * n;
    const float* sr = s + r * ng;
    float acc = 0.0f;
    for (long g = 0; g < ng; ++g) {
      const int8_t* wg = wr + g * gs;
      const float* xg = x + g * gs;
      float part = 0.0f;
#pragma omp simd reduction(+ : part)
      for (int j = 0; j < gs; ++j) part += (float)wg[j] * xg[j];
      acc += part * sr[g];
    }
    y[r] = acc;
  }
}

int cpu_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
