// ref_harness.cu -- TEST INFRASTRUCTURE ONLY.  Links against the reference's
// own src/model_cuda_v2_shared.cu (compiled unmodified from the reference
// tree by oracle/Makefile) and re-exports its three launchers with C linkage
// so tests and the reference arm of bench.py can call them through ctypes.
// Nothing in the product library links this file.
#include <cuda_runtime.h>
#include <stdint.h>

#include "model.h"  // the reference's include/model.h (found with -I)

extern "C" {

// src/model_cuda_v2_shared.cu:64-69
void ref_matmul_int8(float* xout, float* x, int8_t* w_q, float* w_s, int n,
                     int d, int group_size) {
  matmul_int8(xout, x, w_q, w_s, n, d, group_size);
}

// src/model_cuda_v2_shared.cu:503-509
void ref_matmul_dp4a(float* xout, const int8_t* x_q, const float* x_s,
                     const int8_t* w_q, const float* w_s, int n, int d,
                     int group_size) {
  matmul_dp4a(xout, x_q, x_s, w_q, w_s, n, d, group_size);
}

// src/model_cuda_v2_shared.cu:457-460
void ref_quantize_activation(int8_t* xq, float* xs, const float* x, int n) {
  quantize_activation(xq, xs, x, n);
}

int ref_last_error(void) { return static_cast<int>(cudaGetLastError()); }
int ref_device_synchronize(void) { return static_cast<int>(cudaDeviceSynchronize()); }

}  // extern "C"
