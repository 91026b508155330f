// dropin_shim.cpp -- libmli_dropin.so: the reference's GEMV launchers with
// their exact C++ signatures (include/model.h:61-64 of MiniLlama-Infra),
// forwarding to the C ABI on the legacy default stream.
//
// The reference launchers (src/model_cuda_v2_shared.cu:21-25, 64-69, 457-460,
// 503-509) return void and check nothing.  These keep the void signature and
// leave the call's status in mli_last_status() for callers that want it.
#include "../../include/mli_gemv.h"

void matmul_int8(float* xout, float* x, int8_t* w_q, float* w_s, int n, int d,
                 int group_size) {
  (void)mli_gemv_w8a32(xout, x, w_q, w_s, n, d, group_size, nullptr);
}

void matmul_dp4a(float* xout, const int8_t* x_q, const float* x_s,
                 const int8_t* w_q, const float* w_s, int n, int d,
                 int group_size) {
  (void)mli_gemv_w8a8(xout, x_q, x_s, w_q, w_s, n, d, group_size, nullptr);
}

void quantize_activation(int8_t* xq, float* xs, const float* x, int n) {
  (void)mli_quantize_activation(xq, xs, x, n, nullptr);
}

void matmul(float* xout, float* x, float* w, int n, int d) {
  (void)mli_gemv_f32(xout, x, w, n, d, nullptr);
}
