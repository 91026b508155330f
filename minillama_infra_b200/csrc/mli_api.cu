// mli_api.cu -- library state behind the C ABI: status bookkeeping, the
// per-device property cache, launch options and the device error word.
#include <atomic>
#include <mutex>

#include "mli_common.cuh"
#include "mli_internal.h"

namespace mli {

__device__ unsigned int g_device_error = 0;

namespace {
thread_local int t_last_status = MLI_OK;
thread_local int t_last_cuda = 0;
std::atomic<unsigned> g_launch_flags{MLI_LAUNCH_PDL};

constexpr int kMaxDevices = 64;
DeviceInfo g_devices[kMaxDevices];
std::once_flag g_device_once[kMaxDevices];
cudaError_t g_device_err[kMaxDevices];
}  // namespace

unsigned int* device_error_word() {
  static std::once_flag once[kMaxDevices];
  static unsigned int* addr[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::call_once(once[dev], [dev]() {
    void* p = nullptr;
    addr[dev] = cudaGetSymbolAddress(&p, g_device_error) == cudaSuccess ? static_cast<unsigned int*>(p) : nullptr;
  });
  return addr[dev];
}

int set_status(int status, cudaError_t err) {
  t_last_status = status;
  if (status == MLI_ERR_CUDA) t_last_cuda = static_cast<int>(err);
  return status;
}

int check_cuda(cudaError_t err) {
  if (err == cudaSuccess) return set_status(MLI_OK);
  return set_status(MLI_ERR_CUDA, err);
}

namespace {
struct SmemAttr {
  const void* kernel;
  int device;
  size_t bytes;
};
std::mutex g_smem_mu;
SmemAttr g_smem_attrs[256];
int g_smem_count = 0;
}  // namespace

cudaError_t ensure_dynamic_smem(const void* kernel, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_smem_mu);
  SmemAttr* slot = nullptr;
  for (int i = 0; i < g_smem_count; ++i)
    if (g_smem_attrs[i].kernel == kernel && g_smem_attrs[i].device == dev) slot = &g_smem_attrs[i];
  if (slot != nullptr && slot->bytes >= smem) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  if (slot == nullptr && g_smem_count < 256) slot = &g_smem_attrs[g_smem_count++];
  if (slot != nullptr) *slot = SmemAttr{kernel, dev, smem};
  return cudaSuccess;
}

unsigned launch_flags() { return g_launch_flags.load(std::memory_order_relaxed); }

const DeviceInfo& current_device(cudaError_t* err) {
  static DeviceInfo invalid;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *err = (e != cudaSuccess) ? e : cudaErrorInvalidDevice;
    return invalid;
  }
  std::call_once(g_device_once[dev], [dev]() {
    DeviceInfo& d = g_devices[dev];
    d.device = dev;
    cudaError_t r = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (r == cudaSuccess)
      r = cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (r == cudaSuccess)
      r = cudaDeviceGetAttribute(&d.smem_optin_per_cta, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (r == cudaSuccess)
      r = cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev);
    if (r == cudaSuccess)
      r = cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev);
    g_device_err[dev] = r;
  });
  *err = g_device_err[dev];
  return g_devices[dev];
}

}  // namespace mli

extern "C" {

const char* mli_status_string(int status) {
  switch (status) {
    case MLI_OK: return "ok";
    case MLI_ERR_INVALID_ARG: return "invalid argument";
    case MLI_ERR_UNSUPPORTED: return "unsupported shape or layout";
    case MLI_ERR_CUDA: return "CUDA error";
    case MLI_ERR_DEVICE: return "device-side wait gave up";
    default: return "unknown status";
  }
}

int mli_last_status(void) { return mli::t_last_status; }
int mli_last_cuda_error(void) { return mli::t_last_cuda; }
int mli_version(void) { return 100; }
unsigned mli_get_launch_flags(void) { return mli::launch_flags(); }
void mli_set_launch_flags(unsigned flags) {
  mli::g_launch_flags.store(flags, std::memory_order_relaxed);
}

int mli_device_error(unsigned* code_out) {
  unsigned code = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&code, mli::g_device_error, sizeof(code));
  if (e != cudaSuccess) return mli::check_cuda(e);
  if (code != 0) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(mli::g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess) return mli::check_cuda(e);
  }
  if (code_out) *code_out = code;
  return mli::set_status(code == 0 ? MLI_OK : MLI_ERR_DEVICE);
}

}  // extern "C"
