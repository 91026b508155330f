// mli_internal.h -- host-side plumbing shared by the library's translation
// units: status bookkeeping, per-device properties and the kernel launcher.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#include "../../include/mli_gemv.h"

namespace mli {

// Records `status` (and the CUDA error behind it) as this thread's last status
// and returns it, so entry points can `return set_status(...)`.
int set_status(int status, cudaError_t err = cudaSuccess);

// Maps a CUDA error (from a launch or a runtime call) onto the status codes.
int check_cuda(cudaError_t err);

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int smem_per_sm = 0;         // bytes usable by resident CTAs
  int smem_optin_per_cta = 0;  // max dynamic smem one CTA may opt into
  int cc_major = 0, cc_minor = 0;
};

// Properties of the current device, cached after the first query.
const DeviceInfo& current_device(cudaError_t* err);

// Launch-time options (MLI_LAUNCH_* bits).
unsigned launch_flags();

// Device address of the library's error word on the current device, for
// kernels of a translation unit built as its own device module (they cannot
// name the symbol); nullptr if the lookup failed.
unsigned int* device_error_word();

// cudaLaunchKernelEx wrapper: adds the programmatic-dependent-launch
// attribute when enabled, and returns the launch's cudaError_t.  Launches on
// the legacy default stream (NULL), which the reference's forward pass uses,
// never carry it: they keep the plain stream order of <<<>>> launches.
// `cluster_x` > 1 groups consecutive blocks into thread-block clusters of
// that many blocks along x (the grid must be a multiple of it).
template <typename... KArgs, typename... Args>
cudaError_t launch_clustered(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                             size_t smem, cudaStream_t stream, bool allow_pdl,
                             unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (allow_pdl && stream != nullptr && stream != cudaStreamLegacy &&
      (launch_flags() & MLI_LAUNCH_PDL)) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++cfg.numAttrs;
  }
  if (cluster_x > 1) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = cluster_x;
    attr[cfg.numAttrs].val.clusterDim.y = 1;
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    ++cfg.numAttrs;
  }
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block,
                   size_t smem, cudaStream_t stream, bool allow_pdl,
                   Args&&... args) {
  return launch_clustered(kernel, grid, block, smem, stream, allow_pdl, 1u, std::forward<Args>(args)...);
}

// Raises the kernel's dynamic shared memory limit to at least `smem` bytes on
// the current device.  The runtime call is made once per (kernel, device,
// size increase), so launches inside a CUDA-graph capture make none.
cudaError_t ensure_dynamic_smem(const void* kernel, size_t smem);

inline bool aligned(const void* p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

}  // namespace mli
