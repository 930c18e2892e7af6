// Host-side helpers shared by the C-ABI launchers: error reporting, device
// properties, the device status word, and TMA tensor-map encoding.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <string>
#include <utility>

#include "../../include/qvggt_b200.h"
#include "common.cuh"

namespace qv {

// Records a human-readable message for qvggt_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);
// Adds n to the library's launch counter (qvggt_launch_count).
void count_launch(int n);
// Maps a CUDA error to QVGGT_ERR_CUDA with the CUDA message; 0 if success.
int check_cuda(cudaError_t e, const char* what);

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int device = -1;
  int num_sms = 0;
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
};
// Properties of the current device, queried once per device (std::call_once,
// so a second host thread never sees a half-filled entry).
const DeviceInfo& device_info();

// Once-per-device host set-up flags (kernel attributes).  A thread that sees a
// device's flag set also sees the set-up published before it; two threads that
// both find it clear both run the (idempotent) set-up.  Devices beyond
// kMaxDevices never cache: their set-up runs on every call.
struct DeviceFlags {
  std::atomic<bool> done[kMaxDevices];
  bool test(int dev) const { return dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire); }
  void set(int dev) {
    if (dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
  }
};

// Raises a kernel's dynamic shared-memory limit to `bytes`, once per device.
template <class Kernel>
int ensure_smem(DeviceFlags& flags, Kernel kernel, int bytes, const char* what) {
  const int dev = device_info().device;
  if (flags.test(dev)) return QVGGT_OK;
  const int rc = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (rc == QVGGT_OK) flags.set(dev);
  return rc;
}

// Device status word of the current device (library-owned; see capi.cu) and
// the wait budget every bounded device-side wait uses.
Ctl make_ctl();

// cuTensorMapEncodeTiled through the runtime's driver entry point.
int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides_bytes /* rank-1 entries */, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

// 2-D row-major [rows, cols] tile map: box = box_cols x box_rows.
inline int tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t cols, uint64_t rows,
                   uint64_t row_stride_bytes, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw) {
  uint64_t dims[2] = {cols, rows};
  uint64_t strides[1] = {row_stride_bytes};
  uint32_t box[2] = {box_cols, box_rows};
  return encode_tmap(map, dtype, 2, base, dims, strides, box, sw);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether launches use programmatic dependent launch (default on;
// QVGGT_PDL=0 turns it off for the whole process).
bool pdl_enabled();

// Launches `kernel` on `stream` with programmatic stream serialisation (when
// enabled) and, for cluster_x > 1, clusters of cluster_x CTAs.  The kernel must
// call pdl_wait() before its first global memory access.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[n].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  ++n;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = cluster_x;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace qv
