// Host-side helpers shared by the C-ABI entry points (status messages, device checks,
// tensor-map encoding).  Internal to libvitfp4.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vitfp4.h"

namespace vf4 {

// Record a printf-style message for vf4_last_error_string() and return `status`.
int fail(int status, const char* fmt, ...);

// VF4_OK when the current device is sm_100 (B200 class); caches per device.
int check_device();

// Streaming multiprocessors of the current device (cached).
int num_sms();

// Last CUDA launch error -> status (with the kernel name in the message).
int launch_status(const char* what);

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry point.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();

// ID of the calling thread's current CUDA context (driver API, resolved through the runtime so
// the library loads on hosts without a driver).
int current_context_id(unsigned long long* id);

// Per-family readers of the device error word (defined in each .cu).
int cast_device_error(int clear);
int gemm_device_error(int clear);
int attn_device_error(int clear);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Opt kernel `kern` into `bytes` of dynamic shared memory on the current device.  The attribute
// lives with the kernel in the device's context, so the driver call is made only when a kernel
// needs more than it was last given on that device (a process that resets the device must not
// rely on this cache).
int smem_optin_raw(const void* kern, int bytes);
template <typename Kern>
inline int smem_optin(Kern kern, int bytes) {
  return smem_optin_raw(reinterpret_cast<const void*>(kern), bytes);
}

}  // namespace vf4
