// Library-wide runtime pieces of libvitfp4.so: version, status messages, device checks,
// and the driver entry point used to build TMA tensor maps.
#include <stdarg.h>
#include <stdio.h>

#include <map>
#include <mutex>

#include "vf4_host.h"

namespace vf4 {

static thread_local char g_msg[512] = "ok";

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return status;
}

namespace {
constexpr int kMaxDev = 64;
int g_arch_ok[kMaxDev];  // 0 unknown, 1 ok, -1 bad
int g_sms[kMaxDev];
std::mutex g_mu;
}  // namespace

int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(VF4_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDev) return fail(VF4_ERR_CUDA, "device index %d out of range", dev);
  int s = __atomic_load_n(&g_arch_ok[dev], __ATOMIC_ACQUIRE);
  if (s == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    std::lock_guard<std::mutex> lk(g_mu);
    g_sms[dev] = sms;
    s = (major == 10 && minor == 0) ? 1 : -1;
    __atomic_store_n(&g_arch_ok[dev], s, __ATOMIC_RELEASE);
    if (s < 0)
      return fail(VF4_ERR_ARCH, "device %d is sm_%d%d; libvitfp4 is built for sm_100a only", dev,
                  major, minor);
  }
  if (s < 0) return fail(VF4_ERR_ARCH, "device %d is not sm_100", dev);
  return VF4_OK;
}

int num_sms() {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDev || g_sms[dev] == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms > 0 ? sms : 148;
  }
  return g_sms[dev];
}

int smem_optin_raw(const void* kern, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> given;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  int& have = given[{kern, dev}];
  if (have >= bytes) return VF4_OK;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return fail(VF4_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
  have = bytes;
  return VF4_OK;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(VF4_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return VF4_OK;
}

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int current_context_id(unsigned long long* id) {
  using GetCurrentFn = CUresult (*)(CUcontext*);
  using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, id) != CUDA_SUCCESS)
    return fail(VF4_ERR_CUDA, "no current CUDA context");
  return VF4_OK;
}

}  // namespace vf4

extern "C" {

int vf4_version(void) { return 100; }

const char* vf4_last_error_string(void) { return vf4::g_msg; }

int vf4_device_error(int clear) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return -1;
  int a = vf4::cast_device_error(clear);
  int b = vf4::gemm_device_error(clear);
  int c = vf4::attn_device_error(clear);
  return a ? a : (b ? b : c);
}

}  // extern "C"
