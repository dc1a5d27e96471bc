// Library-wide C-ABI pieces: status strings, version, per-device property
// cache and the per-device error word that bounded waits report through.
#include <cudaTypedefs.h>

#include <mutex>

#include "ng_common.cuh"

namespace ngb {
namespace {
// One word per device (each device that loads the module has its own copy).
__device__ unsigned int g_error_word;


DeviceInfo g_info[kMaxDevices];
std::once_flag g_once[kMaxDevices];
int g_status[kMaxDevices];
}  // namespace

int current_device_info(DeviceInfo* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NG_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return NG_ERR_CUDA;
  std::call_once(g_once[dev], [dev] {
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) {
      g_status[dev] = NG_ERR_CUDA;
      return;
    }
    DeviceInfo& d = g_info[dev];
    d.device = dev;
    d.sm_count = p.multiProcessorCount;
    d.cc_major = p.major;
    d.cc_minor = p.minor;
    d.smem_optin = p.sharedMemPerBlockOptin;
    d.l2_bytes = p.l2CacheSize;
    if (p.major != 10 || p.minor != 0) {
      g_status[dev] = NG_ERR_UNSUPPORTED_DEVICE;
      return;
    }
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_error_word) != cudaSuccess || ptr == nullptr) {
      g_status[dev] = NG_ERR_CUDA;
      return;
    }
    d.err = static_cast<unsigned int*>(ptr);
    g_status[dev] = NG_OK;
  });
  if (g_status[dev] != NG_OK) return g_status[dev];
  *out = g_info[dev];
  return NG_OK;
}

void* tensor_map_encode_fn() {
  static void* fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = p;
  });
  return fn;
}

}  // namespace ngb

extern "C" int ng_abi_version(void) { return 3; }

extern "C" int ng_device_status(void* stream) {
  ngb::DeviceInfo dev;
  if (int st = ngb::current_device_info(&dev)) return st;
  auto s = static_cast<cudaStream_t>(stream);
  if (cudaStreamSynchronize(s) != cudaSuccess) return NG_ERR_CUDA;
  unsigned int word = 0;
  if (cudaMemcpy(&word, dev.err, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess)
    return NG_ERR_CUDA;
  if (word != 0) {
    const unsigned int zero = 0;
    if (cudaMemcpy(dev.err, &zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess)
      return NG_ERR_CUDA;
    return (word & ngb::kErrWaitTimeout) ? NG_ERR_DEVICE_TIMEOUT : NG_ERR_BAD_INDEX;
  }
  return NG_OK;
}

extern "C" const char* ng_status_string(int status) {
  switch (status) {
    case NG_OK: return "ok";
    case NG_ERR_NULL_POINTER: return "a required pointer is NULL";
    case NG_ERR_BAD_DTYPE: return "unsupported dtype (expected fp16 or bf16)";
    case NG_ERR_BAD_SHAPE: return "inconsistent or unsupported shape / group size";
    case NG_ERR_MISALIGNED: return "a pointer lacks the alignment its vector loads need";
    case NG_ERR_BAD_ARGUMENT: return "an option is out of range";
    case NG_ERR_LAUNCH: return "kernel launch failed";
    case NG_ERR_UNSUPPORTED_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case NG_ERR_CUDA: return "a CUDA runtime call failed";
    case NG_ERR_DEVICE_TIMEOUT: return "a kernel gave up on a bounded pipeline wait";
    case NG_ERR_BAD_INDEX: return "a kernel met an index outside its table";
    default: return "unknown status";
  }
}
