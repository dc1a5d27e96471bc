// Shared host/device helpers for the nibblegemm_b200 kernels (sm_100a only).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "nibblegemm_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nibblegemm_b200 kernels are written for sm_100a only"
#endif

namespace ngb {

// ---------------------------------------------------------------------------
// Device-side loads with explicit cache behaviour.
// ---------------------------------------------------------------------------

// Streamed-once weights: read-only path, do not allocate in L1 (each packed
// word is used by exactly one thread), and mark the L2 line evict-first so a
// 30 MB weight sweep does not push activations and scales out of L2.
__device__ __forceinline__ uint4 ld_stream_v4(const void* p, uint64_t policy) {
  uint4 v;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;\n"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(p), "l"(policy));
  return v;
}

__device__ __forceinline__ uint64_t make_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
  return pol;
}

// Small re-read operands (scales, activations): read-only path, L1-cached.
__device__ __forceinline__ uint2 ld_ro_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

__device__ __forceinline__ uint4 ld_ro_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100: one instruction, two lanes of fp32).
// ---------------------------------------------------------------------------
struct f2 {
  uint64_t v;
};

__device__ __forceinline__ f2 f2_make(float lo, float hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ f2 f2_from_bits(uint32_t lo, uint32_t hi) {
  f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r.v) : "r"(lo), "r"(hi));
  return r;
}

__device__ __forceinline__ void f2_split(f2 a, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(a.v));
}

// d = a * b + c, lane-wise, round to nearest even, single rounding per lane.
__device__ __forceinline__ f2 f2_fma(f2 a, f2 b, f2 c) {
  f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.v) : "l"(a.v), "l"(b.v), "l"(c.v));
  return d;
}

__device__ __forceinline__ f2 f2_mul(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.v) : "l"(a.v), "l"(b.v));
  return d;
}

// ---------------------------------------------------------------------------
// lop3 with the immediate for (a & b) | c.
// The LUT byte is the truth table evaluated on a=0xF0, b=0xCC, c=0xAA.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  constexpr uint32_t kLut = (0xF0u & 0xCCu) | 0xAAu;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(kLut));
  return d;
}

// Kernels OR this code into the per-device error word (DeviceInfo::err, a
// device address) when a bounded wait expires; ng_device_status reads it back.
constexpr unsigned int kErrWaitTimeout = 1u;
// ... and this one when an index (a token id) lies outside its table.
constexpr unsigned int kErrBadIndex = 2u;

}  // namespace ngb

// ---------------------------------------------------------------------------
// Host-side helpers (defined in capi.cu).
// ---------------------------------------------------------------------------
namespace ngb {

// Per-device host state (property cache, one-time kernel attributes) is held in
// arrays of this many entries; current_device_info rejects larger ordinals.
constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0;
  int cc_minor = 0;
  size_t smem_optin = 0;
  size_t l2_bytes = 0;
  unsigned int* err = nullptr;  // device address of this device's error word
};

// Cached properties of the current device; returns NG_OK or an error status.
int current_device_info(DeviceInfo* out);

// The driver's cuTensorMapEncodeTiled (fetched once through the runtime's
// driver entry-point query, so the library needs no libcuda link), as an
// opaque pointer; nullptr if unavailable.
void* tensor_map_encode_fn();

// Tensor-pipe decode GEMV (gemv_tc.cu); arguments already validated.
size_t gemv_tc_workspace_bytes(int N, const DeviceInfo& dev);
int gemv_tc(const void* x, int x_dtype, const uint32_t* q, const __half* s, void* y, int M, int K,
            int N, int G, void* ws, const DeviceInfo& dev, cudaStream_t strm);


// Bulk-copy tensor-pipe GEMV (gemv_stream.cu), M <= 16; arguments already
// validated.  splits = cluster size (0 = heuristic).  Needs
// gemv_stream_supported (N % 8 == 0, 16-byte aligned scales).
bool gemv_stream_supported(int N, const void* scales);

int gemv_stream(const void* x, int x_dtype, const uint32_t* q, const __half* s, void* y, int M,
                int K, int N, int G, int splits, const DeviceInfo& dev, cudaStream_t strm);

// Bulk-copy ring GEMV (gemv_ring.cu), M <= 8; arguments already validated.
int gemv_ring(const void* x, int x_dtype, bool tensor_pipe, const uint32_t* q, const __half* s,
              void* y, int M, int K, int N, int G, int splits, void* ws, size_t ws_bytes,
              const DeviceInfo& dev, cudaStream_t strm);
// Workspace bytes ng_gemv_w4a16 needs for every schedule (tensor-pipe
// persistent GEMV region, then the stream-K ring's partials and flags).
size_t gemv_ring_workspace_bytes(int N, const DeviceInfo& dev);

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

inline int launch_status(cudaError_t e) { return e == cudaSuccess ? NG_OK : NG_ERR_LAUNCH; }

inline int launch_status() { return launch_status(cudaGetLastError()); }

}  // namespace ngb
