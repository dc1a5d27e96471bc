// One-shot all-reduce (sum) of small fp16/bf16 vectors across the GPUs of one
// node over NVLink peer memory -- the reduction after each row-parallel
// projection of the tensor-parallel decode step (8 KB per call at Llama-3-8B
// batch 1).  At these sizes the cost is latency, not bandwidth: NCCL's ring
// takes ~2(world-1) dependent hops; here every rank pushes its vector straight
// into a slot of every peer's buffer (plain P2P stores, one NVLink crossing),
// raises a flag there, waits for the peers' flags in its own memory, and sums
// its own vector and the peers' slots in rank order -- so every rank computes the identical, deterministic
// result in fp32 and rounds once.
//
// Buffer of each rank (mapped into every peer with CUDA IPC):
//   data  [2 parity][kMaxCtas][world][chunk elems]   (chunk = this CTA's share)
//   flags [2 parity][kMaxCtas][world] uint32
// Each CTA works on its own chunk with its own flags and its own call counter
// (epoch, in local memory), so CTAs never wait on each other.  Parity = epoch
// & 1 double-buffers the slots: a rank can only reuse a parity after every
// peer has set its flag for the next call, i.e. after every peer finished
// reading the previous use.  Flags hold the epoch + 1 of the call that set
// them, so they never need clearing.  Waits are bounded (1 s of %globaltimer)
// and report through the device error word.  No multimem, no TMA.
#include <cstring>

#include "ng_common.cuh"
#include "sm100_primitives.cuh"

namespace ngb {
namespace {

constexpr int kArThreads = 512;
constexpr int kMaxCtas = 16;
constexpr int kMaxWorld = 8;

struct PeerPtrs {
  unsigned short* data[kMaxWorld];  // each rank's buffer base (this process's mapping)
};

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <bool BF16>
__global__ void __launch_bounds__(kArThreads)
    allreduce_kernel(unsigned short* __restrict__ io, long long n, PeerPtrs peers, int rank,
                     int world, long long slot_elems, unsigned int* __restrict__ epochs,
                     unsigned int* __restrict__ err) {
  // Launched with programmatic stream serialisation: let the next kernel (the
  // next projection's GEMV, which prefetches weights before its own
  // griddepcontrol.wait) launch now, and wait for the producer of `io`.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int c = blockIdx.x;
  const long long per = (n + gridDim.x - 1) / gridDim.x;
  const long long e0 = c * per, e1 = e0 + per < n ? e0 + per : n;
  const long long cnt = e1 > e0 ? e1 - e0 : 0;
  __shared__ unsigned int s_epoch;
  if (threadIdx.x == 0) s_epoch = epochs[c];
  __syncthreads();
  const unsigned int epoch = s_epoch;
  const int par = epoch & 1;
  const size_t data_elems = static_cast<size_t>(2) * kMaxCtas * world * slot_elems;
  auto slot = [&](unsigned short* base, int src) {
    return base + ((static_cast<size_t>(par) * kMaxCtas + c) * world + src) * slot_elems;
  };
  auto flag = [&](unsigned short* base, int src) {
    unsigned int* f = reinterpret_cast<unsigned int*>(base + data_elems);
    return f + (static_cast<size_t>(par) * kMaxCtas + c) * kMaxWorld + src;
  };

  // 1. push this rank's chunk into slot `rank` of every peer's buffer (our
  //    own contribution is read straight from `io` in step 4)
  const unsigned short* src = io + e0;
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    unsigned short* dst = slot(peers.data[p], rank);
    if ((cnt & 7) == 0 && ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0) {
      for (long long i = threadIdx.x; i < cnt / 8; i += kArThreads)
        reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
    } else {
      for (long long i = threadIdx.x; i < cnt; i += kArThreads) dst[i] = src[i];
    }
  }
  // 2. raise our flag in every peer's buffer.  The CTA barrier orders every
  //    thread's pushes before the flag writers' system-scope release stores
  //    (release is cumulative over what the barrier made visible to them).
  __syncthreads();
  if (threadIdx.x < world && threadIdx.x != rank)
    st_release_sys(flag(peers.data[threadIdx.x], rank), epoch + 1);
  // 3. wait (bounded) for every peer's flag in our own buffer
  if (threadIdx.x < world && threadIdx.x != rank) {
    const unsigned int* f = flag(peers.data[rank], threadIdx.x);
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_sys(f) != epoch + 1) {
      if (global_timer_ns() - t0 > 1000000000ull) {
        atomicOr(err, kErrWaitTimeout);
        break;
      }
    }
  }
  __syncthreads();
  // 4. sum the world's contributions in rank order (identical on every rank)
  const unsigned short* mine = slot(peers.data[rank], 0);
  for (long long i = threadIdx.x; i < cnt; i += kArThreads) {
    float acc = 0.f;
    for (int s = 0; s < world; ++s) {
      const unsigned short v = s == rank ? src[i] : mine[s * slot_elems + i];
      acc += BF16 ? __uint_as_float(static_cast<uint32_t>(v) << 16) : __half2float(__ushort_as_half(v));
    }
    io[e0 + i] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(acc)) : __half_as_ushort(__float2half_rn(acc));
  }
  __syncthreads();
  if (threadIdx.x == 0) epochs[c] = epoch + 1;
}

// Elements per (parity, CTA, source) slot: a CTA's share of the largest
// message, rounded up to 16 bytes so chunks move as 16-byte vectors.
size_t ar_slot_elems(size_t max_elems) {
  return ((max_elems + kMaxCtas - 1) / kMaxCtas + 7) / 8 * 8;
}

}  // namespace
}  // namespace ngb

extern "C" size_t ng_allreduce_buffer_bytes(int world, size_t max_elems) {
  using namespace ngb;
  if (world < 1 || world > kMaxWorld) return 0;
  const size_t slot = ar_slot_elems(max_elems);
  return static_cast<size_t>(2) * kMaxCtas * world * slot * 2 +
         static_cast<size_t>(2) * kMaxCtas * kMaxWorld * 4;
}

extern "C" int ng_allreduce_sum(void* data, int dtype, size_t n, void* const* peer_buffers,
                                int rank, int world, size_t max_elems, unsigned int* epochs,
                                void* stream) {
  using namespace ngb;
  if (!data || !peer_buffers || !epochs) return NG_ERR_NULL_POINTER;
  if (dtype != NG_DTYPE_F16 && dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world) return NG_ERR_BAD_ARGUMENT;
  if (n == 0 || n > max_elems) return NG_ERR_BAD_SHAPE;
  if (!aligned(data, 2)) return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  PeerPtrs peers = {};
  for (int p = 0; p < world; ++p) {
    if (!peer_buffers[p]) return NG_ERR_NULL_POINTER;
    peers.data[p] = static_cast<unsigned short*>(peer_buffers[p]);
  }
  const long long slot = static_cast<long long>(ar_slot_elems(max_elems));
  // One CTA per 4096 elements, at most kMaxCtas; a chunk never exceeds a slot.
  int ctas = static_cast<int>((n + 4095) / 4096);
  ctas = ctas < 1 ? 1 : (ctas > kMaxCtas ? kMaxCtas : ctas);
  while ((static_cast<long long>(n) + ctas - 1) / ctas > slot) ++ctas;
  if (ctas > kMaxCtas) return NG_ERR_BAD_SHAPE;
  auto* io = static_cast<unsigned short*>(data);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas, 1, 1);
  cfg.blockDim = dim3(kArThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const long long nn = static_cast<long long>(n);
  if (dtype == NG_DTYPE_BF16)
    return launch_status(cudaLaunchKernelEx(&cfg, allreduce_kernel<true>, io, nn, peers, rank, world,
                                            slot, epochs, dev.err));
  return launch_status(cudaLaunchKernelEx(&cfg, allreduce_kernel<false>, io, nn, peers, rank, world,
                                          slot, epochs, dev.err));
}

extern "C" int ng_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  if (!dev_ptr || !handle) return NG_ERR_NULL_POINTER;
  if (bytes == 0) return NG_ERR_BAD_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return NG_ERR_CUDA;
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaFree(p);
    return NG_ERR_CUDA;
  }
  memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return NG_OK;
}

extern "C" int ng_ipc_free(void* dev_ptr) {
  if (!dev_ptr) return NG_ERR_NULL_POINTER;
  return cudaFree(dev_ptr) == cudaSuccess ? NG_OK : NG_ERR_CUDA;
}

extern "C" int ng_ipc_open(const void* handle, void** dev_ptr) {
  if (!handle || !dev_ptr) return NG_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? NG_OK
                                                                                         : NG_ERR_CUDA;
}

extern "C" int ng_ipc_close(void* dev_ptr) {
  if (!dev_ptr) return NG_ERR_NULL_POINTER;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? NG_OK : NG_ERR_CUDA;
}
