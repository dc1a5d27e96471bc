// The decode step's output head and input gather, as library kernels:
//
//   ng_lm_head_argmax: logits = X @ W^T for a dense fp16 / bf16 head weight
//     W [V, H] (row-major, one vocabulary row per output), with the argmax over
//     the vocabulary fused into the epilogue -- the logits never need to be
//     written (optional) nor read back.  Per token the winner is kept as one
//     64-bit key, (order-preserving float bits << 32) | (2^32 - 1 - index), so
//     the largest key is the largest logit and, among equal logits, the
//     smallest index; keys are combined with one 64-bit atomicMax per CTA and
//     token, and across tensor-parallel ranks with one MAX all-reduce of M
//     int64 values.
//   ng_embed_tokens: out[m] = table[token[m]], with the token either given or
//     decoded from such a key (the previous step's argmax); decoding re-arms
//     the key for the next step's head.
//
// Head kernel (bandwidth-bound: V x H x 2 bytes, 1.05 GB per token at
// Llama-3-8B, 128256 x 4096):
//   * Weights as the A operand of mma.sync m16n8k16 (fp32 accumulation): a
//     warp owns 16 vocabulary rows; lane (g = lane / 4, q = lane % 4) loads
//     16 bytes of rows g and g + 8 at K offset 8q of each 32-value window, so
//     a warp load reads 8 rows x 64 contiguous bytes and the 4 pairs of a chunk
//     feed the K slots of lane q in a permuted order that X (the B operand,
//     read from shared memory in the same order) follows.
//   * 16 warps per CTA, one CTA per SM, warps take 16-row tiles round-robin;
//     each lane keeps 8 loads (128 bytes) in flight and the first ones are
//     issued before `griddepcontrol.wait` (the weights are read-only).
//   * Up to 8 tokens per launch (the host splits larger batches).
#include <algorithm>
#include <climits>
#include <mutex>

#include "ng_common.cuh"

namespace ngb {
namespace {

constexpr int kHWarps = 16;
constexpr int kHThreads = kHWarps * 32;
constexpr int kHInFlight = 4;  // 32-value K windows in flight per lane (2 loads each)

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1, bool bf16) {
  if (bf16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Order-preserving map of a float to an unsigned int (larger float -> larger
// integer), then to a signed 64-bit key whose signed order is that order.
__device__ __forceinline__ long long argmax_key(float v, long long index) {
  const uint32_t b = __float_as_uint(v);
  const uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  const uint64_t k = (static_cast<uint64_t>(ord) << 32) |
                     (0xFFFFFFFFull - (static_cast<uint64_t>(index) & 0xFFFFFFFFull));
  return static_cast<long long>(k ^ 0x8000000000000000ull);
}

__device__ __forceinline__ long long key_index(long long key) {
  const uint64_t k = static_cast<uint64_t>(key) ^ 0x8000000000000000ull;
  return static_cast<long long>(0xFFFFFFFFull - (k & 0xFFFFFFFFull));
}

__device__ __forceinline__ long long max_ll(long long a, long long b) { return a > b ? a : b; }

template <bool BF16>
__global__ void __launch_bounds__(kHThreads, 1)
    lm_head_kernel(const unsigned short* __restrict__ x, const unsigned short* __restrict__ w,
                   int M, int V, int H, long long index_offset, unsigned short* __restrict__ logits,
                   long long* __restrict__ keys) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int g = lane >> 2;
  const int q = lane & 3;
  const int tiles = (V + 15) / 16;
  const int nwin = H / 32;                       // 32-value K windows per row
  const int gwarp = blockIdx.x * kHWarps + warp;
  const int nwarps = gridDim.x * kHWarps;
  const uint64_t pol = make_evict_first_policy();
  const int xrow = H * 2 + 64;                   // staged X row stride (bytes), 64 mod 128
  long long* s_best = reinterpret_cast<long long*>(smem + 8 * static_cast<size_t>(xrow));  // [warps][8]

  // Loads of one window of the current tile: rows g and g + 8 (clamped to V;
  // rows past V are computed and discarded).
  auto row_ptr = [&](int tile, int r) {
    const int row = min(tile * 16 + r, V - 1);
    return w + static_cast<size_t>(row) * H + 8 * q;
  };

  long long best[2] = {LLONG_MIN, LLONG_MIN};    // tokens 2q, 2q + 1
  int tile = gwarp;
  uint4 ra[kHInFlight], rb[kHInFlight];
  const unsigned short* pa = tile < tiles ? row_ptr(tile, g) : w;
  const unsigned short* pb = tile < tiles ? row_ptr(tile, g + 8) : w;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (tile < tiles) {
#pragma unroll
    for (int i = 0; i < kHInFlight; ++i) {
      ra[i] = ld_stream_v4(pa + 32 * i, pol);
      rb[i] = ld_stream_v4(pb + 32 * i, pol);
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = threadIdx.x; i < M * (H / 8); i += kHThreads) {
    const int m = i / (H / 8), c = i - m * (H / 8);
    *reinterpret_cast<uint4*>(smem + static_cast<size_t>(m) * xrow + c * 16) =
        ld_ro_v4(x + static_cast<size_t>(m) * H + c * 8);
  }
  __syncthreads();
  const bool have_x = g < M;
  const unsigned char* xp = smem + static_cast<size_t>(g) * xrow + q * 16;

  for (; tile < tiles; tile += nwarps) {
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int next = tile + nwarps;
    const unsigned short* na = next < tiles ? row_ptr(next, g) : pa;
    const unsigned short* nb = next < tiles ? row_ptr(next, g + 8) : pb;
    for (int w0 = 0; w0 < nwin; w0 += kHInFlight) {
#pragma unroll
      for (int i = 0; i < kHInFlight; ++i) {
        const int win = w0 + i;
        const uint4 a = ra[i], b = rb[i];
        // Refill: window win + kHInFlight of this tile, else the next tile's first.
        const int nw = win + kHInFlight;
        if (nw < nwin) {
          ra[i] = ld_stream_v4(pa + 32 * nw, pol);
          rb[i] = ld_stream_v4(pb + 32 * nw, pol);
        } else if (next < tiles) {
          ra[i] = ld_stream_v4(na + 32 * (nw - nwin), pol);
          rb[i] = ld_stream_v4(nb + 32 * (nw - nwin), pol);
        }
        uint4 xv = make_uint4(0u, 0u, 0u, 0u);
        if (have_x) xv = *reinterpret_cast<const uint4*>(xp + win * 64);
        mma_f16(acc[i & 1], a.x, b.x, a.y, b.y, xv.x, xv.y, BF16);
        mma_f16(acc[i & 1], a.z, b.z, a.w, b.w, xv.z, xv.w, BF16);
      }
    }
    // d0: (row g, token 2q), d1: (row g, token 2q + 1), d2 / d3: row g + 8.
    float d[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] = acc[0][e] + acc[1][e];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int row = tile * 16 + g + (e >= 2 ? 8 : 0);
      const int tok = 2 * q + (e & 1);
      if (row < V && tok < M) {
        best[e & 1] = max_ll(best[e & 1], argmax_key(d[e], index_offset + row));
        if (logits != nullptr)
          logits[static_cast<size_t>(tok) * V + row] =
              BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(d[e])) : __half_as_ushort(__float2half_rn(d[e]));
      }
    }
    pa = na;
    pb = nb;
  }
  // Warp: lanes with the same q hold the same tokens.
#pragma unroll
  for (int e = 0; e < 2; ++e)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1)
      best[e] = max_ll(best[e], __shfl_xor_sync(0xffffffffu, best[e], o));
  if (g == 0) {
    s_best[warp * 8 + 2 * q] = best[0];
    s_best[warp * 8 + 2 * q + 1] = best[1];
  }
  __syncthreads();
  if (threadIdx.x < M) {
    long long b = LLONG_MIN;
    for (int k = 0; k < kHWarps; ++k) b = max_ll(b, s_best[k * 8 + threadIdx.x]);
    if (b != LLONG_MIN) atomicMax(keys + threadIdx.x, b);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(256)
    embed_kernel(const long long* __restrict__ tokens_in, long long* __restrict__ keys,
                 long long* __restrict__ tokens_out, const unsigned short* __restrict__ table,
                 long long V, int H, unsigned short* __restrict__ out,
                 unsigned short* __restrict__ zero_out, unsigned int* __restrict__ err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int m = blockIdx.x;
  __shared__ long long s_tok;
  if (threadIdx.x == 0) {
    long long t = keys != nullptr ? key_index(keys[m]) : tokens_in[m];
    if (t < 0 || t >= V) {
      atomicOr(err, kErrBadIndex);
      t = -1;
    }
    s_tok = t;
    if (tokens_out != nullptr) tokens_out[m] = t;
  }
  __syncthreads();
  const long long t = s_tok;
  if (threadIdx.x == 0 && keys != nullptr) keys[m] = LLONG_MIN;  // re-arm for the next head
  if (out == nullptr && zero_out == nullptr) return;
  uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(m) * H);
  const uint4* src = reinterpret_cast<const uint4*>(table + static_cast<size_t>(t < 0 ? 0 : t) * H);
  for (int i = threadIdx.x; i < H / 8; i += blockDim.x) {
    if (out != nullptr) dst[i] = t < 0 ? make_uint4(0u, 0u, 0u, 0u) : ld_ro_v4(src + i);
    if (zero_out != nullptr)
      reinterpret_cast<uint4*>(zero_out + static_cast<size_t>(m) * H)[i] = make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace
}  // namespace ngb

extern "C" int ng_lm_head_argmax(const void* x, const void* weight, int dtype, int M, int V, int H,
                                 long long index_offset, void* logits, long long* keys,
                                 void* stream) {
  using namespace ngb;
  if (!x || !weight || !keys) return NG_ERR_NULL_POINTER;
  if (dtype != NG_DTYPE_F16 && dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 64 || V < 1 || H < 128 || H % 128 != 0 || H > 16384) return NG_ERR_BAD_SHAPE;
  if (index_offset < 0 || index_offset + V > 0xFFFFFFFFll) return NG_ERR_BAD_ARGUMENT;
  if (!aligned(x, 16) || !aligned(weight, 16) || (logits && !aligned(logits, 2)) || !aligned(keys, 8))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  const auto* xs = static_cast<const unsigned short*>(x);
  const auto* ws = static_cast<const unsigned short*>(weight);
  auto* ls = static_cast<unsigned short*>(logits);
  const size_t smem = 8 * static_cast<size_t>(H * 2 + 64) + kHWarps * 8 * sizeof(long long);
  auto kern = dtype == NG_DTYPE_BF16 ? lm_head_kernel<true> : lm_head_kernel<false>;
  static std::once_flag once[kMaxDevices];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(lm_head_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(lm_head_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
  });
  const int tiles = (V + 15) / 16;
  const int grid = std::max(1, std::min(dev.sm_count, (tiles + kHWarps - 1) / kHWarps));
  // Eight tokens per launch: the B operand of one MMA (larger batches re-read the weight).
  for (int m0 = 0; m0 < M; m0 += 8) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kHThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int mb = std::min(8, M - m0);
    if (int st = launch_status(cudaLaunchKernelEx(&cfg, kern, xs + static_cast<size_t>(m0) * H, ws, mb, V, H,
                                                  index_offset, ls ? ls + static_cast<size_t>(m0) * V : nullptr,
                                                  keys + m0)))
      return st;
  }
  return NG_OK;
}

extern "C" int ng_embed_tokens(const long long* tokens, long long* keys, long long* tokens_out,
                               const void* table, int dtype, int M, int H, long long V, void* out,
                               void* zero_out, void* stream) {
  using namespace ngb;
  if ((!tokens && !keys) || !table) return NG_ERR_NULL_POINTER;
  if (dtype != NG_DTYPE_F16 && dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || H < 8 || H % 8 != 0 || V < 1) return NG_ERR_BAD_SHAPE;
  if (!aligned(table, 16) || (out && !aligned(out, 16)) || (zero_out && !aligned(zero_out, 16)))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(M, 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kern = dtype == NG_DTYPE_BF16 ? embed_kernel<true> : embed_kernel<false>;
  return launch_status(cudaLaunchKernelEx(&cfg, kern, tokens, keys, tokens_out,
                                          static_cast<const unsigned short*>(table), V, H,
                                          static_cast<unsigned short*>(out),
                                          static_cast<unsigned short*>(zero_out), dev.err));
}
