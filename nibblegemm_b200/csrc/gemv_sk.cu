// Decode-regime GEMV, stream-K over TMA-fed shared-memory rings (default path
// when the caller supplies a workspace).
//
// The weight matrix is cut into units of 32 packed rows (256 values of K) x
// 128 columns (16 KB).  The units are ordered column-tile-major and the list
// is split into one contiguous, equal-length range per CTA (one CTA per SM,
// gridDim = #SMs), so every SM streams the same number of bytes whatever the
// shape -- no wave-quantisation tail.  A producer thread issues one TMA tile
// load per unit into a ring of up to ~12 stages, so at launch each SM already
// has ~200 KB of loads outstanding: the whole 30 MB config-1 weight is in
// flight across the machine from the first microsecond, which is what a
// ~5 us kernel needs to approach HBM bandwidth (no per-warp load-use chains).
// The unit's activation slice [M x 256] rides along in the same stage.
//
// Eight consumer warps decode: warp w takes rows 4w..4w+3 of every unit
// (one 32-value half2 window), lanes own 4 columns each (a 512-byte
// conflict-free shared-memory row read per warp).  When a CTA's range ends
// inside a column tile, its partial sums go to the workspace and a per-tile
// arrival counter decides which CTA finishes the tile: the last to arrive
// sums every contributor's partial in CTA order (deterministic regardless of
// arrival order), writes Y, and resets the counter to zero -- the workspace
// is left as it was found.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "ng_decode.cuh"
#include "sm100_primitives.cuh"

namespace ngb {
namespace {

constexpr int kCols = 128;     // columns per unit / tile
constexpr int kRows = 32;      // packed rows per unit (256 values of K)
constexpr int kCW = 8;         // consumer warps
constexpr int kThreads = 32 * (kCW + 1);
constexpr int kWBytes = kCols * kRows * 4;  // 16 KB
constexpr int kMaxStages = 16;
constexpr int kSmemBudget = 200 * 1024;

enum Path { kHalf2 = 0, kFloat2 = 1 };

struct SkBarriers {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  int last;
  int abort;
};

struct Partition {
  long long units;
  int P;
  __host__ __device__ long long start(int b) const { return static_cast<long long>(b) * units / P; }
  // The CTA whose range contains unit u.
  __host__ __device__ int owner(long long u) const {
    int b = static_cast<int>(((u + 1) * P - 1) / units);
    if (b >= P) b = P - 1;
    while (b + 1 < P && start(b + 1) <= u) ++b;
    while (b > 0 && start(b) > u) --b;
    return b;
  }
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kCW * 32) : "memory");
}

template <int MT, bool XBF16, int PATH>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_sk_kernel(const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_x, const __half* __restrict__ scales,
                   void* __restrict__ y, int M, int K, int N, int G, long long units, int chunks,
                   int stages, unsigned int* __restrict__ counters, float* __restrict__ partials,
                   unsigned int* __restrict__ err) {
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int kXBytes = MT * kRows * 8 * 2;
  constexpr int kStage = kWBytes + kXBytes;
  constexpr int E = MT * kCols;
  float* red = reinterpret_cast<float*>(smem + stages * kStage);
  SkBarriers* bars = reinterpret_cast<SkBarriers*>(smem + stages * kStage + kCW * E * 4);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Partition part{units, static_cast<int>(gridDim.x)};
  const int b = blockIdx.x;
  const long long u0 = part.start(b), u1 = part.start(b + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], kCW);
    }
    bars->abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_x);
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      for (long long u = u0; u < u1; ++u, ++it) {
        const int s = it % stages;
        const uint32_t ph = (it / stages) & 1;
        if (!mbar_wait_bounded(&bars->empty[s], ph ^ 1, err, abort)) break;
        const int tile = static_cast<int>(u / chunks), c = static_cast<int>(u % chunks);
        unsigned char* st = smem + s * kStage;
        mbar_arrive_expect_tx(&bars->full[s], kStage);
        tma_load_2d(st, &tmap_w, &bars->full[s], tile * kCols, c * kRows);
        tma_load_2d(st + kWBytes, &tmap_x, &bars->full[s], c * kRows * 8, 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ consumers
    const int cw = warp - 1;
    const int ct = threadIdx.x - 32;  // 0..255
    const int ngroups = K / G;
    float acc[4][MT];
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[c][m] = 0.f;

    auto scale_of = [&](long long u) -> uint2 {
      if (u >= u1) return make_uint2(0u, 0u);
      const int tile = static_cast<int>(u / chunks), c = static_cast<int>(u % chunks);
      const int col = tile * kCols + lane * 4;
      const int g = ((c * kRows + cw * 4) * 8) / G;
      if (col >= N || g >= ngroups) return make_uint2(0u, 0u);
      return ld_ro_v2(scales + static_cast<size_t>(g) * N + col);
    };
    uint2 pre0 = scale_of(u0), pre1 = scale_of(u0 + 1);
    long long seg_first = u0;
    int it = 0;
    bool ok = true;
    for (long long u = u0; u < u1; ++u, ++it) {
      const int s = it % stages;
      const uint32_t ph = (it / stages) & 1;
      const uint2 sv = pre0;
      pre0 = pre1;
      pre1 = scale_of(u + 2);
      if (!warp_wait_bounded(&bars->full[s], ph, err, abort)) {
        ok = false;
        break;
      }
      const unsigned char* st = smem + s * kStage;
      const uint4* wrow = reinterpret_cast<const uint4*>(st) + (cw * 4) * (kCols / 4) + lane;
      const unsigned char* xs = st + kWBytes + cw * 4 * 16;  // row r of X slice at +16 r bytes
      float sc[4];
      sc[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x & 0xFFFF)));
      sc[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x >> 16)));
      sc[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y & 0xFFFF)));
      sc[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y >> 16)));
      uint4 q[4];
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) q[rr] = wrow[rr * (kCols / 4)];

      if constexpr (PATH == kHalf2) {
        __half2 h[4][MT];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int m = 0; m < MT; ++m) h[c][m] = __float2half2_rn(0.f);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const uint32_t words[4] = {q[rr].x, q[rr].y, q[rr].z, q[rr].w};
          __half2 wv[4][4];
#pragma unroll
          for (int c = 0; c < 4; ++c) decode8_f16(words[c], wv[c]);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * (kRows * 16) + rr * 16);
            const __half2 xh[4] = {h2_from_bits(xv.x), h2_from_bits(xv.y), h2_from_bits(xv.z),
                                   h2_from_bits(xv.w)};
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
              for (int i = 0; i < 4; ++i) h[c][m] = __hfma2(wv[c][i], xh[i], h[c][m]);
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const float2 f = __half22float2(h[c][m]);
            acc[c][m] = fmaf(f.x + f.y, sc[c], acc[c][m]);
          }
      } else {
        f2 a2[4][MT];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int m = 0; m < MT; ++m) a2[c][m] = f2_make(0.f, 0.f);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const uint32_t words[4] = {q[rr].x, q[rr].y, q[rr].z, q[rr].w};
          f2 wv[4][4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint32_t w16 = words[c] >> 16;
            wv[c][0] = decode_pair_f32<0>(words[c], w16);
            wv[c][1] = decode_pair_f32<1>(words[c], w16);
            wv[c][2] = decode_pair_f32<2>(words[c], w16);
            wv[c][3] = decode_pair_f32<3>(words[c], w16);
          }
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * (kRows * 16) + rr * 16);
            const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
            f2 xp[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if constexpr (XBF16) {
                xp[j] = f2_from_bits(xw[j] << 16, xw[j] & 0xFFFF0000u);
              } else {
                const float2 t = __half22float2(h2_from_bits(xw[j]));
                xp[j] = f2_make(t.x, t.y);
              }
            }
#pragma unroll
            for (int c = 0; c < 4; ++c)
#pragma unroll
              for (int j = 0; j < 4; ++j) a2[c][m] = f2_fma(wv[c][j], xp[j], a2[c][m]);
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float lo, hi;
            f2_split(a2[c][m], lo, hi);
            acc[c][m] = fmaf(lo + hi, sc[c], acc[c][m]);
          }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->empty[s]);

      // ---- end of a column-tile segment: reduce and emit ------------------------
      const int tile = static_cast<int>(u / chunks);
      if (u + 1 == u1 || (u + 1) / chunks != tile) {
        consumer_sync();  // red[] free
#pragma unroll
        for (int m = 0; m < MT; ++m)
          *reinterpret_cast<float4*>(red + (cw * MT + m) * kCols + lane * 4) =
              make_float4(acc[0][m], acc[1][m], acc[2][m], acc[3][m]);
        consumer_sync();
        const bool whole = (seg_first % chunks == 0) && ((u + 1) % chunks == 0);
        unsigned short* yo = static_cast<unsigned short*>(y);
        auto emit = [&](int e, float v) {
          const int m = e / kCols, n = tile * kCols + (e % kCols);
          if (m < M && n < N)
            yo[static_cast<size_t>(m) * N + n] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                       : __half_as_ushort(__float2half_rn(v));
        };
        if (whole) {
          for (int e = ct; e < E; e += kCW * 32) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) v += red[w * E + e];
            emit(e, v);
          }
        } else {
          const int first_tile_of_b = static_cast<int>(u0 / chunks);
          const int slot = 2 * b + (tile == first_tile_of_b ? 0 : 1);
          for (int e = ct; e < E; e += kCW * 32) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) v += red[w * E + e];
            partials[static_cast<size_t>(slot) * E + e] = v;
          }
          __threadfence();
          consumer_sync();
          const int bf = part.owner(static_cast<long long>(tile) * chunks);
          const int bl = part.owner(static_cast<long long>(tile + 1) * chunks - 1);
          if (ct == 0) {
            const unsigned int prev = atomicAdd(&counters[tile], 1u);
            bars->last = (prev == static_cast<unsigned int>(bl - bf));
          }
          consumer_sync();
          if (bars->last) {
            __threadfence();
            for (int e = ct; e < E; e += kCW * 32) {
              float v = 0.f;
              for (int bb = bf; bb <= bl; ++bb) {
                const int tfirst = static_cast<int>(part.start(bb) / chunks);
                const int sl = 2 * bb + (tile == tfirst ? 0 : 1);
                v += __ldcg(&partials[static_cast<size_t>(sl) * E + e]);
              }
              emit(e, v);
            }
            if (ct == 0) counters[tile] = 0u;
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int m = 0; m < MT; ++m) acc[c][m] = 0.f;
        seg_first = u + 1;
      }
    }
    (void)ok;
  }
  __syncthreads();
  if (*abort) {
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) {
    }
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Workspace layout, fixed for a device whatever M and N are (so calls with
// different shapes can share one workspace): partial-sum slots for the
// largest M tile first (2 per CTA), then one arrival counter per column tile.
// Only the counters must be zero between calls; the kernel re-zeroes them.
size_t ws_counter_offset(int P) { return static_cast<size_t>(2) * P * 16 * kCols * 4; }

size_t ws_bytes(int /*MT*/, int N, int P) {
  return ws_counter_offset(P) + static_cast<size_t>((N + kCols - 1) / kCols) * 4;
}

int mt_of(int M) { return M <= 1 ? 1 : M <= 2 ? 2 : M <= 4 ? 4 : M <= 8 ? 8 : 16; }

template <int MT, bool XBF16, int PATH>
int run_sk(const void* x, const uint32_t* q, const __half* s, void* y, int M, int K, int N, int G,
           void* ws, const DeviceInfo& dev, cudaStream_t stream) {
  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
  if (!enc) return NG_ERR_CUDA;
  CUtensorMap mw, mx;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K / 8)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 4};
    const cuuint32_t box[2] = {kCols, kRows};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&mw, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {kRows * 8, MT};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&mx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  const int chunks = (K / 8 + kRows - 1) / kRows;
  const long long units = static_cast<long long>((N + kCols - 1) / kCols) * chunks;
  const int P = static_cast<int>(std::min<long long>(dev.sm_count, units));
  constexpr int stage = kWBytes + MT * kRows * 16;
  const int red = kCW * MT * kCols * 4;
  const int stages = std::min(kMaxStages, (kSmemBudget - red - static_cast<int>(sizeof(SkBarriers))) / stage);
  const size_t smem = static_cast<size_t>(stages) * stage + red + sizeof(SkBarriers);
  auto kern = gemv_sk_kernel<MT, XBF16, PATH>;
  static std::once_flag once[64];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 8192);
  });
  auto* partials = static_cast<float*>(ws);
  auto* counters = reinterpret_cast<unsigned int*>(static_cast<unsigned char*>(ws) +
                                                   ws_counter_offset(dev.sm_count));
  kern<<<P, kThreads, smem, stream>>>(mw, mx, s, y, M, K, N, G, units, chunks, stages, counters,
                                      partials, dev.err);
  return launch_status();
}

template <bool XBF16, int PATH>
int sk_dispatch_m(const void* x, const uint32_t* q, const __half* s, void* y, int M, int K, int N,
                  int G, void* ws, const DeviceInfo& dev, cudaStream_t st) {
  switch (mt_of(M)) {
    case 1: return run_sk<1, XBF16, PATH>(x, q, s, y, M, K, N, G, ws, dev, st);
    case 2: return run_sk<2, XBF16, PATH>(x, q, s, y, M, K, N, G, ws, dev, st);
    case 4: return run_sk<4, XBF16, PATH>(x, q, s, y, M, K, N, G, ws, dev, st);
    case 8: return run_sk<8, XBF16, PATH>(x, q, s, y, M, K, N, G, ws, dev, st);
    default: return run_sk<16, XBF16, PATH>(x, q, s, y, M, K, N, G, ws, dev, st);
  }
}

}  // namespace
}  // namespace ngb

// Experimental entry (not in the public header): stream-K schedule.
extern "C" size_t ngx_gemv_sk_workspace_bytes(int M, int N) {
  ngb::DeviceInfo dev;
  if (M < 1 || M > 16 || N <= 0 || ngb::current_device_info(&dev) != NG_OK) return 0;
  return ngb::ws_bytes(ngb::mt_of(M), N, dev.sm_count);
}

extern "C" int ngx_gemv_sk(const void* x, int x_dtype, const int32_t* qweight,
                           const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                           void* workspace, void* stream) {
  using namespace ngb;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  const auto* q = reinterpret_cast<const uint32_t*>(qweight);
  const auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  if (x_dtype == NG_DTYPE_BF16)
    return sk_dispatch_m<true, kFloat2>(x, q, s, y, M, K, N, group_size, workspace, dev, strm);
  return sk_dispatch_m<false, kHalf2>(x, q, s, y, M, K, N, group_size, workspace, dev, strm);
}
