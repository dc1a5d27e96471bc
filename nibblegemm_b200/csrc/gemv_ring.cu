// Decode-regime fused dequant GEMV with a bulk-copy shared-memory ring:
// Y[M, N] = X[M, K] @ W for M <= 8, one launch.
//
// Why a ring: at M = 1 a GEMV is a 30 MB read that should take ~4.6 us, and a
// kernel whose warps load weights into registers keeps only as many bytes in
// flight as it has warps x registers; with few chunks per warp the load
// latency, the activation staging and the reductions are paid in series.
// Here one producer warp per CTA streams the CTA's whole weight slice with
// `cp.async.bulk` (one 512-byte row segment per lane, completion counted on
// an mbarrier) into a ring of 16 KB stages, and it starts doing so *before*
// `griddepcontrol.wait`: weights are read-only, so under programmatic
// dependent launch the slice is already in flight while the previous kernel
// on the stream drains.  With one CTA per SM the ring holds most or all of
// the slice, so the whole matrix is requested at once; the consumer warps
// then decode from shared memory at on-chip latency.
//
// Work decomposition (packed rows: one packed row = 8 values of K)
//   * A CTA owns a 128-column tile and a K slice of `rows_per_cta` rows; the
//     CTAs sharing a column tile form a thread-block cluster along gridDim.y
//     and reduce their partial sums through distributed shared memory in
//     fixed rank order (deterministic; no workspace, no second launch).
//   * Stage = kStageRows packed rows x 128 columns.  Consumer warp w decodes
//     rows [4w, 4w + 4) of every stage; lane l owns columns 4l..4l+3 (one
//     conflict-free 16-byte shared load per row).  Four packed rows = 32
//     values of K always lie inside one quantisation group (G >= 64).
//   * Scales for the slice are fetched into shared memory with cp.async and
//     activations are staged after `griddepcontrol.wait`, both while the
//     weight stream is in flight.
//   * Arithmetic per 4-row window is that of the cluster GEMV (gemv.cu): fp16
//     magic decode + packed half2 FMA flushed into fp32 by the group scale, or
//     the exact fp32 decode + packed fp32x2 FMA.
//   * Every mbarrier wait is bounded (1 s); on expiry the CTA records
//     kErrWaitTimeout, stops, waits (bounded) for the copies it issued, and
//     returns through the normal reduction path.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "ng_decode.cuh"
#include "sm100_primitives.cuh"

namespace cg = cooperative_groups;

namespace ngb {
namespace {

constexpr int kRCols = 128;                       // columns per tile
constexpr int kRowsPerWarp = 4;                   // packed rows per consumer warp per stage
constexpr int kMaxRingCluster = 8;

enum RPath { kRHalf2 = 0, kRFloat2 = 1 };

template <int CW>
struct RingCfg {
  static constexpr int kStageRows = CW * kRowsPerWarp;
  static constexpr int kStageBytes = kStageRows * kRCols * 4;
  static constexpr int kThreads = (CW + 1) * 32;  // + one producer warp
};

// Shared-memory carve-up, identical on host and device.
struct RingLayout {
  size_t ring, xs, sc, red, fin, total;
  __host__ __device__ RingLayout(int stages, int stage_bytes, int MT, int rows_per_cta, int xs_elem,
                                 int groups, int cw) {
    size_t off = 1024;  // mbarriers + abort flag
    ring = off;
    off += static_cast<size_t>(stages) * stage_bytes;
    xs = off;
    off += (static_cast<size_t>(MT) * rows_per_cta * 8 * xs_elem + 15) / 16 * 16;
    sc = off;
    off += static_cast<size_t>(groups) * kRCols * 2;
    red = off;
    off += static_cast<size_t>(cw) * MT * kRCols * 4;
    fin = off;
    off += static_cast<size_t>(MT) * kRCols * 4;
    total = off;
  }
};

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void cp_async_8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// Wait for a phase regardless of the abort flag (used only to drain copies).
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity, unsigned int* err) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 1000000000ull) {
      atomicOr(err, kErrWaitTimeout);
      return;
    }
  }
}

template <int MT, bool XBF16, int PATH, int CW>
__global__ void __launch_bounds__(RingCfg<CW>::kThreads, 1)
    gemv_ring_kernel(const void* __restrict__ x, const uint32_t* __restrict__ qw,
                     const __half* __restrict__ scales, void* __restrict__ y, int M, int K, int N,
                     int G, int rows_per_cta, int csize, int stages, unsigned int* __restrict__ err) {
  using Cfg = RingCfg<CW>;
  using XS = typename std::conditional<PATH == kRFloat2, float, __half>::type;
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + stages);

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int krows = K >> 3;
  const int kr0 = blockIdx.y * rows_per_cta;
  const int kr1 = min(krows, kr0 + rows_per_cta);
  const int nrows = max(0, kr1 - kr0);
  const int nst = (nrows + Cfg::kStageRows - 1) / Cfg::kStageRows;
  const int c0 = blockIdx.x * kRCols;
  const int g0 = (kr0 * 8) / G;
  const int ngroups = nrows > 0 ? (kr1 * 8 - 1) / G - g0 + 1 : 0;
  const RingLayout L(stages, Cfg::kStageBytes, MT, rows_per_cta, sizeof(XS),
                     rows_per_cta * 8 / G + 2, CW);
  unsigned char* ring = smem + L.ring;
  XS* xs = reinterpret_cast<XS*>(smem + L.xs);
  __half* ssm = reinterpret_cast<__half*>(smem + L.sc);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* fin = reinterpret_cast<float*>(smem + L.fin);
  const int xstride = rows_per_cta * 8;

  if (tid == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  float acc[4][MT];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[c][m] = 0.f;

  if (warp == CW) {
    // ---------------- producer: stream the slice through the ring ----------------
    const int ncols = min(kRCols, N - c0);
    const uint32_t row_bytes = static_cast<uint32_t>(ncols) * 4u;
    const uint64_t pol = make_evict_first_policy();
    int issued = 0;
    for (int s = 0; s < nst; ++s) {
      const int slot = s % stages;
      if (s >= stages) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait_bounded(&empty[slot], ((s / stages) - 1) & 1, err, abort_flag);
        if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) break;
      }
      const int rows_here = min(Cfg::kStageRows, nrows - s * Cfg::kStageRows);
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], rows_here * row_bytes);
      __syncwarp();
      unsigned char* dst = ring + static_cast<size_t>(slot) * Cfg::kStageBytes;
      for (int r = lane; r < rows_here; r += 32) {
        const int grow = kr0 + s * Cfg::kStageRows + r;
        bulk_g2s(dst + r * (kRCols * 4), qw + static_cast<size_t>(grow) * N + c0, row_bytes,
                 &full[slot], pol);
      }
      issued = s + 1;
    }
    // Drain: every copy this CTA issued has landed before shared memory is
    // reused or released (a no-op when the consumers saw every stage).
    if (lane == 0) {
      for (int s = max(0, issued - stages); s < issued; ++s)
        mbar_wait_drain(&full[s % stages], (s / stages) & 1, err);
    }
  } else {
    // ---------------- consumers ----------------
    // Scales of the slice (read-only: fetched before the dependency wait).
    for (int i = tid; i < ngroups * 32; i += CW * 32) {
      const int g = i >> 5, l = i & 31;
      const int col = c0 + l * 4;
      if (col < N) cp_async_8(ssm + g * kRCols + l * 4, scales + static_cast<size_t>(g0 + g) * N + col);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const unsigned short* xin = static_cast<const unsigned short*>(x);
    for (int i = tid; i < MT * nrows; i += CW * 32) {
      const int m = i / nrows;
      const int r = i - m * nrows;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (m < M) v = ld_ro_v4(xin + static_cast<size_t>(m) * K + static_cast<size_t>(kr0 + r) * 8);
      XS* dst = xs + m * xstride + r * 8;
      if constexpr (PATH == kRFloat2) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float f[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (XBF16) {
            f[2 * j] = __uint_as_float(w[j] << 16);
            f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
          } else {
            const float2 t = __half22float2(h2_from_bits(w[j]));
            f[2 * j] = t.x;
            f[2 * j + 1] = t.y;
          }
        }
        reinterpret_cast<float4*>(dst)[0] = make_float4(f[0], f[1], f[2], f[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(f[4], f[5], f[6], f[7]);
      } else {
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");  // consumers only

    for (int s = 0; s < nst; ++s) {
      const int slot = s % stages;
      if (!mbar_wait_bounded(&full[slot], (s / stages) & 1, err, abort_flag)) break;
      const int rows_here = min(Cfg::kStageRows, nrows - s * Cfg::kStageRows);
      const int rr0 = warp * kRowsPerWarp;
      if (rr0 < rows_here) {
        const unsigned char* src = ring + static_cast<size_t>(slot) * Cfg::kStageBytes;
        uint4 q[kRowsPerWarp];
#pragma unroll
        for (int u = 0; u < kRowsPerWarp; ++u)
          q[u] = *reinterpret_cast<const uint4*>(src + (rr0 + u) * (kRCols * 4) + lane * 16);
        const int lrow = s * Cfg::kStageRows + rr0;  // slice-local packed row
        const int grp = ((kr0 + lrow) * 8) / G - g0;
        const uint2 sv = *reinterpret_cast<const uint2*>(ssm + grp * kRCols + lane * 4);
        float sc[4];
        sc[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x & 0xFFFF)));
        sc[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x >> 16)));
        sc[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y & 0xFFFF)));
        sc[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y >> 16)));
        const XS* xc = xs + lrow * 8;
        if constexpr (PATH == kRHalf2) {
          __half2 h[4][MT];
#pragma unroll
          for (int c = 0; c < 4; ++c)
#pragma unroll
            for (int m = 0; m < MT; ++m) h[c][m] = __float2half2_rn(0.f);
#pragma unroll
          for (int u = 0; u < kRowsPerWarp; ++u) {
            const uint32_t words[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
            __half2 wv[4][4];
#pragma unroll
            for (int c = 0; c < 4; ++c) decode8_f16(words[c], wv[c]);
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              const uint4 xv = *reinterpret_cast<const uint4*>(xc + m * xstride + u * 8);
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
          for (int u = 0; u < kRowsPerWarp; ++u) {
            const uint32_t words[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
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
              const float4 xa = *reinterpret_cast<const float4*>(xc + m * xstride + u * 8);
              const float4 xb = *reinterpret_cast<const float4*>(xc + m * xstride + u * 8 + 4);
              const f2 xp[4] = {f2_make(xa.x, xa.y), f2_make(xa.z, xa.w), f2_make(xb.x, xb.y),
                                f2_make(xb.z, xb.w)};
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
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
#pragma unroll
    for (int m = 0; m < MT; ++m)
      *reinterpret_cast<float4*>(red + (warp * MT + m) * kRCols + lane * 4) =
          make_float4(acc[0][m], acc[1][m], acc[2][m], acc[3][m]);
  }
  __syncthreads();

  // ---------------- CTA reduction over consumer warps (fixed order) ----------------
  constexpr int E = MT * kRCols;
  auto store = [&](int e, float v) {
    const int m = e / kRCols;
    const int cn = c0 + (e % kRCols);
    if (m < M && cn < N) {
      unsigned short* yo = static_cast<unsigned short*>(y);
      yo[static_cast<size_t>(m) * N + cn] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                  : __half_as_ushort(__float2half_rn(v));
    }
  };
  for (int e = tid; e < E; e += Cfg::kThreads) {
    float v = 0.f;
#pragma unroll 4
    for (int w = 0; w < CW; ++w) v += red[w * E + e];
    if (csize == 1)
      store(e, v);
    else
      fin[e] = v;
  }
  if (csize == 1) return;
  // ---------------- cluster reduction over K slices through DSMEM ----------------
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int rank = static_cast<int>(cluster.block_rank());
  const int per = (E + csize - 1) / csize;
  const int e0 = rank * per;
  const int e1 = min(E, e0 + per);
  for (int e = e0 + tid; e < e1; e += Cfg::kThreads) {
    float v = 0.f;
    for (int r = 0; r < csize; ++r) v += cluster.map_shared_rank(fin, r)[e];
    store(e, v);
  }
  cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
constexpr int kCW = 8;

template <int MT, bool XBF16, int PATH>
int run_ring(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N, int G,
             int splits, const DeviceInfo& dev, cudaStream_t stream) {
  using Cfg = RingCfg<kCW>;
  auto kern = gemv_ring_kernel<MT, XBF16, PATH, kCW>;
  constexpr int esz = PATH == kRFloat2 ? 4 : 2;
  const int krows = K / 8;
  const int tiles = (N + kRCols - 1) / kRCols;
  const int sms = dev.sm_count;
  const size_t smem_cap = dev.smem_optin ? dev.smem_optin : 227 * 1024;

  static std::once_flag once[64];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem_cap));
  });

  auto layout = [&](int stages, int rows) {
    return RingLayout(stages, Cfg::kStageBytes, MT, rows, esz, rows * 8 / G + 2, kCW);
  };
  // Choose the K split C (cluster size): minimise the rows the busiest SM
  // streams, assuming CTAs spread evenly over the SMs, plus a small charge per
  // cluster rank for the DSMEM reduction.
  int C = 1;
  if (splits > 0) {
    C = splits;
  } else {
    long best = -1;
    for (int c = 1; c <= kMaxRingCluster; ++c) {
      const int rows = (((krows + c - 1) / c) + 7) / 8 * 8;
      if (rows < 8) break;
      const int ceff = (krows + rows - 1) / rows;
      if (ceff != c) continue;
      const long per_sm = static_cast<long>((tiles * c + sms - 1) / sms) * rows;
      const long cost = per_sm + 8L * c;
      if (best < 0 || cost < best) {
        best = cost;
        C = c;
      }
    }
  }
  C = std::max(1, std::min(C, std::min(kMaxRingCluster, krows / 8)));
  int rows_per_cta = (((krows + C - 1) / C) + 7) / 8 * 8;
  C = (krows + rows_per_cta - 1) / rows_per_cta;
  const int nst = (rows_per_cta + Cfg::kStageRows - 1) / Cfg::kStageRows;
  const int ctas_per_sm = std::max(1, std::min(2, (tiles * C + sms - 1) / sms));
  const size_t budget = smem_cap / ctas_per_sm - (ctas_per_sm > 1 ? 1024 : 0);
  int stages = std::min(nst, 12);
  while (stages > 2 && layout(stages, rows_per_cta).total > budget) --stages;
  if (stages < 1) stages = 1;
  if (layout(stages, rows_per_cta).total > smem_cap) return NG_ERR_BAD_SHAPE;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, C, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = layout(stages, rows_per_cta).total;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = C;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return launch_status(cudaLaunchKernelEx(&cfg, kern, x, qw, s, y, M, K, N, G, rows_per_cta, C,
                                          stages, dev.err));
}

template <bool XBF16, int PATH>
int ring_dispatch_m(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N,
                    int G, int splits, const DeviceInfo& dev, cudaStream_t st) {
  if (M <= 1) return run_ring<1, XBF16, PATH>(x, qw, s, y, M, K, N, G, splits, dev, st);
  if (M <= 2) return run_ring<2, XBF16, PATH>(x, qw, s, y, M, K, N, G, splits, dev, st);
  if (M <= 4) return run_ring<4, XBF16, PATH>(x, qw, s, y, M, K, N, G, splits, dev, st);
  return run_ring<8, XBF16, PATH>(x, qw, s, y, M, K, N, G, splits, dev, st);
}

}  // namespace

int gemv_ring(const void* x, int x_dtype, bool float_path, const uint32_t* q, const __half* s,
              void* y, int M, int K, int N, int G, int splits, const DeviceInfo& dev,
              cudaStream_t strm) {
  if (M > 8 || splits > kMaxRingCluster) return NG_ERR_BAD_ARGUMENT;
  if (x_dtype == NG_DTYPE_BF16)
    return ring_dispatch_m<true, kRFloat2>(x, q, s, y, M, K, N, G, splits, dev, strm);
  if (float_path) return ring_dispatch_m<false, kRFloat2>(x, q, s, y, M, K, N, G, splits, dev, strm);
  return ring_dispatch_m<false, kRHalf2>(x, q, s, y, M, K, N, G, splits, dev, strm);
}

}  // namespace ngb
