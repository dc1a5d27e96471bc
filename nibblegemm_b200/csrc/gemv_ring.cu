// Decode-regime fused dequant GEMV with a bulk-copy shared-memory ring:
// Y[M, N] = X[M, K] @ W for M <= 8, one launch.
//
// Why a ring: at M = 1 a GEMV is a 30 MB read that should take ~4.6 us, and a
// kernel whose warps load weights into registers keeps only as many bytes in
// flight as it has warps x registers; with few chunks per warp the load
// latency, the activation staging and the reductions are paid in series.
// Here one producer warp per CTA streams the CTA's whole weight slice with
// 2-D TMA loads (4 KB boxes of 128 columns x 8 packed rows, completion counted
// on an mbarrier) into a ring of stages, and it starts doing so *before*
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
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <type_traits>

#include "ng_decode.cuh"
#include "sm100_primitives.cuh"

namespace cg = cooperative_groups;

namespace ngb {
namespace {

constexpr int kRCols = 128;                       // columns per tile
constexpr int kMaxRingCluster = 8;

// Consumer arithmetic: CUDA-core half2 / fp32x2 (4 packed rows per warp per
// stage), or mma.sync on magic-number operands (16 rows per warp per stage).
enum RPath { kRHalf2 = 0, kRFloat2 = 1, kRMma = 2 };

// Stage geometry: SR packed rows per stage.  SR = CW x RW: every consumer warp
// takes RW rows of every stage.  SR < CW x RW: a stage is taken by SR / RW
// warps and the warp groups take consecutive stages round-robin (smaller
// stages, released as soon as their few warps are done).  Measured on B200:
// whole-CTA 64 KB stages are faster up to M = 8 (config 1: 9.3 us vs 11.0 us
// with 16 KB stages), 16 KB stages at M = 9..16, where the staged activations
// leave room for only a few large stages (14336 x 4096: 26 us vs 52 us).
template <int MT, int PATH>
constexpr int ring_stage_rows(int CW, int RW) { return (PATH == kRMma && MT > 8) ? 32 : CW * RW; }

template <int CW, int PATH, int RW, int SR = CW * RW>
struct RingCfg {
  static constexpr int kRowsPerWarp = RW;
  static constexpr int kStageRows = SR;
  static constexpr int kWarpsPerStage = kStageRows / RW;
  static constexpr int kStageGroups = CW / kWarpsPerStage;
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

constexpr int kBoxRows = 8;  // packed rows per TMA box: 128 x 8 words = 4 KB

// 2-D tiled TMA load of one (128-column, 8-row) box of the packed weight,
// L2 evict-first (each weight byte is read once).
__device__ __forceinline__ void tma_box_g2s(void* dst, const CUtensorMap* map, uint64_t* bar, int col,
                                            int row, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(col), "r"(row), "r"(smem_u32(bar)), "l"(policy)
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

template <bool BF16>
__device__ __forceinline__ void ring_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Magic-number MMA operands of one packed word, no subtract: h[p] holds the
// code pair p (k = 2p, 2p + 1) as two 16-bit values.
//   fp16: pairs 0 and 2 as 1024 + u; pairs 1 and 3 as 1024 + 16u, read in
//         place from nibble bits 4..7 of each half (one AND/OR, no shift) --
//         the matching activations are staged pre-divided by 16, so the
//         product is (64 + u) * x.  1 shift + 4 AND/OR per word.
//   bf16: every pair as 128 + u (bit 7 of a bf16 is exponent, so the high
//         nibbles are shifted down).  3 shifts + 4 AND/OR per word.
// Either way the product with x is exact in the fp32 accumulator; the offsets
// (fp16: 1032 x on pairs 0/2, 72 * 16 (x/16) on pairs 1/3; bf16: 136 x) are
// removed by a correction MMA with those constants as the A operand.
template <bool BF16>
__device__ __forceinline__ void decode_mma_operands(uint32_t q, uint32_t (&h)[4]) {
  if constexpr (BF16) {
    h[0] = and_or(q, 0x000F000Fu, 0x43004300u);
    h[1] = and_or(q >> 4, 0x000F000Fu, 0x43004300u);
    h[2] = and_or(q >> 8, 0x000F000Fu, 0x43004300u);
    h[3] = and_or(q >> 12, 0x000F000Fu, 0x43004300u);
  } else {
    const uint32_t q8 = q >> 8;
    h[0] = and_or(q, 0x000F000Fu, 0x64006400u);
    h[1] = and_or(q, 0x00F000F0u, 0x64006400u);
    h[2] = and_or(q8, 0x000F000Fu, 0x64006400u);
    h[3] = and_or(q8, 0x00F000F0u, 0x64006400u);
  }
}

template <int MT, bool XBF16, int PATH, int CW, int RW>
__global__ void __launch_bounds__(RingCfg<CW, PATH, RW, ring_stage_rows<MT, PATH>(CW, RW)>::kThreads, 1)
    gemv_ring_kernel(const __grid_constant__ CUtensorMap tmap_q, const void* __restrict__ x,
                     const __half* __restrict__ scales, void* __restrict__ y, int M, int K, int N,
                     int G, int rows_per_cta, int csize, int stages, unsigned int* __restrict__ err) {
  using Cfg = RingCfg<CW, PATH, RW, ring_stage_rows<MT, PATH>(CW, RW)>;
  constexpr int kRowsPerWarp = Cfg::kRowsPerWarp;
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
  if (nst > stages && stages % Cfg::kStageGroups != 0) {  // host guarantees this; never wait ambiguously
    if (threadIdx.x == 0) atomicOr(err, kErrWaitTimeout);
    return;
  }
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
      mbar_init(&empty[i], Cfg::kWarpsPerStage);
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
      const int boxes = rows_here / kBoxRows;  // slices are whole multiples of 8 rows
      if (lane == 0) mbar_arrive_expect_tx(&full[slot], boxes * (kBoxRows * kRCols * 4));
      __syncwarp();
      unsigned char* dst = ring + static_cast<size_t>(slot) * Cfg::kStageBytes;
      for (int b = lane; b < boxes; b += 32)
        tma_box_g2s(dst + b * (kBoxRows * kRCols * 4), &tmap_q, &full[slot], c0,
                    kr0 + s * Cfg::kStageRows + b * kBoxRows, pol);
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
      } else if constexpr (PATH == kRMma && !XBF16) {
        // pairs 1 and 3 (k = 2,3 and 6,7 of the row) meet the 16u operands
        const __half2 sixteenth = __float2half2_rn(0.0625f);
        v.y = h2_bits(__hmul2(h2_from_bits(v.y), sixteenth));
        v.w = h2_bits(__hmul2(h2_from_bits(v.w), sixteenth));
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        *reinterpret_cast<uint4*>(dst) = v;
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");  // consumers only

    if constexpr (PATH == kRMma) {
      // Fragment mapping (m16n8k16; lane = 4g + t).  Per 4-row step the lane
      // holds packed row (step + t), 16-byte runs at columns 64h + 4g and
      // 64h + 32 + 4g (h = 0, 1):  A row g <-> column 64h + 4g + i and A row
      // g + 8 <-> column 64h + 32 + 4g + i for the i-th word of the runs.
      // Virtual k pairs t / t + 4 of the first MMA are real pairs 0 / 1 of that
      // packed row, of the second MMA pairs 2 / 3, so the B fragment of lane
      // (g, t) is the staged activation row g, values 8 (step + t) .. + 7.
      const int g = lane >> 2, t = lane & 3;
      constexpr uint32_t kC0 = XBF16 ? 0x43084308u : 0x64086408u;  // 136 (bf16) / 1032 (fp16)
      constexpr uint32_t kC1 = XBF16 ? 0x43084308u : 0x64806480u;  // 136 (bf16) / 1152 (fp16)
      // NT tiles of 8 tokens (MMA N = 8): tokens 8 nt + g feed the B fragment
      constexpr int NT = (MT + 7) / 8;
      float tot[2][4][NT][4], c[2][4][NT][4], cv[NT][4];
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) tot[h][i][nt][r] = c[h][i][nt][r] = 0.f;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) cv[nt][r] = 0.f;
      for (int s = warp / Cfg::kWarpsPerStage; s < nst; s += Cfg::kStageGroups) {
        const int slot = s % stages;
        if (!mbar_wait_bounded(&full[slot], (s / stages) & 1, err, abort_flag)) break;
        const int rows_here = min(Cfg::kStageRows, nrows - s * Cfg::kStageRows);
        const int rr0 = (warp % Cfg::kWarpsPerStage) * kRowsPerWarp;
        const int rend = min(rr0 + kRowsPerWarp, rows_here);
        const unsigned char* stage_base = ring + static_cast<size_t>(slot) * Cfg::kStageBytes;
#pragma unroll
        for (int step = 0; step < kRowsPerWarp / 4; ++step) {
          const int row = rr0 + 4 * step;
          if (row >= rend) break;
          const unsigned char* src = stage_base + (row + t) * (kRCols * 4);
          uint4 w[4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            w[2 * h] = *reinterpret_cast<const uint4*>(src + (64 * h + 4 * g) * 4);
            w[2 * h + 1] = *reinterpret_cast<const uint4*>(src + (64 * h + 32 + 4 * g) * 4);
          }
          const int lrow = s * Cfg::kStageRows + row;  // slice-local packed row of the step
          uint4 xv[NT];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            xv[nt] = make_uint4(0u, 0u, 0u, 0u);
            if (8 * nt + g < MT)
              xv[nt] = *reinterpret_cast<const uint4*>(xs + (8 * nt + g) * xstride + (lrow + t) * 8);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t wa[4] = {w[2 * h].x, w[2 * h].y, w[2 * h].z, w[2 * h].w};
            const uint32_t wb[4] = {w[2 * h + 1].x, w[2 * h + 1].y, w[2 * h + 1].z, w[2 * h + 1].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t ha[4], hb[4];
              decode_mma_operands<XBF16>(wa[i], ha);
              decode_mma_operands<XBF16>(wb[i], hb);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) {
                ring_mma<XBF16>(c[h][i][nt], ha[0], hb[0], ha[1], hb[1], xv[nt].x, xv[nt].y);
                ring_mma<XBF16>(c[h][i][nt], ha[2], hb[2], ha[3], hb[3], xv[nt].z, xv[nt].w);
              }
            }
          }
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            ring_mma<XBF16>(cv[nt], kC0, kC0, kC1, kC1, xv[nt].x, xv[nt].y);
            ring_mma<XBF16>(cv[nt], kC0, kC0, kC1, kC1, xv[nt].z, xv[nt].w);
          }
          // flush at the end of a quantisation group or of this warp's rows
          const int gnext = kr0 + lrow + 4;
          if ((gnext * 8) % G == 0 || row + 4 >= rend) {
            const int grp = ((kr0 + lrow) * 8) / G - g0;
            const __half* sg = ssm + grp * kRCols;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint2 sa = *reinterpret_cast<const uint2*>(sg + 64 * h + 4 * g);
              const uint2 sb = *reinterpret_cast<const uint2*>(sg + 64 * h + 32 + 4 * g);
              const float2 a01 = __half22float2(h2_from_bits(sa.x)), a23 = __half22float2(h2_from_bits(sa.y));
              const float2 b01 = __half22float2(h2_from_bits(sb.x)), b23 = __half22float2(h2_from_bits(sb.y));
              const float fa[4] = {a01.x, a01.y, a23.x, a23.y};
              const float fb[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                  for (int r = 0; r < 4; ++r) {
                    if (MT == 1 && (r & 1)) continue;  // token 2t + 1 >= 1: nothing to keep
                    tot[h][i][nt][r] = fmaf(r < 2 ? fa[i] : fb[i], c[h][i][nt][r] - cv[nt][r & 1], tot[h][i][nt][r]);
                    c[h][i][nt][r] = 0.f;
                  }
            }
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
              for (int r = 0; r < 4; ++r) cv[nt][r] = 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      // warp partials: lane (g, t) holds tokens 2t, 2t + 1 of 16 columns
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
              const int m = 8 * nt + 2 * t + (r & 1);
              const int col = 64 * h + (r < 2 ? 0 : 32) + 4 * g + i;
              if (m < MT) red[(warp * MT + m) * kRCols + col] = tot[h][i][nt][r];
            }
    } else {
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
// Stream-K ring (tensor-pipe consumer; M <= 4; X fits on chip; workspace).
//
// The grid above gives each 128-column tile the same K split, so a shape with
// T tiles keeps only T x C of the 148 SMs busy (config 1: 112).  Here the
// work is the list of 16-row blocks in tile-major order, split into equal
// contiguous ranges over one persistent CTA per SM.  Each stage holds up to 8
// consecutive blocks of one tile (consumer warp w takes block w, exactly the
// per-warp arithmetic of the ring above).  When a CTA's range leaves a tile it
// reduces its warps' partials for that tile (a "segment"):
//   * a segment covering the whole tile is written to Y directly;
//   * a segment that starts inside the tile (only a CTA's first segment can)
//     is published to the workspace: partial sums, then a flag (release);
//   * a segment that starts at the tile's first row but stops short is
//     finished by this CTA: it waits (bounded) for the flags of the later
//     CTAs holding the rest of the tile, adds their partials in CTA order
//     (deterministic), writes Y and clears the flags.
// A CTA reaches the tile it finishes at the end of its range, while the later
// CTAs publish theirs at the start of their ranges, so the wait is short and
// never circular.  The grid is at most one CTA per SM, so all CTAs become
// resident once the previous kernel drains.
// Measured trade-off: CTAs here stream different rows at the same time,
// which costs DRAM locality against the clustered grid (whose CTAs sweep the
// matrix rows in lockstep); it wins where the clustered grid would leave most
// SMs idle (few column tiles, long K) at M = 3..4.
// ---------------------------------------------------------------------------
constexpr int kSkRB = 16;                          // packed rows per block
constexpr int kSkCW = 8;                           // consumer warps
constexpr int kSkStageRows = kSkCW * kSkRB;        // 128
constexpr int kSkStageBytes = kSkStageRows * kRCols * 4;
constexpr int kSkThreads = (kSkCW + 1) * 32;
constexpr int kSkMaxM = 4;

struct SkPart {  // U blocks over P CTAs: the first r get q + 1, the rest q
  int q, r;
  __host__ __device__ int start(int b) const { return b * q + (b < r ? b : r); }
  __host__ __device__ int owner(int u) const {
    const int big = r * (q + 1);
    return u < big ? u / (q + 1) : r + (u - big) / q;
  }
};

// Work plan, shared by host and device.  Two modes:
//   * stream-K (ht = 0): the tile-major list of T x RT blocks split into equal
//     contiguous ranges over the P CTAs (`part`); slot b = CTA b's published
//     partial; the first CTA of a split tile finishes it.
//   * head/tail (ht = 1, T < P): CTA t < T streams the first B0 blocks of tile
//     t (its head, in lockstep with the other tile CTAs) and finishes the
//     tile; the P - T helper CTAs split the tile-major list of tails (RT - B0
//     blocks each) into equal contiguous ranges (`part`, at least a whole tail
//     each, so a tail has at most two helpers) and publish to slot 2t + part,
//     part 0 for the helper holding the tail's first block.  Balances the work
//     per SM over all SMs while every CTA still sweeps rows in order.
struct SkPlan {
  int ht, T, RT, B0, P;
  SkPart part;
  // number of segments (runs of blocks inside one tile) of CTA b
  __host__ __device__ int nseg(int b) const {
    if (ht) {
      if (b < T) return 1;
      const int TL = RT - B0, v0 = part.start(b - T), v1 = part.start(b - T + 1);
      return v1 > v0 ? (v1 - 1) / TL - v0 / TL + 1 : 0;
    }
    const int u0 = part.start(b), u1 = part.start(b + 1);
    return u1 > u0 ? (u1 - 1) / RT - u0 / RT + 1 : 0;
  }
  // segment k of CTA b: tile, first block, blocks, role (0 store, 1 finish
  // from slots [s_lo, s_hi], 2 publish to slot s_lo)
  __host__ __device__ void seg(int b, int k, int& tile, int& blk0, int& nblk, int& role, int& s_lo,
                      int& s_hi) const {
    if (ht) {
      const int TL = RT - B0;
      if (b < T) {
        tile = b, blk0 = 0, nblk = B0;
        role = TL == 0 ? 0 : 1;
        s_lo = 2 * tile;
        s_hi = 2 * tile + (part.owner(tile * TL) != part.owner(tile * TL + TL - 1) ? 1 : 0);
        return;
      }
      const int v0 = part.start(b - T), v1 = part.start(b - T + 1);
      tile = v0 / TL + k;
      const int lo = (v0 > tile * TL ? v0 : tile * TL), hi = (v1 < (tile + 1) * TL ? v1 : (tile + 1) * TL);
      blk0 = B0 + lo - tile * TL, nblk = hi - lo, role = 2;
      s_lo = s_hi = 2 * tile + (lo == tile * TL ? 0 : 1);
      return;
    }
    const int u0 = part.start(b), u1 = part.start(b + 1);
    tile = u0 / RT + k;
    const int lo = (u0 > tile * RT ? u0 : tile * RT), hi = (u1 < (tile + 1) * RT ? u1 : (tile + 1) * RT);
    blk0 = lo - tile * RT, nblk = hi - lo;
    const bool starts = lo == tile * RT, ends = hi == (tile + 1) * RT;
    role = starts && ends ? 0 : (starts ? 1 : 2);
    if (role == 2) {
      s_lo = s_hi = b;
    } else {
      s_lo = b + 1;
      s_hi = part.owner((tile + 1) * RT - 1);
    }
  }
};

struct SkLayout {
  size_t ring, xs, sc, red, fin, total;
  __host__ __device__ SkLayout(int stages, int MT, int K, int groups) {
    size_t off = 1024;
    ring = off;
    off += static_cast<size_t>(stages) * kSkStageBytes;
    xs = off;
    off += (static_cast<size_t>(MT) * K * 2 + 15) / 16 * 16;
    sc = off;
    off += static_cast<size_t>(groups) * kRCols * 2;
    red = off;
    off += static_cast<size_t>(kSkCW) * MT * kRCols * 4;
    fin = off;
    off += static_cast<size_t>(MT) * kRCols * 4;
    total = off;
  }
};

__device__ __forceinline__ unsigned int sk_ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void sk_st_release(unsigned int* p, unsigned int v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int MT, bool XBF16>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemv_ring_sk_kernel(const __grid_constant__ CUtensorMap tmap_q, const void* __restrict__ x,
                        const __half* __restrict__ scales, void* __restrict__ y, int M, int K,
                        int N, int G, SkPlan plan, int stages, int sc_groups,
                        float* __restrict__ ws_part, unsigned int* __restrict__ ws_flag,
                        unsigned int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + stages);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int krows = K >> 3;
  const int b = blockIdx.x;
  const int nseg = plan.nseg(b);
  const int GR = G / 8;  // packed rows per quantisation group
  const SkLayout L(stages, MT, K, sc_groups);
  unsigned char* ring = smem + L.ring;
  __half* xs = reinterpret_cast<__half*>(smem + L.xs);
  __half* ssm = reinterpret_cast<__half*>(smem + L.sc);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* fin = reinterpret_cast<float*>(smem + L.fin);

  if (tid == 0) {
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kSkCW);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == kSkCW) {
    // ---------------- producer: the segments' blocks, 8 per stage ----------------
    const uint64_t pol = make_evict_first_policy();
    int s = 0, issued = 0;
    bool stop = false;
    for (int k = 0; k < nseg && !stop; ++k) {
      int tile, blk0, nblk, role, s_lo, s_hi;
      plan.seg(b, k, tile, blk0, nblk, role, s_lo, s_hi);
      for (int o = 0; o < nblk; o += kSkCW, ++s) {
        const int n = min(kSkCW, nblk - o);
        const int slot = s % stages;
        if (s >= stages) {
          bool ok = true;
          if (lane == 0) ok = mbar_wait_bounded(&empty[slot], ((s / stages) - 1) & 1, err, abort_flag);
          if (!__shfl_sync(0xffffffffu, ok ? 1 : 0, 0)) {
            stop = true;
            break;
          }
        }
        const int boxes = n * (kSkRB / kBoxRows);
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], boxes * (kBoxRows * kRCols * 4));
        __syncwarp();
        unsigned char* dst = ring + static_cast<size_t>(slot) * kSkStageBytes;
        if (lane < boxes)
          tma_box_g2s(dst + lane * (kBoxRows * kRCols * 4), &tmap_q, &full[slot], tile * kRCols,
                      (blk0 + o) * kSkRB + lane * kBoxRows, pol);
        issued = s + 1;
      }
    }
    if (lane == 0)
      for (int t = max(0, issued - stages); t < issued; ++t)
        mbar_wait_drain(&full[t % stages], (t / stages) & 1, err);
    return;  // segment barriers below are consumer-only (named barrier 1)
  }

  // ---------------- consumers ----------------
  // Scales of every segment, packed segment after segment.
  {
    int base = 0;
    for (int k = 0; k < nseg; ++k) {
      int tile, blk0, nblk, role, s_lo, s_hi;
      plan.seg(b, k, tile, blk0, nblk, role, s_lo, s_hi);
      const int gs = (blk0 * kSkRB) / GR, ge = ((blk0 + nblk) * kSkRB - 1) / GR;
      for (int i = tid; i < (ge - gs + 1) * 32; i += kSkCW * 32) {
        const int gg = i >> 5, l = i & 31;
        const int col = tile * kRCols + l * 4;
        if (col < N)
          cp_async_8(ssm + (base + gg) * kRCols + l * 4, scales + static_cast<size_t>(gs + gg) * N + col);
      }
      base += ge - gs + 1;
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  {
    const unsigned short* xin = static_cast<const unsigned short*>(x);
    for (int i = tid; i < MT * krows; i += kSkCW * 32) {
      const int m = i / krows, r = i - m * krows;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (m < M) v = ld_ro_v4(xin + static_cast<size_t>(m) * K + static_cast<size_t>(r) * 8);
      if constexpr (!XBF16) {
        const __half2 sixteenth = __float2half2_rn(0.0625f);
        v.y = h2_bits(__hmul2(h2_from_bits(v.y), sixteenth));
        v.w = h2_bits(__hmul2(h2_from_bits(v.w), sixteenth));
      }
      *reinterpret_cast<uint4*>(xs + static_cast<size_t>(m) * K + r * 8) = v;
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  asm volatile("bar.sync 1, %0;" ::"n"(kSkCW * 32) : "memory");

  const int g = lane >> 2, t = lane & 3;
  constexpr uint32_t kC0 = XBF16 ? 0x43084308u : 0x64086408u;
  constexpr uint32_t kC1 = XBF16 ? 0x43084308u : 0x64806480u;
  float tot[2][4][4], c[2][4][4], cv[4];
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int r = 0; r < 4; ++r) tot[h][i][r] = c[h][i][r] = 0.f;
#pragma unroll
  for (int r = 0; r < 4; ++r) cv[r] = 0.f;

  constexpr int E = MT * kRCols;
  constexpr size_t kSlot = kSkMaxM * kRCols;  // floats per workspace slot
  unsigned short* yo = static_cast<unsigned short*>(y);
  int s = 0, base = 0;
  bool aborted = false;
  for (int k = 0; k < nseg; ++k) {
    int tile, blk0, nblk, role, s_lo, s_hi;
    plan.seg(b, k, tile, blk0, nblk, role, s_lo, s_hi);
    const int gs = (blk0 * kSkRB) / GR;
    for (int o = 0; o < nblk; o += kSkCW, ++s) {
      const int n = min(kSkCW, nblk - o);
      const int slot = s % stages;
      if (!aborted && !mbar_wait_bounded(&full[slot], (s / stages) & 1, err, abort_flag)) aborted = true;
      if (!aborted && warp < n) {
        const int row0 = (blk0 + o + warp) * kSkRB;  // tile row of this warp's block
        const unsigned char* blk = ring + static_cast<size_t>(slot) * kSkStageBytes +
                                   warp * (kSkRB * kRCols * 4);
#pragma unroll
        for (int step = 0; step < kSkRB / 4; ++step) {
          const int row = row0 + 4 * step;
          const unsigned char* src = blk + (4 * step + t) * (kRCols * 4);
          uint4 w[4];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            w[2 * h] = *reinterpret_cast<const uint4*>(src + (64 * h + 4 * g) * 4);
            w[2 * h + 1] = *reinterpret_cast<const uint4*>(src + (64 * h + 32 + 4 * g) * 4);
          }
          uint4 xv = make_uint4(0u, 0u, 0u, 0u);
          if (g < MT) xv = *reinterpret_cast<const uint4*>(xs + static_cast<size_t>(g) * K + (row + t) * 8);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint32_t wa[4] = {w[2 * h].x, w[2 * h].y, w[2 * h].z, w[2 * h].w};
            const uint32_t wb[4] = {w[2 * h + 1].x, w[2 * h + 1].y, w[2 * h + 1].z, w[2 * h + 1].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint32_t ha[4], hb[4];
              decode_mma_operands<XBF16>(wa[i], ha);
              decode_mma_operands<XBF16>(wb[i], hb);
              ring_mma<XBF16>(c[h][i], ha[0], hb[0], ha[1], hb[1], xv.x, xv.y);
              ring_mma<XBF16>(c[h][i], ha[2], hb[2], ha[3], hb[3], xv.z, xv.w);
            }
          }
          ring_mma<XBF16>(cv, kC0, kC0, kC1, kC1, xv.x, xv.y);
          ring_mma<XBF16>(cv, kC0, kC0, kC1, kC1, xv.z, xv.w);
          if ((row + 4) % GR == 0 || step == kSkRB / 4 - 1) {  // group or block end
            const __half* sg = ssm + (base + row / GR - gs) * kRCols;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint2 sa = *reinterpret_cast<const uint2*>(sg + 64 * h + 4 * g);
              const uint2 sb = *reinterpret_cast<const uint2*>(sg + 64 * h + 32 + 4 * g);
              const float2 a01 = __half22float2(h2_from_bits(sa.x)), a23 = __half22float2(h2_from_bits(sa.y));
              const float2 b01 = __half22float2(h2_from_bits(sb.x)), b23 = __half22float2(h2_from_bits(sb.y));
              const float fa[4] = {a01.x, a01.y, a23.x, a23.y};
              const float fb[4] = {b01.x, b01.y, b23.x, b23.y};
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                  if (MT == 1 && (r & 1)) continue;
                  tot[h][i][r] = fmaf(r < 2 ? fa[i] : fb[i], c[h][i][r] - cv[r & 1], tot[h][i][r]);
                  c[h][i][r] = 0.f;
                }
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) cv[r] = 0.f;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
    base += ((blk0 + nblk) * kSkRB - 1) / GR - gs + 1;

    // ---- segment end: this CTA's share of `tile` is complete ----
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int m = 2 * t + (r & 1);
          const int col = 64 * h + (r < 2 ? 0 : 32) + 4 * g + i;
          if (m < MT) red[(warp * MT + m) * kRCols + col] = tot[h][i][r];
          tot[h][i][r] = 0.f;
        }
    asm volatile("bar.sync 1, %0;" ::"n"(kSkCW * 32) : "memory");  // (1) warp partials visible
    auto store = [&](int e, float v) {
      const int m = e / kRCols, cn = tile * kRCols + (e % kRCols);
      if (m < M && cn < N)
        yo[static_cast<size_t>(m) * N + cn] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                    : __half_as_ushort(__float2half_rn(v));
    };
    for (int e = tid; e < E; e += kSkCW * 32) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kSkCW; ++w) v += red[w * E + e];
      if (role == 0)
        store(e, v);
      else if (role == 1)
        fin[e] = v;
      else
        ws_part[static_cast<size_t>(s_lo) * kSlot + e] = v;
    }
    if (role == 2) __threadfence();
    asm volatile("bar.sync 1, %0;" ::"n"(kSkCW * 32) : "memory");  // (2)
    if (role == 2) {
      if (tid == 0) sk_st_release(&ws_flag[s_lo], 1u);
    } else if (role == 1) {
      if (tid == 0) {
        for (int o = s_lo; o <= s_hi; ++o) {
          const uint64_t ts = global_timer_ns();
          while (sk_ld_acquire(&ws_flag[o]) == 0u) {
            if (global_timer_ns() - ts > 1000000000ull) {
              atomicOr(err, kErrWaitTimeout);
              break;
            }
          }
        }
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSkCW * 32) : "memory");
      for (int e = tid; e < E; e += kSkCW * 32) {
        float v = fin[e];
        for (int o = s_lo; o <= s_hi; ++o) v += __ldcg(ws_part + static_cast<size_t>(o) * kSlot + e);
        store(e, v);
      }
      asm volatile("bar.sync 1, %0;" ::"n"(kSkCW * 32) : "memory");
      if (tid == 0)
        for (int o = s_lo; o <= s_hi; ++o) ws_flag[o] = 0u;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kSkCW * 32) : "memory");  // (3) red / fin reusable
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
constexpr int kCW = 8;

template <int MT, bool XBF16, int PATH, int RW>
int run_ring(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N, int G,
             int splits, const DeviceInfo& dev, cudaStream_t stream) {
  using Cfg = RingCfg<kCW, PATH, RW, ring_stage_rows<MT, PATH>(kCW, RW)>;
  auto kern = gemv_ring_kernel<MT, XBF16, PATH, kCW, RW>;
  constexpr int esz = PATH == kRFloat2 ? 4 : 2;
  const int krows = K / 8;
  const int tiles = (N + kRCols - 1) / kRCols;
  const int sms = dev.sm_count;
  const size_t smem_cap = dev.smem_optin ? dev.smem_optin : 227 * 1024;

  static std::once_flag once[kMaxDevices];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem_cap));
  });

  auto layout = [&](int stages, int rows) {
    return RingLayout(stages, Cfg::kStageBytes, MT, rows, esz, rows * 8 / G + 2, kCW);
  };
  // K split C (= cluster size): the largest of 1, 2, 4 that keeps the grid
  // within one CTA per SM and at least 128 packed rows per CTA (measured on
  // B200: a second CTA per SM, or clusters of 3, 6 or 8, cost more than they
  // hide; thinner slices pay the fixed per-CTA cost).  Huge N: C = 1.
  int C = 1;
  if (splits > 0) {
    C = splits;
  } else {
    for (int c : {2, 4})
      if (tiles * c <= sms && krows / c >= 128) C = c;
  }
  // The slice's staged activations plus two ring stages must fit on chip
  // (M = 9..16 at long K): the split count is raised if needed (a request, not
  // a promise, as for the cluster GEMV).
  constexpr int SG = Cfg::kStageGroups;
  constexpr int kMinStages = SG > 2 ? SG : 2;
  auto slice_rows = [&](int c) { return (((krows + c - 1) / c) + 7) / 8 * 8; };
  while (C < kMaxRingCluster && layout(kMinStages, slice_rows(C)).total > smem_cap)
    C = std::min(kMaxRingCluster, C * 2);
  C = std::max(1, std::min(C, std::min(kMaxRingCluster, krows / 8)));
  int rows_per_cta = (((krows + C - 1) / C) + 7) / 8 * 8;
  C = (krows + rows_per_cta - 1) / rows_per_cta;
  const int nst = (rows_per_cta + Cfg::kStageRows - 1) / Cfg::kStageRows;
  // Shared memory: as deep a ring as fits (measured: a ring under half the SM,
  // which would let the next kernel's CTA become resident early, is slower).
  const int ctas_per_sm = std::max(1, std::min(2, (tiles * C + sms - 1) / sms));
  size_t budget = ctas_per_sm == 1 ? smem_cap : smem_cap / 2 - 1024;
  int stages = std::min(nst, 12);
  while (stages > 1 && layout(stages, rows_per_cta).total > budget) --stages;
  if (stages < 1) stages = 1;
  // Ring slots are reused (nst > stages) only with a stage count that is a
  // multiple of the warp groups taking stages round-robin: then every slot
  // belongs to one group, which waits on that slot's phases strictly in order.
  // Otherwise a group could wait on a slot two phases ahead of its current one
  // and the parity test of the mbarrier wait would pass early.
  if (nst > stages) {
    stages = stages / SG * SG;
    if (stages < SG) stages = SG;
  }
  if (nst > stages && stages % SG != 0) return NG_ERR_BAD_SHAPE;
  if (layout(stages, rows_per_cta).total > smem_cap) return NG_ERR_BAD_SHAPE;

  CUtensorMap tmap;
  {
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
    if (!enc) return NG_ERR_CUDA;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(krows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRCols), static_cast<cuuint32_t>(kBoxRows)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(qw), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
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
  return launch_status(cudaLaunchKernelEx(&cfg, kern, tmap, x, s, y, M, K, N, G, rows_per_cta, C,
                                          stages, dev.err));
}

template <bool XBF16, int PATH, int RW>
int ring_dispatch_m(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N,
                    int G, int splits, const DeviceInfo& dev, cudaStream_t st) {
  if (M <= 1) return run_ring<1, XBF16, PATH, RW>(x, qw, s, y, M, K, N, G, splits, dev, st);
  if (M <= 2) return run_ring<2, XBF16, PATH, RW>(x, qw, s, y, M, K, N, G, splits, dev, st);
  if (M <= 4) return run_ring<4, XBF16, PATH, RW>(x, qw, s, y, M, K, N, G, splits, dev, st);
  if (M <= 8 || PATH != kRMma) return run_ring<8, XBF16, PATH, RW>(x, qw, s, y, M, K, N, G, splits, dev, st);
  return run_ring<16, XBF16, kRMma, RW>(x, qw, s, y, M, K, N, G, splits, dev, st);
}

// Tensor-pipe consumer: packed rows per warp per stage (16 = fewest flushes,
// 4 / 8 = smaller stages, more of them in the ring).
template <bool XBF16>
int ring_mma_dispatch(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K,
                      int N, int G, int splits, const DeviceInfo& dev, cudaStream_t st) {
  // 16 rows per warp (fewest flushes) unless the staged activations of 8
  // rows of X leave room for only ~2 of those 64 KB stages.
  int rw = M > 4 ? 8 : 16;
  if (rw == 4) return ring_dispatch_m<XBF16, kRMma, 4>(x, qw, s, y, M, K, N, G, splits, dev, st);
  if (rw == 8) return ring_dispatch_m<XBF16, kRMma, 8>(x, qw, s, y, M, K, N, G, splits, dev, st);
  return ring_dispatch_m<XBF16, kRMma, 16>(x, qw, s, y, M, K, N, G, splits, dev, st);
}


// Workspace of the stream-K ring: partial sums then flags, after the region
// the tensor-pipe persistent GEMV (algo 3) uses, so the two never overlap.
size_t sk_ws_offset(int N, const DeviceInfo& dev) {
  return (gemv_tc_workspace_bytes(N, dev) + 255) / 256 * 256;
}
size_t sk_ws_bytes(const DeviceInfo& dev) {  // 2 x SMs slots (head/tail uses 2 per tile) + flags
  return static_cast<size_t>(2 * dev.sm_count) * (kSkMaxM * kRCols * 4 + 4);
}

// The work plan for an N x K weight: head/tail when the tiles fill between
// half and all of the SMs and every helper's share covers a whole tail,
// stream-K otherwise.  Returns false when neither applies.
bool make_sk_plan(int tiles, int RT, int sms, SkPlan* plan) {
  const int U = tiles * RT;
  if (tiles * 2 >= sms && tiles < sms && RT >= 2) {
    const int H = sms - tiles;
    int B0 = (tiles * RT + sms / 2) / sms;  // blocks per SM if all SMs did the same
    B0 = B0 < 1 ? 1 : (B0 > RT - 1 ? RT - 1 : B0);
    const int TL = RT - B0, tail = tiles * TL;
    if (tail / H >= TL) {
      *plan = SkPlan{1, tiles, RT, B0, sms, SkPart{tail / H, tail % H}};
      return true;
    }
  }
  const int P = sms < U ? sms : U;
  *plan = SkPlan{0, tiles, RT, 0, P, SkPart{U / P, U % P}};
  return true;
}

// Returns NG_OK, an error, or -1 when the stream-K ring does not apply.
template <int MT, bool XBF16>
int run_ring_sk(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N,
                int G, void* ws, size_t ws_bytes, const DeviceInfo& dev, cudaStream_t stream) {
  const int krows = K / 8;
  if (krows % kSkRB != 0) return -1;
  if (static_cast<size_t>(MT) * K * 2 > 64 * 1024) return -1;
  const size_t off = sk_ws_offset(N, dev);
  if (ws == nullptr || ws_bytes < off + sk_ws_bytes(dev)) return -1;
  const int RT = krows / kSkRB;
  const int tiles = (N + kRCols - 1) / kRCols;
  SkPlan plan;
  if (!make_sk_plan(tiles, RT, dev.sm_count, &plan)) return -1;
  const int P = plan.P;
  // shared-memory scale rows and ring depth: the largest any CTA needs
  int sc_groups = 1, max_blocks = 1;
  for (int b = 0; b < P; ++b) {
    int groups = 0, blocks = 0;
    for (int k = 0; k < plan.nseg(b); ++k) {
      int tile, blk0, nblk, role, s_lo, s_hi;
      plan.seg(b, k, tile, blk0, nblk, role, s_lo, s_hi);
      groups += ((blk0 + nblk) * kSkRB - 1) / (G / 8) - (blk0 * kSkRB) / (G / 8) + 1;
      blocks += (nblk + kSkCW - 1) / kSkCW;  // stages of this segment
    }
    sc_groups = std::max(sc_groups, groups);
    max_blocks = std::max(max_blocks, blocks);
  }
  const size_t smem_cap = dev.smem_optin ? dev.smem_optin : 227 * 1024;
  int stages = std::min(4, max_blocks);
  while (stages > 1 && SkLayout(stages, MT, K, sc_groups).total > smem_cap) --stages;
  const size_t smem = SkLayout(stages, MT, K, sc_groups).total;
  if (smem > smem_cap) return -1;

  auto kern = gemv_ring_sk_kernel<MT, XBF16>;
  static std::once_flag once[kMaxDevices];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem_cap));
  });
  CUtensorMap tmap;
  {
    auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
    if (!enc) return NG_ERR_CUDA;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(krows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kRCols), static_cast<cuuint32_t>(kBoxRows)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(qw), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  float* ws_part = reinterpret_cast<float*>(static_cast<unsigned char*>(ws) + off);
  unsigned int* ws_flag =
      reinterpret_cast<unsigned int*>(ws_part + static_cast<size_t>(2 * dev.sm_count) * kSkMaxM * kRCols);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P, 1, 1);
  cfg.blockDim = dim3(kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Cooperative: a tile's finisher waits for the CTAs holding its other blocks,
  // so every CTA must be resident at once; the launch fails (no hang) when they
  // cannot be, e.g. while another kernel holds the SMs.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return launch_status(cudaLaunchKernelEx(&cfg, kern, tmap, x, s, y, M, K, N, G, plan, stages,
                                          sc_groups, ws_part, ws_flag, dev.err));
}

template <bool XBF16>
int ring_sk_dispatch(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N,
                     int G, void* ws, size_t ws_bytes, const DeviceInfo& dev, cudaStream_t st) {
  if (M <= 1) return run_ring_sk<1, XBF16>(x, qw, s, y, M, K, N, G, ws, ws_bytes, dev, st);
  if (M <= 2) return run_ring_sk<2, XBF16>(x, qw, s, y, M, K, N, G, ws, ws_bytes, dev, st);
  if (M <= 4) return run_ring_sk<4, XBF16>(x, qw, s, y, M, K, N, G, ws, ws_bytes, dev, st);
  return -1;
}

}  // namespace

size_t gemv_ring_workspace_bytes(int N, const DeviceInfo& dev) {
  return sk_ws_offset(N, dev) + sk_ws_bytes(dev);
}

int gemv_ring(const void* x, int x_dtype, bool tensor_pipe, const uint32_t* q, const __half* s,
              void* y, int M, int K, int N, int G, int splits, void* ws, size_t ws_bytes,
              const DeviceInfo& dev, cudaStream_t strm) {
  if (M > (tensor_pipe ? 16 : 8) || splits > kMaxRingCluster) return NG_ERR_BAD_ARGUMENT;
  // Stream-K over all SMs when it applies (tensor pipe, M <= 4, X on chip, a
  // workspace, no explicit split); the clustered K split otherwise.
  if (tensor_pipe && splits == 0 && M <= kSkMaxM) {
    const int st = x_dtype == NG_DTYPE_BF16
                       ? ring_sk_dispatch<true>(x, q, s, y, M, K, N, G, ws, ws_bytes, dev, strm)
                       : ring_sk_dispatch<false>(x, q, s, y, M, K, N, G, ws, ws_bytes, dev, strm);
    if (st != -1) return st;
  }
  if (x_dtype == NG_DTYPE_BF16) {
    if (tensor_pipe) return ring_mma_dispatch<true>(x, q, s, y, M, K, N, G, splits, dev, strm);
    return ring_dispatch_m<true, kRFloat2, 4>(x, q, s, y, M, K, N, G, splits, dev, strm);
  }
  if (tensor_pipe) return ring_mma_dispatch<false>(x, q, s, y, M, K, N, G, splits, dev, strm);
  return ring_dispatch_m<false, kRHalf2, 4>(x, q, s, y, M, K, N, G, splits, dev, strm);
}

}  // namespace ngb
