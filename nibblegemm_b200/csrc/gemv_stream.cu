// Decode-regime fused dequant GEMV, bulk-copy tensor-pipe schedule (algo 6):
// Y[M, N] = X[M, K] @ W for M <= 16, one launch.
//
// What sets the time (measured on B200, config 1 = 30.3 MB of weights, CUDA
// graph of back-to-back launches): 9.3 us per launch, the same as the ring
// schedule (algo 5).  With the consumers' arithmetic compiled out the same
// TMA pipeline reads config 1 in 6.2-6.8 us, so the consumers (decode + MMA at
// about 0.5 IPC on the 112 SMs that 112 column tiles occupy) set the time,
// not the copies.  Variants measured and not kept: deeper rings (4-6 stages),
// 8 instead of 16 consumer warps (14.6 us), K split over clusters of 2-8 CTAs
// (10.5-19.7 us), registers instead of a shared-memory ring (11-21 us), and a
// stream-K grid over all 148 SMs (slower still, 21 us).
//
// Work decomposition (packed row = one int32 word = 8 values of K, one column)
//   * CTA tile = 128 columns x a K slice of whole quantisation groups; the
//     CTAs of a column tile form a thread-block cluster along gridDim.y and
//     reduce through distributed shared memory in fixed rank order
//     (deterministic, no workspace, one launch).
//   * One producer warp: per stage of 64 packed rows it issues four 2-D TMA
//     boxes (32 columns x 64 rows, 128-byte swizzle) and one box of the
//     stage's scales, completion counted on the stage's `full` mbarrier.
//   * Eight consumer warps: warp w takes column strip w % 4 and the half w / 4
//     of every stage (32 rows = whole groups), then arrives on `empty`.
//     Lane (g = lane / 4, q = lane % 4) reads the 16-byte chunk of columns
//     [4g, 4g + 4) of rows q, q + 4, ... -- with the swizzle (chunk ^ row % 8)
//     the eight lanes of a quarter-warp hit eight different bank groups.
//
// Tensor-pipe arithmetic (mma.sync m16n8k16, fp32 accumulation)
//   * The weights are the A operand (16 "rows" = 16 columns of W), X is the B
//     operand (8 tokens).  Lane (g, q) supplies A rows g and g + 8 from two of
//     its four words (word 2t -> row g, word 2t + 1 -> row g + 8 of tile t) and
//     its own K pairs; the summation order along K is permuted accordingly and
//     X is read in the same order (lane (g, q) reads X[g, 8 (r + q) .. + 8)).
//     A 16-byte chunk therefore feeds 4 MMAs (2 tiles x 2 pair halves) and a
//     lane accumulates its own 4 columns for tokens 2q and 2q + 1.  M > 8 runs a
//     second token tile on the same A fragments.
//   * Operand decode without conversions or subtractions: fp16 magic numbers
//     0x6400 (1024, ulp 1) for codes in nibble bits 0..3 of each half and
//     0x5400 (64, ulp 1/16) for codes in bits 4..7, so one AND/OR per pair
//     gives 1024 + u or 64 + u exactly (5 instructions per word); bf16 uses
//     0x4300 (128, ulp 1) with shifts (7 per word).  The MMA computes
//     sum x * (offset + u) with exact products; the offsets are removed once
//     per (group, token) by subtracting the precomputed sum x * (offset + 8)
//     over the group, and the group scale is applied in fp32.
//   * Every mbarrier wait is bounded (1 s); on expiry the CTA records
//     kErrWaitTimeout, stops, the producer waits (bounded) for the copies it
//     issued, and the CTA leaves through the normal reduction path.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "ng_decode.cuh"
#include "sm100_primitives.cuh"

namespace cg = cooperative_groups;

namespace ngb {
namespace {

constexpr int kSStrips = 4;                 // 32-column strips per CTA tile
constexpr int kSCols = kSStrips * 32;       // columns per CTA tile
constexpr int kSStageRows = 64;             // packed rows per stage
constexpr int kSBoxBytes = kSStageRows * 128;             // one strip's box: 64 rows x 128 B
constexpr int kSStageBytes = kSStrips * kSBoxBytes;       // 32 KB
constexpr int kSMaxStages = 6;              // ring depth: 3 (96 KB) or up to 6 (192 KB)
constexpr int kSMaxCluster = 16;
constexpr int kSStageBudget = 48 * 1024;    // staged activations per CTA (bytes)

__device__ __forceinline__ void sgrid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void sgrid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
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

// Word -> four operand pairs (k0,k1) (k2,k3) (k4,k5) (k6,k7), each half equal
// to offset + u exactly (fp16: offsets 1024, 64, 1024, 64; bf16: 128).
template <bool BF16>
__device__ __forceinline__ void decode_operands(uint32_t w, uint32_t (&p)[4]) {
  if constexpr (BF16) {
    p[0] = and_or(w, 0x000F000Fu, 0x43004300u);
    p[1] = and_or(w >> 4, 0x000F000Fu, 0x43004300u);
    p[2] = and_or(w >> 8, 0x000F000Fu, 0x43004300u);
    p[3] = and_or(w >> 12, 0x000F000Fu, 0x43004300u);
  } else {
    const uint32_t w8 = w >> 8;
    p[0] = and_or(w, 0x000F000Fu, 0x64006400u);   // 1024 + u
    p[1] = and_or(w, 0x00F000F0u, 0x54005400u);   // 64 + u
    p[2] = and_or(w8, 0x000F000Fu, 0x64006400u);
    p[3] = and_or(w8, 0x00F000F0u, 0x54005400u);
  }
}

// offset + 8 for position k % 8 (what sum x * operand over-counts, per x).
template <bool BF16>
__device__ __forceinline__ float off8(int k8) {
  if constexpr (BF16) return 136.f;
  return ((k8 >> 1) & 1) ? 72.f : 1032.f;
}

template <bool BF16>
__device__ __forceinline__ float x_to_f(unsigned short b) {
  if constexpr (BF16) return __uint_as_float(static_cast<uint32_t>(b) << 16);
  return __half2float(__ushort_as_half(b));
}

// 2-D TMA box load into this CTA's shared memory, L2 evict-first.
__device__ __forceinline__ void stream_tma_hint(uint32_t dst, const CUtensorMap* map, uint64_t* bar,
                                                int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Wait for a phase regardless of the abort flag (draining issued copies), bounded.
__device__ __forceinline__ void stream_drain(uint64_t* bar, uint32_t parity, unsigned int* err) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > 1000000000ull) {
      atomicOr(err, kErrWaitTimeout);
      return;
    }
  }
}

// SPG: steps of 4 packed rows per quantisation group (G / 32).  TT: token
// tiles of 8 (1: M <= 8, 2: M <= 16).  P: stage parts (2: 32 rows per consumer
// warp, 4: 16 rows), so 4 P consumer warps + 1 producer warp.  Cluster = csize
// CTAs along gridDim.y.
template <bool BF16, int TT, int SPG, int P>
__global__ void __launch_bounds__((4 * P + 1) * 32, P == 2 ? 3 : 1)
    gemv_stream_kernel(const __grid_constant__ CUtensorMap tmap_q,
                       const __grid_constant__ CUtensorMap tmap_s,
                       const unsigned short* __restrict__ x, unsigned short* __restrict__ y, int M,
                       int K, int N, int csize, int nstages, unsigned int* __restrict__ err) {
  constexpr int kSConsumers = kSStrips * P;   // consumer warps
  constexpr int kSThreads = (kSConsumers + 1) * 32;
  constexpr int RPG = SPG * 4;                 // packed rows per group
  constexpr int NCH = 2;                       // independent MMA chains per A tile
  constexpr int PR = kSStageRows / P;          // packed rows per stage part
  static_assert(PR % RPG == 0, "a stage part holds whole groups");
  constexpr int HG = PR / RPG;                 // groups per stage part
  constexpr int SGR = kSStageRows / RPG;       // groups per stage
  constexpr int kScaleStage = SGR * kSCols * 2;  // scale bytes per stage
  constexpr int MT = 8 * TT;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled boxes.
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + kSMaxStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 128);
  unsigned char* ring = smem + 1024;
  unsigned char* sring = ring + nstages * kSStageBytes;
  unsigned char* xs = sring + nstages * kScaleStage;

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int NG = K / (RPG * 8);
  const int ck = blockIdx.y;
  const int cg0 = static_cast<int>((static_cast<long long>(ck) * NG) / csize);
  const int cg1 = static_cast<int>((static_cast<long long>(ck + 1) * NG) / csize);
  const int ngc = cg1 - cg0;
  const int nst = (ngc + SGR - 1) / SGR;
  const int tile0 = blockIdx.x * kSCols;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nstages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSConsumers);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  __syncthreads();
  sgrid_launch_dependents();

  const int xrow = ngc * RPG * 16 + 64;        // staged X row stride (bytes), 64 mod 128
  // corr rows M..MT-1 are read by lanes whose tokens do not exist; their sums are discarded
  float* corr = reinterpret_cast<float*>(xs + static_cast<size_t>(M) * xrow);  // [MT][ngc]

  float tot[TT][4][2];                         // consumer partial sums [token tile][column][parity]
#pragma unroll
  for (int t = 0; t < TT; ++t)
#pragma unroll
    for (int c = 0; c < 4; ++c) tot[t][c][0] = tot[t][c][1] = 0.f;

  if (warp == kSConsumers) {
    // ---------------- producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tmap_q);
      tma_prefetch_desc(&tmap_s);
      uint64_t pol;
      asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(pol));
      auto issue = [&](int st) {
        const int slot = st % nstages;
        mbar_arrive_expect_tx(&full[slot], kSStageBytes + kScaleStage);
        const uint32_t dst = smem_u32(ring + slot * kSStageBytes);
        const int row0 = (cg0 + st * SGR) * RPG;
#pragma unroll
        for (int sp = 0; sp < kSStrips; ++sp)
          stream_tma_hint(dst + sp * kSBoxBytes, &tmap_q, &full[slot], tile0 + 32 * sp, row0, pol);
        tma_load_2d(sring + slot * kScaleStage, &tmap_s, &full[slot], tile0, cg0 + st * SGR);
      };
      int issued = 0;
      // Weights and scales are read-only: the first stages go out before the
      // previous kernel on the stream has finished.
      for (; issued < nst && issued < nstages; ++issued) issue(issued);
      for (; issued < nst; ++issued) {
        const int slot = issued % nstages;
        if (!mbar_wait_bounded(&empty[slot], ((issued / nstages) - 1) & 1, err, abort_flag)) break;
        issue(issued);
      }
      // Every copy issued must land before the CTA's shared memory is reused.
      for (int st = issued - 1; st >= 0 && st >= issued - nstages; --st)
        stream_drain(&full[st % nstages], (st / nstages) & 1, err);
    }
  } else {
    // ---------------- consumers ----------------
    sgrid_wait();
    // Stage X[:, cg0 * G : cg1 * G) and the per-(token, group) offsets.
    {
      const int nrows = ngc * RPG;
      const int total = M * nrows;
      const int r0 = cg0 * RPG;
      for (int i0 = 0; i0 < total; i0 += kSConsumers * 32) {
        const int i = i0 + threadIdx.x;
        float part = 0.f;
        if (i < total) {
          const int m = i / nrows;
          const int r = i - m * nrows;
          const uint4 v = ld_ro_v4(x + static_cast<size_t>(m) * K + static_cast<size_t>(r0 + r) * 8);
          *reinterpret_cast<uint4*>(xs + static_cast<size_t>(m) * xrow + r * 16) = v;
          const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            part += (x_to_f<BF16>(static_cast<unsigned short>(wv[j] & 0xFFFFu)) +
                     x_to_f<BF16>(static_cast<unsigned short>(wv[j] >> 16))) * off8<BF16>(2 * j);
        }
        // RPG consecutive threads hold one (token, group); nrows % RPG == 0 and
        // RPG divides 32, so a group never straddles two warps.
#pragma unroll
        for (int o = 1; o < RPG; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (i < total && (i % RPG) == 0) {
          const int m = i / nrows;
          corr[m * ngc + (i - m * nrows) / RPG] = part;
        }
      }
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kSConsumers * 32) : "memory");  // consumers only

    const int strip = warp % kSStrips;
    const int part = warp / kSStrips;
    const int g = lane >> 2;
    const int q = lane & 3;
    const int ctok = 2 * q;                    // this lane's first token (per token tile)
    const bool have_lo = g < M;
    const bool have_hi = TT == 2 && g + 8 < M;
    const unsigned char* xlo = xs + static_cast<size_t>(g) * xrow + q * 16;
    const unsigned char* xhi = xs + static_cast<size_t>(TT == 2 ? g + 8 : g) * xrow + q * 16;

    for (int st = 0; st < nst; ++st) {
      const int slot = st % nstages;
      if (!mbar_wait_bounded(&full[slot], (st / nstages) & 1, err, abort_flag)) break;
      const unsigned char* box = ring + slot * kSStageBytes + strip * kSBoxBytes;
      const unsigned char* sbox = sring + slot * kScaleStage + (strip * 32 + 4 * g) * 2;
#pragma unroll
      for (int i = 0; i < HG; ++i) {
        const int lg = st * SGR + part * HG + i;   // group within the CTA's slice
        if (lg < ngc) {
          // [token tile][A tile][pair half]: four independent MMA chains per tile
          float acc[TT][2][NCH][4];
#pragma unroll
          for (int t = 0; t < TT; ++t)
#pragma unroll
            for (int p = 0; p < 2; ++p)
#pragma unroll
              for (int h = 0; h < NCH; ++h)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[t][p][h][e] = 0.f;
#pragma unroll
          for (int j = 0; j < SPG; ++j) {
            // Step j covers rows 8 (j / 2) + (j % 2) + 2q of the group: with the
            // 128-byte swizzle (chunk ^ row % 8) the eight lanes of a
            // quarter-warp (g = 0..1, q = 0..3) then read eight distinct chunks.
            const int gr = 8 * (j >> 1) + (j & 1) + 2 * q;     // row within the group
            const int rr = part * PR + i * RPG + gr;             // row within the stage box
            const uint4 w = *reinterpret_cast<const uint4*>(box + rr * 128 + ((g ^ (rr & 7)) << 4));
            const int xo = (lg * RPG + gr) * 16 - q * 16;        // xlo / xhi already add q * 16
            uint4 xa = make_uint4(0u, 0u, 0u, 0u), xb = make_uint4(0u, 0u, 0u, 0u);
            if (have_lo) xa = *reinterpret_cast<const uint4*>(xlo + xo);
            if (TT == 2 && have_hi) xb = *reinterpret_cast<const uint4*>(xhi + xo);
            const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int p = 0; p < 2; ++p) {        // A tile p: words 2p (row g), 2p + 1 (row g + 8)
              uint32_t lo[4], hi[4];
              decode_operands<BF16>(words[2 * p], lo);
              decode_operands<BF16>(words[2 * p + 1], hi);
              mma16816<BF16>(acc[0][p][0], lo[0], hi[0], lo[1], hi[1], xa.x, xa.y);
              mma16816<BF16>(acc[0][p][NCH - 1], lo[2], hi[2], lo[3], hi[3], xa.z, xa.w);
              if constexpr (TT == 2) {
                mma16816<BF16>(acc[TT - 1][p][0], lo[0], hi[0], lo[1], hi[1], xb.x, xb.y);
                mma16816<BF16>(acc[TT - 1][p][NCH - 1], lo[2], hi[2], lo[3], hi[3], xb.z, xb.w);
              }
            }
          }
          // tot += scale * (acc - sum x * (offset + 8)) per (column, token).
          const uint2 sv = *reinterpret_cast<const uint2*>(sbox + (part * HG + i) * kSCols * 2);
          const float2 s01 = __half22float2(h2_from_bits(sv.x));
          const float2 s23 = __half22float2(h2_from_bits(sv.y));
          const float sc[4] = {s01.x, s01.y, s23.x, s23.y};
#pragma unroll
          for (int t = 0; t < TT; ++t) {
            const float c0 = corr[(8 * t + ctok) * ngc + lg];
            const float c1 = corr[(8 * t + ctok + 1) * ngc + lg];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
              float a[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) a[e] = NCH == 2 ? acc[t][p][0][e] + acc[t][p][NCH - 1][e] : acc[t][p][0][e];
              tot[t][2 * p][0] = fmaf(sc[2 * p], a[0] - c0, tot[t][2 * p][0]);
              tot[t][2 * p][1] = fmaf(sc[2 * p], a[1] - c1, tot[t][2 * p][1]);
              tot[t][2 * p + 1][0] = fmaf(sc[2 * p + 1], a[2] - c0, tot[t][2 * p + 1][0]);
              tot[t][2 * p + 1][1] = fmaf(sc[2 * p + 1], a[3] - c1, tot[t][2 * p + 1][1]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
  }
  // Every issued copy has landed (producer drain) and every consumer is done
  // with the ring: reuse it for the partial sums, red[part][token][column].
  __syncthreads();
  float* red = reinterpret_cast<float*>(ring);
  if (warp < kSConsumers) {
    const int strip = warp % kSStrips;
    const int part = warp / kSStrips;
    const int g = lane >> 2;
    const int ctok = 2 * (lane & 3);
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int m = 8 * t + ctok + e;
        float* dst = red + (static_cast<size_t>(part) * MT + m) * kSCols + strip * 32 + 4 * g;
        *reinterpret_cast<float4*>(dst) =
            make_float4(tot[t][0][e], tot[t][1][e], tot[t][2][e], tot[t][3][e]);
      }
  }
  __syncthreads();

  // ---- reduction: the stage parts, then the cluster's K slices ---------------
  float* fin = red + P * MT * kSCols;                        // [MT][kSCols]
  const int E = M * kSCols;
  for (int e = threadIdx.x; e < E; e += kSThreads) {
    float v = 0.f;
#pragma unroll
    for (int p = 0; p < P; ++p) v += red[p * MT * kSCols + e];  // fixed order
    fin[e] = v;
  }
  auto store = [&](int e, float v) {
    const int m = e / kSCols;
    const int cn = tile0 + (e % kSCols);
    if (cn < N)
      y[static_cast<size_t>(m) * N + cn] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                : __half_as_ushort(__float2half_rn(v));
  };
  if (csize == 1) {
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kSThreads) store(e, fin[e]);
    return;
  }
  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const int rank = static_cast<int>(cluster.block_rank());
  const int per = (E + csize - 1) / csize;
  const int e0 = rank * per;
  const int e1 = min(E, e0 + per);
  for (int e = e0 + static_cast<int>(threadIdx.x); e < e1; e += kSThreads) {
    float v = 0.f;
    for (int r = 0; r < csize; ++r) v += cluster.map_shared_rank(fin, r)[e];
    store(e, v);
  }
  cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Cluster size (K slices per column tile).  Default: the largest power of two
// (<= 16) with tiles * C <= SMs, raised until a CTA's activation slice fits the
// staging budget; `splits` > 0 requests C.
int stream_cluster(int M, int K, int N, int G, int splits, const DeviceInfo& dev) {
  const int NG = K / G;
  const int tiles = (N + kSCols - 1) / kSCols;
  int C = splits;
  if (C <= 0) {
    C = 1;
    while (C * 2 <= kSMaxCluster && tiles * C * 2 <= dev.sm_count) C *= 2;
  }
  const long long per_group = static_cast<long long>(M) * G * 2;
  const int max_groups = static_cast<int>(std::max(1LL, kSStageBudget / per_group));
  C = std::max(C, (NG + max_groups - 1) / max_groups);
  return std::max(1, std::min(C, std::min(NG, kSMaxCluster)));
}

size_t stream_smem_bytes(int M, int NG, int C, int G, int nstages) {
  const int RPG = G / 8;
  const int MT = M > 8 ? 16 : 8;
  const int gmax = (NG + C - 1) / C;
  const size_t scale_stage = static_cast<size_t>(2 * (32 / RPG)) * kSCols * 2;
  return 2048 + static_cast<size_t>(nstages) * (kSStageBytes + scale_stage) +
         static_cast<size_t>(M) * (gmax * RPG * 16 + 64) + static_cast<size_t>(MT) * gmax * 4;
}

template <bool BF16, int TT, int SPG, int P>
int run_stream(const void* x, const uint32_t* q, const __half* s, void* y, int M, int K, int N,
               int C, const DeviceInfo& dev, cudaStream_t stream) {
  auto kern = gemv_stream_kernel<BF16, TT, SPG, P>;
  constexpr int RPG = SPG * 4;
  constexpr int G = RPG * 8;
  const int NG = K / G;
  const int tiles = (N + kSCols - 1) / kSCols;
  static std::once_flag once[kMaxDevices];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  });
  int nstages = 3;  // measured: deeper rings (4-6 stages) are not faster
  while (nstages > 2 && stream_smem_bytes(M, NG, C, G, nstages) > 200 * 1024) --nstages;
  const size_t smem = stream_smem_bytes(M, NG, C, G, nstages);
  if (smem > 200 * 1024) return NG_ERR_BAD_SHAPE;

  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
  if (!enc) return NG_ERR_CUDA;
  CUtensorMap tq, ts;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K / 8)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 4};
    const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(kSStageRows)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(NG)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kSCols), static_cast<cuuint32_t>(2 * (32 / RPG))};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&ts, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<__half*>(s), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, C, 1);
  cfg.blockDim = dim3((4 * P + 1) * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
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
  return launch_status(cudaLaunchKernelEx(&cfg, kern, tq, ts, static_cast<const unsigned short*>(x),
                                          static_cast<unsigned short*>(y), M, K, N, C, nstages, dev.err));
}

template <bool BF16, int TT>
int stream_g(const void* x, const uint32_t* q, const __half* s, void* y, int M, int K, int N, int G,
             int C, const DeviceInfo& dev, cudaStream_t st) {
  // 16 consumer warps when the grid leaves each SM to one CTA, 8 when two CTAs
  // must share an SM (or a group is 32 rows, G = 256).
  const int tiles = (N + kSCols - 1) / kSCols;
  int P = (tiles * C <= dev.sm_count && G <= 128) ? 4 : 2;
  if (G == 64)
    return P == 4 ? run_stream<BF16, TT, 2, 4>(x, q, s, y, M, K, N, C, dev, st)
                  : run_stream<BF16, TT, 2, 2>(x, q, s, y, M, K, N, C, dev, st);
  if (G == 128)
    return P == 4 ? run_stream<BF16, TT, 4, 4>(x, q, s, y, M, K, N, C, dev, st)
                  : run_stream<BF16, TT, 4, 2>(x, q, s, y, M, K, N, C, dev, st);
  return run_stream<BF16, TT, 8, 2>(x, q, s, y, M, K, N, C, dev, st);
}

}  // namespace

bool gemv_stream_supported(int N, const void* scales) {
  // TMA boxes of the scales need a 16-byte row stride and base.
  return N % 8 == 0 && aligned(scales, 16);
}

int gemv_stream(const void* x, int x_dtype, const uint32_t* q, const __half* s, void* y, int M,
                int K, int N, int G, int splits, const DeviceInfo& dev, cudaStream_t strm) {
  if (!gemv_stream_supported(N, s)) return NG_ERR_BAD_SHAPE;
  const bool bf = x_dtype == NG_DTYPE_BF16;
  const int C = stream_cluster(M, K, N, G, splits, dev);
  if (M > 8)
    return bf ? stream_g<true, 2>(x, q, s, y, M, K, N, G, C, dev, strm)
              : stream_g<false, 2>(x, q, s, y, M, K, N, G, C, dev, strm);
  return bf ? stream_g<true, 1>(x, q, s, y, M, K, N, G, C, dev, strm)
            : stream_g<false, 1>(x, q, s, y, M, K, N, G, C, dev, strm);
}

}  // namespace ngb
