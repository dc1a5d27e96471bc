// Decode-regime GEMV on the tensor pipe: Y[M, N] = X[M, K] @ W, M <= 16.
//
// Why tensor cores for a bandwidth-bound GEMV: at B200's ~7 TB/s the SMs must
// retire ~45 weights per cycle each, and the CUDA-core path spends ~1.7
// instructions per weight (decode + packed FMA + flush).  Here each packed word
// is decoded with 3 shifts + 4 AND/OR and fed straight to mma.sync as fp16
// (or bf16) values 1024 + u (128 + u), the magic-number representation, with
// no subtract: the zero point and the magic offset are removed once per
// quantisation group, from a correction column the same MMA computes
// (a constant-weight row gives magic * sum_k x).  ~1.1 instructions per weight,
// and M = 2..16 costs almost nothing extra.
//
// Fragment mapping (m16n8k16, A row-major 16x16, B 16x8, fp32 C):
//   lane = 4g + t.  The reduction order inside an MMA is free, so the "virtual"
//   k of the MMA is mapped to real k such that each thread's fragment is
//   exactly what one packed word decodes to:
//   * thread (g, t) loads, for packed row j0 + t, the 16-byte runs of columns
//     c0 + 4g .. +3 and c0 + 32 + 4g .. +3;  A row g <-> column c0 + 4g + i and
//     A row g + 8 <-> column c0 + 32 + 4g + i for the i-th word of each run;
//   * virtual k pairs t and t + 4 of MMA #1 are real pairs 0 and 1 of packed
//     row j0 + t, those of MMA #2 real pairs 2 and 3;
//   * so the B fragment of thread (g, t) is X[m = g][8 (j0 + t) .. + 7]: one
//     16-byte load.
//   One step = 4 packed rows (32 values of K) x 64 columns per warp:
//   2 x 16-byte weight loads, 1 x 16-byte activation load (per 8 rows of X),
//   8 word decodes, 8 + 2 MMAs per 8-row tile of X.
//
// Schedule: persistent and balanced.  Work units are (64-column tile,
// quantisation group); the unit list (tile-major) is split into equal
// contiguous ranges, one per CTA (all CTAs resident at once), and a CTA's
// range into equal contiguous ranges per warp.  A warp prefetches the next
// unit's weights before decoding the current one.  Warp partials are reduced
// per tile in shared memory in warp order; a tile split between CTAs is
// finished by the last CTA to arrive (per-tile counter in the workspace),
// which sums the CTAs' partials in CTA order -- deterministic -- and resets
// the counter.  Launched with programmatic stream serialisation: the first
// unit's weights are requested before griddepcontrol.wait.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "ng_decode.cuh"
#include "sm100_primitives.cuh"

namespace ngb {
namespace {

constexpr int kTN = 64;       // columns per tile
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxTiles = 4;  // distinct tiles one CTA range may touch
constexpr int kMaxM = 16;

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

// Magic-number operand for the MMA: each 16-bit lane of the result is
// magic + u (exact) for the code pair (k = 2j, 2j + 1) of the word.
// fp16 magic 1024 (0x6400), bf16 magic 128 (0x4300): both have an ulp of 1.
template <bool BF16>
__device__ __forceinline__ void decode_raw(uint32_t q, uint32_t (&h)[4]) {
  constexpr uint32_t kMagic = BF16 ? 0x43004300u : 0x64006400u;
  h[0] = and_or(q, 0x000F000Fu, kMagic);        // slots 0,4 -> k 0,1
  h[1] = and_or(q >> 4, 0x000F000Fu, kMagic);   // slots 1,5 -> k 2,3
  h[2] = and_or(q >> 8, 0x000F000Fu, kMagic);   // slots 2,6 -> k 4,5
  h[3] = and_or(q >> 12, 0x000F000Fu, kMagic);  // slots 3,7 -> k 6,7
}

// Balanced split of `units` work units over P CTAs: the first r CTAs get
// q + 1 units, the rest q (q, r precomputed on the host) -- 32-bit math only.
struct Part {
  int q, r;
  __device__ __forceinline__ int start(int b) const { return b * q + min(b, r); }
  __device__ __forceinline__ int owner(int u) const {
    const int big = r * (q + 1);
    return u < big ? u / (q + 1) : r + (u - big) / q;
  }
};

template <int NT, int GS, bool XBF16>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 2 : 1)
    gemv_tc_kernel(const unsigned short* __restrict__ x, const uint32_t* __restrict__ qw,
                   const __half* __restrict__ scales, unsigned short* __restrict__ y, int M, int K,
                   int N, int G, int part_q, int part_r, int gpt, float* __restrict__ partials,
                   unsigned int* __restrict__ counters) {
  constexpr int MR = NT * 8;              // rows of X covered
  constexpr int kSlot = MR * kTN;         // floats per (tile, warp) slot
  // (magic + 8) / magic: removes the magic offset and the zero point at once.
  constexpr float kCorr = XBF16 ? (136.0f / 128.0f) : (1032.0f / 1024.0f);
  extern __shared__ __align__(16) float red[];  // [kMaxTiles][kWarps][MR][kTN]
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const Part part{part_q, part_r};
  const int b = blockIdx.x;
  const int u0 = part.start(b), u1 = part.start(b + 1);
  const int n_my = u1 - u0;
  const int wu0 = u0 + (n_my * warp) / kWarps, wu1 = u0 + (n_my * (warp + 1)) / kWarps;
  const int tile_first = u0 / gpt;
  constexpr int UK = GS * 32;  // values of K per unit (64 or 128; a G = 256 group is two units)

  griddep_launch_dependents();

  // ---- weight ring: one slot per step of a unit (GS x 2 x 16 B per lane).  Slot
  // st of the next unit is refilled as soon as step st of the current one is
  // decoded, so GS steps stay in flight per warp at all times.
  const uint64_t pol = make_evict_first_policy();
  uint4 wa[GS], wb[GS];
  uint2 sa[2], sb[2];
  const size_t rows4 = static_cast<size_t>(4) * N;  // 4 packed rows
  // Addressing of one unit for this lane (all 32-bit index math but one
  // 64-bit offset per unit; no divisions inside the loop).
  struct Ptrs {
    const uint32_t* a;
    const uint32_t* b;
    const __half* sa;
    const __half* sb;
    bool oka, okb;
  };
  auto unit_ptrs = [&](int tile, int sub) {
    Ptrs p;
    const int ca = tile * kTN + 4 * g, cb = ca + 32;
    p.oka = ca < N;
    p.okb = cb < N;
    p.a = qw + static_cast<size_t>(sub * (UK / 8) + t) * N + ca;
    p.b = p.a + 32;
    const size_t grp = static_cast<size_t>((sub * UK) / G);
    p.sa = scales + grp * N + ca;
    p.sb = p.sa + 32;
    return p;
  };
  auto load_step = [&](const Ptrs& p, int st) {
    const uint4 pad = make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
    wa[st] = p.oka ? ld_stream_v4(p.a + st * rows4, pol) : pad;
    wb[st] = p.okb ? ld_stream_v4(p.b + st * rows4, pol) : pad;
  };
  auto load_scales = [&](const Ptrs& p, auto bufc) {
    constexpr int B = decltype(bufc)::value;
    sa[B] = p.oka ? ld_ro_v2(p.sa) : make_uint2(0u, 0u);
    sb[B] = p.okb ? ld_ro_v2(p.sb) : make_uint2(0u, 0u);
  };

  // zero the per-tile warp slots (this warp's own slots only)
  for (int i = lane; i < kMaxTiles * kSlot; i += 32)
    red[(i / kSlot) * kWarps * kSlot + warp * kSlot + (i % kSlot)] = 0.f;

  float tot[4][NT][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) tot[i][nt][r] = 0.f;

  auto deposit = [&](int tile) {
    float* slot = red + ((tile - tile_first) * kWarps + warp) * kSlot;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int m = nt * 8 + 2 * t + (r & 1);
          const int c = (r < 2 ? 4 * g : 32 + 4 * g) + i;
          slot[m * kTN + c] = tot[i][nt][r];
          tot[i][nt][r] = 0.f;
        }
  };

  int cur_tile = -1;
  constexpr uint32_t kMagic2 = XBF16 ? 0x43004300u : 0x64006400u;
  // Decode + MMA of one unit from the ring; refills each ring slot with the
  // next unit's step as soon as it is consumed.
  auto process = [&](int tile, int sub, bool has_next, const Ptrs& nxt, auto bufc) {
    constexpr int B = decltype(bufc)::value;
    if (tile != cur_tile) {
      if (cur_tile >= 0) deposit(cur_tile);
      cur_tile = tile;
    }
    float c[4][NT][4], cv[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        cv[nt][r] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i][nt][r] = 0.f;
      }
    const unsigned short* xrow = x + static_cast<size_t>(g) * K + sub * UK + 8 * t;
#pragma unroll
    for (int st = 0; st < GS; ++st) {
      // activations: rows m = nt*8 + g, k = sub*UK + st*32 + 8t .. +7
      uint4 xv[NT];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        xv[nt] = nt * 8 + g < M ? ld_ro_v4(xrow + static_cast<size_t>(nt * 8) * K + st * 32)
                                : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t wA[4] = {wa[st].x, wa[st].y, wa[st].z, wa[st].w};
      const uint32_t wB[4] = {wb[st].x, wb[st].y, wb[st].z, wb[st].w};
      if (has_next) load_step(nxt, st);  // slot st is free again
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t ha[4], hb[4];
        decode_raw<XBF16>(wA[i], ha);
        decode_raw<XBF16>(wB[i], hb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816<XBF16>(c[i][nt], ha[0], hb[0], ha[1], hb[1], xv[nt].x, xv[nt].y);
          mma16816<XBF16>(c[i][nt], ha[2], hb[2], ha[3], hb[3], xv[nt].z, xv[nt].w);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma16816<XBF16>(cv[nt], kMagic2, kMagic2, kMagic2, kMagic2, xv[nt].x, xv[nt].y);
        mma16816<XBF16>(cv[nt], kMagic2, kMagic2, kMagic2, kMagic2, xv[nt].z, xv[nt].w);
      }
    }
    // unit flush: tot += s * (c - corr * cv)
    const __half2 ha01 = h2_from_bits(sa[B].x), ha23 = h2_from_bits(sa[B].y);
    const __half2 hb01 = h2_from_bits(sb[B].x), hb23 = h2_from_bits(sb[B].y);
    const float2 fa01 = __half22float2(ha01), fa23 = __half22float2(ha23);
    const float2 fb01 = __half22float2(hb01), fb23 = __half22float2(hb23);
    const float fa[4] = {fa01.x, fa01.y, fa23.x, fa23.y};
    const float fb[4] = {fb01.x, fb01.y, fb23.x, fb23.y};
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      float corr[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) corr[r] = kCorr * cv[nt][r];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          tot[i][nt][r] = fmaf(r < 2 ? fa[i] : fb[i], c[i][nt][r] - corr[r], tot[i][nt][r]);
    }
  };

  using B0 = std::integral_constant<int, 0>;
  using B1 = std::integral_constant<int, 1>;
  const int nunits_w = wu1 - wu0;
  int tile = wu0 / gpt, sub = wu0 - (wu0 / gpt) * gpt;
  auto advance = [&](int& tl, int& sb_) {
    if (++sb_ == gpt) { sb_ = 0; ++tl; }
  };
  Ptrs cur = unit_ptrs(tile, sub);
  if (nunits_w > 0) {
#pragma unroll
    for (int st = 0; st < GS; ++st) load_step(cur, st);
    load_scales(cur, B0{});
  }
  griddep_wait();  // x, y and the workspace belong to the previous kernel until here
  for (int k = 0; k < nunits_w; k += 2) {
    int t1 = tile, s1 = sub;
    advance(t1, s1);
    const bool has1 = k + 1 < nunits_w;
    const Ptrs p1 = unit_ptrs(t1, s1);
    if (has1) load_scales(p1, B1{});
    process(tile, sub, has1, p1, B0{});
    if (!has1) break;
    int t2 = t1, s2 = s1;
    advance(t2, s2);
    const bool has2 = k + 2 < nunits_w;
    const Ptrs p2 = unit_ptrs(t2, s2);
    if (has2) load_scales(p2, B0{});
    process(t1, s1, has2, p2, B1{});
    tile = t2;
    sub = s2;
  }
  if (cur_tile >= 0) deposit(cur_tile);
  __syncthreads();

  // ---- per-tile reduction over warps (warp order), emit or hand off -----------
  const int tile_last = n_my > 0 ? (u1 - 1) / gpt : tile_first - 1;
  for (int tile = tile_first; tile <= tile_last; ++tile) {
    const int tu0 = tile * gpt, tu1 = tu0 + gpt;
    const bool whole = tu0 >= u0 && tu1 <= u1;
    const float* base = red + (tile - tile_first) * kWarps * kSlot;
    const int slot = 2 * b + (tile == tile_first ? 0 : 1);
    for (int e = threadIdx.x; e < kSlot; e += kThreads) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) v += base[w * kSlot + e];
      const int m = e / kTN, n = tile * kTN + (e % kTN);
      if (whole) {
        if (m < M && n < N)
          y[static_cast<size_t>(m) * N + n] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                    : __half_as_ushort(__float2half_rn(v));
      } else {
        partials[static_cast<size_t>(slot) * (kMaxM * kTN) + e] = v;
      }
    }
    if (whole) continue;
    __threadfence();
    __syncthreads();
    const int bf = part.owner(tu0), bl = part.owner(tu1 - 1);
    if (threadIdx.x == 0) {
      const unsigned int prev = atomicAdd(&counters[tile], 1u);
      s_last = (prev == static_cast<unsigned int>(bl - bf));
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      for (int e = threadIdx.x; e < kSlot; e += kThreads) {
        float v = 0.f;
        for (int bb = bf; bb <= bl; ++bb) {
          // contributor bb wrote this tile to its first slot iff the tile is
          // the first one of its range
          const int sl = 2 * bb + (part.start(bb) >= tu0 ? 0 : 1);
          v += __ldcg(&partials[static_cast<size_t>(sl) * (kMaxM * kTN) + e]);
        }
        const int m = e / kTN, n = tile * kTN + (e % kTN);
        if (m < M && n < N)
          y[static_cast<size_t>(m) * N + n] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                    : __half_as_ushort(__float2half_rn(v));
      }
      if (threadIdx.x == 0) counters[tile] = 0u;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Workspace: partial-sum slots (2 per CTA, up to 4 CTAs per SM, 16 x 64 floats
// each) followed by one arrival counter per 64-column tile.  The layout does
// not depend on M; only the counters must be zero between calls and every
// call leaves them zero.
size_t tc_counter_offset(int sm_count) {
  return static_cast<size_t>(2) * 4 * sm_count * kMaxM * kTN * sizeof(float);
}

template <int NT, int GS, bool XBF16>
int run_tc(const void* x, const uint32_t* q, const __half* s, void* y, int M, int K, int N, int G,
           void* ws, const DeviceInfo& dev, cudaStream_t stream) {
  auto kern = gemv_tc_kernel<NT, GS, XBF16>;
  constexpr size_t smem = static_cast<size_t>(kMaxTiles) * kWarps * NT * 8 * kTN * sizeof(float);
  static std::once_flag once[64];
  static int resident[64];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem) != cudaSuccess) occ = 1;
    resident[dev.device] = std::max(1, std::min(occ, 4));
  });
  const int tiles = (N + kTN - 1) / kTN;
  const int gpt = K / (GS * 32);  // units per tile
  const long long units = static_cast<long long>(tiles) * gpt;
  if (units >= (1LL << 30)) return NG_ERR_BAD_SHAPE;
  // All CTAs resident; enough CTAs that a range touches at most kMaxTiles tiles.
  long long P = static_cast<long long>(dev.sm_count) * resident[dev.device];
  P = std::max<long long>(P, (tiles + kMaxTiles - 3) / (kMaxTiles - 2));
  P = std::min<long long>(P, units);
  if (P > 4LL * dev.sm_count) return NG_ERR_BAD_SHAPE;
  auto* partials = static_cast<float*>(ws);
  auto* counters = reinterpret_cast<unsigned int*>(static_cast<unsigned char*>(ws) +
                                                   tc_counter_offset(dev.sm_count));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(P), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int pq = static_cast<int>(units / P), pr = static_cast<int>(units % P);
  return launch_status(cudaLaunchKernelEx(&cfg, kern, static_cast<const unsigned short*>(x), q, s,
                                          static_cast<unsigned short*>(y), M, K, N, G, pq, pr, gpt,
                                          partials, counters));
}

}  // namespace

size_t gemv_tc_workspace_bytes(int N, const DeviceInfo& dev) {
  return tc_counter_offset(dev.sm_count) + static_cast<size_t>((N + kTN - 1) / kTN) * 4;
}

int gemv_tc(const void* x, int x_dtype, const uint32_t* q, const __half* s, void* y, int M, int K,
            int N, int G, void* ws, const DeviceInfo& dev, cudaStream_t strm) {
  const bool bf = x_dtype == NG_DTYPE_BF16;
#define NG_TC(NT, GS)                                                    \
  return bf ? run_tc<NT, GS, true>(x, q, s, y, M, K, N, G, ws, dev, strm) \
            : run_tc<NT, GS, false>(x, q, s, y, M, K, N, G, ws, dev, strm)
  if (G == 64) {
    if (M <= 8) NG_TC(1, 2);
    NG_TC(2, 2);
  }
  if (M <= 8) NG_TC(1, 4);
  NG_TC(2, 4);
#undef NG_TC
}

}  // namespace ngb
