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

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kRing = 2;  // units of weights in flight per warp (shared-memory ring)
constexpr int kWarpSlots = 3;  // distinct tiles one warp's range may touch

template <int NT, int GS>
struct TcSmem {
  static constexpr int kSlot = NT * 8 * kTN;                       // floats per warp-tile partial
  static constexpr int kRingBytes = kWarps * kRing * GS * 2 * 32 * 16;
  static constexpr int kRedBytes = kWarps * kWarpSlots * kSlot * 4;
  static constexpr int kBytes = kRingBytes + kRedBytes;
};

template <int NT, int GS, bool XBF16>
__global__ void __launch_bounds__(kThreads, NT == 1 ? 2 : 1)
    gemv_tc_kernel(const unsigned short* __restrict__ x, const uint32_t* __restrict__ qw,
                   const __half* __restrict__ scales, unsigned short* __restrict__ y, int M, int K,
                   int N, int G, int part_q, int part_r, int gpt, float* __restrict__ partials,
                   unsigned int* __restrict__ counters, unsigned int* __restrict__ err) {
  using L = TcSmem<NT, GS>;
  constexpr int kSlot = L::kSlot;
  constexpr int UK = GS * 32;  // values of K per unit (64 or 128; a G = 256 group is two units)
  // (magic + 8) / magic: removes the magic offset and the zero point at once.
  constexpr float kCorr = XBF16 ? (136.0f / 128.0f) : (1032.0f / 1024.0f);
  constexpr uint32_t kMagic2 = XBF16 ? 0x43004300u : 0x64006400u;
  extern __shared__ __align__(16) unsigned char smem[];
  uint4* ring = reinterpret_cast<uint4*>(smem);                       // [warp][kRing][GS*2][32]
  float* red = reinterpret_cast<float*>(smem + L::kRingBytes);         // [warp][kWarpSlots][kSlot]
  __shared__ int s_arrive[kMaxTiles];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const Part part{part_q, part_r};
  const int b = blockIdx.x;
  const int u0 = part.start(b), u1 = part.start(b + 1);
  const int n_my = u1 - u0;
  auto wstart = [&](int w) { return u0 + (n_my * w) / kWarps; };
  const int wu0 = wstart(warp), wu1 = wstart(warp + 1);
  const int tile_first = u0 / gpt;
  const int my_first_tile = wu0 / gpt;
  if (threadIdx.x < kMaxTiles) s_arrive[threadIdx.x] = 0;

  griddep_launch_dependents();

  // ---- addressing of one unit for this lane -------------------------------------
  const size_t rows4 = static_cast<size_t>(4) * N;  // 4 packed rows
  auto issue_unit = [&](int tile, int sub, int d) {
    const int ca = tile * kTN + 4 * g, cb = ca + 32;
    const uint32_t* pa = qw + static_cast<size_t>(sub * (UK / 8) + t) * N + ca;
    uint4* dst = ring + ((warp * kRing + d) * (GS * 2)) * 32 + lane;
#pragma unroll
    for (int st = 0; st < GS; ++st) {
      cp_async_16(dst + (2 * st) * 32, ca < N ? pa + st * rows4 : qw, ca < N);
      cp_async_16(dst + (2 * st + 1) * 32, cb < N ? pa + 32 + st * rows4 : qw, cb < N);
    }
  };
  auto load_scales = [&](int tile, int sub, uint2& sa, uint2& sb) {
    const int ca = tile * kTN + 4 * g, cb = ca + 32;
    const size_t grp = static_cast<size_t>((sub * UK) / G);
    sa = ca < N ? ld_ro_v2(scales + grp * N + ca) : make_uint2(0u, 0u);
    sb = cb < N ? ld_ro_v2(scales + grp * N + cb) : make_uint2(0u, 0u);
  };
  auto load_x = [&](int sub, uint4 (&xv)[GS][NT]) {
    const unsigned short* xrow = x + static_cast<size_t>(g) * K + sub * UK + 8 * t;
#pragma unroll
    for (int st = 0; st < GS; ++st)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
        xv[st][nt] = nt * 8 + g < M ? ld_ro_v4(xrow + static_cast<size_t>(nt * 8) * K + st * 32)
                                    : make_uint4(0u, 0u, 0u, 0u);
  };

  // Number of warps of this CTA whose range touches `tile` (contiguous split).
  auto warps_on_tile = [&](int tile) {
    int n = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const int a0 = wstart(w), a1 = wstart(w + 1);
      n += (a0 < a1 && a0 < (tile + 1) * gpt && a1 > tile * gpt) ? 1 : 0;
    }
    return n;
  };

  // The last warp of this CTA to finish its part of `tile` reduces the warps'
  // partials (in warp order) and then: writes Y (tile entirely in this CTA's
  // range), publishes a partial (the tile began in an earlier CTA's range:
  // that CTA finishes it), or waits for the later CTAs' partials and finishes
  // the tile (it owns the tile's first unit) -- deterministic in every case.
  auto finish_tile = [&](int tile) {
    const int tu0 = tile * gpt, tu1 = tu0 + gpt;
    const bool starts_here = tu0 >= u0;
    const bool ends_here = tu1 <= u1;
    const int bl = ends_here ? b : part.owner(tu1 - 1);
    if (starts_here && bl > b) {
      // finisher: wait (bounded) until every later contributor has published
      if (lane == 0) {
        const unsigned int need = static_cast<unsigned int>(bl - b);
        const uint64_t t0 = global_timer_ns();
        unsigned int v;
        for (;;) {
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(counters + tile) : "memory");
          if (v >= need) break;
          if (global_timer_ns() - t0 > 1000000000ull) {
            atomicOr(err, kErrWaitTimeout);
            break;
          }
        }
      }
      __syncwarp();
      __threadfence();
    }
    for (int e = lane; e < kSlot; e += 32) {
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const int a0 = wstart(w), a1 = wstart(w + 1);
        if (a0 < a1 && a0 < tu1 && a1 > tu0)
          v += red[(w * kWarpSlots + (tile - a0 / gpt)) * kSlot + e];
      }
      if (!starts_here) {
        partials[static_cast<size_t>(b) * (kMaxM * kTN) + e] = v;
        continue;
      }
      for (int bb = b + 1; bb <= bl; ++bb)
        v += __ldcg(&partials[static_cast<size_t>(bb) * (kMaxM * kTN) + e]);
      const int m = e / kTN, n = tile * kTN + (e % kTN);
      if (m < M && n < N)
        y[static_cast<size_t>(m) * N + n] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                  : __half_as_ushort(__float2half_rn(v));
    }
    if (!starts_here) {
      __threadfence();
      __syncwarp();
      if (lane == 0)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(counters + tile) : "memory");
    } else if (bl > b) {
      __syncwarp();
      if (lane == 0) counters[tile] = 0u;  // every contributor has arrived: reset for the next call
    }
  };

  float tot[4][NT][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) tot[i][nt][r] = 0.f;

  auto deposit = [&](int tile) {
    float* slot = red + (warp * kWarpSlots + (tile - my_first_tile)) * kSlot;
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
    __threadfence_block();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&s_arrive[tile - tile_first], 1) == warps_on_tile(tile) - 1;
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
      __threadfence_block();
      finish_tile(tile);
    }
  };

  // ---- main loop ---------------------------------------------------------------
  const int nw = wu1 - wu0;
  int tile = wu0 / gpt, sub = wu0 - (wu0 / gpt) * gpt;
  // weights for the first kRing units go out before the dependency wait
  {
    int tl = tile, sb = sub;
#pragma unroll
    for (int d = 0; d < kRing; ++d) {
      if (d < nw) issue_unit(tl, sb, d);
      cp_async_commit();
      if (++sb == gpt) { sb = 0; ++tl; }
    }
  }
  __syncthreads();  // s_arrive initialised
  griddep_wait();   // x, y and the workspace belong to the previous kernel until here

  uint4 xv[2][GS][NT];
  uint2 sa[2], sb2[2];
  if (nw > 0) {
    load_x(sub, xv[0]);
    load_scales(tile, sub, sa[0], sb2[0]);
  }
  int cur_tile = -1;
  auto process = [&](int k, auto bufc) {
    constexpr int B = decltype(bufc)::value;
    if (tile != cur_tile) {
      if (cur_tile >= 0) deposit(cur_tile);
      cur_tile = tile;
    }
    int nt_tile = tile, nt_sub = sub;
    if (++nt_sub == gpt) { nt_sub = 0; ++nt_tile; }
    if (k + 1 < nw) {  // next unit's activations and scales into the other register buffer
      load_x(nt_sub, xv[B ^ 1]);
      load_scales(nt_tile, nt_sub, sa[B ^ 1], sb2[B ^ 1]);
    }
    cp_async_wait<kRing - 1>();  // this unit's weights have landed (this lane's own copies)
    const uint4* src = ring + ((warp * kRing + (k % kRing)) * (GS * 2)) * 32 + lane;
    float c[4][NT][4], cv[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        cv[nt][r] = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) c[i][nt][r] = 0.f;
      }
    uint32_t consumed = 0;  // ties the ring refill below to the completion of these reads
#pragma unroll
    for (int st = 0; st < GS; ++st) {
      const uint4 qa = src[(2 * st) * 32], qb = src[(2 * st + 1) * 32];
      consumed ^= qa.x ^ qb.x;
      const uint32_t wA[4] = {qa.x, qa.y, qa.z, qa.w};
      const uint32_t wB[4] = {qb.x, qb.y, qb.z, qb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t ha[4], hb[4];
        decode_raw<XBF16>(wA[i], ha);
        decode_raw<XBF16>(wB[i], hb);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma16816<XBF16>(c[i][nt], ha[0], hb[0], ha[1], hb[1], xv[B][st][nt].x, xv[B][st][nt].y);
          mma16816<XBF16>(c[i][nt], ha[2], hb[2], ha[3], hb[3], xv[B][st][nt].z, xv[B][st][nt].w);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        mma16816<XBF16>(cv[nt], kMagic2, kMagic2, kMagic2, kMagic2, xv[B][st][nt].x, xv[B][st][nt].y);
        mma16816<XBF16>(cv[nt], kMagic2, kMagic2, kMagic2, kMagic2, xv[B][st][nt].z, xv[B][st][nt].w);
      }
    }
    // ring slot consumed: refill it with the unit kRing ahead.  The empty asm
    // takes the values read from the slot as inputs, so the copies that
    // overwrite it are issued only after those reads have returned.
    asm volatile("" ::"r"(consumed) : "memory");
    {
      int tl = tile, sb = sub;
#pragma unroll
      for (int d = 0; d < kRing; ++d)
        if (++sb == gpt) { sb = 0; ++tl; }
      if (k + kRing < nw) issue_unit(tl, sb, k % kRing);
      cp_async_commit();
    }
    // unit flush: tot += s * (c - corr * cv)
    const float2 fa01 = __half22float2(h2_from_bits(sa[B].x)), fa23 = __half22float2(h2_from_bits(sa[B].y));
    const float2 fb01 = __half22float2(h2_from_bits(sb2[B].x)), fb23 = __half22float2(h2_from_bits(sb2[B].y));
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
    tile = nt_tile;
    sub = nt_sub;
  };
  using B0 = std::integral_constant<int, 0>;
  using B1 = std::integral_constant<int, 1>;
  for (int k = 0; k < nw; k += 2) {
    process(k, B0{});
    if (k + 1 >= nw) break;
    process(k + 1, B1{});
  }
  if (cur_tile >= 0) deposit(cur_tile);
  cp_async_wait<0>();
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
// Workspace: one partial-sum slot per CTA (up to 4 CTAs per SM, 16 x 64
// floats each) followed by one arrival counter per 64-column tile.  The layout
// does not depend on M; only the counters must be zero between calls and
// every call leaves them zero.
size_t tc_counter_offset(int sm_count) {
  return static_cast<size_t>(4) * sm_count * kMaxM * kTN * sizeof(float);
}

template <int NT, int GS, bool XBF16>
int run_tc(const void* x, const uint32_t* q, const __half* s, void* y, int M, int K, int N, int G,
           void* ws, const DeviceInfo& dev, cudaStream_t stream) {
  auto kern = gemv_tc_kernel<NT, GS, XBF16>;
  constexpr size_t smem = TcSmem<NT, GS>::kBytes;
  static std::once_flag once[kMaxDevices];
  static int resident[kMaxDevices];
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
  // Every CTA resident at once (the finisher of a split tile waits for the
  // later CTAs; a cooperative launch guarantees they are running).  A CTA's
  // range must touch at most kMaxTiles tiles and a warp's at most kWarpSlots.
  const long long P = std::min<long long>(static_cast<long long>(dev.sm_count) * resident[dev.device], units);
  const long long per_cta = (units + P - 1) / P;
  if ((per_cta + gpt - 1) / gpt + 1 > kMaxTiles) return NG_ERR_BAD_SHAPE;
  if ((per_cta / kWarps + 1 + gpt - 1) / gpt + 1 > kWarpSlots) return NG_ERR_BAD_SHAPE;
  auto* partials = static_cast<float*>(ws);
  auto* counters = reinterpret_cast<unsigned int*>(static_cast<unsigned char*>(ws) +
                                                   tc_counter_offset(dev.sm_count));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(P), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeCooperative;
  attr[1].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const int pq = static_cast<int>(units / P), pr = static_cast<int>(units % P);
  return launch_status(cudaLaunchKernelEx(&cfg, kern, static_cast<const unsigned short*>(x), q, s,
                                          static_cast<unsigned short*>(y), M, K, N, G, pq, pr, gpt,
                                          partials, counters, dev.err));
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

// ---------------------------------------------------------------------------
// Allocation-free entry point.
//
// Some callers cannot allocate device memory when they call the GEMV: code
// running inside a host allocator's or a framework's own memory hook (where a
// cudaMalloc would re-enter it), plugins whose host owns every allocation and
// hands out none, and inference loops that must not touch the allocator on the
// critical path.  They cannot provide the tensor-pipe GEMV's workspace, so this
// entry point takes it from a fixed array in the library's device data
// instead.  The array exists once per GPU that loads the library and stays
// allocated until the process exits.
// ---------------------------------------------------------------------------
namespace ngb {
namespace {

// 3 MiB: partial-sum slots for up to 4 CTAs per SM on up to 160 SMs (2.5 MiB)
// plus arrival counters for ~131k 64-column tiles.
constexpr size_t kNoAllocScratchBytes = 3u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on each device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up with
// cudaGetSymbolAddress, once per device, with that device current.
void* g_noalloc_ptr[kMaxDevices];
int g_noalloc_status[kMaxDevices];
std::once_flag g_noalloc_once[kMaxDevices];

}  // namespace
}  // namespace ngb

extern "C" int ng_gemv_w4a16_noalloc(const void* x, int x_dtype, const int32_t* qweight,
                                     const uint16_t* scales, void* y, int M, int K, int N,
                                     int group_size, void* stream) {
  using namespace ngb;
  if (!x || !qweight || !scales || !y) return NG_ERR_NULL_POINTER;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 16 || K <= 0 || N <= 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (static_cast<long long>(K) * N >= (1LL << 40)) return NG_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(qweight, 16) || !aligned(scales, 8) || !aligned(y, 2))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  const int d = dev.device;
  std::call_once(g_noalloc_once[d], [d] {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    g_noalloc_ptr[d] = p;
    g_noalloc_status[d] = (e == cudaSuccess && p != nullptr) ? NG_OK : NG_ERR_CUDA;
  });
  if (g_noalloc_status[d] != NG_OK) return g_noalloc_status[d];
  // The workspace this call needs must fit the fixed array.
  const size_t need = gemv_tc_workspace_bytes(N, dev);
  if (need > kNoAllocScratchBytes) return NG_ERR_BAD_SHAPE;
  auto strm = static_cast<cudaStream_t>(stream);
  // The arrival counters must start at zero.  A successful call leaves them at
  // zero, but one that gave up on a bounded wait may not, so clear them on the
  // stream first (a memset, not an allocation).
  unsigned char* base = static_cast<unsigned char*>(g_noalloc_ptr[d]);
  const size_t counters = tc_counter_offset(dev.sm_count);
  if (cudaMemsetAsync(base + counters, 0, need - counters, strm) != cudaSuccess) return NG_ERR_CUDA;
  return gemv_tc(x, x_dtype, reinterpret_cast<const uint32_t*>(qweight),
                 reinterpret_cast<const __half*>(scales), y, M, K, N, group_size, base, dev, strm);
}
