// Prefill-regime fused dequant GEMM on the sm_100 tensor cores.
//
// Y[M, N] = X[M, K] @ W.  The product is computed transposed, Y^T = W^T X^T,
// so that the *weights* are the MMA's 128-row A operand and the activations
// are its N operand (BT = 16..256 rows of X per tile):
//   * a tile is 128 output columns (n) x BT rows of X (tokens); its fp32
//     accumulator is a 128-lane x BT-column block of tensor memory;
//   * each decoded weight (one value of W) feeds 2*BT flops, twice what a
//     128-token x 256-column tile of the untransposed product would get, so the
//     CUDA-core decode needed per tensor-core flop is halved;
//   * small batches (M = 16 .. 128) use a narrow N side instead of padding a
//     128-row M side.
//
// Warp roles (512 threads, one CTA per SM, persistent over tiles):
//   warp 0      TMA producer: packed weight tile [8 words x 128 columns] and
//               the X tile [BT rows x 64 values, 128-byte swizzle] per k-step
//   warp 1      MMA issuer: 4 x tcgen05.mma (K = 16 each) per k-step, commit
//               to the stage's "empty" barrier; per tile, commit to "acc full"
//   warp 2      tensor-memory allocator (2 x BT columns: double-buffered acc)
//   warps 4-7   epilogue: tcgen05.ld 128 lanes x BT columns -> fp16/bf16 -> Y
//   warps 8-15  dequant: two groups of four warps taking alternate k-steps (so
//               each warp has two k-steps of time per stage); thread t owns
//               weight column n0 + t and decodes the step's 8 packed rows with the magic-number
//               method, applies the group scale (one rounding, so the fp16
//               operand equals the reference's dequantised weight bit for
//               bit), and writes one 128-byte row of the A tile in the
//               tensor cores' 128-byte-swizzled K-major layout.
// Pipelines: S stages of {A 16 KB, X BT*128 B, raw 4 KB} guarded by
// full (TMA tx) / afull (dequant) / empty (MMA commit) mbarriers; two
// accumulator buffers guarded by tfull / tempty.  Every wait is bounded.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "ng_decode.cuh"
#include "sm100_primitives.cuh"

namespace ngb {
namespace {

constexpr int kTileN = 128;        // weight columns per tile (MMA M)
constexpr int kBK = 64;            // values of K per k-step (one 128-byte swizzle row)
#ifndef NG_GEMM_DQ_GROUPS
#define NG_GEMM_DQ_GROUPS 2
#endif
// Dequant warps 8.. form kDequantGroups groups of 4 warps taking k-steps round-robin.
constexpr int kDequantGroups = NG_GEMM_DQ_GROUPS;
constexpr int kDequantWarps = 4;   // warps per group (one thread per weight column)
constexpr int kThreads = 256 + kDequantGroups * kDequantWarps * 32;
constexpr int kATileBytes = kTileN * kBK * 2;   // 16 KB decoded weights
constexpr int kRawBytes = (kBK / 8) * kTileN * 4;  // 4 KB packed words
constexpr int kSmemBudget = 220 * 1024;

struct Barriers {
  uint64_t full[16];
  uint64_t afull[16];
  uint64_t empty[16];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint32_t tmem_slot;
  int abort;
  int last;  // split-K: this CTA's epilogue finishes the current tile
};

// tcgen05.alloc takes a power-of-two column count in [32, 512]: the two
// BT-column accumulators are placed in the smallest such allocation.
template <int BT>
constexpr uint32_t tmem_cols() {
  uint32_t c = 32;
  while (c < 2u * BT) c <<= 1;
  return c;
}

template <int BT, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmap_x,
                const __grid_constant__ CUtensorMap tmap_q, const __half* __restrict__ scales,
                void* __restrict__ y, int M, int K, int N, int G, int stages, int splits,
                float* __restrict__ ws_part, unsigned int* __restrict__ ws_cnt,
                unsigned int* __restrict__ err) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 1024-byte alignment for the swizzled operand tiles.
  unsigned char* smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  constexpr int kBTileBytes = BT * kBK * 2;
  constexpr int kStageBytes = kATileBytes + kBTileBytes + kRawBytes;
  Barriers* bars = reinterpret_cast<Barriers*>(smem + stages * kStageBytes);
  volatile int* abort = &bars->abort;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = (N + kTileN - 1) / kTileN;
  const int m_tiles = (M + BT - 1) / BT;
  const int tiles = n_tiles * m_tiles;
  const int kb_count = K / kBK;
  // Work units: (tile, K split); unit u covers k-steps [kbs * (u % splits), + kbs).
  const int units = tiles * splits;
  const int kbs = kb_count / splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->afull[s], kDequantWarps);
      mbar_init(&bars->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&bars->tfull[a], 1);
      mbar_init(&bars->tempty[a], 4);
    }
    bars->abort = 0;
    mbar_fence_init();
    tma_prefetch_desc(&tmap_x);
    tma_prefetch_desc(&tmap_q);
  }
  static_assert(tmem_cols<BT>() <= 512, "two accumulators must fit in tensor memory");
  if (warp == 2) tmem_alloc(&bars->tmem_slot, tmem_cols<BT>());
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = bars->tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x) {
        const int tile = u / splits, kb0 = (u % splits) * kbs;
        const int n0 = (tile % n_tiles) * kTileN;
        const int m0 = (tile / n_tiles) * BT;
        for (int kb = kb0; kb < kb0 + kbs; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t ph = (it / stages) & 1;
          if (!mbar_wait_bounded(&bars->empty[s], ph ^ 1, err, abort)) break;
          unsigned char* st = smem + s * kStageBytes;
          mbar_arrive_expect_tx(&bars->full[s], kBTileBytes + kRawBytes);
          tma_load_2d(st + kATileBytes + kBTileBytes, &tmap_q, &bars->full[s], n0, kb * (kBK / 8));
          tma_load_2d(st + kATileBytes, &tmap_x, &bars->full[s], kb * kBK, m0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BF16, kTileN, BT);
      int it = 0, lt = 0;
      for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x, ++lt) {
        const int acc = lt & 1;
        const uint32_t aph = (lt >> 1) & 1;
        if (!mbar_wait_bounded(&bars->tempty[acc], aph ^ 1, err, abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BT;
        bool ok = true;
        for (int kb = 0; kb < kbs; ++kb, ++it) {
          const int s = it % stages;
          const uint32_t ph = (it / stages) & 1;
          if (!mbar_wait_bounded(&bars->full[s], ph, err, abort) ||
              !mbar_wait_bounded(&bars->afull[s], ph, err, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * kStageBytes);
          const uint32_t b_addr = a_addr + kATileBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // Advancing 16 values (32 bytes) along K inside the swizzle atom
            // is a plain start-address offset: the hardware applies the XOR
            // pattern to the absolute address bits.
            umma_f16(d_tmem, sw128_kmajor_desc(a_addr + kk * 32), sw128_kmajor_desc(b_addr + kk * 32),
                     idesc, (kb | kk) != 0);
          }
          umma_commit(&bars->empty[s]);
        }
        if (!ok) break;
        umma_commit(&bars->tfull[acc]);
      }
    }
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 4;  // TMEM lanes 32e .. 32e+31
    int lt = 0;
    unsigned short* yo = static_cast<unsigned short*>(y);
    for (int u = blockIdx.x; u < units && !*abort; u += gridDim.x, ++lt) {
      const int tile = u / splits;
      const int n0 = (tile % n_tiles) * kTileN;
      const int m0 = (tile / n_tiles) * BT;
      const int acc = lt & 1;
      const uint32_t aph = (lt >> 1) & 1;
      if (!mbar_wait_bounded(&bars->tfull[acc], aph, err, abort)) break;
      tc_fence_after();
      const int n = n0 + e * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(e * 32) << 16) + acc * BT;
#pragma unroll 1
      for (int c0 = 0; c0 < BT; c0 += 16) {
        uint32_t r[16];
        tmem_ld_16(taddr + c0, r);
        tmem_ld_wait();
        if (splits > 1) {  // fp32 partial of this unit, [BT][128] (coalesced over n)
          float* part = ws_part + static_cast<size_t>(u) * BT * kTileN;
#pragma unroll
          for (int j = 0; j < 16; ++j) part[(c0 + j) * kTileN + e * 32 + lane] = __uint_as_float(r[j]);
        } else if (n < N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c0 + j;
            if (m < M) {
              const float v = __uint_as_float(r[j]);
              yo[static_cast<size_t>(m) * N + n] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                        : __half_as_ushort(__float2half_rn(v));
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tempty[acc]);
      if (splits > 1) {
        // Last unit of the tile to arrive sums the partials in split order
        // (deterministic), writes Y, and re-arms the tile's counter.
        __threadfence();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (warp == 4 && lane == 0)
          bars->last = atomicAdd(&ws_cnt[tile], 1u) == static_cast<unsigned int>(splits - 1);
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (bars->last) {
          __threadfence();
          const float* base = ws_part + static_cast<size_t>(tile) * splits * BT * kTileN;
          for (int m = 0; m < BT && m0 + m < M; ++m) {
            float v = 0.f;
            for (int sp = 0; sp < splits; ++sp)
              v += __ldcg(base + (static_cast<size_t>(sp) * BT + m) * kTileN + e * 32 + lane);
            if (n < N)
              yo[static_cast<size_t>(m0 + m) * N + n] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                             : __half_as_ushort(__float2half_rn(v));
          }
          if (warp == 4 && lane == 0) ws_cnt[tile] = 0u;
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ dequant
    const int t = (threadIdx.x - 256) & (kTileN - 1);  // weight column within the tile
    const int grp = (threadIdx.x - 256) >> 7;            // this group decodes k-steps it % kDequantGroups == grp
    const int atom = t >> 3, r8 = t & 7;
    const int my_units = units > static_cast<int>(blockIdx.x)
                             ? (units - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                             : 0;
    const int total = my_units * kbs;
    // Scale of iteration i (flattened over this CTA's tiles x k-steps); loaded
    // kPrefetch iterations ahead so its global-memory latency never sits
    // between a stage landing and its decode.
    auto scale_at = [&](int i) -> __half {
      if (i >= total) return __float2half(0.f);
      const int u = static_cast<int>(blockIdx.x) + (i / kbs) * static_cast<int>(gridDim.x);
      const int tile = u / splits;
      const int n = (tile % n_tiles) * kTileN + t;
      const int g = (((u % splits) * kbs + i % kbs) * kBK) / G;
      return n < N ? scales[static_cast<size_t>(g) * N + n] : __float2half(0.f);
    };
    constexpr int kPrefetch = 4;
    __half pf[kPrefetch];
#pragma unroll
    for (int j = 0; j < kPrefetch; ++j) pf[j] = scale_at(grp + j * kDequantGroups);
    for (int it = grp; it < total; it += kDequantGroups) {
      const int s = it % stages;
      const uint32_t ph = (it / stages) & 1;
      const __half sc = pf[0];
#pragma unroll
      for (int j = 0; j + 1 < kPrefetch; ++j) pf[j] = pf[j + 1];
      pf[kPrefetch - 1] = scale_at(it + kPrefetch * kDequantGroups);
      if (!mbar_wait_bounded(&bars->full[s], ph, err, abort)) break;
      unsigned char* st = smem + s * kStageBytes;
      const uint32_t* raw = reinterpret_cast<const uint32_t*>(st + kATileBytes + kBTileBytes);
      unsigned char* arow = st + atom * 1024 + r8 * 128;
      constexpr int kRowsPer = kBK / 8;  // all 8 packed rows of the k-step
      uint32_t qv[kRowsPer];
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i) qv[i] = raw[i * kTileN + t];
#pragma unroll
      for (int i = 0; i < kRowsPer; ++i) {
        const int r = i;
        const uint32_t q = qv[i];
        uint4 v;
        if constexpr (!BF16) {
          __half2 w[4];
          decode8_f16(q, w);
          const __half2 s2 = __half2half2(sc);
          v.x = h2_bits(__hmul2(w[0], s2));
          v.y = h2_bits(__hmul2(w[1], s2));
          v.z = h2_bits(__hmul2(w[2], s2));
          v.w = h2_bits(__hmul2(w[3], s2));
        } else {
          const uint32_t q16 = q >> 16;
          const float sf = __half2float(sc);
          const f2 s2 = f2_make(sf, sf);
          const f2 p[4] = {decode_pair_f32<0>(q, q16), decode_pair_f32<1>(q, q16),
                           decode_pair_f32<2>(q, q16), decode_pair_f32<3>(q, q16)};
          uint32_t bw[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float lo, hi;
            f2_split(f2_mul(p[j], s2), lo, hi);
            const __nv_bfloat162 bb = __floats2bfloat162_rn(lo, hi);
            bw[j] = *reinterpret_cast<const uint32_t*>(&bb);
          }
          v = make_uint4(bw[0], bw[1], bw[2], bw[3]);
        }
        *reinterpret_cast<uint4*>(arow + ((r ^ r8) << 4)) = v;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->afull[s]);
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (*abort) {
    // Let any TMA copy still in flight land before the CTA's shared memory is
    // released (bounded: copies complete in microseconds).
    const uint64_t t0 = global_timer_ns();
    while (global_timer_ns() - t0 < 200000ull) {
    }
  }
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols<BT>());
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
int make_maps(const void* x, const int32_t* q, int M, int K, int N, int BT, CUtensorMap* mx,
              CUtensorMap* mq) {
  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(tensor_map_encode_fn());
  if (!enc) return NG_ERR_CUDA;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(M)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(BT)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(mx, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(x), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K / 8)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(N) * 4};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileN), static_cast<cuuint32_t>(kBK / 8)};
    const cuuint32_t es[2] = {1, 1};
    if (enc(mq, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<int32_t*>(q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return NG_ERR_CUDA;
  }
  return NG_OK;
}

// K splits for grids that would leave SMs idle: the largest divisor d of the
// k-step count with tiles * d <= SMs, d <= 16 and >= 8 k-steps per unit
// (1 without a large enough workspace).
int pick_splits(int tiles, int kb_count, int sm_count) {
  int best = 1;
  for (int d = 2; d <= 16; ++d)
    if (kb_count % d == 0 && kb_count / d >= 8 && tiles * d <= sm_count) best = d;
  return best;
}

// Workspace layout: per-tile arrival counters at a fixed offset (a split grid
// has at most SMs / 2 tiles), then the fp32 partials.  The counters' place must
// not depend on the call's shape: a later call must find them where an
// earlier call of any shape left them (at zero).
size_t gemm_ws_counter_bytes(int sm_count) { return (static_cast<size_t>(sm_count) * 4 + 255) / 256 * 256; }
size_t gemm_ws_bytes(int tiles, int splits, int BT, int sm_count) {
  return splits > 1 ? gemm_ws_counter_bytes(sm_count) + static_cast<size_t>(tiles) * splits * BT * kTileN * 4
                    : 0;
}

template <int BT, bool BF16>
int run_gemm(const void* x, const int32_t* q, const __half* s, void* y, int M, int K, int N, int G,
             void* ws, size_t ws_bytes, const DeviceInfo& dev, cudaStream_t stream) {
  CUtensorMap mx, mq;
  if (int st = make_maps(x, q, M, K, N, BT, &mx, &mq)) return st;
  constexpr int stage_bytes = kATileBytes + BT * kBK * 2 + kRawBytes;
  int stages = std::min(16, (kSmemBudget - 1024 - static_cast<int>(sizeof(Barriers))) / stage_bytes);
  const size_t smem = 1024 + static_cast<size_t>(stages) * stage_bytes + sizeof(Barriers);
  auto kern = gemm_kernel<BT, BF16>;
  static std::once_flag once[kMaxDevices];
  std::call_once(once[dev.device], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget + 4096);
  });
  const int tiles = ((N + kTileN - 1) / kTileN) * ((M + BT - 1) / BT);
  int splits = pick_splits(tiles, K / kBK, dev.sm_count);
  if (ws == nullptr || ws_bytes < gemm_ws_bytes(tiles, splits, BT, dev.sm_count)) splits = 1;
  unsigned int* ws_cnt = splits > 1 ? static_cast<unsigned int*>(ws) : nullptr;
  float* ws_part = splits > 1 ? reinterpret_cast<float*>(static_cast<unsigned char*>(ws) +
                                                         gemm_ws_counter_bytes(dev.sm_count))
                              : nullptr;
  const int grid = std::min(tiles * splits, dev.sm_count);
  kern<<<grid, kThreads, smem, stream>>>(mx, mq, s, y, M, K, N, G, stages, splits, ws_part, ws_cnt,
                                         dev.err);
  return launch_status();
}

template <bool BF16>
int dispatch_bt(int bt, const void* x, const int32_t* q, const __half* s, void* y, int M, int K,
                int N, int G, void* ws, size_t wsb, const DeviceInfo& dev, cudaStream_t st) {
  switch (bt) {
    case 16: return run_gemm<16, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    case 32: return run_gemm<32, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    case 64: return run_gemm<64, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    case 128: return run_gemm<128, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    case 192: return run_gemm<192, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    case 224: return run_gemm<224, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    case 240: return run_gemm<240, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
    default: return run_gemm<256, BF16>(x, q, s, y, M, K, N, G, ws, wsb, dev, st);
  }
}

// Token-tile heuristic: the smallest BT that covers M, capped at 256; for
// larger M pick between 128 and 256 by the number of tile waves.
int pick_bt(int M, int N, int sm_count) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128) return 128;
  const int nt = (N + kTileN - 1) / kTileN;
  auto cost = [&](int bt) {
    const long long tiles = static_cast<long long>(nt) * ((M + bt - 1) / bt);
    const long long waves = (tiles + sm_count - 1) / sm_count;
    return waves * (bt + 32);  // per-tile time ~ BT plus a fixed pipeline fill
  };
  // 192 / 224 / 240 (multiples of 16 and of the 8-row swizzle atom) are
  // accepted as tile_tokens but not picked: they fill the last wave better, yet
  // measured no faster at M = 2048 and slower at M = 8192 -- the k-step time is
  // set by shared-memory traffic and decode, which do not shrink with BT.
  return cost(128) < cost(256) ? 128 : 256;
}

}  // namespace
}  // namespace ngb

extern "C" size_t ng_gemm_workspace_bytes(int M, int N) {
  using namespace ngb;
  DeviceInfo dev;
  if (M < 1 || N <= 0 || current_device_info(&dev) != NG_OK) return 0;
  // split-K is used only while units = tiles x splits <= SMs
  const int bt = pick_bt(M, N, dev.sm_count);
  return gemm_ws_counter_bytes(dev.sm_count) + static_cast<size_t>(dev.sm_count) * bt * kTileN * 4;
}

extern "C" int ng_gemm_w4a16(const void* x, int x_dtype, const int32_t* qweight,
                             const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                             int tile_tokens, void* workspace, size_t workspace_bytes,
                             void* stream) {
  using namespace ngb;
  if (!x || !qweight || !scales || !y) return NG_ERR_NULL_POINTER;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || K <= 0 || N <= 0 || K % kBK != 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (static_cast<long long>(M) * N >= (1LL << 40) || K / 8 > (1 << 30)) return NG_ERR_BAD_SHAPE;
  if (tile_tokens != 0 && tile_tokens != 16 && tile_tokens != 32 && tile_tokens != 64 &&
      tile_tokens != 128 && tile_tokens != 192 && tile_tokens != 224 && tile_tokens != 240 &&
      tile_tokens != 256)
    return NG_ERR_BAD_ARGUMENT;
  if (!aligned(x, 16) || !aligned(qweight, 16) || !aligned(scales, 2) || !aligned(y, 2) ||
      !aligned(workspace, 256))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  const int bt = tile_tokens ? tile_tokens : pick_bt(M, N, dev.sm_count);
  auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  if (x_dtype == NG_DTYPE_BF16)
    return dispatch_bt<true>(bt, x, qweight, s, y, M, K, N, group_size, workspace, workspace_bytes,
                             dev, strm);
  return dispatch_bt<false>(bt, x, qweight, s, y, M, K, N, group_size, workspace, workspace_bytes,
                            dev, strm);
}
