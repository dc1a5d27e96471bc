// Causal GQA attention for the prefill of a Llama-style decoder (head_dim 128):
// out[b, s, h, :] = softmax(q[b, s, h] . K[b, 0 .. pos0[b] + s]^T * scale) V
// where K / V are read from the KV cache that ng_rope_prefill has just filled
// (one cache per sequence, [B, max_ctx, Hkv, 128], query head h reading KV head
// h / (Hq / Hkv)).  The prompt's queries also see any rows the cache already
// held before pos0[b] (a prefill that continues a sequence).
//
// FlashAttention-2 structure on the warp-level tensor-core MMA (m16n8k16,
// fp32 accumulation):
//   * CTA = 4 warps = 64 query rows of one (sequence, query head); warp w owns
//     rows 16w .. 16w + 15 and keeps their Q fragments (16 x 128) and output
//     accumulators (16 x 128 fp32) in registers for the whole key sweep;
//   * keys in blocks of 64: K and V tiles (64 x 128 each) double-buffered in
//     shared memory by cp.async, rows XOR-swizzled in 16-byte chunks so the
//     ldmatrix reads are conflict-free;
//   * S = Q K^T per block (64 MMAs per warp), causal mask on the blocks that
//     reach past a row's position, online softmax in fp32 (exp2 with the
//     scale folded into log2 e), P rounded to the activation type and fed from
//     the S accumulators straight into O += P V (64 MMAs per warp);
//   * query blocks are issued heaviest (latest) first.
// Attention is a small share of a 2048-token prefill (the projections through
// ng_gemm_w4a16 are ~95 % of the FLOPs), so this kernel stays on the legacy
// MMA path rather than tcgen05.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>

#include "ng_common.cuh"

namespace ngb {
namespace {

constexpr int kPD = 128;                 // head dim
constexpr int kPQ = 64;                  // query rows per CTA
constexpr int kPK = 64;                  // keys per block
constexpr int kPThreads = 128;           // 4 warps x 16 query rows
constexpr int kPTileBytes = kPK * kPD * 2;  // one K or V tile
constexpr int kPSmem = 4 * kPTileBytes;  // K and V, double-buffered

__device__ __forceinline__ uint32_t psmem(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// Byte offset of 16-byte chunk c (0..15) of tile row r: chunks XOR-swizzled
// by the row's low 3 bits.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 256 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void cp16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm4t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <bool BF16>
__device__ __forceinline__ void pmma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                     uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  } else {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

template <bool BF16>
__global__ void __launch_bounds__(kPThreads)
    attn_prefill_kernel(const unsigned short* __restrict__ q, const unsigned short* __restrict__ kc,
                        const unsigned short* __restrict__ vc, const int* __restrict__ pos0,
                        unsigned short* __restrict__ out, int S, int Hq, int Hkv, int max_ctx,
                        float scale_log2) {
  extern __shared__ __align__(128) unsigned char smem[];
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, qd = lane & 3;
  const int qb = gridDim.x - 1 - blockIdx.x;  // latest (most keys) first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (Hq / Hkv);
  const int p0 = pos0[b];
  const int s0 = qb * kPQ;
  // keys this CTA needs: up to the position of its last valid query row
  const int last_q = min(s0 + kPQ, S) - 1;
  const int nkeys = min(p0 + last_q + 1, max_ctx);
  const int nblocks = (nkeys + kPK - 1) / kPK;

  const size_t krow = static_cast<size_t>(Hkv) * kPD;  // elements between cache rows
  const unsigned short* kbase = kc + (static_cast<size_t>(b) * max_ctx * Hkv + kh) * kPD;
  const unsigned short* vbase = vc + (static_cast<size_t>(b) * max_ctx * Hkv + kh) * kPD;
  const uint32_t sbase = psmem(smem);

  auto load_block = [&](int blk, int buf) {
    const int key0 = blk * kPK;
    const uint32_t kd = sbase + buf * 2 * kPTileBytes, vd = kd + kPTileBytes;
#pragma unroll
    for (int j = 0; j < (kPK * 16) / kPThreads; ++j) {
      const int i = tid + j * kPThreads;
      const int r = i >> 4, c = i & 15;
      const int key = key0 + r;
      const bool ok = key < nkeys;
      const size_t off = static_cast<size_t>(ok ? key : 0) * krow + c * 8;
      cp16(kd + swz(r, c), kbase + off, ok);
      cp16(vd + swz(r, c), vbase + off, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  load_block(0, 0);

  // Q fragments of this warp's 16 rows (zero for rows past S)
  const int r_lo = s0 + warp * 16 + g, r_hi = r_lo + 8;
  uint32_t qf[8][4];
  {
    const unsigned short* qlo = q + (static_cast<size_t>(b) * S + r_lo) * Hq * kPD + static_cast<size_t>(h) * kPD;
    const unsigned short* qhi = q + (static_cast<size_t>(b) * S + r_hi) * Hq * kPD + static_cast<size_t>(h) * kPD;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d = 16 * kk + 2 * qd;
      qf[kk][0] = r_lo < S ? *reinterpret_cast<const uint32_t*>(qlo + d) : 0u;
      qf[kk][1] = r_hi < S ? *reinterpret_cast<const uint32_t*>(qhi + d) : 0u;
      qf[kk][2] = r_lo < S ? *reinterpret_cast<const uint32_t*>(qlo + d + 8) : 0u;
      qf[kk][3] = r_hi < S ? *reinterpret_cast<const uint32_t*>(qhi + d + 8) : 0u;
    }
  }
  const int qp_lo = p0 + r_lo, qp_hi = p0 + r_hi;  // query positions

  float o[16][4];
#pragma unroll
  for (int t = 0; t < 16; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;

  for (int blk = 0; blk < nblocks; ++blk) {
    const int buf = blk & 1;
    if (blk + 1 < nblocks) {
      load_block(blk + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint32_t kt = sbase + buf * 2 * kPTileBytes, vt = kt + kPTileBytes;
    const int key0 = blk * kPK;

    // ---- S = Q K^T (16 rows x 64 keys per warp)
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
      for (int kp = 0; kp < 4; ++kp) {  // two k-steps (32 values of d) per ldmatrix.x4
        uint32_t b0, b1, b2, b3;
        ldsm4(kt + swz(8 * j + (lane & 7), 4 * kp + (lane >> 3)), b0, b1, b2, b3);
        pmma<BF16>(sc[j], qf[2 * kp][0], qf[2 * kp][1], qf[2 * kp][2], qf[2 * kp][3], b0, b1);
        pmma<BF16>(sc[j], qf[2 * kp + 1][0], qf[2 * kp + 1][1], qf[2 * kp + 1][2], qf[2 * kp + 1][3], b2, b3);
      }
    }
    // ---- causal mask (blocks reaching past the earliest row of this warp)
    if (key0 + kPK - 1 > p0 + s0 + warp * 16) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int kp = key0 + 8 * j + 2 * qd;
        if (kp > qp_lo) sc[j][0] = -INFINITY;
        if (kp + 1 > qp_lo) sc[j][1] = -INFINITY;
        if (kp > qp_hi) sc[j][2] = -INFINITY;
        if (kp + 1 > qp_hi) sc[j][3] = -INFINITY;
      }
    }
    // ---- online softmax (rows g and g + 8; the quad's 4 lanes share a row)
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx_lo = fmaxf(mx_lo, fmaxf(sc[j][0], sc[j][1]));
      mx_hi = fmaxf(mx_hi, fmaxf(sc[j][2], sc[j][3]));
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo * scale_log2), mn_hi = fmaxf(m_hi, mx_hi * scale_log2);
    // a row with nothing unmasked yet keeps a -inf maximum: use 0 as its base
    const float base_lo = mn_lo == -INFINITY ? 0.f : mn_lo, base_hi = mn_hi == -INFINITY ? 0.f : mn_hi;
    const float corr_lo = exp2f(m_lo - base_lo), corr_hi = exp2f(m_hi - base_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    l_lo *= corr_lo;
    l_hi *= corr_hi;
#pragma unroll
    for (int t = 0; t < 16; ++t) {
      o[t][0] *= corr_lo;
      o[t][1] *= corr_lo;
      o[t][2] *= corr_hi;
      o[t][3] *= corr_hi;
    }
    uint32_t pa[4][4];  // P as the A operand of P V, per 16-key step
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float e0 = exp2f(sc[j][0] * scale_log2 - base_lo), e1 = exp2f(sc[j][1] * scale_log2 - base_lo);
      const float e2 = exp2f(sc[j][2] * scale_log2 - base_hi), e3 = exp2f(sc[j][3] * scale_log2 - base_hi);
      l_lo += e0 + e1;
      l_hi += e2 + e3;
      pa[j >> 1][(j & 1) * 2 + 0] = pack2<BF16>(e0, e1);
      pa[j >> 1][(j & 1) * 2 + 1] = pack2<BF16>(e2, e3);
    }
    // ---- O += P V (16 rows x 128 dims per warp)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int t = 0; t < 16; t += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm4t(vt + swz(16 * kk + (lane & 15), t + (lane >> 4)), b0, b1, b2, b3);
        pmma<BF16>(o[t], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        pmma<BF16>(o[t + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
      }
    }
    __syncthreads();  // this buffer is refilled by the next iteration's load
  }

  // ---- normalise and store (rows past S are not written)
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  unsigned short* olo = out + (static_cast<size_t>(b) * S + r_lo) * Hq * kPD + static_cast<size_t>(h) * kPD;
  unsigned short* ohi = out + (static_cast<size_t>(b) * S + r_hi) * Hq * kPD + static_cast<size_t>(h) * kPD;
#pragma unroll
  for (int t = 0; t < 16; ++t) {
    const int d = 8 * t + 2 * qd;
    if (r_lo < S) *reinterpret_cast<uint32_t*>(olo + d) = pack2<BF16>(o[t][0] * inv_lo, o[t][1] * inv_lo);
    if (r_hi < S) *reinterpret_cast<uint32_t*>(ohi + d) = pack2<BF16>(o[t][2] * inv_hi, o[t][3] * inv_hi);
  }
}

}  // namespace
}  // namespace ngb

extern "C" int ng_attn_prefill(const void* q, const void* k_cache, const void* v_cache, const int* pos0,
                               void* out, int dtype, int B, int S, int Hq, int Hkv, int D, int max_ctx,
                               float scale, void* stream) {
  using namespace ngb;
  if (!q || !k_cache || !v_cache || !pos0 || !out) return NG_ERR_NULL_POINTER;
  if (dtype != NG_DTYPE_F16 && dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (D != kPD || B < 1 || B > 65535 || S < 1 || Hq < 1 || Hq > 65535 || Hkv < 1 || Hq % Hkv ||
      max_ctx < 1)
    return NG_ERR_BAD_SHAPE;
  if (!aligned(q, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) || !aligned(out, 4))
    return NG_ERR_MISALIGNED;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((S + kPQ - 1) / kPQ, Hq, B);
  cfg.blockDim = dim3(kPThreads, 1, 1);
  cfg.dynamicSmemBytes = kPSmem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float sl2 = scale * 1.4426950408889634f;  // softmax in base 2
  const auto* qq = static_cast<const unsigned short*>(q);
  const auto* kk = static_cast<const unsigned short*>(k_cache);
  const auto* vv = static_cast<const unsigned short*>(v_cache);
  auto* oo = static_cast<unsigned short*>(out);
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  static std::once_flag once[kMaxDevices];
  std::call_once(once[dev.device], [] {
    cudaFuncSetAttribute(attn_prefill_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
    cudaFuncSetAttribute(attn_prefill_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem);
  });
  if (dtype == NG_DTYPE_BF16)
    return launch_status(cudaLaunchKernelEx(&cfg, attn_prefill_kernel<true>, qq, kk, vv, pos0, oo, S, Hq,
                                            Hkv, max_ctx, sl2));
  return launch_status(cudaLaunchKernelEx(&cfg, attn_prefill_kernel<false>, qq, kk, vv, pos0, oo, S, Hq,
                                          Hkv, max_ctx, sl2));
}
