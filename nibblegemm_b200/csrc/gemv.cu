// Decode-regime fused dequant GEMV: Y[M, N] = X[M, K] @ W, M <= 16, one launch.
//
// Work decomposition (all sizes in packed rows: one packed row = 8 values of K)
//   * A CTA owns a 128-column tile (32 lanes x 4 columns, one 16-byte packed
//     load per lane per row) and a contiguous K slice of `rows_per_cta` rows.
//   * The CTAs sharing a column tile form one thread-block cluster along
//     gridDim.y (cluster size = number of K slices, up to 16).  Each CTA reduces
//     its warps' partial sums in shared memory, then the cluster reduces the
//     slices through distributed shared memory: CTA r of the cluster sums a
//     1/C share of the tile's outputs over ranks 0..C-1 in fixed order and
//     writes them.  No global workspace, no second launch, deterministic.
//   * Inside a CTA, warps take 8-row chunks (64 values of K, always inside one
//     quantisation group because G >= 64) round-robin.  A chunk issues its eight
//     16-byte weight loads back to back before decoding any of them, so every
//     lane keeps 128 bytes in flight; at 2-4 resident CTAs of 8 warps per SM
//     that is 64-128 KB per SM, comfortably above the bandwidth-latency product.
//   * Activations for the CTA's K slice are staged once in shared memory (in
//     the accumulation type) and read as broadcasts.
//   * Each warp software-pipelines its chunks: the next chunk's eight loads
//     are issued before the current chunk is decoded.
//   * Programmatic dependent launch: the kernel is launched with programmatic
//     stream serialisation, signals `griddepcontrol.launch_dependents` on
//     entry and issues its first weight loads *before* `griddepcontrol.wait`.
//     Weights are read-only, so a GEMV streams its weights while the kernel
//     before it on the stream drains; activations are read and Y written only
//     after the wait, so the data dependency on the previous kernel holds.
//     Back-to-back decode GEMVs (a model's layer sequence) thereby hide the
//     launch and ramp-up latency that dominates a ~5 us kernel.
//
// Two accumulation paths:
//   * kHalf2 (fp16 activations): the fp16 magic-number decode, packed half2
//     FMA over 32 values of K, then a flush into fp32 multiplied by the group
//     scale.  9 decode instructions + 4 HFMA2 per word per row of X.
//   * kFloat2 (bf16 activations; optional for fp16): the fp32 magic-number
//     decode (exact u - 8 as fp32x2 pairs) and packed fp32x2 FMA, scale applied
//     once per 8-row chunk (or per word for M >= 8, to bound registers).
//     Accumulation is fp32 throughout.
#include <cooperative_groups.h>

#include <algorithm>
#include <mutex>
#include <type_traits>

#include "ng_decode.cuh"

namespace cg = cooperative_groups;

namespace ngb {
namespace {

constexpr int kCols = 128;  // columns per CTA tile
constexpr int kU = 8;       // packed rows per chunk
constexpr int kWin = 4;     // half2 path: packed rows per fp16 accumulation window
constexpr int kMaxCluster = 16;
constexpr int kStageBudget = 160 * 1024;  // activation staging limit (bytes)
constexpr int kAttnHeadDim = 128;         // head dimension of the folded attention combine

// Shared-memory offset of the folded attention-combine weights: after the
// staged activations / warp partials and the CTA's final sums.
__host__ __device__ inline size_t na_attw_offset(int MT, int rows_per_cta, int esz, int warps) {
  const size_t stage = static_cast<size_t>(MT) * rows_per_cta * 8 * esz;
  const size_t red = static_cast<size_t>(warps) * MT * kCols * 4;
  return (stage > red ? stage : red) + static_cast<size_t>(MT) * kCols * 4;
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

enum Path { kHalf2 = 0, kFloat2 = 1 };

// Optional RMSNorm of the activations, folded into the staging of X (the
// decode step's norm before the q|k|v and gate|up projections):
//   h = x + res_in;  X = act(h * rsqrt(mean(h^2) + eps) * w);  res_out = h
// with `act` the rounding to the activation type.  Every CTA re-reduces the
// whole row (a few KB from L2); CTA (0, 0) writes res_out, which must not
// alias res_in (the caller ping-pongs two residual buffers).  w == nullptr:
// plain GEMV.
//
// Two more foldings replace the kernel that would produce X (mode):
//   kStageSilu: X[m, k] = act(silu(g) * u) with g = src[m, k], u = src[m, K + k]
//     of the gate|up projection's output [M, 2K] (the SwiGLU before `down`);
//   kStageAttn: X[m, h * 128 + d] = the split-context attention partials
//     part[m][h][s] = (max_s, sum_s, o_s[128]) combined in split order,
//     sum_s w_s o_s[d] / sum_s w_s sum_s with w_s = exp(max_s - max), exactly as
//     the standalone combine kernel (the attention output before `o`).
constexpr int kArMaxWorld = 8;
constexpr int kArMaxSlices = 16;  // cluster ranks (K slices) per column tile

// Exchange buffer of the fused GEMV + all-reduce, per rank (sized for any M <= 16):
//   data  fp32 [2 parity][world][tiles][16 x 128]   (each source rank's partial Y)
//   flags u32  [2 parity][tiles][16 slices][world]  (call counter + 1 per source)
//   ctr   u32  [tiles][16 slices]                   (this rank's call counter per slice)
struct ArLayout {
  size_t data, flags, ctr, total;
  __host__ __device__ ArLayout(int world, int tiles) {
    data = static_cast<size_t>(2) * world * tiles * 16 * 128 * 4;
    flags = static_cast<size_t>(2) * tiles * kArMaxSlices * world * 4;
    ctr = static_cast<size_t>(tiles) * kArMaxSlices * 4;
    total = data + flags + ctr;
  }
};

__device__ __forceinline__ unsigned int ar_ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ar_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void ar_st_release(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

enum StageMode { kStagePlain = 0, kStageNorm = 1, kStageSilu = 2, kStageAttn = 3 };

struct NormArgs {
  const unsigned short* res_in = nullptr;
  unsigned short* res_out = nullptr;
  const unsigned short* w = nullptr;
  float eps = 0.f;
  int mode = kStagePlain;
  const float* part = nullptr;  // kStageAttn: [M][K / 128][splits][2 + 128]
  int splits = 0;
  // Fused tensor-parallel reduction (world > 1): every rank's buffer, as mapped
  // in this process (layout: see gemv_ar_layout).
  unsigned char* peers[kArMaxWorld] = {};
  int ar_rank = 0;
  int ar_world = 1;
  unsigned int* ar_err = nullptr;  // device error word (bounded flag waits)
};

template <bool XBF16>
__device__ __forceinline__ void unpack8(uint4 v, float (&f)[8]) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
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
}

template <bool XBF16>
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if constexpr (XBF16) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&b);
    } else {
      w[j] = h2_bits(__floats2half2_rn(f[2 * j], f[2 * j + 1]));
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int MT, bool XBF16, int PATH, int WARPS>
__global__ void __launch_bounds__(WARPS * 32)
    gemv_kernel(const void* __restrict__ x, const uint32_t* __restrict__ qw,
                const __half* __restrict__ scales, void* __restrict__ y, int M, int K, int N,
                int G, int rows_per_cta, int csize, NormArgs na) {
  extern __shared__ __align__(16) unsigned char smem[];
  using XS = typename std::conditional<PATH == kFloat2, float, __half>::type;
  XS* xs = reinterpret_cast<XS*>(smem);
  const int xstride = rows_per_cta * 8;  // staged elements per row of X

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int krows = K >> 3;
  const int kr0 = blockIdx.y * rows_per_cta;
  const int kr1 = min(krows, kr0 + rows_per_cta);
  const int col = blockIdx.x * kCols + lane * 4;
  const bool col_ok = col < N;
  const uint64_t pol = make_evict_first_policy();
  const unsigned short* xin = static_cast<const unsigned short*>(x);

  float acc[4][MT];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[c][m] = 0.f;

  griddep_launch_dependents();
  const int nrows = max(0, kr1 - kr0);
  const int nch = nrows / kU;
  auto load_chunk = [&](int ch, uint4 (&q)[kU], uint2& sv) {
    const int r0 = kr0 + ch * kU;
#pragma unroll
    for (int u = 0; u < kU; ++u)
      q[u] = col_ok ? ld_stream_v4(qw + static_cast<size_t>(r0 + u) * N + col, pol)
                    : make_uint4(0x88888888u, 0x88888888u, 0x88888888u, 0x88888888u);
    const int grp = (r0 * 8) / G;
    sv = col_ok ? ld_ro_v2(scales + static_cast<size_t>(grp) * N + col) : make_uint2(0u, 0u);
  };
  auto process = [&](int ch, const uint4 (&q)[kU], uint2 sv) {
    const int r0 = kr0 + ch * kU;
    float sc[4];
    sc[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x & 0xFFFF)));
    sc[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.x >> 16)));
    sc[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y & 0xFFFF)));
    sc[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(sv.y >> 16)));
    const XS* xc = xs + (r0 - kr0) * 8;

    if constexpr (PATH == kHalf2) {
#pragma unroll
      for (int win = 0; win < kU / kWin; ++win) {
        __half2 h[4][MT];
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int m = 0; m < MT; ++m) h[c][m] = __float2half2_rn(0.f);
#pragma unroll
        for (int rr = 0; rr < kWin; ++rr) {
          const int u = win * kWin + rr;
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
      }
    } else {
      constexpr bool kScaleEarly = MT >= 8;
      f2 a2[4][MT];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int m = 0; m < MT; ++m) a2[c][m] = f2_make(0.f, 0.f);
      f2 s2[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) s2[c] = f2_make(sc[c], sc[c]);
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const uint32_t words[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
        f2 wv[4][4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t w16 = words[c] >> 16;
          wv[c][0] = decode_pair_f32<0>(words[c], w16);
          wv[c][1] = decode_pair_f32<1>(words[c], w16);
          wv[c][2] = decode_pair_f32<2>(words[c], w16);
          wv[c][3] = decode_pair_f32<3>(words[c], w16);
          if constexpr (kScaleEarly) {
#pragma unroll
            for (int j = 0; j < 4; ++j) wv[c][j] = f2_mul(wv[c][j], s2[c]);
          }
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
          if constexpr (kScaleEarly)
            acc[c][m] += lo + hi;
          else
            acc[c][m] = fmaf(lo + hi, sc[c], acc[c][m]);
        }
    }

  };

  uint4 qa[kU], qb[kU];
  uint2 sa = make_uint2(0u, 0u), sb = make_uint2(0u, 0u);
  int ch = warp;
  if (ch < nch) load_chunk(ch, qa, sa);  // weights only: no dependency on the previous kernel
  griddep_wait();                          // activations / outputs of the previous kernel
  __shared__ float s_inv[MT];
  if (na.w != nullptr) {  // ---- folded RMSNorm: per-token 1/rms over the whole row ----
    __shared__ float s_red[WARPS][MT];
    float ss[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m) ss[m] = 0.f;
    for (int c = tid; c < K / 8; c += WARPS * 32) {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < M) {
          float a[8], b[8];
          unpack8<XBF16>(ld_ro_v4(xin + static_cast<size_t>(m) * K + static_cast<size_t>(c) * 8), a);
          unpack8<XBF16>(ld_ro_v4(na.res_in + static_cast<size_t>(m) * K + static_cast<size_t>(c) * 8), b);
#pragma unroll
          for (int j = 0; j < 8; ++j) ss[m] += (a[j] + b[j]) * (a[j] + b[j]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      for (int o = 16; o > 0; o >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], o);
      if (lane == 0) s_red[warp][m] = ss[m];
    }
    __syncthreads();
    if (tid < MT) {
      float t = 0.f;
      for (int w2 = 0; w2 < WARPS; ++w2) t += s_red[w2][tid];  // fixed order
      s_inv[tid] = rsqrtf(t / static_cast<float>(K) + na.eps);
    }
    if (na.res_out != nullptr && blockIdx.x == 0 && blockIdx.y == 0) {
      for (int i = tid; i < M * (K / 8); i += WARPS * 32) {
        const int m = i / (K / 8), c = i - m * (K / 8);
        float a[8], b[8];
        unpack8<XBF16>(ld_ro_v4(xin + static_cast<size_t>(m) * K + static_cast<size_t>(c) * 8), a);
        unpack8<XBF16>(ld_ro_v4(na.res_in + static_cast<size_t>(m) * K + static_cast<size_t>(c) * 8), b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[j] += b[j];
        *reinterpret_cast<uint4*>(na.res_out + static_cast<size_t>(m) * K + static_cast<size_t>(c) * 8) =
            pack8<XBF16>(a);
      }
    }
    __syncthreads();
  }
  // ---- folded attention combine: per (token, head of the slice) split weights ----
  const int h0 = (kr0 * 8) / kAttnHeadDim;
  const int nh = nrows > 0 ? ((kr1 * 8 + kAttnHeadDim - 1) / kAttnHeadDim) - h0 : 0;
  float* attw = nullptr;  // [MT][nh][splits + 1]: w_s, then the denominator
  if (na.mode == kStageAttn) {
    attw = reinterpret_cast<float*>(smem + na_attw_offset(MT, rows_per_cta, sizeof(XS), WARPS));
    const int hq = K / kAttnHeadDim;
    for (int i = tid; i < M * nh; i += WARPS * 32) {
      const int m = i / nh, hl = i - m * nh;
      const float* p = na.part + (static_cast<size_t>(m) * hq + h0 + hl) * na.splits * (2 + kAttnHeadDim);
      float mx = -INFINITY;
      for (int sp = 0; sp < na.splits; ++sp) mx = fmaxf(mx, p[sp * (2 + kAttnHeadDim)]);
      float den = 0.f;
      float* wv = attw + static_cast<size_t>(i) * (na.splits + 1);
      for (int sp = 0; sp < na.splits; ++sp) {
        const float ms = p[sp * (2 + kAttnHeadDim)];
        const float w = ms == -INFINITY ? 0.f : __expf(ms - mx);  // empty split: weight 0
        wv[sp] = w;
        if (ms != -INFINITY) den += w * p[sp * (2 + kAttnHeadDim) + 1];
      }
      wv[na.splits] = den;
    }
    __syncthreads();
  }
  // ---- stage X[:, kr0*8 : kr1*8) ------------------------------------------------
  for (int i = tid; i < MT * nrows; i += WARPS * 32) {
    const int m = i / nrows;
    const int r = i - m * nrows;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    const size_t k0 = static_cast<size_t>(kr0 + r) * 8;
    if (m < M && (na.mode == kStagePlain || na.mode == kStageNorm))
      v = ld_ro_v4(xin + static_cast<size_t>(m) * K + k0);
    if (m < M && na.mode == kStageSilu) {  // act(silu(gate) * up), as the SwiGLU kernel rounds it
      float gt[8], up[8];
      unpack8<XBF16>(ld_ro_v4(xin + static_cast<size_t>(m) * 2 * K + k0), gt);
      unpack8<XBF16>(ld_ro_v4(xin + static_cast<size_t>(m) * 2 * K + K + k0), up);
#pragma unroll
      for (int j = 0; j < 8; ++j) gt[j] = gt[j] / (1.f + __expf(-gt[j])) * up[j];
      v = pack8<XBF16>(gt);
    }
    if (m < M && na.mode == kStageAttn) {  // combine the splits in split order
      const int head = static_cast<int>(k0 / kAttnHeadDim);
      const int d0 = static_cast<int>(k0 % kAttnHeadDim);
      const float* wv = attw + (static_cast<size_t>(m) * nh + (head - h0)) * (na.splits + 1);
      const float* p = na.part + (static_cast<size_t>(m) * (K / kAttnHeadDim) + head) * na.splits * (2 + kAttnHeadDim) + 2 + d0;
      float num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int sp = 0; sp < na.splits; ++sp) {
        const float w = wv[sp];
        if (w == 0.f) continue;
        // a record is 130 floats: 8-byte aligned (d0 is a multiple of 8), not 16
        const float2* o = reinterpret_cast<const float2*>(p + static_cast<size_t>(sp) * (2 + kAttnHeadDim));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 t = o[j];
          num[2 * j] += w * t.x;
          num[2 * j + 1] += w * t.y;
        }
      }
      const float den = wv[na.splits];
#pragma unroll
      for (int j = 0; j < 8; ++j) num[j] = num[j] / den;
      v = pack8<XBF16>(num);
    }
    if (na.mode == kStageNorm && m < M) {  // h = x + res_in, normalised, rounded to the activation type
      float a[8], b[8], wf[8];
      unpack8<XBF16>(v, a);
      unpack8<XBF16>(ld_ro_v4(na.res_in + static_cast<size_t>(m) * K + static_cast<size_t>(kr0 + r) * 8), b);
      unpack8<XBF16>(ld_ro_v4(na.w + static_cast<size_t>(kr0 + r) * 8), wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = (a[j] + b[j]) * s_inv[m] * wf[j];
      v = pack8<XBF16>(a);
    }
    XS* dst = xs + m * xstride + r * 8;
    if constexpr (PATH == kFloat2) {
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
  __syncthreads();
  // ---- stream the weights, one chunk ahead ------------------------------------
  while (ch < nch) {
    int nx = ch + WARPS;
    if (nx < nch) load_chunk(nx, qb, sb);
    process(ch, qa, sa);
    ch = nx;
    if (ch >= nch) break;
    nx = ch + WARPS;
    if (nx < nch) load_chunk(nx, qa, sa);
    process(ch, qb, sb);
    ch = nx;
  }

  // ---- CTA reduction over warps (fixed order) ---------------------------------
  constexpr int E = MT * kCols;
  const size_t stage_bytes = static_cast<size_t>(MT) * xstride * sizeof(XS);  // staged X
  const size_t red_bytes = static_cast<size_t>(WARPS) * E * sizeof(float);
  float* red = reinterpret_cast<float*>(smem);
  float* fin = reinterpret_cast<float*>(smem + (stage_bytes > red_bytes ? stage_bytes : red_bytes));
  __syncthreads();
#pragma unroll
  for (int m = 0; m < MT; ++m)
    *reinterpret_cast<float4*>(red + (warp * MT + m) * kCols + lane * 4) =
        make_float4(acc[0][m], acc[1][m], acc[2][m], acc[3][m]);
  __syncthreads();

  auto store = [&](int e, float v) {
    const int m = e / kCols;
    const int cn = blockIdx.x * kCols + (e % kCols);
    if (m < M && cn < N) {
      unsigned short* yo = static_cast<unsigned short*>(y);
      yo[static_cast<size_t>(m) * N + cn] = XBF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                                                  : __half_as_ushort(__float2half_rn(v));
    }
  };

  const bool fused_ar = na.ar_world > 1;
  float* vals = nullptr;  // this CTA's reduced outputs [e0, e1) (fused all-reduce only)
  int e0 = 0, e1 = E, slice = 0;
  if (csize == 1) {
    for (int e = tid; e < E; e += WARPS * 32) {
      float v = 0.f;
#pragma unroll 4
      for (int w = 0; w < WARPS; ++w) v += red[w * E + e];
      if (fused_ar)
        fin[e] = v;
      else
        store(e, v);
    }
    if (!fused_ar) return;
    vals = fin;
  } else {
    for (int e = tid; e < E; e += WARPS * 32) {
      float v = 0.f;
#pragma unroll 4
      for (int w = 0; w < WARPS; ++w) v += red[w * E + e];
      fin[e] = v;
    }
    // ---- cluster reduction over K slices through DSMEM ---------------------------
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    slice = static_cast<int>(cluster.block_rank());
    const int per = (E + csize - 1) / csize;
    e0 = slice * per;
    e1 = min(E, e0 + per);
    for (int e = e0 + tid; e < e1; e += WARPS * 32) {
      float v = 0.f;
      for (int r = 0; r < csize; ++r) v += cluster.map_shared_rank(fin, r)[e];
      if (fused_ar)
        red[e - e0] = v;  // red is private to this CTA: peers read only fin
      else
        store(e, v);
    }
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
    if (!fused_ar) return;
    vals = red;
  }

  // ---- fused tensor-parallel all-reduce of this CTA's outputs over peer memory ----
  // Push the slice to every rank's buffer (plain stores), raise this rank's
  // flag there, wait (bounded) for every rank's flag here, sum in rank order:
  // every rank ends with bit-identical Y.  One counter per (tile, slice) makes
  // calls capturable in a CUDA graph; parity double-buffers the slots (a slot
  // is rewritten only after every peer has passed the next call's flags).
  {
    const int W = na.ar_world, me = na.ar_rank;
    const int tiles = (N + kCols - 1) / kCols;
    const ArLayout L(W, tiles);
    const int tile = blockIdx.x;
    unsigned char* own = na.peers[me];
    unsigned int* ctr = reinterpret_cast<unsigned int*>(own + L.data + L.flags) + tile * kArMaxSlices + slice;
    __shared__ unsigned int s_ep;
    __syncthreads();
    if (tid == 0) s_ep = *ctr;
    __syncthreads();
    const unsigned int ep = s_ep;
    const int par = static_cast<int>(ep & 1u);
    auto data = [&](unsigned char* base, int src) {
      return reinterpret_cast<float*>(base) + ((static_cast<size_t>(par) * W + src) * tiles + tile) * 2048;
    };
    auto flag = [&](unsigned char* base, int src) {
      return reinterpret_cast<unsigned int*>(base + L.data) +
             ((static_cast<size_t>(par) * tiles + tile) * kArMaxSlices + slice) * W + src;
    };
    for (int e = e0 + tid; e < e1; e += WARPS * 32) {
      const float v = vals[e - e0];
      for (int p = 0; p < W; ++p) data(na.peers[p], me)[e] = v;
    }
    __syncthreads();  // every push before the release stores (release is cumulative)
    if (tid < W) ar_st_release(flag(na.peers[tid], me), ep + 1);
    if (tid < W) {
      const unsigned int* f = flag(own, tid);
      const uint64_t t0 = ar_timer_ns();
      while (ar_ld_acquire(f) != ep + 1) {
        if (ar_timer_ns() - t0 > 1000000000ull) {
          atomicOr(na.ar_err, kErrWaitTimeout);
          break;
        }
      }
    }
    __syncthreads();
    for (int e = e0 + tid; e < e1; e += WARPS * 32) {
      float v = 0.f;
      for (int src = 0; src < W; ++src) v += __ldcg(data(own, src) + e);  // rank order
      store(e, v);
    }
    if (tid == 0) *ctr = ep + 1;
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int MT, bool XBF16, int PATH, int WARPS>
int run(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N, int G,
        int splits, const DeviceInfo& dev, cudaStream_t stream, NormArgs na = {}) {
  auto kern = gemv_kernel<MT, XBF16, PATH, WARPS>;
  constexpr int threads = WARPS * 32;
  constexpr int esz = PATH == kFloat2 ? 4 : 2;
  const int krows = K / 8;
  const int col_tiles = (N + kCols - 1) / kCols;

  // Per-device one-time attribute set-up for this instantiation.
  static std::once_flag once[kMaxDevices];
  static int occ_cache[kMaxDevices];
  const int d = dev.device;
  std::call_once(once[d], [&] {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    int occ = 0;
    const size_t probe_smem = static_cast<size_t>(WARPS) * MT * kCols * 4 * 2;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, probe_smem) != cudaSuccess)
      occ = 1;
    occ_cache[d] = std::max(1, occ);
  });

  int C;
  if (splits > 0) {
    C = splits;
  } else {
    // Fill the resident CTA slots, but with a power-of-two cluster of at most
    // 8: measured on B200, clusters of 6, 12 or 16 schedule badly (up to 1.7x
    // slower than 8 for the same shape).
    const int target = dev.sm_count * occ_cache[d];
    const int want = std::max(1, target / std::max(1, col_tiles));
    C = 1;
    while (C * 2 <= std::min(want, 8)) C *= 2;
  }
  // The CTA's whole activation slice is staged on chip: raise the split count
  // (a request, not a promise) until it fits the staging budget.
  const int max_rows = kStageBudget / (MT * 8 * esz);
  C = std::max(C, (krows + max_rows - 1) / max_rows);
  C = std::min(C, kMaxCluster);
  C = std::max(1, std::min(C, krows / kU));
  int rows_per_cta = (krows + C - 1) / C;
  rows_per_cta = (rows_per_cta + kU - 1) / kU * kU;
  C = (krows + rows_per_cta - 1) / rows_per_cta;  // trim empty slices
  if (static_cast<long long>(rows_per_cta) * MT * 8 * esz > kStageBudget) return NG_ERR_BAD_SHAPE;
  const size_t stage = static_cast<size_t>(MT) * rows_per_cta * 8 * esz;
  const size_t red = static_cast<size_t>(WARPS) * MT * kCols * 4;
  size_t smem = std::max(stage, red) + static_cast<size_t>(MT) * kCols * 4;
  if (na.mode == kStageAttn) {  // split weights of the heads a slice touches
    const int nh = (rows_per_cta * 8 + kAttnHeadDim - 1) / kAttnHeadDim + 1;
    smem = na_attw_offset(MT, rows_per_cta, esz, WARPS) + static_cast<size_t>(MT) * nh * (na.splits + 1) * 4;
    if (smem > 200 * 1024) return NG_ERR_BAD_SHAPE;
  }

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(col_tiles, C, 1);
  cfg.blockDim = dim3(threads, 1, 1);
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
  return launch_status(cudaLaunchKernelEx(&cfg, kern, x, qw, s, y, M, K, N, G, rows_per_cta, C, na));
}

template <bool XBF16, int PATH, int WARPS>
int dispatch_m(const void* x, const uint32_t* qw, const __half* s, void* y, int M, int K, int N,
               int G, int splits, const DeviceInfo& dev, cudaStream_t st, NormArgs na = {}) {
  if (M <= 1) return run<1, XBF16, PATH, WARPS>(x, qw, s, y, M, K, N, G, splits, dev, st, na);
  if (M <= 2) return run<2, XBF16, PATH, WARPS>(x, qw, s, y, M, K, N, G, splits, dev, st, na);
  if (M <= 4) return run<4, XBF16, PATH, WARPS>(x, qw, s, y, M, K, N, G, splits, dev, st, na);
  if (M <= 8) return run<8, XBF16, PATH, WARPS>(x, qw, s, y, M, K, N, G, splits, dev, st, na);
  return run<16, XBF16, PATH, WARPS>(x, qw, s, y, M, K, N, G, splits, dev, st, na);
}

template <bool XBF16, int PATH>
int dispatch_w(int threads, const void* x, const uint32_t* qw, const __half* s, void* y, int M,
               int K, int N, int G, int splits, const DeviceInfo& dev, cudaStream_t st) {
  if (threads == 128) return dispatch_m<XBF16, PATH, 4>(x, qw, s, y, M, K, N, G, splits, dev, st);
  return dispatch_m<XBF16, PATH, 8>(x, qw, s, y, M, K, N, G, splits, dev, st);
}

}  // namespace
}  // namespace ngb

extern "C" int ng_gemv_w4a16(const void* x, int x_dtype, const int32_t* qweight,
                             const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                             int splits, int block_threads, int algo, void* workspace,
                             size_t workspace_bytes, void* stream) {
  using namespace ngb;
  if (!x || !qweight || !scales || !y) return NG_ERR_NULL_POINTER;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 16 || K <= 0 || N <= 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (static_cast<long long>(K) * N >= (1LL << 40)) return NG_ERR_BAD_SHAPE;
  if (splits < 0 || splits > 16) return NG_ERR_BAD_ARGUMENT;
  if (block_threads != 0 && block_threads != 128 && block_threads != 256) return NG_ERR_BAD_ARGUMENT;
  if (algo < 0 || algo > 6) return NG_ERR_BAD_ARGUMENT;
  if (algo >= 4 && algo <= 5 && (M > (algo == 5 ? 16 : 8) || splits > 8)) return NG_ERR_BAD_ARGUMENT;
  if (x_dtype == NG_DTYPE_BF16 && algo == 1) return NG_ERR_BAD_ARGUMENT;
  if (!aligned(x, 16) || !aligned(qweight, 16) || !aligned(scales, 8) || !aligned(y, 2) ||
      !aligned(workspace, 256))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  const auto* q = reinterpret_cast<const uint32_t*>(qweight);
  const auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  const bool tensor_path = algo == 3;
  if (tensor_path) {
    if (workspace == nullptr) {
      if (algo == 3) return NG_ERR_NULL_POINTER;
    } else {
      if (workspace_bytes < gemv_tc_workspace_bytes(N, dev)) return NG_ERR_BAD_ARGUMENT;
      return gemv_tc(x, x_dtype, q, s, y, M, K, N, group_size, workspace, dev, strm);
    }
  }
  // Default schedule (measured on B200, M <= 8, no cluster-kernel options):
  //   * 96 column tiles (N >= 12288) up to one per SM, M <= 8 and M >= 2 or
  //     K <= 4096: the ring with one CTA per tile (its CTAs sweep the rows in
  //     lockstep);
  //   * more column tiles than SMs, M <= 8: the ring with its own K split;
  //   * M = 3..4 and a packed weight >= 12 MiB: the stream-K ring (all SMs);
  //   * M > 4 (up to 16): the ring with its own K split;
  //   * otherwise the cluster kernel.
  if (algo == 0 && block_threads == 0 && splits <= 8) {
    const int tiles = (N + 127) / 128;
    const double wbytes = static_cast<double>(K) * N / 2.0;
    if (tiles >= 96 && tiles <= dev.sm_count && M <= 8 && (M > 1 || K <= 4096)) {
      // One K slice per tile: the grid leaves SMs free, where the next kernel's
      // CTAs start streaming early (measured: faster in a chain than the
      // all-SM head/tail plan, 9.3 vs 16.2 us at config 1).
      algo = 5;
      if (splits == 0) splits = 1;
    } else if (tiles > dev.sm_count && M <= 8) {
      // More tiles than SMs: one slice per tile runs in two unbalanced waves
      // (measured K=4096 N=57344 M=1: 55.8 us vs 29.5 us with the ring's own
      // K split; M=8 is equal either way).
      algo = 5;
    } else if (M > 4 || (M >= 3 && wbytes >= 12.0 * (1 << 20))) {  // includes M = 9..16
      algo = 5;
    }
  }
  if (algo == 6) {
    if (gemv_stream_supported(N, s))
      return gemv_stream(x, x_dtype, q, s, y, M, K, N, group_size, splits, dev, strm);
    algo = 5;  // scales without a 16-byte row stride: the ring streams them itself
    if (splits > 8) splits = 8;
  }
  if (algo >= 4)
    return gemv_ring(x, x_dtype, algo == 5, q, s, y, M, K, N, group_size, splits, workspace,
                     workspace_bytes, dev, strm);
  const int threads = block_threads ? block_threads : 256;
  if (x_dtype == NG_DTYPE_BF16)
    return dispatch_w<true, kFloat2>(threads, x, q, s, y, M, K, N, group_size, splits, dev, strm);
  if (algo == 2)
    return dispatch_w<false, kFloat2>(threads, x, q, s, y, M, K, N, group_size, splits, dev, strm);
  return dispatch_w<false, kHalf2>(threads, x, q, s, y, M, K, N, group_size, splits, dev, strm);
}

extern "C" size_t ng_gemv_workspace_bytes(int M, int N) {
  ngb::DeviceInfo dev;
  if (M < 1 || M > 16 || N <= 0 || ngb::current_device_info(&dev) != NG_OK) return 0;
  return ngb::gemv_ring_workspace_bytes(N, dev);
}

extern "C" int ng_gemv_w4a16_rmsnorm(const void* x, const void* residual_in, void* residual_out,
                                     const void* norm_weight, float eps, int x_dtype,
                                     const int32_t* qweight, const uint16_t* scales, void* y, int M,
                                     int K, int N, int group_size, void* stream) {
  using namespace ngb;
  if (!x || !residual_in || !norm_weight || !qweight || !scales || !y) return NG_ERR_NULL_POINTER;
  if (residual_out == residual_in) return NG_ERR_BAD_ARGUMENT;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 16 || K <= 0 || K % 8 != 0 || N <= 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (!aligned(x, 16) || !aligned(residual_in, 16) || !aligned(norm_weight, 16) ||
      (residual_out && !aligned(residual_out, 16)) || !aligned(qweight, 16) || !aligned(scales, 8) ||
      !aligned(y, 2))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  NormArgs na;
  na.res_in = static_cast<const unsigned short*>(residual_in);
  na.res_out = static_cast<unsigned short*>(residual_out);
  na.w = static_cast<const unsigned short*>(norm_weight);
  na.eps = eps;
  na.mode = kStageNorm;
  const auto* q = reinterpret_cast<const uint32_t*>(qweight);
  const auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  if (x_dtype == NG_DTYPE_BF16)
    return dispatch_m<true, kFloat2, 8>(x, q, s, y, M, K, N, group_size, 0, dev, strm, na);
  return dispatch_m<false, kHalf2, 8>(x, q, s, y, M, K, N, group_size, 0, dev, strm, na);
}

extern "C" int ng_gemv_w4a16_silu(const void* gate_up, int x_dtype, const int32_t* qweight,
                                  const uint16_t* scales, void* y, int M, int K, int N,
                                  int group_size, void* stream) {
  using namespace ngb;
  if (!gate_up || !qweight || !scales || !y) return NG_ERR_NULL_POINTER;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 16 || K <= 0 || K % 8 != 0 || N <= 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (!aligned(gate_up, 16) || !aligned(qweight, 16) || !aligned(scales, 8) || !aligned(y, 2))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  NormArgs na;
  na.mode = kStageSilu;
  const auto* q = reinterpret_cast<const uint32_t*>(qweight);
  const auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  if (x_dtype == NG_DTYPE_BF16)
    return dispatch_m<true, kFloat2, 8>(gate_up, q, s, y, M, K, N, group_size, 0, dev, strm, na);
  return dispatch_m<false, kHalf2, 8>(gate_up, q, s, y, M, K, N, group_size, 0, dev, strm, na);
}

extern "C" int ng_gemv_w4a16_attn(const float* partials, int splits, int x_dtype,
                                  const int32_t* qweight, const uint16_t* scales, void* y, int M,
                                  int K, int N, int group_size, void* stream) {
  using namespace ngb;
  if (!partials || !qweight || !scales || !y) return NG_ERR_NULL_POINTER;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 16 || K <= 0 || K % kAttnHeadDim != 0 || N <= 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (splits < 1 || splits > 256) return NG_ERR_BAD_ARGUMENT;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (!aligned(partials, 16) || !aligned(qweight, 16) || !aligned(scales, 8) || !aligned(y, 2))
    return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  NormArgs na;
  na.mode = kStageAttn;
  na.part = partials;
  na.splits = splits;
  const auto* q = reinterpret_cast<const uint32_t*>(qweight);
  const auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  if (x_dtype == NG_DTYPE_BF16)
    return dispatch_m<true, kFloat2, 8>(partials, q, s, y, M, K, N, group_size, 0, dev, strm, na);
  return dispatch_m<false, kHalf2, 8>(partials, q, s, y, M, K, N, group_size, 0, dev, strm, na);
}

extern "C" size_t ng_gemv_allreduce_buffer_bytes(int world, int N) {
  if (world < 2 || world > ngb::kArMaxWorld || N <= 0) return 0;
  return ngb::ArLayout(world, (N + ngb::kCols - 1) / ngb::kCols).total;
}

extern "C" int ng_gemv_w4a16_allreduce(const void* x, int x_dtype, const int32_t* qweight,
                                       const uint16_t* scales, void* y, int M, int K, int N, int group_size,
                                       int stage_mode, void* const* peer_buffers, int rank, int world,
                                       void* stream) {
  using namespace ngb;
  if (!x || !qweight || !scales || !y || !peer_buffers) return NG_ERR_NULL_POINTER;
  if (x_dtype != NG_DTYPE_F16 && x_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 16 || K <= 0 || K % 8 != 0 || N <= 0 || N % 4 != 0) return NG_ERR_BAD_SHAPE;
  if (group_size != 64 && group_size != 128 && group_size != 256) return NG_ERR_BAD_SHAPE;
  if (K % group_size != 0) return NG_ERR_BAD_SHAPE;
  if (world < 2 || world > kArMaxWorld || rank < 0 || rank >= world) return NG_ERR_BAD_ARGUMENT;
  if (stage_mode != kStagePlain && stage_mode != kStageSilu) return NG_ERR_BAD_ARGUMENT;
  if (!aligned(x, 16) || !aligned(qweight, 16) || !aligned(scales, 8) || !aligned(y, 2))
    return NG_ERR_MISALIGNED;
  for (int p = 0; p < world; ++p)
    if (!peer_buffers[p] || !aligned(peer_buffers[p], 16)) return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  NormArgs na;
  na.mode = stage_mode;
  for (int p = 0; p < world; ++p) na.peers[p] = static_cast<unsigned char*>(peer_buffers[p]);
  na.ar_rank = rank;
  na.ar_world = world;
  na.ar_err = dev.err;
  const auto* q = reinterpret_cast<const uint32_t*>(qweight);
  const auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  if (x_dtype == NG_DTYPE_BF16)
    return dispatch_m<true, kFloat2, 8>(x, q, s, y, M, K, N, group_size, 0, dev, strm, na);
  return dispatch_m<false, kHalf2, 8>(x, q, s, y, M, K, N, group_size, 0, dev, strm, na);
}
