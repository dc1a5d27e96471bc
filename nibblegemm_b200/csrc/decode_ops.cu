// Non-GEMM kernels of a Llama-style decode step (batch M <= 16 tokens, one
// position each): fused residual + RMSNorm, RoPE + KV-cache append, GQA
// decode attention (split over the context, then combined), SwiGLU.  All are
// HBM- or latency-bound elementwise / reduction kernels; activations are
// fp16 or bf16 with fp32 arithmetic.  Each entry point validates its
// arguments, enqueues on the caller's stream and returns an NG_* status.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "ng_common.cuh"

namespace ngb {
namespace {

template <bool BF16>
__device__ __forceinline__ float ld_act(const void* p, size_t i) {
  const unsigned short v = static_cast<const unsigned short*>(p)[i];
  return BF16 ? __uint_as_float(static_cast<uint32_t>(v) << 16) : __half2float(__ushort_as_half(v));
}
// Four consecutive activations (8 bytes, 8-byte aligned) as fp32.
template <bool BF16>
__device__ __forceinline__ void ld_act4(const void* p, size_t i, float (&f)[4]) {
  const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const unsigned short*>(p) + i);
  const uint32_t w[2] = {v.x, v.y};
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if constexpr (BF16) {
      f[2 * j] = __uint_as_float(w[j] << 16);
      f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    } else {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&w[j]));
      f[2 * j] = t.x;
      f[2 * j + 1] = t.y;
    }
  }
}
template <bool BF16>
__device__ __forceinline__ void st_act(void* p, size_t i, float v) {
  static_cast<unsigned short*>(p)[i] =
      BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v)) : __half_as_ushort(__float2half_rn(v));
}

// Programmatic dependent launch: let the next kernel on the stream launch
// now (a following GEMV starts streaming its weights), then wait for the
// producer of this kernel's inputs.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += red[i];  // fixed order: deterministic
  return t;
}

// h = x + residual (if residual != null; h is written back to residual),
// y = h * rsqrt(mean(h^2) + eps) * w.  One CTA per token.
constexpr int kNormThreads = 512;
constexpr int kNormMaxPer = 16;  // H <= 8192 elements per token held in registers

template <bool BF16>
__global__ void __launch_bounds__(kNormThreads)
    rmsnorm_kernel(const void* __restrict__ x, void* __restrict__ residual,
                   const void* __restrict__ w, void* __restrict__ y, int H, float eps) {
  pdl_enter();
  __shared__ float red[32];
  const size_t base = static_cast<size_t>(blockIdx.x) * H;
  float h[kNormMaxPer];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormMaxPer; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    h[j] = 0.f;
    if (i < H) {
      h[j] = ld_act<BF16>(x, base + i);
      if (residual) h[j] += ld_act<BF16>(residual, base + i);
      ss += h[j] * h[j];
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / static_cast<float>(H) + eps);
#pragma unroll
  for (int j = 0; j < kNormMaxPer; ++j) {
    const int i = threadIdx.x + j * kNormThreads;
    if (i < H) {
      if (residual) st_act<BF16>(residual, base + i, h[j]);
      st_act<BF16>(y, base + i, h[j] * inv * ld_act<BF16>(w, i));
    }
  }
}

// qkv[M, (Hq + 2 Hkv) * D] -> q[M, Hq, D] with RoPE, and K / V rows of every
// token appended at its position in its own sequence's cache: cache[m, pos, Hkv, D].  Rotary pairs (i,
// i + D/2) ("rotate half"), angle pos * theta^(-2i/D) computed in fp32.
template <bool BF16>
__global__ void rope_append_kernel(const void* __restrict__ qkv, void* __restrict__ q_out,
                                   void* __restrict__ k_cache, void* __restrict__ v_cache,
                                   const int* __restrict__ pos, int Hq, int Hkv, int D, float theta,
                                   int max_ctx, int T) {
  pdl_enter();
  // Token m is number s = m % T of sequence seq = m / T, at position pos[seq] + s
  // (decode: T = 1, one token per sequence; prefill: T tokens per sequence).
  const int m = blockIdx.y, head = blockIdx.x;  // head in [0, Hq + Hkv): q heads then k heads
  const int seq = m / T;
  const int p = pos[seq] + (m - seq * T);
  const bool in_cache = p >= 0 && p < max_ctx;  // cache rows outside [0, max_ctx) are never written
  if (head >= Hq && !in_cache) return;
  const int row = (Hq + 2 * Hkv) * D;
  const size_t src = static_cast<size_t>(m) * row + static_cast<size_t>(head) * D;
  const int half = D / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float inv_freq = exp2f(-2.f * i / D * log2f(theta));
    float sn, cs;
    sincosf(static_cast<float>(p) * inv_freq, &sn, &cs);
    const float a = ld_act<BF16>(qkv, src + i), b = ld_act<BF16>(qkv, src + i + half);
    const float ra = a * cs - b * sn, rb = b * cs + a * sn;
    if (head < Hq) {
      const size_t dst = (static_cast<size_t>(m) * Hq + head) * D;
      st_act<BF16>(q_out, dst + i, ra);
      st_act<BF16>(q_out, dst + i + half, rb);
    } else {
      const int kh = head - Hq;
      const size_t dst = ((static_cast<size_t>(seq) * max_ctx + p) * Hkv + kh) * D;
      st_act<BF16>(k_cache, dst + i, ra);
      st_act<BF16>(k_cache, dst + i + half, rb);
    }
  }
  if (head >= Hq) {  // V rows: copied unrotated
    const int kh = head - Hq;
    const size_t vsrc = static_cast<size_t>(m) * row + static_cast<size_t>(Hq + Hkv + kh) * D;
    const size_t dst = ((static_cast<size_t>(seq) * max_ctx + p) * Hkv + kh) * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x)
      static_cast<unsigned short*>(v_cache)[dst + i] = static_cast<const unsigned short*>(qkv)[vsrc + i];
  }
}

// The same operation with one CTA per token, for D % 8 == 0 and D <= 256 (the
// prefill case: thousands of tokens).  The D/2 angles' sines and cosines are
// computed once per token into shared memory and shared by all of its heads;
// each thread then rotates 4 consecutive pairs of one head with 8-byte loads
// and stores, and the V rows are copied 16 bytes at a time.
template <bool BF16>
__device__ __forceinline__ void st_act4(void* p, size_t i, const float (&f)[4]) {
  uint32_t w[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    if constexpr (BF16) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    } else {
      const __half2 h = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<const uint32_t*>(&h);
    }
  }
  *reinterpret_cast<uint2*>(static_cast<unsigned short*>(p) + i) = make_uint2(w[0], w[1]);
}

constexpr int kRopeTokThreads = 256;

template <bool BF16>
__global__ void __launch_bounds__(kRopeTokThreads)
    rope_append_tok_kernel(const void* __restrict__ qkv, void* __restrict__ q_out,
                           void* __restrict__ k_cache, void* __restrict__ v_cache,
                           const int* __restrict__ pos, int Hq, int Hkv, int D, float theta,
                           int max_ctx, int T) {
  __shared__ float cs[128], sn[128];
  pdl_enter();
  const int m = blockIdx.x;
  const int seq = m / T;
  const int p = pos[seq] + (m - seq * T);
  const bool in_cache = p >= 0 && p < max_ctx;  // cache rows outside [0, max_ctx) are never written
  const int half = D / 2;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float inv_freq = exp2f(-2.f * i / D * log2f(theta));
    sincosf(static_cast<float>(p) * inv_freq, &sn[i], &cs[i]);
  }
  __syncthreads();
  const int row = (Hq + 2 * Hkv) * D;
  const int q4 = half / 4;                       // 4-pair chunks per head
  const int heads = in_cache ? Hq + Hkv : Hq;    // K heads only when the row is stored
  for (int it = threadIdx.x; it < heads * q4; it += blockDim.x) {
    const int head = it / q4, i = (it - head * q4) * 4;
    const size_t src = static_cast<size_t>(m) * row + static_cast<size_t>(head) * D;
    float a[4], b[4], ra[4], rb[4];
    ld_act4<BF16>(qkv, src + i, a);
    ld_act4<BF16>(qkv, src + i + half, b);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ra[j] = a[j] * cs[i + j] - b[j] * sn[i + j];
      rb[j] = b[j] * cs[i + j] + a[j] * sn[i + j];
    }
    size_t dst;
    void* base;
    if (head < Hq) {
      dst = (static_cast<size_t>(m) * Hq + head) * D;
      base = q_out;
    } else {
      dst = ((static_cast<size_t>(seq) * max_ctx + p) * Hkv + (head - Hq)) * D;
      base = k_cache;
    }
    st_act4<BF16>(base, dst + i, ra);
    st_act4<BF16>(base, dst + i + half, rb);
  }
  if (!in_cache) return;
  const int c8 = D / 8;  // V rows: copied unrotated, 16 bytes at a time
  for (int it = threadIdx.x; it < Hkv * c8; it += blockDim.x) {
    const int kh = it / c8, c = it - kh * c8;
    const size_t vsrc = static_cast<size_t>(m) * row + static_cast<size_t>(Hq + Hkv + kh) * D + 8 * c;
    const size_t dst = ((static_cast<size_t>(seq) * max_ctx + p) * Hkv + kh) * D + 8 * c;
    *reinterpret_cast<uint4*>(static_cast<unsigned short*>(v_cache) + dst) =
        *reinterpret_cast<const uint4*>(static_cast<const unsigned short*>(qkv) + vsrc);
  }
}

// Split-context GQA decode attention, D = 128.  Grid (Hkv, splits, M): a CTA
// owns one KV head, one contiguous chunk of the context and one token; its
// G = Hq / Hkv warps are the query heads sharing that KV head (lane l holds
// dims 4l..4l+3).  Online softmax in fp32; partial (max, sum, acc[D]) per
// (token, q head, split) go to the workspace for the combine kernel.
constexpr int kAttnD = 128;
template <bool BF16>
__global__ void attn_partial_kernel(const void* __restrict__ q, const void* __restrict__ k_cache,
                                    const void* __restrict__ v_cache, const int* __restrict__ ctx,
                                    float* __restrict__ part, int Hq, int Hkv, int chunk,
                                    int splits, float scale, int max_ctx) {
  pdl_enter();
  const int kh = blockIdx.x, sp = blockIdx.y, m = blockIdx.z;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = kh * G + warp;
  const int len = min(ctx[m], max_ctx);  // never read past the cache
  const int t0 = sp * chunk, t1 = min(len, t0 + chunk);
  float qv[4];
  const size_t qb = (static_cast<size_t>(m) * Hq + qh) * kAttnD + lane * 4;
#pragma unroll
  for (int j = 0; j < 4; ++j) qv[j] = ld_act<BF16>(q, qb + j) * scale;
  float mx = -INFINITY, sum = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  constexpr int kB = 8;  // positions whose K / V rows are loaded together
  for (int tb = t0; tb < t1; tb += kB) {
    float kv[kB][4], vv[kB][4], sc[kB];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      if (tb + u < t1) {
        const size_t kb = ((static_cast<size_t>(m) * max_ctx + tb + u) * Hkv + kh) * kAttnD + lane * 4;
        ld_act4<BF16>(k_cache, kb, kv[u]);
        ld_act4<BF16>(v_cache, kb, vv[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      sc[u] = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) sc[u] += qv[j] * kv[u][j];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < kB; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      if (tb + u >= t1) break;
      const float nm = fmaxf(mx, sc[u]);
      const float corr = __expf(mx - nm), pw = __expf(sc[u] - nm);
      sum = sum * corr + pw;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = acc[j] * corr + pw * vv[u][j];
      mx = nm;
    }
  }
  // part layout: [M][Hq][splits][2 + D]
  float* o = part + ((static_cast<size_t>(m) * Hq + qh) * splits + sp) * (2 + kAttnD);
  if (lane == 0) {
    o[0] = mx;
    o[1] = sum;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) o[2 + lane * 4 + j] = acc[j];
}

// attn_partial_kernel with RoPE and the KV append folded in: q is read from
// qkv [M, (Hq + 2 Hkv) * D] and rotated in registers (the rotation partner of
// lane l's dims 4l..4l+3 is lane l ^ 16); the CTA whose chunk holds the new
// position rotates K, writes K and V there, and only then reads the chunk.
// The context is pos[m] + 1 positions, clamped to the cache.
template <bool BF16, int GQ>
__global__ void __launch_bounds__(GQ * 32)
    attn_rope_partial_kernel(const void* __restrict__ qkv, void* __restrict__ k_cache,
                                         void* __restrict__ v_cache, const int* __restrict__ pos,
                                         float* __restrict__ part, int Hq, int Hkv, int chunk,
                                         int splits, float scale, int max_ctx, float theta) {
  pdl_enter();
  const int kh = blockIdx.x, sp = blockIdx.y, m = blockIdx.z;
  constexpr int G = GQ;  // query heads per KV head (compile time)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qh = kh * G + warp;
  const int p = pos[m];
  const int len = min(p + 1, max_ctx);
  const int t0 = sp * chunk, t1 = min(len, t0 + chunk);
  const size_t row = static_cast<size_t>(Hq + 2 * Hkv) * kAttnD;
  // rotation of the 4 dims this lane holds: dims d = 4 lane + j pair with d +- 64
  const bool lo = lane < 16;
  float cs[4], sn[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = (lo ? 4 * lane : 4 * lane - kAttnD / 2) + j;  // frequency index 0..63
    const float inv_freq = exp2f(-2.f * i / kAttnD * log2f(theta));
    sincosf(static_cast<float>(p) * inv_freq, &sn[j], &cs[j]);
  }
  auto rotate = [&](float (&v)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[j], 16);
      v[j] = lo ? v[j] * cs[j] - partner * sn[j] : v[j] * cs[j] + partner * sn[j];
    }
  };
  float qv[4];
  ld_act4<BF16>(qkv, static_cast<size_t>(m) * row + static_cast<size_t>(qh) * kAttnD + lane * 4, qv);
  rotate(qv);
#pragma unroll
  for (int j = 0; j < 4; ++j) qv[j] *= scale;
  if (p >= 0 && p < max_ctx && p >= t0 && p < t1) {  // this chunk holds the new row: append it
    if (warp == 0) {
      float kn[4], vn[4];
      ld_act4<BF16>(qkv, static_cast<size_t>(m) * row + static_cast<size_t>(Hq + kh) * kAttnD + lane * 4, kn);
      ld_act4<BF16>(qkv, static_cast<size_t>(m) * row + static_cast<size_t>(Hq + Hkv + kh) * kAttnD + lane * 4, vn);
      rotate(kn);
      const size_t dst = ((static_cast<size_t>(m) * max_ctx + p) * Hkv + kh) * kAttnD + lane * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        st_act<BF16>(k_cache, dst + j, kn[j]);
        st_act<BF16>(v_cache, dst + j, vn[j]);
      }
    }
    __syncthreads();
  }
  // Warps take interleaved positions; each K / V row is loaded once and used
  // for all G query heads of this KV head (q of every head held by each warp).
  constexpr int kMaxG = GQ;
  float qa[kMaxG][4];
  // share the rotated, scaled q of every head through shared memory
  __shared__ float qs[kMaxG][kAttnD];
#pragma unroll
  for (int j = 0; j < 4; ++j) qs[warp][lane * 4 + j] = qv[j];
  __syncthreads();
#pragma unroll
  for (int h = 0; h < kMaxG; ++h)
#pragma unroll
    for (int j = 0; j < 4; ++j) qa[h][j] = h < G ? qs[h][lane * 4 + j] : 0.f;
  float mx[kMaxG], sum[kMaxG], acc[kMaxG][4];
#pragma unroll
  for (int h = 0; h < kMaxG; ++h) {
    mx[h] = -INFINITY;
    sum[h] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[h][j] = 0.f;
  }
  const int nw = blockDim.x >> 5;
  constexpr int kB = 4;  // positions per warp loaded together
  for (int tb = t0 + warp; tb < t1; tb += kB * nw) {
    float kv[kB][4], vv[kB][4];
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      const int t = tb + u * nw;
      if (t < t1) {
        const size_t kb = ((static_cast<size_t>(m) * max_ctx + t) * Hkv + kh) * kAttnD + lane * 4;
        ld_act4<BF16>(k_cache, kb, kv[u]);
        ld_act4<BF16>(v_cache, kb, vv[u]);
      }
    }
    float sc[kB][kMaxG];
#pragma unroll
    for (int u = 0; u < kB; ++u)
#pragma unroll
      for (int h = 0; h < kMaxG; ++h) {
        sc[u][h] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) sc[u][h] += qa[h][j] * kv[u][j];
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < kB; ++u)
#pragma unroll
        for (int h = 0; h < kMaxG; ++h)
          if (h < G) sc[u][h] += __shfl_xor_sync(0xffffffffu, sc[u][h], o);
#pragma unroll
    for (int u = 0; u < kB; ++u) {
      if (tb + u * nw >= t1) break;
#pragma unroll
      for (int h = 0; h < kMaxG; ++h) {
        if (h >= G) continue;
        const float nm = fmaxf(mx[h], sc[u][h]);
        const float corr = __expf(mx[h] - nm), pw = __expf(sc[u][h] - nm);
        sum[h] = sum[h] * corr + pw;
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[h][j] = acc[h][j] * corr + pw * vv[u][j];
        mx[h] = nm;
      }
    }
  }
  // merge the warps' states per head (fixed warp order) and write the partial
  __shared__ float ms_[kMaxG][kMaxG][2];          // [warp][head][max, sum]
  __shared__ float as_[kMaxG][kMaxG][kAttnD];     // [warp][head][dim]
#pragma unroll
  for (int h = 0; h < kMaxG; ++h) {
    if (h >= G) continue;
    if (lane == 0) {
      ms_[warp][h][0] = mx[h];
      ms_[warp][h][1] = sum[h];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) as_[warp][h][lane * 4 + j] = acc[h][j];
  }
  __syncthreads();
  {
    const int h = warp;  // warp h writes head h of this group
    float M_ = -INFINITY;
    for (int w2 = 0; w2 < nw; ++w2) M_ = fmaxf(M_, ms_[w2][h][0]);
    float S = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w2 = 0; w2 < nw; ++w2) {
      const float mw = ms_[w2][h][0];
      if (mw == -INFINITY) continue;
      const float f = __expf(mw - M_);
      S += f * ms_[w2][h][1];
#pragma unroll
      for (int j = 0; j < 4; ++j) A[j] += f * as_[w2][h][lane * 4 + j];
    }
    float* o = part + ((static_cast<size_t>(m) * Hq + kh * G + h) * splits + sp) * (2 + kAttnD);
    if (lane == 0) {
      o[0] = M_;
      o[1] = S;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) o[2 + lane * 4 + j] = A[j];
  }
}

// Combine the splits of one (token, q head) in split order: out[M, Hq, D].
template <bool BF16>
__global__ void attn_combine_kernel(const float* __restrict__ part, void* __restrict__ out,
                                    int Hq, int splits) {
  pdl_enter();
  const int qh = blockIdx.x, m = blockIdx.y, d = threadIdx.x;  // blockDim = D
  const float* p = part + (static_cast<size_t>(m) * Hq + qh) * splits * (2 + kAttnD);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, p[s * (2 + kAttnD)]);
  float den = 0.f, num = 0.f;
  for (int s = 0; s < splits; ++s) {
    const float ms = p[s * (2 + kAttnD)];
    if (ms == -INFINITY) continue;  // empty split
    const float w = __expf(ms - mx);
    den += w * p[s * (2 + kAttnD) + 1];
    num += w * p[s * (2 + kAttnD) + 2 + d];
  }
  st_act<BF16>(out, (static_cast<size_t>(m) * Hq + qh) * kAttnD + d, num / den);
}

// gate_up[M, 2I] (gate | up) -> out[M, I] = silu(gate) * up.
template <bool BF16>
__global__ void silu_mul_kernel(const void* __restrict__ gu, void* __restrict__ out, int M, int I) {
  pdl_enter();
  const size_t n = static_cast<size_t>(M) * I;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t m = i / I, j = i - m * I;
    const float g = ld_act<BF16>(gu, m * 2 * I + j), u = ld_act<BF16>(gu, m * 2 * I + I + j);
    st_act<BF16>(out, i, g / (1.f + __expf(-g)) * u);
  }
}

// Row-wise argmax of logits [M, V]: every block folds a strided slice of
// the row into one (value, index) key -- float bits mapped to an unsigned
// order, index complemented so the smallest index wins ties -- and takes
// atomicMax into best[m]; the order of the atomics cannot change the result.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  uint32_t b = __float_as_uint(v);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | static_cast<uint32_t>(~static_cast<uint32_t>(i));
}

template <bool BF16>
__global__ void argmax_partial_kernel(const void* __restrict__ logits, int V,
                                      unsigned long long* __restrict__ best) {
  pdl_enter();
  const int m = blockIdx.y;
  unsigned long long k = 0ull;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < V; i += gridDim.x * blockDim.x) {
    const unsigned long long c = argmax_key(ld_act<BF16>(logits, static_cast<size_t>(m) * V + i), i);
    k = c > k ? c : k;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long c = __shfl_xor_sync(0xffffffffu, k, o);
    k = c > k ? c : k;
  }
  if ((threadIdx.x & 31) == 0 && k) atomicMax(&best[m], k);
}

// best[m] -> (value, index + offset); best[m] re-armed to 0 for the next call.
__global__ void argmax_final_kernel(unsigned long long* __restrict__ best, float* __restrict__ value,
                                    long long* __restrict__ index, int M, long long offset) {
  pdl_enter();
  const int m = threadIdx.x;
  if (m >= M) return;
  const unsigned long long k = best[m];
  uint32_t b = static_cast<uint32_t>(k >> 32);
  b = (b & 0x80000000u) ? (b & 0x7FFFFFFFu) : ~b;
  value[m] = __uint_as_float(b);
  index[m] = static_cast<long long>(~static_cast<uint32_t>(k)) + offset;
  best[m] = 0ull;
}

bool dtype_ok(int d) { return d == NG_DTYPE_F16 || d == NG_DTYPE_BF16; }

// Launch with programmatic stream serialisation (see pdl_enter).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launch_status(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...));
}

}  // namespace
}  // namespace ngb

using namespace ngb;

extern "C" int ng_rmsnorm(const void* x, void* residual, const void* weight, void* y, int dtype,
                          int M, int H, float eps, void* stream) {
  if (!x || !weight || !y) return NG_ERR_NULL_POINTER;
  if (!dtype_ok(dtype)) return NG_ERR_BAD_DTYPE;
  if (M < 1 || H < 1 || H > kNormThreads * kNormMaxPer) return NG_ERR_BAD_SHAPE;
  auto st = static_cast<cudaStream_t>(stream);
  if (dtype == NG_DTYPE_BF16)
    return launch_pdl(rmsnorm_kernel<true>, dim3(M), dim3(kNormThreads), st, x, residual, weight, y, H, eps);
  else
    return launch_pdl(rmsnorm_kernel<false>, dim3(M), dim3(kNormThreads), st, x, residual, weight, y, H, eps);
}

namespace {
int rope_append_launch(const void* qkv, void* q_out, void* k_cache, void* v_cache, const int* pos,
                       int dtype, int M, int T, int Hq, int Hkv, int D, float theta, int max_ctx,
                       void* stream) {
  if (!qkv || !q_out || !k_cache || !v_cache || !pos) return NG_ERR_NULL_POINTER;
  if (!dtype_ok(dtype)) return NG_ERR_BAD_DTYPE;
  if (M < 1 || T < 1 || M % T || (T == 1 && M > 65535) || Hq < 1 || Hkv < 1 || D < 2 || D % 2 || Hq % Hkv ||
      max_ctx < 1)
    return NG_ERR_BAD_SHAPE;
  auto st = static_cast<cudaStream_t>(stream);
  const bool vec = D % 8 == 0 && D <= 256 && aligned(qkv, 16) && aligned(q_out, 8) &&
                   aligned(k_cache, 16) && aligned(v_cache, 16);
  if (vec && T > 1) {  // many tokens: one CTA per token
    if (dtype == NG_DTYPE_BF16)
      return launch_pdl(rope_append_tok_kernel<true>, dim3(M), dim3(kRopeTokThreads), st, qkv, q_out,
                        k_cache, v_cache, pos, Hq, Hkv, D, theta, max_ctx, T);
    return launch_pdl(rope_append_tok_kernel<false>, dim3(M), dim3(kRopeTokThreads), st, qkv, q_out,
                      k_cache, v_cache, pos, Hq, Hkv, D, theta, max_ctx, T);
  }
  if (M > 65535) return NG_ERR_BAD_SHAPE;  // the per-head grid's y extent
  const dim3 grid(Hq + Hkv, M);
  if (dtype == NG_DTYPE_BF16)
    return launch_pdl(rope_append_kernel<true>, dim3(grid), dim3(64), st, qkv, q_out, k_cache, v_cache,
                      pos, Hq, Hkv, D, theta, max_ctx, T);
  return launch_pdl(rope_append_kernel<false>, dim3(grid), dim3(64), st, qkv, q_out, k_cache, v_cache,
                    pos, Hq, Hkv, D, theta, max_ctx, T);
}
}  // namespace

extern "C" int ng_rope_append(const void* qkv, void* q_out, void* k_cache, void* v_cache,
                              const int* pos, int dtype, int M, int Hq, int Hkv, int D, float theta,
                              int max_ctx, void* stream) {
  return rope_append_launch(qkv, q_out, k_cache, v_cache, pos, dtype, M, 1, Hq, Hkv, D, theta, max_ctx,
                            stream);
}

extern "C" int ng_rope_prefill(const void* qkv, void* q_out, void* k_cache, void* v_cache,
                               const int* pos, int dtype, int B, int S, int Hq, int Hkv, int D,
                               float theta, int max_ctx, void* stream) {
  if (B < 1 || S < 1) return NG_ERR_BAD_SHAPE;
  return rope_append_launch(qkv, q_out, k_cache, v_cache, pos, dtype, B * S, S, Hq, Hkv, D, theta,
                            max_ctx, stream);
}

extern "C" size_t ng_attn_workspace_bytes(int M, int Hq, int splits) {
  return static_cast<size_t>(M) * Hq * splits * (2 + kAttnD) * sizeof(float);
}

extern "C" int ng_attn_decode(const void* q, const void* k_cache, const void* v_cache,
                              const int* ctx_len, void* out, int dtype, int M, int Hq, int Hkv,
                              int D, int max_ctx, int splits, float scale, void* workspace,
                              size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !ctx_len || !out || !workspace) return NG_ERR_NULL_POINTER;
  if (!dtype_ok(dtype)) return NG_ERR_BAD_DTYPE;
  if (D != kAttnD || M < 1 || Hkv < 1 || Hq % Hkv || Hq / Hkv > 32 || max_ctx < 1) return NG_ERR_BAD_SHAPE;
  if (splits < 1 || splits > 256) return NG_ERR_BAD_ARGUMENT;
  if (workspace_bytes < ng_attn_workspace_bytes(M, Hq, splits)) return NG_ERR_BAD_ARGUMENT;
  auto st = static_cast<cudaStream_t>(stream);
  const int chunk = (max_ctx + splits - 1) / splits;
  const dim3 g1(Hkv, splits, M), g2(Hq, M);
  const int threads = (Hq / Hkv) * 32;
  auto* part = static_cast<float*>(workspace);
  if (dtype == NG_DTYPE_BF16) {
    if (int e = launch_pdl(attn_partial_kernel<true>, g1, dim3(threads), st, q, k_cache, v_cache,
                           ctx_len, part, Hq, Hkv, chunk, splits, scale, max_ctx))
      return e;
    return launch_pdl(attn_combine_kernel<true>, g2, dim3(kAttnD), st, part, out, Hq, splits);
  }
  if (int e = launch_pdl(attn_partial_kernel<false>, g1, dim3(threads), st, q, k_cache, v_cache,
                         ctx_len, part, Hq, Hkv, chunk, splits, scale, max_ctx))
    return e;
  return launch_pdl(attn_combine_kernel<false>, g2, dim3(kAttnD), st, part, out, Hq, splits);
}

extern "C" int ng_silu_mul(const void* gate_up, void* out, int dtype, int M, int I, void* stream) {
  if (!gate_up || !out) return NG_ERR_NULL_POINTER;
  if (!dtype_ok(dtype)) return NG_ERR_BAD_DTYPE;
  if (M < 1 || I < 1) return NG_ERR_BAD_SHAPE;
  auto st = static_cast<cudaStream_t>(stream);
  const size_t n = static_cast<size_t>(M) * I;
  const int blocks = static_cast<int>(std::min<size_t>((n + 255) / 256, 148 * 8));
  if (dtype == NG_DTYPE_BF16)
    return launch_pdl(silu_mul_kernel<true>, dim3(blocks), dim3(256), st, gate_up, out, M, I);
  else
    return launch_pdl(silu_mul_kernel<false>, dim3(blocks), dim3(256), st, gate_up, out, M, I);
  return launch_status();
}

extern "C" int ng_argmax(const void* logits, int dtype, int M, int V, long long index_offset,
                         void* best_scratch, float* value, long long* index, void* stream) {
  if (!logits || !best_scratch || !value || !index) return NG_ERR_NULL_POINTER;
  if (!dtype_ok(dtype)) return NG_ERR_BAD_DTYPE;
  if (M < 1 || M > 1024 || V < 1) return NG_ERR_BAD_SHAPE;
  auto st = static_cast<cudaStream_t>(stream);
  auto* best = static_cast<unsigned long long*>(best_scratch);
  const int blocks = std::max(1, std::min(148, (V + 255) / 256));
  const dim3 grid(blocks, M);
  int e = dtype == NG_DTYPE_BF16 ? launch_pdl(argmax_partial_kernel<true>, grid, dim3(256), st, logits, V, best)
                                 : launch_pdl(argmax_partial_kernel<false>, grid, dim3(256), st, logits, V, best);
  if (e) return e;
  return launch_pdl(argmax_final_kernel, dim3(1), dim3(std::max(32, (M + 31) / 32 * 32)), st, best, value,
                    index, M, index_offset);
}

extern "C" int ng_attn_decode_rope(const void* qkv, void* k_cache, void* v_cache, const int* pos,
                                   void* out, int dtype, int M, int Hq, int Hkv, int D, int max_ctx,
                                   int splits, float scale, float theta, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  if (!qkv || !k_cache || !v_cache || !pos || !workspace) return NG_ERR_NULL_POINTER;
  if (!dtype_ok(dtype)) return NG_ERR_BAD_DTYPE;
  if (D != kAttnD || M < 1 || Hkv < 1 || Hq % Hkv || max_ctx < 1) return NG_ERR_BAD_SHAPE;
  if (Hq / Hkv != 1 && Hq / Hkv != 2 && Hq / Hkv != 4 && Hq / Hkv != 8) return NG_ERR_BAD_SHAPE;
  if (splits < 1 || splits > 256) return NG_ERR_BAD_ARGUMENT;
  if (workspace_bytes < ng_attn_workspace_bytes(M, Hq, splits)) return NG_ERR_BAD_ARGUMENT;
  if (out != nullptr && !aligned(out, 2)) return NG_ERR_MISALIGNED;
  auto st = static_cast<cudaStream_t>(stream);
  const int chunk = (max_ctx + splits - 1) / splits;
  const dim3 g1(Hkv, splits, M), g2(Hq, M);
  auto* part = static_cast<float*>(workspace);
  const int G = Hq / Hkv;
  auto partial = [&](auto bf, auto gq) -> int {
    constexpr bool B = decltype(bf)::value;
    constexpr int GQ = decltype(gq)::value;
    return launch_pdl(attn_rope_partial_kernel<B, GQ>, g1, dim3(GQ * 32), st, qkv, k_cache, v_cache,
                      pos, part, Hq, Hkv, chunk, splits, scale, max_ctx, theta);
  };
  auto by_g = [&](auto bf) -> int {
    switch (G) {
      case 1: return partial(bf, std::integral_constant<int, 1>{});
      case 2: return partial(bf, std::integral_constant<int, 2>{});
      case 4: return partial(bf, std::integral_constant<int, 4>{});
      default: return partial(bf, std::integral_constant<int, 8>{});
    }
  };
  // out == NULL: partials only (a consumer such as ng_gemv_w4a16_attn combines them)
  if (dtype == NG_DTYPE_BF16) {
    if (int e = by_g(std::true_type{})) return e;
    if (out == nullptr) return NG_OK;
    return launch_pdl(attn_combine_kernel<true>, g2, dim3(kAttnD), st, part, out, Hq, splits);
  }
  if (int e = by_g(std::false_type{})) return e;
  if (out == nullptr) return NG_OK;
  return launch_pdl(attn_combine_kernel<false>, g2, dim3(kAttnD), st, part, out, Hq, splits);
}
