// Dense dequantisation: out[K, N] = round((u - 8) * scale) in fp16 or bf16.
//
// Write-bound (four output bytes per input byte).  Each thread owns one packed
// row-word position and VEC adjacent columns: one 16-byte load (VEC = 4) of
// codes, one 8-byte load of scales, eight 8-byte stores -- a warp writes 256
// contiguous bytes per output row.  VEC = 1 covers N % 4 != 0.
#include "ng_decode.cuh"

namespace ngb {
namespace {

template <int VEC, bool FAST, bool BF16>
__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ qw,
                                                     const __half* __restrict__ scales,
                                                     void* __restrict__ out, int K, int N,
                                                     int group_size) {
  const int ncol = (N + VEC - 1) / VEC;
  const long long total = static_cast<long long>(K / 8) * ncol;
  for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int row = static_cast<int>(idx / ncol);  // packed row = k / 8
    const int col = static_cast<int>(idx % ncol) * VEC;
    const int grp = (row * 8) / group_size;
    uint32_t q[VEC];
    __half s[VEC];
    if constexpr (VEC == 4) {
      const uint4 v = *reinterpret_cast<const uint4*>(qw + static_cast<size_t>(row) * N + col);
      q[0] = v.x; q[1] = v.y; q[2] = v.z; q[3] = v.w;
      const uint2 sv = *reinterpret_cast<const uint2*>(scales + static_cast<size_t>(grp) * N + col);
      s[0] = __ushort_as_half(static_cast<unsigned short>(sv.x & 0xFFFF));
      s[1] = __ushort_as_half(static_cast<unsigned short>(sv.x >> 16));
      s[2] = __ushort_as_half(static_cast<unsigned short>(sv.y & 0xFFFF));
      s[3] = __ushort_as_half(static_cast<unsigned short>(sv.y >> 16));
    } else {
      q[0] = qw[static_cast<size_t>(row) * N + col];
      s[0] = scales[static_cast<size_t>(grp) * N + col];
    }
    unsigned short vals[8][VEC];  // raw 16-bit patterns, [k][column]
#pragma unroll
    for (int c = 0; c < VEC; ++c) {
      if constexpr (FAST && !BF16) {
        __half2 w[4];
        decode8_f16(q[c], w);
        const __half2 s2 = __half2half2(s[c]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t b = h2_bits(__hmul2(w[i], s2));  // one rounding of an exact product
          vals[2 * i][c] = static_cast<unsigned short>(b & 0xFFFF);
          vals[2 * i + 1][c] = static_cast<unsigned short>(b >> 16);
        }
      } else if constexpr (FAST && BF16) {
        const uint32_t q16 = q[c] >> 16;
        const float sf = __half2float(s[c]);
        const f2 s2 = f2_make(sf, sf);
        const f2 p[4] = {decode_pair_f32<0>(q[c], q16), decode_pair_f32<1>(q[c], q16),
                         decode_pair_f32<2>(q[c], q16), decode_pair_f32<3>(q[c], q16)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float lo, hi;
          f2_split(f2_mul(p[j], s2), lo, hi);
          vals[2 * j][c] = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
          vals[2 * j + 1][c] = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
        }
      } else {
        const float sf = __half2float(s[c]);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float v = static_cast<float>(code_minus8(q[c], k)) * sf;
          vals[k][c] = BF16 ? __bfloat16_as_ushort(__float2bfloat16_rn(v))
                            : __half_as_ushort(__float2half_rn(v));
        }
      }
    }
    unsigned short* o = static_cast<unsigned short*>(out);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      unsigned short* dst = o + static_cast<size_t>(row * 8 + k) * N + col;
      if constexpr (VEC == 4) {
        uint2 v;
        v.x = static_cast<uint32_t>(vals[k][0]) | (static_cast<uint32_t>(vals[k][1]) << 16);
        v.y = static_cast<uint32_t>(vals[k][2]) | (static_cast<uint32_t>(vals[k][3]) << 16);
        *reinterpret_cast<uint2*>(dst) = v;
      } else {
        *dst = vals[k][0];
      }
    }
  }
}

template <int VEC, bool FAST, bool BF16>
int launch_dequant(const uint32_t* qw, const __half* s, void* out, int K, int N, int G,
                   const DeviceInfo& dev, cudaStream_t stream) {
  const long long total = static_cast<long long>(K / 8) * ((N + VEC - 1) / VEC);
  const int threads = 256;
  long long blocks = (total + threads - 1) / threads;
  const long long cap = static_cast<long long>(dev.sm_count) * 8 * 4;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  dequant_kernel<VEC, FAST, BF16>
      <<<static_cast<unsigned>(blocks), threads, 0, stream>>>(qw, s, out, K, N, G);
  return launch_status();
}

}  // namespace
}  // namespace ngb

extern "C" int ng_dequant_w4(const int32_t* qweight, const uint16_t* scales, void* out,
                             int out_dtype, int K, int N, int group_size, int fast, void* stream) {
  using namespace ngb;
  if (!qweight || !scales || !out) return NG_ERR_NULL_POINTER;
  if (out_dtype != NG_DTYPE_F16 && out_dtype != NG_DTYPE_BF16) return NG_ERR_BAD_DTYPE;
  if (K <= 0 || N <= 0 || K % 8 != 0 || group_size <= 0 || group_size % 8 != 0 ||
      K % group_size != 0)
    return NG_ERR_BAD_SHAPE;
  if (static_cast<long long>(K) * N >= (1LL << 40)) return NG_ERR_BAD_SHAPE;
  if (!aligned(out, 2) || !aligned(scales, 2) || !aligned(qweight, 4)) return NG_ERR_MISALIGNED;
  DeviceInfo dev;
  if (int st = current_device_info(&dev)) return st;
  auto* q = reinterpret_cast<const uint32_t*>(qweight);
  auto* s = reinterpret_cast<const __half*>(scales);
  auto strm = static_cast<cudaStream_t>(stream);
  const bool vec = (N % 4 == 0) && aligned(qweight, 16) && aligned(scales, 8) && aligned(out, 8);
  const bool bf = out_dtype == NG_DTYPE_BF16;
#define NG_DQ(V)                                                                              \
  return fast ? (bf ? launch_dequant<V, true, true>(q, s, out, K, N, group_size, dev, strm)   \
                    : launch_dequant<V, true, false>(q, s, out, K, N, group_size, dev, strm)) \
              : (bf ? launch_dequant<V, false, true>(q, s, out, K, N, group_size, dev, strm)  \
                    : launch_dequant<V, false, false>(q, s, out, K, N, group_size, dev, strm))
  if (vec) NG_DQ(4);
  NG_DQ(1);
#undef NG_DQ
}
