/*
 * Plain-C restatement of the reference nibblegemm CPU oracle.
 * TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and the
 * CPU legs of bench.py through ctypes, never by the nibblegemm_b200 package.
 *
 * It computes exactly what arvindcr4/nibblegemm python/nibblegemm/quant.py
 * computes, in C so that full BASELINE shapes check in milliseconds:
 *   - unpack of the interleaved nibble word (quant.py:185-196, slot table
 *     quant.py:48: logical k lives in slot (k odd ? 4 + k/2 : k/2));
 *   - dequantize: fp16((u - 8) * float(scale)), a single rounding
 *     (quant.py:199-204);
 *   - reference_matmul: fp32 X @ fp32(dequantized fp16 W), then one cast to
 *     fp16 (quant.py:207-215).  Summation runs over k in ascending order per
 *     output; the reference's BLAS order differs only in fp32 rounding.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -shared), output oracle/_build/.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float half_bits_to_float(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static inline uint16_t float_to_half_bits(float f) {
  _Float16 v = (_Float16)f; /* IEEE round-to-nearest-even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

static inline float bf16_bits_to_float(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline int slot_of_k(int k) { return (k & 1) ? 4 + (k >> 1) : (k >> 1); }

int ngo_abi_version(void) { return 1; }

/* out[K,N] fp16 bits = fp16((u - 8) * scale). */
void ngo_dequantize_f16(const uint32_t* q, const uint16_t* s, uint16_t* out, int K, int N,
                        int G) {
#pragma omp parallel for schedule(static)
  for (int k = 0; k < K; ++k) {
    const uint32_t* qrow = q + (size_t)(k >> 3) * N;
    const uint16_t* srow = s + (size_t)(k / G) * N;
    const int shift = 4 * slot_of_k(k & 7);
    uint16_t* orow = out + (size_t)k * N;
    for (int n = 0; n < N; ++n) {
      const float u = (float)(int)((qrow[n] >> shift) & 0xFu) - 8.0f;
      orow[n] = float_to_half_bits(u * half_bits_to_float(srow[n]));
    }
  }
}

/*
 * y[M,N] (fp32) = x[M,K] @ W, where W is the fp16-rounded dequantised weight.
 * x_kind: 0 = fp16 bit patterns, 1 = bf16 bit patterns, 2 = fp32 values.
 * Parallel over column blocks; each output sums k = 0..K-1 in order.
 * threads <= 0 leaves the OpenMP default.
 */
void ngo_matmul_f32(const void* x, int x_kind, const uint32_t* q, const uint16_t* s, float* y,
                    int M, int K, int N, int G, int threads) {
  float* xf = (float*)malloc(sizeof(float) * (size_t)M * K);
  for (size_t i = 0; i < (size_t)M * K; ++i) {
    if (x_kind == 0) xf[i] = half_bits_to_float(((const uint16_t*)x)[i]);
    else if (x_kind == 1) xf[i] = bf16_bits_to_float(((const uint16_t*)x)[i]);
    else xf[i] = ((const float*)x)[i];
  }
  const int NB = 256;
  const int nblocks = (N + NB - 1) / NB;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel
  {
    float* w = (float*)malloc(sizeof(float) * NB);
    float* acc = (float*)malloc(sizeof(float) * (size_t)NB * (M > 0 ? M : 1));
#pragma omp for schedule(dynamic, 1)
    for (int b = 0; b < nblocks; ++b) {
      const int n0 = b * NB;
      const int nn = (N - n0) < NB ? (N - n0) : NB;
      memset(acc, 0, sizeof(float) * (size_t)NB * M);
      for (int k = 0; k < K; ++k) {
        const uint32_t* qrow = q + (size_t)(k >> 3) * N + n0;
        const uint16_t* srow = s + (size_t)(k / G) * N + n0;
        const int shift = 4 * slot_of_k(k & 7);
        for (int j = 0; j < nn; ++j) {
          const float u = (float)(int)((qrow[j] >> shift) & 0xFu) - 8.0f;
          w[j] = half_bits_to_float(float_to_half_bits(u * half_bits_to_float(srow[j])));
        }
        for (int m = 0; m < M; ++m) {
          const float xv = xf[(size_t)m * K + k];
          float* a = acc + (size_t)m * NB;
          for (int j = 0; j < nn; ++j) a[j] += xv * w[j];
        }
      }
      for (int m = 0; m < M; ++m)
        memcpy(y + (size_t)m * N + n0, acc + (size_t)m * NB, sizeof(float) * nn);
    }
    free(w);
    free(acc);
  }
  free(xf);
}
