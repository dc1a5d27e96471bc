// Placeholder until the tcgen05 GEMM lands.
#include "ng_common.cuh"
extern "C" int ng_gemm_w4a16(const void* x, int, const int32_t* q, const uint16_t* s, void* y, int,
                             int, int, int, int, void*) {
  if (!x || !q || !s || !y) return NG_ERR_NULL_POINTER;
  return NG_ERR_BAD_ARGUMENT;
}
