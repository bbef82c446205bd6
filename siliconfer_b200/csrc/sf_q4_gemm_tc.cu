// sf_q4_gemm_tc.cu -- prefill GEMM on the tcgen05 tensor cores (T > 8).
#include "sf_q4.h"
#include "sf_q4_internal.h"

namespace sf {
SF_DEFINE_ERROR_READER(take_dev_error_tc)
int run_tc_gemm(const uint8_t*, const float*, const float*, const float*, const void*, int,
                void*, int, int, int, int, int, int, cudaStream_t) {
  return SF_ERR_UNSUPPORTED;
}
}  // namespace sf
