// K1 -- code projection GEMM with a sign/bit-pack epilogue (tcgen05 + TMA + TMEM).
#include <cuda_runtime.h>

#include "common.cuh"

namespace lema {

int proj_codes(const void*, const void*, int64_t, int64_t, int64_t, int, int, int, uint32_t*,
               uint32_t*, cudaStream_t) {
  return fail(LEMA_ERR_UNSUPPORTED, "lema_proj_codes is not built yet");
}

}  // namespace lema
