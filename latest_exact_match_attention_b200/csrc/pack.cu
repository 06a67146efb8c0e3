// pack_codes: sign bits of pre-activations -> one integer code per row.
// code = sum_d [z_d >= 0] << d, the rule of code/lema/attention.py:82-97 (sign(0) = +1, a
// float comparison, so NaN gives 0 and -0.0 gives 1). Reads a strided [d0, d1, d2, D] view
// (the [B, H, T, d_qk] transpose of a projection output) and writes codes densely.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace lema {
namespace pack {

constexpr int kThreads = 256;

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }

template <typename In, typename CodeT>
__global__ void __launch_bounds__(kThreads) pack_kernel(const In* __restrict__ z, int64_t d0, int64_t d1,
                                                        int64_t d2, int64_t s0, int64_t s1, int64_t s2,
                                                        int D, CodeT* __restrict__ out) {
  const int64_t total = d0 * d1 * d2;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; r < total;
       r += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t i2 = r % d2;
    const int64_t t = r / d2;
    const int64_t i1 = t % d1;
    const int64_t i0 = t / d1;
    const In* row = z + i0 * s0 + i1 * s1 + i2 * s2;
    CodeT c = 0;
    for (int d = 0; d < D; ++d) {
      if (to_float(row[d]) >= 0.0f) c |= CodeT(1) << d;
    }
    out[r] = c;
  }
}

template <typename In, typename CodeT>
int launch(const void* z, int64_t d0, int64_t d1, int64_t d2, int64_t s0, int64_t s1, int64_t s2,
           int D, void* codes, cudaStream_t stream, int sms) {
  const int64_t total = d0 * d1 * d2;
  const int64_t blocks = std::min<int64_t>((total + kThreads - 1) / kThreads, int64_t(sms) * 16);
  pack_kernel<In, CodeT><<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(
      static_cast<const In*>(z), d0, d1, d2, s0, s1, s2, D, static_cast<CodeT*>(codes));
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

}  // namespace pack

int pack_codes(const void* z, int dtype, int64_t d0, int64_t d1, int64_t d2, int64_t s0, int64_t s1,
               int64_t s2, int D, void* codes, int code_bytes, cudaStream_t stream) {
  if (code_bytes != 4 && code_bytes != 8) return fail(LEMA_ERR_INVALID_ARGUMENT, "code_bytes must be 4 or 8, got %d", code_bytes);
  if (D < 1 || D > 8 * code_bytes) return fail(LEMA_ERR_INVALID_ARGUMENT, "d_qk %d does not pack into %d-byte codes", D, code_bytes);
  if (d0 < 0 || d1 < 0 || d2 < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "negative shape");
  if (d0 * d1 * d2 == 0) return LEMA_OK;
  if (z == nullptr || codes == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned(codes, code_bytes)) return fail(LEMA_ERR_INVALID_ARGUMENT, "codes not aligned to their width");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
  const bool c4 = code_bytes == 4;
  switch (dtype) {
    case LEMA_F32:
      return c4 ? pack::launch<float, uint32_t>(z, d0, d1, d2, s0, s1, s2, D, codes, stream, dev->sms)
                : pack::launch<float, uint64_t>(z, d0, d1, d2, s0, s1, s2, D, codes, stream, dev->sms);
    case LEMA_BF16:
      return c4 ? pack::launch<__nv_bfloat16, uint32_t>(z, d0, d1, d2, s0, s1, s2, D, codes, stream, dev->sms)
                : pack::launch<__nv_bfloat16, uint64_t>(z, d0, d1, d2, s0, s1, s2, D, codes, stream, dev->sms);
    case LEMA_F16:
      return c4 ? pack::launch<__half, uint32_t>(z, d0, d1, d2, s0, s1, s2, D, codes, stream, dev->sms)
                : pack::launch<__half, uint64_t>(z, d0, d1, d2, s0, s1, s2, D, codes, stream, dev->sms);
    default:
      return fail(LEMA_ERR_INVALID_ARGUMENT, "unknown dtype tag %d", dtype);
  }
}

}  // namespace lema
