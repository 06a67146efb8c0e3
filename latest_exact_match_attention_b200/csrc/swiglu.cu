// SwiGLU activation of the model's MLP (code/lema/model.py:85-93, `SwiGLU.forward`:
// down(silu(gate(x)) * up(x))) for the fused gate/up GEMM output: gu[m] = [gate(x) | up(x)],
// out[m][f] = silu(gu[m][f]) * gu[m][F + f], computed in fp32 and rounded once. One pass over
// gu instead of torch's silu and mul kernels (two passes and an intermediate).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace lema {
namespace {

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T>
__global__ void swiglu_kernel(const T* gu, T* out, int64_t M, int64_t F) {
  const int64_t n = M * F;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / F, f = i - m * F;
    const float g = to_f(gu[m * 2 * F + f]);
    const float u = to_f(gu[m * 2 * F + F + f]);
    out[i] = from_f<T>(g / (1.0f + expf(-g)) * u);
  }
}

}  // namespace
}  // namespace lema

extern "C" int lema_swiglu(const void* gu, int dtype, int64_t M, int64_t F, void* out, void* stream) {
  using namespace lema;
  clear_error();
  if (M < 0 || F <= 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "swiglu: bad shape M=%lld F=%lld", (long long)M, (long long)F);
  if (M == 0) return LEMA_OK;
  if (gu == nullptr || out == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "swiglu: null pointer");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>((M * F + 255) / 256, int64_t(dev->sms) * 16));
  switch (dtype) {
    case LEMA_F32: swiglu_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(gu), static_cast<float*>(out), M, F); break;
    case LEMA_BF16: swiglu_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), M, F); break;
    case LEMA_F16: swiglu_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(gu), static_cast<__half*>(out), M, F); break;
    default: return fail(LEMA_ERR_INVALID_ARGUMENT, "swiglu: dtype tag %d", dtype);
  }
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}
