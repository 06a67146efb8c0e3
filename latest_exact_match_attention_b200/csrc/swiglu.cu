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
  griddep_wait();  // launched as a dependent: the gate/up GEMM first
  const int64_t n = M * F;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / F, f = i - m * F;
    const float g = to_f(gu[m * 2 * F + f]);
    const float u = to_f(gu[m * 2 * F + F + f]);
    out[i] = from_f<T>(g / (1.0f + expf(-g)) * u);
  }
}

// bf16, F % 8 == 0, 16-byte aligned: 8 outputs per thread from two 16-byte loads.
__global__ void swiglu_bf16x8_kernel(const uint4* gu, uint4* out, uint32_t M, uint32_t F8) {
  griddep_wait();  // launched as a dependent: the gate/up GEMM first
  const uint32_t n = M * F8;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const uint32_t m = i / F8, f = i - m * F8;
    const uint4 g4 = gu[static_cast<uint64_t>(m) * 2 * F8 + f];
    const uint4 u4 = gu[static_cast<uint64_t>(m) * 2 * F8 + F8 + f];
    const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&g4);
    const __nv_bfloat162* u = reinterpret_cast<const __nv_bfloat162*>(&u4);
    uint4 o4;
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(&o4);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 gf = __bfloat1622float2(g[e]);
      const float2 uf = __bfloat1622float2(u[e]);
      o[e] = __floats2bfloat162_rn(gf.x / (1.0f + expf(-gf.x)) * uf.x, gf.y / (1.0f + expf(-gf.y)) * uf.y);
    }
    out[i] = o4;
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
  if (dtype == LEMA_BF16 && F % 8 == 0 && aligned(gu, 16) && aligned(out, 16) && M * (F / 8) < (int64_t(1) << 31)) {
    const int64_t n = M * (F / 8);
    const int64_t b8 = std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, int64_t(dev->sms) * 16));
    LEMA_CUDA_TRY(launch_dependent(swiglu_bf16x8_kernel, dim3(static_cast<unsigned>(b8)), dim3(256), 0, s,
                                   static_cast<const uint4*>(gu), static_cast<uint4*>(out),
                                   static_cast<uint32_t>(M), static_cast<uint32_t>(F / 8)));
    return LEMA_OK;
  }
  switch (dtype) {
    case LEMA_F32: swiglu_kernel<float><<<blocks, 256, 0, s>>>(static_cast<const float*>(gu), static_cast<float*>(out), M, F); break;
    case LEMA_BF16: swiglu_kernel<__nv_bfloat16><<<blocks, 256, 0, s>>>(static_cast<const __nv_bfloat16*>(gu), static_cast<__nv_bfloat16*>(out), M, F); break;
    case LEMA_F16: swiglu_kernel<__half><<<blocks, 256, 0, s>>>(static_cast<const __half*>(gu), static_cast<__half*>(out), M, F); break;
    default: return fail(LEMA_ERR_INVALID_ARGUMENT, "swiglu: dtype tag %d", dtype);
  }
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}
