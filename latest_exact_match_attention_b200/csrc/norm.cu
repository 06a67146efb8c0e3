// RMSNorm of the model's blocks and head (code/lema/model.py:215-217 and 264, nn.RMSNorm
// before the attention, the MLP and the LM head): out[m] = (x[m] * rstd[m]) * w with
// rstd[m] = 1 / sqrt(mean(x[m]^2) + eps), computed in fp32 and rounded once to the row type.
// One warp per row, 16-byte loads and streaming stores: one read and one write of the rows
// (torch's kernel at config 3's 524,288 x 1024 bf16 rows runs at ~43% of HBM bandwidth).
// Rows of up to kCached * 256 elements stay in registers between the sum and the scaling;
// longer rows are read a second time (from L1/L2: the warp has just read them).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"

namespace lema {
namespace {

constexpr int kRowsPerBlock = 8;  // 8 warps
constexpr int kCached = 8;        // 16-byte chunks per lane kept in registers (D <= 2048)

template <typename T> struct Vec8;
template <> struct Vec8<__nv_bfloat16> {
  using P = __nv_bfloat162;
  __device__ static float2 f2(P p) { return __bfloat1622float2(p); }
  __device__ static P p2(float a, float b) { return __floats2bfloat162_rn(a, b); }
};
template <> struct Vec8<__half> {
  using P = __half2;
  __device__ static float2 f2(P p) { return __half22float2(p); }
  __device__ static P p2(float a, float b) { return __floats2half2_rn(a, b); }
};

template <typename T>
__device__ __forceinline__ float sumsq8(const uint4& v) {
  using V = Vec8<T>;
  const typename V::P* p = reinterpret_cast<const typename V::P*>(&v);
  float s = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = V::f2(p[e]);
    s = fmaf(f.x, f.x, s);
    s = fmaf(f.y, f.y, s);
  }
  return s;
}

template <typename T>
__device__ __forceinline__ uint4 scale8(const uint4& v, const uint4& w, float rstd) {
  using V = Vec8<T>;
  const typename V::P* p = reinterpret_cast<const typename V::P*>(&v);
  const typename V::P* q = reinterpret_cast<const typename V::P*>(&w);
  uint4 o;
  typename V::P* r = reinterpret_cast<typename V::P*>(&o);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = V::f2(p[e]);
    const float2 g = V::f2(q[e]);
    r[e] = V::p2((f.x * rstd) * g.x, (f.y * rstd) * g.y);
  }
  return o;
}

// 16-bit rows, D % 8 == 0, rows and weight 16-byte aligned; C = D / 8 chunks per row.
template <typename T>
__global__ void __launch_bounds__(32 * kRowsPerBlock) rms_norm_x8_kernel(const uint4* x, const uint4* w, uint4* out,
                                                                        int64_t M, uint32_t C, float d, float eps) {
  griddep_wait();    // launched as a dependent: the rows' producer first
  griddep_launch();  // and the next kernel (K1 after norm1) may set itself up meanwhile
  const int lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + (threadIdx.x >> 5);
  if (m >= M) return;
  const uint4* xr = x + m * C;
  uint4* orow = out + m * C;
  uint4 cache[kCached];
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kCached; ++k) {
    const uint32_t c = lane + 32u * k;
    if (c < C) {
      cache[k] = __ldcs(xr + c);
      s += sumsq8<T>(cache[k]);
    }
  }
  for (uint32_t c = lane + 32u * kCached; c < C; c += 32) s += sumsq8<T>(xr[c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float rstd = rsqrtf(s / d + eps);
#pragma unroll
  for (int k = 0; k < kCached; ++k) {
    const uint32_t c = lane + 32u * k;
    if (c < C) __stcs(orow + c, scale8<T>(cache[k], __ldg(w + c), rstd));
  }
  for (uint32_t c = lane + 32u * kCached; c < C; c += 32) __stcs(orow + c, scale8<T>(xr[c], __ldg(w + c), rstd));
}

}  // namespace
}  // namespace lema

extern "C" int lema_rms_norm(const void* x, const void* weight, int dtype, int64_t M, int64_t D, float eps,
                             void* out, void* stream) {
  using namespace lema;
  clear_error();
  if (M < 0 || D <= 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "rms_norm: bad shape M=%lld D=%lld", (long long)M, (long long)D);
  if (M == 0) return LEMA_OK;
  if (x == nullptr || weight == nullptr || out == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "rms_norm: null pointer");
  if (dtype != LEMA_BF16 && dtype != LEMA_F16) return fail(LEMA_ERR_UNSUPPORTED, "rms_norm: 16-bit rows only (dtype tag %d)", dtype);
  if (D % 8 != 0 || !aligned(x, 16) || !aligned(weight, 16) || !aligned(out, 16))
    return fail(LEMA_ERR_UNSUPPORTED, "rms_norm: rows of a multiple of 8 elements, 16-byte aligned, only (D=%lld)", (long long)D);
  if (D / 8 >= (int64_t(1) << 31)) return fail(LEMA_ERR_INVALID_ARGUMENT, "rms_norm: D too large");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  const int64_t blocks = (M + kRowsPerBlock - 1) / kRowsPerBlock;
  if (blocks >= (int64_t(1) << 31)) return fail(LEMA_ERR_INVALID_ARGUMENT, "rms_norm: M too large");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint32_t C = static_cast<uint32_t>(D / 8);
  const float d = static_cast<float>(D);
  const dim3 grid(static_cast<unsigned>(blocks)), block(32 * kRowsPerBlock);
  const uint4* xv = static_cast<const uint4*>(x);
  const uint4* wv = static_cast<const uint4*>(weight);
  uint4* ov = static_cast<uint4*>(out);
  if (dtype == LEMA_BF16) {
    LEMA_CUDA_TRY(launch_dependent(rms_norm_x8_kernel<__nv_bfloat16>, grid, block, 0, s, xv, wv, ov, M, C, d, eps));
  } else {
    LEMA_CUDA_TRY(launch_dependent(rms_norm_x8_kernel<__half>, grid, block, 0, s, xv, wv, ov, M, C, d, eps));
  }
  return LEMA_OK;
}
