// Shared helpers of the LEMA B200 kernels: hashing, warp utilities, status
// reporting and host-side error handling.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "lema_b200.h"

namespace lema {

constexpr unsigned kFullMask = 0xFFFFFFFFu;

// MurmurHash3's 32- and 64-bit finalizers (Appleby, public domain): cheap
// full-avalanche mixers. Codes are what a model chose, not random bits, so they
// are mixed before they index a table.
__host__ __device__ __forceinline__ uint32_t fmix32(uint32_t h) {
  h ^= h >> 16;
  h *= 0x85EBCA6Bu;
  h ^= h >> 13;
  h *= 0xC2B2AE35u;
  h ^= h >> 16;
  return h;
}

__host__ __device__ __forceinline__ uint64_t fmix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xFF51AFD7ED558CCDull;
  k ^= k >> 33;
  k *= 0xC4CEB9FE1A85EC53ull;
  k ^= k >> 33;
  return k;
}

template <typename CodeT>
__device__ __forceinline__ uint32_t code_hash32(CodeT c);
template <>
__device__ __forceinline__ uint32_t code_hash32<uint32_t>(uint32_t c) {
  return fmix32(c);
}
template <>
__device__ __forceinline__ uint32_t code_hash32<uint64_t>(uint64_t c) {
  return static_cast<uint32_t>(fmix64(c) >> 32);
}

__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ void raise_status(uint32_t* status, uint32_t bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// Streaming (evict-first) store of one vector word: outputs are written once
// and never re-read by the kernel that writes them.
template <typename Vec>
__device__ __forceinline__ void store_stream(Vec* p, const Vec& v) {
  __stcs(p, v);
}
template <>
__device__ __forceinline__ void store_stream<unsigned short>(unsigned short* p,
                                                             const unsigned short& v) {
  *p = v;
}

template <typename Vec>
__device__ __forceinline__ Vec zero_vec() {
  Vec v;
  memset(&v, 0, sizeof(Vec));
  return v;
}

// ------------------------------------------------------------------ host side
// Thread-local message of the last failing entry point (lema_last_error()).
void set_error(const char* fmt, ...);
void clear_error();
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);

struct DeviceInfo {
  int device = -1;
  int sms = 0;
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
};
// Cached per device; queried once. Returns nullptr (and sets the error) on failure.
const DeviceInfo* current_device_info();

// Bound, in nanoseconds, of every device-side wait on another warp's, CTA's or pipeline
// stage's progress: 4 s, or LEMA_WAIT_NS from the environment (read at each launch; tests
// shorten it to make a wait run out on purpose). A wait that runs out sets
// LEMA_STATUS_PROBE_LIMIT and returns; it never traps.
unsigned long long wait_limit_ns();

// Propagates a LEMA_* status code (not a CUDA error) from a call of this library.
#define LEMA_TRY(expr)                \
  do {                                \
    const int _rc = (expr);           \
    if (_rc != LEMA_OK) return _rc;   \
  } while (0)

#define LEMA_CUDA_TRY(expr)                                \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return ::lema::cuda_fail(_e, #expr); \
  } while (0)

inline bool aligned(const void* p, size_t a) {
  return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline uint64_t next_pow2(uint64_t x) {
  uint64_t p = 1;
  while (p < x) p <<= 1;
  return p;
}

inline int log2_exact(uint64_t p) {
  int l = 0;
  while ((uint64_t(1) << l) < p) ++l;
  return l;
}

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

}  // namespace lema

namespace lema {
__host__ __device__ constexpr size_t round_up16(size_t x) { return (x + 15) / 16 * 16; }

// Programmatic dependent launch. A kernel launched by launch_dependent may start while the
// kernel before it in the stream is finishing (its launch and CTA placement overlap that
// kernel's tail); it calls griddep_wait() before its first global memory access, which returns
// once the previous kernel has completed and its writes are visible. Launched the ordinary
// way, griddep_wait() returns at once. LEMA_PDL=0 in the environment launches ordinarily.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// In the kernel before it: lets the dependent kernel be placed on free SM slots once every CTA
// of this grid has started (it still waits in griddep_wait for this grid to complete).
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool pdl_enabled();

// Launch facts of a kernel on the current device, worked out on the first call per (kernel,
// device, dynamic shared memory, threads, cluster size) and remembered: the first call sets
// the kernel's dynamic shared memory limit, then `out` (if not null) receives the resident
// CTAs per SM (cluster == 0, threads > 0) or the resident clusters of `cluster` CTAs. A call
// after the first costs a lookup instead of runtime queries (small launches are host-bound).
int kernel_facts(const void* kernel, size_t smem, int threads, int cluster, int* out);

template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t stream, Args... args) {
  if (!pdl_enabled()) {
    kernel<<<grid, block, smem, stream>>>(args...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
}  // namespace lema
