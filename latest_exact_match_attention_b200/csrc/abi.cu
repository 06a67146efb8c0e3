// The C ABI of liblema_b200.so (declared in include/lema_b200.h): argument checks, error
// reporting, per-device facts, and dispatch to the kernels.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "match.cuh"

namespace lema {

// Implemented next to their kernels.
int pack_codes(const void* z, int dtype, int64_t d0, int64_t d1, int64_t d2, int64_t s0, int64_t s1,
               int64_t s2, int D, void* codes, int code_bytes, cudaStream_t stream);
int64_t store_slot_bytes(int64_t vbytes);
size_t store_workspace_bytes(int64_t n, int64_t T, int code_bytes);
int store_exchange(void* table, int64_t cap, int64_t vbytes, const void* qc, const void* kc,
                   int code_bytes, const void* values, void* out, int64_t n, int64_t T, int64_t g0,
                   int64_t* counts, uint32_t* status, void* ws, size_t ws_bytes, cudaStream_t stream,
                   int64_t seg_groups, int64_t seg_slots, const int64_t* rows, int phase);
int proj_codes(const void* x, const void* w_qk, int64_t M, int64_t K, int64_t T, int hq, int hk,
               int d_qk, uint32_t* qcodes, uint32_t* kcodes, uint32_t* status, cudaStream_t stream);

namespace {
thread_local char g_err[512] = {0};
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];
}  // namespace

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  snprintf(g_err, sizeof(g_err), "CUDA error %d (%s) in %s", static_cast<int>(e),
           cudaGetErrorString(e), what);
  return LEMA_ERR_CUDA;
}

unsigned long long wait_limit_ns() {
  const char* e = std::getenv("LEMA_WAIT_NS");
  if (e != nullptr) {
    const unsigned long long v = std::strtoull(e, nullptr, 10);
    if (v > 0) return v;
  }
  return 4000000000ull;
}

bool pdl_enabled() {
  const char* e = std::getenv("LEMA_PDL");
  return e == nullptr || e[0] != '0';
}

int kernel_facts(const void* kernel, size_t smem, int threads, int cluster, int* out) {
  int dev = -1;
  LEMA_CUDA_TRY(cudaGetDevice(&dev));
  struct Fact {
    const void* kernel;
    int dev;
    size_t smem;
    int threads, cluster, value;
  };
  static std::mutex mu;
  static std::vector<Fact> memo;
  {
    std::lock_guard<std::mutex> g(mu);
    for (const Fact& f : memo) {
      if (f.kernel == kernel && f.dev == dev && f.smem == smem && f.threads == threads && f.cluster == cluster) {
        if (out != nullptr) *out = f.value;
        return LEMA_OK;
      }
    }
  }
  LEMA_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  int value = 0;
  if (cluster > 0) {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(cluster), 1, 1);
    cfg.blockDim = dim3(static_cast<unsigned>(threads), 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    LEMA_CUDA_TRY(cudaOccupancyMaxActiveClusters(&value, kernel, &cfg));
  } else if (threads > 0) {
    LEMA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&value, kernel, threads, smem));
  }
  {
    std::lock_guard<std::mutex> g(mu);
    memo.push_back(Fact{kernel, dev, smem, threads, cluster, value});
  }
  if (out != nullptr) *out = value;
  return LEMA_OK;
}

const DeviceInfo* current_device_info() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_fail(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    fail(LEMA_ERR_UNSUPPORTED, "device index %d out of range", dev);
    return nullptr;
  }
  std::call_once(g_dev_once[dev], [dev]() {
    DeviceInfo d;
    d.device = dev;
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
      d.sms = 0;
    }
    g_dev[dev] = d;
  });
  if (g_dev[dev].sms <= 0) {
    fail(LEMA_ERR_CUDA, "could not query device %d", dev);
    return nullptr;
  }
  return &g_dev[dev];
}

}  // namespace lema

extern "C" {

const char* lema_last_error(void) { return lema::g_err; }

int lema_version(void) { return 100; }

int lema_pack_codes(const void* z, int dtype, int64_t d0, int64_t d1, int64_t d2, int64_t s0, int64_t s1,
                    int64_t s2, int d_qk, void* codes, int code_bytes, void* stream) {
  lema::clear_error();
  return lema::pack_codes(z, dtype, d0, d1, d2, s0, s1, s2, d_qk, codes, code_bytes,
                          static_cast<cudaStream_t>(stream));
}

int lema_proj_codes(const void* x, const void* w_qk, int64_t M, int64_t K, int64_t T, int hq, int hk,
                    int d_qk, uint32_t* qcodes, uint32_t* kcodes, uint32_t* status, void* stream) {
  lema::clear_error();
  return lema::proj_codes(x, w_qk, M, K, T, hq, hk, d_qk, qcodes, kcodes, status,
                          static_cast<cudaStream_t>(stream));
}

size_t lema_prefill_workspace_bytes(int64_t n_streams, int64_t T, int code_bytes) {
  return lema::match_workspace_bytes(n_streams, T, code_bytes, true, true);
}

int lema_prefill_match(const void* qcodes, const void* kcodes, int code_bytes, int64_t n_streams,
                       int64_t T, int32_t* src, const void* values, int64_t vbytes, void* out,
                       void* workspace, size_t workspace_bytes, uint32_t* status, void* stream) {
  lema::clear_error();
  lema::MatchLaunch m;
  m.qc = qcodes;
  m.kc = kcodes;
  m.code_bytes = code_bytes;
  m.N = n_streams;
  m.T = T;
  m.src = src;
  m.v = values;
  m.vbytes = vbytes;
  m.out = out;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.status = status;
  m.stream = static_cast<cudaStream_t>(stream);
  return lema::launch_match(m);
}

int lema_prefill_match_strided(const void* qcodes, const void* kcodes, int code_bytes, int64_t n_streams,
                               int64_t T, int32_t* src, const void* values, int64_t vbytes, void* out,
                               int64_t heads, int64_t v_sb, int64_t v_sh, int64_t v_st, int64_t o_sb,
                               int64_t o_sh, int64_t o_st, void* workspace, size_t workspace_bytes,
                               uint32_t* status, void* stream) {
  lema::clear_error();
  if (heads < 1 || (n_streams > 0 && n_streams % heads != 0))
    return lema::fail(LEMA_ERR_INVALID_ARGUMENT, "streams (%lld) must be whole groups of heads (%lld)",
                      (long long)n_streams, (long long)heads);
  if (v_sb < 0 || v_sh < 0 || v_st < 0 || o_sb < 0 || o_sh < 0 || o_st < 0)
    return lema::fail(LEMA_ERR_INVALID_ARGUMENT, "negative stride");
  lema::MatchLaunch m;
  m.qc = qcodes;
  m.kc = kcodes;
  m.code_bytes = code_bytes;
  m.N = n_streams;
  m.T = T;
  m.src = src;
  m.v = values;
  m.vbytes = vbytes;
  m.out = out;
  m.heads = heads;
  m.v_sb = v_sb;
  m.v_sh = v_sh;
  m.v_st = v_st;
  m.o_sb = o_sb;
  m.o_sh = o_sh;
  m.o_st = o_st;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.status = status;
  m.stream = static_cast<cudaStream_t>(stream);
  return lema::launch_match(m);
}

int64_t lema_store_slot_bytes(int64_t vbytes) { return lema::store_slot_bytes(vbytes); }

size_t lema_store_workspace_bytes(int64_t n, int64_t T, int code_bytes) {
  return lema::store_workspace_bytes(n, T, code_bytes);
}

int lema_store_exchange(void* table, int64_t cap, int64_t vbytes, const void* qcodes, const void* kcodes,
                        int code_bytes, const void* values, void* out, int64_t n, int64_t T, int64_t g0,
                        int64_t* counts, uint32_t* status, void* workspace, size_t workspace_bytes,
                        void* stream) {
  lema::clear_error();
  return lema::store_exchange(table, cap, vbytes, qcodes, kcodes, code_bytes, values, out, n, T, g0,
                              counts, status, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream), 0, 0, nullptr, 3);
}

int lema_store_exchange_seg(void* table, int64_t cap, int64_t vbytes, const void* qcodes,
                            const void* kcodes, int code_bytes, const void* values, void* out, int64_t n,
                            int64_t T, int64_t g0, int64_t* counts, uint32_t* status, void* workspace,
                            size_t workspace_bytes, int64_t seg_groups, int64_t seg_slots, void* stream) {
  lema::clear_error();
  return lema::store_exchange(table, cap, vbytes, qcodes, kcodes, code_bytes, values, out, n, T, g0,
                              counts, status, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream), seg_groups, seg_slots, nullptr, 3);
}

int lema_store_exchange_strided(void* table, int64_t cap, int64_t vbytes, const void* qcodes,
                                const void* kcodes, int code_bytes, const void* values, void* out,
                                int64_t n, int64_t T, int64_t g0, int64_t* counts, uint32_t* status,
                                void* workspace, size_t workspace_bytes, int64_t seg_groups,
                                int64_t seg_slots, int64_t heads, int64_t v_sb, int64_t v_sh,
                                int64_t v_st, int64_t o_sb, int64_t o_sh, int64_t o_st, void* stream) {
  lema::clear_error();
  const int64_t rows[7] = {heads, v_sb, v_sh, v_st, o_sb, o_sh, o_st};
  return lema::store_exchange(table, cap, vbytes, qcodes, kcodes, code_bytes, values, out, n, T, g0,
                              counts, status, workspace, workspace_bytes,
                              static_cast<cudaStream_t>(stream), seg_groups, seg_slots, rows, 3);
}

int lema_store_exchange_phase(void* table, int64_t cap, int64_t vbytes, const void* qcodes,
                              const void* kcodes, int code_bytes, const void* values, void* out,
                              int64_t n, int64_t g0, int64_t* counts, uint32_t* status,
                              int64_t seg_groups, int64_t seg_slots, int phase, void* stream) {
  lema::clear_error();
  return lema::store_exchange(table, cap, vbytes, qcodes, kcodes, code_bytes, values, out, n, 1, g0,
                              counts, status, nullptr, 0, static_cast<cudaStream_t>(stream), seg_groups,
                              seg_slots, nullptr, phase);
}

}  // extern "C"
