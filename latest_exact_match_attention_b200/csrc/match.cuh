// Internal interface of the prefill matcher (K2), shared by the C ABI and the
// store's chunked exchange.
#pragma once

#include "common.cuh"

namespace lema {

struct MatchLaunch {
  const void* qc = nullptr;  // [N][T] codes
  const void* kc = nullptr;
  int code_bytes = 4;        // 4 or 8
  int64_t N = 0, T = 0;
  int32_t* src = nullptr;    // [N][T] latest earlier match or -1 (optional)
  const void* v = nullptr;   // [N][T] rows of vbytes (needed iff out)
  int64_t vbytes = 0;
  void* out = nullptr;       // [N][T] gathered rows, zeros on a miss (optional)
  // Last-occurrence table per stream (optional, all three or none): the
  // distinct key codes of stream n with the position of their last occurrence,
  // lt_code[n*T + e], lt_pos[n*T + e] for e < lt_count[n], in no particular order.
  void* lt_code = nullptr;
  int32_t* lt_pos = nullptr;
  int32_t* lt_count = nullptr;
  // optional strided value rows (heads > 0): row (n, t) at v + (n / heads) * v_sb +
  // (n % heads) * v_sh + t * v_st bytes, out likewise; heads = 0: [N][T] rows of vbytes
  int64_t heads = 0, v_sb = 0, v_sh = 0, v_st = 0, o_sb = 0, o_sh = 0, o_st = 0;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  uint32_t* status = nullptr;
  cudaStream_t stream = nullptr;
};

// need_src = false: the caller passes src, so no index scratch is counted. pipe = true also
// counts the pipelined mode's control words (calls that gather rows; without them such a
// call takes the two-kernel path).
size_t match_workspace_bytes(int64_t N, int64_t T, int code_bytes, bool need_src = true, bool pipe = false);
int launch_match(const MatchLaunch& a);

}  // namespace lema
