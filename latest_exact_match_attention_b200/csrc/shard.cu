// Sequence-sharded prefill: the latest exact match over sequences too long for one pass or
// one GPU (config 5: one sequence of 2^26 positions, 16 heads, sharded over 2-8 GPUs).
//
// Replaces, for one sequence cut into contiguous shards, what code/lema/attention.py:100-132
// (`latest_prev_match`) computes in one pass over the whole sequence. Each rank owns positions
// [base, base + L) of every head and runs:
//   1. segment match (K2): the shard is cut into segments of seg_len positions, each matched
//      on its own by the shared-memory matcher, which also emits the segment's
//      last-occurrence table (LT): its distinct key codes and their last positions;
//   2. sweep (lema_shard_sweep): one CTA cluster per head walks the segments in order against a hash
//      of {code -> latest position so far}, starting empty: the queries a segment could not
//      resolve on its own look the hash up, then the segment's LT is inserted. Indices become
//      global positions. Afterwards the hash holds the shard's LT (lema_lt_extract), which the
//      ranks all-gather: no rank waits for another before this point;
//   3. resolve (lema_lt_resolve): the queries still without a match look up a hash of the
//      earlier ranks' LTs (lema_lt_insert), all in parallel;
//   4. gather (lema_shard_gather): rows of this shard's own positions from its values, rows of
//      earlier shards' positions from a buffer the caller fetched from their owners.
// The result is bit-identical to one pass over the whole sequence: the latest earlier key of a
// query is in its own segment (1), else it is the last occurrence of the code in the latest
// earlier segment of the shard holding it (2), else in the latest earlier shard holding it (3).
//
// Hash tables: per head, `slots` (a power of two) 64-bit words, zero = empty, else
// (code << 32) | (position + 1); linear probing from fmix32(code). An insert keeps the larger
// position. Slots are never freed, so a probe that meets an empty slot has seen every slot
// its code could occupy. Codes are 32-bit (d_qk <= 32).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "match.cuh"

namespace lema {
namespace k5 {

__device__ __forceinline__ uint64_t lt_word(uint32_t code, int32_t pos) {
  return (static_cast<uint64_t>(code) << 32) | static_cast<uint32_t>(pos + 1);
}

// Inserts code -> pos keeping the larger position. False when every slot was probed.
__device__ bool lt_insert_max(uint64_t* tab, uint32_t mask, uint32_t code, int32_t pos) {
  const unsigned long long want = lt_word(code, pos);
  uint32_t i = fmix32(code) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe, i = (i + 1) & mask) {
    unsigned long long* slot = reinterpret_cast<unsigned long long*>(tab + i);
    unsigned long long cur = __ldcg(slot);
    for (;;) {
      if (cur == 0) {
        const unsigned long long prev = atomicCAS(slot, 0ull, want);
        if (prev == 0) return true;
        cur = prev;
        continue;
      }
      if (static_cast<uint32_t>(cur >> 32) != code) break;
      if (static_cast<uint32_t>(cur) >= static_cast<uint32_t>(want)) return true;
      const unsigned long long prev = atomicCAS(slot, cur, want);
      if (prev == cur) return true;
      cur = prev;
    }
  }
  return false;
}

// Latest position stored for code, or -1.
__device__ __forceinline__ int32_t lt_find(const uint64_t* tab, uint32_t mask, uint32_t code) {
  uint32_t i = fmix32(code) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe, i = (i + 1) & mask) {
    const uint64_t cur = __ldcg(reinterpret_cast<const unsigned long long*>(tab + i));
    if (cur == 0) return -1;
    if (static_cast<uint32_t>(cur >> 32) == code) return static_cast<int32_t>(static_cast<uint32_t>(cur)) - 1;
  }
  return -1;
}

// ------------------------------------------------------------------ inserts
struct InsertParams {
  uint64_t* table;
  int64_t slots;
  int64_t n_heads;
  const int32_t* heads;
  const uint32_t* codes;
  const int32_t* pos;
  int64_t n;
  uint32_t* status;
};

__global__ void insert_entries_kernel(const InsertParams p) {
  const uint32_t mask = static_cast<uint32_t>(p.slots - 1);
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < p.n; i += int64_t(gridDim.x) * blockDim.x) {
    const int32_t h = p.heads[i];
    if (h < 0 || h >= p.n_heads) {
      raise_status(p.status, LEMA_STATUS_PROBE_LIMIT);
      continue;
    }
    if (!lt_insert_max(p.table + h * p.slots, mask, p.codes[i], p.pos[i]))
      raise_status(p.status, LEMA_STATUS_TABLE_FULL);
  }
}

// Entries with position >= lo as one flat list (head, code, position), in no particular order.
struct ExtractParams {
  const uint64_t* table;
  int64_t slots, n_heads;
  int32_t lo;
  int32_t* out_heads;
  uint32_t* out_codes;
  int32_t* out_pos;
  int32_t* out_count;
  int64_t cap;
  uint32_t* status;
};

__global__ void extract_kernel(const ExtractParams p) {
  const int64_t total = p.n_heads * p.slots;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const uint64_t w = p.table[i];
    if (w == 0) continue;
    const int32_t pos = static_cast<int32_t>(static_cast<uint32_t>(w)) - 1;
    if (pos < p.lo) continue;
    const int32_t k = atomicAdd(p.out_count, 1);
    if (k >= p.cap) {
      raise_status(p.status, LEMA_STATUS_TABLE_FULL);
      continue;
    }
    p.out_heads[k] = static_cast<int32_t>(i / p.slots);
    p.out_codes[k] = static_cast<uint32_t>(w >> 32);
    p.out_pos[k] = pos;
  }
}

// ------------------------------------------------------------------ resolve
// src[h][i] == -1: the latest position of qc[h][i] in the table (earlier shards), or -1.
struct ResolveParams {
  const uint64_t* table;
  int64_t slots, n_heads, L;
  const uint32_t* qc;
  int32_t* src;
};

__global__ void resolve_kernel(const ResolveParams p) {
  const uint32_t mask = static_cast<uint32_t>(p.slots - 1);
  const int64_t total = p.n_heads * p.L;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    if (p.src[i] >= 0) continue;
    const int64_t h = i / p.L;
    p.src[i] = lt_find(p.table + h * p.slots, mask, p.qc[i]);
  }
}

// Queries with src == -1 probe the earlier shards' tables, newest shard first; the first
// shard holding the code has its latest occurrence. tables[t] holds n_heads x slots[t] words.
struct ResolveTablesParams {
  const uint64_t* const* tables;
  const int64_t* slots;
  int n_tables;
  int64_t n_heads, L;
  const uint32_t* qc;
  int32_t* src;
};

__device__ __forceinline__ void resolve_one(const ResolveTablesParams& p, int64_t i) {
  const int64_t h = i / p.L;
  const uint32_t q = p.qc[i];
  int32_t r = -1;
  for (int t = p.n_tables - 1; t >= 0 && r < 0; --t) {
    const int64_t sl = p.slots[t];
    r = lt_find(p.tables[t] + h * sl, static_cast<uint32_t>(sl - 1), q);
  }
  p.src[i] = r;
}

// Only a few positions in a hundred are still unmatched, so instead of one thread per
// position (each waiting on its index load, then on a rare dependent probe chain), every warp
// scans 4 x 32 positions per round (four coalesced loads in flight), queues the unmatched ones
// in shared memory, and probes them 32 at a time, one per lane: the probes of a warp are
// independent and in flight together.
constexpr int kResolveThreads = 256;
__global__ void __launch_bounds__(kResolveThreads) resolve_tables_kernel(const ResolveTablesParams p) {
  constexpr int kWarps = kResolveThreads / 32, kLoads = 4;
  __shared__ int64_t queue[kWarps][64];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t total = p.n_heads * p.L;
  const uint32_t below = (1u << lane) - 1u;
  int n = 0;  // queued, the same in every lane
  const int64_t stride = int64_t(gridDim.x) * kWarps * 32 * kLoads;
  for (int64_t base = (int64_t(blockIdx.x) * kWarps + warp) * 32 * kLoads; base < total; base += stride) {
    int32_t sv[kLoads];
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int64_t i = base + u * 32 + lane;
      sv[u] = i < total ? __ldcs(p.src + i) : 0;
    }
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int64_t i = base + u * 32 + lane;
      const bool miss = i < total && sv[u] < 0;
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, miss);
      if (miss) queue[warp][n + __popc(m & below)] = i;
      n += __popc(m);
      __syncwarp();
      if (n >= 32) {  // 32 probes at once; the rest (< 32) stay queued
        n -= 32;
        resolve_one(p, queue[warp][n + lane]);
        __syncwarp();
      }
    }
  }
  if (lane < n) resolve_one(p, queue[warp][lane]);
}

// A head swept as vrows rows (sub-shards) of L positions: queries of row r (v = r % vrows)
// still without a match probe the rows r - 1, ..., r - v of the same head in the sweep's table,
// newest first.
struct ResolveRowsParams {
  const uint64_t* table;
  int64_t slots, n_rows, vrows, L;
  const uint32_t* qc;
  int32_t* src;
};

__global__ void resolve_rows_kernel(const ResolveRowsParams p) {
  const uint32_t mask = static_cast<uint32_t>(p.slots - 1);
  const int64_t total = p.n_rows * p.L;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / p.L;
    const int64_t v = r % p.vrows;
    if (v == 0 || p.src[i] >= 0) continue;
    const uint32_t q = p.qc[i];
    int32_t res = -1;
    for (int64_t rr = r - 1; rr >= r - v && res < 0; --rr) res = lt_find(p.table + rr * p.slots, mask, q);
    p.src[i] = res;
  }
}

// ------------------------------------------------------------------ sweep
// One 8-CTA cluster per head: the segment's lookups and inserts are spread over the cluster's
// 4096 threads, and cluster barriers (release / acquire at cluster scope) separate the two
// phases of a segment and the segments from one another. The barrier is the hardware's own
// (every CTA of a cluster is resident at once and every CTA takes the same number of steps).
constexpr int kClusterCtas = 8;
constexpr int kSweepThreads = 512;

struct SweepParams {
  uint64_t* table;
  int64_t slots;
  const uint32_t* qc;  // [H][L]
  int32_t* src;        // [H][L]: in, segment-relative index or -1; out, global position or -1
  int64_t L, seg_len, n_seg, base;
  const uint32_t* lt_code;
  const int32_t* lt_pos;
  const int32_t* lt_count;
  uint32_t* status;
  int64_t vrows;       // rows per head: row r's positions start at base + (r % vrows) * L
};

// After the inserts: release, so every insert is visible to the next segment's lookups.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// After the lookups: they have all returned (their values are in registers), so the barrier
// need not wait for this thread's stores; it only keeps the inserts behind every lookup.
__device__ __forceinline__ void cluster_sync_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Insert for the sweep: a blind claim of the probed slot first (one round trip for a new code);
// where the slot already holds the code, the larger position is kept by a 64-bit atomicMax
// (both words carry the same code in their high half), which nothing waits for.
__device__ __forceinline__ bool lt_put(uint64_t* tab, uint32_t mask, uint32_t code, int32_t pos) {
  const unsigned long long want = lt_word(code, pos);
  uint32_t i = fmix32(code) & mask;
  for (uint32_t probe = 0; probe <= mask; ++probe, i = (i + 1) & mask) {
    unsigned long long* slot = reinterpret_cast<unsigned long long*>(tab + i);
    const unsigned long long old = atomicCAS(slot, 0ull, want);
    if (old == 0) return true;
    if (static_cast<uint32_t>(old >> 32) == code) {
      atomicMax(slot, want);
      return true;
    }
  }
  return false;
}

constexpr int kSweepPer = 2;  // positions (and LT entries) per thread per segment: seg_len <= 8192

__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kSweepThreads)
    sweep_kernel(const SweepParams p) {
  const int64_t h = blockIdx.x / kClusterCtas;
  const int t = static_cast<int>(cluster_rank()) * kSweepThreads + threadIdx.x;
  constexpr int kStride = kClusterCtas * kSweepThreads;
  uint64_t* tab = p.table + h * p.slots;
  const uint32_t mask = static_cast<uint32_t>(p.slots - 1);
  const uint32_t* qc = p.qc + h * p.L;
  int32_t* src = p.src + h * p.L;
  // the next segment's inputs, loaded one segment ahead: query index and code, the LT count
  // and this thread's LT entries (entries past the count are read but never used)
  int32_t ns[kSweepPer], np_[kSweepPer], ncnt = 0;
  uint32_t nq[kSweepPer], nc[kSweepPer];
  auto load = [&](int64_t seg) {
    const int64_t s0 = seg * p.seg_len;
    const int64_t st = h * p.n_seg + seg;
    ncnt = p.lt_count[st];
#pragma unroll
    for (int k = 0; k < kSweepPer; ++k) {
      const int64_t i = t + int64_t(k) * kStride;
      const bool in = i < p.seg_len;
      ns[k] = in ? src[s0 + i] : 0;
      nq[k] = in ? qc[s0 + i] : 0;
      nc[k] = in ? p.lt_code[st * p.seg_len + i] : 0;
      np_[k] = in ? p.lt_pos[st * p.seg_len + i] : 0;
    }
  };
  if (p.n_seg > 0) load(0);
  for (int64_t seg = 0; seg < p.n_seg; ++seg) {
    const int64_t s0 = seg * p.seg_len;
    const int64_t g0 = p.base + (h % p.vrows) * p.L + s0;
    int32_t cs[kSweepPer], cp[kSweepPer];
    uint32_t cq[kSweepPer], cc[kSweepPer];
    const int32_t cnt = ncnt;
#pragma unroll
    for (int k = 0; k < kSweepPer; ++k) {
      cs[k] = ns[k];
      cq[k] = nq[k];
      cc[k] = nc[k];
      cp[k] = np_[k];
    }
    if (seg + 1 < p.n_seg) load(seg + 1);
    // queries: in-segment hits become global; misses look up the earlier segments. The
    // results are stored after this segment's inserts, so no barrier waits for the stores.
    int32_t res[kSweepPer];
#pragma unroll
    for (int k = 0; k < kSweepPer; ++k) {
      const int64_t i = t + int64_t(k) * kStride;
      res[k] = (i < p.seg_len && cs[k] < 0) ? lt_find(tab, mask, cq[k]) : static_cast<int32_t>(g0 + cs[k]);
    }
    cluster_sync_relaxed();
    // the segment's keys: each distinct code once, at its last position in the segment
#pragma unroll
    for (int k = 0; k < kSweepPer; ++k) {
      const int e = t + k * kStride;
      if (e < cnt && !lt_put(tab, mask, cc[k], static_cast<int32_t>(g0 + cp[k])))
        raise_status(p.status, LEMA_STATUS_TABLE_FULL);
    }
    cluster_sync();
#pragma unroll
    for (int k = 0; k < kSweepPer; ++k) {
      const int64_t i = t + int64_t(k) * kStride;
      if (i < p.seg_len) src[s0 + i] = res[k];
    }
  }
}

// ------------------------------------------------------------------ gather
constexpr int kMaxPeers = 16;  // ranks whose values one peer gather reads
struct GatherParams {
  const int32_t* src;  // [H][L] global positions or -1
  int64_t base, L, H;
  const unsigned char* v;       // [H][L] rows of this shard
  const unsigned char* remote;  // rows fetched from earlier shards
  const int32_t* remote_idx;    // [H][L] row of `remote` for a position before base
  // peer mode (n_peers > 0): rank k's [H][L] values at peers[k] (this GPU's memory or a peer
  // GPU's, mapped into this process); a position before base is read from its owner's rows
  const unsigned char* peers[kMaxPeers];
  int n_peers;
  unsigned char* out;
  uint32_t wpr;        // vector words per row
  uint32_t words;      // words per head = L * wpr (< 2^32)
  int div_shift;       // log2(wpr) when a power of two, else -1
  uint32_t div_magic;  // floor(2^32 / wpr) + 1 when exact for every word index, else 0
  uint32_t* status;
};

constexpr int kGThreads = 256, kGUnroll = 4;  // as the prefill gather: 4 loads in flight measured best

// Word-parallel, like the prefill gather: each CTA owns a run of output words of one head
// (blockIdx.y), kGUnroll loads in flight per thread, consecutive lanes on consecutive words
// of a row, streaming stores.
template <typename Vec>
__global__ void __launch_bounds__(kGThreads) shard_gather_kernel(const GatherParams g) {
  const uint32_t w0 = blockIdx.x * (kGThreads * kGUnroll) + threadIdx.x;
  for (int64_t h = blockIdx.y; h < g.H; h += gridDim.y) {
    const int32_t* src = g.src + h * g.L;
    const int32_t* ridx = g.remote_idx ? g.remote_idx + h * g.L : nullptr;
    const Vec* v = reinterpret_cast<const Vec*>(g.v) + h * static_cast<int64_t>(g.words);
    const Vec* rem = reinterpret_cast<const Vec*>(g.remote);
    Vec* o = reinterpret_cast<Vec*>(g.out) + h * static_cast<int64_t>(g.words);
    Vec val[kGUnroll];
#pragma unroll
    for (int u = 0; u < kGUnroll; ++u) {
      const uint32_t w = w0 + u * kGThreads;
      val[u] = zero_vec<Vec>();
      if (w < g.words) {
        const uint32_t r = g.div_shift >= 0 ? (w >> g.div_shift)
                                            : (g.div_magic ? __umulhi(w, g.div_magic) : w / g.wpr);
        const uint32_t col = w - r * g.wpr;
        const int32_t s = __ldg(src + r);
        if (s >= g.base) {
          val[u] = __ldg(v + (static_cast<int64_t>(s) - g.base) * g.wpr + col);
        } else if (s >= 0 && g.n_peers > 0) {
          // owner = s / L < base / L = this rank; its row h * L + (s - owner * L)
          const uint32_t owner = static_cast<uint32_t>(s) / static_cast<uint32_t>(g.L);
          const Vec* pv = reinterpret_cast<const Vec*>(g.peers[owner]) + h * static_cast<int64_t>(g.words);
          val[u] = pv[(static_cast<int64_t>(s) - static_cast<int64_t>(owner) * g.L) * g.wpr + col];
        } else if (s >= 0) {
          const int32_t ri = ridx ? __ldg(ridx + r) : -1;
          if (ri >= 0)
            val[u] = __ldg(rem + static_cast<int64_t>(ri) * g.wpr + col);
          else if (col == 0)
            raise_status(g.status, LEMA_STATUS_PROBE_LIMIT);  // a remote row nobody fetched
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kGUnroll; ++u) {
      const uint32_t w = w0 + u * kGThreads;
      if (w < g.words) store_stream(o + w, val[u]);
    }
  }
}

template <typename Vec>
int launch_shard_gather(GatherParams g, int64_t vbytes, cudaStream_t stream) {
  const uint64_t wpr = static_cast<uint64_t>(vbytes) / sizeof(Vec);
  const uint64_t words = static_cast<uint64_t>(g.L) * wpr;
  if (words >= (uint64_t(1) << 32)) return fail(LEMA_ERR_INVALID_ARGUMENT, "L * row words = %llu exceeds 2^32", (unsigned long long)words);
  g.wpr = static_cast<uint32_t>(wpr);
  g.words = static_cast<uint32_t>(words);
  g.div_shift = -1;
  g.div_magic = 0;
  if ((wpr & (wpr - 1)) == 0) {
    g.div_shift = log2_exact(wpr);
  } else if (words * wpr < (uint64_t(1) << 32)) {  // multiply-high is exact for w * wpr < 2^32
    g.div_magic = static_cast<uint32_t>(0xFFFFFFFFull / wpr + 1);
  }
  const uint64_t per_cta = kGThreads * kGUnroll;
  const dim3 grid(static_cast<unsigned>((words + per_cta - 1) / per_cta), static_cast<unsigned>(std::min<int64_t>(g.H, 65535)));
  shard_gather_kernel<Vec><<<grid, kGThreads, 0, stream>>>(g);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

int grid_for(int64_t work, int threads, const DeviceInfo& dev, int per_sm = 8) {
  const int64_t want = (work + threads - 1) / threads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(dev.sms) * per_sm)));
}

const DeviceInfo* sm100() {
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return nullptr;
  if (dev->cc_major != 10) {
    fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
    return nullptr;
  }
  return dev;
}

bool pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

}  // namespace k5
}  // namespace lema

using namespace lema;

extern "C" size_t lema_segment_workspace_bytes(int64_t n_streams, int64_t T, int code_bytes) {
  return match_workspace_bytes(n_streams, T, code_bytes, false);
}

extern "C" int lema_segment_match(const void* qcodes, const void* kcodes, int code_bytes, int64_t n_streams,
                                  int64_t T, int32_t* src, void* lt_code, int32_t* lt_pos, int32_t* lt_count,
                                  void* workspace, size_t workspace_bytes, uint32_t* status, void* stream) {
  clear_error();
  if (src == nullptr || lt_code == nullptr || lt_pos == nullptr || lt_count == nullptr)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "src and the three last-occurrence outputs are required");
  MatchLaunch m;
  m.qc = qcodes;
  m.kc = kcodes;
  m.code_bytes = code_bytes;
  m.N = n_streams;
  m.T = T;
  m.src = src;
  m.lt_code = lt_code;
  m.lt_pos = lt_pos;
  m.lt_count = lt_count;
  m.ws = workspace;
  m.ws_bytes = workspace_bytes;
  m.status = status;
  m.stream = static_cast<cudaStream_t>(stream);
  return launch_match(m);
}

extern "C" int64_t lema_lt_table_slots(int64_t max_entries) {
  return static_cast<int64_t>(next_pow2(static_cast<uint64_t>(std::max<int64_t>(64, 2 * max_entries))));
}

extern "C" int lema_lt_insert(uint64_t* table, int64_t n_heads, int64_t slots, const int32_t* heads,
                              const uint32_t* codes, const int32_t* pos, int64_t n, uint32_t* status,
                              void* stream) {
  clear_error();
  if (n_heads <= 0 || !k5::pow2(slots) || slots > (int64_t(1) << 31) || n < 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad table shape (heads %lld, slots %lld) or count", (long long)n_heads, (long long)slots);
  if (n == 0) return LEMA_OK;
  if (table == nullptr || heads == nullptr || codes == nullptr || pos == nullptr)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::InsertParams p{};
  p.table = table;
  p.slots = slots;
  p.n_heads = n_heads;
  p.heads = heads;
  p.codes = codes;
  p.pos = pos;
  p.n = n;
  p.status = status;
  k5::insert_entries_kernel<<<k5::grid_for(n, 256, *dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_lt_resolve(const uint64_t* table, int64_t n_heads, int64_t slots, const uint32_t* qcodes,
                               int32_t* src, int64_t L, void* stream) {
  clear_error();
  if (n_heads <= 0 || !k5::pow2(slots) || slots > (int64_t(1) << 31) || L < 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape (heads %lld, slots %lld, L %lld)", (long long)n_heads,
                (long long)slots, (long long)L);
  if (L == 0) return LEMA_OK;
  if (table == nullptr || qcodes == nullptr || src == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::ResolveParams p{table, slots, n_heads, L, qcodes, src};
  k5::resolve_kernel<<<k5::grid_for(n_heads * L, 256, *dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_lt_resolve_rows(const uint64_t* table, int64_t n_rows, int64_t slots, int64_t vrows,
                                    const uint32_t* qcodes, int32_t* src, int64_t L, void* stream) {
  clear_error();
  if (n_rows <= 0 || !k5::pow2(slots) || slots > (int64_t(1) << 31) || L < 0 || vrows < 1 || n_rows % vrows)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape (rows %lld, slots %lld, rows per head %lld)", (long long)n_rows,
                (long long)slots, (long long)vrows);
  if (L == 0 || vrows == 1) return LEMA_OK;
  if (table == nullptr || qcodes == nullptr || src == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::ResolveRowsParams p{table, slots, n_rows, vrows, L, qcodes, src};
  k5::resolve_rows_kernel<<<k5::grid_for(n_rows * L, 256, *dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_lt_resolve_tables(const uint64_t* const* tables, const int64_t* slots, int n_tables,
                                      int64_t n_heads, const uint32_t* qcodes, int32_t* src, int64_t L,
                                      void* stream) {
  clear_error();
  if (n_tables < 0 || n_heads <= 0 || L < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape");
  if (n_tables == 0 || L == 0) return LEMA_OK;
  if (tables == nullptr || slots == nullptr || qcodes == nullptr || src == nullptr)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::ResolveTablesParams p{tables, slots, n_tables, n_heads, L, qcodes, src};
  k5::resolve_tables_kernel<<<k5::grid_for((n_heads * L + 3) / 4, k5::kResolveThreads, *dev), k5::kResolveThreads, 0,
                              static_cast<cudaStream_t>(stream)>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_lt_extract(const uint64_t* table, int64_t n_heads, int64_t slots, int32_t lo,
                               int32_t* out_heads, uint32_t* out_codes, int32_t* out_pos, int32_t* out_count,
                               int64_t cap, uint32_t* status, void* stream) {
  clear_error();
  if (n_heads <= 0 || !k5::pow2(slots) || cap < 0 || cap >= (int64_t(1) << 31))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad table shape or capacity");
  if (table == nullptr || out_heads == nullptr || out_codes == nullptr || out_pos == nullptr || out_count == nullptr)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::ExtractParams p{table, slots, n_heads, lo, out_heads, out_codes, out_pos, out_count, cap, status};
  LEMA_CUDA_TRY(cudaMemsetAsync(out_count, 0, sizeof(int32_t), static_cast<cudaStream_t>(stream)));
  k5::extract_kernel<<<k5::grid_for(n_heads * slots, 256, *dev), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_shard_sweep(uint64_t* table, int64_t n_heads, int64_t slots, const uint32_t* qcodes,
                                int32_t* src, int64_t L, int64_t seg_len, const uint32_t* lt_code,
                                const int32_t* lt_pos, const int32_t* lt_count, int64_t base, int64_t vrows,
                                uint32_t* status, void* stream) {
  clear_error();
  if (n_heads <= 0 || !k5::pow2(slots) || slots > (int64_t(1) << 31) || L < 0 || seg_len <= 0 || base < 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape (heads %lld, slots %lld, L %lld, segment %lld)",
                (long long)n_heads, (long long)slots, (long long)L, (long long)seg_len);
  if (L % seg_len != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "L = %lld is not whole segments of %lld", (long long)L, (long long)seg_len);
  if (seg_len > int64_t(k5::kClusterCtas) * k5::kSweepThreads * k5::kSweepPer)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "seg_len = %lld: at most %d positions per segment", (long long)seg_len,
                k5::kClusterCtas * k5::kSweepThreads * k5::kSweepPer);
  if (vrows < 1 || n_heads % vrows != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "rows (%lld) must be whole heads of %lld rows", (long long)n_heads, (long long)vrows);
  if (base + vrows * L >= (int64_t(1) << 31) - 1) return fail(LEMA_ERR_INVALID_ARGUMENT, "positions must stay below 2^31 - 1");
  if (L == 0) return LEMA_OK;
  if (table == nullptr || qcodes == nullptr || src == nullptr || lt_code == nullptr || lt_pos == nullptr || lt_count == nullptr)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::SweepParams p{table, slots, qcodes, src, L, seg_len, L / seg_len, base, lt_code, lt_pos, lt_count, status, vrows};
  k5::sweep_kernel<<<static_cast<unsigned>(n_heads * k5::kClusterCtas), k5::kSweepThreads, 0,
                     static_cast<cudaStream_t>(stream)>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

extern "C" int lema_shard_gather_peer(const int32_t* src, int64_t base, const void* const* peer_values,
                                      int n_ranks, int64_t vbytes, void* out, int64_t n_heads, int64_t L,
                                      uint32_t* status, void* stream) {
  clear_error();
  if (n_heads < 0 || L <= 0 || base < 0 || vbytes <= 0 || vbytes % 2 != 0 || base % L != 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape (heads %lld, L %lld, base %lld) or value row of %lld bytes",
                (long long)n_heads, (long long)L, (long long)base, (long long)vbytes);
  const int64_t rank = base / L;
  if (n_ranks < 1 || n_ranks > k5::kMaxPeers || rank >= n_ranks)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "rank %lld of %d ranks (at most %d)", (long long)rank, n_ranks, k5::kMaxPeers);
  if (n_heads == 0) return LEMA_OK;
  if (src == nullptr || peer_values == nullptr || out == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::GatherParams g{};
  g.src = src;
  g.base = base;
  g.L = L;
  g.H = n_heads;
  g.out = static_cast<unsigned char*>(out);
  g.status = status;
  g.n_peers = static_cast<int>(rank) + 1;  // this rank and the earlier ones
  uintptr_t a = reinterpret_cast<uintptr_t>(out) | static_cast<uintptr_t>(vbytes);
  for (int k = 0; k < g.n_peers; ++k) {
    if (peer_values[k] == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "rank %d's values: null pointer", k);
    g.peers[k] = static_cast<const unsigned char*>(peer_values[k]);
    a |= reinterpret_cast<uintptr_t>(peer_values[k]);
  }
  g.v = g.peers[rank];
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (a % 16 == 0) return k5::launch_shard_gather<uint4>(g, vbytes, s);
  if (a % 8 == 0) return k5::launch_shard_gather<uint2>(g, vbytes, s);
  if (a % 4 == 0) return k5::launch_shard_gather<unsigned int>(g, vbytes, s);
  return k5::launch_shard_gather<unsigned short>(g, vbytes, s);
}

// CUDA IPC of one tensor's memory: the handle names the whole allocation holding `ptr`, so
// the exporter also reports ptr's offset in it (allocation base from the driver).
extern "C" int lema_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  clear_error();
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  using GetRange = int (*)(unsigned long long*, size_t*, unsigned long long);
  static GetRange get_range = nullptr;
  if (get_range == nullptr) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || f == nullptr)
      return fail(LEMA_ERR_CUDA, "cuMemGetAddressRange is not available from the driver");
    get_range = reinterpret_cast<GetRange>(f);
  }
  unsigned long long base = 0;
  size_t size = 0;
  if (get_range(&base, &size, reinterpret_cast<unsigned long long>(ptr)) != 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "not device memory of this process");
  cudaIpcMemHandle_t h;
  LEMA_CUDA_TRY(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<unsigned long long>(ptr) - base);
  return LEMA_OK;
}

extern "C" int lema_ipc_import(const void* handle, int64_t offset, void** ptr) {
  clear_error();
  if (handle == nullptr || ptr == nullptr || offset < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "bad argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  LEMA_CUDA_TRY(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<unsigned char*>(base) + offset;
  return LEMA_OK;
}

extern "C" int lema_ipc_close(void* ptr, int64_t offset) {
  clear_error();
  if (ptr == nullptr || offset < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "bad argument");
  LEMA_CUDA_TRY(cudaIpcCloseMemHandle(static_cast<unsigned char*>(ptr) - offset));
  return LEMA_OK;
}

extern "C" int lema_shard_gather(const int32_t* src, int64_t base, const void* values, const void* remote_rows,
                                 const int32_t* remote_idx, int64_t vbytes, void* out, int64_t n_heads, int64_t L,
                                 uint32_t* status, void* stream) {
  clear_error();
  if (n_heads < 0 || L < 0 || base < 0 || vbytes <= 0 || vbytes % 2 != 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape or value row of %lld bytes (positive, even)", (long long)vbytes);
  if (n_heads == 0 || L == 0) return LEMA_OK;
  if (src == nullptr || values == nullptr || out == nullptr || (base > 0 && (remote_idx == nullptr)))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  const DeviceInfo* dev = k5::sm100();
  if (dev == nullptr) return LEMA_ERR_UNSUPPORTED;
  k5::GatherParams g{};
  g.src = src;
  g.base = base;
  g.L = L;
  g.H = n_heads;
  g.v = static_cast<const unsigned char*>(values);
  g.remote = static_cast<const unsigned char*>(remote_rows);
  g.remote_idx = remote_idx;
  g.out = static_cast<unsigned char*>(out);
  g.status = status;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uintptr_t a = reinterpret_cast<uintptr_t>(values) | reinterpret_cast<uintptr_t>(out) |
                      reinterpret_cast<uintptr_t>(remote_rows) | static_cast<uintptr_t>(vbytes);
  if (a % 16 == 0) return k5::launch_shard_gather<uint4>(g, vbytes, s);
  if (a % 8 == 0) return k5::launch_shard_gather<uint2>(g, vbytes, s);
  if (a % 4 == 0) return k5::launch_shard_gather<unsigned int>(g, vbytes, s);
  return k5::launch_shard_gather<unsigned short>(g, vbytes, s);
}
