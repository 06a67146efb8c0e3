// K3 -- the HBM-resident LEMA store and its exchange.
//
// Semantics are those of code/lema/csrc/store.cpp:122-162: one open-addressing table shared
// by every (layer, stream, head) partition, keyed by (group, code); each partition, in
// position order, looks its query up (zeros on a miss) and then inserts its key (latest write
// wins); counts[p] grows by the slots partition p newly claims; a table with no free slot
// left reports "full" instead of growing.
//
// Table layout: cap slots in cap * (16 + row) bytes, row = vbytes rounded up to 16 -- the
// reference's size for the same capacity -- arranged as two arrays:
//   headers  [0, 16 * cap):       per slot code (8 bytes, zero-extended) and state (8 bytes):
//                                 0 = EMPTY, 1 = LOCKED (being claimed), group + 2 = published
//   rows     [16 * cap, ...):     per slot one value row of `row` bytes, opaque
// Headers are dense (eight per 128-byte line), so a probe chain at high load costs a few lines
// instead of one 64-byte round trip per slot. A zero-filled allocation is an empty table. Claims are a compare-and-swap EMPTY -> LOCKED,
// then the code and value are written and the state is published with a release store;
// probers read the state with acquire loads, so a published slot's code and value are
// complete when seen. The home slot is a 64-bit mix of (group, code) mapped onto [0, cap)
// by a multiply-high (Lemire's range reduction), so the capacity is any slot count.
//
// Exchange on the GPU:
//   T == 1 (decode step): every item is its own partition; a group of lanes per item (below)
//           walks its lookup and its insert probes, interleaved round trip by round trip. No
//           ordering between items is needed.
//   T > 1 (prefill chunk): the order inside a partition only matters between equal codes, so
//           the call is decomposed exactly:
//             (1) the matcher (K2) finds each query's latest earlier key INSIDE the chunk and
//                 each key code's last position in the chunk;
//             (2) a query with an in-chunk match copies that value row; any other query
//                 looks the store up (the state before this call);
//             (3) each partition's distinct key codes are inserted once, with the value row
//                 of their last position -- what a position-ordered sequence of overwrites
//                 leaves behind.
//           Kernel boundaries order (2) before (3).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "match.cuh"

namespace lema {
namespace k3 {

constexpr uint64_t kEmpty = 0, kLocked = 1;
constexpr int kThreads = 256;

struct Args {
  unsigned char* table;  // the header array
  unsigned char* rows;   // the row array, table + 16 * cap
  uint64_t cap;
  int64_t stride;        // bytes per row in the row array
  int64_t vbytes;
  const void* qc;
  const void* kc;
  const unsigned char* v;
  unsigned char* out;
  int64_t n, T;
  uint64_t g0;
  int64_t* counts;
  uint32_t* status;
  const int32_t* src;
  const void* lt_code;
  const int32_t* lt_pos;
  const int32_t* lt_count;
  uint64_t seg_groups;  // > 0: groups [k * seg_groups, (k + 1) * seg_groups) have their home
  uint64_t seg_slots;   //   slots in [k * seg_slots, (k + 1) * seg_slots); probing still wraps cap
  // strided value and output rows (heads > 0): item (partition p = b * heads + h, position t)
  // reads its value row at v + b * v_sb + h * v_sh + t * v_st and writes its output row at
  // out + b * o_sb + h * o_sh + t * o_st (bytes); heads = 0: rows of item i at i * vbytes
  int64_t heads, v_sb, v_sh, v_st, o_sb, o_sh, o_st;
  int phase;  // T == 1: 3 = look up then insert, 1 = look up only, 2 = insert only
};

__device__ __forceinline__ int64_t row_off(const Args& a, int64_t p, int64_t t, bool out) {
  if (a.heads == 0) return (p * a.T + t) * a.vbytes;
  const int64_t b = p / a.heads, h = p - b * a.heads;
  return out ? b * a.o_sb + h * a.o_sh + t * a.o_st : b * a.v_sb + h * a.v_sh + t * a.v_st;
}
template <typename Vec>
__device__ __forceinline__ const Vec* v_row(const Args& a, int64_t p, int64_t t) {
  return reinterpret_cast<const Vec*>(a.v + row_off(a, p, t, false));
}
template <typename Vec>
__device__ __forceinline__ Vec* out_row(const Args& a, int64_t p, int64_t t) {
  return reinterpret_cast<Vec*>(a.out + row_off(a, p, t, true));
}

// Home slot of (group, code): a 64-bit mix mapped by multiply-high onto the whole table, or,
// when the table is segmented, onto the group's segment. Probing continues across segment
// ends and wraps at cap either way, so capacity and fullness are those of one shared table;
// segmenting only keeps one layer's exchange (its groups) inside a slice of the table.
__device__ __forceinline__ uint64_t home(uint64_t code, uint64_t group, const Args& a) {
  const uint64_t h = fmix64(code ^ fmix64(group ^ 0x5851F42D4C957F2Dull));
  if (a.seg_groups == 0) return __umul64hi(h, a.cap);
  return (group / a.seg_groups) * a.seg_slots + __umul64hi(h, a.seg_slots);
}

__device__ __forceinline__ uint64_t ld_acquire(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Probing is done by a GROUP of kG = 8 lanes per item: each round trip the group reads the
// next kG consecutive headers (one per lane, 16 bytes each: 128 contiguous bytes) and decides
// with one ballot which slot, in probe order, ends the probe (its entry, or an empty slot).
// A chain of c slots then costs about c / 8 dependent round trips instead of c: at load 0.95
// an unsuccessful linear probe averages ~200 slots. Calls with few items (a batch-1 decode
// step has 64 per layer) use whole warps instead (kWideG = 32 slots per round trip): the
// lanes are there for free; mid-sized calls (a batch-256 decode step: 16384 items per layer)
// use 16 lanes, measured 3.5% faster per step than 32 (fewer waves of warps) and 8% faster
// than 8 (fewer round trips at load 0.65).
constexpr int kG = 8;
constexpr int kWideG = 32;
constexpr int kMidG = 16;
constexpr int64_t kWideMaxItems = 4096;   // up to this many items per call: 32-lane groups
constexpr int64_t kMidMaxItems = 16384;   // up to this many: 16-lane groups

template <int G>
struct Lane {
  int j;           // index in the group
  int gbase;       // the group's first lane in the warp
  unsigned gmask;  // the group's lanes
  __device__ __forceinline__ unsigned bits(unsigned ballot) const {
    return G == 32 ? ballot : (ballot >> gbase) & ((1u << G) - 1u);
  }
};
template <int G>
__device__ __forceinline__ Lane<G> group_lane() {
  const int lane = threadIdx.x & 31;
  const int base = lane & ~(G - 1);
  return Lane<G>{lane & (G - 1), base, G == 32 ? 0xFFFFFFFFu : (((1u << G) - 1u) << base)};
}

__device__ __forceinline__ uint64_t wrap_add(uint64_t s, uint64_t d, uint64_t cap) {
  s += d;
  while (s >= cap) s -= cap;
  return s;
}

__device__ __forceinline__ uint64_t* header(const Args& a, uint64_t s) {
  return reinterpret_cast<uint64_t*>(a.table) + 2 * s;
}
template <typename Vec>
__device__ __forceinline__ Vec* row_of(const Args& a, uint64_t s) {
  return reinterpret_cast<Vec*>(a.rows + s * a.stride);
}
// (code, state) of slot s, through L2: other items of the same launch may claim slots of it
__device__ __forceinline__ void read_header(const Args& a, uint64_t s, uint64_t& code, uint64_t& state) {
  const ulonglong2 h = __ldcg(reinterpret_cast<const ulonglong2*>(header(a, s)));
  code = h.x;
  state = h.y;
}

// The group's lanes copy / zero the row's vector words j, j + G, ...
template <int G, typename Vec>
__device__ __forceinline__ void copy_row_g(Vec* dst, const Vec* src, int wpr, int j) {
  for (int k = j; k < wpr; k += G) dst[k] = src[k];
}
template <int G, typename Vec>
__device__ __forceinline__ void zero_row_g(Vec* dst, int wpr, int j) {
  const Vec z = zero_vec<Vec>();
  for (int k = j; k < wpr; k += G) dst[k] = z;
}

// Copies the value stored under (group, code) into dst, or zeros; all kG lanes of the group
// call it. Returns whether it hit. The first round also reads the home slot's row (rows of up
// to kG vector words), so a hit at home costs one round trip. A slot seen empty ends the
// probe: slots are never freed, so every slot between an entry's home and the entry was
// occupied before this launch (slots other items claim meanwhile only lengthen the scan).
template <int G, typename Vec>
__device__ bool lookup(const Args& a, uint64_t code, uint64_t group, Vec* dst, const Lane<G>& L) {
  const int wpr = static_cast<int>(a.vbytes / static_cast<int64_t>(sizeof(Vec)));
  const uint64_t tag = group + 2;
  uint64_t s = home(code, group, a);
  Vec spec = zero_vec<Vec>();
  if (wpr <= G && L.j < wpr) spec = row_of<const Vec>(a, s)[L.j];
  for (uint64_t t = 0; t < a.cap; t += G) {
    uint64_t cd, st;
    read_header(a, wrap_add(s, L.j, a.cap), cd, st);
    const bool valid = t + L.j < a.cap;  // no slot twice within one cycle of the table
    const unsigned hit = L.bits(__ballot_sync(L.gmask, valid && st == tag && cd == code));
    const unsigned emp = L.bits(__ballot_sync(L.gmask, valid && st == kEmpty));
    const unsigned stop = hit | emp;
    if (stop) {
      const int k = __ffs(stop) - 1;
      if ((hit >> k) & 1u) {
        if (t == 0 && k == 0 && wpr <= G) {
          if (L.j < wpr) dst[L.j] = spec;
        } else {
          copy_row_g<G>(dst, row_of<const Vec>(a, wrap_add(s, k, a.cap)), wpr, L.j);
        }
        return true;
      }
      break;
    }
    s = wrap_add(s, G, a.cap);
  }
  zero_row_g<G>(dst, wpr, L.j);
  return false;
}

// (group, code) -> row, latest write wins; all kG lanes of the group call it. Returns 1 for a
// newly claimed slot, 0 for an overwrite, -1 when every slot was probed (the table is full).
// Only this item inserts this (group, code) in this launch (a decode step's items have
// distinct groups; a chunk inserts each distinct code of a partition once), so an entry seen
// for it was published by an earlier launch. A claim is one compare-and-swap EMPTY -> LOCKED
// by the lane at the slot; the group writes code and row, then that lane publishes the state
// with a release store (cumulative over the group's writes, ordered by the group barrier).
// A lost claim (another item took the slot) continues from the next slot.
template <int G, typename Vec>
__device__ int insert(const Args& a, uint64_t code, uint64_t group, const Vec* row, const Lane<G>& L) {
  const int wpr = static_cast<int>(a.vbytes / static_cast<int64_t>(sizeof(Vec)));
  const uint64_t tag = group + 2;
  uint64_t s = home(code, group, a);
  uint64_t t = 0;
  while (t < a.cap) {
    uint64_t cd, st;
    read_header(a, wrap_add(s, L.j, a.cap), cd, st);
    const bool valid = t + L.j < a.cap;
    const unsigned mine = L.bits(__ballot_sync(L.gmask, valid && st == tag && cd == code));
    const unsigned emp = L.bits(__ballot_sync(L.gmask, valid && st == kEmpty));
    const unsigned stop = mine | emp;
    if (!stop) {
      s = wrap_add(s, G, a.cap);
      t += G;
      continue;
    }
    const int k = __ffs(stop) - 1;
    const uint64_t slot = wrap_add(s, k, a.cap);
    uint64_t* hdr = header(a, slot);
    if ((mine >> k) & 1u) {
      copy_row_g<G>(row_of<Vec>(a, slot), row, wpr, L.j);
      return 0;
    }
    int won = 0;
    if (L.j == k) won = atomicCAS(reinterpret_cast<unsigned long long*>(hdr + 1), kEmpty, kLocked) == kEmpty;
    won = __shfl_sync(L.gmask, won, L.gbase + k);
    if (won) {
      if (L.j == k) hdr[0] = code;
      copy_row_g<G>(row_of<Vec>(a, slot), row, wpr, L.j);
      __syncwarp(L.gmask);
      if (L.j == k) st_release(hdr + 1, tag);
      return 1;
    }
    s = wrap_add(slot, 1, a.cap);
    t += static_cast<uint64_t>(k) + 1;
  }
  return -1;
}

template <typename CodeT>
__device__ __forceinline__ uint64_t load_code(const void* p, int64_t i) {
  return static_cast<uint64_t>(static_cast<const CodeT*>(p)[i]);
}

// T == 1: item i is partition i; look up, then insert. G lanes per item.
template <typename CodeT, typename Vec, int G>
__global__ void __launch_bounds__(kThreads) exchange_step(const Args a) {
  griddep_wait();  // launched as a dependent: the codes and values first
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / G;
  if (i >= a.n) return;  // whole groups
  const Lane<G> L = group_lane<G>();
  const uint64_t g = a.g0 + static_cast<uint64_t>(i);
  if (a.phase & 1) lookup<G, Vec>(a, load_code<CodeT>(a.qc, i), g, out_row<Vec>(a, i, 0), L);
  if (!(a.phase & 2)) return;
  const int r = insert<G, Vec>(a, load_code<CodeT>(a.kc, i), g, v_row<Vec>(a, i, 0), L);
  if (L.j == 0) {
    if (r < 0) {
      raise_status(a.status, LEMA_STATUS_TABLE_FULL);
    } else if (r > 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(a.counts + i), 1ull);
    }
  }
}

// T == 1, both phases with the two probes interleaved: the lookup (query code) and the insert
// (key code) walk independent probe sequences, so each round trip reads the next window of
// both, and a lookup hit away from home loads its row before the insert's claim is issued.
// Same results as exchange_step: the lookup's decisions rest on headers read before this
// item's claim, and where both probes reach the same slot (query code == key code) each lane
// reads the old row word before it writes the new one.
template <typename CodeT, typename Vec, int G>
__global__ void __launch_bounds__(kThreads, 4) exchange_both(const Args a) {
  griddep_wait();  // launched as a dependent: the codes and values first
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / G;
  if (i >= a.n) return;  // whole groups
  const Lane<G> L = group_lane<G>();
  const int wpr = static_cast<int>(a.vbytes / static_cast<int64_t>(sizeof(Vec)));
  const uint64_t g = a.g0 + static_cast<uint64_t>(i);
  const uint64_t tag = g + 2;
  const uint64_t qcode = load_code<CodeT>(a.qc, i), kcode = load_code<CodeT>(a.kc, i);
  Vec* dst = out_row<Vec>(a, i, 0);
  const Vec* src = v_row<Vec>(a, i, 0);
  uint64_t sq = home(qcode, g, a), sk = home(kcode, g, a);
  uint64_t tq = 0, tk = 0;
  const bool one = wpr <= G;  // one vector word per lane at most
  Vec spec = zero_vec<Vec>(), mine_row = zero_vec<Vec>();
  if (one && L.j < wpr) {
    spec = row_of<const Vec>(a, sq)[L.j];
    mine_row = src[L.j];
  }
  bool qdone = false;
  int kres = 2;  // 2: probing; then 1 claimed, 0 overwritten, -1 full
  while (!qdone || kres == 2) {
    uint64_t qcd = 0, qst = 0, kcd = 0, kst = 0;
    if (!qdone) read_header(a, wrap_add(sq, L.j, a.cap), qcd, qst);
    if (kres == 2) read_header(a, wrap_add(sk, L.j, a.cap), kcd, kst);
    bool deferred = false;
    Vec got = zero_vec<Vec>();
    if (!qdone) {
      const bool valid = tq + L.j < a.cap;
      const unsigned hit = L.bits(__ballot_sync(L.gmask, valid && qst == tag && qcd == qcode));
      const unsigned emp = L.bits(__ballot_sync(L.gmask, valid && qst == kEmpty));
      const unsigned stop = hit | emp;
      if (stop) {
        const int k = __ffs(stop) - 1;
        qdone = true;
        if ((hit >> k) & 1u) {
          if (tq == 0 && k == 0 && one) {
            got = spec;
            deferred = true;
          } else if (one) {
            if (L.j < wpr) got = row_of<const Vec>(a, wrap_add(sq, k, a.cap))[L.j];
            deferred = true;
          } else {
            copy_row_g<G>(dst, row_of<const Vec>(a, wrap_add(sq, k, a.cap)), wpr, L.j);
          }
        } else {
          zero_row_g<G>(dst, wpr, L.j);
        }
      } else {
        sq = wrap_add(sq, G, a.cap);
        tq += G;
        if (tq >= a.cap) {
          zero_row_g<G>(dst, wpr, L.j);
          qdone = true;
        }
      }
    }
    if (kres == 2) {
      const bool valid = tk + L.j < a.cap;
      const unsigned mine = L.bits(__ballot_sync(L.gmask, valid && kst == tag && kcd == kcode));
      const unsigned emp = L.bits(__ballot_sync(L.gmask, valid && kst == kEmpty));
      const unsigned stop = mine | emp;
      if (stop) {
        const int k = __ffs(stop) - 1;
        const uint64_t slot = wrap_add(sk, k, a.cap);
        if ((mine >> k) & 1u) {
          if (one) {
            if (L.j < wpr) row_of<Vec>(a, slot)[L.j] = mine_row;
          } else {
            copy_row_g<G>(row_of<Vec>(a, slot), src, wpr, L.j);
          }
          kres = 0;
        } else {
          uint64_t* hdr = header(a, slot);
          int won = 0;
          if (L.j == k) won = atomicCAS(reinterpret_cast<unsigned long long*>(hdr + 1), kEmpty, kLocked) == kEmpty;
          won = __shfl_sync(L.gmask, won, L.gbase + k);
          if (won) {
            if (L.j == k) hdr[0] = kcode;
            if (one) {
              if (L.j < wpr) row_of<Vec>(a, slot)[L.j] = mine_row;
            } else {
              copy_row_g<G>(row_of<Vec>(a, slot), src, wpr, L.j);
            }
            __syncwarp(L.gmask);
            if (L.j == k) st_release(hdr + 1, tag);
            kres = 1;
          } else {
            sk = wrap_add(slot, 1, a.cap);
            tk += static_cast<uint64_t>(k) + 1;
            if (tk >= a.cap) kres = -1;
          }
        }
      } else {
        sk = wrap_add(sk, G, a.cap);
        tk += G;
        if (tk >= a.cap) kres = -1;
      }
    }
    if (deferred && L.j < wpr) dst[L.j] = got;
  }
  if (L.j == 0) {
    if (kres < 0) {
      raise_status(a.status, LEMA_STATUS_TABLE_FULL);
    } else if (kres > 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(a.counts + i), 1ull);
    }
  }
}

// T > 1, phase (2): in-chunk match or store lookup. G lanes per item.
template <typename CodeT, typename Vec, int G>
__global__ void __launch_bounds__(kThreads) exchange_resolve(const Args a) {
  griddep_wait();  // launched as a dependent: the codes and values first
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / G;
  if (i >= a.n) return;
  const Lane<G> L = group_lane<G>();
  const int64_t wpr = a.vbytes / static_cast<int64_t>(sizeof(Vec));
  const int64_t p = i / a.T;
  Vec* dst = out_row<Vec>(a, p, i - p * a.T);
  const int32_t s = a.src[i];
  if (s >= 0) {
    copy_row_g<G>(dst, v_row<Vec>(a, p, s), static_cast<int>(wpr), L.j);
  } else {
    lookup<G, Vec>(a, load_code<CodeT>(a.qc, i), a.g0 + static_cast<uint64_t>(p), dst, L);
  }
}

// T > 1, phase (3): insert each partition's distinct key codes with their last row.
template <typename CodeT, typename Vec, int G>
__global__ void __launch_bounds__(kThreads) exchange_insert(const Args a) {
  griddep_wait();  // launched as a dependent: the codes and values first
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / G;
  if (i >= a.n) return;
  const int64_t p = i / a.T;
  const int64_t e = i - p * a.T;
  if (e >= a.lt_count[p]) return;  // whole groups
  const Lane<G> L = group_lane<G>();
  const int32_t pos = a.lt_pos[i];
  const int r = insert<G, Vec>(a, load_code<CodeT>(a.lt_code, i), a.g0 + static_cast<uint64_t>(p),
                            v_row<Vec>(a, p, pos), L);
  if (L.j == 0) {
    if (r < 0) {
      raise_status(a.status, LEMA_STATUS_TABLE_FULL);
    } else if (r > 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(a.counts + p), 1ull);
    }
  }
}

struct WsLayout {
  size_t src = 0, lt_code = 0, lt_pos = 0, lt_count = 0, match = 0, total = 0;
};

WsLayout layout(int64_t n, int64_t T, int code_bytes) {
  WsLayout w;
  if (T <= 1 || n <= 0) return w;
  const int64_t P = n / T;
  size_t off = 0;
  w.src = off;
  off = round_up(off + 4 * static_cast<size_t>(n), 256);
  w.lt_code = off;
  off = round_up(off + static_cast<size_t>(code_bytes) * n, 256);
  w.lt_pos = off;
  off = round_up(off + 4 * static_cast<size_t>(n), 256);
  w.lt_count = off;
  off = round_up(off + 4 * static_cast<size_t>(P), 256);
  w.match = off;
  off += match_workspace_bytes(P, T, code_bytes);
  w.total = off;
  return w;
}

// LEMA_K3_INTERLEAVE=0 runs a decode step's lookup and insert probes one after the other
// (exchange_step) instead of interleaved (exchange_both); the same results either way.
inline bool interleave() {
  const char* e = std::getenv("LEMA_K3_INTERLEAVE");
  return e == nullptr || e[0] != '0';
}

template <typename CodeT, typename Vec, int G>
int run(Args a, int64_t T, void* ws, size_t ws_bytes, int code_bytes, cudaStream_t stream) {
  const unsigned blocks = static_cast<unsigned>((a.n * G + kThreads - 1) / kThreads);
  if (T == 1) {
    if (a.phase == 3 && interleave())
      LEMA_CUDA_TRY(launch_dependent(exchange_both<CodeT, Vec, G>, dim3(blocks), dim3(kThreads), 0, stream, a));
    else
      LEMA_CUDA_TRY(launch_dependent(exchange_step<CodeT, Vec, G>, dim3(blocks), dim3(kThreads), 0, stream, a));
    return LEMA_OK;
  }
  const WsLayout w = layout(a.n, T, code_bytes);
  unsigned char* base = static_cast<unsigned char*>(ws);
  MatchLaunch m;
  m.qc = a.qc;
  m.kc = a.kc;
  m.code_bytes = code_bytes;
  m.N = a.n / T;
  m.T = T;
  m.src = reinterpret_cast<int32_t*>(base + w.src);
  m.lt_code = base + w.lt_code;
  m.lt_pos = reinterpret_cast<int32_t*>(base + w.lt_pos);
  m.lt_count = reinterpret_cast<int32_t*>(base + w.lt_count);
  m.ws = (ws_bytes > w.match) ? base + w.match : nullptr;
  m.ws_bytes = ws_bytes - w.match;
  m.status = a.status;
  m.stream = stream;
  const int rc = launch_match(m);
  if (rc != LEMA_OK) return rc;
  a.src = m.src;
  a.lt_code = m.lt_code;
  a.lt_pos = m.lt_pos;
  a.lt_count = m.lt_count;
  LEMA_CUDA_TRY(launch_dependent(exchange_resolve<CodeT, Vec, G>, dim3(blocks), dim3(kThreads), 0, stream, a));
  LEMA_CUDA_TRY(launch_dependent(exchange_insert<CodeT, Vec, G>, dim3(blocks), dim3(kThreads), 0, stream, a));
  return LEMA_OK;
}

template <typename CodeT, typename Vec>
int run_g(int G, const Args& a, int64_t T, void* ws, size_t ws_bytes, int code_bytes, cudaStream_t stream) {
  if (G == 32) return run<CodeT, Vec, 32>(a, T, ws, ws_bytes, code_bytes, stream);
  if (G == 16) return run<CodeT, Vec, 16>(a, T, ws, ws_bytes, code_bytes, stream);
  return run<CodeT, Vec, 8>(a, T, ws, ws_bytes, code_bytes, stream);
}

}  // namespace k3

int64_t store_slot_bytes(int64_t vbytes) {
  return 16 + static_cast<int64_t>(round_up(static_cast<size_t>(vbytes), 16));
}

size_t store_workspace_bytes(int64_t n, int64_t T, int code_bytes) {
  return k3::layout(n, T, code_bytes).total;
}

int store_exchange(void* table, int64_t cap, int64_t vbytes, const void* qc, const void* kc,
                   int code_bytes, const void* values, void* out, int64_t n, int64_t T, int64_t g0,
                   int64_t* counts, uint32_t* status, void* ws, size_t ws_bytes,
                   cudaStream_t stream, int64_t seg_groups, int64_t seg_slots, const int64_t* rows,
                   int phase) {
  if (code_bytes != 4 && code_bytes != 8) return fail(LEMA_ERR_INVALID_ARGUMENT, "code_bytes must be 4 or 8, got %d", code_bytes);
  if (vbytes <= 0 || vbytes % 8 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "value row of %lld bytes: vbytes must be a positive multiple of 8", (long long)vbytes);
  if (cap < 1) return fail(LEMA_ERR_INVALID_ARGUMENT, "capacity must be >= 1 slot, got %lld", (long long)cap);
  if (n < 0 || T <= 0 || n % T != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "items must be partitions x T (n = %lld, T = %lld)", (long long)n, (long long)T);
  if (g0 < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "negative group offset");
  if (seg_groups < 0 || seg_slots < 0 || (seg_groups > 0) != (seg_slots > 0))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "segments: groups and slots per segment both positive or both 0");
  if (seg_groups > 0 && n > 0 && ((g0 + n / T - 1) / seg_groups + 1) * seg_slots > cap)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "group %lld's segment lies past the table's %lld slots",
                (long long)(g0 + n / T - 1), (long long)cap);
  if (phase < 1 || phase > 3 || (phase != 3 && T != 1))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "phase %d: 3 (both), or 1 / 2 (lookups / inserts only, T = 1)", phase);
  if (n == 0) return LEMA_OK;
  if (table == nullptr || !aligned(table, 16)) return fail(LEMA_ERR_INVALID_ARGUMENT, "table must be a 16-byte aligned device pointer");
  if (counts == nullptr || ((phase & 1) && (qc == nullptr || out == nullptr)) || ((phase & 2) && (kc == nullptr || values == nullptr)))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned(qc, code_bytes) || !aligned(kc, code_bytes)) return fail(LEMA_ERR_INVALID_ARGUMENT, "codes not aligned to their width");
  if (!aligned(values, 8) || !aligned(out, 8) || !aligned(counts, 8)) return fail(LEMA_ERR_INVALID_ARGUMENT, "values, out and counts must be 8-byte aligned");
  if (phase != 3) {  // the unused side of a split step: any aligned stand-in
    if (qc == nullptr) qc = kc;
    if (kc == nullptr) kc = qc;
    if (values == nullptr) values = out;
    if (out == nullptr) out = const_cast<void*>(values);
  }
  const size_t need = store_workspace_bytes(n, T, code_bytes);
  if (ws_bytes < need || (need > 0 && ws == nullptr)) return fail(LEMA_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", ws_bytes, need);
  if (need > 0 && !aligned(ws, 256)) return fail(LEMA_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  if (rows != nullptr) {
    const int64_t heads = rows[0];
    if (heads <= 0 || (n / T) % heads != 0)
      return fail(LEMA_ERR_INVALID_ARGUMENT, "strided rows: %lld partitions are not whole groups of heads = %lld",
                  (long long)(n / T), (long long)heads);
    for (int k = 1; k < 7; ++k)
      if (rows[k] % 8 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "strided rows: strides must be multiples of 8 bytes");
  }
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);

  k3::Args a{};
  a.phase = phase;
  if (rows != nullptr) {
    a.heads = rows[0];
    a.v_sb = rows[1]; a.v_sh = rows[2]; a.v_st = rows[3];
    a.o_sb = rows[4]; a.o_sh = rows[5]; a.o_st = rows[6];
  }
  a.table = static_cast<unsigned char*>(table);
  a.cap = static_cast<uint64_t>(cap);
  a.rows = a.table + 16 * a.cap;
  a.stride = store_slot_bytes(vbytes) - 16;
  a.vbytes = vbytes;
  a.qc = qc;
  a.kc = kc;
  a.v = static_cast<const unsigned char*>(values);
  a.out = static_cast<unsigned char*>(out);
  a.n = n;
  a.T = T;
  a.g0 = static_cast<uint64_t>(g0);
  a.counts = counts;
  a.status = status;
  a.seg_groups = static_cast<uint64_t>(seg_groups);
  a.seg_slots = static_cast<uint64_t>(seg_slots);
  const uint64_t st = rows ? static_cast<uint64_t>(rows[1] | rows[2] | rows[3] | rows[4] | rows[5] | rows[6]) : 0;
  const bool v16 = vbytes % 16 == 0 && st % 16 == 0 && aligned(values, 16) && aligned(out, 16);
  // LEMA_K3_WIDE_MAX overrides the item count up to which 32-lane groups probe (same results)
  int64_t wide_max = k3::kWideMaxItems;
  if (const char* e = std::getenv("LEMA_K3_WIDE_MAX")) wide_max = std::atoll(e);
  int G = n <= wide_max ? k3::kWideG : (n <= k3::kMidMaxItems ? k3::kMidG : k3::kG);
  // LEMA_K3_GROUP=8/16/32 sets the lanes per item for every call (same results)
  if (const char* e = std::getenv("LEMA_K3_GROUP")) {
    const int g = std::atoi(e);
    if (g == 8 || g == 16 || g == 32) G = g;
  }
  if (code_bytes == 4) {
    if (v16) return k3::run_g<uint32_t, uint4>(G, a, T, ws, ws_bytes, code_bytes, stream);
    return k3::run_g<uint32_t, uint2>(G, a, T, ws, ws_bytes, code_bytes, stream);
  }
  if (v16) return k3::run_g<uint64_t, uint4>(G, a, T, ws, ws_bytes, code_bytes, stream);
  return k3::run_g<uint64_t, uint2>(G, a, T, ws, ws_bytes, code_bytes, stream);
}

}  // namespace lema
