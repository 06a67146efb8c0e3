// K2 -- latest exact match over position-ordered streams, and the value gather.
//
// For stream n and position i:  src[n][i] = max{ j < i : kc[n][j] == qc[n][i] } or -1,
// out[n][i] = v[n][src] (zeros when -1). This is the rule of code/lema/attention.py:100-158,
// which the reference computes with two stable argsorts over 2T events per stream; here it is
// one pass in position order with a hash table of the stream's key codes in shared memory.
//
// One CTA owns one stream at a time (persistent grid-stride over streams) and walks it in
// chunks of kChunk positions through a three-stage pipeline of warp roles; stage boundaries are
// CTA-wide barriers ("rounds"), and in round r:
//
//   preparers (7 warps) -- chunk r
//     1. insert  the chunk's key codes (loaded in one batch) are inserted into -- or found in --
//                the stream's table, giving each a SLOT id. Equal codes of a warp are first
//                deduplicated with match_any, so one lane per distinct code touches the table.
//     2. lookup  each query code is looked up; a code that no key up to the end of this chunk
//                has used gets no slot, and -1 is already its final answer.
//     3. in-step inside each 32-position step, the latest key lane j < i with the query's
//                slot (32 shuffles), and whether each key lane is the last of its slot.
//   sweeper (1 warp) -- chunk r-1, the only ordered part: 32 positions per step, a query with
//                an in-step match takes it, any other reads meta[slot] (the position of the
//                latest key of its slot swept so far); then the last key lane of each slot
//                writes its position into meta[slot]. Two __syncwarp()s per step order the
//                reads before the step's writes and the writes before the next step's reads.
//   gatherers (8 warps) -- chunk r-2: indices out, value rows copied with 16-byte vectors,
//                eight loads in flight per thread, streaming stores; zeros for misses.
//
// The stages touch the table without conflict: inserts only claim free words, lookups compare
// codes only, and the sweep writes the position half of words claimed in earlier rounds.
//
// The shared-memory table has a fixed capacity (kSmemCap slots). A stream whose distinct key
// codes would load it beyond kOverflowFrac is handed over whole to the same kernel running
// with a CTA-private table in global memory sized 2*T (the overflow path): it appends itself
// to an overflow list in the workspace, and a second launch processes the list. No input
// can make the result wrong; an unusual one only takes the slower path.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "match.cuh"

namespace lema {
namespace k2 {

constexpr int kThreads = 512;
constexpr int kChunk = 2048;
constexpr int kSweepWarp = 0;                        // warp 0: the ordered sweep
constexpr int kPrepWarp0 = 1, kPrepWarps = 7;        // warps 1..7: insert / lookup / in-step
constexpr int kGathWarp0 = 8, kGathWarps = 8;        // warps 8..15: indices and rows out
constexpr int kPrepThreads = kPrepWarps * 32;
constexpr int kGathThreads = kGathWarps * 32;
constexpr int kPerPrep = (kChunk + kPrepThreads - 1) / kPrepThreads;
constexpr int kGatherUnroll = 8;
constexpr int kMini = 64;  // per-warp code -> lane-mask hash of one step's key codes
static_assert((kPrepWarp0 + kPrepWarps) * 32 <= kThreads && kGathWarp0 * 32 + kGathThreads == kThreads, "roles");

constexpr uint32_t kEmpty = 0xFFFFFFFFu;   // meta of a free slot
constexpr uint32_t kLocked = 0xFFFFFFFEu;  // meta of a slot being claimed (64-bit codes only)
constexpr uint32_t kNone = 0xFFFFFFFDu;    // code present, no key position swept yet
constexpr uint32_t kNoSlot = 0xFFFFFFFFu;  // query code absent from the table
constexpr uint32_t kBadKey = 0xFFFFFFFEu;  // key slot of an out-of-range lane
constexpr uint32_t kInStep = 0x80000000u;  // query slot word: in-step match, lane in low bits
constexpr uint32_t kSpinLimit = 1u << 22;  // bound on waiting for a LOCKED slot

// Shared-memory table capacity (slots) per code width, and the load above which a stream
// moves to the global-memory path.
template <typename CodeT>
struct SmemCap;
template <>
struct SmemCap<uint32_t> {
  static constexpr uint32_t kLog2 = 13;
};
template <>
struct SmemCap<uint64_t> {
  static constexpr uint32_t kLog2 = 12;
};
constexpr double kOverflowFrac = 0.75;

template <typename CodeT>
__host__ __device__ constexpr uint32_t overflow_limit() {
  return static_cast<uint32_t>((1u << SmemCap<CodeT>::kLog2) * kOverflowFrac);
}

// ---------------------------------------------------------------- the tables
// Slot -> (code, meta). meta is kEmpty, kLocked, kNone, or the stream position of the latest
// key with that code swept so far.
template <typename CodeT>
struct Table;

// 32-bit codes: one 64-bit word per slot, code in the low half and meta in the high half, so
// a claim is a single compare-and-swap of an all-ones (free) word and no reader ever waits.
template <>
struct Table<uint32_t> {
  unsigned long long* w;
  uint32_t mask;
  static constexpr size_t kBytesPerSlot = 8;

  __device__ void init(void* base, uint32_t cap) {
    w = static_cast<unsigned long long*>(base);
    mask = cap - 1;
  }
  __device__ void clear(int tid, int nthr) {
    for (uint32_t s = tid; s <= mask; s += nthr) w[s] = ~0ull;
  }
  __device__ uint32_t* meta(uint32_t s) const { return reinterpret_cast<uint32_t*>(w + s) + 1; }
  __device__ bool used(uint32_t s, uint32_t& code, uint32_t& m) const {
    const unsigned long long x = w[s];
    code = static_cast<uint32_t>(x);
    m = static_cast<uint32_t>(x >> 32);
    return x != ~0ull;
  }
  // Insert-or-find. Returns the slot, or kNoSlot when every slot was probed.
  __device__ uint32_t insert(uint32_t code, uint32_t& claimed, uint32_t*) {
    const unsigned long long fresh =
        static_cast<unsigned long long>(code) | (static_cast<unsigned long long>(kNone) << 32);
    uint32_t s = code_hash32(code) & mask;
    for (uint32_t n = 0; n <= mask; ++n, s = (s + 1) & mask) {
      unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(w + s);
      if (cur == ~0ull) {
        cur = atomicCAS(w + s, ~0ull, fresh);
        if (cur == ~0ull) {
          claimed = 1;
          return s;
        }
      }
      if (static_cast<uint32_t>(cur) == code) return s;
    }
    return kNoSlot;
  }
  // Find after a barrier that ended all inserts of this chunk (the sweep may be writing
  // position halves meanwhile; codes never change once claimed).
  __device__ uint32_t find(uint32_t code) const {
    uint32_t s = code_hash32(code) & mask;
    for (uint32_t n = 0; n <= mask; ++n, s = (s + 1) & mask) {
      const unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(w + s);
      if (cur == ~0ull) return kNoSlot;
      if (static_cast<uint32_t>(cur) == code) return s;
    }
    return kNoSlot;
  }
};

// 64-bit codes: codes and metas in two arrays. A claim CASes meta kEmpty -> kLocked, writes
// the code, then publishes kNone; a prober that meets kLocked waits (bounded) for it.
template <>
struct Table<uint64_t> {
  unsigned long long* code;
  uint32_t* m;
  uint32_t mask;
  static constexpr size_t kBytesPerSlot = 12;

  __device__ void init(void* base, uint32_t cap) {
    code = static_cast<unsigned long long*>(base);
    m = reinterpret_cast<uint32_t*>(code + cap);
    mask = cap - 1;
  }
  __device__ void clear(int tid, int nthr) {
    for (uint32_t s = tid; s <= mask; s += nthr) m[s] = kEmpty;
  }
  __device__ uint32_t* meta(uint32_t s) const { return m + s; }
  __device__ bool used(uint32_t s, uint64_t& c, uint32_t& mm) const {
    mm = m[s];
    c = code[s];
    return mm != kEmpty;
  }
  __device__ uint32_t insert(uint64_t c, uint32_t& claimed, uint32_t* status) {
    uint32_t s = code_hash32(c) & mask;
    for (uint32_t n = 0; n <= mask; ++n, s = (s + 1) & mask) {
      uint32_t cur = *reinterpret_cast<volatile uint32_t*>(m + s);
      if (cur == kEmpty) {
        cur = atomicCAS(m + s, kEmpty, kLocked);
        if (cur == kEmpty) {
          *reinterpret_cast<volatile unsigned long long*>(code + s) = c;
          __threadfence_block();
          atomicExch(m + s, kNone);
          claimed = 1;
          return s;
        }
      }
      if (cur == kLocked) {
        uint32_t k = 0;
        while ((cur = *reinterpret_cast<volatile uint32_t*>(m + s)) == kLocked && ++k < kSpinLimit) {
        }
        if (cur == kLocked) {
          raise_status(status, LEMA_STATUS_PROBE_LIMIT);
          return kNoSlot;
        }
      }
      __threadfence_block();
      if (*reinterpret_cast<volatile unsigned long long*>(code + s) == c) return s;
    }
    return kNoSlot;
  }
  __device__ uint32_t find(uint64_t c) const {
    uint32_t s = code_hash32(c) & mask;
    for (uint32_t n = 0; n <= mask; ++n, s = (s + 1) & mask) {
      if (*reinterpret_cast<volatile uint32_t*>(m + s) == kEmpty) return kNoSlot;
      if (code[s] == c) return s;
    }
    return kNoSlot;
  }
};

// ---------------------------------------------------------------- the kernel
struct Params {
  const void* qc;
  const void* kc;
  int64_t N, T;
  int32_t* src;
  const unsigned char* v;
  unsigned char* out;
  int64_t vbytes;
  void* lt_code;
  int32_t* lt_pos;
  int32_t* lt_count;
  uint32_t* status;
  // overflow bookkeeping (workspace)
  uint32_t* ovf_count;
  uint32_t* ovf_list;
  // global-memory tables (overflow path): one per CTA
  unsigned char* gtables;
  int64_t gtable_bytes;
  uint32_t gcap_log2;
  int list_mode;  // global path: 1 = streams from ovf_list, 0 = all streams
  int div_shift;       // log2(words per row) when a power of two, else -1
  uint32_t div_magic;  // floor(2^32 / words per row) + 1 when usable, else 0
};

template <typename CodeT>
__device__ __forceinline__ uint32_t mini_hash(CodeT c) {
  return code_hash32(c) >> (32 - 6);  // top bits: independent of the table's low-bit home
}
static_assert(kMini == 64, "mini_hash yields 6 bits");

__device__ __forceinline__ void prep_barrier() {
  asm volatile("bar.sync 1, %0;" ::"n"(kPrepThreads) : "memory");
}

// Gatherers: indices of one chunk to global memory, then its value rows, kGatherUnroll vector
// loads in flight per thread before the streaming stores.
template <typename Vec>
__device__ __forceinline__ void gather_chunk(const Params& p, int64_t row0, int64_t base, int cnt,
                                             const int32_t* src_s, int gtid) {
  if (p.src != nullptr) {
    for (int i = gtid; i < cnt; i += kGathThreads) p.src[row0 + base + i] = src_s[i];
  }
  if (p.out == nullptr) return;
  const int wpr = static_cast<int>(p.vbytes / static_cast<int64_t>(sizeof(Vec)));
  const int total = cnt * wpr;
  const Vec* v = reinterpret_cast<const Vec*>(p.v) + row0 * wpr;
  Vec* o = reinterpret_cast<Vec*>(p.out) + (row0 + base) * wpr;
  // row of word w: a shift for power-of-two rows, else a multiply-high by a magic reciprocal
  // (exact for w * wpr < 2^32, which the host guarantees), else a division
  const int dshift = p.div_shift;
  const uint32_t dmagic = p.div_magic;
  for (int w0 = gtid; w0 < total; w0 += kGathThreads * kGatherUnroll) {
    Vec val[kGatherUnroll];
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      const int w = w0 + u * kGathThreads;
      val[u] = zero_vec<Vec>();
      if (w < total) {
        const int r = dshift >= 0 ? (w >> dshift)
                                  : (dmagic ? static_cast<int>(__umulhi(static_cast<uint32_t>(w), dmagic))
                                            : w / wpr);
        const int32_t s = src_s[r];
        if (s >= 0) val[u] = __ldg(v + static_cast<int64_t>(s) * wpr + (w - r * wpr));
      }
    }
#pragma unroll
    for (int u = 0; u < kGatherUnroll; ++u) {
      const int w = w0 + u * kGathThreads;
      if (w < total) store_stream(o + w, val[u]);
    }
  }
}

template <typename CodeT, bool kSmemTable, typename Vec>
__global__ void __launch_bounds__(kThreads) match_kernel(const Params p) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr uint32_t kCap = 1u << SmemCap<CodeT>::kLog2;
  const size_t table_bytes = kSmemTable ? kCap * Table<CodeT>::kBytesPerSlot : 0;
  uint32_t* kbuf = reinterpret_cast<uint32_t*>(smem + table_bytes);  // [2][kChunk] key slots
  uint32_t* qbuf = kbuf + 2 * kChunk;                                // [2][kChunk] query words
  int32_t* sbuf = reinterpret_cast<int32_t*>(qbuf + 2 * kChunk);     // [2][kChunk] src
  CodeT* mini_key = reinterpret_cast<CodeT*>(sbuf + 2 * kChunk);      // [kPrepWarps][kMini]
  uint32_t* mini_mask = reinterpret_cast<uint32_t*>(mini_key + kPrepWarps * kMini);
  __shared__ uint32_t s_used, s_ovf, s_abort, s_lt;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const CodeT* qc = static_cast<const CodeT*>(p.qc);
  const CodeT* kc = static_cast<const CodeT*>(p.kc);

  Table<CodeT> tab;
  if (kSmemTable) {
    tab.init(smem, kCap);
  } else {
    tab.init(p.gtables + static_cast<int64_t>(blockIdx.x) * p.gtable_bytes, 1u << p.gcap_log2);
  }
  for (int i = tid; i < kPrepWarps * kMini; i += kThreads) mini_mask[i] = 0u;  // 0 = free entry
  const int64_t n_work = (!kSmemTable && p.list_mode) ? static_cast<int64_t>(*p.ovf_count) : p.N;
  const int64_t n_chunks = (p.T + kChunk - 1) / kChunk;

  for (int64_t wi = blockIdx.x; wi < n_work; wi += gridDim.x) {
    const int64_t n = (!kSmemTable && p.list_mode) ? static_cast<int64_t>(p.ovf_list[wi]) : wi;
    const int64_t row0 = n * p.T;
    tab.clear(tid, kThreads);
    if (tid == 0) {
      s_used = 0;
      s_ovf = 0;
      s_abort = 0;
      s_lt = 0;
    }
    __syncthreads();

    bool aborted = false;
    for (int64_t r = 0; r < n_chunks + 2; ++r) {
      if (warp >= kPrepWarp0 && warp < kPrepWarp0 + kPrepWarps && r < n_chunks) {
        // ------------------------------------------------ preparers: chunk r
        const int ptid = tid - kPrepWarp0 * 32;
        const int pwarp = warp - kPrepWarp0;
        const int64_t base = r * kChunk;
        const int cnt = static_cast<int>(min(static_cast<int64_t>(kChunk), p.T - base));
        const int cnt32 = (cnt + 31) & ~31;
        uint32_t* kb = kbuf + (r & 1) * kChunk;
        uint32_t* qb = qbuf + (r & 1) * kChunk;
        CodeT* mkey = mini_key + pwarp * kMini;
        uint32_t* mmask = mini_mask + pwarp * kMini;
        CodeT kr[kPerPrep], qr[kPerPrep];
#pragma unroll
        for (int u = 0; u < kPerPrep; ++u) {
          const int i = ptid + u * kPrepThreads;
          kr[u] = i < cnt ? kc[row0 + base + i] : CodeT(0);
          qr[u] = i < cnt ? qc[row0 + base + i] : CodeT(0);
        }
        // 1. One aligned 32-position step per warp-iteration. The lanes holding one key code
        //    (match_any) elect their lowest lane, which inserts the code into the table and
        //    publishes code -> lane mask in the warp's 64-entry mini hash; each query lane
        //    then finds the latest key lane j < i of its code in the step, if any.
        uint32_t qpend = 0;  // bit u: the query of iteration u needs a table lookup
#pragma unroll
        for (int u = 0; u < kPerPrep; ++u) {
          const int i = ptid + u * kPrepThreads;
          if (i < cnt32) {  // uniform per warp: a warp covers an aligned run of 32 positions
            const bool valid = i < cnt;
            const uint32_t vm = __ballot_sync(kFullMask, valid);
            uint32_t mine = kMini;  // mini-hash entry this lane claimed
            if (valid) {
              const uint32_t peers = __match_any_sync(vm, kr[u]);
              const int leader = __ffs(peers) - 1;
              uint32_t slot = kNoSlot, claimed = 0;
              if (lane == leader) {
                slot = tab.insert(kr[u], claimed, p.status);
                if (claimed) atomicAdd(&s_used, 1u);
                if (slot == kNoSlot) s_ovf = 1;
                uint32_t h = mini_hash(kr[u]);
                for (int t = 0; t < kMini; ++t, h = (h + 1) & (kMini - 1)) {
                  if (atomicCAS(mmask + h, 0u, peers) == 0u) {
                    mkey[h] = kr[u];
                    mine = h;
                    break;
                  }
                }
              }
              slot = __shfl_sync(vm, slot, leader);
              kb[i] = ((peers >> lane) == 1u) ? slot : kNoSlot;  // last key lane of its code
            }
            __syncwarp();
            if (valid) {
              uint32_t mm = 0;
              uint32_t h = mini_hash(qr[u]);
              for (int t = 0; t < kMini; ++t, h = (h + 1) & (kMini - 1)) {
                const uint32_t m = mmask[h];
                if (m == 0u) break;
                if (mkey[h] == qr[u]) {
                  mm = m & lanemask_lt();
                  break;
                }
              }
              if (mm) {
                qb[i] = kInStep | (31u - __clz(mm));
              } else {
                qpend |= 1u << u;
              }
            }
            __syncwarp();
            if (mine < kMini) mmask[mine] = 0u;
            __syncwarp();
          }
        }
        prep_barrier();
        if (s_ovf != 0 || (kSmemTable && s_used > overflow_limit<CodeT>())) {
          if (ptid == 0) s_abort = 1;
        } else {
          // 2. queries without an in-step match read their code's slot (or none: then no key
          //    of the code has appeared up to the end of this chunk, and the answer is -1)
#pragma unroll
          for (int u = 0; u < kPerPrep; ++u) {
            if ((qpend >> u) & 1u) qb[ptid + u * kPrepThreads] = tab.find(qr[u]);
          }
        }
      } else if (warp == kSweepWarp && r >= 1 && r <= n_chunks) {
        // ------------------------------------------------ sweeper: chunk r-1, in order
        const int64_t c = r - 1;
        const int64_t base = c * kChunk;
        const int cnt = static_cast<int>(min(static_cast<int64_t>(kChunk), p.T - base));
        const int nsteps = (cnt + 31) >> 5;
        const uint32_t* kb = kbuf + (c & 1) * kChunk;
        const uint32_t* qb = qbuf + (c & 1) * kChunk;
        int32_t* sb = sbuf + (c & 1) * kChunk;
        uint32_t qn = kNoSlot, kn = kNoSlot;
        if (lane < cnt) {
          qn = qb[lane];
          kn = kb[lane];
        }
        for (int s = 0; s < nsteps; ++s) {
          const int i = s * 32 + lane;
          const bool valid = i < cnt;
          const uint32_t qv = qn, kv = kn;
          if (i + 32 < cnt) {
            qn = qb[i + 32];
            kn = kb[i + 32];
          }
          int32_t sv = -1;
          if (valid && qv != kNoSlot) {
            if (qv & kInStep) {
              sv = static_cast<int32_t>(base + s * 32 + static_cast<int>(qv & 31u));
            } else {
              const uint32_t m = *reinterpret_cast<volatile uint32_t*>(tab.meta(qv));
              sv = (m == kNone) ? -1 : static_cast<int32_t>(m);
            }
          }
          if (valid) sb[i] = sv;
          __syncwarp();
          if (valid && kv != kNoSlot) {
            *reinterpret_cast<volatile uint32_t*>(tab.meta(kv)) = static_cast<uint32_t>(base + i);
          }
          __syncwarp();
        }
      } else if (warp >= kGathWarp0 && r >= 2) {
        // ------------------------------------------------ gatherers: chunk r-2
        const int64_t c = r - 2;
        const int64_t base = c * kChunk;
        const int cnt = static_cast<int>(min(static_cast<int64_t>(kChunk), p.T - base));
        gather_chunk<Vec>(p, row0, base, cnt, sbuf + (c & 1) * kChunk, tid - kGathWarp0 * 32);
      }
      __syncthreads();
      if (s_abort != 0) {
        aborted = true;
        break;
      }
    }

    if (aborted) {
      if (tid == 0) {
        if (kSmemTable) {
          const uint32_t k = atomicAdd(p.ovf_count, 1u);
          p.ovf_list[k] = static_cast<uint32_t>(n);
        } else {
          // a global table holds 2T slots, so this cannot happen; report, never loop
          raise_status(p.status, LEMA_STATUS_PROBE_LIMIT);
        }
      }
      __syncthreads();
      continue;
    }

    // last-occurrence table: every key code of the stream with its last position
    if (p.lt_count != nullptr) {
      CodeT* ltc = static_cast<CodeT*>(p.lt_code) + row0;
      int32_t* ltp = p.lt_pos + row0;
      for (uint32_t s = tid; s <= tab.mask; s += kThreads) {
        CodeT c;
        uint32_t m;
        if (tab.used(s, c, m) && m < kNone) {
          const uint32_t k = atomicAdd(&s_lt, 1u);
          ltc[k] = c;
          ltp[k] = static_cast<int32_t>(m);
        }
      }
      __syncthreads();
      if (tid == 0) p.lt_count[n] = static_cast<int32_t>(s_lt);
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------- host side
constexpr size_t kChunkSmem = 6 * kChunk * sizeof(uint32_t);
constexpr int64_t kMaxOverflowTables = 64;
constexpr uint64_t kOverflowTableBudget = uint64_t(1) << 30;  // bytes of global tables
constexpr int64_t kFastMaxT = int64_t(1) << 20;               // beyond: global path directly

template <typename CodeT>
size_t smem_bytes(bool smem_table) {
  return (smem_table ? (size_t(1) << SmemCap<CodeT>::kLog2) * Table<CodeT>::kBytesPerSlot : 0) +
         kChunkSmem + kPrepWarps * kMini * (sizeof(CodeT) + sizeof(uint32_t));
}

struct Plan {
  bool fast = false;       // run the shared-memory kernel
  bool global = false;     // run the global-table kernel
  bool list_mode = false;  // global kernel reads the overflow list
  uint32_t gcap_log2 = 0;
  int64_t gtable_bytes = 0;
  int64_t n_gtables = 0;
  size_t off_list = 0, off_tables = 0, total = 0;
};

Plan make_plan(int64_t N, int64_t T, int code_bytes) {
  Plan pl;
  if (N <= 0 || T <= 0) return pl;
  const uint32_t limit = code_bytes == 4 ? overflow_limit<uint32_t>() : overflow_limit<uint64_t>();
  pl.fast = T <= kFastMaxT;
  const bool may_overflow = !pl.fast || T > static_cast<int64_t>(limit);
  if (!may_overflow) return pl;
  pl.global = true;
  pl.list_mode = pl.fast;
  const uint64_t cap = next_pow2(static_cast<uint64_t>(2 * T));
  pl.gcap_log2 = static_cast<uint32_t>(log2_exact(cap));
  const size_t per_slot = code_bytes == 4 ? Table<uint32_t>::kBytesPerSlot : Table<uint64_t>::kBytesPerSlot;
  pl.gtable_bytes = static_cast<int64_t>(round_up(cap * per_slot, 256));
  pl.n_gtables = std::max<int64_t>(
      1, std::min<int64_t>({N, kMaxOverflowTables,
                            static_cast<int64_t>(kOverflowTableBudget / pl.gtable_bytes)}));
  pl.off_list = 256;
  pl.off_tables = round_up(pl.off_list + 4 * static_cast<size_t>(N), 256);
  pl.total = pl.off_tables + static_cast<size_t>(pl.n_gtables * pl.gtable_bytes);
  return pl;
}

template <typename CodeT, typename Vec>
int run(const MatchLaunch& a, const Plan& pl, const DeviceInfo& dev) {
  Params p{};
  p.qc = a.qc;
  p.kc = a.kc;
  p.N = a.N;
  p.T = a.T;
  p.src = a.src;
  p.v = static_cast<const unsigned char*>(a.v);
  p.out = static_cast<unsigned char*>(a.out);
  p.vbytes = a.vbytes;
  p.lt_code = a.lt_code;
  p.lt_pos = a.lt_pos;
  p.lt_count = a.lt_count;
  p.status = a.status;
  {
    const int64_t wpr = a.out ? a.vbytes / static_cast<int64_t>(sizeof(Vec)) : 1;
    p.div_shift = -1;
    p.div_magic = 0;
    if ((wpr & (wpr - 1)) == 0) {
      p.div_shift = log2_exact(static_cast<uint64_t>(wpr));
    } else if (static_cast<uint64_t>(kChunk) * wpr * wpr < (uint64_t(1) << 32)) {
      p.div_magic = static_cast<uint32_t>(0xFFFFFFFFull / static_cast<uint64_t>(wpr) + 1);
    }
  }
  unsigned char* ws = static_cast<unsigned char*>(a.ws);
  if (pl.global) {
    p.ovf_count = reinterpret_cast<uint32_t*>(ws);
    p.ovf_list = reinterpret_cast<uint32_t*>(ws + pl.off_list);
    p.gtables = ws + pl.off_tables;
    p.gtable_bytes = pl.gtable_bytes;
    p.gcap_log2 = pl.gcap_log2;
    if (pl.list_mode) LEMA_CUDA_TRY(cudaMemsetAsync(p.ovf_count, 0, sizeof(uint32_t), a.stream));
  }
  if (pl.fast) {
    auto kern = match_kernel<CodeT, true, Vec>;
    const size_t sm = smem_bytes<CodeT>(true);
    LEMA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm)));
    int per_sm = 0;
    LEMA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, sm));
    const int64_t grid = std::min<int64_t>(a.N, static_cast<int64_t>(std::max(per_sm, 1)) * dev.sms);
    kern<<<static_cast<unsigned>(grid), kThreads, sm, a.stream>>>(p);
    LEMA_CUDA_TRY(cudaGetLastError());
  }
  if (pl.global) {
    p.list_mode = pl.list_mode ? 1 : 0;
    auto kern = match_kernel<CodeT, false, Vec>;
    const size_t sm = smem_bytes<CodeT>(false);
    LEMA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(sm)));
    kern<<<static_cast<unsigned>(pl.n_gtables), kThreads, sm, a.stream>>>(p);
    LEMA_CUDA_TRY(cudaGetLastError());
  }
  return LEMA_OK;
}

template <typename CodeT>
int run_code(const MatchLaunch& a, const Plan& pl, const DeviceInfo& dev) {
  if (a.out == nullptr) return run<CodeT, uint4>(a, pl, dev);
  const bool a16 = a.vbytes % 16 == 0 && aligned(a.v, 16) && aligned(a.out, 16);
  const bool a8 = a.vbytes % 8 == 0 && aligned(a.v, 8) && aligned(a.out, 8);
  const bool a4 = a.vbytes % 4 == 0 && aligned(a.v, 4) && aligned(a.out, 4);
  if (a16) return run<CodeT, uint4>(a, pl, dev);
  if (a8) return run<CodeT, uint2>(a, pl, dev);
  if (a4) return run<CodeT, uint32_t>(a, pl, dev);
  return run<CodeT, unsigned short>(a, pl, dev);
}

}  // namespace k2

size_t match_workspace_bytes(int64_t N, int64_t T, int code_bytes) {
  return k2::make_plan(N, T, code_bytes).total;
}

int launch_match(const MatchLaunch& a) {
  if (a.code_bytes != 4 && a.code_bytes != 8) return fail(LEMA_ERR_INVALID_ARGUMENT, "code_bytes must be 4 or 8, got %d", a.code_bytes);
  if (a.N < 0 || a.T < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "negative shape (%lld, %lld)", (long long)a.N, (long long)a.T);
  if (a.T > (int64_t(1) << 31) - 16) return fail(LEMA_ERR_INVALID_ARGUMENT, "T = %lld exceeds 2^31 - 16", (long long)a.T);
  if (a.N == 0 || a.T == 0) return LEMA_OK;
  if (a.qc == nullptr || a.kc == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null code pointer");
  if (!aligned(a.qc, a.code_bytes) || !aligned(a.kc, a.code_bytes)) return fail(LEMA_ERR_INVALID_ARGUMENT, "codes not aligned to their width");
  if (a.out != nullptr) {
    if (a.v == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "out given without values");
    if (a.vbytes <= 0 || a.vbytes % 2 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "vbytes must be a positive multiple of 2, got %lld", (long long)a.vbytes);
    if (!aligned(a.v, 2) || !aligned(a.out, 2)) return fail(LEMA_ERR_INVALID_ARGUMENT, "value rows must be 2-byte aligned");
    if (a.vbytes / 2 * k2::kChunk > (int64_t(1) << 31)) return fail(LEMA_ERR_INVALID_ARGUMENT, "vbytes %lld too large", (long long)a.vbytes);
  }
  const bool lt_any = a.lt_code || a.lt_pos || a.lt_count;
  if (lt_any && !(a.lt_code && a.lt_pos && a.lt_count)) return fail(LEMA_ERR_INVALID_ARGUMENT, "last-occurrence outputs: all three or none");
  const k2::Plan pl = k2::make_plan(a.N, a.T, a.code_bytes);
  if (a.ws_bytes < pl.total || (pl.total > 0 && a.ws == nullptr)) {
    return fail(LEMA_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", a.ws_bytes, pl.total);
  }
  if (pl.total > 0 && !aligned(a.ws, 256)) return fail(LEMA_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
  return a.code_bytes == 4 ? k2::run_code<uint32_t>(a, pl, *dev) : k2::run_code<uint64_t>(a, pl, *dev);
}

}  // namespace lema
