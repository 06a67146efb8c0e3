// K2 -- latest exact match over position-ordered streams, and the value gather.
//
// For stream n and position i:  src[n][i] = max{ j < i : kc[n][j] == qc[n][i] } or -1,
// out[n][i] = v[n][src] (zeros when -1). This is the rule of code/lema/attention.py:100-158,
// which the reference computes with two stable argsorts over 2T events per stream. Here a
// stream is walked in chunks of kChunk positions against a hash table of its key codes, and
// every phase inside a chunk is parallel; only chunk-to-chunk is ordered.
//
// Table state per slot (one slot per distinct key code of the stream):
//   carry[slot]  1 + position of the latest key with that code BEFORE the current chunk (0: none)
//   mask[slot]   bit s set iff a key with that code occurs in step s (32 positions) of the
//                current chunk
// A chunk is 32 steps of 32 positions and three phases, all parallel:
//   P1 (keys)    each key inserts its code into -- or finds it in -- the table (its SLOT), sets
//                its step's bit in mask[slot], records its slot in the step's key-slot array
//                and ORs its lane into the step's lane-set bucket of the slot (slot % 64).
//   P2 (queries) each query looks its code up; no slot means no key of that code so far (-1).
//                If the query's own step holds the code (mask bit), the highest lane below its
//                own in the step's bucket whose recorded slot is the query's answers it;
//                otherwise the highest mask bit below its step names the latest earlier step
//                holding the code, whose highest such lane is the answer; with no such step the
//                answer is carry[slot].
//   P3 (keys)    carry[slot] = max(carry, 1 + position) by an atomic max, mask[slot] = 0, and
//                every key clears its bucket for the next chunk.
// Two slots sharing a bucket in one step only cost a second look; no warp-wide ballot or match
// instruction is needed (on this part those cost far more than the table traffic).
// All 32 warps of a CTA run the phases (one step each per chunk); CTA barriers separate them.
// The value rows are copied by CTAs on other SMs of the same launch as the matchers publish
// their progress (the pipelined mode, below), or by a separate kernel afterwards
// (gather_kernel: the two-kernel path).
//
// The table is bucketed: 8 slots per bucket, read with vector loads, linear probing over
// buckets; a claim is one compare-and-swap of a free code word (all ones), and the all-ones
// code itself lives in a dedicated side slot, so every code value is an ordinary key.
//
// One CTA owns one stream at a time (persistent grid-stride over streams). The shared-memory
// table has a fixed capacity. A stream whose distinct key codes would load it beyond
// kOverflowFrac is handed over whole to the same kernel running with a CTA-private table in
// global memory sized for 2*T (the overflow path). No input can make the result wrong; an
// unusual one only takes the slower path.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "match.cuh"

namespace lema {
namespace k2 {

constexpr int kThreads = 1024;  // 32 warps: one step of 32 positions each per chunk
constexpr int kChunk = 1024;                   // positions per chunk: 32 steps of 32
constexpr int kSteps = kChunk / 32;
constexpr int kMatchWarps = kThreads / 32;                         // every warp matches
constexpr int kPerLane = (kSteps + kMatchWarps - 1) / kMatchWarps;  // steps per warp
constexpr int kBucket = 8;  // slots per table bucket
static_assert(kSteps == 32, "step masks are 32-bit");

constexpr uint32_t kNoSlot = 0xFFFFFFFFu;

// Shared-memory table capacity (slots) per code width; above kOverflowFrac of it a stream
// moves to the global-memory path.
template <typename CodeT>
struct SmemCap;
template <>
struct SmemCap<uint32_t> {
  static constexpr uint32_t kSlots = 8192;
};
template <>
struct SmemCap<uint64_t> {
  static constexpr uint32_t kSlots = 4096;
};
constexpr double kOverflowFrac = 0.75;

static_assert(SmemCap<uint32_t>::kSlots < (1u << 14) && SmemCap<uint64_t>::kSlots < (1u << 14),
              "shared-memory slot indices (and the side slot) stay small");

template <typename CodeT>
__host__ __device__ constexpr uint32_t overflow_limit() {
  return static_cast<uint32_t>(SmemCap<CodeT>::kSlots * kOverflowFrac);
}

// ---------------------------------------------------------------- the table
__device__ __forceinline__ uint32_t cas_code(uint32_t* p, uint32_t cmp, uint32_t val) {
  return atomicCAS(p, cmp, val);
}
__device__ __forceinline__ uint64_t cas_code(uint64_t* p, uint64_t cmp, uint64_t val) {
  return atomicCAS(reinterpret_cast<unsigned long long*>(p), static_cast<unsigned long long>(cmp),
                   static_cast<unsigned long long>(val));
}
template <typename CodeT>
__device__ __forceinline__ void load_bucket(const CodeT* p, CodeT (&w)[kBucket]) {
  static_assert(sizeof(CodeT) * kBucket % 16 == 0, "bucket = whole 16-byte vectors");
  const uint4* v = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int k = 0; k < static_cast<int>(sizeof(CodeT) * kBucket / 16); ++k) {
    const uint4 x = v[k];
    memcpy(reinterpret_cast<char*>(w) + 16 * k, &x, 16);
  }
}

// Slot -> (code, carry, mask). Slots [0, cap) form cap / kBucket buckets; slot `cap` holds the
// all-ones code, whose presence is the side flag.
template <typename CodeT, typename CarryT>
struct Table {
  static constexpr CodeT kFree = static_cast<CodeT>(~CodeT(0));
  static constexpr CarryT kNoCarry = 0;  // carries hold position + 1
  CodeT* code;      // [cap]
  CarryT* carry;    // [cap + 1]
  uint32_t* mask;   // [cap + 1]
  uint32_t* side;   // 1 word
  uint32_t cap;
  uint32_t bmask;   // buckets - 1
  uint32_t bshift;  // 32 - log2(buckets): the bucket is the top bits of mix(code)

  __host__ __device__ static constexpr size_t bytes(uint32_t slots) {
    return round_up16(slots * sizeof(CodeT)) + round_up16((slots + 1) * sizeof(CarryT)) +
           round_up16((slots + 1) * sizeof(uint32_t)) + 16;
  }
  // codes and the side word only (the dictionary of the sweep path: no carries, no masks)
  __device__ void init_dict(void* base, uint32_t slots) {
    cap = slots;
    bmask = slots / kBucket - 1;
    bshift = 32 - (31 - __clz(slots / kBucket));
    code = static_cast<CodeT*>(base);
    side = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(base) + slots * sizeof(CodeT));
    carry = nullptr;
    mask = nullptr;
  }
  __device__ void init(void* base, uint32_t slots) {
    cap = slots;
    bmask = slots / kBucket - 1;
    bshift = 32 - (31 - __clz(slots / kBucket));  // buckets: a power of two, >= 2
    unsigned char* b = static_cast<unsigned char*>(base);
    code = reinterpret_cast<CodeT*>(b);
    b += round_up16(slots * sizeof(CodeT));
    carry = reinterpret_cast<CarryT*>(b);
    b += round_up16((slots + 1) * sizeof(CarryT));
    mask = reinterpret_cast<uint32_t*>(b);
    b += round_up16((slots + 1) * sizeof(uint32_t));
    side = reinterpret_cast<uint32_t*>(b);
  }
  __device__ void clear(int tid, int nthr) {
    for (uint32_t s = tid; s < cap; s += nthr) code[s] = kFree;
    for (uint32_t s = tid; s <= cap; s += nthr) {
      carry[s] = kNoCarry;
      mask[s] = 0u;
    }
    if (tid == 0) *side = 0;
  }
  // Fibonacci (multiplicative) hashing: one multiply; the bucket is the product's top bits and
  // the code's own slot in it the next three. Placement only, never results.
  __device__ static uint32_t mix(uint32_t c) { return c * 0x9E3779B1u; }
  __device__ static uint32_t mix(uint64_t c) {
    return static_cast<uint32_t>((c * 0x9E3779B97F4A7C15ull) >> 32);
  }
  __device__ uint32_t home(CodeT c) const { return mix(c) >> bshift; }
  // Insert-or-find from the bucket contents `w` already loaded from `home(c)`; the general
  // probe (CAS races, full buckets) continues from there. Returns the slot, or kNoSlot when
  // every bucket was full.
  __device__ uint32_t insert_from(CodeT c, uint32_t b, CodeT (&w)[kBucket], uint32_t& claimed) {
    if (c == kFree) {
      claimed = atomicCAS(side, 0u, 1u) == 0u;
      return cap;
    }
    for (uint32_t n = 0; n <= bmask; ++n) {
      CodeT* bk = code + b * kBucket;
#pragma unroll
      for (int k = 0; k < kBucket; ++k) {
        if (w[k] == c) return b * kBucket + k;
      }
#pragma unroll
      for (int k = 0; k < kBucket; ++k) {
        if (w[k] == kFree) {
          const CodeT old = cas_code(bk + k, kFree, c);
          if (old == kFree) {
            claimed = 1;
            return b * kBucket + k;
          }
          if (old == c) return b * kBucket + k;
          // another code took slot k: the later slots are judged by their fresh contents
#pragma unroll
          for (int j = k + 1; j < kBucket; ++j) w[j] = *reinterpret_cast<volatile CodeT*>(bk + j);
#pragma unroll
          for (int j = k + 1; j < kBucket; ++j) {
            if (w[j] == c) return b * kBucket + j;
          }
        }
      }
      b = (b + 1) & bmask;
      load_bucket(code + b * kBucket, w);
    }
    return kNoSlot;
  }
  // Find (after a barrier that ended the inserts). A bucket with a free slot ends the search:
  // codes fill a bucket's slots in order and reach a bucket only when the buckets before it on
  // their chain were full.
  __device__ uint32_t find_from(CodeT c, uint32_t b, CodeT (&w)[kBucket]) const {
    if (c == kFree) return *side ? cap : kNoSlot;
    for (uint32_t n = 0; n <= bmask; ++n) {
      bool open = false;
#pragma unroll
      for (int k = 0; k < kBucket; ++k) {
        if (w[k] == c) return b * kBucket + k;
        open |= (w[k] == kFree);
      }
      if (open) return kNoSlot;
      b = (b + 1) & bmask;
      load_bucket(code + b * kBucket, w);
    }
    return kNoSlot;
  }
  // One-bucket fast paths, branch-free in the common case; a full bucket or a lost claim race
  // falls back to the general probe.
  // A code's own slot in its home bucket (hash bits below the bucket's). A code is
  // placed there whenever that slot is free at its insertion, so most inserts and finds touch
  // one slot; a free own slot also proves the code absent (slots are never freed in a stream).
  __device__ uint32_t own(uint32_t h, uint32_t b) const { return b * kBucket + ((h >> (bshift - 3)) & 7u); }
  __device__ uint32_t insert_fast(CodeT c, uint32_t& claimed) {
    static_assert(kBucket == 8, "own slot = 3 hash bits");
    if (c == kFree) {
      claimed = atomicCAS(side, 0u, 1u) == 0u;
      return cap;
    }
    const uint32_t h = mix(c);
    const uint32_t b = h >> bshift;
    {
      const uint32_t hs = own(h, b);
      const CodeT cur = code[hs];
      if (cur == c) return hs;
      if (cur == kFree) {
        const CodeT old = cas_code(code + hs, kFree, c);
        if (old == kFree) {
          claimed = 1;
          return hs;
        }
        if (old == c) return hs;
      }
    }
    CodeT w[kBucket];
    load_bucket(code + b * kBucket, w);
    uint32_t eq = 0, fr = 0;
#pragma unroll
    for (int k = 0; k < kBucket; ++k) {
      eq |= static_cast<uint32_t>(w[k] == c) << k;
      fr |= static_cast<uint32_t>(w[k] == kFree) << k;
    }
    if (eq) return b * kBucket + (__ffs(eq) - 1);
    if (fr) {
      const int k = __ffs(fr) - 1;
      const CodeT old = cas_code(code + b * kBucket + k, kFree, c);
      if (old == kFree) {
        claimed = 1;
        return b * kBucket + k;
      }
      if (old == c) return b * kBucket + k;
    }
    load_bucket(code + b * kBucket, w);
    return insert_from(c, b, w, claimed);
  }
  __device__ uint32_t find_fast(CodeT c) const {
    if (c == kFree) return *side ? cap : kNoSlot;
    const uint32_t h = mix(c);
    const uint32_t b = h >> bshift;
    {
      const CodeT cur = code[own(h, b)];
      if (cur == c) return own(h, b);
      if (cur == kFree) return kNoSlot;
    }
    CodeT w[kBucket];
    load_bucket(code + b * kBucket, w);
    uint32_t eq = 0, fr = 0;
#pragma unroll
    for (int k = 0; k < kBucket; ++k) {
      eq |= static_cast<uint32_t>(w[k] == c) << k;
      fr |= static_cast<uint32_t>(w[k] == kFree) << k;
    }
    if (eq) return b * kBucket + (__ffs(eq) - 1);
    if (fr) return kNoSlot;
    return find_from(c, b, w);
  }
  __device__ bool used(uint32_t s, CodeT& c, CarryT& m) const {
    m = carry[s];
    if (s == cap) {
      c = kFree;
      return *side != 0;
    }
    c = code[s];
    return c != kFree;
  }
};

// ---------------------------------------------------------------- the kernel
// Rows to gather: out[n][i] = v[n][src[n][i]] (zeros where src is -1), in Vec words.
struct GatherParams {
  const int32_t* src;
  const unsigned char* v;
  unsigned char* out;
  int64_t N, T;
  // row (n, t) of the values at v + (n / heads) * v_sb + (n % heads) * v_sh + t * v_st, of the
  // output likewise (bytes); a plain [N][T] layout is heads = 1, sb = T * row, st = row
  int64_t heads, v_sb, v_sh, v_st, o_sb, o_sh, o_st;
  uint32_t wpr;        // vector words per row
  uint32_t words;      // words per stream = T * wpr (< 2^32)
  int div_shift;       // log2(wpr) when a power of two, else -1
  uint32_t div_magic;  // floor(2^32 / wpr) + 1 when exact for every word index, else 0
};

// Pipelined mode: ONE launch matches and gathers. The CTAs of the first `match_sms` SMs to
// start match streams (taken from a counter, so they run in claim order); the other SMs' CTAs
// copy value rows of the positions already matched, a unit (kUnitChunks chunks of one stream)
// at a time, as the matchers publish their progress; a matcher with no stream left turns to
// the rows too. The row traffic then overlaps the issue-bound matching, and the two never
// share an SM (value loads beside a shared-memory table slow every table access).
constexpr int kUnitChunks = 4;                    // chunks per gather unit and per publication
constexpr uint32_t kProgOvf = 0x80000000u;        // progress word of a stream handed to the overflow path
constexpr int kMaxSmIds = 512;                    // %smid values with a role slot
constexpr uint32_t kRoleMatch = 1, kRoleGather = 2;
struct PipeCtl {
  uint32_t sm_seen[kMaxSmIds];  // CTAs started per SM
  uint32_t sm_role[kMaxSmIds];  // the role of each SM, set by its first CTA
  uint32_t sm_ticket;           // SMs seen
  uint32_t next_stream;         // streams claimed by matchers
  uint32_t next_unit;           // gather units claimed
  uint32_t failed;              // a wait ran out: every later wait gives up at once
};

struct Params {
  const void* qc;
  const void* kc;
  int64_t N, T;
  int32_t* src;
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
  uint32_t gslots;
  int list_mode;  // global path: 1 = streams from ovf_list, 0 = all streams
  // pipelined mode (zeroed control block and per-stream progress in the workspace)
  PipeCtl* ctl;
  uint32_t* progress;     // [N]: chunks matched and published, or kProgOvf
  uint32_t match_sms;     // SMs whose CTAs match
  uint32_t wave;          // streams matched at once: the gather units' order
  int gather_inline;      // overflow path: gather each stream right after matching it
  GatherParams g;         // uint4 words (pipelined and inline gathers)
  unsigned long long wait_ns;  // bound of every wait on another warp's or CTA's progress
};

__device__ __forceinline__ void st_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Rows [t0, t1) of stream n by the kThr threads of a CTA, kGUnroll loads in flight per thread.
// The indices come through L2 (__ldcg): other CTAs of the same launch may have written them.
// loads in flight per thread in the gather kernel (the two-kernel path: calls below one wave of
// matchers). Measured on config 2's streams with the current matcher: 2 / 4 / 8 give 0.1039 /
// 0.1068 / 0.1135 ms per call at 128 streams and 0.1657 / 0.1697 / 0.1826 at 256
constexpr int kGUnroll = 2;
template <typename Vec, int kThr>
__device__ __forceinline__ void gather_span(const GatherParams& g, int64_t n, uint32_t t0, uint32_t t1,
                                            int tid) {
  const int32_t* src = g.src + n * g.T;
  const int64_t b = n / g.heads, h = n - b * g.heads;
  const unsigned char* v = g.v + b * g.v_sb + h * g.v_sh;
  unsigned char* o = g.out + b * g.o_sb + h * g.o_sh;
  const uint32_t w_end = t1 * g.wpr;
  for (uint32_t w0 = t0 * g.wpr + tid; w0 < w_end; w0 += kThr * kGUnroll) {
    Vec val[kGUnroll];
#pragma unroll
    for (int u = 0; u < kGUnroll; ++u) {
      const uint32_t w = w0 + u * kThr;
      val[u] = zero_vec<Vec>();
      if (w < w_end) {
        const uint32_t r = g.div_shift >= 0 ? (w >> g.div_shift)
                                            : (g.div_magic ? __umulhi(w, g.div_magic) : w / g.wpr);
        const int32_t s = __ldcg(src + r);
        if (s >= 0) val[u] = __ldg(reinterpret_cast<const Vec*>(v + s * g.v_st) + (w - r * g.wpr));
      }
    }
#pragma unroll
    for (int u = 0; u < kGUnroll; ++u) {
      const uint32_t w = w0 + u * kThr;
      if (w < w_end) {
        const uint32_t r = g.div_shift >= 0 ? (w >> g.div_shift)
                                            : (g.div_magic ? __umulhi(w, g.div_magic) : w / g.wpr);
        store_stream(reinterpret_cast<Vec*>(o + r * g.o_st) + (w - r * g.wpr), val[u]);
      }
    }
  }
}

// Per step of a chunk, two small shared arrays replace any warp-wide matching:
//   ls[step][b]   bit j set iff key lane j of the step holds a slot with (slot % kLsBuckets) == b
//   ks[step][j]   the slot of key lane j (kNoSlot for none)
// The key lanes of a step holding slot s are the bits of ls[step][s % kLsBuckets] whose ks is s;
// two slots sharing a bucket in one step only cost a second look.
constexpr int kLsBuckets = 64;

// The highest lane of `cand` whose key slot is s, or -1.
__device__ __forceinline__ int lane_with_slot(uint32_t cand, const uint32_t* ks, uint32_t s) {
  while (cand) {
    const int j = 31 - __clz(cand);
    if (ks[j] == s) return j;
    cand &= ~(1u << j);
  }
  return -1;
}

__device__ __forceinline__ void match_barrier() { __syncthreads(); }


__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool fill) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(gsrc), "r"(fill ? 16 : 0)
               : "memory");
}

// Rows [t0, t1) of stream n through this CTA's shared memory (kThr threads; `buf` holds
// `rows_per_pass` <= 2 * kThr rows): every thread fetches its rows of a pass with
// asynchronous 16-byte copies (zero fill on a miss), so a pass keeps the whole buffer in
// flight without holding registers; the indices of the next pass load meanwhile; then the
// CTA writes the pass out with coalesced streaming stores. A CTA whose table is idle (a
// row-copying CTA, or a matcher with no stream left) lends its shared memory to this.
template <int kThr>
__device__ void gather_unit_staged(const GatherParams& g, int64_t n, uint32_t t0, uint32_t t1, int tid,
                                   uint4* buf, uint32_t rows_per_pass) {
  const int32_t* src = g.src + n * g.T;
  const int64_t b = n / g.heads, h = n - b * g.heads;
  const unsigned char* v = g.v + b * g.v_sb + h * g.v_sh;
  unsigned char* o = g.out + b * g.o_sb + h * g.o_sh;
  const uint32_t wpr = g.wpr;
  int32_t s0 = -1, s1 = -1;  // indices of this thread's two rows of the coming pass
  {
    const uint32_t lim = min(t1, t0 + rows_per_pass);
    if (t0 + tid < lim) s0 = __ldcg(src + t0 + tid);
    if (t0 + kThr + tid < lim) s1 = __ldcg(src + t0 + kThr + tid);
  }
  for (uint32_t r0 = t0; r0 < t1; r0 += rows_per_pass) {
    const uint32_t cnt = min(rows_per_pass, t1 - r0);
    if (static_cast<uint32_t>(tid) < cnt) {
      const unsigned char* row = v + static_cast<int64_t>(max(s0, 0)) * g.v_st;
      for (uint32_t c = 0; c < wpr; ++c) cp_async16(buf + tid * wpr + c, row + 16 * c, s0 >= 0);
    }
    if (static_cast<uint32_t>(kThr + tid) < cnt) {
      const unsigned char* row = v + static_cast<int64_t>(max(s1, 0)) * g.v_st;
      for (uint32_t c = 0; c < wpr; ++c) cp_async16(buf + (kThr + tid) * wpr + c, row + 16 * c, s1 >= 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint32_t r1 = r0 + rows_per_pass;
    s0 = s1 = -1;
    if (r1 < t1) {
      const uint32_t lim = min(t1, r1 + rows_per_pass);
      if (r1 + tid < lim) s0 = __ldcg(src + r1 + tid);
      if (r1 + kThr + tid < lim) s1 = __ldcg(src + r1 + kThr + tid);
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();
    for (uint32_t w = tid; w < cnt * wpr; w += kThr) {
      const uint32_t r = g.div_shift >= 0 ? (w >> g.div_shift)
                                          : (g.div_magic ? __umulhi(w, g.div_magic) : w / wpr);
      store_stream(reinterpret_cast<uint4*>(o + static_cast<int64_t>(r0 + r) * g.o_st) + (w - r * wpr), buf[w]);
    }
    __syncthreads();  // the buffer is refilled by the next pass
  }
}

// Pipelined mode: this CTA's role, the same for both CTAs of an SM (the first to start on an
// SM draws it: the first match_sms SMs match).
__device__ uint32_t pipe_role(const Params& p, int tid) {
  __shared__ uint32_t s_role;
  if (tid == 0) {
    uint32_t smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    uint32_t role = kRoleMatch;
    if (smid < static_cast<uint32_t>(kMaxSmIds)) {
      if (atomicAdd(&p.ctl->sm_seen[smid], 1u) == 0u) {
        role = atomicAdd(&p.ctl->sm_ticket, 1u) < p.match_sms ? kRoleMatch : kRoleGather;
        st_release(&p.ctl->sm_role[smid], role);
      } else {
        // the SM's first CTA publishes its role right after drawing it
        uint32_t r = 0;
        const unsigned long long t0 = global_ns();
        while ((r = ld_acquire(&p.ctl->sm_role[smid])) == 0u && global_ns() - t0 < 1000000ull) __nanosleep(64);
        role = r != 0u ? r : kRoleMatch;
      }
    }
    s_role = role;
  }
  __syncthreads();
  return s_role;
}

// Pipelined mode: gather units until none is left. Unit u covers kUnitChunks chunks of one
// stream; units are numbered wave by wave (streams [k * wave, (k + 1) * wave) are matched at
// about the same time), chunk group by chunk group, so a unit's turn comes about when its
// rows are matched. A unit waits for its stream's published progress (bounded); a stream
// handed to the overflow path is gathered there.
template <int kThr>
__device__ void pipe_gather(const Params& p, int tid, uint4* buf, uint32_t rows_per_pass) {
  __shared__ uint32_t s_n, s_t0, s_t1;
  __shared__ int s_go;
  const uint32_t n_chunks = static_cast<uint32_t>((p.T + kChunk - 1) / kChunk);
  const uint32_t ng = (n_chunks + kUnitChunks - 1) / kUnitChunks;
  const uint32_t N = static_cast<uint32_t>(p.N);
  const uint32_t total = N * ng;  // < 2^31 (host)
  for (;;) {
    if (tid == 0) {
      const uint32_t u = atomicAdd(&p.ctl->next_unit, 1u);
      s_go = -1;
      if (u < total) {
        const uint32_t full = p.wave * ng;
        const uint32_t blk = u / full, rem = u - blk * full;
        const uint32_t n0 = blk * p.wave, bsz = min(p.wave, N - n0);
        const uint32_t cg = rem / bsz, n = n0 + (rem - cg * bsz);
        const uint32_t need = min((cg + 1) * kUnitChunks, n_chunks);
        uint32_t v = ld_acquire(p.progress + n);
        if (v < need) {
          const unsigned long long t0 = global_ns();
          while ((v = ld_acquire(p.progress + n)) < need) {
            if (ld_acquire(&p.ctl->failed) != 0u || global_ns() - t0 > p.wait_ns) {
              atomicExch(&p.ctl->failed, 1u);
              raise_status(p.status, LEMA_STATUS_PROBE_LIMIT);
              break;
            }
            __nanosleep(256);
          }
        }
        s_go = (v >= need && (v & kProgOvf) == 0u) ? 1 : 0;
        s_n = n;
        s_t0 = cg * kUnitChunks * kChunk;
        s_t1 = static_cast<uint32_t>(min(static_cast<int64_t>(need) * kChunk, p.T));
      }
    }
    __syncthreads();
    const int go = s_go;
    if (go < 0) break;
    if (go) gather_unit_staged<kThr>(p.g, s_n, s_t0, s_t1, tid, buf, rows_per_pass);
    __syncthreads();  // s_* are rewritten for the next unit
  }
}

// Segmented mode, after a CTA's run of chunks [r_lo, r_hi) of stream n: a cluster barrier
// (every run's table complete), then, unless some run of the stream overflowed its table
// (the stream then goes once to the overflow path, which redoes it whole), every position of
// this run still at -1 looks its query code up in the tables of the earlier runs, newest
// first; a second cluster barrier keeps every table intact until the last remote read.
template <typename CodeT, typename Tab>
__device__ void seg_resolve(const Params& p, const Tab& tab, int64_t n, int64_t r_lo, int64_t r_hi,
                            uint32_t rank, uint32_t count, int tid, uint32_t* s_abort) {
  const cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
  cl.sync();
  bool any = false;
  for (uint32_t k = 0; k < count; ++k) any |= *cl.map_shared_rank(s_abort, k) != 0u;
  if (any) {
    if (rank == 0 && tid == 0 && p.ovf_list != nullptr) {
      const uint32_t k = atomicAdd(p.ovf_count, 1u);
      p.ovf_list[k] = static_cast<uint32_t>(n);
    }
  } else if (rank > 0) {  // (rank 0's run starts the stream: nothing earlier to look up)
    const CodeT* qc = static_cast<const CodeT*>(p.qc) + n * p.T;
    int32_t* src = p.src + n * p.T;
    const int64_t lo = r_lo * kChunk, hi = std::min<int64_t>(p.T, r_hi * kChunk);
    for (int64_t i = lo + tid; i < hi; i += kThreads) {
      if (src[i] != -1) continue;
      const CodeT c = qc[i];
      for (int k = static_cast<int>(rank) - 1; k >= 0; --k) {
        Tab rt = tab;  // run k's table, through distributed shared memory
        rt.code = cl.map_shared_rank(tab.code, k);
        rt.carry = cl.map_shared_rank(tab.carry, k);
        rt.side = cl.map_shared_rank(tab.side, k);
        const uint32_t sl = rt.find_fast(c);
        if (sl == kNoSlot) continue;
        const uint32_t m = rt.carry[sl];
        if (m != 0u) {
          src[i] = static_cast<int32_t>(m) - 1;
          break;
        }
      }
    }
  }
  cl.sync();
}

// kSeg: segmented mode (launched in clusters of S CTAs, S = the cluster size). The S CTAs of a
// cluster share one stream: CTA k matches the k-th run of whole chunks with its own shared-
// memory table, then, after a cluster barrier, resolves its positions that found no earlier
// key inside its run against the tables of runs k - 1, ..., 0 (newest first, read through
// distributed shared memory): a table's carry is 1 + the latest key position of that run.
// That is the latest earlier key over the whole stream, as one CTA walking every chunk finds.
template <typename CodeT, bool kSmemTable, bool kPipe = false, bool kSeg = false>
__global__ void __launch_bounds__(kThreads, 2) match_kernel(const Params p) {
  static_assert(!kSeg || (kSmemTable && !kPipe), "segments: shared-memory tables, two-kernel path");
  griddep_wait();  // launched as a dependent (the overflow path): the matcher's results first
  griddep_launch();
  using Tab = Table<CodeT, uint32_t>;
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr uint32_t kCap = SmemCap<CodeT>::kSlots;
  constexpr size_t kTableBytes = kSmemTable ? round_up16(Tab::bytes(kCap)) : 0;
  uint32_t* s_ls = reinterpret_cast<uint32_t*>(smem + kTableBytes);  // [kSteps][kLsBuckets]
  uint32_t* s_ks = s_ls + kSteps * kLsBuckets;                         // [kSteps][32]
  __shared__ uint32_t s_ovf, s_lt;
  __shared__ uint32_t s_used[2];  // slots claimed in the stream before chunk r: s_used[r & 1]
  __shared__ uint32_t s_claim;
  __shared__ uint32_t s_abort;  // segmented mode: this CTA's run overflowed its table

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // segmented mode: this CTA's rank in its cluster, the cluster's index and count
  uint32_t seg_rank = 0, seg_count = 1;
  int64_t seg_first = blockIdx.x, seg_stride = gridDim.x;
  if constexpr (kSeg) {
    const cooperative_groups::cluster_group cl = cooperative_groups::this_cluster();
    seg_rank = cl.block_rank();
    seg_count = cl.num_blocks();
    seg_first = blockIdx.x / seg_count;
    seg_stride = gridDim.x / seg_count;
  }
  const CodeT* qc = static_cast<const CodeT*>(p.qc);
  const CodeT* kc = static_cast<const CodeT*>(p.kc);

  Tab tab;
  if (kSmemTable) {
    tab.init(smem, kCap);
  } else {
    tab.init(p.gtables + static_cast<int64_t>(blockIdx.x) * p.gtable_bytes, p.gslots);
  }
  const int64_t n_work = (!kSmemTable && p.list_mode) ? static_cast<int64_t>(*p.ovf_count) : p.N;
  const int64_t n_chunks = (p.T + kChunk - 1) / kChunk;
  // pipelined: streams in claim order from a counter (each CTA takes the next when it is free)
  auto claim = [&]() -> int64_t {
    if (tid == 0) s_claim = atomicAdd(&p.ctl->next_stream, 1u);
    __syncthreads();
    const int64_t w = s_claim;
    __syncthreads();
    return w;
  };
  // pipelined: the whole dynamic shared memory stages rows once this CTA copies them
  const uint32_t stage_rows = kPipe ? min(2u * kThreads, static_cast<uint32_t>(
                                              (kTableBytes + kSteps * (kLsBuckets + 32) * sizeof(uint32_t)) /
                                              (16u * p.g.wpr))) : 0u;
  if constexpr (kPipe) {
    if (pipe_role(p, tid) != kRoleMatch) {
      pipe_gather<kThreads>(p, tid, reinterpret_cast<uint4*>(smem), stage_rows);
      return;
    }
  }

  // segmented mode: this CTA's run of chunks [r_lo, r_hi)
  const int64_t seg_chunks = (n_chunks + seg_count - 1) / seg_count;
  const int64_t r_lo = kSeg ? std::min<int64_t>(n_chunks, seg_rank * seg_chunks) : 0;
  const int64_t r_hi = kSeg ? std::min<int64_t>(n_chunks, r_lo + seg_chunks) : n_chunks;

  for (int64_t wi = kPipe ? claim() : seg_first; wi < n_work;
       wi = kPipe ? claim() : wi + seg_stride) {
    const int64_t n = (!kSmemTable && p.list_mode) ? static_cast<int64_t>(p.ovf_list[wi]) : wi;
    const int64_t row0 = n * p.T;
    tab.clear(tid, kThreads);
    for (int k = tid; k < kSteps * kLsBuckets; k += kThreads) s_ls[k] = 0u;
    if (tid == 0) {
      s_ovf = 0;
      s_lt = 0;
      s_used[r_lo & 1] = 0;
    }
    __syncthreads();

    bool aborted = false;
    for (int64_t r = r_lo; r < r_hi; ++r) {
      {
        // ==================================================== chunk r
        const int64_t base = r * kChunk;
        const int cnt = static_cast<int>(min(static_cast<int64_t>(kChunk), p.T - base));
        int32_t* ab = p.src + row0 + base;
        CodeT kr[kPerLane], qr[kPerLane];
#pragma unroll
        for (int u = 0; u < kPerLane; ++u) {
          const int i = (warp + u * kMatchWarps) * 32 + lane;
          kr[u] = (i < cnt && warp + u * kMatchWarps < kSteps) ? kc[row0 + base + i] : CodeT(0);
          qr[u] = (i < cnt && warp + u * kMatchWarps < kSteps) ? qc[row0 + base + i] : CodeT(0);
        }
        {
          // the next chunk's codes into L2 meanwhile: its loads then wait on L2, not on HBM
          // (which row copies elsewhere on the chip may keep busy)
          constexpr int kLines = kChunk * static_cast<int>(sizeof(CodeT)) / 128;
          if (tid < 2 * kLines) {
            const int64_t e = base + kChunk + (tid % kLines) * (128 / static_cast<int>(sizeof(CodeT)));
            if (e < p.T) prefetch_l2((tid < kLines ? kc : qc) + row0 + e);
          }
        }
        // ---------------------------------------------- P1: keys into the table, step bits
        const int32_t base32 = static_cast<int32_t>(base);
        uint32_t kslot[kPerLane];
        uint32_t claims = 0;  // 0 or 1: one key per thread
        static_assert(kPerLane == 1, "one key per thread per chunk: the barrier counts claims");
#pragma unroll
        for (int u = 0; u < kPerLane; ++u) {
          const int step = warp + u * kMatchWarps;
          const int i = step * 32 + lane;
          kslot[u] = kNoSlot;
          if (step >= kSteps || step * 32 >= cnt) continue;  // uniform per warp
          const bool valid = i < cnt;
          uint32_t claimed = 0;
          if (valid) {
            kslot[u] = tab.insert_fast(kr[u], claimed);
            if (!kSmemTable && kslot[u] == kNoSlot) s_ovf = 1;
          }
          claims += claimed;
          // the step's key lanes per slot bucket, and each lane's slot; every key lane sets its
          // step's bit in the slot's mask (lanes sharing a slot set the same bit)
          const uint32_t ks = kslot[u];
          s_ks[step * 32 + lane] = ks;
          if (ks != kNoSlot) {
            atomicOr(s_ls + step * kLsBuckets + (ks & (kLsBuckets - 1)), 1u << lane);
            atomicOr(tab.mask + ks, 1u << step);
          }
        }
        // claims counted by the barrier; every thread stores the same new total (the other
        // word of the pair, read only after the next chunk's count). A key that finds no slot
        // at all means every slot is claimed, which is past the limit too.
        const uint32_t used = s_used[r & 1] + static_cast<uint32_t>(__syncthreads_count(claims != 0));
        s_used[(r + 1) & 1] = used;
        const bool over = kSmemTable ? used > overflow_limit<CodeT>() : s_ovf != 0;
        if (over) {
          // the whole CTA learns it after the round barrier; P2/P3 are skipped
        } else {
          // ---------------------------------------------- P2: queries
#pragma unroll
          for (int u = 0; u < kPerLane; ++u) {
            const int step = warp + u * kMatchWarps;
            const int i = step * 32 + lane;
            if (step >= kSteps || step * 32 >= cnt) continue;  // uniform per warp
            const bool valid = i < cnt;
            // the query's slot, looked up once every key of the chunk is in the table
            const uint32_t sl = valid ? tab.find_fast(qr[u]) : kNoSlot;
            int32_t a = -1;
            if (valid && sl != kNoSlot) {
              const uint32_t m = tab.mask[sl];
              const uint32_t bk = sl & (kLsBuckets - 1);
              int j = -1, st = step;
              // own step: the highest key lane below this one holding the slot
              if ((m >> step) & 1u)
                j = lane_with_slot(s_ls[step * kLsBuckets + bk] & lanemask_lt(), s_ks + step * 32, sl);
              // else the latest earlier step holding it: its highest lane with the slot
              const uint32_t me = m & ((1u << step) - 1u);
              if (j < 0 && me) {
                st = 31 - __clz(me);
                j = lane_with_slot(s_ls[st * kLsBuckets + bk], s_ks + st * 32, sl);
              }
              a = j >= 0 ? base32 + st * 32 + j
                         : static_cast<int32_t>(tab.carry[sl]) - 1;  // 0 (none) gives -1
            }
            if (valid) ab[i] = a;
          }
          match_barrier();
          // ---------------------------------------------- P3: carries
#pragma unroll
          for (int u = 0; u < kPerLane; ++u) {
            const int step = warp + u * kMatchWarps;
            if (step >= kSteps || kslot[u] == kNoSlot) continue;
            s_ls[step * kLsBuckets + (kslot[u] & (kLsBuckets - 1))] = 0u;  // clean for the next chunk
            // every key of the chunk: the latest one per slot becomes the carry (one atomic max
            // per key is cheaper than finding each slot's last step first)
            atomicMax(tab.carry + kslot[u], static_cast<uint32_t>(base32 + step * 32 + lane + 1));
            tab.mask[kslot[u]] = 0u;
          }
        }
      }
      __syncthreads();
      if (kSmemTable ? s_used[(r + 1) & 1] > overflow_limit<CodeT>() : s_ovf != 0) {
        aborted = true;
        break;
      }
      if (kPipe && tid == 0 && ((r + 1) % kUnitChunks == 0 || r + 1 == n_chunks)) {
        // every thread's indices of chunks <= r are stored (barrier above): a release store
        // by one thread after the barrier publishes them
        st_release(p.progress + n, static_cast<uint32_t>(r + 1));
      }
    }

    if constexpr (kSeg) {
      if (tid == 0) s_abort = aborted ? 1u : 0u;
      seg_resolve<CodeT>(p, tab, n, r_lo, r_hi, seg_rank, seg_count, tid, &s_abort);
      continue;
    }
    if (aborted) {
      if (tid == 0) {
        if (kSmemTable) {
          const uint32_t k = atomicAdd(p.ovf_count, 1u);
          p.ovf_list[k] = static_cast<uint32_t>(n);
          if (kPipe) st_release(p.progress + n, kProgOvf);  // its rows are gathered there
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
      for (uint32_t s = tid; s <= tab.cap; s += kThreads) {
        CodeT c;
        uint32_t m;
        if (tab.used(s, c, m) && m != Tab::kNoCarry) {
          const uint32_t k = atomicAdd(&s_lt, 1u);
          ltc[k] = c;
          ltp[k] = static_cast<int32_t>(m - 1);
        }
      }
      __syncthreads();
      if (tid == 0) p.lt_count[n] = static_cast<int32_t>(s_lt);
    }
    __syncthreads();
    if (!kSmemTable && p.gather_inline) {
      // overflow path of a pipelined call: this CTA's own indices, visible after the barrier
      gather_span<uint4, kThreads>(p.g, n, 0u, static_cast<uint32_t>(p.T), tid);
      __syncthreads();
    }
  }
  // no stream left: copy rows with the others
  if constexpr (kPipe) pipe_gather<kThreads>(p, tid, reinterpret_cast<uint4*>(smem), stage_rows);
}


// ---------------------------------------------------------------- dictionary + sweep
// A second matcher for streams of at most kSweepMaxT positions. One CTA of kSwThreads threads
// owns a stream at a time (kSwPerSm CTAs per SM):
//   A (dictionary, order-free). Every key code goes into a shared-memory table of the stream's
//     distinct key codes, all threads at once; its slot is the key's ID. After a barrier every
//     query code is looked up: its ID is that slot, or kNone when no key of the stream holds
//     the code. Position i's two IDs (key | query << 16) are written over src[i], which the
//     sweep then reads and overwrites with the answer. Each lookup first tries the code's own
//     slot (one shared load); the lanes that need more (a slot held by another code) are
//     queued per warp and served together after each round, so a warp pays for the longer
//     probe once per round instead of once per position.
//   B (sweep, ordered). One warp walks the stream in steps of 32 positions with two arrays
//     indexed by ID, laid over the table's memory:
//       last[id]   1 + the latest key position with that ID before the step (0: none)
//       lanes[id]  the step's key lanes holding that ID (cleared after every step)
//     Per step: keys OR their lane into lanes[id]; a query answers with the highest key lane
//     below its own in lanes[its id], else last[its id] - 1; the highest key lane of each ID
//     writes last[id]. About twenty warp instructions per 32 positions, no divergence.
// Used for calls without value rows (src only) of at least one wave of CTAs (kSwPerSm per SM
// on half the SMs): measured on config 2 (512 streams x 16384) 0.149 ms against the chunked
// matcher's 0.181 ms. Its cost per stream is a latency chain (phase B: ~64 us at T = 16384)
// rather than issue slots, so with fewer streams the chunked matcher, whose 32 warps share a
// stream, is faster, and with value rows the row copy (bandwidth-bound, ~0.13 ms) dominates
// either way: row traffic on the same SM slows the sweep's shared-memory chain, and copying
// rows through the bulk-copy engine instead topped out at ~2 TB/s for 48-byte rows.
// A stream whose distinct key codes would load the table beyond kOverflowFrac goes to the
// overflow path (the global-table match_kernel) as in the chunked path; results never depend
// on the path.
constexpr int kSwThreads = 256;
constexpr int kSwWarps = kSwThreads / 32;
constexpr int kSwPerSm = 4;
constexpr int64_t kSweepMaxT = 65535;  // 1 + a position fits the 16-bit last[] words
constexpr int kSwBatch = 16;           // steps whose IDs the sweep loads at once
constexpr uint32_t kPending = 0xFFFFFFFEu;  // own-slot attempt inconclusive: queued

template <typename CodeT>
struct SweepLayout {
  static constexpr uint32_t kSlots = SmemCap<CodeT>::kSlots;
  static constexpr uint32_t kSide = kSlots;       // slot of the all-ones code
  static constexpr uint32_t kDummy = kSlots + 1;  // key ID of lanes past the end
  static constexpr uint32_t kNone = kSlots + 2;   // query ID: no key holds the code
  static constexpr uint32_t kIds = kSlots + 3;
  static constexpr int kRound = sizeof(CodeT) == 4 ? 8 : 4;  // positions per thread per round
  static constexpr size_t kDictBytes = round_up16(kSlots * sizeof(CodeT) + sizeof(uint32_t));
  // per warp during phase A: codes and positions of the queued lanes of one round
  static constexpr size_t kQueueCodeBytes = round_up16(kRound * 32 * sizeof(CodeT));
  static constexpr size_t kQueueBytes = kQueueCodeBytes + round_up16(kRound * 32 * sizeof(uint16_t));
  static constexpr size_t kPhaseABytes = kDictBytes + kSwWarps * kQueueBytes;
  static constexpr size_t kLanesBytes = round_up16(kIds * sizeof(uint32_t));
  static constexpr size_t kLastBytes = round_up16(kIds * sizeof(uint16_t));
  static constexpr size_t kBytes =
      kPhaseABytes > kLanesBytes + kLastBytes ? kPhaseABytes : kLanesBytes + kLastBytes;
  static_assert(kIds < 65536, "IDs are 16-bit");
};

// The code's own slot only: the slot, kNoSlot (find: the own slot is free, so the code is
// absent), or kPending (the slot holds another code; the all-ones code always queues).
template <typename Tab, typename CodeT>
__device__ __forceinline__ uint32_t own_insert(Tab& tab, CodeT c, uint32_t& claimed) {
  if (c == Tab::kFree) return kPending;
  const uint32_t h = Tab::mix(c);
  const uint32_t o = tab.own(h, h >> tab.bshift);
  const CodeT cur = tab.code[o];
  if (cur == c) return o;
  if (cur == Tab::kFree) {
    const CodeT old = cas_code(tab.code + o, Tab::kFree, c);
    if (old == Tab::kFree) {
      claimed = 1;
      return o;
    }
    if (old == c) return o;
  }
  return kPending;
}
template <typename Tab, typename CodeT>
__device__ __forceinline__ uint32_t own_find(const Tab& tab, CodeT c) {
  if (c == Tab::kFree) return kPending;
  const uint32_t h = Tab::mix(c);
  const uint32_t o = tab.own(h, h >> tab.bshift);
  const CodeT cur = tab.code[o];
  if (cur == c) return o;
  return cur == Tab::kFree ? kNoSlot : kPending;
}

// Queue the lanes whose slot[u] is kPending (their code and position) in this warp's queue;
// returns the count. Entry order: round item u, then lane.
template <typename L, typename CodeT>
__device__ __forceinline__ uint32_t queue_pending(const uint32_t (&slot)[L::kRound], const CodeT (&c)[L::kRound],
                                                  uint32_t i0, int tid, CodeT* qcode, uint16_t* qpos) {
  uint32_t n = 0;
#pragma unroll
  for (int u = 0; u < L::kRound; ++u) {
    const bool pend = slot[u] == kPending;
    const uint32_t m = __ballot_sync(kFullMask, pend);
    if (pend) {
      const uint32_t e = n + __popc(m & lanemask_lt());
      qcode[e] = c[u];
      qpos[e] = static_cast<uint16_t>(i0 + u * kSwThreads + tid);
    }
    n += __popc(m);
  }
  __syncwarp();
  return n;
}

// Phase A, keys: every key code of the stream into the table; the low half of ids[i] = the
// key's slot. No barrier between rounds (a barrier would wait for the next round's code loads,
// issued one round ahead): a thread whose claims push the table past the overflow limit
// raises s_over, and every warp stops at its next round. Ends with a barrier; the caller then
// reads s_over.
template <typename L, typename CodeT, typename Tab>
__device__ __forceinline__ void dict_keys(Tab& tab, const CodeT* kc, uint32_t T, uint32_t* ids, int tid,
                                          CodeT* qcode, uint16_t* qpos, uint32_t* s_claims,
                                          volatile uint32_t* s_over) {
  constexpr uint32_t kLimit = overflow_limit<CodeT>();
  constexpr int R = L::kRound;
  constexpr uint32_t kStride = kSwThreads * R;
  const int lane = tid & 31;
  CodeT nxt[R];
#pragma unroll
  for (int u = 0; u < R; ++u) {
    const uint32_t i = u * kSwThreads + tid;
    nxt[u] = i < T ? kc[i] : CodeT(0);
  }
  for (uint32_t i0 = 0; i0 < T; i0 += kStride) {
    // one read per warp, broadcast: the whole warp leaves together
    if (__shfl_sync(kFullMask, *s_over, 0) != 0u) break;
    CodeT c[R];
    uint32_t slot[R];
    uint32_t claims = 0;
#pragma unroll
    for (int u = 0; u < R; ++u) {
      c[u] = nxt[u];
      const uint32_t i = i0 + kStride + u * kSwThreads + tid;
      nxt[u] = i < T ? kc[i] : CodeT(0);
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const uint32_t i = i0 + u * kSwThreads + tid;
      slot[u] = kNoSlot;
      if (i < T) {
        uint32_t cl = 0;
        slot[u] = own_insert(tab, c[u], cl);
        claims += cl;
        if (slot[u] != kPending) reinterpret_cast<uint16_t*>(ids + i)[0] = static_cast<uint16_t>(slot[u]);
      }
    }
    const uint32_t nq = queue_pending<L>(slot, c, i0, tid, qcode, qpos);
    bool bad = false;
    for (uint32_t e = lane; e < nq; e += 32) {
      uint32_t cl = 0;
      const uint32_t sl = tab.insert_fast(qcode[e], cl);
      claims += cl;
      bad |= sl == kNoSlot;
      reinterpret_cast<uint16_t*>(ids + qpos[e])[0] = static_cast<uint16_t>(sl);
    }
    if ((claims != 0 && atomicAdd(s_claims, claims) + claims > kLimit) || bad) *s_over = 1u;
    __syncwarp();  // the queue is refilled next round
  }
  __syncthreads();
}

// Phase A, queries (after the keys): the high half of ids[i] = the slot of the query's code,
// or kNone.
template <typename L, typename CodeT, typename Tab>
__device__ __forceinline__ void dict_queries(const Tab& tab, const CodeT* qc, uint32_t T, uint32_t* ids,
                                             int tid, CodeT* qcode, uint16_t* qpos) {
  constexpr int R = L::kRound;
  constexpr uint32_t kStride = kSwThreads * R;
  const int lane = tid & 31;
  CodeT nxt[R];
#pragma unroll
  for (int u = 0; u < R; ++u) {
    const uint32_t i = u * kSwThreads + tid;
    nxt[u] = i < T ? qc[i] : CodeT(0);
  }
  for (uint32_t i0 = 0; i0 < T; i0 += kStride) {
    CodeT c[R];
    uint32_t slot[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      c[u] = nxt[u];
      const uint32_t i = i0 + kStride + u * kSwThreads + tid;
      nxt[u] = i < T ? qc[i] : CodeT(0);
    }
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const uint32_t i = i0 + u * kSwThreads + tid;
      slot[u] = kNoSlot;
      if (i < T) {
        slot[u] = own_find(tab, c[u]);
        if (slot[u] != kPending)
          reinterpret_cast<uint16_t*>(ids + i)[1] = static_cast<uint16_t>(slot[u] == kNoSlot ? L::kNone : slot[u]);
      }
    }
    const uint32_t nq = queue_pending<L>(slot, c, i0, tid, qcode, qpos);
    for (uint32_t e = lane; e < nq; e += 32) {
      const uint32_t sl = tab.find_fast(qcode[e]);
      reinterpret_cast<uint16_t*>(ids + qpos[e])[1] = static_cast<uint16_t>(sl == kNoSlot ? L::kNone : sl);
    }
    __syncwarp();  // the queue is refilled next round
  }
}

// Phase B by one warp: ids[i] (key ID | query ID << 16) becomes the answer for position i.
// The IDs of kSwBatch steps are loaded at once and their answers stored at once: a global
// access pending at a __syncwarp costs the step its whole latency.
template <typename L>
__device__ __forceinline__ void sweep_warp(uint32_t* ids, uint32_t T, uint32_t* lanes, uint16_t* last,
                                           int lane) {
  constexpr uint32_t kTail = (L::kNone << 16) | L::kDummy;
  const uint32_t steps = (T + 31) / 32;
  const uint32_t below = lanemask_lt();
  int32_t* ans_out = reinterpret_cast<int32_t*>(ids);
  for (uint32_t s0 = 0; s0 < steps; s0 += kSwBatch) {
    uint32_t id[kSwBatch];
    int32_t a[kSwBatch];
#pragma unroll
    for (int d = 0; d < kSwBatch; ++d) {
      const uint32_t i = (s0 + d) * 32 + lane;
      id[d] = i < T ? ids[i] : kTail;
    }
    // steps past the end (last batch) run on the tail IDs: a dummy key and a query of no code
#pragma unroll
    for (int d = 0; d < kSwBatch; ++d) {
      const uint32_t st = s0 + d;
      const uint32_t k = id[d] & 0xFFFFu, q = id[d] >> 16;
      atomicOr(lanes + k, 1u << lane);
      __syncwarp();
      const uint32_t mq = lanes[q], mk = lanes[k];
      const uint32_t lq = last[q];
      const uint32_t bel = mq & below;
      a[d] = bel ? static_cast<int32_t>(st * 32 + 31 - __clz(bel)) : static_cast<int32_t>(lq) - 1;
      __syncwarp();
      if (31 - __clz(mk) == lane) last[k] = static_cast<uint16_t>(st * 32 + lane + 1);
      lanes[k] = 0u;
      __syncwarp();
    }
#pragma unroll
    for (int d = 0; d < kSwBatch; ++d) {
      const uint32_t i = (s0 + d) * 32 + lane;
      if (i < T) ans_out[i] = a[d];
    }
  }
}

template <typename CodeT>
__global__ void __launch_bounds__(kSwThreads, kSwPerSm) sweep_kernel(const Params p) {
  griddep_launch();  // the overflow path may be placed once every sweep CTA runs
  using L = SweepLayout<CodeT>;
  using Tab = Table<CodeT, uint32_t>;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint32_t s_claims, s_lt;
  __shared__ volatile uint32_t s_over;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const CodeT* qc = static_cast<const CodeT*>(p.qc);
  const CodeT* kc = static_cast<const CodeT*>(p.kc);
  const uint32_t T = static_cast<uint32_t>(p.T);
  Tab tab;
  tab.init_dict(smem, L::kSlots);
  CodeT* qcode = reinterpret_cast<CodeT*>(smem + L::kDictBytes + warp * L::kQueueBytes);
  uint16_t* qpos = reinterpret_cast<uint16_t*>(smem + L::kDictBytes + warp * L::kQueueBytes + L::kQueueCodeBytes);
  uint32_t* lanes = reinterpret_cast<uint32_t*>(smem);
  uint16_t* last = reinterpret_cast<uint16_t*>(smem + L::kLanesBytes);
  for (int64_t n = blockIdx.x; n < p.N; n += gridDim.x) {
    const int64_t row0 = n * p.T;
    uint32_t* ids = reinterpret_cast<uint32_t*>(p.src + row0);
    // ------------------------------------------------ A: the dictionary
    for (uint32_t s = tid; s < L::kSlots; s += kSwThreads) tab.code[s] = Tab::kFree;
    if (tid == 0) {
      *tab.side = 0u;
      s_claims = 0u;
      s_over = 0u;
      s_lt = 0u;
    }
    __syncthreads();
    dict_keys<L>(tab, kc + row0, T, ids, tid, qcode, qpos, &s_claims, &s_over);
    const bool over = s_over != 0u;
    if (!over) dict_queries<L>(tab, qc + row0, T, ids, tid, qcode, qpos);
    __syncthreads();
    if (over) {
      if (tid == 0) {
        const uint32_t k = atomicAdd(p.ovf_count, 1u);
        p.ovf_list[k] = static_cast<uint32_t>(n);
      }
      continue;  // every thread is past the last read of the table
    }
    // ------------------------------------------------ B: the sweep, over the table's memory
    for (uint32_t s = tid; s < L::kIds; s += kSwThreads) {
      lanes[s] = 0u;
      last[s] = 0;
    }
    __syncthreads();
    if (warp == 0) sweep_warp<L>(ids, T, lanes, last, lane);
    __syncthreads();
    if (p.lt_count != nullptr) {
      // last-occurrence table: every key code of the stream with its last position
      CodeT* ltc = static_cast<CodeT*>(p.lt_code) + row0;
      int32_t* ltp = p.lt_pos + row0;
      for (uint32_t s = tid; s <= L::kSide; s += kSwThreads) {
        const uint32_t l = last[s];
        if (l != 0u) {
          const uint32_t k = atomicAdd(&s_lt, 1u);
          ltc[k] = kc[row0 + l - 1];
          ltp[k] = static_cast<int32_t>(l - 1);
        }
      }
      __syncthreads();
      if (tid == 0) p.lt_count[n] = static_cast<int32_t>(s_lt);
    }
    __syncthreads();  // the arrays are cleared for the next stream
  }
}

// ---------------------------------------------------------------- the value gather
// out[n][i] = v[n][src[n][i]] (vbytes-byte rows), zeros where src is -1: the two-kernel path
// (rows not 16-byte aligned, 64-bit codes, no room for the pipelined mode's control words).
// Value traffic in the same SM as the matcher's shared-memory table multiplies the latency of
// every table access, so the two never share SMs. Each CTA owns one
// contiguous run of output words of one stream (blockIdx.y), kGUnroll loads in flight per
// thread, streaming stores.
constexpr int kGThreads = 256;
template <typename Vec>
__global__ void __launch_bounds__(kGThreads) gather_kernel(const GatherParams g) {
  griddep_wait();  // the indices of the kernels before it
  const uint32_t w0 = blockIdx.x * (kGThreads * kGUnroll) + threadIdx.x;
  for (int64_t n = blockIdx.y; n < g.N; n += gridDim.y) {
    const int32_t* src = g.src + n * g.T;
    const int64_t b = n / g.heads, h = n - b * g.heads;
    const unsigned char* v = g.v + b * g.v_sb + h * g.v_sh;
    unsigned char* o = g.out + b * g.o_sb + h * g.o_sh;
    Vec val[kGUnroll];
    uint32_t row[kGUnroll], col[kGUnroll];
#pragma unroll
    for (int u = 0; u < kGUnroll; ++u) {
      const uint32_t w = w0 + u * kGThreads;
      val[u] = zero_vec<Vec>();
      row[u] = 0;
      col[u] = 0;
      if (w < g.words) {
        const uint32_t r = g.div_shift >= 0 ? (w >> g.div_shift)
                                            : (g.div_magic ? __umulhi(w, g.div_magic) : w / g.wpr);
        row[u] = r;
        col[u] = w - r * g.wpr;
        const int32_t s = __ldg(src + r);
        if (s >= 0) val[u] = __ldg(reinterpret_cast<const Vec*>(v + s * g.v_st) + col[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < kGUnroll; ++u) {
      const uint32_t w = w0 + u * kGThreads;
      if (w < g.words) store_stream(reinterpret_cast<Vec*>(o + row[u] * g.o_st) + col[u], val[u]);
    }
  }
}

template <typename Vec>
int make_gather(const MatchLaunch& a, const int32_t* src, GatherParams& g) {
  g = GatherParams{};
  g.src = src;
  g.v = static_cast<const unsigned char*>(a.v);
  g.out = static_cast<unsigned char*>(a.out);
  g.N = a.N;
  g.T = a.T;
  if (a.heads > 0) {
    g.heads = a.heads;
    g.v_sb = a.v_sb; g.v_sh = a.v_sh; g.v_st = a.v_st;
    g.o_sb = a.o_sb; g.o_sh = a.o_sh; g.o_st = a.o_st;
  } else {
    g.heads = 1;
    g.v_sb = g.o_sb = a.T * a.vbytes;
    g.v_sh = g.o_sh = 0;
    g.v_st = g.o_st = a.vbytes;
  }
  const uint64_t wpr = static_cast<uint64_t>(a.vbytes) / sizeof(Vec);
  const uint64_t words = static_cast<uint64_t>(a.T) * wpr;
  if (words >= (uint64_t(1) << 32)) return fail(LEMA_ERR_INVALID_ARGUMENT, "T * row words = %llu exceeds 2^32", (unsigned long long)words);
  g.wpr = static_cast<uint32_t>(wpr);
  g.words = static_cast<uint32_t>(words);
  g.div_shift = -1;
  g.div_magic = 0;
  if ((wpr & (wpr - 1)) == 0) {
    g.div_shift = log2_exact(wpr);
  } else if (words * wpr < (uint64_t(1) << 32)) {  // multiply-high is exact for w * wpr < 2^32
    g.div_magic = static_cast<uint32_t>(0xFFFFFFFFull / wpr + 1);
  }
  return LEMA_OK;
}

template <typename Vec>
int launch_gather(const MatchLaunch& a, const int32_t* src) {
  GatherParams g;
  const int rc = make_gather<Vec>(a, src, g);
  if (rc != LEMA_OK) return rc;
  const uint64_t words = g.words;
  const uint64_t per_cta = kGThreads * kGUnroll;
  const dim3 grid(static_cast<unsigned>((words + per_cta - 1) / per_cta),
                  static_cast<unsigned>(std::min<int64_t>(a.N, 65535)));
  LEMA_CUDA_TRY(launch_dependent(gather_kernel<Vec>, grid, dim3(kGThreads), 0, a.stream, g));
  return LEMA_OK;
}

// every row starts on a 16-byte boundary: pointers, row size and (strided) strides
bool rows_16(const MatchLaunch& a) {
  const uint64_t st = a.heads > 0 ? static_cast<uint64_t>(a.v_sb | a.v_sh | a.v_st | a.o_sb | a.o_sh | a.o_st) : 0;
  return a.vbytes % 16 == 0 && st % 16 == 0 && aligned(a.v, 16) && aligned(a.out, 16);
}

int run_gather(const MatchLaunch& a, const int32_t* src) {
  // every row must start on the vector boundary: pointers, row size and (strided) strides
  const uint64_t st = a.heads > 0 ? static_cast<uint64_t>(a.v_sb | a.v_sh | a.v_st | a.o_sb | a.o_sh | a.o_st) : 0;
  const bool a16 = rows_16(a);
  const bool a8 = a.vbytes % 8 == 0 && st % 8 == 0 && aligned(a.v, 8) && aligned(a.out, 8);
  const bool a4 = a.vbytes % 4 == 0 && st % 4 == 0 && aligned(a.v, 4) && aligned(a.out, 4);
  if (a16) return launch_gather<uint4>(a, src);
  if (a8) return launch_gather<uint2>(a, src);
  if (a4) return launch_gather<uint32_t>(a, src);
  return launch_gather<unsigned short>(a, src);
}

// ---------------------------------------------------------------- host side
// per-step lane sets and key slots
template <bool kSmemTable>
constexpr size_t chunk_smem() {
  return kSteps * (kLsBuckets + 32) * sizeof(uint32_t);  // lane-set buckets and key slots
}
constexpr int64_t kMaxOverflowTables = 64;
constexpr uint64_t kOverflowTableBudget = uint64_t(1) << 30;  // bytes of global tables

template <typename CodeT>
size_t smem_bytes(bool smem_table) {
  return smem_table ? round_up16(Table<CodeT, uint32_t>::bytes(SmemCap<CodeT>::kSlots)) + chunk_smem<true>()
                    : chunk_smem<false>();
}

struct Plan {
  size_t off_src = 0;      // index scratch (used when the caller passes no src)
  bool fast = false;       // run the shared-memory kernel
  bool global = false;     // run the global-table kernel
  bool list_mode = false;  // global kernel reads the overflow list
  uint32_t gslots = 0;
  int64_t gtable_bytes = 0;
  int64_t n_gtables = 0;
  size_t off_list = 0, off_tables = 0, total = 0;
  // pipelined mode's control block and progress words, last; a workspace of min_total bytes
  // (without them) runs the two-kernel path
  size_t off_ctl = 0, ctl_bytes = 0, min_total = 0;
};

void add_ctl(Plan& pl, int64_t N) {
  pl.min_total = pl.total;
  pl.off_ctl = round_up(pl.total, 256);
  pl.ctl_bytes = round_up(sizeof(PipeCtl) + 4 * static_cast<size_t>(N), 256);
  pl.total = pl.off_ctl + pl.ctl_bytes;
}

// need_src: the caller passes no index output, so the indices live in the workspace.
Plan make_plan(int64_t N, int64_t T, int code_bytes, bool need_src = true) {
  Plan pl;
  if (N <= 0 || T <= 0) return pl;
  const uint32_t limit = code_bytes == 4 ? overflow_limit<uint32_t>() : overflow_limit<uint64_t>();
  pl.fast = true;  // any T: a stream with too many distinct keys moves to the global path
  const size_t src_bytes =
      need_src ? round_up(4 * static_cast<size_t>(N) * static_cast<size_t>(T), 256) : 0;
  pl.total = src_bytes;
  const bool may_overflow = T > static_cast<int64_t>(limit);
  if (!may_overflow) {
    add_ctl(pl, N);
    return pl;
  }
  pl.global = true;
  pl.list_mode = pl.fast;
  pl.gslots = static_cast<uint32_t>(next_pow2(static_cast<uint64_t>(std::max<int64_t>(2 * T, 2 * kBucket))));
  const size_t tb = code_bytes == 4 ? Table<uint32_t, uint32_t>::bytes(pl.gslots)
                                    : Table<uint64_t, uint32_t>::bytes(pl.gslots);
  pl.gtable_bytes = static_cast<int64_t>(round_up(tb, 256));
  pl.n_gtables = std::max<int64_t>(
      1, std::min<int64_t>({N, kMaxOverflowTables,
                            static_cast<int64_t>(kOverflowTableBudget / pl.gtable_bytes)}));
  pl.off_list = src_bytes + 256;
  pl.off_tables = round_up(pl.off_list + 4 * static_cast<size_t>(N), 256);
  pl.total = pl.off_tables + static_cast<size_t>(pl.n_gtables * pl.gtable_bytes);
  add_ctl(pl, N);
  return pl;
}

// The pipelined mode serves calls that gather 16-byte-aligned rows of at most 4 KiB (27 or more
// staged per pass), with the control words in the workspace, streams short enough that a
// unit's wait stays far below its bound, and unit and word counts inside 32 bits; and calls
// of at least one full wave of matchers (2 per SM): with fewer streams the two-kernel path
// runs each matcher alone on its SM, faster than two per SM on fewer SMs (measured: 128
// streams of config 2 take 0.185 ms in two kernels, 0.224 ms pipelined; 512 streams 0.344
// and 0.322). LEMA_K2_PIPELINE=0 in the environment selects the two-kernel path (the same
// results).
constexpr int64_t kPipeMaxT = int64_t(1) << 22;
bool use_pipe(const MatchLaunch& a, const Plan& pl, int sms) {
  const char* e = std::getenv("LEMA_K2_PIPELINE");
  const bool enabled = !(e != nullptr && e[0] == '0');
  if (!enabled || a.out == nullptr || pl.ctl_bytes == 0 || a.ws == nullptr || a.ws_bytes < pl.total ||
      !aligned(a.ws, 256))
    return false;
  if (!rows_16(a) || a.T > kPipeMaxT || a.vbytes > 4096 || a.N < 2 * static_cast<int64_t>(sms)) return false;
  const uint64_t ng = (static_cast<uint64_t>(a.T) + kChunk * kUnitChunks - 1) / (kChunk * kUnitChunks);
  const uint64_t words = static_cast<uint64_t>(a.T) * static_cast<uint64_t>(a.vbytes / 16);
  return static_cast<uint64_t>(a.N) * ng < (uint64_t(1) << 31) &&
         words + static_cast<uint64_t>(kThreads) * kGUnroll < (uint64_t(1) << 32);
}

// SMs that match: enough CTAs for the streams in whole waves, at most kMatchFrac of the SMs
// (LEMA_K2_MATCH_FRAC overrides), so that the others copy rows while the matching runs.
uint32_t match_sms(int64_t N, int per_sm, int sms) {
  const char* e = std::getenv("LEMA_K2_MATCH_FRAC");
  const double f = e != nullptr ? std::atof(e) : 0.0;
  const double frac = (f > 0.0 && f <= 1.0) ? f : 0.87;
  const int64_t cap = std::max<int64_t>(1, static_cast<int64_t>(frac * sms));
  const int64_t per_wave = static_cast<int64_t>(per_sm) * cap;
  const int64_t waves = (N + per_wave - 1) / per_wave;
  const int64_t per = static_cast<int64_t>(per_sm) * waves;
  return static_cast<uint32_t>(std::min<int64_t>(sms, (N + per - 1) / per));
}

template <typename CodeT>
int run_pipe(const MatchLaunch& a, const Plan& pl, const DeviceInfo& dev, Params p) {
  unsigned char* ws = static_cast<unsigned char*>(a.ws);
  int rc = make_gather<uint4>(a, p.src, p.g);
  if (rc != LEMA_OK) return rc;
  p.ctl = reinterpret_cast<PipeCtl*>(ws + pl.off_ctl);
  p.progress = reinterpret_cast<uint32_t*>(ws + pl.off_ctl + sizeof(PipeCtl));
  LEMA_CUDA_TRY(cudaMemsetAsync(ws + pl.off_ctl, 0, pl.ctl_bytes, a.stream));
  auto kern = match_kernel<CodeT, true, true>;
  const size_t sm = smem_bytes<CodeT>(true);
  int per_sm = 0;
  LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(kern), sm, kThreads, 0, &per_sm));
  per_sm = std::max(per_sm, 1);
  p.match_sms = match_sms(a.N, per_sm, dev.sms);
  p.wave = p.match_sms * static_cast<uint32_t>(per_sm);
  kern<<<static_cast<unsigned>(per_sm * dev.sms), kThreads, sm, a.stream>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  if (pl.global) {
    // streams that overflowed the shared-memory table: matched and gathered here
    p.list_mode = pl.list_mode ? 1 : 0;
    p.gather_inline = 1;
    auto gk = match_kernel<CodeT, false>;
    const size_t gsm = smem_bytes<CodeT>(false);
    LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(gk), gsm, 0, 0, nullptr));
    LEMA_CUDA_TRY(launch_dependent(gk, dim3(static_cast<unsigned>(pl.n_gtables)), dim3(kThreads), gsm, a.stream, p));
  }
  return LEMA_OK;
}

// The dictionary + sweep path serves calls without value rows of at least one wave of sweep
// CTAs and streams of at most kSweepMaxT positions. LEMA_K2_SWEEP=0 turns it off, =1 takes it
// for every call it can serve (rows then copied by the gather kernel); same results.
bool use_sweep(const MatchLaunch& a, const Plan& pl, int sms) {
  if (!pl.fast || a.T > kSweepMaxT) return false;
  const char* e = std::getenv("LEMA_K2_SWEEP");
  if (e != nullptr && e[0] == '0') return false;
  if (e != nullptr && e[0] == '1') return true;
  return a.out == nullptr && a.N >= static_cast<int64_t>(kSwPerSm) * sms / 2;
}

template <typename CodeT>
int run_sweep(const MatchLaunch& a, const Plan& pl, const DeviceInfo& dev, Params p) {
  auto kern = sweep_kernel<CodeT>;
  const size_t sm = SweepLayout<CodeT>::kBytes;
  int per_sm = 0;
  LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(kern), sm, kSwThreads, 0, &per_sm));
  const int64_t grid = std::min<int64_t>(a.N, static_cast<int64_t>(std::max(per_sm, 1)) * dev.sms);
  kern<<<static_cast<unsigned>(grid), kSwThreads, sm, a.stream>>>(p);
  LEMA_CUDA_TRY(cudaGetLastError());
  if (pl.global) {
    // streams that outgrew the shared-memory table are matched here
    p.list_mode = 1;
    p.gather_inline = 0;
    auto gk = match_kernel<CodeT, false>;
    const size_t gsm = smem_bytes<CodeT>(false);
    LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(gk), gsm, 0, 0, nullptr));
    LEMA_CUDA_TRY(launch_dependent(gk, dim3(static_cast<unsigned>(pl.n_gtables)), dim3(kThreads), gsm, a.stream, p));
  }
  if (a.out != nullptr) return run_gather(a, p.src);
  return LEMA_OK;
}

// Segments per stream for the two-kernel path: calls of fewer streams than SMs split each
// stream's chunks over a cluster of S CTAs (S = 2, 4 or 8: the most that keeps one CTA per SM,
// with runs of at least 2 chunks), so the chain of chunks each CTA walks is S times shorter.
// Measured on config 2's streams (T = 16384, rows gathered): 64 streams 0.084 -> 0.066 ms
// (S = 2 or 4); at 128 and 256 streams two CTAs per SM gain nothing (the matcher is then
// bound by its instruction issue, not its chain): 0.108 / 0.110 ms (S = 1 / 2), 0.174 / 0.202.
// Not for calls that export last-occurrence tables. LEMA_K2_SEGMENTS=1/2/4/8 overrides (the
// same results).
int seg_count(const MatchLaunch& a, int sms) {
  if (a.lt_count != nullptr) return 1;
  const int64_t n_chunks = (a.T + kChunk - 1) / kChunk;
  if (const char* e = std::getenv("LEMA_K2_SEGMENTS")) {
    const int s = std::atoi(e);
    if (s == 1 || s == 2 || s == 4 || s == 8) return n_chunks >= s ? s : 1;
  }
  int best = 1;
  for (int s = 2; s <= 8; s *= 2)
    if (a.N * s <= static_cast<int64_t>(sms) && n_chunks >= 2 * s) best = s;
  return best;
}

template <typename CodeT>
int run(const MatchLaunch& a, const Plan& pl, const DeviceInfo& dev) {
  unsigned char* ws = static_cast<unsigned char*>(a.ws);
  Params p{};
  p.wait_ns = wait_limit_ns();
  p.qc = a.qc;
  p.kc = a.kc;
  p.N = a.N;
  p.T = a.T;
  p.src = a.src ? a.src : reinterpret_cast<int32_t*>(ws + pl.off_src);
  p.lt_code = a.lt_code;
  p.lt_pos = a.lt_pos;
  p.lt_count = a.lt_count;
  p.status = a.status;
  if (pl.global) {
    p.ovf_count = reinterpret_cast<uint32_t*>(ws + pl.off_list - 256);
    p.ovf_list = reinterpret_cast<uint32_t*>(ws + pl.off_list);
    p.gtables = ws + pl.off_tables;
    p.gtable_bytes = pl.gtable_bytes;
    p.gslots = pl.gslots;
    if (pl.list_mode) LEMA_CUDA_TRY(cudaMemsetAsync(p.ovf_count, 0, sizeof(uint32_t), a.stream));
  }
  if (use_sweep(a, pl, dev.sms)) return run_sweep<CodeT>(a, pl, dev, p);
  if constexpr (sizeof(CodeT) == 4) {  // 64-bit codes: the two-kernel path (no spare registers)
    if (pl.fast && use_pipe(a, pl, dev.sms)) return run_pipe<CodeT>(a, pl, dev, p);
  }
  const int segs = pl.fast ? seg_count(a, dev.sms) : 1;
  bool seg_done = false;
  if (segs > 1) {
    auto kern = match_kernel<CodeT, true, false, true>;
    const size_t sm = smem_bytes<CodeT>(true);
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(segs);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = sm;
    cfg.stream = a.stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3(static_cast<unsigned>(a.N * segs), 1, 1);
    int clusters = 0;
    LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(kern), sm, kThreads, segs, &clusters));
    if (clusters >= 1) {  // else: one CTA per stream
      cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>(a.N, clusters) * segs), 1, 1);
      LEMA_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
      seg_done = true;
    }
  }
  if (pl.fast && !seg_done) {
    auto kern = match_kernel<CodeT, true>;
    const size_t sm = smem_bytes<CodeT>(true);
    int per_sm = 0;
    LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(kern), sm, kThreads, 0, &per_sm));
    const int64_t grid = std::min<int64_t>(a.N, static_cast<int64_t>(std::max(per_sm, 1)) * dev.sms);
    kern<<<static_cast<unsigned>(grid), kThreads, sm, a.stream>>>(p);
    LEMA_CUDA_TRY(cudaGetLastError());
  }
  if (pl.global) {
    p.list_mode = pl.list_mode ? 1 : 0;
    auto kern = match_kernel<CodeT, false>;
    const size_t sm = smem_bytes<CodeT>(false);
    LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(kern), sm, 0, 0, nullptr));
    LEMA_CUDA_TRY(launch_dependent(kern, dim3(static_cast<unsigned>(pl.n_gtables)), dim3(kThreads), sm, a.stream, p));
  }
  if (a.out != nullptr) return run_gather(a, p.src);
  return LEMA_OK;
}

}  // namespace k2

size_t match_workspace_bytes(int64_t N, int64_t T, int code_bytes, bool need_src, bool pipe) {
  const k2::Plan pl = k2::make_plan(N, T, code_bytes, need_src);
  return pipe ? pl.total : pl.min_total;
}

int launch_match(const MatchLaunch& a) {
  if (a.code_bytes != 4 && a.code_bytes != 8) return fail(LEMA_ERR_INVALID_ARGUMENT, "code_bytes must be 4 or 8, got %d", a.code_bytes);
  if (a.N < 0 || a.T < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "negative shape (%lld, %lld)", (long long)a.N, (long long)a.T);
  if (a.T > (int64_t(1) << 30)) return fail(LEMA_ERR_INVALID_ARGUMENT, "T = %lld exceeds 2^30", (long long)a.T);
  if (a.N == 0 || a.T == 0) return LEMA_OK;
  if (a.qc == nullptr || a.kc == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null code pointer");
  if (!aligned(a.qc, a.code_bytes) || !aligned(a.kc, a.code_bytes)) return fail(LEMA_ERR_INVALID_ARGUMENT, "codes not aligned to their width");
  if (a.out != nullptr) {
    if (a.v == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "out given without values");
    if (a.vbytes <= 0 || a.vbytes % 2 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "vbytes must be a positive multiple of 2, got %lld", (long long)a.vbytes);
    if (!aligned(a.v, 2) || !aligned(a.out, 2)) return fail(LEMA_ERR_INVALID_ARGUMENT, "value rows must be 2-byte aligned");
    if (static_cast<uint64_t>(a.T) * static_cast<uint64_t>(a.vbytes / 2) >= (uint64_t(1) << 32)) return fail(LEMA_ERR_INVALID_ARGUMENT, "T * vbytes too large for one stream (%lld x %lld)", (long long)a.T, (long long)a.vbytes);
  }
  const bool lt_any = a.lt_code || a.lt_pos || a.lt_count;
  if (lt_any && !(a.lt_code && a.lt_pos && a.lt_count)) return fail(LEMA_ERR_INVALID_ARGUMENT, "last-occurrence outputs: all three or none");
  const k2::Plan pl = k2::make_plan(a.N, a.T, a.code_bytes, a.src == nullptr);
  if (a.ws_bytes < pl.min_total || (pl.min_total > 0 && a.ws == nullptr)) {
    return fail(LEMA_ERR_WORKSPACE, "workspace of %zu bytes, %zu needed", a.ws_bytes, pl.min_total);
  }
  if (pl.min_total > 0 && !aligned(a.ws, 256)) return fail(LEMA_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
  return a.code_bytes == 4 ? k2::run<uint32_t>(a, pl, *dev) : k2::run<uint64_t>(a, pl, *dev);
}


// ---------------------------------------------------------------- no-allocation variant
// lema_prefill_match_noalloc: the same latest-match and gather for callers that cannot
// allocate device memory at all -- a plugin handed only its input and output tensors by a
// host engine that owns every byte of device memory, a C program without a device allocator,
// or a latency-critical loop where a cudaMalloc (which may block) or a cudaFree (which
// synchronises the device) is not allowed. Its scratch (the index scratch when the caller
// passes no src, the overflow list and the overflow-path tables) lives in the fixed array
// below: every GPU that loads this library holds these bytes until the process exits.
namespace k2 {

constexpr size_t kNoallocScratchBytes = size_t(32) << 20;  // 32 MiB, LEMA_NOALLOC_SCRATCH_BYTES
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoallocScratchBytes];

// make_plan for a fixed scratch size: the overflow path gets as many CTA-private tables as
// fit (at least one). `fits` is false when even the index scratch plus one table does not.
Plan make_plan_within(int64_t N, int64_t T, int code_bytes, bool need_src, size_t budget, bool& fits) {
  Plan pl;
  fits = true;
  if (N <= 0 || T <= 0) return pl;
  const uint32_t limit = code_bytes == 4 ? overflow_limit<uint32_t>() : overflow_limit<uint64_t>();
  pl.fast = true;
  const size_t src_bytes = need_src ? round_up(4 * static_cast<size_t>(N) * static_cast<size_t>(T), 256) : 0;
  pl.off_src = 0;
  pl.total = src_bytes;
  if (T > static_cast<int64_t>(limit)) {
    pl.global = true;
    pl.list_mode = true;
    pl.gslots = static_cast<uint32_t>(next_pow2(static_cast<uint64_t>(std::max<int64_t>(2 * T, 2 * kBucket))));
    const size_t tb = code_bytes == 4 ? Table<uint32_t, uint32_t>::bytes(pl.gslots)
                                      : Table<uint64_t, uint32_t>::bytes(pl.gslots);
    pl.gtable_bytes = static_cast<int64_t>(round_up(tb, 256));
    pl.off_list = src_bytes + 256;  // the overflow count sits in the 256 bytes before the list
    pl.off_tables = round_up(pl.off_list + 4 * static_cast<size_t>(N), 256);
    if (pl.off_tables + static_cast<size_t>(pl.gtable_bytes) > budget) {
      fits = false;
      pl.total = pl.off_tables + static_cast<size_t>(pl.gtable_bytes);
      pl.min_total = pl.total;
      return pl;
    }
    pl.n_gtables = std::min<int64_t>(
        {N, kMaxOverflowTables, static_cast<int64_t>((budget - pl.off_tables) / pl.gtable_bytes)});
    pl.total = pl.off_tables + static_cast<size_t>(pl.n_gtables * pl.gtable_bytes);
  }
  fits = pl.total <= budget;
  pl.min_total = pl.total;
  if (fits) {
    Plan q = pl;
    add_ctl(q, N);
    if (q.total <= budget) pl = q;  // room for the pipelined mode's control words
  }
  return pl;
}

// Device address of the array on each device, looked up with that device current (in host
// code the array's name is only a host-side stand-in for it) by the first call on the device
// and kept; a failed look-up is not kept, so the next call tries again. The address does not
// survive cudaDeviceReset.
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64];

}  // namespace k2
}  // namespace lema

extern "C" int lema_prefill_match_noalloc(const void* qcodes, const void* kcodes, int code_bytes,
                                          int64_t n_streams, int64_t T, int32_t* src,
                                          const void* values, int64_t vbytes, void* out,
                                          uint32_t* status, void* stream) {
  using namespace lema;
  clear_error();
  if (code_bytes != 4 && code_bytes != 8) return fail(LEMA_ERR_INVALID_ARGUMENT, "code_bytes must be 4 or 8, got %d", code_bytes);
  if (n_streams < 0 || T < 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "negative shape (%lld, %lld)", (long long)n_streams, (long long)T);
  if (T > (int64_t(1) << 30)) return fail(LEMA_ERR_INVALID_ARGUMENT, "T = %lld exceeds 2^30", (long long)T);
  if (n_streams == 0 || T == 0) return LEMA_OK;
  if (qcodes == nullptr || kcodes == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null code pointer");
  if (!aligned(qcodes, code_bytes) || !aligned(kcodes, code_bytes)) return fail(LEMA_ERR_INVALID_ARGUMENT, "codes not aligned to their width");
  if (out != nullptr) {
    if (values == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "out given without values");
    if (vbytes <= 0 || vbytes % 2 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "vbytes must be a positive multiple of 2, got %lld", (long long)vbytes);
    if (!aligned(values, 2) || !aligned(out, 2)) return fail(LEMA_ERR_INVALID_ARGUMENT, "value rows must be 2-byte aligned");
    if (static_cast<uint64_t>(T) * static_cast<uint64_t>(vbytes / 2) >= (uint64_t(1) << 32)) return fail(LEMA_ERR_INVALID_ARGUMENT, "T * vbytes too large for one stream (%lld x %lld)", (long long)T, (long long)vbytes);
  }
  bool fits = true;
  const k2::Plan pl = k2::make_plan_within(n_streams, T, code_bytes, src == nullptr, k2::kNoallocScratchBytes, fits);
  if (!fits) {
    return fail(LEMA_ERR_WORKSPACE,
                "%lld streams x %lld positions need %zu bytes of scratch, more than the %zu of "
                "lema_prefill_match_noalloc: pass src, split the streams over several calls, or "
                "use lema_prefill_match with a caller-owned workspace",
                (long long)n_streams, (long long)T, pl.total, k2::kNoallocScratchBytes);
  }
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
  const int d = dev->device;
  if (d < 0 || d >= 64) return fail(LEMA_ERR_UNSUPPORTED, "device ordinal %d: lema_prefill_match_noalloc serves devices 0..63", d);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(k2::g_noalloc_mu);
    if (k2::g_noalloc_ptr[d] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, k2::g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(noalloc scratch)");
      k2::g_noalloc_ptr[d] = p;
    }
    scratch = k2::g_noalloc_ptr[d];
  }
  MatchLaunch m;
  m.qc = qcodes;
  m.kc = kcodes;
  m.code_bytes = code_bytes;
  m.N = n_streams;
  m.T = T;
  m.src = src;
  m.v = values;
  m.vbytes = vbytes;
  m.out = out;
  m.ws = scratch;
  m.ws_bytes = k2::kNoallocScratchBytes;
  m.status = status;
  m.stream = static_cast<cudaStream_t>(stream);
  return code_bytes == 4 ? k2::run<uint32_t>(m, pl, *dev) : k2::run<uint64_t>(m, pl, *dev);
}
