/*
 * CPU ORACLE of the LEMA inference hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the algorithm of the reference
 * (moritzbroe/latest_exact_match_attention) for the paths the B200 library
 * implements. It exists to CHECK the CUDA library: only tests/, the smoke test of
 * __graft_entry__.py and the cpu_baseline leg of bench.py may load it. It is never
 * part of the product path and never a fallback for it.
 *
 * Pinning: the outputs of these functions are compared, in tests/, against golden
 * vectors produced by the reference's own code (code/lema/attention.py and
 * code/lema/csrc/store.cpp, run in the build container by
 * tests/golden/make_golden.py) and against the reference's C++ store compiled from
 * its own source (oracle/build_ref.py -> oracle/_ref/).
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* A 64-bit mixer (MurmurHash3 fmix64) -- any full-avalanche mixer serves: slot
 * placement is not observable through any of the functions below. */
static uint64_t mix64(uint64_t k) {
  k ^= k >> 33;
  k *= 0xFF51AFD7ED558CCDull;
  k ^= k >> 33;
  k *= 0xC4CEB9FE1A85EC53ull;
  k ^= k >> 33;
  return k;
}

static uint64_t load_code(const void* p, int code_bytes, int64_t i) {
  if (code_bytes == 2) return ((const uint16_t*)p)[i];
  if (code_bytes == 4) return ((const uint32_t*)p)[i];
  return ((const uint64_t*)p)[i];
}

/*
 * latest_prev_match: src[n][i] = max{ j < i : kc[n][j] == qc[n][i] }, else -1.
 *
 * Follows the definition of code/lema/attention.py:100-132 ("For each i, the largest
 * j < i with kc[j] == qc[i], else -1") in the dictionary form the reference states at
 * verification/lema.py:19-33 and executes at code/lema/csrc/store.cpp:151-157: walk the
 * positions in order, look the query up in {code -> last key position}, then record
 * the key. The reference's batched version sorts events instead; both compute the
 * same function, which the golden vectors pin.
 * Returns 0, or -1 if memory could not be allocated.
 */
int oracle_latest_prev_match(const void* qc, const void* kc, int code_bytes, int64_t N,
                             int64_t T, int64_t* src) {
  if (N <= 0 || T <= 0) return 0;
  uint64_t cap = 16;
  while (cap < (uint64_t)(2 * T)) cap <<= 1;
  uint64_t* codes = (uint64_t*)malloc(cap * sizeof(uint64_t));
  int64_t* last = (int64_t*)malloc(cap * sizeof(int64_t));
  if (!codes || !last) {
    free(codes);
    free(last);
    return -1;
  }
  const uint64_t mask = cap - 1;
  for (int64_t n = 0; n < N; ++n) {
    for (uint64_t s = 0; s < cap; ++s) last[s] = -2; /* -2 = free slot */
    const int64_t row = n * T;
    for (int64_t i = 0; i < T; ++i) {
      /* look the query up */
      const uint64_t q = load_code(qc, code_bytes, row + i);
      int64_t hit = -1;
      for (uint64_t s = mix64(q) & mask;; s = (s + 1) & mask) {
        if (last[s] == -2) break;
        if (codes[s] == q) {
          hit = last[s];
          break;
        }
      }
      src[row + i] = hit;
      /* then record the key: latest wins */
      const uint64_t k = load_code(kc, code_bytes, row + i);
      for (uint64_t s = mix64(k) & mask;; s = (s + 1) & mask) {
        if (last[s] == -2) {
          codes[s] = k;
          last[s] = i;
          break;
        }
        if (codes[s] == k) {
          last[s] = i;
          break;
        }
      }
    }
  }
  free(codes);
  free(last);
  return 0;
}

/*
 * The value gather of code/lema/attention.py:157-158: out[n][i] = v[n][src] or zeros.
 * Rows are opaque bytes (vbytes each).
 */
void oracle_gather(const int64_t* src, const uint8_t* v, int64_t N, int64_t T, int64_t vbytes,
                   uint8_t* out) {
  for (int64_t n = 0; n < N; ++n) {
    for (int64_t i = 0; i < T; ++i) {
      const int64_t s = src[n * T + i];
      uint8_t* o = out + (n * T + i) * vbytes;
      if (s >= 0)
        memcpy(o, v + (n * T + s) * vbytes, (size_t)vbytes);
      else
        memset(o, 0, (size_t)vbytes);
    }
  }
}

/*
 * The store exchange of code/lema/csrc/store.cpp:122-162, single-threaded.
 *
 * One table of `cap` slots shared by every group; slot = [code u64 | state u64 | value]
 * with state 0 = empty and group + 2 = occupied (store.cpp:3-16), linear probing. Items
 * are partition-major: item i is position i % T of partition i / T, group g0 + i / T.
 * Each item looks its query up into out[i] (zeros on a miss, store.cpp:84-93) and then
 * inserts its key with its value, latest write wins (store.cpp:97-117); added[p] counts
 * the slots partition p newly claims. Returns 0, or 1 when an insert found every slot
 * taken ("hash table full", store.cpp:159-160) -- the remaining items still run.
 * `table` is caller-owned, cap * (16 + vbytes) bytes, zero-filled before first use.
 */
int oracle_store_exchange(uint8_t* table, int64_t cap, int64_t vbytes, const void* qc,
                          const void* kc, int code_bytes, const uint8_t* values, uint8_t* out,
                          int64_t n, int64_t T, int64_t g0, int64_t* added) {
  const int64_t stride = 16 + vbytes;
  int full = 0;
  if (T <= 0 || n % T) return 2;
  for (int64_t p = 0; p < n / T; ++p) added[p] = 0;
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t g = (uint64_t)(g0 + i / T), tag = g + 2;
    const uint64_t hg = mix64(g ^ 0x2545F4914F6CDD1Dull);
    /* lookup */
    const uint64_t q = load_code(qc, code_bytes, i);
    int64_t s = (int64_t)(mix64(q ^ hg) % (uint64_t)cap);
    int hit = 0;
    for (int64_t t = 0; t < cap; ++t, s = (s + 1 == cap) ? 0 : s + 1) {
      uint64_t* h = (uint64_t*)(table + s * stride);
      if (h[1] == 0) break;
      if (h[1] == tag && h[0] == q) {
        memcpy(out + i * vbytes, table + s * stride + 16, (size_t)vbytes);
        hit = 1;
        break;
      }
    }
    if (!hit) memset(out + i * vbytes, 0, (size_t)vbytes);
    /* insert */
    const uint64_t k = load_code(kc, code_bytes, i);
    s = (int64_t)(mix64(k ^ hg) % (uint64_t)cap);
    int done = 0;
    for (int64_t t = 0; t < cap; ++t, s = (s + 1 == cap) ? 0 : s + 1) {
      uint64_t* h = (uint64_t*)(table + s * stride);
      if (h[1] == 0) {
        h[0] = k;
        h[1] = tag;
        memcpy(table + s * stride + 16, values + i * vbytes, (size_t)vbytes);
        added[i / T] += 1;
        done = 1;
        break;
      }
      if (h[1] == tag && h[0] == k) {
        memcpy(table + s * stride + 16, values + i * vbytes, (size_t)vbytes);
        done = 1;
        break;
      }
    }
    if (!done) full = 1;
  }
  return full;
}

/* pack_codes of code/lema/attention.py:82-97 on fp32 rows: bit d = (z[d] >= 0). */
void oracle_pack_codes_f32(const float* z, int64_t rows, int d, uint64_t* codes) {
  for (int64_t r = 0; r < rows; ++r) {
    uint64_t c = 0;
    for (int j = 0; j < d; ++j)
      if (z[r * d + j] >= 0.0f) c |= (uint64_t)1 << j;
    codes[r] = c;
  }
}
