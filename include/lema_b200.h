/*
 * lema_b200.h -- C ABI of the B200 (sm_100a) LEMA inference hot path.
 *
 * LEMA ("latest exact match attention"): a head turns its query and key
 * pre-activations into sign codes, code(z) = sum_d [z_d >= 0] << d, and query i
 * reads the value row of the LARGEST j < i (strictly causal) whose key code
 * equals its query code, or zeros when there is none.
 *
 * Every entry point:
 *   - takes plain device pointers and sizes (no framework types), and a CUDA
 *     stream as `void*` (NULL = the legacy default stream);
 *   - is asynchronous and stream-ordered: it validates its arguments on the host,
 *     launches, and returns; it never synchronises and never allocates device
 *     memory, so it can be captured into a CUDA graph after the first call on a
 *     device (which sets kernel attributes);
 *   - returns LEMA_OK or an error code; lema_last_error() gives the message of the
 *     last failing call on this host thread;
 *   - reports conditions found ON THE DEVICE (a full store, an exhausted probe)
 *     by OR-ing LEMA_STATUS_* bits into a caller-owned, zero-initialised uint32
 *     status word in device memory. Kernels never trap.
 *
 * Codes are unsigned integers of `code_bytes` = 4 (d_qk <= 32) or 8 (d_qk <= 64)
 * bytes; only equality is ever used, so the int64 codes of the reference (uint64
 * bit patterns) are passed as code_bytes = 8 unchanged.
 *
 * Value rows are opaque byte rows of `vbytes` bytes: the library copies them and
 * never interprets them, so fp32, fp16 and bf16 rows are all the same call.
 */
#ifndef LEMA_B200_H
#define LEMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
enum {
  LEMA_OK = 0,
  LEMA_ERR_INVALID_ARGUMENT = 1, /* shapes, sizes, alignment or null pointers */
  LEMA_ERR_CUDA = 2,             /* a CUDA runtime call failed                 */
  LEMA_ERR_WORKSPACE = 3,        /* workspace smaller than *_workspace_bytes() */
  LEMA_ERR_UNSUPPORTED = 4       /* no kernel for this device or this case     */
};

/* Bits OR-ed into the device status word by kernels. */
#define LEMA_STATUS_TABLE_FULL 0x1u  /* store: an insert probed every slot       */
#define LEMA_STATUS_PROBE_LIMIT 0x2u /* internal: a bounded probe or wait ran out */

/* Message of the last failing call on the calling host thread ("" if none). */
const char* lema_last_error(void);

/* Library version, major * 10000 + minor * 100 + patch. */
int lema_version(void);

/* ------------------------------------------------------------ (a) codes */
/* Element type tags of pre-activations. */
enum { LEMA_F32 = 0, LEMA_BF16 = 1, LEMA_F16 = 2 };

/*
 * pack_codes: one code per row of a strided [d0, d1, d2, d_qk] pre-activation
 * tensor (the innermost dimension contiguous), written densely as codes[d0][d1][d2].
 * Bit d of a code is (z[..., d] >= 0); NaN packs to 0 and -0.0 to 1, exactly as a
 * float comparison `z >= 0` does.
 *
 * Replaces: code/lema/attention.py:82-97 (`pack_codes`), applied to the
 * [B, H, T, d_qk] views that code/lema/model.py:168-175 (`Attention.project`)
 * returns and code/lema/model.py:224-227 (`Block.gpu_pre`) packs.
 *   z           device pointer, element type `dtype`
 *   s0, s1, s2  strides of the three outer dimensions, in elements
 *   d_qk        1..32 for code_bytes = 4, 1..64 for code_bytes = 8
 */
int lema_pack_codes(const void* z, int dtype, int64_t d0, int64_t d1, int64_t d2,
                    int64_t s0, int64_t s1, int64_t s2, int d_qk, void* codes,
                    int code_bytes, void* stream);

/*
 * Code projection (K1): for rows x[M][K] (bf16, row-major) and the stacked query
 * and key projection weights w_qk[(hq + hk) * d_qk][K] (bf16, row-major, nn.Linear
 * layout), computes z = x * w_qk^T with fp32 accumulation on the tcgen05 tensor
 * cores and packs the signs of each head's d_qk = 32 columns in the epilogue, so
 * z never reaches memory. Row m = b * T + t; the codes are written head-major,
 * as the matcher consumes them:
 *   qcodes[(b * hq + h) * T + t], kcodes[(b * hk + h) * T + t]   (uint32)
 * Requires d_qk = 32, K % 64 == 0, M % T == 0, 16-byte aligned x and w_qk.
 * Bit d of a code is (z_d >= 0) for the fp32 z; codes can differ from a bf16
 * GEMM followed by pack_codes only where |z_d| is within rounding of zero.
 * status (optional, device): LEMA_STATUS_PROBE_LIMIT is OR-ed in if a pipeline
 * wait inside the kernel ran out (the codes are then incomplete).
 *
 * Replaces: the q_proj/k_proj GEMMs of code/lema/model.py:160-175 plus
 * code/lema/attention.py:82-97, i.e. code/lema/model.py:224-227 minus the norm
 * and the value projection.
 */
int lema_proj_codes(const void* x, const void* w_qk, int64_t M, int64_t K,
                    int64_t T, int hq, int hk, int d_qk, uint32_t* qcodes,
                    uint32_t* kcodes, uint32_t* status, void* stream);

/*
 * lema_proj_codes with the value projection and the norm folded in: w_all stacks the
 * query and key weights ((hq + hk) * 32 rows) and n_v value rows (v_proj.weight), each
 * column-scaled by the RMSNorm weight; x is the UN-normalised residual stream. The
 * codes are those of the normalised input (the norm's positive row scale cannot change
 * a sign); the n_v value columns are written as bf16 v_out[m][c] = row_scale[m] * z,
 * row_scale = 1 / sqrt(mean(x[m]^2) + eps) from lema_row_rms (NULL: 1). n_v = 0 is
 * lema_proj_codes. v_out 16-byte aligned.
 * Replaces: code/lema/model.py:224-227 (`Block.gpu_pre`: norm1, q/k/v projections,
 * pack_codes) in one GEMM.
 */
int lema_proj_codes_v(const void* x, const void* w_all, int64_t M, int64_t K, int64_t T,
                      int hq, int hk, int d_qk, uint32_t* qcodes, uint32_t* kcodes,
                      int64_t n_v, void* v_out, const float* row_scale, uint32_t* status,
                      void* stream);

/* out[m] = 1 / sqrt(mean over K of x[m][k]^2 + eps) for bf16 rows x[M][K] (K % 8 == 0),
 * fp32 sums: the RMSNorm row scale. */
int lema_row_rms(const void* x, int64_t M, int64_t K, float eps, float* out, void* stream);

/* SwiGLU activation on a fused gate/up GEMM output gu[M][2F] (gate columns first):
 * out[m][f] = silu(gu[m][f]) * gu[m][F + f], fp32 inside, dtype LEMA_F32/BF16/F16.
 * Replaces: the silu and product of code/lema/model.py:85-93 (`SwiGLU.forward`). */
int lema_swiglu(const void* gu, int dtype, int64_t M, int64_t F, void* out, void* stream);

/* The MLP's gate/up GEMM with SwiGLU in its epilogue (K1's tcgen05 pipeline):
 * act[m][f] = bf16(silu(x[m] . gate[f]) * (x[m] . up[f])), fp32 accumulators, for bf16 x
 * [M][K] and w_il [2F][K] holding the gate and up rows interleaved in blocks of 128 (rows
 * 256 b .. 256 b + 127 = gate rows 128 b ..; the next 128 = up rows 128 b ..). K a multiple
 * of 64, F of 128; pointers 16-byte aligned. The [M][2F] product never reaches HBM.
 * Replaces: gate(x), up(x) and silu(.) * (.) of code/lema/model.py:85-93 (SwiGLU.forward);
 * the down projection stays a GEMM. status as for lema_proj_codes. */
int lema_gemm_swiglu(const void* x, const void* w_il, int64_t M, int64_t K, int64_t F, void* act_out,
                     uint32_t* status, void* stream);

/* RMSNorm of 16-bit rows: out[m] = (x[m] * rstd) * weight, rstd = 1 / sqrt(mean(x[m]^2) +
 * eps), fp32 inside, rounded once; dtype LEMA_BF16 or LEMA_F16, D a multiple of 8, x, weight
 * and out 16-byte aligned (else LEMA_ERR_UNSUPPORTED: use the framework's own norm).
 * Replaces: nn.RMSNorm of code/lema/model.py:215-217, 264 (norm1, norm2, norm_f). */
int lema_rms_norm(const void* x, const void* weight, int dtype, int64_t M, int64_t D, float eps,
                  void* out, void* stream);

/* ---------------------------------------------- (b) prefill latest match */
/*
 * Bytes of device workspace lema_prefill_match needs for n_streams x T
 * positions: room for the indices (used when src is NULL) plus, when a stream can
 * hold more distinct key codes than the on-chip table takes, the overflow-path
 * tables, plus the control words (4 KiB + 4 bytes per stream) of the pipelined
 * mode, in which one launch matches and copies the value rows at once. A smaller
 * workspace that still holds the first two runs the matcher and the row copy as
 * two kernels: the same results. 256-byte aligned workspace required.
 */
size_t lema_prefill_workspace_bytes(int64_t n_streams, int64_t T, int code_bytes);

/*
 * Latest exact match over n_streams independent streams (batch x heads) of T
 * positions each, stream-major:
 *   src[n][i] = max { j < i : kcodes[n][j] == qcodes[n][i] }, or -1
 *   out[n][i] = values[n][src[n][i]]  (vbytes bytes), or zeros when src is -1
 * src (int32) and out are each optional (NULL skips it); values may be NULL
 * only when out is. vbytes must be a positive multiple of 2.
 *
 * Replaces: code/lema/attention.py:100-132 (`latest_prev_match`, int64 indices
 * there) and the gather of code/lema/attention.py:150-158 (`lema_hard` without
 * a store).
 */
int lema_prefill_match(const void* qcodes, const void* kcodes, int code_bytes,
                       int64_t n_streams, int64_t T, int32_t* src,
                       const void* values, int64_t vbytes, void* out,
                       void* workspace, size_t workspace_bytes, uint32_t* status,
                       void* stream);

/*
 * lema_prefill_match with strided value rows: stream n = b * heads + h (codes stay
 * [n_streams][T]); value row t of stream n at values + b * v_sb + h * v_sh + t * v_st
 * bytes, output row at out + b * o_sb + h * o_sh + t * o_st. This reads a projection's
 * [B][T][H][d_v] output and writes the [B][T][H][d_v] rows the output projection takes,
 * with no transposing copy either side. n_streams must be a multiple of heads.
 * Replaces: code/lema/attention.py:150-158 on the transposed views of
 * code/lema/model.py:168-180 (`project`, `merge`).
 */
int lema_prefill_match_strided(const void* qcodes, const void* kcodes, int code_bytes,
                               int64_t n_streams, int64_t T, int32_t* src,
                               const void* values, int64_t vbytes, void* out, int64_t heads,
                               int64_t v_sb, int64_t v_sh, int64_t v_st, int64_t o_sb,
                               int64_t o_sh, int64_t o_st, void* workspace,
                               size_t workspace_bytes, uint32_t* status, void* stream);

/*
 * lema_prefill_match_noalloc: lema_prefill_match without a workspace argument, for callers
 * that cannot allocate device memory -- a plugin that is handed only its input and output
 * tensors by a host engine owning all device memory, a C program with no device allocator,
 * or a latency-critical loop in which cudaMalloc (may block) and cudaFree (synchronises the
 * device) are not allowed. It allocates nothing: its scratch is a fixed array of
 * LEMA_NOALLOC_SCRATCH_BYTES inside this library, which every GPU that loads the library
 * holds until the process exits.
 *   - The first call on a device looks up that array's device address (with the device
 *     current); make that first call before any CUDA-graph stream capture.
 *   - All calls share the one array and it keeps the last call's contents: each call
 *     clears what it needs at zero (the overflow counter and, when it runs the pipelined
 *     mode, the control block and per-stream progress words) and assumes nothing else
 *     about it. Calls that overlap on the GPU -- on different streams, or from different
 *     host threads -- race on it: order them on one stream.
 *   - The address looked up on a device is kept for the life of the process; it does not
 *     survive cudaDeviceReset on that device. A failed look-up is retried by the next call.
 *   - A call whose scratch does not fit is rejected with LEMA_ERR_WORKSPACE: the scratch is
 *     4 * n_streams * T bytes when src is NULL, plus, when T > 6144 (32-bit codes) or
 *     T > 3072 (64-bit codes), room for at least one overflow-path table of about
 *     12 * next_pow2(2 * T) bytes (16 * ... for 64-bit codes). Passing src avoids the
 *     first part.
 * Same arguments, results and status behaviour as lema_prefill_match otherwise.
 * No counterpart in the reference: it is an addition for allocation-free callers.
 */
#define LEMA_NOALLOC_SCRATCH_BYTES (32u << 20)
int lema_prefill_match_noalloc(const void* qcodes, const void* kcodes, int code_bytes,
                               int64_t n_streams, int64_t T, int32_t* src,
                               const void* values, int64_t vbytes, void* out,
                               uint32_t* status, void* stream);

/* ---------------------------------------------------- (c) the HBM store */
/*
 * The store is ONE open-addressing table in device memory shared by every
 * (layer, stream, head) partition ("group"), keyed by (group, code), holding the
 * value row of the latest key written under that key. The caller owns the table:
 * cap slots of lema_store_slot_bytes(vbytes) bytes each, ZERO-FILLED before first
 * use (a zeroed table is an empty table). It never grows; an insert that finds
 * no free slot sets LEMA_STATUS_TABLE_FULL.
 *
 * Replaces: the host table of code/lema/cache.py:129-201 (`HashStore`), whose
 * slots are [code | state | value] at code/lema/csrc/store.cpp:3-16. The size per
 * slot is the reference's (16 + the row); inside, the bytes are a dense array of
 * 16-byte slot headers (code, state) followed by the rows, so probing at high
 * load walks few cache lines.
 */
int64_t lema_store_slot_bytes(int64_t vbytes);

/* Bytes of device workspace lema_store_exchange needs for n = P * T items. */
size_t lema_store_workspace_bytes(int64_t n, int64_t T, int code_bytes);

/*
 * One exchange of P = n / T partitions x T positions against the store. Item i
 * is position i % T of partition i / T, group g0 + i / T. Each partition, in
 * position order, looks qcodes[i] up into out[i] (zeros on a miss) and then
 * inserts kcodes[i] -> values[i] (latest write wins), so a query sees every
 * earlier key of its partition -- this call's and all earlier calls' -- and not
 * its own. A prefill chunk (T > 1) and a decode step (T = 1) are the same call.
 * counts[p] (int64, device, P entries) is increased by the number of slots
 * partition p newly claimed.
 *
 * Replaces: code/lema/csrc/store.cpp:127-162 (`exchange`, which returns the
 * per-partition `added` the caller adds into code/lema/cache.py:200's counts).
 *   table      device, cap * lema_store_slot_bytes(vbytes) bytes
 *   vbytes     positive multiple of 8 (as code/lema/cache.py:161-165 requires)
 */
int lema_store_exchange(void* table, int64_t cap, int64_t vbytes,
                        const void* qcodes, const void* kcodes, int code_bytes,
                        const void* values, void* out, int64_t n, int64_t T,
                        int64_t g0, int64_t* counts, uint32_t* status,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * lema_store_exchange on a SEGMENTED table: the home slot of a group g lies in segment
 * g / seg_groups, slots [seg * seg_slots, (seg + 1) * seg_slots); probing continues past
 * the segment and wraps at cap as before, so capacity and "full" are still those of one
 * shared table. With one segment per layer (seg_groups = the partitions of a layer), a
 * layer's exchange touches 1/depth of a large table instead of all of it. A table must be
 * used with one segmentation throughout. (0, 0) = lema_store_exchange.
 * Replaces: code/lema/csrc/store.cpp:127-162 like lema_store_exchange; the segmentation
 * is a placement choice of this build, invisible in results.
 */
int lema_store_exchange_seg(void* table, int64_t cap, int64_t vbytes,
                            const void* qcodes, const void* kcodes, int code_bytes,
                            const void* values, void* out, int64_t n, int64_t T,
                            int64_t g0, int64_t* counts, uint32_t* status,
                            void* workspace, size_t workspace_bytes, int64_t seg_groups,
                            int64_t seg_slots, void* stream);

/*
 * lema_store_exchange_seg with strided value and output rows: partition p = b * heads + h
 * (n / T partitions, a multiple of heads), item (p, t) reads its value row at values +
 * b * v_sb + h * v_sh + t * v_st and writes its retrieved row at out + b * o_sb + h * o_sh +
 * t * o_st (bytes, multiples of 8). This takes a projection's [B][T][H][d_v] output as it is
 * and writes the [B][T][H][d_v] rows the output projection reads, with no transposing copy
 * either side of a prefill chunk.
 * Replaces: code/lema/csrc/store.cpp:127-162 (`exchange`) on the item-major copies that
 * code/lema/cache.py:272-291 makes of the [B, H, T, d_v] views, and the merge of
 * code/lema/model.py:229-232 (`Block.gpu_post`).
 */
int lema_store_exchange_strided(void* table, int64_t cap, int64_t vbytes,
                                const void* qcodes, const void* kcodes, int code_bytes,
                                const void* values, void* out, int64_t n, int64_t T,
                                int64_t g0, int64_t* counts, uint32_t* status,
                                void* workspace, size_t workspace_bytes, int64_t seg_groups,
                                int64_t seg_slots, int64_t heads, int64_t v_sb, int64_t v_sh,
                                int64_t v_st, int64_t o_sb, int64_t o_sh, int64_t o_st,
                                void* stream);

/*
 * One decode step (T = 1) of lema_store_exchange_seg in two launches: phase 1 looks every
 * item's query up into out (qcodes, out used), phase 2 inserts every item's key and value
 * (kcodes, values, counts used). Phase 1 then phase 2 on the same items equals phase 3 (both,
 * what lema_store_exchange_seg does): a decode step's items are distinct partitions, so no
 * lookup of the step depends on an insert of the step. The inserts can then run beside later
 * work that needs only the retrieved rows, as long as they finish before the next lookups of
 * the same groups. No workspace (T = 1).
 * Replaces: code/lema/csrc/store.cpp:84-117 (`Table::read`, `Table::insert`) as
 * code/lema/csrc/store.cpp:150-156 calls them per item, split into its two halves.
 */
int lema_store_exchange_phase(void* table, int64_t cap, int64_t vbytes, const void* qcodes,
                              const void* kcodes, int code_bytes, const void* values, void* out,
                              int64_t n, int64_t g0, int64_t* counts, uint32_t* status,
                              int64_t seg_groups, int64_t seg_slots, int phase, void* stream);

/* ----------------------------------- (d) sequence-sharded prefill (config 5) */
/*
 * One sequence too long for one pass (or one GPU) is cut into contiguous shards of L
 * positions per head; a rank owns positions [base, base + L) of all n_heads heads,
 * laid out [n_heads][L]. Together the calls below give, bit for bit, what one
 * lema_prefill_match over the whole sequence gives, with src as global positions:
 *   lema_segment_match   K2 per segment of seg_len positions, with each segment's
 *                        last-occurrence table (LT: distinct key codes, last position)
 *   lema_shard_sweep     segments in order against an empty table: misses look up the
 *                        earlier segments; the table ends up holding the shard's LT
 *   lema_lt_extract      that LT, for the other ranks (all-gathered by the caller)
 *   lema_lt_insert       + lema_lt_resolve: queries still unmatched look up the LTs of
 *                        the earlier ranks
 *   lema_shard_gather    rows from this shard or from rows fetched from earlier shards
 *   lema_shard_gather_peer  rows from this shard or read in place from the earlier shards'
 *                        values (peer GPUs' memory over NVLink, mapped by lema_ipc_import)
 * Hash tables: n_heads x slots uint64 words (slots a power of two, see
 * lema_lt_table_slots), ZERO-FILLED by the caller; an insert keeps the larger position.
 * Codes are 32-bit; global positions stay below 2^31 - 1.
 *
 * Replaces: code/lema/attention.py:100-132 (`latest_prev_match`) over the whole
 * sequence and the gather of code/lema/attention.py:150-158, for a sharded sequence.
 */
size_t lema_segment_workspace_bytes(int64_t n_streams, int64_t T, int code_bytes);

/* lema_prefill_match with src required and the per-stream last-occurrence tables:
 * lt_code[n * T + e] (code_bytes wide), lt_pos[n * T + e] (position in the stream),
 * e < lt_count[n], in no particular order. */
int lema_segment_match(const void* qcodes, const void* kcodes, int code_bytes,
                       int64_t n_streams, int64_t T, int32_t* src, void* lt_code,
                       int32_t* lt_pos, int32_t* lt_count, void* workspace,
                       size_t workspace_bytes, uint32_t* status, void* stream);

/* Slots per head for a table that may hold max_entries codes (load <= 0.5). */
int64_t lema_lt_table_slots(int64_t max_entries);

/* Insert n entries (heads[i], codes[i]) -> pos[i] (global positions). */
int lema_lt_insert(uint64_t* table, int64_t n_heads, int64_t slots, const int32_t* heads,
                   const uint32_t* codes, const int32_t* pos, int64_t n,
                   uint32_t* status, void* stream);

/* src[h][i] == -1 only: probe the tables of earlier shards, newest (index n_tables - 1)
 * first; the first holding qcodes[h][i] gives its latest position, else -1. `tables`
 * and `slots` are DEVICE arrays of n_tables table pointers (each n_heads x slots[t]
 * words, slots a power of two) and slot counts. */
int lema_lt_resolve_tables(const uint64_t* const* tables, const int64_t* slots, int n_tables,
                           int64_t n_heads, const uint32_t* qcodes, int32_t* src, int64_t L,
                           void* stream);

/* src[h][i] == -1 only: the latest position of qcodes[h][i] in the table, or -1. */
int lema_lt_resolve(const uint64_t* table, int64_t n_heads, int64_t slots,
                    const uint32_t* qcodes, int32_t* src, int64_t L, void* stream);

/* Entries with position >= lo as one flat list: out_heads/out_codes/out_pos[k],
 * k < *out_count (a single int32), in no particular order; more than cap entries sets
 * LEMA_STATUS_TABLE_FULL (the first cap are written). */
int lema_lt_extract(const uint64_t* table, int64_t n_heads, int64_t slots, int32_t lo,
                    int32_t* out_heads, uint32_t* out_codes, int32_t* out_pos,
                    int32_t* out_count, int64_t cap, uint32_t* status, void* stream);

/* One 8-CTA cluster per head walks the L / seg_len segments in order: src (in: index within
 * the segment or -1, from lema_segment_match) becomes the global position of the
 * latest earlier key of the shard with the query's code, or -1; then the segment's
 * LT goes into the table (zero-filled before the call; slots for the shard's
 * distinct key codes). */
int lema_shard_sweep(uint64_t* table, int64_t n_heads, int64_t slots, const uint32_t* qcodes,
                     int32_t* src, int64_t L, int64_t seg_len, const uint32_t* lt_code,
                     const int32_t* lt_pos, const int32_t* lt_count, int64_t base,
                     int64_t vrows, uint32_t* status, void* stream);
/* (vrows > 1: each head is swept as vrows independent rows of L positions -- "n_heads" then
 * counts rows, row r starting at position base + (r % vrows) * L -- and
 * lema_lt_resolve_rows then lets a row's remaining misses probe the earlier rows of its
 * head, newest first.) */
int lema_lt_resolve_rows(const uint64_t* table, int64_t n_rows, int64_t slots, int64_t vrows,
                         const uint32_t* qcodes, int32_t* src, int64_t L, void* stream);

/* out[h][i] = values[h][src - base] for src >= base, remote_rows[remote_idx[h][i]]
 * for 0 <= src < base, zeros for -1. */
int lema_shard_gather(const int32_t* src, int64_t base, const void* values,
                      const void* remote_rows, const int32_t* remote_idx, int64_t vbytes,
                      void* out, int64_t n_heads, int64_t L, uint32_t* status, void* stream);

/* The same, with every earlier shard's rows read where they lie: peer_values is a HOST array
 * of n_ranks pointers, rank k's [n_heads][L] values (k < this rank: this process's mapping of
 * rank k's tensor, from lema_ipc_import; k = base / L: this rank's own values). All ranks
 * share n_heads, L and vbytes; n_ranks <= 16. Plain loads only: the peers' values must stay
 * unchanged until every rank's call has completed (the caller's collective after the call).
 * Replaces the row request and exchange of lema_shard_gather's caller. */
int lema_shard_gather_peer(const int32_t* src, int64_t base, const void* const* peer_values,
                           int n_ranks, int64_t vbytes, void* out, int64_t n_heads, int64_t L,
                           uint32_t* status, void* stream);

/* CUDA IPC of a device tensor for lema_shard_gather_peer: export writes the 64-byte handle of
 * the allocation holding ptr and ptr's offset in it; import (in another process of the same
 * node) maps it and returns the tensor's address there; close unmaps it. */
int lema_ipc_export(const void* ptr, void* handle, int64_t* offset);
int lema_ipc_import(const void* handle, int64_t offset, void** ptr);
int lema_ipc_close(void* ptr, int64_t offset);

#ifdef __cplusplus
}
#endif

#endif /* LEMA_B200_H */
