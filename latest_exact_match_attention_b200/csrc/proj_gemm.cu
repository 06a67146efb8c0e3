// K1 -- code projection: z = x * w_qk^T on the tcgen05 tensor cores, with the sign/bit-pack
// of every head's 32 columns in the epilogue, so z never leaves the SM.
//
// Replaces the q_proj / k_proj GEMMs of code/lema/model.py:160-175 (Attention.project) and the
// pack_codes of code/lema/attention.py:82-97 that code/lema/model.py:224-227 (Block.gpu_pre)
// applies to their outputs: there a bf16 z goes to HBM and is read back to be packed.
//
// One persistent CTA per SM walks output tiles of 128 rows x 256 columns (8 heads of 32).
// Warp roles:
//   warp 0     TMA producer: 128x64 tiles of x and 256x64 tiles of w_qk (bf16, 128-byte
//              swizzle) into a 4-stage shared-memory ring, one mbarrier pair per stage;
//   warp 1     MMA issuer: per stage, 4 x tcgen05.mma M128 N256 K16 (bf16 in, fp32 out)
//              into one of two 256-column TMEM accumulators; tcgen05.commit frees the stage;
//   warps 2-5  epilogue: each reads its 32 TMEM lanes (= 32 output rows), one head (32 fp32
//              columns) per tcgen05.ld, packs the 32 signs into a uint32 code and stores it
//              head-major, 32 consecutive positions of one head per warp store.
// Two accumulators let the epilogue of one tile run under the main loop of the next.
//
// Every wait on an mbarrier is bounded in time: a wait that runs out sets a shared abort flag
// (the other roles then stop at their next wait) and LEMA_STATUS_PROBE_LIMIT in the caller's
// status word; before the CTA exits, the producer waits (bounded again) for its copies in
// flight, the MMA warp for its tensor-core work, and the TMEM is released.
#include <cuda.h>  // CUtensorMap and its enums (types only; the encoder comes from the runtime)
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace lema {
namespace k1 {

constexpr int kBM = 128, kBK = 64;  // tile rows, K per stage
constexpr int kABytes = kBM * kBK * 2;  // 16 KiB
constexpr int kThreads = 192;           // 6 warps: producer, MMA, 4 x epilogue
constexpr uint64_t kDrainNs = 4000000000ull;  // a wait for work already in flight at exit: 4 s

// A tile is 128 rows x BN columns (BN / 32 heads). Per width: as many stages as fit in about
// 192 KiB of shared memory (at most 8), two BN-column fp32 TMEM accumulators, and the
// instruction descriptor of tcgen05.mma kind::f16 (32-bit form): fp32 accumulator (bits 4-5
// = 1), A and B bf16 (bits 7-9 = 1, bits 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3
// at bits 17-22, M >> 4 at bits 24-28. The widest tile (256) is for large M; narrower ones
// give small M (decode: a few hundred rows) enough tiles to occupy the SMs.
template <int BN>
struct Tile {
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes < 8 ? (192 * 1024) / kStageBytes : 8;
  static constexpr int kHeads = BN / 32;
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr size_t kSmemBytes = size_t(kStages) * kStageBytes + 1024 /* alignment */ + 256 /* barriers */;
  static constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(BN >> 3) << 17) |
                                         (uint32_t(kBM >> 4) << 24);
};

struct Params {
  uint32_t* qcodes;
  uint32_t* kcodes;
  uint32_t* status;
  uint64_t wait_ns;  // bound of a pipeline wait (wait_limit_ns(): 4 s unless LEMA_WAIT_NS)
  int64_t M, T;
  int64_t n_tiles;
  int k_blocks;
  int n_blocks;
  int hq, hk;
  // optional value columns after the code heads: v_out[m][c] = bf16(row_scale[m] * z[m][c]),
  // c < n_v (row_scale NULL: 1)
  __nv_bfloat16* v_out;
  const float* row_scale;
  int n_v;
  // SwiGLU mode (act_out set, no codes, BN = 256): the weight rows of tile column block nb are
  // 128 gate rows then the 128 up rows of the same features f = 128 nb ...;
  // act_out[m][f] = bf16(silu(gate) * up) from the fp32 accumulators, act_f = F features
  __nv_bfloat16* act_out;
  int64_t act_f;
};

// ------------------------------------------------------------------ PTX wrappers
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// The same with a bound (ns) on how long the thread may be suspended in one try: the caller
// then checks its deadline at least that often.
__device__ __forceinline__ bool mbar_try_wait_for(uint32_t bar, uint32_t parity, uint32_t suspend_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(suspend_ns)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Shared-memory matrix descriptor of a K-major tile written by TMA with the 128-byte swizzle:
// rows of 128 bytes (64 bf16), 8-row swizzle atoms of 1024 bytes stacked along M/N (stride
// byte offset 1024), leading byte offset unused for this layout (1), descriptor version 1
// (bits 46-47), layout type 2 = 128-byte swizzle (bits 61-63). The start address is in 16-byte
// units; a K slice of 16 elements (32 bytes) inside the atom is start + 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) |
         (uint64_t(1024 >> 4) << 32) | (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// 32 consecutive fp32 columns of this thread's TMEM lane, waited for before returning.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Waits for the phase of `bar` with parity `parity`. Returns false when another role has
// given up, or after wait_ns (then this wait raises the abort flag and the status bit).
__device__ bool wait_phase(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag, uint32_t* status,
                           uint64_t wait_ns) {
  // each try suspends at most ~wait_ns (between 32 ns and 1 ms); the deadline is checked
  // every 4 tries, so a short bound (LEMA_WAIT_NS) is honoured within a few microseconds
  const uint32_t suspend = static_cast<uint32_t>(wait_ns < 32 ? 32 : (wait_ns > 1000000 ? 1000000 : wait_ns));
  uint64_t deadline = 0;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_for(bar, parity, suspend)) return true;
    if ((i & 3) == 0) {
      if (*abort_flag) return false;
      const uint64_t now = globaltimer();
      if (deadline == 0) {
        deadline = now + wait_ns;
      } else if (now > deadline) {
        *abort_flag = 1;
        raise_status(status, LEMA_STATUS_PROBE_LIMIT);
        return false;
      }
    }
  }
}

// The same wait for draining work already in flight at exit: ignores the abort flag and keeps
// its own bound (kDrainNs), whatever wait_ns is: copies and MMAs in flight always complete.
__device__ void drain_phase(uint32_t bar, uint32_t parity, uint32_t* status) {
  uint64_t deadline = 0;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 63) == 0) {
      const uint64_t now = globaltimer();
      if (deadline == 0) {
        deadline = now + kDrainNs;
      } else if (now > deadline) {
        raise_status(status, LEMA_STATUS_PROBE_LIMIT);
        return;
      }
    }
  }
}

__device__ __forceinline__ uint32_t pack_signs(const uint32_t (&r)[32]) {
  uint32_t code = 0;
#pragma unroll
  for (int d = 0; d < 32; ++d) code |= (__uint_as_float(r[d]) >= 0.0f ? 1u : 0u) << d;
  return code;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    proj_codes_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
                      const Params p) {
  using TL = Tile<BN>;
  constexpr int kStages = TL::kStages, kStageBytes = TL::kStageBytes;
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment of the stage buffers (the swizzle atom), done on the shared address
  const uint32_t raw = smem_addr(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw & 1023u)) & 1023u);
  const uint32_t sbase = smem_addr(smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  // barriers: full[kStages], empty[kStages], acc_full[2], acc_empty[2], drain
  const uint32_t bar0 = smem_addr(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto accf_bar = [&](int a) { return bar0 + 8u * (2 * kStages + a); };
  auto acce_bar = [&](int a) { return bar0 + 8u * (2 * kStages + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kStages + 4);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  volatile uint32_t* s_abort = s_tmem + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), 4);  // one arrival per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
  }
  if (warp == 0) {  // TMEM: 512 columns, written to s_tmem; the same warp frees it at exit
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(s_tmem)),
                 "r"(TL::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  // launched as a dependent: the set-up above overlaps the previous kernel; its outputs (x)
  // are read only from here on
  griddep_wait();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, issued = 0, last_ph = 0;  // per-stage bits: issued at least once, parity
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x) {
        const int m0 = static_cast<int>(tile / p.n_blocks) * kBM;
        const int n0 = static_cast<int>(tile % p.n_blocks) * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_phase(empty_bar(s), ph ^ 1u, s_abort, p.status, p.wait_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(s), kStageBytes);
          const uint32_t a_dst = sbase + s * kStageBytes;
          tma_load_2d(a_dst, &map_x, full_bar(s), kb * kBK, m0);
          tma_load_2d(a_dst + kABytes, &map_w, full_bar(s), kb * kBK, n0);
          issued |= 1u << s;
          last_ph = (last_ph & ~(1u << s)) | (ph << s);
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // copies still in flight must land before the CTA's shared memory goes away
      for (int i = 0; i < kStages; ++i)
        if (issued & (1u << i)) drain_phase(full_bar(i), (last_ph >> i) & 1u, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; ok && tile < p.n_tiles; tile += gridDim.x) {
        if (!wait_phase(acce_bar(acc), aph ^ 1u, s_abort, p.status, p.wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!wait_phase(full_bar(s), ph, s_abort, p.status, p.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = sbase + s * kStageBytes;
          const uint64_t a_desc = sw128_desc(a_addr), b_desc = sw128_desc(a_addr + kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16(d_tmem, a_desc + 2u * kk, b_desc + 2u * kk, TL::kInstrDesc, (kb | kk) != 0 ? 1u : 0u);
          mma_commit(empty_bar(s));  // the stage is free once these MMAs have read it
          if (++s == kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(accf_bar(acc));  // the accumulator is ready once every MMA of the tile is done
        if (++acc == 2) {
          acc = 0;
          aph ^= 1u;
        }
      }
      mma_commit(drain_bar);  // nothing this thread issued may still run at exit
      drain_phase(drain_bar, 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // a warp reads TMEM lanes 32 * (warp % 4) ... + 31
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int n_heads = p.hq + p.hk;
    const int n_groups = n_heads + (p.n_v + 31) / 32;  // 32-column groups: code heads, then values
    int acc = 0;
    uint32_t aph = 0;
    for (int64_t tile = blockIdx.x; tile < p.n_tiles; tile += gridDim.x) {
      if (!wait_phase(accf_bar(acc), aph, s_abort, p.status, p.wait_ns)) break;
      tc_fence_after();
      const int64_t m = (tile / p.n_blocks) * kBM + quarter * 32 + lane;
      const int h0 = static_cast<int>(tile % p.n_blocks) * TL::kHeads;
      const bool live = m < p.M;
      const int64_t b = live ? m / p.T : 0;
      const int64_t t = live ? m - b * p.T : 0;
      const float scale = (live && p.row_scale != nullptr) ? p.row_scale[m] : 1.0f;
      if (p.act_out != nullptr) {
        // SwiGLU: gate columns j * 32 ... and up columns BN / 2 + j * 32 ... of the same 32
        // features; silu(g) * u in fp32 (the formula of lema_swiglu), rounded once
        const int64_t f0 = (tile % p.n_blocks) * (BN / 2);
        for (int j = 0; j < BN / 64; ++j) {
          uint32_t g[32], u[32];
          tmem_load32(tmem_base + lane_base + static_cast<uint32_t>(acc * BN + j * 32), g);
          tmem_load32(tmem_base + lane_base + static_cast<uint32_t>(acc * BN + BN / 2 + j * 32), u);
          if (live) {
            uint4* dst = reinterpret_cast<uint4*>(p.act_out + m * p.act_f + f0 + j * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float g0 = __uint_as_float(g[8 * q + 2 * e]), g1 = __uint_as_float(g[8 * q + 2 * e + 1]);
                const float u0 = __uint_as_float(u[8 * q + 2 * e]), u1 = __uint_as_float(u[8 * q + 2 * e + 1]);
                const __nv_bfloat162 pr =
                    __floats2bfloat162_rn(g0 / (1.0f + expf(-g0)) * u0, g1 / (1.0f + expf(-g1)) * u1);
                wp[e] = *reinterpret_cast<const uint32_t*>(&pr);
              }
              dst[q] = w;
            }
          }
        }
      }
      for (int j = 0; p.act_out == nullptr && j < TL::kHeads; ++j) {
        const int h = h0 + j;
        if (h >= n_groups) break;  // warp-uniform
        uint32_t r[32];
        tmem_load32(tmem_base + lane_base + static_cast<uint32_t>(acc * BN + j * 32), r);
        if (h < n_heads) {
          const uint32_t code = pack_signs(r);
          if (live) {
            if (h < p.hq)
              p.qcodes[(b * p.hq + h) * p.T + t] = code;
            else
              p.kcodes[(b * p.hk + (h - p.hq)) * p.T + t] = code;
          }
        } else if (live) {
          // value columns: scaled, rounded to bf16, one row's 32 columns per thread
          const int c0 = (h - n_heads) * 32;
          __nv_bfloat16* dst = p.v_out + m * static_cast<int64_t>(p.n_v) + c0;
          if (c0 + 32 <= p.n_v && (p.n_v % 8) == 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 w;
              uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const __nv_bfloat162 pr = __floats2bfloat162_rn(__uint_as_float(r[8 * q + 2 * e]) * scale,
                                                               __uint_as_float(r[8 * q + 2 * e + 1]) * scale);
                wp[e] = *reinterpret_cast<const uint32_t*>(&pr);
              }
              reinterpret_cast<uint4*>(dst)[q] = w;
            }
          } else {
#pragma unroll
            for (int d = 0; d < 32; ++d)
              if (c0 + d < p.n_v) dst[d] = __float2bfloat16_rn(__uint_as_float(r[d]) * scale);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(acc));
      if (++acc == 2) {
        acc = 0;
        aph ^= 1u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TL::kTmemCols)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// A 2-D bf16 tensor map of a row-major [rows][K] matrix, boxes of box_rows x 64 with the
// 128-byte swizzle; rows past the end read as zeros.
bool encode_kmajor(EncodeTiledFn enc, CUtensorMap* map, const void* base, int64_t rows, int64_t K, int box_rows) {
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN>
int launch(const CUtensorMap& map_x, const CUtensorMap& map_w, const Params& prm, int64_t grid, cudaStream_t stream) {
  LEMA_TRY(kernel_facts(reinterpret_cast<const void*>(proj_codes_kernel<BN>), Tile<BN>::kSmemBytes, 0, 0, nullptr));
  LEMA_CUDA_TRY(launch_dependent(proj_codes_kernel<BN>, dim3(static_cast<unsigned>(grid)), dim3(kThreads),
                                 Tile<BN>::kSmemBytes, stream, map_x, map_w, prm));
  return LEMA_OK;
}

}  // namespace k1

int proj_codes_v(const void* x, const void* w_all, int64_t M, int64_t K, int64_t T, int hq, int hk, int d_qk,
                 uint32_t* qcodes, uint32_t* kcodes, int64_t n_v, void* v_out, const float* row_scale,
                 uint32_t* status, cudaStream_t stream);

int proj_codes(const void* x, const void* w_qk, int64_t M, int64_t K, int64_t T, int hq, int hk, int d_qk,
               uint32_t* qcodes, uint32_t* kcodes, uint32_t* status, cudaStream_t stream) {
  return proj_codes_v(x, w_qk, M, K, T, hq, hk, d_qk, qcodes, kcodes, 0, nullptr, nullptr, status, stream);
}

int proj_codes_v(const void* x, const void* w_all, int64_t M, int64_t K, int64_t T, int hq, int hk, int d_qk,
                 uint32_t* qcodes, uint32_t* kcodes, int64_t n_v, void* v_out, const float* row_scale,
                 uint32_t* status, cudaStream_t stream) {
  using namespace k1;
  const void* w_qk = w_all;
  if (n_v < 0 || n_v > (int64_t(1) << 20) || (n_v > 0 && v_out == nullptr))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "value columns: n_v = %lld (0 .. 2^20), v_out required", (long long)n_v);
  if (n_v > 0 && !aligned(v_out, 16)) return fail(LEMA_ERR_INVALID_ARGUMENT, "v_out must be 16-byte aligned");
  if (d_qk != 32)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "lema_proj_codes packs d_qk = 32 only (got %d); "
                "use lema_pack_codes on a projected z for other widths", d_qk);
  if (M < 0 || K <= 0 || T <= 0 || hq < 0 || hk < 0)
    return fail(LEMA_ERR_INVALID_ARGUMENT, "bad shape M=%lld K=%lld T=%lld hq=%d hk=%d", (long long)M,
                (long long)K, (long long)T, hq, hk);
  if (K % kBK != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "K = %lld is not a multiple of 64", (long long)K);
  if (M % T != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "M = %lld rows is not whole sequences of T = %lld", (long long)M, (long long)T);
  if (M >= (int64_t(1) << 31) || K >= (int64_t(1) << 24) || hq + hk > (1 << 16))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "shape too large (M=%lld K=%lld heads=%d)", (long long)M, (long long)K, hq + hk);
  if (M == 0 || hq + hk + n_v == 0) return LEMA_OK;
  if (x == nullptr || w_qk == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "null x or w_qk");
  if ((hq > 0 && qcodes == nullptr) || (hk > 0 && kcodes == nullptr))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "null code output");
  if (!aligned(x, 16) || !aligned(w_qk, 16)) return fail(LEMA_ERR_INVALID_ARGUMENT, "x and w_qk must be 16-byte aligned");
  if (!aligned(qcodes, 4) || !aligned(kcodes, 4)) return fail(LEMA_ERR_INVALID_ARGUMENT, "code outputs must be 4-byte aligned");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return fail(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");

  const int64_t n_cols = static_cast<int64_t>(hq + hk) * 32 + n_v;
  // the widest tile that still gives every SM a tile; narrower tiles only for small M
  const int64_t m_blocks = (M + kBM - 1) / kBM;
  int bn = 256;
  while (bn > 64 && m_blocks * ((n_cols + bn - 1) / bn) < dev->sms) bn /= 2;
  CUtensorMap map_x, map_w;
  if (!encode_kmajor(enc, &map_x, x, M, K, kBM) || !encode_kmajor(enc, &map_w, w_qk, n_cols, K, bn))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "tensor map encoding failed (M=%lld K=%lld N=%lld)", (long long)M,
                (long long)K, (long long)n_cols);

  Params prm{};
  prm.qcodes = qcodes;
  prm.kcodes = kcodes;
  prm.status = status;
  prm.wait_ns = wait_limit_ns();
  prm.M = M;
  prm.T = T;
  prm.hq = hq;
  prm.hk = hk;
  prm.k_blocks = static_cast<int>(K / kBK);
  prm.v_out = static_cast<__nv_bfloat16*>(v_out);
  prm.row_scale = row_scale;
  prm.n_v = static_cast<int>(n_v);
  prm.n_blocks = static_cast<int>((n_cols + bn - 1) / bn);
  prm.n_tiles = m_blocks * prm.n_blocks;
  const int64_t grid = std::min<int64_t>(prm.n_tiles, dev->sms);
  switch (bn) {
    case 256: return launch<256>(map_x, map_w, prm, grid, stream);
    case 128: return launch<128>(map_x, map_w, prm, grid, stream);
    default: return launch<64>(map_x, map_w, prm, grid, stream);
  }
}

// The MLP's gate/up GEMM with SwiGLU in the epilogue: act[m][f] = silu(x[m] . gate[f]) *
// (x[m] . up[f]) for x [M][K] and w_il [2F][K], the gate and up rows interleaved in blocks of
// 128 (rows 256 nb ... 256 nb + 127: gate rows 128 nb ...; the next 128: the up rows of the
// same features). The [M][2F] product never goes to HBM.
int gemm_swiglu(const void* x, const void* w_il, int64_t M, int64_t K, int64_t F, void* act_out,
                uint32_t* status, cudaStream_t stream) {
  using namespace k1;
  if (M < 0 || K <= 0 || F <= 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "gemm_swiglu: bad shape M=%lld K=%lld F=%lld", (long long)M, (long long)K, (long long)F);
  if (K % kBK != 0 || F % 128 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "gemm_swiglu: K (%lld) a multiple of 64, F (%lld) of 128", (long long)K, (long long)F);
  if (M >= (int64_t(1) << 31) || K >= (int64_t(1) << 24) || F >= (int64_t(1) << 24))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "gemm_swiglu: shape too large");
  if (M == 0) return LEMA_OK;
  if (x == nullptr || w_il == nullptr || act_out == nullptr) return fail(LEMA_ERR_INVALID_ARGUMENT, "gemm_swiglu: null pointer");
  if (!aligned(x, 16) || !aligned(w_il, 16) || !aligned(act_out, 16))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "gemm_swiglu: x, w and act must be 16-byte aligned");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  if (dev->cc_major != 10) return fail(LEMA_ERR_UNSUPPORTED, "built for sm_100a; device is sm_%d%d", dev->cc_major, dev->cc_minor);
  EncodeTiledFn enc = encode_tiled();
  if (enc == nullptr) return fail(LEMA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  CUtensorMap map_x, map_w;
  if (!encode_kmajor(enc, &map_x, x, M, K, kBM) || !encode_kmajor(enc, &map_w, w_il, 2 * F, K, 256))
    return fail(LEMA_ERR_INVALID_ARGUMENT, "gemm_swiglu: tensor map encoding failed (M=%lld K=%lld F=%lld)", (long long)M, (long long)K, (long long)F);
  Params prm{};
  prm.status = status;
  prm.wait_ns = wait_limit_ns();
  prm.M = M;
  prm.T = M;
  prm.k_blocks = static_cast<int>(K / kBK);
  prm.act_out = static_cast<__nv_bfloat16*>(act_out);
  prm.act_f = F;
  prm.n_blocks = static_cast<int>(2 * F / 256);
  prm.n_tiles = ((M + kBM - 1) / kBM) * prm.n_blocks;
  const int64_t grid = std::min<int64_t>(prm.n_tiles, dev->sms);
  return launch<256>(map_x, map_w, prm, grid, stream);
}

// RMS scale of each row: out[m] = 1 / sqrt(mean(x[m]^2) + eps), fp32 sums; one warp per row.
__global__ void row_rms_kernel(const __nv_bfloat16* x, int64_t M, int64_t K, float eps, float* out) {
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (int64_t m = (blockIdx.x * int64_t(blockDim.x) + threadIdx.x) >> 5; m < M; m += warps) {
    const uint4* row = reinterpret_cast<const uint4*>(x + m * K);
    float acc = 0.f;
    for (int64_t k = lane; k < K / 8; k += 32) {
      const uint4 w = row[k];
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(h[e]);
        acc += f.x * f.x + f.y * f.y;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, o);
    if (lane == 0) out[m] = rsqrtf(acc / static_cast<float>(K) + eps);
  }
}

int row_rms(const void* x, int64_t M, int64_t K, float eps, float* out, cudaStream_t stream) {
  if (M < 0 || K <= 0 || K % 8 != 0) return fail(LEMA_ERR_INVALID_ARGUMENT, "row_rms: K = %lld must be a positive multiple of 8", (long long)K);
  if (M == 0) return LEMA_OK;
  if (x == nullptr || out == nullptr || !aligned(x, 16)) return fail(LEMA_ERR_INVALID_ARGUMENT, "row_rms: null or unaligned pointer");
  const DeviceInfo* dev = current_device_info();
  if (dev == nullptr) return LEMA_ERR_CUDA;
  const int64_t blocks = std::min<int64_t>((M + 7) / 8, int64_t(dev->sms) * 16);
  row_rms_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), M, K, eps, out);
  LEMA_CUDA_TRY(cudaGetLastError());
  return LEMA_OK;
}

}  // namespace lema

extern "C" int lema_proj_codes_v(const void* x, const void* w_all, int64_t M, int64_t K, int64_t T, int hq, int hk,
                                 int d_qk, uint32_t* qcodes, uint32_t* kcodes, int64_t n_v, void* v_out,
                                 const float* row_scale, uint32_t* status, void* stream) {
  lema::clear_error();
  return lema::proj_codes_v(x, w_all, M, K, T, hq, hk, d_qk, qcodes, kcodes, n_v, v_out, row_scale, status,
                            static_cast<cudaStream_t>(stream));
}

extern "C" int lema_gemm_swiglu(const void* x, const void* w_il, int64_t M, int64_t K, int64_t F, void* act_out,
                                uint32_t* status, void* stream) {
  lema::clear_error();
  return lema::gemm_swiglu(x, w_il, M, K, F, act_out, status, static_cast<cudaStream_t>(stream));
}

extern "C" int lema_row_rms(const void* x, int64_t M, int64_t K, float eps, float* out, void* stream) {
  lema::clear_error();
  return lema::row_rms(x, M, K, eps, out, static_cast<cudaStream_t>(stream));
}
