// 4-bit MatMulNBits prefill GEMM for sm_100a on tcgen05 tensor cores.
//
// Y[m, n] = sum_k A[m, k] * W[n, k] + bias[n], W[n, k] = (q[n, k] - z[n, k / bs]) * s[n, k / bs]
// (nbitWeight / packedMatmul of kernels/_shared/extended/shaders/complex_kernel.glsl:80,83).
//
// Orientation. One MMA computes D[n, m] += W[n, k] * A[m, k] for 128 weight rows (the MMA's M)
// and T activation rows (the MMA's N, 16 <= T <= 192, chosen per problem): the weight tile is
// operand A and lives in tensor memory, the activation tile is operand B in shared memory.
// Dequantized weights therefore never touch shared memory: the dequantizing warps unpack the
// TMA-staged nibbles in registers and write float16 straight into TMEM with tcgen05.st. The
// only shared-memory operand traffic is the activation tile (1/128 byte per flop).
//
// Warp roles (26 warps, one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer (one lane): activation tile [T x 64] (128-byte swizzle, the UMMA
//               K-major canonical layout), packed nibbles [128 x 32 B], an 8-block window of
//               scales and of zero points per 64-wide K step, into a ring of `stages` buffers.
//   warp 1      TMEM allocator and single-lane MMA issuer (4 x tcgen05.mma K=16, one commit
//               per step).
//   warps 2-17  dequantizers, four groups of four warps: group j handles the K steps g with
//               g % 4 == j (each warp has four steps of MMA time per step it dequantizes);
//               warp w owns TMEM lane quadrant w % 4, one weight row per thread.
//   warps 18-25 epilogue: lane quadrant w % 4, half of the T accumulator columns; adds the
//               bias, rounds to float16 and stores Y (masked at the M / N edges).
//
// Tensor memory (512 columns, allocated once): two fp32 accumulator buffers of 192 columns
// (tile i accumulates in buffer i % 2 while the epilogue drains the other), then four
// 32-column weight stages (64 float16 per lane each), stage j owned by dequant group j.
//
// Only the two issuing lanes poll their mbarriers; the dequant and epilogue warps wait with a
// hardware-suspending probe so that they take no issue slots from the issuers while idle.
//
// Every mbarrier wait is bounded (1 s of device time); on expiry the kernel records an error
// code in the device error word, raises a CTA-wide abort flag, waits (bounded) for its own
// copies and MMAs in flight, frees its tensor memory and returns.
#include <cuda.h>
#include <cuda_fp16.h>

#include <climits>
#include <cstdio>
#include <mutex>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kRows = 128;                // weight rows per tile (MMA M)
constexpr int kStepK = 64;                // K per pipeline step: one 128-byte swizzle row of fp16
constexpr int kMaxT = 192;                // activation rows per tile (MMA N) at most
constexpr int kAccCols = kMaxT;           // columns per accumulator buffer (two buffers)
constexpr int kWStages = 4;               // dequantized weight stages in TMEM
constexpr int kWCols = 32;                // TMEM columns per weight stage (64 f16 per lane)
constexpr int kWCol0 = 2 * kAccCols;      // first weight-stage column
constexpr int kTmemCols = 512;
static_assert(kWCol0 + kWStages * kWCols == kTmemCols, "TMEM map must fill the 512 columns");
constexpr int kDqGroups = kWStages;       // dequant group g % 4 owns weight stage g % 4
constexpr int kDequantWarps = 4 * kDqGroups;
constexpr int kEpilogueWarps = 8;
constexpr int kWarps = 2 + kDequantWarps + kEpilogueWarps;
constexpr int kThreads = kWarps * 32;
constexpr uint32_t kPackedStage = kRows * 32;  // 64 codes per row per step
constexpr uint32_t kMetaStage = kRows * 16;    // 16-byte window per row (scales or zero points)
constexpr int kMaxStages = 8;
constexpr int kStepOverheadCols = 128;  // per-step fixed cost in MMA columns (tile-height model)
constexpr int kSmemBudget = 227 * 1024;
constexpr size_t kOneCtaSmem = 120 * 1024;  // > half of the SM's 228 KB

// Device error codes of this kernel (first error wins in the device error word).
constexpr unsigned kErrWaitProducer = 0x301;
constexpr unsigned kErrWaitMma = 0x302;
constexpr unsigned kErrWaitDequant = 0x303;
constexpr unsigned kErrWaitEpilogue = 0x304;
constexpr unsigned kErrDrain = 0x305;
constexpr unsigned kSuspendHintNs = 0x989680;  // longest hardware suspension per mbarrier probe

enum ZpMode : int { kZDefault = 0, kZPacked = 1, kZHalf = 2 };

struct GemmArgs {
  int M, N, ksteps, T, n_ttiles, tiles, stages, bs_log2;
  uint32_t tok_stage_bytes;  // T * 128
  uint32_t tx_bytes;         // bytes landing per stage
  int64_t ldy;
  const __half* bias;
  __half* y;
  unsigned* err;
};

// ------------------------------------------------------------------ tcgen05 / TMA wrappers
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem_d] (+)= A[tmem_a] (128 x 16 f16, lanes = rows) * B[smem desc] (T x 16 f16, K-major)^T
__device__ __forceinline__ void mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
// Waits for this thread's tcgen05.ld; the registers are in/out operands so that no use of
// them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&a)[8], uint32_t (&b)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]),
                 "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7])
               ::"memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

// UMMA shared-memory descriptor, K-major operand in the 128-byte swizzle canonical layout:
// rows of 128 bytes, 8-row atoms 1024 bytes apart (stride byte offset), version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;             // leading byte offset (unused for swizzled K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;     // stride byte offset
  d |= static_cast<uint64_t>(1u) << 46;             // descriptor version
  d |= static_cast<uint64_t>(2u) << 61;             // SWIZZLE_128B
  return d;
}

// Instruction descriptor: f16 x f16 -> f32, both operands K-major, M = 128, N = T.
__device__ __forceinline__ uint32_t umma_idesc(int T) {
  return (1u << 4) | (static_cast<uint32_t>(T >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
}

struct Ctl {
  volatile int* abort;
  unsigned* err;
};

// Non-blocking probe of an mbarrier phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// mbarrier probe that may suspend the thread in hardware until the phase completes (or the
// time hint, in ns, passes).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done != 0;
}

// Single-lane bounded spin for the latency-critical roles (TMA producer, MMA issuer).
// Gives up on the abort flag or after the wait limit (raising it).
__device__ __forceinline__ bool thread_wait(uint64_t* bar, uint32_t parity, const Ctl& c, unsigned code) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  for (;;) {
    if (mbar_test_wait(bar, parity)) return true;
    if (*c.abort) return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_device_error(c.err, code);
      *c.abort = 1;
      return false;
    }
  }
}

// Whole-warp bounded wait (dequant and epilogue warps): every lane observes the phase and the
// warp agrees on the outcome, so the .sync.aligned tcgen05 instructions after it stay
// converged; the probes suspend the warp in hardware, leaving issue slots to the producer and
// the MMA issuer. Gives up on the abort flag or after the wait limit (raising it).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const Ctl& c, unsigned code) {
  if (__all_sync(~0u, mbar_try_wait_suspend(bar, parity))) return true;
  const uint64_t start = global_timer_ns();
  for (;;) {
    if (__all_sync(~0u, mbar_try_wait_suspend(bar, parity))) return true;
    const bool aborted = *c.abort != 0;
    const bool expired = global_timer_ns() - start > kWaitLimitNs;
    if (__any_sync(~0u, aborted || expired)) {
      if (__any_sync(~0u, expired) && (threadIdx.x & 31) == 0) {
        record_device_error(c.err, code);
        *c.abort = 1;
      }
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag: used to drain copies / MMAs before exit.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, unsigned* err) {
  const uint64_t start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_device_error(err, kErrDrain);
      return;
    }
  }
}

// float16x2 constant pair for an integer zero point z: adds -(1024 + z) to the low half
// (1024 + q) and -(64 + z) to the high half (1024 + 16 q) / 16, both exact.
__device__ __forceinline__ uint32_t zero_add_pair(uint32_t z) {
  return (0xE400u + z) | ((0xD400u + (z << 4)) << 16);
}

// Dequantizes the 8 codes of one little-endian word (k = 8i .. 8i+7, low nibble first) to
// four float16x2 registers in K order: out[j] = (w[8i+2j], w[8i+2j+1]).
template <int ZM>
__device__ __forceinline__ void dequant_word(uint32_t w, uint32_t add, uint32_t zz, uint32_t s2, uint32_t* out) {
  constexpr uint32_t kMul = 0x2C003C00u;  // (1, 1/16)
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    // byte j duplicated into both halves: low half keeps its low nibble, high half its high
    // nibble at bits 4..7, each OR-ed into the float16 1024: (1024 + q_lo, 1024 + 16 q_hi).
    uint32_t x = prmt(w, 0u, 0x4040u + 0x0101u * j);
    x = lop3_and_or(x, 0x00F0000Fu, 0x64006400u);
    uint32_t d = hfma2_u32(x, kMul, add);  // exact: (q_lo - z, q_hi - z) or (q_lo, q_hi)
    if (ZM == kZHalf) d = hsub2_u32(d, zz);
    out[j] = hmul2_u32(d, s2);
  }
}

template <int ZM>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_q4_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                      const __grid_constant__ CUtensorMap map_s, const __grid_constant__ CUtensorMap map_z,
                      const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = args.stages;

  // ---- shared memory carve-up (base rounded up to 1024 bytes for the swizzled tiles)
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t tok_s = base;
  const uint32_t pk_s = tok_s + S * args.tok_stage_bytes;
  const uint32_t sc_s = pk_s + S * kPackedStage;
  const uint32_t zp_s = sc_s + S * kMetaStage;
  const uint32_t bar_off = (zp_s + (ZM != kZDefault ? S * kMetaStage : 0u)) - base;
  uint64_t* full = reinterpret_cast<uint64_t*>(gbase + bar_off);
  uint64_t* empty = full + S;
  uint64_t* wfull = empty + S;
  uint64_t* accfull = wfull + kWStages;  // [2]
  uint64_t* accempty = accfull + 2;        // [2]
  uint64_t* drain = accempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);  // the MMA commit + the 4 warps of the step's dequant group
    }
    for (int s = 0; s < kWStages; ++s) mbar_init(&wfull[s], 4);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], kEpilogueWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(tmem_slot)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  const Ctl ctl{abort_flag, args.err};
  const int ksteps = args.ksteps;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int g = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x) {
        const int n0 = (tile / args.n_ttiles) * kRows;
        const int m0 = (tile % args.n_ttiles) * args.T;
        for (int ks = 0; ks < ksteps; ++ks, ++g) {
          if (!thread_wait(&empty[s], ph ^ 1, ctl, kErrWaitProducer)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], args.tx_bytes);
          const int blk = (ks * kStepK) >> args.bs_log2;
          tma_load_2d(tok_s + s * args.tok_stage_bytes, &map_a, ks * kStepK, m0, &full[s]);
          tma_load_2d(pk_s + s * kPackedStage, &map_b, ks * (kStepK / 2), n0, &full[s]);
          tma_load_2d(sc_s + s * kMetaStage, &map_s, blk & ~7, n0, &full[s]);
          if (ZM == kZPacked) tma_load_2d(zp_s + s * kMetaStage, &map_z, (blk & ~31) >> 1, n0, &full[s]);
          if (ZM == kZHalf) tma_load_2d(zp_s + s * kMetaStage, &map_z, blk & ~7, n0, &full[s]);
          if (++s == S) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) {
        // Wait for the copies still in flight (the last `S` issued steps) before exiting.
        for (int h = (g > S ? g - S : 0); h < g; ++h) drain_wait(&full[h % S], (h / S) & 1, args.err);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc(args.T);
      const uint64_t desc0 = umma_desc_sw128(tok_s);
      const uint32_t desc_stage = args.tok_stage_bytes >> 4;
      int i = 0, s = 0, ws = 0;
      uint32_t wph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < args.tiles; tile += gridDim.x, ++i) {
        const int b = i & 1;  // accumulator buffer: the epilogue drains the other one meanwhile
        if (!thread_wait(&accempty[b], ((i >> 1) & 1) ^ 1, ctl, kErrWaitMma)) break;
        tc_fence_after();
        const uint32_t d_col = tmem + b * kAccCols;
        for (int ks = 0; ks < ksteps; ++ks) {
          // wfull of step g implies full[s] of step g: the dequant group read this stage's
          // nibbles (after the stage's TMA completed) before it arrived.
          if (!thread_wait(&wfull[ws], wph, ctl, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = desc0 + s * desc_stage;
          const uint32_t a_col = tmem + kWCol0 + ws * kWCols;
#pragma unroll
          for (int j = 0; j < kStepK / 16; ++j)
            mma_ts(d_col, a_col + 8 * j, bdesc + 2 * j, idesc, (ks | j) != 0);
          // One commit per step: frees input stage s and, for the dequant group of step g + 4,
          // weight stage ws (both read by exactly these MMAs).
          mma_commit(&empty[s]);
          if (++s == S) s = 0;
          if (++ws == kWStages) {
            ws = 0;
            wph ^= 1;
          }
        }
        if (ok) mma_commit(&accfull[b]);
      }
      // Every MMA this thread issued has completed once `drain` flips.
      mma_commit(drain);
      drain_wait(drain, 0, args.err);
    }
  } else if (warp < 2 + kDequantWarps) {
    // ------------------------------------------------------------ dequantizers
    // Group `grp` dequantizes the K steps g = grp, grp + 4, ... into its own TMEM weight stage;
    // warp w % 4 covers TMEM lanes (weight rows) 32 (w % 4) .. 32 (w % 4) + 31. Step g is K step
    // g % ksteps of the CTA's tile number g / ksteps, in input stage g % S (S >= 4, so the
    // stage wraps at most once per advance).
    const int q = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int r = 32 * q + lane;  // weight row within the tile
    const uint32_t w_addr = tmem + (static_cast<uint32_t>(32 * q) << 16) + kWCol0 + grp * kWCols;
    const int bs_log2 = args.bs_log2;
    int tile = blockIdx.x, ks = grp, s = grp;
    uint32_t ph = 0;
    int prev_s = -1;  // input stage of this group's previous step g - 4 (none yet)
    uint32_t prev_ph = 0;
    while (ks >= ksteps) {
      ks -= ksteps;
      tile += gridDim.x;
    }
    while (tile < args.tiles) {
      if (!warp_wait(&full[s], ph, ctl, kErrWaitDequant)) break;
      const uint32_t prow = pk_s + s * kPackedStage + r * 32;
      const uint4 p0 = lds128(prow), p1 = lds128(prow + 16);
      // Word pair j (codes 16j .. 16j+15 of the step) lies in block bj (bs >= 16).
      const int kbase = ks * kStepK;
      const int w8 = (kbase >> bs_log2) & ~7;
      const uint32_t srow = sc_s + s * kMetaStage + r * 16;
      uint32_t s2[4], add[4], zz[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int bj = (kbase + 16 * j) >> bs_log2;
        const uint32_t sv = lds_u16(srow + (bj - w8) * 2);
        s2[j] = sv | (sv << 16);
        zz[j] = 0;
        if (ZM == kZDefault) {
          add[j] = zero_add_pair(8u);
        } else if (ZM == kZPacked) {
          const int w32 = (kbase >> bs_log2) & ~31;
          const uint32_t zb = lds_u8(zp_s + s * kMetaStage + r * 16 + ((bj - w32) >> 1));
          add[j] = zero_add_pair(((bj - w32) & 1) ? (zb >> 4) : (zb & 15u));
        } else {
          const uint32_t zh = lds_u16(zp_s + s * kMetaStage + r * 16 + (bj - w8) * 2);
          zz[j] = zh | (zh << 16);
          add[j] = 0xD400E400u;  // (-1024, -64): exact codes, zero point subtracted after
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done reading stage s

      // Weight stage `grp` is free once the MMAs of step g - 4 completed: their commit (with
      // this group's own earlier arrivals) completes the empty phase of that step's stage.
      if (prev_s >= 0 && !warp_wait(&empty[prev_s], prev_ph, ctl, kErrWaitDequant)) break;
      tc_fence_after();
      uint32_t v[32];
      dequant_word<ZM>(p0.x, add[0], zz[0], s2[0], v + 0);
      dequant_word<ZM>(p0.y, add[0], zz[0], s2[0], v + 4);
      dequant_word<ZM>(p0.z, add[1], zz[1], s2[1], v + 8);
      dequant_word<ZM>(p0.w, add[1], zz[1], s2[1], v + 12);
      dequant_word<ZM>(p1.x, add[2], zz[2], s2[2], v + 16);
      dequant_word<ZM>(p1.y, add[2], zz[2], s2[2], v + 20);
      dequant_word<ZM>(p1.z, add[3], zz[3], s2[3], v + 24);
      dequant_word<ZM>(p1.w, add[3], zz[3], s2[3], v + 28);
      tmem_st32(w_addr, v);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&wfull[grp]);

      prev_s = s;
      prev_ph = ph;
      s += kDqGroups;
      if (s >= S) {
        s -= S;
        ph ^= 1;
      }
      ks += kDqGroups;
      while (ks >= ksteps) {
        ks -= ksteps;
        tile += gridDim.x;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2 - kDequantWarps;
    const int q = warp & 3;
    const int c = e >> 2;  // which half of the accumulator columns
    const uint32_t lane_addr = static_cast<uint32_t>(32 * q) << 16;
    const int T = args.T;
    const int half_cols = T >> 1;  // multiple of 8
    int i = 0;
    for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++i) {
      const int b = i & 1;
      const int n = (tile / args.n_ttiles) * kRows + 32 * q + lane;
      const int mbase = (tile % args.n_ttiles) * T + c * half_cols;
      const float bias = (args.bias != nullptr && n < args.N) ? __half2float(args.bias[n]) : 0.0f;
      if (!warp_wait(&accfull[b], (i >> 1) & 1, ctl, kErrWaitEpilogue)) break;
      tc_fence_after();
      __half* ycol = args.y + n;
      for (int c0 = 0; c0 < half_cols; c0 += 16) {
        uint32_t va[8] = {}, vb[8] = {};
        const uint32_t taddr = tmem + lane_addr + b * kAccCols + c * half_cols + c0;
        tmem_ld8(taddr, va);
        if (c0 + 8 < half_cols) tmem_ld8(taddr + 8, vb);
        tmem_wait_ld(va, vb);
        if (n < args.N) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = mbase + c0 + j;
            if ((j < 8 || c0 + 8 < half_cols) && m < args.M) {
              const float acc = __uint_as_float(j < 8 ? va[j] : vb[j - 8]);
              ycol[static_cast<int64_t>(m) * args.ldy] = __float2half_rn(acc + bias);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accempty[b]);
    }
  }

  // ---- teardown: every role has stopped issuing; free tensor memory.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ------------------------------------------------------------------ host side
struct GemmShape {
  int T, n_ttiles, tiles, grid, stages;
  uint32_t tok_stage_bytes, tx_bytes;
  size_t smem;
};

int zp_mode(const Problem& p) {
  return p.zp == kZpPacked ? kZPacked : p.zp == kZpF16 ? kZHalf : kZDefault;
}

// Picks the activation-tile height T (a multiple of 16 up to 192) that minimises the number of
// persistent rounds times the per-tile cost: T columns of MMA per K step plus a fixed per-step
// cost of the pipeline (synchronisation and MMA issue), measured at about 128 columns' worth.
GemmShape gemm_shape(const Problem& p, int sms) {
  const int64_t n_w = ceil_div(p.N, kRows);
  GemmShape best{};
  double best_cost = 0.0;
  for (int T = 16; T <= kMaxT; T += 16) {
    const int64_t nt = ceil_div(p.M, T);
    const int64_t tiles = n_w * nt;
    if (tiles > INT_MAX) continue;
    const int64_t rounds = ceil_div(tiles, sms);
    const double cost = static_cast<double>(rounds) * (T + kStepOverheadCols);
    if (best.T == 0 || cost < best_cost || (cost == best_cost && T > best.T)) {
      best.T = T;
      best.n_ttiles = static_cast<int>(nt);
      best.tiles = static_cast<int>(tiles);
      best_cost = cost;
    }
  }
  best.grid = static_cast<int>(best.tiles < sms ? best.tiles : sms);
  best.tok_stage_bytes = static_cast<uint32_t>(best.T) * 128u;
  const uint32_t meta = kMetaStage * (zp_mode(p) != kZDefault ? 2u : 1u);
  const uint32_t stage = best.tok_stage_bytes + kPackedStage + meta;
  best.tx_bytes = stage;
  const size_t fixed = 1024 /* alignment slack */ + 512 /* barriers, TMEM slot, abort flag */;
  int stages = static_cast<int>((kSmemBudget - fixed) / stage);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < kDqGroups) stages = 0;  // the dequant groups' stage walk needs S >= 4 (never at T <= 192)
  best.stages = stages;
  best.smem = fixed + static_cast<size_t>(stages) * stage;
  // Each CTA allocates all 512 TMEM columns: request enough shared memory that a second CTA
  // can never be co-resident on the SM (it would stall in tcgen05.alloc).
  if (best.smem < kOneCtaSmem) best.smem = kOneCtaSmem;
  return best;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, resolved through the runtime so that the library has no
// link-time dependency on libcuda (it loads on machines without a driver).
EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

bool encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* ptr, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swz) {
  const EncodeTiledFn encode = encode_tiled_fn();
  if (encode == nullptr) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return encode(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int ZM>
cudaError_t launch_mode(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& msc, const CUtensorMap& mz,
                        const GemmArgs& args, const GemmShape& sh, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(gemm_q4_tc_kernel<ZM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(sh.smem));
  if (e != cudaSuccess) return e;
  gemm_q4_tc_kernel<ZM><<<sh.grid, kThreads, sh.smem, stream>>>(ma, mb, msc, mz, args);
  return cudaGetLastError();
}

}  // namespace

bool encode_tensor_map_2d(void* map, int dtype, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                          uint32_t box_inner, uint32_t box_outer, bool swizzle_128b) {
  return encode_2d(static_cast<CUtensorMap*>(map), dtype == 1 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                   ptr, inner, outer, row_bytes, box_inner, box_outer,
                   swizzle_128b ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE);
}

bool gemm_supported(const Problem& p) {
  if (!p.f16 || p.bits != 4 || p.M < 1 || p.N < 1) return false;
  if (p.K < kStepK || p.K % kStepK != 0 || p.K > (int64_t(1) << 30)) return false;
  if (p.bs < 16 || (p.bs & (p.bs - 1)) != 0 || p.K % p.bs != 0) return false;
  if (p.kb % 8 != 0) return false;                        // 16-byte rows of scales for TMA
  if (p.zp == kZpF32) return false;
  if (p.zp == kZpPacked && p.kb % 32 != 0) return false;  // 16-byte rows of packed zero points
  if (p.M > INT_MAX || p.N > INT_MAX || p.ldy < p.N) return false;
  if (!aligned(p.a, 16) || !aligned(p.b, 16) || !aligned(p.scales, 16)) return false;
  if (p.zp != kZpNone && !aligned(p.zp_ptr, 16)) return false;
  if (!aligned(p.y, 2) || (p.bias != nullptr && !aligned(p.bias, 2))) return false;
  return true;
}

uint64_t gemm_workspace_bytes(const Problem&) { return 0; }

cudaError_t launch_gemm(const Problem& p, void*, cudaStream_t stream) {
  if (!gemm_supported(p)) return cudaErrorNotSupported;
  if (p.M == 0) return cudaSuccess;
  const GemmShape sh = gemm_shape(p, device_sm_count());
  if (sh.stages == 0) return cudaErrorNotSupported;

  CUtensorMap ma, mb, msc, mz;
  const uint64_t K = static_cast<uint64_t>(p.K), N = static_cast<uint64_t>(p.N);
  const uint64_t kb = static_cast<uint64_t>(p.kb);
  bool ok = encode_2d(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, p.a, K, static_cast<uint64_t>(p.M), K * 2, kStepK,
                      static_cast<uint32_t>(sh.T), CU_TENSOR_MAP_SWIZZLE_128B);
  ok = ok && encode_2d(&mb, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.b, K / 2, N, K / 2, kStepK / 2, kRows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  ok = ok && encode_2d(&msc, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, p.scales, kb, N, kb * 2, 8, kRows,
                       CU_TENSOR_MAP_SWIZZLE_NONE);
  const int zm = zp_mode(p);
  if (zm == kZPacked) {
    ok = ok && encode_2d(&mz, CU_TENSOR_MAP_DATA_TYPE_UINT8, p.zp_ptr, kb / 2, N, kb / 2, 16, kRows,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
  } else if (zm == kZHalf) {
    ok = ok && encode_2d(&mz, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, p.zp_ptr, kb, N, kb * 2, 8, kRows,
                         CU_TENSOR_MAP_SWIZZLE_NONE);
  } else {
    mz = msc;  // unused by the kernel
  }
  if (!ok) return cudaErrorInvalidValue;

  GemmArgs args{};
  args.M = static_cast<int>(p.M);
  args.N = static_cast<int>(p.N);
  args.ksteps = static_cast<int>(p.K / kStepK);
  args.T = sh.T;
  args.n_ttiles = sh.n_ttiles;
  args.tiles = sh.tiles;
  args.stages = sh.stages;
  int lg = 0;
  while ((int64_t(1) << lg) < p.bs) ++lg;
  args.bs_log2 = lg;
  args.tok_stage_bytes = sh.tok_stage_bytes;
  args.tx_bytes = sh.tx_bytes;
  args.ldy = p.ldy;
  args.bias = static_cast<const __half*>(p.bias);
  args.y = static_cast<__half*>(p.y);
  args.err = p.err;
  switch (zm) {
    case kZPacked: return launch_mode<kZPacked>(ma, mb, msc, mz, args, sh, stream);
    case kZHalf: return launch_mode<kZHalf>(ma, mb, msc, mz, args, sh, stream);
    default: return launch_mode<kZDefault>(ma, mb, msc, mz, args, sh, stream);
  }
}

}  // namespace xrgpu
