// 4-bit MatMulNBits decode GEMV for sm_100a (M <= 16 rows, float16 activations).
//
// The kernel streams the packed weights once, unpacks nibbles to float16 in registers and
// multiplies them on the tensor cores (mma.sync m16n8k16, float32 accumulation). Exactness:
//   * each nibble becomes float16 (q - z) exactly: LOP3 places it in the mantissa of 1024.0
//     (0x6400), then one float16 subtract / fused multiply-add removes 1024 + z (z integer:
//     the default 2^(bits-1) or a packed uint8 zero point);
//   * a float zero point (reference contract, possibly non-integer) is applied instead as
//     sum(q*x) - z*sum(x) in float32, sum(x) coming from the same MMA against a ones operand;
//   * the tensor core multiplies exact float16 operands and accumulates in float32, and the
//     per-block scale is applied in float32 once per block.
// This restates packedMatmul/nbitWeight (complex_kernel.glsl:80,83) with the exact
// association sum_b s_b * sum_{k in b} (q_k - z_b) * x_k.
//
// Decomposition. A warp owns one tile of 16 output columns and a block-aligned range of
// 64-wide k "regions". Lane (g = lane/4, c = lane%4) handles columns n0+g and n0+g+8. The
// warp streams its weights with cp.async (16 bytes per lane, L1 bypassed) into its own
// kStages-deep shared-memory ring, one batch of 4 regions (128 bytes per column) per stage,
// so about 8 KB per warp are in flight without holding registers; each lane then reads the
// exact 32-bit words its mma fragments need (word c of each 16-byte block for block size
// 32). A CTA of 4 warps holds `tpc` column tiles and splits its k range into 4/tpc slices;
// it stages its activations once (cp.async, permuted in place into mma B-fragment order).
// Per-block scales and zero points go, 8 regions at a time, into a per-warp window of
// 16-byte records (float32 scale, float16x2 unpack constants, float32 zero point), loaded one
// chunk ahead (vectorised when the block size is 32 and K is a multiple of 256). Split-K CTAs
// of one column group form a thread-block cluster and combine their partial sums in a fixed
// order through distributed shared memory: no global workspace, deterministic results.
#include <cuda_fp16.h>

#include <algorithm>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kCols = 16;
constexpr int kRegionK = 64;              // k per region: 32 bytes of one column
constexpr int kBatch = 4;                 // regions per ring stage
constexpr int kStages = 4;                // ring depth (batches)
constexpr int kRowBytes = kBatch * 32 + 16;             // one column's bytes in a stage, padded
constexpr int kStageBytes = kCols * kRowBytes;          // 2304
constexpr int kRingBytes = kStages * kStageBytes;       // per warp
constexpr int kChunk = 8;                 // regions per metadata chunk (512 k) = 2 batches
constexpr int kMaxSplits = 8;             // portable cluster size
constexpr int kSmemBudget = 160 * 1024;   // dynamic shared memory per CTA
constexpr int kTargetWarps = 24;          // per SM

enum ZpMode : int { kModeDefault = 0, kModeInt = 1, kModeFloat = 2 };

struct GemvParams {
  const __half* x;        // [M, K]
  const uint8_t* b;       // [N, K/2]
  const __half* scales;   // [N, kb]
  const void* zp;         // zero points (kind zp_kind) or nullptr
  const __half* bias;     // [N] or nullptr
  __half* y;              // [M, ldy]
  int64_t ldy;
  int M, K, N, kb, zp_kind;
  int log2_bs;
  int groups;             // block-aligned k groups
  int group_regions;      // regions per group
  int splits, tpc;
  int xrow_bytes;         // staged activation row stride (bytes)
  int smem_x_bytes;       // bytes of the staged activations
  int nb_chunk;           // blocks per 8-region chunk: max(1, 512 / bs)
  int win_stride;         // records per column in a window
};

// k offset (within a 64-wide region) of the 8 consecutive k that lane c holds in half h:
// block size 32: half h is block h and lane c holds its word c; otherwise lane c holds the
// 8 bytes at 8c, i.e. k in [16c, 16c+16) and half h = [16c + 8h, 16c + 8h + 8).
__host__ __device__ __forceinline__ constexpr int koff(bool exch, int h, int c) {
  return exch ? 32 * h + 8 * c : 16 * c + 8 * h;
}

// Nibbles of one 32-bit word (k0..k7, k_i in bits 4i..4i+3) as float16 pairs
// q[0] = (k0,k4), q[1] = (k1,k5), q[2] = (k2,k6), q[3] = (k3,k7), each equal to k_i - z.
// c_lo = (1024+z, 1024+z); c_hi = (-(64+z), -(64+z)) in float16.
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t c_lo, uint32_t c_hi, uint32_t (&q)[4]) {
  constexpr uint32_t kLo = 0x000F000Fu, kHi = 0x00F000F0u, kExp = 0x64006400u, kSixteenth = 0x2C002C00u;
  const uint32_t w8 = w >> 8;
  q[0] = hsub2_u32(lop3_and_or(w, kLo, kExp), c_lo);
  q[1] = hfma2_u32(lop3_and_or(w, kHi, kExp), kSixteenth, c_hi);
  q[2] = hsub2_u32(lop3_and_or(w8, kLo, kExp), c_lo);
  q[3] = hfma2_u32(lop3_and_or(w8, kHi, kExp), kSixteenth, c_hi);
}

// float16x2 unpack constants for an integer zero point z in [0, 15] (4-bit codes):
// (1024 + z, 1024 + z) (ulp 1) and (-(64 + z), -(64 + z)) (64 + z < 128 has ulp 1/16).
__host__ __device__ __forceinline__ constexpr uint32_t zconst_lo(uint32_t z) { return (0x6400u + z) * 0x00010001u; }
__host__ __device__ __forceinline__ constexpr uint32_t zconst_hi(uint32_t z) {
  return (0xD400u + (z << 4)) * 0x00010001u;
}

__device__ __forceinline__ void cp_async_16(uint32_t smem_addr, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float ld_dsmem_f32(const float* local_addr, unsigned rank) {
  uint32_t remote;
  float v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(local_addr)), "r"(rank));
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
}

// D = A * B with a zero accumulator input.
__device__ __forceinline__ void mma_16816_zc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// Region range [r0, r1) of (part s of S) over block-aligned groups.
__host__ __device__ __forceinline__ void split_range(int groups, int group_regions, int s, int S, int& r0, int& r1) {
  r0 = static_cast<int>(static_cast<int64_t>(groups) * s / S) * group_regions;
  r1 = static_cast<int>(static_cast<int64_t>(groups) * (s + 1) / S) * group_regions;
}

template <int MT>
struct Acc {
  float y[MT][4];   // output partial sums
  float d[MT][4];   // current block's sum(q*x) (or sum((q-z)*x))
  float xs[MT][4];  // current block's sum(x) (float zero points)
};

// One half-region (32 k of columns A and B, one word each) into the block sums d.
template <int MT, int ZM>
__device__ __forceinline__ void mma_half(Acc<MT>& acc, uint32_t wa, uint32_t wb, uint32_t clo_a, uint32_t chi_a,
                                         uint32_t clo_b, uint32_t chi_b, uint32_t xaddr, uint32_t xrow8,
                                         bool row_ok0, bool row_ok1, bool first) {
  uint32_t qa[4], qb[4];
  unpack8(wa, clo_a, chi_a, qa);
  unpack8(wb, clo_b, chi_b, qb);
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    uint4 xf = make_uint4(0u, 0u, 0u, 0u);
    if (t == 0 ? row_ok0 : row_ok1) xf = lds128(xaddr + t * xrow8);
    if (first) mma_16816_zc(acc.d[t], qa[0], qb[0], qa[2], qb[2], xf.x, xf.y);
    else mma_16816(acc.d[t], qa[0], qb[0], qa[2], qb[2], xf.x, xf.y);
    mma_16816(acc.d[t], qa[1], qb[1], qa[3], qb[3], xf.z, xf.w);
    if (ZM == kModeFloat) {
      constexpr uint32_t kOnes = 0x3C003C00u;
      if (first) mma_16816_zc(acc.xs[t], kOnes, kOnes, kOnes, kOnes, xf.x, xf.y);
      else mma_16816(acc.xs[t], kOnes, kOnes, kOnes, kOnes, xf.x, xf.y);
      mma_16816(acc.xs[t], kOnes, kOnes, kOnes, kOnes, xf.z, xf.w);
    }
  }
}

// y += s * (d - z * sum(x)) with the block records ra (column A) and rb (column B):
// record = {float32 scale, unpack constant lo, unpack constant hi, float32 zero point}.
template <int MT, int ZM>
__device__ __forceinline__ void finish_block(Acc<MT>& acc, uint4 ra, uint4 rb) {
  const float sa = __uint_as_float(ra.x), sb = __uint_as_float(rb.x);
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    float d0 = acc.d[t][0], d1 = acc.d[t][1], d2 = acc.d[t][2], d3 = acc.d[t][3];
    if (ZM == kModeFloat) {
      const float za = __uint_as_float(ra.w), zb = __uint_as_float(rb.w);
      d0 = fmaf(-za, acc.xs[t][0], d0);
      d1 = fmaf(-za, acc.xs[t][1], d1);
      d2 = fmaf(-zb, acc.xs[t][0], d2);
      d3 = fmaf(-zb, acc.xs[t][1], d3);
    }
    acc.y[t][0] = fmaf(sa, d0, acc.y[t][0]);
    acc.y[t][1] = fmaf(sa, d1, acc.y[t][1]);
    acc.y[t][2] = fmaf(sb, d2, acc.y[t][2]);
    acc.y[t][3] = fmaf(sb, d3, acc.y[t][3]);
  }
}

template <int ZM>
__device__ __forceinline__ void block_consts(uint4 ra, uint4 rb, uint32_t& clo_a, uint32_t& chi_a, uint32_t& clo_b,
                                             uint32_t& chi_b) {
  if (ZM == kModeInt) {
    clo_a = ra.y; chi_a = ra.z;
    clo_b = rb.y; chi_b = rb.z;
  } else {
    clo_a = clo_b = zconst_lo(ZM == kModeFloat ? 0u : 8u);
    chi_a = chi_b = zconst_hi(ZM == kModeFloat ? 0u : 8u);
  }
}

// Stores one 16-byte record (scale, zero point) for the given mode.
template <int ZM>
__device__ __forceinline__ void store_record(uint32_t addr, float scale, float z) {
  uint32_t lo = 0u, hi = 0u;
  if (ZM == kModeInt) {
    lo = zconst_lo(static_cast<uint32_t>(z));
    hi = zconst_hi(static_cast<uint32_t>(z));
  }
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(__float_as_uint(scale)), "r"(lo), "r"(hi),
               "r"(__float_as_uint(z))
               : "memory");
}

// ----------------------------------------------------------------- metadata chunks
// Vectorised form (block size 32, kb % 8 == 0, chunk starts on a multiple of 4 regions):
// lane l holds column l & 15, blocks [8 (l >> 4), +8) of the chunk's 16 blocks.
struct MetaVec {
  uint4 s;      // 8 float16 scales
  uint4 z;      // 8 zero-point nibbles in z.x (int) or 8 float16 zero points (float16)
};

template <int ZM>
__device__ __forceinline__ void meta_vec_load(const GemvParams& p, MetaVec& mv, int n0, int blk_first, int lane) {
  const int col = min(n0 + (lane & 15), p.N - 1);
  const int blk = blk_first + 8 * (lane >> 4);
  mv.s = make_uint4(0u, 0u, 0u, 0u);
  mv.z = make_uint4(0u, 0u, 0u, 0u);
  if (blk < p.kb) {
    const int64_t idx = static_cast<int64_t>(col) * p.kb + blk;
    mv.s = *reinterpret_cast<const uint4*>(p.scales + idx);
    if (ZM == kModeInt) mv.z.x = *reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(p.zp) + (idx >> 1));
    if (ZM == kModeFloat) mv.z = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(p.zp) + idx);
  }
}

template <int ZM>
__device__ __forceinline__ void meta_vec_store(const MetaVec& mv, uint32_t win_u32, int win_stride, int lane) {
  const uint32_t base = win_u32 + static_cast<uint32_t>((lane & 15) * win_stride + 8 * (lane >> 4)) * 16u;
  const uint32_t sw[4] = {mv.s.x, mv.s.y, mv.s.z, mv.s.w};
  const uint32_t zw[4] = {mv.z.x, mv.z.y, mv.z.z, mv.z.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 s2 = *reinterpret_cast<const __half2*>(&sw[i]);
    float z0 = 0.f, z1 = 0.f;
    if (ZM == kModeInt) {
      z0 = static_cast<float>((zw[0] >> (8 * i)) & 15u);
      z1 = static_cast<float>((zw[0] >> (8 * i + 4)) & 15u);
    } else if (ZM == kModeFloat) {
      const __half2 z2 = *reinterpret_cast<const __half2*>(&zw[i]);
      z0 = __low2float(z2);
      z1 = __high2float(z2);
    }
    store_record<ZM>(base + 32u * i, __low2float(s2), z0);
    store_record<ZM>(base + 32u * i + 16u, __high2float(s2), z1);
  }
}

// General form: lane l holds elements e = l + 32 i of the (16 x nb) chunk.
constexpr int kMetaPerLane = 8;
struct MetaScalar {
  float s[kMetaPerLane];
  float z[kMetaPerLane];
};

template <int ZM>
__device__ __forceinline__ void meta_scalar_load(const GemvParams& p, MetaScalar& mr, int n0, int blk_first, int lane,
                                                 int log2_nb) {
  const int nb = 1 << log2_nb;
#pragma unroll
  for (int i = 0; i < kMetaPerLane; ++i) {
    const int e = lane + 32 * i;
    mr.s[i] = mr.z[i] = 0.f;
    if (e < kCols * nb) {
      const int col = min(n0 + (e >> log2_nb), p.N - 1);
      const int blk = blk_first + (e & (nb - 1));
      if (blk < p.kb) {
        const int64_t idx = static_cast<int64_t>(col) * p.kb + blk;
        mr.s[i] = __half2float(p.scales[idx]);
        if (ZM == kModeInt) {
          const int64_t stride = (p.kb + 1) >> 1;
          const uint32_t byte = reinterpret_cast<const uint8_t*>(p.zp)[static_cast<int64_t>(col) * stride + (blk >> 1)];
          mr.z[i] = static_cast<float>((byte >> (4 * (blk & 1))) & 15u);
        } else if (ZM == kModeFloat) {
          mr.z[i] = p.zp_kind == kZpF32 ? reinterpret_cast<const float*>(p.zp)[idx]
                                        : __half2float(reinterpret_cast<const __half*>(p.zp)[idx]);
        }
      }
    }
  }
}

template <int ZM>
__device__ __forceinline__ void meta_scalar_store(const MetaScalar& mr, uint32_t win_u32, int win_stride, int lane,
                                                  int log2_nb) {
  const int nb = 1 << log2_nb;
#pragma unroll
  for (int i = 0; i < kMetaPerLane; ++i) {
    const int e = lane + 32 * i;
    if (e < kCols * nb)
      store_record<ZM>(win_u32 + static_cast<uint32_t>((e >> log2_nb) * win_stride + (e & (nb - 1))) * 16u, mr.s[i],
                       mr.z[i]);
  }
}

// MT: 8-row activation tiles (M <= 8*MT). EXCH: block_size == 32. ZM: zero-point mode.
// VEC: vectorised metadata (block size 32 only).
template <int MT, bool EXCH, int ZM, bool VEC>
__global__ void __launch_bounds__(kThreads) gemv_q4_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[kWarps][kCols][8 * MT];
  __shared__ float part[kWarps][kCols * 8 * MT];

  const int M = p.M;
  const int split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int tpc = p.tpc, slices = kWarps / tpc;
  const int tile = blockIdx.x * tpc + warp % tpc, slice = warp / tpc;
  const int n0 = tile * kCols;
  int r0, r1;  // this CTA's regions
  split_range(p.groups, p.group_regions, split, p.splits, r0, r1);
  int wr0, wr1;  // this warp's regions (absolute)
  {
    int a, b;
    split_range((r1 - r0) / p.group_regions, p.group_regions, slice, slices, a, b);
    wr0 = r0 + a;
    wr1 = r0 + b;
  }
  const bool tile_ok = n0 < p.N;
  const int colA = min(n0 + g, p.N - 1), colB = min(n0 + g + 8, p.N - 1);
  const int64_t colbytes = static_cast<int64_t>(p.K) / 2;
  const int log2_nb = 31 - __clz(p.nb_chunk);

  unsigned char* xs = smem_raw;
  const uint32_t win_u32 = smem_u32(smem_raw + p.smem_x_bytes) + static_cast<uint32_t>(warp * kCols * p.win_stride) * 16u;
  const uint32_t ring_u32 =
      smem_u32(smem_raw + p.smem_x_bytes + kWarps * kCols * p.win_stride * 16) + static_cast<uint32_t>(warp * kRingBytes);

  // Programmatic dependent launch: let the next kernel in the stream start its own weight
  // prefetch while this one runs; everything that may depend on earlier kernels (the
  // activations read below, the output written at the end) comes after griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---- weight stream: batch j (regions wr0 + 4j ..) goes to stage j % kStages. Lane (g, c)
  // copies 16 bytes of columns A and B for each pair of regions: region 2jj + (c >> 1) of the
  // batch, bytes 16 (c & 1) within it, landing at row offset 64 jj + 16 c.
  const int nbatches = (wr1 - wr0 + kBatch - 1) / kBatch;
  const uint8_t* srcA = p.b + colA * colbytes + static_cast<int64_t>(wr0) * 32 + (c >> 1) * 32 + (c & 1) * 16;
  const uint8_t* srcB = p.b + colB * colbytes + static_cast<int64_t>(wr0) * 32 + (c >> 1) * 32 + (c & 1) * 16;
  const uint32_t dstA = ring_u32 + static_cast<uint32_t>(g * kRowBytes + 16 * c);
  const uint32_t dstB = ring_u32 + static_cast<uint32_t>((g + 8) * kRowBytes + 16 * c);
  auto issue = [&](int j) {
    if (tile_ok && j < nbatches) {
      const uint32_t so = static_cast<uint32_t>(j % kStages) * kStageBytes;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int r = wr0 + kBatch * j + 2 * jj + (c >> 1);
        if (r < wr1) {
          const int64_t off = static_cast<int64_t>(kBatch * j + 2 * jj) * 32;
          cp_async_16(dstA + so + 64 * jj, srcA + off);
          cp_async_16(dstB + so + 64 * jj, srcB + off);
        }
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int j = 0; j < kStages - 1; ++j) issue(j);

  MetaVec mv;
  MetaScalar ms;
  if (tile_ok && wr0 < wr1) {
    if (VEC) meta_vec_load<ZM>(p, mv, n0, (wr0 * kRegionK) >> p.log2_bs, lane);
    else meta_scalar_load<ZM>(p, ms, n0, (wr0 * kRegionK) >> p.log2_bs, lane, log2_nb);
  }

  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- stage the CTA's activations (cp.async, 16-byte chunks) and permute them in place
  // into mma B-fragment order: (x0,x4), (x2,x6), (x1,x5), (x3,x7).
  const int chunks_per_row = (r1 - r0) * (kRegionK / 8);
  const int xchunks = M * chunks_per_row;
  {
    int m = 0, ch = threadIdx.x;
    while (ch >= chunks_per_row && m < M) { ch -= chunks_per_row; ++m; }
    for (int e = threadIdx.x; e < xchunks; e += kThreads) {
      cp_async_16(smem_u32(xs + m * p.xrow_bytes + ch * 16),
                  p.x + static_cast<int64_t>(m) * p.K + static_cast<int64_t>(r0) * kRegionK + ch * 8);
      ch += kThreads;
      while (ch >= chunks_per_row && m < M) { ch -= chunks_per_row; ++m; }
    }
  }
  cp_async_commit();
  cp_async_wait<0>();  // activations (and the first weight stages) have landed
  __syncthreads();
  {
    int m = 0, ch = threadIdx.x;
    while (ch >= chunks_per_row && m < M) { ch -= chunks_per_row; ++m; }
    for (int e = threadIdx.x; e < xchunks; e += kThreads) {
      uint4* ptr = reinterpret_cast<uint4*>(xs + m * p.xrow_bytes + ch * 16);
      const uint4 v = *ptr;
      *ptr = make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.y, v.w, 0x5410), prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x7632));
      ch += kThreads;
      while (ch >= chunks_per_row && m < M) { ch -= chunks_per_row; ++m; }
    }
  }
  __syncthreads();

  Acc<MT> acc;
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc.y[t][i] = acc.d[t][i] = acc.xs[t][i] = 0.f;
  uint32_t clo_a, chi_a, clo_b, chi_b;
  block_consts<ZM>(make_uint4(0u, 0u, 0u, 0u), make_uint4(0u, 0u, 0u, 0u), clo_a, chi_a, clo_b, chi_b);
  const bool row_ok0 = g < M, row_ok1 = g + 8 < M;

  if (tile_ok) {
    const uint32_t recA0 = win_u32 + static_cast<uint32_t>(g * p.win_stride) * 16u;
    const uint32_t recB0 = win_u32 + static_cast<uint32_t>((g + 8) * p.win_stride) * 16u;
    const uint32_t xrow8 = static_cast<uint32_t>(8 * p.xrow_bytes);
    const uint32_t xbase = smem_u32(xs) + static_cast<uint32_t>(g * p.xrow_bytes + koff(EXCH, 0, c) * 2);
    constexpr uint32_t kHalfStep = EXCH ? 64u : 16u;  // bytes between the halves' activation chunks
    const uint32_t rdA = ring_u32 + static_cast<uint32_t>(g * kRowBytes) + (EXCH ? 4u * c : 8u * c);
    const uint32_t rdB = ring_u32 + static_cast<uint32_t>((g + 8) * kRowBytes) + (EXCH ? 4u * c : 8u * c);
    const int bmask = (1 << p.log2_bs) - 1;
    int blk_first = 0;

    for (int j = 0; j < nbatches; ++j) {
      const int reg = wr0 + kBatch * j;
      const bool chunk_start = (j & 1) == 0;
      if (chunk_start) {
        // Records of this chunk into the window; the next chunk's metadata goes in flight.
        __syncwarp();
        if (VEC) meta_vec_store<ZM>(mv, win_u32, p.win_stride, lane);
        else meta_scalar_store<ZM>(ms, win_u32, p.win_stride, lane, log2_nb);
        blk_first = (reg * kRegionK) >> p.log2_bs;
        if (reg + kChunk < wr1) {
          if (VEC) meta_vec_load<ZM>(p, mv, n0, ((reg + kChunk) * kRegionK) >> p.log2_bs, lane);
          else meta_scalar_load<ZM>(p, ms, n0, ((reg + kChunk) * kRegionK) >> p.log2_bs, lane, log2_nb);
        }
      }
      // Batch j is in shared memory once every lane's copies for it completed.
      cp_async_wait<kStages - 2>();
      __syncwarp();
      const uint32_t so = static_cast<uint32_t>(j % kStages) * kStageBytes;
      const int cend = min(reg - ((reg - wr0) & (kChunk - 1)) + kChunk, wr1);
      const uint32_t xb = xbase + static_cast<uint32_t>((reg - r0) * kRegionK * 2);
#pragma unroll
      for (int u = 0; u < kBatch; ++u) {
        const int r = reg + u;
        if (r < wr1) {
          const uint32_t xa = xb + u * (kRegionK * 2);
          if (EXCH) {
            const uint32_t rec = static_cast<uint32_t>(2 * r - blk_first) * 16u;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const uint32_t wa = lds32(rdA + so + 32u * u + 16u * h);
              const uint32_t wb = lds32(rdB + so + 32u * u + 16u * h);
              const uint4 ma = lds128(recA0 + rec + 16u * h), mb = lds128(recB0 + rec + 16u * h);
              block_consts<ZM>(ma, mb, clo_a, chi_a, clo_b, chi_b);
              mma_half<MT, ZM>(acc, wa, wb, clo_a, chi_a, clo_b, chi_b, xa + kHalfStep * h, xrow8, row_ok0, row_ok1, true);
              finish_block<MT, ZM>(acc, ma, mb);
            }
          } else {
            const uint2 wa = lds64(rdA + so + 32u * u), wb = lds64(rdB + so + 32u * u);
            const int gk = r * kRegionK;
            const uint32_t rec = static_cast<uint32_t>((gk >> p.log2_bs) - blk_first) * 16u;
            const bool starts = (gk & bmask) == 0 || (u == 0 && chunk_start);
            const bool ends = ((gk + kRegionK) & bmask) == 0 || r + 1 == cend;
            const uint4 ma = lds128(recA0 + rec), mb = lds128(recB0 + rec);
            if (starts) block_consts<ZM>(ma, mb, clo_a, chi_a, clo_b, chi_b);
            mma_half<MT, ZM>(acc, wa.x, wb.x, clo_a, chi_a, clo_b, chi_b, xa, xrow8, row_ok0, row_ok1, starts);
            mma_half<MT, ZM>(acc, wa.y, wb.y, clo_a, chi_a, clo_b, chi_b, xa + kHalfStep, xrow8, row_ok0, row_ok1, false);
            if (ends) finish_block<MT, ZM>(acc, ma, mb);
          }
        }
      }
      // Stage (j + kStages - 1) % kStages held batch j - 1, which every lane finished reading
      // before the __syncwarp above: refill it.
      issue(j + kStages - 1);
    }
  }
  cp_async_wait<0>();

  // ---- reduce the k slices of each tile (fixed order), then the split-K CTAs of this
  // cluster through distributed shared memory.
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    red[warp][g][8 * t + 2 * c] = acc.y[t][0];
    red[warp][g][8 * t + 2 * c + 1] = acc.y[t][1];
    red[warp][g + 8][8 * t + 2 * c] = acc.y[t][2];
    red[warp][g + 8][8 * t + 2 * c + 1] = acc.y[t][3];
  }
  __syncthreads();
  const int per_tile = kCols * M;
  for (int idx = threadIdx.x; idx < tpc * per_tile; idx += kThreads) {
    const int t = idx / per_tile, rem = idx - t * per_tile;
    const int col = rem % kCols, m = rem / kCols;
    float v = 0.f;
    for (int sl = 0; sl < slices; ++sl) v += red[t + sl * tpc][col][m];
    part[t][rem] = v;
  }
  if (p.splits > 1) cluster_sync();
  else __syncthreads();
  if (split == 0) {
    for (int idx = threadIdx.x; idx < tpc * per_tile; idx += kThreads) {
      const int t = idx / per_tile, rem = idx - t * per_tile;
      const int col = rem % kCols, m = rem / kCols;
      const int n = (blockIdx.x * tpc + t) * kCols + col;
      float v = part[t][rem];
      for (int s = 1; s < p.splits; ++s) v += ld_dsmem_f32(&part[t][rem], static_cast<unsigned>(s));
      if (n < p.N) {
        if (p.bias) v += __half2float(p.bias[n]);
        p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(v);
      }
    }
  }
  if (p.splits > 1) cluster_sync();  // keep every CTA's shared memory alive until it is read
}

struct GemvShape {
  int tiles, tpc, splits, mt, groups, group_regions, xrow_bytes, smem_x_bytes, nb_chunk, win_stride;
  bool vec;
  size_t smem;
};

int ilog2(int64_t v) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= v) ++r;
  return r;
}

GemvShape gemv_shape(const Problem& p) {
  GemvShape s{};
  const int regions = static_cast<int>(p.K / kRegionK);
  s.tiles = static_cast<int>(ceil_div(p.N, kCols));
  s.mt = p.M <= 8 ? 1 : 2;
  const int block_regions = static_cast<int>(std::max<int64_t>(1, p.bs / kRegionK));
  // Vectorised metadata needs chunk starts on multiples of 4 regions (16-byte aligned scales).
  s.vec = p.bs == 32 && p.kb % 8 == 0 && regions % 4 == 0 && p.zp != kZpF32 &&
          (reinterpret_cast<uintptr_t>(p.scales) % 16) == 0 &&
          (p.zp == kZpNone || (reinterpret_cast<uintptr_t>(p.zp_ptr) % 16) == 0);
  s.group_regions = s.vec ? std::max(block_regions, 4) : block_regions;
  s.groups = regions / s.group_regions;
  s.nb_chunk = static_cast<int>(std::max<int64_t>(1, kChunk * kRegionK / p.bs));
  // 16-byte records; rows of nb + 1 records keep the 8 rows a warp reads in distinct banks.
  s.win_stride = s.nb_chunk >= 2 ? s.nb_chunk + 1 : 3;
  const int sms = device_sm_count();
  const int target = sms * kTargetWarps;
  s.tpc = s.tiles >= target ? 4 : (s.tiles >= target / 2 ? 2 : 1);
  const int slices = kWarps / s.tpc;
  int splits = static_cast<int>(ceil_div(target, static_cast<int64_t>(s.tiles) * slices));
  splits = std::max(1, std::min({splits, kMaxSplits, std::max(1, s.groups / slices)}));
  for (;; ++splits) {
    const int cta_regions = static_cast<int>(ceil_div(s.groups, splits)) * s.group_regions;
    s.xrow_bytes = cta_regions * kRegionK * 2 + 64;  // +64 B: rows alternate shared-memory bank halves
    s.smem_x_bytes = static_cast<int>(p.M) * s.xrow_bytes;
    s.smem = static_cast<size_t>(s.smem_x_bytes) + static_cast<size_t>(kWarps) * kCols * s.win_stride * 16 +
             static_cast<size_t>(kWarps) * kRingBytes;
    if (s.smem <= static_cast<size_t>(kSmemBudget) || splits >= std::min(kMaxSplits, s.groups)) break;
  }
  s.splits = splits;
  return s;
}

template <int MT, bool EXCH, int ZM, bool VEC>
cudaError_t launch_variant(const GemvShape& s, const GemvParams& gp, cudaStream_t stream) {
  auto kernel = gemv_q4_kernel<MT, EXCH, ZM, VEC>;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBudget);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(s.tiles, s.tpc)), static_cast<unsigned>(s.splits), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = s.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(s.splits);
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, gp);
}

template <int MT, bool EXCH, int ZM>
cudaError_t launch_vec(const GemvShape& s, const GemvParams& gp, cudaStream_t stream) {
  if (EXCH && s.vec) return launch_variant<MT, EXCH, ZM, true>(s, gp, stream);
  return launch_variant<MT, EXCH, ZM, false>(s, gp, stream);
}

}  // namespace

bool gemv_supported(const Problem& p) {
  if (!(p.f16 && p.bits == 4 && p.M >= 1 && p.M <= 16 && p.bs >= 32 && (p.bs & (p.bs - 1)) == 0 &&
        p.K % kRegionK == 0 && p.K % p.bs == 0 && p.K < (1ll << 30) && p.N < (1ll << 30) &&
        (reinterpret_cast<uintptr_t>(p.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 &&
        (reinterpret_cast<uintptr_t>(p.scales) % 2) == 0))
    return false;
  return gemv_shape(p).smem <= static_cast<size_t>(kSmemBudget);
}

uint64_t gemv_workspace_bytes(const Problem&) { return 0; }

cudaError_t launch_gemv(const Problem& p, void* /*workspace*/, cudaStream_t stream) {
  if (p.N == 0 || p.M == 0) return cudaSuccess;
  const GemvShape s = gemv_shape(p);
  GemvParams gp{};
  gp.x = static_cast<const __half*>(p.a);
  gp.b = p.b;
  gp.scales = static_cast<const __half*>(p.scales);
  gp.zp = p.zp_ptr;
  gp.bias = static_cast<const __half*>(p.bias);
  gp.y = static_cast<__half*>(p.y);
  gp.ldy = p.ldy;
  gp.M = static_cast<int>(p.M);
  gp.K = static_cast<int>(p.K);
  gp.N = static_cast<int>(p.N);
  gp.kb = static_cast<int>(p.kb);
  gp.zp_kind = p.zp;
  gp.log2_bs = ilog2(p.bs);
  gp.groups = s.groups;
  gp.group_regions = s.group_regions;
  gp.splits = s.splits;
  gp.tpc = s.tpc;
  gp.xrow_bytes = s.xrow_bytes;
  gp.smem_x_bytes = s.smem_x_bytes;
  gp.nb_chunk = s.nb_chunk;
  gp.win_stride = s.win_stride;
  const bool exch = p.bs == 32;
  const int zm = p.zp == kZpNone ? kModeDefault : (p.zp == kZpPacked ? kModeInt : kModeFloat);
#define XRGPU_GEMV_CASE(MT, EX, ZM) \
  if (s.mt == MT && exch == EX && zm == ZM) return launch_vec<MT, EX, ZM>(s, gp, stream);
  XRGPU_GEMV_CASE(1, true, kModeDefault)
  XRGPU_GEMV_CASE(1, true, kModeInt)
  XRGPU_GEMV_CASE(1, true, kModeFloat)
  XRGPU_GEMV_CASE(1, false, kModeDefault)
  XRGPU_GEMV_CASE(1, false, kModeInt)
  XRGPU_GEMV_CASE(1, false, kModeFloat)
  XRGPU_GEMV_CASE(2, true, kModeDefault)
  XRGPU_GEMV_CASE(2, true, kModeInt)
  XRGPU_GEMV_CASE(2, true, kModeFloat)
  XRGPU_GEMV_CASE(2, false, kModeDefault)
  XRGPU_GEMV_CASE(2, false, kModeInt)
  XRGPU_GEMV_CASE(2, false, kModeFloat)
#undef XRGPU_GEMV_CASE
  return cudaErrorInvalidValue;
}

}  // namespace xrgpu
