// 4-bit MatMulNBits decode GEMV for sm_100a (M <= 16 rows, float16 activations).
//
// Decode is a pure stream of the packed weights (each byte is used once), so the kernel is
// built to spend as few instructions per weight byte as possible while keeping enough bytes in
// flight to saturate HBM:
//   * weights go straight from global memory into registers with 128-bit streaming loads
//     (L1 bypassed), one iteration of prefetch per warp; no shared-memory staging;
//   * each 32-bit word (8 codes) is dequantized in registers to four float16x2 values
//     w = (q - z) * s: LOP3 drops a nibble into the mantissa of 1024.0 (0x6400), one float16
//     subtract / fused multiply-add removes 1024 + z exactly (z an integer: the default 8 or a
//     packed zero point), one float16 multiply applies the block scale (w is the float16
//     nearest to the reference's float32 weight (q - z) * s, complex_kernel.glsl:80);
//   * the tensor cores (mma.sync m16n8k16) multiply the weights by the activations and
//     accumulate in float32 over the warp's whole K slice (packedMatmul, complex_kernel.glsl:83);
//     activations are read from L1 in natural order and paired with the nibble order by PRMT.
//
// Decomposition. A warp owns 16 output columns (lane g = lane/4 handles columns n0+g and
// n0+g+8) and a contiguous slice of 128-wide k iterations; in an iteration lane c = lane%4
// holds 16 bytes of each of its columns, the 32 codes k in [32c, 32c+32), which lie in a single
// quantization block for block sizes >= 32. The tile's slices are spread over the warps of a
// CTA (tpc tiles x spc slices = 8 warps) and, for short K or few columns, over the CTAs of a
// thread-block cluster; partial sums are combined in a fixed order through shared memory and
// distributed shared memory, so results are deterministic and no global workspace is used.
#include <cuda_fp16.h>

#include <algorithm>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kCols = 16;          // output columns per warp tile
constexpr int kIterK = 128;        // k per iteration: 64 bytes of a column, 16 per lane
constexpr int kMaxSplits = 8;      // portable cluster size
constexpr int kMaxSlices = 64;     // slices per tile (spc * splits)

enum ZpMode : int { kZDefault = 0, kZPacked = 1, kZFloat = 2 };

struct GemvParams {
  const __half* x;        // [M, K]
  const uint8_t* b;       // [N, K/2]
  const __half* scales;   // [N, kb]
  const void* zp;         // zero points or nullptr
  const __half* bias;     // [N] or nullptr
  __half* y;              // [M, ldy]
  int64_t ldy;
  int M, K, N, kb, log2_bs;
  int zp_f32;             // float zero points stored as float32 (else float16)
  int zp_row_bytes;       // packed zero points: bytes per column
  int iters;              // full 128-wide k iterations
  int tail;               // 1 when a final 64-wide region remains (K % 128 == 64)
  int tpc, spc, splits;   // tiles per CTA, slices per CTA (tpc * spc == 8), CTAs per cluster
};

// 16-byte streaming load of read-only weights (L1 bypassed, 256-byte L2 fetch).
__device__ __forceinline__ uint4 ldg_w128(const void* ptr) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(ptr));
  return v;
}
__device__ __forceinline__ uint2 ldg_w64(const void* ptr) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(ptr));
  return v;
}
// 16-byte activation load (cached in L1: every warp of the SM reads the same rows). Volatile
// with a memory clobber so that it stays after griddepcontrol.wait.
__device__ __forceinline__ uint4 ldg_x128(const void* ptr) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr)
               : "memory");
  return v;
}

__device__ __forceinline__ void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
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

// Quantization metadata of one (column, block), as loaded: the float16 scale in the low half
// of `s`, the zero point in `z` (an integer code for packed / default zero points, the float16
// bits of a float zero point otherwise).
struct BlockMeta {
  uint32_t s, z;
};

// `srow` = col * kb, `zrow` = col * zp_row_bytes (32-bit: N * kb < 2^31 is checked by the planner).
template <int ZM>
__device__ __forceinline__ BlockMeta block_meta(const GemvParams& p, int srow, int zrow, int blk) {
  BlockMeta m;
  const int idx = srow + blk;
  m.s = __half_as_ushort(__ldg(p.scales + idx));
  m.z = 8u;
  if (ZM == kZPacked) {
    const uint32_t byte = __ldg(reinterpret_cast<const uint8_t*>(p.zp) + zrow + (blk >> 1));
    m.z = (byte >> ((blk & 1) * 4)) & 15u;
  }
  if (ZM == kZFloat) {
    const __half zh = p.zp_f32 ? __float2half_rn(__ldg(reinterpret_cast<const float*>(p.zp) + idx))
                               : __ldg(reinterpret_cast<const __half*>(p.zp) + idx);
    m.z = __half_as_ushort(zh);
  }
  return m;
}

// Dequantization constants: float16x2 scale (s, s); for integer zero points
// zlo = (1024 + z, 1024 + z), zhi = (-(64 + z), -(64 + z)) (64 + z < 128 has ulp 1/16); for float
// zero points zlo = (1024, 1024), zhi = (-64, -64) and zf = (z, z) is subtracted after.
struct BlockConsts {
  uint32_t s2, zlo, zhi, zf;
};

template <int ZM>
__device__ __forceinline__ BlockConsts block_consts(BlockMeta m) {
  BlockConsts bc;
  bc.s2 = m.s * 0x00010001u;
  const uint32_t z = ZM == kZFloat ? 0u : m.z;
  bc.zf = ZM == kZFloat ? m.z * 0x00010001u : 0u;
  bc.zlo = z * 0x00010001u + 0x64006400u;
  bc.zhi = z * 0x00100010u + 0xD400D400u;
  return bc;
}

// One 32-bit word (codes k0..k7, k_i in bits 4i..4i+3) to float16x2 weights in the pair order
// q[0] = (k0,k4), q[1] = (k1,k5), q[2] = (k2,k6), q[3] = (k3,k7).
template <int ZM>
__device__ __forceinline__ void dequant_word(uint32_t w, const BlockConsts& bc, uint32_t (&q)[4]) {
  constexpr uint32_t kLo = 0x000F000Fu, kHi = 0x00F000F0u, kExp = 0x64006400u, kSixteenth = 0x2C002C00u;
  const uint32_t w8 = w >> 8;
  uint32_t d0 = hsub2_u32(lop3_and_or(w, kLo, kExp), bc.zlo);
  uint32_t d1 = hfma2_u32(lop3_and_or(w, kHi, kExp), kSixteenth, bc.zhi);
  uint32_t d2 = hsub2_u32(lop3_and_or(w8, kLo, kExp), bc.zlo);
  uint32_t d3 = hfma2_u32(lop3_and_or(w8, kHi, kExp), kSixteenth, bc.zhi);
  if (ZM == kZFloat) {
    d0 = hsub2_u32(d0, bc.zf);
    d1 = hsub2_u32(d1, bc.zf);
    d2 = hsub2_u32(d2, bc.zf);
    d3 = hsub2_u32(d3, bc.zf);
  }
  q[0] = hmul2_u32(d0, bc.s2);
  q[1] = hmul2_u32(d1, bc.s2);
  q[2] = hmul2_u32(d2, bc.s2);
  q[3] = hmul2_u32(d3, bc.s2);
}

// Words wa[i], wb[i] (columns A and B, codes k0 + 8 i .. k0 + 8 i + 7) times the activations:
// lane (g, c) supplies the B fragments of activation row g (and g + 8 when MT == 2), read in
// natural order and paired as (x0,x4), (x2,x6) / (x1,x5), (x3,x7) to match the nibble pairs.
template <int MT, int ZM, int NW>
__device__ __forceinline__ void mma_words(float (&acc)[MT][4], const uint32_t* wa, const uint32_t* wb, BlockMeta ma,
                                          BlockMeta mb, const __half* x0, const __half* x1, bool row0, bool row1) {
  const BlockConsts ca = block_consts<ZM>(ma), cb = block_consts<ZM>(mb);
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    uint4 xv[MT];
    // Lanes whose activation row is >= M read row 0 instead: B column g only feeds output
    // row g, which is never stored, so no predication is needed.
    xv[0] = ldg_x128(x0 + 8 * i);
    if (MT == 2) xv[MT - 1] = ldg_x128(x1 + 8 * i);
    uint32_t qa[4], qb[4];
    dequant_word<ZM>(wa[i], ca, qa);
    dequant_word<ZM>(wb[i], cb, qb);
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const uint4 v = xv[t];
      mma_acc(acc[t], qa[0], qb[0], qa[2], qb[2], prmt(v.x, v.z, 0x5410), prmt(v.y, v.w, 0x5410));
      mma_acc(acc[t], qa[1], qb[1], qa[3], qb[3], prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x7632));
    }
  }
}

// MT: 8-row activation tiles (M <= 8 MT). ZM: zero-point mode.
template <int MT, int ZM>
__global__ void __launch_bounds__(kThreads, MT == 1 ? 4 : 3) gemv_q4_kernel(const __grid_constant__ GemvParams p) {
  __shared__ float red[kWarps][kCols * 8 * MT];
  __shared__ float part[kWarps][kCols * 8 * MT];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int t_local = warp % p.tpc, s_local = warp / p.tpc;
  const int n0 = (blockIdx.x * p.tpc + t_local) * kCols;
  const int S = p.spc * p.splits;
  const int slice = static_cast<int>(blockIdx.y) * p.spc + s_local;
  const int it0 = static_cast<int>(static_cast<int64_t>(p.iters) * slice / S);
  const int it1 = static_cast<int>(static_cast<int64_t>(p.iters) * (slice + 1) / S);
  const bool do_tail = p.tail && slice == S - 1;
  const bool tile_ok = n0 < p.N;
  const int colA = min(n0 + g, p.N - 1), colB = min(n0 + g + 8, p.N - 1);
  // 32-bit offsets (N * K / 2 < 2^31 and N * kb < 2^31 are checked by the planner).
  const uint8_t* wA = p.b + (colA * (p.K / 2) + 16 * c);
  const uint8_t* wB = p.b + (colB * (p.K / 2) + 16 * c);
  const int sA = colA * p.kb, sB = colB * p.kb, zA = colA * p.zp_row_bytes, zB = colB * p.zp_row_bytes;
  const bool row0 = g < p.M, row1 = g + 8 < p.M;
  const __half* xr0 = p.x + static_cast<int64_t>(row0 ? g : 0) * p.K + 32 * c;
  const __half* xr1 = p.x + static_cast<int64_t>(row1 ? g + 8 : 0) * p.K + 32 * c;

  // Programmatic dependent launch: the next kernel in the stream may start (and prefetch its
  // weights) while this one runs. Weights, scales and zero points are read before
  // griddepcontrol.wait; the activations and the output only after it.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  float acc[MT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[t][i] = 0.f;

  // Block of lane c's codes in iteration it: (128 it + 32 c) / bs.
  auto blk_of = [&](int it) { return (it * kIterK + 32 * c) >> p.log2_bs; };
  // Two register slots alternate (2-way unrolled loop): the weights of iteration it + 1 are in
  // flight while iteration it is computed, with no copies between slots.
  uint4 wa[2], wb[2];
  BlockMeta ma[2], mb[2];
  auto fetch = [&](int it, int slot) {
    wa[slot] = ldg_w128(wA + it * 64);
    wb[slot] = ldg_w128(wB + it * 64);
    const int blk = blk_of(it);
    ma[slot] = block_meta<ZM>(p, sA, zA, blk);
    mb[slot] = block_meta<ZM>(p, sB, zB, blk);
  };
  if (tile_ok && it0 < it1) fetch(it0, 0);
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (tile_ok) {
    auto compute = [&](int it, int slot) {
      const uint32_t a[4] = {wa[slot].x, wa[slot].y, wa[slot].z, wa[slot].w};
      const uint32_t b[4] = {wb[slot].x, wb[slot].y, wb[slot].z, wb[slot].w};
      mma_words<MT, ZM, 4>(acc, a, b, ma[slot], mb[slot], xr0 + it * kIterK, xr1 + it * kIterK, row0, row1);
    };
    int it = it0;
    for (; it + 2 <= it1; it += 2) {
      fetch(it + 1, 1);
      compute(it, 0);
      if (it + 2 < it1) fetch(it + 2, 0);
      compute(it + 1, 1);
    }
    if (it < it1) compute(it, 0);
    if (do_tail) {
      // Final 64-wide region: lane c holds 8 bytes per column, codes [16c, 16c+16) of it.
      const int kr = p.iters * kIterK;
      const uint2 a2 = ldg_w64(wA - 16 * c + kr / 2 + 8 * c);
      const uint2 b2 = ldg_w64(wB - 16 * c + kr / 2 + 8 * c);
      const int blk = (kr + 16 * c) >> p.log2_bs;
      const BlockMeta ma = block_meta<ZM>(p, sA, zA, blk), mb = block_meta<ZM>(p, sB, zB, blk);
      const uint32_t wa[2] = {a2.x, a2.y}, wb[2] = {b2.x, b2.y};
      mma_words<MT, ZM, 2>(acc, wa, wb, ma, mb, xr0 - 32 * c + kr + 16 * c, xr1 - 32 * c + kr + 16 * c, row0, row1);
    }
  }

  // ---- reduce: the slices of each tile in this CTA (fixed order), then the cluster's CTAs.
  // d0 = (column g, row 2c), d1 = (g, 2c+1), d2 = (g+8, 2c), d3 = (g+8, 2c+1), per 8-row tile t.
  constexpr int kTileOut = kCols * 8 * MT;
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    red[warp][g * 8 * MT + 8 * t + 2 * c] = acc[t][0];
    red[warp][g * 8 * MT + 8 * t + 2 * c + 1] = acc[t][1];
    red[warp][(g + 8) * 8 * MT + 8 * t + 2 * c] = acc[t][2];
    red[warp][(g + 8) * 8 * MT + 8 * t + 2 * c + 1] = acc[t][3];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.tpc * kTileOut; idx += kThreads) {
    const int t = idx / kTileOut, rem = idx - t * kTileOut;
    float v = 0.f;
    for (int sl = 0; sl < p.spc; ++sl) v += red[t + sl * p.tpc][rem];
    part[t][rem] = v;
  }
  if (p.splits > 1) cluster_sync();
  else __syncthreads();
  if (blockIdx.y == 0) {
    for (int idx = threadIdx.x; idx < p.tpc * kTileOut; idx += kThreads) {
      const int t = idx / kTileOut, rem = idx - t * kTileOut;
      const int col = rem / (8 * MT), m = rem - col * (8 * MT);
      const int n = (blockIdx.x * p.tpc + t) * kCols + col;
      if (m < p.M && n < p.N) {
        float v = part[t][rem];
        for (int s = 1; s < p.splits; ++s) v += ld_dsmem_f32(&part[t][rem], static_cast<unsigned>(s));
        if (p.bias) v += __half2float(p.bias[n]);
        p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(v);
      }
    }
  }
  if (p.splits > 1) cluster_sync();  // keep every CTA's shared memory alive until it is read
}

struct GemvShape {
  int tiles, tpc, spc, splits, mt;
};

int ilog2(int64_t v) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= v) ++r;
  return r;
}

// Slices per tile: about one warp per resident warp slot of the GPU (32 per SM), a power of
// two, at most one slice per 128-wide iteration, at most 8 warps x 8 cluster CTAs.
GemvShape gemv_shape(const Problem& p) {
  GemvShape s{};
  s.tiles = static_cast<int>(ceil_div(p.N, kCols));
  s.mt = p.M <= 8 ? 1 : 2;
  const int iters = static_cast<int>(p.K / kIterK);
  const int64_t capacity = static_cast<int64_t>(device_sm_count()) * 32;
  int S = 1;
  while (S * 2 <= kMaxSlices && static_cast<int64_t>(s.tiles) * S * 2 <= capacity && S * 2 <= std::max(1, iters)) S *= 2;
  s.spc = std::min(S, kWarps);
  s.splits = S / s.spc;
  s.tpc = kWarps / s.spc;
  return s;
}

template <int MT, int ZM>
cudaError_t launch_variant(const GemvShape& s, const GemvParams& gp, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(s.tiles, s.tpc)), static_cast<unsigned>(s.splits), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
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
  return cudaLaunchKernelEx(&cfg, gemv_q4_kernel<MT, ZM>, gp);
}

}  // namespace

bool gemv_supported(const Problem& p) {
  return p.f16 && p.bits == 4 && p.M >= 1 && p.M <= 16 && p.bs >= 32 && (p.bs & (p.bs - 1)) == 0 &&
         p.K % 64 == 0 && p.K % p.bs == 0 && p.N * (p.K / 2) < (1ll << 31) && p.N * p.kb < (1ll << 31) &&
         (reinterpret_cast<uintptr_t>(p.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(p.scales) % 2) == 0;
}

uint64_t gemv_workspace_bytes(const Problem&) { return 0; }

cudaError_t launch_gemv(const Problem& p, void* /*workspace*/, cudaStream_t stream) {
  if (p.N == 0 || p.M == 0) return cudaSuccess;
  if (gemv_staged_supported(p)) return launch_gemv_staged(p, stream);
  if (gemv_mr_supported(p)) return launch_gemv_mr(p, stream);
  if (gemv_m1_supported(p)) return launch_gemv_m1(p, stream);
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
  gp.log2_bs = ilog2(p.bs);
  gp.zp_f32 = p.zp == kZpF32;
  gp.zp_row_bytes = static_cast<int>((p.kb + 1) / 2);
  gp.iters = static_cast<int>(p.K / kIterK);
  gp.tail = static_cast<int>((p.K % kIterK) / 64);
  gp.tpc = s.tpc;
  gp.spc = s.spc;
  gp.splits = s.splits;
  const int zm = p.zp == kZpNone ? kZDefault : (p.zp == kZpPacked ? kZPacked : kZFloat);
  if (s.mt == 1) {
    if (zm == kZDefault) return launch_variant<1, kZDefault>(s, gp, stream);
    if (zm == kZPacked) return launch_variant<1, kZPacked>(s, gp, stream);
    return launch_variant<1, kZFloat>(s, gp, stream);
  }
  if (zm == kZDefault) return launch_variant<2, kZDefault>(s, gp, stream);
  if (zm == kZPacked) return launch_variant<2, kZPacked>(s, gp, stream);
  return launch_variant<2, kZFloat>(s, gp, stream);
}

}  // namespace xrgpu
