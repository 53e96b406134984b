// 4-bit MatMulNBits decode GEMV for sm_100a (M <= 16 rows, float16 activations).
//
// The kernel streams the packed weights once, unpacks nibbles to float16 in registers and
// multiplies them on the tensor cores (mma.sync m16n8k16, float32 accumulation). Exactness:
//   * each nibble becomes float16 (q - z) (or q) exactly: LOP3 places it in the mantissa of
//     1024.0 (0x6400), then one float16 subtract / fused multiply-add removes the offset;
//   * the tensor core multiplies exact float16 operands and accumulates in float32;
//   * the per-block scale (and a float zero point, via sum(q*x) - z*sum(x)) is applied in
//     float32 once per block, so (q - z) * s is never rounded to float16.
// This restates packedMatmul/nbitWeight (complex_kernel.glsl:80,83) with a different, exact
// association: sum_b s_b * sum_{k in b} (q_k - z_b) * x_k.
//
// Work decomposition: a CTA owns 16 output columns and a contiguous range of 64-wide k
// "regions" (split-K across CTAs, within a CTA across its 4 warps). Within a warp, lane
// (g = lane/4, c = lane%4) handles columns n0+g and n0+g+8; each quad reads one 32-byte
// sector per column per region (8 bytes per lane). Split-K partial sums are combined in a
// fixed order by the last CTA of each column tile (deterministic).
#include <cuda_fp16.h>

#include <algorithm>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kCols = 16;
constexpr int kRegionK = 64;            // k per region: 32 bytes of one column
constexpr int kSmemBudget = 40 * 1024;  // dynamic shared memory per CTA for staged activations
constexpr int kUnroll = 4;

struct GemvParams {
  const __half* x;        // [M, K]
  const uint8_t* b;       // [N, K/2]
  const __half* scales;   // [N, kb]
  const void* zp;         // zero points (kind zp_kind) or nullptr
  const __half* bias;     // [N] or nullptr
  __half* y;              // [M, ldy]
  float* partial;         // [splits, M, N] (splits > 1)
  unsigned* counters;     // [tiles] (splits > 1)
  int64_t ldy;
  int M, K, N, bs, kb, zp_kind, regions, splits;
};

// Per-region k offset (within the 64-wide region) of the 8 consecutive k values that lane
// c holds in half h. With bs == 32 ("exchange"): half h is block h of the region and lanes
// hold words in the order 0, 2, 1, 3 after the pair exchange. Otherwise lane c's 8 bytes
// are k in [16c, 16c+16): half h is [16c + 8h, 16c + 8h + 8).
__device__ __forceinline__ int koff(bool exch, int h, int c) {
  if (exch) {
    const int perm = (c == 1) ? 2 : (c == 2) ? 1 : c;
    return 32 * h + 8 * perm;
  }
  return 16 * c + 8 * h;
}

// Nibbles of one 32-bit word (k0..k7, k_i in bits 4i..4i+3) as float16 pairs
// q[0] = (k0,k4), q[1] = (k1,k5), q[2] = (k2,k6), q[3] = (k3,k7), each minus z0.
// c_lo = (1024+z0, 1024+z0); c_hi = (-(64+z0), -(64+z0)).
__device__ __forceinline__ void unpack8(uint32_t w, uint32_t c_lo, uint32_t c_hi, uint32_t (&q)[4]) {
  constexpr uint32_t kLo = 0x000F000Fu, kHi = 0x00F000F0u, kExp = 0x64006400u, kSixteenth = 0x2C002C00u;
  const uint32_t w8 = w >> 8;
  q[0] = hsub2_u32(lop3_and_or(w, kLo, kExp), c_lo);
  q[1] = hfma2_u32(lop3_and_or(w, kHi, kExp), kSixteenth, c_hi);
  q[2] = hsub2_u32(lop3_and_or(w8, kLo, kExp), c_lo);
  q[3] = hfma2_u32(lop3_and_or(w8, kHi, kExp), kSixteenth, c_hi);
}

__device__ __forceinline__ float zero_point_at(const GemvParams& p, int col, int blk) {
  switch (p.zp_kind) {
    case kZpF32: return reinterpret_cast<const float*>(p.zp)[static_cast<int64_t>(col) * p.kb + blk];
    case kZpF16: return __half2float(reinterpret_cast<const __half*>(p.zp)[static_cast<int64_t>(col) * p.kb + blk]);
    case kZpPacked: {
      const int64_t stride = (p.kb * 4 + 7) / 8;
      const uint32_t byte = reinterpret_cast<const uint8_t*>(p.zp)[static_cast<int64_t>(col) * stride + blk / 2];
      return static_cast<float>((byte >> (4 * (blk & 1))) & 15u);
    }
    default: return 8.f;
  }
}

// MT: 8-row tiles of activations (M <= 8*MT). EXCH: block_size == 32. ZPX: zero points
// given (applied in float32 via sum(x)); otherwise the default zero point 8 is folded
// into the float16 unpack.
template <int MT, bool EXCH, bool ZPX>
__global__ void __launch_bounds__(kThreads) gemv_q4_kernel(GemvParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float red[kWarps][kCols][8 * MT];
  __shared__ int s_last;

  constexpr int MP = 8 * MT;
  const int M = p.M;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int n0 = tile * kCols;
  const int r0 = static_cast<int>(static_cast<int64_t>(p.regions) * split / p.splits);
  const int r1 = static_cast<int>(static_cast<int64_t>(p.regions) * (split + 1) / p.splits);
  const int nreg = r1 - r0;

  // ---- stage this CTA's activations, permuted into mma B-fragment order, plus sum(x).
  uint4* xs = reinterpret_cast<uint4*>(smem_raw);                          // [nreg][2][M][4]
  float* xsum = reinterpret_cast<float*>(xs + static_cast<size_t>(nreg) * 2 * M * 4);  // [nreg][2][MP]
  for (int e = threadIdx.x; e < nreg * 2 * MP; e += kThreads) {
    const int m = e % MP, t = e / MP, h = t & 1, reg = t >> 1;
    float sum = 0.f;
    if (m < M) {
      const __half* xrow = p.x + static_cast<int64_t>(m) * p.K + static_cast<int64_t>(r0 + reg) * kRegionK;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 v = *reinterpret_cast<const uint4*>(xrow + koff(EXCH, h, c));
        uint4 o;
        o.x = prmt(v.x, v.z, 0x5410);  // (x0, x4)
        o.y = prmt(v.y, v.w, 0x5410);  // (x2, x6)
        o.z = prmt(v.x, v.z, 0x7632);  // (x1, x5)
        o.w = prmt(v.y, v.w, 0x7632);  // (x3, x7)
        xs[((reg * 2 + h) * M + m) * 4 + c] = o;
        if (ZPX) {
          const __half2* hv = reinterpret_cast<const __half2*>(&v);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(hv[i]);
            sum += f.x + f.y;
          }
        }
      }
    }
    if (ZPX) xsum[(reg * 2 + h) * MP + m] = sum;
  }
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int wr0 = nreg * warp / kWarps, wr1 = nreg * (warp + 1) / kWarps;
  const int colA = min(n0 + g, p.N - 1), colB = min(n0 + g + 8, p.N - 1);
  const int64_t colbytes = static_cast<int64_t>(p.K) / 2;
  const uint8_t* bA = p.b + colA * colbytes + static_cast<int64_t>(r0) * 32 + c * 8;
  const uint8_t* bB = p.b + colB * colbytes + static_cast<int64_t>(r0) * 32 + c * 8;
  const __half* sA = p.scales + static_cast<int64_t>(colA) * p.kb;
  const __half* sB = p.scales + static_cast<int64_t>(colB) * p.kb;

  // Unpack constants: subtract 1024 (and the default zero point 8 when no zero points).
  const uint32_t c_lo = ZPX ? 0x64006400u : 0x64086408u;  // 1024 or 1032
  const uint32_t c_hi = ZPX ? 0xD400D400u : 0xD480D480u;  // -64 or -72

  float y[MT][4];
  float d[MT][4];
  float xacc[MT][2];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
#pragma unroll
    for (int i = 0; i < 4; ++i) y[t][i] = d[t][i] = 0.f;
    xacc[t][0] = xacc[t][1] = 0.f;
  }

  // Applies scale (and zero point) of block `blk` to the accumulated block sums d.
  auto finish_block = [&](int blk) {
    const float scA = __half2float(sA[blk]), scB = __half2float(sB[blk]);
    float zA = 0.f, zB = 0.f;
    if (ZPX) {
      zA = zero_point_at(p, colA, blk);
      zB = zero_point_at(p, colB, blk);
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      float d0 = d[t][0], d1 = d[t][1], d2 = d[t][2], d3 = d[t][3];
      if (ZPX) {
        d0 = fmaf(-zA, xacc[t][0], d0);
        d1 = fmaf(-zA, xacc[t][1], d1);
        d2 = fmaf(-zB, xacc[t][0], d2);
        d3 = fmaf(-zB, xacc[t][1], d3);
        xacc[t][0] = xacc[t][1] = 0.f;
      }
      y[t][0] = fmaf(scA, d0, y[t][0]);
      y[t][1] = fmaf(scA, d1, y[t][1]);
      y[t][2] = fmaf(scB, d2, y[t][2]);
      y[t][3] = fmaf(scB, d3, y[t][3]);
      d[t][0] = d[t][1] = d[t][2] = d[t][3] = 0.f;
    }
  };

  // One region: 64 k of columns colA/colB, words already loaded.
  auto do_region = [&](int reg, uint2 wa, uint2 wb) {
    uint32_t a_h[2], b_h[2];  // [half] word of column A / B
    if (EXCH) {
      const bool upper = (c & 2) != 0;
      const uint32_t sa = upper ? wa.x : wa.y, sb = upper ? wb.x : wb.y;
      const uint32_t ra = __shfl_xor_sync(0xffffffffu, sa, 2), rb = __shfl_xor_sync(0xffffffffu, sb, 2);
      a_h[0] = upper ? ra : wa.x;
      a_h[1] = upper ? wa.y : ra;
      b_h[0] = upper ? rb : wb.x;
      b_h[1] = upper ? wb.y : rb;
    } else {
      a_h[0] = wa.x; a_h[1] = wa.y;
      b_h[0] = wb.x; b_h[1] = wb.y;
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t qa[4], qb[4];
      unpack8(a_h[h], c_lo, c_hi, qa);
      unpack8(b_h[h], c_lo, c_hi, qb);
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const int m = g + 8 * t;
        uint4 xf = make_uint4(0u, 0u, 0u, 0u);
        if (m < M) xf = xs[((reg * 2 + h) * M + m) * 4 + c];
        mma_16816(d[t], qa[0], qb[0], qa[2], qb[2], xf.x, xf.y);
        mma_16816(d[t], qa[1], qb[1], qa[3], qb[3], xf.z, xf.w);
        if (ZPX) {
          const float2 s2 = *reinterpret_cast<const float2*>(&xsum[(reg * 2 + h) * MP + 8 * t + 2 * c]);
          xacc[t][0] += s2.x;
          xacc[t][1] += s2.y;
        }
      }
      if (EXCH) finish_block((r0 + reg) * 2 + h);
    }
    if (!EXCH) {
      const int kend = (r0 + reg + 1) * kRegionK;
      if (kend % p.bs == 0 || reg + 1 == wr1) finish_block(((r0 + reg) * kRegionK) / p.bs);
    }
  };

  int reg = wr0;
  for (; reg + kUnroll <= wr1; reg += kUnroll) {
    uint2 wa[kUnroll], wb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      wa[u] = ldg_stream_u2(bA + static_cast<int64_t>(reg + u) * 32);
      wb[u] = ldg_stream_u2(bB + static_cast<int64_t>(reg + u) * 32);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) do_region(reg + u, wa[u], wb[u]);
  }
  for (; reg < wr1; ++reg) {
    const uint2 wa = ldg_stream_u2(bA + static_cast<int64_t>(reg) * 32);
    const uint2 wb = ldg_stream_u2(bB + static_cast<int64_t>(reg) * 32);
    do_region(reg, wa, wb);
  }

  // ---- reduce the 4 warps' partial sums (fixed order), then across split-K CTAs.
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    red[warp][g][8 * t + 2 * c] = y[t][0];
    red[warp][g][8 * t + 2 * c + 1] = y[t][1];
    red[warp][g + 8][8 * t + 2 * c] = y[t][2];
    red[warp][g + 8][8 * t + 2 * c + 1] = y[t][3];
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < kCols * M; idx += kThreads) {
    const int col = idx % kCols, m = idx / kCols, n = n0 + col;
    if (n >= p.N) continue;
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) v += red[w][col][m];
    if (p.splits == 1) {
      if (p.bias) v += __half2float(p.bias[n]);
      p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(v);
    } else {
      __stcg(&p.partial[(static_cast<int64_t>(split) * M + m) * p.N + n], v);
    }
  }
  if (p.splits == 1) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&p.counters[tile], 1u) == static_cast<unsigned>(p.splits - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < kCols * M; idx += kThreads) {
    const int col = idx % kCols, m = idx / kCols, n = n0 + col;
    if (n >= p.N) continue;
    float v = 0.f;
    for (int s = 0; s < p.splits; ++s) v += __ldcg(&p.partial[(static_cast<int64_t>(s) * M + m) * p.N + n]);
    if (p.bias) v += __half2float(p.bias[n]);
    p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2half_rn(v);
  }
  if (threadIdx.x == 0) p.counters[tile] = 0u;  // leave the workspace zero-filled
}

struct GemvShape {
  int tiles, splits, mt;
  size_t smem;
  uint64_t partial_bytes, counter_bytes;
};

GemvShape gemv_shape(const Problem& p) {
  GemvShape s{};
  const int regions = static_cast<int>(p.K / kRegionK);
  s.tiles = static_cast<int>(ceil_div(p.N, kCols));
  s.mt = p.M <= 8 ? 1 : 2;
  const int mp = 8 * s.mt;
  const size_t per_region = static_cast<size_t>(2) * p.M * 4 * 16 + static_cast<size_t>(2) * mp * 4;
  const int target_ctas = device_sm_count() * 4;
  int splits = static_cast<int>(ceil_div(target_ctas, s.tiles));
  splits = std::min(splits, std::max(1, regions / kWarps));
  const int smem_splits = static_cast<int>(ceil_div(static_cast<int64_t>(regions) * per_region, kSmemBudget));
  splits = std::max(splits, smem_splits);
  splits = std::max(1, std::min(splits, regions));
  s.splits = splits;
  s.smem = per_region * static_cast<size_t>(ceil_div(regions, splits));
  s.partial_bytes = splits > 1 ? align_up(static_cast<uint64_t>(splits) * p.M * p.N * 4, 256) : 0;
  s.counter_bytes = splits > 1 ? align_up(static_cast<uint64_t>(s.tiles) * 4, 256) : 0;
  return s;
}

template <int MT, bool EXCH, bool ZPX>
cudaError_t launch_variant(const GemvShape& s, const GemvParams& gp, cudaStream_t stream) {
  auto kernel = gemv_q4_kernel<MT, EXCH, ZPX>;
  if (s.smem > 32 * 1024) {  // static + dynamic may pass the 48 KB default: opt in
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s.smem));
    if (e != cudaSuccess) return e;
  }
  kernel<<<dim3(s.tiles, s.splits), kThreads, s.smem, stream>>>(gp);
  return cudaGetLastError();
}

}  // namespace

bool gemv_supported(const Problem& p) {
  return p.f16 && p.bits == 4 && p.M >= 1 && p.M <= 16 && p.bs >= 32 && (p.bs & (p.bs - 1)) == 0 &&
         p.K % kRegionK == 0 && p.K % p.bs == 0 && p.K / kRegionK < (1 << 30) && p.N < (1 << 30) &&
         (reinterpret_cast<uintptr_t>(p.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 &&
         (reinterpret_cast<uintptr_t>(p.scales) % 2) == 0;
}

uint64_t gemv_workspace_bytes(const Problem& p) {
  if (!gemv_supported(p)) return 0;
  const GemvShape s = gemv_shape(p);
  return s.partial_bytes + s.counter_bytes;
}

cudaError_t launch_gemv(const Problem& p, void* workspace, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
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
  gp.bs = static_cast<int>(p.bs);
  gp.kb = static_cast<int>(p.kb);
  gp.zp_kind = p.zp;
  gp.regions = static_cast<int>(p.K / kRegionK);
  gp.splits = s.splits;
  if (s.splits > 1) {
    if (!workspace) return cudaErrorInvalidValue;
    gp.partial = static_cast<float*>(workspace);
    gp.counters = reinterpret_cast<unsigned*>(static_cast<char*>(workspace) + s.partial_bytes);
  }
  const bool exch = p.bs == 32, zpx = p.zp != kZpNone;
#define XRGPU_GEMV_CASE(MT, EX, ZX) \
  if (s.mt == MT && exch == EX && zpx == ZX) return launch_variant<MT, EX, ZX>(s, gp, stream);
  XRGPU_GEMV_CASE(1, true, false)
  XRGPU_GEMV_CASE(1, true, true)
  XRGPU_GEMV_CASE(1, false, false)
  XRGPU_GEMV_CASE(1, false, true)
  XRGPU_GEMV_CASE(2, true, false)
  XRGPU_GEMV_CASE(2, true, true)
  XRGPU_GEMV_CASE(2, false, false)
  XRGPU_GEMV_CASE(2, false, true)
#undef XRGPU_GEMV_CASE
  return cudaErrorInvalidValue;
}

}  // namespace xrgpu
