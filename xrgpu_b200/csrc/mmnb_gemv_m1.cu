// 4-bit MatMulNBits decode GEMV for a single activation row (M == 1), sm_100a.
//
// With one activation row the whole cost is streaming the packed weights, so the inner loop is
// cut down to the fewest instructions per weight byte:
//   * a 32-bit word of 8 codes becomes four float16x2 operands with four ANDs and one shift
//     and nothing else: (w & 0x000F000F) is the pair (q0, q4) as float16 subnormals q * 2^-24,
//     (w & 0x00F000F0) the pair (q1, q5) as 16 q * 2^-24, and the same on w >> 8 gives
//     (q2, q6) and (q3, q7). Subnormal float16 operands are exact, so the tensor cores form the
//     exact products q * x * 2^-24 (and 16 q * x * 2^-24) and sum them in float32;
//   * zero point and scale are applied after the MMA, in float32, once per (column, 32 codes):
//     sum_k (q_k - z) s x_k = s * (sum_k q_k x_k - z * sum_k x_k) (complex_kernel.glsl:80-83),
//     with sum_k x_k precomputed per 32 codes when the activations are staged;
//   * for that the MMA must keep each lane's 32 codes apart: in mma.sync m16n8k16 a lane c of a
//     quad supplies k in {2c, 2c+1, 2c+8, 2c+9}, so the B operand routes lane c's activations to
//     output column 2c only (lane 9c holds them, every other lane reads zeros). Output column 2c
//     of the accumulator is then the partial sum of lane c's own quantization block.
// Per 128 codes of 16 columns a lane issues about 80 instructions (2 weight loads, 4 shared
// activation loads, 40 bit operations, 8 MMAs, scale/zero-point math), a third of the
// dequantize-then-multiply form. Six register slots per lane keep five 128-code steps of
// weights in flight per warp (two CTAs of 8 warps per SM).
//
// Decomposition (as in the general GEMV): a warp owns 16 output columns (lane g = lane/4 holds
// columns n0+g and n0+g+8) and a contiguous slice of 128-wide k iterations, in which lane c
// holds the 16 bytes k in [32c, 32c+32) of each of its columns; slices are spread over the warps
// of a CTA and the CTAs of a thread-block cluster and combined in a fixed order through shared
// and distributed shared memory (deterministic, no global workspace). The activations of the
// CTA's k range are staged once per CTA in shared memory, permuted into MMA operand order.
#include <cuda_fp16.h>

#include <algorithm>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kCols = 16;            // output columns per warp tile
constexpr int kIterK = 128;          // k per iteration: 64 bytes of a column, 16 per lane
constexpr int kMaxSlices = 64;       // slices per tile (spc * splits)
constexpr int kSlots = 6;            // weight register slots per lane (prefetch distance 5)
constexpr int kMinBlocks = 2;        // resident CTAs per SM the register budget is set for
constexpr int kZeroBytes = 256;      // zero operands read by the lanes that carry no activations
constexpr int kMaxSmem = 96 * 1024;  // dynamic shared memory cap (staged activations)

enum ZpMode : int { kZDefault = 0, kZPacked = 1, kZFloat = 2 };

struct M1Params {
  const __half* x;        // [K]
  const uint8_t* b;       // [N, K/2]
  const __half* scales;   // [N, kb]
  const void* zp;         // zero points or nullptr
  const __half* bias;     // [N] or nullptr
  __half* y;              // [N]
  int K, N, kb, log2_bs;
  int zp_f32;             // float zero points stored as float32 (else float16)
  int zp_row_bytes;       // packed zero points: bytes per column
  int iters;              // 128-wide k iterations (K % 128 == 0)
  int tpc, spc, splits;   // tiles per CTA, slices per CTA (tpc * spc == 8), CTAs per cluster
};

__device__ __forceinline__ uint4 ldg_w128(const void* ptr) {
  uint4 v;
  asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(ptr));
  return v;
}

// Activation load for staging (after griddepcontrol.wait; volatile keeps it there).
__device__ __forceinline__ uint4 ldg_x128(const void* ptr) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(ptr)
               : "memory");
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// D += A * B (float32 accumulate).
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
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

// Metadata of one (column, block) as loaded: the float16 scale bits in the low half of `s` (a
// packed zero-point byte above them), float zero points in their stored bits in `z`.
struct Meta {
  uint32_t s, z;
};

template <int ZM>
__device__ __forceinline__ Meta load_meta(const M1Params& p, int srow, int zrow, int blk) {
  Meta m;
  m.s = __half_as_ushort(__ldg(p.scales + srow + blk));
  m.z = 0u;
  if (ZM == kZPacked) m.s |= static_cast<uint32_t>(__ldg(reinterpret_cast<const uint8_t*>(p.zp) + zrow + (blk >> 1))) << 16;
  if (ZM == kZFloat) {
    m.z = p.zp_f32 ? __float_as_uint(__ldg(reinterpret_cast<const float*>(p.zp) + srow + blk))
                   : static_cast<uint32_t>(__half_as_ushort(__ldg(reinterpret_cast<const __half*>(p.zp) + srow + blk)));
  }
  return m;
}

// Zero point as float: 8 when absent, the nibble of block blk when packed (low nibble first,
// complex_kernel.glsl:85), the stored value for float zero points.
template <int ZM>
__device__ __forceinline__ float zero_value(const M1Params& p, const Meta& m, int blk) {
  if (ZM == kZPacked) return static_cast<float>((m.s >> (16 + (blk & 1) * 4)) & 15u);
  if (ZM == kZFloat) return p.zp_f32 ? __uint_as_float(m.z) : __half2float(__ushort_as_half(static_cast<unsigned short>(m.z)));
  return 8.f;
}

__device__ __forceinline__ float scale_value(const Meta& m) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(m.s & 0xFFFFu)));
}


__device__ __forceinline__ float hsum2(uint32_t u) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
  return f.x + f.y;
}

// Shared memory (dynamic): [zeros: kZeroBytes][activations: n_stage * 256 B]
//                          [sums: n_stage * 4 floats][red: kWarps * 16 floats][part: kWarps * 16 floats]
template <int ZM>
__global__ void __launch_bounds__(kThreads, kMinBlocks) gemv_m1_kernel(const __grid_constant__ M1Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const int t_local = warp % p.tpc, s_local = warp / p.tpc;
  const int n0 = (static_cast<int>(blockIdx.x) * p.tpc + t_local) * kCols;
  const int S = p.spc * p.splits;
  const int y = static_cast<int>(blockIdx.y);
  const int slice = y * p.spc + s_local;
  const int it0 = static_cast<int>(static_cast<int64_t>(p.iters) * slice / S);
  const int it1 = static_cast<int>(static_cast<int64_t>(p.iters) * (slice + 1) / S);
  const int cta0 = static_cast<int>(static_cast<int64_t>(p.iters) * (y * p.spc) / S);
  const int cta1 = static_cast<int>(static_cast<int64_t>(p.iters) * ((y + 1) * p.spc) / S);
  const int n_stage = cta1 - cta0;
  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_x = s_base + kZeroBytes;
  float* sums = reinterpret_cast<float*>(smem + kZeroBytes + n_stage * 256);
  float* red = sums + n_stage * 4;
  float* part = red + kWarps * kCols;

  const bool tile_ok = n0 < p.N;
  const int colA = min(n0 + g, p.N - 1), colB = min(n0 + g + 8, p.N - 1);
  // 32-bit offsets (N * K / 2 < 2^31 and N * kb < 2^31 are checked by the planner).
  const uint8_t* wA = p.b + (colA * (p.K / 2) + 16 * c);
  const uint8_t* wB = p.b + (colB * (p.K / 2) + 16 * c);
  const int sA = colA * p.kb, sB = colB * p.kb, zA = colA * p.zp_row_bytes, zB = colB * p.zp_row_bytes;

  // Programmatic dependent launch: weights, scales and zero points are fetched before
  // griddepcontrol.wait, the activations and the output only after it.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  auto blk_of = [&](int it) { return (it * kIterK + 32 * c) >> p.log2_bs; };
  uint4 wa[kSlots], wb[kSlots];
  Meta ma[kSlots], mb[kSlots];
  auto fetch = [&](int it, int slot) {
    wa[slot] = ldg_w128(wA + it * 64);
    wb[slot] = ldg_w128(wB + it * 64);
    const int blk = blk_of(it);
    ma[slot] = load_meta<ZM>(p, sA, zA, blk);
    mb[slot] = load_meta<ZM>(p, sB, zB, blk);
  };
  const bool work = tile_ok && it0 < it1;
  const int n_it = work ? it1 - it0 : 0;
#pragma unroll
  for (int j = 0; j < kSlots - 1; ++j)
    if (j < n_it) fetch(it0 + j, j);

  asm volatile("griddepcontrol.wait;" ::: "memory");

  // Stage the CTA's activations: each 16-byte group (x0..x7) is stored as the B operands
  // (x0,x4), (x2,x6) | (x1,x5), (x3,x7) of the low- and high-nibble MMAs; the sum of every
  // 32 activations is kept times 2^-24 (the scale of the subnormal weight operands).
  if (threadIdx.x < kZeroBytes / 16) sts128(s_base + 16 * threadIdx.x, make_uint4(0u, 0u, 0u, 0u));
  {
    const int groups = n_stage * 16;
    const __half* xs = p.x + static_cast<int64_t>(cta0) * kIterK;
    for (int base = 0; base < groups; base += kThreads) {
      const int idx = base + static_cast<int>(threadIdx.x);
      const bool ok = idx < groups;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (ok) v = ldg_x128(xs + 8 * idx);
      float sum = (hsum2(v.x) + hsum2(v.y)) + (hsum2(v.z) + hsum2(v.w));
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if (ok) {
        sts128(s_x + 16 * idx, make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.y, v.w, 0x5410), prmt(v.x, v.z, 0x7632),
                                          prmt(v.y, v.w, 0x7632)));
        if ((idx & 3) == 0) sums[idx >> 2] = sum * 5.9604644775390625e-8f;  // 2^-24
      }
    }
  }
  __syncthreads();

  float tot0 = 0.f, tot1 = 0.f;  // columns colA and colB, this lane's 32-code chunks, times 2^-24
  if (work) {
    // Lane 9c (g == 2c) carries the activations of chunk c into B column 2c; every other lane
    // reads zeros, at an address whose banks differ from those of its 8-lane phase's carrier.
    const bool carrier = g == 2 * c;
    const uint32_t xlane = carrier ? s_x + (it0 - cta0) * 256 + 64 * c : s_base + ((64 * (lane >> 3) + 32) & 127);
    const uint32_t xstep = carrier ? 256u : 0u;
    const float* sum_lane = sums + (it0 - cta0) * 4 + c;
    auto compute = [&](int i, int slot) {
      const uint32_t xa = xlane + static_cast<uint32_t>(i) * xstep;
      const uint32_t a[4] = {wa[slot].x, wa[slot].y, wa[slot].z, wa[slot].w};
      const uint32_t b[4] = {wb[slot].x, wb[slot].y, wb[slot].z, wb[slot].w};
      float lo[4] = {0.f, 0.f, 0.f, 0.f}, hi[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint4 xv = lds128(xa + 16 * w);
        const uint32_t a8 = a[w] >> 8, b8 = b[w] >> 8;
        mma_f16(lo, a[w] & 0x000F000Fu, b[w] & 0x000F000Fu, a8 & 0x000F000Fu, b8 & 0x000F000Fu, xv.x, xv.y);
        mma_f16(hi, a[w] & 0x00F000F0u, b[w] & 0x00F000F0u, a8 & 0x00F000F0u, b8 & 0x00F000F0u, xv.z, xv.w);
      }
      const int blk = blk_of(it0 + i);
      const float sx = sum_lane[4 * i];
      const float za = zero_value<ZM>(p, ma[slot], blk), zb = zero_value<ZM>(p, mb[slot], blk);
      const float va = fmaf(hi[0], 0.0625f, lo[0]), vb = fmaf(hi[2], 0.0625f, lo[2]);
      tot0 = fmaf(scale_value(ma[slot]), fmaf(-za, sx, va), tot0);
      tot1 = fmaf(scale_value(mb[slot]), fmaf(-zb, sx, vb), tot1);
    };
    for (int i = 0; i < n_it; i += kSlots) {
#pragma unroll
      for (int s = 0; s < kSlots; ++s) {
        if (i + s < n_it) {
          if (i + s + kSlots - 1 < n_it) fetch(it0 + i + s + kSlots - 1, (s + kSlots - 1) % kSlots);
          compute(i + s, s);
        }
      }
    }
  }

  // ---- reduce: the quad's chunks, the slices of each tile in this CTA (fixed order), then the
  // cluster's CTAs through distributed shared memory.
  tot0 += __shfl_xor_sync(0xffffffffu, tot0, 1);
  tot0 += __shfl_xor_sync(0xffffffffu, tot0, 2);
  tot1 += __shfl_xor_sync(0xffffffffu, tot1, 1);
  tot1 += __shfl_xor_sync(0xffffffffu, tot1, 2);
  if (c == 0) {
    red[warp * kCols + g] = tot0;
    red[warp * kCols + g + 8] = tot1;
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.tpc * kCols; idx += kThreads) {
    const int t = idx / kCols, col = idx - t * kCols;
    float v = 0.f;
    for (int sl = 0; sl < p.spc; ++sl) v += red[(t + sl * p.tpc) * kCols + col];
    part[idx] = v;
  }
  if (p.splits > 1) cluster_sync();
  else __syncthreads();
  if (y == 0) {
    for (int idx = threadIdx.x; idx < p.tpc * kCols; idx += kThreads) {
      const int t = idx / kCols, col = idx - t * kCols;
      const int n = (static_cast<int>(blockIdx.x) * p.tpc + t) * kCols + col;
      if (n < p.N) {
        float v = part[idx];
        for (int s = 1; s < p.splits; ++s) v += ld_dsmem_f32(&part[idx], static_cast<unsigned>(s));
        v *= 16777216.f;  // 2^24
        if (p.bias) v += __half2float(p.bias[n]);
        p.y[n] = __float2half_rn(v);
      }
    }
  }
  if (p.splits > 1) cluster_sync();  // keep every CTA's shared memory alive until it is read
}

struct M1Shape {
  int tiles, tpc, spc, splits;
  size_t smem;
};

size_t m1_smem_bytes(int iters, int splits) {
  const int64_t max_stage = ceil_div(iters, splits);
  return static_cast<size_t>(kZeroBytes + max_stage * (256 + 16) + 2 * kWarps * kCols * 4);
}

// Slices per tile: the largest power of two whose warps all fit in one wave of resident CTAs
// (kMinBlocks per SM, fewer when the staged activations do not fit), at most one slice per
// 128-wide iteration, at most 8 warps x 8 cluster CTAs.
M1Shape m1_shape(const Problem& p) {
  M1Shape s{};
  s.tiles = static_cast<int>(ceil_div(p.N, kCols));
  const int iters = static_cast<int>(p.K / kIterK);
  auto fits = [&](int S) {
    const int spc = std::min(S, kWarps), splits = S / spc;
    const int64_t per_sm = std::min<int64_t>(kMinBlocks, (227 * 1024) / (m1_smem_bytes(iters, splits) + 1024));
    return static_cast<int64_t>(s.tiles) * S <= static_cast<int64_t>(device_sm_count()) * kWarps * per_sm;
  };
  int S = 1;
  while (S * 2 <= kMaxSlices && S * 2 <= std::max(1, iters) && fits(S * 2)) S *= 2;
  s.spc = std::min(S, kWarps);
  s.splits = S / s.spc;
  s.tpc = kWarps / s.spc;
  s.smem = m1_smem_bytes(iters, s.splits);
  return s;
}

template <int ZM>
cudaError_t launch_m1_variant(const M1Shape& s, const M1Params& gp, cudaStream_t stream) {
  if (s.smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemv_m1_kernel<ZM>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(s.smem));
    if (e != cudaSuccess) return e;
  }
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
  return cudaLaunchKernelEx(&cfg, gemv_m1_kernel<ZM>, gp);
}

int ilog2_m1(int64_t v) {
  int r = 0;
  while ((int64_t(1) << (r + 1)) <= v) ++r;
  return r;
}

}  // namespace

bool gemv_m1_supported(const Problem& p) {
  if (!(p.f16 && p.bits == 4 && p.M == 1 && p.bs >= 32 && (p.bs & (p.bs - 1)) == 0 && p.K % kIterK == 0 &&
        p.K % p.bs == 0 && p.N * (p.K / 2) < (1ll << 31) && p.N * p.kb < (1ll << 31) &&
        (reinterpret_cast<uintptr_t>(p.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 &&
        (reinterpret_cast<uintptr_t>(p.scales) % 2) == 0))
    return false;
  return m1_shape(p).smem <= static_cast<size_t>(kMaxSmem);
}

cudaError_t launch_gemv_m1(const Problem& p, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  const M1Shape s = m1_shape(p);
  M1Params gp{};
  gp.x = static_cast<const __half*>(p.a);
  gp.b = p.b;
  gp.scales = static_cast<const __half*>(p.scales);
  gp.zp = p.zp_ptr;
  gp.bias = static_cast<const __half*>(p.bias);
  gp.y = static_cast<__half*>(p.y);
  gp.K = static_cast<int>(p.K);
  gp.N = static_cast<int>(p.N);
  gp.kb = static_cast<int>(p.kb);
  gp.log2_bs = ilog2_m1(p.bs);
  gp.zp_f32 = p.zp == kZpF32;
  gp.zp_row_bytes = static_cast<int>((p.kb + 1) / 2);
  gp.iters = static_cast<int>(p.K / kIterK);
  gp.tpc = s.tpc;
  gp.spc = s.spc;
  gp.splits = s.splits;
  if (p.zp == kZpNone) return launch_m1_variant<kZDefault>(s, gp, stream);
  if (p.zp == kZpPacked) return launch_m1_variant<kZPacked>(s, gp, stream);
  return launch_m1_variant<kZFloat>(s, gp, stream);
}

}  // namespace xrgpu
