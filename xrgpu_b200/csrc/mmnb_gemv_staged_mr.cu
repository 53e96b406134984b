// 4-bit MatMulNBits decode GEMV for 1..16 activation rows with block size 128 or 256, weights staged
// through shared memory by asynchronous copies, sm_100a.
//
// The batched-decode form of the staged single-row GEMV (mmnb_gemv_staged.cu), for the shapes it
// leaves out: several activation rows (M = 4 / 16, K = 4096, N = 14336, bs 128,
// packed zero points) and single rows at bs >= 128 with packed zero points.
//   * Same copy side: one CTA per SM owns a contiguous range of 16-column tiles, whose 16-column x
//     128-code units are cut into one contiguous range per warp; each warp streams its units through
//     its own ring of shared-memory stages with cp.async (a stage = up to four units of one 512-code
//     window: 16 rows x 256 contiguous bytes, plus the window's scales and zero points).
//   * Same unpack: codes become exact float16 subnormal operands with ANDs and a shift
//     ((w & 0x000F000F) is (q0, q4) * 2^-24, (w & 0x00F000F0) is (q1, q5) * 16 * 2^-24, and so on).
//   * The activation rows are the MMA's B columns. In mma.sync m16n8k16 lane (g, c) supplies B for
//     column g and k in {2c, 2c+1, 2c+8, 2c+9}, i.e. for activation row 8t + g and the codes of its
//     own 32-code chunk c; with MT = ceil(M / 8) tiles of 8 rows each weight fragment feeds MT MMAs.
//     Each lane reads its row from shared memory: rows at a pitch of 2K + 16 bytes and 16-byte groups
//     swizzled (group i at i ^ 2 ((i >> 3) & 1)) so the eight lanes of a load phase hit distinct bank
//     groups.
//   * A block size of 128 or 256 puts a whole unit in one quantization block, so every unit's MMA sum
//     is scaled on its own: sum_k (q_k - z) s x_k = s (sum_k q_k x_k - z sum_k x_k)
//     (complex_kernel.glsl:80-83), with the activation sums per row and unit precomputed. Each
//     (row, column) of Y then sits in exactly one lane's accumulator: no reduction across lanes.
// Tiles cut between warps are summed at the end of the CTA through shared memory in warp order
// (deterministic, no global workspace).
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kNst = 2;               // stages per warp ring
constexpr int kRows = 16;             // output columns per tile
constexpr int kUnitK = 128;           // codes per work unit
constexpr int kWinUnits = 4;          // units per 512-code window (one stage at most)
constexpr int kPitch = 256;           // shared-memory row pitch of a stage (swizzled)
constexpr int kStageWBytes = kRows * kPitch;
constexpr int kMaxSmem = 227 * 1024;

enum ZpMode : int { kZDefault = 0, kZPacked = 1, kZFloat = 2 };

struct MrParams {
  const __half* x;       // [M][K]
  const uint8_t* b;      // [N, K/2]
  const __half* scales;  // [N, kb]
  const void* zp;        // zero points or nullptr
  const __half* bias;    // [N] or nullptr
  __half* y;             // [M][ldy]
  int M, K, N, kb, ldy;
  int zp_f32;            // float zero points stored as float32 (else float16)
  int zrow;              // packed zero points: bytes per column
  int tiles, upt;        // 16-column tiles; units per tile (K / 128)
  int bs_shift;          // log2(block size): 7 or 8
  int sb;                // scale bytes per row per window (8 or 4)
  int zb;                // zero-point bytes per row per window as copied (packed: the 4-byte word)
  int slot_bytes;        // bytes of one stage
  int xpitch;            // bytes per staged activation row (2K + 16)
  int ring_off;          // byte offset of the rings in shared memory
};

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_bytes(uint32_t dst, const void* src, int bytes) {
  if (bytes == 16) asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
  else if (bytes == 8) asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
  else asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 lds64f(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float half_lo(uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v))); }
__device__ __forceinline__ float nibble_f(uint32_t n) { return __uint_as_float(0x4B000000u | n) - 8388608.f; }
__device__ __forceinline__ float hsum2(uint32_t u) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
  return f.x + f.y;
}

// D = A * B (fresh accumulator) and D += A * B, float16 operands, float32 accumulation.
__device__ __forceinline__ void mma_first(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}
__device__ __forceinline__ void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Stage row swizzle (as in the single-row kernel): 16-byte chunk k of row r at chunk k ^ f(r).
__host__ __device__ constexpr int row_swizzle(int r) { return (r & 7) ^ (4 * (r & 1)); }
// Activation row swizzle: 16-byte group i of a row at group i ^ 2 ((i >> 3) & 1).
__host__ __device__ constexpr int x_swizzle(int i) { return i ^ (((i >> 3) & 1) << 1); }

__device__ __forceinline__ int range_lo(int q, int base, int r) { return q * base + min(q, r); }
__device__ __forceinline__ int owner_of(int i, int base, int r) {
  const int split = r * (base + 1);
  return i < split ? i / (base + 1) : r + (i - split) / base;
}

// Shared memory (dynamic), offsets from the 1024-byte aligned base:
//   [0, 8 MT xpitch)           activation rows (rows >= M zero), each 16-byte group (x0..x7) stored as
//                              (x0,x4) (x2,x6) (x1,x5) (x3,x7) at its swizzled position
//   [.., + upt 8 MT 4)         sums[unit][row] of every 128 activations times 2^-24
//   [ring_off, ..)             W rings of kNst stages: [16 rows x 256 B][16 x sb scales][16 x zb zero points];
//                              after the last stage, partial sums of tiles cut between warps
//                              [warp][first / last][16][8 MT]
template <int MT, int ZM, int W>
__global__ void __launch_bounds__(W * 32, 1) gemv_staged_mr_kernel(const __grid_constant__ MrParams p) {
  constexpr int kRowsPad = 8 * MT;
  constexpr int kThreads = W * 32;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_x = s_base;
  const uint32_t s_sums = s_x + kRowsPad * p.xpitch;
  // partial sums of tiles cut between warps, [warp][first / last][16][8 MT]: in the ring area,
  // written only after every warp has finished streaming
  float* red = reinterpret_cast<float*>(smem + p.ring_off);
  const uint32_t s_ring = s_base + p.ring_off + warp * kNst * p.slot_bytes;

  const int tile_lo = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.tiles / gridDim.x);
  const int tile_hi = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.tiles / gridDim.x);
  const int cu = (tile_hi - tile_lo) * p.upt;
  const int act = min(W, cu), base = cu / act, rem = cu % act;
  const int u_lo = tile_lo * p.upt + range_lo(min(warp, act), base, rem);
  const int u_hi = tile_lo * p.upt + range_lo(min(warp + 1, act), base, rem);
  const int tile0 = u_lo / p.upt;
  const int tu0 = u_lo - tile0 * p.upt;

  // ---- copy side (as the single-row kernel): copy instruction i moves rows 2i and 2i+1 of the window,
  // lane: row 2i + (lane >> 4), 16-byte chunk k = lane & 15, stored at chunk k ^ f(row).
  const int wh = lane >> 4, wk = lane & 15;
  uint32_t w_dst[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) w_dst[j] = wh * kPitch + 16u * static_cast<uint32_t>((wk ^ (5 * wh)) ^ (2 * j));
  const int w_unit = wk >> 2;
  int is_tile = tile0, is_tu = tu0, is_slot = 0;
  int is_left = u_hi - u_lo;
  const uint8_t *w_src = nullptr, *s_src = nullptr, *z_src = nullptr;
  const int zcopy = ZM == kZPacked ? 4 : p.zb;  // bytes per row per window copied for the zero points
  auto set_tile = [&](int tile) {
    const int nbase = tile * kRows;
    w_src = p.b + static_cast<int64_t>(nbase + wh) * (p.K / 2) + 16 * wk;
    const int r = min(nbase + (lane & 15), p.N - 1);
    s_src = reinterpret_cast<const uint8_t*>(p.scales) + static_cast<int64_t>(r) * p.kb * 2;
    if (ZM == kZPacked) z_src = reinterpret_cast<const uint8_t*>(p.zp) + static_cast<int64_t>(r) * p.zrow;
    if (ZM == kZFloat) z_src = reinterpret_cast<const uint8_t*>(p.zp) + static_cast<int64_t>(r) * p.kb * (p.zp_f32 ? 4 : 2);
  };
  if (is_left > 0) set_tile(is_tile);
  auto issue = [&]() {
    if (is_left > 0) {
      const int win = is_tu >> 2, j0 = is_tu & 3;
      const int n = min(min(kWinUnits - j0, p.upt - is_tu), is_left);
      const uint32_t slot = s_ring + is_slot * p.slot_bytes;
      if (w_unit >= j0 && w_unit < j0 + n) {
        const uint32_t d0 = slot + w_dst[0], d1 = slot + w_dst[1], d2 = slot + w_dst[2], d3 = slot + w_dst[3];
        const int win_off = win * (kWinUnits * kUnitK / 2);
        if ((is_tile + 1) * kRows <= p.N) {
          const uint8_t* src = w_src + win_off;
          const int64_t brow2 = p.K;  // two rows
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t d = (i & 3) == 0 ? d0 : (i & 3) == 1 ? d1 : (i & 3) == 2 ? d2 : d3;
            cp_async_16(d + 512u * i, src + i * brow2);
          }
        } else {  // ragged last tile: rows past N re-read row N - 1
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t d = (i & 3) == 0 ? d0 : (i & 3) == 1 ? d1 : (i & 3) == 2 ? d2 : d3;
            const int n_row = min(is_tile * kRows + 2 * i + wh, p.N - 1);
            cp_async_16(d + 512u * i, p.b + static_cast<int64_t>(n_row) * (p.K / 2) + win_off + 16 * wk);
          }
        }
      }
      if (lane < kRows) {
        cp_async_bytes(slot + kStageWBytes + lane * p.sb, s_src + win * p.sb, p.sb);
        if (ZM == kZPacked)  // the aligned 4-byte word holding the window's packed zero points
          cp_async_bytes(slot + kStageWBytes + kRows * p.sb + lane * 4, z_src + ((win * p.zb) & ~3), 4);
        if (ZM == kZFloat) cp_async_bytes(slot + kStageWBytes + kRows * p.sb + lane * zcopy, z_src + win * zcopy, zcopy);
      }
      is_left -= n;
      is_tu += n;
      if (is_tu == p.upt && is_left > 0) {
        is_tu = 0;
        set_tile(++is_tile);
      }
    }
    cp_async_commit();
    if (++is_slot == kNst) is_slot = 0;
  };

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#pragma unroll
  for (int j = 0; j < kNst - 1; ++j) issue();
  asm volatile("griddepcontrol.wait;" ::: "memory");

  {  // Activations: every 16-byte group copied into place by cp.async (rows >= M zero-filled), then
     // one pass per (row, unit) turns the unit's 16 groups into MMA order in place -- (x0..x7) to
     // (x0,x4) (x2,x6) (x1,x5) (x3,x7), the second 8 groups swapped in pairs (the row swizzle keeps
     // a unit's groups inside the unit) -- and adds its 128 activations. Lanes start at different
     // groups of their unit so the eight lanes of a phase hit different bank groups.
    const int gpr = p.K / 8;  // 16-byte groups per row
    for (int gi = threadIdx.x; gi < kRowsPad * gpr; gi += kThreads) {
      const int row = gi / gpr, idx = gi - row * gpr;
      const bool real = row < p.M;
      const void* src = real ? static_cast<const void*>(p.x + static_cast<int64_t>(row) * p.K + 8 * idx) : p.x;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s_x + row * p.xpitch + 16 * idx), "l"(src),
                   "r"(real ? 16 : 0)
                   : "memory");
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncthreads();
    for (int ru = threadIdx.x; ru < kRowsPad * p.upt; ru += kThreads) {
      const int row = ru / p.upt, u = ru - row * p.upt;
      const uint32_t ub = s_x + row * p.xpitch + 256 * u;
      float sum = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = lds128(ub + 16 * (8 * half + ((j + ru) & 7)));
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = 8 * half + ((j + ru) & 7);
          sum += (hsum2(v[j].x) + hsum2(v[j].y)) + (hsum2(v[j].z) + hsum2(v[j].w));
          sts128(ub + 16 * x_swizzle(i), make_uint4(prmt(v[j].x, v[j].z, 0x5410), prmt(v[j].y, v[j].w, 0x5410),
                                                    prmt(v[j].x, v[j].z, 0x7632), prmt(v[j].y, v[j].w, 0x7632)));
        }
      }
      asm volatile("st.shared.f32 [%0], %1;" ::"r"(s_sums + 4u * (u * kRowsPad + row)), "f"(sum * 5.9604644775390625e-8f)
                   : "memory");
    }
  }
  __syncthreads();

  // ---- compute side
  const uint32_t w_lane = g * kPitch + 16u * static_cast<uint32_t>(c ^ row_swizzle(g));
  const int cs = 2 * (c >> 1);  // the activation swizzle of this lane's chunk
  uint32_t x_row[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) x_row[t] = s_x + (8 * t + g) * p.xpitch + 64 * c;

  float tot[MT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int j = 0; j < 4; ++j) tot[t][j] = 0.f;

  auto consume = [&](uint32_t slot, int win, int j0, int n) {
    const uint32_t sslot = slot + kStageWBytes, zslot = sslot + kRows * p.sb;
    const uint32_t wl = slot + w_lane;
#pragma unroll
    for (int jl = 0; jl < kWinUnits; ++jl) {
      if (jl < j0 || jl >= j0 + n) continue;
      const uint32_t wad = wl ^ (64u * jl);
      const uint4 wa = lds128(wad), wb = lds128(wad + 8 * kPitch);
      const uint32_t a[4] = {wa.x, wa.y, wa.z, wa.w}, b[4] = {wb.x, wb.y, wb.z, wb.w};
      float lo[MT][4], hi[MT][4];
      const uint32_t xo = 1024u * win + 256u * jl;
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint32_t a8 = a[w] >> 8, b8 = b[w] >> 8;
        const uint32_t l0 = a[w] & 0x000F000Fu, l1 = b[w] & 0x000F000Fu, l2 = a8 & 0x000F000Fu, l3 = b8 & 0x000F000Fu;
        const uint32_t h0 = a[w] & 0x00F000F0u, h1 = b[w] & 0x00F000F0u, h2 = a8 & 0x00F000F0u, h3 = b8 & 0x00F000F0u;
        const uint32_t xw = xo + 16u * static_cast<uint32_t>(w ^ cs);
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const uint4 xv = lds128(x_row[t] + xw);
          if (w == 0) {
            mma_first(lo[t], l0, l1, l2, l3, xv.x, xv.y);
            mma_first(hi[t], h0, h1, h2, h3, xv.z, xv.w);
          } else {
            mma_acc(lo[t], l0, l1, l2, l3, xv.x, xv.y);
            mma_acc(hi[t], h0, h1, h2, h3, xv.z, xv.w);
          }
        }
      }
      // the unit's quantization block, its scales and zero points for columns g and g + 8
      const int blk = (jl * kUnitK) >> p.bs_shift;  // block within the window
      const float sa = half_lo(lds_u16(sslot + g * p.sb + 2 * blk));
      const float sbv = half_lo(lds_u16(sslot + (g + 8) * p.sb + 2 * blk));
      float za = 8.f, zb = 8.f;
      if (ZM == kZPacked) {
        const int nib = ((win * p.zb) & 3) * 2 + blk;  // nibble index within the copied word
        za = nibble_f((lds_u32(zslot + g * 4) >> (4 * nib)) & 15u);
        zb = nibble_f((lds_u32(zslot + (g + 8) * 4) >> (4 * nib)) & 15u);
      }
      if (ZM == kZFloat) {
        const uint32_t ra = zslot + g * p.zb + (p.zp_f32 ? 4 : 2) * blk, rb = ra + 8 * p.zb;
        za = p.zp_f32 ? __uint_as_float(lds_u32(ra)) : half_lo(lds_u16(ra));
        zb = p.zp_f32 ? __uint_as_float(lds_u32(rb)) : half_lo(lds_u16(rb));
      }
      const int u = win * kWinUnits + jl;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        const float2 sx = lds64f(s_sums + 4u * (u * kRowsPad + 8 * t + 2 * c));
        const float v0 = fmaf(hi[t][0], 0.0625f, lo[t][0]), v1 = fmaf(hi[t][1], 0.0625f, lo[t][1]);
        const float v2 = fmaf(hi[t][2], 0.0625f, lo[t][2]), v3 = fmaf(hi[t][3], 0.0625f, lo[t][3]);
        tot[t][0] = fmaf(sa, fmaf(-za, sx.x, v0), tot[t][0]);
        tot[t][1] = fmaf(sa, fmaf(-za, sx.y, v1), tot[t][1]);
        tot[t][2] = fmaf(sbv, fmaf(-zb, sx.x, v2), tot[t][2]);
        tot[t][3] = fmaf(sbv, fmaf(-zb, sx.y, v3), tot[t][3]);
      }
    }
  };

  // Y[row][n] from its scaled sum (bias added), rows < M and columns < N only.
  auto store = [&](int row, int n, float v) {
    if (row < p.M && n < p.N) {
      v *= 16777216.f;  // 2^24
      if (p.bias) v += __half2float(p.bias[n]);
      p.y[static_cast<int64_t>(row) * p.ldy + n] = __float2half_rn(v);
    }
  };
  // Lane (g, c) holds, for tile t, columns g / g + 8 and rows 8t + 2c / 8t + 2c + 1. A segment that
  // covers only part of its tile (the warp's first and/or last) is kept in registers until the end.
  float keep0[MT][4], keep1[MT][4];  // the first / last cut segment
  bool kept0 = false, kept1 = false;
  auto emit = [&](int tile, bool whole, bool first) {
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int r0 = 8 * t + 2 * c;
      if (whole) {
        store(r0, tile * kRows + g, tot[t][0]);
        store(r0 + 1, tile * kRows + g, tot[t][1]);
        store(r0, tile * kRows + g + 8, tot[t][2]);
        store(r0 + 1, tile * kRows + g + 8, tot[t][3]);
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (!whole && first) keep0[t][j] = tot[t][j];
        if (!whole && !first) keep1[t][j] = tot[t][j];
        tot[t][j] = 0.f;
      }
    }
    kept0 |= !whole && first;
    kept1 |= !whole && !first;
  };
  auto spill = [&](int slot, const float (&kv)[MT][4]) {  // red[warp][slot][column][row]
    float* mine = red + (warp * 2 + slot) * kRows * kRowsPad;
#pragma unroll
    for (int t = 0; t < MT; ++t) {
      const int r0 = 8 * t + 2 * c;
      mine[g * kRowsPad + r0] = kv[t][0];
      mine[g * kRowsPad + r0 + 1] = kv[t][1];
      mine[(g + 8) * kRowsPad + r0] = kv[t][2];
      mine[(g + 8) * kRowsPad + r0 + 1] = kv[t][3];
    }
  };
  auto finish = [&](int tile) {
    const int t0 = (tile - tile_lo) * p.upt;
    const int qa = owner_of(t0, base, rem), qb = owner_of(t0 + p.upt - 1, base, rem);
    if (qb != warp || qa == qb) return;
    const int qa_slot = range_lo(qa, base, rem) < t0 ? 1 : 0;
    for (int e = lane; e < kRows * kRowsPad; e += 32) {
      float v = 0.f;
      for (int qq = qa; qq <= qb; ++qq) v += red[(qq * 2 + (qq == qa ? qa_slot : 0)) * kRows * kRowsPad + e];
      store(e % kRowsPad, tile * kRows + e / kRowsPad, v);
    }
  };

  int left = u_hi - u_lo;
  int tile = tile0, tu = tu0, seg0 = tu0, slot_i = 0;
  bool first = true;
  while (left > 0) {
    const int win = tu >> 2, j0 = tu & 3;
    const int n = min(min(kWinUnits - j0, p.upt - tu), left);
    cp_async_wait<kNst - 2>();
    __syncwarp();
    issue();
    consume(s_ring + slot_i * p.slot_bytes, win, j0, n);
    if (++slot_i == kNst) slot_i = 0;
    left -= n;
    tu += n;
    if (tu == p.upt || left == 0) {
      emit(tile, seg0 == 0 && tu == p.upt, first);
      first = false;
      seg0 = 0;
      tu = 0;
      ++tile;
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the rings are free: cut-tile partials go there
  if (kept0) spill(0, keep0);
  if (kept1) spill(1, keep1);
  __syncthreads();
  if (u_lo < u_hi) {
    finish(tile0);
    const int last = (u_hi - 1) / p.upt;
    if (last != tile0) finish(last);
  }
}

struct MrShape {
  int mt, warps, sb, zb, slot_bytes, xpitch, ring_off;
  size_t smem;
};

MrShape mr_shape(const Problem& p) {
  MrShape s{};
  s.mt = p.M <= 8 ? 1 : 2;
  s.warps = s.mt == 1 ? 16 : 11;
  const int win_blocks = static_cast<int>((kWinUnits * kUnitK) / p.bs);  // 4 or 2
  s.sb = 2 * win_blocks;
  s.zb = p.zp == kZpPacked ? win_blocks / 2 : (p.zp == kZpF32 ? 4 * win_blocks : (p.zp == kZpF16 ? 2 * win_blocks : 0));
  const int zcopy = p.zp == kZpPacked ? 4 : s.zb;
  s.slot_bytes = (kStageWBytes + kRows * (s.sb + zcopy) + 255) & ~255;
  s.xpitch = static_cast<int>(2 * p.K + 16);
  const int rows_pad = 8 * s.mt;
  const int64_t upt = p.K / kUnitK;
  const int64_t head = static_cast<int64_t>(rows_pad) * s.xpitch + upt * rows_pad * 4;
  s.ring_off = static_cast<int>((head + 255) & ~int64_t{255});
  const size_t rings = static_cast<size_t>(s.warps) * kNst * s.slot_bytes;
  const size_t red = static_cast<size_t>(s.warps) * 2 * kRows * rows_pad * 4;  // aliases the rings
  s.smem = static_cast<size_t>(s.ring_off) + std::max(rings, red);
  return s;
}

template <int MT, int ZM, int W>
cudaError_t launch_mr_variant(const MrParams& mp, int grid, size_t smem, cudaStream_t stream) {
  static std::atomic<uint64_t> raised{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (smem > 48 * 1024 && !(raised.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(gemv_staged_mr_kernel<MT, ZM, W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kMaxSmem);
    if (e != cudaSuccess) return e;
    raised.fetch_or(bit, std::memory_order_acq_rel);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(W * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_staged_mr_kernel<MT, ZM, W>, mp);
}

template <int MT, int W>
cudaError_t launch_mr_mt(const Problem& p, const MrParams& mp, int grid, size_t smem, cudaStream_t s) {
  if (p.zp == kZpNone) return launch_mr_variant<MT, kZDefault, W>(mp, grid, smem, s);
  if (p.zp == kZpPacked) return launch_mr_variant<MT, kZPacked, W>(mp, grid, smem, s);
  return launch_mr_variant<MT, kZFloat, W>(mp, grid, smem, s);
}

}  // namespace

bool gemv_mr_supported(const Problem& p) {
  if (!(p.f16 && p.bits == 4 && p.M >= 1 && p.M <= 16 && (p.bs == 128 || p.bs == 256) && p.K % (kWinUnits * kUnitK) == 0 &&
        p.N >= 1 && p.N * (p.K / 2) < (1ll << 31) && p.N * p.kb < (1ll << 31) && p.ldy >= p.N &&
        (reinterpret_cast<uintptr_t>(p.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 &&
        (reinterpret_cast<uintptr_t>(p.scales) % 16) == 0))
    return false;
  if (p.zp == kZpPacked && ((p.kb + 1) / 2 % 4 != 0 || reinterpret_cast<uintptr_t>(p.zp_ptr) % 4 != 0)) return false;
  if ((p.zp == kZpF16 || p.zp == kZpF32) && (reinterpret_cast<uintptr_t>(p.zp_ptr) % 16) != 0) return false;
  return mr_shape(p).smem <= static_cast<size_t>(kMaxSmem);
}

cudaError_t launch_gemv_mr(const Problem& p, cudaStream_t stream) {
  if (p.N == 0 || p.M == 0) return cudaSuccess;
  const MrShape s = mr_shape(p);
  MrParams mp{};
  mp.x = static_cast<const __half*>(p.a);
  mp.b = p.b;
  mp.scales = static_cast<const __half*>(p.scales);
  mp.zp = p.zp_ptr;
  mp.bias = static_cast<const __half*>(p.bias);
  mp.y = static_cast<__half*>(p.y);
  mp.M = static_cast<int>(p.M);
  mp.K = static_cast<int>(p.K);
  mp.N = static_cast<int>(p.N);
  mp.kb = static_cast<int>(p.kb);
  mp.ldy = static_cast<int>(p.ldy);
  mp.zp_f32 = p.zp == kZpF32;
  mp.zrow = static_cast<int>((p.kb + 1) / 2);
  mp.tiles = static_cast<int>(ceil_div(p.N, kRows));
  mp.upt = static_cast<int>(p.K / kUnitK);
  mp.bs_shift = p.bs == 128 ? 7 : 8;
  mp.sb = s.sb;
  mp.zb = s.zb;
  mp.slot_bytes = s.slot_bytes;
  mp.xpitch = s.xpitch;
  mp.ring_off = s.ring_off;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(device_sm_count(), mp.tiles)));
  return s.mt == 1 ? launch_mr_mt<1, 16>(p, mp, grid, s.smem, stream) : launch_mr_mt<2, 11>(p, mp, grid, s.smem, stream);
}

}  // namespace xrgpu
