// 4-bit MatMulNBits decode GEMV for a single activation row (M == 1), weights staged through
// shared memory by asynchronous copies, sm_100a.
//
// A decode GEMV of a 4096 x 14336 projection gives each SM only ~200 KB of weights, so the kernel
// is built around three things: little instruction work per weight byte, enough warps per SM to
// hide instruction latency, and an even split of the bytes over the SMs.
//   * Work unit: 16 output columns x 128 codes (1 KB of packed weights). Each CTA (one per SM)
//     owns a contiguous range of 16-column tiles, and the units of that range, tile-major, are cut
//     into one contiguous range per warp, so the warps of a CTA stream the same number of units
//     (+-1) whatever the shape. A tile cut between warps is summed at the end of the CTA through
//     shared memory, in warp order (fixed, so results are deterministic): no global workspace.
//   * Each warp drives its own ring of shared-memory stages with cp.async (LDGSTS): a stage is up
//     to four consecutive units of one 512-code window of its tile (256 bytes of each of the 16
//     rows, one lane copying 128 contiguous bytes of a row) plus the window's scales and zero
//     points. Rows are stored at a 320-byte pitch, which makes the MMA operand reads below
//     conflict-free at fixed offsets. Completion is per thread (cp.async.wait_group), then
//     __syncwarp: no barrier waits.
//   * Arithmetic: codes become exact float16 subnormal operands with four ANDs and a shift per 8
//     codes ((w & 0x000F000F) is the pair (q0, q4) as q * 2^-24, (w & 0x00F000F0) the pair (q1, q5)
//     as 16 q * 2^-24, the same on w >> 8 gives (q2, q6), (q3, q7)); in mma.sync m16n8k16 lane c of
//     a quad supplies k in {2c, 2c+1, 2c+8, 2c+9}, and lane 9c routes the activations of lane c's
//     32 codes (unit chunk c) to accumulator column 2c only, so each column of the accumulator is
//     the partial sum of one quantization block; scale and zero point are then applied in float32:
//     sum_k (q_k - z) s x_k = s (sum_k q_k x_k - z sum_k x_k) (complex_kernel.glsl:80-83), with the
//     activation sums per 32 codes precomputed when the activations are staged.
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>

#include "mmnb_common.cuh"

namespace xrgpu {
namespace {

constexpr int kW = 16;                // warps per CTA, one CTA per SM (each warp copies its own stages)
constexpr int kThreads = kW * 32;
constexpr int kNst = 2;               // stages per warp ring (one in flight while one is read)
constexpr int kMinCtas = 1;           // CTAs per SM the register budget allows (2: two kernels' CTAs co-reside)
constexpr int kRows = 16;             // output columns per warp tile
constexpr int kUnitK = 128;           // codes per work unit (64 bytes of each row)
constexpr int kWinUnits = 4;          // units per 512-code window (one stage at most)
constexpr int kPitch = 256;           // shared-memory row pitch of a stage (swizzled)
constexpr int kStageWBytes = kRows * kPitch;
constexpr int kZeroRegion = 1024;     // zero B operands for the lanes that carry no activations
constexpr int kMaxSmem = 227 * 1024;

enum ZpMode : int { kZDefault = 0, kZPacked = 1, kZFloat = 2 };

struct StagedParams {
  const __half* x;       // [K]
  const uint8_t* b;      // [N, K/2]
  const __half* scales;  // [N, kb]
  const void* zp;        // zero points or nullptr
  const __half* bias;    // [N] or nullptr
  __half* y;             // [N]
  int K, N, kb;
  int zp_f32;            // float zero points stored as float32 (else float16)
  int zrow;              // packed zero points: bytes per column
  int tiles, upt;        // 16-column tiles; units per tile (K / 128)
  int sb, zb;            // scale / zero-point bytes per row per window
  int slot_bytes;        // bytes of one stage: weights, scales, zero points
  StagedPush push;       // sharded form: output columns also sent to the other ranks (world 0: off)
};

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_volatile_u64(void* p, uint64_t v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Columns (n, n + 1) of this rank's shard as one word (float16 bits of n | bits of n + 1 << 16 |
// epoch << 32) into words[e & 1][rank] of every other rank, at byte 4 n: the layout of the peer
// all-gather's flag-in-word form, whose receive kernel takes the words. One 64-bit store each, so
// the receiver sees data and epoch together; no fence is needed. Columns at or past the shard
// width (ragged last tile) are not sent.
__device__ __forceinline__ void push_pair(const StagedPush& q, uint32_t e, int n, uint32_t two) {
  if (n >= q.cols) return;
  const int64_t off = q.words_off + (static_cast<int64_t>(e & 1u) * q.world + q.rank) * q.ll_bytes + 4 * static_cast<int64_t>(n);
  const uint64_t w = (static_cast<uint64_t>(e) << 32) | two;
  for (int r = 0; r < q.world; ++r)
    if (r != q.rank) st_volatile_u64(q.region[r] + off, w);
}

__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_small(uint32_t dst, const void* src, int bytes) {
  if (bytes >= 16) asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
  else if (bytes == 8) asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
  else asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
template <int kBytes>
__device__ __forceinline__ void cp_async_n(uint32_t dst, const void* src) {
  if (kBytes == 16) asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
  else if (kBytes == 8) asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
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
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 lds128f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}
__device__ __forceinline__ float half_lo(uint32_t v) { return __half2float(__ushort_as_half(static_cast<unsigned short>(v))); }
// Integer 0..15 to float without the conversion unit: 2^23 + n as bits, minus 2^23.
__device__ __forceinline__ float nibble_f(uint32_t n) { return __uint_as_float(0x4B000000u | n) - 8388608.f; }

// D = A * B (float32, accumulator starting from zero).
__device__ __forceinline__ void mma_f16_first(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
}

// D += A * B (float32 accumulate).
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}


__device__ __forceinline__ float hsum2(uint32_t u) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
  return f.x + f.y;
}

// Swizzle of row r in a stage: 16-byte chunk k is stored at chunk k ^ f(r). Rows 2p and 2p+1 then
// put the four chunks an MMA step reads from each in different bank groups, and the 16 rows of one
// copy instruction land in all eight bank groups.
__host__ __device__ constexpr int row_swizzle(int r) { return (r & 7) ^ (4 * (r & 1)); }

// Shared memory (dynamic), offsets from the 1024-byte aligned base:
//   [0, 1 KB)          zeros (B operands of the lanes that carry no activations)
//   [1 KB, +2K)        activations, each 16-byte group (x0..x7) as (x0,x4) (x2,x6) (x1,x5) (x3,x7)
//   [.., +K/8)         sum of every 32 activations times 2^-24, ordered [window][chunk c][unit]
//   [.., +kW 128 B)    partial sums of the tiles cut between warps, [warp][first / last][16]
//   [256-aligned, ..)  kW rings of kNst stages: [16 rows x 256 B][16 x sb scales][16 x zb zero points]
__host__ __device__ inline int ring_offset(int K) { return (kZeroRegion + 2 * K + K / 8 + kW * 2 * kRows * 4 + 255) & ~255; }

// Window geometry of one block size (a window is 512 codes of a row).
template <int BS>
struct WinGeom {
  static constexpr int kSb = 2 * kWinUnits * kUnitK / BS;        // scale bytes per row: 32, 16, 8, 4
  static constexpr int kScs = kSb < 16 ? kSb : 16;                 // copy size of the scales
  static constexpr int kSparts = kSb / kScs;                       // copies per row: 2, 1, 1, 1
  static constexpr int kScopies = kRows * kSparts;                 // 32, 16, 16, 16
  static constexpr int kZbPacked = kWinUnits * kUnitK / BS / 2;    // packed zero-point bytes per row (BS <= 64)
};

// Warp ranges in a CTA: with U = Q base + r, warps q < r take base + 1 units and the others base, so
// warp q starts at q base + min(q, r); owner_of(i) is the warp whose range holds unit i.
__device__ __forceinline__ int range_lo(int q, int base, int r) { return q * base + min(q, r); }
__device__ __forceinline__ int owner_of(int i, int base, int r) {
  const int split = r * (base + 1);
  return i < split ? i / (base + 1) : r + (i - split) / base;
}

template <int BS, int ZM>
__global__ void __launch_bounds__(kThreads, kMinCtas) gemv_staged_kernel(const __grid_constant__ StagedParams p) {
  using G = WinGeom<BS>;
  extern __shared__ __align__(1024) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const uint32_t s_base = smem_u32(smem);
  const uint32_t s_x = s_base + kZeroRegion, s_sums = s_x + 2 * p.K;
  const uint32_t s_ring = s_base + ring_offset(p.K) + warp * kNst * p.slot_bytes;

  float* red = reinterpret_cast<float*>(smem + kZeroRegion + 2 * p.K + p.K / 8);
  // This CTA's tiles [tile_lo, tile_hi) and their cu units, cut over the first `act` warps (every
  // one of them non-empty; the others idle).
  const int tile_lo = static_cast<int>(static_cast<int64_t>(blockIdx.x) * p.tiles / gridDim.x);
  const int tile_hi = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * p.tiles / gridDim.x);
  const int cu = (tile_hi - tile_lo) * p.upt;
  const int act = min(kW, cu), base = cu / act, rem = cu % act;
  const int u_lo = tile_lo * p.upt + range_lo(min(warp, act), base, rem);
  const int u_hi = tile_lo * p.upt + range_lo(min(warp + 1, act), base, rem);
  const int tile0 = u_lo / p.upt;
  const int tu0 = u_lo - tile0 * p.upt;

  // ---- copy side. Weights: copy instruction i moves rows 2i and 2i+1 of the window, 256 contiguous
  // bytes each (lane: row 2i + (lane >> 4), 16-byte chunk k = lane & 15), which DRAM serves at
  // close to copy bandwidth. Chunk k of row r goes to chunk k ^ f(r): for r = 2i + h that is
  // (k ^ 5h) ^ 2 (i & 3), so the four destinations e[i & 3] + 512 i are fixed per lane.
  // Scales: lane l < kScopies copies part l % kSparts of row l / kSparts. Packed zero points:
  // lane l < 16 copies row l.
  const int wh = lane >> 4, wk = lane & 15;
  uint32_t w_dst[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) w_dst[j] = wh * kPitch + 16u * static_cast<uint32_t>((wk ^ (5 * wh)) ^ (2 * j));
  const int w_unit = wk >> 2;  // unit of the window this lane's chunk belongs to
  const int srow = lane / G::kSparts, spart = lane % G::kSparts;
  int is_tile = tile0, is_tu = tu0, is_slot = 0;
  int is_left = u_hi - u_lo;  // units still to request
  const uint8_t *w_src = nullptr, *s_src = nullptr, *z_src = nullptr;
  auto set_tile = [&](int tile) {
    const int nbase = tile * kRows;
    w_src = p.b + static_cast<int64_t>(nbase + wh) * (p.K / 2) + 16 * wk;
    s_src = reinterpret_cast<const uint8_t*>(p.scales) + static_cast<int64_t>(min(nbase + srow, p.N - 1)) * p.kb * 2 +
            spart * G::kScs;
    if (ZM == kZPacked)
      z_src = reinterpret_cast<const uint8_t*>(p.zp) + static_cast<int64_t>(min(nbase + lane, p.N - 1)) * p.zrow;
  };
  if (is_left > 0) set_tile(is_tile);
  auto issue = [&]() {
    if (is_left > 0) {
      const int win = is_tu >> 2, j0 = is_tu & 3;
      const int n = min(min(kWinUnits - j0, p.upt - is_tu), is_left);
      const uint32_t slot = s_ring + is_slot * p.slot_bytes;
      if (w_unit >= j0 && w_unit < j0 + n) {  // this lane's chunk is in the stage
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
      if (lane < G::kScopies)
        cp_async_n<G::kScs>(slot + kStageWBytes + srow * G::kSb + spart * G::kScs, s_src + win * G::kSb);
      if (ZM == kZPacked && lane < kRows)
        cp_async_n<G::kZbPacked>(slot + kStageWBytes + kRows * G::kSb + lane * G::kZbPacked,
                                 z_src + win * G::kZbPacked);
      if (ZM == kZFloat) {  // zb = 2 or 4 bytes x blocks per window, per row
        const int zcs = p.zb < 16 ? p.zb : 16, zparts = p.zb / zcs;
        const int64_t zstride = static_cast<int64_t>(p.kb) * (p.zp_f32 ? 4 : 2);
        for (int e = lane; e < kRows * zparts; e += 32) {
          const int r = e / zparts, part = e - r * zparts;
          cp_async_small(slot + kStageWBytes + kRows * G::kSb + r * p.zb + part * zcs,
                         reinterpret_cast<const uint8_t*>(p.zp) + min(is_tile * kRows + r, p.N - 1) * zstride +
                             static_cast<int64_t>(win) * p.zb + part * zcs,
                         zcs);
        }
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

  // Programmatic dependent launch: the first stage of weights and metadata is requested before
  // griddepcontrol.wait; the activations, the workspace and the output only after it.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#pragma unroll
  for (int j = 0; j < kNst - 1; ++j) issue();
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Sharded form: this call's epoch, one past the value the previous call's receive left (read
  // only now, after the previous kernel in the stream has completed).
  const bool pushing = p.push.world > 1;
  const uint32_t push_e = pushing ? ld_volatile_u32(p.push.epoch) + 1u : 0u;

  for (int i = threadIdx.x; i < kZeroRegion / 16; i += kThreads) sts128(s_base + 16 * i, make_uint4(0u, 0u, 0u, 0u));
  {  // Activations: up to eight 16-byte loads per thread are in flight before any is used, so staging
     // costs one L2 round trip for K <= 8 * 8 * kThreads.
    constexpr int kBatch = 8;
    const int groups16 = p.K / 8;
    for (int base = 0; base < groups16; base += kThreads * kBatch) {
      uint4 v[kBatch];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int idx = base + j * kThreads + static_cast<int>(threadIdx.x);
        v[j] = idx < groups16 ? __ldg(reinterpret_cast<const uint4*>(p.x) + idx) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        if (base + j * kThreads >= groups16) break;  // warp-uniform: groups16 is a multiple of 64
        const int idx = base + j * kThreads + static_cast<int>(threadIdx.x);
        float sum = (hsum2(v[j].x) + hsum2(v[j].y)) + (hsum2(v[j].z) + hsum2(v[j].w));
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if (idx < groups16) {
          sts128(s_x + 16 * idx, make_uint4(prmt(v[j].x, v[j].z, 0x5410), prmt(v[j].y, v[j].w, 0x5410),
                                            prmt(v[j].x, v[j].z, 0x7632), prmt(v[j].y, v[j].w, 0x7632)));
          if ((idx & 3) == 0) {
            const int chunk = idx >> 2, unit = chunk >> 2, cc = chunk & 3;  // unit = 4 win + jl
            const uint32_t at = s_sums + 4u * (((unit >> 2) * 4 + cc) * 4 + (unit & 3));
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(at), "f"(sum * 5.9604644775390625e-8f) : "memory");
          }
        }
      }
    }
  }
  __syncthreads();

  // ---- compute side. Lane 9c (g == 2c) carries the activations of lane c's chunk into B column
  // 2c; the other lanes read zeros two 16-byte slots away from the carrier of their 8-lane phase.
  const bool carrier = g == 2 * c;
  const uint32_t x_lane = carrier ? s_x + 64 * c : s_base + ((64 * (lane >> 3) + 32) & 127);
  const uint32_t x_win = carrier ? 1024u : 0u;
  const uint32_t w_lane = g * kPitch + 16u * static_cast<uint32_t>(c ^ row_swizzle(g));  // row g+8: same swizzle
  const uint32_t s_lane = g * G::kSb + 2 * ((32 * c) / BS);  // (32 c) / BS: 0 unless BS == 32 or 64

  auto consume = [&](uint32_t slot, int win, int j0, int n, float& tot0, float& tot1) {
    const uint32_t sslot = slot + kStageWBytes, zslot = sslot + kRows * G::kSb;
    const float4 sx4 = lds128f(s_sums + 64u * win + 16u * c);
    const float sx[4] = {sx4.x, sx4.y, sx4.z, sx4.w};
    const uint32_t xa = x_lane + win * x_win;
    const uint32_t wl = slot + w_lane;
#pragma unroll
    for (int jl = 0; jl < kWinUnits; ++jl) {
      if (jl < j0 || jl >= j0 + n) continue;
      const uint32_t wad = wl ^ (64u * jl);
      const uint4 wa = lds128(wad), wb = lds128(wad + 8 * kPitch);
      const uint32_t a[4] = {wa.x, wa.y, wa.z, wa.w}, b[4] = {wb.x, wb.y, wb.z, wb.w};
      float lo[4], hi[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const uint4 xv = lds128(xa + 256 * jl + 16 * w);
        const uint32_t a8 = a[w] >> 8, b8 = b[w] >> 8;
        if (w == 0) {
          mma_f16_first(lo, a[w] & 0x000F000Fu, b[w] & 0x000F000Fu, a8 & 0x000F000Fu, b8 & 0x000F000Fu, xv.x, xv.y);
          mma_f16_first(hi, a[w] & 0x00F000F0u, b[w] & 0x00F000F0u, a8 & 0x00F000F0u, b8 & 0x00F000F0u, xv.z, xv.w);
        } else {
          mma_f16(lo, a[w] & 0x000F000Fu, b[w] & 0x000F000Fu, a8 & 0x000F000Fu, b8 & 0x000F000Fu, xv.x, xv.y);
          mma_f16(hi, a[w] & 0x00F000F0u, b[w] & 0x00F000F0u, a8 & 0x00F000F0u, b8 & 0x00F000F0u, xv.z, xv.w);
        }
      }
      // Block of lane c's chunk: (128 jl + 32 c) / BS of the window.
      const int blk = (kUnitK * jl + 32 * c) / BS;
      const uint32_t soff = s_lane + 2 * ((kUnitK * jl) / BS);
      const float sa = half_lo(lds_u16(sslot + soff)), sbv = half_lo(lds_u16(sslot + soff + 8 * G::kSb));
      float za = 8.f, zb = 8.f;
      if (ZM == kZPacked) {
        const uint32_t zo = g * G::kZbPacked + (blk >> 1), sh = 4 * (blk & 1);
        za = nibble_f((lds_u8(zslot + zo) >> sh) & 15u);
        zb = nibble_f((lds_u8(zslot + zo + 8 * G::kZbPacked) >> sh) & 15u);
      }
      if (ZM == kZFloat) {
        const uint32_t ra = zslot + g * p.zb + (p.zp_f32 ? 4 : 2) * blk, rb = ra + 8 * p.zb;
        za = p.zp_f32 ? __uint_as_float(lds_u32(ra)) : half_lo(lds_u16(ra));
        zb = p.zp_f32 ? __uint_as_float(lds_u32(rb)) : half_lo(lds_u16(rb));
      }
      const float va = fmaf(hi[0], 0.0625f, lo[0]), vb = fmaf(hi[2], 0.0625f, lo[2]);
      tot0 = fmaf(sa, fmaf(-za, sx[jl], va), tot0);
      tot1 = fmaf(sbv, fmaf(-zb, sx[jl], vb), tot1);
    }
  };

  // Output column n from its scaled sum: float16 bits (bias added for columns inside N).
  auto half_bits = [&](int n, float v) -> uint32_t {
    v *= 16777216.f;  // 2^24
    if (p.bias && n < p.N) v += __half2float(p.bias[n]);
    return __half_as_ushort(__float2half_rn(v));
  };
  auto put = [&](int n, uint32_t h) {
    if (n < p.N) p.y[n] = __ushort_as_half(static_cast<unsigned short>(h));
  };
  // A finished segment of this warp's range inside `tile`: stored directly when the warp covered
  // the whole tile, otherwise kept in shared memory (slot 0: the warp's first tile, 1: its last)
  // for the fixed-order sum at the end of the CTA.
  auto emit = [&](int tile, bool whole, bool first, float tot0, float tot1) {
    tot0 += __shfl_xor_sync(0xffffffffu, tot0, 1);
    tot0 += __shfl_xor_sync(0xffffffffu, tot0, 2);
    tot1 += __shfl_xor_sync(0xffffffffu, tot1, 1);
    tot1 += __shfl_xor_sync(0xffffffffu, tot1, 2);
    if (whole) {
      const int n0 = tile * kRows + g;
      const uint32_t h0 = half_bits(n0, tot0), h1 = half_bits(n0 + 8, tot1);
      if (c == 0) {
        put(n0, h0);
        put(n0 + 8, h1);
      }
      if (pushing) {  // lane 4g + 4 holds column g + 1 (and g + 9)
        const uint32_t o0 = __shfl_down_sync(0xffffffffu, h0, 4), o1 = __shfl_down_sync(0xffffffffu, h1, 4);
        if (c == 0 && (g & 1) == 0) {
          push_pair(p.push, push_e, n0, h0 | (o0 << 16));
          push_pair(p.push, push_e, n0 + 8, h1 | (o1 << 16));
        }
      }
    } else if (c == 0) {
      float* mine = red + (warp * 2 + (first ? 0 : 1)) * kRows;
      mine[g] = tot0;
      mine[g + 8] = tot1;
    }
  };
  // Tile `tile` of this CTA was cut between warps qa..qb: the last of them adds the parts in order.
  auto finish = [&](int tile) {
    const int t0 = (tile - tile_lo) * p.upt;
    const int qa = owner_of(t0, base, rem), qb = owner_of(t0 + p.upt - 1, base, rem);
    if (qb != warp || qa == qb) return;
    const int qa_slot = range_lo(qa, base, rem) < t0 ? 1 : 0;  // the tile is qa's last when qa began before it
    float v = 0.f;
    if (lane < kRows)
      for (int qq = qa; qq <= qb; ++qq) v += red[(qq * 2 + (qq == qa ? qa_slot : 0)) * kRows + lane];
    const int n = tile * kRows + lane;
    const uint32_t h = half_bits(n, v);
    if (lane < kRows) put(n, h);
    if (pushing) {
      const uint32_t o = __shfl_down_sync(0xffffffffu, h, 1);
      if (lane < kRows && (lane & 1) == 0) push_pair(p.push, push_e, n, h | (o << 16));
    }
  };

  int left = u_hi - u_lo;
  int tile = tile0, tu = tu0, seg0 = tu0, slot_i = 0;
  bool first = true;
  float tot0 = 0.f, tot1 = 0.f;
  while (left > 0) {
    const int win = tu >> 2, j0 = tu & 3;
    const int n = min(min(kWinUnits - j0, p.upt - tu), left);
    cp_async_wait<kNst - 2>();
    __syncwarp();
    issue();  // refills the slot read in the previous step
    consume(s_ring + slot_i * p.slot_bytes, win, j0, n, tot0, tot1);
    if (++slot_i == kNst) slot_i = 0;
    left -= n;
    tu += n;
    if (tu == p.upt || left == 0) {
      emit(tile, seg0 == 0 && tu == p.upt, first, tot0, tot1);
      first = false;
      tot0 = tot1 = 0.f;
      seg0 = 0;
      tu = 0;
      ++tile;
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  if (u_lo < u_hi) {
    finish(tile0);                                  // the warp's first tile
    const int last = (u_hi - 1) / p.upt;
    if (last != tile0) finish(last);                // and its last
  }
}

int staged_grid(const Problem& p) {
  // One CTA per SM, each a contiguous range of tiles.
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(device_sm_count(), ceil_div(p.N, kRows))));
}

int meta_bytes_per_window(int64_t bs, int zp, int* sb, int* zb) {
  const int64_t win_k = kWinUnits * kUnitK;
  *sb = static_cast<int>(2 * win_k / bs);
  *zb = zp == kZpPacked ? static_cast<int>(win_k / bs / 2)
                        : (zp == kZpF32 ? static_cast<int>(4 * win_k / bs) : (zp == kZpF16 ? static_cast<int>(2 * win_k / bs) : 0));
  return kRows * (*sb + *zb);
}

size_t staged_smem(const Problem& p) {
  int sb = 0, zb = 0;
  const int slot = (kStageWBytes + meta_bytes_per_window(p.bs, p.zp, &sb, &zb) + 255) & ~255;
  return static_cast<size_t>(ring_offset(static_cast<int>(p.K))) + static_cast<size_t>(kW) * kNst * slot;
}

template <int BS, int ZM>
cudaError_t launch_staged_variant(const StagedParams& gp, int grid, size_t smem, cudaStream_t stream) {
  // The dynamic shared-memory limit is raised to the maximum once per device (a host call per
  // launch would add microseconds to every decode step launched eagerly).
  static std::atomic<uint64_t> raised{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
  if (smem > 48 * 1024 && !(raised.load(std::memory_order_acquire) & bit)) {
    const cudaError_t e = cudaFuncSetAttribute(gemv_staged_kernel<BS, ZM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kMaxSmem);
    if (e != cudaSuccess) return e;
    raised.fetch_or(bit, std::memory_order_acq_rel);
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, gemv_staged_kernel<BS, ZM>, gp);
}

template <int BS>
cudaError_t launch_staged_bs(const Problem& p, const StagedParams& gp, int grid, size_t smem, cudaStream_t stream) {
  if (p.zp == kZpNone) return launch_staged_variant<BS, kZDefault>(gp, grid, smem, stream);
  if (p.zp == kZpPacked) {
    if constexpr (BS <= 64) return launch_staged_variant<BS, kZPacked>(gp, grid, smem, stream);
    return cudaErrorInvalidValue;  // excluded by gemv_staged_supported
  }
  return launch_staged_variant<BS, kZFloat>(gp, grid, smem, stream);
}

}  // namespace

bool gemv_staged_supported(const Problem& p) {
  if (!(p.f16 && p.bits == 4 && p.M == 1 && p.bs >= 32 && p.bs <= 256 && (p.bs & (p.bs - 1)) == 0 &&
        p.K % (kWinUnits * kUnitK) == 0 && p.N >= 1 && p.N * (p.K / 2) < (1ll << 31) && p.N * p.kb < (1ll << 31) &&
        (reinterpret_cast<uintptr_t>(p.b) % 16) == 0 && (reinterpret_cast<uintptr_t>(p.a) % 16) == 0 &&
        (reinterpret_cast<uintptr_t>(p.scales) % 16) == 0))
    return false;
  if (p.zp == kZpPacked && (p.bs > 64 || (reinterpret_cast<uintptr_t>(p.zp_ptr) % 8) != 0)) return false;
  if ((p.zp == kZpF16 || p.zp == kZpF32) && (reinterpret_cast<uintptr_t>(p.zp_ptr) % 16) != 0) return false;
  return staged_smem(p) <= static_cast<size_t>(kMaxSmem);
}

cudaError_t launch_gemv_staged(const Problem& p, cudaStream_t stream) { return launch_gemv_staged_push(p, nullptr, stream); }

cudaError_t launch_gemv_staged_push(const Problem& p, const StagedPush* push, cudaStream_t stream) {
  if (p.N == 0) return cudaSuccess;
  const int grid = staged_grid(p);
  StagedParams gp{};
  gp.x = static_cast<const __half*>(p.a);
  gp.b = p.b;
  gp.scales = static_cast<const __half*>(p.scales);
  gp.zp = p.zp_ptr;
  gp.bias = static_cast<const __half*>(p.bias);
  gp.y = static_cast<__half*>(p.y);
  gp.K = static_cast<int>(p.K);
  gp.N = static_cast<int>(p.N);
  gp.kb = static_cast<int>(p.kb);
  gp.zp_f32 = p.zp == kZpF32;
  gp.zrow = static_cast<int>((p.kb + 1) / 2);
  gp.tiles = static_cast<int>(ceil_div(p.N, kRows));
  gp.upt = static_cast<int>(p.K / kUnitK);
  int sb = 0, zb = 0;
  const int meta = meta_bytes_per_window(p.bs, p.zp, &sb, &zb);
  gp.sb = sb;
  gp.zb = zb;
  gp.slot_bytes = (kStageWBytes + meta + 255) & ~255;
  if (push) gp.push = *push;
  const size_t smem = staged_smem(p);
  switch (p.bs) {
    case 32: return launch_staged_bs<32>(p, gp, grid, smem, stream);
    case 64: return launch_staged_bs<64>(p, gp, grid, smem, stream);
    case 128: return launch_staged_bs<128>(p, gp, grid, smem, stream);
    default: return launch_staged_bs<256>(p, gp, grid, smem, stream);
  }
}

}  // namespace xrgpu
