// Kernels of the operators that call or share MatMulNBits' quantized formats (sm_100a):
//   * the normalisation prologue of MatMulNBitsQkv (1028) / MatMulNBitsMlp (1027):
//     packedInput, complex_kernel.glsl:81 -- h = a + skip, residual = h,
//     x = h * (1 / sqrt(sum(h^2) / K + eps) * normScale[k]); the projections then run on x through
//     the MatMulNBits kernels (GEMV / tcgen05 GEMM / generic);
//   * the Mlp combine, packedMatmul's 1027 branch (complex_kernel.glsl:83):
//     y = fused(gate + gateBias) * (up + upBias), fused = complex_kernel.glsl:41-47;
//   * MatMulBnb4 (1026): bnbWeight, complex_kernel.glsl:82 (NF4 / FP4 codebooks, high nibble first,
//     absmax per block of flat weight indices);
//   * GatherBlockQuantized (1031): gatherQuant, complex_kernel.glsl:85 (an out-of-range index records
//     code 55 in the device error word and leaves its row zero, like the reference's fail(55));
//   * QMoE (1030): moe / expertRank / expertWeight, complex_kernel.glsl:158-160 (top-k by the rank
//     rule, softmax over the chosen experts, symmetric int4/int8 expert weights).
// Every kernel accumulates in float32 and stores in the output's dtype with one rounding.
#include <cuda_fp16.h>

#include <cstdint>

#include "mmnb_common.cuh"
#include "mmnb_family.h"

namespace xrgpu {
namespace {

__device__ __forceinline__ void store_f(void* p, int f16, int64_t i, float v) {
  if (f16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// logistic and fused as complex_kernel.glsl:39-47 (gelu: erf form for 1027, tanh form otherwise).
__device__ __forceinline__ float logistic_f(float x) {
  return x >= 0.f ? 1.f / (1.f + expf(-x)) : expf(x) / (1.f + expf(x));
}
__device__ __forceinline__ float fused_f(float x, int kind, int gelu_erf) {
  switch (kind) {
    case 1: return fmaxf(x, 0.f);
    case 2: return x * logistic_f(x);
    case 3:
      return gelu_erf ? 0.5f * x * (1.f + erff(x * 0.7071067811865475f))
                      : 0.5f * x * (1.f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x)));
    case 4: return tanhf(x);
    case 5: return logistic_f(x);
    default: return x;
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x == 0) {
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];  // fixed order
    red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// ---------------------------------------------------------------- normalisation prologue
__global__ void __launch_bounds__(256) norm_rows_kernel(const NormProblem p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float red[33];
  const int64_t row = blockIdx.x;
  const int64_t base = row * p.K;
  float sq = 0.f;
  for (int64_t k = threadIdx.x; k < p.K; k += blockDim.x) {
    float h = load_f(p.a, p.f16, base + k);
    if (p.skip) h = h + load_f(p.skip, p.f16, base + k);  // one float32 add (packedInput)
    if (p.residual) store_f(p.residual, p.f16, base + k, h);
    if (!p.norm_scale) {
      store_f(p.x, p.f16, base + k, h);
    } else {
      sq = fmaf(h, h, sq);
    }
  }
  if (!p.norm_scale) return;
  const float total = block_sum(sq, red);
  const float inv = 1.f / sqrtf(total / static_cast<float>(p.K) + p.epsilon);
  for (int64_t k = threadIdx.x; k < p.K; k += blockDim.x) {
    float h = load_f(p.a, p.f16, base + k);
    if (p.skip) h = h + load_f(p.skip, p.f16, base + k);
    store_f(p.x, p.f16, base + k, h * (inv * load_f(p.norm_scale, p.f16, k)));
  }
}

// ---------------------------------------------------------------- Mlp combine
__global__ void mlp_combine_kernel(const void* g, const void* u, void* y, int64_t count, int f16, int act) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    store_f(y, f16, i, fused_f(load_f(g, f16, i), act, 1) * load_f(u, f16, i));
}

// ---------------------------------------------------------------- MatMulBnb4
__constant__ float kBnbTables[2][16] = {
    // FP4 (quant_type 0)
    {0.0f, 0.0052083333333333f, 0.6666666666666666f, 1.0f, 0.3333333333333333f, 0.5f, 0.1666666666666666f, 0.25f,
     -0.0f, -0.0052083333333333f, -0.6666666666666666f, -1.0f, -0.3333333333333333f, -0.5f, -0.1666666666666666f,
     -0.25f},
    // NF4 (quant_type 1)
    {-1.0f, -0.6961928009986877f, -0.5250730514526367f, -0.3949174880981445f, -0.28444138169288635f,
     -0.18477343022823334f, -0.09105003625154495f, 0.0f, 0.07958029955625534f, 0.16093020141124725f,
     0.24611230194568634f, 0.33791524171829224f, 0.44070982933044434f, 0.5626170039176941f, 0.7229568362236023f,
     1.0f}};

constexpr int kBnbRows = 8;  // activation rows per warp pass

// One warp per output column n (transB: weight index n*K + k), up to 8 activation rows per pass.
// Lanes take 32 consecutive codes (16 bytes) per step when rows are 16-byte aligned, else one code each.
__global__ void __launch_bounds__(256) bnb4_kernel(const Bnb4Problem p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float table[16];
  if (threadIdx.x < 16) table[threadIdx.x] = kBnbTables[p.quant_type == 1 ? 1 : 0][threadIdx.x];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (n >= p.N) return;
  const bool vec = p.vector_ok;
  for (int64_t m0 = 0; m0 < p.M; m0 += kBnbRows) {
    const int rows = static_cast<int>(p.M - m0 < kBnbRows ? p.M - m0 : kBnbRows);
    float acc[kBnbRows];
#pragma unroll
    for (int r = 0; r < kBnbRows; ++r) acc[r] = 0.f;
    if (vec) {  // K % 32 == 0: row n is K/2 whole bytes at offset n*K/2 (16-byte aligned)
      const uint4* row = reinterpret_cast<const uint4*>(p.b + n * (p.K / 2));
      for (int64_t c = lane; c < p.K / 32; c += 32) {
        const uint4 w = __ldg(row + c);
        const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
          for (int byte = 0; byte < 4; ++byte) {
            const uint32_t v = (words[wi] >> (8 * byte)) & 0xffu;
            const int64_t k = c * 32 + wi * 8 + byte * 2;  // codes k (high nibble) and k + 1 (low)
            const int64_t idx = n * p.K + k;
            const float w0 = table[v >> 4] * load_f(p.absmax, p.f16, idx / p.block_size);
            const float w1 = table[v & 15u] * load_f(p.absmax, p.f16, (idx + 1) / p.block_size);
#pragma unroll
            for (int r = 0; r < kBnbRows; ++r)
              if (r < rows) {
                const int64_t ab = (m0 + r) * p.K + k;
                acc[r] = fmaf(load_f(p.a, p.f16, ab), w0, acc[r]);
                acc[r] = fmaf(load_f(p.a, p.f16, ab + 1), w1, acc[r]);
              }
          }
        }
      }
    } else {
      for (int64_t k = lane; k < p.K; k += 32) {
        const int64_t idx = n * p.K + k;
        const uint32_t byte = p.b[idx / 2];
        const float w = table[(idx & 1) ? (byte & 15u) : (byte >> 4)] * load_f(p.absmax, p.f16, idx / p.block_size);
#pragma unroll
        for (int r = 0; r < kBnbRows; ++r)
          if (r < rows) acc[r] = fmaf(load_f(p.a, p.f16, (m0 + r) * p.K + k), w, acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kBnbRows; ++r) {
      float v = acc[r];
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0 && r < rows) store_f(p.y, p.f16, (m0 + r) * p.N + n, v);
    }
  }
}

// ---------------------------------------------------------------- GatherBlockQuantized
__device__ __forceinline__ int64_t load_index(const void* idx, int idx64, int64_t i) {
  if (!idx64) return reinterpret_cast<const int32_t*>(idx)[i];
  const int64_t v = reinterpret_cast<const int64_t*>(idx)[i];
  // controlIndex (complex_kernel.glsl:31) saturates 64-bit indices to the int32 range
  return v > 0x7fffffffll ? 0x7fffffffll : (v < -0x80000000ll ? -0x80000000ll : v);
}

// grid (gathered rows, column blocks); each thread writes one output value.
__global__ void __launch_bounds__(256) gather_quant_kernel(const GatherProblem p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t r = blockIdx.y;
  const int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (j >= p.width) return;
  const int64_t sel = load_index(p.indices, p.idx64, r);
  float out = 0.f;
  if (sel < 0 || sel >= p.rows) {
    if (j == 0) record_device_error(p.err, 55u);
  } else {
    const uint32_t mask = (1u << p.bits) - 1u;
    const uint32_t packed = p.data[sel * p.row_bytes + (j * p.bits) / 8];
    const uint32_t q = (packed >> ((j * p.bits) % 8)) & mask;
    const int64_t blk = j / p.block_size;
    uint32_t z = 1u << (p.bits - 1);
    if (p.zero_points) z = (p.zero_points[sel * p.zp_row + (blk * p.bits) / 8] >> ((blk * p.bits) % 8)) & mask;
    out = (static_cast<float>(q) - static_cast<float>(z)) * p.scales[sel * p.blocks + blk];
  }
  p.out[r * p.width + j] = out;
}

// ---------------------------------------------------------------- QMoE
// expertWeight for opcode 1030: (q - 2^(bits-1)) * scale, q packed low-first.
__device__ __forceinline__ float expert_weight(const uint8_t* w, const float* scales, int64_t scales_per_row, int bits,
                                               int64_t block_size, int64_t e, int64_t rows, int64_t row, int64_t cols,
                                               int64_t col) {
  const int64_t packed_cols = (cols * bits + 7) / 8;
  const uint32_t byte = w[(e * rows + row) * packed_cols + (col * bits) / 8];
  const uint32_t q = (byte >> ((col * bits) % 8)) & ((1u << bits) - 1u);
  const int64_t s = (e * rows + row) * scales_per_row + (scales_per_row > 1 ? col / (block_size > 0 ? block_size : 1) : 0);
  return (static_cast<float>(q) - static_cast<float>(1u << (bits - 1))) * scales[s];
}

// One warp per token: expertRank (ties rank the higher expert index first), softmax over the chosen.
__global__ void qmoe_route_kernel(const QmoeProblem p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= p.tokens) return;
  // Every slot starts empty: with NaN scores several experts can share a rank and some ranks stay
  // unused; an empty slot (-1) contributes nothing downstream.
  for (int64_t r = lane; r < p.k; r += 32) {
    p.route_expert[t * p.k + r] = -1;
    p.route_weight[t * p.k + r] = 0.f;
  }
  __syncwarp();
  const float* s = p.router + t * p.experts;
  float mx = __uint_as_float(0xff800000u);
  for (int64_t e = lane; e < p.experts; e += 32) {
    int64_t rank = 0;
    for (int64_t o = 0; o < p.experts; ++o) rank += (s[o] > s[e] || (s[o] == s[e] && o > e)) ? 1 : 0;
    if (rank < p.k) {
      p.route_expert[t * p.k + rank] = static_cast<int32_t>(e);
      mx = fmaxf(mx, s[e]);
    }
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  __syncwarp();
  if (lane == 0) {
    float den = 0.f;
    for (int64_t r = 0; r < p.k; ++r) {  // rank order
      const int32_t e = p.route_expert[t * p.k + r];
      if (e >= 0) den += expf(s[e] - mx);
    }
    for (int64_t r = 0; r < p.k; ++r) {
      const int32_t e = p.route_expert[t * p.k + r];
      if (e >= 0) p.route_weight[t * p.k + r] = expf(s[e] - mx) / den;
    }
  }
}

// One warp per (token, slot, intermediate j): fc1 row(s), then the activation.
__global__ void qmoe_fc1_kernel(const QmoeProblem p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t w_id = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const int64_t total = p.tokens * p.k * p.inter;
  if (w_id >= total) return;
  const int64_t j = w_id % p.inter, ts = w_id / p.inter, t = ts / p.k;
  const int64_t e = p.route_expert[ts];
  if (e < 0 || e >= p.experts) {  // an empty routing slot
    if (lane == 0) p.act_buf[ts * p.inter + j] = 0.f;
    return;
  }
  const bool swiglu = p.act == 6 && p.swiglu_fusion != 0;
  const int64_t gate_row = (p.act == 6 && p.swiglu_fusion == 1) ? 2 * j : j;
  const int64_t lin_row = p.swiglu_fusion == 1 ? 2 * j + 1 : p.inter + j;
  float g = 0.f, l = 0.f;
  for (int64_t c = lane; c < p.hidden; c += 32) {
    const float x = p.x[t * p.hidden + c];
    g = fmaf(x, expert_weight(p.fc1, p.fc1_scales, p.fc1_spr, p.bits, p.block_size, e, p.fc1_rows, gate_row, p.hidden, c), g);
    if (swiglu)
      l = fmaf(x, expert_weight(p.fc1, p.fc1_scales, p.fc1_spr, p.bits, p.block_size, e, p.fc1_rows, lin_row, p.hidden, c), l);
  }
  for (int o = 16; o > 0; o >>= 1) {
    g += __shfl_xor_sync(0xffffffffu, g, o);
    l += __shfl_xor_sync(0xffffffffu, l, o);
  }
  if (lane != 0) return;
  float a;
  if (p.act == 6) {
    if (p.has_limit) {
      g = fminf(g, p.swiglu_limit);
      l = fminf(fmaxf(l, -p.swiglu_limit), p.swiglu_limit);
    }
    a = g * logistic_f(p.alpha * g) * (l + p.beta);
  } else {
    a = fused_f(g, p.act, 0);
  }
  p.act_buf[ts * p.inter + j] = a;
}

// One warp per (token, output column): sum over the chosen experts in rank order.
__global__ void qmoe_fc2_kernel(const QmoeProblem p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int64_t w_id = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w_id >= p.tokens * p.hidden) return;
  const int64_t t = w_id / p.hidden, col = w_id % p.hidden;
  float result = 0.f;
  for (int64_t r = 0; r < p.k; ++r) {
    const int64_t ts = t * p.k + r, e = p.route_expert[ts];
    if (e < 0 || e >= p.experts) continue;  // an empty routing slot
    float v = 0.f;
    for (int64_t j = lane; j < p.inter; j += 32)
      v = fmaf(p.act_buf[ts * p.inter + j],
               expert_weight(p.fc2, p.fc2_scales, p.fc2_spr, p.bits, p.block_size, e, p.hidden, col, p.inter, j), v);
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    result = fmaf(p.route_weight[ts], v, result);
  }
  if (lane == 0) p.out[t * p.hidden + col] = result;
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, void** args, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace

cudaError_t launch_norm_rows(const NormProblem& p, cudaStream_t s) {
  if (p.M == 0 || p.K == 0) return cudaSuccess;
  NormProblem q = p;
  void* args[] = {&q};
  return launch_pdl(reinterpret_cast<const void*>(norm_rows_kernel), dim3(static_cast<unsigned>(p.M)), dim3(256), args, s);
}

cudaError_t launch_mlp_combine(const void* g, const void* u, void* y, int64_t count, int f16, int act, cudaStream_t s) {
  if (count == 0) return cudaSuccess;
  const int64_t blocks = (count + 255) / 256;
  unsigned grid = static_cast<unsigned>(blocks < 4096 ? blocks : 4096);
  void* args[] = {&g, &u, &y, &count, &f16, &act};
  return launch_pdl(reinterpret_cast<const void*>(mlp_combine_kernel), dim3(grid), dim3(256), args, s);
}

cudaError_t launch_bnb4(const Bnb4Problem& p, cudaStream_t s) {
  if (p.M == 0 || p.N == 0) return cudaSuccess;
  Bnb4Problem q = p;
  q.vector_ok = (p.K % 32 == 0) && (reinterpret_cast<uintptr_t>(p.b) % 16 == 0);
  void* args[] = {&q};
  const unsigned grid = static_cast<unsigned>((p.N + 7) / 8);
  return launch_pdl(reinterpret_cast<const void*>(bnb4_kernel), dim3(grid), dim3(256), args, s);
}

cudaError_t launch_gather_quant(const GatherProblem& p, cudaStream_t s) {
  if (p.count == 0 || p.width == 0) return cudaSuccess;
  GatherProblem q = p;
  void* args[] = {&q};
  const dim3 grid(static_cast<unsigned>((p.width + 255) / 256), static_cast<unsigned>(p.count));
  return launch_pdl(reinterpret_cast<const void*>(gather_quant_kernel), grid, dim3(256), args, s);
}

cudaError_t launch_qmoe(const QmoeProblem& p, cudaStream_t s) {
  if (p.tokens == 0) return cudaSuccess;
  QmoeProblem q = p;
  void* args[] = {&q};
  cudaError_t e = cudaSuccess;
  if (p.k > 0) {
    e = launch_pdl(reinterpret_cast<const void*>(qmoe_route_kernel), dim3(static_cast<unsigned>((p.tokens + 7) / 8)),
                   dim3(256), args, s);
    if (e != cudaSuccess) return e;
    if (p.inter > 0) {
      const int64_t warps = p.tokens * p.k * p.inter;
      e = launch_pdl(reinterpret_cast<const void*>(qmoe_fc1_kernel), dim3(static_cast<unsigned>((warps + 7) / 8)),
                     dim3(256), args, s);
      if (e != cudaSuccess) return e;
    }
  }
  const int64_t warps = p.tokens * p.hidden;
  if (p.k == 0 || p.inter == 0) {  // no chosen expert or an empty projection: output zeros
    return cudaMemsetAsync(p.out, 0, static_cast<size_t>(p.tokens * p.hidden) * sizeof(float), s);
  }
  return launch_pdl(reinterpret_cast<const void*>(qmoe_fc2_kernel), dim3(static_cast<unsigned>((warps + 7) / 8)),
                    dim3(256), args, s);
}

}  // namespace xrgpu
