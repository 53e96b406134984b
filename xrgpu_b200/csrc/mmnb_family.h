// Device-pointer problems and launchers of the MatMulNBits family kernels (mmnb_family.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace xrgpu {

// packedInput's normalisation (complex_kernel.glsl:81): x = (a + skip) * (1/sqrt(mean + eps) * ns[k]).
// norm_scale == nullptr: x = a + skip (no normalisation). residual (optional) receives a + skip.
struct NormProblem {
  int f16;
  int64_t M, K;
  float epsilon;
  const void* a;
  const void* skip;        // [M, K] or nullptr
  const void* norm_scale;  // [K] or nullptr
  void* x;                 // [M, K]
  void* residual;          // [M, K] or nullptr
};
cudaError_t launch_norm_rows(const NormProblem& p, cudaStream_t s);

// y[i] = fused(g[i], act) * u[i] over `count` elements (the 1027 branch of packedMatmul).
cudaError_t launch_mlp_combine(const void* g, const void* u, void* y, int64_t count, int f16, int act, cudaStream_t s);

// MatMulBnb4 (transB = 1): y[m, n] = sum_k a[m, k] * table[code(n*K + k)] * absmax[(n*K + k) / block_size].
struct Bnb4Problem {
  int f16, quant_type, vector_ok;
  int64_t M, K, N, block_size;
  const void* a;
  const uint8_t* b;      // [ceil(N*K/2)]
  const void* absmax;    // [ceil(N*K/block_size)]
  void* y;               // [M, N]
};
cudaError_t launch_bnb4(const Bnb4Problem& p, cudaStream_t s);

// GatherBlockQuantized (gather_axis 0, quantize_axis 1): out[r, j] = (q - z) * scales[sel, j / bs].
struct GatherProblem {
  int bits, idx64;
  int64_t rows, row_bytes, width, blocks, zp_row, block_size, count;
  const uint8_t* data;         // [rows, row_bytes]
  const void* indices;         // [count] int32 or int64
  const float* scales;         // [rows, blocks]
  const uint8_t* zero_points;  // [rows, zp_row] or nullptr
  float* out;                  // [count, width]
  unsigned* err;               // device error word (code 55: index out of range)
};
cudaError_t launch_gather_quant(const GatherProblem& p, cudaStream_t s);

// QMoE (opcode 1030), float32.
struct QmoeProblem {
  int bits, act, swiglu_fusion, has_limit;
  int64_t tokens, hidden, experts, k, fc1_rows, inter, block_size, fc1_spr, fc2_spr;
  float alpha, beta, swiglu_limit;
  const float* x;            // [tokens, hidden]
  const float* router;       // [tokens, experts]
  const uint8_t* fc1;        // [experts, fc1_rows, ceil(hidden*bits/8)]
  const float* fc1_scales;   // [experts, fc1_rows(, blocks)]
  const uint8_t* fc2;        // [experts, hidden, ceil(inter*bits/8)]
  const float* fc2_scales;   // [experts, hidden(, blocks)]
  float* out;                // [tokens, hidden]
  int32_t* route_expert;     // scratch [tokens, k]
  float* route_weight;       // scratch [tokens, k]
  float* act_buf;            // scratch [tokens, k, inter]
};
cudaError_t launch_qmoe(const QmoeProblem& p, cudaStream_t s);

}  // namespace xrgpu
