// Generic MatMulNBits kernel and the exact float32 dequantization kernel.
//
// The generic kernel covers every contract-legal configuration (bits 2/4/8, any power-of-two
// block size, tail K, float32 or float16 activations, every zero-point form, bias). It
// restates packedMatmul (complex_kernel.glsl:83) with the k loop split across a warp's lanes
// and float32 accumulation; each dequantized weight is nbitWeight (complex_kernel.glsl:80).
#include <cuda_fp16.h>

#include <algorithm>

#include "mmnb_common.cuh"

namespace xrgpu {

namespace {
__device__ unsigned int g_device_error = 0;
}  // namespace

unsigned* device_error_word() {
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, g_device_error) != cudaSuccess) return nullptr;
  return static_cast<unsigned*>(ptr);
}

namespace {

constexpr int kGenericRows = 8;   // output rows per warp
constexpr int kGenericWarps = 8;  // columns per CTA

// One dequantized weight, exactly as nbitWeight: (float(q) - z) * s in two float32 roundings.
__device__ __forceinline__ float nbit_weight(const Problem& p, const uint8_t* col_bytes, int64_t n, int64_t k) {
  const int64_t blk = k / p.bs, e = k - blk * p.bs;
  const uint32_t packed = col_bytes[blk * p.blob + (e * p.bits) / 8];
  const uint32_t q = (packed >> ((e * p.bits) % 8)) & ((1u << p.bits) - 1u);
  const float z = load_zero_point(p, n, blk);
  const float s = load_f(p.scales, p.f16, n * p.kb + blk);
  return __fmul_rn(__fsub_rn(static_cast<float>(q), z), s);
}

__global__ void __launch_bounds__(kGenericWarps * 32) generic_kernel(Problem p) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = static_cast<int64_t>(blockIdx.x) * kGenericWarps + warp;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kGenericRows;
  if (n >= p.N) return;
  const uint8_t* col_bytes = p.b + n * p.kb * p.blob;
  const int rows = static_cast<int>(p.M - m0 < kGenericRows ? p.M - m0 : kGenericRows);
  float acc[kGenericRows];
#pragma unroll
  for (int r = 0; r < kGenericRows; ++r) acc[r] = 0.f;
  for (int64_t k = lane; k < p.K; k += 32) {
    const float w = nbit_weight(p, col_bytes, n, k);
#pragma unroll
    for (int r = 0; r < kGenericRows; ++r)
      if (r < rows) acc[r] = fmaf(load_f(p.a, p.f16, (m0 + r) * p.K + k), w, acc[r]);
  }
#pragma unroll
  for (int r = 0; r < kGenericRows; ++r) {
    float v = acc[r];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    acc[r] = v;
  }
  if (lane == 0) {
    const float bias = p.bias ? load_f(p.bias, p.f16, n) : 0.f;
    for (int r = 0; r < rows; ++r) {
      const float v = acc[r] + bias;
      const int64_t o = (m0 + r) * p.ldy + n;
      if (p.f16) reinterpret_cast<__half*>(p.y)[o] = __float2half_rn(v);
      else reinterpret_cast<float*>(p.y)[o] = v;
    }
  }
}

__global__ void dequant_kernel(Problem p, float* __restrict__ w) {
  const int64_t total = p.N * p.K;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t n = i / p.K, k = i - n * p.K;
    w[i] = nbit_weight(p, p.b + n * p.kb * p.blob, n, k);
  }
}

}  // namespace

cudaError_t launch_generic(const Problem& p, cudaStream_t s) {
  if (p.M == 0 || p.N == 0) return cudaSuccess;
  const int64_t gx = ceil_div(p.N, kGenericWarps), gy = ceil_div(p.M, kGenericRows);
  if (gx > 0x7fffffff || gy > 65535) return cudaErrorInvalidConfiguration;
  generic_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), kGenericWarps * 32, 0, s>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_dequant(const Problem& p, float* w, cudaStream_t s) {
  if (p.N == 0 || p.K == 0) return cudaSuccess;
  const int64_t total = p.N * p.K;
  const int64_t blocks = std::min<int64_t>(ceil_div(total, 256), static_cast<int64_t>(device_sm_count()) * 16);
  dequant_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(p, w);
  return cudaGetLastError();
}

cudaError_t read_device_error(uint32_t* code, bool clear) {
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v));
  if (e != cudaSuccess) return e;
  if (code) *code = v;
  if (clear && v) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(zero));
  }
  return e;
}

}  // namespace xrgpu
