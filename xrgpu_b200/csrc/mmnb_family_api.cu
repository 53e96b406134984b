// Host side of the operators around MatMulNBits: the zero-copy device API (xrgpu_mlp_forward,
// xrgpu_qkv_forward, xrgpu_bnb4_forward, xrgpu_gather_block_quantized_forward, xrgpu_qmoe_forward)
// and their plans for the operator API (xrgpu_plan_ex / xrgpu_prepare_ex, mmnb_api.cu).
//
// Planning follows the reference's plan_complex branches (kernels/_shared/extended/complex_plan.cpp):
//   1026-1028 (:117-120): K defaults to A's last dim, block_size to 32, bits to 4, quant_type to 1,
//     transB to 1, epsilon to 1e-5 (1e-6 for 1028), activation to "silu"; 1028 reads Nq and Nkv;
//     outputs replace A's last dim (residualT optional, A's shape);
//   1030 (:121-128): k 1, expert_weight_bits 4, block_size 0, activation_type "relu", swiglu_fusion 0,
//     activation_alpha 1, activation_beta 0, optional swiglu_limit; the geometry checks in order;
//   1031 (:129): bits 4, block_size 128, gather_axis 0, quantize_axis 1; output
//     [len(indices), cols * 8 / bits] in the scales' dtype;
// with the contracts' dtype and rank rules (kernels/<operation>/contract.json) checked up front.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

#include "mmnb_family.h"
#include "mmnb_family_ops.h"
#include "mmnb_internal.h"
#include "xrgpu_mmnb.h"

namespace xrgpu {
namespace {

int fail(int status, const std::string& m) { return api_fail(status, m); }

uint64_t al256(uint64_t v) { return (v + 255) / 256 * 256; }

int t1_code(int32_t dtype, int* f16) {
  if (dtype == XRGPU_FLOAT16) *f16 = 1;
  else if (dtype == XRGPU_FLOAT32) *f16 = 0;
  else return fail(XRGPU_INVALID_ARGUMENT, "T1 must be float32 or float16");
  return XRGPU_OK;
}

// One MatMulNBits projection without zero points (nbitWeight's default z = 2^(bits-1)), run by the
// planner's kernel.
Problem projection(int f16, int64_t M, int64_t K, int64_t N, int64_t bs, int64_t bits, const void* x, const uint8_t* b,
                   const void* scales, const void* bias, void* y) {
  Problem q{};
  q.f16 = f16;
  q.zp = kZpNone;
  q.M = M; q.K = K; q.N = N; q.bs = bs; q.bits = bits;
  q.kb = ceil_div(K, bs);
  q.blob = (bs * bits + 7) / 8;
  q.ldy = N;
  q.a = x; q.b = b; q.scales = scales; q.zp_ptr = nullptr; q.bias = bias; q.y = y;
  q.err = device_error_word();
  return q;
}

uint64_t projection_workspace(const Problem& p) {
  const int path = select_path(p, kPathAuto);
  return path < 0 ? 0 : workspace_for(p, path);
}

int run_projection(const Problem& p, void* ws, cudaStream_t s) {
  const int path = select_path(p, kPathAuto);
  const cudaError_t e = launch_path(p, path, ws, s);
  if (e != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, std::string("kernel launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

int launched(cudaError_t e) {
  if (e != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, std::string("kernel launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

int check_geometry(int64_t M, int64_t K, int64_t N, int64_t bs, int64_t bits) {
  if (M < 0 || K <= 0 || bs <= 0 || K > 0xffffffffll || N > 0xffffffffll)
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid packed matmul geometry");
  if (bits != 2 && bits != 4 && bits != 8) return fail(XRGPU_INVALID_ARGUMENT, "bits must be 2, 4 or 8");
  return XRGPU_OK;
}

// Workspace: [normalised x, M*K] [gate, M*N] [up, M*N] [projection scratch].
struct MlpLayout {
  uint64_t x = 0, g = 0, u = 0, proj = 0, total = 0;
  bool norm = false;
};
MlpLayout mlp_layout(const xrgpu_mlp_problem& c, int f16) {
  MlpLayout l;
  const uint64_t es = f16 ? 2 : 4;
  l.norm = c.skip || c.norm_scale;
  uint64_t at = 0;
  if (l.norm) { l.x = at; at += al256(static_cast<uint64_t>(c.M * c.K) * es); }
  l.g = at; at += al256(static_cast<uint64_t>(c.M * c.N) * es);
  l.u = at; at += al256(static_cast<uint64_t>(c.M * c.N) * es);
  l.proj = at;
  const Problem g = projection(f16, c.M, c.K, c.N, c.block_size, c.bits, c.a, c.gate_b, c.gate_scales, c.gate_bias, nullptr);
  at += al256(projection_workspace(g));
  l.total = at;
  return l;
}

int mlp_check(const xrgpu_mlp_problem* c, int* f16) {
  if (!c) return fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  int st = t1_code(c->dtype, f16);
  if (st) return st;
  if ((st = check_geometry(c->M, c->K, c->N, c->block_size, c->bits))) return st;
  if (c->N <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Packed matmul N required");
  if (c->activation < XRGPU_ACT_NONE || c->activation > XRGPU_ACT_SWIGLU) return fail(XRGPU_INVALID_ARGUMENT, "Unknown fused activation");
  if (c->M > 0 && (!c->a || !c->y)) return fail(XRGPU_INVALID_ARGUMENT, "null tensor pointer");
  if (!c->gate_b || !c->gate_scales || !c->up_b || !c->up_scales) return fail(XRGPU_INVALID_ARGUMENT, "null weight pointer");
  return XRGPU_OK;
}

int resolve_workspace(uint64_t need, void* given, uint64_t given_bytes, void** out) {
  *out = given;
  if (!need) return XRGPU_OK;
  if (!given) return library_workspace(need, out);
  if (given_bytes < need) return fail(XRGPU_INVALID_ARGUMENT, "workspace too small: need " + std::to_string(need) + " bytes");
  return XRGPU_OK;
}

}  // namespace

// ---------------------------------------------------------------- forwards (shared with the operator API)
int mlp_forward(const xrgpu_mlp_problem& c, void* ws, uint64_t ws_bytes, cudaStream_t s) {
  int f16 = 0;
  int st = mlp_check(&c, &f16);
  if (st) return st;
  if (c.M == 0) return XRGPU_OK;
  const MlpLayout l = mlp_layout(c, f16);
  void* base = nullptr;
  if ((st = resolve_workspace(l.total, ws, ws_bytes, &base))) return st;
  char* w = static_cast<char*>(base);
  const void* x = c.a;
  if (l.norm) {
    NormProblem n{f16, c.M, c.K, c.epsilon, c.a, c.skip, c.norm_scale, w + l.x, c.residual};
    if ((st = launched(launch_norm_rows(n, s)))) return st;
    x = w + l.x;
  } else if (c.residual) {  // residual = a + 0
    if ((st = launched(cudaMemcpyAsync(c.residual, c.a, static_cast<size_t>(c.M * c.K) * (f16 ? 2 : 4),
                                       cudaMemcpyDeviceToDevice, s))))
      return st;
  }
  const Problem g = projection(f16, c.M, c.K, c.N, c.block_size, c.bits, x, c.gate_b, c.gate_scales, c.gate_bias, w + l.g);
  const Problem u = projection(f16, c.M, c.K, c.N, c.block_size, c.bits, x, c.up_b, c.up_scales, c.up_bias, w + l.u);
  if ((st = run_projection(g, w + l.proj, s)) || (st = run_projection(u, w + l.proj, s))) return st;
  return launched(launch_mlp_combine(w + l.g, w + l.u, c.y, c.M * c.N, f16, c.activation, s));
}

uint64_t qkv_workspace(const xrgpu_qkv_problem& c, int f16) {
  const uint64_t es = f16 ? 2 : 4;
  uint64_t at = al256(static_cast<uint64_t>(c.M * c.K) * es);
  uint64_t proj = 0;
  const int64_t ns[3] = {c.Nq, c.Nkv, c.Nkv};
  for (int64_t n : ns)
    if (n > 0) proj = std::max(proj, projection_workspace(projection(f16, c.M, c.K, n, c.block_size, c.bits, nullptr,
                                                                     c.q_b, c.q_scales, nullptr, nullptr)));
  return at + al256(proj);
}

int qkv_check(const xrgpu_qkv_problem* c, int* f16) {
  if (!c) return fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  int st = t1_code(c->dtype, f16);
  if (st) return st;
  if ((st = check_geometry(c->M, c->K, std::max(c->Nq, c->Nkv), c->block_size, c->bits))) return st;
  if (c->Nq < 0 || c->Nkv < 0) return fail(XRGPU_INVALID_ARGUMENT, "Nq and Nkv must be >= 0");
  if (!c->norm_scale) return fail(XRGPU_INVALID_ARGUMENT, "Missing complex input: normScaleT");
  if (c->M > 0 && (!c->a || (c->Nq && !c->q) || (c->Nkv && (!c->k || !c->v))))
    return fail(XRGPU_INVALID_ARGUMENT, "null tensor pointer");
  if ((c->Nq && (!c->q_b || !c->q_scales)) || (c->Nkv && (!c->k_b || !c->k_scales || !c->v_b || !c->v_scales)))
    return fail(XRGPU_INVALID_ARGUMENT, "null weight pointer");
  return XRGPU_OK;
}

int qkv_forward(const xrgpu_qkv_problem& c, void* ws, uint64_t ws_bytes, cudaStream_t s) {
  int f16 = 0;
  int st = qkv_check(&c, &f16);
  if (st) return st;
  if (c.M == 0) return XRGPU_OK;
  const uint64_t need = qkv_workspace(c, f16);
  void* base = nullptr;
  if ((st = resolve_workspace(need, ws, ws_bytes, &base))) return st;
  char* w = static_cast<char*>(base);
  NormProblem n{f16, c.M, c.K, c.epsilon, c.a, c.skip, c.norm_scale, w, c.residual};
  if ((st = launched(launch_norm_rows(n, s)))) return st;
  char* proj = w + al256(static_cast<uint64_t>(c.M * c.K) * (f16 ? 2 : 4));
  const struct { int64_t n; const uint8_t* b; const void* sc; void* y; } outs[3] = {
      {c.Nq, c.q_b, c.q_scales, c.q}, {c.Nkv, c.k_b, c.k_scales, c.k}, {c.Nkv, c.v_b, c.v_scales, c.v}};
  for (const auto& o : outs)
    if (o.n > 0 && (st = run_projection(projection(f16, c.M, c.K, o.n, c.block_size, c.bits, w, o.b, o.sc, nullptr, o.y),
                                        proj, s)))
      return st;
  return XRGPU_OK;
}

int bnb4_forward(const xrgpu_bnb4_problem& c, cudaStream_t s) {
  int f16 = 0;
  int st = t1_code(c.dtype, &f16);
  if (st) return st;
  if (c.M < 0 || c.K <= 0 || c.N <= 0 || c.block_size <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Invalid packed matmul geometry");
  if (c.quant_type != 0 && c.quant_type != 1) return fail(XRGPU_INVALID_ARGUMENT, "quant_type must be 0 (FP4) or 1 (NF4)");
  if (c.M > 0 && (!c.a || !c.b || !c.absmax || !c.y)) return fail(XRGPU_INVALID_ARGUMENT, "null tensor pointer");
  Bnb4Problem p{f16, c.quant_type, 0, c.M, c.K, c.N, c.block_size, c.a, c.b, c.absmax, c.y};
  return launched(launch_bnb4(p, s));
}

int gather_forward(const xrgpu_gather_problem& c, cudaStream_t s) {
  if ((c.bits != 4 && c.bits != 8) || c.block_size < 16 || (c.block_size & (c.block_size - 1)))
    return fail(XRGPU_INVALID_ARGUMENT, "Unsupported GatherBlockQuantized geometry");
  if (c.index_dtype != XRGPU_INT64 && c.index_dtype != XRGPU_INT32) return fail(XRGPU_INVALID_ARGUMENT, "indices must be int64 or int32");
  if (c.rows < 0 || c.row_bytes < 0 || c.count < 0) return fail(XRGPU_INVALID_ARGUMENT, "invalid GatherBlockQuantized sizes");
  const int64_t width = c.row_bytes * (8 / c.bits);
  if (c.count > 0 && width > 0 && (!c.data || !c.indices || !c.scales || !c.out))
    return fail(XRGPU_INVALID_ARGUMENT, "null tensor pointer");
  if (c.count > 65535) return fail(XRGPU_INVALID_ARGUMENT, "at most 65535 indices per call");
  GatherProblem p{};
  p.bits = c.bits;
  p.idx64 = c.index_dtype == XRGPU_INT64;
  p.rows = c.rows; p.row_bytes = c.row_bytes; p.width = width;
  p.blocks = (width + c.block_size - 1) / c.block_size;
  p.zp_row = (p.blocks * c.bits + 7) / 8;
  p.block_size = c.block_size; p.count = c.count;
  p.data = c.data; p.indices = c.indices; p.scales = c.scales; p.zero_points = c.zero_points; p.out = c.out;
  p.err = device_error_word();
  return launched(launch_gather_quant(p, s));
}

int qmoe_geometry(const xrgpu_qmoe_problem& c, int64_t* inter) {
  if (c.bits != 4 && c.bits != 8) return fail(XRGPU_INVALID_ARGUMENT, "Unsupported QMoE integer layout");
  if (!((c.activation == XRGPU_ACT_RELU && c.swiglu_fusion == 0) || (c.activation == XRGPU_ACT_SWIGLU && c.swiglu_fusion == 1)))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid quantized SwiGLU fusion");
  if (c.tokens < 0 || c.hidden <= 0 || c.k < 1 || c.k > c.experts) return fail(XRGPU_INVALID_ARGUMENT, "Invalid MoE input or routing geometry");
  const int64_t fusion = c.activation == XRGPU_ACT_SWIGLU ? 2 : 1;
  if (c.fc1_rows < 0 || c.fc1_rows % fusion) return fail(XRGPU_INVALID_ARGUMENT, "Invalid MoE weight geometry");
  *inter = c.fc1_rows / fusion;
  const int64_t bs = c.block_size;
  if (bs != 0 && (bs < 16 || (bs & (bs - 1)) || c.hidden % bs || *inter % bs))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid quantized expert block size");
  return XRGPU_OK;
}

uint64_t qmoe_workspace(const xrgpu_qmoe_problem& c, int64_t inter) {
  const uint64_t tk = static_cast<uint64_t>(c.tokens * c.k);
  return al256(tk * 4) + al256(tk * 4) + al256(tk * static_cast<uint64_t>(inter) * 4);
}

int qmoe_forward(const xrgpu_qmoe_problem& c, void* ws, uint64_t ws_bytes, cudaStream_t s) {
  int64_t inter = 0;
  int st = qmoe_geometry(c, &inter);
  if (st) return st;
  if (c.tokens == 0) return XRGPU_OK;
  if (!c.input || !c.router || !c.output || (inter > 0 && (!c.fc1 || !c.fc1_scales || !c.fc2 || !c.fc2_scales)))
    return fail(XRGPU_INVALID_ARGUMENT, "null tensor pointer");
  void* base = nullptr;
  if ((st = resolve_workspace(qmoe_workspace(c, inter), ws, ws_bytes, &base))) return st;
  char* w = static_cast<char*>(base);
  const uint64_t tk = static_cast<uint64_t>(c.tokens * c.k);
  QmoeProblem p{};
  p.bits = c.bits; p.act = c.activation; p.swiglu_fusion = c.swiglu_fusion; p.has_limit = c.has_swiglu_limit;
  p.tokens = c.tokens; p.hidden = c.hidden; p.experts = c.experts; p.k = c.k; p.fc1_rows = c.fc1_rows; p.inter = inter;
  p.block_size = c.block_size;
  p.fc1_spr = c.block_size ? c.hidden / c.block_size : 1;
  p.fc2_spr = c.block_size ? inter / c.block_size : 1;
  p.alpha = c.activation_alpha; p.beta = c.activation_beta; p.swiglu_limit = c.swiglu_limit;
  p.x = c.input; p.router = c.router; p.fc1 = c.fc1; p.fc1_scales = c.fc1_scales; p.fc2 = c.fc2;
  p.fc2_scales = c.fc2_scales; p.out = c.output;
  p.route_expert = reinterpret_cast<int32_t*>(w);
  p.route_weight = reinterpret_cast<float*>(w + al256(tk * 4));
  p.act_buf = reinterpret_cast<float*>(w + 2 * al256(tk * 4));
  return launched(launch_qmoe(p, s));
}

}  // namespace xrgpu

extern "C" {

int xrgpu_mlp_workspace_size(const xrgpu_mlp_problem* p, uint64_t* bytes) {
  int f16 = 0;
  const int st = xrgpu::mlp_check(p, &f16);
  if (st) return st;
  if (bytes) *bytes = p->M ? xrgpu::mlp_layout(*p, f16).total : 0;
  return XRGPU_OK;
}

int xrgpu_mlp_forward(const xrgpu_mlp_problem* p, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!p) return xrgpu::api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  return xrgpu::mlp_forward(*p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int xrgpu_qkv_workspace_size(const xrgpu_qkv_problem* p, uint64_t* bytes) {
  int f16 = 0;
  const int st = xrgpu::qkv_check(p, &f16);
  if (st) return st;
  if (bytes) *bytes = p->M ? xrgpu::qkv_workspace(*p, f16) : 0;
  return XRGPU_OK;
}

int xrgpu_qkv_forward(const xrgpu_qkv_problem* p, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!p) return xrgpu::api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  return xrgpu::qkv_forward(*p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int xrgpu_bnb4_forward(const xrgpu_bnb4_problem* p, void* stream) {
  if (!p) return xrgpu::api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  return xrgpu::bnb4_forward(*p, static_cast<cudaStream_t>(stream));
}

int xrgpu_gather_block_quantized_forward(const xrgpu_gather_problem* p, void* stream) {
  if (!p) return xrgpu::api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  return xrgpu::gather_forward(*p, static_cast<cudaStream_t>(stream));
}

int xrgpu_qmoe_workspace_size(const xrgpu_qmoe_problem* p, uint64_t* bytes) {
  if (!p) return xrgpu::api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  int64_t inter = 0;
  const int st = xrgpu::qmoe_geometry(*p, &inter);
  if (st) return st;
  if (bytes) *bytes = xrgpu::qmoe_workspace(*p, inter);
  return XRGPU_OK;
}

int xrgpu_qmoe_forward(const xrgpu_qmoe_problem* p, void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!p) return xrgpu::api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  return xrgpu::qmoe_forward(*p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
