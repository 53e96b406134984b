// Plans of the operators around MatMulNBits for the operator API: contract checks, attributes,
// output inference, device snapshots and launches (xrgpu_prepare_ex in mmnb_api.cu calls these).
//
// Layers, as in the reference:
//   validate_contract (kernels/_shared/extended/contracts.cpp:14-20): every input name belongs to the
//     operation, required inputs are present, dtype in the tensor's mask, fixed ranks, one dtype per
//     type variable -- the rows below restate contract_data.h:659-663,718-721,728-751,821-827;
//   plan_complex (complex_plan.cpp:58-143): canonical input order, attribute defaults and the
//     operation's geometry checks, optional outputs only when requested, requested output order;
//   shape rules the shaders leave to their bounds checks (framework.glsl:44) are rejected up front.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <map>
#include <set>
#include <string>

#include "mmnb_family_ops.h"
#include "mmnb_internal.h"

namespace xrgpu {
namespace {

int fail(int status, const std::string& m) { return api_fail(status, m); }

struct Row {
  const char* op;
  const char* name;
  const char* var;   // type variable (upper case) or a fixed dtype name
  uint32_t mask;     // allowed dtypes, bit = xrgpu_dtype
  int rank;          // -1: any
  bool optional;
  bool output;
};
constexpr uint32_t kF = 1u << XRGPU_FLOAT32, kFH = (1u << XRGPU_FLOAT32) | (1u << XRGPU_FLOAT16),
                   kU8 = 1u << XRGPU_UINT8, kI64 = 1u << XRGPU_INT64;
const Row kRows[] = {
    {"com.microsoft.GatherBlockQuantized", "dataT", "T1", kU8, 2, false, false},
    {"com.microsoft.GatherBlockQuantized", "indicesT", "Tind", kI64, 1, false, false},
    {"com.microsoft.GatherBlockQuantized", "scalesT", "T2", kF, 2, false, false},
    {"com.microsoft.GatherBlockQuantized", "zeroPointsT", "T1", kU8, 2, true, false},
    {"com.microsoft.GatherBlockQuantized", "outputT", "T2", kF, 2, false, true},
    {"com.microsoft.MatMulBnb4", "aT", "T1", kFH, 2, false, false},
    {"com.microsoft.MatMulBnb4", "bT", "T2", kU8, 1, false, false},
    {"com.microsoft.MatMulBnb4", "absmaxT", "T1", kFH, 1, false, false},
    {"com.microsoft.MatMulBnb4", "yT", "T1", kFH, 2, false, true},
    {"com.microsoft.MatMulNBitsMlp", "aT", "T1", kFH, -1, false, false},
    {"com.microsoft.MatMulNBitsMlp", "skipT", "T1", kFH, -1, true, false},
    {"com.microsoft.MatMulNBitsMlp", "normScaleT", "T1", kFH, 1, true, false},
    {"com.microsoft.MatMulNBitsMlp", "gateBT", "uint8", kU8, 3, false, false},
    {"com.microsoft.MatMulNBitsMlp", "gateScalesT", "T1", kFH, 2, false, false},
    {"com.microsoft.MatMulNBitsMlp", "gateBiasT", "T1", kFH, 1, true, false},
    {"com.microsoft.MatMulNBitsMlp", "upBT", "uint8", kU8, 3, false, false},
    {"com.microsoft.MatMulNBitsMlp", "upScalesT", "T1", kFH, 2, false, false},
    {"com.microsoft.MatMulNBitsMlp", "upBiasT", "T1", kFH, 1, true, false},
    {"com.microsoft.MatMulNBitsMlp", "yT", "T1", kFH, -1, false, true},
    {"com.microsoft.MatMulNBitsMlp", "residualT", "T1", kFH, -1, true, true},
    {"com.microsoft.MatMulNBitsQkv", "aT", "T1", kFH, -1, false, false},
    {"com.microsoft.MatMulNBitsQkv", "skipT", "T1", kFH, -1, true, false},
    {"com.microsoft.MatMulNBitsQkv", "normScaleT", "T1", kFH, 1, false, false},
    {"com.microsoft.MatMulNBitsQkv", "qBT", "T2", kU8, 3, false, false},
    {"com.microsoft.MatMulNBitsQkv", "qScalesT", "T1", kFH, 2, false, false},
    {"com.microsoft.MatMulNBitsQkv", "kBT", "T2", kU8, 3, false, false},
    {"com.microsoft.MatMulNBitsQkv", "kScalesT", "T1", kFH, 2, false, false},
    {"com.microsoft.MatMulNBitsQkv", "vBT", "T2", kU8, 3, false, false},
    {"com.microsoft.MatMulNBitsQkv", "vScalesT", "T1", kFH, 2, false, false},
    {"com.microsoft.MatMulNBitsQkv", "qT", "T1", kFH, -1, false, true},
    {"com.microsoft.MatMulNBitsQkv", "kT", "T1", kFH, -1, false, true},
    {"com.microsoft.MatMulNBitsQkv", "vT", "T1", kFH, -1, false, true},
    {"com.microsoft.MatMulNBitsQkv", "residualT", "T1", kFH, -1, true, true},
    {"com.microsoft.QMoE", "inputT", "T", kF, -1, false, false},
    {"com.microsoft.QMoE", "routerT", "T", kF, 2, false, false},
    {"com.microsoft.QMoE", "fc1T", "T1", kU8, 3, false, false},
    {"com.microsoft.QMoE", "fc1ScalesT", "T2", kF, -1, false, false},
    {"com.microsoft.QMoE", "fc2T", "T1", kU8, 3, false, false},
    {"com.microsoft.QMoE", "fc2ScalesT", "T2", kF, -1, false, false},
    {"com.microsoft.QMoE", "outputT", "T", kF, -1, false, true},
};

// Canonical input and output order (complex_plan.cpp:33-37,39-40).
struct Spec {
  const char* op;
  int code;
  std::vector<std::string> inputs, outputs;
};
const Spec& spec_of(const std::string& op, bool* found) {
  static const Spec specs[] = {
      {"com.microsoft.MatMulBnb4", 1026, {"aT", "bT", "absmaxT"}, {"yT"}},
      {"com.microsoft.MatMulNBitsMlp", 1027,
       {"aT", "skipT", "normScaleT", "gateBT", "gateScalesT", "gateBiasT", "upBT", "upScalesT", "upBiasT"},
       {"yT", "residualT"}},
      {"com.microsoft.MatMulNBitsQkv", 1028,
       {"aT", "skipT", "normScaleT", "qBT", "qScalesT", "kBT", "kScalesT", "vBT", "vScalesT"},
       {"qT", "kT", "vT", "residualT"}},
      {"com.microsoft.QMoE", 1030, {"inputT", "routerT", "fc1T", "fc1ScalesT", "fc2T", "fc2ScalesT"}, {"outputT"}},
      {"com.microsoft.GatherBlockQuantized", 1031, {"dataT", "indicesT", "scalesT", "zeroPointsT"}, {"outputT"}},
  };
  for (const auto& s : specs)
    if (op == s.op) { *found = true; return s; }
  *found = false;
  return specs[0];
}

const Row* row_of(const std::string& op, const std::string& name, bool output) {
  for (const auto& r : kRows)
    if (op == r.op && name == r.name && output == r.output) return &r;
  return nullptr;
}

uint64_t dtype_size(int dt) {
  switch (dt) {
    case XRGPU_FLOAT32: case XRGPU_INT32: case XRGPU_UINT32: return 4;
    case XRGPU_FLOAT16: case XRGPU_INT16: return 2;
    case XRGPU_INT64: return 8;
    case XRGPU_INT8: case XRGPU_UINT8: case XRGPU_BOOL: return 1;
    default: return 0;
  }
}

uint64_t numel(const std::vector<int64_t>& s) {
  uint64_t n = 1;
  for (auto d : s) n *= static_cast<uint64_t>(d);
  return n;
}

bool int_attr(const xrgpu_request_ex* r, const char* name, int64_t* v) {
  for (int i = 0; i < r->num_args; ++i)  // args override attrs (planner.cpp:72-85)
    if (r->args[i].name && !std::strcmp(r->args[i].name, name)) { *v = r->args[i].value; return true; }
  for (int i = 0; i < r->num_attrs; ++i)
    if (r->attrs[i].name && !std::strcmp(r->attrs[i].name, name)) { *v = r->attrs[i].value; return true; }
  return false;
}
int64_t attr_i(const xrgpu_request_ex* r, const char* name, int64_t fallback) {
  int64_t v = fallback;
  int_attr(r, name, &v);
  return v;
}
bool float_attr(const xrgpu_request_ex* r, const char* name, double* v) {
  for (int i = 0; i < r->num_float_attrs; ++i)
    if (r->float_attrs[i].name && !std::strcmp(r->float_attrs[i].name, name)) { *v = r->float_attrs[i].value; return true; }
  int64_t iv = 0;
  if (int_attr(r, name, &iv)) { *v = static_cast<double>(iv); return true; }
  return false;
}
double attr_f(const xrgpu_request_ex* r, const char* name, double fallback) {
  double v = fallback;
  float_attr(r, name, &v);
  return v;
}
std::string attr_s(const xrgpu_request_ex* r, const char* name, const char* fallback) {
  for (int i = 0; i < r->num_string_attrs; ++i)
    if (r->string_attrs[i].name && !std::strcmp(r->string_attrs[i].name, name))
      return r->string_attrs[i].value ? r->string_attrs[i].value : "";
  return fallback;
}

// activation_lower (complex_plan.cpp:50).
int activation_code(const std::string& name, int* code) {
  if (name == "none" || name.empty() || name == "identity") *code = XRGPU_ACT_NONE;
  else if (name == "relu") *code = XRGPU_ACT_RELU;
  else if (name == "silu" || name == "swish") *code = XRGPU_ACT_SILU;
  else if (name == "gelu") *code = XRGPU_ACT_GELU;
  else if (name == "tanh") *code = XRGPU_ACT_TANH;
  else if (name == "sigmoid") *code = XRGPU_ACT_SIGMOID;
  else if (name == "swiglu") *code = XRGPU_ACT_SWIGLU;
  else return fail(XRGPU_INVALID_ARGUMENT, "Unknown fused activation: " + name);
  return XRGPU_OK;
}

std::vector<int64_t> replace_last(const std::vector<int64_t>& s, int64_t n) {
  auto out = s;
  out.back() = n;
  return out;
}

const FamilyTensor& T(const FamilyOp& op, const char* name) {
  for (const auto& t : op.in)
    if (t.name == name) return t;
  static FamilyTensor none;
  return none;
}

int check_packed_weights(const FamilyOp& op, const char* b, const char* s, int64_t N) {
  const int64_t kb = ceil_div(op.K, op.bs), blob = (op.bs * op.bits + 7) / 8;
  const auto& bt = T(op, b);
  const auto& st = T(op, s);
  if (bt.shape[0] != N || bt.shape[1] != kb || bt.shape[2] != blob)
    return fail(XRGPU_INVALID_ARGUMENT, std::string(b) + " shape must be [N, ceil(K/block_size), ceil(block_size*bits/8)]");
  if (st.shape[0] != N || st.shape[1] != kb) return fail(XRGPU_INVALID_ARGUMENT, std::string(s) + " shape must be [N, ceil(K/block_size)]");
  return XRGPU_OK;
}

int plan_packed(const xrgpu_request_ex* r, FamilyOp& op) {
  const auto& a = T(op, "aT");
  if (a.shape.empty()) return fail(XRGPU_INVALID_ARGUMENT, "Rank-one or greater tensor required");
  op.K = attr_i(r, "K", a.shape.back());
  op.N = attr_i(r, "N", 0);
  op.bs = attr_i(r, "block_size", 32);
  op.bits = attr_i(r, "bits", 4);
  op.quant_type = attr_i(r, "quant_type", 1);
  op.epsilon = attr_f(r, "epsilon", op.code == 1028 ? 1e-6 : 1e-5);
  int st = activation_code(attr_s(r, "activation", "silu"), &op.act);
  if (st) return st;
  if (op.K <= 0 || op.bs <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Invalid packed matmul geometry");
  if (op.code != 1028 && op.N <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Packed matmul N required");
  if (a.shape.back() != op.K) return fail(XRGPU_INVALID_ARGUMENT, "aT last dimension must equal attribute K");
  op.M = static_cast<int64_t>(numel(a.shape) / static_cast<uint64_t>(op.K));
  if (op.code == 1026) {
    if (op.quant_type != 0 && op.quant_type != 1) return fail(XRGPU_INVALID_ARGUMENT, "Attribute quant_type must be 0 or 1");
    if (attr_i(r, "transB", 1) != 1) return fail(XRGPU_INVALID_ARGUMENT, "Attribute transB must be 1");
    if (attr_i(r, "training_mode", 0) != 0) return fail(XRGPU_INVALID_ARGUMENT, "Attribute training_mode must be 0");
    const uint64_t w = static_cast<uint64_t>(op.N) * static_cast<uint64_t>(op.K);
    if (numel(T(op, "bT").shape) < (w + 1) / 2) return fail(XRGPU_INVALID_ARGUMENT, "bT must hold ceil(N*K/2) bytes");
    if (numel(T(op, "absmaxT").shape) < (w + op.bs - 1) / op.bs)
      return fail(XRGPU_INVALID_ARGUMENT, "absmaxT must hold ceil(N*K/block_size) values");
    return XRGPU_OK;
  }
  if (op.bits != 2 && op.bits != 4 && op.bits != 8) return fail(XRGPU_INVALID_ARGUMENT, "Attribute bits must be 2, 4 or 8");
  const auto& skip = T(op, "skipT");
  if (skip.present && skip.shape != a.shape) return fail(XRGPU_INVALID_ARGUMENT, "skipT shape must equal aT's");
  const auto& ns = T(op, "normScaleT");
  if (ns.present && ns.shape[0] != op.K) return fail(XRGPU_INVALID_ARGUMENT, "normScaleT shape must be [K]");
  if (op.code == 1027) {
    if ((st = check_packed_weights(op, "gateBT", "gateScalesT", op.N)) || (st = check_packed_weights(op, "upBT", "upScalesT", op.N)))
      return st;
    for (const char* b : {"gateBiasT", "upBiasT"})
      if (T(op, b).present && T(op, b).shape[0] != op.N) return fail(XRGPU_INVALID_ARGUMENT, std::string(b) + " shape must be [N]");
    return XRGPU_OK;
  }
  op.Nq = attr_i(r, "Nq", 0);
  op.Nkv = attr_i(r, "Nkv", 0);
  if (op.Nq <= 0 || op.Nkv <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Positive attributes Nq and Nkv required");
  if ((st = check_packed_weights(op, "qBT", "qScalesT", op.Nq)) || (st = check_packed_weights(op, "kBT", "kScalesT", op.Nkv)) ||
      (st = check_packed_weights(op, "vBT", "vScalesT", op.Nkv)))
    return st;
  return XRGPU_OK;
}

// complex_plan.cpp:121-128 (QMoE branch).
int plan_qmoe(const xrgpu_request_ex* r, FamilyOp& op) {
  const auto& x = T(op, "inputT");
  const auto& router = T(op, "routerT");
  const auto& fc1 = T(op, "fc1T");
  const auto& fc2 = T(op, "fc2T");
  const auto& s1 = T(op, "fc1ScalesT");
  const auto& s2 = T(op, "fc2ScalesT");
  op.k = attr_i(r, "k", 1);
  op.swiglu_fusion = attr_i(r, "swiglu_fusion", 0);
  op.bits = attr_i(r, "expert_weight_bits", 4);
  op.bs = attr_i(r, "block_size", 0);
  const int64_t prepacked = attr_i(r, "weights_prepacked", -1);
  int st = activation_code(attr_s(r, "activation_type", "relu"), &op.act);
  if (st) return st;
  op.alpha = attr_f(r, "activation_alpha", 1.0);
  op.beta = attr_f(r, "activation_beta", 0.0);
  op.has_limit = float_attr(r, "swiglu_limit", &op.limit);
  const int64_t rank = static_cast<int64_t>(x.shape.size());
  op.hidden = rank ? x.shape.back() : 1;
  op.experts = router.shape[1];
  op.fc1_rows = fc1.shape[1];
  const int64_t fusion = (op.act == XRGPU_ACT_SWIGLU && op.swiglu_fusion) ? 2 : 1;
  const int64_t inter = op.fc1_rows / fusion;
  if (!((rank == 2 || rank == 3) && op.hidden > 0 && op.k >= 1 && op.k <= op.experts && attr_i(r, "use_sparse_mixer", 0) == 0))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid MoE input or routing geometry");
  op.M = static_cast<int64_t>(numel(x.shape) / static_cast<uint64_t>(op.hidden));
  if (!(router.shape[0] == op.M && fc1.shape[0] == op.experts && fc2.shape[0] == op.experts && fc2.shape[1] == op.hidden &&
        op.fc1_rows % fusion == 0))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid MoE weight geometry");
  if (!((op.bits == 4 || op.bits == 8) && (prepacked == -1 || prepacked == 0) && attr_s(r, "quant_type", "int") == "int"))
    return fail(XRGPU_INVALID_ARGUMENT, "Unsupported QMoE integer layout");
  if (!((op.act == XRGPU_ACT_RELU && op.swiglu_fusion == 0) || (op.act == XRGPU_ACT_SWIGLU && op.swiglu_fusion == 1)))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid quantized SwiGLU fusion");
  if (!(fc1.shape[2] * (8 / op.bits) == op.hidden && fc2.shape[2] * (8 / op.bits) == inter))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid packed expert projection");
  if (!(op.bs == 0 || (op.bs >= 16 && (op.bs & (op.bs - 1)) == 0 && op.hidden % op.bs == 0 && inter % op.bs == 0)))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid quantized expert block size");
  for (int which = 0; which < 2; ++which) {
    const auto& s = which ? s2 : s1;
    const auto& w = which ? fc2 : fc1;
    const int64_t cols = which ? inter : op.hidden;
    const bool ok = static_cast<int64_t>(s.shape.size()) == (op.bs ? 3 : 2) && s.shape[0] == op.experts &&
                    s.shape[1] == w.shape[1] && (!op.bs || s.shape[2] == cols / op.bs);
    if (!ok) return fail(XRGPU_INVALID_ARGUMENT, "Invalid quantized expert scales");
  }
  return XRGPU_OK;
}

// complex_plan.cpp:129 (GatherBlockQuantized branch).
int plan_gather(const xrgpu_request_ex* r, FamilyOp& op) {
  op.bits = attr_i(r, "bits", 4);
  op.bs = attr_i(r, "block_size", 128);
  if (!((op.bits == 4 || op.bits == 8) && op.bs >= 16 && (op.bs & (op.bs - 1)) == 0 && attr_i(r, "gather_axis", 0) == 0 &&
        attr_i(r, "quantize_axis", 1) == 1))
    return fail(XRGPU_INVALID_ARGUMENT, "Unsupported GatherBlockQuantized geometry");
  const auto& data = T(op, "dataT");
  const int64_t width = data.shape[1] * (8 / op.bits), blocks = (width + op.bs - 1) / op.bs;
  const auto& sc = T(op, "scalesT");
  if (sc.shape[0] != data.shape[0] || sc.shape[1] != blocks)
    return fail(XRGPU_INVALID_ARGUMENT, "scalesT shape must be [rows, ceil(width/block_size)]");
  const auto& zp = T(op, "zeroPointsT");
  if (zp.present && (zp.shape[0] != data.shape[0] || zp.shape[1] != (blocks * op.bits + 7) / 8))
    return fail(XRGPU_INVALID_ARGUMENT, "zeroPointsT shape must be [rows, ceil(blocks*bits/8)]");
  op.M = T(op, "indicesT").shape[0];
  if (op.M > 65535) return fail(XRGPU_INVALID_ARGUMENT, "at most 65535 indices");
  return XRGPU_OK;
}

}  // namespace

bool is_family_operation(const char* operation) {
  bool found = false;
  if (operation) spec_of(operation, &found);
  return found;
}

int family_plan(const xrgpu_request_ex* r, bool need_data, FamilyOp* out) {
  if (!r || !r->operation) return fail(XRGPU_INVALID_ARGUMENT, "Null request");
  bool found = false;
  const Spec& spec = spec_of(r->operation, &found);
  if (!found) return fail(XRGPU_INVALID_ARGUMENT, std::string("Unsupported extended operator: ") + r->operation);
  if (r->num_inputs < 0 || (r->num_inputs > 0 && !r->inputs) || r->num_attrs < 0 || (r->num_attrs > 0 && !r->attrs) ||
      r->num_args < 0 || (r->num_args > 0 && !r->args) || r->num_float_attrs < 0 ||
      (r->num_float_attrs > 0 && !r->float_attrs) || r->num_string_attrs < 0 ||
      (r->num_string_attrs > 0 && !r->string_attrs) || r->num_requested_outputs < 0 ||
      (r->num_requested_outputs > 0 && !r->requested_outputs))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid request arrays");
  FamilyOp op;
  op.code = spec.code;
  op.operation = spec.op;
  op.in.resize(spec.inputs.size());
  for (size_t i = 0; i < spec.inputs.size(); ++i) op.in[i].name = spec.inputs[i];
  // validate_contract: names, dtypes, ranks, type variables, required inputs.
  std::map<std::string, int> types;
  std::set<std::string> seen;
  for (int i = 0; i < r->num_inputs; ++i) {
    const xrgpu_tensor& t = r->inputs[i];
    if (!t.name || !seen.insert(t.name).second) return fail(XRGPU_INVALID_ARGUMENT, "Duplicate or unnamed extended input");
    const Row* row = row_of(op.operation, t.name, false);
    if (!row) return fail(XRGPU_INVALID_ARGUMENT, std::string("Unknown input outside frozen contract: ") + t.name);
    if (t.dtype < 0 || t.dtype > XRGPU_BOOL || !(row->mask & (1u << t.dtype)))
      return fail(XRGPU_INVALID_ARGUMENT, std::string("Logical dtype outside frozen contract: ") + t.name);
    if (t.rank < 0 || t.rank > XRGPU_MAX_RANK || (row->rank >= 0 && t.rank != row->rank))
      return fail(XRGPU_INVALID_ARGUMENT, std::string("Rank outside frozen contract: ") + t.name);
    if (row->var[0] >= 'A' && row->var[0] <= 'Z') {
      auto prior = types.find(row->var);
      if (prior != types.end() && prior->second != t.dtype)
        return fail(XRGPU_INVALID_ARGUMENT, std::string("Type variable differs between tensors: ") + row->var);
      types[row->var] = t.dtype;
    }
    for (auto& slot : op.in)
      if (slot.name == t.name) {
        slot.present = true;
        slot.dtype = t.dtype;
        slot.shape.assign(t.shape, t.shape + t.rank);
        for (auto d : slot.shape)
          if (d < 0 || d > 0xffffffffll) return fail(XRGPU_INVALID_ARGUMENT, "Invalid extended tensor dimension");
        slot.nbytes = t.nbytes;
        slot.host = t.data;
      }
  }
  for (const auto& slot : op.in) {
    const Row* row = row_of(op.operation, slot.name, false);
    if (!row->optional && !slot.present)
      return fail(XRGPU_INVALID_ARGUMENT, "Missing required frozen-contract input: " + slot.name);
  }
  int st = XRGPU_OK;
  if (op.code == 1030) st = plan_qmoe(r, op);
  else if (op.code == 1031) st = plan_gather(r, op);
  else st = plan_packed(r, op);
  if (st) return st;
  // Outputs (complex_plan.cpp:54-57 O(), :131-132 requested order).
  const auto& first = op.in[0];
  int t1 = first.dtype;
  std::vector<FamilyTensor> cand(spec.outputs.size());
  for (size_t i = 0; i < spec.outputs.size(); ++i) cand[i].name = spec.outputs[i];
  if (op.code == 1028) {
    cand[0].shape = replace_last(first.shape, op.Nq);
    cand[1].shape = replace_last(first.shape, op.Nkv);
    cand[2].shape = replace_last(first.shape, op.Nkv);
    cand[3].shape = first.shape;
  } else if (op.code == 1027) {
    cand[0].shape = replace_last(first.shape, op.N);
    cand[1].shape = first.shape;
  } else if (op.code == 1026) {
    cand[0].shape = {first.shape[0], op.N};
  } else if (op.code == 1030) {
    cand[0].shape = first.shape;
  } else {
    cand[0].shape = {op.M, T(op, "dataT").shape[1] * (8 / op.bits)};
    t1 = T(op, "scalesT").dtype;
  }
  auto requested = [&](const std::string& n) {
    for (int i = 0; i < r->num_requested_outputs; ++i)
      if (r->requested_outputs[i] && n == r->requested_outputs[i]) return true;
    return false;
  };
  std::vector<FamilyTensor> planned;
  std::vector<int> slots;
  for (size_t i = 0; i < cand.size(); ++i) {
    const bool optional = row_of(op.operation, cand[i].name, true)->optional;
    const bool req = requested(cand[i].name);
    if ((optional && !req) || (r->num_requested_outputs > 0 && !req)) continue;
    cand[i].dtype = t1;
    cand[i].nbytes = numel(cand[i].shape) * dtype_size(t1);
    planned.push_back(cand[i]);
    slots.push_back(static_cast<int>(i));
  }
  if (r->num_requested_outputs > 0) {
    std::vector<FamilyTensor> ordered;
    std::vector<int> oslots;
    for (int i = 0; i < r->num_requested_outputs; ++i) {
      bool hit = false;
      for (size_t j = 0; j < planned.size(); ++j)
        if (r->requested_outputs[i] && planned[j].name == r->requested_outputs[i]) {
          ordered.push_back(planned[j]);
          oslots.push_back(slots[j]);
          hit = true;
        }
      if (!hit) return fail(XRGPU_INVALID_ARGUMENT, "Unknown requested complex output");
    }
    planned = ordered;
    slots = oslots;
  }
  for (size_t i = 0; i < cand.size(); ++i) {  // required outputs must be planned
    const Row* row = row_of(op.operation, cand[i].name, true);
    if (!row->optional && std::find(slots.begin(), slots.end(), static_cast<int>(i)) == slots.end())
      return fail(XRGPU_INVALID_ARGUMENT, "Missing required frozen-contract output: " + cand[i].name);
  }
  op.out = planned;
  op.out_slot = slots;
  if (need_data) {
    for (const auto& t : op.in) {
      if (!t.present) continue;
      if (t.nbytes != numel(t.shape) * dtype_size(t.dtype))
        return fail(XRGPU_INVALID_ARGUMENT, "Extended input byte count mismatch: " + t.name);
      if (t.nbytes && !t.host) return fail(XRGPU_INVALID_ARGUMENT, "Missing data for input: " + t.name);
    }
  }
  *out = std::move(op);
  return XRGPU_OK;
}

namespace {

void* in_dev(const FamilyOp& op, const char* name) { return T(op, name).dev; }

void* out_dev(const FamilyOp& op, int slot) {
  for (size_t i = 0; i < op.out.size(); ++i)
    if (op.out_slot[i] == slot) return op.out[i].dev;
  return nullptr;
}

xrgpu_mlp_problem mlp_of(const FamilyOp& op) {
  xrgpu_mlp_problem c{};
  c.dtype = T(op, "aT").dtype;
  c.activation = op.act;
  c.M = op.M; c.K = op.K; c.N = op.N; c.block_size = op.bs; c.bits = op.bits;
  c.epsilon = static_cast<float>(op.epsilon);
  c.a = in_dev(op, "aT"); c.skip = in_dev(op, "skipT"); c.norm_scale = in_dev(op, "normScaleT");
  c.gate_b = static_cast<const uint8_t*>(in_dev(op, "gateBT")); c.gate_scales = in_dev(op, "gateScalesT");
  c.gate_bias = in_dev(op, "gateBiasT");
  c.up_b = static_cast<const uint8_t*>(in_dev(op, "upBT")); c.up_scales = in_dev(op, "upScalesT");
  c.up_bias = in_dev(op, "upBiasT");
  c.y = out_dev(op, 0); c.residual = out_dev(op, 1);
  return c;
}

xrgpu_qkv_problem qkv_of(const FamilyOp& op) {
  xrgpu_qkv_problem c{};
  c.dtype = T(op, "aT").dtype;
  c.M = op.M; c.K = op.K; c.Nq = op.Nq; c.Nkv = op.Nkv; c.block_size = op.bs; c.bits = op.bits;
  c.epsilon = static_cast<float>(op.epsilon);
  c.a = in_dev(op, "aT"); c.skip = in_dev(op, "skipT"); c.norm_scale = in_dev(op, "normScaleT");
  c.q_b = static_cast<const uint8_t*>(in_dev(op, "qBT")); c.q_scales = in_dev(op, "qScalesT");
  c.k_b = static_cast<const uint8_t*>(in_dev(op, "kBT")); c.k_scales = in_dev(op, "kScalesT");
  c.v_b = static_cast<const uint8_t*>(in_dev(op, "vBT")); c.v_scales = in_dev(op, "vScalesT");
  c.q = out_dev(op, 0); c.k = out_dev(op, 1); c.v = out_dev(op, 2); c.residual = out_dev(op, 3);
  return c;
}

xrgpu_qmoe_problem qmoe_of(const FamilyOp& op) {
  xrgpu_qmoe_problem c{};
  c.bits = static_cast<int32_t>(op.bits);
  c.activation = op.act;
  c.swiglu_fusion = static_cast<int32_t>(op.swiglu_fusion);
  c.has_swiglu_limit = op.has_limit;
  c.tokens = op.M; c.hidden = op.hidden; c.experts = op.experts; c.k = op.k; c.fc1_rows = op.fc1_rows;
  c.block_size = op.bs;
  c.activation_alpha = static_cast<float>(op.alpha);
  c.activation_beta = static_cast<float>(op.beta);
  c.swiglu_limit = static_cast<float>(op.limit);
  c.input = static_cast<const float*>(in_dev(op, "inputT"));
  c.router = static_cast<const float*>(in_dev(op, "routerT"));
  c.fc1 = static_cast<const uint8_t*>(in_dev(op, "fc1T"));
  c.fc1_scales = static_cast<const float*>(in_dev(op, "fc1ScalesT"));
  c.fc2 = static_cast<const uint8_t*>(in_dev(op, "fc2T"));
  c.fc2_scales = static_cast<const float*>(in_dev(op, "fc2ScalesT"));
  c.output = static_cast<float*>(out_dev(op, 0));
  return c;
}

uint64_t workspace_need(const FamilyOp& op) {
  uint64_t need = 0;
  if (op.code == 1027) {
    const xrgpu_mlp_problem c = mlp_of(op);
    xrgpu_mlp_workspace_size(&c, &need);
  } else if (op.code == 1028) {
    const xrgpu_qkv_problem c = qkv_of(op);
    xrgpu_qkv_workspace_size(&c, &need);
  } else if (op.code == 1030) {
    const xrgpu_qmoe_problem c = qmoe_of(op);
    xrgpu_qmoe_workspace_size(&c, &need);
  }
  return need;
}

}  // namespace

int family_allocate(FamilyOp* op, uint64_t memory_limit) {
  uint64_t total = 0;
  for (const auto& t : op->in) total += t.present ? align_up(t.nbytes, 256) : 0;
  for (const auto& t : op->out) total += align_up(t.nbytes, 256);
  if (total > memory_limit) return fail(XRGPU_INVALID_ARGUMENT, "Extended heap memory limit exceeded");
  for (auto& t : op->in) {
    if (!t.present) continue;
    if (cudaMalloc(&t.dev, std::max<uint64_t>(t.nbytes, 16)) != cudaSuccess)
      return fail(XRGPU_RUNTIME_ERROR, "device allocation failed: " + t.name);
    if (t.nbytes && cudaMemcpy(t.dev, t.host, t.nbytes, cudaMemcpyHostToDevice) != cudaSuccess)
      return fail(XRGPU_RUNTIME_ERROR, "host to device copy failed: " + t.name);
    t.host = nullptr;  // the handle owns its device snapshot
  }
  for (auto& t : op->out)
    if (cudaMalloc(&t.dev, std::max<uint64_t>(t.nbytes, 16)) != cudaSuccess)
      return fail(XRGPU_RUNTIME_ERROR, "device allocation failed: " + t.name);
  op->workspace_bytes = workspace_need(*op);
  if (total + op->workspace_bytes > memory_limit) return fail(XRGPU_INVALID_ARGUMENT, "Extended heap memory limit exceeded");
  if (op->workspace_bytes) {
    if (cudaMalloc(&op->workspace, op->workspace_bytes) != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, "workspace allocation failed");
    if (cudaMemset(op->workspace, 0, op->workspace_bytes) != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, "workspace clear failed");
  }
  return XRGPU_OK;
}

int family_launch(FamilyOp* op, cudaStream_t s) {
  switch (op->code) {
    case 1027: return mlp_forward(mlp_of(*op), op->workspace, op->workspace_bytes, s);
    case 1028: return qkv_forward(qkv_of(*op), op->workspace, op->workspace_bytes, s);
    case 1030: return qmoe_forward(qmoe_of(*op), op->workspace, op->workspace_bytes, s);
    case 1026: {
      xrgpu_bnb4_problem c{};
      c.dtype = T(*op, "aT").dtype;
      c.quant_type = static_cast<int32_t>(op->quant_type);
      c.M = op->M; c.K = op->K; c.N = op->N; c.block_size = op->bs;
      c.a = in_dev(*op, "aT"); c.b = static_cast<const uint8_t*>(in_dev(*op, "bT")); c.absmax = in_dev(*op, "absmaxT");
      c.y = out_dev(*op, 0);
      return bnb4_forward(c, s);
    }
    default: {
      const auto& data = T(*op, "dataT");
      xrgpu_gather_problem c{};
      c.bits = static_cast<int32_t>(op->bits);
      c.index_dtype = T(*op, "indicesT").dtype;
      c.rows = data.shape[0]; c.row_bytes = data.shape[1]; c.count = op->M; c.block_size = op->bs;
      c.data = static_cast<const uint8_t*>(data.dev); c.indices = in_dev(*op, "indicesT");
      c.scales = static_cast<const float*>(in_dev(*op, "scalesT"));
      c.zero_points = static_cast<const uint8_t*>(in_dev(*op, "zeroPointsT"));
      c.out = static_cast<float*>(out_dev(*op, 0));
      return gather_forward(c, s);
    }
  }
}

void family_release(FamilyOp* op) {
  for (auto& t : op->in) { if (t.dev) cudaFree(t.dev); t.dev = nullptr; }
  for (auto& t : op->out) { if (t.dev) cudaFree(t.dev); t.dev = nullptr; }
  if (op->workspace) cudaFree(op->workspace);
  op->workspace = nullptr;
}

}  // namespace xrgpu
