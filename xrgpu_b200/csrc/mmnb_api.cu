// Host side of the MatMulNBits CUDA backend: contract validation, shape planning, path
// selection, the prepared-operator handle and the C ABI declared in include/xrgpu_mmnb.h.
//
// Validation follows the reference's layers in order:
//   validate_contract (kernels/_shared/extended/contracts.cpp:14-20) with the MatMulNBits rows of
//     contract_data.h:722-727: aT T1 (f32|f16, any rank), bT uint8 rank 3, scalesT T1 rank 2,
//     zeroPointsT T3 (f32|f16) rank 2 optional, biasT T1 rank 1 optional;
//   plan() (planner.cpp:67-99): unique names, args override attrs;
//   plan_complex 1025 (complex_plan.cpp:58-62,117-120): canonical order aT,bT,scalesT,
//     zeroPointsT?,biasT?; K defaults to A's last dim, N required, block_size defaults to 32,
//     bits to 4; yT = A.shape[:-1] + [N] with A's dtype;
//   plus the contract's attribute constraints (contract.json:2-40) and the shape rules the
//     upstream manifest states (manifest.json:47-48,68-71): bT [N, ceil(K/bs), ceil(bs*bits/8)],
//     scalesT and zeroPointsT [N, ceil(K/bs)], biasT [N]. The reference leaves these to its shader's
//     bounds checks (framework.glsl:44); here they are rejected up front with INVALID_ARGUMENT.
// Extension: a uint8 zeroPointsT of shape [N, ceil(ceil(K/bs)*bits/8)] is accepted as the packed
// ONNX Runtime form.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "mmnb_family_ops.h"
#include "mmnb_internal.h"
#include "xrgpu_mmnb.h"

namespace xrgpu {
namespace {

thread_local std::string g_last_error;

int fail(int status, const std::string& message) {
  g_last_error = message;
  return status;
}

const char* kOperation = "com.microsoft.MatMulNBits";
const char* kInputNames[5] = {"aT", "bT", "scalesT", "zeroPointsT", "biasT"};

uint64_t dtype_bytes(int dt) {
  switch (dt) {
    case XRGPU_FLOAT32: case XRGPU_INT32: case XRGPU_UINT32: return 4;
    case XRGPU_FLOAT16: case XRGPU_INT16: return 2;
    case XRGPU_INT8: case XRGPU_UINT8: case XRGPU_BOOL: return 1;
    case XRGPU_INT64: return 8;
    default: return 0;
  }
}

const char* dtype_name(int dt) {
  static const char* names[] = {"float32", "float16", "int32", "uint32", "int16", "int8", "uint8", "int64", "bool", "unspecified"};
  return (dt >= 0 && dt <= 9) ? names[dt] : "invalid";
}

struct TensorMeta {
  bool present = false;
  int dtype = XRGPU_UNSPECIFIED;
  std::vector<int64_t> shape;
  const void* data = nullptr;
  uint64_t nbytes = 0;
  uint64_t numel() const {
    uint64_t n = 1;
    for (auto d : shape) n *= static_cast<uint64_t>(d);
    return n;
  }
};

struct Plan {
  TensorMeta in[5];  // canonical order
  int64_t K = 0, N = 0, bs = 0, bits = 0, accuracy = 0, kb = 0, blob = 0, M = 0;
  int f16 = 0, zp = kZpNone;
  std::vector<int64_t> y_shape;
  int y_dtype = XRGPU_FLOAT32;
};

int lookup_int(const xrgpu_request* r, const char* name, bool* found, int64_t* value) {
  *found = false;
  for (int i = 0; i < r->num_args; ++i)  // args override attrs (planner.cpp:72-85)
    if (r->args[i].name && std::strcmp(r->args[i].name, name) == 0) { *found = true; *value = r->args[i].value; }
  if (*found) return 0;
  for (int i = 0; i < r->num_attrs; ++i)
    if (r->attrs[i].name && std::strcmp(r->attrs[i].name, name) == 0) { *found = true; *value = r->attrs[i].value; }
  return 0;
}

int make_plan(const xrgpu_request* r, bool need_data, Plan* out) {
  if (!r) return fail(XRGPU_INVALID_ARGUMENT, "Null request");
  if (!r->operation || std::strcmp(r->operation, kOperation) != 0)
    return fail(XRGPU_INVALID_ARGUMENT, std::string("Unsupported extended operator: ") + (r->operation ? r->operation : "(null)"));
  if (r->num_inputs < 0 || (r->num_inputs > 0 && !r->inputs) || r->num_attrs < 0 || (r->num_attrs > 0 && !r->attrs) ||
      r->num_args < 0 || (r->num_args > 0 && !r->args))
    return fail(XRGPU_INVALID_ARGUMENT, "Invalid request arrays");
  Plan p;
  std::set<std::string> names;
  for (int i = 0; i < r->num_inputs; ++i) {
    const xrgpu_tensor& t = r->inputs[i];
    if (!t.name || !*t.name || !names.insert(t.name).second)
      return fail(XRGPU_INVALID_ARGUMENT, "Duplicate or unnamed extended input");
    int slot = -1;
    for (int s = 0; s < 5; ++s)
      if (std::strcmp(t.name, kInputNames[s]) == 0) slot = s;
    if (slot < 0) return fail(XRGPU_INVALID_ARGUMENT, std::string("Unknown input outside frozen contract: ") + t.name);
    if (t.rank < 0 || t.rank > XRGPU_MAX_RANK) return fail(XRGPU_INVALID_ARGUMENT, "Extended tensor rank exceeds 16");
    TensorMeta& m = p.in[slot];
    m.present = true;
    m.dtype = t.dtype;
    m.shape.assign(t.shape, t.shape + t.rank);
    for (auto d : m.shape)
      if (d < 0 || d > 0xffffffffll) return fail(XRGPU_INVALID_ARGUMENT, "Invalid extended tensor dimension");
    m.data = t.data;
    m.nbytes = t.nbytes;
  }
  for (int s = 0; s < 3; ++s)
    if (!p.in[s].present) return fail(XRGPU_INVALID_ARGUMENT, std::string("Missing required frozen-contract input: ") + kInputNames[s]);
  // Dtype masks and type variables (contract_data.h:722-727).
  const int t1 = p.in[0].dtype;
  if (t1 != XRGPU_FLOAT32 && t1 != XRGPU_FLOAT16) return fail(XRGPU_INVALID_ARGUMENT, "Logical dtype outside frozen contract: aT");
  if (p.in[1].dtype != XRGPU_UINT8) return fail(XRGPU_INVALID_ARGUMENT, "Logical dtype outside frozen contract: bT");
  if (p.in[2].dtype != XRGPU_FLOAT32 && p.in[2].dtype != XRGPU_FLOAT16)
    return fail(XRGPU_INVALID_ARGUMENT, "Logical dtype outside frozen contract: scalesT");
  if (p.in[2].dtype != t1) return fail(XRGPU_INVALID_ARGUMENT, "Type variable differs between tensors: T1");
  if (p.in[4].present) {
    if (p.in[4].dtype != XRGPU_FLOAT32 && p.in[4].dtype != XRGPU_FLOAT16)
      return fail(XRGPU_INVALID_ARGUMENT, "Logical dtype outside frozen contract: biasT");
    if (p.in[4].dtype != t1) return fail(XRGPU_INVALID_ARGUMENT, "Type variable differs between tensors: T1");
  }
  if (p.in[3].present && p.in[3].dtype != XRGPU_FLOAT32 && p.in[3].dtype != XRGPU_FLOAT16 && p.in[3].dtype != XRGPU_UINT8)
    return fail(XRGPU_INVALID_ARGUMENT, "Logical dtype outside frozen contract: zeroPointsT");
  // Ranks.
  if (p.in[0].shape.empty()) return fail(XRGPU_INVALID_ARGUMENT, "Rank-one or greater tensor required");
  if (p.in[1].shape.size() != 3) return fail(XRGPU_INVALID_ARGUMENT, "Rank outside frozen contract: bT");
  if (p.in[2].shape.size() != 2) return fail(XRGPU_INVALID_ARGUMENT, "Rank outside frozen contract: scalesT");
  if (p.in[3].present && p.in[3].shape.size() != 2) return fail(XRGPU_INVALID_ARGUMENT, "Rank outside frozen contract: zeroPointsT");
  if (p.in[4].present && p.in[4].shape.size() != 1) return fail(XRGPU_INVALID_ARGUMENT, "Rank outside frozen contract: biasT");
  // Attributes (complex_plan.cpp:117-120 defaults; contract.json constraints).
  bool found = false;
  int64_t v = 0;
  lookup_int(r, "K", &found, &v);
  p.K = found ? v : p.in[0].shape.back();
  lookup_int(r, "N", &found, &v);
  p.N = found ? v : 0;
  lookup_int(r, "block_size", &found, &v);
  p.bs = found ? v : 32;
  lookup_int(r, "bits", &found, &v);
  p.bits = found ? v : 4;
  lookup_int(r, "accuracy_level", &found, &v);
  p.accuracy = found ? v : 0;
  if (p.K <= 0 || p.bs <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Invalid packed matmul geometry");
  if (p.N <= 0) return fail(XRGPU_INVALID_ARGUMENT, "Packed matmul N required");
  if (p.K > 0xffffffffll || p.N > 0xffffffffll) return fail(XRGPU_INVALID_ARGUMENT, "Positive complex operator attribute required: K/N");
  if (p.bits != 2 && p.bits != 4 && p.bits != 8) return fail(XRGPU_INVALID_ARGUMENT, "Attribute bits must be 2, 4 or 8");
  if (p.bs < 16 || (p.bs & (p.bs - 1)) != 0) return fail(XRGPU_INVALID_ARGUMENT, "Attribute block_size must be a power of two >= 16");
  if (p.accuracy < 0 || p.accuracy > 4) return fail(XRGPU_INVALID_ARGUMENT, "Attribute accuracy_level must be in [0, 4]");
  p.kb = ceil_div(p.K, p.bs);
  p.blob = (p.bs * p.bits + 7) / 8;
  const auto& a = p.in[0].shape;
  if (a.back() != p.K) return fail(XRGPU_INVALID_ARGUMENT, "aT last dimension must equal attribute K");
  p.M = 1;
  for (size_t i = 0; i + 1 < a.size(); ++i) p.M *= a[i];
  const auto& b = p.in[1].shape;
  if (b[0] != p.N || b[1] != p.kb || b[2] != p.blob) {
    std::ostringstream o;
    o << "bT shape must be [N, ceil(K/block_size), block_size*bits/8] = [" << p.N << ", " << p.kb << ", " << p.blob << "]";
    return fail(XRGPU_INVALID_ARGUMENT, o.str());
  }
  if (p.in[2].shape[0] != p.N || p.in[2].shape[1] != p.kb) return fail(XRGPU_INVALID_ARGUMENT, "scalesT shape must be [N, ceil(K/block_size)]");
  if (p.in[3].present) {
    const auto& z = p.in[3].shape;
    if (p.in[3].dtype == XRGPU_UINT8) {
      if (z[0] != p.N || z[1] != (p.kb * p.bits + 7) / 8)
        return fail(XRGPU_INVALID_ARGUMENT, "packed uint8 zeroPointsT shape must be [N, ceil(ceil(K/block_size)*bits/8)]");
      p.zp = kZpPacked;
    } else {
      if (z[0] != p.N || z[1] != p.kb) return fail(XRGPU_INVALID_ARGUMENT, "zeroPointsT shape must be [N, ceil(K/block_size)]");
      p.zp = p.in[3].dtype == XRGPU_FLOAT32 ? kZpF32 : kZpF16;
    }
  }
  if (p.in[4].present && p.in[4].shape[0] != p.N) return fail(XRGPU_INVALID_ARGUMENT, "biasT shape must be [N]");
  if (need_data) {
    for (int s = 0; s < 5; ++s) {
      const TensorMeta& m = p.in[s];
      if (!m.present) continue;
      if (m.nbytes != m.numel() * dtype_bytes(m.dtype))
        return fail(XRGPU_INVALID_ARGUMENT, std::string("Extended input byte count mismatch: ") + kInputNames[s]);
      if (m.nbytes && !m.data) return fail(XRGPU_INVALID_ARGUMENT, std::string("Missing data for input: ") + kInputNames[s]);
    }
  }
  p.f16 = t1 == XRGPU_FLOAT16;
  p.y_shape = a;
  p.y_shape.back() = p.N;
  p.y_dtype = t1;
  *out = std::move(p);
  return XRGPU_OK;
}

// ---------------------------------------------------------------- zero-copy problems
int problem_from_c(const xrgpu_mmnb_problem* c, Problem* p, bool need_y) {
  if (!c) return fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  if (c->dtype != XRGPU_FLOAT32 && c->dtype != XRGPU_FLOAT16) return fail(XRGPU_INVALID_ARGUMENT, "problem dtype must be float32 or float16");
  if (c->bits != 2 && c->bits != 4 && c->bits != 8) return fail(XRGPU_INVALID_ARGUMENT, "bits must be 2, 4 or 8");
  if (c->block_size < 16 || (c->block_size & (c->block_size - 1)) != 0) return fail(XRGPU_INVALID_ARGUMENT, "block_size must be a power of two >= 16");
  if (c->M < 0 || c->K <= 0 || c->N <= 0 || c->K > 0xffffffffll || c->N > 0xffffffffll) return fail(XRGPU_INVALID_ARGUMENT, "invalid M/K/N");
  if (c->path < XRGPU_PATH_AUTO || c->path > XRGPU_PATH_GEMM) return fail(XRGPU_INVALID_ARGUMENT, "invalid path");
  Problem q{};
  q.f16 = c->dtype == XRGPU_FLOAT16;
  switch (c->zero_point_dtype) {
    case XRGPU_UNSPECIFIED: q.zp = kZpNone; break;
    case XRGPU_FLOAT32: q.zp = kZpF32; break;
    case XRGPU_FLOAT16: q.zp = kZpF16; break;
    case XRGPU_UINT8: q.zp = kZpPacked; break;
    default: return fail(XRGPU_INVALID_ARGUMENT, "invalid zero_point_dtype");
  }
  if (q.zp != kZpNone && !c->zero_points) return fail(XRGPU_INVALID_ARGUMENT, "zero_points pointer required");
  q.M = c->M; q.K = c->K; q.N = c->N; q.bs = c->block_size; q.bits = c->bits;
  q.kb = ceil_div(q.K, q.bs);
  q.blob = (q.bs * q.bits + 7) / 8;
  q.ldy = c->ldy ? c->ldy : c->N;
  if (q.ldy < q.N) return fail(XRGPU_INVALID_ARGUMENT, "ldy must be >= N");
  q.a = c->a; q.b = c->b; q.scales = c->scales; q.zp_ptr = q.zp == kZpNone ? nullptr : c->zero_points;
  q.bias = c->bias; q.y = c->y;
  if (!q.b || !q.scales || (need_y && q.M > 0 && (!q.a || !q.y))) return fail(XRGPU_INVALID_ARGUMENT, "null tensor pointer");
  *p = q;
  return XRGPU_OK;
}

}  // namespace

// ---------------------------------------------------------------- shared with the family operators
int problem_from_api(const xrgpu_mmnb_problem* c, Problem* p, bool need_y) { return problem_from_c(c, p, need_y); }

int select_path(const Problem& p, int forced) {
  if (forced == kPathGeneric) return kPathGeneric;
  if (forced == kPathGemv) return gemv_supported(p) ? kPathGemv : -1;
  if (forced == kPathGemm) return gemm_supported(p) ? kPathGemm : -1;
  // Planner (replaces the reference's single serial dispatch, complex_plan.cpp:60):
  // decode rows (M <= 16) stream the weights through the GEMV; prefill rows use the
  // tensor-core GEMM; everything else runs the generic kernel.
  if (p.M <= 16 && gemv_supported(p)) return kPathGemv;
  if (p.M > 16 && gemm_supported(p)) return kPathGemm;
  return kPathGeneric;
}

const char* path_name(int path) {
  switch (path) {
    case kPathGeneric: return "generic";
    case kPathGemv: return "gemv";
    case kPathGemm: return "gemm";
    default: return "none";
  }
}

uint64_t workspace_for(const Problem& p, int path) {
  if (path == kPathGemv) return gemv_workspace_bytes(p);
  if (path == kPathGemm) return gemm_workspace_bytes(p);
  return 0;
}

cudaError_t launch_path(const Problem& p, int path, void* ws, cudaStream_t s) {
  if (p.M == 0) return cudaSuccess;
  switch (path) {
    case kPathGemv: return launch_gemv(p, ws, s);
    case kPathGemm: return launch_gemm(p, ws, s);
    default: return launch_generic(p, s);
  }
}

// Per-device library workspace for callers that pass none (zero-filled; grows on demand).
struct DeviceWorkspace {
  std::mutex mu;
  void* ptr = nullptr;
  uint64_t bytes = 0;
  std::vector<void*> retired;  // kept alive: may still be referenced by enqueued work
};
DeviceWorkspace g_workspaces[64];

int library_workspace(uint64_t need, void** out) {
  *out = nullptr;
  if (need == 0) return XRGPU_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return fail(XRGPU_RUNTIME_ERROR, "cudaGetDevice failed");
  DeviceWorkspace& w = g_workspaces[dev];
  std::lock_guard<std::mutex> lock(w.mu);
  if (w.bytes < need) {
    void* fresh = nullptr;
    const uint64_t bytes = std::max<uint64_t>(need, w.bytes * 2);
    if (cudaMalloc(&fresh, bytes) != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, "workspace allocation failed");
    if (cudaMemset(fresh, 0, bytes) != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, "workspace clear failed");
    if (w.ptr) w.retired.push_back(w.ptr);
    w.ptr = fresh;
    w.bytes = bytes;
  }
  *out = w.ptr;
  return XRGPU_OK;
}

std::string json_escape(const std::string& s) {
  std::ostringstream o;
  for (unsigned char ch : s) {
    if (ch == '"' || ch == '\\') o << '\\' << ch;
    else if (ch < 32) { char buf[8]; std::snprintf(buf, sizeof buf, "\\u%04x", ch); o << buf; }
    else o << ch;
  }
  return o.str();
}

int write_json(const std::string& s, char* out, uint64_t capacity, uint64_t* needed) {
  if (needed) *needed = s.size() + 1;
  if (out && capacity) {
    const uint64_t n = std::min<uint64_t>(capacity - 1, s.size());
    std::memcpy(out, s.data(), n);
    out[n] = 0;
    if (n < s.size()) return fail(XRGPU_INVALID_ARGUMENT, "JSON buffer too small");
  }
  return XRGPU_OK;
}

std::string device_description(int dev) {
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return "unknown";
  std::ostringstream o;
  o << prop.name << " (sm_" << prop.major << prop.minor << ", " << prop.multiProcessorCount << " SMs)";
  return o.str();
}

int api_fail(int status, const std::string& message) { return fail(status, message); }

int device_sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!counts[dev]) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    counts[dev] = c > 0 ? c : 148;
  }
  return counts[dev];
}

}  // namespace xrgpu

// =================================================================== prepared operator
struct xrgpu_operator {
  xrgpu::Plan plan;
  xrgpu_options options{};
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
  void* dev_in[5] = {nullptr, nullptr, nullptr, nullptr, nullptr};
  void* dev_y = nullptr;
  uint64_t y_bytes = 0;
  void* workspace = nullptr;
  uint64_t workspace_bytes = 0;
  int path = 0;
  bool closed = false, poisoned = false, executed = false;
  double execution_ms = 0, gpu_ms = -1;
  uint64_t dispatch_count = 0;
  std::string poison_reason;
  xrgpu::FamilyOp* family = nullptr;  // the operations around MatMulNBits (mmnb_family_plan.cu)
};

namespace {

using namespace xrgpu;

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

Problem operator_problem(const xrgpu_operator* op) {
  const Plan& p = op->plan;
  Problem q{};
  q.f16 = p.f16; q.zp = p.zp;
  q.M = p.M; q.K = p.K; q.N = p.N; q.bs = p.bs; q.bits = p.bits; q.kb = p.kb; q.blob = p.blob; q.ldy = p.N;
  q.a = op->dev_in[0]; q.b = static_cast<const uint8_t*>(op->dev_in[1]); q.scales = op->dev_in[2];
  q.zp_ptr = op->dev_in[3]; q.bias = op->dev_in[4]; q.y = op->dev_y;
  q.err = device_error_word();
  return q;
}

void release(xrgpu_operator* op) {
  DeviceGuard guard(op->device);
  if (op->stream) cudaStreamSynchronize(op->stream);
  if (op->family) family_release(op->family);
  for (auto& ptr : op->dev_in) { if (ptr) cudaFree(ptr); ptr = nullptr; }
  if (op->dev_y) cudaFree(op->dev_y);
  op->dev_y = nullptr;
  if (op->workspace) cudaFree(op->workspace);
  op->workspace = nullptr;
  if (op->ev_start) cudaEventDestroy(op->ev_start);
  if (op->ev_stop) cudaEventDestroy(op->ev_stop);
  op->ev_start = op->ev_stop = nullptr;
  if (op->stream) cudaStreamDestroy(op->stream);
  op->stream = nullptr;
}

// A request with integer attributes only, in the extended form.
xrgpu_request_ex extend_request(const xrgpu_request* r) {
  xrgpu_request_ex ex{};
  ex.operation = r->operation;
  ex.inputs = r->inputs;
  ex.num_inputs = r->num_inputs;
  ex.attrs = r->attrs;
  ex.num_attrs = r->num_attrs;
  ex.args = r->args;
  ex.num_args = r->num_args;
  return ex;
}

// The plain request of a MatMulNBits request given in the extended form (its attributes are integers).
xrgpu_request plain_request(const xrgpu_request_ex* r) {
  xrgpu_request p{};
  p.operation = r->operation;
  p.inputs = r->inputs;
  p.num_inputs = r->num_inputs;
  p.attrs = r->attrs;
  p.num_attrs = r->num_attrs;
  p.args = r->args;
  p.num_args = r->num_args;
  return p;
}

int check_open(const xrgpu_operator* op) {
  if (!op) return fail(XRGPU_INVALID_ARGUMENT, "Null operator");
  if (op->closed) return fail(XRGPU_RUNTIME_ERROR, "Operator is closed");
  if (op->poisoned) return fail(XRGPU_RUNTIME_ERROR, "Operator failed earlier and must be closed: " + op->poison_reason);
  return XRGPU_OK;
}

int poison(xrgpu_operator* op, int status, const std::string& why) {
  op->poisoned = true;
  op->poison_reason = why;
  return fail(status, why);
}

int wait_bounded(xrgpu_operator* op, cudaEvent_t ev) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(op->options.timeout_ns);
  for (;;) {
    const cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) break;
    if (e != cudaErrorNotReady) return poison(op, XRGPU_RUNTIME_ERROR, std::string("CUDA execution failed: ") + cudaGetErrorString(e));
    if (std::chrono::steady_clock::now() > deadline) return poison(op, XRGPU_TIMEOUT, "GPU operator timed out");
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  uint32_t code = 0;
  if (read_device_error(&code, true) != cudaSuccess) return poison(op, XRGPU_RUNTIME_ERROR, "device error word unreadable");
  if (code) return poison(op, XRGPU_DEVICE_ERROR, "GPU operator contract validation failed: code " + std::to_string(code));
  return XRGPU_OK;
}

}  // namespace

extern "C" {

const char* xrgpu_last_error(void) { return xrgpu::g_last_error.c_str(); }

const char* xrgpu_version(void) { return "xrgpu-b200-mmnb 0.1 (sm_100a)"; }

void xrgpu_default_options(xrgpu_options* o) {
  if (!o) return;
  o->profiling = 0;
  o->timeout_ns = 15000000000ull;
  o->memory_limit_bytes = 268435456ull;
  o->device = 0;
}

int xrgpu_probe(char* json, uint64_t capacity, uint64_t* needed) {
  int count = 0;
  const cudaError_t e = cudaGetDeviceCount(&count);
  std::ostringstream o;
  o << "{\"backend\":\"cuda\",\"target\":\"sm_100a\",\"cpu_compute_fallback\":false,";
  if (e != cudaSuccess || count == 0) {
    o << "\"available\":false,\"device\":null,\"reason\":\"" << json_escape(e != cudaSuccess ? cudaGetErrorString(e) : "no CUDA device")
      << "\"}";
    write_json(o.str(), json, capacity, needed);
    return fail(XRGPU_UNAVAILABLE, "no usable CUDA device");
  }
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceProp prop{};
  cudaGetDeviceProperties(&prop, dev);
  const bool ok = prop.major == 10 && prop.minor == 0;
  o << "\"available\":" << (ok ? "true" : "false") << ",\"device\":\"" << json_escape(device_description(dev)) << "\",\"device_count\":"
    << count << ",\"reason\":\"" << (ok ? "" : "kernels are built for sm_100a only") << "\"}";
  const int s = write_json(o.str(), json, capacity, needed);
  if (!ok) return fail(XRGPU_UNAVAILABLE, "kernels are built for sm_100a only");
  return s;
}

int xrgpu_plan(const xrgpu_request* request, xrgpu_tensor* outputs, int32_t capacity, int32_t* count) {
  if (request && is_family_operation(request->operation)) {
    const xrgpu_request_ex ex = extend_request(request);
    return xrgpu_plan_ex(&ex, outputs, capacity, count);
  }
  Plan p;
  const int st = make_plan(request, false, &p);
  if (st) return st;
  if (count) *count = 1;
  if (capacity >= 1 && outputs) {
    xrgpu_tensor& y = outputs[0];
    std::memset(&y, 0, sizeof(y));
    y.name = "yT";
    y.dtype = p.y_dtype;
    y.rank = static_cast<int32_t>(p.y_shape.size());
    for (size_t i = 0; i < p.y_shape.size(); ++i) y.shape[i] = p.y_shape[i];
    uint64_t n = 1;
    for (auto d : p.y_shape) n *= static_cast<uint64_t>(d);
    y.nbytes = n * dtype_bytes(p.y_dtype);
  }
  return XRGPU_OK;
}

int xrgpu_prepare(const char* package_directory, const xrgpu_request* request, const xrgpu_options* options,
                  xrgpu_operator** out) {
  if (!out) return fail(XRGPU_INVALID_ARGUMENT, "Null output handle");
  *out = nullptr;
  if (request && is_family_operation(request->operation)) {
    const xrgpu_request_ex ex = extend_request(request);
    return xrgpu_prepare_ex(package_directory, &ex, options, out);
  }
  Plan plan;
  int st = make_plan(request, true, &plan);
  if (st) return st;
  xrgpu_options opt;
  xrgpu_default_options(&opt);
  if (options) opt = *options;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return fail(XRGPU_UNAVAILABLE, "no usable CUDA device");
  if (opt.device < 0 || opt.device >= count) return fail(XRGPU_INVALID_ARGUMENT, "Invalid CUDA device ordinal");
  auto* op = new xrgpu_operator();
  op->plan = std::move(plan);
  op->options = opt;
  op->device = opt.device;
  DeviceGuard guard(op->device);
  // Memory limit over everything the handle keeps on the device (operators.h:27).
  uint64_t total = 0;
  for (int s = 0; s < 5; ++s) total += op->plan.in[s].present ? align_up(op->plan.in[s].nbytes, 256) : 0;
  uint64_t ny = 1;
  for (auto d : op->plan.y_shape) ny *= static_cast<uint64_t>(d);
  op->y_bytes = ny * dtype_bytes(op->plan.y_dtype);
  total += align_up(op->y_bytes, 256);
  Problem probe_problem = operator_problem(op);
  probe_problem.a = reinterpret_cast<const void*>(uintptr_t(256));  // aligned placeholders for path selection
  probe_problem.b = reinterpret_cast<const uint8_t*>(uintptr_t(256));
  probe_problem.scales = reinterpret_cast<const void*>(uintptr_t(256));
  op->path = select_path(probe_problem, kPathAuto);
  op->workspace_bytes = workspace_for(probe_problem, op->path);
  total += op->workspace_bytes;
  if (total > opt.memory_limit_bytes) {
    delete op;
    return fail(XRGPU_INVALID_ARGUMENT, "Extended heap memory limit exceeded");
  }
  auto cleanup = [&](const std::string& why) {
    release(op);
    delete op;
    return fail(XRGPU_RUNTIME_ERROR, why);
  };
  if (cudaStreamCreateWithFlags(&op->stream, cudaStreamNonBlocking) != cudaSuccess) return cleanup("cudaStreamCreate failed");
  if (cudaEventCreate(&op->ev_start) != cudaSuccess || cudaEventCreate(&op->ev_stop) != cudaSuccess) return cleanup("cudaEventCreate failed");
  for (int s = 0; s < 5; ++s) {
    const TensorMeta& m = op->plan.in[s];
    if (!m.present) continue;
    if (cudaMalloc(&op->dev_in[s], std::max<uint64_t>(m.nbytes, 16)) != cudaSuccess) return cleanup(std::string("device allocation failed: ") + kInputNames[s]);
    if (m.nbytes && cudaMemcpy(op->dev_in[s], m.data, m.nbytes, cudaMemcpyHostToDevice) != cudaSuccess)
      return cleanup(std::string("host to device copy failed: ") + kInputNames[s]);
    op->plan.in[s].data = nullptr;  // the handle owns its device snapshot
  }
  if (cudaMalloc(&op->dev_y, std::max<uint64_t>(op->y_bytes, 16)) != cudaSuccess) return cleanup("device allocation failed: yT");
  if (op->workspace_bytes) {
    if (cudaMalloc(&op->workspace, op->workspace_bytes) != cudaSuccess) return cleanup("workspace allocation failed");
    if (cudaMemset(op->workspace, 0, op->workspace_bytes) != cudaSuccess) return cleanup("workspace clear failed");
  }
  // Re-select with the real (aligned) device pointers.
  const Problem real = operator_problem(op);
  const int path = select_path(real, kPathAuto);
  if (path != op->path) {
    op->path = path;
    if (workspace_for(real, path) > op->workspace_bytes) return cleanup("workspace size changed after allocation");
  }
  *out = op;
  return XRGPU_OK;
}

int xrgpu_run_async(xrgpu_operator* op, void* stream) {
  int st = check_open(op);
  if (st) return st;
  DeviceGuard guard(op->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : op->stream;
  if (op->family) {
    st = family_launch(op->family, s);
    if (st) return poison(op, st == XRGPU_INVALID_ARGUMENT ? XRGPU_RUNTIME_ERROR : st, xrgpu_last_error());
    op->dispatch_count += 1;
    op->executed = true;
    return XRGPU_OK;
  }
  const Problem p = operator_problem(op);
  const cudaError_t e = launch_path(p, op->path, op->workspace, s);
  if (e != cudaSuccess) return poison(op, XRGPU_RUNTIME_ERROR, std::string("kernel launch failed: ") + cudaGetErrorString(e));
  op->dispatch_count += 1;
  op->executed = true;
  return XRGPU_OK;
}

int xrgpu_run(xrgpu_operator* op) {
  int st = check_open(op);
  if (st) return st;
  DeviceGuard guard(op->device);
  const auto t0 = std::chrono::steady_clock::now();
  cudaEventRecord(op->ev_start, op->stream);
  st = xrgpu_run_async(op, nullptr);
  if (st) return st;
  cudaEventRecord(op->ev_stop, op->stream);
  st = wait_bounded(op, op->ev_stop);
  const auto t1 = std::chrono::steady_clock::now();
  op->execution_ms = std::chrono::duration<double, std::milli>(t1 - t0).count();
  if (st) return st;
  if (op->options.profiling) {
    float ms = 0;
    if (cudaEventElapsedTime(&ms, op->ev_start, op->ev_stop) == cudaSuccess) op->gpu_ms = ms;
  }
  return XRGPU_OK;
}

int xrgpu_sync(xrgpu_operator* op) {
  int st = check_open(op);
  if (st) return st;
  DeviceGuard guard(op->device);
  cudaEventRecord(op->ev_stop, op->stream);
  return wait_bounded(op, op->ev_stop);
}

int xrgpu_read_outputs(const xrgpu_operator* op, int32_t index, void* dst, uint64_t capacity) {
  int st = check_open(op);
  if (st) return st;
  void* src = op->dev_y;
  uint64_t bytes = op->y_bytes;
  if (op->family) {
    if (index < 0 || index >= static_cast<int32_t>(op->family->out.size()))
      return fail(XRGPU_INVALID_ARGUMENT, "output index outside the planned outputs");
    src = op->family->out[index].dev;
    bytes = op->family->out[index].nbytes;
  } else if (index != 0) {
    return fail(XRGPU_INVALID_ARGUMENT, "MatMulNBits has one output (index 0, yT)");
  }
  if (capacity < bytes || (bytes && !dst)) return fail(XRGPU_INVALID_ARGUMENT, "output buffer too small");
  DeviceGuard guard(op->device);
  if (!op->executed) return fail(XRGPU_RUNTIME_ERROR, "Operator has not run");
  if (bytes && cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, op->stream) != cudaSuccess)
    return fail(XRGPU_RUNTIME_ERROR, "device to host copy failed");
  if (cudaStreamSynchronize(op->stream) != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, "device to host copy failed");
  return XRGPU_OK;
}

int xrgpu_output_device_ptr(const xrgpu_operator* op, int32_t index, void** ptr) {
  int st = check_open(op);
  if (st) return st;
  if (!ptr) return fail(XRGPU_INVALID_ARGUMENT, "invalid output index or pointer");
  if (op->family) {
    if (index < 0 || index >= static_cast<int32_t>(op->family->out.size()))
      return fail(XRGPU_INVALID_ARGUMENT, "invalid output index or pointer");
    *ptr = op->family->out[index].dev;
    return XRGPU_OK;
  }
  if (index != 0) return fail(XRGPU_INVALID_ARGUMENT, "invalid output index or pointer");
  *ptr = op->dev_y;
  return XRGPU_OK;
}

int xrgpu_write_input(xrgpu_operator* op, const char* name, const void* data, uint64_t nbytes) {
  int st = check_open(op);
  if (st) return st;
  if (!name) return fail(XRGPU_INVALID_ARGUMENT, "Null input name");
  if (op->family) {
    for (auto& t : op->family->in) {
      if (t.name != name || !t.present) continue;
      if (nbytes != t.nbytes || (nbytes && !data))
        return fail(XRGPU_INVALID_ARGUMENT, std::string("Extended input byte count mismatch: ") + name);
      DeviceGuard guard(op->device);
      if (nbytes && cudaMemcpyAsync(t.dev, data, nbytes, cudaMemcpyHostToDevice, op->stream) != cudaSuccess)
        return poison(op, XRGPU_RUNTIME_ERROR, "host to device copy failed");
      if (cudaStreamSynchronize(op->stream) != cudaSuccess) return poison(op, XRGPU_RUNTIME_ERROR, "host to device copy failed");
      return XRGPU_OK;
    }
    return fail(XRGPU_INVALID_ARGUMENT, std::string("Unknown prepared input: ") + name);
  }
  int slot = -1;
  for (int s = 0; s < 5; ++s)
    if (std::strcmp(name, kInputNames[s]) == 0) slot = s;
  if (slot < 0 || !op->plan.in[slot].present) return fail(XRGPU_INVALID_ARGUMENT, std::string("Unknown prepared input: ") + name);
  if (nbytes != op->plan.in[slot].nbytes || (nbytes && !data)) return fail(XRGPU_INVALID_ARGUMENT, std::string("Extended input byte count mismatch: ") + name);
  DeviceGuard guard(op->device);
  if (nbytes && cudaMemcpyAsync(op->dev_in[slot], data, nbytes, cudaMemcpyHostToDevice, op->stream) != cudaSuccess)
    return poison(op, XRGPU_RUNTIME_ERROR, "host to device copy failed");
  if (cudaStreamSynchronize(op->stream) != cudaSuccess) return poison(op, XRGPU_RUNTIME_ERROR, "host to device copy failed");
  return XRGPU_OK;
}

int xrgpu_info(const xrgpu_operator* op, char* json, uint64_t capacity, uint64_t* needed) {
  if (!op) return fail(XRGPU_INVALID_ARGUMENT, "Null operator");
  std::ostringstream o;
  if (op->family) {
    const FamilyOp& f = *op->family;
    o << "{\"backend\":\"cuda\",\"operation\":\"" << f.operation << "\",\"device\":\""
      << json_escape(device_description(op->device)) << "\",\"cpu_compute_fallback\":false,\"execution_ms\":"
      << op->execution_ms << ",\"gpu_ms\":";
    if (op->gpu_ms >= 0) o << op->gpu_ms; else o << "null";
    o << ",\"dispatch_count\":" << op->dispatch_count << ",\"executed\":" << (op->executed ? "true" : "false")
      << ",\"closed\":" << (op->closed ? "true" : "false") << ",\"poisoned\":" << (op->poisoned ? "true" : "false")
      << ",\"workspace_bytes\":" << f.workspace_bytes << ",\"inputs\":[";
    bool first_in = true;
    for (const auto& t : f.in) {
      if (!t.present) continue;
      o << (first_in ? "" : ",") << "{\"name\":\"" << t.name << "\",\"dtype\":\"" << dtype_name(t.dtype) << "\",\"shape\":[";
      for (size_t i = 0; i < t.shape.size(); ++i) o << (i ? "," : "") << t.shape[i];
      o << "]}";
      first_in = false;
    }
    o << "],\"outputs\":[";
    for (size_t j = 0; j < f.out.size(); ++j) {
      o << (j ? "," : "") << "{\"name\":\"" << f.out[j].name << "\",\"dtype\":\"" << dtype_name(f.out[j].dtype) << "\",\"shape\":[";
      for (size_t i = 0; i < f.out[j].shape.size(); ++i) o << (i ? "," : "") << f.out[j].shape[i];
      o << "]}";
    }
    o << "]}";
    return write_json(o.str(), json, capacity, needed);
  }
  const Plan& p = op->plan;
  o << "{\"backend\":\"cuda\",\"operation\":\"" << kOperation << "\",\"device\":\"" << json_escape(device_description(op->device))
    << "\",\"cpu_compute_fallback\":false,\"path\":\"" << path_name(op->path) << "\",\"execution_ms\":" << op->execution_ms
    << ",\"gpu_ms\":";
  if (op->gpu_ms >= 0) o << op->gpu_ms; else o << "null";
  o << ",\"dispatch_count\":" << op->dispatch_count << ",\"executed\":" << (op->executed ? "true" : "false")
    << ",\"closed\":" << (op->closed ? "true" : "false") << ",\"poisoned\":" << (op->poisoned ? "true" : "false")
    << ",\"workspace_bytes\":" << op->workspace_bytes << ",\"attributes\":{\"K\":" << p.K << ",\"N\":" << p.N
    << ",\"block_size\":" << p.bs << ",\"bits\":" << p.bits << ",\"accuracy_level\":" << p.accuracy << "},\"inputs\":[";
  bool first = true;
  for (int s = 0; s < 5; ++s) {
    if (!p.in[s].present) continue;
    o << (first ? "" : ",") << "{\"name\":\"" << kInputNames[s] << "\",\"dtype\":\"" << dtype_name(p.in[s].dtype) << "\",\"shape\":[";
    for (size_t i = 0; i < p.in[s].shape.size(); ++i) o << (i ? "," : "") << p.in[s].shape[i];
    o << "]}";
    first = false;
  }
  o << "],\"outputs\":[{\"name\":\"yT\",\"dtype\":\"" << dtype_name(p.y_dtype) << "\",\"shape\":[";
  for (size_t i = 0; i < p.y_shape.size(); ++i) o << (i ? "," : "") << p.y_shape[i];
  o << "]}]}";
  return write_json(o.str(), json, capacity, needed);
}

int xrgpu_close(xrgpu_operator* op) {
  if (!op) return fail(XRGPU_INVALID_ARGUMENT, "Null operator");
  if (op->closed) return XRGPU_OK;
  release(op);
  op->closed = true;
  return XRGPU_OK;
}

void xrgpu_destroy(xrgpu_operator* op) {
  if (!op) return;
  if (!op->closed) xrgpu_close(op);
  delete op->family;
  delete op;
}

int xrgpu_plan_ex(const xrgpu_request_ex* request, xrgpu_tensor* outputs, int32_t capacity, int32_t* count) {
  if (!request) return fail(XRGPU_INVALID_ARGUMENT, "Null request");
  if (!is_family_operation(request->operation)) {
    const xrgpu_request plain = plain_request(request);
    return xrgpu_plan(&plain, outputs, capacity, count);
  }
  FamilyOp plan;
  const int st = family_plan(request, false, &plan);
  if (st) return st;
  static const char* kNames[] = {"yT", "residualT", "qT", "kT", "vT", "outputT"};
  if (count) *count = static_cast<int32_t>(plan.out.size());
  for (int32_t i = 0; outputs && i < capacity && i < static_cast<int32_t>(plan.out.size()); ++i) {
    xrgpu_tensor& y = outputs[i];
    std::memset(&y, 0, sizeof(y));
    for (const char* n : kNames)
      if (plan.out[i].name == n) y.name = n;  // names with static storage
    y.dtype = plan.out[i].dtype;
    y.rank = static_cast<int32_t>(plan.out[i].shape.size());
    for (size_t d = 0; d < plan.out[i].shape.size(); ++d) y.shape[d] = plan.out[i].shape[d];
    y.nbytes = plan.out[i].nbytes;
  }
  return XRGPU_OK;
}

int xrgpu_prepare_ex(const char* package_directory, const xrgpu_request_ex* request, const xrgpu_options* options,
                     xrgpu_operator** out) {
  if (!out) return fail(XRGPU_INVALID_ARGUMENT, "Null output handle");
  *out = nullptr;
  if (!request) return fail(XRGPU_INVALID_ARGUMENT, "Null request");
  if (!is_family_operation(request->operation)) {
    const xrgpu_request plain = plain_request(request);
    return xrgpu_prepare(package_directory, &plain, options, out);
  }
  FamilyOp plan;
  int st = family_plan(request, true, &plan);
  if (st) return st;
  xrgpu_options opt;
  xrgpu_default_options(&opt);
  if (options) opt = *options;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return fail(XRGPU_UNAVAILABLE, "no usable CUDA device");
  if (opt.device < 0 || opt.device >= count) return fail(XRGPU_INVALID_ARGUMENT, "Invalid CUDA device ordinal");
  auto* op = new xrgpu_operator();
  op->options = opt;
  op->device = opt.device;
  op->family = new FamilyOp(std::move(plan));
  DeviceGuard guard(op->device);
  auto cleanup = [&](int status, const std::string& why) {
    release(op);
    delete op->family;
    delete op;
    return fail(status, why);
  };
  if (cudaStreamCreateWithFlags(&op->stream, cudaStreamNonBlocking) != cudaSuccess)
    return cleanup(XRGPU_RUNTIME_ERROR, "cudaStreamCreate failed");
  if (cudaEventCreate(&op->ev_start) != cudaSuccess || cudaEventCreate(&op->ev_stop) != cudaSuccess)
    return cleanup(XRGPU_RUNTIME_ERROR, "cudaEventCreate failed");
  st = family_allocate(op->family, opt.memory_limit_bytes);
  if (st) return cleanup(st, xrgpu_last_error());
  *out = op;
  return XRGPU_OK;
}

// ------------------------------------------------------------------ zero-copy API
int xrgpu_mmnb_workspace_size(const xrgpu_mmnb_problem* c, uint64_t* bytes) {
  Problem p;
  const int st = problem_from_c(c, &p, false);
  if (st) return st;
  const int path = select_path(p, c->path);
  if (path < 0) return fail(XRGPU_INVALID_ARGUMENT, "requested kernel path does not support this problem");
  if (bytes) *bytes = workspace_for(p, path);
  return XRGPU_OK;
}

int xrgpu_mmnb_select_path(const xrgpu_mmnb_problem* c, char* name, uint64_t capacity) {
  Problem p;
  const int st = problem_from_c(c, &p, false);
  if (st) return st;
  const int path = select_path(p, c->path);
  if (path < 0) return fail(XRGPU_INVALID_ARGUMENT, "requested kernel path does not support this problem");
  return write_json(path_name(path), name, capacity, nullptr);
}

int xrgpu_mmnb_forward(const xrgpu_mmnb_problem* c, void* workspace, uint64_t workspace_bytes, void* stream) {
  Problem p;
  int st = problem_from_c(c, &p, true);
  if (st) return st;
  const int path = select_path(p, c->path);
  if (path < 0) return fail(XRGPU_INVALID_ARGUMENT, "requested kernel path does not support this problem");
  const uint64_t need = workspace_for(p, path);
  void* ws = workspace;
  if (need) {
    if (!ws) {
      st = library_workspace(need, &ws);
      if (st) return st;
    } else if (workspace_bytes < need) {
      return fail(XRGPU_INVALID_ARGUMENT, "workspace too small: need " + std::to_string(need) + " bytes");
    }
  }
  p.err = device_error_word();
  const cudaError_t e = launch_path(p, path, ws, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, std::string("kernel launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

int xrgpu_mmnb_dequantize(const xrgpu_mmnb_problem* c, float* w, void* stream) {
  Problem p;
  const int st = problem_from_c(c, &p, false);
  if (st) return st;
  if (!w) return fail(XRGPU_INVALID_ARGUMENT, "null output pointer");
  const cudaError_t e = launch_dequant(p, w, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, std::string("kernel launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

int xrgpu_device_error(int32_t device, uint32_t* code, int32_t clear) {
  DeviceGuard guard(device);
  const cudaError_t e = read_device_error(code, clear != 0);
  if (e != cudaSuccess) return fail(XRGPU_RUNTIME_ERROR, std::string("device error word unreadable: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

}  // extern "C"
