// Internal declarations shared by the host API and the kernel translation units.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <string>

#include "xrgpu_mmnb.h"

namespace xrgpu {

enum ZpKind : int { kZpNone = 0, kZpF32 = 1, kZpF16 = 2, kZpPacked = 3 };
enum Path : int { kPathAuto = 0, kPathGeneric = 1, kPathGemv = 2, kPathGemm = 3 };

// A fully validated MatMulNBits problem over device pointers.
struct Problem {
  int f16;            // 1: aT/scalesT/biasT/yT are float16, 0: float32
  int zp;             // ZpKind
  int64_t M, K, N, bs, bits, kb, blob, ldy;
  const void* a;
  const uint8_t* b;
  const void* scales;
  const void* zp_ptr;
  const void* bias;
  void* y;
  unsigned* err;      // device error word (see device_error_word())
};

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Generic path: any bits / block size / dtype / zero-point form, float32 accumulation.
cudaError_t launch_generic(const Problem& p, cudaStream_t s);
// Exact float32 dequantization W[N, K] (nbitWeight).
cudaError_t launch_dequant(const Problem& p, float* w, cudaStream_t s);

// 4-bit decode GEMV on mma.sync tensor cores, M <= 16, float16 activations.
bool gemv_supported(const Problem& p);
uint64_t gemv_workspace_bytes(const Problem& p);
cudaError_t launch_gemv(const Problem& p, void* workspace, cudaStream_t s);
// Its single-row (M == 1) form: scale and zero point applied after the MMA.
bool gemv_m1_supported(const Problem& p);
cudaError_t launch_gemv_m1(const Problem& p, cudaStream_t s);
// Its single-row form with the weights staged through shared memory by asynchronous copies.
bool gemv_staged_supported(const Problem& p);
cudaError_t launch_gemv_staged(const Problem& p, cudaStream_t s);
// Sharded form of the staged GEMV (peer all-gather, flag-in-word layout): every output column
// n < cols is also sent to each other rank r as part of the word of columns (n & ~1, n | 1), at
// region[r] + words_off + ((e & 1) world + rank) ll_bytes + 4 (n & ~1), e = *epoch + 1.
struct StagedPush {
  int world, rank, cols;
  const uint32_t* epoch;  // the group's epoch (a slot the all-gather's receive advances once per call)
  char* region[16];       // every rank's peer-memory region, as mapped on this device
  int64_t words_off, ll_bytes;
};
cudaError_t launch_gemv_staged_push(const Problem& p, const StagedPush* push, cudaStream_t s);

// Its multi-row form (1..16 rows, block size 128 or 256), weights staged like the single-row form.
bool gemv_mr_supported(const Problem& p);
cudaError_t launch_gemv_mr(const Problem& p, cudaStream_t s);

// 4-bit prefill GEMM on tcgen05 tensor cores (sm_100a), float16 activations.
bool gemm_supported(const Problem& p);
uint64_t gemm_workspace_bytes(const Problem& p);
cudaError_t launch_gemm(const Problem& p, void* workspace, cudaStream_t s);

// Encodes a 2-D TMA tensor map into `map` (a CUtensorMap, 64-byte aligned, 128 bytes) through the
// driver entry point resolved at run time. dtype: 0 = uint8, 1 = float16. Returns false on failure.
bool encode_tensor_map_2d(void* map, int dtype, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                          uint32_t box_inner, uint32_t box_outer, bool swizzle_128b);

// Records `message` as the calling thread's last error (xrgpu_last_error) and returns `status`.
int api_fail(int status, const std::string& message);

// Device error word of the current device (nonzero after a kernel's bounded wait expired).
unsigned* device_error_word();
cudaError_t read_device_error(uint32_t* code, bool clear);

// Validates a C-ABI problem and converts it (need_y: A and Y must be given when M > 0).
int problem_from_api(const xrgpu_mmnb_problem* c, Problem* p, bool need_y);

// The planner's kernel choice for a problem (forced: a Path, kPathAuto = the planner's), -1 when a
// forced path does not support it; its name; its scratch bytes; and its launch.
int select_path(const Problem& p, int forced);
const char* path_name(int path);
uint64_t workspace_for(const Problem& p, int path);
cudaError_t launch_path(const Problem& p, int path, void* ws, cudaStream_t s);
// Per-device library workspace for callers that pass none (zero-filled, grows on demand).
int library_workspace(uint64_t need, void** out);
std::string json_escape(const std::string& s);
int write_json(const std::string& s, char* out, uint64_t capacity, uint64_t* needed);
std::string device_description(int dev);

}  // namespace xrgpu
