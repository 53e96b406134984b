// Internal interface between the operator API (mmnb_api.cu) and the operators around MatMulNBits
// (mmnb_family_api.cu): their plans, device snapshots and launches.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "xrgpu_mmnb.h"

namespace xrgpu {

struct FamilyTensor {
  std::string name;
  bool present = false;
  int dtype = XRGPU_UNSPECIFIED;
  std::vector<int64_t> shape;
  uint64_t nbytes = 0;
  const void* host = nullptr;  // prepare's source (not kept)
  void* dev = nullptr;
};

struct FamilyOp {
  int code = 0;  // 1026 MatMulBnb4, 1027 MatMulNBitsMlp, 1028 MatMulNBitsQkv, 1030 QMoE, 1031 GatherBlockQuantized
  std::string operation;
  std::vector<FamilyTensor> in;   // canonical input order (complex_plan.cpp:33-40)
  std::vector<FamilyTensor> out;  // planned output order
  std::vector<int> out_slot;      // canonical output slot of each planned output
  int64_t M = 0, K = 0, N = 0, Nq = 0, Nkv = 0, bs = 0, bits = 4, quant_type = 1;
  int64_t k = 1, swiglu_fusion = 0, experts = 0, fc1_rows = 0, hidden = 0;
  int act = XRGPU_ACT_SILU;
  double epsilon = 1e-5, alpha = 1.0, beta = 0.0, limit = 0.0;
  bool has_limit = false;
  void* workspace = nullptr;
  uint64_t workspace_bytes = 0;
};

bool is_family_operation(const char* operation);
// Validation and output inference (need_data: also check byte counts and data pointers).
int family_plan(const xrgpu_request_ex* r, bool need_data, FamilyOp* op);
// Device snapshot of every input, output buffers and workspace, bounded by memory_limit.
int family_allocate(FamilyOp* op, uint64_t memory_limit);
int family_launch(FamilyOp* op, cudaStream_t s);
void family_release(FamilyOp* op);

// Zero-copy forwards (also used by family_launch).
int mlp_forward(const xrgpu_mlp_problem& c, void* ws, uint64_t ws_bytes, cudaStream_t s);
int qkv_forward(const xrgpu_qkv_problem& c, void* ws, uint64_t ws_bytes, cudaStream_t s);
int bnb4_forward(const xrgpu_bnb4_problem& c, cudaStream_t s);
int gather_forward(const xrgpu_gather_problem& c, cudaStream_t s);
int qmoe_forward(const xrgpu_qmoe_problem& c, void* ws, uint64_t ws_bytes, cudaStream_t s);

}  // namespace xrgpu
