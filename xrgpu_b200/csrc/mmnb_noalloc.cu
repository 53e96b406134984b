// MatMulNBitsMlp with scratch the library never allocates: a fixed array in device memory.
//
// Some callers cannot let a library allocate device memory in the middle of their work: a serving
// engine that plans every byte of the GPU up front and gives a library none of it, a real-time
// decode loop where cudaMalloc's implicit device synchronisation would stall the stream, or code
// that runs where the CUDA allocator must not be called at all. xrgpu_mlp_forward needs scratch for
// the normalised activations and the two projections; given no workspace it takes the library's
// per-device workspace, which it allocates on first use. xrgpu_mlp_forward_static runs the same
// kernels on a file-scope __device__ array instead and calls no allocator.
//
// The array is XRGPU_STATIC_SCRATCH_BYTES (4 MiB) and every GPU that loads the library holds it
// until the process exits. Host code cannot use the array's name as a device address: the first
// call on a device looks up the address with cudaGetSymbolAddress (that device current) and keeps
// it. Every call shares the array and it keeps the last call's contents; the Mlp writes each region
// before reading it, so nothing needs clearing. Calls that overlap on the GPU (different streams,
// or different host threads) race on the array.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "mmnb_family_ops.h"
#include "mmnb_internal.h"
#include "xrgpu_mmnb.h"

namespace xrgpu {
namespace {

constexpr uint64_t kStaticScratchBytes = XRGPU_STATIC_SCRATCH_BYTES;

// One array per GPU, alive until the process exits.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_address[kMaxDevices];  // device address of g_static_scratch per device (set once)
std::mutex g_scratch_mutex;

// The array's device address on the current device, looked up on that device's first call.
int static_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return api_fail(XRGPU_RUNTIME_ERROR, "cudaGetDevice failed");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_address[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return api_fail(XRGPU_RUNTIME_ERROR,
                      std::string("static scratch: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    g_scratch_address[dev] = ptr;
  }
  *out = g_scratch_address[dev];
  return XRGPU_OK;
}

}  // namespace
}  // namespace xrgpu

extern "C" {

int xrgpu_mlp_forward_static(const xrgpu_mlp_problem* p, void* stream) {
  using namespace xrgpu;
  if (!p) return api_fail(XRGPU_INVALID_ARGUMENT, "Null problem");
  uint64_t need = 0;
  int st = xrgpu_mlp_workspace_size(p, &need);
  if (st) return st;
  if (need > kStaticScratchBytes)
    return api_fail(XRGPU_INVALID_ARGUMENT,
                    "MatMulNBitsMlp needs " + std::to_string(need) + " bytes of scratch, more than the " +
                        std::to_string(kStaticScratchBytes) +
                        " bytes of static scratch; use xrgpu_mlp_forward with a caller workspace");
  void* scratch = nullptr;
  if (need > 0 && (st = static_scratch(&scratch))) return st;
  return mlp_forward(*p, scratch, kStaticScratchBytes, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
