// All-gather of Y shards over NVLink peer memory for column-sharded MatMulNBits (one process per
// GPU on one node). The reference backend is single-device; this is the exchange step of the
// N-sharded form, written to replace one NCCL all-gather per projection with a single small kernel
// that CUDA graphs can capture.
//
// Each rank owns one region (cudaMalloc, shared with the other ranks by CUDA IPC):
//   [0, 4 KB)       done flags: done[q][c] = last epoch in which rank q finished writing chunk c here
//   [4 KB, ...)     staging[2][world][slot_bytes]: rank q's shard of epoch e lands in staging[e & 1][q]
//   then            words[2][world][ll_bytes]: the same for the low-latency form below (kept apart, so
//                   that raw shard bytes are never read as words)
// The shard (rows x row bytes, contiguous) is cut into `chunks` byte chunks (4 for decode shards,
// up to 64 of ~256 KB for large ones; every rank derives the same count from the same size). Every
// call advances ONE epoch per peer, whatever its chunk count: epoch[p][c] holds the same value for
// all 64 chunk slots c of peer p, and the CTA of chunk c advances the slots c, c + chunks, c + 2 chunks,
// ... so that each slot is advanced exactly once per call. A call on rank r (epoch e) runs one CTA per
// (peer p, chunk c):
//   * p == r: the CTA copies chunk c of r's own shard into r's block of Y;
//   * p != r: the CTA stores chunk c of r's shard into p's staging[e & 1][r] (peer stores over
//     NVLink), and after a CTA barrier one thread sets p's done[r][c] = e with a release store at
//     system scope (the barrier orders every thread's stores before it, and release is cumulative);
//     it then waits until its own done[p][c] >= e (acquire, bounded) and copies chunk c of p's shard
//     from its own staging into p's block of Y.
// Staging is double-buffered by epoch parity, so no "ready" handshake is needed. Rank r writes any
// byte of p's staging[e & 1][r] in call e only after its call e - 1 completed, and that call saw
// done[p][c] >= e - 1 for at least one chunk c. p sets that flag in its call e - 1, which starts
// (griddepcontrol.wait, stream order) after p's call e - 2 -- the last reader of staging[e & 1] --
// has finished. Because the epoch is per call, not per chunk, this holds whatever byte ranges the
// chunks of calls e - 2 and e cover (shards of different sizes on one group).
// Shards up to kLLMaxBytes (decode) take a lower-latency form of the same exchange: every 8-byte
// word sent carries 4 bytes of the shard and the call's epoch, written with one 64-bit store (single-
// copy atomic), so the receiver polls the words themselves until each holds epoch e and no fence,
// release or separate flag is needed on either side. Such a shard takes twice its size in staging;
// the same parity and per-call epoch argument covers it (a word of an older call holds an older
// epoch and is not taken).
// Every rank must make the same sequence of calls on its group. Waits give up after 1 s and record
// kErrPeerWait in the device error word; the group is then out of step and must be destroyed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <string>

#include "mmnb_common.cuh"
#include "mmnb_internal.h"
#include "xrgpu_mmnb.h"

struct xrgpu_p2p {
  int device = 0, world = 0, rank = 0;
  uint64_t slot_bytes = 0;   // largest shard a call may pass (raw staging per parity and rank)
  uint64_t ll_bytes = 0;     // word staging per parity and rank: 2 x min(slot_bytes, kLLMaxBytes)
  uint64_t region_bytes = 0;
  char* local = nullptr;
  char* peers[XRGPU_P2P_MAX_WORLD] = {};
  bool opened[XRGPU_P2P_MAX_WORLD] = {};
  uint32_t* epoch = nullptr;  // device [XRGPU_P2P_MAX_WORLD][64]: epoch of the last call per peer, one copy
                              // per chunk slot (all 64 copies of a peer are equal between calls)
};

namespace xrgpu {
namespace {

constexpr int kMaxChunks = 64;                              // CTAs per peer at most
constexpr int kFlagBytes = XRGPU_P2P_MAX_WORLD * kMaxChunks * 4;  // one done flag per (rank, chunk)
// Threads per CTA: 256 for large shards (copy bandwidth), 128 for decode-sized ones, so that a CTA
// (40 registers a thread: 5,120 a CTA) fits in the 8,192 registers a decode GEMV CTA leaves free on
// its SM and a spinning all-gather never holds an SM that the next GEMV's CTA is waiting for.
constexpr int kThreads = 256;
constexpr int kSmallThreads = 128;
constexpr int64_t kSmallShardBytes = 1 << 20;
constexpr int64_t kLLMaxBytes = 1 << 20;  // shards up to 1 MB travel as (4 data bytes, epoch) words
constexpr int64_t kLLPairsPerThread = 4;  // 16-byte word pairs a thread sends per chunk at most
constexpr int kMinChunks = 4;  // CTAs per peer for small shards: the peer stores spread over 4 SMs
constexpr int64_t kChunkBytes = 256 * 1024;  // target chunk size for large shards
constexpr unsigned kErrPeerWait = 0x401;

struct P2PParams {
  char* peers[XRGPU_P2P_MAX_WORLD];
  uint32_t* epoch;
  const char* shard;  // [rows][srb]
  char* out;          // [rows][orb], rank q's block at byte q * srb, first ovb bytes of a row valid
  int64_t rows, srb, orb, ovb, slot_bytes, ll_bytes;
  int world, rank, chunks;
  unsigned* err;
};

// One 16-byte vector of two 64-bit elements: each element is written and read as one single-copy
// atomic access, so a word's data and epoch are always seen together.
__device__ __forceinline__ void st_ll_pair(void* p, uint64_t w0, uint64_t w1) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
}
__device__ __forceinline__ void ld_ll_pair(const void* p, uint64_t& w0, uint64_t& w1) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Copies bytes [lo, hi) of a contiguous [rows][srb] shard (lo, hi and srb multiples of 16) into
// the rows of dst (row stride orb), keeping only the first `valid` bytes of each row. kCg: read
// the source through L2 only (it was written by another GPU).
template <bool kCg>
__device__ void copy_chunk(char* dst, int64_t orb, const char* src, int64_t srb, int64_t lo, int64_t hi, int64_t valid) {
  if (valid <= 0) return;
  const int64_t width = valid < srb ? valid : srb;
  for (int64_t o = lo + 16 * static_cast<int64_t>(threadIdx.x); o < hi; o += 16 * static_cast<int64_t>(blockDim.x)) {
    const int64_t m = o / srb, j = o - m * srb;
    if (j >= width) continue;
    const uint4* s = reinterpret_cast<const uint4*>(src + o);
    if (j + 16 <= width) {
      const uint4 v = kCg ? __ldcg(s) : *s;
      *reinterpret_cast<uint4*>(dst + m * orb + j) = v;
    } else {  // ragged end of the last block
      for (int64_t t = j; t < width; ++t)
        dst[m * orb + t] = kCg ? static_cast<char>(__ldcg(reinterpret_cast<const unsigned char*>(src + m * srb + t)))
                               : src[m * srb + t];
    }
  }
}

__global__ void __launch_bounds__(kThreads) p2p_allgather_kernel(const __grid_constant__ P2PParams q) {
  // Programmatic dependent launch: the next kernel may start (its own griddepcontrol.wait then
  // waits for this one); this kernel reads the shard only after the previous kernel completed.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int p = static_cast<int>(blockIdx.x) / q.chunks, c = static_cast<int>(blockIdx.x) % q.chunks;
  const int64_t bytes = q.rows * q.srb;
  const int64_t per = (bytes / 16 + q.chunks - 1) / q.chunks * 16;
  const int64_t lo = per * c < bytes ? per * c : bytes, hi = per * (c + 1) < bytes ? per * (c + 1) : bytes;
  const int64_t block_off = static_cast<int64_t>(p) * q.srb;
  const int64_t valid = q.ovb - block_off;
  if (p == q.rank) {
    copy_chunk<false>(q.out + block_off, q.orb, q.shard, q.srb, lo, hi, valid);
    return;
  }
  __shared__ uint32_t epoch_s;
  __shared__ int ok_s;
  uint32_t* epoch = q.epoch + p * kMaxChunks;  // kMaxChunks equal slots of peer p
  if (threadIdx.x == 0) epoch_s = epoch[c] + 1u;
  __syncthreads();
  const uint32_t e = epoch_s;
  const int64_t slot_off = kFlagBytes + (static_cast<int64_t>(e & 1u) * q.world + q.rank) * q.slot_bytes;
  // 1. chunk c of this rank's shard into p's staging (16-byte vectors)
  {
    const uint4* src = reinterpret_cast<const uint4*>(q.shard + lo);
    uint4* dst = reinterpret_cast<uint4*>(q.peers[p] + slot_off + lo);
    for (int64_t i = threadIdx.x; i < (hi - lo) / 16; i += blockDim.x) dst[i] = src[i];
  }
  __syncthreads();
  // 2. publish (release, system scope), then wait for p's chunk in this rank's staging
  if (threadIdx.x == 0) {
    st_release_sys(reinterpret_cast<uint32_t*>(q.peers[p]) + q.rank * kMaxChunks + c, e);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(q.peers[q.rank]) + p * kMaxChunks + c;
    int ok = 1;
    if (static_cast<int32_t>(ld_acquire_sys(mine) - e) < 0) {
      const uint64_t start = global_timer_ns();
      while (static_cast<int32_t>(ld_acquire_sys(mine) - e) < 0) {
        if (global_timer_ns() - start > kWaitLimitNs) {
          record_device_error(q.err, kErrPeerWait);
          ok = 0;
          break;
        }
        __nanosleep(32);
      }
    }
    ok_s = ok;
    for (int slot = c; slot < kMaxChunks; slot += q.chunks) epoch[slot] = e;  // every slot once per call
  }
  __syncthreads();
  // 3. chunk c of p's shard from this rank's staging into p's block of Y
  if (ok_s) {
    const char* src = q.peers[q.rank] + kFlagBytes + (static_cast<int64_t>(e & 1u) * q.world + p) * q.slot_bytes;
    copy_chunk<true>(q.out + block_off, q.orb, src, q.srb, lo, hi, valid);
  }
}

// Low-latency form (shards of at most kLLMaxBytes). CTA (p, c) handles 8-byte pair range
// [lo, hi) of the shard. p == rank: copies it into Y. p != rank: sends it to p as words
// (data | e << 32) into p's staging[e & 1][rank] (16 bytes per 8 data bytes), then polls its own
// staging[e & 1][p] until both words of each of its pairs hold epoch e and writes their data into
// p's block of Y. No fence is needed: a word carries its own validity.
__global__ void __launch_bounds__(kThreads) p2p_allgather_ll_kernel(const __grid_constant__ P2PParams q) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int p = static_cast<int>(blockIdx.x) / q.chunks, c = static_cast<int>(blockIdx.x) % q.chunks;
  const int64_t pairs = q.rows * q.srb / 8;
  const int64_t per = (pairs + q.chunks - 1) / q.chunks;
  const int64_t lo = per * c < pairs ? per * c : pairs, hi = per * (c + 1) < pairs ? per * (c + 1) : pairs;
  const int64_t block_off = static_cast<int64_t>(p) * q.srb;
  const int64_t valid = q.ovb - block_off;
  if (p == q.rank) {  // copy_chunk wants 16-byte bounds: split the bytes in 16-byte units instead
    const int64_t bytes = q.rows * q.srb, per16 = (bytes / 16 + q.chunks - 1) / q.chunks * 16;
    const int64_t blo = per16 * c < bytes ? per16 * c : bytes, bhi = per16 * (c + 1) < bytes ? per16 * (c + 1) : bytes;
    copy_chunk<false>(q.out + block_off, q.orb, q.shard, q.srb, blo, bhi, valid);
    return;
  }
  __shared__ uint32_t epoch_s;
  uint32_t* epoch = q.epoch + p * kMaxChunks;
  if (threadIdx.x == 0) epoch_s = epoch[c] + 1u;
  __syncthreads();
  const uint32_t e = epoch_s;
  const uint64_t tag = static_cast<uint64_t>(e) << 32;
  const int64_t ll_base = kFlagBytes + 2 * static_cast<int64_t>(q.world) * q.slot_bytes;
  const int64_t par_off = ll_base + static_cast<int64_t>(e & 1u) * q.world * q.ll_bytes;
  // 1. send: 8 data bytes -> one 16-byte pair of words
  {
    char* dst = q.peers[p] + par_off + static_cast<int64_t>(q.rank) * q.ll_bytes;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
      const uint2 d = *reinterpret_cast<const uint2*>(q.shard + 8 * i);
      st_ll_pair(dst + 16 * i, tag | d.x, tag | d.y);
    }
  }
  // 2. receive p's pairs of this range from this rank's staging
  const char* src = q.peers[q.rank] + par_off + static_cast<int64_t>(p) * q.ll_bytes;
  const int64_t width = valid < q.srb ? valid : q.srb;
  bool ok = true;
  for (int64_t i = lo + threadIdx.x; i < hi && ok; i += blockDim.x) {
    if ((8 * i) % q.srb >= width) continue;  // past this block's valid columns: nothing to take
    uint64_t w0, w1;
    ld_ll_pair(src + 16 * i, w0, w1);
    if (static_cast<uint32_t>(w0 >> 32) != e || static_cast<uint32_t>(w1 >> 32) != e) {
      const uint64_t start = global_timer_ns();
      do {
        if (global_timer_ns() - start > kWaitLimitNs) {
          record_device_error(q.err, kErrPeerWait);
          ok = false;
          break;
        }
        ld_ll_pair(src + 16 * i, w0, w1);
      } while (static_cast<uint32_t>(w0 >> 32) != e || static_cast<uint32_t>(w1 >> 32) != e);
      if (!ok) break;
    }
    const int64_t m = (8 * i) / q.srb, j = 8 * i - m * q.srb;
    char* o = q.out + block_off + m * q.orb + j;
    const uint32_t d0 = static_cast<uint32_t>(w0), d1 = static_cast<uint32_t>(w1);
    if (j + 8 <= width) {
      *reinterpret_cast<uint2*>(o) = make_uint2(d0, d1);
    } else {  // ragged end of the last block
      for (int64_t t = 0; t < width - j; ++t) o[t] = static_cast<char>((t < 4 ? d0 >> (8 * t) : d1 >> (8 * (t - 4))) & 0xff);
    }
  }
  __syncthreads();  // every thread has read epoch_s
  if (threadIdx.x == 0)
    for (int slot = c; slot < kMaxChunks; slot += q.chunks) epoch[slot] = e;  // every slot once per call
}

// Receive side of the fused form (the decode GEMV sent the words), for up to kMaxRecvGroups groups in
// one launch. Group gi has (world - 1) * chunks CTAs; CTA (p, c) takes pairs [lo, hi) of peer p's
// single-row block from this rank's words[e & 1][p] and writes them into Y. The epoch slot and the
// first pair of both parities are loaded together, so the epoch costs no extra round trip.
constexpr int kMaxRecvGroups = 8;
struct RecvGroup {
  const char* words;  // this rank's words[0][0] (region + words offset)
  uint32_t* epoch;    // the group's epoch slots [XRGPU_P2P_MAX_WORLD][kMaxChunks]
  char* out;          // Y: one row, rank q's block at byte q * srb
  int64_t srb, ovb, ll_bytes;
  int world, rank, chunks, first_cta;
};
struct RecvManyParams {
  RecvGroup g[kMaxRecvGroups];
  int count;
  unsigned* err;
};

__device__ __forceinline__ uint32_t ld_volatile_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kSmallThreads) p2p_recv_many_kernel(const __grid_constant__ RecvManyParams P) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int gi = 0;
  while (gi + 1 < P.count && static_cast<int>(blockIdx.x) >= P.g[gi + 1].first_cta) ++gi;
  const RecvGroup& G = P.g[gi];
  const int local = static_cast<int>(blockIdx.x) - G.first_cta;
  int p = local / G.chunks;
  const int c = local % G.chunks;
  if (p >= G.rank) ++p;  // peers only
  const int64_t pairs = G.srb / 8;
  const int64_t per = (pairs + G.chunks - 1) / G.chunks;
  const int64_t lo = per * c < pairs ? per * c : pairs, hi = per * (c + 1) < pairs ? per * (c + 1) : pairs;
  const int64_t block_off = static_cast<int64_t>(p) * G.srb;
  const int64_t valid = G.ovb - block_off;
  const int64_t width = valid < G.srb ? valid : G.srb;
  uint32_t* epoch = G.epoch + p * kMaxChunks;
  const char* par0 = G.words + static_cast<int64_t>(p) * G.ll_bytes;
  const char* par1 = G.words + (static_cast<int64_t>(G.world) + p) * G.ll_bytes;
  int64_t i = lo + threadIdx.x;
  uint64_t a0 = 0, a1 = 0, b0 = 0, b1 = 0;
  if (i < hi && 8 * i < width) {
    ld_ll_pair(par0 + 16 * i, a0, a1);
    ld_ll_pair(par1 + 16 * i, b0, b1);
  }
  const uint32_t e = ld_volatile_u32(epoch + c) + 1u;
  const char* src = (e & 1u) ? par1 : par0;
  uint64_t w0 = (e & 1u) ? b0 : a0, w1 = (e & 1u) ? b1 : a1;
  bool ok = true, first = true;
  for (; i < hi && ok; i += blockDim.x, first = false) {
    if (8 * i >= width) continue;  // past this block's valid columns: never sent
    if (!first) ld_ll_pair(src + 16 * i, w0, w1);
    if (static_cast<uint32_t>(w0 >> 32) != e || static_cast<uint32_t>(w1 >> 32) != e) {
      const uint64_t start = global_timer_ns();
      do {
        if (global_timer_ns() - start > kWaitLimitNs) {
          record_device_error(P.err, kErrPeerWait);
          ok = false;
          break;
        }
        ld_ll_pair(src + 16 * i, w0, w1);
      } while (static_cast<uint32_t>(w0 >> 32) != e || static_cast<uint32_t>(w1 >> 32) != e);
      if (!ok) break;
    }
    char* o = G.out + block_off + 8 * i;
    const uint32_t d0 = static_cast<uint32_t>(w0), d1 = static_cast<uint32_t>(w1);
    if (8 * i + 8 <= width) {
      *reinterpret_cast<uint2*>(o) = make_uint2(d0, d1);
    } else {  // ragged end of the last block
      for (int64_t t = 0; t < width - 8 * i; ++t) o[t] = static_cast<char>((t < 4 ? d0 >> (8 * t) : d1 >> (8 * (t - 4))) & 0xff);
    }
  }
  __syncthreads();  // every thread has read the epoch slot
  if (threadIdx.x == 0)
    for (int slot = c; slot < kMaxChunks; slot += G.chunks) epoch[slot] = e;  // every slot once per call
}

}  // namespace
}  // namespace xrgpu

extern "C" {

int xrgpu_p2p_create(int32_t device, int32_t world, int32_t rank, uint64_t slot_bytes, xrgpu_p2p** group,
                     void* ipc_handle) {
  using namespace xrgpu;
  if (!group || !ipc_handle) return api_fail(XRGPU_INVALID_ARGUMENT, "null group or handle pointer");
  *group = nullptr;
  if (world < 1 || world > XRGPU_P2P_MAX_WORLD || rank < 0 || rank >= world)
    return api_fail(XRGPU_INVALID_ARGUMENT, "world must be in [1, 16] and rank in [0, world)");
  if (slot_bytes == 0 || slot_bytes % 16) return api_fail(XRGPU_INVALID_ARGUMENT, "slot_bytes must be a positive multiple of 16");
  int prev = 0;
  cudaGetDevice(&prev);
  if (cudaSetDevice(device) != cudaSuccess) return api_fail(XRGPU_UNAVAILABLE, "cannot select the CUDA device");
  xrgpu_p2p* g = new (std::nothrow) xrgpu_p2p();
  int st = XRGPU_OK;
  if (!g) {
    st = api_fail(XRGPU_RUNTIME_ERROR, "out of host memory");
  } else {
    g->device = device;
    g->world = world;
    g->rank = rank;
    g->slot_bytes = align_up(slot_bytes, 256);
    g->ll_bytes = 2 * std::min<uint64_t>(g->slot_bytes, kLLMaxBytes);
    g->region_bytes = kFlagBytes + 2 * static_cast<uint64_t>(world) * (g->slot_bytes + g->ll_bytes);
    cudaIpcMemHandle_t h;
    if (cudaMalloc(&g->local, g->region_bytes) != cudaSuccess || cudaMemset(g->local, 0, g->region_bytes) != cudaSuccess ||
        cudaMalloc(&g->epoch, sizeof(uint32_t) * XRGPU_P2P_MAX_WORLD * kMaxChunks) != cudaSuccess ||
        cudaMemset(g->epoch, 0, sizeof(uint32_t) * XRGPU_P2P_MAX_WORLD * kMaxChunks) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess || cudaIpcGetMemHandle(&h, g->local) != cudaSuccess) {
      st = api_fail(XRGPU_RUNTIME_ERROR, "peer-memory region allocation or IPC export failed");
    } else {
      std::memcpy(ipc_handle, &h, sizeof(h));
      g->peers[rank] = g->local;
      *group = g;
    }
  }
  if (st != XRGPU_OK && g) {
    if (g->local) cudaFree(g->local);
    if (g->epoch) cudaFree(g->epoch);
    delete g;
  }
  cudaSetDevice(prev);
  return st;
}

int xrgpu_p2p_connect(xrgpu_p2p* g, const void* ipc_handles) {
  using namespace xrgpu;
  if (!g || !ipc_handles) return api_fail(XRGPU_INVALID_ARGUMENT, "null group or handles");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  int st = XRGPU_OK;
  for (int p = 0; p < g->world && st == XRGPU_OK; ++p) {
    if (p == g->rank || g->opened[p]) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const char*>(ipc_handles) + static_cast<size_t>(p) * XRGPU_P2P_HANDLE_BYTES, sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      st = api_fail(XRGPU_RUNTIME_ERROR, "cannot open rank " + std::to_string(p) + "'s peer-memory region");
    } else {
      g->peers[p] = static_cast<char*>(ptr);
      g->opened[p] = true;
    }
  }
  cudaSetDevice(prev);
  return st;
}

int xrgpu_p2p_allgather(xrgpu_p2p* g, const void* shard, int64_t rows, int64_t shard_row_bytes, void* out,
                        int64_t out_row_bytes, int64_t out_valid_bytes, void* stream) {
  using namespace xrgpu;
  if (!g || !shard || !out) return api_fail(XRGPU_INVALID_ARGUMENT, "null group, shard or output");
  for (int p = 0; p < g->world; ++p)
    if (!g->peers[p]) return api_fail(XRGPU_INVALID_ARGUMENT, "group not connected (xrgpu_p2p_connect)");
  if (rows < 0 || shard_row_bytes <= 0 || shard_row_bytes % 16 || (rows > 1 && out_row_bytes % 16) ||
      out_valid_bytes > out_row_bytes || out_valid_bytes > shard_row_bytes * g->world ||
      out_valid_bytes <= shard_row_bytes * (g->world - 1))
    return api_fail(XRGPU_INVALID_ARGUMENT,
                    "need shard_row_bytes % 16 == 0, out_row_bytes % 16 == 0 (more than one row) and "
                    "(world-1)*shard < valid <= min(out_row_bytes, world*shard)");
  if (static_cast<uint64_t>(rows * shard_row_bytes) > g->slot_bytes)
    return api_fail(XRGPU_INVALID_ARGUMENT, "shard larger than the group's slot_bytes");
  if ((reinterpret_cast<uintptr_t>(shard) | reinterpret_cast<uintptr_t>(out)) % 16)
    return api_fail(XRGPU_INVALID_ARGUMENT, "shard and output must be 16-byte aligned");
  if (rows == 0) return XRGPU_OK;
  P2PParams q{};
  for (int p = 0; p < g->world; ++p) q.peers[p] = g->peers[p];
  q.epoch = g->epoch;
  q.shard = static_cast<const char*>(shard);
  q.out = static_cast<char*>(out);
  q.rows = rows;
  q.srb = shard_row_bytes;
  q.orb = out_row_bytes;
  q.ovb = out_valid_bytes;
  q.slot_bytes = static_cast<int64_t>(g->slot_bytes);
  q.ll_bytes = static_cast<int64_t>(g->ll_bytes);
  q.world = g->world;
  q.rank = g->rank;
  const int64_t bytes = rows * shard_row_bytes;
  const bool ll = bytes <= kLLMaxBytes;
  if (ll) {  // enough CTAs per peer that a thread sends at most kLLPairsPerThread pairs
    const int64_t per_cta = kSmallThreads * kLLPairsPerThread;
    q.chunks = static_cast<int>(std::min<int64_t>(kMaxChunks, std::max<int64_t>(1, (bytes / 8 + per_cta - 1) / per_cta)));
  } else {
    q.chunks = static_cast<int>(std::min<int64_t>(kMaxChunks, std::max<int64_t>(kMinChunks, (bytes + kChunkBytes - 1) / kChunkBytes)));
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  q.err = device_error_word();
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(g->world * q.chunks), 1, 1);
  cfg.blockDim = dim3(bytes <= kSmallShardBytes ? kSmallThreads : kThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = ll ? cudaLaunchKernelEx(&cfg, p2p_allgather_ll_kernel, q) : cudaLaunchKernelEx(&cfg, p2p_allgather_kernel, q);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return api_fail(XRGPU_RUNTIME_ERROR, std::string("peer all-gather launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

}  // extern "C"

namespace xrgpu {
namespace {

// Checks for the fused form; on success *prob is this rank's problem with y = out + rank * shard_cols.
int fused_check(xrgpu_p2p* g, const xrgpu_mmnb_problem* c, int64_t shard_cols, void* out, Problem* prob,
                std::string* why) {
  if (!g || !c) { *why = "null group or problem"; return XRGPU_INVALID_ARGUMENT; }
  for (int p = 0; p < g->world; ++p)
    if (!g->peers[p]) { *why = "group not connected (xrgpu_p2p_connect)"; return XRGPU_INVALID_ARGUMENT; }
  if (g->world < 2) { *why = "the fused form needs at least two ranks"; return XRGPU_INVALID_ARGUMENT; }
  if (shard_cols <= 0 || shard_cols % 8 || shard_cols < c->N || static_cast<uint64_t>(4 * shard_cols) > g->ll_bytes) {
    *why = "shard_cols must be a multiple of 8, at least N, with 2 * shard_cols <= min(slot_bytes, 1 MiB)";
    return XRGPU_INVALID_ARGUMENT;
  }
  if (reinterpret_cast<uintptr_t>(out) % 16) { *why = "out must be 16-byte aligned"; return XRGPU_INVALID_ARGUMENT; }
  xrgpu_mmnb_problem mine = *c;
  mine.y = out ? static_cast<char*>(out) + 2 * shard_cols * g->rank : nullptr;
  mine.ldy = 0;
  const int st = problem_from_api(&mine, prob, out != nullptr);
  if (st) { *why = "invalid problem"; return st; }
  if (!(prob->f16 && prob->M == 1 && select_path(*prob, c->path) == kPathGemv && gemv_staged_supported(*prob))) {
    *why = "the fused form runs single-row float16 problems of the staged decode GEMV only";
    return XRGPU_INVALID_ARGUMENT;
  }
  return XRGPU_OK;
}

}  // namespace
}  // namespace xrgpu

extern "C" {

int xrgpu_p2p_forward_supported(xrgpu_p2p* g, const xrgpu_mmnb_problem* p, int64_t shard_cols, int32_t* yes) {
  using namespace xrgpu;
  if (!yes) return api_fail(XRGPU_INVALID_ARGUMENT, "null result pointer");
  *yes = 0;
  if (!g || !p) return api_fail(XRGPU_INVALID_ARGUMENT, "null group or problem");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  Problem prob;
  std::string why;
  // a 16-byte aligned stand-in for out: only the problem's own pointers are checked
  *yes = fused_check(g, p, shard_cols, reinterpret_cast<void*>(uintptr_t{256}), &prob, &why) == XRGPU_OK ? 1 : 0;
  cudaSetDevice(prev);
  return XRGPU_OK;
}

int xrgpu_p2p_forward_send(xrgpu_p2p* g, const xrgpu_mmnb_problem* c, int64_t shard_cols, void* out, void* stream) {
  using namespace xrgpu;
  if (!out) return api_fail(XRGPU_INVALID_ARGUMENT, "null output");
  int prev = 0;
  cudaGetDevice(&prev);
  if (g) cudaSetDevice(g->device);
  Problem prob;
  std::string why;
  int st = fused_check(g, c, shard_cols, out, &prob, &why);
  if (st) {
    cudaSetDevice(prev);
    return api_fail(st, why);
  }
  StagedPush push{};
  push.world = g->world;
  push.rank = g->rank;
  push.cols = static_cast<int>(shard_cols);
  push.epoch = g->epoch + ((g->rank + 1) % g->world) * kMaxChunks;  // slot 0 of another rank (all equal)
  for (int p = 0; p < g->world; ++p) push.region[p] = g->peers[p];
  push.words_off = kFlagBytes + 2 * static_cast<int64_t>(g->world) * static_cast<int64_t>(g->slot_bytes);
  push.ll_bytes = static_cast<int64_t>(g->ll_bytes);
  prob.err = device_error_word();
  const cudaError_t e = launch_gemv_staged_push(prob, &push, static_cast<cudaStream_t>(stream));
  cudaSetDevice(prev);
  if (e != cudaSuccess) return api_fail(XRGPU_RUNTIME_ERROR, std::string("fused GEMV launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

int xrgpu_p2p_forward_recv_many(int32_t count, xrgpu_p2p* const* groups, const int64_t* shard_cols, void* const* outs,
                                const int64_t* out_valid_cols, void* stream) {
  using namespace xrgpu;
  if (count < 1 || count > kMaxRecvGroups || !groups || !shard_cols || !outs || !out_valid_cols)
    return api_fail(XRGPU_INVALID_ARGUMENT, "need 1 to 8 groups with their shard widths, outputs and valid widths");
  RecvManyParams P{};
  P.count = count;
  int ctas = 0;
  for (int k = 0; k < count; ++k) {
    xrgpu_p2p* g = groups[k];
    const int64_t S = shard_cols[k], valid = out_valid_cols[k];
    if (!g || !outs[k]) return api_fail(XRGPU_INVALID_ARGUMENT, "null group or output");
    if (g->device != groups[0]->device) return api_fail(XRGPU_INVALID_ARGUMENT, "groups of one receive must share a device");
    for (int p = 0; p < g->world; ++p)
      if (!g->peers[p]) return api_fail(XRGPU_INVALID_ARGUMENT, "group not connected (xrgpu_p2p_connect)");
    if (g->world < 2 || S <= 0 || S % 8 || static_cast<uint64_t>(4 * S) > g->ll_bytes || valid <= (g->world - 1) * S ||
        valid > g->world * S || reinterpret_cast<uintptr_t>(outs[k]) % 16)
      return api_fail(XRGPU_INVALID_ARGUMENT,
                      "need world >= 2, shard_cols a multiple of 8 within the word staging, "
                      "(world-1)*shard_cols < out_valid_cols <= world*shard_cols and a 16-byte aligned out");
    RecvGroup& G = P.g[k];
    G.words = g->local + kFlagBytes + 2 * static_cast<int64_t>(g->world) * static_cast<int64_t>(g->slot_bytes);
    G.epoch = g->epoch;
    G.out = static_cast<char*>(outs[k]);
    G.srb = 2 * S;
    G.ovb = 2 * valid;
    G.ll_bytes = static_cast<int64_t>(g->ll_bytes);
    G.world = g->world;
    G.rank = g->rank;
    const int64_t per_cta = kSmallThreads * kLLPairsPerThread;
    G.chunks = static_cast<int>(std::min<int64_t>(kMaxChunks, std::max<int64_t>(1, (G.srb / 8 + per_cta - 1) / per_cta)));
    G.first_cta = ctas;
    ctas += (g->world - 1) * G.chunks;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(groups[0]->device);
  P.err = device_error_word();
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ctas), 1, 1);
  cfg.blockDim = dim3(kSmallThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, p2p_recv_many_kernel, P);
  cudaSetDevice(prev);
  if (e != cudaSuccess) return api_fail(XRGPU_RUNTIME_ERROR, std::string("peer receive launch failed: ") + cudaGetErrorString(e));
  return XRGPU_OK;
}

int xrgpu_p2p_forward_recv(xrgpu_p2p* g, int64_t shard_cols, void* out, int64_t out_valid_cols, void* stream) {
  return xrgpu_p2p_forward_recv_many(1, &g, &shard_cols, &out, &out_valid_cols, stream);
}

int xrgpu_stream_capture_id(void* stream, uint64_t* id) {
  using namespace xrgpu;
  if (!id) return api_fail(XRGPU_INVALID_ARGUMENT, "null result pointer");
  *id = 0;
  cudaStreamCaptureStatus status = cudaStreamCaptureStatusNone;
  unsigned long long seq = 0;
  const cudaError_t e = cudaStreamGetCaptureInfo(static_cast<cudaStream_t>(stream), &status, &seq);
  if (e != cudaSuccess) return api_fail(XRGPU_RUNTIME_ERROR, std::string("cudaStreamGetCaptureInfo failed: ") + cudaGetErrorString(e));
  if (status == cudaStreamCaptureStatusActive) *id = seq;
  return XRGPU_OK;
}

int xrgpu_p2p_destroy(xrgpu_p2p* g) {
  using namespace xrgpu;
  if (!g) return XRGPU_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(g->device);
  int st = XRGPU_OK;
  for (int p = 0; p < g->world; ++p)
    if (g->opened[p] && cudaIpcCloseMemHandle(g->peers[p]) != cudaSuccess)
      st = api_fail(XRGPU_RUNTIME_ERROR, "closing a peer-memory mapping failed");
  if (g->local) cudaFree(g->local);
  if (g->epoch) cudaFree(g->epoch);
  cudaSetDevice(prev);
  delete g;
  return st;
}

}  // extern "C"
