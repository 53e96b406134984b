/*
 * xrgpu_mmnb.h -- C ABI of the B200 (sm_100a) backend for com.microsoft.MatMulNBits.
 *
 *   Y[M, N] = A[M, K] . dequant(B)^T (+ bias),
 *   dequant(B)[n, k] = (float(q[n, k]) - z[n, k / bs]) * scales[n, k / bs],
 *
 * B is uint8 [N, ceil(K/bs), ceil(bs*bits/8)] with codes packed low-first, bits in {2,4,8}.
 *
 * Two call styles:
 *   1. The operator API of the reference backend (prepare / run / read_outputs / info / close)
 *      over named host tensors, mirroring xrgpu::operators::extended
 *      (runtime/include/xrgpu/extended_operators.h:22-61, runtime/include/xrgpu/operators.h:9-55).
 *   2. A zero-copy call over device pointers on a caller's CUDA stream (xrgpu_mmnb_forward).
 *
 * Every function returns an xrgpu_status; on failure xrgpu_last_error() holds a message
 * (thread-local). No function falls back to CPU computation.
 */
#ifndef XRGPU_MMNB_H
#define XRGPU_MMNB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define XRGPU_API __attribute__((visibility("default")))
#else
#define XRGPU_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Logical dtypes, same numbering as xrgpu::operators::DType (operators.h:9). */
typedef enum {
  XRGPU_FLOAT32 = 0,
  XRGPU_FLOAT16 = 1,
  XRGPU_INT32 = 2,
  XRGPU_UINT32 = 3,
  XRGPU_INT16 = 4,
  XRGPU_INT8 = 5,
  XRGPU_UINT8 = 6,
  XRGPU_INT64 = 7,
  XRGPU_BOOL = 8,
  XRGPU_UNSPECIFIED = 9
} xrgpu_dtype;

/* Status codes in place of the reference's exceptions:
 *   XRGPU_INVALID_ARGUMENT  <- std::invalid_argument (contracts.cpp:9-20, complex_plan.cpp:52-120,
 *                              planner.cpp:12-99)
 *   XRGPU_RUNTIME_ERROR     <- std::runtime_error (vulkan.cpp:24-26, 115); also a poisoned handle
 *   XRGPU_TIMEOUT           <- the fence wait exceeding Options.timeout_ns (vulkan.cpp:115)
 *   XRGPU_DEVICE_ERROR      <- a nonzero device error word (vulkan.cpp:115 "contract validation failed")
 *   XRGPU_UNAVAILABLE       <- no usable CUDA device (operators.h:34 probe: available=false)        */
typedef enum {
  XRGPU_OK = 0,
  XRGPU_INVALID_ARGUMENT = 1,
  XRGPU_RUNTIME_ERROR = 2,
  XRGPU_TIMEOUT = 3,
  XRGPU_DEVICE_ERROR = 4,
  XRGPU_UNAVAILABLE = 5
} xrgpu_status;

#define XRGPU_MAX_RANK 16

/* Named tensor: xrgpu::operators::Tensor (operators.h:16-23). Logical dtype, shape and
 * contiguous little-endian row-major bytes. For xrgpu_prepare, data is a HOST pointer. */
typedef struct {
  const char* name;
  int32_t dtype;                 /* xrgpu_dtype */
  int32_t rank;
  int64_t shape[XRGPU_MAX_RANK];
  const void* data;
  uint64_t nbytes;
} xrgpu_tensor;

/* One integer attribute (MatMulNBits has integer attributes only: K, N, bits, block_size,
 * accuracy_level; contract.json:2-40). */
typedef struct {
  const char* name;
  int64_t value;
} xrgpu_int_attr;

/* extended::Request (extended_operators.h:22-28). args override attrs (planner.cpp:72-85). */
typedef struct {
  const char* operation;         /* "com.microsoft.MatMulNBits" */
  const xrgpu_tensor* inputs;
  int32_t num_inputs;
  const xrgpu_int_attr* attrs;
  int32_t num_attrs;
  const xrgpu_int_attr* args;
  int32_t num_args;
} xrgpu_request;

/* xrgpu::operators::Options (operators.h:24-28) plus the CUDA device ordinal. */
typedef struct {
  int32_t profiling;             /* nonzero: time each run() with CUDA events (info "gpu_ms") */
  uint64_t timeout_ns;           /* bound on run()'s wait; default 15 s */
  uint64_t memory_limit_bytes;   /* bound on device bytes prepare() may hold; default 256 MiB */
  int32_t device;                /* CUDA device ordinal; default 0 */
} xrgpu_options;

typedef struct xrgpu_operator xrgpu_operator;

/* Message of the last failure on the calling thread ("" when none). */
XRGPU_API const char* xrgpu_last_error(void);

/* Fills o with the reference defaults (operators.h:24-28): profiling off, 15 s, 256 MiB, device 0. */
XRGPU_API void xrgpu_default_options(xrgpu_options* o);

/* JSON {"available","backend","device","reason",...}; replaces operators.h:34 probe().
 * Writes at most capacity bytes (NUL-terminated); *needed (if non-NULL) gets the full size. */
XRGPU_API int xrgpu_probe(char* json, uint64_t capacity, uint64_t* needed);

/* Metadata-only validation and output inference; replaces extended::plan(Request)
 * (extended_operators.h:48, planner.cpp:67 -> complex_plan.cpp:58,117-120). Reads no
 * tensor bytes. outputs[0] receives yT's name/dtype/rank/shape (data NULL, nbytes set). */
XRGPU_API int xrgpu_plan(const xrgpu_request* request, xrgpu_tensor* outputs, int32_t capacity, int32_t* count);

/* Validates, plans and copies every input to the device; replaces Operator::prepare
 * (extended_operators.h:51, vulkan.cpp:109-114,119). package_directory is accepted for
 * signature parity and may be NULL (kernels are linked into this library). */
XRGPU_API int xrgpu_prepare(const char* package_directory, const xrgpu_request* request,
                  const xrgpu_options* options, xrgpu_operator** out);

/* Synchronous execution bounded by options.timeout_ns; replaces Operator::run (vulkan.cpp:115,120).
 * A failure poisons the handle until xrgpu_close (vulkan.cpp:105). */
XRGPU_API int xrgpu_run(xrgpu_operator* op);

/* Copies output `index` (0 = yT) to host memory; replaces Operator::read_outputs (vulkan.cpp:121). */
XRGPU_API int xrgpu_read_outputs(const xrgpu_operator* op, int32_t index, void* dst, uint64_t capacity);

/* JSON statistics; replaces Operator::info (vulkan.cpp:123): backend, operation, device,
 * execution_ms, gpu_ms, dispatch_count, path, cpu_compute_fallback (always false), closed. */
XRGPU_API int xrgpu_info(const xrgpu_operator* op, char* json, uint64_t capacity, uint64_t* needed);

/* Waits for submitted work and releases device memory; replaces Operator::close (vulkan.cpp:122).
 * The handle stays valid for xrgpu_info until xrgpu_destroy. */
XRGPU_API int xrgpu_close(xrgpu_operator* op);

/* Frees the handle (closing it first if needed); the reference's ~Operator. */
XRGPU_API void xrgpu_destroy(xrgpu_operator* op);

/* Extension (no reference counterpart): replaces the bytes of one prepared input of the same
 * name, dtype and size (e.g. a new activation for the next decode step) without re-preparing
 * the weights. Host pointer; the copy completes before return. */
XRGPU_API int xrgpu_write_input(xrgpu_operator* op, const char* name, const void* data, uint64_t nbytes);

/* Extension: enqueue run() on `stream` (cudaStream_t; NULL = the handle's own stream)
 * without waiting. Errors raised on the device surface at the next xrgpu_run/xrgpu_sync. */
XRGPU_API int xrgpu_run_async(xrgpu_operator* op, void* stream);

/* Extension: waits for the handle's work; checks the device error word. */
XRGPU_API int xrgpu_sync(xrgpu_operator* op);

/* Extension: device pointer of output `index` (valid until xrgpu_close). */
XRGPU_API int xrgpu_output_device_ptr(const xrgpu_operator* op, int32_t index, void** ptr);

/* ---------------------------------------------------------------------------------------
 * Zero-copy device API (extension). Pointers are device pointers of the current context.
 * ------------------------------------------------------------------------------------- */

/* Kernel selection for xrgpu_mmnb_forward (the planner's choice unless forced). */
typedef enum {
  XRGPU_PATH_AUTO = 0,
  XRGPU_PATH_GENERIC = 1,   /* any bits/block size/dtype; float32 CUDA-core accumulation */
  XRGPU_PATH_GEMV = 2,      /* 4-bit decode GEMV, M <= 16, float16 A */
  XRGPU_PATH_GEMM = 3       /* 4-bit prefill GEMM on tcgen05 tensor cores, float16 A */
} xrgpu_mmnb_path;

typedef struct {
  int32_t dtype;            /* T1 of aT/scalesT/biasT/yT: XRGPU_FLOAT32 or XRGPU_FLOAT16 */
  int32_t zero_point_dtype; /* XRGPU_UNSPECIFIED: absent (z = 2^(bits-1));
                               XRGPU_FLOAT32 / XRGPU_FLOAT16: [N, ceil(K/bs)] (reference contract);
                               XRGPU_UINT8: packed [N, ceil(ceil(K/bs)*bits/8)] (ONNX Runtime form) */
  int32_t path;             /* xrgpu_mmnb_path */
  int32_t reserved;
  int64_t M, K, N, block_size, bits;
  const void* a;            /* [M, K] T1 */
  const uint8_t* b;         /* [N, ceil(K/bs), ceil(bs*bits/8)] */
  const void* scales;       /* [N, ceil(K/bs)] T1 */
  const void* zero_points;  /* see zero_point_dtype; NULL when absent */
  const void* bias;         /* [N] T1 or NULL */
  void* y;                  /* [M, ldy] T1 */
  int64_t ldy;              /* row stride of y in elements; 0 means N */
} xrgpu_mmnb_problem;

/* Device scratch bytes xrgpu_mmnb_forward needs for this problem. Every kernel path of this
 * build reports 0: the GEMV's K slices meet in shared memory and the GEMM keeps whole K per tile.
 * The argument stays so that a path which needs global scratch can be added without an ABI change. */
XRGPU_API int xrgpu_mmnb_workspace_size(const xrgpu_mmnb_problem* p, uint64_t* bytes);

/* Enqueues Y = A.dequant(B)^T (+bias) on `stream` (cudaStream_t, NULL = legacy default).
 * workspace: device scratch of at least xrgpu_mmnb_workspace_size bytes, zero-filled before its
 * first use and left zero-filled by every completed call; NULL = a per-device workspace owned by
 * the library (grown on demand, so that call may allocate). Calls sharing a workspace must not
 * overlap on the GPU. */
XRGPU_API int xrgpu_mmnb_forward(const xrgpu_mmnb_problem* p, void* workspace, uint64_t workspace_bytes,
                       void* stream);

/* Enqueues W[n, k] = (float(q) - z) * s as float32 [N, K] (bit-exact nbitWeight,
 * complex_kernel.glsl:80). Uses p->b, scales, zero_points, K, N, block_size, bits, dtype. */
XRGPU_API int xrgpu_mmnb_dequantize(const xrgpu_mmnb_problem* p, float* w, void* stream);

/* Name of the kernel path the planner selects for p ("generic", "gemv", "gemm"). */
XRGPU_API int xrgpu_mmnb_select_path(const xrgpu_mmnb_problem* p, char* name, uint64_t capacity);

/* Reads (and optionally clears) the device error word of `device`: 0 = no error; otherwise the
 * code of the first bounded wait that expired in a kernel (each wait gives up after about 1 s):
 *   0x301..0x305  prefill GEMM: producer, MMA, dequantisation, epilogue wait, final drain;
 *   0x401         peer all-gather: a peer's flag did not arrive. The group's epochs have then
 *                 advanced past the failed call, so the group must be destroyed, not reused.
 * The kernel that gave up returns normally and leaves the context usable; its output is undefined. */
XRGPU_API int xrgpu_device_error(int32_t device, uint32_t* code, int32_t clear);

/* ---- Peer-memory all-gather for column-sharded MatMulNBits (no counterpart in the reference,
 * whose backend is single-device). One process per GPU on one node; every rank of a group makes
 * the same sequence of calls. The all-gather is one kernel, so CUDA graphs can capture it. */
#define XRGPU_P2P_MAX_WORLD 16
#define XRGPU_P2P_HANDLE_BYTES 64
typedef struct xrgpu_p2p xrgpu_p2p;

/* Allocates this rank's staging region on `device` (4 KB of flags, 2 * world * slot_bytes of shard
 * staging and 2 * world * 2 * min(slot_bytes, 1 MiB) of word staging, zero-filled) and writes its
 * 64-byte CUDA IPC handle to ipc_handle. slot_bytes: largest shard in bytes (a multiple of 16). */
XRGPU_API int xrgpu_p2p_create(int32_t device, int32_t world, int32_t rank, uint64_t slot_bytes, xrgpu_p2p** group,
                               void* ipc_handle);

/* Maps the other ranks' regions: ipc_handles holds world handles of 64 bytes in rank order (this
 * rank's own entry is ignored). */
XRGPU_API int xrgpu_p2p_connect(xrgpu_p2p* group, const void* ipc_handles);

/* Enqueues on `stream`: out[m, q * shard_row_bytes + j] = shard of rank q [m, j] for every rank q,
 * m < rows, keeping the first out_valid_bytes of each output row (the last shard may be padded).
 * shard is this rank's [rows, shard_row_bytes] (contiguous); shard_row_bytes is a multiple of 16, and
 * so is out_row_bytes when rows > 1; rows * shard_row_bytes <= slot_bytes. A peer that does not arrive within 1 s
 * leaves code 0x401 in the device error word (xrgpu_device_error). */
XRGPU_API int xrgpu_p2p_allgather(xrgpu_p2p* group, const void* shard, int64_t rows, int64_t shard_row_bytes,
                                  void* out, int64_t out_row_bytes, int64_t out_valid_bytes, void* stream);

/* Sharded single-row MatMulNBits with the send half of the all-gather fused into the GEMV, in two
 * enqueues. xrgpu_p2p_forward_send runs this rank's shard p (M == 1, float16, a problem the planner
 * gives to the staged decode GEMV; p->y is ignored) writing its columns to out + rank * shard_cols
 * and, from the same epilogue, to every other rank's word staging as epoch-tagged words.
 * xrgpu_p2p_forward_recv then waits (bounded, 0x401 on expiry) for the other ranks' words and writes
 * their columns into out. out: float16 [out_valid_cols], 16-byte aligned; shard_cols: columns per
 * rank (a multiple of 8, at least p->N, 2 * shard_cols <= min(slot_bytes, 1 MiB)); out_valid_cols in
 * ((world - 1) * shard_cols, world * shard_cols]. Each send must be followed by its receive before
 * the group's next call of any kind (same stream, or ordered by an event); every rank makes the same
 * sequence of calls. xrgpu_p2p_forward_supported sets *yes to 1 when send accepts (group, p,
 * shard_cols). */
XRGPU_API int xrgpu_p2p_forward_supported(xrgpu_p2p* group, const xrgpu_mmnb_problem* p, int64_t shard_cols,
                                          int32_t* yes);
XRGPU_API int xrgpu_p2p_forward_send(xrgpu_p2p* group, const xrgpu_mmnb_problem* p, int64_t shard_cols, void* out,
                                     void* stream);
XRGPU_API int xrgpu_p2p_forward_recv(xrgpu_p2p* group, int64_t shard_cols, void* out, int64_t out_valid_cols,
                                     void* stream);
/* The receives of up to 8 groups (each after its own send) in one kernel, e.g. the projections
 * that share one input; groups[k] with shard_cols[k], outs[k] and out_valid_cols[k] as above. */
XRGPU_API int xrgpu_p2p_forward_recv_many(int32_t count, xrgpu_p2p* const* groups, const int64_t* shard_cols,
                                          void* const* outs, const int64_t* out_valid_cols, void* stream);

/* Identifier of the CUDA graph capture `stream` takes part in (0 when it is not capturing), so a
 * host can tell whether two enqueues belong to one capture (cross-stream ordering is only legal
 * inside one). No reference counterpart. */
XRGPU_API int xrgpu_stream_capture_id(void* stream, uint64_t* id);

/* Unmaps the peers' regions and frees this rank's. Call only after every rank has finished its
 * last all-gather on the group (synchronise, then a host barrier). */
XRGPU_API int xrgpu_p2p_destroy(xrgpu_p2p* group);

/* ---------------------------------------------------------------------------------------
 * Operators around MatMulNBits: its fused callers and the operators that share its quantized
 * formats. Same request model as above, with the reference's floating-point and string
 * attributes and its requested-output list (xrgpu::operators::extended::Request and Attributes,
 * runtime/include/xrgpu/extended_operators.h:8-28; attributes read by complex_plan.cpp:44-47).
 *   com.microsoft.MatMulNBitsMlp (1027)  aT, skipT?, normScaleT?, gateBT, gateScalesT, gateBiasT?, upBT,
 *                                         upScalesT, upBiasT?  -> yT, residualT?
 *   com.microsoft.MatMulNBitsQkv (1028)  aT, skipT?, normScaleT, qBT, qScalesT, kBT, kScalesT, vBT, vScalesT
 *                                         -> qT, kT, vT, residualT?
 *   com.microsoft.MatMulBnb4 (1026)      aT, bT, absmaxT -> yT
 *   com.microsoft.GatherBlockQuantized (1031)  dataT, indicesT, scalesT, zeroPointsT? -> outputT
 *   com.microsoft.QMoE (1030)            inputT, routerT, fc1T, fc1ScalesT, fc2T, fc2ScalesT -> outputT
 * (input lists: complex_plan.cpp:33-37,39-40; contracts: kernels/<operation>/contract.json).
 * xrgpu_prepare / xrgpu_plan accept these operations too (integer attributes only);
 * xrgpu_read_outputs / xrgpu_output_device_ptr take the output's index in the planned order.
 * ------------------------------------------------------------------------------------- */
typedef struct {
  const char* name;
  double value;
} xrgpu_float_attr;

typedef struct {
  const char* name;
  const char* value;
} xrgpu_string_attr;

/* extended::Request with every attribute kind (planner.cpp:72-85 precedence: args over attrs). */
typedef struct {
  const char* operation;
  const xrgpu_tensor* inputs;
  int32_t num_inputs;
  const xrgpu_int_attr* attrs;
  int32_t num_attrs;
  const xrgpu_int_attr* args;
  int32_t num_args;
  const xrgpu_float_attr* float_attrs;
  int32_t num_float_attrs;
  const xrgpu_string_attr* string_attrs;
  int32_t num_string_attrs;
  const char* const* requested_outputs;  /* names in the wanted order; NULL/0 = the required outputs */
  int32_t num_requested_outputs;
} xrgpu_request_ex;

/* extended::plan for every supported operation (complex_plan.cpp:58-143). */
XRGPU_API int xrgpu_plan_ex(const xrgpu_request_ex* request, xrgpu_tensor* outputs, int32_t capacity, int32_t* count);

/* Operator::prepare for every supported operation (extended_operators.h:51). */
XRGPU_API int xrgpu_prepare_ex(const char* package_directory, const xrgpu_request_ex* request,
                               const xrgpu_options* options, xrgpu_operator** out);

/* Activation codes of the fused operators (complex_plan.cpp:50 activation_lower; fused,
 * complex_kernel.glsl:41-47). */
typedef enum {
  XRGPU_ACT_NONE = 0,
  XRGPU_ACT_RELU = 1,
  XRGPU_ACT_SILU = 2,
  XRGPU_ACT_GELU = 3,
  XRGPU_ACT_TANH = 4,
  XRGPU_ACT_SIGMOID = 5,
  XRGPU_ACT_SWIGLU = 6
} xrgpu_activation;

/* MatMulNBitsMlp over device pointers (packedMatmul opcode 1027, complex_kernel.glsl:81,83):
 *   h = a + skip; x = norm_scale ? h * (1/sqrt(sum(h^2)/K + epsilon) * norm_scale[k]) : h;
 *   y = fused(x . dequant(gate)^T + gate_bias, activation) * (x . dequant(up)^T + up_bias);
 *   residual (optional) = h. Weights use nbitWeight without zero points (z = 2^(bits-1)). */
typedef struct {
  int32_t dtype;           /* T1: XRGPU_FLOAT32 or XRGPU_FLOAT16 */
  int32_t activation;      /* xrgpu_activation */
  int64_t M, K, N, block_size, bits;
  float epsilon;
  int32_t reserved;
  const void* a;           /* [M, K] */
  const void* skip;        /* [M, K] or NULL */
  const void* norm_scale;  /* [K] or NULL */
  const uint8_t* gate_b;   /* [N, ceil(K/bs), ceil(bs*bits/8)] */
  const void* gate_scales; /* [N, ceil(K/bs)] */
  const void* gate_bias;   /* [N] or NULL */
  const uint8_t* up_b;
  const void* up_scales;
  const void* up_bias;
  void* y;                 /* [M, N] */
  void* residual;          /* [M, K] or NULL */
} xrgpu_mlp_problem;

/* Device scratch bytes of xrgpu_mlp_forward (the normalised activations and the two projections). */
XRGPU_API int xrgpu_mlp_workspace_size(const xrgpu_mlp_problem* p, uint64_t* bytes);
/* workspace NULL: the library's per-device workspace (grown on demand). */
XRGPU_API int xrgpu_mlp_forward(const xrgpu_mlp_problem* p, void* workspace, uint64_t workspace_bytes, void* stream);

/* xrgpu_mlp_forward for callers that must not have the library allocate device memory (a serving
 * engine that plans all GPU memory itself, a decode loop that cannot take cudaMalloc's implicit
 * synchronisation). No counterpart in the reference, whose Operator owns every buffer it uses.
 * The scratch is a fixed array of XRGPU_STATIC_SCRATCH_BYTES in device memory, held by every GPU that
 * loads the library until the process exits; problems whose xrgpu_mlp_workspace_size is larger are
 * rejected with XRGPU_INVALID_ARGUMENT. The caller still passes inputs and outputs. The first call on
 * a device looks up the array's device address (make that call before any stream capture). All calls
 * share the array: calls that overlap on the GPU race. Calls no allocator. */
#define XRGPU_STATIC_SCRATCH_BYTES (4u << 20)
XRGPU_API int xrgpu_mlp_forward_static(const xrgpu_mlp_problem* p, void* stream);

/* MatMulNBitsQkv over device pointers (packedMatmul opcode 1028): x normalised as above (norm_scale
 * required), q/k/v = x . dequant(W)^T (no zero points, no bias), residual (optional) = a + skip. */
typedef struct {
  int32_t dtype;
  int32_t reserved;
  int64_t M, K, Nq, Nkv, block_size, bits;
  float epsilon;
  int32_t reserved2;
  const void* a;
  const void* skip;
  const void* norm_scale;
  const uint8_t* q_b;
  const void* q_scales;
  const uint8_t* k_b;
  const void* k_scales;
  const uint8_t* v_b;
  const void* v_scales;
  void* q;                 /* [M, Nq] */
  void* k;                 /* [M, Nkv] */
  void* v;                 /* [M, Nkv] */
  void* residual;          /* [M, K] or NULL */
} xrgpu_qkv_problem;

XRGPU_API int xrgpu_qkv_workspace_size(const xrgpu_qkv_problem* p, uint64_t* bytes);
XRGPU_API int xrgpu_qkv_forward(const xrgpu_qkv_problem* p, void* workspace, uint64_t workspace_bytes, void* stream);

/* MatMulBnb4 over device pointers (bnbWeight, complex_kernel.glsl:82; transB = 1):
 * y[m, n] = sum_k a[m, k] * table[code(n*K + k)] * absmax[(n*K + k) / block_size], NF4 for
 * quant_type 1, FP4 for 0, the high nibble of a byte first. */
typedef struct {
  int32_t dtype;
  int32_t quant_type;
  int64_t M, K, N, block_size;
  const void* a;           /* [M, K] */
  const uint8_t* b;        /* [ceil(N*K/2)] */
  const void* absmax;      /* [ceil(N*K/block_size)] */
  void* y;                 /* [M, N] */
} xrgpu_bnb4_problem;

XRGPU_API int xrgpu_bnb4_forward(const xrgpu_bnb4_problem* p, void* stream);

/* GatherBlockQuantized over device pointers (gatherQuant, complex_kernel.glsl:85; gather_axis 0,
 * quantize_axis 1): out[r, j] = (q - z) * scales[idx[r], j / block_size] as float32, zero points
 * packed low-first (default 2^(bits-1)). An index outside [0, rows) leaves its row 0 and code 55
 * in the device error word (the reference's fail(55)). */
typedef struct {
  int32_t bits;            /* 4 or 8 */
  int32_t index_dtype;     /* XRGPU_INT64 or XRGPU_INT32 */
  int64_t rows, row_bytes, count, block_size;
  const uint8_t* data;     /* [rows, row_bytes] */
  const void* indices;     /* [count] */
  const float* scales;     /* [rows, ceil(width/block_size)], width = row_bytes * 8 / bits */
  const uint8_t* zero_points; /* [rows, ceil(blocks*bits/8)] or NULL */
  float* out;              /* [count, width] */
} xrgpu_gather_problem;

XRGPU_API int xrgpu_gather_block_quantized_forward(const xrgpu_gather_problem* p, void* stream);

/* QMoE over device pointers (moe, complex_kernel.glsl:158-160), float32: the k experts of highest
 * router score (ties: the higher expert index first) are weighted by a softmax over their scores;
 * expert weights are symmetric (q - 2^(bits-1)) * scale with one scale per row (block_size 0) or
 * per block of block_size columns; activation XRGPU_ACT_RELU, or XRGPU_ACT_SWIGLU with
 * swiglu_fusion 1 (gate/linear rows interleaved), alpha/beta and an optional limit. */
typedef struct {
  int32_t bits;
  int32_t activation;
  int32_t swiglu_fusion;
  int32_t has_swiglu_limit;
  int64_t tokens, hidden, experts, k, fc1_rows, block_size;
  float activation_alpha, activation_beta, swiglu_limit;
  int32_t reserved;
  const float* input;      /* [tokens, hidden] */
  const float* router;     /* [tokens, experts] */
  const uint8_t* fc1;      /* [experts, fc1_rows, ceil(hidden*bits/8)] */
  const float* fc1_scales; /* [experts, fc1_rows] or [experts, fc1_rows, hidden/block_size] */
  const uint8_t* fc2;      /* [experts, hidden, ceil(inter*bits/8)], inter = fc1_rows / (swiglu ? 2 : 1) */
  const float* fc2_scales;
  float* output;           /* [tokens, hidden] */
} xrgpu_qmoe_problem;

XRGPU_API int xrgpu_qmoe_workspace_size(const xrgpu_qmoe_problem* p, uint64_t* bytes);
XRGPU_API int xrgpu_qmoe_forward(const xrgpu_qmoe_problem* p, void* workspace, uint64_t workspace_bytes, void* stream);

/* Library version string. */
XRGPU_API const char* xrgpu_version(void);

#ifdef __cplusplus
}
#endif

#endif /* XRGPU_MMNB_H */
