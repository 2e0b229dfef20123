/*
 * qraf_cuda.h — C ABI of the B200 quantized matvec library (libqraf_cuda.so).
 *
 * The library replaces the body of one seam of QRAF (simonpierreboucher02/qraf):
 * the block-quantized Q8_0 / Q4_0 weight x fp32 activation matvec behind
 * `qraf::dispatch_matvec_q` (src/nn/backend.cpp:131-199, declared at
 * include/nn/backend.h:31-34) and its per-row primitives `dot_q8_0_f32` /
 * `dot_q4_0_f32` (src/tensor/quantize.cpp:187-239, include/tensor/quantize.h:60-61).
 * The on-device weight layout is the reference's native block layout, byte for
 * byte (include/tensor/quantize.h:11-31):
 *
 *   Q8_0 block: [f32 scale][block_size x int8]                 4 + bs bytes
 *   Q4_0 block: [f16 scale][block_size/2 x u8, element 2i in
 *               the low nibble, 2i+1 in the high, +8 bias]      2 + bs/2 bytes
 *   weight:     rows x ceil(cols / bs) blocks, rows back to back.
 *
 * Conventions: every function returns a status (QRAF_OK = 0).  Pointers named
 * `*_dev` are device memory of the current device; `*_host` are host memory.
 * `stream` is a cudaStream_t passed as void* (NULL = the legacy default
 * stream).  Device entry points are asynchronous on `stream`; host entry points
 * are synchronous.  On error, qraf_cuda_last_error() returns a message for the
 * calling thread.
 */
#ifndef QRAF_CUDA_H
#define QRAF_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── status codes ───────────────────────────────────────────────────────── */
#define QRAF_OK              0
#define QRAF_ERR_INVALID     1   /* an argument is out of range or inconsistent */
#define QRAF_ERR_UNSUPPORTED 2   /* unknown dtype, or a mode this shape has no kernel for */
#define QRAF_ERR_CUDA        3   /* a CUDA runtime call failed */
#define QRAF_ERR_TIMEOUT     4   /* a bounded device-side wait expired (see qraf_cuda_device_status) */
#define QRAF_ERR_COMM        5   /* a collective / peer-exchange step failed */
#define QRAF_ERR_NOMEM       6   /* device or pinned-host allocation failed */

/* ── weight dtypes: the reference's DType values (include/core/types.h:27-39) */
#define QRAF_DTYPE_Q8_0 10u
#define QRAF_DTYPE_Q4_0 20u

/* ── arithmetic modes ───────────────────────────────────────────────────── */
#define QRAF_MODE_EXACT 0  /* bit-identical to the reference's Linux scalar path */
#define QRAF_MODE_FAST  1  /* exact per-block integer sums (activations as 8-bit limbs),
                              reordered fp32 sums; allclose(rtol 1e-5, atol 1e-6) */
#define QRAF_MODE_TC    2  /* tcgen05 tensor-core tile (exact per-block integer sums, fp32
                              epilogue); same tolerance as FAST.  Needs block size 32,
                              K % 128 == 0 (Q8_0) or K % 256 == 0 (Q4_0) and 16-byte-aligned
                              weights.  One vector with K a multiple of 1024 up to 4096, a
                              16-byte-aligned x and at most 32 x (SM count) rows runs a
                              batch-1 tensor-core kernel instead (int8 MMAs on the FAST
                              path's activation limbs). */
/* Per-stream scratch.  QRAF_MODE_TC, and QRAF_MODE_FAST (also the sharded FAST
 * path) when a row has at least 320 blocks (K >= 10240) and a CTA gets at most 96
 * rows (long-K projections, row shards), use scratch memory that the library
 * allocates per (device, stream) at the stream's first call that needs that much.
 * Make one call of each such shape on a stream before capturing the stream in a
 * CUDA graph: a capture that would need more scratch fails with
 * QRAF_ERR_UNSUPPORTED.  Scratch areas are never freed before qraf_cuda_shutdown
 * (graphs hold their addresses); a graph captured on a stream uses that stream's
 * scratch, so it must not run concurrently with other work of that stream. */
#define QRAF_MODE_AUTO  3  /* FAST for M <= 2, TC from M = 3 where the weight allows (else FAST) */
/* Or-able flag: the kernel may start while the previous kernel in the stream is
 * still running and fetch the weight before waiting for it (programmatic
 * dependent launch).  Only valid when that previous kernel does not write the
 * weight - true for model weights in a decode loop.  Activations are always
 * read after the wait. */
#define QRAF_MODE_FLAG_OVERLAP 0x100

/* A quantized weight on one device: a plain descriptor, no hidden state. */
typedef struct qraf_weight {
    const void* data;     /* device pointer to rows * row_bytes bytes */
    uint64_t bytes;       /* rows * row_bytes */
    uint64_t row_bytes;   /* ceil(cols / block_size) * block bytes */
    uint32_t dtype;       /* QRAF_DTYPE_Q8_0 or QRAF_DTYPE_Q4_0 */
    uint32_t block_size;  /* elements per block (QuantScheme::block_size, format.h:91) */
    uint32_t rows;        /* N = out_dim */
    uint32_t cols;        /* K = in_dim */
    int32_t device;       /* CUDA device that holds `data` */
    uint32_t owned;       /* 1 when the library allocated `data` (qraf_cuda_weight_upload) */
} qraf_weight_t;

/* ── library ────────────────────────────────────────────────────────────── */
const char* qraf_cuda_version(void);
/* Select `device` for the calling thread and prepare the kernels on it. */
int qraf_cuda_init(int device);
/* Free the host-pointer weight cache and staging buffers of every device. */
int qraf_cuda_shutdown(void);
/* Kernels the library has launched in this process, all devices and streams (a
 * launch captured into a CUDA graph counts once, at capture). */
uint64_t qraf_cuda_launch_count(void);
/* Copy the calling thread's last error message into buf (always NUL-terminated). */
int qraf_cuda_last_error(char* buf, size_t len);
/* Synchronise the current device and return QRAF_ERR_TIMEOUT if a kernel
 * reported an expired wait since the last clear; `clear` resets the word. */
int qraf_cuda_device_status(int clear);

/* Bytes of one row: ceil(cols / block_size) blocks (backend.cpp:138-139,167-168).
 * 0 for an unknown dtype or block_size 0. */
uint64_t qraf_row_bytes(uint32_t dtype, uint32_t block_size, uint32_t cols);

/* ── weights ────────────────────────────────────────────────────────────── */
/* Describe native blocks already on the device (nothing is copied). */
int qraf_cuda_weight_wrap(const void* data_dev, uint64_t bytes, uint32_t dtype, uint32_t block_size,
                          uint32_t rows, uint32_t cols, qraf_weight_t* out);
/* Copy native blocks from host memory to a new device allocation. */
int qraf_cuda_weight_upload(const void* data_host, uint64_t bytes, uint32_t dtype, uint32_t block_size,
                            uint32_t rows, uint32_t cols, qraf_weight_t* out);
/* Free a weight made by qraf_cuda_weight_upload (no-op for wrapped weights). */
int qraf_cuda_weight_free(qraf_weight_t* w);
/* Rows [rank*rows/world, (rank+1)*rows/world) of `full` as a view (no copy).
 * Row sharding keeps each row's bytes intact, so every shard is a valid weight. */
int qraf_cuda_weight_shard(const qraf_weight_t* full, uint32_t world, uint32_t rank, qraf_weight_t* out);

/* ── the hot path ───────────────────────────────────────────────────────── */
/* Y[m][n] = dispatch_matvec_q(W, X[m])[n] for m < M (backend.cpp:131-199 per
 * vector; the reference's batching is M independent batch-1 forwards,
 * include/runtime/batch_scheduler.h:187-228).  x_dev is [M][cols] fp32,
 * y_dev is [M][rows] fp32. */
int qraf_cuda_matvec_q(const qraf_weight_t* w, const float* x_dev, float* y_dev, uint32_t M, int mode,
                       void* stream);

/* Several projections of the same activations in one launch: ys_dev[i] =
 * W_i X for the `count` weights ws[0..count) (1 to QRAF_MULTI_MAX_WEIGHTS, same
 * dtype, block size, cols and device; each ys_dev[i] is [M][ws[i].rows]).  The
 * reference makes one dispatch_matvec_q call per projection on one input
 * (src/nn/attention.cpp:92-97: Q, K and V of the normalised hidden state;
 * :172-174: gate and up); here the weights are one row range of one launch, so
 * the activations are staged once and there is one launch instead of `count`.
 * EXACT (any M) and FAST (M <= 2) run fused and give the same bits as separate
 * qraf_cuda_matvec_q calls; other modes and shapes run one call per weight. */
#define QRAF_MULTI_MAX_WEIGHTS 4
int qraf_cuda_matvec_q_multi(const qraf_weight_t* ws, uint32_t count, const float* x_dev, float* const* ys_dev,
                             uint32_t M, int mode, void* stream);

/* qraf_cuda_matvec_q_multi with the steps the reference runs around those
 * projections folded in: norm_w (non-NULL) replaces X[m] by
 * RMSNorm(X[m]) = X[m] * (1 / sqrt(mean(X[m]^2) + norm_eps)) * norm_w first
 * (dispatch_rms_norm, src/nn/backend.cpp:203-223 / src/nn/ops.cpp:107-118, as
 * src/nn/transformer.cpp:588-590 runs it before Q, K and V); biases[i]
 * (non-NULL array, entries may be NULL) is added to weight i's outputs,
 * fl(y + b) (src/nn/attention.cpp:100-102).  FAST (M <= 2) folds both into the
 * one launch (RMSNorm's sum of squares in fp64 by every CTA); EXACT folds the
 * biases and runs RMSNorm first in the reference's order, so its results are
 * the reference's bits; other modes run the steps around the projections.  x is
 * not modified. */
int qraf_cuda_matvec_q_multi_ex(const qraf_weight_t* ws, uint32_t count, const float* x_dev, const float* norm_w,
                                float norm_eps, const float* const* biases, float* const* ys_dev, uint32_t M, int mode,
                                void* stream);

/* SwiGLU of one input: h[m][i] = silu((W_gate X[m])[i]) * (W_up X[m])[i], with
 * silu(g) = g / (1 + exp(-g)) - the reference's gate and up projections, silu and
 * product (mlp_forward, src/nn/attention.cpp:172-179; silu_inplace,
 * src/nn/ops.cpp:218-221).  gate and up have one dtype, block size and shape; h is
 * [M][rows].  FAST (and AUTO for one or two vectors) runs one launch: the row
 * kernel streams each gate row beside its up row and writes the product, so
 * gate and up never reach memory.  Other modes run the two projections in that
 * mode and an elementwise pass (through a per-stream buffer that, like the
 * scratch above, is sized at a stream's first call of the shape).  exp is CUDA's
 * expf (within 2 ulp of the C library's). */
int qraf_cuda_matvec_q_swiglu(const qraf_weight_t* gate, const qraf_weight_t* up, const float* x_dev, float* h_dev,
                              uint32_t M, int mode, void* stream);
/* The same after an RMSNorm of x (norm_w, norm_eps as in qraf_cuda_matvec_q_multi_ex;
 * src/nn/transformer.cpp:597-600 normalises before the MLP): one launch in FAST. */
int qraf_cuda_matvec_q_swiglu_ex(const qraf_weight_t* gate, const qraf_weight_t* up, const float* x_dev,
                                 const float* norm_w, float norm_eps, float* h_dev, uint32_t M, int mode,
                                 void* stream);

/* The tensor-core path of qraf_cuda_matvec_q (QRAF_MODE_TC, same kernels and
 * results) for callers that may not allocate device memory: its scratch (the
 * prepared activation tiles, the stream-K partial sums and tile counters) lives
 * in one fixed device array of QRAF_NOALLOC_SCRATCH_BYTES inside the library,
 * and the call makes no cudaMalloc, cudaFree or other allocating call.  No
 * counterpart in the reference (its CPU path needs no scratch).
 *  - A call whose scratch would exceed QRAF_NOALLOC_SCRATCH_BYTES is rejected
 *    with QRAF_ERR_INVALID and a message naming both sizes (among the
 *    BASELINE shapes: only K = 28672 with more than 60 vectors in one call).
 *  - The first call on a device does the set-up (looks up the array's device
 *    address); make that first call before any stream capture.
 *  - Every call on a device shares the array: calls that overlap on the GPU
 *    (on different streams, or from different threads without ordering) race.
 *    What must start at zero is cleared by each call's own first kernel.
 *  - flags: QRAF_MODE_FLAG_OVERLAP or 0. */
#define QRAF_NOALLOC_SCRATCH_BYTES (16u << 20)
int qraf_cuda_matmul_tc_noalloc(const qraf_weight_t* w, const float* x_dev, float* y_dev, uint32_t M, int flags,
                                void* stream);

/* One quantized row dotted with x (dot_q8_0_f32 / dot_q4_0_f32,
 * quantize.cpp:187-239); *out_dev receives the fp32 result. */
int qraf_cuda_dot_q(uint32_t dtype, const void* q_dev, const float* x_dev, uint64_t count, uint32_t block_size,
                    float* out_dev, int mode, void* stream);

/* Per-block integer partial sums of the FAST batch-1 arithmetic, for bit-exact
 * checks against a CPU restatement (verification entry; no counterpart in the
 * reference, whose path has no integer sums).  For one vector x and every (row
 * n, block b): d_dev[n][b][j] = sum_i q_i * L_j,i (int32, j = 0..3; codes with
 * their bias removed; L_j the balanced signed 8-bit digits, most significant
 * first, of X_i = rint(x_i 2^(30-e_b)), max |x| (1 + 2^-8) < 2^e_b over the block)
 * and c_dev[b] = 2^(e_b - 30), exactly as the FAST kernels form them.  Block
 * size 32, K % 32 == 0, 4-byte-aligned rows, K up to the shared memory (176 B per
 * block). */
int qraf_cuda_limb_partials(const qraf_weight_t* w, const float* x_dev, int32_t* d_dev, float* c_dev, void* stream);

/* Per-block partial products p[n][b] = fl(block_sum * scale) exactly as the
 * reference forms them before `total += ...` (quantize.cpp:201-205, 226-234).
 * partials_dev is [rows][ceil(cols / block_size)].  For bit-exact checking. */
int qraf_cuda_block_partials(const qraf_weight_t* w, const float* x_dev, float* partials_dev, void* stream);

/* ── quantizer (byte-exact with the reference) ──────────────────────────── */
/* quantize_q8_0 / quantize_q4_0 over `count` contiguous values
 * (quantize.cpp:105-183); out_dev receives qraf_row_bytes(dtype, bs, count) bytes. */
int qraf_cuda_quantize(uint32_t dtype, const float* x_dev, uint64_t count, uint32_t block_size, void* out_dev,
                       void* stream);
/* The same applied to each of `rows` rows of `cols` values (the layout a
 * weight has when each output row is quantized on its own). */
int qraf_cuda_quantize_rows(uint32_t dtype, const float* x_dev, uint32_t rows, uint32_t cols, uint32_t block_size,
                            void* out_dev, void* stream);
/* dequantize_tensor for Q8_0 / Q4_0 (quantize.cpp:55-101). */
int qraf_cuda_dequantize(uint32_t dtype, const void* q_dev, uint64_t count, uint32_t block_size, float* out_dev,
                         void* stream);

/* ── row-sharded matvec over several GPUs (one process per GPU) ─────────── */
/* A weight too large for one GPU's bandwidth budget is partitioned by output
 * rows (qraf_cuda_weight_shard); each rank computes its rows and the kernel
 * itself stores every output element into this rank's y and, as one 8-byte
 * word (call number << 32 | value bits), into every peer's receive array over
 * NVLink (CUDA IPC peer mappings, plain stores, no fence and no flag: an
 * aligned 8-byte store is seen whole or not at all).  Before it ends, the
 * kernel copies the other ranks' rows from its own receive array into y,
 * polling each word (bounded) until it carries this call's number: the
 * all-gather is fused into the matvec.  The library does no networking: the
 * caller exchanges the opaque handles (e.g. with torch.distributed or MPI).
 * Waits that run out set the device status (qraf_cuda_device_status returns
 * QRAF_ERR_TIMEOUT). */
#define QRAF_COMM_HANDLE_BYTES 512
#define QRAF_COMM_BUFFERS 4
#define QRAF_COMM_MAX_WORLD 8
typedef struct qraf_comm* qraf_comm_t;
/* Allocate this rank's QRAF_COMM_BUFFERS output buffers of `capacity_floats`
 * floats each (used in turn, call by call) and its receive array (2 x
 * capacity_floats 8-byte words that the peers write) on the current device.
 * A call's activations may be the output of any of the previous
 * QRAF_COMM_BUFFERS - 1 calls. */
int qraf_cuda_comm_create(int world, int rank, uint64_t capacity_floats, qraf_comm_t* out);
/* This rank's CUDA IPC handle (its receive array), QRAF_COMM_HANDLE_BYTES bytes. */
int qraf_cuda_comm_handle(qraf_comm_t comm, void* handle_out);
/* Map every peer's receive array; `all_handles` holds world handles in rank order. */
int qraf_cuda_comm_open(qraf_comm_t comm, const void* all_handles);
/* Link `n` comms created by this one process (one per GPU, or several on one
 * GPU) directly, without IPC: peer access is enabled between distinct devices.
 * comms[i] must have rank i and world n. */
int qraf_cuda_comm_open_local(qraf_comm_t* comms, int n);
int qraf_cuda_comm_destroy(qraf_comm_t comm);
/* Rows [row_offset, row_offset + shard->rows) of a weight with total_rows rows
 * (the ranks' row ranges partition [0, total_rows)).  The kernel stores each of
 * its outputs into this rank's buffer and, with the call's number, into every
 * peer's receive array over NVLink; before it ends it copies the other ranks'
 * rows into this rank's buffer, so Y[m][n] for all n is in *y_out (this rank's
 * buffer for this call, valid for the next QRAF_COMM_BUFFERS - 1 calls) when
 * the launch completes.  Same arguments as qraf_cuda_matvec_q, modes EXACT,
 * FAST and TC; AUTO runs TC from three vectors (where the tensor-core path
 * applies) and FAST below.  EXACT and FAST need block size 32, K a multiple of
 * 32 and 16-byte-aligned rows and pointers; TC what qraf_cuda_matvec_q's TC mode
 * needs.  Any M: the vectors go in groups of one launch each (FAST: two; TC: up
 * to 64, the tile storing into the peers from its epilogue), every launch one
 * numbered call of the protocol.  EXACT and FAST give exactly the unsharded
 * result's bits; TC gives on each rank the bits of its shard's own TC call
 * (the tile's split of K among CTAs depends on the shard's row count).
 * The calls of one comm go to one stream, in the same order on every rank.  Calls are numbered on the device, so a sequence of
 * calls may be captured in a CUDA graph and replayed; capture a multiple of
 * QRAF_COMM_BUFFERS calls per comm so that replays keep the buffer rotation
 * (the buffers are chosen at capture).  A peer that does not deliver its rows
 * within about a second leaves the status QRAF_ERR_TIMEOUT. */
int qraf_cuda_matvec_q_sharded(qraf_comm_t comm, const qraf_weight_t* shard, uint32_t total_rows, uint32_t row_offset,
                               const float* x_dev, uint32_t M, int mode, void* stream, float** y_out);

/* ── host-pointer entry: the drop-in body of qraf::dispatch_matvec_q ────── */
/* Same arguments as the reference's dispatch_matvec_q (backend.h:31-34) plus M
 * and mode.  The first call with a given (w_host, w_size, dtype, bs, rows,
 * cols) uploads the weight to the current device and caches it (weights are
 * immutable model data, mmap'd read-only by the reference, loader.cpp:80);
 * each call copies x in, runs the kernel and copies y out before returning.
 * Thread-safe; calls on one device are serialised. */
int qraf_cuda_matvec_q_host(const void* w_host, uint64_t w_size, uint32_t dtype, uint32_t block_size,
                            uint32_t out_dim, uint32_t in_dim, const float* x_host, float* y_host, uint32_t M,
                            int mode);
/* Drop every cached device copy made by qraf_cuda_matvec_q_host. */
int qraf_cuda_host_cache_clear(void);
/* Upload one weight into that cache now, under the key a later
 * qraf_cuda_matvec_q_host call with the same arguments looks up, so the first
 * decode step pays no upload.  The call a host integration adds where the
 * reference's Transformer::init takes each weight's mapped bytes
 * (setup_layer_llama's set_w / set_mlp, src/nn/transformer.cpp:96-126, and the
 * lm_head, :374-389): out_dim = shape[0], in_dim = shape[1], block_size from the
 * tensor's QuantScheme (0 = 32).  w_size, when non-zero, must cover the rows. */
int qraf_cuda_host_cache_add(const void* w_host, uint64_t w_size, uint32_t dtype, uint32_t block_size,
                             uint32_t out_dim, uint32_t in_dim);
/* Number of cached weights and their device bytes (either pointer may be NULL). */
int qraf_cuda_host_cache_info(uint32_t* entries, uint64_t* device_bytes);

/* ── .qraf model files on the device ────────────────────────────────────── */
/* A .qraf file (the reference's format, include/qraf/format.h) with its Q8_0 /
 * Q4_0 tensors resident on one device.  qraf_cuda_model_open maps the file,
 * checks it as the reference's loader does (validate_header,
 * src/qraf/header.cpp:8-55; tensor bounds, src/qraf/loader.cpp:178-211; plus
 * every section and string this reader touches) and copies every quantized
 * tensor into one device allocation on the current device (256-byte aligned
 * tensors); rows = the product of the leading dimensions, cols = the last,
 * block size from the tensor's QuantScheme (32 without one).  F32 tensors are
 * not uploaded.  A malformed file returns QRAF_ERR_INVALID before any device
 * work.  Weights handed out are views (owned = 0), valid until
 * qraf_cuda_model_close. */
typedef struct qraf_model* qraf_model_t;
int qraf_cuda_model_open(const char* path, qraf_model_t* out);
/* The descriptor of the quantized tensor `name` (QRAF_ERR_INVALID if absent). */
int qraf_cuda_model_weight(qraf_model_t m, const char* name, qraf_weight_t* out);
/* Number of quantized tensors, bytes of the device allocation, device (each may be NULL). */
int qraf_cuda_model_info(qraf_model_t m, uint32_t* num_weights, uint64_t* device_bytes, int* device);
/* Name of quantized tensor `index` in directory order; NULL past the end. */
const char* qraf_cuda_model_weight_name(qraf_model_t m, uint32_t index);
/* Raw 32-bit value of a u32 or f32 config entry (ConfigEntry, format.h:61-65). */
int qraf_cuda_model_config_u32(qraf_model_t m, const char* key, uint32_t* value);
/* Free the device copy. */
int qraf_cuda_model_close(qraf_model_t m);
/* qraf_cuda_model_open with flags.  QRAF_MODEL_F32: the F32 tensors (embedding,
 * norms, biases, an F32 LM head) join the same device allocation, read by
 * qraf_cuda_model_tensor_f32 (the reference's Transformer::init loads them with
 * load_tensor_f32, src/nn/transformer.cpp:300-440). */
#define QRAF_MODEL_F32 1u
int qraf_cuda_model_open_ex(const char* path, uint32_t flags, qraf_model_t* out);
/* Device address and element count of the F32 tensor `name` of a model opened
 * with QRAF_MODEL_F32 (QRAF_ERR_INVALID if absent). */
int qraf_cuda_model_tensor_f32(qraf_model_t m, const char* name, const float** data, uint64_t* count);

/* ── decode engine ─────────────────────────────────────────────────────── */
/* A Llama / Qwen2 / Mistral decoder over a .qraf file, resident on the current
 * device: replaces Transformer::init + Transformer::forward(token, pos)
 * (src/nn/transformer.cpp:300-440, :573-620) and the request-at-a-time loop of
 * BatchScheduler (include/runtime/batch_scheduler.h:187-228).  open reads the
 * model (qraf_cuda_model_open_ex with QRAF_MODEL_F32; tensor names as
 * Transformer::init reads them; lm_head.weight quantized or F32, else the
 * embedding tied), allocates an F32 KV cache of max_slots x layers x max_seq
 * x kv_dim per K and V and the RoPE angles of every position. */
typedef struct qraf_decoder* qraf_decoder_t;
int qraf_cuda_decoder_open(const char* path, uint32_t max_slots, uint32_t max_seq, qraf_decoder_t* out);
/* qraf_cuda_decoder_open with flags.  QRAF_DECODER_KV_INT8: the KV cache holds
 * int8 codes with an fp32 scale per (position, KV head), quantized as the
 * reference's QuantizedKVCache::store does (include/nn/kv_cache_quant.h:61-94:
 * scale = max |x| / 127, codes clamp(round(x / scale), -127, 127)); attention
 * reads the codes (scores dot(q, codes) * scale, kv_cache_quant.h:113-123).
 * A quarter of the cache's bytes; needs head_dim % 16 == 0. */
#define QRAF_DECODER_KV_INT8 1u
int qraf_cuda_decoder_open_ex(const char* path, uint32_t max_slots, uint32_t max_seq, uint32_t flags,
                              qraf_decoder_t* out);
/* Copy one cache row (slot, layer, position) to host memory: kv_dim floats of K
 * and of V, or with the int8 cache kv_dim codes of each and kv_heads scales of each. */
int qraf_cuda_decoder_kv_read(qraf_decoder_t d, uint32_t slot, uint32_t layer, uint32_t pos, void* k_out, void* v_out,
                              float* k_scales, float* v_scales);
/* One decode step for M <= max_slots slots at once: slot slots_dev[m] takes
 * token tokens_dev[m] at position pos_dev[m] (all device int32 arrays of M;
 * slots distinct within a step; positions < max_seq), writes K/V at that
 * position of its cache, attends over positions 0 .. pos, and leaves the
 * logits in logits_dev[m][vocab].  `mode` picks the projections' arithmetic
 * (QRAF_MODE_*).  A token, position or slot out of range raises the device
 * status (qraf_cuda_device_status). */
int qraf_cuda_decoder_step(qraf_decoder_t d, uint32_t M, const int32_t* tokens_dev, const int32_t* pos_dev,
                           const int32_t* slots_dev, float* logits_dev, int mode, void* stream);
/* Sizes of the decoder (each pointer may be NULL). */
int qraf_cuda_decoder_info(qraf_decoder_t d, uint32_t* vocab, uint32_t* hidden, uint32_t* layers, uint32_t* max_slots,
                           uint32_t* max_seq);
/* Free the decoder, its caches and its model. */
int qraf_cuda_decoder_close(qraf_decoder_t d);

/* ── host utility ───────────────────────────────────────────────────────── */
/* Seeded synthetic data with the reference's idiom: std::mt19937(seed) and
 * std::normal_distribution<float>(mean, stddev) (tools/dummy_model.cpp:12-16). */
void qraf_fill_normal(uint32_t seed, float mean, float stddev, float* out_host, uint64_t n);

#ifdef __cplusplus
}
#endif
#endif /* QRAF_CUDA_H */
