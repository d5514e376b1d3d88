/*
 * glm5x_moe.h -- C ABI of the B200 routed-expert MoE sublayer.
 *
 * Drop-in for the expert-sublayer boundary of rsb1813/project-glm5x. Every
 * entry point names the reference interface it replaces (paths inside the
 * reference project). Plain pointers and sizes only; `stream` arguments are
 * cudaStream_t handles passed as void* (NULL = the engine's own stream).
 *
 * Conventions (runtime/include/k3x/backend.hpp:170-298):
 *  - Every function returns a glm5x_status; codes 0..19 keep the values of
 *    k3x::ErrorCode (runtime/include/k3x/status.hpp:9-30). The message of the
 *    last failure is available from glm5x_moe_error_message() (per engine) or
 *    glm5x_last_error_message() (per thread, for calls without an engine).
 *  - Bad inputs are rejected before any device work.
 *  - One engine = one device, one stream; not thread-safe, like CudaBackend.
 *  - Weights are NVFP4 ([out, in] packed two E2M1 per byte, low nibble first,
 *    E4M3 block-16 scales in the 128x4 blocked layout, one FP32 global
 *    scale) exactly as the reference's packer and .pn4 sidecars store them
 *    (reference/glm5x_ref/nvfp4.py:58-198, packed_cache.py:277-309), or
 *    MXFP4 (E8M0 group-32 scales, row-major, mxfp4.py:31-107).
 */
#ifndef GLM5X_MOE_H_
#define GLM5X_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* k3x::ErrorCode values (status.hpp:9-30) plus engine-specific codes. */
typedef enum glm5x_status {
  GLM5X_OK = 0,
  GLM5X_IO_ERROR = 1,
  GLM5X_BAD_MAGIC = 2,
  GLM5X_UNSUPPORTED_VERSION = 3,
  GLM5X_UNSUPPORTED_REQUIRED_FEATURE = 4,
  GLM5X_SUPERBLOCK_CRC_MISMATCH = 6,
  GLM5X_TRUNCATED_FILE = 7,
  GLM5X_INVALID_DIRECTORY = 8,
  GLM5X_INVALID_EXTENT = 9,
  GLM5X_DATA_CRC_MISMATCH = 10,
  GLM5X_AUXILIARY_CRC_MISMATCH = 11,
  GLM5X_DIRECTORY_SHA256_MISMATCH = 12,
  GLM5X_ROOT_SHA256_MISMATCH = 13,
  GLM5X_TENSOR_NOT_FOUND = 14,
  GLM5X_INVALID_MXFP4 = 15,
  GLM5X_INVALID_STATE = 16,
  GLM5X_BACKEND_UNAVAILABLE = 17,
  GLM5X_UNSUPPORTED_ARCHITECTURE = 19,
  GLM5X_DEVICE_ERROR = 100,    /* CUDA error or a device-side error word */
  GLM5X_OUT_OF_MEMORY = 101,
  GLM5X_WAIT_TIMEOUT = 102     /* a bounded device wait gave up */
} glm5x_status;

typedef enum glm5x_precision {
  GLM5X_PRECISION_NVFP4 = 0,   /* E2M1 + E4M3/16 + FP32 global */
  GLM5X_PRECISION_MXFP4 = 1    /* E2M1 + E8M0/32 */
} glm5x_precision;

typedef enum glm5x_scale_mode {
  GLM5X_SCALE_MAX_ABS = 0,     /* nvfp4.py:164-170, mxfp4.py:70-79 */
  GLM5X_SCALE_MSE = 1          /* nvfp4.py:139-163, mxfp4.py:80-97 */
} glm5x_scale_mode;

/* Layer shape and policy. Replaces the constructor arguments of
 * GLM5XLayer10MoEReference (reference/glm5x_ref/layer10_moe.py:352-374) and
 * the fixed constants of build_learned_routes
 * (runtime/src/cuda_glm5x_real_expert_bench.cpp:291-293). */
typedef struct glm5x_moe_config {
  int32_t hidden;            /* 6144 */
  int32_t intermediate;      /* 2048 */
  int32_t num_experts;       /* 256 routed experts (global count) */
  int32_t top_k;             /* 8 */
  int32_t has_shared;        /* 1: one always-on shared expert */
  float routed_scaling;      /* 2.5 */
  int32_t precision;         /* glm5x_precision */
  int32_t max_tokens;        /* largest T per forward on this engine */
  int32_t expert_begin;      /* first expert held here (expert parallel) */
  int32_t expert_count;      /* experts held here; num_experts on one GPU */
} glm5x_moe_config;

/* One NVFP4 matrix [rows, cols] (GLM5XNVFP4Weight, nvfp4.py:58-98). */
typedef struct glm5x_nvfp4_matrix {
  const uint8_t* packed;     /* rows * cols / 2 bytes */
  const uint8_t* scales;     /* blocked E4M3, ceil(rows/128)*ceil(cols/64)*512 bytes */
  float global_scale;
  int64_t rows;
  int64_t cols;
} glm5x_nvfp4_matrix;

/* One MXFP4 matrix (Mxfp4WeightView, runtime/include/k3x/backend.hpp:114-121). */
typedef struct glm5x_mxfp4_matrix {
  const uint8_t* packed;     /* rows * cols / 2 bytes */
  const uint8_t* scales;     /* row-major E8M0, rows * cols / group bytes */
  int64_t rows;
  int64_t cols;
  int64_t group_size;        /* 32 */
} glm5x_mxfp4_matrix;

typedef struct glm5x_moe_stats {
  /* subset of k3x::BackendRuntimeStats (backend.hpp:55-105) */
  uint64_t forward_calls;
  uint64_t kernel_launches;
  uint64_t resident_weight_bytes;
  uint64_t activation_h2d_bytes;
  uint64_t device_to_host_bytes;
  uint64_t stream_synchronization_count;
  uint64_t workspace_bytes;
  uint64_t loaded_experts;
} glm5x_moe_stats;

typedef struct glm5x_moe glm5x_moe;

/* ---------------------------------------------------------------- engine */

/* make_cuda_backend (backend.hpp:296-298; backend_cuda.cu:5091-5168).
 * Fails with GLM5X_UNSUPPORTED_ARCHITECTURE on anything but sm_100. */
glm5x_status glm5x_moe_create(const glm5x_moe_config* config, int device, glm5x_moe** out);
void glm5x_moe_destroy(glm5x_moe* moe);
const char* glm5x_moe_error_message(const glm5x_moe* moe);
const char* glm5x_last_error_message(void);

/* Router weight [num_experts, hidden] BF16 and correction bias [num_experts]
 * FP32, host memory (GLM5XLayer10MoEReference router_weight /
 * correction_bias, layer10_moe.py:375-380, 411-413). */
glm5x_status glm5x_moe_set_router(glm5x_moe* moe, const uint16_t* weight_bf16,
                                  const float* bias);

/* Admit one expert's gate/up [I, H] and down [H, I] NVFP4 matrices.
 * expert = global expert id, or -1 for the shared expert. Host pointers
 * (load_glm5x_bf16_expert, runtime/include/k3x/glm5x_bundle.hpp:21-26;
 * GLM5XPackedExpertCache.get, packed_cache.py:506-617). */
glm5x_status glm5x_moe_load_expert_nvfp4(glm5x_moe* moe, int32_t expert,
                                         const glm5x_nvfp4_matrix* gate,
                                         const glm5x_nvfp4_matrix* up,
                                         const glm5x_nvfp4_matrix* down);
/* Same, with the matrices already in device memory (no host staging). */
glm5x_status glm5x_moe_load_expert_nvfp4_device(glm5x_moe* moe, int32_t expert,
                                                const glm5x_nvfp4_matrix* gate,
                                                const glm5x_nvfp4_matrix* up,
                                                const glm5x_nvfp4_matrix* down);
/* MXFP4 expert (Mxfp4MlpView, backend.hpp:154-158), host pointers: packed
 * [rows, cols/2] low nibble first and row-major E8M0 scales [rows, cols/32]
 * (encode_mxfp4, k3x_ref/mxfp4.py:31-107). group_size must be 32. A 0xFF
 * scale is rejected with GLM5X_INVALID_MXFP4 (decode_mxfp4,
 * runtime/src/ops.cpp:40-63). The engine must be created with
 * GLM5X_PRECISION_MXFP4; its forward feeds the experts four MXFP4 residual
 * terms per activation row (the reference's MXFP4 path keeps activations in
 * full precision, backend_cuda.cu:1878-2171). */
glm5x_status glm5x_moe_load_expert_mxfp4(glm5x_moe* moe, int32_t expert,
                                         const glm5x_mxfp4_matrix* gate,
                                         const glm5x_mxfp4_matrix* up,
                                         const glm5x_mxfp4_matrix* down);
/* Same, with the matrices already in device memory (no host staging). */
glm5x_status glm5x_moe_load_expert_mxfp4_device(glm5x_moe* moe, int32_t expert,
                                                const glm5x_mxfp4_matrix* gate,
                                                const glm5x_mxfp4_matrix* up,
                                                const glm5x_mxfp4_matrix* down);
/* BF16 expert (load_glm5x_bf16_expert's roles, runtime/include/k3x/
 * glm5x_bundle.hpp:15-26; RawBf16MlpView, backend.hpp:129-140): gate/up [I, H]
 * and down [H, I] BF16 row-major, host pointers, packed on the device at
 * admission. NVFP4 engines pack each projection with quantize_nvfp4_weight
 * (the reference's NVFP4 mode does this when it loads float experts,
 * _quantize_expert_nvfp4, layer10_moe.py:603-619; GLM5X_SCALE_MSE is its
 * default), bit-identical to the reference's packer; MXFP4 engines encode
 * with encode_mxfp4, group 32 (k3x_ref/mxfp4.py:31-107). The packed bytes are
 * then admitted as by glm5x_moe_load_expert_nvfp4 / _mxfp4. Synchronizes. */
glm5x_status glm5x_moe_load_expert_bf16(glm5x_moe* moe, int32_t expert, const uint16_t* gate,
                                        const uint16_t* up, const uint16_t* down,
                                        int32_t scale_mode);
/* Same, with the BF16 projections already in device memory. */
glm5x_status glm5x_moe_load_expert_bf16_device(glm5x_moe* moe, int32_t expert,
                                               const uint16_t* gate, const uint16_t* up,
                                               const uint16_t* down, int32_t scale_mode);
/* Parse and admit a .pn4 / .pm4 packed sidecar of the engine's precision
 * (GLM5XPackedExpertCache.get / _decode_role, packed_cache.py:506-617,
 * 407-504): glm5x_sidecar_open(path, engine precision, NULL) then
 * glm5x_moe_load_expert_sidecar. */
glm5x_status glm5x_moe_load_sidecar(glm5x_moe* moe, int32_t expert, const char* path);

/* ---------------------------------------------------------------- packed sidecars */

/* An open, fully checked packed expert sidecar (host memory only; no device
 * work). Layout of GLM5XPackedExpertCache.put (packed_cache.py:327-404):
 * header "<8sII" = ("GLM5XPI4", 1, json_len), compact sorted-key JSON
 * {format "glm5x-<nvfp4|mxfp4>-expert-v1", source_digest, roles [gate, up,
 * down], payload_bytes}, then the payload (per role: packed E2M1 bytes, then
 * qparams = blocked E4M3 scales + FP32 global for NVFP4, row-major E8M0 for
 * MXFP4). The checks run in the order of the reference's get / _decode_role
 * (packed_cache.py:518-545, 407-423, 476-479), and the message of a failure
 * (glm5x_last_error_message) starts with the reference's error code:
 *   GLM5X_PACKED_CACHE_HEADER       TRUNCATED_FILE    file shorter than 16 bytes
 *   GLM5X_PACKED_CACHE_FORMAT       BAD_MAGIC / UNSUPPORTED_VERSION / INVALID_STATE
 *                                   (magic, version, format string vs `precision`)
 *   GLM5X_PACKED_CACHE_METADATA     INVALID_DIRECTORY metadata not a JSON object
 *   GLM5X_PACKED_CACHE_SOURCE_MISMATCH INVALID_STATE  source_digest differs
 *   GLM5X_PACKED_CACHE_ROLES        INVALID_DIRECTORY roles not three complete records
 *   GLM5X_PACKED_CACHE_PAYLOAD_EXTENT INVALID_EXTENT  payload size / a section outside it
 *   GLM5X_PACKED_CACHE_PACKED_CRC   DATA_CRC_MISMATCH
 *   GLM5X_PACKED_CACHE_QPARAM_CRC   AUXILIARY_CRC_MISMATCH
 *   GLM5X_PACKED_CACHE_NVFP4_QPARAM_EXTENT INVALID_EXTENT scale + global bytes != qparams
 * precision: GLM5X_PRECISION_NVFP4 / _MXFP4, or -1 to take the file's;
 * source_digest: the digest get() is given, or NULL to skip that check. */
typedef struct glm5x_sidecar glm5x_sidecar;

typedef struct glm5x_sidecar_role {
  int32_t precision;       /* glm5x_precision of the file */
  int32_t reserved;
  int64_t rows, cols, group_size;
  const uint8_t* packed;   /* rows * cols / 2 bytes, inside the reader */
  int64_t packed_bytes;
  const uint8_t* scales;   /* NVFP4: blocked E4M3; MXFP4: row-major E8M0 */
  int64_t scale_bytes;
  float global_scale;      /* NVFP4; 1 for MXFP4 */
} glm5x_sidecar_role;

glm5x_status glm5x_sidecar_open(const char* path, int32_t precision, const char* source_digest,
                                glm5x_sidecar** out);
void glm5x_sidecar_close(glm5x_sidecar* sidecar);
/* role 0 gate, 1 up, 2 down; the pointers stay valid until close. */
glm5x_status glm5x_sidecar_get_role(const glm5x_sidecar* sidecar, int32_t role,
                                    glm5x_sidecar_role* out);
/* "<root>/layer-LLLL-expert-EEEE.<pn4|pm4>" (GLM5XPackedExpertCache._path,
 * packed_cache.py:198-214); GLM5X_INVALID_STATE for a negative key. */
glm5x_status glm5x_sidecar_path(const char* root, int32_t layer, int32_t expert,
                                int32_t precision, char* buf, size_t capacity);
/* Admits expert slot `expert` (-1 = shared) from an open sidecar of the
 * engine's precision through glm5x_moe_load_expert_nvfp4 / _mxfp4. */
glm5x_status glm5x_moe_load_expert_sidecar(glm5x_moe* moe, int32_t expert,
                                           const glm5x_sidecar* sidecar);

/* ---------------------------------------------------------------- .k3x containers */

/* An open K3X v1 checkpoint container (.k3x), the reference runtime's weight
 * file: opened with the checks of k3x::Reader::open (runtime/src/reader.cpp:
 * 420-702) and its status codes (BAD_MAGIC, UNSUPPORTED_VERSION,
 * SUPERBLOCK_CRC_MISMATCH, TRUNCATED_FILE, INVALID_DIRECTORY, INVALID_EXTENT,
 * ...). verify_checksums = 1 is the reader's checksums mode: every extent's
 * CRC32C and the directory and root SHA-256 (a pass over the whole file);
 * 0 checks the metadata only. Host memory only. */
typedef struct glm5x_k3x glm5x_k3x;

/* One tensor record (converter/k3x_converter/format.py:155-210): dtype 1 FP32,
 * 2 UINT8, 3 BF16; quantization 1 = MXFP4 (UINT8 packed E2M1 data, E8M0
 * auxiliary extent); dimensions[0..rank) = the logical shape. */
typedef struct glm5x_k3x_tensor_info {
  uint64_t tensor_id; /* FNV-1a 64 of the tensor name */
  int32_t dtype;
  int32_t quantization;
  int32_t rank;
  int32_t layer_id;   /* -1 = none */
  int32_t expert_id;  /* -1 = none */
  int32_t reserved;
  uint64_t dimensions[4];
  uint64_t data_length;
  uint64_t logical_length;
  uint64_t auxiliary_length;
} glm5x_k3x_tensor_info;

glm5x_status glm5x_k3x_open(const char* path, int32_t verify_checksums, glm5x_k3x** out);
void glm5x_k3x_close(glm5x_k3x* file);
/* The record of tensor `name` (looked up by FNV-1a 64 of the name, as
 * runtime/src/model.cpp:538-551 does); TENSOR_NOT_FOUND if absent. */
glm5x_status glm5x_k3x_tensor(const glm5x_k3x* file, const char* name,
                              glm5x_k3x_tensor_info* info);
/* Reads tensor `name`'s data (and auxiliary extent, when it has one and
 * `auxiliary` is not NULL) into host buffers of at least their lengths
 * (Reader::read_tensor / read_auxiliary, runtime/src/reader.cpp:749-778). */
glm5x_status glm5x_k3x_read(const glm5x_k3x* file, const char* name, void* data,
                            uint64_t data_capacity, void* auxiliary, uint64_t auxiliary_capacity);
/* Admits expert slot `expert` (-1 = shared) from the three MXFP4 records
 * `<prefix>.gate`, `<prefix>.up`, `<prefix>.down` of an open container (the
 * names runtime/src/model.cpp:538-551 builds, e.g.
 * "model.layers.1.feed_forward.experts.3"), through
 * glm5x_moe_load_expert_mxfp4: row-major E8M0 scales are reordered into the
 * MMA's blocked layout, 0xFF scales rejected. The engine must be MXFP4. */
glm5x_status glm5x_moe_load_expert_k3x(glm5x_moe* moe, int32_t expert, const glm5x_k3x* file,
                                       const char* prefix);

/* Full sublayer on device buffers: hidden [T, hidden] BF16 -> out [T, hidden]
 * FP32 = sum over top-k of weight * expert(x) + shared(x). Asynchronous on
 * `stream`. (GLM5XLayer10MoEReference.__call__, layer10_moe.py:942-968;
 * CudaBackend::raw_bf16_situ_mlp_expert_major_with_shared,
 * backend_cuda.cu:1545-1867.) */
glm5x_status glm5x_moe_forward(glm5x_moe* moe, const void* hidden_bf16, int64_t tokens,
                               float* out, void* stream);
/* Same with host buffers (H2D, forward, D2H, synchronize): the reference's
 * ComputeBackend convention of host spans in and host vectors out. */
glm5x_status glm5x_moe_forward_host(glm5x_moe* moe, const uint16_t* hidden_bf16,
                                    int64_t tokens, float* out);
/* Pipelined form of glm5x_moe_forward_host for callers with a stream of
 * batches (no reference counterpart: ComputeBackend calls are synchronous).
 * Enqueues the upload of `hidden_bf16`, the forward and the download into
 * `out` and returns a ticket without waiting. The upload runs on a copy
 * stream, the forward on the engine's stream and the download on a second
 * copy stream, ordered by events over two staging slots, so the upload of one
 * batch, the forward of the previous one and the download of the one before
 * overlap. Both host buffers must stay valid and unchanged until
 * glm5x_moe_wait_host(ticket) returns; page-locked buffers let the copies
 * run asynchronously. Results equal glm5x_moe_forward_host's. */
glm5x_status glm5x_moe_submit_host(glm5x_moe* moe, const uint16_t* hidden_bf16, int64_t tokens,
                                   float* out, int64_t* ticket);
/* Copies n <= 4096 int64 words from device memory to `dst` (host) after the
 * work already on `stream` (NULL = the engine's stream), through page-locked
 * mapped memory the device writes with ordinary stores, then synchronizes
 * `stream`. A read-back of a few counts this way uses no copy engine, so it
 * does not wait behind a large download running on another stream (the
 * expert-parallel dispatch reads its all-to-all counts with it). */
glm5x_status glm5x_moe_read_ints(glm5x_moe* moe, const int64_t* src, int64_t n, int64_t* dst,
                                 void* stream);
/* Blocks until the download of `ticket` is done and returns the status of its
 * forward's device checks (the error words glm5x_moe_check reports).
 * GLM5X_INVALID_STATE for a ticket not yet submitted or older than the last
 * 64 submissions. */
glm5x_status glm5x_moe_wait_host(glm5x_moe* moe, int64_t ticket);
/* Expert path only, with caller-supplied routing (device buffers): ids
 * [T, top_k] int32 global expert ids, weights [T, top_k] FP32 (the
 * contribution of each slot, already scaled). Replaces
 * mxfp4_situ_mlp_grid / raw_bf16_situ_mlp_expert_major
 * (backend.hpp:220-252) for callers that route themselves. */
glm5x_status glm5x_moe_forward_routed(glm5x_moe* moe, const void* hidden_bf16, int64_t tokens,
                                      const int32_t* ids, const float* weights, float* out,
                                      void* stream);
/* Expert-parallel building blocks (experts sharded across
 * ranks by config.expert_begin / expert_count, tokens exchanged by the
 * caller's all-to-all). The reference has no expert-parallel API; these
 * replace the per-rank halves of its single-process expert path
 * (layer10_moe.py:760-847 + 954-961).
 *
 * glm5x_moe_route: router only (logits, sigmoid + bias, top-k, renormalize,
 * x routed_scaling) over `tokens` BF16 rows on the device; ids/weights
 * [tokens, top_k], logits [tokens, num_experts] (NULL: internal buffer). */
glm5x_status glm5x_moe_route(glm5x_moe* moe, const void* hidden_bf16, int64_t tokens,
                             int32_t* ids, float* weights, float* logits, void* stream);
/* glm5x_moe_forward_expert_rows: rows [R, hidden] BF16 dispatched to this
 * engine, ids [R, top_k] GLOBAL expert ids (slots whose expert this engine
 * does not hold, or -1, are skipped), weights [R, top_k]. out[r] = sum over
 * the held slots of weight * expert(row r), plus the shared expert for rows
 * r < shared_rows. FP32 out [R, hidden]. */
glm5x_status glm5x_moe_forward_expert_rows(glm5x_moe* moe, const void* rows_bf16, int64_t rows,
                                           const int32_t* ids, const float* weights,
                                           int64_t shared_rows, float* out, void* stream);

/* ---------------------------------------------------------------- expert parallelism */

/* Expert-parallel MoE sublayer over the GPUs of one node (no counterpart in
 * the reference, which runs every expert in one process; this is the
 * multi-GPU form of layer10_moe.py:791-847 + 954-961, the drop-in's EP entry
 * glm5x_moe_create_ep). One object per rank, one process per GPU: rank r of
 * `world` holds experts [r * E/world, (r + 1) * E/world) plus a replica of the
 * shared expert and the router (load them through glm5x_moe_ep_engine with
 * GLOBAL expert ids). Tokens are exchanged by the library's own kernels over
 * NVLink peer memory, mapped through CUDA IPC: each rank stores every token
 * row once into each destination rank that holds one of its experts, and
 * pulls each destination's weighted partial sum back (see ep_peer.cu); no
 * host synchronization inside a forward. The result equals the NCCL
 * all-to-all form (glm5x_moe/ep.py) bit for bit.
 *
 * Every rank must call glm5x_moe_ep_forward the same number of times (T may
 * differ per rank, and may be 0); its waits on peers are bounded, and a peer
 * that does not take part makes glm5x_moe_ep_check report
 * GLM5X_WAIT_TIMEOUT. All ranks must have finished their last forward (e.g.
 * a barrier) before any rank calls glm5x_moe_ep_destroy. */
typedef struct glm5x_moe_ep glm5x_moe_ep;
#define GLM5X_EP_HANDLE_BYTES 64

/* Creates rank `rank` of `world` (<= 16) with room for max_local_tokens
 * local tokens per forward (the receive area holds world times that). The
 * config is the whole layer's (num_experts = all experts; expert_begin /
 * expert_count / max_tokens are set here). Not usable until connected. */
glm5x_status glm5x_moe_ep_create(const glm5x_moe_config* config, int device, int32_t rank,
                                 int32_t world, int64_t max_local_tokens, glm5x_moe_ep** out);
/* This rank's GLM5X_EP_HANDLE_BYTES-byte memory handle, for the caller to
 * gather from every rank (any transport). */
glm5x_status glm5x_moe_ep_handle(glm5x_moe_ep* ep, void* handle);
/* Maps every peer's memory: handles = world * GLM5X_EP_HANDLE_BYTES bytes in
 * rank order (this rank's own entry is not used). */
glm5x_status glm5x_moe_ep_connect(glm5x_moe_ep* ep, const void* handles);
/* glm5x_moe_ep_create + handle exchange over the caller's NCCL communicator
 * (an ncclComm_t of exactly these `world` ranks, this process being `rank`;
 * one ncclAllGather of the handles) + glm5x_moe_ep_connect. NCCL is taken
 * from the process (the library that made `nccl_comm`), else libnccl.so.2. */
glm5x_status glm5x_moe_create_ep(const glm5x_moe_config* config, int device, void* nccl_comm,
                                 int32_t rank, int32_t world, int64_t max_local_tokens,
                                 glm5x_moe_ep** out);
/* The rank's engine (owned by the EP object): glm5x_moe_set_router,
 * glm5x_moe_load_expert_* (global ids of the held experts, -1 = shared). */
glm5x_moe* glm5x_moe_ep_engine(glm5x_moe_ep* ep);
/* hidden [T, H] BF16 (device) -> out [T, H] FP32 (device) = sum over top-k
 * of weight * expert(x) + shared(x), experts on whichever rank holds them.
 * Asynchronous on `stream` (NULL = the EP object's stream). */
glm5x_status glm5x_moe_ep_forward(glm5x_moe_ep* ep, const void* hidden_bf16, int64_t tokens,
                                  float* out, void* stream);
/* Synchronizes the device and reports the engine's and the exchange's error
 * words (GLM5X_WAIT_TIMEOUT when a peer did not answer in time). */
glm5x_status glm5x_moe_ep_check(glm5x_moe_ep* ep);
const char* glm5x_moe_ep_error_message(const glm5x_moe_ep* ep);
/* Stage times of later forwards, with CUDA events on the forward's stream
 * (each event adds a few microseconds): 0 route, 1 plan + count exchange, 2
 * dispatch + the wait for every source's rows, 3 experts, 4 ready + the
 * partial-sum pull. glm5x_moe_ep_stage_times synchronizes and writes the
 * milliseconds summed per stage since its last call and the forwards counted. */
#define GLM5X_EP_STAGES 5
glm5x_status glm5x_moe_ep_set_profiling(glm5x_moe_ep* ep, int32_t enable);
glm5x_status glm5x_moe_ep_stage_times(glm5x_moe_ep* ep, float* ms, int32_t* forwards);
/* Rows the last forward sent to each rank (sent[world]) and received in all
 * (synchronizes the device). */
glm5x_status glm5x_moe_ep_last_counts(glm5x_moe_ep* ep, int64_t* sent, int64_t* received);
void glm5x_moe_ep_destroy(glm5x_moe_ep* ep);

/* Expert-parallel FP4 dispatch (no counterpart in the reference, which runs
 * every expert in one process). The slab of a routed expert is every rank's
 * tokens routed to it, as one GPU would see the concatenated batch; its NVFP4
 * global scale needs the slab's max |x| over all ranks. So:
 *  1. glm5x_moe_slab_amax: amax[e] (device, num_experts floats) = max |x| of
 *     this rank's tokens routed to e (ids [T, top_k] global ids, -1 skipped);
 *     the caller reduces it with MAX over the ranks;
 *  2. glm5x_moe_quantize_rows: NVFP4 codes (packed [n, H/2]) and row-major
 *     E4M3 scales ([n, H/16]) of token row_token[r] for expert row_expert[r]
 *     with that expert's reduced slab scale: the bits the single-GPU segment
 *     quantizer gives the row; these rows travel instead of BF16 rows;
 *  3. glm5x_moe_forward_quantized_rows on the rank holding the experts: the
 *     T local tokens take the shared expert (out_local [T, H] FP32, their own
 *     slab) and the R received rows their expert (row_expert global ids held
 *     here, row_weight the routing weights); out_groups[g] (FP32 [groups, H])
 *     = the sum, in listed order, of the weighted expert rows of received rows
 *     group_rows[g, 0 .. slots) (-1 = none), e.g. one group per source token.
 * T + R must not exceed max_tokens. NVFP4 engines only. */
glm5x_status glm5x_moe_slab_amax(glm5x_moe* moe, const void* hidden_bf16, int64_t tokens,
                                 const int32_t* ids, float* amax, void* stream);
glm5x_status glm5x_moe_quantize_rows(glm5x_moe* moe, const void* hidden_bf16, int64_t tokens,
                                     const int32_t* row_token, const int32_t* row_expert,
                                     int64_t rows, const float* amax, void* packed,
                                     void* scales, void* stream);
glm5x_status glm5x_moe_forward_quantized_rows(glm5x_moe* moe, const void* hidden_bf16,
                                              int64_t tokens, const void* packed,
                                              const void* scales, const int32_t* row_expert,
                                              const float* row_weight, int64_t rows,
                                              const float* amax, float* out_local,
                                              const int32_t* group_rows, int64_t groups,
                                              int32_t slots, float* out_groups, void* stream);
/* Routing of the last forward (synchronizes): ids/weights [T, top_k] in
 * descending choice order, logits [T, num_experts] (may be NULL). */
glm5x_status glm5x_moe_last_routing(glm5x_moe* moe, int32_t* ids, float* weights,
                                    float* logits, int64_t tokens);
/* Synchronizes and turns the device error word into a status. */
glm5x_status glm5x_moe_check(glm5x_moe* moe);
glm5x_status glm5x_moe_get_stats(const glm5x_moe* moe, glm5x_moe_stats* out);
/* Device pointer and size of an internal buffer of the last forward, for
 * parity tests: 0 act packed, 1 act scales (blocked), 2 act global [nseg],
 * 3 h BF16 [rows, I], 4 h packed, 5 h scales, 6 h global, 7 y BF16 [rows, H],
 * 8 segment starts [nseg+1] int32, 9 segment counts [nseg], 10 row_token,
 * 11 pos [T, k+1], 12 row_weight. */
glm5x_status glm5x_moe_debug_buffer(glm5x_moe* moe, int32_t which, void** ptr, size_t* bytes);
/* Phase timing with CUDA events on the forward's stream (the per-projection
 * device times the reference records, backend_cuda.cu:2034-2040, 2151-2168).
 * Phases: 0 row amax, 1 router (tcgen05 logits + top-k), 2 (unused), 3 permutation, 4 activation
 * quantize, 5 gate/up GEMM, 6 h quantize, 7 down GEMM, 8 combine. */
#define GLM5X_NUM_PHASES 9
glm5x_status glm5x_moe_set_profiling(glm5x_moe* moe, int32_t enable);
/* Synchronizes; writes the milliseconds accumulated per phase since the last
 * call (ms[GLM5X_NUM_PHASES]) and the number of profiled forwards, then resets. */
glm5x_status glm5x_moe_phase_times(glm5x_moe* moe, float* ms, int32_t* forwards);
/* Token-tile width of the expert GEMMs: 32, 64, 128 or 256 rows, or 0 to
 * choose from the batch (the default). */
glm5x_status glm5x_moe_set_tile_n(glm5x_moe* moe, int32_t bn);
/* 256-row token tiles run on CTA pairs (tcgen05 cta_group::2, enable = 1,
 * the default) or on single CTAs (enable = 0); both give the same results to
 * within accumulation order. */
glm5x_status glm5x_moe_set_pair_mma(glm5x_moe* moe, int32_t enable);
/* Down projection of batches with >= 128-row token tiles: token-major tiles
 * (enable = 1: each epilogue thread stores one token's output features) or
 * weight-major tiles like the gate/up GEMM (the default, enable = 0); same
 * results to within accumulation order. */
glm5x_status glm5x_moe_set_token_major_down(glm5x_moe* moe, int32_t enable);
/* Weight-major down projection of batches with >= 128-row token tiles: token
 * tile width 128 or 256 (0 = the gate/up GEMM's). Used when token-major tiles
 * are off. */
glm5x_status glm5x_moe_set_down_tile_n(glm5x_moe* moe, int32_t bn);
/* CTA-pair GEMMs (256-row token tiles) with pipeline stages of 512 of K
 * (enable = 1, the default: one barrier wait and one commit of the
 * MMA-issuing thread per eight MMAs, operand, token and scale copies from
 * three threads) or of 256 (0). Same results: every output sums the same
 * products in the same order. */
glm5x_status glm5x_moe_set_pair_wide_stages(glm5x_moe* moe, int32_t enable);
/* Weight rows per tile of the GEMMs for 32- and 64-row token tiles (small
 * batches such as decode): 256 (the default: two 128-row halves with their
 * own accumulators in one stage, so each stage hand-off streams twice the
 * weight bytes) or 128 (one M = 128 MMA per K step). Both give the same
 * results: every output element sums the same products in the same order. */
glm5x_status glm5x_moe_set_weight_tile_rows(glm5x_moe* moe, int32_t rows);
/* Tile order of the CTA-pair GEMMs (256-row token tiles), per GEMM: 0 runs
 * a segment's weight tiles in turn; g > 0 cuts the segments into groups of
 * about g token tiles and runs each group weight-tile-major (weight tile 0
 * of every segment in the group, then tile 1, ...), so light and heavy
 * experts share the GPU at every moment. Defaults: 8 (gate/up) and 16
 * (down). Results do not depend on it: every tile computes the same sums. */
glm5x_status glm5x_moe_set_pair_tile_order(glm5x_moe* moe, int32_t up_group, int32_t down_group);
/* The engine's own stream (used by glm5x_moe_forward_host and by forwards
 * given a NULL stream), as a cudaStream_t. */
glm5x_status glm5x_moe_get_stream(glm5x_moe* moe, void** stream);
/* Synchronizes, then copies the first `bytes` of debug buffer `which` to the
 * device pointer `dst`. */
glm5x_status glm5x_moe_debug_copy(glm5x_moe* moe, int32_t which, void* dst, size_t bytes);

/* ---------------------------------------------------------------- kernels */
/* Stand-alone device kernels. All pointers are device pointers. */

/* Converter NVFP4 packing of one matrix (quantize_nvfp4_weight,
 * nvfp4.py:180-198; scale_mode GLM5X_SCALE_MSE is the reference default).
 * src FP32 or BF16 [rows, cols]; packed [rows, cols/2]; scales blocked;
 * global_out one float (device). */
glm5x_status glm5x_nvfp4_quantize_f32(const float* src, int64_t rows, int64_t cols,
                                      int32_t scale_mode, uint8_t* packed, uint8_t* scales,
                                      float* global_out, void* stream);
glm5x_status glm5x_nvfp4_quantize_bf16(const uint16_t* src, int64_t rows, int64_t cols,
                                       int32_t scale_mode, uint8_t* packed, uint8_t* scales,
                                       float* global_out, void* stream);
/* Activation quantization of expert-major slabs (layer10_moe.py:729 ->
 * nvfp4.py:236-252): rows seg_start[s] .. + seg_count[s] of the output take
 * src rows row_token[row]; each segment gets its own global scale
 * (seg_global[s]). Scales are written in the blocked layout of the output
 * row space. nseg <= 1024; cols a multiple of 512. */
glm5x_status glm5x_nvfp4_quantize_slabs_bf16(const uint16_t* src, int64_t cols,
                                             const int32_t* row_token, const int32_t* seg_start,
                                             const int32_t* seg_count, int32_t nseg,
                                             int64_t out_rows, uint8_t* packed,
                                             uint8_t* scales, float* seg_global, void* stream);
/* dequantize_nvfp4 (nvfp4.py:201-217). */
glm5x_status glm5x_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales,
                                    float global_scale, int64_t rows, int64_t cols, float* out,
                                    void* stream);
/* encode_mxfp4 (k3x_ref/mxfp4.py:31-107); synchronizes to report
 * GLM5X_INVALID_MXFP4 for exponents above 126. */
glm5x_status glm5x_mxfp4_encode_f32(const float* src, int64_t rows, int64_t cols,
                                    int64_t group_size, int32_t scale_mode, uint8_t* packed,
                                    uint8_t* scales, void* stream);
/* decode_mxfp4 (mxfp4.py:110-144; runtime/src/ops.cpp:40-63); synchronizes
 * to report GLM5X_INVALID_MXFP4 for the reserved scale 0xFF. */
glm5x_status glm5x_mxfp4_decode(const uint8_t* packed, const uint8_t* scales, int64_t rows,
                                int64_t cols, int64_t group_size, float* out, void* stream);
/* select_routing natural mode over given sigmoid scores (routing_policy.cpp:
 * 31-159) for T tokens at once: scores/bias -> ids [T,k], weights [T,k]
 * multiplied by routed_scale (1.0 reproduces select_routing itself). */
glm5x_status glm5x_select_routing(const float* scores, const float* bias, int64_t tokens,
                                  int32_t num_experts, int32_t top_k, float routed_scale,
                                  int32_t* ids, float* weights, void* stream);
/* ---------------------------------------------------------------- activation files */

/* GLM5XACT BF16 activation batches, the reference's hidden-state hand-off
 * between its Python layer and C++ runtime (load_glm5x_bf16_activation,
 * runtime/src/glm5x_activation.cpp:53-109; write_bf16_activation,
 * converter/glm5x_converter/activation.py:21-57): a 40-byte header
 * "<8sIIIIHHQI" = ("GLM5XACT", 1, 40, tokens, hidden, 3 = BF16, 0, payload
 * bytes, CRC32C) then BF16 [tokens, hidden]. Reading with out = NULL checks
 * the header and file size and returns the extents; with a buffer of
 * out_elems >= tokens * hidden values it also reads the payload and checks
 * its CRC. Non-zero expected_* must match. Status codes are the reference's:
 * IO_ERROR, TRUNCATED_FILE, BAD_MAGIC, UNSUPPORTED_VERSION, INVALID_EXTENT,
 * DATA_CRC_MISMATCH. Host memory only. */
glm5x_status glm5x_read_bf16_activation(const char* path, uint32_t expected_tokens,
                                        uint32_t expected_hidden, uint32_t* tokens,
                                        uint32_t* hidden, uint16_t* out, uint64_t out_elems);
/* Writes [tokens, hidden] BF16 values as a GLM5XACT file (beside the path,
 * then renamed over it). */
glm5x_status glm5x_write_bf16_activation(const char* path, const uint16_t* data,
                                         uint32_t tokens, uint32_t hidden);

/* ---------------------------------------------------------------- routing policy */

/* k3x::RoutingMode / RoutingPolicyConfig (runtime/include/k3x/
 * routing_policy.hpp:11-19). fixed: fixed_k of the ladder 4/6/8/12/16 (<= the
 * natural top-k); adaptive (natural top-k 16): the smallest ladder K whose
 * natural probability mass reaches mass_target, that covers the entropy's
 * effective support and whose boundary gap reaches minimum_boundary_gap
 * (routing_policy.cpp:111-135); quality_floor_k raises fixed / adaptive K.
 * Slots past a token's selected K hold id -1 and weight 0, and the selected
 * weights are renormalized over the selected scores. collect_diagnostics keeps
 * the per-token decision scalars in natural mode as well (the other modes
 * always keep them). */
typedef enum glm5x_routing_mode {
  GLM5X_ROUTING_NATURAL = 0,
  GLM5X_ROUTING_FIXED = 1,
  GLM5X_ROUTING_ADAPTIVE = 2,
} glm5x_routing_mode;

typedef struct glm5x_routing_policy {
  int32_t mode;                 /* glm5x_routing_mode */
  int32_t fixed_k;
  float mass_target;            /* (0, 1]; the reference's default is 0.9 */
  float minimum_boundary_gap;   /* [0, 1] */
  int32_t quality_floor_k;      /* 0 or a ladder K */
  int32_t collect_diagnostics;
} glm5x_routing_policy;

/* Routing counters of the last router pass with diagnostics, as the
 * reference's session exports them (runtime/src/model.cpp:102-113). */
typedef struct glm5x_routing_stats {
  uint64_t decisions;
  uint64_t selected_experts;
  uint64_t quality_escalated_decisions;
  double normalized_entropy_sum;
  double selected_mass_sum;
  double boundary_confidence_sum;
} glm5x_routing_stats;

/* Validates like select_routing (GLM5X_INVALID_STATE with the reference's
 * message for an invalid threshold, floor, fixed K or adaptive without a
 * natural Top-16) and applies to later forwards and glm5x_moe_route. */
glm5x_status glm5x_moe_set_routing_policy(glm5x_moe* moe, const glm5x_routing_policy* policy);
/* Sums of the last router pass's per-token decisions (synchronizes). */
glm5x_status glm5x_moe_routing_stats(glm5x_moe* moe, glm5x_routing_stats* out);
/* Per-token decisions of the last router pass over `tokens` tokens, host
 * buffers (either may be NULL): sel [tokens, 2] = selected K, quality-floor
 * escalated; diag [tokens, 4] = normalized entropy, entropy effective support,
 * selected cumulative mass, boundary confidence. Synchronizes. */
glm5x_status glm5x_moe_routing_decisions(glm5x_moe* moe, int64_t tokens, int32_t* sel,
                                         float* diag);
/* select_routing with a policy over given sigmoid scores for T tokens at once
 * (device buffers): ids / weights [T, natural_top_k] (weights times
 * routed_scale), sel [T, 2] and diag [T, 4] as above (either may be NULL).
 * Synchronizes; invalid scores (outside [0, 1] or non-finite) and a zero
 * selected mass are GLM5X_INVALID_STATE as in the reference. */
glm5x_status glm5x_select_routing_policy(const float* scores, const float* bias, int64_t tokens,
                                         int32_t num_experts, int32_t natural_top_k,
                                         const glm5x_routing_policy* policy, float routed_scale,
                                         int32_t* ids, float* weights, int32_t* sel,
                                         float* diag, void* stream);

/* Greedy verification of speculative draft blocks for S sequences at once
 * (verify_greedy_target_block, runtime/src/speculative.cpp:75-113): sequence
 * s proposed draft_counts[s] <= max_draft_tokens candidates after
 * anchors[s], and targets[s, 0 .. n] are the target's argmax tokens after the
 * anchor and after each candidate (one expert-major block per sequence, as
 * runtime/src/model.cpp:1640-1690 runs them). Outputs: accepted[s] = the
 * length of the matching prefix, committed[s, 0 .. accepted[s]] = the
 * accepted candidates then the first mismatching (or bonus) target token,
 * status[s] = 0, GLM5X_INVALID_EXTENT (anchor or candidate outside the
 * vocabulary, n outside [0, max]) or GLM5X_INVALID_STATE (a target token
 * outside the vocabulary), as the reference returns them per sequence.
 * Device buffers: candidates [S, max], targets / committed [S, max + 1].
 * Asynchronous on `stream`. */
glm5x_status glm5x_verify_greedy_target_blocks(const uint32_t* anchors, const uint32_t* candidates,
                                               const int32_t* draft_counts,
                                               const uint32_t* targets, int64_t sequences,
                                               int32_t max_draft_tokens, uint32_t vocabulary_size,
                                               int32_t* accepted, uint32_t* committed,
                                               int32_t* status, void* stream);

/* out[t] (+)= sum over s < slots of rows[pos[t, s]] (BF16 rows, FP32 sums in
 * slot order; pos < 0 = absent), device buffers: the weighted scatter of
 * scatter_expert_major_outputs (runtime/src/expert_major.cpp:148-196) /
 * index_add_ (layer10_moe.py:843-846) in gather form with a fixed order. The
 * expert-parallel layer adds each token's per-rank partial sums with it. */
glm5x_status glm5x_combine_rows(const void* rows_bf16, const int32_t* pos, int64_t tokens,
                                int32_t slots, int64_t hidden, float* out, int32_t accumulate,
                                void* stream);
/* The device expert-major permutation (build_expert_major_plan,
 * runtime/src/expert_major.cpp:12-98): ids [T,k] -> seg_count [E],
 * seg_start [E+1] (128-aligned), pos [T,k], row_token [rows]. */
glm5x_status glm5x_expert_major_plan(const int32_t* ids, int64_t tokens, int32_t top_k,
                                     int32_t num_experts, int32_t* seg_count,
                                     int32_t* seg_start, int32_t* pos, int32_t* row_token,
                                     void* stream);

/* Same plan as glm5x_expert_major_plan, for callers that cannot allocate
 * device memory (an allocator-owning host framework, a process at its memory
 * cap, or a serving loop that cannot take cudaFree's device-wide
 * synchronization). No counterpart in the reference: its planner runs on
 * the host. Scratch is a fixed __device__ array (about 1 MB per GPU, held
 * until exit); tokens <= 8192 and tokens * top_k <= 65536, else
 * GLM5X_INVALID_EXTENT. The first call on a device looks the array up
 * (make it before capturing a stream there); calls whose GPU work overlaps
 * share the array and race. Synchronizes `stream` to report errors. */
glm5x_status glm5x_expert_major_plan_noalloc(const int32_t* ids, int64_t tokens, int32_t top_k,
                                             int32_t num_experts, int32_t* seg_count,
                                             int32_t* seg_start, int32_t* pos,
                                             int32_t* row_token, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* GLM5X_MOE_H_ */
