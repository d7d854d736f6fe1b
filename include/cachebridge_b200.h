/*
 * cachebridge_b200 — C ABI of the B200 (sm_100a) CacheBridge handoff hot path.
 *
 * The reference implements this path in PyTorch (src/cachebridge/mapper.py,
 * src/cachebridge/online/blocks.py and the SGLang runtime adapters). Every
 * entry point below replaces one reference interface; the comment above each
 * declaration names the reference file:line it stands in for.
 *
 * Conventions
 *  - All pointers to tensor data are DEVICE pointers owned by the caller,
 *    except where a parameter is documented as a host array.
 *  - Calls that launch work are asynchronous on the caller's CUDA stream
 *    (`stream` is a cudaStream_t passed as void*; NULL = legacy default stream).
 *  - Return value: CB_OK (0) or a negative CB_ERR_* code. No call throws across
 *    the ABI. cb_last_error() returns a thread-local message for the last
 *    failure on the calling thread.
 *  - Hot-path calls (cb_map_install, cb_derotate_keys, cb_map_install_packed,
 *    cb_pack_rows, cb_install_rows, cb_rope_table) never allocate device or
 *    host memory. cb_mapper_create is
 *    the only allocating call besides the IPC helpers.
 *  - Rows and blocks may live on another GPU of the process (for example a
 *    target pool opened through CUDA IPC). The first call that meets such a
 *    pointer enables peer access from the launching device to its owner, or
 *    fails with CB_ERR_UNSUPPORTED when the two devices cannot reach each
 *    other; kernels then load and store peer memory directly over NVLink.
 *  - Row indices (slots) are validated on the device: an index outside
 *    [0, rows) is skipped and CB_DEV_ERR_SLOT_RANGE is OR-ed into the caller's
 *    device status word, which the caller reads after the stream completes.
 *
 * Data model
 *  A "row set" (cb_rows) is a per-layer array of row-addressed buffers, which
 *  is exactly an SGLang MHATokenToKVPool (k_buffer[l] / v_buffer[l] with rows
 *  of [heads, head_dim]) or a dense page [2, layers, tokens, heads, head_dim]
 *  seen as per-layer pointers with slot = token.
 */
#ifndef CACHEBRIDGE_B200_H
#define CACHEBRIDGE_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Host status codes. */
#define CB_OK 0
#define CB_ERR_INVALID -1     /* bad geometry, pointer alignment or argument */
#define CB_ERR_UNSUPPORTED -2 /* valid request outside what this build supports */
#define CB_ERR_CUDA -3        /* a CUDA runtime call failed */
#define CB_ERR_ALIAS -4       /* destination rows alias (install) */

/*
 * Device status bits, OR-ed into the caller's int32 status word. Once
 * CB_DEV_ERR_TIMEOUT is set in a status word, the map, pack and install
 * kernels given that word do nothing (a chunk whose receive slot never filled
 * is neither mapped nor installed, and the chunks queued after it are skipped)
 * until the caller reads and clears the word. Rows those kernels would have
 * written keep whatever they held; after a failed publication vote they are
 * undefined until the caller frees or rewrites them.
 */
#define CB_DEV_ERR_SLOT_RANGE 1 /* a source or destination slot was outside [0, rows) */
#define CB_DEV_ERR_TIMEOUT 2    /* a bounded pipeline wait inside a kernel expired */

/* Storage dtypes. */
#define CB_DTYPE_F32 0
#define CB_DTYPE_BF16 1

/* Slot index dtypes (0 = no index array: row t of the set is row t). */
#define CB_INDEX_NONE 0
#define CB_INDEX_I32 32
#define CB_INDEX_I64 64

/* Maximum layers in one row set (kernel parameter arrays are sized by it). */
#define CB_MAX_LAYERS 128

typedef struct cb_rows {
  int32_t layers;          /* number of per-layer buffers */
  int32_t heads;           /* heads per row (row = heads * head_dim elements) */
  void* const* k;          /* HOST array [layers] of device pointers to K rows */
  void* const* v;          /* HOST array [layers] of device pointers to V rows */
  int64_t row_stride;      /* elements between consecutive rows */
  int64_t rows;            /* addressable rows per layer (bound for slots) */
  int32_t head_offset;     /* head index inside a row of this call's head 0 */
  int32_t slot_dtype;      /* CB_INDEX_* */
  const void* slots;       /* device [n_tokens] row indices, or NULL */
} cb_rows;

/*
 * Split-half (Qwen) RoPE of one model. Token t of a call sits at absolute
 * position position_start + t; frequency i < half_dim has the FP32 phase
 * float(position) * inv_freq[i] and the coefficients cos(phase) * magnitude,
 * sin(phase) * magnitude: the table of qwen_rope (src/cachebridge/rope.py:16-72),
 * whose cat(phase, phase) duplicate half is implied. inv_freq and magnitude
 * (YaRN included, rope.py:28-69) are computed by the caller; the kernels
 * evaluate the coefficients themselves, so no table crosses the ABI.
 */
typedef struct cb_rope {
  int32_t half_dim;      /* head_dim / 2, at most 128 */
  float magnitude;       /* YaRN attention magnitude, 1.0 without scaling */
  float inv_freq[128];   /* first half_dim entries used */
} cb_rope;

typedef struct cb_mapper cb_mapper;

/* Library version (major*10000 + minor*100 + patch). */
CB_API int cb_version(void);
/* Human-readable text for a host status code. */
CB_API const char* cb_status_string(int status);
/* Thread-local message describing the last failing call on this thread. */
CB_API const char* cb_last_error(void);

/*
 * Upload one head-local (CacheBridge, "headwise") mapper for a target TP rank.
 * Replaces PageMapper.__init__ (src/cachebridge/mapper.py:35-110): the caller
 * has already loaded layer_NNN.safetensors and sliced its target heads
 * (mapper.py:75-107); this call takes the sliced FP32 tensors (host memory):
 *   selected [target_layers][num_selected] int64   (mapper.py:95)
 *   k_weight, v_weight [target_layers][heads][num_selected*head_dim][head_dim]
 *   k_bias,   v_bias   [target_layers][heads][head_dim]
 * Weights are kept on `device` in FP32 (generic kernel) and, for head_dim 128,
 * also as a BF16 tensor-core image (rounded to nearest even).
 */
CB_API int cb_mapper_create(cb_mapper** out, int device, int target_layers, int heads,
                     int head_dim, int num_selected, const int64_t* selected,
                     const float* k_weight, const float* k_bias,
                     const float* v_weight, const float* v_bias);
/*
 * Upload one dense ("nv_transfer") mapper for a target TP rank. Replaces
 * PageMapper.__init__ for non-headwise layer files (src/cachebridge/mapper.py:59-110
 * with the dense branch of map_page, mapper.py:182-203): every target head
 * reads all source_heads heads of each selected source layer.
 *   selected [target_layers][num_selected] int64
 *   k_weight, v_weight [target_layers][num_selected*source_heads*head_dim][target_heads][head_dim]
 *     (the reference's k_weight[:, head_slice])
 *   k_bias, v_bias [target_layers][target_heads][head_dim]
 * head_dim must be 128 and num_selected*source_heads at most 64; the map runs
 * on the tensor-core path only (BF16 storage). cb_map_install then reads
 * source heads src->head_offset .. +source_heads of every source row.
 */
CB_API int cb_mapper_create_dense(cb_mapper** out, int device, int target_layers, int target_heads,
                                  int source_heads, int head_dim, int num_selected,
                                  const int64_t* selected, const float* k_weight, const float* k_bias,
                                  const float* v_weight, const float* v_bias);
/* Free a mapper and its device memory. */
CB_API int cb_mapper_destroy(cb_mapper* mapper);
/* Geometry of an uploaded mapper (any output pointer may be NULL). */
CB_API int cb_mapper_info(const cb_mapper* mapper, int* target_layers, int* heads,
                   int* head_dim, int* num_selected, int* used_source_layers);
/*
 * Which kernel a map + install call with these arguments runs; no
 * counterpart in the reference (an introspection helper for callers and
 * benchmarks). Returns CB_PATH_CUDA_CORE (FP32 storage or head_dim != 128),
 * CB_PATH_TENSOR_CORE (map_install_tc_kernel: more than four 128-feature
 * blocks per head, a caller token order, or target-RoPE phases beyond 4e5)
 * or CB_PATH_TENSOR_MEMORY (map_install_tm_kernel: weights in tensor
 * memory), or a negative status.
 */
#define CB_PATH_CUDA_CORE 0
#define CB_PATH_TENSOR_CORE 1
#define CB_PATH_TENSOR_MEMORY 2
CB_API int cb_mapper_path(const cb_mapper* mapper, int dtype, int64_t n_tokens, int64_t position_start,
                          const cb_rope* dst_rope, int has_token_order);

/*
 * Bytes of caller-provided scratch that cb_map_install needs for n_tokens
 * tokens of `dtype` storage (0 when the call needs none).
 */
CB_API size_t cb_mapper_workspace_bytes(const cb_mapper* mapper, int dtype,
                                 int64_t n_tokens);

/*
 * RoPE coefficient tables (a utility; the handoff kernels do not need them):
 * for i < rope->half_dim and t < n,
 *   out_cos[i * out_stride + t] = cos(float(position_start + t) * inv_freq[i]) * magnitude
 * and out_sin likewise, out_stride >= n (frequency-major). Equals
 * qwen_rope (src/cachebridge/rope.py:16-72) transposed, without its
 * duplicated second half.
 */
CB_API int cb_rope_table(void* stream, const cb_rope* rope, int64_t position_start,
                  int64_t n, float* out_cos, float* out_sin, int64_t out_stride);

/*
 * Fused pack + mapper apply + install for n_tokens tokens.
 * Replaces, in one call, pack_source_block (src/cachebridge/online/blocks.py:47-82),
 * PageMapper.map_page headwise branch (src/cachebridge/mapper.py:116-181, 207-239;
 * head narrowing src/cachebridge/online/mapping.py:7-33) and the install
 * (blocks.py:86-111 map_write_block / set_kv_buffer, and
 * backends/sglang/runtime/source_mapper_adapter.py:389-425 _DirectMappedPoolCodec.copy).
 *   src: source rows, src->layers >= 1 + max(selected); token t reads row
 *        src->slots[t]; target head h reads source head src->head_offset + h.
 *   dst: target rows, dst->layers == target_layers; token t of target head h
 *        is written to row dst->slots[t], head dst->head_offset + h. dst
 *        pointers may be peer-device pointers (CUDA IPC / peer access).
 *   position_start: absolute position of token 0 of this call (token t is at
 *        position_start + t, mapper.py:131-136).
 *   src_rope, dst_rope: source and target model RoPE (mapper.py:137-142,
 *        209-214).
 *   dtype: storage dtype of src and dst rows (CB_DTYPE_BF16 or CB_DTYPE_F32).
 *   workspace: >= cb_mapper_workspace_bytes(mapper, dtype, n_tokens) bytes.
 *   token_order: NULL, or a device int32 array [n_tokens] holding a
 *        permutation of 0..n_tokens-1: the order in which the tensor-core path
 *        processes the tokens (128 per tile). Results do not depend on it.
 *        An order that sorts dst->slots makes each tile's stores land in a few
 *        memory pages. Entries outside [0, n_tokens) are skipped and flag
 *        CB_DEV_ERR_SLOT_RANGE.
 *   dev_status: device int32 status word (CB_DEV_ERR_* bits are OR-ed in).
 * Compute: keys have the source RoPE removed in FP32, features of the S
 * selected source layers are concatenated, y = x W + b is accumulated in FP32,
 * target RoPE is applied to keys in FP32, and the result is rounded to the
 * storage dtype. BF16 rows with head_dim 128 run on tcgen05 tensor cores
 * (BF16 operands, FP32 accumulation); other geometries on a CUDA-core kernel.
 */
CB_API int cb_map_install(cb_mapper* mapper, void* stream, const cb_rows* src,
                   const cb_rows* dst, int64_t n_tokens, int64_t position_start,
                   const cb_rope* src_rope, const cb_rope* dst_rope, int dtype, void* workspace,
                   size_t workspace_bytes, const int32_t* token_order, int32_t* dev_status);

/*
 * cb_map_install without a caller workspace; no counterpart in the reference.
 * For callers that cannot allocate device memory when a handoff runs: a
 * serving engine whose KV pool was sized at start-up to fill the GPU, or an
 * FFI host that holds raw device pointers but no device allocator. The key
 * workspace is instead a fixed array of CB_NOALLOC_SCRATCH_BYTES (64 MiB) per
 * device inside this library, so one call maps at most
 * CB_NOALLOC_SCRATCH_BYTES / cb_mapper_workspace_bytes(mapper, dtype, 1)
 * tokens; a larger n_tokens is rejected with CB_ERR_UNSUPPORTED before any
 * work is queued. The call itself allocates nothing (no cudaMalloc, cudaFree
 * or allocating library routine). Its first call on a device performs a
 * one-time set-up (cudaGetSymbolAddress of the array, which can make CUDA
 * load this library's device code on that device); make that first call
 * before any stream capture. Every call on a device shares the one array:
 * calls whose GPU work can overlap (streams not ordered with one another,
 * concurrent host threads) race on it and must be serialised by the caller.
 * Nothing in the array needs to start at zero. The array is part of the
 * library's device code: every device on which that code is loaded (with
 * CUDA's eager module loading, every device the process uses with this
 * library loaded) holds the 64 MiB until the process exits, whether or not
 * this entry point is ever called. Arguments and results are those of
 * cb_map_install with token_order NULL.
 */
#define CB_NOALLOC_SCRATCH_BYTES (64 << 20)
CB_API int cb_map_install_noalloc(cb_mapper* mapper, void* stream, const cb_rows* src,
                           const cb_rows* dst, int64_t n_tokens, int64_t position_start,
                           const cb_rope* src_rope, const cb_rope* dst_rope, int dtype,
                           int32_t* dev_status);

/*
 * The two phases of cb_map_install's tensor-core path as separate calls
 * (head_dim 128, BF16 storage only), mirroring the reference's pack -> map
 * split (online/blocks.py:47-82 then mapper.py:116-239):
 *  cb_derotate_keys: gather the source key rows of every used source layer
 *    through src->slots, remove the source RoPE in FP32 (rope.py:82-89,
 *    mapper.py:143-144) and store BF16 content-space keys in `workspace`
 *    ([used_layers][n_tokens][heads][128]).
 *  cb_map_install_packed: map keys from `workspace` and values from the
 *    source rows, add the bias, apply the target RoPE and install into dst rows.
 * cb_map_install(...) == cb_derotate_keys(...) then cb_map_install_packed(...)
 * on the same stream, with the same workspace, position_start and token_order
 * (the workspace holds the keys in processing order).
 */
CB_API int cb_derotate_keys(cb_mapper* mapper, void* stream, const cb_rows* src,
                     int64_t n_tokens, int64_t position_start, const cb_rope* src_rope,
                     void* workspace, size_t workspace_bytes, const int32_t* token_order,
                     int32_t* dev_status);
CB_API int cb_map_install_packed(cb_mapper* mapper, void* stream, const cb_rows* src,
                          const cb_rows* dst, int64_t n_tokens, int64_t position_start,
                          const cb_rope* dst_rope, const void* workspace,
                          size_t workspace_bytes, const int32_t* token_order, int32_t* dev_status);

/*
 * Row gather: out[kind][l][t][:] = src.{k,v}[l][src.slots[t]][row] for all
 * src.layers layers, kinds K then V; `row` = src.heads*head_dim elements
 * starting at head src.head_offset. out is a dense device buffer
 * [2][layers][n_tokens][heads*head_dim].
 * Replaces pack_source_block (src/cachebridge/online/blocks.py:47-82).
 */
CB_API int cb_pack_rows(void* stream, const cb_rows* src, int head_dim, int dtype,
                 int64_t n_tokens, void* out, int32_t* dev_status);

/*
 * Row scatter: dst.{k,v}[l][dst.slots[t]][row] = block[kind][l][t][:].
 * block is dense [2][layers][n_tokens][heads*head_dim] and may live on a peer
 * device. Replaces _DirectMappedPoolCodec.copy
 * (backends/sglang/runtime/source_mapper_adapter.py:389-425) and the
 * cudaMemcpyPeerAsync span loop (backends/sglang/runtime/peer_adapter.py:211-282,
 * peer_runtime.py:55-64) with one launch.
 */
CB_API int cb_install_rows(void* stream, const void* block, const cb_rows* dst,
                    int head_dim, int dtype, int64_t n_tokens,
                    int32_t* dev_status);

/*
 * CUDA IPC helpers for the tensor-parallel transfer. They stand in for torch's
 * reduce_tensor / rebuild_cuda_tensor used by
 * backends/sglang/runtime/bounded_handoff_channel.py:83-123, with one
 * difference that matters for kernels: the importer maps the allocation into
 * the context of the device that will access it (`device`), with lazy peer
 * access, so a kernel on that device can store into it directly.
 *  cb_ipc_export: 64-byte handle of the allocation holding device_ptr, and
 *    the byte offset of device_ptr inside it.
 *  cb_ipc_open: map a peer allocation on `device`; *ptr_out is its base (add
 *    the exporter's offset).
 *  cb_ipc_close: unmap a base returned by cb_ipc_open.
 */
CB_API int cb_ipc_export(const void* device_ptr, void* handle_out /* 64 bytes */, uint64_t* offset_out);
CB_API int cb_ipc_open(const void* handle /* 64 bytes */, int device, void** ptr_out);
CB_API int cb_ipc_close(void* ptr);
/*
 * One asynchronous copy of `bytes` contiguous bytes on `stream` (the copy
 * engines; either side may be a peer device's memory, with peer access
 * enabled first). Replaces the ctypes cudaMemcpyPeerAsync of
 * backends/sglang/runtime/peer_runtime.py:34-64 for whole packed chunks.
 */
CB_API int cb_copy_async(void* stream, void* dst, const void* src, size_t bytes);

/*
 * Device-side chunk handshake between two GPUs (the double-buffered
 * source -> target pipeline). Both launch one thread on the caller's stream
 * on the current device; `flag` is an 8-byte aligned int64 counter in device
 * memory, local or a peer's mapped through cb_ipc_open.
 *  cb_chunk_signal: after all earlier work on `stream`, store `value` into
 *    *flag with release semantics at system scope.
 *  cb_chunk_wait: later work on `stream` starts once *flag >= value
 *    (acquire, system scope). The wait gives up after timeout_ns, ORs
 *    CB_DEV_ERR_TIMEOUT into *dev_status and lets the stream continue.
 * They replace the per-block ready / acknowledge messages of
 * backends/sglang/runtime/source_mapper_adapter.py:197-232 (_DoubleBufferedSender.offer)
 * and :282-324 (_DoubleBufferedReceiver.next / acknowledge).
 */
CB_API int cb_chunk_signal(void* stream, int64_t* flag, int64_t value);
CB_API int cb_chunk_wait(void* stream, const int64_t* flag, int64_t value, int64_t timeout_ns,
                         int32_t* dev_status);

/* Enable direct peer access from `device` to `peer` (idempotent). */
CB_API int cb_enable_peer_access(int device, int peer);

#ifdef __cplusplus
}
#endif

#endif /* CACHEBRIDGE_B200_H */
