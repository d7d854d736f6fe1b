// Host implementation of the C ABI declared in include/cachebridge_b200.h.
//
// Validates every request on the host (geometry, alignment, layer counts),
// packs kernel parameter blocks and launches on the caller's stream. Hot-path
// entry points allocate nothing; cb_mapper_create owns all device memory of a
// mapper. Errors are reported by status code plus a thread-local message.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/cachebridge_b200.h"
#include "cb_kernels.cuh"
#include "cb_map_tc.cuh"
#include "cb_map_tm.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(CB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return static_cast<uint16_t>((u >> 16) | 0x40);
  const uint32_t rounding = 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>((u + rounding) >> 16);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Rows or blocks may live on another GPU (a target pool opened through CUDA
// IPC, a peer staging block). Kernels on `device` can only touch them once
// peer access device -> owner is enabled, so every launch that takes such a
// pointer enables it first (once per device pair) or refuses the call.
constexpr int kMaxPeerDevices = 64;
std::mutex g_peer_mu;
bool g_peer_on[kMaxPeerDevices][kMaxPeerDevices] = {};

int ensure_access(int device, const void* ptr, const char* what) {
  cudaPointerAttributes a{};
  cudaError_t e = cudaPointerGetAttributes(&a, ptr);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(CB_ERR_INVALID, std::string(what) + ": not a CUDA pointer");
  }
  if (a.type == cudaMemoryTypeManaged) return CB_OK;
  if (a.type != cudaMemoryTypeDevice) return fail(CB_ERR_INVALID, std::string(what) + ": must be device memory");
  if (a.device == device) return CB_OK;
  if (device < 0 || device >= kMaxPeerDevices || a.device < 0 || a.device >= kMaxPeerDevices)
    return fail(CB_ERR_UNSUPPORTED, std::string(what) + ": device index beyond the 64 this build tracks");
  std::lock_guard<std::mutex> lock(g_peer_mu);
  if (g_peer_on[device][a.device]) return CB_OK;
  int can = 0;
  e = cudaDeviceCanAccessPeer(&can, device, a.device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
  if (!can)
    return fail(CB_ERR_UNSUPPORTED, std::string(what) + ": lives on device " + std::to_string(a.device) +
                                        ", which device " + std::to_string(device) + " cannot access");
  DeviceGuard guard(device);
  if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  e = cudaDeviceEnablePeerAccess(a.device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
  } else if (e != cudaSuccess) {
    return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  }
  g_peer_on[device][a.device] = true;
  return CB_OK;
}

// Peer access for the first K and V buffers of a row set (the layers of one
// row set share a device).
// True when the row set's buffers are memory of `device` itself rather than a
// peer GPU's mapping. A row set's layers share one device (the same rule as
// ensure_rows_access), so layer 0's K and V buffers decide.
bool rows_on_device(int device, const cb_rows* r) {
  for (const void* ptr : {static_cast<const void*>(r->k[0]), static_cast<const void*>(r->v[0])}) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (a.type != cudaMemoryTypeDevice || a.device != device) return false;
  }
  return true;
}

int ensure_rows_access(int device, const cb_rows* r, const char* what) {
  int rc = ensure_access(device, r->k[0], what);
  if (rc != CB_OK) return rc;
  return ensure_access(device, r->v[0], what);
}

int elem_size(int dtype) { return dtype == CB_DTYPE_F32 ? 4 : 2; }

int check_rows(const cb_rows* r, const char* name, int head_dim, int heads_used, int dtype,
               bool need_16b) {
  if (r == nullptr) return fail(CB_ERR_INVALID, std::string(name) + ": null row set");
  if (r->layers <= 0 || r->layers > CB_MAX_LAYERS)
    return fail(CB_ERR_UNSUPPORTED, std::string(name) + ": layers must be in [1, 128]");
  if (r->k == nullptr || r->v == nullptr) return fail(CB_ERR_INVALID, std::string(name) + ": null layer arrays");
  if (r->heads <= 0 || r->head_offset < 0 || r->head_offset + heads_used > r->heads)
    return fail(CB_ERR_INVALID, std::string(name) + ": head range outside the row");
  if (r->row_stride < static_cast<int64_t>(r->heads) * head_dim)
    return fail(CB_ERR_INVALID, std::string(name) + ": row_stride smaller than a row");
  if (r->rows <= 0) return fail(CB_ERR_INVALID, std::string(name) + ": rows must be positive");
  if (r->slot_dtype != CB_INDEX_NONE && r->slot_dtype != CB_INDEX_I32 && r->slot_dtype != CB_INDEX_I64)
    return fail(CB_ERR_INVALID, std::string(name) + ": unknown slot dtype");
  if (r->slot_dtype != CB_INDEX_NONE && r->slots == nullptr)
    return fail(CB_ERR_INVALID, std::string(name) + ": slot dtype given without slots");
  const int es = elem_size(dtype);
  for (int l = 0; l < r->layers; ++l) {
    if (r->k[l] == nullptr || r->v[l] == nullptr)
      return fail(CB_ERR_INVALID, std::string(name) + ": null layer pointer");
    if (reinterpret_cast<uintptr_t>(r->k[l]) % es || reinterpret_cast<uintptr_t>(r->v[l]) % es)
      return fail(CB_ERR_INVALID, std::string(name) + ": layer pointer not element aligned");
    if (need_16b && (!aligned16(r->k[l]) || !aligned16(r->v[l])))
      return fail(CB_ERR_INVALID, std::string(name) + ": layer pointer not 16-byte aligned");
  }
  if (need_16b && (r->row_stride * es) % 16 != 0)
    return fail(CB_ERR_INVALID, std::string(name) + ": row stride not a multiple of 16 bytes");
  return CB_OK;
}

// cudaFuncSetAttribute result for the tensor-core kernels' shared-memory
// opt-in, per device: set once, and its result (success or the error) is
// returned to every later call on that device.
struct AttrOnce {
  std::once_flag once;
  cudaError_t result = cudaSuccess;
};
AttrOnce g_tc_attr[64];
AttrOnce g_tm_attr[64];

cudaError_t set_smem_attr_once(AttrOnce& a, const void* kernel) {
  std::call_once(a.once, [&] {
    a.result = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, cbk::kTcMaxSmem);
  });
  return a.result;
}

int check_rope(const cb_rope* r, int head_dim, const char* name) {
  if (r == nullptr) return fail(CB_ERR_INVALID, std::string(name) + ": null RoPE descriptor");
  if (r->half_dim * 2 != head_dim || r->half_dim > 128)
    return fail(CB_ERR_INVALID, std::string(name) + ": RoPE half_dim does not match head_dim");
  if (!std::isfinite(r->magnitude)) return fail(CB_ERR_INVALID, std::string(name) + ": non-finite RoPE magnitude");
  return CB_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (the
// library does not link libcuda directly).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

int encode_bf16_map(CUtensorMap* map, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
                    const cuuint32_t* box) {
  auto enc = tensor_map_encoder();
  if (enc == nullptr) return fail(CB_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box,
                   elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CB_ERR_INVALID, "cuTensorMapEncodeTiled rejected a map (error " + std::to_string(r) + ")");
  return CB_OK;
}

cbk::RopeDev rope_dev(const cb_rope* r) {
  cbk::RopeDev d{};
  std::memcpy(d.inv_freq, r->inv_freq, sizeof(float) * r->half_dim);
  d.magnitude = r->magnitude;
  d.half_dim = r->half_dim;
  return d;
}

}  // namespace

struct cb_mapper {
  int device = 0;
  int L_t = 0, H = 0, D = 0, S = 0, U = 0;
  // Dense (nv_transfer) mappers read every source head: Hs source heads per
  // selected layer feed each target head, so a unit has KB = S * Hs k-blocks.
  // Headwise mappers: Hs = 0 (target head h reads source head h), KB = S.
  int Hs = 0, KB = 0;
  int num_sms = 0;
  int max_sel = 0;
  std::vector<int> used;  // sorted unique selected source layers
  float* w32 = nullptr;   // [2][L_t][H][S*D][D]
  float* b32 = nullptr;   // [2][L_t][H][D]
  int* sel = nullptr;     // [L_t][S]
  int* sel_local = nullptr;
  int* used_dev = nullptr;
  uint8_t* w_img = nullptr;  // head_dim 128 only: [2][L_t][H][S][32 KB]
  // head_dim 128 and KB <= 4 only: per unit KB * 16 chunks x 128 lanes x 16 B,
  // the tensor-memory weight image of map_install_tm_kernel.
  uint8_t* w_tm = nullptr;
};

namespace {

int mapper_create(cb_mapper** out, int device, int target_layers, int heads, int head_dim, int num_selected,
                  const int64_t* selected, const float* k_weight, const float* k_bias, const float* v_weight,
                  const float* v_bias, int src_heads);
int check_tc_extras(const cb_mapper* m, int dtype, int64_t n_tokens, const void* workspace,
                    size_t workspace_bytes);

// Source heads a call reads per source layer (all of them for a dense mapper).
int ws_heads(const cb_mapper* m) { return m->Hs > 0 ? m->Hs : m->H; }

// Tensor-core workspace: BF16 content-space keys [U][n][ws_heads][128].
size_t ws_total_bytes(const cb_mapper* m, int64_t n) {
  return static_cast<size_t>(m->U) * static_cast<size_t>(n) * ws_heads(m) * cbk::kD * 2;
}

int launch_rope_table(cudaStream_t st, const cb_rope* rope, int64_t position_start, int64_t n, float* out_cos,
                      float* out_sin, int64_t out_stride);

int launch_derotate(const cb_mapper* m, cudaStream_t st, const cb_rows* src, int64_t n_tokens,
                    int64_t position_start, const cb_rope* src_rope, void* workspace, const int32_t* order,
                    int32_t* dev_status) {
  cbk::DerotateParams dp{};
  dp.n_tokens = n_tokens;
  dp.H = ws_heads(m);
  dp.U = m->U;
  for (int l = 0; l < src->layers; ++l) dp.src_k[l] = src->k[l];
  dp.used = m->used_dev;
  dp.src_row_stride = src->row_stride;
  dp.src_rows = src->rows;
  dp.src_head_offset = src->head_offset;
  dp.src_slot_dtype = src->slot_dtype;
  dp.src_slots = src->slots;
  dp.rope = rope_dev(src_rope);
  dp.position_start = position_start;
  dp.order = order;
  dp.ws = static_cast<__nv_bfloat16*>(workspace);
  dp.status = dev_status;
  // Small calls: split each token's U*H rows over several warps, as far as
  // the grid still fits one resident wave (3 blocks of 8 warps per SM); a
  // split that spills into a second, nearly empty wave is slower than none
  // (2048 tokens x 8 heads in 2 parts: 66 -> 81 us). Calls of at least one
  // wave of tokens keep one warp per token.
  const int total_rows = dp.U * dp.H;
  const int max_parts = (total_rows + 15) / 16;
  const int64_t wave_warps = 24ll * (m->num_sms > 0 ? m->num_sms : 148);
  const int parts = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(max_parts, wave_warps / std::max<int64_t>(n_tokens, 1))));
  dp.rows_per_part = ((total_rows + parts - 1) / parts + 15) / 16 * 16;
  dp.parts = (total_rows + dp.rows_per_part - 1) / dp.rows_per_part;
  const int blocks = static_cast<int>((n_tokens * dp.parts + 7) / 8);
  cbk::derotate_pack_kernel<<<blocks, 256, 0, st>>>(dp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "derotate_pack launch");
  return CB_OK;
}

// True when a target-RoPE phase of the call can reach 4e5 rad, beyond the
// reduced-range trigonometry of the tensor-core epilogues.
bool needs_exact_trig(const cb_rope* dst_rope, int64_t position_start, int64_t n_tokens) {
  float max_inv = 0.f;
  for (int i = 0; i < dst_rope->half_dim; ++i) max_inv = std::max(max_inv, std::fabs(dst_rope->inv_freq[i]));
  return static_cast<double>(position_start + n_tokens) * max_inv > 4.0e5;
}

// M-tiles per work item of the tensor-core kernel. An item is one (target
// layer, head, kind) over a run of R m-tiles; its weights and bias are loaded
// into shared memory once, and the MMA pipeline drains at each item boundary
// while the next item's weights arrive (about five m-tiles of tensor time).
// Items are spread round-robin over the persistent CTAs, so the busiest CTA
// runs ceil(items / grid) of them: pick the R that minimises
// ceil(items / grid) * (R + 5). Runs are capped at kMaxRunMtiles: the CTAs
// that read the same source rows (the ~L_t*S/U target layers selecting a
// source layer) then stay within one 1024-token window, so a row's later
// readers find it in L2. Measured at the 8192-token Qwen3 shapes: runs of 64
// / 32 / 16 / 8 m-tiles take 1.099 / 1.089 / 1.077 / 1.070 ms.
// The tensor-memory kernel with a single weight buffer (S >= 3) reloads its
// weights between items with the MMA stalled, and those reloads are about a
// tenth of its L2 -> shared-memory bytes: it takes runs of up to 32 m-tiles
// (one 16384-token config-4 request: 3.82 -> 3.43 ms; config 2, double
// buffered, unchanged at any cap).
constexpr int64_t kMaxRunMtiles = 8;
constexpr int64_t kMaxRunMtilesOneWeightBuffer = 32;

int tc_chunk_mtiles(int64_t n_tokens, int64_t groups, int grid, int64_t max_run = kMaxRunMtiles) {
  const int64_t mt = (n_tokens + cbk::kBM - 1) / cbk::kBM;
  int best_r = 1;
  int64_t best_cost = -1;
  for (int64_t r = 1; r <= mt && r <= max_run; ++r) {
    const int64_t items = groups * ((mt + r - 1) / r);
    const int64_t cost = ((items + grid - 1) / grid) * (r + 5);
    if (best_cost < 0 || cost <= best_cost) {
      best_cost = cost;
      best_r = static_cast<int>(r);
    }
  }
  return best_r;
}

int launch_tc(const cb_mapper* m, cudaStream_t st, const cb_rows* src, const cb_rows* dst,
              int64_t n_tokens, int64_t position_start, const cb_rope* dst_rope, const void* workspace,
              const int32_t* order, int32_t* dev_status) {
  cbk::MapTcParams p{};
  p.n_tokens = static_cast<int>(n_tokens);
  p.L_t = m->L_t;
  p.H = m->H;
  p.S = m->S;
  p.KB = m->KB;
  p.kb_heads = m->Hs > 0 ? m->Hs : 1;
  p.dense = m->Hs > 0 ? 1 : 0;
  p.ws_heads = ws_heads(m);
  p.R = tc_chunk_mtiles(n_tokens, 2ll * m->H * m->L_t, m->num_sms);
  p.n_chunks = static_cast<int>((n_tokens + p.R * cbk::kBM - 1) / (p.R * cbk::kBM));
  const int64_t items = 2ll * m->H * p.n_chunks * m->L_t;
  if (items > (int64_t(1) << 31) - 1) return fail(CB_ERR_UNSUPPORTED, "work too large for one call");
  p.num_items = static_cast<int>(items);
  // Weights stay resident for a whole item when they leave room for >= 2 A
  // stages; otherwise two weight slots are streamed per m-tile.
  const int res_stages = (cbk::kTcMaxSmem - cbk::tc_smem_bytes(m->KB, 0)) / cbk::kKBlockBytes;
  p.w_resident = (m->KB <= 4 && res_stages >= 2) ? 1 : 0;
  p.w_slots = p.w_resident ? m->KB : 2;
  const int stages = (cbk::kTcMaxSmem - cbk::tc_smem_bytes(p.w_slots, 0)) / cbk::kKBlockBytes;
  p.stages = std::min(stages, 4);
  if (p.stages < 2) return fail(CB_ERR_UNSUPPORTED, "shared memory too small for the pipeline");
  p.w_img = m->w_img;
  p.unit_bytes = static_cast<int64_t>(m->KB) * cbk::kKBlockBytes + cbk::kBiasBlockBytes;
  p.sel_global = m->sel;
  p.sel_local = m->sel_local;
  p.ws_k = static_cast<const __nv_bfloat16*>(workspace);
  for (int l = 0; l < src->layers; ++l) p.src_v[l] = src->v[l];
  p.src_row_stride = src->row_stride;
  p.src_rows = src->rows;
  {
    const cuuint64_t kdims[4] = {128, static_cast<cuuint64_t>(ws_heads(m)), static_cast<cuuint64_t>(n_tokens),
                                 static_cast<cuuint64_t>(m->U)};
    const cuuint64_t kstr[3] = {256, static_cast<cuuint64_t>(ws_heads(m)) * 256,
                                static_cast<cuuint64_t>(n_tokens) * ws_heads(m) * 256};
    const cuuint32_t kbox[4] = {64, 1, 128, 1};
    int rc = encode_bf16_map(&p.kmap, 4, workspace, kdims, kstr, kbox);
    if (rc != CB_OK) return rc;
  }
  p.src_head_offset = src->head_offset;
  p.src_slot_dtype = src->slot_dtype;
  p.src_slots = src->slots;
  for (int l = 0; l < dst->layers; ++l) {
    p.dst_k[l] = dst->k[l];
    p.dst_v[l] = dst->v[l];
  }
  p.dst_row_stride = dst->row_stride;
  p.dst_rows = dst->rows;
  p.dst_head_offset = dst->head_offset;
  p.dst_slot_dtype = dst->slot_dtype;
  p.dst_slots = dst->slots;
  p.dst_evict_first = rows_on_device(m->device, dst) ? 1 : 0;
  std::memcpy(p.dst_inv_freq, dst_rope->inv_freq, sizeof(p.dst_inv_freq));
  p.dst_magnitude = dst_rope->magnitude;
  p.position_start = position_start;
  p.order = order;
  p.trig_exact = needs_exact_trig(dst_rope, position_start, n_tokens) ? 1 : 0;
  p.status = dev_status;
  const int smem = cbk::tc_smem_bytes(p.w_slots, p.stages);
  const cudaError_t attr_err =
      set_smem_attr_once(g_tc_attr[m->device & 63], reinterpret_cast<const void*>(cbk::map_install_tc_kernel));
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute");
  const int grid = static_cast<int>(std::min<int64_t>(items, m->num_sms));
  cbk::map_install_tc_kernel<<<grid, cbk::kTcThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "map_install_tc launch");
  return CB_OK;
}

// map_install_tm_kernel (weights in tensor memory) serves mappers of at most
// four 128-feature blocks per unit, tokens in call order and phases inside the
// reduced trigonometry range; map_install_tc_kernel takes every other call.
bool tm_eligible(const cb_mapper* m, const cb_rope* dst_rope, int64_t position_start, int64_t n_tokens,
                 const int32_t* order) {
  return m->w_tm != nullptr && m->KB <= cbk::kTmMaxKB && order == nullptr &&
         !needs_exact_trig(dst_rope, position_start, n_tokens);
}

int launch_tm(const cb_mapper* m, cudaStream_t st, const cb_rows* src, const cb_rows* dst, int64_t n_tokens,
              int64_t position_start, const cb_rope* dst_rope, const void* workspace, int32_t* dev_status) {
  cbk::MapTmParams p{};
  p.n_tokens = static_cast<int>(n_tokens);
  p.L_t = m->L_t;
  p.H = m->H;
  p.S = m->S;
  p.KB = m->KB;
  p.kb_heads = m->Hs > 0 ? m->Hs : 1;
  p.dense = m->Hs > 0 ? 1 : 0;
  // Two weight buffers when both fit beside the accumulators (S <= 2).
  p.w_bufs = (512 - cbk::kTmWeightCol0) / (64 * m->KB) >= 2 ? 2 : 1;
  p.R = tc_chunk_mtiles(n_tokens, 2ll * m->H * m->L_t, m->num_sms,
                        p.w_bufs == 1 ? kMaxRunMtilesOneWeightBuffer : kMaxRunMtiles);
  p.n_chunks = static_cast<int>((n_tokens + p.R * cbk::kBM - 1) / (p.R * cbk::kBM));
  const int64_t items = 2ll * m->H * p.n_chunks * m->L_t;
  if (items > (int64_t(1) << 31) - 1) return fail(CB_ERR_UNSUPPORTED, "work too large for one call");
  p.num_items = static_cast<int>(items);
  p.stages = std::min(8, (cbk::kTcMaxSmem - cbk::tm_smem_bytes(0)) / cbk::kKBlockBytes);
  if (p.stages < 2) return fail(CB_ERR_UNSUPPORTED, "shared memory too small for the pipeline");
  p.w_tm = m->w_tm;
  p.unit_bytes = static_cast<int64_t>(m->KB) * cbk::kKBlockBytes;
  p.bias = m->b32;
  p.sel_global = m->sel;
  p.sel_local = m->sel_local;
  for (int l = 0; l < src->layers; ++l) p.src_v[l] = src->v[l];
  p.src_row_stride = src->row_stride;
  p.src_rows = src->rows;
  p.src_head_offset = src->head_offset;
  p.src_slot_dtype = src->slot_dtype;
  p.src_slots = src->slots;
  {
    const cuuint64_t kdims[4] = {128, static_cast<cuuint64_t>(ws_heads(m)), static_cast<cuuint64_t>(n_tokens),
                                 static_cast<cuuint64_t>(m->U)};
    const cuuint64_t kstr[3] = {256, static_cast<cuuint64_t>(ws_heads(m)) * 256,
                                static_cast<cuuint64_t>(n_tokens) * ws_heads(m) * 256};
    const cuuint32_t kbox[4] = {64, 1, 128, 1};
    int rc = encode_bf16_map(&p.kmap, 4, workspace, kdims, kstr, kbox);
    if (rc != CB_OK) return rc;
  }
  for (int l = 0; l < dst->layers; ++l) {
    p.dst_k[l] = dst->k[l];
    p.dst_v[l] = dst->v[l];
  }
  p.dst_row_stride = dst->row_stride;
  p.dst_rows = dst->rows;
  p.dst_head_offset = dst->head_offset;
  p.dst_slot_dtype = dst->slot_dtype;
  p.dst_slots = dst->slots;
  p.dst_evict_first = rows_on_device(m->device, dst) ? 1 : 0;
  // 32-byte stores only into this GPU's own memory; rows of a peer's pool
  // (stores over NVLink) take 16-byte stores.
  p.dst_v8 = (p.dst_evict_first && (dst->row_stride * 2) % 32 == 0) ? 1 : 0;
  for (int l = 0; l < dst->layers && p.dst_v8; ++l)
    if (reinterpret_cast<uintptr_t>(dst->k[l]) % 32 || reinterpret_cast<uintptr_t>(dst->v[l]) % 32) p.dst_v8 = 0;
  for (int i = 0; i < 64; ++i) {
    const float inv = dst_rope->inv_freq[i];
    p.dst_inv_freq[i] = inv;
    // Unit rotations by one and by eight positions of the exact angle.
    p.rot1_c[i] = static_cast<float>(std::cos(static_cast<double>(inv)));
    p.rot1_s[i] = static_cast<float>(std::sin(static_cast<double>(inv)));
    p.rot8_c[i] = static_cast<float>(std::cos(8.0 * static_cast<double>(inv)));
    p.rot8_s[i] = static_cast<float>(std::sin(8.0 * static_cast<double>(inv)));
  }
  p.dst_magnitude = dst_rope->magnitude;
  p.position_start = position_start;
  p.order = nullptr;
  p.status = dev_status;
  const cudaError_t attr_err =
      set_smem_attr_once(g_tm_attr[m->device & 63], reinterpret_cast<const void*>(cbk::map_install_tm_kernel));
  if (attr_err != cudaSuccess) return cuda_fail(attr_err, "cudaFuncSetAttribute");
  const int grid = static_cast<int>(std::min<int64_t>(items, m->num_sms));
  cbk::map_install_tm_kernel<<<grid, cbk::kTmThreads, cbk::tm_smem_bytes(p.stages), st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "map_install_tm launch");
  return CB_OK;
}

// The tensor-core map + install phase: the transposed kernel where it
// applies, else the general one.
int launch_map(const cb_mapper* m, cudaStream_t st, const cb_rows* src, const cb_rows* dst, int64_t n_tokens,
               int64_t position_start, const cb_rope* dst_rope, const void* workspace, const int32_t* order,
               int32_t* dev_status) {
  if (tm_eligible(m, dst_rope, position_start, n_tokens, order))
    return launch_tm(m, st, src, dst, n_tokens, position_start, dst_rope, workspace, dev_status);
  return launch_tc(m, st, src, dst, n_tokens, position_start, dst_rope, workspace, order, dev_status);
}

int check_tc_extras(const cb_mapper* m, int dtype, int64_t n_tokens, const void* workspace,
                    size_t workspace_bytes) {
  const size_t need = ws_total_bytes(m, n_tokens);
  if (m->D != cbk::kD || dtype != CB_DTYPE_BF16)
    return fail(CB_ERR_UNSUPPORTED, "tensor-core path needs head_dim 128 and bf16 storage");
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(CB_ERR_INVALID, "workspace missing, too small or misaligned");
  return CB_OK;
}

// Shared validation of a tensor-core call's row sets.
int check_tc_call(const cb_mapper* m, const cb_rows* src, const cb_rows* dst, int64_t n_tokens) {
  if (m == nullptr) return fail(CB_ERR_INVALID, "null mapper");
  if (n_tokens < 0) return fail(CB_ERR_INVALID, "negative token count");
  if (n_tokens > (int64_t(1) << 31) - 1) return fail(CB_ERR_UNSUPPORTED, "too many tokens in one call");
  int rc = check_rows(src, "src", m->D, ws_heads(m), CB_DTYPE_BF16, true);
  if (rc != CB_OK) return rc;
  if (src->layers <= m->max_sel) return fail(CB_ERR_INVALID, "mapper selected layer exceeds source page depth");
  if (dst != nullptr) {
    if ((rc = check_rows(dst, "dst", m->D, m->H, CB_DTYPE_BF16, true)) != CB_OK) return rc;
    if (dst->layers != m->L_t) return fail(CB_ERR_INVALID, "destination layer count != mapper target layers");
  }
  return CB_OK;
}

int launch_rope_table(cudaStream_t st, const cb_rope* rope, int64_t position_start, int64_t n, float* out_cos,
                      float* out_sin, int64_t out_stride) {
  cbk::RopeTableParams p{};
  p.rope = rope_dev(rope);
  p.position_start = position_start;
  p.n = n;
  p.out_cos = out_cos;
  p.out_sin = out_sin;
  p.out_stride = out_stride;
  const int64_t total = n * rope->half_dim;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16));
  cbk::rope_table_kernel<<<blocks, 256, 0, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "rope_table launch");
  return CB_OK;
}

}  // namespace

extern "C" {

int cb_version(void) { return 100; }

const char* cb_status_string(int status) {
  switch (status) {
    case CB_OK: return "ok";
    case CB_ERR_INVALID: return "invalid argument or geometry";
    case CB_ERR_UNSUPPORTED: return "unsupported geometry";
    case CB_ERR_CUDA: return "CUDA runtime error";
    case CB_ERR_ALIAS: return "destination rows alias";
    default: return "unknown status";
  }
}

const char* cb_last_error(void) { return g_last_error.c_str(); }

int cb_mapper_create(cb_mapper** out, int device, int target_layers, int heads, int head_dim,
                     int num_selected, const int64_t* selected, const float* k_weight,
                     const float* k_bias, const float* v_weight, const float* v_bias) {
  return mapper_create(out, device, target_layers, heads, head_dim, num_selected, selected, k_weight, k_bias,
                       v_weight, v_bias, 0);
}

int cb_mapper_create_dense(cb_mapper** out, int device, int target_layers, int target_heads, int source_heads,
                           int head_dim, int num_selected, const int64_t* selected, const float* k_weight,
                           const float* k_bias, const float* v_weight, const float* v_bias) {
  if (out == nullptr) return fail(CB_ERR_INVALID, "null output handle");
  *out = nullptr;
  if (head_dim != cbk::kD) return fail(CB_ERR_UNSUPPORTED, "dense (nv_transfer) mappers need head_dim 128");
  if (source_heads <= 0 || target_heads <= 0 || num_selected <= 0 || target_layers <= 0)
    return fail(CB_ERR_INVALID, "dense mapper: counts must be positive");
  if (static_cast<int64_t>(num_selected) * source_heads > 64)
    return fail(CB_ERR_UNSUPPORTED, "dense mapper: at most 64 (selected layer, source head) feature blocks");
  if (!k_weight || !v_weight) return fail(CB_ERR_INVALID, "null mapper tensor");
  // [L_t][F][H][D] (F = S * Hs * D, the reference's k_weight[:, head_slice]) ->
  // [L_t][H][F][D]: per target head, the same shape as a headwise map.
  const int64_t F = static_cast<int64_t>(num_selected) * source_heads * head_dim;
  const size_t per_layer = static_cast<size_t>(F) * target_heads * head_dim;
  std::vector<float> kw(per_layer * target_layers), vw(per_layer * target_layers);
  for (int l = 0; l < target_layers; ++l)
    for (int64_t f = 0; f < F; ++f)
      for (int h = 0; h < target_heads; ++h) {
        const size_t from = l * per_layer + (static_cast<size_t>(f) * target_heads + h) * head_dim;
        const size_t to = l * per_layer + (static_cast<size_t>(h) * F + f) * head_dim;
        std::memcpy(&kw[to], k_weight + from, head_dim * sizeof(float));
        std::memcpy(&vw[to], v_weight + from, head_dim * sizeof(float));
      }
  return mapper_create(out, device, target_layers, target_heads, head_dim, num_selected, selected, kw.data(),
                       k_bias, vw.data(), v_bias, source_heads);
}

}  // extern "C"

namespace {

// Shared by the headwise and dense constructors: weights arrive per target
// head as [L_t][H][KB * D][D] (KB = S headwise, S * src_heads dense).
int mapper_create(cb_mapper** out, int device, int target_layers, int heads, int head_dim, int num_selected,
                  const int64_t* selected, const float* k_weight, const float* k_bias, const float* v_weight,
                  const float* v_bias, int src_heads) {
  if (out == nullptr) return fail(CB_ERR_INVALID, "null output handle");
  *out = nullptr;
  if (target_layers <= 0 || target_layers > CB_MAX_LAYERS)
    return fail(CB_ERR_UNSUPPORTED, "target_layers must be in [1, 128]");
  if (heads <= 0 || head_dim <= 0 || head_dim % 2 || head_dim > 256)
    return fail(CB_ERR_INVALID, "heads must be positive and head_dim even and <= 256");
  if (num_selected <= 0 || num_selected > 16) return fail(CB_ERR_UNSUPPORTED, "num_selected must be in [1, 16]");
  if (!selected || !k_weight || !k_bias || !v_weight || !v_bias)
    return fail(CB_ERR_INVALID, "null mapper tensor");
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return fail(CB_ERR_INVALID, "device index out of range");

  auto* m = new cb_mapper();
  m->device = device;
  m->L_t = target_layers;
  m->H = heads;
  m->D = head_dim;
  m->S = num_selected;
  m->Hs = src_heads;
  m->KB = num_selected * (src_heads > 0 ? src_heads : 1);
  std::vector<int> sel(static_cast<size_t>(target_layers) * num_selected);
  for (size_t i = 0; i < sel.size(); ++i) {
    if (selected[i] < 0 || selected[i] >= CB_MAX_LAYERS) {
      delete m;
      return fail(CB_ERR_INVALID, "selected source layer outside [0, 128)");
    }
    sel[i] = static_cast<int>(selected[i]);
    m->max_sel = std::max(m->max_sel, sel[i]);
  }
  m->used = sel;
  std::sort(m->used.begin(), m->used.end());
  m->used.erase(std::unique(m->used.begin(), m->used.end()), m->used.end());
  m->U = static_cast<int>(m->used.size());
  std::vector<int> sel_local(sel.size());
  for (size_t i = 0; i < sel.size(); ++i)
    sel_local[i] = static_cast<int>(std::lower_bound(m->used.begin(), m->used.end(), sel[i]) - m->used.begin());

  const int F = m->KB * head_dim;
  const size_t w_per_kind = static_cast<size_t>(target_layers) * heads * F * head_dim;
  const size_t b_per_kind = static_cast<size_t>(target_layers) * heads * head_dim;

  DeviceGuard guard(device);
  if (!guard.ok) {
    delete m;
    return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  }
  cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device);

  auto cleanup = [&](cudaError_t err, const char* what) {
    cb_mapper_destroy(m);
    return cuda_fail(err, what);
  };
  // FP32 weights feed the CUDA-core kernel, which is headwise only.
  const bool keep_f32 = src_heads == 0;
  if (keep_f32 && (e = cudaMalloc(&m->w32, 2 * w_per_kind * sizeof(float))) != cudaSuccess) return cleanup(e, "cudaMalloc w32");
  if ((e = cudaMalloc(&m->b32, 2 * b_per_kind * sizeof(float))) != cudaSuccess) return cleanup(e, "cudaMalloc b32");
  if ((e = cudaMalloc(&m->sel, sel.size() * sizeof(int))) != cudaSuccess) return cleanup(e, "cudaMalloc sel");
  if ((e = cudaMalloc(&m->sel_local, sel.size() * sizeof(int))) != cudaSuccess) return cleanup(e, "cudaMalloc sel_local");
  if ((e = cudaMalloc(&m->used_dev, m->used.size() * sizeof(int))) != cudaSuccess) return cleanup(e, "cudaMalloc used");
  if (keep_f32 && (e = cudaMemcpy(m->w32, k_weight, w_per_kind * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload k_weight");
  if (keep_f32 && (e = cudaMemcpy(m->w32 + w_per_kind, v_weight, w_per_kind * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload v_weight");
  if ((e = cudaMemcpy(m->b32, k_bias, b_per_kind * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload k_bias");
  if ((e = cudaMemcpy(m->b32 + b_per_kind, v_bias, b_per_kind * sizeof(float), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload v_bias");
  if ((e = cudaMemcpy(m->sel, sel.data(), sel.size() * sizeof(int), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload sel");
  if ((e = cudaMemcpy(m->sel_local, sel_local.data(), sel.size() * sizeof(int), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload sel_local");
  if ((e = cudaMemcpy(m->used_dev, m->used.data(), m->used.size() * sizeof(int), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload used");

  if (head_dim == cbk::kD) {
    // Tensor-core image, one unit per (kind, layer, head): S blocks of 32 KB
    // holding W^T (rows = output dim d, K-major = input feature) as two
    // 128B-swizzled panels of 64 features (16-byte chunk c of row d at chunk
    // position c ^ (d & 7) of its 128-byte row), then a 4 KB bias block: one
    // K=16 step in no-swizzle K-major layout whose columns 0 and 1 hold
    // bf16(bias) and bf16(bias - bf16(bias)), so ones @ block == bias to ~2^-17.
    const size_t units = 2ull * target_layers * heads;
    const size_t unit_halfs = (static_cast<size_t>(m->KB) * cbk::kKBlockBytes + cbk::kBiasBlockBytes) / 2;
    std::vector<uint16_t> img(units * unit_halfs, 0);
    for (int kind = 0; kind < 2; ++kind) {
      const float* W = kind ? v_weight : k_weight;
      const float* B = kind ? v_bias : k_bias;
      for (int l = 0; l < target_layers; ++l)
        for (int h = 0; h < heads; ++h) {
          const float* wh = W + (static_cast<size_t>(l) * heads + h) * F * head_dim;
          const float* bh = B + (static_cast<size_t>(l) * heads + h) * head_dim;
          const size_t unit = (static_cast<size_t>(kind) * target_layers + l) * heads + h;
          uint16_t* base = img.data() + unit * unit_halfs;
          for (int j = 0; j < m->KB; ++j) {
            uint16_t* blk = base + static_cast<size_t>(j) * (cbk::kKBlockBytes / 2);
            for (int f = 0; f < 128; ++f) {
              const int panel = f >> 6, chunk = (f & 63) >> 3, e8 = f & 7;
              const float* wrow = wh + static_cast<size_t>(j * 128 + f) * head_dim;
              for (int d = 0; d < 128; ++d) {
                const size_t byte = static_cast<size_t>(panel) * cbk::kPanelBytes + d * 128 +
                                    ((chunk ^ (d & 7)) << 4) + e8 * 2;
                blk[byte / 2] = f32_to_bf16_rne(wrow[d]);
              }
            }
          }
          uint16_t* bias_blk = base + static_cast<size_t>(m->KB) * (cbk::kKBlockBytes / 2);
          for (int d = 0; d < 128; ++d) {
            const uint16_t hi = f32_to_bf16_rne(bh[d]);
            uint32_t hbits = static_cast<uint32_t>(hi) << 16;
            float hf;
            std::memcpy(&hf, &hbits, 4);
            const uint16_t lo = f32_to_bf16_rne(bh[d] - hf);
            const size_t b0 = (d / 8) * 256 + (d % 8) * 16;  // k = 0 and k = 1 of row d
            bias_blk[b0 / 2] = hi;
            bias_blk[b0 / 2 + 1] = lo;
          }
        }
    }
    if ((e = cudaMalloc(&m->w_img, img.size() * sizeof(uint16_t))) != cudaSuccess) return cleanup(e, "cudaMalloc w_img");
    if ((e = cudaMemcpy(m->w_img, img.data(), img.size() * sizeof(uint16_t), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload w_img");
    if (m->KB <= cbk::kTmMaxKB) {
      // Tensor-memory image: per unit, chunk c (input features 8c..8c+7) of
      // lane L (output feature tm_lane_feature(L)) at (c * 128 + L) * 16 B.
      const size_t unit_halfs_tm = static_cast<size_t>(m->KB) * cbk::kKBlockBytes / 2;
      std::vector<uint16_t> tm(units * unit_halfs_tm, 0);
      for (int kind = 0; kind < 2; ++kind) {
        const float* W = kind ? v_weight : k_weight;
        for (int l = 0; l < target_layers; ++l)
          for (int h = 0; h < heads; ++h) {
            const float* wh = W + (static_cast<size_t>(l) * heads + h) * F * head_dim;
            const size_t unit = (static_cast<size_t>(kind) * target_layers + l) * heads + h;
            uint16_t* base = tm.data() + unit * unit_halfs_tm;
            for (int c = 0; c < F / 8; ++c)
              for (int L = 0; L < 128; ++L) {
                const int f = cbk::tm_lane_feature(L);
                for (int e8 = 0; e8 < 8; ++e8)
                  base[(static_cast<size_t>(c) * 128 + L) * 8 + e8] =
                      f32_to_bf16_rne(wh[static_cast<size_t>(8 * c + e8) * head_dim + f]);
              }
          }
      }
      if ((e = cudaMalloc(&m->w_tm, tm.size() * sizeof(uint16_t))) != cudaSuccess) return cleanup(e, "cudaMalloc w_tm");
      if ((e = cudaMemcpy(m->w_tm, tm.data(), tm.size() * sizeof(uint16_t), cudaMemcpyHostToDevice)) != cudaSuccess) return cleanup(e, "upload w_tm");
    }
  }
  *out = m;
  return CB_OK;
}

}  // namespace

extern "C" {

int cb_mapper_destroy(cb_mapper* m) {
  if (m == nullptr) return CB_OK;
  DeviceGuard guard(m->device);
  cudaFree(m->w32);
  cudaFree(m->b32);
  cudaFree(m->sel);
  cudaFree(m->sel_local);
  cudaFree(m->used_dev);
  cudaFree(m->w_img);
  cudaFree(m->w_tm);
  delete m;
  return CB_OK;
}

int cb_mapper_info(const cb_mapper* m, int* target_layers, int* heads, int* head_dim,
                   int* num_selected, int* used_source_layers) {
  if (m == nullptr) return fail(CB_ERR_INVALID, "null mapper");
  if (target_layers) *target_layers = m->L_t;
  if (heads) *heads = m->H;
  if (head_dim) *head_dim = m->D;
  if (num_selected) *num_selected = m->S;
  if (used_source_layers) *used_source_layers = m->U;
  return CB_OK;
}

int cb_mapper_path(const cb_mapper* m, int dtype, int64_t n_tokens, int64_t position_start, const cb_rope* dst_rope,
                   int has_token_order) {
  if (m == nullptr || dst_rope == nullptr) return fail(CB_ERR_INVALID, "null mapper or RoPE descriptor");
  if (m->D != cbk::kD || dtype != CB_DTYPE_BF16) return CB_PATH_CUDA_CORE;
  const int32_t dummy_order = 0;
  return tm_eligible(m, dst_rope, position_start, n_tokens, has_token_order ? &dummy_order : nullptr)
             ? CB_PATH_TENSOR_MEMORY
             : CB_PATH_TENSOR_CORE;
}

size_t cb_mapper_workspace_bytes(const cb_mapper* m, int dtype, int64_t n_tokens) {
  if (m == nullptr || n_tokens <= 0) return 0;
  if (m->D != cbk::kD || dtype != CB_DTYPE_BF16) return 0;
  return ws_total_bytes(m, n_tokens);
}

int cb_rope_table(void* stream, const cb_rope* rope, int64_t position_start, int64_t n, float* out_cos,
                  float* out_sin, int64_t out_stride) {
  if (rope == nullptr || rope->half_dim <= 0 || rope->half_dim > 128 || n < 0 || position_start < 0)
    return fail(CB_ERR_INVALID, "rope table: bad arguments");
  if (n == 0) return CB_OK;
  if (out_cos == nullptr || out_sin == nullptr) return fail(CB_ERR_INVALID, "rope table: null output");
  if (out_stride < n) return fail(CB_ERR_INVALID, "rope table: stride smaller than n");
  return launch_rope_table(static_cast<cudaStream_t>(stream), rope, position_start, n, out_cos, out_sin,
                           out_stride);
}

int cb_map_install(cb_mapper* m, void* stream, const cb_rows* src, const cb_rows* dst,
                   int64_t n_tokens, int64_t position_start, const cb_rope* src_rope,
                   const cb_rope* dst_rope, int dtype, void* workspace, size_t workspace_bytes,
                   const int32_t* token_order, int32_t* dev_status) {
  if (m == nullptr) return fail(CB_ERR_INVALID, "null mapper");
  if (dtype != CB_DTYPE_BF16 && dtype != CB_DTYPE_F32) return fail(CB_ERR_UNSUPPORTED, "dtype must be bf16 or fp32");
  if (n_tokens < 0) return fail(CB_ERR_INVALID, "negative token count");
  if (n_tokens > (int64_t(1) << 31) - 1) return fail(CB_ERR_UNSUPPORTED, "too many tokens in one call");
  const bool tc = (m->D == cbk::kD && dtype == CB_DTYPE_BF16);
  int rc;
  if (m->Hs > 0 && !tc)
    return fail(CB_ERR_UNSUPPORTED, "dense (nv_transfer) mappers run on the tensor-core path only (bf16, head_dim 128)");
  if ((rc = check_rows(src, "src", m->D, ws_heads(m), dtype, tc)) != CB_OK) return rc;
  if ((rc = check_rows(dst, "dst", m->D, m->H, dtype, tc)) != CB_OK) return rc;
  if (src->layers <= m->max_sel) return fail(CB_ERR_INVALID, "mapper selected layer exceeds source page depth");
  if (dst->layers != m->L_t) return fail(CB_ERR_INVALID, "destination layer count != mapper target layers");
  if (n_tokens == 0) return CB_OK;
  if ((rc = check_rope(src_rope, m->D, "source RoPE")) != CB_OK) return rc;
  if ((rc = check_rope(dst_rope, m->D, "target RoPE")) != CB_OK) return rc;
  if (position_start < 0) return fail(CB_ERR_INVALID, "negative position_start");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DeviceGuard guard(m->device);
  if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  if ((rc = ensure_rows_access(m->device, src, "src rows")) != CB_OK) return rc;
  if ((rc = ensure_rows_access(m->device, dst, "dst rows")) != CB_OK) return rc;

  if (tc) {
    if ((rc = check_tc_extras(m, dtype, n_tokens, workspace, workspace_bytes)) != CB_OK) return rc;
    if ((rc = launch_derotate(m, st, src, n_tokens, position_start, src_rope, workspace, token_order,
                              dev_status)) != CB_OK)
      return rc;
    return launch_map(m, st, src, dst, n_tokens, position_start, dst_rope, workspace, token_order, dev_status);
  }

  // Generic CUDA-core path.
  cbk::SimtParams p{};
  p.L_t = m->L_t;
  p.H = m->H;
  p.S = m->S;
  p.D = m->D;
  p.w32 = m->w32;
  p.b32 = m->b32;
  p.sel = m->sel;
  for (int l = 0; l < src->layers; ++l) {
    p.src_k[l] = src->k[l];
    p.src_v[l] = src->v[l];
  }
  p.src_row_stride = src->row_stride;
  p.src_rows = src->rows;
  p.src_head_offset = src->head_offset;
  p.src_slot_dtype = src->slot_dtype;
  p.src_slots = src->slots;
  for (int l = 0; l < dst->layers; ++l) {
    p.dst_k[l] = dst->k[l];
    p.dst_v[l] = dst->v[l];
  }
  p.dst_row_stride = dst->row_stride;
  p.dst_rows = dst->rows;
  p.dst_head_offset = dst->head_offset;
  p.dst_slot_dtype = dst->slot_dtype;
  p.dst_slots = dst->slots;
  p.src_rope = rope_dev(src_rope);
  p.dst_rope = rope_dev(dst_rope);
  p.position_start = position_start;
  p.status = dev_status;
  const size_t smem = static_cast<size_t>(m->H) * (m->S * m->D + m->D) * sizeof(float);
  if (smem > static_cast<size_t>(cbk::kTcMaxSmem)) return fail(CB_ERR_UNSUPPORTED, "generic mapper: heads*features too large");
  if (n_tokens > 2147483647ll) return fail(CB_ERR_UNSUPPORTED, "too many tokens");
  dim3 grid(static_cast<unsigned>(n_tokens), static_cast<unsigned>(m->L_t), 2);
  cudaError_t e = cbk::launch_map_simt(dtype == CB_DTYPE_F32, p, grid, smem, st);
  if (e != cudaSuccess) return cuda_fail(e, "map_install_simt launch");
  return CB_OK;
}

int cb_derotate_keys(cb_mapper* m, void* stream, const cb_rows* src, int64_t n_tokens,
                     int64_t position_start, const cb_rope* src_rope, void* workspace,
                     size_t workspace_bytes, const int32_t* token_order,
                     int32_t* dev_status) {
  int rc = check_tc_call(m, src, nullptr, n_tokens);
  if (rc != CB_OK) return rc;
  if ((rc = check_rope(src_rope, m->D, "source RoPE")) != CB_OK) return rc;
  if (position_start < 0) return fail(CB_ERR_INVALID, "negative position_start");
  if (n_tokens == 0) return CB_OK;
  if ((rc = check_tc_extras(m, CB_DTYPE_BF16, n_tokens, workspace, workspace_bytes)) != CB_OK) return rc;
  DeviceGuard guard(m->device);
  if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  if ((rc = ensure_rows_access(m->device, src, "src rows")) != CB_OK) return rc;
  return launch_derotate(m, static_cast<cudaStream_t>(stream), src, n_tokens, position_start, src_rope, workspace,
                         token_order,
                         dev_status);
}

int cb_map_install_packed(cb_mapper* m, void* stream, const cb_rows* src, const cb_rows* dst,
                          int64_t n_tokens, int64_t position_start, const cb_rope* dst_rope,
                          const void* workspace, size_t workspace_bytes,
                          const int32_t* token_order, int32_t* dev_status) {
  int rc = check_tc_call(m, src, dst, n_tokens);
  if (rc != CB_OK) return rc;
  if ((rc = check_rope(dst_rope, m->D, "target RoPE")) != CB_OK) return rc;
  if (position_start < 0) return fail(CB_ERR_INVALID, "negative position_start");
  if (n_tokens == 0) return CB_OK;
  if ((rc = check_tc_extras(m, CB_DTYPE_BF16, n_tokens, workspace, workspace_bytes)) != CB_OK) return rc;
  DeviceGuard guard(m->device);
  if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  if ((rc = ensure_rows_access(m->device, src, "src rows")) != CB_OK) return rc;
  if ((rc = ensure_rows_access(m->device, dst, "dst rows")) != CB_OK) return rc;
  return launch_map(m, static_cast<cudaStream_t>(stream), src, dst, n_tokens, position_start, dst_rope, workspace,
                   token_order,
                   dev_status);
}

static int launch_copy_rows(cudaStream_t st, cbk::CopyRowsParams& p, int64_t n) {
  if (n == 0) return CB_OK;
  int vec = 16;
  auto ok_for = [&](int v) {
    if (p.row_bytes % v) return false;
    if (p.src_stride_bytes % v || p.dst_stride_bytes % v || p.src_offset_bytes % v || p.dst_offset_bytes % v) return false;
    for (int l = 0; l < p.layers; ++l) {
      if (reinterpret_cast<uintptr_t>(p.src_k[l]) % v || reinterpret_cast<uintptr_t>(p.src_v[l]) % v) return false;
      if (reinterpret_cast<uintptr_t>(p.dst_k[l]) % v || reinterpret_cast<uintptr_t>(p.dst_v[l]) % v) return false;
    }
    return true;
  };
  while (vec > 2 && !ok_for(vec)) vec >>= 1;
  if (!ok_for(vec)) return fail(CB_ERR_INVALID, "row copy: rows not 2-byte aligned");
  const int64_t rows = 2 * static_cast<int64_t>(p.layers) * n;
  const int blocks = static_cast<int>(std::min<int64_t>((rows + 7) / 8, 148 * 32));
  cudaError_t e = cbk::launch_copy_rows(vec, p, blocks, st);
  if (e != cudaSuccess) return cuda_fail(e, "copy_rows launch");
  return CB_OK;
}

int cb_pack_rows(void* stream, const cb_rows* src, int head_dim, int dtype, int64_t n_tokens,
                 void* out, int32_t* dev_status) {
  if (dtype != CB_DTYPE_BF16 && dtype != CB_DTYPE_F32) return fail(CB_ERR_UNSUPPORTED, "dtype must be bf16 or fp32");
  if (head_dim <= 0) return fail(CB_ERR_INVALID, "head_dim must be positive");
  if (src == nullptr) return fail(CB_ERR_INVALID, "null row set");
  const int heads = src->heads - src->head_offset;
  int rc = check_rows(src, "src", head_dim, heads, dtype, false);
  if (rc != CB_OK) return rc;
  if (n_tokens < 0) return fail(CB_ERR_INVALID, "negative token count");
  if (n_tokens > 0 && out == nullptr) return fail(CB_ERR_INVALID, "null output block");
  if (n_tokens > 0) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(CB_ERR_CUDA, "cudaGetDevice failed");
    if ((rc = ensure_rows_access(device, src, "src rows")) != CB_OK) return rc;
    if ((rc = ensure_access(device, out, "output block")) != CB_OK) return rc;
  }
  const int es = elem_size(dtype);
  cbk::CopyRowsParams p{};
  p.layers = src->layers;
  p.row_bytes = heads * head_dim * es;
  p.n = n_tokens;
  for (int l = 0; l < src->layers; ++l) {
    p.src_k[l] = src->k[l];
    p.src_v[l] = src->v[l];
    p.dst_k[l] = static_cast<char*>(out) + (static_cast<int64_t>(l) * n_tokens) * p.row_bytes;
    p.dst_v[l] = static_cast<char*>(out) + (static_cast<int64_t>(src->layers + l) * n_tokens) * p.row_bytes;
  }
  p.src_stride_bytes = src->row_stride * es;
  p.src_offset_bytes = static_cast<int64_t>(src->head_offset) * head_dim * es;
  p.src_rows = src->rows;
  p.src_slot_dtype = src->slot_dtype;
  p.src_slots = src->slots;
  p.dst_stride_bytes = p.row_bytes;
  p.dst_offset_bytes = 0;
  p.dst_rows = n_tokens;
  p.dst_slot_dtype = CB_INDEX_NONE;
  p.dst_slots = nullptr;
  p.status = dev_status;
  return launch_copy_rows(static_cast<cudaStream_t>(stream), p, n_tokens);
}

int cb_install_rows(void* stream, const void* block, const cb_rows* dst, int head_dim, int dtype,
                    int64_t n_tokens, int32_t* dev_status) {
  if (dtype != CB_DTYPE_BF16 && dtype != CB_DTYPE_F32) return fail(CB_ERR_UNSUPPORTED, "dtype must be bf16 or fp32");
  if (head_dim <= 0) return fail(CB_ERR_INVALID, "head_dim must be positive");
  if (dst == nullptr) return fail(CB_ERR_INVALID, "null row set");
  const int heads = dst->heads - dst->head_offset;
  int rc = check_rows(dst, "dst", head_dim, heads, dtype, false);
  if (rc != CB_OK) return rc;
  if (n_tokens < 0) return fail(CB_ERR_INVALID, "negative token count");
  if (n_tokens > 0 && block == nullptr) return fail(CB_ERR_INVALID, "null source block");
  if (n_tokens > 0) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return fail(CB_ERR_CUDA, "cudaGetDevice failed");
    if ((rc = ensure_access(device, block, "source block")) != CB_OK) return rc;
    if ((rc = ensure_rows_access(device, dst, "dst rows")) != CB_OK) return rc;
  }
  const int es = elem_size(dtype);
  cbk::CopyRowsParams p{};
  p.layers = dst->layers;
  p.row_bytes = heads * head_dim * es;
  p.n = n_tokens;
  for (int l = 0; l < dst->layers; ++l) {
    p.src_k[l] = static_cast<const char*>(block) + (static_cast<int64_t>(l) * n_tokens) * p.row_bytes;
    p.src_v[l] = static_cast<const char*>(block) + (static_cast<int64_t>(dst->layers + l) * n_tokens) * p.row_bytes;
    p.dst_k[l] = dst->k[l];
    p.dst_v[l] = dst->v[l];
  }
  p.src_stride_bytes = p.row_bytes;
  p.src_offset_bytes = 0;
  p.src_rows = n_tokens;
  p.src_slot_dtype = CB_INDEX_NONE;
  p.src_slots = nullptr;
  p.dst_stride_bytes = dst->row_stride * es;
  p.dst_offset_bytes = static_cast<int64_t>(dst->head_offset) * head_dim * es;
  p.dst_rows = dst->rows;
  p.dst_slot_dtype = dst->slot_dtype;
  p.dst_slots = dst->slots;
  p.status = dev_status;
  return launch_copy_rows(static_cast<cudaStream_t>(stream), p, n_tokens);
}

int cb_ipc_export(const void* device_ptr, void* handle_out, uint64_t* offset_out) {
  if (device_ptr == nullptr || handle_out == nullptr || offset_out == nullptr)
    return fail(CB_ERR_INVALID, "null pointer");
  // The handle names the whole allocation that holds device_ptr (a caching
  // allocator hands out pieces of larger ones): report where inside it the
  // pointer sits.
  static PFN_cuMemGetAddressRange_v3020 range = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      ptr = nullptr;
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(ptr);
  }();
  if (range == nullptr) return fail(CB_ERR_CUDA, "cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(device_ptr)) != CUDA_SUCCESS)
    return fail(CB_ERR_INVALID, "cb_ipc_export: pointer is not inside a device allocation");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle_out, &h, 64);
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(device_ptr) - base);
  return CB_OK;
}

int cb_ipc_open(const void* handle, int device, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) return fail(CB_ERR_INVALID, "null pointer");
  DeviceGuard guard(device);
  if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, 64);
  cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  return CB_OK;
}

int cb_ipc_close(void* ptr) {
  if (ptr == nullptr) return CB_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcCloseMemHandle");
  return CB_OK;
}

int cb_copy_async(void* stream, void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return CB_OK;
  if (dst == nullptr || src == nullptr) return fail(CB_ERR_INVALID, "null copy pointer");
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail(CB_ERR_CUDA, "cudaGetDevice failed");
  int rc = ensure_access(device, dst, "copy destination");
  if (rc != CB_OK) return rc;
  if ((rc = ensure_access(device, src, "copy source")) != CB_OK) return rc;
  const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpyAsync");
  return CB_OK;
}

int cb_chunk_signal(void* stream, int64_t* flag, int64_t value) {
  if (flag == nullptr) return fail(CB_ERR_INVALID, "null flag");
  if (reinterpret_cast<uintptr_t>(flag) % 8) return fail(CB_ERR_INVALID, "flag not 8-byte aligned");
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail(CB_ERR_CUDA, "cudaGetDevice failed");
  int rc = ensure_access(device, flag, "flag");
  if (rc != CB_OK) return rc;
  cudaError_t e = cbk::launch_signal(reinterpret_cast<unsigned long long*>(flag), value,
                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "signal launch");
  return CB_OK;
}

int cb_chunk_wait(void* stream, const int64_t* flag, int64_t value, int64_t timeout_ns, int32_t* dev_status) {
  if (flag == nullptr || dev_status == nullptr) return fail(CB_ERR_INVALID, "null flag or status");
  if (reinterpret_cast<uintptr_t>(flag) % 8) return fail(CB_ERR_INVALID, "flag not 8-byte aligned");
  if (timeout_ns <= 0) return fail(CB_ERR_INVALID, "timeout must be positive");
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return fail(CB_ERR_CUDA, "cudaGetDevice failed");
  int rc = ensure_access(device, flag, "flag");
  if (rc != CB_OK) return rc;
  cudaError_t e = cbk::launch_wait(reinterpret_cast<const unsigned long long*>(flag), value, timeout_ns,
                                   dev_status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "wait launch");
  return CB_OK;
}

int cb_enable_peer_access(int device, int peer) {
  DeviceGuard guard(device);
  if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
  int can = 0;
  cudaError_t e = cudaDeviceCanAccessPeer(&can, device, peer);
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceCanAccessPeer");
  if (!can) return fail(CB_ERR_UNSUPPORTED, "peer access not possible between these devices");
  e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return CB_OK;
  }
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceEnablePeerAccess");
  return CB_OK;
}

}  // extern "C"

// ------------------------- no-allocation map + install -------------------------
// cb_map_install_noalloc: cb_map_install with its key workspace taken from a
// fixed device array that belongs to this library instead of from the caller.
// It serves callers that cannot allocate device memory at handoff time: a
// serving engine that sized its KV pool to fill the GPU at start-up and so has
// no headroom left for per-handoff scratch, and hosts that bind the C ABI
// without any device allocator of their own (an FFI caller holding only raw
// pointers), where a cudaMalloc/cudaFree pair per call would also stall the
// device. The array is CB_NOALLOC_SCRATCH_BYTES (64 MiB) per device; it holds
// the BF16 content-space keys [used_layers][n_tokens][heads][128], so one call
// maps at most 64 MiB / (used_layers * heads * 256 B) tokens. Every call on a
// device shares it, so calls whose GPU work overlaps (unordered streams,
// concurrent host threads) race on it. No part of it must start at zero: the
// key phase writes every element that the map phase reads.
static __device__ __align__(256) unsigned char g_noalloc_scratch[CB_NOALLOC_SCRATCH_BYTES];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on `device`, which the caller has made
// current. Looked up once per device, on that device's first call.
int noalloc_scratch(int device, void** out) {
  if (device < 0 || device >= kNoAllocMaxDevices)
    return fail(CB_ERR_UNSUPPORTED, "cb_map_install_noalloc: device index beyond the 64 this build tracks");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
    g_noalloc_ptr[device] = ptr;
  }
  *out = g_noalloc_ptr[device];
  return CB_OK;
}

}  // namespace

extern "C" {

int cb_map_install_noalloc(cb_mapper* m, void* stream, const cb_rows* src, const cb_rows* dst,
                           int64_t n_tokens, int64_t position_start, const cb_rope* src_rope,
                           const cb_rope* dst_rope, int dtype, int32_t* dev_status) {
  if (m == nullptr) return fail(CB_ERR_INVALID, "null mapper");
  if (n_tokens < 0) return fail(CB_ERR_INVALID, "negative token count");
  const size_t need = cb_mapper_workspace_bytes(m, dtype, n_tokens);
  if (need > static_cast<size_t>(CB_NOALLOC_SCRATCH_BYTES)) {
    const size_t per_token = cb_mapper_workspace_bytes(m, dtype, 1);
    char msg[320];
    std::snprintf(msg, sizeof msg,
                  "cb_map_install_noalloc: %lld tokens need %zu bytes of key scratch, above its fixed %d bytes "
                  "(at most %zu tokens per call for this mapper); split the tokens over several calls or use "
                  "cb_map_install with a caller workspace",
                  static_cast<long long>(n_tokens), need, CB_NOALLOC_SCRATCH_BYTES,
                  per_token ? static_cast<size_t>(CB_NOALLOC_SCRATCH_BYTES) / per_token : size_t(0));
    return fail(CB_ERR_UNSUPPORTED, msg);
  }
  void* scratch = nullptr;
  {
    DeviceGuard guard(m->device);
    if (!guard.ok) return fail(CB_ERR_CUDA, "cudaSetDevice failed");
    const int rc = noalloc_scratch(m->device, &scratch);
    if (rc != CB_OK) return rc;
  }
  return cb_map_install(m, stream, src, dst, n_tokens, position_start, src_rope, dst_rope, dtype, scratch,
                        static_cast<size_t>(CB_NOALLOC_SCRATCH_BYTES), nullptr, dev_status);
}

}  // extern "C"
