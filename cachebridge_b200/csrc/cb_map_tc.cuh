// Parameter block and constants of the tcgen05 fused map+install kernel.
#pragma once

#include <stdint.h>

#include "cb_device.cuh"

namespace cbk {

constexpr int kD = 128;                        // head_dim of the tensor-core path
constexpr int kBM = 128;                       // tokens per m-tile (UMMA M)
constexpr int kPanelBytes = 128 * 128;         // 128 rows x 64 bf16 (one 128B-swizzle panel)
constexpr int kKBlockBytes = 2 * kPanelBytes;  // 128 rows x 128 bf16: one source layer's head
constexpr int kEpiWarps = 8;                   // two groups of 4 (one warp per TMEM lane quarter)
constexpr int kEpiWarpBytes = 32 * 128;        // 32 token rows x 128 B staging per epilogue warp
constexpr int kAccBufs = 4;                    // FP32 accumulators in TMEM (128 columns each)
constexpr int kTcThreads = 32 * (4 + kEpiWarps + 2);  // producers, epilogue, MMA, loader
constexpr int kTmemCols = 128 * kAccBufs;      // all 512 TMEM columns
constexpr int kTcMaxSmem = 232448;             // sm_100 opt-in dynamic shared memory per block

struct MapTcParams {
  int n_tokens;
  int L_t;       // target layers
  int H;         // heads mapped by this call
  int S;         // selected source layers per target layer
  int R;         // m-tiles per chunk
  int n_chunks;
  int num_items;
  int w_slots;   // weight k-block slots in shared memory
  int stages;    // A stages (ring)
  int w_resident;

  const uint8_t* w_img;     // [2 kinds][L_t][H][S][32 KB] pre-swizzled bf16 W^T k-blocks
  const float* bias;        // [2 kinds][L_t][H][128] fp32
  const int* sel_global;    // [L_t][S] source layer ids
  const int* sel_local;     // [L_t][S] index into the workspace's used-layer list

  const __nv_bfloat16* ws_k;  // [U][n_tokens][H][128] content-space keys
  const void* src_v[CB_MAX_LAYERS];
  int64_t src_row_stride;   // elements
  int64_t src_rows;
  int src_head_offset;
  int src_slot_dtype;
  const void* src_slots;

  void* dst_k[CB_MAX_LAYERS];
  void* dst_v[CB_MAX_LAYERS];
  int64_t dst_row_stride;   // elements
  int64_t dst_rows;
  int dst_head_offset;
  int dst_slot_dtype;
  const void* dst_slots;

  const float* dcos;  // [64][n_tokens] target RoPE coefficients (workspace tail)
  const float* dsin;
  int32_t* status;
};

__global__ void map_install_tc_kernel(const __grid_constant__ MapTcParams p);

// Shared-memory bytes the kernel needs for a given weight-slot / stage split.
inline int tc_smem_bytes(int w_slots, int stages) {
  return 1024 /* alignment slack */ + (w_slots + stages) * kKBlockBytes + kEpiWarps * kEpiWarpBytes +
         512 /* barriers, TMEM holder, abort flag */;
}

}  // namespace cbk
