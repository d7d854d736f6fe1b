// Parameter block and constants of the tcgen05 fused map+install kernel.
#pragma once

#include <stdint.h>

#include "cb_device.cuh"

namespace cbk {

constexpr int kD = 128;                        // head_dim of the tensor-core path
constexpr int kBM = 128;                       // tokens per m-tile (UMMA M)
constexpr int kPanelBytes = 128 * 128;         // 128 rows x 64 bf16 (one 128B-swizzle panel)
constexpr int kKBlockBytes = 2 * kPanelBytes;  // 128 rows x 128 bf16: one source layer's head
constexpr int kBiasBlockBytes = 128 * 32;      // one K=16 step x 128 rows (no swizzle): bias rows
constexpr int kOnesBytes = 128 * 32;           // one K=16 step x 128 rows: constant 1.0 columns
constexpr int kProdWarps = 4;                  // producer warps (cp.async value gathers, TMA keys)
constexpr int kEpiGroups = 3;                  // epilogue groups (one m-tile each in flight)
constexpr int kEpiWarps = 4 * kEpiGroups;      // one warp per TMEM lane quarter per group
constexpr int kMmaWarp = kProdWarps + kEpiWarps;
constexpr int kLoaderWarp = kMmaWarp + 1;
constexpr int kTcThreads = 32 * (kLoaderWarp + 1);
constexpr int kAccBufs = 4;                    // FP32 accumulators in TMEM (128 columns each)
constexpr int kTmemCols = 128 * kAccBufs;      // all 512 TMEM columns
constexpr int kEpiWarpBytes = 32 * 128;        // 32 token rows x 128 B staging per epilogue warp
constexpr int kTcMaxSmem = 232448;             // sm_100 opt-in dynamic shared memory per block

struct MapTcParams {
  int n_tokens;
  int L_t;       // target layers
  int H;         // heads mapped by this call
  int S;         // selected source layers per target layer
  int KB;        // 128-feature blocks per unit: S (headwise) or S * source heads (dense)
  int kb_heads;  // source heads per selected layer in the block sequence (1 headwise)
  int dense;     // 1: block kb reads source head kb % kb_heads; 0: the target head
  int ws_heads;  // heads per row of the key workspace and of the source rows read
  int R;         // m-tiles per chunk
  int n_chunks;
  int num_items;
  int w_slots;   // weight k-block slots in shared memory
  int stages;    // A stages (ring)
  int w_resident;

  const uint8_t* w_img;     // per unit: KB x 32 KB W^T k-blocks (128B-swizzled) + 4 KB bias block
  int64_t unit_bytes;       // KB * 32 KB + 4 KB
  const int* sel_global;    // [L_t][S] source layer ids
  const int* sel_local;     // [L_t][S] index into the workspace's used-layer list

  const __nv_bfloat16* ws_k;  // [U][n_tokens][H][128] content-space keys, processing order
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
  int dst_evict_first;      // 1: the target rows are this GPU's memory; store them with an
                            // L2 evict-first policy (peer pools get plain stores)

  float dst_inv_freq[64];   // target RoPE
  float dst_magnitude;
  int64_t position_start;   // absolute position of token 0
  const int32_t* order;     // token at each processing index (null: identity)
  int trig_exact;           // 1 when a phase can exceed the reduced method's range: use sincosf
  int32_t* status;
  // 4-D map of the key workspace {128, H, n_tokens, U}, box {64, 1, 128, 1},
  // 128B-swizzled, so a box lands in the UMMA K-major SW128 layout.
  CUtensorMap kmap;
};

__global__ void map_install_tc_kernel(const __grid_constant__ MapTcParams p);

// Shared memory bytes of everything but the weight slots and A stages.
constexpr int kTcFixedSmem = 1024 /* alignment slack */ + kBiasBlockBytes + kOnesBytes +
                             kEpiWarps * kEpiWarpBytes + 512 /* barriers */;

// Shared-memory bytes the kernel needs for a given weight-slot / stage split.
inline int tc_smem_bytes(int w_slots, int stages) {
  return kTcFixedSmem + (w_slots + stages) * kKBlockBytes;
}

}  // namespace cbk
