// Parameter block and constants of the transposed tensor-core map+install
// kernel (mapper weights resident in tensor memory).
#pragma once

#include <stdint.h>

#include "cb_device.cuh"
#include "cb_map_tc.cuh"

namespace cbk {

constexpr int kTmProdWarps = 4;                     // producer warps (TMA keys, cp.async values)
constexpr int kTmEpiGroups = 2;                     // epilogue groups, one accumulator each
constexpr int kTmEpiWarps = 4 * kTmEpiGroups;       // one warp per TMEM lane quarter per group
constexpr int kTmMmaWarp = kTmProdWarps + kTmEpiWarps;
constexpr int kTmLoadWarp0 = kTmMmaWarp + 1;        // four weight-loader warps (one per lane quarter)
constexpr int kTmThreads = 32 * (kTmLoadWarp0 + 4);
constexpr int kTmAccCols = 128;                     // one FP32 accumulator: 128 features x 128 tokens
constexpr int kTmWeightCol0 = kTmEpiGroups * kTmAccCols;  // weights start after the accumulators
constexpr int kTmRowPitch = 256 + 16;               // staging row pitch (bytes): one 256 B row + 16
constexpr int kTmStageBytes = 128 * kTmRowPitch;    // epilogue staging: 128 token rows
constexpr int kTmMaxKB = 4;                         // k-blocks whose weights fit in tensor memory

struct MapTmParams {
  int n_tokens;
  int L_t;
  int H;
  int S;
  int KB;        // 128-feature blocks per unit (S headwise, S * source heads dense)
  int kb_heads;  // source heads per selected layer in the block sequence (1 headwise)
  int dense;
  int R;         // m-tiles per work item
  int n_chunks;
  int num_items;
  int stages;    // token-tile stages in shared memory (ring)
  int w_bufs;    // weight buffers in tensor memory (2: next item's weights load during this one)

  // Per unit (kind, layer, head): KB * 16 chunks of 128 lanes x 16 B. Chunk c
  // of lane L holds bf16 W[8c .. 8c+8)[f(L)] (input features 8c..8c+7 of
  // output feature f(L)), f(L) = 8 (L / 16) + L % 8 + 64 ((L / 8) % 2): tensor
  // memory lanes L and L + 8 hold the RoPE pair (i, i + 64).
  const uint8_t* w_tm;
  int64_t unit_bytes;        // KB * 32 KB
  const float* bias;         // [2][L_t][H][128] FP32 (split into BF16 hi + lo for the bias step)
  const int* sel_global;     // [L_t][S]
  const int* sel_local;      // [L_t][S]

  const void* src_v[CB_MAX_LAYERS];
  int64_t src_row_stride;    // elements
  int64_t src_rows;
  int src_head_offset;
  int src_slot_dtype;
  const void* src_slots;

  void* dst_k[CB_MAX_LAYERS];
  void* dst_v[CB_MAX_LAYERS];
  int64_t dst_row_stride;    // elements
  int64_t dst_rows;
  int dst_head_offset;
  int dst_slot_dtype;
  const void* dst_slots;
  int dst_evict_first;
  int dst_v8;                // 1: every destination row is this GPU's and 32-byte aligned (32-byte stores)

  // Target RoPE: per frequency i, inv_freq, and the unit rotations by one and
  // by eight positions (cos, sin of inv_freq and 8 inv_freq, from the exact
  // product, rounded once); the YaRN magnitude scales the recurrence.
  float dst_inv_freq[64];
  float rot1_c[64], rot1_s[64], rot8_c[64], rot8_s[64];
  float dst_magnitude;
  int64_t position_start;
  const int32_t* order;      // always null: this kernel processes tokens in order
  int32_t* status;
  CUtensorMap kmap;          // content-space key workspace, as for map_install_tc_kernel
};

__global__ void map_install_tm_kernel(const __grid_constant__ MapTmParams p);

// Fixed shared memory: staging tiles, two bias blocks (one per weight buffer)
// and the constant ones block of the bias step, barriers.
constexpr int kTmFixedSmem =
    1024 /* alignment */ + kTmEpiGroups * kTmStageBytes + 2 * kBiasBlockBytes + kOnesBytes + 512 /* barriers */;

inline int tm_smem_bytes(int stages) { return kTmFixedSmem + stages * kKBlockBytes; }

// Output feature held by tensor-memory lane L of a weight block.
__host__ __device__ constexpr int tm_lane_feature(int L) { return 8 * (L / 16) + (L % 8) + 64 * ((L / 8) % 2); }

}  // namespace cbk
