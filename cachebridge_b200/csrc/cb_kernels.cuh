// Parameter blocks of the bandwidth kernels and the generic mapper.
#pragma once

#include <stdint.h>

#include "cb_device.cuh"

namespace cbk {

struct RopeTableParams {
  RopeDev rope;
  int64_t position_start;
  int64_t n;
  float* out_cos;  // [half_dim][out_stride]
  float* out_sin;
  int64_t out_stride;
};

struct DerotateParams {
  int64_t n_tokens;
  int H;  // heads packed (this call's heads)
  int U;  // used source layers
  const void* src_k[CB_MAX_LAYERS];
  const int* used;  // [U] source layer ids
  int64_t src_row_stride;
  int64_t src_rows;
  int src_head_offset;
  int src_slot_dtype;
  const void* src_slots;
  RopeDev rope;  // source RoPE
  int64_t position_start;
  const int32_t* order;  // processing order of the tokens, or null
  __nv_bfloat16* ws;  // [U][n][H][128], rows in processing order
  int parts;          // warps per token: part p takes rows [p, p + 1) * rows_per_part of its U*H
  int rows_per_part;  // a multiple of 16
  int32_t* status;
};

struct CopyRowsParams {
  int layers;
  int row_bytes;
  int64_t n;
  const void* src_k[CB_MAX_LAYERS];
  const void* src_v[CB_MAX_LAYERS];
  int64_t src_stride_bytes;
  int64_t src_offset_bytes;
  int64_t src_rows;
  int src_slot_dtype;
  const void* src_slots;
  void* dst_k[CB_MAX_LAYERS];
  void* dst_v[CB_MAX_LAYERS];
  int64_t dst_stride_bytes;
  int64_t dst_offset_bytes;
  int64_t dst_rows;
  int dst_slot_dtype;
  const void* dst_slots;
  int32_t* status;
};

struct SimtParams {
  int L_t, H, S, D;
  const float* w32;  // [2][L_t][H][S*D][D]
  const float* b32;  // [2][L_t][H][D]
  const int* sel;    // [L_t][S]
  const void* src_k[CB_MAX_LAYERS];
  const void* src_v[CB_MAX_LAYERS];
  int64_t src_row_stride, src_rows;
  int src_head_offset, src_slot_dtype;
  const void* src_slots;
  void* dst_k[CB_MAX_LAYERS];
  void* dst_v[CB_MAX_LAYERS];
  int64_t dst_row_stride, dst_rows;
  int dst_head_offset, dst_slot_dtype;
  const void* dst_slots;
  RopeDev src_rope;
  RopeDev dst_rope;
  int64_t position_start;
  int32_t* status;
};

__global__ void rope_table_kernel(const __grid_constant__ RopeTableParams p);
__global__ void derotate_pack_kernel(const __grid_constant__ DerotateParams p);

// Host launchers for the templated kernels (kept in the defining translation unit).
// vec_bytes in {16, 8, 4, 2}.
cudaError_t launch_copy_rows(int vec_bytes, const CopyRowsParams& p, int blocks, cudaStream_t stream);
cudaError_t launch_signal(unsigned long long* flag, long long value, cudaStream_t stream);
cudaError_t launch_wait(const unsigned long long* flag, long long value, long long timeout_ns, int32_t* status,
                        cudaStream_t stream);
cudaError_t launch_map_simt(bool fp32_storage, const SimtParams& p, dim3 grid, size_t smem_bytes,
                            cudaStream_t stream);

}  // namespace cbk
