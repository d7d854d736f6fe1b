// Bandwidth kernels of the handoff path and the generic CUDA-core mapper.
//
//  - rope_table_kernel      qwen_rope tables (src/cachebridge/rope.py:16-72)
//  - derotate_pack_kernel   gather source key rows through the slot table,
//                           remove source RoPE in FP32 (rope.py:82-89) and
//                           store BF16 content-space keys for the tensor-core
//                           mapper (the key half of pack_source_block,
//                           online/blocks.py:47-82, fused with mapper.py:143-144)
//  - copy_rows_kernel       row gather / scatter between row sets (pack_source_block
//                           and _DirectMappedPoolCodec.copy)
//  - map_install_simt_kernel  the full headwise mapper for geometries outside
//                           the tensor-core path (head_dim != 128 or FP32 storage)
#include "cb_device.cuh"
#include "cb_kernels.cuh"

namespace cbk {

// ---------------------------------------------------------------------------
// RoPE tables
// ---------------------------------------------------------------------------
__global__ void rope_table_kernel(const __grid_constant__ RopeTableParams p) {
  const int half = p.rope.half_dim;
  const int64_t total = p.n * half;
  // Token-fastest order: consecutive threads write consecutive columns of one
  // frequency row (coalesced stores into the frequency-major table).
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(idx / p.n);
    const int64_t t = idx - static_cast<int64_t>(i) * p.n;
    float c, s;
    rope_coeff(static_cast<float>(p.position_start + t), p.rope.inv_freq[i], p.rope.magnitude, c, s);
    p.out_cos[i * p.out_stride + t] = c;
    p.out_sin[i * p.out_stride + t] = s;
  }
}

// ---------------------------------------------------------------------------
// Key gather + source-RoPE removal -> BF16 content-space workspace
// ---------------------------------------------------------------------------
// One warp per (token, part): the U*H rows of a token are split into `parts`
// runs of rows_per_part so that small calls still fill the GPU. Lane = (row
// group g = lane/8, pair index j = lane%8):
// it owns elements [8j, 8j+8) and [64+8j, 64+8j+8) of one 128-wide head row,
// i.e. 8 complete RoPE pairs, so the rotation needs no data exchange. Four
// consecutive heads of the same slot row are read per warp instruction (1 KB
// contiguous per instruction pair).
//
// The reference divides by max(cos^2 + sin^2, FLT_MIN) per element
// (rope.py:86-89). The result here is rounded to BF16 (the tensor-core operand),
// so the division is folded once per (token, frequency) into the coefficients
// cos/m and sin/m; the two forms differ by at most a few FP32 ulps before the
// BF16 rounding.
__global__ void __launch_bounds__(256, 3) derotate_pack_kernel(const __grid_constant__ DerotateParams p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t wg = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  const int64_t t = wg / p.parts;
  const int part = static_cast<int>(wg - t * p.parts);
  if (t >= p.n_tokens || status_timed_out(p.status)) return;
  const int g = lane >> 3;
  const int j = lane & 7;

  // Processing index t holds token `tok` (the caller's order, or t itself).
  const int tok = token_at(p.order, static_cast<int>(t), static_cast<int>(p.n_tokens), lane == 0 ? p.status : nullptr);
  int64_t slot = tok < 0 ? -1 : load_slot(p.src_slots, p.src_slot_dtype, tok);
  if (tok >= 0 && (slot < 0 || slot >= p.src_rows)) {
    if (lane == 0) flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
    slot = -1;
  }
  float c[8], s[8];
  {
    const float pos = static_cast<float>(p.position_start + (tok < 0 ? 0 : tok));
#pragma unroll
    for (int e = 0; e < 8; ++e) rope_coeff(pos, p.rope.inv_freq[8 * j + e], p.rope.magnitude, c[e], s[e]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float m = fmaxf(__fadd_rn(__fmul_rn(c[e], c[e]), __fmul_rn(s[e], s[e])), 1.17549435e-38f);
      const float inv = __frcp_rn(m);
      c[e] = __fmul_rn(c[e], inv);
      s[e] = __fmul_rn(s[e], inv);
    }
  }
  const int r_begin = part * p.rows_per_part;
  const int rows = min(p.U * p.H, r_begin + p.rows_per_part);  // end of this warp's rows
  const int64_t src_off = slot * p.src_row_stride;
  constexpr int kUnroll = 4;
  for (int r0 = r_begin; r0 < rows; r0 += 4 * kUnroll) {
    uint4 a[kUnroll], b[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int r = r0 + 4 * k + g;
      a[k] = make_uint4(0, 0, 0, 0);
      b[k] = make_uint4(0, 0, 0, 0);
      if (r < rows && slot >= 0) {
        const int u = r / p.H;
        const int h = r - u * p.H;
        const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(p.src_k[__ldg(p.used + u)]) +
                                   src_off + static_cast<int64_t>(p.src_head_offset + h) * 128;
        a[k] = __ldg(reinterpret_cast<const uint4*>(row + 8 * j));
        b[k] = __ldg(reinterpret_cast<const uint4*>(row + 64 + 8 * j));
      }
    }
#pragma unroll
    for (int k = 0; k < kUnroll; ++k) {
      const int r = r0 + 4 * k + g;
      if (r >= rows) continue;
      const int u = r / p.H;
      const int h = r - u * p.H;
      const uint32_t av[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
      const uint32_t bv[4] = {b[k].x, b[k].y, b[k].z, b[k].w};
      uint32_t oa[4], ob[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float x0l = bf16_lo(av[e]), x0h = bf16_hi(av[e]);
        const float x1l = bf16_lo(bv[e]), x1h = bf16_hi(bv[e]);
        // (x0*c + x1*s)/m and (x1*c - x0*s)/m with c, s pre-divided by m.
        const float y0l = __fmaf_rn(x0l, c[2 * e], __fmul_rn(x1l, s[2 * e]));
        const float y1l = __fmaf_rn(x1l, c[2 * e], -__fmul_rn(x0l, s[2 * e]));
        const float y0h = __fmaf_rn(x0h, c[2 * e + 1], __fmul_rn(x1h, s[2 * e + 1]));
        const float y1h = __fmaf_rn(x1h, c[2 * e + 1], -__fmul_rn(x0h, s[2 * e + 1]));
        oa[e] = pack_bf16x2(y0l, y0h);
        ob[e] = pack_bf16x2(y1l, y1h);
      }
      __nv_bfloat16* out = p.ws + ((static_cast<int64_t>(u) * p.n_tokens + t) * p.H + h) * 128;
      *reinterpret_cast<uint4*>(out + 8 * j) = make_uint4(oa[0], oa[1], oa[2], oa[3]);
      *reinterpret_cast<uint4*>(out + 64 + 8 * j) = make_uint4(ob[0], ob[1], ob[2], ob[3]);
    }
  }
}

// ---------------------------------------------------------------------------
// Row copies (gather / scatter)
// ---------------------------------------------------------------------------
// Warps walk groups of RPW consecutive tokens of one (kind, layer); V-byte
// vectors across lanes. Short rows (one vector per lane or less) take RPW = 4
// so each lane keeps four independent loads in flight and the (kind, layer,
// token) decomposition is paid once per group; longer rows take RPW = 1 and
// loop over their vectors.
template <typename V, int RPW>
__global__ void __launch_bounds__(256) copy_rows_kernel(const __grid_constant__ CopyRowsParams p) {
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t groups_per_kl = (p.n + RPW - 1) / RPW;
  const int64_t groups_total = 2 * static_cast<int64_t>(p.layers) * groups_per_kl;
  const int lane = threadIdx.x & 31;
  if (status_timed_out(p.status)) return;
  const int nvec = p.row_bytes / static_cast<int>(sizeof(V));
  for (int64_t w = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
       w < groups_total; w += warps_total) {
    const int64_t kl = w / groups_per_kl;
    const int64_t t0 = (w - kl * groups_per_kl) * RPW;
    const int layer = static_cast<int>(kl % p.layers);
    const int kind = static_cast<int>(kl / p.layers);
    const char* src_base = reinterpret_cast<const char*>(kind ? p.src_v[layer] : p.src_k[layer]) + p.src_offset_bytes;
    char* dst_base = reinterpret_cast<char*>(kind ? p.dst_v[layer] : p.dst_k[layer]) + p.dst_offset_bytes;
    const char* src[RPW];
    char* dst[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
      src[r] = nullptr;
      dst[r] = nullptr;
      const int64_t t = t0 + r;
      if (t >= p.n) continue;
      const int64_t ss = load_slot(p.src_slots, p.src_slot_dtype, t);
      const int64_t ds = load_slot(p.dst_slots, p.dst_slot_dtype, t);
      if (ss < 0 || ss >= p.src_rows || ds < 0 || ds >= p.dst_rows) {
        if (lane == 0) flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
        continue;
      }
      src[r] = src_base + ss * p.src_stride_bytes;
      dst[r] = dst_base + ds * p.dst_stride_bytes;
    }
    if (RPW > 1) {
      V v[RPW];
#pragma unroll
      for (int r = 0; r < RPW; ++r)
        if (src[r] != nullptr && lane < nvec) v[r] = reinterpret_cast<const V*>(src[r])[lane];
#pragma unroll
      for (int r = 0; r < RPW; ++r)
        if (src[r] != nullptr && lane < nvec) reinterpret_cast<V*>(dst[r])[lane] = v[r];
    } else {
      // Long rows: four vectors per lane in flight, all loaded before any is
      // stored (the stores could otherwise alias the next loads and serialise
      // them behind one another).
#pragma unroll
      for (int r = 0; r < RPW; ++r) {
        if (src[r] == nullptr) continue;
        const V* s = reinterpret_cast<const V*>(src[r]);
        V* d = reinterpret_cast<V*>(dst[r]);
        for (int e0 = 0; e0 < nvec; e0 += 128) {
          V v[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e = e0 + lane + 32 * i;
            if (e < nvec) v[i] = s[e];
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e = e0 + lane + 32 * i;
            if (e < nvec) d[e] = v[i];
          }
        }
      }
    }
  }
}

template <typename V>
static void copy_rows_dispatch(const CopyRowsParams& p, int blocks, cudaStream_t st) {
  if (p.row_bytes <= 32 * static_cast<int>(sizeof(V)))
    copy_rows_kernel<V, 4><<<blocks, 256, 0, st>>>(p);
  else
    copy_rows_kernel<V, 1><<<blocks, 256, 0, st>>>(p);
}

cudaError_t launch_copy_rows(int vec_bytes, const CopyRowsParams& p, int blocks, cudaStream_t st) {
  switch (vec_bytes) {
    case 16: copy_rows_dispatch<uint4>(p, blocks, st); break;
    case 8: copy_rows_dispatch<uint2>(p, blocks, st); break;
    case 4: copy_rows_dispatch<uint32_t>(p, blocks, st); break;
    default: copy_rows_dispatch<uint16_t>(p, blocks, st); break;
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Generic (CUDA-core) headwise mapper
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float to_f32(T v);
template <>
__device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// grid (n_tokens, L_t, 2 kinds). Shared memory: X [H][S*D] then Y [H][D] floats.
template <typename T>
__global__ void __launch_bounds__(256) map_install_simt_kernel(const __grid_constant__ SimtParams p) {
  extern __shared__ float sm_f[];
  __shared__ int skip;
  if (threadIdx.x == 0) skip = status_timed_out(p.status) ? 1 : 0;
  __syncthreads();
  if (skip) return;
  const int64_t t = blockIdx.x;
  const int l = blockIdx.y;
  const int kind = blockIdx.z;
  const int D = p.D;
  const int half = D / 2;
  const int F = p.S * D;
  float* X = sm_f;
  float* Y = sm_f + p.H * F;

  const int64_t ss = load_slot(p.src_slots, p.src_slot_dtype, t);
  const int64_t ds = load_slot(p.dst_slots, p.dst_slot_dtype, t);
  if (ss < 0 || ss >= p.src_rows || ds < 0 || ds >= p.dst_rows) {
    if (threadIdx.x == 0) flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
    return;
  }
  for (int idx = threadIdx.x; idx < p.H * F; idx += blockDim.x) {
    const int h = idx / F;
    const int f = idx - h * F;
    const int j = f / D;
    const int e = f - j * D;
    const int layer = __ldg(p.sel + l * p.S + j);
    const T* row = reinterpret_cast<const T*>(kind ? p.src_v[layer] : p.src_k[layer]) +
                   ss * p.src_row_stride + static_cast<int64_t>(p.src_head_offset + h) * D;
    float x = to_f32<T>(row[e]);
    if (kind == 0) {
      const int i = e < half ? e : e - half;
      float c, s;
      rope_coeff(static_cast<float>(p.position_start + t), p.src_rope.inv_freq[i], p.src_rope.magnitude, c, s);
      float o0, o1;
      if (e < half) {
        rope_remove_pair(x, to_f32<T>(row[e + half]), c, s, o0, o1);
        x = o0;
      } else {
        rope_remove_pair(to_f32<T>(row[e - half]), x, c, s, o0, o1);
        x = o1;
      }
    }
    X[idx] = x;
  }
  __syncthreads();
  const float* W = p.w32 + ((static_cast<int64_t>(kind) * p.L_t + l) * p.H) * F * D;
  const float* B = p.b32 + ((static_cast<int64_t>(kind) * p.L_t + l) * p.H) * D;
  for (int idx = threadIdx.x; idx < p.H * D; idx += blockDim.x) {
    const int h = idx / D;
    const int d = idx - h * D;
    const float* wh = W + static_cast<int64_t>(h) * F * D + d;
    const float* xh = X + h * F;
    float acc = 0.f;
    for (int f = 0; f < F; ++f) acc = fmaf(xh[f], __ldg(wh + static_cast<int64_t>(f) * D), acc);
    Y[idx] = __fadd_rn(acc, __ldg(B + idx));
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < p.H * D; idx += blockDim.x) {
    const int h = idx / D;
    const int d = idx - h * D;
    float y = Y[idx];
    if (kind == 0) {
      const int i = d < half ? d : d - half;
      float c, s;
      rope_coeff(static_cast<float>(p.position_start + t), p.dst_rope.inv_freq[i], p.dst_rope.magnitude, c, s);
      float o0, o1;
      if (d < half) {
        rope_apply_pair(y, Y[idx + half], c, s, o0, o1);
        y = o0;
      } else {
        rope_apply_pair(Y[idx - half], y, c, s, o0, o1);
        y = o1;
      }
    }
    T* out = reinterpret_cast<T*>(kind ? p.dst_v[l] : p.dst_k[l]) + ds * p.dst_row_stride +
             static_cast<int64_t>(p.dst_head_offset + h) * D;
    out[d] = from_f32<T>(y);
  }
}

cudaError_t launch_map_simt(bool fp32_storage, const SimtParams& p, dim3 grid, size_t smem, cudaStream_t st) {
  cudaError_t e = cudaSuccess;
  if (fp32_storage) {
    if (smem > 48 * 1024)
      e = cudaFuncSetAttribute(map_install_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    map_install_simt_kernel<float><<<grid, 256, smem, st>>>(p);
  } else {
    if (smem > 48 * 1024)
      e = cudaFuncSetAttribute(map_install_simt_kernel<__nv_bfloat16>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    map_install_simt_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(p);
  }
  return cudaGetLastError();
}

// ------------------------- cross-GPU chunk handshake -------------------------
// One-thread kernels that order a chunk pipeline between two GPUs through a
// 64-bit counter in device memory (the counter may be a peer's, mapped
// through CUDA IPC). They replace the reference's per-block ready / ACK
// messages over a Unix socket (source_mapper_adapter.py:197-232
// _DoubleBufferedSender.offer, :282-324 _DoubleBufferedReceiver.next /
// acknowledge) with device-side signals, so no host round trip sits between
// chunks.

// Publish `value` after every write of the preceding kernels on this stream:
// the fence orders them (system scope, peers included) before the store.
__global__ void signal_kernel(unsigned long long* flag, long long value) {
  __threadfence_system();
  asm volatile("st.release.sys.global.b64 [%0], %1;" ::"l"(flag), "l"(value) : "memory");
}

// Wait until *flag >= value (acquire, system scope). Bounded: after
// timeout_ns the kernel records CB_DEV_ERR_TIMEOUT and returns, so a lost peer
// ends the pipeline with an error instead of a hung stream.
__global__ void wait_kernel(const unsigned long long* flag, long long value, long long timeout_ns,
                            int32_t* status) {
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    long long v;
    asm volatile("ld.acquire.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
    if (v >= value) return;
    if (static_cast<long long>(global_timer_ns() - t0) > timeout_ns) {
      flag_error(status, CB_DEV_ERR_TIMEOUT);
      return;
    }
    __nanosleep(256);
  }
}

cudaError_t launch_signal(unsigned long long* flag, long long value, cudaStream_t st) {
  signal_kernel<<<1, 1, 0, st>>>(flag, value);
  return cudaGetLastError();
}

cudaError_t launch_wait(const unsigned long long* flag, long long value, long long timeout_ns, int32_t* status,
                        cudaStream_t st) {
  wait_kernel<<<1, 1, 0, st>>>(flag, value, timeout_ns, status);
  return cudaGetLastError();
}

}  // namespace cbk
