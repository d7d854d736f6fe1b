// Fused CacheBridge mapper apply + paged-KV install on tcgen05 tensor cores.
//
// Computes, for every target layer l, target head h of this rank, kind
// (K or V) and token t, the headwise affine map of the reference
// (src/cachebridge/mapper.py:153-181, 207-239):
//     y[t] = concat_j x_kind[sel[l][j]][t][h] @ W_kind[l][h] + b_kind[l][h]
// then target RoPE on keys, BF16 rounding, and a store of the 256-byte head
// row straight into the target pool row dst_slots[t]
// (online/blocks.py:86-111 set_kv_buffer; source_mapper_adapter.py:389-425).
// Keys read the content-space (source-RoPE-removed, BF16-rounded) rows that
// cb_derotate.cu packed into the workspace; values read the source pool rows
// directly through src_slots (the gather of online/blocks.py:47-82).
//
// Work unit ("item"): (head h, kind, chunk of R*128 tokens, target layer l).
// Items are ordered head/kind-major, then chunk, then layer, so the CTAs that
// run concurrently share one head/kind's source rows of one token window
// (each source row feeds ~L_t*S/L_s target layers and is read from HBM once)
// and that head/kind's weights (L_t*S*32 KB) stay resident in L2.
//
// CTA (persistent, one per SM, 320 threads) roles:
//   warps 0-3  producers: 16-byte cp.async gathers of 128 token rows x 256 B
//              per k-block into a 128B-swizzled K-major stage (ring of NS).
//   warps 4-7  epilogue: tcgen05.ld of the FP32 accumulator (one token row per
//              thread), + bias, target RoPE (K), BF16, staging through a
//              swizzled 8 KB/warp buffer, then row-coalesced 16-byte stores
//              (two 256-byte rows per warp instruction) to the pool rows.
//   warp 8     TMEM owner + single-thread tcgen05.mma issuer (M=128, N=128,
//              K=16 steps; 8 steps per 128-feature k-block).
//   warp 9     weight loader: one bulk copy per 32 KB weight k-block (the
//              pre-swizzled image built at upload); resident for the whole
//              item when S <= 4, streamed per m-tile otherwise.
// Accumulators: 2 x (128 lanes x 128 fp32 columns) in TMEM, so the epilogue of
// m-tile i overlaps the MMAs of m-tile i+1.
#include "cb_device.cuh"
#include "cb_map_tc.cuh"

namespace cbk {

namespace {

constexpr int kBarFull = 0;       // [4]  producers -> MMA (A stage filled)
constexpr int kBarEmpty = 4;      // [4]  MMA -> producers (A stage consumed)
constexpr int kBarWFull = 8;      // [4]  loader -> MMA (weight slot filled)
constexpr int kBarWEmpty = 12;    // [4]  MMA -> loader (weight slot consumed)
constexpr int kBarAccFull = 16;   // [2]  MMA -> epilogue (accumulator ready)
constexpr int kBarAccEmpty = 18;  // [2]  epilogue -> MMA (accumulator drained)
constexpr int kBarDone = 20;      // [1]  MMA drain at exit
constexpr int kNumBars = 24;

struct Item {
  int kind;   // 0 = K, 1 = V
  int h;      // head within this call
  int l;      // target layer
  int tok0;   // first token of the chunk
  int mtiles; // valid 128-token m-tiles in the chunk
};

__device__ __forceinline__ Item decode_item(const MapTcParams& p, int i) {
  Item it;
  const int per_hk = p.n_chunks * p.L_t;
  const int hk = i / per_hk;
  const int rem = i - hk * per_hk;
  const int c = rem / p.L_t;
  it.l = rem - c * p.L_t;
  it.h = hk >> 1;
  it.kind = hk & 1;
  it.tok0 = c * p.R * kBM;
  const int remaining = p.n_tokens - it.tok0;
  const int mt = (remaining + kBM - 1) / kBM;
  it.mtiles = mt < p.R ? mt : p.R;
  return it;
}

struct Smem {
  uint32_t w;     // weight slots base (shared::cta address)
  uint32_t a;     // A stages base
  uint32_t e;     // epilogue staging base
  uint8_t* e_gen; // generic pointer to epilogue staging
  uint32_t bars;  // mbarrier array base
  uint32_t* tmem_holder;
  volatile int* abort_flag;
};

__device__ __forceinline__ uint32_t bar_at(const Smem& s, int idx) { return s.bars + 8u * idx; }

// ------------------------------- producers ---------------------------------
__device__ void run_producer(const MapTcParams& p, const Smem& s, int pw, int lane) {
  const int NS = p.stages;
  const int LAG = p.stages - 1;
  int issued = 0, finished = 0;
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    for (int m = 0; m < it.mtiles && ok; ++m) {
      // This lane's token row of the m-tile (row = pw*32 + lane).
      const int t = it.tok0 + m * kBM + pw * 32 + lane;
      int valid = t < p.n_tokens;
      int64_t srow = t;
      if (it.kind == 1 && valid) {
        srow = load_slot(p.src_slots, p.src_slot_dtype, t);
        if (srow < 0 || srow >= p.src_rows) {
          flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
          valid = 0;
        }
      }
      for (int j = 0; j < p.S; ++j) {
        const int stage = issued % NS;
        // Warp-uniform outcome: the gather below uses full-warp shuffles.
        const bool got = mbar_wait(bar_at(s, kBarEmpty + stage), ((issued / NS) & 1) ^ 1,
                                   s.abort_flag, p.status);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const char* base;
        int64_t stride_bytes;
        if (it.kind == 0) {
          const int u = __ldg(p.sel_local + it.l * p.S + j);
          base = reinterpret_cast<const char*>(p.ws_k) +
                 ((static_cast<int64_t>(u) * p.n_tokens) * p.H + it.h) * (kD * 2);
          stride_bytes = static_cast<int64_t>(p.H) * kD * 2;
        } else {
          const int sl = __ldg(p.sel_global + it.l * p.S + j);
          base = reinterpret_cast<const char*>(p.src_v[sl]) +
                 static_cast<int64_t>(p.src_head_offset + it.h) * (kD * 2);
          stride_bytes = p.src_row_stride * 2;
        }
        const uint32_t stage_addr = s.a + stage * kKBlockBytes;
        const int c = lane & 15;
#pragma unroll
        for (int ii = 0; ii < 16; ++ii) {
          const int r = 2 * ii + (lane >> 4);
          const int64_t rr = __shfl_sync(0xffffffffu, srow, r);
          const int vv = __shfl_sync(0xffffffffu, valid, r);
          const int row = pw * 32 + r;
          const char* g = base + (vv ? rr * stride_bytes : 0) + c * 16;
          const uint32_t dst =
              stage_addr + (c >> 3) * kPanelBytes + row * 128 + (((c & 7) ^ (row & 7)) << 4);
          cp_async_16(dst, g, vv ? 16u : 0u);
        }
        cp_async_commit();
        ++issued;
        if (issued - finished > LAG) {
          cp_async_wait_dyn(LAG);
          fence_proxy_async_smem();
          mbar_arrive(bar_at(s, kBarFull + (finished % NS)));
          ++finished;
        }
      }
    }
  }
  // Drain: every issued group completes (plain loads always finish).
  cp_async_wait<0>();
  fence_proxy_async_smem();
  while (finished < issued) {
    mbar_arrive(bar_at(s, kBarFull + (finished % NS)));
    ++finished;
  }
}

// ------------------------------ weight loader ------------------------------
__device__ void run_weight_loader(const MapTcParams& p, const Smem& s) {
  const uint64_t policy = l2_policy_evict_last();
  int wq = 0, itc = 0;
  bool ok = true;
  // Track the last load issued into each slot so an aborted CTA can wait for
  // its own bulk copies before exiting.
  int last_par[4] = {-1, -1, -1, -1};
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    const uint8_t* wu =
        p.w_img + (static_cast<int64_t>((it.kind * p.L_t + it.l) * p.H + it.h) * p.S) * kKBlockBytes;
    if (p.w_resident) {
      for (int j = 0; j < p.S; ++j) {
        if (!mbar_wait(bar_at(s, kBarWEmpty + j), (itc & 1) ^ 1, s.abort_flag, p.status)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_at(s, kBarWFull + j), kKBlockBytes);
        bulk_copy_g2s(s.w + j * kKBlockBytes, wu + static_cast<int64_t>(j) * kKBlockBytes,
                      kKBlockBytes, bar_at(s, kBarWFull + j), policy);
        last_par[j] = itc & 1;
      }
    } else {
      for (int m = 0; m < it.mtiles && ok; ++m) {
        for (int j = 0; j < p.S; ++j) {
          const int slot = wq & 1;
          if (!mbar_wait(bar_at(s, kBarWEmpty + slot), ((wq >> 1) & 1) ^ 1, s.abort_flag,
                         p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_at(s, kBarWFull + slot), kKBlockBytes);
          bulk_copy_g2s(s.w + slot * kKBlockBytes, wu + static_cast<int64_t>(j) * kKBlockBytes,
                        kKBlockBytes, bar_at(s, kBarWFull + slot), policy);
          last_par[slot] = (wq >> 1) & 1;
          ++wq;
        }
      }
    }
    ++itc;
  }
  if (!ok) {
    // Aborted: wait (bounded) for this thread's own copies still in flight.
    const uint64_t t0 = global_timer_ns();
    for (int slot = 0; slot < 4; ++slot) {
      if (last_par[slot] < 0) continue;
      while (!mbar_try_wait(bar_at(s, kBarWFull + slot), last_par[slot])) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) break;
      }
    }
  }
}

// ------------------------------- MMA issuer --------------------------------
__device__ void run_mma(const MapTcParams& p, const Smem& s, uint32_t tmem_base) {
  constexpr uint32_t idesc = make_idesc_bf16_f32(kBM, kD);
  const int NS = p.stages;
  int q = 0, wq = 0, accc = 0, itc = 0;
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    for (int m = 0; m < it.mtiles && ok; ++m) {
      const int acc = accc & 1;
      if (!mbar_wait(bar_at(s, kBarAccEmpty + acc), ((accc >> 1) & 1) ^ 1, s.abort_flag,
                     p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kD;
      for (int j = 0; j < p.S; ++j) {
        int wslot;
        if (p.w_resident) {
          wslot = j;
          if (m == 0) {
            if (!mbar_wait(bar_at(s, kBarWFull + j), itc & 1, s.abort_flag, p.status)) {
              ok = false;
              break;
            }
          }
        } else {
          wslot = wq & 1;
          if (!mbar_wait(bar_at(s, kBarWFull + wslot), (wq >> 1) & 1, s.abort_flag, p.status)) {
            ok = false;
            break;
          }
        }
        const int stage = q % NS;
        if (!mbar_wait(bar_at(s, kBarFull + stage), (q / NS) & 1, s.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = s.a + stage * kKBlockBytes;
        const uint32_t b0 = s.w + wslot * kKBlockBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kPanelBytes + (kk & 3) * 32;
          umma_bf16(d_tmem, make_sw128_kmajor_desc(a0 + off), make_sw128_kmajor_desc(b0 + off),
                    idesc, (j | kk) != 0 ? 1u : 0u);
        }
        umma_commit(bar_at(s, kBarEmpty + stage));
        if (!p.w_resident) {
          umma_commit(bar_at(s, kBarWEmpty + wslot));
          ++wq;
        }
        ++q;
      }
      if (!ok) break;
      umma_commit(bar_at(s, kBarAccFull + acc));
      ++accc;
    }
    if (ok && p.w_resident) {
      for (int j = 0; j < p.S; ++j) umma_commit(bar_at(s, kBarWEmpty + j));
    }
    ++itc;
  }
  // Drain every MMA issued by this thread before TMEM is released.
  umma_commit(bar_at(s, kBarDone));
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar_at(s, kBarDone), 0)) {
    if (global_timer_ns() - t0 > kWaitTimeoutNs) {
      flag_error(p.status, CB_DEV_ERR_TIMEOUT);
      break;
    }
  }
}

// -------------------------------- epilogue ---------------------------------
__device__ void run_epilogue(const MapTcParams& p, const Smem& s, uint32_t tmem_base, int eq,
                             int lane) {
  uint8_t* stage_gen = s.e_gen + eq * kEpiWarpBytes;
  const uint32_t stage_s = s.e + eq * kEpiWarpBytes;
  int accc = 0;
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    const float* bias = p.bias + (static_cast<int64_t>(it.kind * p.L_t + it.l) * p.H + it.h) * kD;
    char* dst_layer = reinterpret_cast<char*>(it.kind ? p.dst_v[it.l] : p.dst_k[it.l]) +
                      static_cast<int64_t>(p.dst_head_offset + it.h) * (kD * 2);
    const int64_t dst_stride_bytes = p.dst_row_stride * 2;
    for (int m = 0; m < it.mtiles; ++m) {
      const int acc = accc & 1;
      // Warp-uniform outcome: tcgen05.ld is .sync.aligned across the warp.
      const bool got = mbar_wait(bar_at(s, kBarAccFull + acc), (accc >> 1) & 1, s.abort_flag, p.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int row = eq * 32 + lane;
      const int t = it.tok0 + m * kBM + row;
      int valid = t < p.n_tokens;
      int64_t dslot = 0;
      if (valid) {
        dslot = load_slot(p.dst_slots, p.dst_slot_dtype, t);
        if (dslot < 0 || dslot >= p.dst_rows) {
          flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
          valid = 0;
        }
      }
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(eq * 32) << 16) + acc * kD;
      uint8_t* my_row = stage_gen + lane * 256;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t lo[32], hi[32];
        tmem_ld_32x32b_x32(tbase + half * 32, lo);
        tmem_ld_32x32b_x32(tbase + 64 + half * 32, hi);
        tmem_wait_ld();
        if (half == 1) {
          // Accumulator fully read into registers: hand it back to the MMA.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_at(s, kBarAccEmpty + acc));
        }
        float ylo[32], yhi[32];
#pragma unroll
        for (int q4 = 0; q4 < 8; ++q4) {
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + half * 32) + q4);
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + 64 + half * 32) + q4);
          ylo[4 * q4 + 0] = __fadd_rn(__uint_as_float(lo[4 * q4 + 0]), b0.x);
          ylo[4 * q4 + 1] = __fadd_rn(__uint_as_float(lo[4 * q4 + 1]), b0.y);
          ylo[4 * q4 + 2] = __fadd_rn(__uint_as_float(lo[4 * q4 + 2]), b0.z);
          ylo[4 * q4 + 3] = __fadd_rn(__uint_as_float(lo[4 * q4 + 3]), b0.w);
          yhi[4 * q4 + 0] = __fadd_rn(__uint_as_float(hi[4 * q4 + 0]), b1.x);
          yhi[4 * q4 + 1] = __fadd_rn(__uint_as_float(hi[4 * q4 + 1]), b1.y);
          yhi[4 * q4 + 2] = __fadd_rn(__uint_as_float(hi[4 * q4 + 2]), b1.z);
          yhi[4 * q4 + 3] = __fadd_rn(__uint_as_float(hi[4 * q4 + 3]), b1.w);
        }
        if (it.kind == 0 && valid) {
          const float4* cp = reinterpret_cast<const float4*>(p.dcos + static_cast<int64_t>(t) * 64 + half * 32);
          const float4* sp = reinterpret_cast<const float4*>(p.dsin + static_cast<int64_t>(t) * 64 + half * 32);
#pragma unroll
          for (int q4 = 0; q4 < 8; ++q4) {
            const float4 c4 = __ldg(cp + q4);
            const float4 s4 = __ldg(sp + q4);
            const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
            const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float o0, o1;
              rope_apply_pair(ylo[4 * q4 + e], yhi[4 * q4 + e], cc[e], ss[e], o0, o1);
              ylo[4 * q4 + e] = o0;
              yhi[4 * q4 + e] = o1;
            }
          }
        }
        // Stage this thread's row: logical 16-byte chunk c of the 256-byte row
        // sits at physical chunk (c & 8) | ((c & 7) ^ (lane & 7)).
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          uint4 vlo, vhi;
          vlo.x = pack_bf16x2(ylo[8 * k + 0], ylo[8 * k + 1]);
          vlo.y = pack_bf16x2(ylo[8 * k + 2], ylo[8 * k + 3]);
          vlo.z = pack_bf16x2(ylo[8 * k + 4], ylo[8 * k + 5]);
          vlo.w = pack_bf16x2(ylo[8 * k + 6], ylo[8 * k + 7]);
          vhi.x = pack_bf16x2(yhi[8 * k + 0], yhi[8 * k + 1]);
          vhi.y = pack_bf16x2(yhi[8 * k + 2], yhi[8 * k + 3]);
          vhi.z = pack_bf16x2(yhi[8 * k + 4], yhi[8 * k + 5]);
          vhi.w = pack_bf16x2(yhi[8 * k + 6], yhi[8 * k + 7]);
          const int clo = half * 4 + k;       // chunks 0..7
          const int chi = 8 + half * 4 + k;   // chunks 8..15
          *reinterpret_cast<uint4*>(my_row + ((((clo & 7) ^ (lane & 7))) << 4)) = vlo;
          *reinterpret_cast<uint4*>(my_row + ((8 | ((chi & 7) ^ (lane & 7))) << 4)) = vhi;
        }
      }
      __syncwarp();
      // Row-coalesced stores: lanes 0-15 write row 2i, lanes 16-31 row 2i+1.
      const int c = lane & 15;
#pragma unroll 4
      for (int ii = 0; ii < 16; ++ii) {
        const int r = 2 * ii + (lane >> 4);
        const int64_t sl = __shfl_sync(0xffffffffu, dslot, r);
        const int vv = __shfl_sync(0xffffffffu, valid, r);
        const uint4 v = *reinterpret_cast<const uint4*>(stage_gen + r * 256 +
                                                        (((c & 8) | ((c & 7) ^ (r & 7))) << 4));
        if (vv) {
          *reinterpret_cast<uint4*>(dst_layer + sl * dst_stride_bytes + c * 16) = v;
        }
      }
      __syncwarp();
      ++accc;
    }
  }
  (void)stage_s;
}

}  // namespace

__global__ void __launch_bounds__(kTcThreads, 1) map_install_tc_kernel(const __grid_constant__ MapTcParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align the dynamic window to 1024 B (128B-swizzle atoms need it).
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_gen = smem_raw + (base - raw);

  Smem s;
  s.w = base;
  s.a = base + p.w_slots * kKBlockBytes;
  s.e = s.a + p.stages * kKBlockBytes;
  s.e_gen = base_gen + (s.e - base);
  s.bars = s.e + 4 * kEpiWarpBytes;
  uint8_t* bars_gen = base_gen + (s.bars - base);
  s.tmem_holder = reinterpret_cast<uint32_t*>(bars_gen + 8 * kNumBars);
  s.abort_flag = reinterpret_cast<volatile int*>(bars_gen + 8 * kNumBars + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(bar_at(s, kBarFull + i), 128);
      mbar_init(bar_at(s, kBarEmpty + i), 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(bar_at(s, kBarWFull + i), 1);
      mbar_init(bar_at(s, kBarWEmpty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_at(s, kBarAccFull + i), 1);
      mbar_init(bar_at(s, kBarAccEmpty + i), 4);
    }
    mbar_init(bar_at(s, kBarDone), 1);
    *s.abort_flag = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 8) {
    tmem_alloc(smem_u32(s.tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_holder;

  if (warp < 4) {
    run_producer(p, s, warp, lane);
  } else if (warp < 8) {
    run_epilogue(p, s, tmem_base, warp - 4, lane);
  } else if (warp == 8) {
    if (lane == 0) run_mma(p, s, tmem_base);
    __syncwarp();
  } else {
    if (lane == 0) run_weight_loader(p, s);
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace cbk
