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
// derotate_pack_kernel (cb_kernels.cu) packed into the workspace; values read the source pool rows
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
//   warps 4-11 epilogue, two groups of four warps that take alternate
//              m-tiles; in a group, warp q reads TMEM lane quarter q (token
//              rows 32q..32q+31, one row per thread). Per 32-pair half row:
//              two tcgen05.ld rounds of 16 RoPE pairs (columns i and i+64),
//              + bias, target RoPE (K), BF16, staging into the warp's
//              swizzled 32 x 128 B tile, then 16-byte stores of 4 rows x
//              (2 x 64 B) per warp instruction.
//   warp 12    TMEM owner + single-thread tcgen05.mma issuer (M=128, N=128,
//              K=16 steps; 8 steps per 128-feature k-block).
//   warp 13    weight loader: one bulk copy per 32 KB weight k-block (the
//              pre-swizzled image built at upload); resident for the whole
//              item when S <= 4, streamed per m-tile otherwise.
// Accumulators: 4 x (128 lanes x 128 fp32 columns) in TMEM (all 512 columns),
// so the MMAs run up to three m-tiles ahead of the two epilogue groups.
#include "cb_device.cuh"
#include "cb_map_tc.cuh"

namespace cbk {

namespace {

constexpr int kBarFull = 0;       // [4]  producers -> MMA (A stage filled)
constexpr int kBarEmpty = 4;      // [4]  MMA -> producers (A stage consumed)
constexpr int kBarWFull = 8;      // [4]  loader -> MMA (weight slot filled)
constexpr int kBarWEmpty = 12;    // [4]  MMA -> loader (weight slot consumed)
constexpr int kBarAccFull = 16;   // [4]  MMA -> epilogue (accumulator ready)
constexpr int kBarAccEmpty = 20;  // [4]  epilogue -> MMA (accumulator drained)
constexpr int kBarDone = 24;      // [1]  MMA drain at exit
constexpr int kNumBars = 32;

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
  int issued = 0;
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    // Slot of this lane's token row, prefetched one m-tile ahead.
    const int lane_row = pw * 32 + lane;
    int next_t = it.tok0 + lane_row;
    int next_valid = next_t < p.n_tokens;
    int64_t next_row = next_t;
    if (it.kind == 1 && next_valid) next_row = load_slot(p.src_slots, p.src_slot_dtype, next_t);
    for (int m = 0; m < it.mtiles && ok; ++m) {
      int valid = next_valid;
      int64_t srow = next_row;
      if (m + 1 < it.mtiles) {
        next_t += kBM;
        next_valid = next_t < p.n_tokens;
        next_row = next_t;
        if (it.kind == 1 && next_valid) next_row = load_slot(p.src_slots, p.src_slot_dtype, next_t);
      }
      if (it.kind == 1 && valid && (srow < 0 || srow >= p.src_rows)) {
        flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
        valid = 0;
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
        // The stage's full barrier (count 128) completes when every producer
        // thread's copies have landed, independently of the producer's progress.
        cp_async_arrive_noinc(bar_at(s, kBarFull + stage));
        ++issued;
      }
    }
  }
  // Never exit with copies in flight into shared memory.
  cp_async_wait_all();
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
      const int acc = accc & 3;
      if (!mbar_wait(bar_at(s, kBarAccEmpty + acc), ((accc >> 2) & 1) ^ 1, s.abort_flag,
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
__device__ __forceinline__ void load16(const float* src, float (&out)[16]) {
  const float4* v = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 x = __ldg(v + q);
    out[4 * q + 0] = x.x;
    out[4 * q + 1] = x.y;
    out[4 * q + 2] = x.z;
    out[4 * q + 3] = x.w;
  }
}

// Warp (group g, quarter eq): m-tiles n with n % 2 == g, token rows eq*32 + lane.
// Target RoPE coefficients come from the frequency-major table [64][n] that
// phase 1 wrote: one load instruction fetches one frequency for the warp's 32
// consecutive tokens (one 128-byte line); the next round's 16 are fetched while
// the current round computes.
__device__ __forceinline__ void load_rope16(const float* cos_row0, const float* sin_row0, int64_t rs,
                                            float (&c)[16], float (&s)[16]) {
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    c[e] = __ldg(cos_row0 + e * rs);
    s[e] = __ldg(sin_row0 + e * rs);
  }
}

__device__ void run_epilogue(const MapTcParams& p, const Smem& s, uint32_t tmem_base, int g, int eq,
                             int lane) {
  uint8_t* stage = s.e_gen + (g * 4 + eq) * kEpiWarpBytes;  // 32 rows x 128 B, this warp only
  uint8_t* my_row = stage + lane * 128;
  const int64_t dst_stride_bytes = p.dst_row_stride * 2;
  const int64_t rs = p.n_tokens;
  int accc = 0;  // CTA-wide m-tile counter (both groups count every m-tile)
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    const float* bias = p.bias + (static_cast<int64_t>(it.kind * p.L_t + it.l) * p.H + it.h) * kD;
    char* dst_layer = reinterpret_cast<char*>(it.kind ? p.dst_v[it.l] : p.dst_k[it.l]) +
                      static_cast<int64_t>(p.dst_head_offset + it.h) * (kD * 2);
    for (int m = 0; m < it.mtiles; ++m, ++accc) {
      if ((accc & 1) != g) continue;
      const int t = it.tok0 + m * kBM + eq * 32 + lane;
      int valid = t < p.n_tokens;
      int64_t dslot = valid ? load_slot(p.dst_slots, p.dst_slot_dtype, t) : 0;
      if (valid && (dslot < 0 || dslot >= p.dst_rows)) {
        flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
        valid = 0;
      }
      const bool do_rope = it.kind == 0 && valid;
      const float* cbase = p.dcos + t;
      const float* sbase = p.dsin + t;
      float ca[16], sa[16];  // coefficients of the current 16-pair round
      if (do_rope) load_rope16(cbase, sbase, rs, ca, sa);
      const int acc = accc & 3;
      // Warp-uniform outcome: tcgen05.ld is .sync.aligned across the warp.
      const bool got = mbar_wait(bar_at(s, kBarAccFull + acc), (accc >> 2) & 1, s.abort_flag, p.status);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(eq * 32) << 16) + acc * kD;
#pragma unroll
      for (int hb = 0; hb < 2; ++hb) {  // RoPE pairs [32hb, 32hb+32)
#pragma unroll
        for (int sr = 0; sr < 2; ++sr) {  // 16-pair round
          const int p0 = 32 * hb + 16 * sr;  // first pair of the round
          uint32_t lo[16], hi[16];
          tmem_ld_32x32b_x16(tbase + p0, lo);
          tmem_ld_32x32b_x16(tbase + 64 + p0, hi);
          float cb[16], sb[16];  // next round's coefficients, fetched while this one computes
          const bool prefetch = do_rope && p0 + 16 < 64;
          if (prefetch) load_rope16(cbase + (p0 + 16) * rs, sbase + (p0 + 16) * rs, rs, cb, sb);
          tmem_wait_ld();
          if (hb == 1 && sr == 1) {
            // Accumulator fully read into registers: hand it back to the MMA.
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_at(s, kBarAccEmpty + acc));
          }
          float blo[16], bhi[16];
          load16(bias + p0, blo);
          load16(bias + 64 + p0, bhi);
          float ylo[16], yhi[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            ylo[e] = __fadd_rn(__uint_as_float(lo[e]), blo[e]);
            yhi[e] = __fadd_rn(__uint_as_float(hi[e]), bhi[e]);
          }
          if (do_rope) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              float o0, o1;
              rope_apply_pair(ylo[e], yhi[e], ca[e], sa[e], o0, o1);
              ylo[e] = o0;
              yhi[e] = o1;
            }
          }
          if (prefetch) {
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              ca[e] = cb[e];
              sa[e] = sb[e];
            }
          }
          // Local chunk lc of the warp's 128-byte row piece: 0-3 = columns
          // [32hb, 32hb+32), 4-7 = [64+32hb, ...); it sits at lc ^ (row & 7).
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            uint4 vlo, vhi;
            vlo.x = pack_bf16x2(ylo[8 * k + 0], ylo[8 * k + 1]);
            vlo.y = pack_bf16x2(ylo[8 * k + 2], ylo[8 * k + 3]);
            vlo.z = pack_bf16x2(ylo[8 * k + 4], ylo[8 * k + 5]);
            vlo.w = pack_bf16x2(ylo[8 * k + 6], ylo[8 * k + 7]);
            vhi.x = pack_bf16x2(yhi[8 * k + 0], yhi[8 * k + 1]);
            vhi.y = pack_bf16x2(yhi[8 * k + 2], yhi[8 * k + 3]);
            vhi.z = pack_bf16x2(yhi[8 * k + 4], yhi[8 * k + 5]);
            vhi.w = pack_bf16x2(yhi[8 * k + 6], yhi[8 * k + 7]);
            const int llo = 2 * sr + k;
            const int lhi = 4 + 2 * sr + k;
            *reinterpret_cast<uint4*>(my_row + ((llo ^ (lane & 7)) << 4)) = vlo;
            *reinterpret_cast<uint4*>(my_row + ((lhi ^ (lane & 7)) << 4)) = vhi;
          }
        }
        __syncwarp();
        // Stores: 4 rows x (2 x 64 contiguous bytes) per warp instruction.
        const int lc = lane & 7;
        const int gchunk = lc < 4 ? 4 * hb + lc : 8 + 4 * hb + (lc - 4);
#pragma unroll
        for (int ii = 0; ii < 8; ++ii) {
          const int rr = 4 * ii + (lane >> 3);
          const int64_t sl = __shfl_sync(0xffffffffu, dslot, rr);
          const int vv = __shfl_sync(0xffffffffu, valid, rr);
          const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((lc ^ (rr & 7)) << 4));
          if (vv) *reinterpret_cast<uint4*>(dst_layer + sl * dst_stride_bytes + gchunk * 16) = v;
        }
        __syncwarp();
      }
    }
  }
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
  s.bars = s.e + kEpiWarps * kEpiWarpBytes;
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
    for (int i = 0; i < kAccBufs; ++i) {
      mbar_init(bar_at(s, kBarAccFull + i), 1);
      mbar_init(bar_at(s, kBarAccEmpty + i), 4);  // the 4 warps of the group that owns the m-tile
    }
    mbar_init(bar_at(s, kBarDone), 1);
    *s.abort_flag = 0;
    fence_mbarrier_init();
    fence_proxy_async_smem();
  }
  constexpr int kMmaWarp = 4 + kEpiWarps;
  constexpr int kLoaderWarp = kMmaWarp + 1;
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(s.tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_holder;

  if (warp < 4) {
    run_producer(p, s, warp, lane);
  } else if (warp < kMmaWarp) {
    // TMEM lane quarter = warp % 4 (tcgen05.ld lane-access rule); group = (warp - 4) / 4.
    run_epilogue(p, s, tmem_base, (warp - 4) >> 2, warp & 3, lane);
  } else if (warp == kMmaWarp) {
    if (lane == 0) run_mma(p, s, tmem_base);
    __syncwarp();
  } else if (warp == kLoaderWarp) {
    if (lane == 0) run_weight_loader(p, s);
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

}  // namespace cbk
