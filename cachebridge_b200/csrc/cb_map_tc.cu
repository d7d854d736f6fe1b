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
// derotate_pack_kernel (cb_kernels.cu) packed into the workspace; values read
// the source pool rows directly through src_slots (the gather of
// online/blocks.py:47-82).
//
// Work unit ("item"): (head h, kind, chunk of R*128 tokens, target layer l).
// Items are ordered head/kind-major, then chunk, then layer, so the CTAs that
// run concurrently share one head/kind's source rows of one token window
// (each source row feeds ~L_t*S/L_s target layers and is read from HBM once)
// and that head/kind's weights stay resident in L2.
//
// CTA (persistent, one per SM, 576 threads) roles:
//   warps 0-3   producers: per k-block one 32 KB stage (ring of NS) in the
//               UMMA 128B-swizzled K-major layout: keys by two 4-D TMA tiled
//               loads from the workspace, values by 16-byte cp.async gathers
//               of the source pool rows through the slot table.
//   warps 4-15  epilogue: three groups of four warps; group g takes the m-tiles
//               n with n % 3 == g (TMEM accumulator n % 4). In a
//               group, warp w reads TMEM lane quarter w % 4 (token rows, one
//               per thread), in four rounds of 16 RoPE pairs (columns i and
//               i+64): target RoPE for keys (sin/cos of the exact FP32 phase
//               after a Cody-Waite reduction by pi), BF16 packing into a
//               swizzled 32 x 128 B staging tile that collects two rounds,
//               then 16-byte stores of 4 rows x (2 x 64 B) per warp
//               instruction, so two store instructions touch each row per
//               m-tile; into this GPU's own pool with an L2 evict-first
//               policy, so the stores do not push shared source rows out.
//   warp 16     TMEM owner + single-thread tcgen05.mma issuer: per m-tile one
//               K=16 step that loads the bias (a constant ones column times a
//               [bias_hi, bias_lo] block), then 8 K=16 steps per 128-feature
//               k-block (M=128, N=128, BF16 in, FP32 accumulate).
//   warp 17     weight loader: bulk copies of the unit's 4 KB bias block and
//               its 32 KB W^T k-blocks (the pre-swizzled image built at
//               upload); resident for the whole item when they fit, streamed
//               per m-tile otherwise.
// Every wait is bounded (kWaitTimeoutNs): an expired wait flags
// CB_DEV_ERR_TIMEOUT and the CTA unwinds instead of hanging.
#include "cb_device.cuh"
#include "cb_map_tc.cuh"
#include "cb_pipeline.cuh"

namespace cbk {

namespace {

constexpr int kBarFull = 0;       // [4]  producers -> MMA (A stage filled)
constexpr int kBarEmpty = 4;      // [4]  MMA -> producers (A stage consumed)
constexpr int kBarWFull = 8;      // [4]  loader -> MMA (weight slot filled)
constexpr int kBarWEmpty = 12;    // [4]  MMA -> loader (weight slot consumed)
constexpr int kBarAccFull = 16;   // [4]  MMA -> epilogue group (accumulator ready)
constexpr int kBarAccEmpty = 20;  // [4]  epilogue group -> MMA (accumulator drained)
constexpr int kBarBFull = 24;     // [1]  loader -> MMA (bias block filled)
constexpr int kBarBEmpty = 25;    // [1]  MMA -> loader (bias block consumed)
constexpr int kBarDone = 26;      // [1]  MMA drain at exit
constexpr int kNumBars = 32;

struct Smem {
  uint32_t w;      // weight slots (shared::cta address)
  uint32_t bias;   // bias block slot
  uint32_t a;      // A stages
  uint32_t ones;   // constant ones block
  uint8_t* e_gen;  // epilogue staging (generic pointer)
  uint32_t bars;   // mbarrier array
  uint32_t* tmem_holder;
  volatile int* abort_flag;
};

__device__ __forceinline__ uint32_t bar_at(const Smem& s, int idx) { return s.bars + 8u * idx; }

// cos and sin of an FP32 phase up to a sign: Cody-Waite reduction by pi
// (k = rint(phi / pi); r = phi - k*P1 - k*P2 with P1 = fl(pi) and
// P2 = fl(pi - P1); phi - k*P1 is exact inside the FMA), then the hardware
// sin/cos approximations on |r| <= pi/2 (__sincosf: absolute error below
// 2^-21 on [-pi, pi]). cos(phi) = (-1)^k cos(r) and sin(phi) = (-1)^k sin(r);
// `sign` is (-1)^k as an FP32 sign-bit mask, applied by the caller to the
// rotated pair. Within 4e-7 of cos/sin(phi) for |phi| < 4e5 (k stays an exact
// FP32 integer), far below the BF16 rounding of the output; calls with larger
// phases use sincosf (MapTcParams::trig_exact). Few issue slots and no shared
// memory: the epilogue warps share their schedulers with the MMA issuer.
__device__ __forceinline__ void sincos_half_turns(float phi, float& c, float& s, uint32_t& sign) {
  const float kOneOverPi = 0x1.45f306p-2f;  // fl(1 / pi)
  const float kP1 = 0x1.921fb6p+1f;         // fl(pi)
  const float kP2 = -0x1.777a5cp-24f;       // fl(pi - kP1)
  const float kf = rintf(phi * kOneOverPi);
  float r = fmaf(-kf, kP1, phi);
  r = fmaf(-kf, kP2, r);
  __sincosf(r, &s, &c);
  sign = static_cast<uint32_t>(static_cast<int>(kf)) << 31;
}

// ------------------------------ weight loader ------------------------------
__device__ void run_weight_loader(const MapTcParams& p, const Smem& s) {
  const uint64_t policy = l2_policy_evict_last();
  int wq = 0, itc = 0;
  bool ok = true;
  // The last load issued into each weight slot (and the bias slot, index 4),
  // so an aborted CTA can wait for its own bulk copies before exiting.
  int last_par[5] = {-1, -1, -1, -1, -1};
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    const uint8_t* wu = p.w_img + static_cast<int64_t>((it.kind * p.L_t + it.l) * p.H + it.h) * p.unit_bytes;
    if (!mbar_wait(bar_at(s, kBarBEmpty), (itc & 1) ^ 1, s.abort_flag, p.status)) break;
    mbar_arrive_expect_tx(bar_at(s, kBarBFull), kBiasBlockBytes);
    bulk_copy_g2s(s.bias, wu + static_cast<int64_t>(p.KB) * kKBlockBytes, kBiasBlockBytes, bar_at(s, kBarBFull),
                  policy);
    last_par[4] = itc & 1;
    if (p.w_resident) {
      for (int j = 0; j < p.KB; ++j) {
        if (!mbar_wait(bar_at(s, kBarWEmpty + j), (itc & 1) ^ 1, s.abort_flag, p.status)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_at(s, kBarWFull + j), kKBlockBytes);
        bulk_copy_g2s(s.w + j * kKBlockBytes, wu + static_cast<int64_t>(j) * kKBlockBytes, kKBlockBytes,
                      bar_at(s, kBarWFull + j), policy);
        last_par[j] = itc & 1;
      }
    } else {
      for (int m = 0; m < it.mtiles && ok; ++m) {
        for (int j = 0; j < p.KB; ++j) {
          const int slot = wq & 1;
          if (!mbar_wait(bar_at(s, kBarWEmpty + slot), ((wq >> 1) & 1) ^ 1, s.abort_flag, p.status)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_at(s, kBarWFull + slot), kKBlockBytes);
          bulk_copy_g2s(s.w + slot * kKBlockBytes, wu + static_cast<int64_t>(j) * kKBlockBytes, kKBlockBytes,
                        bar_at(s, kBarWFull + slot), policy);
          last_par[slot] = (wq >> 1) & 1;
          ++wq;
        }
      }
    }
    ++itc;
  }
  if (*s.abort_flag) {
    // Aborted: wait (bounded) for this thread's own copies still in flight.
    const uint64_t t0 = global_timer_ns();
    for (int k = 0; k < 5; ++k) {
      if (last_par[k] < 0) continue;
      const uint32_t bar = k < 4 ? bar_at(s, kBarWFull + k) : bar_at(s, kBarBFull);
      while (!mbar_try_wait(bar, last_par[k])) {
        if (global_timer_ns() - t0 > kWaitTimeoutNs) break;
      }
    }
  }
}

// ------------------------------- MMA issuer --------------------------------
__device__ void run_mma(const MapTcParams& p, const Smem& s, uint32_t tmem_base) {
  constexpr uint32_t idesc = make_idesc_bf16_f32(kBM, kD);
  const uint64_t ones_desc = make_noswizzle_k16_desc(s.ones);
  const uint64_t bias_desc = make_noswizzle_k16_desc(s.bias);
  // Descriptors of A stage 0 and weight slot 0: the start-address field holds
  // address >> 4 in 14 bits and every shared address here is below 256 KB, so
  // stage, slot and K-step offsets are plain additions of (bytes >> 4).
  const uint64_t a_desc0 = make_sw128_kmajor_desc(s.a);
  const uint64_t w_desc0 = make_sw128_kmajor_desc(s.w);
  constexpr uint64_t kBlockDesc = kKBlockBytes >> 4;
  const int NS = p.stages;
  int stage = 0;
  uint32_t phase = 0;
  int wq = 0, n = 0, itc = 0;
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    if (!mbar_wait(bar_at(s, kBarBFull), itc & 1, s.abort_flag, p.status)) break;
    for (int m = 0; m < it.mtiles && ok; ++m, ++n) {
      const int acc = n & 3;
      if (!mbar_wait(bar_at(s, kBarAccEmpty + acc), ((n >> 2) & 1) ^ 1, s.abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kD;
      // Accumulator := ones[:, 0:2] @ [bias_hi; bias_lo] = bias (FP32).
      umma_bf16(d_tmem, ones_desc, bias_desc, idesc, 0u);
      for (int j = 0; j < p.KB; ++j) {
        int wslot;
        if (p.w_resident) {
          wslot = j;
          if (m == 0 && !mbar_wait(bar_at(s, kBarWFull + j), itc & 1, s.abort_flag, p.status)) {
            ok = false;
            break;
          }
        } else {
          wslot = wq & 1;
          if (!mbar_wait(bar_at(s, kBarWFull + wslot), (wq >> 1) & 1, s.abort_flag, p.status)) {
            ok = false;
            break;
          }
        }
        if (!mbar_wait(bar_at(s, kBarFull + stage), phase, s.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Value stages were written by cp.async (generic proxy); the MMA reads
        // them through the async proxy.
        if (it.kind == 1) fence_proxy_async_smem();
        const uint64_t ad = a_desc0 + stage * kBlockDesc;
        const uint64_t bd = w_desc0 + wslot * kBlockDesc;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t off = static_cast<uint64_t>((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4;
          umma_bf16(d_tmem, ad + off, bd + off, idesc, 1u);
        }
        umma_commit(bar_at(s, kBarEmpty + stage));
        if (++stage == NS) {
          stage = 0;
          phase ^= 1u;
        }
        if (!p.w_resident) {
          umma_commit(bar_at(s, kBarWEmpty + wslot));
          ++wq;
        }
      }
      if (!ok) break;
      umma_commit(bar_at(s, kBarAccFull + acc));
    }
    if (ok) {
      umma_commit(bar_at(s, kBarBEmpty));
      if (p.w_resident)
        for (int j = 0; j < p.KB; ++j) umma_commit(bar_at(s, kBarWEmpty + j));
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
__device__ __forceinline__ uint4 pack8(const float* v) {
  uint4 r;
  r.x = pack_bf16x2(v[0], v[1]);
  r.y = pack_bf16x2(v[2], v[3]);
  r.z = pack_bf16x2(v[4], v[5]);
  r.w = pack_bf16x2(v[6], v[7]);
  return r;
}

// One m-tile of an epilogue group: item index i (decoded in it), m-tile m of
// the item, CTA m-tile counter n.
struct TileCursor {
  int i, m, n;
  Item it;
};

// Moves c forward by `step` m-tiles of the CTA's sequence, across items.
__device__ __forceinline__ void cursor_advance(const MapTcParams& p, TileCursor& c, int step) {
  c.m += step;
  c.n += step;
  while (c.i < p.num_items && c.m >= c.it.mtiles) {
    c.m -= c.it.mtiles;
    c.i += gridDim.x;
    if (c.i < p.num_items) c.it = decode_item(p, c.i);
  }
}

__device__ __forceinline__ int cursor_token_raw(const MapTcParams& p, const TileCursor& c, int row) {
  return c.i < p.num_items ? item_token_raw(p, c.it, c.m, row) : kNoToken;
}

// Warp (group g, lane quarter eq): the m-tiles n with n % 3 == g, token rows
// eq*32 + lane (one per thread), accumulator n % 4. The destination slot of
// the next m-tile is loaded while this one is processed.
__device__ void run_epilogue(const MapTcParams& p, const Smem& s, uint32_t tmem_base, int g, int eq, int lane) {
  uint8_t* stage = s.e_gen + (g * 4 + eq) * kEpiWarpBytes;  // 32 rows x 128 B, this warp only
  uint8_t* my_row = stage + lane * 128;
  const int my_key = lane & 7;  // staging swizzle of this lane's row
  const int64_t dst_stride_bytes = p.dst_row_stride * 2;
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(eq * 32) << 16);
  const int row_in_tile = eq * 32 + lane;
  const uint64_t store_policy = l2_policy_evict_first();  // mapped rows are not read again here
  TileCursor cur;
  cur.i = blockIdx.x;
  cur.m = 0;
  cur.n = 0;
  if (cur.i < p.num_items) cur.it = decode_item(p, cur.i);
  cursor_advance(p, cur, g);
  TileCursor nxt = cur;
  cursor_advance(p, nxt, kEpiGroups);
  int tok = check_token(p, cursor_token_raw(p, cur, row_in_tile));
  int64_t slot = tok >= 0 ? load_slot(p.dst_slots, p.dst_slot_dtype, tok) : 0;
  int raw_nxt = cursor_token_raw(p, nxt, row_in_tile);
  while (cur.i < p.num_items) {
    TileCursor after = nxt;
    cursor_advance(p, after, kEpiGroups);
    const int tok_nxt = check_token(p, raw_nxt);
    const int64_t slot_nxt = tok_nxt >= 0 ? load_slot(p.dst_slots, p.dst_slot_dtype, tok_nxt) : 0;
    raw_nxt = cursor_token_raw(p, after, row_in_tile);

    const Item& it = cur.it;
    const int n = cur.n;
    const int acc = n & 3;  // accumulator buffer of this m-tile
    const uint32_t tbase = lane_base + acc * kD;
    char* row_ptr = nullptr;  // this lane's destination row, or null
    if (tok >= 0) {
      if (slot < 0 || slot >= p.dst_rows)
        flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
      else
        row_ptr = reinterpret_cast<char*>(it.kind ? p.dst_v[it.l] : p.dst_k[it.l]) +
                  static_cast<int64_t>(p.dst_head_offset + it.h) * (kD * 2) + slot * dst_stride_bytes;
    }
    const bool do_rope = it.kind == 0 && row_ptr != nullptr;
    const float pos = static_cast<float>(p.position_start + (tok < 0 ? 0 : tok));
    // Warp-uniform outcome: tcgen05.ld is .sync.aligned across the warp.
    const bool got = mbar_wait(bar_at(s, kBarAccFull + acc), (n >> 2) & 1, s.abort_flag, p.status);
    if (!__all_sync(0xffffffffu, got)) break;
    tc_fence_after();
#pragma unroll 1
    for (int r = 0; r < 4; ++r) {  // RoPE pairs [16r, 16r + 16)
      const int p0 = 16 * r;
      uint32_t lo[16], hi[16];
      tmem_ld_32x32b_x16(tbase + p0, lo);
      tmem_ld_32x32b_x16(tbase + 64 + p0, hi);
      tmem_wait_ld();
      if (r == 3) {
        // Accumulator fully read into registers: hand it back to the MMA.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_at(s, kBarAccEmpty + acc));
      }
      float ylo[16], yhi[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        ylo[e] = __uint_as_float(lo[e]);
        yhi[e] = __uint_as_float(hi[e]);
      }
      if (do_rope && p.trig_exact) {
        for (int e = 0; e < 16; ++e) {
          float c, sn, o0, o1;
          sincosf(__fmul_rn(pos, p.dst_inv_freq[p0 + e]), &sn, &c);
          rope_apply_pair(ylo[e], yhi[e], __fmul_rn(c, p.dst_magnitude), __fmul_rn(sn, p.dst_magnitude), o0, o1);
          ylo[e] = o0;
          yhi[e] = o1;
        }
      } else if (do_rope) {
        // (y_lo + i y_hi) * (cos r + i sin r), then the sign (-1)^k.
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float c, sn;
          uint32_t sg;
          sincos_half_turns(__fmul_rn(pos, p.dst_inv_freq[p0 + e]), c, sn, sg);
          const float o0 = fmaf(ylo[e], c, -__fmul_rn(yhi[e], sn));
          const float o1 = fmaf(yhi[e], c, __fmul_rn(ylo[e], sn));
          ylo[e] = __uint_as_float(__float_as_uint(o0) ^ sg);
          yhi[e] = __uint_as_float(__float_as_uint(o1) ^ sg);
        }
        if (p.dst_magnitude != 1.0f) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            ylo[e] = __fmul_rn(ylo[e], p.dst_magnitude);
            yhi[e] = __fmul_rn(yhi[e], p.dst_magnitude);
          }
        }
      }
      // Staging row (128 B): chunks 0-3 hold columns [32h, 32h+32) and chunks
      // 4-7 columns [64+32h, ...) of the round pair h = r / 2; round r fills
      // chunks 2(r&1), 2(r&1)+1 and 4+2(r&1), 4+2(r&1)+1. Chunk c sits at
      // c ^ (row & 7).
      {
        const int c0 = 2 * (r & 1);
        *reinterpret_cast<uint4*>(my_row + (((c0 + 0) ^ my_key) << 4)) = pack8(ylo);
        *reinterpret_cast<uint4*>(my_row + (((c0 + 1) ^ my_key) << 4)) = pack8(ylo + 8);
        *reinterpret_cast<uint4*>(my_row + (((c0 + 4) ^ my_key) << 4)) = pack8(yhi);
        *reinterpret_cast<uint4*>(my_row + (((c0 + 5) ^ my_key) << 4)) = pack8(yhi + 8);
      }
      if (r & 1) {
        __syncwarp();
        // Stores: 4 rows x (2 x 64 contiguous bytes) per warp instruction.
        const int lc = lane & 7;
        const int half = r >> 1;
        const int gchunk = lc < 4 ? 4 * half + lc : 8 + 4 * half + (lc - 4);
#pragma unroll
        for (int qq = 0; qq < 8; ++qq) {
          const int rr = 4 * qq + (lane >> 3);
          char* dst = reinterpret_cast<char*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(row_ptr), rr));
          const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((lc ^ (rr & 7)) << 4));
          if (dst != nullptr) {
            if (p.dst_evict_first)
              st_global_v4_hint(dst + gchunk * 16, v, store_policy);
            else
              *reinterpret_cast<uint4*>(dst + gchunk * 16) = v;
          }
        }
        __syncwarp();
      }
    }
    cur = nxt;
    nxt = after;
    tok = tok_nxt;
    slot = slot_nxt;
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
  s.a = s.w + p.w_slots * kKBlockBytes;
  s.bias = s.a + p.stages * kKBlockBytes;
  s.ones = s.bias + kBiasBlockBytes;
  const uint32_t e = s.ones + kOnesBytes;
  s.e_gen = base_gen + (e - base);
  s.bars = e + kEpiWarps * kEpiWarpBytes;
  uint8_t* bars_gen = base_gen + (s.bars - base);
  s.tmem_holder = reinterpret_cast<uint32_t*>(bars_gen + 8 * kNumBars);
  s.abort_flag = reinterpret_cast<volatile int*>(bars_gen + 8 * kNumBars + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages; ++i) {
      mbar_init(bar_at(s, kBarFull + i), 32 * kProdWarps + 1);  // producer threads + expect_tx
      mbar_init(bar_at(s, kBarEmpty + i), 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(bar_at(s, kBarWFull + i), 1);
      mbar_init(bar_at(s, kBarWEmpty + i), 1);
      mbar_init(bar_at(s, kBarAccFull + i), 1);
      mbar_init(bar_at(s, kBarAccEmpty + i), 4);  // the 4 warps of the group owning the accumulator
    }
    mbar_init(bar_at(s, kBarBFull), 1);
    mbar_init(bar_at(s, kBarBEmpty), 1);
    mbar_init(bar_at(s, kBarDone), 1);
    // A device timeout before this launch: every role skips its work.
    *s.abort_flag = status_timed_out(p.status) ? 1 : 0;
    fence_mbarrier_init();
  }
  // Constant operands: the ones block (rows of [1, 1, 0 x 14], no-swizzle
  // K-major layout) and the (cos, sin) table.
  {
    uint16_t* ones = reinterpret_cast<uint16_t*>(base_gen + (s.ones - base));
    for (int idx = threadIdx.x; idx < kOnesBytes / 2; idx += blockDim.x) {
      const int kidx = ((idx >> 6) & 1) * 8 + (idx & 7);  // (byte/128 % 2) * 8 + byte%16/2
      ones[idx] = kidx < 2 ? static_cast<uint16_t>(0x3F80) : static_cast<uint16_t>(0);
    }
    fence_proxy_async_smem();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(smem_u32(s.tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_holder;

  if (*s.abort_flag) {
    // Skipped launch (see status_timed_out).
  } else if (warp < kProdWarps) {
    run_producer(p, StageRing{s.a, s.bars, kBarFull, kBarEmpty}, s.abort_flag, warp, lane);
  } else if (warp < kMmaWarp) {
    // TMEM lane quarter = warp % 4 (tcgen05.ld lane-access rule).
    run_epilogue(p, s, tmem_base, (warp - kProdWarps) >> 2, warp & 3, lane);
  } else if (warp == kMmaWarp) {
    if (lane == 0) run_mma(p, s, tmem_base);
    __syncwarp();
  } else {
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
