// Pieces shared by the two tensor-core map+install kernels: work items, token
// lookups and the producer role that fills the token-tile stages.
//
// A work item is (head h, kind, chunk of R*128 tokens, target layer l).
// Items are ordered head/kind-major, then chunk, then layer, so the CTAs that
// run concurrently share one head/kind's source rows of one token window
// (each source row feeds ~L_t*S/L_s target layers and is read from HBM once).
#pragma once

#include <climits>

#include "cb_device.cuh"
#include "cb_map_tc.cuh"

namespace cbk {

struct Item {
  int kind;   // 0 = K, 1 = V
  int h;      // head within this call
  int l;      // target layer
  int tok0;   // first token of the chunk
  int mtiles; // valid 128-token m-tiles in the chunk
};

template <typename P>
__device__ __forceinline__ Item decode_item(const P& p, int i) {
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

// Token lookups. A row's token is order[t] (or t) for processing index t; the
// producers and the epilogue read the order entry two m-tiles ahead and the
// slot one m-tile ahead, so neither dependent load stalls a pipeline role.
// kNoToken marks a row past the call's (or item's) end.
constexpr int kNoToken = INT_MIN;

template <typename P>
__device__ __forceinline__ int item_token_raw(const P& p, const Item& it, int mm, int row) {
  if (mm >= it.mtiles) return kNoToken;
  const int t = it.tok0 + mm * kBM + row;
  if (t >= p.n_tokens) return kNoToken;
  return p.order == nullptr ? t : __ldg(p.order + t);
}

// A token read by item_token_raw, or -1 for none. An order entry outside
// [0, n) flags CB_DEV_ERR_SLOT_RANGE and the row is skipped.
template <typename P>
__device__ __forceinline__ int check_token(const P& p, int raw) {
  if (raw == kNoToken) return -1;
  if (raw < 0 || raw >= p.n_tokens) {
    flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
    return -1;
  }
  return raw;
}

// Stage ring seen by the producers: stage s occupies 32 KB at a_base + s*32 KB;
// its full and empty mbarriers sit at bars + 8*(full0 + s) and bars + 8*(empty0 + s).
struct StageRing {
  uint32_t a_base;
  uint32_t bars;
  int full0, empty0;
  __device__ __forceinline__ uint32_t full(int s) const { return bars + 8u * (full0 + s); }
  __device__ __forceinline__ uint32_t empty(int s) const { return bars + 8u * (empty0 + s); }
};

// Producers: four warps; warp pw owns token rows [32 pw, 32 pw + 32) of every
// stage. Keys: thread 0 loads the stage with two 4-D TMA boxes (128 tokens x
// 64 features) from the content-space workspace (expect_tx 32 KB). Values:
// 16-byte cp.async gathers of the source pool rows through the slot table, 16
// lanes per 256-byte row, two rows per warp instruction, tracked by
// cp.async.mbarrier.arrive.noinc. The stage's full barrier counts 129
// arrivals: one per producer thread plus thread 0's expect_tx. Each stage is
// a 128-token x 128-feature block in the UMMA 128B-swizzled K-major layout.
template <typename P>
__device__ void run_producer(const P& p, const StageRing& ring, volatile int* abort_flag, int pw, int lane) {
  const int NS = p.stages;
  const bool leader = pw == 0 && lane == 0;
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  // The last stage whose key tile the leader requested by TMA, and its phase,
  // so an aborted CTA can wait for those bytes before it exits.
  int tma_stage = -1;
  uint32_t tma_phase = 0;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x) {
    const Item it = decode_item(p, i);
    // Source slot of this lane's row (values only): tok_c / row_c for m-tile
    // m, raw_n the order entry of m-tile m + 1.
    const int row_in_tile = pw * 32 + lane;
    int tok_c = -1, raw_n = kNoToken;
    int64_t row_c = 0;
    if (it.kind == 1) {
      tok_c = check_token(p, item_token_raw(p, it, 0, row_in_tile));
      if (tok_c >= 0) row_c = load_slot(p.src_slots, p.src_slot_dtype, tok_c);
      raw_n = item_token_raw(p, it, 1, row_in_tile);
    }
    for (int m = 0; m < it.mtiles && ok; ++m) {
      const int tok0 = it.tok0 + m * kBM;
      int valid = tok_c >= 0;
      const int64_t srow = row_c;
      if (it.kind == 1) {
        tok_c = check_token(p, raw_n);
        row_c = tok_c >= 0 ? load_slot(p.src_slots, p.src_slot_dtype, tok_c) : 0;
        raw_n = item_token_raw(p, it, m + 2, row_in_tile);
      }
      if (it.kind == 1 && valid && (srow < 0 || srow >= p.src_rows)) {
        flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
        valid = 0;
      }
      for (int kb = 0; kb < p.KB; ++kb) {
        // Feature block kb: selected layer j, source head sh (the target head
        // itself for headwise maps, every source head in turn for dense ones).
        const int j = kb / p.kb_heads;
        const int sh = p.dense ? kb - j * p.kb_heads : it.h;
        // Warp-uniform outcome: the gather below uses full-warp shuffles.
        const bool got = mbar_wait(ring.empty(stage), phase ^ 1u, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint32_t full = ring.full(stage);
        const uint32_t dst = ring.a_base + stage * kKBlockBytes;
        if (it.kind == 0) {
          if (leader) {
            const int u = __ldg(p.sel_local + it.l * p.S + j);
            mbar_arrive_expect_tx(full, kKBlockBytes);
            tma_load_4d(dst, &p.kmap, 0, sh, tok0, u, full);
            tma_load_4d(dst + kPanelBytes, &p.kmap, 64, sh, tok0, u, full);
            tma_stage = stage;
            tma_phase = phase;
          }
          mbar_arrive(full);
        } else {
          const int sl = __ldg(p.sel_global + it.l * p.S + j);
          const char* base = reinterpret_cast<const char*>(p.src_v[sl]) +
                             static_cast<int64_t>(p.src_head_offset + sh) * (kD * 2);
          const int64_t stride_bytes = p.src_row_stride * 2;
          const int c = lane & 15;
#pragma unroll
          for (int ii = 0; ii < 16; ++ii) {
            const int r = 2 * ii + (lane >> 4);
            const int64_t rr = __shfl_sync(0xffffffffu, srow, r);
            const int vv = __shfl_sync(0xffffffffu, valid, r);
            const int row = pw * 32 + r;
            const char* g = base + (vv ? rr * stride_bytes : 0) + c * 16;
            const uint32_t d = dst + (c >> 3) * kPanelBytes + row * 128 + (((c & 7) ^ (row & 7)) << 4);
            cp_async_16(d, g, vv ? 16u : 0u);
          }
          cp_async_arrive_noinc(full);
          if (leader) {
            mbar_arrive(full);
            // This refill of the stage follows the completion of its TMA phase.
            if (stage == tma_stage) tma_stage = -1;
          }
        }
        if (++stage == NS) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  }
  // Never exit with copies in flight into shared memory: cp.async gathers
  // complete under wait_all; an aborted CTA also waits (bounded) for the
  // phase of the last stage the leader armed for TMA key tiles.
  cp_async_wait_all();
  if (leader && tma_stage >= 0 && *abort_flag) {
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(ring.full(tma_stage), tma_phase)) {
      if (global_timer_ns() - t0 > kWaitTimeoutNs) break;
    }
  }
}

}  // namespace cbk
