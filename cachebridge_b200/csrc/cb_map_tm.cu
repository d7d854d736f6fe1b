// Fused CacheBridge mapper apply + paged-KV install, transposed on tcgen05:
// the mapper weights are the MMA's A operand in tensor memory and the token
// tiles are its B operand in shared memory.
//
// For every target layer l, target head h, kind (K or V) and 128-token tile,
//     D^T = W^T . X^T      (D^T: 128 output features x 128 tokens, FP32 in TMEM)
// with X the concatenation of the S selected source layers' rows of head h
// (src/cachebridge/mapper.py:153-181). Each tile starts with one K=16 step that
// writes the bias into the accumulator (the unit's [bias_hi, bias_lo] block,
// the FP32 bias split into two BF16 parts, times a constant ones block); the
// epilogue applies the target RoPE to keys (mapper.py:207-239), rounds to BF16 and stores each
// 256-byte head row into the target pool row dst_slots[t]
// (online/blocks.py:86-111 set_kv_buffer; source_mapper_adapter.py:389-425).
//
// Why transposed: (1) one thread of the epilogue holds one RoPE frequency for
// many consecutive tokens, so the target RoPE coefficients follow an angle
// recurrence on the FMA pipe (two sincos per thread and tile) instead of a
// sincos per (token, frequency); (2) the tensor pipe reads only the token tile
// from shared memory; (3) the weights leave shared memory, which then holds
// full 256-byte staging rows, so every global store writes whole 128-byte lines.
//
// Tensor memory (512 columns): two FP32 accumulators (128 columns each), then
// one or two weight buffers of 64 columns per 128-feature k-block (bf16 pairs;
// lane L holds output feature f(L) = 8 (L/16) + L%8 + 64 ((L/8)%2), so lanes
// L and L+8 hold the RoPE pair (i, i+64)). With S <= 2 the next item's weights
// load while the current item's tiles run.
//
// CTA (persistent, one per SM, 544 threads) roles:
//   warps 0-3    producers (cb_pipeline.cuh): token tiles into a ring of stages.
//   warps 4-11   epilogue: two groups of four warps; group g takes the tiles
//                n with n % 2 == g (accumulator g). Warp w reads TMEM lane
//                quarter w % 4 with tcgen05.ld.16x256b, whose fragment gives
//                each thread lanes (j, j + 8) of a 16-lane block, i.e. one
//                RoPE pair, at two adjacent token columns. RoPE and BF16
//                packing in registers; stmatrix .trans writes token rows into
//                a 128-row staging tile per group (272-byte row pitch: whole
//                rows, no bank conflicts); each warp then stores 32 rows, two
//                whole rows (four 128-byte lines) per instruction. The four warps of a
//                group meet on mbarriers (bounded waits), not bar.sync, so a
//                warp that gives up cannot leave the others blocked.
//   warp 12      TMEM owner + single-thread tcgen05.mma issuer (M=128, N=128,
//                K=16, A from tensor memory; the bias step reads A and B from
//                shared memory).
//   warps 13-16  weight loaders: 16-byte loads of the unit's pre-arranged image,
//                tcgen05.st into the weight buffer (one warp per lane quarter),
//                and the [bias_hi, bias_lo] rows of the buffer's bias block.
// Every wait is bounded (kWaitTimeoutNs): an expired wait flags
// CB_DEV_ERR_TIMEOUT and the CTA unwinds instead of hanging.
#include "cb_device.cuh"
#include "cb_map_tm.cuh"
#include "cb_pipeline.cuh"

namespace cbk {

namespace {

constexpr int kBarFull = 0;       // [8] producers -> MMA (token tile filled)
constexpr int kBarEmpty = 8;      // [8] MMA -> producers (token tile consumed)
constexpr int kBarWFull = 16;     // [2] loaders -> MMA (weight buffer written)
constexpr int kBarWEmpty = 18;    // [2] MMA -> loaders (weight buffer no longer read)
constexpr int kBarAccFull = 20;   // [2] MMA -> epilogue group (accumulator ready)
constexpr int kBarAccEmpty = 22;  // [2] epilogue group -> MMA (accumulator read out)
constexpr int kBarDone = 24;      // [1] MMA drain at exit
constexpr int kBarStaged = 25;    // [2] epilogue group: all four warps staged the tile
constexpr int kBarFree = 27;      // [2] epilogue group: all four warps read the staging tile out
constexpr int kNumBars = 32;
constexpr int kMaxStages = 8;

struct Smem {
  uint32_t a;        // token-tile stages
  uint32_t stage;    // epilogue staging tiles (shared::cta address)
  uint32_t bias;     // bias blocks, one per weight buffer (no-swizzle K=16 layout)
  uint32_t ones;     // constant ones block of the bias step
  uint8_t* stage_gen;
  uint32_t bars;
  uint32_t* tmem_holder;
  volatile int* abort_flag;
};

__device__ __forceinline__ uint32_t bar_at(const Smem& s, int idx) { return s.bars + 8u * idx; }

// UMMA descriptor of a 128-row K-major operand with the 128-byte swizzle (as
// make_sw128_kmajor_desc), here the B operand: 128 token rows.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 16 lanes x 256 bits, repeated 4 times along the columns: thread t receives,
// for repetition k, lanes (base + t/4, base + 8 + t/4) at columns
// base + 8k + 2(t%4) + {0, 1}: r[4k + 0..1] from the first lane, r[4k + 2..3]
// from the second.
__device__ __forceinline__ void tmem_ld_16x256b_x4(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x 32 columns from registers: thread t writes lane (base + t).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Four 8x8 b16 matrices stored transposed: matrix m takes register r_m of
// every thread (thread t holding fragment row t/4, columns 2(t%4), 2(t%4)+1);
// thread 8m + i gives the shared address of stored row i of matrix m.
__device__ __forceinline__ void stmatrix_x4_trans(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0),
               "r"(r1), "r"(r2), "r"(r3)
               : "memory");
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// ------------------------------ weight loaders ------------------------------
// Warp of lane quarter q writes tensor-memory lanes [32q, 32q + 32) of the
// item's weight buffer: per k-block, 16 chunks of 16 bytes (64 columns of bf16
// pairs) per lane, read as 512 contiguous bytes per warp instruction.
__device__ void run_weight_loader(const MapTmParams& p, const Smem& s, uint32_t tmem_base, int q, int lane) {
  const int WB = p.w_bufs;
  const int wcols = 64 * p.KB;
  int itc = 0;
  for (int i = blockIdx.x; i < p.num_items; i += gridDim.x, ++itc) {
    const Item it = decode_item(p, i);
    const int wb = itc % WB;
    const uint32_t par = static_cast<uint32_t>((itc / WB) & 1);
    const bool got = mbar_wait(bar_at(s, kBarWEmpty + wb), par ^ 1u, s.abort_flag, p.status);
    if (!__all_sync(0xffffffffu, got)) break;
    tc_fence_after();
    const uint4* src = reinterpret_cast<const uint4*>(
        p.w_tm + static_cast<int64_t>((it.kind * p.L_t + it.l) * p.H + it.h) * p.unit_bytes);
    const int L = 32 * q + lane;
    const uint32_t taddr = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + kTmWeightCol0 + wb * wcols;
    for (int h8 = 0; h8 < 2 * p.KB; ++h8) {  // eight chunks (32 columns) at a time
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 w = __ldg(src + (h8 * 8 + c) * 128 + L);
        v[4 * c + 0] = w.x;
        v[4 * c + 1] = w.y;
        v[4 * c + 2] = w.z;
        v[4 * c + 3] = w.w;
      }
      tmem_st_32x32b_x32(taddr + h8 * 32, v);
    }
    {
      // Row L of the buffer's bias block: [bias_hi, bias_lo] of output
      // feature f(L) at k = 0, 1 (the rest of the block stays zero).
      const float b = __ldg(p.bias + static_cast<int64_t>((it.kind * p.L_t + it.l) * p.H + it.h) * kD +
                            tm_lane_feature(L));
      const float hi = __bfloat162float(__float2bfloat16_rn(b));
      const uint32_t word = pack_bf16x2(hi, __fsub_rn(b, hi));
      const uint32_t addr = s.bias + wb * kBiasBlockBytes + (L >> 3) * 256 + (L & 7) * 16;
      asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(word) : "memory");
      fence_proxy_async_smem();  // read by the MMA (async proxy)
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_at(s, kBarWFull + wb));
  }
}

// ------------------------------- MMA issuer --------------------------------
__device__ void run_mma(const MapTmParams& p, const Smem& s, uint32_t tmem_base) {
  constexpr uint32_t idesc = make_idesc_bf16_f32(kBM, kBM);  // M = 128 features, N = 128 tokens
  const uint64_t b_desc0 = make_sw128_kmajor_desc(s.a);
  const uint64_t ones_desc = make_noswizzle_k16_desc(s.ones);
  constexpr uint64_t kBlockDesc = kKBlockBytes >> 4;
  const int NS = p.stages;
  const int WB = p.w_bufs;
  const int wcols = 64 * p.KB;
  int stage = 0;
  uint32_t phase = 0;
  int n = 0, itc = 0;
  bool ok = true;
  for (int i = blockIdx.x; i < p.num_items && ok; i += gridDim.x, ++itc) {
    const Item it = decode_item(p, i);
    const int wb = itc % WB;
    if (!mbar_wait(bar_at(s, kBarWFull + wb), static_cast<uint32_t>((itc / WB) & 1), s.abort_flag, p.status)) break;
    tc_fence_after();
    const uint32_t a_base = tmem_base + kTmWeightCol0 + wb * wcols;
    for (int m = 0; m < it.mtiles && ok; ++m, ++n) {
      const int acc = n & 1;
      if (!mbar_wait(bar_at(s, kBarAccEmpty + acc), ((n >> 1) & 1) ^ 1, s.abort_flag, p.status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + acc * kTmAccCols;
      // Accumulator := [bias_hi, bias_lo] @ ones[:, 0:2]^T = the bias of each feature row.
      umma_bf16(d_tmem, make_noswizzle_k16_desc(s.bias + wb * kBiasBlockBytes), ones_desc, idesc, 0u);
      for (int kb = 0; kb < p.KB; ++kb) {
        if (!mbar_wait(bar_at(s, kBarFull + stage), phase, s.abort_flag, p.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // Value tiles were written by cp.async (generic proxy); the MMA reads
        // them through the async proxy.
        if (it.kind == 1) fence_proxy_async_smem();
        const uint64_t bd = b_desc0 + stage * kBlockDesc;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t off = static_cast<uint64_t>((kk >> 2) * kPanelBytes + (kk & 3) * 32) >> 4;
          umma_bf16_ts(d_tmem, a_base + kb * 64 + kk * 8, bd + off, idesc, 1u);
        }
        umma_commit(bar_at(s, kBarEmpty + stage));
        if (++stage == NS) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      umma_commit(bar_at(s, kBarAccFull + acc));
    }
    if (ok) umma_commit(bar_at(s, kBarWEmpty + wb));
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
// Target RoPE coefficient recurrence of one frequency for the token columns
// 2(t%4) + 8k + {0, 1} of a tile: (c, s) track cos/sin (times the YaRN
// magnitude) of the exact angle pos * inv_freq; the reference angle is
// ph = fl(pos * inv_freq) = pos * inv_freq - e with e = fma(pos, inv, -ph)
// exact, so cos(ph) = c + s e and sin(ph) = s - c e to first order (|e| is at
// most half an ulp of the phase, below 1e-3 rad for phases under 4e5).
struct RopeTrack {
  float inv, r1c, r1s, r8c, r8s;
  float c, s;  // at the current column pair's first token
};

__device__ __forceinline__ void rope_start(RopeTrack& rt, float pos0, float magnitude) {
  const float ph = __fmul_rn(pos0, rt.inv);
  const float e = fmaf(pos0, rt.inv, -ph);
  float sn, cs;
  sincosf(ph, &sn, &cs);
  // exact angle = ph + e
  rt.c = __fmul_rn(fmaf(-sn, e, cs), magnitude);
  rt.s = __fmul_rn(fmaf(cs, e, sn), magnitude);
}

// Rotate the pair (y0, y1) = (feature i, feature i + 64) of the token at
// position pos whose exact-angle coefficients are (c, s).
__device__ __forceinline__ void rope_rotate(float& y0, float& y1, float c, float s, float pos, float inv) {
  const float ph = __fmul_rn(pos, inv);
  const float e = fmaf(pos, inv, -ph);
  const float cr = fmaf(s, e, c);
  const float sr = fmaf(-c, e, s);
  const float o0 = fmaf(y0, cr, -__fmul_rn(y1, sr));
  const float o1 = fmaf(y1, cr, __fmul_rn(y0, sr));
  y0 = o0;
  y1 = o1;
}

struct TileCursor {
  int i, m, n;
  Item it;
};

__device__ __forceinline__ void cursor_advance(const MapTmParams& p, TileCursor& c, int step) {
  c.m += step;
  c.n += step;
  while (c.i < p.num_items && c.m >= c.it.mtiles) {
    c.m -= c.it.mtiles;
    c.i += gridDim.x;
    if (c.i < p.num_items) c.it = decode_item(p, c.i);
  }
}

// Epilogue warp of group g, lane quarter q. Tiles n with n % 2 == g. The
// thread's destination row is token row 32q + lane of the tile (the rows this
// warp stores); its slot is loaded one tile ahead.
__device__ void run_epilogue(const MapTmParams& p, const Smem& s, uint32_t tmem_base, int g, int q, int lane) {
  const uint32_t stage = s.stage + g * kTmStageBytes;
  const int64_t dst_stride_bytes = p.dst_row_stride * 2;
  const uint64_t store_policy = l2_policy_evict_first();
  const int quad = lane & 3;    // column pair within an 8-column repetition
  const int j = lane >> 2;      // lane within the 8-lane half block
  // Frequencies of this thread: blocks 2q and 2q + 1, lane j -> i = 8 * block + j.
  RopeTrack rt[2];
#pragma unroll
  for (int b = 0; b < 2; ++b) {
    const int i = 8 * (2 * q + b) + j;
    rt[b].inv = p.dst_inv_freq[i];
    rt[b].r1c = p.rot1_c[i];
    rt[b].r1s = p.rot1_s[i];
    rt[b].r8c = p.rot8_c[i];
    rt[b].r8s = p.rot8_s[i];
  }
  // stmatrix addressing: thread 8m + r gives stored row r of matrix m.
  const int st_m = lane >> 3, st_r = lane & 7;
  TileCursor cur;
  cur.i = blockIdx.x;
  cur.m = 0;
  cur.n = 0;
  if (cur.i < p.num_items) cur.it = decode_item(p, cur.i);
  cursor_advance(p, cur, g);
  TileCursor nxt = cur;
  cursor_advance(p, nxt, kTmEpiGroups);
  const int my_row = 32 * q + lane;
  int tok = cur.i < p.num_items ? check_token(p, item_token_raw(p, cur.it, cur.m, my_row)) : -1;
  int64_t slot = tok >= 0 ? load_slot(p.dst_slots, p.dst_slot_dtype, tok) : 0;
  uint32_t gpar = 0;  // parity of this group's tile counter
  bool first = true;  // no earlier tile of this group has used the staging tile
  while (cur.i < p.num_items) {
    const int tok_nxt = nxt.i < p.num_items ? check_token(p, item_token_raw(p, nxt.it, nxt.m, my_row)) : -1;
    const int64_t slot_nxt = tok_nxt >= 0 ? load_slot(p.dst_slots, p.dst_slot_dtype, tok_nxt) : 0;
    const Item& it = cur.it;
    const int n = cur.n;
    const int acc = n & 1;
    char* row_ptr = nullptr;  // this lane's destination row, or null
    if (tok >= 0) {
      if (slot < 0 || slot >= p.dst_rows)
        flag_error(p.status, CB_DEV_ERR_SLOT_RANGE);
      else
        row_ptr = reinterpret_cast<char*>(it.kind ? p.dst_v[it.l] : p.dst_k[it.l]) +
                  static_cast<int64_t>(p.dst_head_offset + it.h) * (kD * 2) + slot * dst_stride_bytes;
    }
    const bool rope = it.kind == 0;
    const int tile_tok0 = it.tok0 + cur.m * kBM;
    const float pos0 = static_cast<float>(p.position_start + tile_tok0 + 2 * quad);
    if (rope) {
#pragma unroll
      for (int b = 0; b < 2; ++b) rope_start(rt[b], pos0, p.dst_magnitude);
    }
    // Warp-uniform outcome: tcgen05.ld is .sync.aligned across the warp.
    const bool got = mbar_wait(bar_at(s, kBarAccFull + acc), (n >> 1) & 1, s.abort_flag, p.status);
    if (!__all_sync(0xffffffffu, got)) break;
    tc_fence_after();
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + acc * kTmAccCols;
    bool aborted = false;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {  // 32-token chunks of the tile
      uint32_t r[2][16];
      tmem_ld_16x256b_x4(t_lane + 32 * c, r[0]);
      tmem_ld_16x256b_x4(t_lane + (16u << 16) + 32 * c, r[1]);
      tmem_wait_ld();
      if (c == 3) {
        // Accumulator fully read into registers: hand it back to the MMA.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_at(s, kBarAccEmpty + acc));
      }
      if (c == 0) {
        // The group's previous tile has been read out of the staging tile:
        // this warp's reads first, then all four warps'.
        if (!first) {
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_at(s, kBarFree + g));
        }
        const bool free_ok = mbar_wait(bar_at(s, kBarFree + g), gpar ^ 1u, s.abort_flag, p.status);
        if (!__all_sync(0xffffffffu, free_ok)) {
          aborted = true;
          break;
        }
      }
      uint32_t packed[2][8];  // [block][2k + (0: features i, 1: features i + 64)]
#pragma unroll
      for (int b = 0; b < 2; ++b) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float y0a = __uint_as_float(r[b][4 * k + 0]);  // feature i, token 2quad + 8k
          float y0b = __uint_as_float(r[b][4 * k + 1]);  // feature i, token + 1
          float y1a = __uint_as_float(r[b][4 * k + 2]);  // feature i + 64
          float y1b = __uint_as_float(r[b][4 * k + 3]);
          if (rope) {
            const float pa = pos0 + static_cast<float>(32 * c + 8 * k);
            const float ca = rt[b].c, sa = rt[b].s;
            const float cb = fmaf(ca, rt[b].r1c, -__fmul_rn(sa, rt[b].r1s));
            const float sb = fmaf(sa, rt[b].r1c, __fmul_rn(ca, rt[b].r1s));
            rope_rotate(y0a, y1a, ca, sa, pa, rt[b].inv);
            rope_rotate(y0b, y1b, cb, sb, pa + 1.0f, rt[b].inv);
            // Advance to the next repetition (+8 positions).
            rt[b].c = fmaf(ca, rt[b].r8c, -__fmul_rn(sa, rt[b].r8s));
            rt[b].s = fmaf(sa, rt[b].r8c, __fmul_rn(ca, rt[b].r8s));
          }
          packed[b][2 * k + 0] = pack_bf16x2(y0a, y0b);
          packed[b][2 * k + 1] = pack_bf16x2(y1a, y1b);
        }
      }
      // Staging: token row T (0..127) at T * kTmRowPitch, 16-byte chunk lc
      // (features 8 lc .. 8 lc + 7) at 16 lc. The 272-byte pitch puts the 8
      // rows of one stored matrix in 8 different bank quads. Matrix m of an x4
      // store: rep k = k0 + m / 2, features i (m even, chunk 2q + b) or i + 64
      // (m odd, chunk 8 + 2q + b); its stored row st_r is token 32c + 8k + st_r.
#pragma unroll
      for (int b = 0; b < 2; ++b) {
#pragma unroll
        for (int k0 = 0; k0 < 4; k0 += 2) {
          const int k = k0 + (st_m >> 1);
          const int T = 32 * c + 8 * k + st_r;
          const int lc = ((st_m & 1) ? 8 : 0) + 2 * q + b;
          const uint32_t addr = stage + T * kTmRowPitch + (lc << 4);
          stmatrix_x4_trans(addr, packed[b][2 * k0], packed[b][2 * k0 + 1], packed[b][2 * k0 + 2],
                            packed[b][2 * k0 + 3]);
        }
      }
    }
    if (aborted) break;
    // The whole tile is staged once all four warps of the group arrived.
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_at(s, kBarStaged + g));
    const bool staged = mbar_wait(bar_at(s, kBarStaged + g), gpar, s.abort_flag, p.status);
    if (!__all_sync(0xffffffffu, staged)) break;
    first = false;
    {
      // Stores: this warp writes token rows [32q, 32q + 32), four whole rows
      // per instruction: lane (g, L) = (lane / 8, lane % 8) writes bytes
      // [32 L, 32 L + 32) of row 32q + 4i + g with one 32-byte store. Its two
      // 16-byte staging reads fall in bank quad (g + 2L) mod 8 under the
      // 272-byte pitch: four lanes per quad, the minimum of four wavefronts.
      const int gq = lane >> 3, L8 = lane & 7;
#pragma unroll 2
      for (int i = 0; i < 8; ++i) {
        const int rl = 4 * i + gq;  // row within this warp's 32
        char* dst = reinterpret_cast<char*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(row_ptr), rl));
        const uint32_t src = stage + (32 * q + rl) * kTmRowPitch + 32 * L8;
        const uint4 va = ld_shared_v4(src);
        const uint4 vb = ld_shared_v4(src + 16);
        if (dst != nullptr) {
          char* d = dst + 32 * L8;
          if (p.dst_v8) {
            if (p.dst_evict_first)
              st_global_v8_hint(d, va, vb, store_policy);
            else
              st_global_v8(d, va, vb);
          } else if (p.dst_evict_first) {
            st_global_v4_hint(d, va, store_policy);
            st_global_v4_hint(d + 16, vb, store_policy);
          } else {
            *reinterpret_cast<uint4*>(d) = va;
            *reinterpret_cast<uint4*>(d + 16) = vb;
          }
        }
      }
    }
    gpar ^= 1u;
    cur = nxt;
    cursor_advance(p, nxt, kTmEpiGroups);
    tok = tok_nxt;
    slot = slot_nxt;
  }
}

}  // namespace

__global__ void __launch_bounds__(kTmThreads, 1) map_install_tm_kernel(const __grid_constant__ MapTmParams p) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_gen = smem_raw + (base - raw);

  Smem s;
  s.a = base;
  s.stage = s.a + p.stages * kKBlockBytes;
  s.stage_gen = base_gen + (s.stage - base);
  s.bias = s.stage + kTmEpiGroups * kTmStageBytes;
  s.ones = s.bias + 2 * kBiasBlockBytes;
  s.bars = s.ones + kOnesBytes;
  uint8_t* bars_gen = base_gen + (s.bars - base);
  s.tmem_holder = reinterpret_cast<uint32_t*>(bars_gen + 8 * kNumBars);
  s.abort_flag = reinterpret_cast<volatile int*>(bars_gen + 8 * kNumBars + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.stages && i < kMaxStages; ++i) {
      mbar_init(bar_at(s, kBarFull + i), 32 * kTmProdWarps + 1);  // producer threads + expect_tx
      mbar_init(bar_at(s, kBarEmpty + i), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_at(s, kBarWFull + i), 4);     // the four loader warps
      mbar_init(bar_at(s, kBarWEmpty + i), 1);
      mbar_init(bar_at(s, kBarAccFull + i), 1);
      mbar_init(bar_at(s, kBarAccEmpty + i), 4);  // the four warps of the group owning the accumulator
    }
    mbar_init(bar_at(s, kBarDone), 1);
    for (int g = 0; g < kTmEpiGroups; ++g) {
      mbar_init(bar_at(s, kBarStaged + g), 4);
      mbar_init(bar_at(s, kBarFree + g), 4);
    }
    // A device timeout before this launch: every role skips its work.
    *s.abort_flag = status_timed_out(p.status) ? 1 : 0;
    fence_mbarrier_init();
  }
  // Constant operands of the bias step: the ones block (rows of [1, 1, 0 x 14])
  // and two bias blocks whose rows the loaders fill at k = 0, 1 (zero elsewhere).
  // No-swizzle K=16 layout: element (row r, k) at (r/8)*256 + (k/8)*128 + (r%8)*16 + (k%8)*2.
  {
    uint16_t* ones = reinterpret_cast<uint16_t*>(base_gen + (s.ones - base));
    uint16_t* bias = reinterpret_cast<uint16_t*>(base_gen + (s.bias - base));
    for (int idx = threadIdx.x; idx < kOnesBytes / 2; idx += blockDim.x) {
      const int kidx = ((idx >> 6) & 1) * 8 + (idx & 7);  // (byte/128 % 2) * 8 + byte%16/2
      ones[idx] = kidx < 2 ? static_cast<uint16_t>(0x3F80) : static_cast<uint16_t>(0);
    }
    for (int idx = threadIdx.x; idx < kBiasBlockBytes; idx += blockDim.x) bias[idx] = 0;  // both blocks
    fence_proxy_async_smem();
  }
  if (warp == kTmMmaWarp) {
    tmem_alloc(smem_u32(s.tmem_holder), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s.tmem_holder;

  if (*s.abort_flag) {
    // Skipped launch (see status_timed_out).
  } else if (warp < kTmProdWarps) {
    run_producer(p, StageRing{s.a, s.bars, kBarFull, kBarEmpty}, s.abort_flag, warp, lane);
  } else if (warp < kTmMmaWarp) {
    // TMEM lane quarter = warp % 4 (tcgen05.ld lane-access rule).
    run_epilogue(p, s, tmem_base, (warp - kTmProdWarps) >> 2, warp & 3, lane);
  } else if (warp == kTmMmaWarp) {
    if (lane == 0) run_mma(p, s, tmem_base);
    __syncwarp();
  } else {
    run_weight_loader(p, s, tmem_base, warp & 3, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kTmMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace cbk
