// Device-side helpers shared by the cachebridge_b200 kernels (sm_100a only).
//
// Inline PTX wrappers for mbarriers, cp.async, bulk copies and the tcgen05
// (5th-generation tensor core / tensor memory) instructions, plus the row-set
// parameter blocks every kernel receives by value.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cachebridge_b200.h"

namespace cbk {

// ---------------------------------------------------------------------------
// Parameter blocks
// ---------------------------------------------------------------------------

// One per-layer row set as seen by a kernel (the device-side image of cb_rows).
struct RowSet {
  const void* k[CB_MAX_LAYERS];
  const void* v[CB_MAX_LAYERS];
  int64_t row_stride;  // elements
  int64_t rows;
  int32_t head_offset;
  int32_t slot_dtype;
  const void* slots;
};

// Device image of cb_rope.
struct RopeDev {
  float inv_freq[128];
  float magnitude;
  int half_dim;
};

// qwen_rope coefficients of one (position, frequency): the FP32 phase
// float(position) * inv_freq, then cos/sin (CUDA's accurate sincosf) times the
// YaRN magnitude, in the reference's op order (rope.py:70-72).
__device__ __forceinline__ void rope_coeff(float pos, float inv_freq, float magnitude, float& c,
                                           float& s) {
  float sn, cs;
  sincosf(__fmul_rn(pos, inv_freq), &sn, &cs);
  c = __fmul_rn(cs, magnitude);
  s = __fmul_rn(sn, magnitude);
}

__device__ __forceinline__ int64_t load_slot(const void* slots, int dtype, int64_t t) {
  if (dtype == CB_INDEX_I32) return (int64_t)__ldg(reinterpret_cast<const int32_t*>(slots) + t);
  if (dtype == CB_INDEX_I64) return (int64_t)__ldg(reinterpret_cast<const long long*>(slots) + t);
  return t;
}

__device__ __forceinline__ void flag_error(int32_t* status, int bits) {
  if (status != nullptr) atomicOr(reinterpret_cast<int*>(status), bits);
}

// True once a bounded wait on this device has expired (CB_DEV_ERR_TIMEOUT is
// set in the status word). The handoff kernels then do no work: a chunk whose
// receive slot never filled is not mapped or installed, and the chunks after
// it are skipped too, until the caller reads and clears the status word.
__device__ __forceinline__ bool status_timed_out(const int32_t* status) {
  return status != nullptr && (*reinterpret_cast<const volatile int32_t*>(status) & CB_DEV_ERR_TIMEOUT) != 0;
}

// Token handled at processing index i of a call: token_order[i] when the
// caller gave an order (a permutation of [0, n)), else i. An entry outside
// [0, n) flags CB_DEV_ERR_SLOT_RANGE and returns -1 (the row is skipped).
__device__ __forceinline__ int token_at(const int32_t* order, int i, int n, int32_t* status) {
  if (order == nullptr) return i;
  const int t = __ldg(order + i);
  if (t < 0 || t >= n) {
    flag_error(status, CB_DEV_ERR_SLOT_RANGE);
    return -1;
  }
  return t;
}

// ---------------------------------------------------------------------------
// Shared-memory addressing, fences, timers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wall-clock bound of every pipeline wait inside a kernel. A wait that expires
// raises the CTA's abort flag and CB_DEV_ERR_TIMEOUT, and the kernel unwinds
// instead of spinning forever.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

// Bounded wait on an mbarrier phase. Returns false (and aborts the CTA) if the
// phase did not complete within kWaitTimeoutNs, or if another role of the CTA
// has already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int32_t* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 63u) == 0u) {
      if (*abort_flag) return false;
      if (global_timer_ns() - t0 > kWaitTimeoutNs) {
        *abort_flag = 1;
        flag_error(status, CB_DEV_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// cp.async (16-byte global -> shared, L2 only) and bulk copies
// ---------------------------------------------------------------------------

// src_bytes = 16 copies, src_bytes = 0 zero-fills the 16 destination bytes
// without reading global memory.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Arrive on `bar` (without raising its pending count) once every cp.async this
// thread issued so far has completed.
__device__ __forceinline__ void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Wait until at most n (0..3) of this thread's cp.async groups are pending.
__device__ __forceinline__ void cp_async_wait_dyn(int n) {
  switch (n) {
    case 0: cp_async_wait<0>(); break;
    case 1: cp_async_wait<1>(); break;
    case 2: cp_async_wait<2>(); break;
    default: cp_async_wait<3>(); break;
  }
}

// Non-tensor bulk copy global -> this CTA's shared memory, completing `bytes`
// transaction bytes on mbarrier `bar`. Addresses 16-byte aligned, bytes % 16 == 0.
// Carries an L2 evict-last hint: the same weight tiles are re-read by many CTAs.
__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                              uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// TMA tiled load of a 4-D box into this CTA's shared memory.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}


// L2 policy for data written once and not read again by this kernel (the
// mapped target rows): evicted first, so the source rows that other CTAs
// still read stay in L2.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void st_global_v4_hint(void* ptr, uint4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(ptr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w), "l"(policy)
               : "memory");
}

// 32-byte global stores (sm_100): eight 32-bit words, 32-byte aligned.
__device__ __forceinline__ void st_global_v8(void* ptr, uint4 a, uint4 b) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(ptr), "r"(a.x), "r"(a.y), "r"(a.z),
               "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

__device__ __forceinline__ void st_global_v8_hint(void* ptr, uint4 a, uint4 b, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8}, %9;" ::"l"(ptr), "r"(a.x),
               "r"(a.y), "r"(a.z), "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w), "l"(policy)
               : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA, commit, loads
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(holder_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 operands, fp32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on `bar` when all previously issued tcgen05 ops of this thread complete.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i receives lane (base lane + i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// UMMA shared-memory matrix descriptor for a K-major operand stored with the
// 128-byte swizzle: rows of 128 B (64 bf16), 8-row atoms of 1024 B packed
// contiguously (stride byte offset 1024), leading byte offset unused (1).
// Bit layout: start>>4 [0,14), LBO>>4 [16,30), SBO>>4 [32,46), version 1 at
// [46,48), base offset 0, layout type 2 (SWIZZLE_128B) at [61,64).
__device__ __forceinline__ uint64_t make_sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// UMMA descriptor of one K=16 step of a 128-row K-major operand without
// swizzle: 8-row x 16-byte core matrices, the two K halves 128 B apart
// (leading byte offset), consecutive 8-row groups 256 B apart (stride byte
// offset). Element (row r, k) sits at (r/8)*256 + (k/8)*128 + (r%8)*16 + (k%8)*2.
__device__ __forceinline__ uint64_t make_noswizzle_k16_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(128u >> 4) << 16;
  d |= static_cast<uint64_t>(256u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  return d;  // layout type 0: no swizzle
}

// Instruction descriptor for kind::f16: D fp32, A and B bf16, both K-major,
// N = n, M = m.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int m, int n) {
  return (1u << 4)                                   // D format: F32
         | (1u << 7)                                 // A format: BF16
         | (1u << 10)                                // B format: BF16
         | (static_cast<uint32_t>(n >> 3) << 17)     // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);    // M >> 4
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// Split-half RoPE removal for one (i, i + half) pair, in the reference's op
// order: (x*cos - rotate_half(x)*sin) / max(cos^2 + sin^2, FLT_MIN).
__device__ __forceinline__ void rope_remove_pair(float x0, float x1, float c, float s, float& o0,
                                                 float& o1) {
  float m = __fadd_rn(__fmul_rn(c, c), __fmul_rn(s, s));
  m = fmaxf(m, 1.17549435e-38f);
  o0 = __fdiv_rn(__fsub_rn(__fmul_rn(x0, c), __fmul_rn(-x1, s)), m);
  o1 = __fdiv_rn(__fsub_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)), m);
}

// Split-half RoPE application: x*cos + rotate_half(x)*sin.
__device__ __forceinline__ void rope_apply_pair(float x0, float x1, float c, float s, float& o0,
                                                float& o1) {
  o0 = __fadd_rn(__fmul_rn(x0, c), __fmul_rn(-x1, s));
  o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
}

}  // namespace cbk
