// Shared device-side helpers for the sm_100a GQA attention kernels.
//
// Everything here is a thin wrapper over one PTX instruction (mbarrier, TMA,
// tcgen05, mma.sync, ldmatrix) written from the public PTX ISA, plus the
// bounded-wait machinery that turns a lost arrival into an error status
// instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/gqa_sm100.h"

namespace gqa {

// ---------------------------------------------------------------------------
// Device error word. A kernel whose bounded wait expires writes a nonzero
// code here (first writer wins) and returns; gqa_device_error() reads it.
// ---------------------------------------------------------------------------
__device__ int g_device_error = 0;
__device__ int g_device_error_site = 0;

// Upper bound on any single wait inside a kernel (nanoseconds of %globaltimer).
// Every kernel here finishes in well under a second, so hitting this means a
// lost arrival (a bug), never a slow GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_device_error(int code, int site) {
  if (atomicCAS(&g_device_error, 0, code) == 0) g_device_error_site = site;
}

// Ranks of one peer exchange: the GPUs of one node.
constexpr int kMaxPeers = 8;

// System-scope acquire load: orders this thread's later reads after the writes
// (from any GPU) that a matching release made visible.
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

#ifdef GQA_DEBUG_CHECKS
// Test hooks of the checked build (gqa_debug_inject): the wait limit can be
// shortened at run time, and the TMA producer of one CTA can withhold one of its
// loads (no expect-tx, no copy), so the consumer's bounded wait on that load runs
// out and the abort path runs -- no memory is touched that a release build would
// not touch, and nothing is left in flight. Release builds compile these to
// constants.
__device__ unsigned long long g_wait_limit_ns = kWaitLimitNs;
__device__ int g_withhold_cta = -1;
__device__ int g_withhold_load = -1;
__device__ __forceinline__ uint64_t wait_limit_ns() { return g_wait_limit_ns; }
__device__ __forceinline__ bool withheld_load(int t) {
  return (int)blockIdx.x == g_withhold_cta && t == g_withhold_load;
}
#else
__device__ __forceinline__ uint64_t wait_limit_ns() { return kWaitLimitNs; }
__device__ __forceinline__ bool withheld_load(int) { return false; }
#endif

// Debug builds (-DGQA_DEBUG_CHECKS, `build.py --debug`): the TMA, UMMA and TMEM
// helpers below check their addresses and coordinates first. A failed check records
// GQA_ERR_DEBUG_CHECK and a site id in the device error word and skips the access;
// the wait that depended on it then expires (bounded), so a bad index becomes an
// error status instead of a fault. Release builds compile the checks away.
#ifdef GQA_DEBUG_CHECKS
#define GQA_CHECK(cond, site) ((cond) ? true : (report_device_error(GQA_ERR_DEBUG_CHECK, (site)), false))
#else
#define GQA_CHECK(cond, site) true
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok;
}

// As mbar_try_wait, but the warp is suspended in hardware (no issue slots
// taken from the other warps of its SM sub-partition) until the phase
// completes or about kSuspendHintNs pass.
constexpr uint32_t kSuspendHintNs = 1000000;
__device__ __forceinline__ uint32_t mbar_try_wait_suspend(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok;
}

// Wait for the phase with the given parity to complete. Returns false (after
// recording `site` in the device error word and raising the CTA-wide abort
// flag) if it does not complete within kWaitLimitNs, or returns false at once
// if another thread of the CTA has already raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 4; ++i)
      if (mbar_try_wait_suspend(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > wait_limit_ns()) {
      *abort_flag = 1;
      report_device_error(GQA_ERR_TIMEOUT, site);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch. The host launches the prefill and streaming
// kernels with programmatic stream serialisation, so a grid may start while the
// previous kernel on the stream is still finishing. Every thread calls pdl_wait()
// before its first global memory access (read or write): it returns once the
// previous grid has completed and its writes are visible (at once when there is
// none). pdl_trigger() lets the next such grid start its prologue on SMs this grid
// frees; it takes effect when every CTA of this grid has triggered or exited.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor): plain tile loads and stores of this GPU's own memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0,
                                            int c1, int c2, int c3) {
  // 128-byte swizzled tiles start on 128 bytes; x * 2 bytes is a multiple of 16.
  if (!GQA_CHECK((dst & 127u) == 0 && (c0 & 7) == 0 && (bar & 7u) == 0, 900)) return;
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// L2 prefetch of one tensor-map box (no shared-memory destination, no barrier). A
// hint only: the line is fetched into L2 and later loads read it through L2, which
// any write to it also goes through, so it may be issued before the grid dependency
// wait without changing what the kernel reads.
__device__ __forceinline__ void tma_prefetch_l2_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  if (!GQA_CHECK((c0 & 7) == 0, 905)) return;
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                                 int c0, int c1, int c2, int c3, uint64_t policy) {
  if (!GQA_CHECK((dst & 127u) == 0 && (c0 & 7) == 0 && (bar & 7u) == 0, 900)) return;
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, uint32_t src, int c0, int c1, int c2,
                                             int c3) {
  // Stores never start at a negative coordinate.
  if (!GQA_CHECK((src & 127u) == 0 && (c0 & 7) == 0 && c0 >= 0 && c1 >= 0 && c2 >= 0 && c3 >= 0, 901)) return;
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor core + tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]   (kind::f16: f16/bf16 inputs, f32 accumulate)
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  if (!GQA_CHECK((d_tmem & 0xFFFFu) < 512u, 903)) return;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  if (!GQA_CHECK((d_tmem & 0xFFFFu) < 512u && (a_tmem & 0xFFFFu) < 512u, 903)) return;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Instruction descriptor for kind::f16 with f32 accumulation.
//   bits [4,6) D format (1 = f32); [7,10) A format; [10,13) B format (0 = f16, 1 = bf16);
//   bit 15 A major, bit 16 B major (0 = K-major, 1 = MN-major); [17,23) N>>3; [24,29) M>>4.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, bool bf16, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Shared-memory matrix descriptor (tcgen05 form, version field = 1), 128-byte swizzle.
//   [0,14) start>>4; [16,30) leading byte offset>>4; [32,46) stride byte offset>>4;
//   [46,48) version = 1; [49,52) base offset = 0 (tiles are 1024-byte aligned); [61,64) layout = 2 (SW128).
// K-major operand: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO); LBO unused.
__device__ __forceinline__ uint64_t desc_sw128_kmajor(uint32_t saddr) {
  (void)GQA_CHECK((saddr & 15u) == 0, 902);
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// MN-major operand: each 128-byte row holds 64 MN-contiguous elements of one K index;
// consecutive 64-element MN blocks are `lbo_bytes` apart, 8-row K groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_sw128_mnmajor(uint32_t saddr, uint32_t lbo_bytes) {
  (void)GQA_CHECK((saddr & 15u) == 0 && (lbo_bytes & 15u) == 0, 902);
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// tcgen05.ld / st, 32 lanes x 32-bit, repeated 32 / 16 times along columns.
// Each thread of the warp reads (writes) its own TMEM lane.
#define GQA_R8(p, o) "=r"(p[o + 0]), "=r"(p[o + 1]), "=r"(p[o + 2]), "=r"(p[o + 3]), "=r"(p[o + 4]), \
                     "=r"(p[o + 5]), "=r"(p[o + 6]), "=r"(p[o + 7])
#define GQA_W8(p, o) "r"(p[o + 0]), "r"(p[o + 1]), "r"(p[o + 2]), "r"(p[o + 3]), "r"(p[o + 4]), \
                     "r"(p[o + 5]), "r"(p[o + 6]), "r"(p[o + 7])

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  if (!GQA_CHECK((taddr & 0xFFFFu) + 32u <= 512u, 904)) return;  // warp-uniform address
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : GQA_R8(r, 0), GQA_R8(r, 8), GQA_R8(r, 16), GQA_R8(r, 24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  if (!GQA_CHECK((taddr & 0xFFFFu) + 16u <= 512u, 904)) return;  // warp-uniform address
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : GQA_R8(r, 0), GQA_R8(r, 8)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  if (!GQA_CHECK((taddr & 0xFFFFu) + 32u <= 512u, 904)) return;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      GQA_W8(r, 0), GQA_W8(r, 8), GQA_W8(r, 16), GQA_W8(r, 24)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  if (!GQA_CHECK((taddr & 0xFFFFu) + 16u <= 512u, 904)) return;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      GQA_W8(r, 0), GQA_W8(r, 8)
      : "memory");
}
// Registers written by tcgen05.ld are only valid after tcgen05.wait::ld. This
// empty asm ties each register to a point after the wait so the compiler
// cannot hoist a use above it.
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
template <int N>
__device__ __forceinline__ void reg_fence_n(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// ---------------------------------------------------------------------------
// Legacy warp-level MMA path (used by the HBM-bound streaming kernel).
// ---------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Two e4m3 values (low byte -> low half) to two f16, exactly (every e4m3 value is
// an f16 value).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t pair16) {
  uint32_t r;
  const uint16_t x = (uint16_t)pair16;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(x));
  return r;
}

// Transpose of an 8 x 8 matrix of 16-bit values held one row pair per lane in the
// mma fragment layout (lane 4g + t holds row g, columns 2t, 2t + 1).
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t r;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(r) : "r"(x));
  return r;
}

// Byte permute: result byte i = byte (sel >> 4i & 7) of {b:a}.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Two 16-bit values of the I/O type (bf16 when BF16) as two f16.
template <bool BF16>
__device__ __forceinline__ uint32_t to_f16x2(uint32_t x) {
  if constexpr (BF16) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&x));
    const __half2 h = __float22half2_rn(f);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    return x;
  }
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-lane fp32 arithmetic (sm_100: one instruction for two values).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// Three-input maximum (one instruction on sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two values on the FMA pipe instead of the MUFU pipe, so the two
// pipes share the softmax's exponentials. Cody-Waite style range reduction:
// n = round(x) through the 1.5 * 2^23 addend (n lands in the low mantissa bits
// of t), f = x - n in [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted for
// near-equioscillating relative error (tests/exp2_fit.py, which a CPU test binds
// to these constants; max relative error 1.5e-4, far below the 2^-8 step of the
// bf16 P it feeds); the result's
// exponent field then gets n added. x is clamped at -126 so the exponent never
// underflows into the sign bit: x < -126 (masked keys, -inf) gives about 1e-38
// instead of 0, negligible against any visible key; a NaN x (row with no visible
// key) also lands on the clamp, so callers keep MUFU columns in every row for the
// NaN to propagate.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  constexpr float kC0 = 0.9999280571937561f, kC1 = 0.6932609677314758f;
  constexpr float kC2 = 0.2426111251115799f, kC3 = 0.0551716685295105f;
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 t = add2(x, make_float2(kRound, kRound));
  const float2 n = add2(t, make_float2(-kRound, -kRound));
  const float2 f = fma2(n, make_float2(-1.0f, -1.0f), x);
  float2 p = fma2(make_float2(kC3, kC3), f, make_float2(kC2, kC2));
  p = fma2(p, f, make_float2(kC1, kC1));
  p = fma2(p, f, make_float2(kC0, kC0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

// Pack two floats into one 32-bit register of two 16-bit values (lo = a).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a tile whose rows
// are 128 bytes and stored with the TMA / UMMA 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

}  // namespace gqa
