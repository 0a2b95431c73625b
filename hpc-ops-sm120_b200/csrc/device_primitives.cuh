// device_primitives.cuh -- thin inline-PTX wrappers for sm_100a used by the
// decode kernels: mbarriers, TMA tiled loads, ldmatrix/movmatrix, the
// m16n8k16 BF16 tensor-core MMA, exp2, named barriers and programmatic
// dependent launch.  Each wrapper is one PTX instruction (or a bounded loop
// around one) documented in the PTX ISA.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace adb {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
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

__device__ __forceinline__ uint32_t smid() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Sticky per-device error word, set when a bounded wait gives up.  Defined
// here: the library is one translation unit (decode_capi.cu).
__device__ int g_adb_error_flag = 0;

constexpr int kErrWaitTimeout = 1;
constexpr int kErrWorkspace = 2;  // a scheduler counter left its bounds (dirty header)
constexpr int kErrPeerTimeout = 4;  // a peer's partial states did not arrive in time
constexpr int kErrAppendFull = 8;   // append: a sequence's cache had no free position
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait

// Waits for the given phase parity of an mbarrier.  The wait is bounded: if
// `abort_flag` (shared) is already set it returns false at once; after
// kWaitLimitNs it sets `abort_flag` and the device error word and returns
// false, so that no thread of the CTA can spin forever.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t start = 0;
  for (uint32_t i = 0;; ++i) {
    if (*abort_flag) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      const uint64_t now = global_timer_ns();
      if (start == 0) {
        start = now;
      } else if (now - start > kWaitLimitNs) {
        *abort_flag = 1;
        atomicOr(&g_adb_error_flag, kErrWaitTimeout);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
// 3-D tiled bulk tensor load global -> shared, completion via mbarrier
// transaction bytes.  No multicast (plain CTA-local load).
// The copy carries an L2 cache-eviction policy (createpolicy).
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar), "l"(policy)
      : "memory");
}

// 4-D tiled bulk tensor load (paged caches laid out [blocks][page][heads][D]).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int x, int y,
                                            int z, int w, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(bar), "l"(policy)
      : "memory");
}

// Prefetch of one tiled box into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}

// L2 policy for data read once: evict it first (all of the access).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- warp MMA
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// D(16x8, f32) += A(16x16, bf16, row) * B(16x8, bf16, col)
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  const __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Two e4m3 values (the low and high byte of `pair`) to an f16x2 register
// (low half from the low byte), exactly: every e4m3 value is an f16 value
// (cvt.rn.f16x2.e4m3x2, PTX ISA, sm_89 and later; the NaN code stays NaN).
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t pair) {
  uint32_t out;
  const uint16_t lo16 = static_cast<uint16_t>(pair);
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(lo16));
  return out;
}

// Pairs of the four e4m3 bytes (b0, b1, b2, b3) of x as f16x2:
// (b0, b1), (b2, b3) -- consecutive elements -- and (b0, b2), (b1, b3).
__device__ __forceinline__ uint32_t e4m3_01(uint32_t x) { return e4m3x2_to_f16x2(x); }
__device__ __forceinline__ uint32_t e4m3_23(uint32_t x) { return e4m3x2_to_f16x2(x >> 16); }
__device__ __forceinline__ uint32_t e4m3_02(uint32_t x) { return e4m3x2_to_f16x2(__byte_perm(x, 0u, 0x0020u)); }
__device__ __forceinline__ uint32_t e4m3_13(uint32_t x) { return e4m3x2_to_f16x2(__byte_perm(x, 0u, 0x0031u)); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_u16x2(uint16_t lo, uint16_t hi) {
  return static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
}

// 2^x with the SFU instruction (ex2.approx.ftz: 2^-inf = +0, 2^0 = 1).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------- sync
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue; it must call griddep_wait() before touching this grid's output.
// System-scope strong (relaxed) store / load of a 32-bit flag: the flags that
// ranks on other GPUs raise in this GPU's memory (and read in theirs).  With
// fence_acq_rel_sys() they form the PTX memory model's release pattern (a
// fence, then strong writes) and acquire pattern (strong reads, then a
// fence), so a batch of flags costs one system-scope fence, not one per flag
// as st.release.sys / ld.acquire.sys would (a system-scope fence waits for
// every earlier write of the thread, peer writes over NVLink included).
__device__ __forceinline__ void st_relaxed_sys_u32(uint32_t* ptr, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(ptr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_relaxed_sys_u32(const uint32_t* ptr) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ptr) : "memory");
  return v;
}

// Release/acquire fence at system scope (orders this thread's, and by
// cumulativity everything it has observed, earlier memory accesses before
// its later ones for observers on other GPUs); lighter than fence.sc.sys.
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

}  // namespace adb
