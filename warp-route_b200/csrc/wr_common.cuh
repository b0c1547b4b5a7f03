// wr_common.cuh — device helpers shared by the warp-route B200 kernels:
// mbarrier + bulk-copy (TMA) wrappers, L2 cache policies, bounded waits,
// bf16 unpacking and the packed expert layout.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define WR_DEVINL __device__ __forceinline__

namespace wr {

// ---------------------------------------------------------------------------
// Packed expert layout (src/expert_layout.cuh:34-47 of warp-route, with the
// element size as a parameter): per expert [gate I x H][up I x H][down H x I],
// row-major, expert stride rounded up to 128 bytes.
// ---------------------------------------------------------------------------
struct Layout {
  int64_t off_gate;
  int64_t off_up;
  int64_t off_down;
  int64_t stride;
};

__host__ __device__ inline Layout make_layout(int H, int I, int elt) {
  Layout l;
  const int64_t gu = (int64_t)I * H * elt;
  l.off_gate = 0;
  l.off_up = gu;
  l.off_down = 2 * gu;
  const int64_t raw = 2 * gu + (int64_t)H * I * elt;
  l.stride = (raw + 127) & ~int64_t(127);
  return l;
}

// Status bits a kernel ORs into the workspace status word.
enum : uint32_t {
  DEV_TIMEOUT_FULL = 1u << 0,   // consumer gave up waiting for a stage
  DEV_TIMEOUT_EMPTY = 1u << 1,  // producer gave up waiting for a free stage
  DEV_TIMEOUT_GRID = 1u << 2,   // grid-wide barrier gave up
  DEV_TIMEOUT_ACT = 1u << 3,    // activation-window copy never landed
  DEV_TIMEOUT_DRAIN = 1u << 4,  // copies still in flight at exit
  DEV_TIMEOUT_PEER = 1u << 5,   // a peer rank's partial outputs never arrived
};

// Wall-clock bound of every spin in these kernels (ns).  A healthy wait is
// micro-seconds; the bound only turns a lost arrival into an error status.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

WR_DEVINL uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

WR_DEVINL uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------
WR_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
WR_DEVINL void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
WR_DEVINL void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// Arrives `count` times at once (count >= 1).
WR_DEVINL void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
WR_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
WR_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: has the phase with `parity` completed?  (try_wait may
// suspend the thread for a while when the phase is still open; a loop that
// polls several conditions uses this instead.)
WR_DEVINL bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with `parity` to complete.  Gives up after
// kWaitLimitNs, or as soon as *abort is set by another warp; returns false
// then.  `abort` may be null (drain waits ignore it).
WR_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (abort && *abort) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

// ---- bulk async copy (TMA, non-tensor) ------------------------------------
// global -> this CTA's shared memory; completion counted on `bar` in bytes.
// dst, src 16-byte aligned; bytes a multiple of 16.
WR_DEVINL void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                        uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

WR_DEVINL uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
WR_DEVINL uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Brings [p, p + bytes) into L2 without touching shared memory or L1
// (p 16-byte aligned, bytes a multiple of 16).  L2 is the device's point of
// coherence, so a prefetch never makes a later read see stale data.
WR_DEVINL void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetches this CTA's share (CTA b of G) of [p, p + bytes) into L2, in
// 16-byte-aligned pieces; p must be 16-byte aligned.
WR_DEVINL void prefetch_share_l2(const void* p, int64_t bytes, int b, int G) {
  const int64_t units = bytes >> 4;  // whole 16-byte units (a ragged tail is skipped)
  const int64_t u0 = units * b / G, u1 = units * (b + 1) / G;
  if (u1 > u0)
    bulk_prefetch_l2(static_cast<const uint8_t*>(p) + (u0 << 4), (uint32_t)((u1 - u0) << 4));
}

// Orders this thread's generic-proxy accesses against later async-proxy
// (bulk copy) accesses to global / shared memory.
WR_DEVINL void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
WR_DEVINL void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Named barrier among `nthreads` threads (a multiple of 32), id 1..15.
WR_DEVINL void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

WR_DEVINL uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
WR_DEVINL void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// System scope (other GPUs of the node read or write the word), relaxed:
// single-copy atomic for aligned 64-bit words.
WR_DEVINL uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
WR_DEVINL void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// 16-byte read-only global load that does not allocate in L1.
WR_DEVINL uint4 ldg_nc_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ---- element helpers --------------------------------------------------------
WR_DEVINL float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
WR_DEVINL float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }

// A 16-byte chunk of weights widened to fp32 (8 bf16 or 4 fp32 values).
template <typename Tw>
struct Chunk;

template <>
struct Chunk<uint16_t> {  // bf16 bits
  static constexpr int kVec = 8;
  WR_DEVINL static void widen(const uint4& v, float (&f)[8]) {
    f[0] = bf16lo(v.x); f[1] = bf16hi(v.x);
    f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
    f[4] = bf16lo(v.z); f[5] = bf16hi(v.z);
    f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
  }
};

template <>
struct Chunk<float> {
  static constexpr int kVec = 4;
  WR_DEVINL static void widen(const uint4& v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  }
};

template <typename Tw>
WR_DEVINL float load_scalar(const Tw* p, int64_t i);
template <>
WR_DEVINL float load_scalar<uint16_t>(const uint16_t* p, int64_t i) {
  return __uint_as_float(static_cast<uint32_t>(__ldg(p + i)) << 16);
}
template <>
WR_DEVINL float load_scalar<float>(const float* p, int64_t i) {
  return __ldg(p + i);
}

WR_DEVINL float silu(float g) { return g / (1.0f + expf(-g)); }

// Layer output element i (of [T, H]) with the fused residual connection:
// returns v + x[i] and, when next_x is set, stores that sum rounded to the
// layer dtype (round to nearest even) as next_x[i].  x == null: v as is.
template <typename Res>
WR_DEVINL float residual_out(const Res& r, int64_t i, float v) {
  if (!r.x) return v;
  float o;
  if (r.bf16) {
    o = v + __uint_as_float((uint32_t)static_cast<const uint16_t*>(r.x)[i] << 16);
    if (r.next_x)
      static_cast<uint16_t*>(r.next_x)[i] = __bfloat16_as_ushort(__float2bfloat16_rn(o));
  } else {
    o = v + static_cast<const float*>(r.x)[i];
    if (r.next_x) static_cast<float*>(r.next_x)[i] = o;
  }
  return o;
}

// Programmatic dependent launch: wait for the previous kernel on the stream
// (complete, memory visible) / let the next one be scheduled.  Both are
// no-ops for a kernel launched without the programmatic-serialization
// attribute.
WR_DEVINL void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
WR_DEVINL void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace wr
