// Shared device helpers for the 7x7 depthwise / stencil kernels (sm_100a).
//
// Numerical contract of every kernel (it is also what the CPU oracle in
// oracle/pla_oracle.c restates): per output point the 49 taps are
// accumulated in row-major (ky, kx) order with a correctly rounded fused
// multiply-add, starting from +0, in fp32 (fp64 for fp64 data); the bias is
// added once at the end and the sum is rounded to the output type with
// round-to-nearest-even.  Taps that fall on the zero padding contribute an
// exact +-0 and may be skipped without changing the value.  This follows
// torch.nn.Conv2d(C, C, 7, padding=3, groups=C) as used by
// data/depthwise_conv_7x7.py:15-29 and data/stencil_7x7.py:5-12, and the
// "bias in the accumulator type before the output cast" convention of
// data/stencil_direct_cuda_v7/stencil_cuda_kernel.cu:64-71.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace pla {

constexpr int kTaps = 49;
constexpr int kHalo = 3;

// Device fault word (bit 0: an mbarrier wait exceeded its time bound;
// bit 1: a wait for a neighbouring GPU's halo flag timed out).
__device__ unsigned int g_device_faults;

// n / d for 0 <= n < 2^31 by one multiply-high and a shift; the divisor is
// fixed per launch.  m = ceil(2^(31+l) / d) with l = ceil(log2 d) makes the
// quotient exact for every n < 2^31 (tests/test_host_logic.py checks the
// same arithmetic exhaustively on edge cases).
struct FastDiv {
  unsigned int d, m, s;
};
inline FastDiv make_fastdiv(unsigned int d) {
  FastDiv f;
  f.d = d;
  f.m = 0;
  f.s = 0;
  if (d <= 1) return f;
  unsigned int l = 0;
  while ((1ull << l) < d) ++l;
  f.m = static_cast<unsigned int>(((1ull << (31 + l)) + d - 1) / d);
  f.s = l - 1;
  return f;
}
__device__ __forceinline__ int fdiv(int n, const FastDiv& f) {
  return f.d == 1 ? n : static_cast<int>(__umulhi(static_cast<unsigned int>(n), f.m) >> f.s);
}

// One filter passed by value (kernel-parameter / constant bank): the FMA
// instructions read the taps as uniform operands instead of holding 49
// registers per thread.  Filled on the host from fp32 values (16-bit taps
// widen exactly).
struct HostTaps {
  float w[kTaps];
  float b;
  int has_b;
};

template <typename T> struct AccOf { using type = float; };
template <> struct AccOf<double> { using type = double; };

__device__ __forceinline__ float to_acc(float v) { return v; }
__device__ __forceinline__ float to_acc(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_acc(__half v) { return __half2float(v); }
__device__ __forceinline__ double to_acc(double v) { return v; }

template <typename T> __device__ __forceinline__ T from_acc(typename AccOf<T>::type v);
template <> __device__ __forceinline__ float from_acc<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_acc<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_acc<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ double from_acc<double>(double v) { return v; }

__device__ __forceinline__ float fma_rn(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_rn(double a, double b, double c) { return __fma_rn(a, b, c); }

// Mixed-precision FMA of sm_100 (PTX fma.rn.f32.bf16 / fma.rn.f32.f16):
// 16-bit a and b, fp32 c, a * b + c rounded once to fp32.  Widening a 16-bit
// value to fp32 is exact, so this equals fmaf(float(a), float(b), c) bit for
// bit (checked on B200 over 2^24 random operand triples, specials included);
// it lets 16-bit kernels use x and w straight from packed 16-bit storage.
// The tag argument selects the format.
__device__ __forceinline__ float fma_mix(__nv_bfloat16, unsigned short a, unsigned short b, float c) {
  float d;
  asm("fma.rn.f32.bf16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float fma_mix(__half, unsigned short a, unsigned short b, float c) {
  float d;
  asm("fma.rn.f32.f16 %0, %1, %2, %3;" : "=f"(d) : "h"(a), "h"(b), "f"(c));
  return d;
}
// Half `hi` (0: bits 0-15, 1: bits 16-31) of a packed pair.
__device__ __forceinline__ unsigned short half_of(uint32_t w, int hi) {
  unsigned short l, h;
  asm("mov.b32 {%0, %1}, %2;" : "=h"(l), "=h"(h) : "r"(w));
  return hi ? h : l;
}
// The NT taps of filter c as packed 16-bit pairs: tap k in half k & 1 of p[k / 2].
template <int NT, typename T>
__device__ __forceinline__ void load_taps16(const T* w, int c, uint32_t (&p)[(NT + 1) / 2]) {
  const unsigned short* wb = reinterpret_cast<const unsigned short*>(w) + c * NT;
#pragma unroll
  for (int k = 0; k < (NT + 1) / 2; ++k)
    p[k] = static_cast<uint32_t>(wb[2 * k]) | (2 * k + 1 < NT ? static_cast<uint32_t>(wb[2 * k + 1]) << 16 : 0u);
}

// ---------------------------------------------------------------------------
// mbarrier + TMA (cp.async.bulk.tensor) wrappers.  Loads only, never
// multicast: every tensor map in this library covers this GPU's own memory.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Waits for phase `parity` of `bar` for at most ~`limit_ns` nanoseconds.
// On time-out it records bit 0 in the device fault word and returns false;
// the caller then carries on (its results are undefined and the host sees
// the fault through pla_read_device_faults()).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > limit_ns) {
      atomicOr(&g_device_faults, 1u);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// Cluster launch control (sm_100): a running CTA takes over the work of a CTA
// of the same grid that has not started yet.  clc_try_cancel asks for one
// (the 16-byte response lands in `resp`, 16-byte aligned shared memory, and
// completes `bar`); clc_claimed_x reads the response after that phase: the
// cancelled CTA's blockIdx.x, or -1 when no CTA was left to cancel.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void clc_try_cancel(void* resp, uint64_t* bar) {
  mbar_arrive_expect_tx(bar, 16);
  asm volatile("clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];"
               ::"r"(smem_u32(resp)), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ int clc_claimed_x(const void* resp) {
  int ok = 0, x = -1;
  asm volatile(
      "{ .reg .b128 r; .reg .pred p; ld.shared.b128 r, [%2];\n"
      " clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n"
      " selp.s32 %0, 1, 0, p;\n"
      " @p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, r; }"
      : "=r"(ok), "+r"(x)
      : "r"(smem_u32(resp))
      : "memory");
  return ok ? x : -1;
}

// ---------------------------------------------------------------------------
// System-scope flags between GPUs (row-band halo exchange over peer memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
  unsigned int old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Spins until *flag >= target (the flag only grows) for at most ~limit_ns.
// On time-out it records bit 1 in the device fault word and returns false;
// the caller carries on (results undefined, host sees the fault).
__device__ __forceinline__ bool wait_flag_geq(const unsigned int* flag, unsigned int target,
                                              uint64_t limit_ns = 2000000000ull) {
  if (ld_acquire_sys(flag) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (ld_acquire_sys(flag) >= target) return true;
      __nanosleep(128);
    }
    // Past the bound, or another wait already gave up (the neighbour is not
    // answering): record and stop, so later edge tiles do not wait again.
    if (global_timer_ns() - t0 > limit_ns || (*reinterpret_cast<volatile unsigned int*>(&g_device_faults) & 2u)) {
      atomicOr(&g_device_faults, 2u);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Programmatic dependent launch (griddepcontrol): wait for the grids this
// one depends on to complete and flush their memory; let the grids that
// depend on this one start launching (their CTAs then block in their own
// wait).  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// Shared-memory row loads: 12 consecutive elements starting at a 4-element
// aligned position, widened to fp32.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void load_row12(const float* s, float (&r)[12]) {
  const float4 a = *reinterpret_cast<const float4*>(s);
  const float4 b = *reinterpret_cast<const float4*>(s + 4);
  const float4 c = *reinterpret_cast<const float4*>(s + 8);
  r[0] = a.x; r[1] = a.y; r[2] = a.z; r[3] = a.w;
  r[4] = b.x; r[5] = b.y; r[6] = b.z; r[7] = b.w;
  r[8] = c.x; r[9] = c.y; r[10] = c.z; r[11] = c.w;
}

__device__ __forceinline__ void unpack_bf16x2(uint32_t u, float& lo, float& hi) {
  lo = __uint_as_float(u << 16);
  hi = __uint_as_float(u & 0xffff0000u);
}

__device__ __forceinline__ void load_row12(const __nv_bfloat16* s, float (&r)[12]) {
  const uint2 a = *reinterpret_cast<const uint2*>(s);
  const uint2 b = *reinterpret_cast<const uint2*>(s + 4);
  const uint2 c = *reinterpret_cast<const uint2*>(s + 8);
  unpack_bf16x2(a.x, r[0], r[1]); unpack_bf16x2(a.y, r[2], r[3]);
  unpack_bf16x2(b.x, r[4], r[5]); unpack_bf16x2(b.y, r[6], r[7]);
  unpack_bf16x2(c.x, r[8], r[9]); unpack_bf16x2(c.y, r[10], r[11]);
}

__device__ __forceinline__ void unpack_half2(uint32_t u, float& lo, float& hi) {
  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
  lo = f.x;
  hi = f.y;
}

__device__ __forceinline__ void load_row12(const __half* s, float (&r)[12]) {
  const uint2 a = *reinterpret_cast<const uint2*>(s);
  const uint2 b = *reinterpret_cast<const uint2*>(s + 4);
  const uint2 c = *reinterpret_cast<const uint2*>(s + 8);
  unpack_half2(a.x, r[0], r[1]); unpack_half2(a.y, r[2], r[3]);
  unpack_half2(b.x, r[4], r[5]); unpack_half2(b.y, r[6], r[7]);
  unpack_half2(c.x, r[8], r[9]); unpack_half2(c.y, r[10], r[11]);
}

// Four consecutive outputs, one vector store (16 B for fp32, 8 B otherwise).
__device__ __forceinline__ void store4(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}
__device__ __forceinline__ void store4(__nv_bfloat16* p, float a, float b, float c, float d) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(a, b);
  __nv_bfloat162 hi = __floats2bfloat162_rn(c, d);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&lo);
  v.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = v;
}
__device__ __forceinline__ void store4(__half* p, float a, float b, float c, float d) {
  __half2 lo = __floats2half2_rn(a, b);
  __half2 hi = __floats2half2_rn(c, d);
  uint2 v;
  v.x = *reinterpret_cast<uint32_t*>(&lo);
  v.y = *reinterpret_cast<uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(p) = v;
}

}  // namespace pla
