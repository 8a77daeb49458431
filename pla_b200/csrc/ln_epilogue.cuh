// Channel LayerNorm epilogue for the NHWC depthwise kernels (the "dwconv ->
// norm" pair of a ConvNeXt block: nn.LayerNorm(C, eps) over the channels of
// every pixel of the depthwise output).  No reference counterpart: the
// reference's operator is the depthwise half (data/depthwise_conv_7x7.py:15-29).
//
// A stage of the NHWC kernels holds LANES channels of a set of P pixels in
// shared memory ("os", element (p, l) at os[p * LANES + l]).  LayerNorm needs
// all C channels of a pixel, so the kernels run as thread-block clusters: the
// CTA of cluster rank r owns channels [r * LANES, (r + 1) * LANES) of the
// same pixels, and per-pixel partial results travel between the CTAs through
// distributed shared memory (mapa + ld.shared::cluster), one exchange per
// stage:
//
//   ln_local_stats  each CTA reduces every (32-channel group, pixel) of its
//                   stage on its own: sum s_g and, around the group mean
//                   m_g = s_g / n_g, the sum of squared deviations q_g;
//                   -> part[buf][g][p], part2[buf][g][p]; then the cluster
//                   barrier is ARRIVED at (release);
//   ln_combine      after the barrier's WAIT (acquire), every CTA loads all
//                   groups' (s_g, q_g) of its pixels from the owning ranks,
//                   eight loads in flight at a time, and combines them in
//                   group order: mean = sum s_g / C,
//                   M = sum (q_g + n_g (m_g - mean)^2)  (Chan, Golub and
//                   LeVeque's pairwise variance update: stable, one exchange),
//                   inv = 1 / sqrt(M / C + eps);
//   ln_normalize    z = ((v - mean) * inv) * gamma + beta, in place in os.
//
// Every operation is a correctly rounded fp32 add / multiply / divide /
// square root in a fixed tree, which the CPU oracle's
// oracle_depthwise7x7_layernorm_nhwc restates, so the result is the same bit
// for bit.  v is the depthwise output already rounded to T, exactly what the
// unfused pair would hand to the LayerNorm.
//
// Kernels with an output ring split the barrier around the next stage's
// FMAs (arrive after stage i's local statistics, wait after stage i+1's
// convolution), so the exchange's latency hides behind compute; stage i is
// normalised and stored then.  part / part2 alternate between two buffers by
// stage parity: a peer reads stage i's buffer between wait(i) and its own
// arrive(i + 1), and the owner rewrites it at stage i + 2, after wait(i + 1).
// The kernels end with one more cluster barrier so that no CTA exits while
// a peer may still read its shared memory.
#pragma once

#include "pla_common.cuh"

namespace pla {

struct LnArgs {
  const void* gamma;  // [C] or nullptr (scale 1)
  const void* beta;   // [C] or nullptr (shift 0)
  float eps;
};

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Cluster barrier halves; every thread of every CTA of the cluster executes
// them, alternating arrive / wait.  Release / acquire order the shared-memory
// writes before an arrive against the peers' reads after their wait.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}
// Shared-memory address `addr` of this CTA -> the same offset in cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ float dsmem_ld(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Shared memory of the epilogue: part[2][GL][P], part2[2][GL][P] (two
// buffers by stage parity), mean[P], inv[P].
template <int LANES, int P>
struct LnSmem {
  static constexpr int GL = LANES / 32;
  static constexpr uint32_t BYTES = static_cast<uint32_t>((4 * GL * P + 2 * P) * sizeof(float));
};

template <int LANES, int P>
struct LnView {
  static constexpr int GL = LANES / 32;
  float* base;
  __device__ float* part(int buf) const { return base + buf * GL * P; }
  __device__ float* part2(int buf) const { return base + (2 + buf) * GL * P; }
  __device__ float* mean() const { return base + 4 * GL * P; }
  __device__ float* inv() const { return base + 4 * GL * P + P; }
};

// Channels of 32-channel group `gi` of this CTA's stage that exist (0..32).
__device__ __forceinline__ int group_size(int C, int c0, int gi) {
  const int n = C - c0 - gi * 32;
  return n < 0 ? 0 : (n > 32 ? 32 : n);
}

// (s_g, q_g) of every (group, pixel) of the stage in os -> part[buf], part2[buf].
template <typename T, int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_local_stats(const T* os, const LnView<LANES, P>& v, int buf, int c0, int C) {
  constexpr int GL = LANES / 32;
  constexpr int VEC = 16 / sizeof(T);
  float* part = v.part(buf);
  float* part2 = v.part2(buf);
  for (int t = threadIdx.x; t < GL * P; t += THREADS) {
    const int gi = t / P, p = t - gi * P;
    const int n = group_size(C, c0, gi);
    const uint4* row = reinterpret_cast<const uint4*>(os + p * LANES + gi * 32);  // 16-byte aligned
    float x[32];
#pragma unroll
    for (int q = 0; q < 32 / VEC; ++q) {
      const uint4 u = row[q];
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int j = 0; j < VEC; ++j) x[q * VEC + j] = to_acc(e[j]);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < n) s = __fadd_rn(s, x[j]);
    float q2 = 0.f;
    if (n > 0) {
      const float m = __fdiv_rn(s, static_cast<float>(n));
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (j < n) {
          const float d = __fsub_rn(x[j], m);
          q2 = __fadd_rn(q2, __fmul_rn(d, d));
        }
      }
    }
    part[t] = s;
    part2[t] = q2;
  }
}

// After cluster_wait(): mean and 1 / sqrt(var + eps) of every pixel of the
// stage whose partials are in buffer `buf` of every rank -> v.mean(), v.inv().
template <int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_combine(const LnView<LANES, P>& v, int buf, int C, float eps) {
  constexpr int GL = LANES / 32;
  constexpr int CH = 8;  // remote loads in flight per thread
  const int ngroups = (C + 31) / 32;
  const float fc = static_cast<float>(C);
  const uint32_t pa = smem_u32(v.part(buf)), qa = smem_u32(v.part2(buf));
  float* mean_s = v.mean();
  float* inv_s = v.inv();
  for (int p = threadIdx.x; p < P; p += THREADS) {
    float s = 0.f;
    for (int g0 = 0; g0 < ngroups; g0 += CH) {
      float sv[CH];
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = g0 + j;
        sv[j] = g < ngroups ? dsmem_ld(dsmem_map(pa + ((g % GL) * P + p) * 4u, g / GL)) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < CH; ++j)
        if (g0 + j < ngroups) s = __fadd_rn(s, sv[j]);
    }
    const float mean = __fdiv_rn(s, fc);
    float m2 = 0.f;
    for (int g0 = 0; g0 < ngroups; g0 += CH) {
      float sv[CH], qv[CH];
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = g0 + j;
        const uint32_t off = ((g % GL) * P + p) * 4u;
        sv[j] = g < ngroups ? dsmem_ld(dsmem_map(pa + off, g / GL)) : 0.f;
        qv[j] = g < ngroups ? dsmem_ld(dsmem_map(qa + off, g / GL)) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = g0 + j;
        if (g < ngroups) {
          const int n = C - g * 32 < 32 ? C - g * 32 : 32;
          const float fn = static_cast<float>(n);
          const float e = __fsub_rn(__fdiv_rn(sv[j], fn), mean);
          m2 = __fadd_rn(m2, __fadd_rn(qv[j], __fmul_rn(fn, __fmul_rn(e, e))));
        }
      }
    }
    mean_s[p] = mean;
    inv_s[p] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(m2, fc), eps)));
  }
}

// z = ((v - mean) * inv) * gamma + beta in place.  Thread tid handles channel
// c0 + tid % LANES (THREADS is a multiple of LANES), whose scale and shift it
// holds in g / bt.
template <typename T, int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_normalize(T* os, const LnView<LANES, P>& v, int c0, int C, bool has_gamma,
                                             float g, bool has_beta, float bt) {
  static_assert(LANES % 32 == 0 && THREADS % LANES == 0, "fixed channel per thread");
  const float* mean_s = v.mean();
  const float* inv_s = v.inv();
  if (c0 + static_cast<int>(threadIdx.x % LANES) >= C) return;
  for (int i = threadIdx.x; i < P * LANES; i += THREADS) {
    const int p = i / LANES;
    float t = __fmul_rn(__fsub_rn(to_acc(os[i]), mean_s[p]), inv_s[p]);
    if (has_gamma) t = __fmul_rn(t, g);
    if (has_beta) t = __fadd_rn(t, bt);
    os[i] = from_acc<T>(t);
  }
}

}  // namespace pla
