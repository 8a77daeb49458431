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
//                   -> s / m / q [buf][g][p]; then the cluster barrier is
//                   ARRIVED at (release);
//   ln_combine      after the barrier's WAIT (acquire), every CTA loads all
//                   groups' (s_g, m_g, q_g) of its pixels from the owning
//                   ranks, eight groups in flight at a time, and combines them
//                   in group order: mean = sum s_g / C,
//                   M = sum (q_g + n_g (m_g - mean)^2)  (Chan, Golub and
//                   LeVeque's pairwise variance update: stable, one exchange),
//                   inv = 1 / sqrt(M / C + eps);
//   ln_normalize    z = ((v - mean) * inv) * gamma + beta, in place in os,
//                   16 bytes of channels per thread and step.
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
// normalised and stored then.  The partials alternate between two buffers by
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

// Shared memory of the epilogue: sums s[2][GL][P], group means m[2][GL][P]
// and squared deviations q[2][GL][P] (two buffers by stage parity), then
// mean[P], inv[P], and the CTA's scales and shifts gamma[LANES], beta[LANES].
template <int LANES, int P>
struct LnSmem {
  static constexpr int GL = LANES / 32;
  static constexpr uint32_t BYTES = static_cast<uint32_t>((6 * GL * P + 2 * P + 2 * LANES) * sizeof(float));
};

template <int LANES, int P>
struct LnView {
  static constexpr int GL = LANES / 32;
  float* base;
  __device__ float* part(int buf) const { return base + buf * GL * P; }         // s_g
  __device__ float* part_m(int buf) const { return base + (2 + buf) * GL * P; }  // m_g
  __device__ float* part2(int buf) const { return base + (4 + buf) * GL * P; }   // q_g
  __device__ float* mean() const { return base + 6 * GL * P; }
  __device__ float* inv() const { return base + 6 * GL * P + P; }
  __device__ float* gamma() const { return base + 6 * GL * P + 2 * P; }
  __device__ float* beta() const { return gamma() + LANES; }
};

// The CTA's LANES scales and shifts (channels c0 ...) as fp32 in shared
// memory (1 / 0 for NULL vectors or channels past C).  Called once, before
// the first stage; the stage barriers order it before any use.
template <typename T, int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_load_affine(const LnView<LANES, P>& v, const void* gamma, const void* beta,
                                               int c0, int C) {
  for (int l = threadIdx.x; l < LANES; l += THREADS) {
    const int c = c0 + l;
    v.gamma()[l] = gamma && c < C ? to_acc(static_cast<const T*>(gamma)[c]) : 1.f;
    v.beta()[l] = beta && c < C ? to_acc(static_cast<const T*>(beta)[c]) : 0.f;
  }
}

// Channels of 32-channel group `gi` of this CTA's stage that exist (0..32).
__device__ __forceinline__ int group_size(int C, int c0, int gi) {
  const int n = C - c0 - gi * 32;
  return n < 0 ? 0 : (n > 32 ? 32 : n);
}

// (s_g, m_g, q_g) of `n` values, in ascending order from +0.
template <bool FULL>
__device__ __forceinline__ void group_stats(const float (&x)[32], int n, float& s, float& m, float& q2) {
  s = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (FULL || j < n) s = __fadd_rn(s, x[j]);
  m = __fdiv_rn(s, static_cast<float>(FULL ? 32 : n));
  q2 = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (FULL || j < n) {
      const float d = __fsub_rn(x[j], m);
      q2 = __fadd_rn(q2, __fmul_rn(d, d));
    }
  }
}

// (s_g, m_g, q_g) of every (group, pixel) of the stage in os -> buffer `buf`.
template <typename T, int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_local_stats(const T* os, const LnView<LANES, P>& v, int buf, int c0, int C) {
  constexpr int GL = LANES / 32;
  constexpr int VEC = 16 / sizeof(T);
  float* part = v.part(buf);
  float* part_m = v.part_m(buf);
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
    float s = 0.f, m = 0.f, q2 = 0.f;
    if (n == 32)
      group_stats<true>(x, n, s, m, q2);
    else if (n > 0)
      group_stats<false>(x, n, s, m, q2);
    part[t] = s;
    part_m[t] = m;
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
  const uint32_t pa = smem_u32(v.part(buf)), ma = smem_u32(v.part_m(buf)), qa = smem_u32(v.part2(buf));
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
      float mv[CH], qv[CH];
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = g0 + j;
        const uint32_t off = ((g % GL) * P + p) * 4u;
        mv[j] = g < ngroups ? dsmem_ld(dsmem_map(ma + off, g / GL)) : 0.f;
        qv[j] = g < ngroups ? dsmem_ld(dsmem_map(qa + off, g / GL)) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < CH; ++j) {
        const int g = g0 + j;
        if (g < ngroups) {
          const int n = C - g * 32 < 32 ? C - g * 32 : 32;
          const float fn = static_cast<float>(n);
          const float e = __fsub_rn(mv[j], mean);
          m2 = __fadd_rn(m2, __fadd_rn(qv[j], __fmul_rn(fn, __fmul_rn(e, e))));
        }
      }
    }
    mean_s[p] = mean;
    inv_s[p] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(m2, fc), eps)));
  }
}

// z = ((v - mean) * inv) * gamma + beta in place, one 16-byte chunk of
// channels at a time.  Thread tid always handles chunk tid % NQ of a pixel
// (THREADS is a multiple of NQ), channels c0 + VEC * (tid % NQ) + [0, VEC),
// whose scales and shifts it reads from shared memory (ln_load_affine).
// C * sizeof(T) is a multiple of 16 bytes, so a chunk is all in or all out.
template <typename T, int LANES>
struct LnChunk {
  static constexpr int VEC = 16 / sizeof(T);
  static constexpr int NQ = LANES / VEC;  // chunks per pixel
};

template <typename T, int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_normalize(T* os, const LnView<LANES, P>& v, int c0, int C, bool has_gamma,
                                             bool has_beta) {
  using K = LnChunk<T, LANES>;
  static_assert(THREADS % K::NQ == 0, "fixed chunk per thread");
  constexpr int PSTEP = THREADS / K::NQ;
  const float* mean_s = v.mean();
  const float* inv_s = v.inv();
  const int q = threadIdx.x % K::NQ;
  if (c0 + K::VEC * q >= C) return;
  float g[K::VEC], bt[K::VEC];
#pragma unroll
  for (int j = 0; j < K::VEC; ++j) {
    g[j] = v.gamma()[K::VEC * q + j];
    bt[j] = v.beta()[K::VEC * q + j];
  }
  for (int p = threadIdx.x / K::NQ; p < P; p += PSTEP) {
    uint4* cp = reinterpret_cast<uint4*>(os + p * LANES) + q;
    uint4 u = *cp;
    T* e = reinterpret_cast<T*>(&u);
    const float mean = mean_s[p], inv = inv_s[p];
#pragma unroll
    for (int j = 0; j < K::VEC; ++j) {
      float t = __fmul_rn(__fsub_rn(to_acc(e[j]), mean), inv);
      if (has_gamma) t = __fmul_rn(t, g[j]);
      if (has_beta) t = __fadd_rn(t, bt[j]);
      e[j] = from_acc<T>(t);
    }
    *cp = u;
  }
}

}  // namespace pla
