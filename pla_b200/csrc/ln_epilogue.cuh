// Channel LayerNorm epilogue for the NHWC depthwise kernels (the "dwconv ->
// norm" pair of a ConvNeXt block: nn.LayerNorm(C, eps) over the channels of
// every pixel of the depthwise output).  No reference counterpart: the
// reference's operator is the depthwise half (data/depthwise_conv_7x7.py:15-29).
//
// A stage of the NHWC kernels holds LANES channels of a set of P pixels in
// shared memory ("os", element (p, l) at os[p * LANES + l]).  LayerNorm needs
// all C channels of a pixel, so the kernels run as thread-block clusters: the
// CTA of cluster rank r owns channels [r * LANES, (r + 1) * LANES) of the
// same pixels, and the per-pixel partial sums travel between the CTAs
// through distributed shared memory (mapa + ld.shared::cluster), with two
// cluster barriers per stage:
//
//   1. each CTA sums its channels of every pixel, per 32-channel group, in
//      ascending channel order -> part[g][p];
//   2. barrier; every CTA reads all ranks' partials of its pixels and adds
//      them in channel-group order -> mean = S / C;
//   3. each CTA sums (v - mean)^2 the same way -> part2[g][p];
//   4. barrier; every CTA adds all partials -> inv = 1 / sqrt(M / C + eps);
//   5. z = ((v - mean) * inv) * gamma + beta, written back into os (the
//      kernel's TMA store then sends it out).
//
// Every operation is a correctly rounded fp32 add / multiply / divide /
// square root in a fixed tree (the CPU oracle's
// oracle_depthwise7x7_layernorm_nhwc restates it), so the result is the same
// bit for bit.  v is the depthwise output already rounded to T, exactly what
// the unfused pair would hand to the LayerNorm.
//
// Reuse of part / part2 across stages needs no third barrier: a peer reads a
// CTA's part[] between barrier 1 and its own arrival at barrier 2 of the same
// stage, and the owner rewrites part[] only after barrier 2; part2[] is read
// between barrier 2 and the next stage's barrier 1 and rewritten after that
// barrier.  The kernels end with one more cluster barrier so that no CTA
// exits while a peer may still read its shared memory.
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
// All threads of all CTAs of the cluster; release / acquire orders the
// shared-memory writes before it against the peers' reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
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

// Shared-memory footprint of the epilogue: part[GL][P], part2[GL][P], mean[P], inv[P].
template <int LANES, int P>
struct LnSmem {
  static constexpr int GL = LANES / 32;
  static constexpr uint32_t BYTES = static_cast<uint32_t>((2 * GL * P + 2 * P) * sizeof(float));
};

// Sum of v (or of (v - mean)^2 when SQ) over channels [0, nv) of one 32-channel
// group of one pixel, in ascending order from +0.  `row` is 16-byte aligned.
template <typename T, bool SQ>
__device__ __forceinline__ float group_sum(const T* row, int nv, float mean) {
  constexpr int VEC = 16 / sizeof(T);
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 32 / VEC; ++q) {
    const uint4 u = reinterpret_cast<const uint4*>(row)[q];
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < VEC; ++j) {
      if (q * VEC + j < nv) {
        const float v = to_acc(e[j]);
        if (SQ) {
          const float d = __fsub_rn(v, mean);
          s = __fadd_rn(s, __fmul_rn(d, d));
        } else {
          s = __fadd_rn(s, v);
        }
      }
    }
  }
  return s;
}

// The epilogue (all threads of the CTA call it, the same number of times in
// every CTA of the cluster).  os: the stage's LANES x P outputs (rounded to
// T); ln_smem: LnSmem<LANES, P>::BYTES of 16-byte aligned shared memory;
// rank / nranks: this CTA's cluster rank and the cluster size; C: channels.
// Thread tid always handles channel tid % LANES in step 5 (THREADS is a
// multiple of LANES), whose scale and shift the caller passes in g / bt.
template <typename T, int LANES, int P, int THREADS>
__device__ __forceinline__ void ln_epilogue(T* os, float* ln_smem, int rank, int nranks, int C, float eps,
                                            bool has_gamma, float g, bool has_beta, float bt) {
  static_assert(LANES % 32 == 0 && THREADS % LANES == 0, "fixed channel per thread");
  constexpr int GL = LANES / 32;
  float* part = ln_smem;
  float* part2 = part + GL * P;
  float* mean_s = part2 + GL * P;
  float* inv_s = mean_s + P;
  const int tid = threadIdx.x;
  const int c0 = rank * LANES;
  const int ngroups = (C + 31) / 32;  // 32-channel groups over all ranks
  const float fc = static_cast<float>(C);

  __syncthreads();  // os complete
  // 1. partial sums per (group, pixel)
  for (int t = tid; t < GL * P; t += THREADS) {
    const int gi = t / P, p = t - gi * P;
    part[t] = group_sum<T, false>(os + p * LANES + gi * 32, C - c0 - gi * 32, 0.f);
  }
  cluster_sync();
  // 2. mean per pixel: all ranks' partials in channel-group order
  const uint32_t part_a = smem_u32(part), part2_a = smem_u32(part2);
  for (int p = tid; p < P; p += THREADS) {
    float s = 0.f;
    for (int r = 0; r < nranks; ++r) {
#pragma unroll
      for (int gi = 0; gi < GL; ++gi) {
        if (r * GL + gi < ngroups) s = __fadd_rn(s, dsmem_ld(dsmem_map(part_a + (gi * P + p) * 4u, r)));
      }
    }
    mean_s[p] = __fdiv_rn(s, fc);
  }
  __syncthreads();
  // 3. partial sums of squared deviations
  for (int t = tid; t < GL * P; t += THREADS) {
    const int gi = t / P, p = t - gi * P;
    part2[t] = group_sum<T, true>(os + p * LANES + gi * 32, C - c0 - gi * 32, mean_s[p]);
  }
  cluster_sync();
  // 4. 1 / sqrt(var + eps) per pixel
  for (int p = tid; p < P; p += THREADS) {
    float m = 0.f;
    for (int r = 0; r < nranks; ++r) {
#pragma unroll
      for (int gi = 0; gi < GL; ++gi) {
        if (r * GL + gi < ngroups) m = __fadd_rn(m, dsmem_ld(dsmem_map(part2_a + (gi * P + p) * 4u, r)));
      }
    }
    inv_s[p] = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(m, fc), eps)));
  }
  __syncthreads();
  // 5. normalise in place
  const int l = tid % LANES;
  if (c0 + l < C) {
    for (int i = tid; i < P * LANES; i += THREADS) {
      const int p = i / LANES;
      float t = __fmul_rn(__fsub_rn(to_acc(os[i]), mean_s[p]), inv_s[p]);
      if (has_gamma) t = __fmul_rn(t, g);
      if (has_beta) t = __fadd_rn(t, bt);
      os[i] = from_acc<T>(t);
    }
  }
}

}  // namespace pla
