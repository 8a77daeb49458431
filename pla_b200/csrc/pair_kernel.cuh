// Plane-pair kernel: depthwise 7x7 on NCHW stacks of 56 x 56 planes, 16-bit
// data (stage 1 of the ConvNeXt-T sweep of data/depthwise_conv_7x7.py's
// benchmark configurations: N=256, C=96, 56 x 56).
//
// The plane-tile kernel covers a 56-wide plane with one 64-wide tile, so 8 of
// every 64 columns it computes fall outside the plane and are dropped.  Here
// every lane computes outputs that are stored:
//  * stage = two adjacent planes (planes are contiguous in NCHW), loaded as one
//    3-D TMA box of 72 x 62 x 2 elements into a 2-deep shared-memory ring
//    guarded by mbarriers (bounded waits), one stage ahead, by thread 0; the
//    out-of-bounds fill of the box supplies the zero padding (3 rows and
//    columns on every side, plus the plane past the end of an odd stack);
//  * 224 threads = 2 planes x 8 row groups x 14 column groups; a thread owns
//    7 rows x 4 columns of its plane and reads each of its 13 input rows once
//    with three 64-bit shared loads (bank-conflict free: a half-warp's 16
//    loads cover 128 consecutive bytes or two runs that do not share banks);
//  * taps: the 49 taps of the thread's channel packed two per register,
//    mixed-precision FMAs (16-bit x and w, fp32 accumulator) in the fixed
//    (ky, kx) order, first tap added to -0, bias in fp32, one rounding: the
//    same bits as every other kernel of this library and the oracle;
//  * persistent CTAs own contiguous ranges of stages.  With C even a stage
//    index v is (channel pair v / N, image v % N), so the stages of a CTA keep
//    the same two filters in registers; with C odd stages are consecutive
//    plane pairs and the filters change every stage.
#pragma once

#include "pla_common.cuh"

namespace pla {

template <typename T>
struct PairGeom {
  static_assert(sizeof(T) == 2, "16-bit planes");
  static constexpr int S = 56;                   // plane side
  static constexpr int PL = 2;                   // planes per stage
  static constexpr int R = 7;                    // output rows per thread
  static constexpr int RG = S / R;               // row groups per plane
  static constexpr int CG = S / 4;               // column groups per plane
  static constexpr int THREADS = PL * RG * CG;   // 224
  static constexpr int LEFT = 16 / sizeof(T);    // 16-byte aligned TMA x start, >= 3-column halo
  static constexpr int PITCH = S + 2 * LEFT;     // box width (row pitch in shared memory)
  static constexpr int ROWS = S + 6;             // box height
  static_assert((PITCH * sizeof(T)) % 16 == 0, "TMA box inner extent must be a multiple of 16 B");
  static constexpr uint32_t BYTES = PL * ROWS * PITCH * sizeof(T);
  static constexpr uint32_t STAGE = (BYTES + 127u) & ~127u;
  static constexpr int NS = 2;                   // ring stages
  static constexpr uint32_t SMEM = NS * STAGE + 16;
};

struct PairArgs {
  const void* w;      // [C][49]
  const void* b;      // [C] or nullptr
  void* y;            // output planes, dense 56 x 56
  int N, C;
  int planes;         // N * C (< 2^31, host check)
  int stages;         // ceil(planes / 2)
  int cp_major;       // 1: C even, stage v = (channel pair v / N, image v % N)
  FastDiv div_n, div_c;
};

// First plane of stage v.
__device__ __forceinline__ int pair_first_plane(int v, const PairArgs& a) {
  if (!a.cp_major) return 2 * v;
  const int cp = fdiv(v, a.div_n);
  const int n = v - cp * a.N;
  return n * a.C + 2 * cp;
}

template <typename T>
__global__ void __launch_bounds__(PairGeom<T>::THREADS, 4)
    pair_kernel(const __grid_constant__ CUtensorMap tmap, const PairArgs a) {
  using G = PairGeom<T>;
  constexpr int NT = kTaps;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::NS * G::STAGE);

  const int tid = threadIdx.x;
  const int pl = tid / (G::RG * G::CG);
  const int rem = tid - pl * (G::RG * G::CG);
  const int rg = rem / G::CG;
  const int cg = rem - rg * G::CG;

  if (tid == 0) {
    prefetch_tensormap(&tmap);
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Programmatic dependent launch: the set-up above overlaps the previous
  // kernel's drain; every global access below comes after it completed.
  grid_dependency_wait();

  const int v_begin = static_cast<int>((static_cast<long long>(a.stages) * blockIdx.x) / gridDim.x);
  const int v_end = static_cast<int>((static_cast<long long>(a.stages) * (blockIdx.x + 1)) / gridDim.x);

  // Thread 0: load stage v into ring slot s.
  auto issue = [&](int v, int s) {
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[s], G::BYTES);
    tma_load_3d(smem + s * G::STAGE, &tmap, &bars[s], -G::LEFT, -kHalo, pair_first_plane(v, a));
  };
  if (tid == 0 && v_begin < v_end) issue(v_begin, 0);

  const T* wt_base = static_cast<const T*>(a.w);
  const T* b_base = static_cast<const T*>(a.b);
  uint32_t wh[(NT + 1) / 2];
  int cur_c = -1;
  float bias = 0.f;
  constexpr int PLANE_PX = G::S * G::S;

  for (int v = v_begin, it = 0; v < v_end; ++v, ++it) {
    const int s = it & 1;
    // Slot s ^ 1 was last read in iteration it - 1, which every thread left
    // through the barrier that ended it.
    if (tid == 0 && v + 1 < v_end) issue(v + 1, s ^ 1);
    if (tid == 0 && v + 1 == v_end) launch_dependents();  // last load issued

    const int p = pair_first_plane(v, a) + pl;
    const bool ok = p < a.planes;
    const int c = ok ? p - fdiv(p, a.div_c) * a.C : 0;
    if (c != cur_c) {
      cur_c = c;
      load_taps16<NT>(wt_base, c, wh);
      bias = b_base ? to_acc(b_base[c]) : 0.f;
    }

    mbar_wait_bounded(&bars[s], (it >> 1) & 1);

    // u[k / 2] half k & 1 below is input column 4 cg - 4 + k of this plane.
    const T* sp = reinterpret_cast<const T*>(smem + s * G::STAGE) + pl * (G::ROWS * G::PITCH) +
                  (rg * G::R) * G::PITCH + 4 * cg + (G::LEFT - 4);
    float acc[G::R][4];
#pragma unroll
    for (int ir = 0; ir < G::R + 6; ++ir) {
      const uint2 q0 = *reinterpret_cast<const uint2*>(sp + ir * G::PITCH);
      const uint2 q1 = *reinterpret_cast<const uint2*>(sp + ir * G::PITCH + 4);
      const uint2 q2 = *reinterpret_cast<const uint2*>(sp + ir * G::PITCH + 8);
      const uint32_t u[6] = {q0.x, q0.y, q1.x, q1.y, q2.x, q2.y};
#pragma unroll
      for (int kx = 0; kx < 7; ++kx) {
#pragma unroll
        for (int r = 0; r < G::R; ++r) {
          const int ky = ir - r;
          if (ky >= 0 && ky < 7) {
            const int k = ky * 7 + kx;
            const unsigned short wv = half_of(wh[k >> 1], k & 1);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int col = j + kx + 1;  // input column 4 cg + j + kx - 3
              acc[r][j] = fma_mix(T(), half_of(u[col >> 1], col & 1), wv, (ky == 0 && kx == 0) ? -0.0f : acc[r][j]);
            }
          }
        }
      }
    }
    // Every thread is done with slot s before thread 0 refills it.
    __syncthreads();

    if (ok) {
      T* yp = static_cast<T*>(a.y) + static_cast<long long>(p) * PLANE_PX + (rg * G::R) * G::S + 4 * cg;
      const bool has_bias = b_base != nullptr;
#pragma unroll
      for (int r = 0; r < G::R; ++r) {
        float o0 = acc[r][0], o1 = acc[r][1], o2 = acc[r][2], o3 = acc[r][3];
        if (has_bias) {
          o0 += bias; o1 += bias; o2 += bias; o3 += bias;
        }
        store4(yp + r * G::S, o0, o1, o2, o3);
      }
    }
  }
}

}  // namespace pla
