// Channel-minor block kernel: depthwise 7x7 on small planes.
//
// Used for NHWC (channels_last) activations, and for NCHW activations whose
// planes are too narrow for the plane-tile kernel (ConvNeXt-style 56/28/14/7
// planes).  A CTA owns 32 "lanes" (32 consecutive channels of one image for
// NHWC, 32 consecutive (n, c) planes for NCHW) and one TS x TS spatial tile
// (TS = 7 * BT).  The (TS+6)^2 zero-padded input window of all 32 lanes is
// staged in shared memory as fp32 in [y][x][lane] order (lane pitch 33, so
// both the staging stores and the compute loads are bank-conflict free);
// warp w computes the 7x7 output block (w / BT, w % BT) and lane l the
// channel/plane l, so every thread accumulates 49 outputs x 49 taps with its
// filter in registers, reading each of its 13 input rows once.
#pragma once

#include "pla_common.cuh"

namespace pla {

constexpr int kLanePitch = 33;

struct CmArgs {
  const void* x;
  const void* w;   // [C][49]
  const void* b;   // [C] or nullptr
  void* y;
  int N, C, H, W;
  int tiles_x, tiles_y;  // spatial tiles per plane
  int cgroups;           // NHWC: ceil(C / 32) channel groups per image
  long long groups;      // lane groups: NHWC N * cgroups, NCHW ceil(N*C / 32)
};

template <int BT>
struct CmGeom {
  static constexpr int TS = 7 * BT;
  static constexpr int SW = TS + 6;
  static constexpr int THREADS = 32 * BT * BT;
  static constexpr uint32_t SMEM = SW * SW * kLanePitch * sizeof(float);
};

template <typename T, bool NHWC, int BT>
__global__ void __launch_bounds__(CmGeom<BT>::THREADS)
    cm_kernel(const CmArgs a) {
  using G = CmGeom<BT>;
  extern __shared__ __align__(16) float s[];

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int tiles = a.tiles_x * a.tiles_y;
  const long long g = blockIdx.x / tiles;
  const int tile = static_cast<int>(blockIdx.x % tiles);
  const int ty = tile / a.tiles_x, tx = tile % a.tiles_x;
  const int Y0 = ty * G::TS - kHalo, X0 = tx * G::TS - kHalo;

  const T* x = static_cast<const T*>(a.x);
  const long long HW = static_cast<long long>(a.H) * a.W;
  const long long NC = static_cast<long long>(a.N) * a.C;

  // ---- stage the zero-padded window of all 32 lanes -------------------
  if (NHWC) {
    const int n = static_cast<int>(g / a.cgroups);
    const int c0 = static_cast<int>(g % a.cgroups) * 32;
    const int c = c0 + lane;
    const T* xn = x + static_cast<long long>(n) * HW * a.C + c;
    for (int pos = warp; pos < G::SW * G::SW; pos += G::THREADS / 32) {
      const int sy = pos / G::SW, sx = pos % G::SW;
      const int Y = Y0 + sy, X = X0 + sx;
      float v = 0.f;
      if (c < a.C && Y >= 0 && Y < a.H && X >= 0 && X < a.W)
        v = to_acc(xn[(static_cast<long long>(Y) * a.W + X) * a.C]);
      s[pos * kLanePitch + lane] = v;
    }
  } else {
    const long long p0 = g * 32;
    for (int i = tid; i < 32 * G::SW * G::SW; i += G::THREADS) {
      const int sx = i % G::SW;
      const int rest = i / G::SW;
      const int sy = rest % G::SW;
      const int l = rest / G::SW;
      const int Y = Y0 + sy, X = X0 + sx;
      const long long p = p0 + l;
      float v = 0.f;
      if (p < NC && Y >= 0 && Y < a.H && X >= 0 && X < a.W)
        v = to_acc(x[p * HW + static_cast<long long>(Y) * a.W + X]);
      s[(sy * G::SW + sx) * kLanePitch + l] = v;
    }
  }

  // ---- filter of this lane ---------------------------------------------
  int c;
  bool lane_ok;
  long long plane = 0;
  int n_img = 0;
  if (NHWC) {
    n_img = static_cast<int>(g / a.cgroups);
    c = static_cast<int>(g % a.cgroups) * 32 + lane;
    lane_ok = c < a.C;
  } else {
    plane = g * 32 + lane;
    lane_ok = plane < NC;
    c = static_cast<int>(plane % a.C);
  }
  const int cw = lane_ok ? c : 0;
  const T* wp = static_cast<const T*>(a.w) + static_cast<long long>(cw) * kTaps;
  float wt[kTaps];
#pragma unroll
  for (int k = 0; k < kTaps; ++k) wt[k] = to_acc(wp[k]);
  const bool has_bias = a.b != nullptr;
  const float bias = has_bias ? to_acc(static_cast<const T*>(a.b)[cw]) : 0.f;

  __syncthreads();

  // ---- 7x7 output block of this warp ------------------------------------
  const int bh = warp / BT, bw = warp % BT;
  const float* sb = s + ((7 * bh) * G::SW + 7 * bw) * kLanePitch + lane;
  float acc[7][7];
#pragma unroll
  for (int r = 0; r < 7; ++r)
#pragma unroll
    for (int j = 0; j < 7; ++j) acc[r][j] = 0.f;

#pragma unroll
  for (int iy = 0; iy < 13; ++iy) {
    float v[13];
#pragma unroll
    for (int ix = 0; ix < 13; ++ix) v[ix] = sb[(iy * G::SW + ix) * kLanePitch];
#pragma unroll
    for (int kx = 0; kx < 7; ++kx) {
#pragma unroll
      for (int r = 0; r < 7; ++r) {
        const int ky = iy - r;
        if (ky >= 0 && ky < 7) {
          const float wv = wt[ky * 7 + kx];
#pragma unroll
          for (int j = 0; j < 7; ++j) acc[r][j] = fma_rn(v[j + kx], wv, acc[r][j]);
        }
      }
    }
  }

  if (!lane_ok) return;
  T* y = static_cast<T*>(a.y);
  const int Yb = ty * G::TS + 7 * bh, Xb = tx * G::TS + 7 * bw;
#pragma unroll
  for (int r = 0; r < 7; ++r) {
    const int Y = Yb + r;
    if (Y >= a.H) break;
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const int X = Xb + j;
      if (X < a.W) {
        float o = acc[r][j];
        if (has_bias) o += bias;
        long long idx;
        if (NHWC)
          idx = ((static_cast<long long>(n_img) * a.H + Y) * a.W + X) * a.C + c;
        else
          idx = plane * HW + static_cast<long long>(Y) * a.W + X;
        y[idx] = from_acc<T>(o);
      }
    }
  }
}

}  // namespace pla
