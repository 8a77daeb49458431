// Generic strided kernel: any dtype (fp64 included), any input strides.
//
// Covers what the fast kernels do not: non-contiguous or misaligned stencil
// inputs (the strided cases of data/stencil_direct_cuda_v7/test_stencil.py:31-37:
// sliced, transposed and batch-sliced tensors), fp64, and depthwise shapes
// whose rows break the vector-alignment rules, and depthwise filters of any
// odd size K <= 7 in any layout.  One thread per output point, the same tap
// order and rounding as the fast kernels.
#pragma once

#include "pla_common.cuh"

namespace pla {

struct GenericArgs {
  const void* x;
  const void* w;  // [C][K*K]
  const void* b;  // [C] or nullptr
  void* y;
  int N, C, H, W;
  long long xs_n, xs_c, xs_h, xs_w;  // input element strides
  long long ys_n, ys_c, ys_h, ys_w;  // output element strides
  long long total;                   // N*C*H*W
  int K;                             // filter side (odd, <= 7); padding K / 2
};

template <typename T>
__global__ void __launch_bounds__(256) generic_kernel(const GenericArgs a) {
  using Acc = typename AccOf<T>::type;
  const T* x = static_cast<const T*>(a.x);
  const T* w = static_cast<const T*>(a.w);
  const T* b = static_cast<const T*>(a.b);
  T* y = static_cast<T*>(a.y);
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < a.total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int X = static_cast<int>(i % a.W);
    long long q = i / a.W;
    const int Y = static_cast<int>(q % a.H);
    q /= a.H;
    const int c = static_cast<int>(q % a.C);
    const int n = static_cast<int>(q / a.C);
    const T* xp = x + n * a.xs_n + c * a.xs_c;
    const int K = a.K, half = a.K / 2;
    const T* wp = w + static_cast<long long>(c) * K * K;
    Acc acc = Acc(0);
    for (int ky = 0; ky < K; ++ky) {
      const int yy = Y + ky - half;
      if (yy < 0 || yy >= a.H) continue;
      for (int kx = 0; kx < K; ++kx) {
        const int xx = X + kx - half;
        if (xx < 0 || xx >= a.W) continue;
        acc = fma_rn(to_acc(xp[yy * a.xs_h + xx * a.xs_w]), to_acc(wp[ky * K + kx]), acc);
      }
    }
    if (b) acc += to_acc(b[c]);
    y[n * a.ys_n + c * a.ys_c + Y * a.ys_h + X * a.ys_w] = from_acc<T>(acc);
  }
}

}  // namespace pla
