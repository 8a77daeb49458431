/*
 * pla_oracle.c — CPU restatement of the reference's 7x7 depthwise / stencil
 * algorithm.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke check and
 * the CPU-baseline leg of bench.py use it as the checker; the product path
 * never calls it.
 *
 * The reference computes both ops with torch.nn.Conv2d (PyTorch 2.11.0, ATen;
 * a third-party dependency not vendored in the reference tree):
 *   - depthwise: data/depthwise_conv_7x7.py:15-29
 *       nn.Conv2d(C, C, 7, stride=1, padding=3, groups=C, bias)
 *   - stencil:   data/stencil_7x7.py:5-12
 *       nn.Conv2d(1, 1, 7, stride=1, padding=3)   (bias=True)
 * Published algorithm restated here (PyTorch Conv2d documentation:
 * cross-correlation, zero padding, groups=C means one filter per channel):
 *     y[n,c,i,j] = b[c] + sum_{ky,kx} w[c,0,ky,kx] * x[n,c,i+ky-3,j+kx-3],
 * with x == 0 outside [0,H) x [0,W).  The low-precision convention is the
 * reference tests' expected value F.conv2d(x.float(), w.float(),
 * b.float()).to(dtype) (data/stencil_direct_cuda_v7/test_stencil.py:49-54):
 * widen to fp32, accumulate in fp32, add the bias in fp32 (v7 kernel
 * data/stencil_direct_cuda_v7/stencil_cuda_kernel.cu:64-71), round once
 * (round-to-nearest-even).  fp64 data accumulates in fp64.
 *
 * Evaluation order is fixed: taps in row-major (ky, kx) order, each one a
 * correctly rounded fma() starting from +0, then "+ bias".  Taps on the zero
 * padding are skipped (they add an exact +-0).  The CUDA kernels evaluate in
 * the same order, so for identical inputs the two agree bit for bit (up to
 * the sign of an exactly-zero result); against PyTorch (whose order differs)
 * the agreement is within rounding, which tests/test_oracle.py pins against
 * golden vectors produced by the reference modules themselves.
 *
 * The k x k variants (k = 3, 5) restate the operator of the reference's
 * MetaSchedule benchmark, benchmark/MetaSchedule/depthwise_conv.py:32-33
 * (topi.nn.depthwise_conv2d_nchw, stride 1, padding k // 2, no bias), in the
 * same fixed order; its own numpy check (:41-46) sums the k*k products in fp32
 * in the same (ry, rx) order with separate multiply and add.
 *
 * Build: see oracle/Makefile (gcc -O2 -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define TAPS 49
#define HALO 3

/* ---- 16-bit float conversions (IEEE binary16 and bfloat16), RNE ---------- */
static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static inline float f16_to_f32(uint16_t h) {
  _Float16 v;
  memcpy(&v, &h, 2);
  return (float)v;
}

static inline uint16_t f32_to_f16(float f) {
  _Float16 v = (_Float16)f; /* IEEE conversion, round-to-nearest-even */
  uint16_t h;
  memcpy(&h, &v, 2);
  return h;
}

enum { ORACLE_F16 = 0, ORACLE_F32 = 1, ORACLE_F64 = 2, ORACLE_BF16 = 3 };
enum { ORACLE_NCHW = 0, ORACLE_NHWC = 1 };

static inline float load_f(const void* p, int64_t i, int dtype) {
  switch (dtype) {
    case ORACLE_F16: return f16_to_f32(((const uint16_t*)p)[i]);
    case ORACLE_BF16: return bf16_to_f32(((const uint16_t*)p)[i]);
    default: return ((const float*)p)[i];
  }
}

static inline void store_f(void* p, int64_t i, float v, int dtype) {
  switch (dtype) {
    case ORACLE_F16: ((uint16_t*)p)[i] = f32_to_f16(v); break;
    case ORACLE_BF16: ((uint16_t*)p)[i] = f32_to_bf16(v); break;
    default: ((float*)p)[i] = v; break;
  }
}

/*
 * One output point of one plane: plane element (r, c) lives at
 * x[base + r*sh + c*sw].  Rows [0,H), columns [0,W).
 */
static inline float point_f32(const void* x, int64_t base, int64_t sh, int64_t sw, int H, int W, const float* wt,
                              int K, int i, int j, int dtype) {
  float acc = 0.0f;
  const int half = K / 2;
  for (int ky = 0; ky < K; ++ky) {
    const int r = i + ky - half;
    if (r < 0 || r >= H) continue;
    for (int kx = 0; kx < K; ++kx) {
      const int c = j + kx - half;
      if (c < 0 || c >= W) continue;
      acc = fmaf(load_f(x, base + (int64_t)r * sh + (int64_t)c * sw, dtype), wt[ky * K + kx], acc);
    }
  }
  return acc;
}

/*
 * Depthwise 7x7 (stencil == the C == 1 case) on dense N x C x H x W data in
 * `layout`: output rows [row0, row1) of planes p in [p0, p1), p = n*C + c
 * (p0 = 0, p1 = N*C, row0 = 0, row1 = H for the whole tensor).  w: [C][49],
 * b: [C] or NULL, all of `dtype` (f16, f32, bf16).  Nothing else of y is
 * written, so disjoint ranges can run on separate threads (the Python
 * wrapper in oracle/oracle.py does that; ctypes drops the GIL per call).
 */
int oracle_depthwise(const void* x, const void* w, const void* b, void* y, int N, int C, int H, int W, int K,
                     int dtype, int layout, int64_t p0, int64_t p1, int row0, int row1) {
  if (dtype == ORACLE_F64) return -1;
  if (K < 1 || K > 7 || (K & 1) == 0) return -2;
  if (row0 < 0) row0 = 0;
  if (row1 > H) row1 = H;
  const int64_t plane = (int64_t)H * W;
  const int64_t planes = (int64_t)N * C;
  if (p0 < 0) p0 = 0;
  if (p1 > planes) p1 = planes;
  for (int64_t p = p0; p < p1; ++p) {
    const int n = (int)(p / C), ch = (int)(p % C);
    float wt[TAPS];
    for (int k = 0; k < K * K; ++k) wt[k] = load_f(w, (int64_t)ch * K * K + k, dtype);
    const float bias = b ? load_f(b, ch, dtype) : 0.0f;
    int64_t base, sh, sw;
    if (layout == ORACLE_NCHW) {
      base = p * plane;
      sh = W;
      sw = 1;
    } else {
      base = (int64_t)n * plane * C + ch;
      sh = (int64_t)W * C;
      sw = C;
    }
    for (int i = row0; i < row1; ++i)
      for (int j = 0; j < W; ++j) {
        float acc = point_f32(x, base, sh, sw, H, W, wt, K, i, j, dtype);
        if (b) acc = acc + bias;
        store_f(y, base + (int64_t)i * sh + (int64_t)j * sw, acc, dtype);
      }
  }
  return 0;
}

/* The 7x7 case (data/depthwise_conv_7x7.py, data/stencil_7x7.py). */
int oracle_depthwise7x7(const void* x, const void* w, const void* b, void* y, int N, int C, int H, int W,
                        int dtype, int layout, int64_t p0, int64_t p1, int row0, int row1) {
  return oracle_depthwise(x, w, b, y, N, C, H, W, 7, dtype, layout, p0, p1, row0, row1);
}

/* fp64 variant (fp64 accumulation), k x k, NCHW or NHWC. */
int oracle_depthwise_f64(const double* x, const double* w, const double* b, double* y, int N, int C, int H, int W,
                         int K, int layout) {
  if (K < 1 || K > 7 || (K & 1) == 0) return -2;
  const int half = K / 2;
  const int64_t plane = (int64_t)H * W;
  const int64_t planes = (int64_t)N * C;
  for (int64_t p = 0; p < planes; ++p) {
    const int n = (int)(p / C), ch = (int)(p % C);
    int64_t base, sh, sw;
    if (layout == ORACLE_NCHW) {
      base = p * plane;
      sh = W;
      sw = 1;
    } else {
      base = (int64_t)n * plane * C + ch;
      sh = (int64_t)W * C;
      sw = C;
    }
    for (int i = 0; i < H; ++i)
      for (int j = 0; j < W; ++j) {
        double acc = 0.0;
        for (int ky = 0; ky < K; ++ky) {
          const int r = i + ky - half;
          if (r < 0 || r >= H) continue;
          for (int kx = 0; kx < K; ++kx) {
            const int c = j + kx - half;
            if (c < 0 || c >= W) continue;
            acc = fma(x[base + r * sh + c * sw], w[(int64_t)ch * K * K + ky * K + kx], acc);
          }
        }
        if (b) acc = acc + b[ch];
        y[base + i * sh + j * sw] = acc;
      }
  }
  return 0;
}

int oracle_depthwise7x7_f64(const double* x, const double* w, const double* b, double* y, int N, int C, int H,
                            int W, int layout) {
  return oracle_depthwise_f64(x, w, b, y, N, C, H, W, 7, layout);
}

/*
 * Iterated stencil (no reference function: data/stencil_7x7.py:10-12 applied
 * `steps` times, zero padding every step == zero Dirichlet boundary).
 * fp32 data, one plane H x W; `work` is caller scratch of H*W floats; the
 * result lands in y (y may equal x).  b may be NULL.
 */
int oracle_stencil7x7_iterate_f32(const float* x, const float* w, const float* b, float* y, float* work, int H,
                                  int W, int steps) {
  const int64_t plane = (int64_t)H * W;
  if (steps == 0) {
    if (y != x) memcpy(y, x, (size_t)plane * sizeof(float));
    return 0;
  }
  memcpy(work, x, (size_t)plane * sizeof(float)); /* x may alias y */
  float* src = work;
  float* dst = y;
  for (int t = 0; t < steps; ++t) {
    oracle_depthwise7x7(src, w, b, dst, 1, 1, H, W, ORACLE_F32, ORACLE_NCHW, 0, 1, 0, H);
    float* tmp = src;
    src = dst;
    dst = tmp;
  }
  if (src != y) memcpy(y, src, (size_t)plane * sizeof(float));
  return 0;
}

/*
 * Depthwise 7x7 followed by LayerNorm over the channels of every pixel, on
 * channels_last (NHWC) data: the "dwconv -> norm" pair of a ConvNeXt block
 * (nn.Conv2d(C, C, 7, padding=3, groups=C) then nn.LayerNorm(C, eps) on the
 * channels-last view).  The reference has no counterpart; its depthwise
 * operator (data/depthwise_conv_7x7.py:15-29) is the first half, and the
 * LayerNorm restates torch.nn.LayerNorm's published definition
 * (biased variance, eps inside the square root).
 *
 * Images [n0, n1).  The depthwise output is exactly oracle_depthwise's (one
 * rounding to dtype); the normalisation then reads those rounded values v_c
 * (widened to fp32) and evaluates, per pixel, in this fixed order, with the
 * channels split into 32-channel groups g (n_g channels each; the last group
 * may be shorter) and every sum running in ascending order from +0:
 *   s_g  = sum of v_c over group g
 *   m_g  = s_g / n_g
 *   q_g  = sum over group g of d * d, d = v_c - m_g
 *   mean = (sum over g of s_g) / C
 *   M    = sum over g of (q_g + n_g * (e * e)), e = m_g - mean
 *          (the groups' squared deviations combined by Chan, Golub and
 *           LeVeque's pairwise-update formula)
 *   inv  = 1 / sqrt(M / C + eps)
 *   z_c  = ((v_c - mean) * inv) * gamma_c + beta_c   (gamma / beta skipped if NULL)
 * every operation a correctly rounded fp32 add / multiply / divide / square
 * root, then one rounding of z_c to dtype.  The CUDA epilogue evaluates the
 * same expression tree (a group is what one CTA reduces locally before the
 * CTAs of a cluster exchange their partial results).
 */
static void group_stats(const void* y, int64_t base, int g, int n, int dtype, float* s_out, float* q_out) {
  float s = 0.0f;
  for (int c = g; c < g + n; ++c) s = s + load_f(y, base + c, dtype);
  const float m = s / (float)n;
  float q = 0.0f;
  for (int c = g; c < g + n; ++c) {
    const float d = load_f(y, base + c, dtype) - m;
    q = q + d * d;
  }
  *s_out = s;
  *q_out = q;
}

int oracle_depthwise7x7_layernorm_nhwc(const void* x, const void* w, const void* b, const void* gamma,
                                       const void* beta, float eps, void* y, int N, int C, int H, int W,
                                       int dtype, int n0, int n1) {
  if (dtype == ORACLE_F64) return -1;
  if (n0 < 0) n0 = 0;
  if (n1 > N) n1 = N;
  if (n0 >= n1 || C <= 0) return 0;
  int rc = oracle_depthwise(x, w, b, y, N, C, H, W, 7, dtype, ORACLE_NHWC, (int64_t)n0 * C, (int64_t)n1 * C, 0, H);
  if (rc != 0) return rc;
  const float fc = (float)C;
  for (int64_t px = (int64_t)n0 * H * W; px < (int64_t)n1 * H * W; ++px) {
    const int64_t base = px * C;
    float s = 0.0f;
    for (int g = 0; g < C; g += 32) {
      float sg, qg;
      group_stats(y, base, g, C - g < 32 ? C - g : 32, dtype, &sg, &qg);
      s = s + sg;
    }
    const float mean = s / fc;
    float m = 0.0f;
    for (int g = 0; g < C; g += 32) {
      const int n = C - g < 32 ? C - g : 32;
      float sg, qg;
      group_stats(y, base, g, n, dtype, &sg, &qg);
      const float e = sg / (float)n - mean;
      m = m + (qg + (float)n * (e * e));
    }
    const float inv = 1.0f / sqrtf(m / fc + eps);
    for (int c = 0; c < C; ++c) {
      float t = (load_f(y, base + c, dtype) - mean) * inv;
      if (gamma) t = t * load_f(gamma, c, dtype);
      if (beta) t = t + load_f(beta, c, dtype);
      store_f(y, base + c, t, dtype);
    }
  }
  return 0;
}
