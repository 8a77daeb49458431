/*
 * A C caller of the library: no Python, no torch.  Built by tests/test_c_abi.py
 * with gcc against include/pla_b200.h and pla_b200/libpla_b200.so.
 *
 *   abi_example cpu   status strings, version, argument checks (no device)
 *   abi_example gpu   cudaMalloc'd buffers, one stencil step and one 3x3
 *                     depthwise call on the current device, results checked
 *                     against scalar C loops
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "pla_b200.h"

/* The few CUDA runtime entry points used here (libcudart). */
typedef int cudaError_t;
extern cudaError_t cudaMalloc(void** p, size_t n);
extern cudaError_t cudaFree(void* p);
extern cudaError_t cudaMemcpy(void* dst, const void* src, size_t n, int kind);
extern cudaError_t cudaDeviceSynchronize(void);

static int check_cpu(void) {
  if (strcmp(pla_status_string(PLA_OK), "ok") != 0) return 1;
  if ((pla_version() >> 16) != 1) return 2;
  if (pla_stencil7x7_forward(NULL, NULL, NULL, NULL, 1, 1, 1, 1, 1, 1, 42, NULL) != PLA_ERR_UNSUPPORTED) return 3;
  if (pla_depthwise7x7_forward(NULL, NULL, NULL, NULL, -1, 1, 1, 1, PLA_F32, PLA_NCHW, NULL) !=
      PLA_ERR_INVALID_ARGUMENT)
    return 4;
  if (pla_stencil7x7_forward(NULL, NULL, NULL, NULL, 0, 8, 8, 64, 8, 1, PLA_F32, NULL) != PLA_OK) return 5;
  if ((pla_version() & 0xffff) < 1) return 6; /* 1.1: pla_depthwise_forward */
  if (pla_depthwise_forward(NULL, NULL, NULL, NULL, 1, 1, 8, 8, 4, PLA_F32, PLA_NCHW, NULL) != PLA_ERR_UNSUPPORTED)
    return 7;
  printf("cpu ok\n");
  return 0;
}

static int check_gpu(void) {
  const int H = 37, W = 96;
  const size_t n = (size_t)H * W;
  float* hx = (float*)malloc(n * sizeof(float));
  float* hy = (float*)malloc(n * sizeof(float));
  float hw[49], hb = 0.125f;
  for (size_t i = 0; i < n; ++i) hx[i] = (float)((i * 7919u) % 1000u) / 1000.0f - 0.5f;
  for (int k = 0; k < 49; ++k) hw[k] = (float)(k % 7 - 3) / 49.0f + (float)(k / 7) / 100.0f;
  void *dx, *dy, *dw, *db;
  if (cudaMalloc(&dx, n * 4) || cudaMalloc(&dy, n * 4) || cudaMalloc(&dw, 49 * 4) || cudaMalloc(&db, 4)) return 10;
  cudaMemcpy(dx, hx, n * 4, 1);
  cudaMemcpy(dw, hw, 49 * 4, 1);
  cudaMemcpy(db, &hb, 4, 1);
  int st = pla_stencil7x7_forward(dx, dw, db, dy, 1, H, W, (int64_t)n, W, 1, PLA_F32, NULL);
  if (st != PLA_OK) {
    fprintf(stderr, "pla_stencil7x7_forward: %s %s\n", pla_status_string(st), pla_last_cuda_error());
    return 11;
  }
  cudaDeviceSynchronize();
  cudaMemcpy(hy, dy, n * 4, 2);
  /* same arithmetic as the library's contract: row-major taps, fmaf, then + bias */
  for (int i = 0; i < H; ++i)
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int ky = 0; ky < 7; ++ky)
        for (int kx = 0; kx < 7; ++kx) {
          const int r = i + ky - 3, c = j + kx - 3;
          if (r < 0 || r >= H || c < 0 || c >= W) continue;
          acc = fmaf(hx[r * W + c], hw[ky * 7 + kx], acc);
        }
      acc = acc + hb;
      if (acc != hy[i * W + j]) {
        fprintf(stderr, "mismatch at %d,%d: %.9g vs %.9g\n", i, j, acc, hy[i * W + j]);
        return 12;
      }
    }
  /* 3x3 depthwise, one channel, no bias: the first 9 taps as the filter */
  st = pla_depthwise_forward(dx, dw, NULL, dy, 1, 1, H, W, 3, PLA_F32, PLA_NCHW, NULL);
  if (st != PLA_OK) {
    fprintf(stderr, "pla_depthwise_forward: %s %s\n", pla_status_string(st), pla_last_cuda_error());
    return 13;
  }
  cudaDeviceSynchronize();
  cudaMemcpy(hy, dy, n * 4, 2);
  for (int i = 0; i < H; ++i)
    for (int j = 0; j < W; ++j) {
      float acc = 0.0f;
      for (int ky = 0; ky < 3; ++ky)
        for (int kx = 0; kx < 3; ++kx) {
          const int r = i + ky - 1, c = j + kx - 1;
          if (r < 0 || r >= H || c < 0 || c >= W) continue;
          acc = fmaf(hx[r * W + c], hw[ky * 3 + kx], acc);
        }
      if (acc != hy[i * W + j]) {
        fprintf(stderr, "3x3 mismatch at %d,%d: %.9g vs %.9g\n", i, j, acc, hy[i * W + j]);
        return 14;
      }
    }
  cudaFree(dx);
  cudaFree(dy);
  cudaFree(dw);
  cudaFree(db);
  free(hx);
  free(hy);
  printf("gpu ok\n");
  return 0;
}

int main(int argc, char** argv) {
  if (argc > 1 && strcmp(argv[1], "gpu") == 0) return check_gpu();
  return check_cpu();
}
