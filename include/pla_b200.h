/*
 * pla_b200.h — C ABI of the B200 (sm_100a) 7x7 depthwise-convolution and
 * 7x7 stencil library.
 *
 * Every entry point takes plain device pointers, element counts/strides and a
 * CUDA stream, launches asynchronously on that stream and returns a status
 * code (PLA_OK == 0).  Nothing here allocates device memory, synchronises the
 * stream or falls back to a CPU path: a non-zero status means no kernel ran.
 *
 * Numerical contract (shared by every kernel and by the CPU oracle that the
 * tests check against): each output point is
 *
 *     acc = 0;  for ky in 0..6: for kx in 0..6:
 *                   acc = fma(x[i+ky-3][j+kx-3], w[ky][kx], acc)
 *     y[i][j] = round_to_output_dtype(acc + bias)      (bias add skipped if null)
 *
 * with x == 0 outside the plane (zero padding 3, cross-correlation, output size
 * == input size), the accumulator in fp32 for fp32/bf16/fp16 data and fp64 for
 * fp64 data.  This is the semantics of torch.nn.Conv2d(C, C, 7, stride=1,
 * padding=3, groups=C) used by the reference modules, evaluated in one fixed
 * tap order so that results are bit-reproducible.
 */
#ifndef PLA_B200_H_
#define PLA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define PLA_API __attribute__((visibility("default")))
#else
#define PLA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque CUDA stream handle (binary-compatible with cudaStream_t). */
typedef struct CUstream_st* pla_stream_t;

/* Element type codes.  The values are the ones the reference stencil launcher
 * uses for its `type` argument (data/stencil_direct_cuda_v7/stencil_cuda.cpp:30:
 * 0=float16, 1=float32, 2=float64, 3=bfloat16). */
enum pla_dtype {
  PLA_F16 = 0,
  PLA_F32 = 1,
  PLA_F64 = 2,
  PLA_BF16 = 3
};

/* Memory layout of a depthwise activation tensor [N, C, H, W]. */
enum pla_layout {
  PLA_NCHW = 0, /* torch.contiguous_format */
  PLA_NHWC = 1  /* torch.channels_last */
};

/* Status codes. */
enum pla_status {
  PLA_OK = 0,
  PLA_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad enum   */
  PLA_ERR_UNSUPPORTED = 2,      /* dtype/layout/shape outside this library */
  PLA_ERR_TOO_LARGE = 3,        /* size exceeds grid/indexing limits       */
  PLA_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed       */
  PLA_ERR_NO_DEVICE = 5,        /* no sm_100 device current                */
  PLA_ERR_DEVICE_FAULT = 6      /* a kernel recorded a bounded-wait timeout */
};

/* Human-readable text for a status code (static storage, never NULL). */
PLA_API const char* pla_status_string(int status);

/* Detail text of the last failure seen by this thread inside the library
 * (CUDA error strings, size limits). */
PLA_API const char* pla_last_cuda_error(void);

/* Library ABI version: (major << 16) | minor.  1.1 added pla_depthwise_forward,
 * 1.2 pla_depthwise7x7_layernorm_nhwc, 1.3 pla_depthwise7x7_forward_many. */
PLA_API int pla_version(void);

/*
 * Single-step 7x7 stencil, one filter for all planes:
 *     y[n,0,:,:] = stencil(x[n,0,:,:]; w[0..48]) + b[0]
 *
 * Replaces the reference launchers
 *   launch_direct()  data/stencil_direct_cuda_v7/stencil_cuda_kernel.cu:230-244
 *   launch_stencil() data/stencil_cuda_v2/stencil_cuda_kernel.cu:195-209
 * with the argument meaning of launch_direct: x may be strided
 * (element strides sn, sh, sw; sn ignored when n == 1), y is contiguous
 * [n, h, width], w holds 49 taps row-major, b is NULL or one element, all of
 * dtype `dtype` (enum pla_dtype).  y must not overlap x (as with the
 * reference, whose extension allocates a fresh output): overlapping byte
 * spans return PLA_ERR_INVALID_ARGUMENT.  Unlike the reference it returns a
 * status.
 */
PLA_API int pla_stencil7x7_forward(const void* x, const void* w, const void* b, void* y,
                           int n, int h, int width,
                           int64_t sn, int64_t sh, int64_t sw,
                           int dtype, pla_stream_t stream);

/*
 * pla_stencil7x7_forward with the filter given by value: `taps` points to 49
 * fp32 taps in HOST memory (row-major), `bias` to one host fp32 value or is
 * NULL.  The taps travel in the kernel's parameter block, so the kernel reads
 * them as uniform constant operands instead of holding them in registers
 * (the fast path; same results bit for bit).  16-bit filters widen to fp32
 * exactly.  Only inputs that qualify for the TMA path are accepted (unit
 * column stride, 16-byte aligned rows); others return PLA_ERR_UNSUPPORTED
 * and should use pla_stencil7x7_forward.  Same reference counterpart as
 * pla_stencil7x7_forward.
 */
PLA_API int pla_stencil7x7_forward_taps(const void* x, const float* taps, const float* bias, void* y,
                                        int n, int h, int width,
                                        int64_t sn, int64_t sh, int64_t sw,
                                        int dtype, pla_stream_t stream);

/*
 * Depthwise 7x7 convolution (groups = C, stride 1, padding 3):
 *     y[n,c] = stencil(x[n,c]; w[c, 0..48]) + b[c]
 *
 * Replaces launch_depthwise_7x7_cutlass()
 *   data/depthwise_conv_7x7_cuda/model_cutlass_autotune_v6.py:428-458
 *   (and the v1/v5 launchers, model_cutlass.py:263-279,
 *    model_cutlass_autotune_v5.py:403-420).
 * Differences: w is the module's own [C,1,7,7] weight (no [C,8,80] repack),
 * b may be non-NULL ([C]), dtype may be f32/bf16/f16/f64 and layout NCHW or
 * NHWC.  x and y are dense in `layout` and must not overlap
 * (PLA_ERR_INVALID_ARGUMENT otherwise).
 */
PLA_API int pla_depthwise7x7_forward(const void* x, const void* w, const void* b, void* y,
                             int n, int c, int h, int width,
                             int dtype, int layout, pla_stream_t stream);

/*
 * Depthwise k x k convolution, k in {3, 5, 7} (groups = C, stride 1,
 * padding k / 2), w [C,1,k,k], same arguments otherwise.  k = 7 is
 * pla_depthwise7x7_forward.
 *
 * Replaces the operator of the reference's MetaSchedule benchmark
 *   benchmark/MetaSchedule/depthwise_conv.py:7-13 and :32-33
 *   (topi.nn.depthwise_conv2d_nchw(X, W, 1, k // 2, 1), kernel 3 or 7,
 *    NCHW, no bias, fp32/fp16/bf16),
 * whose numpy check (:41-46) accumulates the k*k products in fp32 in
 * row-major (ry, rx) order.  Here every output is one fp32 FMA chain in that
 * order plus the optional bias, rounded once; NHWC, bias and fp64 are also
 * accepted.  Other k: PLA_ERR_UNSUPPORTED.
 */
PLA_API int pla_depthwise_forward(const void* x, const void* w, const void* b, void* y,
                                  int n, int c, int h, int width, int k,
                                  int dtype, int layout, pla_stream_t stream);

/*
 * Several independent depthwise 7x7 problems in one call, for instance the
 * four stages of the ConvNeXt-T-shaped sweep (data/depthwise_conv_7x7.py's
 * benchmark shapes, one launcher call each in the reference,
 * model_cutlass_autotune_v6.py:428-458).  Problem i is
 * pla_depthwise7x7_forward(p[i].x, p[i].w, p[i].b, p[i].y, p[i].n, p[i].c,
 * p[i].h, p[i].width, dtype, layout): same arguments and results.
 *
 * The problems run concurrently: the call forks from `stream` onto up to 4
 * streams of the library (created once per device, on the first call made
 * with that device current), launches the problems round-robin and joins
 * back, so one problem's first tiles overlap another's last ones instead of
 * each launch paying its own ramp and drain.  Problems are launched smallest
 * first (by element count; ties in the given order): a large problem's
 * persistent grid occupies every SM, so a small one queued behind it would
 * start only in its drain.  Work queued on `stream` before
 * the call is finished before any problem starts; work queued after it
 * starts after every problem is done.  No problem's output may overlap any
 * problem's input or output (PLA_ERR_INVALID_ARGUMENT).  Arguments are
 * checked for every problem before anything is launched.
 *
 * The library streams are shared by every caller on the device: calls made
 * on different streams are ordered after one another on them (correct, but
 * not concurrent with each other), and a stream capture that contains a
 * call holds them in capture mode until the capture ends, so while it is
 * open no other thread may call this function on that device.
 */
typedef struct pla_dw_problem {
  const void* x;
  const void* w;
  const void* b; /* NULL: no bias */
  void* y;
  int n, c, h, width;
} pla_dw_problem;
PLA_API int pla_depthwise7x7_forward_many(const pla_dw_problem* problems, int count, int dtype, int layout,
                                          pla_stream_t stream);

/*
 * Depthwise 7x7 followed by LayerNorm over the channels of every pixel, in
 * one pass over HBM: the "dwconv -> norm" pair of a ConvNeXt block,
 *     v = depthwise7x7(x; w, b) rounded to dtype   (pla_depthwise7x7_forward)
 *     y[n,i,j,:] = (v[n,i,j,:] - mean) / sqrt(var + eps) * gamma + beta
 * with mean / biased variance over the C channels of the pixel.
 *
 * No reference counterpart: the reference's operator is the depthwise half
 * (data/depthwise_conv_7x7.py:15-29, whose CUDA launchers
 * pla_depthwise7x7_forward replaces); the LayerNorm is the next layer of the
 * ConvNeXt stages its benchmark shapes come from.
 *
 * x and y are channels_last (NHWC) [n, h, width, c], dense, of dtype f32 /
 * bf16 / f16, and must not overlap; w [c,1,7,7]; b, gamma, beta [c] of the
 * same dtype or NULL (no bias / scale 1 / shift 0); eps >= 0.  The
 * normalisation runs in fp32 on the rounded depthwise outputs in a fixed
 * order (sums per 32-channel group, then over the groups), one rounding of
 * y.  Supported: c * element size a multiple of 16 bytes and at most 16
 * channel groups per pixel (c <= 512; c <= 2048 for 7 x 7 planes, whose
 * groups hold 128 channels); other shapes return PLA_ERR_UNSUPPORTED.
 */
PLA_API int pla_depthwise7x7_layernorm_nhwc(const void* x, const void* w, const void* b,
                                            const void* gamma, const void* beta, float eps,
                                            void* y, int n, int c, int h, int width, int dtype,
                                            pla_stream_t stream);

/*
 * Iterated stencil on one device (no reference counterpart; the reference
 * path is data/stencil_7x7.py:10-12 applied `steps` times with zero padding
 * each step, i.e. a zero Dirichlet boundary):
 *     u_0 = x;  u_{t+1} = stencil(u_t; w) (+ b if non-NULL);  y = u_steps
 * fp32/bf16/f16 planes [h, width], contiguous.  `scratch` is a caller-owned
 * device buffer of at least h*width elements used as the second ping-pong
 * buffer; x is only read; y may be x itself.  A partial overlap of x and y,
 * or a scratch overlapping either, returns PLA_ERR_INVALID_ARGUMENT.
 */
PLA_API int pla_stencil7x7_iterate(const void* x, const void* w, const void* b, void* y,
                           void* scratch, int h, int width, int steps,
                           int dtype, pla_stream_t stream);

/*
 * pla_stencil7x7_iterate without a caller scratch buffer, for callers that
 * cannot allocate device memory: a plugin running inside a host framework
 * that owns every device allocation, a fixed-budget embedded runtime, or a
 * real-time loop that cannot afford cudaMalloc's implicit synchronisation.
 * This entry point has no counterpart in the reference.
 *
 * The second ping-pong plane is a 16 MiB static device array inside this
 * library (PLA_NOALLOC_SCRATCH_BYTES), held by every GPU that loads the
 * library until the process exits.  Grids larger than that (h * width *
 * element size > 16 MiB, e.g. more than 2048 x 2048 fp32) return
 * PLA_ERR_TOO_LARGE with the sizes in pla_last_cuda_error().  Nothing is
 * allocated: no cudaMalloc/cudaFree or allocating library call.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call
 * before any stream capture.  Only a successful lookup is kept: after a
 * failed one the next call tries again.  All calls on a device share the one array and
 * leave the last call's data in it (no call needs it cleared: every step
 * overwrites the whole plane before reading it), so calls that overlap on
 * the GPU (concurrent streams) race on it; serialise them.
 * Arguments and results are those of pla_stencil7x7_iterate.
 */
#define PLA_NOALLOC_SCRATCH_BYTES (16u << 20)
PLA_API int pla_stencil7x7_iterate_noalloc(const void* x, const void* w, const void* b, void* y,
                                           int h, int width, int steps,
                                           int dtype, pla_stream_t stream);

/* pla_stencil7x7_iterate with host taps (see pla_stencil7x7_forward_taps). */
PLA_API int pla_stencil7x7_iterate_taps(const void* x, const float* taps, const float* bias, void* y,
                                        void* scratch, int h, int width, int steps,
                                        int dtype, pla_stream_t stream);

/*
 * One Jacobi step of a row band of a larger grid (building block of the
 * row-band multi-GPU iterated stencil; no reference counterpart).
 * `in` and `out` are band buffers of (rows + 6) x width elements: rows 0..2
 * hold the 3 halo rows above the band, rows 3..rows+2 the band itself and
 * rows rows+3..rows+5 the halo rows below it.  The step writes output band
 * rows [row_begin, row_end) (0 <= row_begin <= row_end <= rows) into
 * out rows 3+row_begin .. 3+row_end-1; halo rows of `out` are not touched.
 * `in` and `out` must not overlap (PLA_ERR_INVALID_ARGUMENT).
 */
PLA_API int pla_stencil7x7_band_step(const void* in, const void* w, const void* b, void* out,
                             int rows, int width, int row_begin, int row_end,
                             int dtype, pla_stream_t stream);

/* pla_stencil7x7_band_step with host taps (see pla_stencil7x7_forward_taps). */
PLA_API int pla_stencil7x7_band_step_taps(const void* in, const float* taps, const float* bias, void* out,
                                          int rows, int width, int row_begin, int row_end,
                                          int dtype, pla_stream_t stream);

/*
 * One band step fused with the halo exchange over peer memory (NVLink), the
 * row-band multi-GPU iterated stencil without a separate collective (no
 * reference counterpart).  Band buffers as in pla_stencil7x7_band_step; the
 * step computes every band row (rows >= 64) with the host taps, and
 *  - before reading its halo, waits (bounded, ~2 s, then fault bit 1) until
 *    flags[0] >= step (neighbour above delivered) / flags[1] >= step (below);
 *  - stores its first 3 band rows into up_out rows up_rows+3..up_rows+5 and
 *    its last 3 into down_out rows 0..2 (the neighbours' `out` buffers, peer
 *    pointers from pla_ipc_import), then raises up_flags[1] / down_flags[0]
 *    (the neighbours' flags) to step+1.
 * up_out/down_out NULL = grid edge (zero halo kept).  flags[2] and counters[2]
 * are this GPU's zero-initialised words; steps must be launched 0, 1, 2, ...
 * on every rank.  Ranks are separate GPUs (never two on one device).
 */
PLA_API int pla_stencil7x7_band_step_halo(const void* in, const float* taps, const float* bias, void* out,
                                          int rows, int width, int dtype,
                                          void* up_out, int up_rows, void* down_out,
                                          unsigned int* flags, unsigned int* up_flags,
                                          unsigned int* down_flags, unsigned int* counters,
                                          unsigned int step, pla_stream_t stream);

/* CUDA IPC: export a device pointer as (64-byte handle of its allocation,
 * byte offset), import it in another process (peer access enabled lazily),
 * close an imported pointer. */
PLA_API int pla_ipc_export(const void* ptr, void* handle, uint64_t* offset);
PLA_API int pla_ipc_import(const void* handle, uint64_t offset, void** ptr);
PLA_API int pla_ipc_close(void* ptr, uint64_t offset);

/*
 * Device-side fault word of the current device: bit 0 = an mbarrier wait in a
 * kernel gave up after its time bound; bit 1 = a wait for a neighbouring
 * GPU's halo flag gave up.  Reading it synchronises the
 * device.  pla_clear_device_faults() zeroes it.
 */
PLA_API int pla_read_device_faults(unsigned int* faults);
PLA_API int pla_clear_device_faults(void);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* PLA_B200_H_ */
