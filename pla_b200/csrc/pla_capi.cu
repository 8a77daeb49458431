// C ABI of the library (declarations and contract: include/pla_b200.h).
//
// Host-side dispatch: validates arguments, picks the kernel family, builds the
// TMA tensor map and launches on the caller's stream.  No allocation, no
// synchronisation, no CPU fallback.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/pla_b200.h"
#include "cm_kernel.cuh"
#include "generic_kernel.cuh"
#include "nhwc_tile_kernel.cuh"
#include "pair_kernel.cuh"
#include "pla_common.cuh"
#include "stack_kernel.cuh"
#include "tile_kernel.cuh"

namespace pla {
namespace {

thread_local char g_last_cuda_error[256] = "";

int cuda_fail(cudaError_t e, const char* where) {
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", where, cudaGetErrorString(e));
  // Reset the runtime's last-error slot (a no-op for sticky errors), so the
  // launch check of a later, unrelated call does not report this failure.
  (void)cudaGetLastError();
  return PLA_ERR_CUDA;
}

#define PLA_CUDA(call)                              \
  do {                                              \
    cudaError_t e_ = (call);                        \
    if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
  } while (0)

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag once;
  int status = PLA_OK;
  int sms = 0;
  int cc_major = 0;
  size_t smem_optin = 0;
};
DeviceInfo g_dev[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return PLA_ERR_NO_DEVICE;
  return PLA_OK;
}

DeviceInfo* device_info(int* status) {
  int dev;
  *status = current_device(&dev);
  if (*status != PLA_OK) return nullptr;
  DeviceInfo& d = g_dev[dev];
  std::call_once(d.once, [&]() {
    cudaDeviceProp p;
    cudaError_t e = cudaGetDeviceProperties(&p, dev);
    if (e != cudaSuccess) {
      d.status = cuda_fail(e, "cudaGetDeviceProperties");
      return;
    }
    d.sms = p.multiProcessorCount;
    d.cc_major = p.major;
    d.smem_optin = p.sharedMemPerBlockOptin;
    if (p.major != 10) d.status = PLA_ERR_NO_DEVICE;
  });
  *status = d.status;
  return d.status == PLA_OK ? &d : nullptr;
}

int encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::call_once(g_encode_once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  *fn = g_encode;
  if (!g_encode) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled unavailable");
    return PLA_ERR_CUDA;
  }
  return PLA_OK;
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case PLA_F16: return 2;
    case PLA_BF16: return 2;
    case PLA_F32: return 4;
    case PLA_F64: return 8;
    default: return 0;
  }
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Byte span [lo, hi) touched by a tensor view; overlap tests between spans.
struct Span {
  uintptr_t lo, hi;
};
Span dense_span(const void* p, long long elems, size_t es) {
  const uintptr_t b = reinterpret_cast<uintptr_t>(p);
  return {b, b + static_cast<uintptr_t>(elems) * es};
}
// (extent, element stride) per dimension; strides may be negative.
Span strided_span(const void* p, size_t es, int nd, const long long* ext, const long long* str) {
  long long lo = 0, hi = 0;
  for (int i = 0; i < nd; ++i) {
    if (ext[i] <= 0) return {0, 0};
    const long long d = (ext[i] - 1) * str[i] * static_cast<long long>(es);
    if (d < 0) lo += d; else hi += d;
  }
  const uintptr_t b = reinterpret_cast<uintptr_t>(p);
  return {b + static_cast<uintptr_t>(lo), b + static_cast<uintptr_t>(hi) + es};
}
bool overlap(Span a, Span b) { return a.lo < b.hi && b.lo < a.hi; }

// Launch with programmatic dependent launch allowed: the kernel may start
// (CTA launch, barrier init, tensor-map prefetch) while the previous kernel
// in the stream drains; it waits for that kernel's completion and memory
// flush (griddepcontrol.wait) before touching global memory.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), int grid, int threads, uint32_t smem, cudaStream_t stream,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Tile-kernel launch: static-striding launches (persistent CTAs, at most a
// few tiles each) with programmatic dependent launch, which measured 6.5 %
// faster on back-to-back 4096^2 steps; tile-claiming launches (one CTA per
// tile) without it: on a 32768^2 band step it measured 10 % slower.
template <typename... KArgs, typename... Args>
cudaError_t launch_tile_kernel(void (*kernel)(KArgs...), bool pdl, int grid, uint32_t smem, cudaStream_t stream,
                               Args&&... args) {
  if (pdl) return launch_pdl(kernel, grid, kTileThreads, smem, stream, std::forward<Args>(args)...);
  kernel<<<grid, kTileThreads, smem, stream>>>(std::forward<Args>(args)...);
  return cudaGetLastError();
}

// Per-(kernel, device) one-time attribute setup (dynamic smem opt-in) and
// the resident-CTA count used to size persistent grids.
template <auto Kernel>
int kernel_setup(int threads, uint32_t smem, int* blocks_per_sm) {
  int dev;
  int st = current_device(&dev);
  if (st != PLA_OK) return st;
  static std::mutex mu;
  static std::atomic<int> cached[kMaxDevices] = {};
  int v = cached[dev].load(std::memory_order_acquire);
  if (v == 0) {
    std::lock_guard<std::mutex> lock(mu);
    v = cached[dev].load(std::memory_order_relaxed);
    if (v == 0) {
      PLA_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      int nb = 0;
      PLA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, Kernel, threads, smem));
      v = nb > 0 ? nb : 1;
      cached[dev].store(v, std::memory_order_release);
    }
  }
  *blocks_per_sm = v;
  return PLA_OK;
}

CUtensorMapDataType tmap_dtype(int dtype) {
  switch (dtype) {
    case PLA_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    case PLA_BF16: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

// Stack of `planes` planes of `rows` x `width` elements; strides in elements.
// The box is G::PITCH x G::ROWS x box_planes.
template <typename T, typename G>
int make_tile_map(CUtensorMap* map, const void* x, int dtype, int width, int rows, int planes,
                  long long row_stride, long long plane_stride, int box_planes = 1) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int st = encoder(&enc);
  if (st != PLA_OK) return st;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(planes)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride) * sizeof(T),
                                 static_cast<cuuint64_t>(plane_stride) * sizeof(T)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(G::PITCH), static_cast<cuuint32_t>(G::ROWS),
                             static_cast<cuuint32_t>(box_planes)};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, tmap_dtype(dtype), 3, const_cast<void*>(x), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled failed (%d)",
                  static_cast<int>(r));
    return PLA_ERR_CUDA;
  }
  return PLA_OK;
}

// Tile shapes: wide planes (stencil grids, big depthwise planes) and
// 33..64-wide planes (one 56 x 64 tile per ConvNeXt stage-1 plane).
constexpr int kWideR = 8, kWideLX = 32;
constexpr int kNarrowR = 7, kNarrowLX = 16;
// Short narrow tiles (16 x 64) for stacks too small to give every SM a
// 56-row tile.
constexpr int kShortR = 2;

// Can the plane-tile kernel read this stack with TMA?
bool tile_path_ok(const void* x, const void* y, int dtype, int width, long long row_stride,
                  long long plane_stride, int planes) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return false;
  const size_t es = dtype_size(dtype);
  if (!aligned(x, 16) || !aligned(y, 16)) return false;
  if (width % 4 != 0) return false;                        // 4-wide vector stores
  if ((row_stride * es) % 16 != 0) return false;           // TMA stride rule
  if (planes > 1 && (plane_stride * es) % 16 != 0) return false;
  if (row_stride * es >= (1ll << 40) || plane_stride * es >= (1ll << 40)) return false;
  return true;
}

template <typename T, int R, int LX, int K = 7>
int launch_tile(const void* x, const void* w, const void* b, const HostTaps* ht, void* y, int dtype, int planes,
                int C, int in_rows, int width, long long x_row_stride, long long x_plane_stride, int row_begin,
                int row_end, int in_row_shift, long long y_plane_stride, long long y_row_stride,
                cudaStream_t stream) {
  using G = TileGeom<T, R, LX, K>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  if (row_end <= row_begin || planes == 0 || width == 0) return PLA_OK;
  if (K != 7 && ht) return PLA_ERR_UNSUPPORTED;  // host taps hold a 7x7 filter
  CUtensorMap map;
  st = make_tile_map<T, G>(&map, x, dtype, width, in_rows, planes, x_row_stride, x_plane_stride);
  if (st != PLA_OK) return st;
  int per_sm = 1;
  if constexpr (K == 7) {
    st = ht ? kernel_setup<tile_kernel<T, R, LX, true>>(kTileThreads, G::SMEM, &per_sm)
            : kernel_setup<tile_kernel<T, R, LX, false>>(kTileThreads, G::SMEM, &per_sm);
  } else {
    st = kernel_setup<tile_kernel<T, R, LX, false, false, K>>(kTileThreads, G::SMEM, &per_sm);
  }
  if (st != PLA_OK) return st;
  TileArgs a;
  a.w = w;
  a.b = b;
  a.y = y;
  a.planes = planes;
  a.C = C;
  a.W = width;
  a.row_begin = row_begin;
  a.row_end = row_end;
  a.in_row_shift = in_row_shift;
  a.tiles_x = (width + G::TW - 1) / G::TW;
  a.tiles_y = (row_end - row_begin + G::TH - 1) / G::TH;
  const long long total = static_cast<long long>(planes) * a.tiles_x * a.tiles_y;
  if (total > 0x7fffffffll) return PLA_ERR_TOO_LARGE;
  a.total_tiles = static_cast<int>(total);
  a.div_tx = make_fastdiv(a.tiles_x);
  a.div_ty = make_fastdiv(a.tiles_y);
  a.div_c = make_fastdiv(C);
  a.y_plane_stride = y_plane_stride;
  a.y_row_stride = y_row_stride;
  const long long slots = static_cast<long long>(d->sms) * per_sm;
  // Long tile lists: one CTA per tile with launch-control claiming (see tile_kernel.cuh).
  a.dyn = total >= 8 * slots ? 1 : 0;
  const int grid = static_cast<int>(a.dyn ? total : (total < slots ? total : slots));
  const HaloLinks no_halo{};
  if constexpr (K == 7) {
    if (ht) {
      PLA_CUDA(launch_tile_kernel(tile_kernel<T, R, LX, true>, !a.dyn, grid, G::SMEM, stream, map, a, *ht, no_halo));
    } else {
      HostTaps unused{};
      PLA_CUDA(launch_tile_kernel(tile_kernel<T, R, LX, false>, !a.dyn, grid, G::SMEM, stream, map, a, unused,
                                  no_halo));
    }
  } else {
    HostTaps unused{};
    PLA_CUDA(launch_tile_kernel(tile_kernel<T, R, LX, false, false, K>, !a.dyn, grid, G::SMEM, stream, map, a,
                                unused, no_halo));
  }
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

template <typename T, int K = 7>
int launch_tile_shape(int shape, const void* x, const void* w, const void* b, const HostTaps* ht, void* y,
                      int dtype, int planes, int C, int in_rows, int width, long long x_row_stride,
                      long long x_plane_stride, int row_begin, int row_end, int in_row_shift,
                      long long y_plane_stride, long long y_row_stride, cudaStream_t stream) {
  if (shape == 1)
    return launch_tile<T, kNarrowR, kNarrowLX, K>(x, w, b, ht, y, dtype, planes, C, in_rows, width, x_row_stride,
                                               x_plane_stride, row_begin, row_end, in_row_shift, y_plane_stride,
                                               y_row_stride, stream);
  if (shape == 2)
    return launch_tile<T, kShortR, kNarrowLX, K>(x, w, b, ht, y, dtype, planes, C, in_rows, width, x_row_stride,
                                              x_plane_stride, row_begin, row_end, in_row_shift, y_plane_stride,
                                              y_row_stride, stream);
  return launch_tile<T, kWideR, kWideLX, K>(x, w, b, ht, y, dtype, planes, C, in_rows, width, x_row_stride,
                                         x_plane_stride, row_begin, row_end, in_row_shift, y_plane_stride,
                                         y_row_stride, stream);
}

// Narrow tiles only pay off for 33..64-wide planes tall enough to fill them.
bool use_narrow_tiles(int width, int rows) { return width > 32 && width <= 64 && rows > 28; }

template <int K = 7>
int launch_tile_dtype(int dtype, const void* x, const void* w, const void* b, const HostTaps* ht, void* y,
                      int planes, int C, int in_rows, int width, long long x_row_stride, long long x_plane_stride,
                      int row_begin, int row_end, int in_row_shift, long long y_plane_stride,
                      long long y_row_stride, cudaStream_t stream) {
  // 0: 32 x 128 tiles; 1: 56 x 64 tiles; 2: 16 x 64 tiles when 56-row tiles
  // would leave SMs idle.
  int narrow = use_narrow_tiles(width, row_end - row_begin) ? 1 : 0;
  if (narrow) {
    int st;
    DeviceInfo* d = device_info(&st);
    if (!d) return st;
    const long long tall = static_cast<long long>(planes) * ((row_end - row_begin + 55) / 56);
    if (tall < 2ll * d->sms) narrow = 2;
  }
  switch (dtype) {
    case PLA_F32:
      return launch_tile_shape<float, K>(narrow, x, w, b, ht, y, dtype, planes, C, in_rows, width, x_row_stride,
                                      x_plane_stride, row_begin, row_end, in_row_shift, y_plane_stride,
                                      y_row_stride, stream);
    case PLA_BF16:
      return launch_tile_shape<__nv_bfloat16, K>(narrow, x, w, b, ht, y, dtype, planes, C, in_rows, width,
                                              x_row_stride, x_plane_stride, row_begin, row_end, in_row_shift,
                                              y_plane_stride, y_row_stride, stream);
    case PLA_F16:
      return launch_tile_shape<__half, K>(narrow, x, w, b, ht, y, dtype, planes, C, in_rows, width, x_row_stride,
                                       x_plane_stride, row_begin, row_end, in_row_shift, y_plane_stride,
                                       y_row_stride, stream);
    default:
      return PLA_ERR_UNSUPPORTED;
  }
}

// One fused band step with the halo exchange over peer memory (wide tiles,
// host taps, one plane).  `links` carries the peer pointers and flags.
// NCHW stacks of 56 x 56 16-bit planes (pair_kernel.cuh).  Below a few
// stages per SM the plane-tile kernel's shorter tiles fill the GPU better.
bool pair_path_ok(const void* x, const void* y, int dtype, long long n, long long c, int h, int w, int sms) {
  if (dtype != PLA_BF16 && dtype != PLA_F16) return false;
  if (h != 56 || w != 56) return false;
  if (!aligned(x, 16) || !aligned(y, 16)) return false;
  const long long planes = n * c;
  return planes <= 0x7fffffffll && planes >= 8ll * sms;
}

template <typename T>
int launch_pair(const void* x, const void* w, const void* b, void* y, int dtype, int n, int c,
                cudaStream_t stream) {
  using G = PairGeom<T>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  PairArgs a;
  a.w = w; a.b = b; a.y = y;
  a.N = n; a.C = c;
  a.planes = n * c;  // < 2^31 (pair_path_ok)
  a.stages = (a.planes + 1) / 2;
  a.cp_major = (c % 2 == 0) ? 1 : 0;
  a.div_n = make_fastdiv(n);
  a.div_c = make_fastdiv(c);
  constexpr long long kPlane = static_cast<long long>(G::S) * G::S;
  CUtensorMap map;
  st = make_tile_map<T, G>(&map, x, dtype, G::S, G::S, a.planes, G::S, kPlane, G::PL);
  if (st != PLA_OK) return st;
  int per_sm = 1;
  st = kernel_setup<pair_kernel<T>>(G::THREADS, G::SMEM, &per_sm);
  if (st != PLA_OK) return st;
  const long long slots = static_cast<long long>(d->sms) * per_sm;
  const int grid = static_cast<int>(a.stages < slots ? a.stages : slots);
  PLA_CUDA(launch_pdl(pair_kernel<T>, grid, G::THREADS, G::SMEM, stream, map, a));
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

template <typename T>
int launch_tile_halo(const void* in, const HostTaps& ht, void* out_rows, int dtype, int rows, int width,
                     HaloLinks links, cudaStream_t stream) {
  using G = TileGeom<T, kWideR, kWideLX>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  if (rows < 2 * G::TH) return PLA_ERR_UNSUPPORTED;  // edge tile rows must not overlap
  CUtensorMap map;
  const long long band = static_cast<long long>(rows + 6) * width;
  st = make_tile_map<T, G>(&map, in, dtype, width, rows + 6, 1, width, band);
  if (st != PLA_OK) return st;
  int per_sm = 1;
  st = kernel_setup<tile_kernel<T, kWideR, kWideLX, true, true>>(kTileThreads, G::SMEM, &per_sm);
  if (st != PLA_OK) return st;
  TileArgs a;
  a.dyn = 0;
  a.w = nullptr;
  a.b = nullptr;
  a.y = out_rows;
  a.planes = 1;
  a.C = 1;
  a.W = width;
  a.row_begin = 0;
  a.row_end = rows;
  a.in_row_shift = 3;
  a.tiles_x = (width + G::TW - 1) / G::TW;
  a.tiles_y = (rows + G::TH - 1) / G::TH;
  const long long total = static_cast<long long>(a.tiles_x) * a.tiles_y;
  if (total > 0x7fffffffll) return PLA_ERR_TOO_LARGE;
  a.total_tiles = static_cast<int>(total);
  a.div_tx = make_fastdiv(a.tiles_x);
  a.div_ty = make_fastdiv(a.tiles_y);
  a.div_c = make_fastdiv(1);
  a.y_plane_stride = band;
  a.y_row_stride = width;
  links.rows = rows;
  links.bot0 = (rows - 3) / G::TH;
  links.n_top = a.tiles_x;
  links.n_bot = a.tiles_x * (a.tiles_y - links.bot0);
  const long long slots = static_cast<long long>(d->sms) * per_sm;
  // Static striding: tile claiming measured 0.6 % slower for the fused
  // halo step (2 GPUs, same box), unlike the plain band step.
  const int grid = static_cast<int>(total < slots ? total : slots);
  PLA_CUDA(launch_pdl(tile_kernel<T, kWideR, kWideLX, true, true>, grid, kTileThreads, G::SMEM, stream, map, a, ht,
                      links));
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

// ---- CUDA IPC for peer buffers ----------------------------------------------
typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);
PfnMemGetAddressRange g_get_range = nullptr;
std::once_flag g_get_range_once;

int alloc_base(const void* ptr, void** base) {
  std::call_once(g_get_range_once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_get_range = reinterpret_cast<PfnMemGetAddressRange>(p);
  });
  if (!g_get_range) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuMemGetAddressRange unavailable");
    return PLA_ERR_CUDA;
  }
  CUdeviceptr b = 0;
  size_t size = 0;
  CUresult r = g_get_range(&b, &size, reinterpret_cast<CUdeviceptr>(ptr));
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuMemGetAddressRange failed (%d)",
                  static_cast<int>(r));
    return PLA_ERR_CUDA;
  }
  *base = reinterpret_cast<void*>(b);
  return PLA_OK;
}

// Host taps (fp32) -> kernel-parameter filter.
HostTaps make_host_taps(const float* taps, const float* bias) {
  HostTaps h;
  for (int k = 0; k < kTaps; ++k) h.w[k] = taps[k];
  h.b = bias ? *bias : 0.f;
  h.has_b = bias != nullptr;
  return h;
}

template <typename T>
int launch_generic(const GenericArgs& a, cudaStream_t stream) {
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  if (a.total == 0) return PLA_OK;
  long long blocks = (a.total + 255) / 256;
  const long long cap = static_cast<long long>(d->sms) * 16;
  if (blocks > cap) blocks = cap;
  generic_kernel<T><<<static_cast<int>(blocks), 256, 0, stream>>>(a);
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

int launch_generic_dtype(int dtype, const GenericArgs& a, cudaStream_t stream) {
  switch (dtype) {
    case PLA_F32: return launch_generic<float>(a, stream);
    case PLA_BF16: return launch_generic<__nv_bfloat16>(a, stream);
    case PLA_F16: return launch_generic<__half>(a, stream);
    case PLA_F64: return launch_generic<double>(a, stream);
    default: return PLA_ERR_UNSUPPORTED;
  }
}

template <typename T, bool NHWC, int BT>
int launch_cm(const CmArgs& in, cudaStream_t stream) {
  using G = CmGeom<BT>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  int per_sm;
  st = kernel_setup<cm_kernel<T, NHWC, BT>>(G::THREADS, G::SMEM, &per_sm);
  if (st != PLA_OK) return st;
  CmArgs a = in;
  a.tiles_x = (a.W + G::TS - 1) / G::TS;
  a.tiles_y = (a.H + G::TS - 1) / G::TS;
  a.cgroups = (a.C + 31) / 32;
  const long long NC = static_cast<long long>(a.N) * a.C;
  a.groups = NHWC ? static_cast<long long>(a.N) * a.cgroups : (NC + 31) / 32;
  const long long blocks = a.groups * a.tiles_x * a.tiles_y;
  if (blocks == 0) return PLA_OK;
  if (blocks > 0x7fffffffll) return PLA_ERR_TOO_LARGE;
  cm_kernel<T, NHWC, BT><<<static_cast<int>(blocks), G::THREADS, G::SMEM, stream>>>(a);
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

template <typename T, bool NHWC>
int launch_cm_bt(const CmArgs& a, cudaStream_t stream) {
  if (a.H <= 7 && a.W <= 7) return launch_cm<T, NHWC, 1>(a, stream);
  return launch_cm<T, NHWC, 2>(a, stream);
}

int launch_cm_dtype(int dtype, bool nhwc, const CmArgs& a, cudaStream_t stream) {
  switch (dtype) {
    case PLA_F32: return nhwc ? launch_cm_bt<float, true>(a, stream) : launch_cm_bt<float, false>(a, stream);
    case PLA_BF16:
      return nhwc ? launch_cm_bt<__nv_bfloat16, true>(a, stream) : launch_cm_bt<__nv_bfloat16, false>(a, stream);
    case PLA_F16: return nhwc ? launch_cm_bt<__half, true>(a, stream) : launch_cm_bt<__half, false>(a, stream);
    default: return PLA_ERR_UNSUPPORTED;
  }
}

// ---- plane-stack kernel (small square planes, NCHW or NHWC) ----------------
template <typename T>
int make_nhwc_map(CUtensorMap* map, const void* base, int dtype, int n, int c, int h, int w, int lanes, int s) {
  PFN_cuTensorMapEncodeTiled_v12000 enc;
  int st = encoder(&enc);
  if (st != PLA_OK) return st;
  const cuuint64_t es = sizeof(T);
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(c), static_cast<cuuint64_t>(w), static_cast<cuuint64_t>(h),
                              static_cast<cuuint64_t>(n)};
  const cuuint64_t strides[3] = {c * es, static_cast<cuuint64_t>(w) * c * es,
                                 static_cast<cuuint64_t>(h) * w * c * es};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(lanes), static_cast<cuuint32_t>(s),
                             static_cast<cuuint32_t>(s), 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, tmap_dtype(dtype), 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "cuTensorMapEncodeTiled (4d) failed (%d)",
                  static_cast<int>(r));
    return PLA_ERR_CUDA;
  }
  return PLA_OK;
}

template <typename T, bool NHWC, int S>
int launch_stack(const void* x, const void* w, const void* b, void* y, int dtype, int n, int c,
                 cudaStream_t stream) {
  using G = StackGeom<S, kMixStack<T>>;
  using M = StackSmem<T, S>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  StackArgs a;
  a.x = x; a.w = w; a.b = b; a.y = y;
  a.N = n; a.C = c;
  a.planes = static_cast<long long>(n) * c;
  CUtensorMap xmap, ymap;
  std::memset(&xmap, 0, sizeof(xmap));
  std::memset(&ymap, 0, sizeof(ymap));
  long long stages;
  if (NHWC) {
    a.cgroups = (c + G::LANES - 1) / G::LANES;
    stages = static_cast<long long>(n) * a.cgroups;
    a.full_stages = 0;
    st = make_nhwc_map<T>(&xmap, x, dtype, n, c, S, S, G::LANES, S);
    if (st != PLA_OK) return st;
    st = make_nhwc_map<T>(&ymap, y, dtype, n, c, S, S, G::LANES, S);
    if (st != PLA_OK) return st;
  } else {
    a.cgroups = 1;
    stages = (a.planes + G::LANES - 1) / G::LANES;
    a.full_stages = static_cast<int>(a.planes / G::LANES);
  }
  if (stages == 0) return PLA_OK;
  a.stages = static_cast<int>(stages);
  if (NHWC) {
    a.cg_major = 1;
  } else {
    // NCHW stages hold whole channel groups only when LANES divides C.
    a.cg_major = (c % G::LANES == 0) ? 1 : 0;
    if (a.cg_major) a.cgroups = c / G::LANES;
  }
  a.div_c = make_fastdiv(c);
  a.div_cg = make_fastdiv(a.cgroups);
  a.div_n = make_fastdiv(n);
  int per_sm;
  st = kernel_setup<stack_kernel<T, NHWC, S>>(G::THREADS, M::TOTAL, &per_sm);
  if (st != PLA_OK) return st;
  const long long slots = static_cast<long long>(d->sms) * per_sm;
  const int grid = static_cast<int>(stages < slots ? stages : slots);
  PLA_CUDA(launch_pdl(stack_kernel<T, NHWC, S>, grid, G::THREADS, M::TOTAL, stream, xmap, ymap, a));
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

// Square planes of side 7, 14 or 28 (and, for NHWC, channel rows that are
// 16-byte multiples so the 4-D TMA map is legal).
// NHWC planes the stack kernel does not take: 14 x 14 spatial tiles x 32
// channels (nhwc_tile_kernel.cuh).  TMA needs 16-byte aligned bases and a
// channel stride (C * element size) that is a multiple of 16 bytes.
bool nhwc_tile_ok(const void* x, const void* y, int dtype, long long n, long long c, int h, int w) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return false;
  if (!aligned(x, 16) || !aligned(y, 16)) return false;
  if ((c * static_cast<long long>(dtype_size(dtype))) % 16 != 0) return false;
  const long long tiles = static_cast<long long>((h + 13) / 14) * ((w + 13) / 14);
  return n * tiles * ((c + 31) / 32) < 0x7fffffffll;
}

template <typename T>
int launch_nhwc_tile(const void* x, const void* w, const void* b, void* y, int dtype, int n, int c, int h,
                     int width, cudaStream_t stream) {
  using G = NhwcTileGeom;
  using M = NhwcTileSmem<T>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  CUtensorMap xmap, ymap;
  st = make_nhwc_map<T>(&xmap, x, dtype, n, c, h, width, G::LANES, G::SW);
  if (st != PLA_OK) return st;
  st = make_nhwc_map<T>(&ymap, y, dtype, n, c, h, width, G::LANES, G::TS);
  if (st != PLA_OK) return st;
  NhwcTileArgs a;
  a.w = w;
  a.b = b;
  a.N = n;
  a.C = c;
  a.cgroups = (c + G::LANES - 1) / G::LANES;
  a.tiles_x = (width + G::TS - 1) / G::TS;
  a.tiles_y = (h + G::TS - 1) / G::TS;
  a.tiles = a.tiles_x * a.tiles_y;
  a.stages = a.cgroups * n * a.tiles;
  a.div_stage_cg = make_fastdiv(n * a.tiles);
  a.div_tiles = make_fastdiv(a.tiles);
  a.div_tx = make_fastdiv(a.tiles_x);
  int per_sm;
  st = kernel_setup<nhwc_tile_kernel<T>>(G::THREADS, M::TOTAL, &per_sm);
  if (st != PLA_OK) return st;
  const long long slots = static_cast<long long>(d->sms) * per_sm;
  const int grid = static_cast<int>(a.stages < slots ? a.stages : slots);
  PLA_CUDA(launch_pdl(nhwc_tile_kernel<T>, grid, G::THREADS, M::TOTAL, stream, xmap, ymap, a));
  PLA_CUDA(cudaGetLastError());
  return PLA_OK;
}

int launch_nhwc_tile_dtype(int dtype, const void* x, const void* w, const void* b, void* y, int n, int c, int h,
                           int width, cudaStream_t stream) {
  switch (dtype) {
    case PLA_F32: return launch_nhwc_tile<float>(x, w, b, y, dtype, n, c, h, width, stream);
    case PLA_BF16: return launch_nhwc_tile<__nv_bfloat16>(x, w, b, y, dtype, n, c, h, width, stream);
    case PLA_F16: return launch_nhwc_tile<__half>(x, w, b, y, dtype, n, c, h, width, stream);
    default: return PLA_ERR_UNSUPPORTED;
  }
}

bool stack_path_ok(const void* x, const void* y, int dtype, int layout, long long n, long long c, int h, int w) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return false;
  if (h != w || (h != 7 && h != 14 && h != 28)) return false;
  if (!aligned(x, 16) || !aligned(y, 16)) return false;
  if (n * c >= 0x7fffffffll || n >= 0x7fffffffll) return false;
  if (layout == PLA_NHWC && (c * static_cast<long long>(dtype_size(dtype))) % 16 != 0) return false;
  // fp32 28x28 stages do not fit in shared memory (2 x 100 KB raw + 100 KB fp32).
  if (h == 28 && dtype == PLA_F32) return false;
  return true;
}

template <typename T, bool NHWC>
int launch_stack_s(const void* x, const void* w, const void* b, void* y, int dtype, int n, int c, int s,
                   cudaStream_t stream) {
  switch (s) {
    case 7: return launch_stack<T, NHWC, 7>(x, w, b, y, dtype, n, c, stream);
    case 14: return launch_stack<T, NHWC, 14>(x, w, b, y, dtype, n, c, stream);
    default: return launch_stack<T, NHWC, 28>(x, w, b, y, dtype, n, c, stream);
  }
}

int launch_stack_dtype(int dtype, bool nhwc, const void* x, const void* w, const void* b, void* y, int n, int c,
                       int s, cudaStream_t stream) {
  switch (dtype) {
    case PLA_F32:
      return nhwc ? launch_stack_s<float, true>(x, w, b, y, dtype, n, c, s, stream)
                  : launch_stack_s<float, false>(x, w, b, y, dtype, n, c, s, stream);
    case PLA_BF16:
      return nhwc ? launch_stack_s<__nv_bfloat16, true>(x, w, b, y, dtype, n, c, s, stream)
                  : launch_stack_s<__nv_bfloat16, false>(x, w, b, y, dtype, n, c, s, stream);
    case PLA_F16:
      return nhwc ? launch_stack_s<__half, true>(x, w, b, y, dtype, n, c, s, stream)
                  : launch_stack_s<__half, false>(x, w, b, y, dtype, n, c, s, stream);
    default:
      return PLA_ERR_UNSUPPORTED;
  }
}

// ---- depthwise 7x7 + channel LayerNorm (NHWC), cluster launches ----------
// Clusters hold one CTA per channel group; the hardware allows up to 16 CTAs
// per cluster (more than 8 needs the non-portable opt-in).
constexpr int kMaxClusterCtas = 16;

// One-time attribute setup of a cluster kernel and the number of clusters of
// `cs` CTAs that can be resident at once on this device (0: none fit).
template <auto Kernel>
int cluster_setup(int threads, uint32_t smem, int cs, int* max_clusters) {
  int dev;
  int st = current_device(&dev);
  if (st != PLA_OK) return st;
  static std::mutex mu;
  static int cached[kMaxDevices][kMaxClusterCtas + 1] = {};  // 0: not yet known; -1: none fit
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev][cs] == 0) {
    PLA_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    PLA_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(cs, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    PLA_CUDA(cudaOccupancyMaxActiveClusters(&n, Kernel, &cfg));
    cached[dev][cs] = n > 0 ? n : -1;
  }
  *max_clusters = cached[dev][cs] > 0 ? cached[dev][cs] : 0;
  return PLA_OK;
}

template <auto Kernel, typename Args>
int launch_clusters(const CUtensorMap& xmap, const CUtensorMap& ymap, const Args& a, int threads, uint32_t smem,
                    int cs, long long units, cudaStream_t stream) {
  int max_cl = 0;
  int st = cluster_setup<Kernel>(threads, smem, cs, &max_cl);
  if (st != PLA_OK) return st;
  if (max_cl == 0) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error),
                  "no cluster of %d CTAs (%u B shared memory each) fits on this device", cs, smem);
    return PLA_ERR_UNSUPPORTED;
  }
  const long long ncl = units < max_cl ? units : max_cl;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(static_cast<unsigned>(cs * ncl), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  PLA_CUDA(cudaLaunchKernelEx(&cfg, Kernel, xmap, ymap, a));
  return PLA_OK;
}

int too_many_channels(int c, int lanes) {
  std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error),
                "depthwise + LayerNorm: %d channels need %d CTAs per cluster, at most %d are possible", c,
                (c + lanes - 1) / lanes, kMaxClusterCtas);
  return PLA_ERR_UNSUPPORTED;
}

template <typename T, int S>
int launch_stack_ln(const void* x, const void* w, const void* b, const LnArgs& ln, void* y, int dtype, int n, int c,
                    cudaStream_t stream) {
  using G = StackGeom<S, kMixStack<T>>;
  using M = StackSmem<T, S, true>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  if (M::TOTAL > d->smem_optin) return PLA_ERR_UNSUPPORTED;
  const int cs = (c + G::LANES - 1) / G::LANES;
  if (cs > kMaxClusterCtas) return too_many_channels(c, G::LANES);
  StackArgs a;
  a.x = x; a.w = w; a.b = b; a.y = y;
  a.N = n; a.C = c;
  a.planes = static_cast<long long>(n) * c;
  a.cgroups = cs;
  a.stages = n * cs;  // n * c < 2^31 (stack_path_ok)
  a.full_stages = 0;
  a.cg_major = 1;
  a.div_c = make_fastdiv(c);
  a.div_cg = make_fastdiv(cs);
  a.div_n = make_fastdiv(n);
  a.ln = ln;
  CUtensorMap xmap, ymap;
  st = make_nhwc_map<T>(&xmap, x, dtype, n, c, S, S, G::LANES, S);
  if (st != PLA_OK) return st;
  st = make_nhwc_map<T>(&ymap, y, dtype, n, c, S, S, G::LANES, S);
  if (st != PLA_OK) return st;
  return launch_clusters<stack_kernel<T, true, S, true>>(xmap, ymap, a, G::THREADS, M::TOTAL, cs, n, stream);
}

template <typename T>
int launch_nhwc_tile_ln(const void* x, const void* w, const void* b, const LnArgs& ln, void* y, int dtype, int n,
                        int c, int h, int width, cudaStream_t stream) {
  using G = NhwcTileGeom;
  using M = NhwcTileSmem<T, true>;
  int st;
  DeviceInfo* d = device_info(&st);
  if (!d) return st;
  const int cs = (c + G::LANES - 1) / G::LANES;
  if (cs > kMaxClusterCtas) return too_many_channels(c, G::LANES);
  NhwcTileArgs a;
  a.w = w;
  a.b = b;
  a.N = n;
  a.C = c;
  a.cgroups = cs;
  a.tiles_x = (width + G::TS - 1) / G::TS;
  a.tiles_y = (h + G::TS - 1) / G::TS;
  a.tiles = a.tiles_x * a.tiles_y;
  a.stages = a.cgroups * n * a.tiles;  // < 2^31 (nhwc_tile_ok)
  a.div_stage_cg = make_fastdiv(n * a.tiles);
  a.div_tiles = make_fastdiv(a.tiles);
  a.div_tx = make_fastdiv(a.tiles_x);
  a.ln = ln;
  CUtensorMap xmap, ymap;
  st = make_nhwc_map<T>(&xmap, x, dtype, n, c, h, width, G::LANES, G::SW);
  if (st != PLA_OK) return st;
  st = make_nhwc_map<T>(&ymap, y, dtype, n, c, h, width, G::LANES, G::TS);
  if (st != PLA_OK) return st;
  return launch_clusters<nhwc_tile_kernel<T, true>>(xmap, ymap, a, G::THREADS, M::TOTAL, cs,
                                                    static_cast<long long>(n) * a.tiles, stream);
}

template <typename T>
int launch_dw_ln(const void* x, const void* w, const void* b, const LnArgs& ln, void* y, int dtype, int n, int c,
                 int h, int width, cudaStream_t stream) {
  if (stack_path_ok(x, y, dtype, PLA_NHWC, n, c, h, width)) {
    switch (h) {
      case 7: return launch_stack_ln<T, 7>(x, w, b, ln, y, dtype, n, c, stream);
      case 14: return launch_stack_ln<T, 14>(x, w, b, ln, y, dtype, n, c, stream);
      default: return launch_stack_ln<T, 28>(x, w, b, ln, y, dtype, n, c, stream);
    }
  }
  if (nhwc_tile_ok(x, y, dtype, n, c, h, width))
    return launch_nhwc_tile_ln<T>(x, w, b, ln, y, dtype, n, c, h, width, stream);
  return PLA_ERR_UNSUPPORTED;
}

bool valid_dtype(int dtype) { return dtype_size(dtype) != 0; }

int stencil_forward_impl(const void* x, const void* w, const void* b, const HostTaps* ht, void* y, int n, int h,
                         int width, int64_t sn, int64_t sh, int64_t sw, int dtype, pla_stream_t stream) {
  if (!valid_dtype(dtype)) return PLA_ERR_UNSUPPORTED;
  if (n < 0 || h < 0 || width < 0) return PLA_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(n) * h * width == 0) return PLA_OK;
  if (!x || (!w && !ht) || !y) return PLA_ERR_INVALID_ARGUMENT;
  if (n > 65535 * 1024 || h > (1 << 30) || width > (1 << 30)) return PLA_ERR_TOO_LARGE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long plane = static_cast<long long>(h) * width;
  if (n == 1) sn = plane;  // ignored for a single plane
  {
    // The output must not overlap the input: a tile's halo rows are read
    // after other CTAs may already have stored their outputs.
    const long long ext[3] = {n, h, width}, str[3] = {sn, sh, sw};
    if (overlap(strided_span(x, dtype_size(dtype), 3, ext, str), dense_span(y, n * plane, dtype_size(dtype))))
      return PLA_ERR_INVALID_ARGUMENT;
  }
  if (sw == 1 && tile_path_ok(x, y, dtype, width, sh, sn, n)) {
    return launch_tile_dtype(dtype, x, w, b, ht, y, n, 1, h, width, sh, sn, 0, h, 0, plane, width, s);
  }
  if (!w) return PLA_ERR_UNSUPPORTED;  // host taps drive the TMA tile path only
  GenericArgs a;
  a.x = x; a.w = w; a.b = b; a.y = y;
  a.N = n; a.C = 1; a.H = h; a.W = width;
  a.xs_n = sn; a.xs_c = 0; a.xs_h = sh; a.xs_w = sw;
  a.ys_n = plane; a.ys_c = 0; a.ys_h = width; a.ys_w = 1;
  a.total = static_cast<long long>(n) * plane;
  a.K = 7;
  return launch_generic_dtype(dtype, a, s);
}

int band_step_impl(const void* in, const void* w, const void* b, const HostTaps* ht, void* out, int rows,
                   int width, int row_begin, int row_end, int dtype, pla_stream_t stream) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return PLA_ERR_UNSUPPORTED;
  if (rows < 0 || width < 0 || row_begin < 0 || row_end < row_begin || row_end > rows)
    return PLA_ERR_INVALID_ARGUMENT;
  if (row_end == row_begin || width == 0) return PLA_OK;
  if (!in || (!w && !ht) || !out) return PLA_ERR_INVALID_ARGUMENT;
  const size_t es = dtype_size(dtype);
  const long long band = static_cast<long long>(rows + 6) * width;
  if (overlap(dense_span(in, band, es), dense_span(out, band, es))) return PLA_ERR_INVALID_ARGUMENT;
  void* out_rows = static_cast<char*>(out) + 3ll * width * es;
  if (!tile_path_ok(in, out_rows, dtype, width, width, band, 1)) return PLA_ERR_UNSUPPORTED;
  return launch_tile_dtype(dtype, in, w, b, ht, out_rows, 1, 1, rows + 6, width, width, band, row_begin, row_end,
                           3, band, width, reinterpret_cast<cudaStream_t>(stream));
}

int iterate_impl(const void* x, const void* w, const void* b, const HostTaps* ht, void* y, void* scratch, int h,
                 int width, int steps, int dtype, pla_stream_t stream) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return PLA_ERR_UNSUPPORTED;
  if (h < 0 || width < 0 || steps < 0) return PLA_ERR_INVALID_ARGUMENT;
  const long long plane = static_cast<long long>(h) * width;
  if (plane == 0) return PLA_OK;
  if (!x || (!w && !ht) || !y || (!scratch && steps > 0)) return PLA_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const size_t bytes = static_cast<size_t>(plane) * dtype_size(dtype);
  {
    // y may be x itself, but not overlap it partially; scratch overlaps neither.
    const Span sx = dense_span(x, plane, dtype_size(dtype)), sy = dense_span(y, plane, dtype_size(dtype));
    if (x != y && overlap(sx, sy)) return PLA_ERR_INVALID_ARGUMENT;
    if (steps > 0) {
      const Span ss = dense_span(scratch, plane, dtype_size(dtype));
      if (overlap(ss, sx) || overlap(ss, sy)) return PLA_ERR_INVALID_ARGUMENT;
    }
  }
  if (steps == 0) {
    if (x != y) PLA_CUDA(cudaMemcpyAsync(y, x, bytes, cudaMemcpyDeviceToDevice, s));
    return PLA_OK;
  }
  if (!tile_path_ok(x, y, dtype, width, width, plane, 1) || !aligned(scratch, 16)) return PLA_ERR_UNSUPPORTED;
  const void* src = x;
  if (x == y && (steps & 1)) {
    // The first step would write into its own input: start from a copy.
    PLA_CUDA(cudaMemcpyAsync(scratch, x, bytes, cudaMemcpyDeviceToDevice, s));
    src = scratch;
  }
  for (int t = 0; t < steps; ++t) {
    void* dst = ((steps - t) & 1) ? y : scratch;
    int st = launch_tile_dtype(dtype, src, w, b, ht, dst, 1, 1, h, width, width, plane, 0, h, 0, plane, width, s);
    if (st != PLA_OK) return st;
    src = dst;
  }
  return PLA_OK;
}

// ---- allocation-free iterate: file-scope scratch ---------------------------
// The ping-pong plane of pla_stencil7x7_iterate_noalloc lives here instead of
// in a caller buffer.  Every GPU that loads this library holds these 16 MiB
// until the process exits; all calls on a device share them.
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static_assert(kNoAllocScratchBytes == PLA_NOALLOC_SCRATCH_BYTES, "header and library agree on the limit");
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocScratch {
  std::mutex mu;
  void* ptr = nullptr;  // set once, by the first successful lookup
};
NoAllocScratch g_noalloc[kMaxDevices];

// Device address of g_noalloc_scratch on the current device.  The host-side
// name of the array is only a stand-in for the symbol, so the address must
// come from cudaGetSymbolAddress, looked up with that device current (on the
// first call made on that device).  Only a successful lookup is kept: a
// failed one (e.g. made during a stream capture) is retried by the next call.
int noalloc_scratch(void** out) {
  int dev;
  int st = current_device(&dev);
  if (st != PLA_OK) return st;
  NoAllocScratch& s = g_noalloc[dev];
  std::lock_guard<std::mutex> lock(s.mu);
  if (!s.ptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    s.ptr = p;
  }
  *out = s.ptr;
  return PLA_OK;
}

// ---- concurrent independent problems: fork / join over library streams ----
constexpr int kForkStreams = 4;

struct ForkJoin {
  std::mutex mu;  // one call at a time per device: the events are reused
  bool ready = false;
  cudaStream_t s[kForkStreams];
  cudaEvent_t fork, done[kForkStreams];
};
ForkJoin g_fork[kMaxDevices];

// Creates the device's streams and events once (called with f.mu held, the
// device current).  A failure leaves nothing behind, so a later call retries.
int fork_join_setup(ForkJoin& f) {
  if (f.ready) return PLA_OK;
  cudaStream_t st[kForkStreams] = {};
  cudaEvent_t ev[kForkStreams + 1] = {};
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < kForkStreams && e == cudaSuccess; ++i)
    e = cudaStreamCreateWithFlags(&st[i], cudaStreamNonBlocking);
  for (int i = 0; i <= kForkStreams && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
  if (e != cudaSuccess) {
    for (cudaEvent_t x : ev)
      if (x) cudaEventDestroy(x);
    for (cudaStream_t x : st)
      if (x) cudaStreamDestroy(x);
    return cuda_fail(e, "fork/join stream setup");
  }
  for (int i = 0; i < kForkStreams; ++i) {
    f.s[i] = st[i];
    f.done[i] = ev[i];
  }
  f.fork = ev[kForkStreams];
  f.ready = true;
  return PLA_OK;
}

// Argument checks of pla_depthwise7x7_forward that need no device.
int dw_check(const void* x, const void* w, const void* y, int n, int c, int h, int width, int dtype, int layout) {
  if (!valid_dtype(dtype)) return PLA_ERR_UNSUPPORTED;
  if (layout != PLA_NCHW && layout != PLA_NHWC) return PLA_ERR_INVALID_ARGUMENT;
  if (n < 0 || c < 0 || h < 0 || width < 0) return PLA_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(n) * c * h * width == 0) return PLA_OK;
  if (!x || !w || !y) return PLA_ERR_INVALID_ARGUMENT;
  if (h > (1 << 30) || width > (1 << 30)) return PLA_ERR_TOO_LARGE;
  return PLA_OK;
}

}  // namespace
}  // namespace pla

using namespace pla;

extern "C" {

const char* pla_status_string(int status) {
  switch (status) {
    case PLA_OK: return "ok";
    case PLA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PLA_ERR_UNSUPPORTED: return "unsupported dtype, layout or shape";
    case PLA_ERR_TOO_LARGE: return "size exceeds supported limits";
    case PLA_ERR_CUDA: return "CUDA error";
    case PLA_ERR_NO_DEVICE: return "no sm_100 device is current";
    case PLA_ERR_DEVICE_FAULT: return "a kernel recorded a device-side fault";
    default: return "unknown status";
  }
}

const char* pla_last_cuda_error(void) { return g_last_cuda_error; }

// 1.1: pla_depthwise_forward (k x k); 1.2: pla_depthwise7x7_layernorm_nhwc;
// 1.3: pla_depthwise7x7_forward_many
int pla_version(void) { return (1 << 16) | 3; }

int pla_stencil7x7_forward(const void* x, const void* w, const void* b, void* y, int n, int h, int width,
                           int64_t sn, int64_t sh, int64_t sw, int dtype, pla_stream_t stream) {
  return stencil_forward_impl(x, w, b, nullptr, y, n, h, width, sn, sh, sw, dtype, stream);
}

int pla_stencil7x7_forward_taps(const void* x, const float* taps, const float* bias, void* y, int n, int h,
                                int width, int64_t sn, int64_t sh, int64_t sw, int dtype, pla_stream_t stream) {
  if (!taps) return PLA_ERR_INVALID_ARGUMENT;
  const HostTaps ht = make_host_taps(taps, bias);
  return stencil_forward_impl(x, nullptr, nullptr, &ht, y, n, h, width, sn, sh, sw, dtype, stream);
}

int pla_depthwise7x7_forward(const void* x, const void* w, const void* b, void* y, int n, int c, int h,
                             int width, int dtype, int layout, pla_stream_t stream) {
  if (!valid_dtype(dtype)) return PLA_ERR_UNSUPPORTED;
  if (layout != PLA_NCHW && layout != PLA_NHWC) return PLA_ERR_INVALID_ARGUMENT;
  if (n < 0 || c < 0 || h < 0 || width < 0) return PLA_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(n) * c * h * width == 0) return PLA_OK;
  if (!x || !w || !y) return PLA_ERR_INVALID_ARGUMENT;
  if (h > (1 << 30) || width > (1 << 30)) return PLA_ERR_TOO_LARGE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long plane = static_cast<long long>(h) * width;
  const long long planes = static_cast<long long>(n) * c;
  if (overlap(dense_span(x, planes * plane, dtype_size(dtype)), dense_span(y, planes * plane, dtype_size(dtype))))
    return PLA_ERR_INVALID_ARGUMENT;
  if (dtype != PLA_F64) {
    if (stack_path_ok(x, y, dtype, layout, n, c, h, width))
      return launch_stack_dtype(dtype, layout == PLA_NHWC, x, w, b, y, n, c, h, s);
    if (layout == PLA_NCHW && dtype != PLA_F32) {
      int st;
      DeviceInfo* d = device_info(&st);
      if (!d) return st;
      if (pair_path_ok(x, y, dtype, n, c, h, width, d->sms))
        return dtype == PLA_BF16 ? launch_pair<__nv_bfloat16>(x, w, b, y, dtype, n, c, s)
                                 : launch_pair<__half>(x, w, b, y, dtype, n, c, s);
    }
    if (layout == PLA_NCHW && (width >= 64 || use_narrow_tiles(width, h)) && planes <= 0x7fffffffll &&
        tile_path_ok(x, y, dtype, width, width, plane, static_cast<int>(planes))) {
      return launch_tile_dtype(dtype, x, w, b, nullptr, y, static_cast<int>(planes), c, h, width, width, plane, 0,
                               h, 0, plane, width, s);
    }
    if (layout == PLA_NHWC && nhwc_tile_ok(x, y, dtype, n, c, h, width))
      return launch_nhwc_tile_dtype(dtype, x, w, b, y, n, c, h, width, s);
    CmArgs a;
    a.x = x; a.w = w; a.b = b; a.y = y;
    a.N = n; a.C = c; a.H = h; a.W = width;
    return launch_cm_dtype(dtype, layout == PLA_NHWC, a, s);
  }
  GenericArgs a;
  a.x = x; a.w = w; a.b = b; a.y = y;
  a.N = n; a.C = c; a.H = h; a.W = width;
  if (layout == PLA_NCHW) {
    a.xs_n = c * plane; a.xs_c = plane; a.xs_h = width; a.xs_w = 1;
  } else {
    a.xs_n = c * plane; a.xs_c = 1; a.xs_h = static_cast<long long>(width) * c; a.xs_w = c;
  }
  a.ys_n = a.xs_n; a.ys_c = a.xs_c; a.ys_h = a.xs_h; a.ys_w = a.xs_w;
  a.total = planes * plane;
  a.K = 7;
  return launch_generic_dtype(dtype, a, s);
}

int pla_depthwise7x7_forward_many(const pla_dw_problem* p, int count, int dtype, int layout, pla_stream_t stream) {
  if (count < 0 || (count > 0 && !p) || count > 1024) return PLA_ERR_INVALID_ARGUMENT;
  const size_t es = dtype_size(dtype);
  for (int i = 0; i < count; ++i) {
    const int st = dw_check(p[i].x, p[i].w, p[i].y, p[i].n, p[i].c, p[i].h, p[i].width, dtype, layout);
    if (st != PLA_OK) return st;
  }
  // No output may overlap any input or output of the call (the problems run
  // concurrently).
  for (int i = 0; i < count; ++i) {
    const long long ei = static_cast<long long>(p[i].n) * p[i].c * p[i].h * p[i].width;
    if (ei == 0) continue;
    const Span yi = dense_span(p[i].y, ei, es);
    for (int j = 0; j < count; ++j) {
      const long long ej = static_cast<long long>(p[j].n) * p[j].c * p[j].h * p[j].width;
      if (ej == 0) continue;
      if (overlap(yi, dense_span(p[j].x, ej, es))) return PLA_ERR_INVALID_ARGUMENT;
      if (j != i && overlap(yi, dense_span(p[j].y, ej, es))) return PLA_ERR_INVALID_ARGUMENT;
    }
  }
  if (count == 0) return PLA_OK;
  if (count == 1)
    return pla_depthwise7x7_forward(p[0].x, p[0].w, p[0].b, p[0].y, p[0].n, p[0].c, p[0].h, p[0].width, dtype,
                                    layout, stream);
  int dev;
  int st = current_device(&dev);
  if (st != PLA_OK) return st;
  ForkJoin& f = g_fork[dev];
  std::lock_guard<std::mutex> lock(f.mu);
  st = fork_join_setup(f);
  if (st != PLA_OK) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int used = count < kForkStreams ? count : kForkStreams;
  PLA_CUDA(cudaEventRecord(f.fork, s));
  for (int i = 0; i < used; ++i) PLA_CUDA(cudaStreamWaitEvent(f.s[i], f.fork, 0));
  // Smallest problems first (stable): a large problem's persistent grid
  // fills every SM, and a small grid launched after it would only start in
  // its drain (ConvNeXt-T sweep at 32 images per GPU: 49.2 vs 52.4 us).
  int order[1024];
  long long elems[1024];
  for (int i = 0; i < count; ++i) {
    order[i] = i;
    elems[i] = static_cast<long long>(p[i].n) * p[i].c * p[i].h * p[i].width;
  }
  std::stable_sort(order, order + count, [&](int a, int b) { return elems[a] < elems[b]; });
  int first_err = PLA_OK;
  for (int j = 0; j < count; ++j) {
    const int i = order[j];
    const int r = pla_depthwise7x7_forward(p[i].x, p[i].w, p[i].b, p[i].y, p[i].n, p[i].c, p[i].h, p[i].width,
                                           dtype, layout, reinterpret_cast<pla_stream_t>(f.s[j % used]));
    if (r != PLA_OK && first_err == PLA_OK) first_err = r;
  }
  // Join every forked stream back, also after a failed launch, so the
  // caller's stream never runs ahead of work this call queued.
  for (int i = 0; i < used; ++i) {
    PLA_CUDA(cudaEventRecord(f.done[i], f.s[i]));
    PLA_CUDA(cudaStreamWaitEvent(s, f.done[i], 0));
  }
  return first_err;
}

int pla_depthwise_forward(const void* x, const void* w, const void* b, void* y, int n, int c, int h, int width,
                          int k, int dtype, int layout, pla_stream_t stream) {
  if (k == 7) return pla_depthwise7x7_forward(x, w, b, y, n, c, h, width, dtype, layout, stream);
  if (k != 3 && k != 5) return PLA_ERR_UNSUPPORTED;
  if (!valid_dtype(dtype)) return PLA_ERR_UNSUPPORTED;
  if (layout != PLA_NCHW && layout != PLA_NHWC) return PLA_ERR_INVALID_ARGUMENT;
  if (n < 0 || c < 0 || h < 0 || width < 0) return PLA_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(n) * c * h * width == 0) return PLA_OK;
  if (!x || !w || !y) return PLA_ERR_INVALID_ARGUMENT;
  if (h > (1 << 30) || width > (1 << 30)) return PLA_ERR_TOO_LARGE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const long long plane = static_cast<long long>(h) * width;
  const long long planes = static_cast<long long>(n) * c;
  if (overlap(dense_span(x, planes * plane, dtype_size(dtype)), dense_span(y, planes * plane, dtype_size(dtype))))
    return PLA_ERR_INVALID_ARGUMENT;
  // Dense NCHW planes wide enough for the tile shapes: the TMA tile kernel
  // with a k x k filter.  Everything else (NHWC, small or misaligned planes,
  // fp64): the one-thread-per-output kernel.
  if (dtype != PLA_F64 && layout == PLA_NCHW && (width >= 64 || use_narrow_tiles(width, h)) &&
      planes <= 0x7fffffffll && tile_path_ok(x, y, dtype, width, width, plane, static_cast<int>(planes))) {
    return k == 3 ? launch_tile_dtype<3>(dtype, x, w, b, nullptr, y, static_cast<int>(planes), c, h, width, width,
                                         plane, 0, h, 0, plane, width, s)
                  : launch_tile_dtype<5>(dtype, x, w, b, nullptr, y, static_cast<int>(planes), c, h, width, width,
                                         plane, 0, h, 0, plane, width, s);
  }
  GenericArgs a;
  a.x = x; a.w = w; a.b = b; a.y = y;
  a.N = n; a.C = c; a.H = h; a.W = width;
  if (layout == PLA_NCHW) {
    a.xs_n = c * plane; a.xs_c = plane; a.xs_h = width; a.xs_w = 1;
  } else {
    a.xs_n = c * plane; a.xs_c = 1; a.xs_h = static_cast<long long>(width) * c; a.xs_w = c;
  }
  a.ys_n = a.xs_n; a.ys_c = a.xs_c; a.ys_h = a.xs_h; a.ys_w = a.xs_w;
  a.total = planes * plane;
  a.K = k;
  return launch_generic_dtype(dtype, a, s);
}

int pla_depthwise7x7_layernorm_nhwc(const void* x, const void* w, const void* b, const void* gamma,
                                    const void* beta, float eps, void* y, int n, int c, int h, int width, int dtype,
                                    pla_stream_t stream) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return PLA_ERR_UNSUPPORTED;
  if (n < 0 || c < 0 || h < 0 || width < 0 || !(eps >= 0.f) || eps == INFINITY) return PLA_ERR_INVALID_ARGUMENT;
  if (static_cast<long long>(n) * c * h * width == 0) return PLA_OK;
  if (!x || !w || !y) return PLA_ERR_INVALID_ARGUMENT;
  if (h > (1 << 30) || width > (1 << 30)) return PLA_ERR_TOO_LARGE;
  {
    const long long elems = static_cast<long long>(n) * c * h * width;
    if (overlap(dense_span(x, elems, dtype_size(dtype)), dense_span(y, elems, dtype_size(dtype))))
      return PLA_ERR_INVALID_ARGUMENT;
  }
  LnArgs ln;
  ln.gamma = gamma;
  ln.beta = beta;
  ln.eps = eps;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PLA_F32: return launch_dw_ln<float>(x, w, b, ln, y, dtype, n, c, h, width, s);
    case PLA_BF16: return launch_dw_ln<__nv_bfloat16>(x, w, b, ln, y, dtype, n, c, h, width, s);
    default: return launch_dw_ln<__half>(x, w, b, ln, y, dtype, n, c, h, width, s);
  }
}

int pla_stencil7x7_band_step(const void* in, const void* w, const void* b, void* out, int rows, int width,
                             int row_begin, int row_end, int dtype, pla_stream_t stream) {
  return band_step_impl(in, w, b, nullptr, out, rows, width, row_begin, row_end, dtype, stream);
}

int pla_stencil7x7_band_step_taps(const void* in, const float* taps, const float* bias, void* out, int rows,
                                  int width, int row_begin, int row_end, int dtype, pla_stream_t stream) {
  if (!taps) return PLA_ERR_INVALID_ARGUMENT;
  const HostTaps ht = make_host_taps(taps, bias);
  return band_step_impl(in, nullptr, nullptr, &ht, out, rows, width, row_begin, row_end, dtype, stream);
}

int pla_stencil7x7_iterate(const void* x, const void* w, const void* b, void* y, void* scratch, int h, int width,
                           int steps, int dtype, pla_stream_t stream) {
  return iterate_impl(x, w, b, nullptr, y, scratch, h, width, steps, dtype, stream);
}

int pla_stencil7x7_iterate_taps(const void* x, const float* taps, const float* bias, void* y, void* scratch, int h,
                                int width, int steps, int dtype, pla_stream_t stream) {
  if (!taps) return PLA_ERR_INVALID_ARGUMENT;
  const HostTaps ht = make_host_taps(taps, bias);
  return iterate_impl(x, nullptr, nullptr, &ht, y, scratch, h, width, steps, dtype, stream);
}

int pla_stencil7x7_iterate_noalloc(const void* x, const void* w, const void* b, void* y, int h, int width,
                                   int steps, int dtype, pla_stream_t stream) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return PLA_ERR_UNSUPPORTED;
  if (h < 0 || width < 0 || steps < 0) return PLA_ERR_INVALID_ARGUMENT;
  const unsigned long long bytes =
      static_cast<unsigned long long>(h) * static_cast<unsigned long long>(width) * dtype_size(dtype);
  if (bytes > kNoAllocScratchBytes) {
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error),
                  "pla_stencil7x7_iterate_noalloc: a %d x %d grid needs %llu scratch bytes, the static "
                  "scratch holds %llu",
                  h, width, bytes, static_cast<unsigned long long>(kNoAllocScratchBytes));
    return PLA_ERR_TOO_LARGE;
  }
  if (bytes == 0) return PLA_OK;
  if (!x || !w || !y) return PLA_ERR_INVALID_ARGUMENT;
  if (x != y && overlap(dense_span(x, bytes / dtype_size(dtype), dtype_size(dtype)),
                        dense_span(y, bytes / dtype_size(dtype), dtype_size(dtype))))
    return PLA_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st != PLA_OK) return st;
  return iterate_impl(x, w, b, nullptr, y, scratch, h, width, steps, dtype, stream);
}

int pla_stencil7x7_band_step_halo(const void* in, const float* taps, const float* bias, void* out, int rows,
                                  int width, int dtype, void* up_out, int up_rows, void* down_out,
                                  unsigned int* flags, unsigned int* up_flags, unsigned int* down_flags,
                                  unsigned int* counters, unsigned int step, pla_stream_t stream) {
  if (dtype != PLA_F32 && dtype != PLA_BF16 && dtype != PLA_F16) return PLA_ERR_UNSUPPORTED;
  if (!in || !taps || !out || !flags || !counters || rows <= 0 || width <= 0) return PLA_ERR_INVALID_ARGUMENT;
  if ((up_out && (!up_flags || up_rows < 3)) || (down_out && !down_flags)) return PLA_ERR_INVALID_ARGUMENT;
  const size_t es = dtype_size(dtype);
  const long long band = static_cast<long long>(rows + 6) * width;
  if (overlap(dense_span(in, band, es), dense_span(out, band, es))) return PLA_ERR_INVALID_ARGUMENT;
  void* out_rows = static_cast<char*>(out) + 3ll * width * es;
  if (!tile_path_ok(in, out_rows, dtype, width, width, band, 1)) return PLA_ERR_UNSUPPORTED;
  if ((up_out && !aligned(up_out, 16)) || (down_out && !aligned(down_out, 16))) return PLA_ERR_UNSUPPORTED;
  const HostTaps ht = make_host_taps(taps, bias);
  HaloLinks links{};
  links.up_out = up_out;
  links.down_out = down_out;
  links.up_rows = up_rows;
  links.flags = flags;
  links.up_flags = up_flags;
  links.down_flags = down_flags;
  links.counters = counters;
  links.step = step;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case PLA_F32: return launch_tile_halo<float>(in, ht, out_rows, dtype, rows, width, links, s);
    case PLA_BF16: return launch_tile_halo<__nv_bfloat16>(in, ht, out_rows, dtype, rows, width, links, s);
    default: return launch_tile_halo<__half>(in, ht, out_rows, dtype, rows, width, links, s);
  }
}

int pla_ipc_export(const void* ptr, void* handle, uint64_t* offset) {
  if (!ptr || !handle || !offset) return PLA_ERR_INVALID_ARGUMENT;
  void* base = nullptr;
  int st = alloc_base(ptr, &base);
  if (st != PLA_OK) return st;
  cudaIpcMemHandle_t h;
  PLA_CUDA(cudaIpcGetMemHandle(&h, base));
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(static_cast<const char*>(ptr) - static_cast<const char*>(base));
  return PLA_OK;
}

int pla_ipc_import(const void* handle, uint64_t offset, void** ptr) {
  if (!handle || !ptr) return PLA_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  PLA_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<char*>(base) + offset;
  return PLA_OK;
}

int pla_ipc_close(void* ptr, uint64_t offset) {
  if (!ptr) return PLA_ERR_INVALID_ARGUMENT;
  PLA_CUDA(cudaIpcCloseMemHandle(static_cast<char*>(ptr) - offset));
  return PLA_OK;
}

int pla_read_device_faults(unsigned int* faults) {
  if (!faults) return PLA_ERR_INVALID_ARGUMENT;
  PLA_CUDA(cudaMemcpyFromSymbol(faults, g_device_faults, sizeof(unsigned int)));
  return PLA_OK;
}

int pla_clear_device_faults(void) {
  const unsigned int zero = 0;
  PLA_CUDA(cudaMemcpyToSymbol(g_device_faults, &zero, sizeof(unsigned int)));
  return PLA_OK;
}

}  // extern "C"
