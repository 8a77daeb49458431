// Plane-tile kernel: K x K correlation (K = 7; 3 and 5 for the depthwise
// filters of the reference's MetaSchedule benchmark) over a stack of dense planes
// (the single-step stencil of data/stencil_7x7.py, NCHW depthwise planes of
// data/depthwise_conv_7x7.py with wide rows, and one Jacobi step of the
// iterated stencil, whole grid or one row band).
//
// Design (sm_100a):
//  * CTAs walk a flat list of TH x TW output tiles, plane-major then
//    row-major.  Short lists: persistent CTAs (grid = #SMs x resident CTAs),
//    tile t, t + grid, ...  Long lists (>= 8 tiles per resident CTA): one CTA
//    per tile, and each running CTA takes over the tiles of CTAs not yet
//    started with Blackwell's cluster launch control
//    (clusterlaunchcontrol.try_cancel), one claim ahead of its TMA prefetch.
//    Claimed tiles come in launch order, so the tiles in flight stay a compact
//    window (DRAM row locality, halo rows still in L2) and SMs finish together:
//    9 % faster on a 32768^2 band step, 14 % on a 3x3 1x32x1024^2 depthwise;
//    with fewer tiles per CTA the per-tile claim costs more than it saves;
//  * each tile's (TH+6) x (TW+2*LEFT) input window is one 3-D TMA tile load
//    (cp.async.bulk.tensor, no multicast) into a shared-memory ring of NS = 2
//    stages (3 or 4 stages measured slower for every filter size: the larger
//    ring leaves room for fewer CTAs per SM)
//    guarded by mbarriers, so the next tile streams in while this one is
//    computed; TMA's out-of-bounds zero fill supplies the zero padding;
//  * 4 warps; a thread owns R rows x 4 columns of outputs, loads
//    each input row of its window once with three 128-bit (fp32) or 64-bit
//    (16-bit types) shared loads and applies it to every output row it
//    touches (the 7-wide window is reused across the 4 columns in registers);
//  * the 49 taps of the current plane's filter live in registers; fp32 FMA
//    in row-major tap order; bias added in fp32; 128/64-bit vector stores;
//  * 16-bit planes with device-resident filters take x and w straight from
//    their packed 16-bit form into mixed-precision FMAs (fp32 accumulator,
//    same bits as widening first), which drops the unpacking and halves the
//    registers the taps need.
#pragma once

#include "pla_common.cuh"

namespace pla {

constexpr int kTileThreads = 128;

// A warp is (32 / LX) row groups x LX column groups; a thread owns R rows x
// 4 columns, so a tile is TH = 4 warps x (32 / LX) x R rows by TW = 4 LX
// columns.  (R, LX) = (8, 32) gives the 32 x 128 tiles of wide planes,
// (7, 16) one 56 x 64 tile per 56-wide plane.
// The TMA box starts LEFT columns left of the tile: LEFT * sizeof(T) == 16 B
// keeps the innermost TMA coordinate 16-byte aligned (a hard TMA rule), and
// LEFT >= 3 covers the halo.  The box is LEFT + TW + LEFT wide.
template <typename T, int R, int LX, int K = 7>
struct TileGeom {
  static constexpr int NS = 2;                          // ring stages
  static_assert(LX == 32 || LX == 16, "column groups per warp");
  static constexpr int TW = 4 * LX;                     // output columns per tile
  static constexpr int TH = (kTileThreads / 32) * (32 / LX) * R;  // output rows per tile
  static constexpr int ROWS = TH + K - 1;    // input rows per tile (K / 2-row halo)
  static constexpr int LEFT = 16 / sizeof(T);
  static constexpr int PITCH = TW + 2 * LEFT;
  static_assert(LEFT >= 4 && (LEFT * sizeof(T)) % 16 == 0, "TMA x must stay 16-byte aligned");
  static_assert((PITCH * sizeof(T)) % 16 == 0, "TMA box inner extent must be a multiple of 16 B");
  static constexpr uint32_t BYTES = ROWS * PITCH * sizeof(T);
  static constexpr uint32_t STAGE = (BYTES + 127u) & ~127u;
  // + NS mbarriers, the launch-control mbarrier, its 16-byte response, 2 tile ids
  static constexpr uint32_t SMEM = NS * STAGE + 64;
};

struct TileArgs {
  const void* w;            // [C][49] taps
  const void* b;            // [C] or nullptr
  void* y;                  // output base (row 0 of output plane 0)
  int planes;               // planes in the stack (tensor-map z extent)
  int C;                    // filter index of plane p is p % C
  int W;                    // plane width (output columns)
  int row_begin, row_end;   // output rows computed: [row_begin, row_end)
  int in_row_shift;         // input row (tensor-map y) of output row r is r + in_row_shift
  int tiles_x, tiles_y;     // tiles per plane
  int dyn;                  // 1: one CTA per tile, pending CTAs' tiles claimed
  int total_tiles;          // planes * tiles_y * tiles_x (< 2^31, checked on the host)
  FastDiv div_tx, div_ty, div_c;
  long long y_plane_stride; // elements
  long long y_row_stride;   // elements
};

// Row-band halo exchange over peer memory (HALO kernels only).  The band of
// this GPU is band rows [0, rows) of buffers laid out as in
// pla_stencil7x7_band_step; its neighbours' `out` buffers are mapped here
// (CUDA IPC).  Step s: tiles holding band rows 0..2 ("top edge") and
// rows-3..rows-1 ("bottom edge") are visited first; before loading its input a
// top (bottom) edge tile waits until flags[0] (flags[1]) >= s, i.e. until the
// neighbour above (below) has delivered its step s-1 rows into this GPU's
// halo; after storing, edge tiles also store their 3 rows into the
// neighbour's halo rows, and the last edge tile of a side raises that
// neighbour's flag to s+1 (release, system scope).  Counters are per side,
// monotonic across steps (expected (s+1) x tiles of that side).
struct HaloLinks {
  void* up_out;             // neighbour above: its out buffer (peer memory), or nullptr
  void* down_out;           // neighbour below: its out buffer (peer memory), or nullptr
  int up_rows;              // band rows of the neighbour above
  int rows;                 // band rows here
  int bot0;                 // first tile row holding band row rows-3
  int n_top, n_bot;         // edge tiles per side
  unsigned int* flags;      // this GPU: [0] delivered by up, [1] delivered by down
  unsigned int* up_flags;   // neighbour above's flags (peer memory)
  unsigned int* down_flags; // neighbour below's flags (peer memory)
  unsigned int* counters;   // this GPU: edge tiles finished, [0] top, [1] bottom
  unsigned int step;
};

// Visit order of tile rows for HALO launches: the top edge row, the bottom
// edge rows, then the rest.
__device__ __forceinline__ int halo_tile_row(int q, int tiles_y, int bot0) {
  if (q == 0) return 0;
  const int nb = tiles_y - bot0;
  return q <= nb ? bot0 + q - 1 : q - nb;
}

// HOST_TAPS: one filter for every plane, read from the HostTaps parameter;
// otherwise plane p uses the device filter a.w[(p % C) * 49 ...] held in
// registers.
template <typename T, int R, int LX, bool HOST_TAPS, bool HALO = false, int K = 7>
__global__ void __launch_bounds__(kTileThreads, HOST_TAPS ? 5 : 4)
    tile_kernel(const __grid_constant__ CUtensorMap tmap, const TileArgs a,
                const __grid_constant__ HostTaps taps, const __grid_constant__ HaloLinks h) {
  static_assert(K == 3 || K == 5 || K == 7, "filter side");
  static_assert(K == 7 || (!HALO && !HOST_TAPS), "halo exchange and host taps are 7x7 only");
  constexpr int NT = K * K;        // taps
  constexpr int CX = 4 - K / 2;    // v[j + kx + CX] is input column ox + j + kx - K / 2
  using G = TileGeom<T, R, LX, K>;
  extern __shared__ __align__(128) unsigned char smem[];
  constexpr int NS = G::NS;
  static_assert(NS == 2, "tile claiming assumes a 2-stage ring");
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NS * G::STAGE);
  uint64_t* claim_bar = bars + NS;                                        // byte 16
  unsigned char* claim_resp = smem + NS * G::STAGE + 32;                  // 16-byte aligned
  int* next_tile = reinterpret_cast<int*>(smem + NS * G::STAGE + 48);     // [2]
  const bool dyn = !HALO && a.dyn;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int rgrp = (tid >> 5) * (32 / LX) + lane / LX;  // row group within the tile
  const int cgrp = lane % LX;                           // column group within the tile

  if (tid == 0) {
    prefetch_tensormap(&tmap);
#pragma unroll
    for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
    mbar_init(claim_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Static-striding launches use programmatic dependent launch: everything
  // above overlaps the previous kernel's drain; every global read or write
  // below comes after that kernel has completed and flushed (a no-op for a
  // launch without the attribute).
  grid_dependency_wait();

  const int total = a.total_tiles;
  const int stride = gridDim.x;
  int t = blockIdx.x;
  bool claiming = dyn;
  // Thread 0: ask for the tile of a CTA that has not started yet; the
  // response (16 bytes) lands in claim_resp and completes claim_bar.
  auto claim = [&]() { clc_try_cancel(claim_resp, claim_bar); };

  auto issue = [&](int tile, int stage) {
    const int q = fdiv(tile, a.div_tx);
    const int tx = tile - q * a.tiles_x;
    const int plane = fdiv(q, a.div_ty);
    int ty = q - plane * a.tiles_y;
    if (HALO) {
      ty = halo_tile_row(ty, a.tiles_y, h.bot0);
      // The halo rows this tile reads arrive from the neighbours.
      if (ty == 0 && h.up_out) wait_flag_geq(&h.flags[0], h.step);
      if (ty >= h.bot0 && h.down_out) wait_flag_geq(&h.flags[1], h.step);
      fence_proxy_async_global();
    }
    const int x0 = tx * G::TW - G::LEFT;
    const int y0 = a.row_begin + ty * G::TH + a.in_row_shift - K / 2;
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[stage], G::BYTES);
    tma_load_3d(smem + stage * G::STAGE, &tmap, &bars[stage], x0, y0, plane);
  };

  // Prologue: the first NS - 1 tiles of this CTA.
  if (tid == 0) {
#pragma unroll
    for (int j = 0; j < NS - 1; ++j)
      if (dyn ? j == 0 : t + j * stride < total) issue(t + j * stride, j);
    if (dyn) claim();
  }

  const T* wt_base = static_cast<const T*>(a.w);
  const T* b_base = static_cast<const T*>(a.b);
  // 16-bit planes, filter from device memory: packed 16-bit taps + mixed FMA.
  constexpr bool MIX = sizeof(T) == 2 && !HOST_TAPS;
  float wt[NT];
  uint32_t wh[(NT + 1) / 2];
  int cur_c = -1;
  float bias = 0.f;

  for (int it = 0; t < total; ++it) {
    const int stage = it % NS;
    if (dyn) {
      // The claim made one tile ago: on success prefetch that tile into the
      // other stage and claim again; a failed claim (or a wait past its
      // bound) ends this CTA after the current tile.  No claim follows a
      // failed one.
      if (tid == 0) {
        int nt = -1;
        if (claiming && mbar_wait_bounded(claim_bar, it & 1)) nt = clc_claimed_x(claim_resp);
        if (nt >= 0) {
          issue(nt, stage ^ 1);
          claim();
        } else {
          claiming = false;
        }
        next_tile[it & 1] = nt;  // read by every thread after this iteration's barrier
      }
    } else if (tid == 0 && t + (NS - 1) * stride < total) {
      // Tile it + NS - 1 goes into the stage that tile it - 1 used; every
      // thread left that stage at the barrier that ended iteration it - 1.
      issue(t + (NS - 1) * stride, (it + NS - 1) % NS);
    } else if (tid == 0) {
      // Static striding, last tile of this CTA: a kernel launched after this
      // one with programmatic dependent launch may start its CTAs now.
      launch_dependents();
    }

    const int q = fdiv(t, a.div_tx);
    const int tx = t - q * a.tiles_x;
    const int plane = fdiv(q, a.div_ty);
    int ty = q - plane * a.tiles_y;
    if (HALO) ty = halo_tile_row(ty, a.tiles_y, h.bot0);
    if (!HOST_TAPS) {
      const int c = plane - fdiv(plane, a.div_c) * a.C;
      if (c != cur_c) {
        cur_c = c;
        if constexpr (MIX) {
          load_taps16<NT>(wt_base, c, wh);
        } else {
#pragma unroll
          for (int k = 0; k < NT; ++k) wt[k] = to_acc(wt_base[c * NT + k]);
        }
        bias = b_base ? to_acc(b_base[c]) : 0.f;
      }
    }

    mbar_wait_bounded(&bars[stage], (it / NS) & 1);

    // v[k] below is input column ox - 4 + k (ox = this thread's first output column).
    const T* s = reinterpret_cast<const T*>(smem + stage * G::STAGE) + (rgrp * R) * G::PITCH + 4 * cgrp +
                 (G::LEFT - 4);
    // The first tap of every output (ky = kx = 0, reached at ir == r) starts
    // its accumulator with a plain product: RN(x * w) == fma(x, w, +0) except
    // for the sign of an exact zero, which no later "+" can tell apart.
    float acc[R][4];
    if constexpr (MIX) {
      // Same loop on packed 16-bit words: u[k / 2] half k & 1 is column ox - 4 + k.
      // The first tap adds its product to -0, which returns RN(x * w) exactly.
#pragma unroll
      for (int ir = 0; ir < R + K - 1; ++ir) {
        const uint2 q0 = *reinterpret_cast<const uint2*>(s + ir * G::PITCH);
        const uint2 q1 = *reinterpret_cast<const uint2*>(s + ir * G::PITCH + 4);
        const uint2 q2 = *reinterpret_cast<const uint2*>(s + ir * G::PITCH + 8);
        const uint32_t u[6] = {q0.x, q0.y, q1.x, q1.y, q2.x, q2.y};
#pragma unroll
        for (int kx = 0; kx < K; ++kx) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = ir - r;
            if (ky >= 0 && ky < K) {
              const int k = ky * K + kx;
              const unsigned short wv = half_of(wh[k >> 1], k & 1);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int c = j + kx + CX;
                acc[r][j] = fma_mix(T(), half_of(u[c >> 1], c & 1), wv, (ky == 0 && kx == 0) ? -0.0f : acc[r][j]);
              }
            }
          }
        }
      }
    } else {
#pragma unroll
      for (int ir = 0; ir < R + K - 1; ++ir) {
        float v[12];
        load_row12(s + ir * G::PITCH, v);
#pragma unroll
        for (int kx = 0; kx < K; ++kx) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = ir - r;
            if (ky >= 0 && ky < K) {
              const float wv = HOST_TAPS ? taps.w[ky * K + kx] : wt[ky * K + kx];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                if (ky == 0 && kx == 0)
                  acc[r][j] = __fmul_rn(v[j + kx + CX], wv);
                else
                  acc[r][j] = fma_rn(v[j + kx + CX], wv, acc[r][j]);
              }
            }
          }
        }
      }
    }
    // Every thread is done with this stage before it is refilled.
    __syncthreads();

    const int ox = tx * G::TW + 4 * cgrp;
    const bool has_bias = HOST_TAPS ? taps.has_b != 0 : b_base != nullptr;
    if (HOST_TAPS) bias = taps.b;
    if (has_bias) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][j] += bias;
    }
    const int oy0 = a.row_begin + ty * G::TH + rgrp * R;
    T* yp = static_cast<T*>(a.y) + static_cast<long long>(plane) * a.y_plane_stride +
            static_cast<long long>(oy0) * a.y_row_stride + ox;
    // Whole tile inside the output (the common case): no per-row tests.
    const bool interior = (tx + 1) * G::TW <= a.W && a.row_begin + (ty + 1) * G::TH <= a.row_end;
    if (interior) {
#pragma unroll
      for (int r = 0; r < R; ++r) store4(yp + r * a.y_row_stride, acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    } else if (ox < a.W) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (oy0 + r < a.row_end) store4(yp + r * a.y_row_stride, acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    }

    if (HALO) {
      const bool top = ty == 0 && h.up_out != nullptr;
      const bool bot = ty >= h.bot0 && h.down_out != nullptr;
      if (top || bot) {
        if (ox < a.W) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int oy = oy0 + r;
            if (top && oy < 3)  // neighbour above: its bottom halo rows up_rows+3 .. up_rows+5
              store4(static_cast<T*>(h.up_out) + static_cast<long long>(h.up_rows + 3 + oy) * a.W + ox,
                     acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
            if (bot && oy >= h.rows - 3 && oy < h.rows)  // neighbour below: its top halo rows 0..2
              store4(static_cast<T*>(h.down_out) + static_cast<long long>(oy - (h.rows - 3)) * a.W + ox,
                     acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
          }
        }
        __syncthreads();
        if (tid == 0) {
          fence_acq_rel_sys();
          if (top && atom_add_acq_rel_gpu(&h.counters[0], 1u) + 1u == (h.step + 1u) * h.n_top) {
            fence_acq_rel_sys();
            st_release_sys(&h.up_flags[1], h.step + 1u);
          }
          if (bot && atom_add_acq_rel_gpu(&h.counters[1], 1u) + 1u == (h.step + 1u) * h.n_bot) {
            fence_acq_rel_sys();
            st_release_sys(&h.down_flags[0], h.step + 1u);
          }
        }
      }
    }
    if (dyn) {
      t = next_tile[it & 1];
      if (t < 0) break;
    } else {
      t += stride;
    }
  }
}

}  // namespace pla
