// NHWC spatial-tile kernel: depthwise 7x7 on channels_last activations whose
// planes are not one of the plane-stack sizes (7, 14, 28), e.g. the 56x56
// planes of ConvNeXt stage 1 (data/depthwise_conv_7x7.py's benchmark cfg4 in
// channels_last).
//
// Work unit ("stage"): 32 consecutive channels of one image x one 14 x 14
// output tile.  Its 20 x 20 input window (3-pixel halo) is one 4-D TMA box
// (32 channels x 20 x 20 x 1 image); the TMA zero fill outside the image is
// the convolution's zero padding, so edge and interior tiles run the same
// code.  Stages stream through a 2-deep input ring (mbarriers, issued one
// stage ahead by thread 0 of a persistent CTA) and leave through a 2-deep
// output ring with one TMA store each (the store clips at the image edge).
//
// Lane l of every warp owns channel 32 cg + l; warp g computes output rows
// 2g, 2g + 1 of the tile, all 14 columns, reading each of its 8 input rows
// once (20 elements: 16-bit elements or fp32 words, conflict-free across
// the warp).  16-bit data feeds mixed-precision FMAs (16-bit x and w, fp32
// accumulator) with the taps packed two per register; fp32 data keeps its
// 49 taps in registers.  Same tap order and rounding as every kernel here.
// CTAs own contiguous runs of stages ordered channel-group-major, so a CTA
// reloads its filters only when its channel group changes.
//
// LN: the stage's outputs go through the channel LayerNorm epilogue of
// ln_epilogue.cuh before the store; the kernel then runs as clusters of
// ceil(C / 32) CTAs, rank r taking channel group r of the (image, tile)
// stages its cluster visits.  A stage is normalised and stored one stage
// late, so the cluster exchange overlaps the next stage's FMAs.
#pragma once

#include "ln_epilogue.cuh"
#include "pla_common.cuh"
#include "stack_kernel.cuh"

namespace pla {

struct NhwcTileGeom {
  static constexpr int TS = 14;              // output tile side
  static constexpr int SW = TS + 6;          // input window side
  static constexpr int LANES = 32;           // channels per stage
  static constexpr int R = 2;                // output rows per thread
  static constexpr int WARPS = TS / R;       // 7
  static constexpr int THREADS = 32 * WARPS;
};

template <typename T, bool LN = false>
struct NhwcTileSmem {
  using G = NhwcTileGeom;
  static constexpr uint32_t IN = ((G::LANES * G::SW * G::SW * sizeof(T)) + 127u) & ~127u;
  static constexpr uint32_t OUT = ((G::LANES * G::TS * G::TS * sizeof(T)) + 127u) & ~127u;
  static constexpr uint32_t OFF_IN = 0;
  static constexpr uint32_t OFF_OUT = 2 * IN;
  static constexpr uint32_t OFF_BAR = OFF_OUT + 2 * OUT;
  static constexpr uint32_t OFF_LN = OFF_BAR + 2 * sizeof(uint64_t);
  static constexpr uint32_t TOTAL = OFF_LN + (LN ? LnSmem<G::LANES, G::TS * G::TS>::BYTES : 0u);
};

struct NhwcTileArgs {
  const void* w;     // [C][49]
  const void* b;     // [C] or nullptr
  int N, C;
  int cgroups;       // ceil(C / 32)
  int tiles_x, tiles_y;
  int tiles;         // tiles_x * tiles_y
  int stages;        // cgroups * N * tiles (< 2^31, host check)
  FastDiv div_stage_cg;  // N * tiles: stage v -> channel group v / (N * tiles)
  FastDiv div_tiles;     // tiles
  FastDiv div_tx;        // tiles_x
  LnArgs ln;             // LN variant only
};

template <typename T, bool LN = false>
__global__ void __launch_bounds__(NhwcTileGeom::THREADS, sizeof(T) == 2 ? 2 : 1)
    nhwc_tile_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                     const NhwcTileArgs a) {
  using G = NhwcTileGeom;
  using M = NhwcTileSmem<T, LN>;
  constexpr bool MIX = sizeof(T) == 2;
  constexpr int TS = G::TS, SW = G::SW, LANES = G::LANES, R = G::R;
  extern __shared__ __align__(128) unsigned char smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + M::OFF_BAR);
  auto in_buf = [&](int s) { return reinterpret_cast<T*>(smem + M::OFF_IN + s * M::IN); };
  auto out_buf = [&](int s) { return reinterpret_cast<T*>(smem + M::OFF_OUT + s * M::OUT); };

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int rg = tid >> 5;  // output rows 2 rg, 2 rg + 1

  if (tid == 0) {
    prefetch_tensormap(&xmap);
    prefetch_tensormap(&ymap);
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Programmatic dependent launch (no-op without the launch attribute): the
  // set-up above overlaps the previous kernel's drain; every global access
  // below comes after that kernel completed.
  grid_dependency_wait();

  // Stage v -> (channel group, image, tile); channel-group-major order.
  auto decode = [&](int v, int& cg, int& n, int& tx, int& ty) {
    cg = fdiv(v, a.div_stage_cg);
    const int r = v - cg * (a.N * a.tiles);
    n = fdiv(r, a.div_tiles);
    const int t = r - n * a.tiles;
    ty = fdiv(t, a.div_tx);
    tx = t - ty * a.tiles_x;
  };
  constexpr uint32_t STAGE_BYTES = LANES * SW * SW * sizeof(T);
  auto issue = [&](int v, int s) {  // thread 0
    int cg, n, tx, ty;
    decode(v, cg, n, tx, ty);
    fence_proxy_async_smem();
    mbar_arrive_expect_tx(&bars[s], STAGE_BYTES);
    tma_load_4d(in_buf(s), &xmap, &bars[s], cg * LANES, tx * TS - kHalo, ty * TS - kHalo, n);
  };

  // LN: the cluster's balanced range of (image, tile) units, in this rank's
  // channel group (stage = channel group * N * tiles + unit); every rank of
  // a cluster runs the same number of stages.
  int v_begin, v_end;
  int rank = 0;
  if constexpr (LN) {
    rank = static_cast<int>(cluster_ctarank());
    const long long units = static_cast<long long>(a.N) * a.tiles;
    const long long cid = cluster_id_x(), ncl = nclusters_x();
    v_begin = static_cast<int>(rank * units + (units * cid) / ncl);
    v_end = static_cast<int>(rank * units + (units * (cid + 1)) / ncl);
  } else {
    v_begin = static_cast<int>((static_cast<long long>(a.stages) * blockIdx.x) / gridDim.x);
    v_end = static_cast<int>((static_cast<long long>(a.stages) * (blockIdx.x + 1)) / gridDim.x);
  }
  if (tid == 0 && v_begin < v_end) issue(v_begin, 0);

  const T* wbase = static_cast<const T*>(a.w);
  const T* bbase = static_cast<const T*>(a.b);
  float wt[kTaps];
  uint32_t wh[(kTaps + 1) / 2];
  int cur_cg = -1;
  float bias = 0.f;
  // LN: the CTA's scales and shifts (rank r always owns channel group r).
  if constexpr (LN) {
    const LnView<LANES, TS * TS> lv{reinterpret_cast<float*>(smem + M::OFF_LN)};
    ln_load_affine<T, LANES, TS * TS, G::THREADS>(lv, a.ln.gamma, a.ln.beta, rank * LANES, a.C);
  }
  int prev_n = 0, prev_tx = 0, prev_ty = 0;  // LN: the stage awaiting its store

  for (int v = v_begin, it = 0; v < v_end; ++v, ++it) {
    const int s = it & 1;
    if (tid == 0 && v + 1 < v_end) issue(v + 1, s ^ 1);  // in[s ^ 1] was released by the last barrier
    if (!LN && tid == 0 && v + 1 == v_end) launch_dependents();  // last load issued

    int cg, n, tx, ty;
    decode(v, cg, n, tx, ty);
    if (cg != cur_cg) {
      cur_cg = cg;
      const int c = cg * LANES + lane;
      const int cw = c < a.C ? c : 0;
      if constexpr (MIX) {
        load_taps16<kTaps>(wbase, cw, wh);
      } else {
#pragma unroll
        for (int t = 0; t < kTaps; ++t) wt[t] = to_acc(wbase[cw * kTaps + t]);
      }
      bias = bbase ? to_acc(bbase[cw]) : 0.f;
    }

    mbar_wait_bounded(&bars[s], (it >> 1) & 1);

    // ---- R output rows x TS columns of channel `lane` -------------------
    const T* src = in_buf(s);
    float acc[R][TS];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int o = 0; o < TS; ++o) acc[r][o] = 0.f;
#pragma unroll
    for (int ir = 0; ir < R + 6; ++ir) {
      const int iy = rg * R + ir;  // window row
      if constexpr (MIX) {
        const unsigned short* r16 = reinterpret_cast<const unsigned short*>(src) + iy * SW * LANES + lane;
        unsigned short xv[SW];
#pragma unroll
        for (int xx = 0; xx < SW; ++xx) xv[xx] = r16[xx * LANES];
#pragma unroll
        for (int kx = 0; kx < 7; ++kx) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = ir - r;
            if (ky < 0 || ky >= 7) continue;
            const int k = ky * 7 + kx;
            const unsigned short wv = half_of(wh[k >> 1], k & 1);
#pragma unroll
            for (int o = 0; o < TS; ++o) acc[r][o] = fma_mix(T(), xv[o + kx], wv, acc[r][o]);
          }
        }
      } else {
        const T* rr = src + iy * SW * LANES + lane;
        float xv[SW];
#pragma unroll
        for (int xx = 0; xx < SW; ++xx) xv[xx] = to_acc(rr[xx * LANES]);
#pragma unroll
        for (int kx = 0; kx < 7; ++kx) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = ir - r;
            if (ky < 0 || ky >= 7) continue;
            const float wv = wt[ky * 7 + kx];
#pragma unroll
            for (int o = 0; o < TS; ++o) acc[r][o] = fma_rn(xv[o + kx], wv, acc[r][o]);
          }
        }
      }
    }

    // ---- + bias, round, into out[s] [y][x][lane]; TMA store -------------
    T* os = out_buf(s);
    if constexpr (LN) {
      // out[s] was last read by the store of stage it - 2, which the LN flow
      // issues one iteration late; it is done before anyone writes out[s].
      if (tid == 0) bulk_wait_read_all();
      __syncthreads();
    }
    const bool has_bias = bbase != nullptr;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int oy = rg * R + r;
#pragma unroll
      for (int o = 0; o < TS; ++o) {
        float val = acc[r][o];
        if (has_bias) val += bias;
        os[(oy * TS + o) * LANES + lane] = from_acc<T>(val);
      }
    }
    if constexpr (LN) {
      // Deferred: finish stage it - 1 (its exchange ran behind this stage's
      // FMAs), then publish this stage's partials.
      const LnView<LANES, TS * TS> lv{reinterpret_cast<float*>(smem + M::OFF_LN)};
      if (it > 0) {
        cluster_wait();
        ln_combine<LANES, TS * TS, G::THREADS>(lv, (it - 1) & 1, a.C, a.ln.eps);
        __syncthreads();
        ln_normalize<T, LANES, TS * TS, G::THREADS>(out_buf(s ^ 1), lv, cg * LANES, a.C, a.ln.gamma != nullptr,
                                                    a.ln.beta != nullptr);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
          tma_store_4d(&ymap, out_buf(s ^ 1), cg * LANES, prev_tx * TS, prev_ty * TS, prev_n);
          bulk_commit();
        }
      } else {
        __syncthreads();
      }
      ln_local_stats<T, LANES, TS * TS, G::THREADS>(os, lv, it & 1, cg * LANES, a.C);
      cluster_arrive();
      prev_n = n;
      prev_tx = tx;
      prev_ty = ty;
      continue;
    }
    fence_proxy_async_smem();
    // The store that read out[s ^ 1] (issued one stage ago) is done before
    // the barrier releases the next stage's writes into it.
    if (tid == 0) bulk_wait_read_all();
    __syncthreads();
    if (tid == 0) {
      tma_store_4d(&ymap, os, cg * LANES, tx * TS, ty * TS, n);
      bulk_commit();
    }
  }
  if constexpr (LN) {
    if (v_end > v_begin) {  // the last stage's deferred exchange
      const LnView<LANES, TS * TS> lv{reinterpret_cast<float*>(smem + M::OFF_LN)};
      const int last = (v_end - v_begin - 1) & 1;
      cluster_wait();
      ln_combine<LANES, TS * TS, G::THREADS>(lv, last, a.C, a.ln.eps);
      __syncthreads();
      ln_normalize<T, LANES, TS * TS, G::THREADS>(out_buf(last), lv, rank * LANES, a.C, a.ln.gamma != nullptr,
                                                    a.ln.beta != nullptr);
      fence_proxy_async_smem();
      __syncthreads();
      if (tid == 0) {
        tma_store_4d(&ymap, out_buf(last), rank * LANES, prev_tx * TS, prev_ty * TS, prev_n);
        bulk_commit();
      }
    }
    cluster_sync();  // peers may still read this CTA's partial sums
  }
  if (tid == 0) bulk_wait_all();
}

}  // namespace pla
