// Plane-stack kernel: depthwise 7x7 on stacks of small square planes
// (S x S with S in {7, 14, 28}: the ConvNeXt-style shapes of
// data/depthwise_conv_7x7.py's benchmark configurations), NCHW or NHWC.
//
// Work unit ("stage"): LANES = 32 * G planes (NCHW: 32*G consecutive (n, c)
// planes, contiguous in memory) or LANES channels of one image (NHWC).  Lane
// l of lane group g owns plane / channel 32 g + l of the stage.
//
//  * Load: NCHW stages are one contiguous chunk -> one cp.async.bulk copy;
//    NHWC stages are one 4-D TMA box (LANES channels x S x S x 1 image).  Both
//    land raw in a 2-deep shared-memory ring guarded by mbarriers, issued one
//    stage ahead by thread 0 of a persistent CTA.
//  * fp32 stacks: the raw stage is first copied into an "x-quad" layout
//    F[y][x/4][lane][x%4], so that one 128-bit shared load gives a thread 4
//    consecutive columns of its own plane and a warp's load is 512 contiguous
//    bytes (bank-conflict free).
//  * 16-bit stacks skip that copy: each thread reads its plane's rows straight
//    from the raw stage (32-bit words of two columns for even-width NCHW
//    planes, 16-bit elements otherwise) into mixed-precision FMAs (16-bit x
//    and w, fp32 accumulator, identical bits), with the taps packed two per
//    register.  Half the registers and no second shared buffer give 3 CTAs
//    per SM instead of 2 at S = 14.
//  * Compute: a thread computes R output rows x S columns of its plane with
//    the 49 taps of its channel in registers.  Rows and columns that fall on
//    the zero padding are skipped (compile-time for columns, a warp-uniform
//    branch for rows): they would add an exact 0, so the fixed (ky, kx) tap
//    order and hence the bits of every output are unchanged, while 23% (S=14)
//    to 43% (S=7) of the FMAs of a padded formulation disappear.
//  * Store: + bias in fp32, one rounding, written in the source layout and
//    sent out with one bulk copy / TMA store.  fp32 stacks reuse the stage's
//    raw buffer (free once F holds it); 16-bit stacks, which read the raw
//    buffer while computing, write to a 2-buffer output ring instead, so one
//    barrier per stage suffices.
//  * LN (NHWC only): the stage's outputs go through the channel LayerNorm
//    epilogue of ln_epilogue.cuh before the store.  The kernel then runs as
//    clusters of C / LANES CTAs: rank r owns channel group r of the images
//    the cluster visits, so its filters never change.  16-bit stages, which
//    have the output ring, are normalised and stored one stage late, so the
//    cluster exchange overlaps the next stage's FMAs.
#pragma once

#include "ln_epilogue.cuh"
#include "pla_common.cuh"

namespace pla {

template <int S, bool MIX>
struct StackGeom {
  static_assert(S == 7 || S == 14 || S == 28, "plane side");
  static constexpr int R = (S == 7) ? 7 : 2;           // output rows per thread
  static constexpr int RG = (S + R - 1) / R;           // row groups per plane
  static constexpr int G = (S == 7) ? 4 : 1;           // lane groups per CTA
  static constexpr int WARPS = RG * G;
  static constexpr int THREADS = 32 * WARPS;
  static constexpr int LANES = 32 * G;                 // planes / channels per stage
  static constexpr int Q = (S + 3) / 4;                // x-quads per row
  static constexpr int F_FLOATS = S * Q * LANES * 4;   // expanded fp32 stage
  static constexpr int MIN_BLOCKS = (S == 7) ? 4 : (S == 14 ? (MIX ? 3 : 2) : 1);
};

// 16-bit stacks compute from the raw stage with mixed-precision FMAs.
template <typename T>
constexpr bool kMixStack = sizeof(T) == 2;

template <typename T, int S, bool LN = false>
struct StackSmem {
  using G = StackGeom<S, kMixStack<T>>;
  static constexpr uint32_t RAW = ((G::LANES * S * S * sizeof(T)) + 127u) & ~127u;
  static constexpr uint32_t F_BYTES = kMixStack<T> ? 0u : G::F_FLOATS * sizeof(float);
  static constexpr uint32_t OFF_F = 0;
  static constexpr uint32_t OFF_RAW = F_BYTES;
  // 16-bit stacks write outputs to their own 2-buffer ring (no in-place reuse).
  static constexpr uint32_t OFF_OUT = OFF_RAW + 2 * RAW;
  static constexpr uint32_t OFF_BAR = OFF_OUT + (kMixStack<T> ? 2 * RAW : 0u);
  static constexpr uint32_t OFF_LN = OFF_BAR + 2 * sizeof(uint64_t);
  static constexpr uint32_t OFF_TAPS = OFF_LN + (LN ? LnSmem<G::LANES, S * S>::BYTES : 0u);
  // 16-bit stacks whose warps share their lanes' filters (several row groups,
  // no LN): the stage's filters, packed 16-bit pairs, [25][LANES] words.
  static constexpr bool STAGE_TAPS = kMixStack<T> && G::RG > 1 && !LN;
  static constexpr uint32_t TOTAL = OFF_TAPS + (STAGE_TAPS ? ((kTaps + 1) / 2) * G::LANES * 4u : 0u);
};

struct StackArgs {
  const void* x;
  const void* w;   // [C][49]
  const void* b;   // [C] or nullptr
  void* y;
  int N, C;
  int stages;          // NCHW: ceil(N*C / LANES); NHWC: N * ceil(C / LANES)
  int cgroups;         // NHWC: ceil(C / LANES)
  long long planes;    // NCHW: N * C
  int full_stages;     // NCHW: stages whose chunk is complete (bulk-copy path)
  int cg_major;        // 1: visit stages channel-group-major (see stage_of)
  FastDiv div_c, div_cg, div_n;
  LnArgs ln;           // LN variant only
};

// CTAs own contiguous ranges of "virtual" stages.  With cg_major, virtual
// stage v is (channel group v / N, image v % N), so consecutive stages of a
// CTA reuse the same 32 (or 128) filters, which then stay in registers; the
// stage index k (the memory order) is n * cgroups + cg.  This needs every
// stage to hold whole channel groups: always true for NHWC, and for NCHW when
// C is a multiple of LANES.
__device__ __forceinline__ int stage_of(int v, const StackArgs& a) {
  if (!a.cg_major) return v;
  const int cg = fdiv(v, a.div_n);
  const int n = v - cg * a.N;
  return n * a.cgroups + cg;
}

// ---- bulk async copies (non-tensor) and 4-D tensor copies ------------------
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c, int x, int y,
                                            int n) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c), "r"(x), "r"(y), "r"(n)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c, int x, int y, int n) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c), "r"(x), "r"(y), "r"(n)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ float raw_to_f(float v) { return v; }
__device__ __forceinline__ float raw_to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float raw_to_f(__half v) { return __half2float(v); }

template <typename T, bool NHWC, int S, bool LN = false>
__global__ void __launch_bounds__(StackGeom<S, kMixStack<T>>::THREADS, StackGeom<S, kMixStack<T>>::MIN_BLOCKS)
    stack_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap ymap,
                 const StackArgs a) {
  static_assert(!LN || NHWC, "the LayerNorm epilogue normalises the channels of NHWC pixels");
  constexpr bool MIX = kMixStack<T>;
  using G = StackGeom<S, MIX>;
  using M = StackSmem<T, S, LN>;
  constexpr int R = G::R, Q = G::Q, LANES = G::LANES;
  extern __shared__ __align__(128) unsigned char smem[];
  float* F = reinterpret_cast<float*>(smem + M::OFF_F);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + M::OFF_BAR);
  auto raw = [&](int s) { return reinterpret_cast<T*>(smem + M::OFF_RAW + s * M::RAW); };
  auto outb = [&](int s) { return MIX ? reinterpret_cast<T*>(smem + M::OFF_OUT + s * M::RAW) : raw(s); };

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const int grp = warp / G::RG;        // lane group
  const int rg = warp % G::RG;         // row group
  const int ln = grp * 32 + lane;      // lane within the stage

  if (tid == 0) {
    if (NHWC) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&ymap);
    }
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  // Programmatic dependent launch (no-op without the launch attribute): the
  // set-up above overlaps the previous kernel's drain; every global access
  // below comes after that kernel completed.
  grid_dependency_wait();

  const T* x = static_cast<const T*>(a.x);
  T* y = static_cast<T*>(a.y);
  constexpr long long PLANE = static_cast<long long>(S) * S;
  constexpr uint32_t STAGE_BYTES = LANES * S * S * sizeof(T);

  // Issue the loads of stage k into raw buffer s (thread 0 only).
  auto issue = [&](int k, int s) {
    if (NHWC) {
      const int n = fdiv(k, a.div_cg);
      const int cg = k - n * a.cgroups;
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars[s], STAGE_BYTES);
      tma_load_4d(raw(s), &xmap, &bars[s], cg * LANES, 0, 0, n);
    } else if (k < a.full_stages) {
      fence_proxy_async_smem();
      mbar_arrive_expect_tx(&bars[s], STAGE_BYTES);
      bulk_load(raw(s), x + static_cast<long long>(k) * LANES * PLANE, STAGE_BYTES, &bars[s]);
    }
  };

  // Balanced contiguous range of virtual stages for this CTA.  LN: the
  // cluster's balanced range of images, in this rank's channel group
  // (virtual stage = channel group * N + image); every rank of a cluster
  // runs the same number of stages.
  int v_begin, v_end;
  int rank = 0;
  if constexpr (LN) {
    rank = static_cast<int>(cluster_ctarank());
    const long long cid = cluster_id_x(), ncl = nclusters_x();
    v_begin = rank * a.N + static_cast<int>((static_cast<long long>(a.N) * cid) / ncl);
    v_end = rank * a.N + static_cast<int>((static_cast<long long>(a.N) * (cid + 1)) / ncl);
  } else {
    v_begin = static_cast<int>((static_cast<long long>(a.stages) * blockIdx.x) / gridDim.x);
    v_end = static_cast<int>((static_cast<long long>(a.stages) * (blockIdx.x + 1)) / gridDim.x);
  }
  if (tid == 0 && v_begin < v_end) issue(stage_of(v_begin, a), 0);

  const T* wbase = static_cast<const T*>(a.w);
  const T* bbase = static_cast<const T*>(a.b);
  float wt[kTaps];
  uint32_t wh[(kTaps + 1) / 2];
  int cur_c = -1;
  int cur_key = -1;  // STAGE_TAPS: channel set whose filters are in registers
  float bias = 0.f;
  // LN: the CTA's scales and shifts (rank r always owns channel group r).
  if constexpr (LN) {
    const LnView<LANES, S * S> lv{reinterpret_cast<float*>(smem + M::OFF_LN)};
    ln_load_affine<T, LANES, S * S, G::THREADS>(lv, a.ln.gamma, a.ln.beta, rank * LANES, a.C);
  }
  int prev_img = 0;              // LN, 16-bit: image of the stage awaiting its store

  for (int v = v_begin, it = 0; v < v_end; ++v, ++it) {
    const int s = it & 1;
    const int k = stage_of(v, a);
    if (tid == 0 && v + 1 < v_end) {
      if (!MIX) bulk_wait_read_all();  // raw[s^1] carried the previous stage's output
      issue(stage_of(v + 1, a), s ^ 1);
    }
    if (!LN && tid == 0 && v + 1 == v_end) launch_dependents();  // last load issued

    // ---- this lane's channel and filter --------------------------------
    int c;
    bool lane_ok;
    long long plane = 0;
    int n_img = 0;
    if (NHWC) {
      n_img = fdiv(k, a.div_cg);
      const int cg = k - n_img * a.cgroups;
      c = cg * LANES + ln;
      lane_ok = c < a.C;
    } else {
      plane = static_cast<long long>(k) * LANES + ln;
      lane_ok = plane < a.planes;
      const int p = static_cast<int>(plane);  // planes < 2^31 (host check)
      c = p - fdiv(p, a.div_c) * a.C;
    }
    const int cw = lane_ok ? c : 0;
    if constexpr (M::STAGE_TAPS) {
      // Every row group (warp) of the CTA uses the same LANES filters, so
      // the CTA loads them once, cooperatively, into shared memory as packed
      // 16-bit pairs, and each thread takes its 25 words from there (instead
      // of every warp issuing 49 scattered 16-bit loads per lane).  The key
      // identifies the stage's channel set; it is the same on every thread.
      const bool part = !NHWC && k >= a.full_stages;
      const int key = NHWC ? (k - n_img * a.cgroups)
                           : (static_cast<int>(plane - ln) - fdiv(static_cast<int>(plane - ln), a.div_c) * a.C) +
                                 (part ? (1 << 30) : 0);
      if (key != cur_key) {
        cur_key = key;
        // The previous filters were read into registers before at least one
        // end-of-stage barrier, so the buffer is free to refill.
        uint32_t* ts = reinterpret_cast<uint32_t*>(smem + M::OFF_TAPS);
        const unsigned short* wb16 = reinterpret_cast<const unsigned short*>(wbase);
        for (int i = tid; i < ((kTaps + 1) / 2) * LANES; i += G::THREADS) {
          const int kk = i / LANES, l = i - kk * LANES;
          int cl;
          if (NHWC) {
            cl = (k - n_img * a.cgroups) * LANES + l;
            cl = cl < a.C ? cl : 0;
          } else {
            const long long pl = static_cast<long long>(k) * LANES + l;
            const int pi = static_cast<int>(pl);
            cl = pl < a.planes ? pi - fdiv(pi, a.div_c) * a.C : 0;
          }
          const unsigned short* wc = wb16 + cl * kTaps;
          ts[i] = static_cast<uint32_t>(wc[2 * kk]) |
                  (2 * kk + 1 < kTaps ? static_cast<uint32_t>(wc[2 * kk + 1]) << 16 : 0u);
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < (kTaps + 1) / 2; ++kk) wh[kk] = ts[kk * LANES + ln];
        bias = bbase ? to_acc(bbase[cw]) : 0.f;
        cur_c = cw;
      }
    } else if (cw != cur_c) {
      cur_c = cw;
      if constexpr (MIX) {
        load_taps16<kTaps>(wbase, cw, wh);
      } else {
#pragma unroll
        for (int t = 0; t < kTaps; ++t) wt[t] = to_acc(wbase[cw * kTaps + t]);
      }
      bias = bbase ? to_acc(bbase[cw]) : 0.f;
    }

    // ---- raw stage in shared memory ------------------------------------
    T* rs = raw(s);
    const bool partial = !NHWC && k >= a.full_stages;
    if (partial) {
      // Tail chunk that a bulk copy cannot move (fewer planes than LANES or a
      // size that is not a multiple of 16 bytes): plain loads, zero fill.
      const long long base = static_cast<long long>(k) * LANES * PLANE;
      const long long left = (a.planes - static_cast<long long>(k) * LANES) * PLANE;
      for (int i = tid; i < LANES * PLANE; i += G::THREADS) rs[i] = i < left ? x[base + i] : T(0.f);
      __syncthreads();
    } else {
      mbar_wait_bounded(&bars[s], (it >> 1) & 1);
    }

    // ---- fp32: widen / copy to the x-quad layout F[y][q][lane][4] --------------
    if constexpr (!MIX) {
      for (int i = tid; i < S * Q * LANES; i += G::THREADS) {
        const int l = i % LANES;
        const int yq = i / LANES;
        const int yy = yq / Q, q = yq % Q;
        float4 v;
        float* vv = reinterpret_cast<float*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int xx = 4 * q + j;
          float f = 0.f;
          if (xx < S) {
            const T e = NHWC ? rs[(yy * S + xx) * LANES + l] : rs[l * PLANE + yy * S + xx];
            f = raw_to_f(e);
          }
          vv[j] = f;
        }
        reinterpret_cast<float4*>(F)[i] = v;
      }
      __syncthreads();
    }

    // ---- R output rows x S columns of plane `ln` -----------------------------
    float acc[R][S];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int o = 0; o < S; ++o) acc[r][o] = 0.f;

    if constexpr (MIX) {
      const unsigned short* r16 = reinterpret_cast<const unsigned short*>(rs);
#pragma unroll
      for (int ir = 0; ir < R + 6; ++ir) {
        const int iy = rg * R + ir - kHalo;
        if (iy < 0 || iy >= S) continue;  // zero-padding row (warp-uniform)
        unsigned short xv[S];           // row iy of plane / channel ln
        if constexpr (NHWC) {
#pragma unroll
          for (int xx = 0; xx < S; ++xx) xv[xx] = r16[(iy * S + xx) * LANES + ln];
        } else if constexpr (S % 2 == 0) {
          const uint32_t* p = reinterpret_cast<const uint32_t*>(r16 + ln * PLANE + iy * S);
#pragma unroll
          for (int q2 = 0; q2 < S / 2; ++q2) {
            const uint32_t u = p[q2];
            xv[2 * q2] = half_of(u, 0);
            xv[2 * q2 + 1] = half_of(u, 1);
          }
        } else {  // odd-width rows are not word aligned
#pragma unroll
          for (int xx = 0; xx < S; ++xx) xv[xx] = r16[ln * PLANE + iy * S + xx];
        }
#pragma unroll
        for (int kx = 0; kx < 7; ++kx) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = ir - r;
            if (ky < 0 || ky >= 7) continue;
            const int k = ky * 7 + kx;
            const unsigned short wv = half_of(wh[k >> 1], k & 1);
#pragma unroll
            for (int o = 0; o < S; ++o) {
              const int ix = o + kx - kHalo;
              if (ix < 0 || ix >= S) continue;  // zero-padding column (compile time)
              acc[r][o] = fma_mix(T(), xv[ix], wv, acc[r][o]);
            }
          }
        }
      }
    } else {
      const float4* F4 = reinterpret_cast<const float4*>(F) + ln;
#pragma unroll
      for (int ir = 0; ir < R + 6; ++ir) {
        const int iy = rg * R + ir - kHalo;
        if (iy < 0 || iy >= S) continue;  // zero-padding row (warp-uniform)
        float v[4 * Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) {
          const float4 t = F4[(iy * Q + q) * LANES];
          v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
        }
#pragma unroll
        for (int kx = 0; kx < 7; ++kx) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int ky = ir - r;
            if (ky < 0 || ky >= 7) continue;
            const float wv = wt[ky * 7 + kx];
#pragma unroll
            for (int o = 0; o < S; ++o) {
              const int ix = o + kx - kHalo;
              if (ix < 0 || ix >= S) continue;  // zero-padding column (compile time)
              acc[r][o] = fma_rn(v[ix], wv, acc[r][o]);
            }
          }
        }
      }
    }

    // ---- + bias, round, stage the output (fp32: in raw[s], whose input is
    // consumed; 16-bit: in out[s], whose last bulk store has been read) ----
    T* os = outb(s);
    if constexpr (LN && MIX) {
      // out[s] was last read by the store of stage it - 2, which the LN flow
      // issues one iteration late; it is done before anyone writes out[s].
      if (tid == 0) bulk_wait_read_all();
      __syncthreads();
    }
    const bool has_bias = bbase != nullptr;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int oy = rg * R + r;
      if (oy >= S) continue;
#pragma unroll
      for (int o = 0; o < S; ++o) {
        float val = acc[r][o];
        if (has_bias) val += bias;
        const T e = from_acc<T>(val);
        if (NHWC)
          os[(oy * S + o) * LANES + ln] = e;
        else
          os[ln * PLANE + oy * S + o] = e;
      }
    }
    if constexpr (LN) {
      const LnView<LANES, S * S> lv{reinterpret_cast<float*>(smem + M::OFF_LN)};
      const int c0 = rank * LANES;
      if constexpr (MIX) {
        // Deferred: finish stage it - 1 (its exchange ran behind this
        // stage's FMAs), then publish this stage's partials.
        if (it > 0) {
          cluster_wait();
          ln_combine<LANES, S * S, G::THREADS>(lv, (it - 1) & 1, a.C, a.ln.eps);
          __syncthreads();
          ln_normalize<T, LANES, S * S, G::THREADS>(outb(s ^ 1), lv, c0, a.C, a.ln.gamma != nullptr,
                                                    a.ln.beta != nullptr);
          fence_proxy_async_smem();
          __syncthreads();
          if (tid == 0) {
            tma_store_4d(&ymap, outb(s ^ 1), rank * LANES, 0, 0, prev_img);
            bulk_commit();
          }
        } else {
          __syncthreads();
        }
        ln_local_stats<T, LANES, S * S, G::THREADS>(os, lv, it & 1, c0, a.C);
        cluster_arrive();
        prev_img = n_img;
        continue;
      } else {
        // fp32 stages are normalised in place (raw[s] is the next load's
        // target), so the exchange is not deferred.
        __syncthreads();
        ln_local_stats<T, LANES, S * S, G::THREADS>(os, lv, it & 1, c0, a.C);
        cluster_sync();
        ln_combine<LANES, S * S, G::THREADS>(lv, it & 1, a.C, a.ln.eps);
        __syncthreads();
        ln_normalize<T, LANES, S * S, G::THREADS>(os, lv, c0, a.C, a.ln.gamma != nullptr,
                                                    a.ln.beta != nullptr);
      }
    }
    fence_proxy_async_smem();
    // 16-bit: before this barrier releases the next stage's writes into
    // out[s ^ 1], the bulk store that read it (issued one stage ago) is done.
    if (MIX && tid == 0) bulk_wait_read_all();
    __syncthreads();

    if (partial) {
      const long long base = static_cast<long long>(k) * LANES * PLANE;
      const long long left = (a.planes - static_cast<long long>(k) * LANES) * PLANE;
      for (int i = tid; i < LANES * PLANE && i < left; i += G::THREADS) y[base + i] = os[i];
    } else if (tid == 0) {
      if (NHWC) {
        const int cg = k - n_img * a.cgroups;
        tma_store_4d(&ymap, os, cg * LANES, 0, 0, n_img);
      } else {
        bulk_store(y + static_cast<long long>(k) * LANES * PLANE, os, STAGE_BYTES);
      }
      bulk_commit();
    }
    (void)lane_ok;
  }
  if constexpr (LN) {
    if constexpr (MIX) {
      if (v_end > v_begin) {  // the last stage's deferred exchange
        const LnView<LANES, S * S> lv{reinterpret_cast<float*>(smem + M::OFF_LN)};
        const int last = (v_end - v_begin - 1) & 1;
        cluster_wait();
        ln_combine<LANES, S * S, G::THREADS>(lv, last, a.C, a.ln.eps);
        __syncthreads();
        ln_normalize<T, LANES, S * S, G::THREADS>(outb(last), lv, rank * LANES, a.C, a.ln.gamma != nullptr,
                                                    a.ln.beta != nullptr);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
          tma_store_4d(&ymap, outb(last), rank * LANES, 0, 0, prev_img);
          bulk_commit();
        }
      }
    }
    cluster_sync();  // peers may still read this CTA's partial sums
  }
  if (tid == 0) bulk_wait_all();
}

}  // namespace pla
