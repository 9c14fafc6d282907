// Fused-loss kernels with a column-streaming vertical pass (sm_100a).
//
// These are the kernels of the fused loss path (fssim_forward / fssim_backward): the
// forward writes the three SSIM partials and the deterministic reductions, the backward
// applies the transposed Gaussian to the partials. They share the work decomposition of
// the map kernels in ssim_kernels.cuh (64-column strips of the batch's planes, column runs
// of H output rows split over a persistent grid in equal amounts of work, TMA staging one
// step ahead), but the vertical pass is organised differently:
//
//   * one output column per thread: a CTA of 64 threads (2 warps) covers one strip;
//   * a step is 8 output rows; its horizontal pass writes its moment rows to a shared
//     buffer that holds only that step's rows;
//   * each thread keeps the last 2*HALO moment rows of its column in registers from one
//     step to the next (a sliding window), and reads each moment value from shared memory
//     exactly once; the vertical halo is never stored, copied or recomputed within a run
//     part;
//   * the first step of every run part ("preload") runs only the horizontal pass over the
//     2*HALO rows above the part's first output row, to fill the window.
//
// Per output pixel this reads 16 bytes of moments from shared memory in the forward (4
// maps) where a 4-row register tile reads 56, and it needs no halo-row copy between steps.
// Arithmetic is the map kernels' (and the reference's) tap for tap: the horizontal pass is
// the same code, and the vertical sum adds symmetric pairs (d = 1..HALO) then the centre,
// so per-pixel results are bitwise identical to the map kernels'; two maps are carried per
// packed FP32 pair ((mu_x, mu_y) and (E[x^2 + y^2], E[xy]) in the forward), which keeps the
// packed instructions without pairing adjacent columns, and the epilogue runs on pairs of
// output rows.
//
// Loop structure: an outer loop over the CTA's parts (one per column run it touches, with
// the part's constants computed once) and an inner loop over the part's steps. Staging is
// double-buffered in two slots of 8 rows: a regular step's rows are staged into the free
// slot while the previous step is processed; a preload (2*HALO rows, both slots) and the
// step after it are staged once the previous step's horizontal pass has finished.
#pragma once

#include "ssim_kernels.cuh"

namespace fssim {

constexpr int kSThreads = 64;                 // one thread per strip column
constexpr int kSWarps = kSThreads / 32;
constexpr int kSStep = 8;                     // output rows per step (and rows per TMA box)
static_assert(kSThreads == kStrip, "one output column per thread");

// Horizontal pass task mapping over a 64-column strip for 2 warps: rows in groups of 8
// (lane % 8) and chunks of 8 columns j = lane / 8 + 4 * warp, one task per thread per
// group. The 8 lanes of a quarter warp read the same chunk of 8 consecutive staged rows.
__device__ __forceinline__ int htask_row(int lane) { return lane & 7; }
__device__ __forceinline__ int htask_chunk(int warp, int lane) { return (lane >> 3) + 4 * warp; }

// Deterministic sum over the CTA of one double per thread (fixed shuffle tree, warps in
// order). red holds NW doubles.
template <int NW>
__device__ __forceinline__ double block_sum_w(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double s = red[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) s += red[w];
  return s;
}

// Start of CTA b's range of strip-rows for the streaming kernels: as cta_range_start, with a
// run part costing its rows plus 2*HALO + 4 rows for its preload (the preload's rows, its
// exposed staging wait and the part's set-up; 2*HALO alone, and 2*HALO + 8, balanced the
// grid slightly worse on a B200).
template <int HALO>
__device__ __forceinline__ int64_t scta_range_start(const Geometry& g, int64_t b, int64_t G) {
  const int64_t runs = g.LT / g.H;
  const int64_t per = g.H + 2 * HALO + 4;
  const int64_t A = (runs * per * b) / G;
  const int64_t r = A / per;
  const int64_t o = A - r * per;
  if (o >= g.H) return (r + 1) * g.H;
  return r * g.H + (o / kSStep) * kSStep;
}

// A CTA's part of one column run: plane (image img, channel chan), strip, output rows
// [t0, t1); rest = strip-rows of the CTA's range after this part.
struct SPart {
  int plane, img, chan, strip, t0, t1, rest;
  bool live;
};

__device__ __forceinline__ SPart sfirst_part(int64_t beg, int64_t end, const Geometry& g) {
  SPart p;
  const int64_t len = end - beg;
  p.live = len > 0;
  if (!p.live) return p;
  const int64_t col = beg / g.H;
  p.t0 = static_cast<int>(beg - col * g.H);
  const int64_t plane = col / g.S;
  p.plane = static_cast<int>(plane);
  p.strip = static_cast<int>(col - plane * g.S);
  p.img = p.plane / g.C;
  p.chan = p.plane - p.img * g.C;
  const int64_t seg = (g.H - p.t0) < len ? (g.H - p.t0) : len;
  p.t1 = p.t0 + static_cast<int>(seg);
  p.rest = static_cast<int>(len - seg);
  return p;
}

// L2 prefetch of the TMA boxes of a part's preload (rows [t0 - HALO, t0 + HALO)), issued
// before the wait for the previous kernel: thread m * 2 + b (m < NMAP, b < 2) prefetches
// box b of map m. A hint: rows are clamped to the image.
template <int HALO, int NMAP>
__device__ __forceinline__ void prefetch_preload(const CUtensorMap* maps, const SPart& p,
                                                 const Geometry& g) {
  const int i = threadIdx.x;
  if (!p.live || i >= 2 * NMAP) return;
  const int y = p.t0 - HALO + (i & 1) * kSStep;
  tma_prefetch_3d(maps + (i >> 1), max(p.strip * kStrip - kLeft, 0),
                  min(max(y, 0), static_cast<int>(g.H) - 1), p.plane);
}

__device__ __forceinline__ SPart snext_part(const SPart& c, const Geometry& g) {
  SPart p = c;
  if (!c.live || c.rest == 0) {
    p.live = false;
    return p;
  }
  if (++p.strip == g.S) {
    p.strip = 0;
    ++p.plane;
    if (++p.chan == g.C) {
      p.chan = 0;
      ++p.img;
    }
  }
  const int H = static_cast<int>(g.H);
  p.t0 = 0;
  p.t1 = c.rest < H ? c.rest : H;
  p.rest = c.rest - p.t1;
  return p;
}

// Rows [h0, h0 + nh) (nh <= 2 * kSStep) of one strip of one plane, into staging slot `slot`.
struct SStage {
  int plane, strip, h0, nh, slot;
};

// Bytes the TMA staging of nh rows delivers for NMAP maps of element type T (boxes of
// kSStep rows).
template <typename T, int NMAP>
__device__ __forceinline__ unsigned sstep_bytes(int nh) {
  const int nbox = (nh + kSStep - 1) / kSStep;
  return static_cast<unsigned>(NMAP * nbox * kSStep * StagePitch<T>::value * sizeof(T));
}

// TMA staging of step st by the lanes of warp 0: lane m * nbox + b copies box b (kSStep rows)
// of map m into rows [slot + b * kSStep, ...) of the layout [NMAP][2 * kSStep][pitch].
template <typename T, int NMAP>
__device__ __forceinline__ void sstage_tma(T* stg, const CUtensorMap* maps, const SStage& st,
                                           uint64_t* bar) {
  constexpr int P = StagePitch<T>::value;
  constexpr int SROWS = 2 * kSStep;
  const int lane = threadIdx.x & 31;
  const int nbox = (st.nh + kSStep - 1) / kSStep;
  if (lane == 0) mbar_arrive_expect_tx(bar, sstep_bytes<T, NMAP>(st.nh));
  if (lane < NMAP * nbox) {
    const int m = lane / nbox;
    const int b = lane - m * nbox;
    fence_proxy_async_smem();
    tma_load_3d(stg + (m * SROWS + st.slot + b * kSStep) * P, maps + m,
                st.strip * kStrip - kLeft, st.h0 + b * kSStep, st.plane, bar);
  }
}

// Horizontal pass of the streaming forward over staged rows [0, nh) of one slot, into moment
// rows [0, nh) of `ring` (maps at column offsets 0: X, 64: X^2+Y^2, 128: Y, 192: XY). The
// arithmetic is fwd_hpass's (merged second moment). L1: |x - y| of the centre pixels of
// staged rows [l1_i0, l1_i1) in the strip's first l1_cols columns.
template <int HALO, typename TIn>
__device__ __forceinline__ void sfwd_hpass(const TIn* sx, const TIn* sy, float* ring, int nh,
                                           const Taps2<HALO, HalfTaps<TIn>::value>& T, bool l1,
                                           int l1_i0, int l1_i1, int l1_cols, float& l1_sum) {
  constexpr int SP = StagePitch<TIn>::value;
  constexpr int RP = RingPitch<4>::value;
  constexpr int HA = (sizeof(TIn) == 2 || HALO > 4) ? 8 : 4;  // aligned left extent
  constexpr int NV = 8 + 2 * HA;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = htask_chunk(warp, lane);
#pragma unroll 1
  for (int rg = 0; rg < nh; rg += kSStep) {
    const int i = rg + htask_row(lane);
    if (i < nh) {
      {
        float xv[NV], yv[NV];
        load_vec(sx + i * SP + 8 * j + kLeft - HA, xv);
        load_vec(sy + i * SP + 8 * j + kLeft - HA, yv);
        PairRow<NV> X, Y, XX, S, XY;
        X.build(xv);
        Y.build(yv);
#pragma unroll
        for (int q = 0; q < NV / 2; ++q) {
          XX.a[q] = mul2(X.a[q], X.a[q]);
          XY.a[q] = mul2(X.a[q], Y.a[q]);
          S.a[q] = fma2(Y.a[q], Y.a[q], XX.a[q]);
        }
        if (l1 && i >= l1_i0 && i < l1_i1) {
          const int nc = l1_cols - 8 * j;  // centre columns of the task inside the image
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 dv = sub2(X.pr(HA + 2 * q), Y.pr(HA + 2 * q));
            l1_sum += (2 * q < nc ? fabsf(dv.x) : 0.f) + (2 * q + 1 < nc ? fabsf(dv.y) : 0.f);
          }
        }
        float* dst = ring + i * RP + 8 * j;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int c = HA + 2 * p;  // first column of the output pair (even)
          const float2 wc = T.w[HALO];
          float2 sX = make_float2(0.f, 0.f), sY = sX, sXY = sX, sS = sX;
#pragma unroll
          for (int d = 1; d <= HALO; ++d) {
            const float2 w = T.w[HALO - d];
            sX = fma2(psum(X, c, d), w, sX);
            sY = fma2(psum(Y, c, d), w, sY);
            sXY = fma2(pfma(X, Y, XY, c, d), w, sXY);
            sS = fma2(psum(S, c, d), w, sS);
          }
          *reinterpret_cast<float2*>(dst + 0 * kStrip + 2 * p) = fma2(X.pr(c), wc, sX);
          *reinterpret_cast<float2*>(dst + 1 * kStrip + 2 * p) = fma2(S.pr(c), wc, sS);
          *reinterpret_cast<float2*>(dst + 2 * kStrip + 2 * p) = fma2(Y.pr(c), wc, sY);
          *reinterpret_cast<float2*>(dst + 3 * kStrip + 2 * p) = fma2(XY.pr(c), wc, sXY);
        }
      }
    }
  }
}

// Vertical 2*HALO+1 tap sum of output row k from window rows k..k+2*HALO (reference order:
// pairs d = 1..HALO, centre last). `row(j)` returns window row j.
template <int HALO, bool HW_, typename RowF>
__device__ __forceinline__ float2 svsum(const Taps2<HALO, HW_>& T, int k, RowF row) {
  float2 acc = make_float2(0.f, 0.f);
#pragma unroll
  for (int d = 1; d <= HALO; ++d) acc = fma2(add2(row(k + HALO - d), row(k + HALO + d)), T.w[HALO - d], acc);
  return fma2(row(k + HALO), T.w[HALO], acc);
}

template <int HALO, bool HW_, typename RowF>
__device__ __forceinline__ float svsum1(const Taps2<HALO, HW_>& T, int k, RowF row) {
  float acc = 0.f;
#pragma unroll
  for (int d = 1; d <= HALO; ++d)
    acc = __fmaf_rn(__fadd_rn(row(k + HALO - d), row(k + HALO + d)), T.w[HALO - d].x, acc);
  return __fmaf_rn(row(k + HALO), T.w[HALO].x, acc);
}

// SSIM value and its three partials of two pixels from their four filtered moments (MERGED
// form), each operand a pair of pixels (packed FP32, identical to the map kernels'
// epilogue).
struct PixelOut2 {
  float2 v, pm, ps, pc;
};
template <bool TRAIN>
__device__ __forceinline__ PixelOut2 ssim_pixel2(float2 mu1, float2 mu2, float2 S, float2 XY,
                                                 float2 C1v, float2 C2v) {
  const float2 neg1 = splat(-1.f), two = splat(2.f);
  const float2 mu1_sq = mul2(mu1, mu1), mu2_sq = mul2(mu2, mu2);
  const float2 msq = add2(mu1_sq, mu2_sq);
  const float2 mu12 = mul2(mu1, mu2);
  const float2 A = add2(msq, C1v);
  const float2 B = add2(fma2(msq, neg1, S), C2v);
  const float2 sigma12 = fma2(mu12, neg1, XY);
  const float2 Cc = fma2(two, mu12, C1v);
  const float2 D = fma2(two, sigma12, C2v);
  const float2 rA = make_float2(rcp_approx(A.x), rcp_approx(A.y));
  const float2 rB = make_float2(rcp_approx(B.x), rcp_approx(B.y));
  const float2 rAB = mul2(rA, rB);
  PixelOut2 o;
  o.v = mul2(mul2(Cc, D), rAB);
  if (TRAIN) {
    o.pm = fma2(mul2(two, mu2), mul2(fma2(Cc, neg1, D), rAB),
                mul2(mul2(two, mu1), mul2(o.v, fma2(rA, neg1, rB))));
    o.ps = mul2(mul2(o.v, neg1), rB);
    o.pc = mul2(mul2(two, Cc), rAB);
  }
  return o;
}

template <typename TP>
__device__ __forceinline__ void store1(TP* p, float v) {
  if constexpr (sizeof(TP) == 4) {
    *p = v;
  } else if constexpr (HalfTaps<TP>::value) {
    *p = __float2half_rn(v);
  } else {
    *p = __float2bfloat16_rn(v);
  }
}

// Last CTA of a reducing forward: turn the per-image fixed-point accumulators into the
// outputs (NaN for every output of a call in which a CTA gave up), zero them again and, for
// a sharded loss, publish the batch sum. Called by every thread of the CTA after its steps.
template <int NT>
__device__ __forceinline__ void finish_reduction(const FwdParams& a, bool failed, double* red,
                                                 unsigned* s_last) {
  const bool l1 = a.l1 != 0;
  __syncthreads();
  if (threadIdx.x == 0) {
    // One atomic per CTA on the ticket word: finished CTAs counted in its low 16 bits,
    // CTAs that gave up in its high 16 bits (grids stay below 2^16 CTAs, checked on the
    // host). Its release half orders this CTA's accumulator atomics before the count; its
    // acquire half, in the last CTA, orders every counted CTA's before what follows. The
    // last CTA leaves the word zero for the next call (the "failed" word after it is not
    // used by these kernels and stays zero).
    const unsigned add = failed ? 0x10001u : 1u;
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;\n"
                 : "=r"(prev)
                 : "l"(a.ticket), "r"(add)
                 : "memory");
    const bool last = (prev & 0xffffu) == gridDim.x - 1;
    if (last) *a.ticket = 0u;
    *s_last = !last ? 0u : ((prev >> 16) != 0u || failed) ? 2u : 1u;
  }
  __syncthreads();
  if (!*s_last) return;
  __threadfence();
  const double poison = *s_last == 2u ? __longlong_as_double(0x7ff8000000000000ll) : 0.0;
  double local = 0.0, local_l1 = 0.0;
  for (int b = threadIdx.x; b < a.g.B; b += NT) {
    const long long q = static_cast<long long>(atomicExch(a.acc + b, 0ull));
    const double s = static_cast<double>(q) * (1.0 / kFixScale) + poison;
    double s1 = 0.0;
    if (l1) s1 = static_cast<double>(static_cast<long long>(atomicExch(a.acc_l1 + b, 0ull))) *
                 (1.0 / kFixScaleL1);
    if (a.image_sums) a.image_sums[b] = s;
    if (a.reduce == 2)
      a.out[b] = static_cast<float>(s * static_cast<double>(a.out_scale) +
                                    s1 * static_cast<double>(a.l1_weight) +
                                    static_cast<double>(a.out_offset));
    local += s;
    local_l1 += s1;
  }
  if (a.reduce == 1) {
    const double total = block_sum_w<NT / 32>(local, red);
    const double total_l1 = block_sum_w<NT / 32>(local_l1, red);
    if (threadIdx.x == 0) {
      a.out[0] = static_cast<float>(total * static_cast<double>(a.out_scale) +
                                    total_l1 * static_cast<double>(a.l1_weight) +
                                    static_cast<double>(a.out_offset));
      if (a.dp.world > 0) dp_publish(a.dp, total);
    }
  }
}

template <int HALO, typename TIn, typename TP, bool TRAIN>
struct SFwdConfig {
  static constexpr bool kHalfW = HalfTaps<TIn>::value;
  static constexpr int kSP = StagePitch<TIn>::value;
  static constexpr int kRP = RingPitch<4>::value;
  static constexpr int kRingRows = 2 * HALO > kSStep ? 2 * HALO : kSStep;
  static_assert(2 * HALO <= 2 * kSStep, "a preload fits the two staging slots");
  static constexpr size_t kStageBytes = 2ull * (2 * kSStep) * kSP * sizeof(TIn);  // 2 maps
  static constexpr size_t kRingBytes = static_cast<size_t>(kRingRows) * kRP * sizeof(float);
  static constexpr size_t kSmem = kStageBytes + kRingBytes + 128;
  static constexpr int kFit = static_cast<int>((228 * 1024) / (kSmem + 1024));
  // Launch bound of 5 CTAs/SM (a register target of 204): every instantiation compiles to
  // at most 168 registers, so 6 CTAs/SM still fit (shared memory allows more), and on a
  // B200 this code ran 2-3 % faster than the same kernels built for a bound of 6 (also 168
  // registers). 7 or 8 CTAs/SM (144 or 128 registers) spill and ran slower; 4 (232
  // registers) ran slower too.
  static constexpr int kMinBlocks = kFit >= 5 ? 5 : kFit;
};

template <int HALO, typename TIn, typename TP, bool TRAIN>
__global__ void __launch_bounds__(kSThreads, (SFwdConfig<HALO, TIn, TP, TRAIN>::kMinBlocks))
    loss_fwd_kernel(const __grid_constant__ FwdParams a) {
  using Cfg = SFwdConfig<HALO, TIn, TP, TRAIN>;
  constexpr int SP = Cfg::kSP;
  constexpr int RP = Cfg::kRP;
  constexpr int SROWS = 2 * kSStep;
  constexpr bool HW_ = Cfg::kHalfW;
  constexpr int W2 = 2 * HALO;  // window rows carried between steps
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
  TIn* stg = reinterpret_cast<TIn*>(smem);
  float* ring = reinterpret_cast<float*>(smem + Cfg::kStageBytes);
  __shared__ double red[kSWarps];
  __shared__ unsigned s_last;
  __shared__ uint64_t bar;

  const Geometry& g = a.g;
  const int64_t beg = scta_range_start<HALO>(g, blockIdx.x, gridDim.x);
  const int64_t end = scta_range_start<HALO>(g, blockIdx.x + 1, gridDim.x);
  const TIn* const src[2] = {static_cast<const TIn*>(a.img1), static_cast<const TIn*>(a.img2)};
  const int warp = threadIdx.x >> 5;
  const int c = threadIdx.x;  // this thread's column in the strip
  Taps2<HALO, HW_> T;
  T.load();

  const bool tma = a.use_tma != 0;
  if (tma && threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  SPart part = sfirst_part(beg, end, g);
  if (tma && threadIdx.x < 2) prefetch_tensormap(a.tmap + threadIdx.x);
  // the first preload's boxes into L2 while the previous kernel finishes (not in the FP32
  // 11-tap forward: there the extra code made ptxas spill 12 bytes in the step loop, which
  // cost 3 % on large batches, more than the prefetch saves at 1080p)
  if constexpr (!(sizeof(TIn) == 4 && HALO == 5)) {
    if (tma) prefetch_preload<HALO, 2>(a.tmap, part, g);
  }
  grid_dependency_wait();
  grid_launch_dependents();
  // staging of rows: TMA boxes issued by warp 0, or cp.async by the whole CTA
  auto stage_rows = [&](const SStage& st) {
    if (tma) {
      if (warp == 0) sstage_tma<TIn, 2>(stg, a.tmap, st, &bar);
    } else {
      Step<HALO> s{};
      s.plane = st.plane;
      s.strip = st.strip;
      s.first = false;
      s.t = st.h0 - HALO;  // Step::h0() = t + HALO for a non-first step
      s.n = st.nh;
      stage<TIn, 2, SROWS, Step<HALO>, kSThreads>(stg + st.slot * SP, src, g, s, a.aligned16);
    }
  };
  unsigned phase = 0;
  // wait for the staging in flight; false (the CTA stops) if the copy did not arrive
  auto wait_staged = [&]() -> bool {
    bool timed_out = false;
    if (tma) {
      timed_out = !mbar_wait_bounded(&bar, phase, a.wait_limit);
      phase ^= 1u;
    } else {
      cp_async_wait_all();
    }
    if (__syncthreads_or(timed_out)) {
      if (threadIdx.x == 0) atomicOr(&g_device_error, kErrStagingTimeout);
      mbar_wait_bounded(&bar, phase ^ 1u, kWaitLimit);
      return false;
    }
    return true;
  };
  if (part.live) stage_rows({part.plane, part.strip, part.t0 - HALO, W2, 0});
  const bool l1 = a.l1 != 0;
  bool failed = false;
  const int W = static_cast<int>(g.W);
  const int H = static_cast<int>(g.H);
  const float2 C1v = splat(a.C1), C2v = splat(a.C2);
  const float* col = ring + c;

  while (part.live) {
    SPart nextp;  // set at the part's last step
    // ---- constants of the part ----
    const int sx0 = part.strip * kStrip;
    const int gx = sx0 + c;
    const bool in_x = gx < W;
    const bool col_ok = in_x && (!a.valid || (gx >= HALO && gx < W - HALO));
    const bool strip_fast = !a.clamp && sx0 + kStrip <= W &&
                            (!a.valid || (sx0 >= HALO && sx0 + kStrip <= W - HALO));
    // this thread's pixel of the part's first row, as an offset into the (B, C, H, W) outputs;
    // the output pointers are formed at the stores, which keeps them out of the registers
    // the step loop carries
    const int64_t pix = static_cast<int64_t>(part.plane) * g.HW + gx;
    const int l1_cols = W - sx0;
    double run_sum = 0.0, run_l1 = 0.0;

    // ---- preload: moment rows [t0 - HALO, t0 + HALO) fill the window ----
    if (!wait_staged()) {
      failed = true;
      break;
    }
    {
      float l1s = 0.f;
      sfwd_hpass<HALO, TIn>(stg, stg + SROWS * SP, ring, W2, T, l1, HALO,
                            part.t1 - part.t0 + HALO, l1_cols, l1s);
      run_l1 += static_cast<double>(l1s);
    }
    __syncthreads();
    // the first regular step's rows fill slot 0 (the preload used both slots)
    stage_rows({part.plane, part.strip, part.t0 + HALO, min(kSStep, part.t1 - part.t0), 0});
    float2 wP[W2], wQ[W2];  // the column's last 2*HALO moment rows: (X, Y), (X^2+Y^2, XY)
#pragma unroll
    for (int j = 0; j < W2; ++j) {
      wP[j] = make_float2(col[j * RP + 0 * kStrip], col[j * RP + 2 * kStrip]);
      wQ[j] = make_float2(col[j * RP + 1 * kStrip], col[j * RP + 3 * kStrip]);
    }
    // (no barrier here: the step's staging wait is a barrier of the whole CTA, and it comes
    // before the next horizontal pass overwrites the moment rows just read)

    // ---- regular steps: output rows [t, t + n) ----
    int slot = 0;
    for (int t = part.t0; t < part.t1; t += kSStep) {
      const int n = min(kSStep, part.t1 - t);
      const bool last = t + kSStep >= part.t1;
      if (!wait_staged()) {
        failed = true;
        break;
      }
      if (!last) stage_rows({part.plane, part.strip, t + kSStep + HALO,
                             min(kSStep, part.t1 - t - kSStep), slot ^ kSStep});
      {
        float l1s = 0.f;
        sfwd_hpass<HALO, TIn>(stg + slot * SP, stg + (SROWS + slot) * SP, ring, n, T, l1, 0,
                              part.t1 - t - HALO, l1_cols, l1s);
        run_l1 += static_cast<double>(l1s);
      }
      __syncthreads();
      // the next part's preload fills both slots once this step's rows are consumed
      if (last) {
        nextp = snext_part(part, g);
        if (nextp.live) stage_rows({nextp.plane, nextp.strip, nextp.t0 - HALO, W2, 0});
      }

      float2 nP[kSStep], nQ[kSStep];
      const int off0 = t * W;  // 32-bit in-plane row offset (planes < 2^31 elements)
      float step_sum = 0.f;
      if (n == kSStep && strip_fast && (!a.valid || (t >= HALO && t + kSStep <= H - HALO))) {
#pragma unroll
        for (int r = 0; r < kSStep; ++r) {
          nP[r] = make_float2(col[r * RP + 0 * kStrip], col[r * RP + 2 * kStrip]);
          nQ[r] = make_float2(col[r * RP + 1 * kStrip], col[r * RP + 3 * kStrip]);
        }
        auto rowP = [&](int j) { return j < W2 ? wP[j] : nP[j - W2]; };
        auto rowQ = [&](int j) { return j < W2 ? wQ[j] : nQ[j - W2]; };
        // two output rows at a time: the epilogue runs on (row k, row k+1) pairs
#pragma unroll
        for (int k = 0; k < kSStep; k += 2) {
          const float2 P0 = svsum<HALO, HW_>(T, k, rowP), P1 = svsum<HALO, HW_>(T, k + 1, rowP);
          const float2 Q0 = svsum<HALO, HW_>(T, k, rowQ), Q1 = svsum<HALO, HW_>(T, k + 1, rowQ);
          const PixelOut2 o = ssim_pixel2<TRAIN>(make_float2(P0.x, P1.x), make_float2(P0.y, P1.y),
                                                 make_float2(Q0.x, Q1.x), make_float2(Q0.y, Q1.y),
                                                 C1v, C2v);
          if (a.reduce) step_sum += o.v.x + o.v.y;
          const int64_t off = pix + off0 + k * W;
          if (a.map) {
            a.map[off] = o.v.x;
            a.map[off + W] = o.v.y;
          }
          if (TRAIN) {
            store1(static_cast<TP*>(a.p0) + off, o.pm.x);
            store1(static_cast<TP*>(a.p0) + off + W, o.pm.y);
            store1(static_cast<TP*>(a.p1) + off, o.ps.x);
            store1(static_cast<TP*>(a.p1) + off + W, o.ps.y);
            store1(static_cast<TP*>(a.p2) + off, o.pc.x);
            store1(static_cast<TP*>(a.p2) + off + W, o.pc.y);
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < kSStep; ++r) {
          if (r < n) {
            nP[r] = make_float2(col[r * RP + 0 * kStrip], col[r * RP + 2 * kStrip]);
            nQ[r] = make_float2(col[r * RP + 1 * kStrip], col[r * RP + 3 * kStrip]);
          } else {
            nP[r] = nQ[r] = make_float2(0.f, 0.f);
          }
        }
        auto rowP = [&](int j) { return j < W2 ? wP[j] : nP[j - W2]; };
        auto rowQ = [&](int j) { return j < W2 ? wQ[j] : nQ[j - W2]; };
        int rlo = 0, rhi = n;
        if (a.valid) {
          rlo = max(0, HALO - t);
          rhi = min(n, H - HALO - t);
        }
        // masked outputs, also two rows at a time; a row at or past n is computed from zero
        // window rows and neither summed nor stored
        auto masked = [&](float v, float pm, float ps, float pc, int k) {
          const bool ok = col_ok && k >= rlo && k < rhi;
          float contrib = 0.f;
          if (a.reduce) contrib = ok ? ((a.clamp && v < 0.f) ? 0.f : v) : 0.f;
          if (in_x && k < n) {
            const int64_t off = pix + off0 + k * W;
            if (a.map) a.map[off] = v;
            if (TRAIN) {
              const bool live = !a.mask_partials || (ok && (!a.clamp || v >= 0.f));
              if (!live) pm = ps = pc = 0.f;
              store1(static_cast<TP*>(a.p0) + off, pm);
              store1(static_cast<TP*>(a.p1) + off, ps);
              store1(static_cast<TP*>(a.p2) + off, pc);
            }
          }
          return contrib;
        };
#pragma unroll
        for (int k = 0; k < kSStep; k += 2) {
          if (k < n) {
            const float2 P0 = svsum<HALO, HW_>(T, k, rowP), P1 = svsum<HALO, HW_>(T, k + 1, rowP);
            const float2 Q0 = svsum<HALO, HW_>(T, k, rowQ), Q1 = svsum<HALO, HW_>(T, k + 1, rowQ);
            const PixelOut2 o = ssim_pixel2<TRAIN>(make_float2(P0.x, P1.x), make_float2(P0.y, P1.y),
                                                   make_float2(Q0.x, Q1.x), make_float2(Q0.y, Q1.y),
                                                   C1v, C2v);
            const float c0 = masked(o.v.x, o.pm.x, o.ps.x, o.pc.x, k);
            const float c1 = masked(o.v.y, o.pm.y, o.ps.y, o.pc.y, k + 1);
            step_sum += c0 + c1;
          }
        }
      }
      run_sum += static_cast<double>(step_sum);
      // carry the window: the last 2*HALO rows of window and step (after a partial step,
      // the last of its part, the next part preloads a new window)
      {
        float2 cP[W2], cQ[W2];
#pragma unroll
        for (int j = 0; j < W2; ++j) {
          cP[j] = j + kSStep < W2 ? wP[j + kSStep] : nP[j + kSStep - W2];
          cQ[j] = j + kSStep < W2 ? wQ[j + kSStep] : nQ[j + kSStep - W2];
        }
#pragma unroll
        for (int j = 0; j < W2; ++j) {
          wP[j] = cP[j];
          wQ[j] = cQ[j];
        }
      }
      if (a.reduce && last) {
        // end of the part: fold its sums into the image's fixed-point accumulators
        const double s_ = block_sum_w<kSWarps>(run_sum, red);
        const double s1 = l1 ? block_sum_w<kSWarps>(run_l1, red) : 0.0;
        if (threadIdx.x == 0) {
          atomicAdd(a.acc + part.img,
                    static_cast<unsigned long long>(__double2ll_rn(s_ * kFixScale)));
          if (l1)
            atomicAdd(a.acc_l1 + part.img,
                      static_cast<unsigned long long>(__double2ll_rn(s1 * kFixScaleL1)));
        }
      }
      // the moment rows of this step were read into registers before the epilogue; the next
      // step's staging wait (a CTA barrier) orders those reads before its horizontal pass
      slot ^= kSStep;
    }
    if (failed) break;
    part = nextp;
  }

  if (!a.reduce) return;
  finish_reduction<kSThreads>(a, failed, red, &s_last);
}

// ---------------------------------------------------------------------------------------
// Streaming backward: transposed Gaussian of the three partial maps, one column per thread
// ---------------------------------------------------------------------------------------
template <int HALO, typename TIn, typename TP>
struct SBwdConfig {
  static constexpr bool kHalfW = HalfTaps<TIn>::value;
  static constexpr int kSP = StagePitch<TP>::value;
  static constexpr int kRP = RingPitch<3>::value;
  static constexpr int kRingRows = 2 * HALO > kSStep ? 2 * HALO : kSStep;
  static constexpr size_t kStageBytes = 3ull * (2 * kSStep) * kSP * sizeof(TP);  // 3 maps
  static constexpr size_t kRingBytes = static_cast<size_t>(kRingRows) * kRP * sizeof(float);
  static constexpr size_t kSmem = kStageBytes + kRingBytes + 128;
  static constexpr int kFit = static_cast<int>((228 * 1024) / (kSmem + 1024));
  static constexpr int kMinBlocks = kFit >= 8 ? 8 : kFit;
};

// Horizontal pass of the streaming backward: the three staged partial maps, rows [0, nh).
template <int HALO, typename TIn, typename TP>
__device__ __forceinline__ void sbwd_hpass(const TP* sp, float* ring, int nh,
                                           const Taps2<HALO, HalfTaps<TIn>::value>& T) {
  constexpr int SP = StagePitch<TP>::value;
  constexpr int RP = RingPitch<3>::value;
  constexpr int SROWS = 2 * kSStep;
  constexpr int HA = (sizeof(TP) == 2 || HALO > 4) ? 8 : 4;
  constexpr int NV = 8 + 2 * HA;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = htask_chunk(warp, lane);
#pragma unroll 1
  for (int rg = 0; rg < nh; rg += kSStep) {
    const int i = rg + htask_row(lane);
    if (i < nh) {
      {
        float* dst = ring + i * RP + 8 * j;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          float v[NV];
          load_vec(sp + (m * SROWS + i) * SP + 8 * j + kLeft - HA, v);
          PairRow<NV> V;
          V.build(v);
          float2 s4[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) s4[p] = make_float2(0.f, 0.f);
#pragma unroll
          for (int d = 1; d <= HALO; ++d) {
#pragma unroll
            for (int p = 0; p < 4; ++p) s4[p] = fma2(psum(V, HA + 2 * p, d), T.w[HALO - d], s4[p]);
          }
#pragma unroll
          for (int p = 0; p < 4; ++p)
            *reinterpret_cast<float2*>(dst + m * kStrip + 2 * p) =
                fma2(V.pr(HA + 2 * p), T.w[HALO], s4[p]);
        }
      }
    }
  }
}

template <typename T>
__device__ __forceinline__ float ldg1(const T* p) {
  if constexpr (sizeof(T) == 4) {
    return __ldg(p);
  } else {
    return to_f(*p);
  }
}

template <int HALO, typename TIn, typename TP>
__global__ void __launch_bounds__(kSThreads, (SBwdConfig<HALO, TIn, TP>::kMinBlocks))
    loss_bwd_kernel(const __grid_constant__ BwdParams a) {
  using Cfg = SBwdConfig<HALO, TIn, TP>;
  constexpr int SP = Cfg::kSP;
  constexpr int RP = Cfg::kRP;
  constexpr int SROWS = 2 * kSStep;
  constexpr bool HW_ = Cfg::kHalfW;
  constexpr int W2 = 2 * HALO;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
  TP* stg = reinterpret_cast<TP*>(smem);
  float* ring = reinterpret_cast<float*>(smem + Cfg::kStageBytes);
  __shared__ uint64_t bar;

  const Geometry& g = a.g;
  const int64_t beg = scta_range_start<HALO>(g, blockIdx.x, gridDim.x);
  const int64_t end = scta_range_start<HALO>(g, blockIdx.x + 1, gridDim.x);
  const TP* const src[3] = {static_cast<const TP*>(a.p0), static_cast<const TP*>(a.p1),
                            static_cast<const TP*>(a.p2)};
  const TIn* img1 = static_cast<const TIn*>(a.img1);
  const TIn* img2 = static_cast<const TIn*>(a.img2);
  const int warp = threadIdx.x >> 5;
  const int c = threadIdx.x;
  Taps2<HALO, HW_> T;
  T.load();

  const bool tma = a.use_tma != 0;
  if (tma && threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  SPart part = sfirst_part(beg, end, g);
  if (tma && threadIdx.x < 3) prefetch_tensormap(a.tmap + threadIdx.x);
  // the first preload's boxes into L2 while the previous kernel finishes
  if (tma) prefetch_preload<HALO, 3>(a.tmap, part, g);
  grid_dependency_wait();
  grid_launch_dependents();
  auto stage_rows = [&](const SStage& st) {
    if (tma) {
      if (warp == 0) sstage_tma<TP, 3>(stg, a.tmap, st, &bar);
    } else {
      Step<HALO> s{};
      s.plane = st.plane;
      s.strip = st.strip;
      s.first = false;
      s.t = st.h0 - HALO;
      s.n = st.nh;
      stage<TP, 3, SROWS, Step<HALO>, kSThreads>(stg + st.slot * SP, src, g, s, a.aligned16);
    }
  };
  unsigned phase = 0;
  auto wait_staged = [&]() -> bool {
    bool timed_out = false;
    if (tma) {
      timed_out = !mbar_wait_bounded(&bar, phase, a.wait_limit);
      phase ^= 1u;
    } else {
      cp_async_wait_all();
    }
    if (__syncthreads_or(timed_out)) {
      if (threadIdx.x == 0) atomicOr(&g_device_error, kErrStagingTimeout);
      mbar_wait_bounded(&bar, phase ^ 1u, kWaitLimit);
      return false;
    }
    return true;
  };
  if (part.live) stage_rows({part.plane, part.strip, part.t0 - HALO, W2, 0});
  const int W = static_cast<int>(g.W);
  const float* col = ring + c;

  while (part.live) {
    const SPart nextp = snext_part(part, g);
    const int gx = part.strip * kStrip + c;
    const bool in_x = gx < W;
    const bool strip_full = part.strip * kStrip + kStrip <= W;
    const int64_t plane_off = static_cast<int64_t>(part.plane) * g.HW + gx;
    const TIn* x_pl = img1 + plane_off;
    const TIn* y_pl = img2 + plane_off;
    float chain = a.chain_scale;
    float l1c = a.l1_scale;
    if (a.grad_out) {
      const float up = a.grad_out[a.grad_per_image ? part.img : 0];
      chain = __fmul_rn(chain, up);
      l1c = __fmul_rn(l1c, up);
    }

    // ---- preload ----
    if (!wait_staged()) return;
    sbwd_hpass<HALO, TIn, TP>(stg, ring, W2, T);
    __syncthreads();
    stage_rows({part.plane, part.strip, part.t0 + HALO, min(kSStep, part.t1 - part.t0), 0});
    float2 wA[W2];  // the column's last 2*HALO rows of filtered (dm_dmu1, dm_dsigma1_sq)
    float wB[W2];   // ... and of filtered dm_dsigma12
#pragma unroll
    for (int j = 0; j < W2; ++j) {
      wA[j] = make_float2(col[j * RP + 0 * kStrip], col[j * RP + 1 * kStrip]);
      wB[j] = col[j * RP + 2 * kStrip];
    }
    // (no barrier: the staging wait of the first step orders these reads before its pass)

    // ---- regular steps ----
    int slot = 0;
    for (int t = part.t0; t < part.t1; t += kSStep) {
      const int n = min(kSStep, part.t1 - t);
      const bool last = t + kSStep >= part.t1;
      const bool full = n == kSStep && strip_full;
      if (!wait_staged()) return;
      if (!last) stage_rows({part.plane, part.strip, t + kSStep + HALO,
                             min(kSStep, part.t1 - t - kSStep), slot ^ kSStep});
      // the epilogue's image values, loaded before the horizontal pass so they are in flight
      const int off0 = t * W;
      float xin[kSStep], yin[kSStep];
      if (full) {
#pragma unroll
        for (int k = 0; k < kSStep; ++k) {
          xin[k] = ldg1(x_pl + off0 + k * W);
          yin[k] = ldg1(y_pl + off0 + k * W);
        }
      } else {
#pragma unroll
        for (int k = 0; k < kSStep; ++k) {
          const bool ld = in_x && k < n;
          xin[k] = ld ? ldg1(x_pl + off0 + k * W) : 0.f;
          yin[k] = ld ? ldg1(y_pl + off0 + k * W) : 0.f;
        }
      }
      sbwd_hpass<HALO, TIn, TP>(stg + slot * SP, ring, n, T);
      __syncthreads();
      if (last && nextp.live) stage_rows({nextp.plane, nextp.strip, nextp.t0 - HALO, W2, 0});

      float2 nA[kSStep];
      float nB[kSStep];
#pragma unroll
      for (int r = 0; r < kSStep; ++r) {
        if (full || r < n) {
          nA[r] = make_float2(col[r * RP + 0 * kStrip], col[r * RP + 1 * kStrip]);
          nB[r] = col[r * RP + 2 * kStrip];
        } else {
          nA[r] = make_float2(0.f, 0.f);
          nB[r] = 0.f;
        }
      }
      auto rowA = [&](int j) { return j < W2 ? wA[j] : nA[j - W2]; };
      auto rowB = [&](int j) { return j < W2 ? wB[j] : nB[j - W2]; };
      float gv[kSStep];
#pragma unroll
      for (int k = 0; k < kSStep; ++k) {
        const float2 r01 = svsum<HALO, HW_>(T, k, rowA);
        const float r2 = svsum1<HALO, HW_>(T, k, rowB);
        // g = s0 + 2 x s1 + y s2 (csrc/ssim.cu:504), then the chain factor
        gv[k] = __fmul_rn(__fmaf_rn(yin[k], r2, __fmaf_rn(__fmul_rn(2.f, xin[k]), r01.y, r01.x)),
                          chain);
      }
      if (a.l1_scale != 0.f) {
        // d|x - y|/dx = sign(x - y), 0 where x == y (torch's abs backward)
#pragma unroll
        for (int k = 0; k < kSStep; ++k) {
          const float dv = __fsub_rn(xin[k], yin[k]);
          gv[k] = __fmaf_rn(dv > 0.f ? 1.f : (dv < 0.f ? -1.f : 0.f), l1c, gv[k]);
        }
      }
      auto store_grad = [&](auto* base) {
        auto* gp = base + plane_off + off0;
        if (full) {
#pragma unroll
          for (int k = 0; k < kSStep; ++k) store1(gp + k * W, gv[k]);
        } else if (in_x) {
#pragma unroll
          for (int k = 0; k < kSStep; ++k)
            if (k < n) store1(gp + k * W, gv[k]);
        }
      };
      if (a.grad_dtype == 0)
        store_grad(static_cast<float*>(a.grad));
      else if (a.grad_dtype == 1)
        store_grad(static_cast<__half*>(a.grad));
      else
        store_grad(static_cast<__nv_bfloat16*>(a.grad));
      {
        float2 cA[W2];
        float cB[W2];
#pragma unroll
        for (int j = 0; j < W2; ++j) {
          cA[j] = j + kSStep < W2 ? wA[j + kSStep] : nA[j + kSStep - W2];
          cB[j] = j + kSStep < W2 ? wB[j + kSStep] : nB[j + kSStep - W2];
        }
#pragma unroll
        for (int j = 0; j < W2; ++j) {
          wA[j] = cA[j];
          wB[j] = cB[j];
        }
      }
      // the next step's staging wait (a CTA barrier) orders this step's reads of the filtered
      // rows before the next horizontal pass overwrites them
      slot ^= kSStep;
    }
    part = nextp;
  }
}

}  // namespace fssim
