// SSIM stencil kernels for sm_100a (B200).
//
// Work decomposition (both kernels)
// ---------------------------------
// The image batch is viewed as P = B*C planes, each cut into S = ceil(W/64) vertical
// strips of 64 output columns. Every (plane, strip) pair is a column of H output rows;
// all columns laid end to end form LT = P*S*H "strip-rows". A persistent grid of G CTAs
// splits [0, LT) into G equal contiguous ranges, so every CTA gets the same number of
// rows whatever the image shape. A CTA walks its range in steps of up to 32 output rows:
//
//   stage   input rows of the step (64 + 16 columns, zero outside the image) -> smem,
//           issued with cp.async one step ahead so the copy overlaps the previous step;
//   H-pass  horizontal Gaussian of every staged row -> a smem ring of moment rows
//           (5 moments forward, 3 chain-weighted partials backward);
//   V-pass  vertical Gaussian of the ring for the step's 32 x 64 outputs, then the
//           per-pixel epilogue (SSIM + partials, or the gradient).
//
// The last 2*HALO moment rows of a step are kept for the next step (copied to the top
// of the ring), so the vertical halo is computed once per column run, not per tile.
// Zero padding ("same") comes from the zero-filled staging of out-of-image pixels.
//
// Arithmetic follows the reference kernels tap for tap (csrc/ssim.cu:200-300,440-503):
// symmetric taps paired as (left + right) * w for d = 1..HALO, centre last, FP32.
//
// Reduction: each CTA sums its pixels' SSIM per column run (FP32 per thread per step,
// FP64 across the block), converts the run's sum to 2^-28 fixed point and adds it with
// a 64-bit integer atomic into a per-image accumulator. Integer addition is associative,
// so the result is bitwise deterministic in any CTA order. The last CTA to finish
// (atomicInc ticket) turns the accumulators into the outputs and zeroes them again.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fssim {

constexpr int kThreads = 128;         // 4 warps per CTA
constexpr int kStrip = 64;            // output columns per strip
constexpr int kRows = 32;             // output rows per step (8 per warp)
constexpr int kLeft = 8;              // staged columns left of the strip (>= HALO, 16-byte aligned)
constexpr int kInCols = kStrip + 2 * kLeft;  // 80 staged columns
constexpr double kFixScale = 268435456.0;    // 2^28 fixed point for the sums

// Staged row pitch in elements. The pitch in 4-byte words is 4 * odd, so the 8 lanes of
// a quarter warp reading 16 bytes each from 8 consecutive rows hit distinct banks.
template <typename T> struct StagePitch;
template <> struct StagePitch<float> { static constexpr int value = 84; };   // 84 words
template <> struct StagePitch<__half> { static constexpr int value = 88; };  // 44 words

// Moment-ring pitch in floats: NMAP rows of 64 plus 4 (again 4 * odd words modulo 32).
template <int NMAP> struct RingPitch { static constexpr int value = NMAP * kStrip + 4; };

template <int HALO> struct MaxRows { static constexpr int value = kRows + 2 * HALO; };

// Gaussian taps: [half-rounded][halo-3][k], k = 0..2*HALO, symmetric.
// Row 0: the reference's FP32 tables (csrc/ssim.cu:28-64).
// Row 1: the same values rounded to IEEE half, as the reference's FP16 kernels use them
//        (csrc/ssim_fp16.cu:55-82, __float2half then __half2float).
__constant__ float c_taps[2][3][11] = {
    {{0.00443304609f, 0.05400558188f, 0.24203622937f, 0.39905029535f, 0.24203622937f,
      0.05400558188f, 0.00443304609f, 0.f, 0.f, 0.f, 0.f},
     {0.00098442685f, 0.00971502065f, 0.04529544711f, 0.11722830242f, 0.19355361462f,
      0.11722830242f, 0.04529544711f, 0.00971502065f, 0.00098442685f, 0.f, 0.f},
     {0.001028380123898387f, 0.0075987582094967365f, 0.036000773310661316f,
      0.10936068743467331f, 0.21300552785396576f, 0.26601171493530273f,
      0.21300552785396576f, 0.10936068743467331f, 0.036000773310661316f,
      0.0075987582094967365f, 0.001028380123898387f}},
    {{0x1.228p-8f, 0x1.ba8p-5f, 0x1.efcp-3f, 0x1.98cp-2f, 0x1.efcp-3f, 0x1.ba8p-5f, 0x1.228p-8f,
      0.f, 0.f, 0.f, 0.f},
     {0x1.02p-10f, 0x1.3e4p-7f, 0x1.73p-5f, 0x1.e04p-4f, 0x1.8c8p-3f, 0x1.e04p-4f, 0x1.73p-5f,
      0x1.3e4p-7f, 0x1.02p-10f, 0.f, 0.f},
     {0x1.0d8p-10f, 0x1.f2p-8f, 0x1.27p-5f, 0x1.cp-4f, 0x1.b44p-3f, 0x1.108p-2f, 0x1.b44p-3f,
      0x1.cp-4f, 0x1.27p-5f, 0x1.f2p-8f, 0x1.0d8p-10f}}};

template <int HALO, bool HALFW>
__device__ __forceinline__ float tap(int k) {
  return c_taps[HALFW ? 1 : 0][HALO - 3][k];
}

// ---------------------------------------------------------------------------------------
// Small device helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool in) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
               "r"(in ? 16 : 0));
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src, bool in) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
               "r"(in ? 4 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

// Load NV consecutive staged elements (16-byte aligned) as floats.
template <int NV>
__device__ __forceinline__ void load_vec(const float* p, float (&v)[NV]) {
#pragma unroll
  for (int q = 0; q < NV / 4; ++q) {
    const float4 t = reinterpret_cast<const float4*>(p)[q];
    v[4 * q + 0] = t.x;
    v[4 * q + 1] = t.y;
    v[4 * q + 2] = t.z;
    v[4 * q + 3] = t.w;
  }
}
template <int NV>
__device__ __forceinline__ void load_vec(const __half* p, float (&v)[NV]) {
#pragma unroll
  for (int q = 0; q < NV / 8; ++q) {
    const uint4 t = reinterpret_cast<const uint4*>(p)[q];
    const __half2* h = reinterpret_cast<const __half2*>(&t);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __half22float2(h[e]);
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
}

// Store a pair of adjacent columns (gx, gx+1) of one row; `pair` means both columns are in
// range and the address is aligned for a vector store.
__device__ __forceinline__ void store2(float* base, int64_t idx, float a, float b, bool pair,
                                      bool in0, bool in1) {
  if (pair) {
    *reinterpret_cast<float2*>(base + idx) = make_float2(a, b);
  } else {
    if (in0) base[idx] = a;
    if (in1) base[idx + 1] = b;
  }
}
__device__ __forceinline__ void store2(__half* base, int64_t idx, float a, float b, bool pair,
                                      bool in0, bool in1) {
  if (pair) {
    *reinterpret_cast<__half2*>(base + idx) = __floats2half2_rn(a, b);
  } else {
    if (in0) base[idx] = __float2half_rn(a);
    if (in1) base[idx + 1] = __float2half_rn(b);
  }
}
__device__ __forceinline__ void store2(__nv_bfloat16* base, int64_t idx, float a, float b,
                                      bool pair, bool in0, bool in1) {
  if (pair) {
    *reinterpret_cast<__nv_bfloat162*>(base + idx) = __floats2bfloat162_rn(a, b);
  } else {
    if (in0) base[idx] = __float2bfloat16_rn(a);
    if (in1) base[idx + 1] = __float2bfloat16_rn(b);
  }
}

template <typename T>
__device__ __forceinline__ void load2(const T* base, int64_t idx, bool pair, bool in0, bool in1,
                                      float& a, float& b) {
  if (pair) {
    if constexpr (sizeof(T) == 4) {
      const float2 t = *reinterpret_cast<const float2*>(base + idx);
      a = t.x;
      b = t.y;
    } else {
      const float2 t = __half22float2(*reinterpret_cast<const __half2*>(base + idx));
      a = t.x;
      b = t.y;
    }
  } else {
    a = in0 ? to_f(base[idx]) : 0.f;
    b = in1 ? to_f(base[idx + 1]) : 0.f;
  }
}

// ---------------------------------------------------------------------------------------
// Geometry and step sequencing
// ---------------------------------------------------------------------------------------
struct Geometry {
  int64_t H, W, HW;  // plane geometry
  int64_t LT;        // strip-rows in the whole batch
  int S;             // strips per plane
  int C;             // channels per image
  int B;             // images
};

struct Step {
  int64_t pos;   // linear strip-row index of the first output row of this step
  int64_t plane;
  int strip;
  int t;         // first output row (image row index)
  int n;         // output rows in this step (1..32)
  int h0;        // first moment row (image row index) computed by this step
  int nh;        // moment rows computed by this step
  int hdst;      // ring row receiving moment row h0
  bool valid;
  bool last;     // last step of its column run
};

template <int HALO>
__device__ __forceinline__ Step make_step(int64_t pos, int64_t beg, int64_t end,
                                          const Geometry& g) {
  Step s;
  s.valid = pos < end;
  s.pos = pos;
  if (!s.valid) {
    s.plane = 0; s.strip = 0; s.t = 0; s.n = 0; s.h0 = 0; s.nh = 0; s.hdst = 0; s.last = true;
    return s;
  }
  const int64_t col = pos / g.H;
  const int r = static_cast<int>(pos - col * g.H);
  const int64_t col_end = (col + 1) * g.H;
  const int64_t run_end = end < col_end ? end : col_end;
  s.plane = col / g.S;
  s.strip = static_cast<int>(col - s.plane * g.S);
  s.t = r;
  const int64_t left = run_end - pos;
  s.n = static_cast<int>(left < kRows ? left : kRows);
  const bool first = (pos == beg) || (r == 0);
  s.last = (pos + s.n == run_end);
  if (first) {
    s.h0 = r - HALO;
    s.nh = s.n + 2 * HALO;
    s.hdst = 0;
  } else {
    s.h0 = r + HALO;
    s.nh = s.n;
    s.hdst = 2 * HALO;
  }
  return s;
}

// Stage moment rows [h0, h0+nh) x columns [x0-8, x0+72) of NMAP planes into smem
// (layout [NMAP][MAXR][PITCH]); out-of-image elements become zero.
template <typename T, int NMAP, int MAXR>
__device__ __forceinline__ void stage(T* sm, const T* const (&src)[NMAP], const Geometry& g,
                                      const Step& s, bool aligned16) {
  constexpr int P = StagePitch<T>::value;
  const int x0 = s.strip * kStrip - kLeft;
  if (aligned16) {
    constexpr int E = 16 / sizeof(T);   // elements per 16-byte chunk
    constexpr int CH = kInCols / E;      // chunks per staged row
    const int total = s.nh * CH;
#pragma unroll
    for (int m = 0; m < NMAP; ++m) {
      const T* plane = src[m] + s.plane * g.HW;
      T* dst = sm + m * MAXR * P;
      for (int i = threadIdx.x; i < total; i += kThreads) {
        const int row = i / CH;
        const int ch = i - row * CH;
        const int gy = s.h0 + row;
        const int gx = x0 + ch * E;
        const bool in = (gy >= 0) && (gy < g.H) && (gx >= 0) && (gx < g.W);
        const T* p = in ? plane + static_cast<int64_t>(gy) * g.W + gx : plane;
        cp_async16(dst + row * P + ch * E, p, in);
      }
    }
  } else if constexpr (sizeof(T) == 4) {
    const int total = s.nh * kInCols;
#pragma unroll
    for (int m = 0; m < NMAP; ++m) {
      const T* plane = src[m] + s.plane * g.HW;
      T* dst = sm + m * MAXR * P;
      for (int i = threadIdx.x; i < total; i += kThreads) {
        const int row = i / kInCols;
        const int c = i - row * kInCols;
        const int gy = s.h0 + row;
        const int gx = x0 + c;
        const bool in = (gy >= 0) && (gy < g.H) && (gx >= 0) && (gx < g.W);
        const T* p = in ? plane + static_cast<int64_t>(gy) * g.W + gx : plane;
        cp_async4(dst + row * P + c, p, in);
      }
    }
  } else {
    // 2-byte elements on an unaligned layout: plain loads.
    const int total = s.nh * kInCols;
#pragma unroll
    for (int m = 0; m < NMAP; ++m) {
      const T* plane = src[m] + s.plane * g.HW;
      T* dst = sm + m * MAXR * P;
      for (int i = threadIdx.x; i < total; i += kThreads) {
        const int row = i / kInCols;
        const int c = i - row * kInCols;
        const int gy = s.h0 + row;
        const int gx = x0 + c;
        const bool in = (gy >= 0) && (gy < g.H) && (gx >= 0) && (gx < g.W);
        dst[row * P + c] = in ? plane[static_cast<int64_t>(gy) * g.W + gx] : T(0.f);
      }
    }
  }
  cp_async_commit();
}

// Copy ring rows [n, n + 2*HALO) to [0, 2*HALO): the vertical halo for the next step.
template <int HALO, int RP>
__device__ __forceinline__ void ring_carry(float* ring, int n) {
  constexpr int V = RP / 4;  // float4 per ring row
  float4* r4 = reinterpret_cast<float4*>(ring);
  for (int i = threadIdx.x; i < 2 * HALO * V; i += kThreads) {
    const int row = i / V;
    const int c = i - row * V;
    r4[row * V + c] = r4[(n + row) * V + c];
  }
}

// Deterministic block sum of a double (fixed shuffle tree, warps combined in order).
__device__ __forceinline__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  return ((red[0] + red[1]) + red[2]) + red[3];
}

// ---------------------------------------------------------------------------------------
// Forward kernel
// ---------------------------------------------------------------------------------------
struct FwdParams {
  const void* img1;
  const void* img2;
  float* map;            // optional per-pixel SSIM (unmasked)
  void* p0;              // optional partials (TP): dm_dmu1, dm_dsigma1_sq, dm_dsigma12
  void* p1;
  void* p2;
  float* out;            // reduction outputs
  double* image_sums;    // optional FP64 per-image sums
  unsigned long long* acc;  // B fixed-point accumulators (workspace)
  unsigned* ticket;         // last-CTA ticket (workspace)
  Geometry g;
  float C1, C2, out_scale;
  int valid, clamp, reduce, mask_partials, aligned16, pair_ok;
};

template <int HALO, typename TIn, typename TP, bool TRAIN>
struct FwdConfig {
  static constexpr bool kHalfW = sizeof(TIn) == 2;
  static constexpr int kMaxR = MaxRows<HALO>::value;
  static constexpr int kSP = StagePitch<TIn>::value;
  static constexpr int kRP = RingPitch<5>::value;
  static constexpr size_t kStageBytes = 2ull * kMaxR * kSP * sizeof(TIn);
  static constexpr size_t kRingBytes = static_cast<size_t>(kMaxR) * kRP * sizeof(float);
  static constexpr size_t kSmem = kStageBytes + kRingBytes;
};

// Horizontal pass of the forward: for staged row i and output columns 8j..8j+7 compute the
// five moments sum w*X, w*X^2, w*Y, w*Y^2, w*XY (order of the reference's xconv features).
template <int HALO, typename TIn, int MAXR>
__device__ __forceinline__ void fwd_hpass(const TIn* sx, const TIn* sy, float* ring, int nh,
                                          int hdst) {
  constexpr bool HW_ = sizeof(TIn) == 2;
  constexpr int SP = StagePitch<TIn>::value;
  constexpr int RP = RingPitch<5>::value;
  constexpr int HA = (sizeof(TIn) == 2 || HALO > 4) ? 8 : 4;  // aligned left extent
  constexpr int NV = 8 + 2 * HA;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int rg = 0; rg < nh; rg += 32) {
    const int i = rg + lane;
    if (i < nh) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = warp + 4 * jj;
        float xv[NV], yv[NV];
        load_vec(sx + i * SP + 8 * j + kLeft - HA, xv);
        load_vec(sy + i * SP + 8 * j + kLeft - HA, yv);
        float xx[NV], yy[NV], xy[NV];
#pragma unroll
        for (int q = HA - HALO; q < HA + 8; ++q) {
          xx[q] = xv[q] * xv[q];
          yy[q] = yv[q] * yv[q];
          xy[q] = xv[q] * yv[q];
        }
        float o[5][8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = HA + k;
          float sX = 0.f, sX2 = 0.f, sY = 0.f, sY2 = 0.f, sXY = 0.f;
#pragma unroll
          for (int d = 1; d <= HALO; ++d) {
            const float w = tap<HALO, HW_>(HALO - d);
            const int l = c - d, r = c + d;
            sX = fmaf(xv[l] + xv[r], w, sX);
            sX2 = fmaf(fmaf(xv[r], xv[r], xx[l]), w, sX2);
            sY = fmaf(yv[l] + yv[r], w, sY);
            sY2 = fmaf(fmaf(yv[r], yv[r], yy[l]), w, sY2);
            sXY = fmaf(fmaf(xv[r], yv[r], xy[l]), w, sXY);
          }
          const float wc = tap<HALO, HW_>(HALO);
          o[0][k] = fmaf(xv[c], wc, sX);
          o[1][k] = fmaf(xx[c], wc, sX2);
          o[2][k] = fmaf(yv[c], wc, sY);
          o[3][k] = fmaf(yy[c], wc, sY2);
          o[4][k] = fmaf(xy[c], wc, sXY);
        }
        float* dst = ring + (hdst + i) * RP + 8 * j;
#pragma unroll
        for (int m = 0; m < 5; ++m) {
          reinterpret_cast<float4*>(dst + m * kStrip)[0] =
              make_float4(o[m][0], o[m][1], o[m][2], o[m][3]);
          reinterpret_cast<float4*>(dst + m * kStrip)[1] =
              make_float4(o[m][4], o[m][5], o[m][6], o[m][7]);
        }
      }
    }
  }
}

template <int HALO, typename TIn, typename TP, bool TRAIN>
__global__ void __launch_bounds__(kThreads, 2) ssim_fwd_kernel(const FwdParams a) {
  using Cfg = FwdConfig<HALO, TIn, TP, TRAIN>;
  constexpr int MAXR = Cfg::kMaxR;
  constexpr int SP = Cfg::kSP;
  constexpr int RP = Cfg::kRP;
  constexpr bool HW_ = Cfg::kHalfW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TIn* stg = reinterpret_cast<TIn*>(smem_raw);
  float* ring = reinterpret_cast<float*>(smem_raw + Cfg::kStageBytes);
  __shared__ double red[4];
  __shared__ unsigned s_last;

  const Geometry& g = a.g;
  const int64_t beg = (g.LT * blockIdx.x) / gridDim.x;
  const int64_t end = (g.LT * (blockIdx.x + 1)) / gridDim.x;
  const TIn* const src[2] = {static_cast<const TIn*>(a.img1), static_cast<const TIn*>(a.img2)};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = warp * 8;

  Step cur = make_step<HALO>(beg, beg, end, g);
  if (cur.valid) stage<TIn, 2, MAXR>(stg, src, g, cur, a.aligned16);
  double run_sum = 0.0;

  while (cur.valid) {
    cp_async_wait_all();
    __syncthreads();
    fwd_hpass<HALO, TIn, MAXR>(stg, stg + MAXR * SP, ring, cur.nh, cur.hdst);
    __syncthreads();
    const Step nxt = make_step<HALO>(cur.pos + cur.n, beg, end, g);
    if (nxt.valid) stage<TIn, 2, MAXR>(stg, src, g, nxt, a.aligned16);

    // ---- V-pass + epilogue: rows r0..r0+7 of the step, columns 2*lane, 2*lane+1 ----
    if (r0 < cur.n) {
      float res[5][8][2];
#pragma unroll
      for (int m = 0; m < 5; ++m) {
        float2 v[8 + 2 * HALO];
#pragma unroll
        for (int q = 0; q < 8 + 2 * HALO; ++q)
          v[q] = *reinterpret_cast<const float2*>(ring + (r0 + q) * RP + m * kStrip + 2 * lane);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float ox = 0.f, oy = 0.f;
#pragma unroll
          for (int d = 1; d <= HALO; ++d) {
            const float w = tap<HALO, HW_>(HALO - d);
            ox = fmaf(v[k + HALO - d].x + v[k + HALO + d].x, w, ox);
            oy = fmaf(v[k + HALO - d].y + v[k + HALO + d].y, w, oy);
          }
          const float wc = tap<HALO, HW_>(HALO);
          res[m][k][0] = fmaf(v[k + HALO].x, wc, ox);
          res[m][k][1] = fmaf(v[k + HALO].y, wc, oy);
        }
      }
      const int gx0 = cur.strip * kStrip + 2 * lane;
      const bool in0 = gx0 < g.W, in1 = gx0 + 1 < g.W;
      const bool pair = a.pair_ok && in1;
      const int64_t plane_off = cur.plane * g.HW;
      float step_sum = 0.f;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int row = r0 + k;
        if (row < cur.n) {
          const int gy = cur.t + row;
          const bool row_ok = !a.valid || (gy >= HALO && gy < g.H - HALO);
          float val[2], pm[2], ps[2], pc[2];
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const float mu1 = res[0][k][c], mu2 = res[2][k][c];
            const float mu1_sq = mu1 * mu1, mu2_sq = mu2 * mu2;
            const float sigma1_sq = res[1][k][c] - mu1_sq;
            const float sigma2_sq = res[3][k][c] - mu2_sq;
            const float sigma12 = res[4][k][c] - mu1 * mu2;
            const float A = mu1_sq + mu2_sq + a.C1;
            const float B = sigma1_sq + sigma2_sq + a.C2;
            const float Cc = 2.f * mu1 * mu2 + a.C1;
            const float D = 2.f * sigma12 + a.C2;
            const float rA = __fdividef(1.f, A);
            const float rB = __fdividef(1.f, B);
            const float rAB = rA * rB;
            const float v = (Cc * D) * rAB;
            val[c] = v;
            const int gx = gx0 + c;
            const bool in = c == 0 ? in0 : in1;
            const bool counted =
                in && row_ok && (!a.valid || (gx >= HALO && gx < g.W - HALO));
            if (a.reduce && counted) step_sum += (a.clamp && v < 0.f) ? 0.f : v;
            if (TRAIN) {
              const bool live = !a.mask_partials || (counted && (!a.clamp || v >= 0.f));
              pm[c] = live ? 2.f * mu2 * (D - Cc) * rAB + 2.f * mu1 * v * (rB - rA) : 0.f;
              ps[c] = live ? -v * rB : 0.f;
              pc[c] = live ? 2.f * Cc * rAB : 0.f;
            }
          }
          const int64_t idx = plane_off + static_cast<int64_t>(gy) * g.W + gx0;
          if (a.map) store2(a.map, idx, val[0], val[1], pair, in0, in1);
          if (TRAIN) {
            store2(static_cast<TP*>(a.p0), idx, pm[0], pm[1], pair, in0, in1);
            store2(static_cast<TP*>(a.p1), idx, ps[0], ps[1], pair, in0, in1);
            store2(static_cast<TP*>(a.p2), idx, pc[0], pc[1], pair, in0, in1);
          }
        }
      }
      run_sum += static_cast<double>(step_sum);
    }

    if (a.reduce && cur.last) {
      // end of a column run: fold its sum into the image's fixed-point accumulator
      const double s = block_sum(run_sum, red);
      run_sum = 0.0;
      if (threadIdx.x == 0) {
        const int64_t b = cur.plane / g.C;
        const long long q = __double2ll_rn(s * kFixScale);
        atomicAdd(a.acc + b, static_cast<unsigned long long>(q));
      }
    }
    __syncthreads();
    if (!cur.last) {
      ring_carry<HALO, RP>(ring, cur.n);
    }
    cur = nxt;
  }

  if (!a.reduce) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicInc(a.ticket, gridDim.x - 1);
    s_last = (prev == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  double local = 0.0;
  for (int b = threadIdx.x; b < g.B; b += kThreads) {
    const long long q = static_cast<long long>(atomicExch(a.acc + b, 0ull));
    const double s = static_cast<double>(q) * (1.0 / kFixScale);
    if (a.image_sums) a.image_sums[b] = s;
    if (a.reduce == 2) a.out[b] = static_cast<float>(s * static_cast<double>(a.out_scale));
    local += s;
  }
  if (a.reduce == 1) {
    const double total = block_sum(local, red);
    if (threadIdx.x == 0) a.out[0] = static_cast<float>(total * static_cast<double>(a.out_scale));
  }
}

// ---------------------------------------------------------------------------------------
// Backward kernel
// ---------------------------------------------------------------------------------------
struct BwdParams {
  const void* img1;
  const void* img2;
  const void* p0;         // partials (TP)
  const void* p1;
  const void* p2;
  const float* dl;        // general path: per-pixel dL/dmap (FP32)
  const float* grad_out;  // fused path: upstream scalar(s) (FP32) or NULL
  void* grad;             // output
  Geometry g;
  float chain_scale;
  int grad_per_image, grad_dtype, aligned16, pair_ok;
};

template <int HALO, typename TIn, typename TP, bool DLMAP>
struct BwdConfig {
  static constexpr bool kHalfW = sizeof(TIn) == 2;
  static constexpr int kMaxR = MaxRows<HALO>::value;
  static constexpr int kSP = StagePitch<TP>::value;
  static constexpr int kRP = RingPitch<3>::value;
  static constexpr size_t kStageBytes = 3ull * kMaxR * kSP * sizeof(TP);
  static constexpr size_t kDlBytes =
      DLMAP ? static_cast<size_t>(kMaxR) * StagePitch<float>::value * sizeof(float) : 0;
  static constexpr size_t kRingBytes = static_cast<size_t>(kMaxR) * kRP * sizeof(float);
  static constexpr size_t kSmem = kStageBytes + kDlBytes + kRingBytes;
};

// Horizontal pass of the backward over the three partial maps (times dL/dmap on the
// general path, as the reference multiplies at load, csrc/ssim.cu:408-411).
template <int HALO, typename TIn, typename TP, bool DLMAP, int MAXR>
__device__ __forceinline__ void bwd_hpass(const TP* sp, const float* sdl, float* ring, int nh,
                                          int hdst) {
  constexpr bool HW_ = sizeof(TIn) == 2;
  constexpr int SP = StagePitch<TP>::value;
  constexpr int RP = RingPitch<3>::value;
  constexpr int HA = (sizeof(TP) == 2 || HALO > 4) ? 8 : 4;
  constexpr int NV = 8 + 2 * HA;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int rg = 0; rg < nh; rg += 32) {
    const int i = rg + lane;
    if (i < nh) {
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int j = warp + 4 * jj;
        // The general path only exists for FP32 partials, so dL and the partials share
        // the staged layout (pitch 84, same aligned left extent HA).
        static_assert(!DLMAP || sizeof(TP) == 4, "per-pixel dL/dmap needs FP32 partials");
        float dl[NV];
        if (DLMAP) load_vec(sdl + i * StagePitch<float>::value + 8 * j + kLeft - HA, dl);
        float o[3][8];
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          float v[NV];
          load_vec(sp + (m * MAXR + i) * SP + 8 * j + kLeft - HA, v);
          if (DLMAP) {
#pragma unroll
            for (int q = HA - HALO; q < HA + 8 + HALO; ++q) v[q] = v[q] * dl[q];
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int c = HA + k;
            float s = 0.f;
#pragma unroll
            for (int d = 1; d <= HALO; ++d) s = fmaf(v[c - d] + v[c + d], tap<HALO, HW_>(HALO - d), s);
            o[m][k] = fmaf(v[c], tap<HALO, HW_>(HALO), s);
          }
        }
        float* dst = ring + (hdst + i) * RP + 8 * j;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          reinterpret_cast<float4*>(dst + m * kStrip)[0] =
              make_float4(o[m][0], o[m][1], o[m][2], o[m][3]);
          reinterpret_cast<float4*>(dst + m * kStrip)[1] =
              make_float4(o[m][4], o[m][5], o[m][6], o[m][7]);
        }
      }
    }
  }
}

template <int HALO, typename TIn, typename TP, bool DLMAP>
__global__ void __launch_bounds__(kThreads, 2) ssim_bwd_kernel(const BwdParams a) {
  using Cfg = BwdConfig<HALO, TIn, TP, DLMAP>;
  constexpr int MAXR = Cfg::kMaxR;
  constexpr int RP = Cfg::kRP;
  constexpr bool HW_ = Cfg::kHalfW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TP* stg = reinterpret_cast<TP*>(smem_raw);
  float* sdl = reinterpret_cast<float*>(smem_raw + Cfg::kStageBytes);
  float* ring = reinterpret_cast<float*>(smem_raw + Cfg::kStageBytes + Cfg::kDlBytes);

  const Geometry& g = a.g;
  const int64_t beg = (g.LT * blockIdx.x) / gridDim.x;
  const int64_t end = (g.LT * (blockIdx.x + 1)) / gridDim.x;
  const TP* const src[3] = {static_cast<const TP*>(a.p0), static_cast<const TP*>(a.p1),
                            static_cast<const TP*>(a.p2)};
  const float* const dsrc[1] = {a.dl};
  const TIn* img1 = static_cast<const TIn*>(a.img1);
  const TIn* img2 = static_cast<const TIn*>(a.img2);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = warp * 8;

  Step cur = make_step<HALO>(beg, beg, end, g);
  if (cur.valid) {
    stage<TP, 3, MAXR>(stg, src, g, cur, a.aligned16);
    if (DLMAP) stage<float, 1, MAXR>(sdl, dsrc, g, cur, a.aligned16);
  }
  while (cur.valid) {
    cp_async_wait_all();
    __syncthreads();
    bwd_hpass<HALO, TIn, TP, DLMAP, MAXR>(stg, sdl, ring, cur.nh, cur.hdst);
    __syncthreads();
    const Step nxt = make_step<HALO>(cur.pos + cur.n, beg, end, g);
    if (nxt.valid) {
      stage<TP, 3, MAXR>(stg, src, g, nxt, a.aligned16);
      if (DLMAP) stage<float, 1, MAXR>(sdl, dsrc, g, nxt, a.aligned16);
    }

    if (r0 < cur.n) {
      const int gx0 = cur.strip * kStrip + 2 * lane;
      const bool in0 = gx0 < g.W, in1 = gx0 + 1 < g.W;
      const bool pair = a.pair_ok && in1;
      const int64_t plane_off = cur.plane * g.HW;
      float chain = a.chain_scale;
      if (!DLMAP && a.grad_out) {
        const int64_t b = cur.plane / g.C;
        chain *= a.grad_out[a.grad_per_image ? b : 0];
      }
      float res[3][8][2];
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        float2 v[8 + 2 * HALO];
#pragma unroll
        for (int q = 0; q < 8 + 2 * HALO; ++q)
          v[q] = *reinterpret_cast<const float2*>(ring + (r0 + q) * RP + m * kStrip + 2 * lane);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float ox = 0.f, oy = 0.f;
#pragma unroll
          for (int d = 1; d <= HALO; ++d) {
            const float w = tap<HALO, HW_>(HALO - d);
            ox = fmaf(v[k + HALO - d].x + v[k + HALO + d].x, w, ox);
            oy = fmaf(v[k + HALO - d].y + v[k + HALO + d].y, w, oy);
          }
          const float wc = tap<HALO, HW_>(HALO);
          res[m][k][0] = fmaf(v[k + HALO].x, wc, ox);
          res[m][k][1] = fmaf(v[k + HALO].y, wc, oy);
        }
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int row = r0 + k;
        if (row < cur.n) {
          const int gy = cur.t + row;
          const int64_t idx = plane_off + static_cast<int64_t>(gy) * g.W + gx0;
          float x0v, x1v, y0v, y1v;
          load2(img1, idx, pair, in0, in1, x0v, x1v);
          load2(img2, idx, pair, in0, in1, y0v, y1v);
          float gv0 = fmaf(y0v, res[2][k][0], fmaf(2.f * x0v, res[1][k][0], res[0][k][0]));
          float gv1 = fmaf(y1v, res[2][k][1], fmaf(2.f * x1v, res[1][k][1], res[0][k][1]));
          if (!DLMAP) {
            gv0 *= chain;
            gv1 *= chain;
          }
          if (a.grad_dtype == 0)
            store2(static_cast<float*>(a.grad), idx, gv0, gv1, pair, in0, in1);
          else if (a.grad_dtype == 1)
            store2(static_cast<__half*>(a.grad), idx, gv0, gv1, pair, in0, in1);
          else
            store2(static_cast<__nv_bfloat16*>(a.grad), idx, gv0, gv1, pair, in0, in1);
        }
      }
    }
    __syncthreads();
    if (!cur.last) ring_carry<HALO, RP>(ring, cur.n);
    cur = nxt;
  }
}

}  // namespace fssim
