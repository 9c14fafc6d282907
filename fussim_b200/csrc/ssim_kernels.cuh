// SSIM stencil kernels for sm_100a (B200).
//
// Work decomposition (both kernels)
// ---------------------------------
// The image batch is viewed as P = B*C planes, each cut into S = ceil(W/64) vertical
// strips of 64 output columns. Every (plane, strip) pair is a column of H output rows;
// all columns laid end to end form LT = P*S*H "strip-rows". A persistent grid of G CTAs
// splits [0, LT) into G equal contiguous ranges, so every CTA gets the same number of
// rows whatever the image shape. A CTA walks its range in steps of up to 16 output rows:
//
//   stage   input rows of the step (64 + 16 columns, zero outside the image) -> smem by
//           TMA boxes (cp.async where the layout does not allow TMA), issued one step
//           ahead so the copy overlaps the previous step;
//   H-pass  horizontal Gaussian of every staged row -> a smem ring of moment rows (4 maps
//           in the fused forward, 5 in the map-producing one, 3 partials backward);
//   V-pass  vertical Gaussian of the ring for the step's 16 x 64 outputs, then the
//           per-pixel epilogue (SSIM + partials, or the gradient).
//
// The last 2*HALO moment rows of a step are kept for the next step (copied to the top
// of the ring), so the vertical halo is computed once per column run, not per tile.
// Zero padding ("same") comes from the zero-filled staging of out-of-image pixels.
//
// Arithmetic follows the reference kernels tap for tap (csrc/ssim.cu:200-300,440-503):
// symmetric taps paired as (left + right) * w for d = 1..HALO, centre last, FP32, with
// the squared/cross moments as fma(right, right, left^2). All stencil and epilogue math
// runs on pairs of adjacent output columns with the sm_100 packed FP32 instructions
// (fma/add/mul .f32x2), which halve the instruction count at the same FMA throughput and
// identical per-component rounding.
//
// Reduction: each CTA sums its pixels' SSIM per column run (FP32 per thread per step,
// FP64 across the block), converts the run's sum to 2^-28 fixed point and adds it with
// a 64-bit integer atomic into a per-image accumulator. Integer addition is associative,
// so the result is bitwise deterministic in any CTA order. The last CTA to finish
// (the count on the ticket word reaches the grid size) turns the accumulators into the
// outputs and zeroes them again.
#pragma once

#include <cuda.h>  // CUtensorMap (type only; the driver API is not linked)
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fssim {

constexpr int kThreads = 128;         // 4 warps per CTA
constexpr int kStrip = 64;            // output columns per strip
constexpr int kRows = 16;             // output rows per step
constexpr int kRPT = kRows / 4;       // output rows per thread in the V-pass (4 warps)
constexpr int kLeft = 8;              // staged columns left of the strip (>= HALO, 16-byte aligned)
constexpr int kInCols = kStrip + 2 * kLeft;  // 80 staged columns
// Fixed-point scales of the per-image sums. SSIM values lie in [-1, 1], so an image's SSIM
// sum stays within 2^34 (the host rejects C*H*W > 2^34 for the reductions) and 2^28 fits it
// in a signed 64-bit word. The L1 sum of |x - y| has no such bound; 2^20 leaves room for
// image sums up to 2^43 (8.8e12) at an absolute resolution of 1e-6 per column run.
constexpr double kFixScale = 268435456.0;    // 2^28: SSIM sums
constexpr double kFixScaleL1 = 1048576.0;    // 2^20: L1 sums

// Staged row pitch in elements. The pitch in 4-byte words is 4 * odd, so the 8 lanes of
// a quarter warp reading 16 bytes each from 8 consecutive rows hit distinct banks.
template <typename T> struct StagePitch;
template <> struct StagePitch<float> { static constexpr int value = 84; };   // 84 words
template <> struct StagePitch<__half> { static constexpr int value = 88; };  // 44 words
template <> struct StagePitch<__nv_bfloat16> { static constexpr int value = 88; };

// Inputs read as IEEE half use the reference's half-rounded Gaussian taps (its FP16 kernels
// do); FP32 and bfloat16 inputs use the FP32 taps. bfloat16 has no reference kernel: it is
// this engine's native path for bfloat16 images, FP32 arithmetic on the widened values.
template <typename T> struct HalfTaps { static constexpr bool value = false; };
template <> struct HalfTaps<__half> { static constexpr bool value = true; };

// Moment-ring pitch in floats: NMAP rows of 64 plus 2. The H-pass stores 8-byte column
// pairs from 16 consecutive rows per half warp; a pitch of 2 mod 32 words puts each half
// warp on 32 distinct banks.
template <int NMAP> struct RingPitch { static constexpr int value = NMAP * kStrip + 2; };

template <int HALO> struct MaxRows { static constexpr int value = kRows + 2 * HALO; };

// H-pass task mapping. A task is (staged row i, output columns 8j..8j+7), j = 0..7; a group
// of kRG rows has 8*kRG tasks, one per thread per chunk iteration: lane l of warp w takes
// row l % kRG of the group and chunks j = w + 4*(l / kRG) + 4*kLG*jj, jj < kJJ.
constexpr int kRG = kRows < 32 ? kRows : 32;  // rows per group
constexpr int kLG = 32 / kRG;                 // lane groups per warp (1 or 2)
constexpr int kJJ = 2 / kLG;                  // chunk iterations per thread per group
static_assert(kRows == 16 || kRows == 32, "steps of 16 or 32 rows");

// Staged rows per map: MaxRows rounded up to whole TMA boxes of 16 rows, and at least two
// slots of kRows rows, so a step can be staged into one slot while the H-pass reads the
// other. The map stride (rows x pitch x element size) is then a multiple of 128 bytes, as
// is every box start.
template <int HALO> struct StageRows {
  static constexpr int kBoxed = (MaxRows<HALO>::value + 15) / 16 * 16;
  static constexpr int value = kBoxed > 2 * kRows ? kBoxed : 2 * kRows;
};

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
// The packed FMA takes its multiplier as a register pair, not as a constant-bank operand.
// The HALO+1 distinct taps are therefore loaded once per kernel into register pairs and
// made opaque to the compiler, so it keeps them live instead of re-materialising a pair
// from constant memory before every packed FMA.
template <int HALO, bool HALFW>
struct Taps2 {
  float2 w[HALO + 1];  // w[k] = (tap k, tap k), k = 0..HALO (the centre is k = HALO)
  __device__ __forceinline__ void load() {
#pragma unroll
    for (int k = 0; k <= HALO; ++k) {
      float t = tap<HALO, HALFW>(k);
      asm volatile("" : "+f"(t));
      w[k] = make_float2(t, t);
    }
  }
};

// ---------------------------------------------------------------------------------------
// Packed FP32 helpers (per component identical to fmaf / + / *)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  return __fadd2_rn(a, make_float2(-b.x, -b.y));
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }

// Single-instruction reciprocal (PTX rcp.approx.ftz.f32, max error 1 ulp). The SSIM
// denominators are >= C1 or C2 - O(1e-8), far above the denormal range.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
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

// ---------------------------------------------------------------------------------------
// Staging with the tensor memory accelerator (TMA)
// ---------------------------------------------------------------------------------------
// When every staged plane is 16-byte aligned with a row pitch that is a multiple of 16
// bytes, warp 0 stages a step with a handful of tiled bulk copies (boxes of kBoxRows
// rows x one staged row pitch of columns, zero-filled outside the image by the copy unit)
// that complete on an mbarrier. This replaces 2-4 cp.async chunks per thread per staged
// row and all their address arithmetic. Each copy reads this GPU's own memory into this CTA only.
constexpr int kBoxRows = 16;  // one box per map for a regular step
// Bounded mbarrier polls before a step reports failure. The kernels take the limit of a
// step's first wait as a parameter (the host default is this value; a limit of 0 makes
// every TMA-staged step fail at once, which tests use to exercise the failure path). The
// wait that drains a failed step's copies before the CTA leaves always uses this bound.
constexpr int kWaitLimit = 1 << 20;

// Device-side failure codes (OR-ed into g_device_error, read by fssim_poll_device_error).
constexpr unsigned kErrStagingTimeout = 1u;
__device__ unsigned g_device_error;

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
// Orders this CTA's earlier generic-proxy shared-memory accesses before later bulk copies.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the mbarrier phase with the given parity to complete; false after `limit` polls
// (the caller reports the failure and stops its work).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, int limit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// Brings a tensor map into the descriptor cache ahead of its first copy.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// L2 prefetch of one tensor-map box (no shared memory, no completion to wait for). L2 is
// the point of coherence of global memory, so a prefetch issued while an earlier kernel may
// still write the same lines cannot make a later load read stale data.
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
// One 3-D tiled bulk copy global -> shared (coordinates: column, row, plane).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// Programmatic dependent launch. The kernels are launched so that they may start while the
// previous kernel on the stream is finishing; their set-up (barrier init, step cursor)
// overlaps that tail, and griddepcontrol.wait, before the first access to global memory,
// waits for the previous kernel to complete and its writes to be visible. (Both are no-ops
// for a regular launch.) A kernel then allows its own dependent to launch.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float2 to_f2(__half2 v) { return __half22float2(v); }
__device__ __forceinline__ float2 to_f2(__nv_bfloat162 v) { return __bfloat1622float2(v); }
template <typename T> struct Pair2;
template <> struct Pair2<__half> { using type = __half2; };
template <> struct Pair2<__nv_bfloat16> { using type = __nv_bfloat162; };

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
template <int NV, typename T2>
__device__ __forceinline__ void load_vec(const T2* p, float (&v)[NV]) {
  static_assert(sizeof(T2) == 2, "2-byte elements");
  using P2 = typename Pair2<T2>::type;
#pragma unroll
  for (int q = 0; q < NV / 8; ++q) {
    const uint4 t = reinterpret_cast<const uint4*>(p)[q];
    const P2* h = reinterpret_cast<const P2*>(&t);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = to_f2(h[e]);
      v[8 * q + 2 * e] = f.x;
      v[8 * q + 2 * e + 1] = f.y;
    }
  }
}

// A loaded row held as aligned column pairs (v[2q], v[2q+1]). Packed operands that start
// at an even column are these pairs. Odd-start pairs are never built: the compiler would
// re-assemble them with register moves at every use. Instead odd taps combine single
// elements with scalar instructions that write the two halves of a result pair directly.
template <int NV>
struct PairRow {
  float2 a[NV / 2];
  __device__ __forceinline__ void build(const float (&v)[NV]) {
#pragma unroll
    for (int q = 0; q < NV / 2; ++q) a[q] = make_float2(v[2 * q], v[2 * q + 1]);
  }
  __device__ __forceinline__ float el(int i) const { return (i & 1) ? a[i >> 1].y : a[i >> 1].x; }
  __device__ __forceinline__ float2 pr(int i) const { return a[i >> 1]; }  // i even
};

// For the output pair at columns (c, c+1), c even, and tap distance d:
// (v[c-d] + v[c+d], v[c+1-d] + v[c+1+d]).
template <int NV>
__device__ __forceinline__ float2 psum(const PairRow<NV>& V, int c, int d) {
  if ((d & 1) == 0) return add2(V.pr(c - d), V.pr(c + d));
  return make_float2(V.el(c - d) + V.el(c + d), V.el(c + 1 - d) + V.el(c + 1 + d));
}

// (fma(A[c+d], B[c+d], L[c-d]), fma(A[c+1+d], B[c+1+d], L[c+1-d])): the reference's
// ((Xl*Yl) + (Xr*Yr)) form of the squared and cross moments with L = A*B precomputed.
template <int NV>
__device__ __forceinline__ float2 pfma(const PairRow<NV>& A, const PairRow<NV>& B,
                                       const PairRow<NV>& L, int c, int d) {
  if ((d & 1) == 0) return fma2(A.pr(c + d), B.pr(c + d), L.pr(c - d));
  return make_float2(fmaf(A.el(c + d), B.el(c + d), L.el(c - d)),
                     fmaf(A.el(c + 1 + d), B.el(c + 1 + d), L.el(c + 1 - d)));
}

// Store a pair of adjacent columns (gx, gx+1) of one row; `pair` means both columns are in
// range and the address is aligned for a vector store.
template <typename I>
__device__ __forceinline__ void store2(float* base, I idx, float2 v, bool pair, bool in0,
                                      bool in1) {
  if (pair) {
    *reinterpret_cast<float2*>(base + idx) = v;
  } else {
    if (in0) base[idx] = v.x;
    if (in1) base[idx + 1] = v.y;
  }
}
template <typename I>
__device__ __forceinline__ void store2(__half* base, I idx, float2 v, bool pair, bool in0,
                                      bool in1) {
  if (pair) {
    *reinterpret_cast<__half2*>(base + idx) = __floats2half2_rn(v.x, v.y);
  } else {
    if (in0) base[idx] = __float2half_rn(v.x);
    if (in1) base[idx + 1] = __float2half_rn(v.y);
  }
}
template <typename I>
__device__ __forceinline__ void store2(__nv_bfloat16* base, I idx, float2 v, bool pair,
                                      bool in0, bool in1) {
  if (pair) {
    *reinterpret_cast<__nv_bfloat162*>(base + idx) = __floats2bfloat162_rn(v.x, v.y);
  } else {
    if (in0) base[idx] = __float2bfloat16_rn(v.x);
    if (in1) base[idx + 1] = __float2bfloat16_rn(v.y);
  }
}

template <typename T, typename I>
__device__ __forceinline__ float2 load2(const T* base, I idx, bool pair, bool in0, bool in1) {
  if (pair) {
    if constexpr (sizeof(T) == 4) {
      return __ldg(reinterpret_cast<const float2*>(base + idx));
    } else {
      using P2 = typename Pair2<T>::type;
      return to_f2(__ldg(reinterpret_cast<const P2*>(base + idx)));
    }
  }
  return make_float2(in0 ? to_f(base[idx]) : 0.f, in1 ? to_f(base[idx + 1]) : 0.f);
}

// ---------------------------------------------------------------------------------------
// Geometry and step sequencing
// ---------------------------------------------------------------------------------------
struct Geometry {
  int64_t H, W, HW;  // plane geometry (HW < 2^31, checked on the host)
  int64_t LT;        // strip-rows in the whole batch
  int S;             // strips per plane
  int C;             // channels per image
  int B;             // images
};

// Position of a CTA in its range: the column run (plane, strip), the part of it that
// belongs to the CTA (rows up to t_end) and the next step. 32-bit throughout (the host
// keeps planes and per-CTA ranges below 2^31) and advanced incrementally, so a step costs
// a handful of integer operations.
template <int HALO>
struct Step {
  int plane;      // plane of the current column run (image img, channel chan)
  int img, chan;
  int strip;
  int t;          // first output row of this step
  int n;          // output rows in this step (1..kRows); 0 = no step
  int t_end;      // end row of the CTA's part of this column run
  int rest;       // strip-rows of the CTA's range after that part
  int slot;       // first staging row of the step (0 or kRows)
  bool first;     // first step of a run part: it also computes the top halo rows
  __device__ __forceinline__ int h0() const { return first ? t - HALO : t + HALO; }  // first moment row
  __device__ __forceinline__ int nh() const { return first ? n + 2 * HALO : n; }     // moment rows
  __device__ __forceinline__ int hdst() const { return first ? 0 : 2 * HALO; }       // ring row of h0
  __device__ __forceinline__ bool last() const { return t + n == t_end; }  // last step of the part
};

// Start of CTA b's range of strip-rows (b = 0..G; b = G gives LT). The split is even in
// "work" rather than in rows: a column run part costs its rows plus about HALO rows for
// the halo rows its first step computes, so each run is counted as H + HALO units and a
// CTA boundary that would fall in a run's extra units moves to the next run's start.
// Boundaries inside a run are rounded down to whole steps, so only a run's last step is
// partial. Adjacent CTAs compute the shared boundary identically.
template <int HALO>
__device__ __forceinline__ int64_t cta_range_start(const Geometry& g, int64_t b, int64_t G) {
  const int64_t runs = g.LT / g.H;
  const int64_t per = g.H + HALO;
  const int64_t A = (runs * per * b) / G;
  const int64_t r = A / per;
  const int64_t o = A - r * per;
  if (o >= g.H) return (r + 1) * g.H;
  return r * g.H + (o / kRows) * kRows;
}

template <int HALO>
__device__ __forceinline__ Step<HALO> first_step(int64_t beg, int64_t end, const Geometry& g) {
  Step<HALO> s;
  const int64_t len = end - beg;
  if (len <= 0) {
    s.n = 0;
    return s;
  }
  const int64_t col = beg / g.H;
  s.t = static_cast<int>(beg - col * g.H);
  const int64_t plane = col / g.S;
  s.plane = static_cast<int>(plane);
  s.strip = static_cast<int>(col - plane * g.S);
  s.img = s.plane / g.C;
  s.chan = s.plane - s.img * g.C;
  const int64_t seg = (g.H - s.t) < len ? (g.H - s.t) : len;
  s.t_end = s.t + static_cast<int>(seg);
  s.rest = static_cast<int>(len - seg);
  s.slot = 0;
  s.first = true;
  s.n = static_cast<int>(seg) < kRows ? static_cast<int>(seg) : kRows;
  return s;
}

template <int HALO>
__device__ __forceinline__ Step<HALO> next_step(const Step<HALO>& c, const Geometry& g) {
  Step<HALO> s = c;
  s.t = c.t + c.n;
  s.first = false;
  if (s.t == c.t_end) {  // the CTA's part of this column run is done
    if (c.rest == 0) {
      s.n = 0;
      return s;
    }
    s.t = 0;
    s.first = true;
    if (++s.strip == g.S) {
      s.strip = 0;
      ++s.plane;
      if (++s.chan == g.C) {
        s.chan = 0;
        ++s.img;
      }
    }
    const int H = static_cast<int>(g.H);
    const int seg = c.rest < H ? c.rest : H;
    s.t_end = seg;
    s.rest = c.rest - seg;
  }
  const int r = s.t_end - s.t;
  s.n = r < kRows ? r : kRows;
  return s;
}

// Stage moment rows [h0, h0+nh) x columns [x0-8, x0+72) of NMAP planes into smem
// (layout [NMAP][MAXR][PITCH]) with the NT threads of the CTA; out-of-image elements
// become zero.
template <typename T, int NMAP, int MAXR, typename StepT, int NT = kThreads>
__device__ __forceinline__ void stage(T* sm, const T* const (&src)[NMAP], const Geometry& g,
                                      const StepT& s, bool aligned16) {
  constexpr int P = StagePitch<T>::value;
  const int x0 = s.strip * kStrip - kLeft;
  const int W = static_cast<int>(g.W);
  const int H = static_cast<int>(g.H);
  const int h0 = s.h0();
  if (aligned16) {
    constexpr int E = 16 / sizeof(T);   // elements per 16-byte chunk
    constexpr int CH = kInCols / E;      // chunks per staged row
    const int total = s.nh() * CH;
#pragma unroll
    for (int m = 0; m < NMAP; ++m) {
      const T* plane = src[m] + static_cast<int64_t>(s.plane) * g.HW;
      T* dst = sm + m * MAXR * P;
      for (int i = threadIdx.x; i < total; i += NT) {
        const int row = i / CH;
        const int ch = i - row * CH;
        const int gy = h0 + row;
        const int gx = x0 + ch * E;
        const bool in = (static_cast<unsigned>(gy) < static_cast<unsigned>(H)) &&
                        (static_cast<unsigned>(gx) < static_cast<unsigned>(W));
        const T* p = in ? plane + (gy * W + gx) : plane;
        cp_async16(dst + row * P + ch * E, p, in);
      }
    }
  } else if constexpr (sizeof(T) == 4) {
    const int total = s.nh() * kInCols;
#pragma unroll
    for (int m = 0; m < NMAP; ++m) {
      const T* plane = src[m] + static_cast<int64_t>(s.plane) * g.HW;
      T* dst = sm + m * MAXR * P;
      for (int i = threadIdx.x; i < total; i += NT) {
        const int row = i / kInCols;
        const int c = i - row * kInCols;
        const int gy = h0 + row;
        const int gx = x0 + c;
        const bool in = (static_cast<unsigned>(gy) < static_cast<unsigned>(H)) &&
                        (static_cast<unsigned>(gx) < static_cast<unsigned>(W));
        const T* p = in ? plane + (gy * W + gx) : plane;
        cp_async4(dst + row * P + c, p, in);
      }
    }
  } else {
    // 2-byte elements on an unaligned layout: plain loads.
    const int total = s.nh() * kInCols;
#pragma unroll
    for (int m = 0; m < NMAP; ++m) {
      const T* plane = src[m] + static_cast<int64_t>(s.plane) * g.HW;
      T* dst = sm + m * MAXR * P;
      for (int i = threadIdx.x; i < total; i += NT) {
        const int row = i / kInCols;
        const int c = i - row * kInCols;
        const int gy = h0 + row;
        const int gx = x0 + c;
        const bool in = (static_cast<unsigned>(gy) < static_cast<unsigned>(H)) &&
                        (static_cast<unsigned>(gx) < static_cast<unsigned>(W));
        dst[row * P + c] = in ? plane[gy * W + gx] : T(0.f);
      }
    }
  }
  cp_async_commit();
}

// Bytes the TMA staging of one step delivers for NMAP maps of element type T.
template <typename T, int NMAP>
__device__ __forceinline__ unsigned tma_step_bytes(int nh) {
  const int nbox = (nh + kBoxRows - 1) / kBoxRows;
  return static_cast<unsigned>(NMAP * nbox * kBoxRows * StagePitch<T>::value * sizeof(T));
}

// TMA staging of one step by the lanes of one warp, one box per lane: rows [h0, h0+nh)
// rounded up to whole boxes, columns [x0-8, x0-8+pitch) of plane s.plane for each of the
// NMAP tensor maps, into rows [slot, slot + nh) of the layout [NMAP][SROWS][pitch]; rows or
// columns outside the image arrive as zeros. Lane lane0 + m*nbox + b issues box b of map m. Every issuing lane first orders the CTA's
// earlier shared-memory reads of the slot (made visible by a CTA barrier) before its copy.
template <typename T, int NMAP, int SROWS, typename StepT>
__device__ __forceinline__ void stage_tma_lanes(T* sm, const CUtensorMap* maps, const StepT& s,
                                                uint64_t* bar, int lane0) {
  constexpr int P = StagePitch<T>::value;
  const int nbox = (s.nh() + kBoxRows - 1) / kBoxRows;
  const int l = static_cast<int>(threadIdx.x & 31) - lane0;
  if (l >= 0 && l < NMAP * nbox) {
    const int m = l / nbox;
    const int b = l - m * nbox;
    fence_proxy_async_smem();
    tma_load_3d(sm + (m * SROWS + s.slot + b * kBoxRows) * P, maps + m,
                s.strip * kStrip - kLeft, s.h0() + b * kBoxRows, s.plane, bar);
  }
}

// L2 prefetch of the boxes stage_tma_lanes would copy for step s (thread l < NMAP * nbox
// takes box l), issued before the wait for the previous kernel so the first staging hits
// L2. A hint: coordinates are clamped to the image.
template <typename StepT, int NMAP>
__device__ __forceinline__ void prefetch_step_boxes(const CUtensorMap* maps, const StepT& s,
                                                    int H) {
  const int nbox = (s.nh() + kBoxRows - 1) / kBoxRows;
  const int l = static_cast<int>(threadIdx.x);
  if (l < NMAP * nbox) {
    const int m = l / nbox;
    const int b = l - m * nbox;
    tma_prefetch_3d(maps + m, max(s.strip * kStrip - kLeft, 0),
                    min(max(s.h0() + b * kBoxRows, 0), H - 1), s.plane);
  }
}

// Copy ring rows [kRows, kRows + 2*HALO) to [0, 2*HALO): the vertical halo for the next
// step. Only full steps carry, and 2*HALO <= kRows, so source and destination are disjoint
// contiguous blocks.
template <int HALO, int RP>
__device__ __forceinline__ void ring_carry(float* ring) {
  static_assert(2 * HALO <= kRows, "carry source and destination must not overlap");
  static_assert((2 * HALO * RP) % 4 == 0 && (kRows * RP) % 4 == 0, "float4 carry");
  constexpr int N4 = 2 * HALO * RP / 4;
  const float4* src = reinterpret_cast<const float4*>(ring + kRows * RP);
  float4* dst = reinterpret_cast<float4*>(ring);
  for (int i = threadIdx.x; i < N4; i += kThreads) dst[i] = src[i];
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

// Deterministic block sums of two doubles at once (red holds 8 doubles).
__device__ __forceinline__ void block_sum2(double& a, double& b, double* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    red[warp] = a;
    red[4 + warp] = b;
  }
  __syncthreads();
  a = ((red[0] + red[1]) + red[2]) + red[3];
  b = ((red[4] + red[5]) + red[6]) + red[7];
}

// Vertical 2*HALO+1 tap sum of column pairs for kRPT consecutive output rows: rows k..k+2HALO
// of `v` feed output k (reference order: pairs d = 1..HALO, centre last).
template <int HALO, bool HW_>
__device__ __forceinline__ void vsumR(const float2 (&v)[kRPT + 2 * HALO], float2 (&o)[kRPT],
                                      const Taps2<HALO, HW_>& T) {
  // Tap distance outermost: the kRPT independent accumulation chains advance together, so
  // consecutive packed FMAs never wait on each other.
  float2 acc[kRPT];
#pragma unroll
  for (int k = 0; k < kRPT; ++k) acc[k] = make_float2(0.f, 0.f);
#pragma unroll
  for (int d = 1; d <= HALO; ++d) {
#pragma unroll
    for (int k = 0; k < kRPT; ++k)
      acc[k] = fma2(add2(v[k + HALO - d], v[k + HALO + d]), T.w[HALO - d], acc[k]);
  }
#pragma unroll
  for (int k = 0; k < kRPT; ++k) o[k] = fma2(v[k + HALO], T.w[HALO], acc[k]);
}

// ---------------------------------------------------------------------------------------
// Forward kernel
// ---------------------------------------------------------------------------------------
// ---------------------------------------------------------------------------------------
// Cross-GPU exchange of the per-rank SSIM sums (batch-sharded loss, one process per GPU)
// ---------------------------------------------------------------------------------------
// Every rank owns a mailbox in its own device memory, mapped into every other rank's
// process (CUDA IPC), of 2 x world slots of {double sum; u64 seq}. At the end of the
// forward, the last CTA stores the rank's sum into slot [seq & 1][rank] of every rank's
// mailbox over NVLink (value, system fence, then seq). A one-warp gather kernel on each rank
// waits, with a bounded poll, until all `world` slots of its own mailbox carry `seq`, then
// sums them in rank order: the same bits on every rank. Two slot sets suffice: a rank
// writes step seq+2 only after its gather of step seq+1, which needs every rank's step
// seq+1 sum, which each rank publishes only after its own gather of step seq.
constexpr int kMaxDpRanks = 8;
constexpr unsigned kErrGatherTimeout = 2u;

struct DpMailSlot {
  double sum;
  unsigned long long seq;
};

struct DpParams {
  DpMailSlot* mail[kMaxDpRanks];  // mailbox of rank r as mapped in this process
  int world;                      // 0: not sharded
  int rank;
  unsigned long long seq;
  unsigned long long timeout_ns;  // gather: give up after this long (device global timer)
};

// Nanoseconds of the device's global timer.
__device__ __forceinline__ unsigned long long global_timer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void dp_publish(const DpParams& dp, double sum) {
  const int set = static_cast<int>(dp.seq & 1ull);
  for (int r = 0; r < dp.world; ++r) {
    DpMailSlot* slot = dp.mail[r] + set * dp.world + dp.rank;
    *reinterpret_cast<volatile double*>(&slot->sum) = sum;
  }
  __threadfence_system();
  for (int r = 0; r < dp.world; ++r) {
    DpMailSlot* slot = dp.mail[r] + set * dp.world + dp.rank;
    *reinterpret_cast<volatile unsigned long long*>(&slot->seq) = dp.seq;
  }
}

// Publishes a sum computed without the forward kernel (an empty shard publishes 0).
__global__ void dp_publish_kernel(const DpParams dp, double sum) {
  if (threadIdx.x == 0 && blockIdx.x == 0) dp_publish(dp, sum);
}

// One warp: lane r < world waits for slot [seq & 1][r] of this rank's mailbox, then lane 0
// writes out[0] = scale * (sum of the world sums in rank order). The wait ends after
// dp.timeout_ns of the device's global timer: out[0] is then NaN and bit 1 of the device
// error flag is set.
__global__ void __launch_bounds__(32) dp_gather_kernel(const DpParams dp, float scale, float* out) {
  const int lane = threadIdx.x;
  const int set = static_cast<int>(dp.seq & 1ull);
  bool ok = true;
  double v = 0.0;
  if (lane < dp.world) {
    const DpMailSlot* slot = dp.mail[dp.rank] + set * dp.world + lane;
    const volatile unsigned long long* seqp =
        reinterpret_cast<const volatile unsigned long long*>(&slot->seq);
    const unsigned long long t0 = global_timer_ns();
    while (*seqp != dp.seq) {
      if (global_timer_ns() - t0 > dp.timeout_ns) break;
      __nanosleep(128);
    }
    ok = (*seqp == dp.seq);
    __threadfence_system();
    v = *reinterpret_cast<const volatile double*>(&slot->sum);
  }
  const bool all_ok = __all_sync(0xffffffffu, ok);
  if (!all_ok) {
    if (lane == 0) {
      atomicOr(&g_device_error, kErrGatherTimeout);
      out[0] = __int_as_float(0x7fc00000);  // NaN
    }
    return;
  }
  // rank-ordered sum (lane 0 reads the others' values through shuffles)
  double total = 0.0;
  for (int r = 0; r < dp.world; ++r) total += __shfl_sync(0xffffffffu, v, r);
  if (lane == 0) out[0] = static_cast<float>(total * static_cast<double>(scale));
}

struct FwdParams {
  CUtensorMap tmap[2];   // img1, img2 as (W, H, planes), boxes of kBoxRows rows (when use_tma)
  DpParams dp;           // sharded loss: publish the batch sum to every rank (dp.world > 0)
  const void* img1;
  const void* img2;
  float* map;            // optional per-pixel SSIM (unmasked)
  void* p0;              // optional partials (TP): dm_dmu1, dm_dsigma1_sq, dm_dsigma12
  void* p1;
  void* p2;
  float* out;            // reduction outputs
  double* image_sums;    // optional FP64 per-image sums
  unsigned long long* acc;  // B fixed-point accumulators (workspace)
  unsigned long long* acc_l1;  // B more for the L1 sums (workspace, used when l1)
  unsigned* ticket;         // last-CTA ticket (workspace)
  Geometry g;
  float C1, C2, out_scale;
  float l1_weight, out_offset;  // out = out_scale*sum(ssim) + l1_weight*sum|x-y| + out_offset
  int l1;                       // accumulate sum |x - y| (fused L1 term)
  int valid, clamp, reduce, mask_partials, aligned16, pair_ok, use_tma;
  int wait_limit;               // polls of a step's staging wait before the step fails
};

// MERGED (the fused loss path): the SSIM value and its partials depend on the second moments
// only through sigma1^2 + sigma2^2 (in B), so one map E[x^2 + y^2] replaces E[x^2] and
// E[y^2]: 4 filtered maps instead of 5. Its FP32 rounding error against an exact result is
// the same size as that of the separate maps (both are dominated by the cancellation in
// E[.] - mu^2). The map-producing reference entry points keep the reference's 5 maps
// (MERGED = false) so their per-pixel outputs follow its arithmetic order exactly.
template <int HALO, typename TIn, typename TP, bool TRAIN, bool MERGED>
struct FwdConfig {
  static constexpr bool kHalfW = HalfTaps<TIn>::value;
  static constexpr int kMaps = MERGED ? 4 : 5;
  static constexpr int kMaxR = MaxRows<HALO>::value;
  static constexpr int kSRows = StageRows<HALO>::value;
  // a first step's boxes fit the staging rows; a regular step's boxes fit one slot
  static_assert(kSRows >= (kMaxR + kBoxRows - 1) / kBoxRows * kBoxRows, "staging rows");
  static_assert(kRows % kBoxRows == 0 && kSRows >= 2 * kRows, "staging slots");
  static constexpr int kSP = StagePitch<TIn>::value;
  static constexpr int kRP = RingPitch<kMaps>::value;
  static constexpr size_t kStageBytes = 2ull * kSRows * kSP * sizeof(TIn);
  static constexpr size_t kRingBytes = static_cast<size_t>(kMaxR) * kRP * sizeof(float);
  // + 128: the dynamic shared memory base is rounded up to 128 bytes for the TMA boxes
  static constexpr size_t kSmem = kStageBytes + kRingBytes + 128;
  // resident CTAs per SM the kernel is compiled for (228 KB of shared memory per SM)
  static constexpr int kFit = static_cast<int>((228 * 1024) / (kSmem + 1024));
  static constexpr int kMinBlocks = kFit >= 4 ? 4 : (kFit >= 3 ? 3 : 2);
};

// Horizontal pass of the forward: for staged row i and output columns 8j..8j+7 compute the
// moments sum w*X, w*X^2, w*Y, w*Y^2, w*XY (order of the reference's xconv features), or
// with MERGED sum w*X, w*(X^2+Y^2), w*Y, w*XY, as four column pairs.
// With l1 set it also adds |x - y| of the task's 8 centre pixels to l1_sum, for staged rows
// [l1_i0, l1_i1) and the strip's first l1_cols columns (each image pixel is counted by
// exactly one task of one step).
template <int HALO, typename TIn, int MAXR, bool MERGED>
__device__ __forceinline__ void fwd_hpass(const TIn* sx, const TIn* sy, float* ring, int nh,
                                          int hdst, const Taps2<HALO, HalfTaps<TIn>::value>& T,
                                          bool l1, int l1_i0, int l1_i1, int l1_cols,
                                          float& l1_sum) {
  constexpr int SP = StagePitch<TIn>::value;
  constexpr int RP = RingPitch<MERGED ? 4 : 5>::value;
  constexpr int HA = (sizeof(TIn) == 2 || HALO > 4) ? 8 : 4;  // aligned left extent
  constexpr int NV = 8 + 2 * HA;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int rg = 0; rg < nh; rg += kRG) {
    const int i = rg + lane % kRG;
    if (i < nh) {
#pragma unroll 1
      for (int jj = 0; jj < kJJ; ++jj) {
        const int j = warp + 4 * (lane / kRG) + 4 * kLG * jj;
        float xv[NV], yv[NV];
        load_vec(sx + i * SP + 8 * j + kLeft - HA, xv);
        load_vec(sy + i * SP + 8 * j + kLeft - HA, yv);
        PairRow<NV> X, Y, XX, YY, XY;
        X.build(xv);
        Y.build(yv);
#pragma unroll
        for (int q = 0; q < NV / 2; ++q) {
          XX.a[q] = mul2(X.a[q], X.a[q]);
          XY.a[q] = mul2(X.a[q], Y.a[q]);
          YY.a[q] = MERGED ? fma2(Y.a[q], Y.a[q], XX.a[q]) : mul2(Y.a[q], Y.a[q]);
        }
        if (l1 && i >= l1_i0 && i < l1_i1) {
          const int nc = l1_cols - 8 * j;  // centre columns of the task inside the image
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 dv = sub2(X.pr(HA + 2 * q), Y.pr(HA + 2 * q));
            l1_sum += (2 * q < nc ? fabsf(dv.x) : 0.f) + (2 * q + 1 < nc ? fabsf(dv.y) : 0.f);
          }
        }
        float* dst = ring + (hdst + i) * RP + 8 * j;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int c = HA + 2 * p;  // first column of the output pair (even)
          const float2 wc = T.w[HALO];
          float2 sX = make_float2(0.f, 0.f), sY = sX, sXY = sX, s2a = sX, s2b = sX;
#pragma unroll
          for (int d = 1; d <= HALO; ++d) {
            const float2 w = T.w[HALO - d];
            sX = fma2(psum(X, c, d), w, sX);
            sY = fma2(psum(Y, c, d), w, sY);
            sXY = fma2(pfma(X, Y, XY, c, d), w, sXY);
            if constexpr (MERGED) {
              s2a = fma2(psum(YY, c, d), w, s2a);  // YY holds x^2 + y^2
            } else {
              s2a = fma2(pfma(X, X, XX, c, d), w, s2a);
              s2b = fma2(pfma(Y, Y, YY, c, d), w, s2b);
            }
          }
          // ring maps: MERGED 0 = X, 1 = X^2+Y^2, 2 = Y, 3 = XY; else X, X^2, Y, Y^2, XY
          *reinterpret_cast<float2*>(dst + 0 * kStrip + 2 * p) = fma2(X.pr(c), wc, sX);
          *reinterpret_cast<float2*>(dst + 2 * kStrip + 2 * p) = fma2(Y.pr(c), wc, sY);
          if constexpr (MERGED) {
            *reinterpret_cast<float2*>(dst + 1 * kStrip + 2 * p) = fma2(YY.pr(c), wc, s2a);
            *reinterpret_cast<float2*>(dst + 3 * kStrip + 2 * p) = fma2(XY.pr(c), wc, sXY);
          } else {
            *reinterpret_cast<float2*>(dst + 1 * kStrip + 2 * p) = fma2(XX.pr(c), wc, s2a);
            *reinterpret_cast<float2*>(dst + 3 * kStrip + 2 * p) = fma2(YY.pr(c), wc, s2b);
            *reinterpret_cast<float2*>(dst + 4 * kStrip + 2 * p) = fma2(XY.pr(c), wc, sXY);
          }
        }
      }
    }
  }
}

template <int HALO, typename TIn, typename TP, bool TRAIN, bool MERGED>
__global__ void __launch_bounds__(kThreads, (FwdConfig<HALO, TIn, TP, TRAIN, MERGED>::kMinBlocks))
    ssim_fwd_kernel(const __grid_constant__ FwdParams a) {
  using Cfg = FwdConfig<HALO, TIn, TP, TRAIN, MERGED>;
  constexpr int NM = Cfg::kMaps;
  constexpr int SROWS = Cfg::kSRows;
  constexpr int SP = Cfg::kSP;
  constexpr int RP = Cfg::kRP;
  constexpr bool HW_ = Cfg::kHalfW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
  TIn* stg = reinterpret_cast<TIn*>(smem);
  float* ring = reinterpret_cast<float*>(smem + Cfg::kStageBytes);
  __shared__ double red[8];
  __shared__ unsigned s_last;
  __shared__ uint64_t bar;

  const Geometry& g = a.g;
  const int64_t beg = cta_range_start<HALO>(g, blockIdx.x, gridDim.x);
  const int64_t end = cta_range_start<HALO>(g, blockIdx.x + 1, gridDim.x);
  const TIn* const src[2] = {static_cast<const TIn*>(a.img1), static_cast<const TIn*>(a.img2)};
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = warp * kRPT;
  const float2 C1v = splat(a.C1), C2v = splat(a.C2), two = splat(2.f);
  Taps2<HALO, HW_> T;
  T.load();

  const bool tma = a.use_tma != 0;
  if (tma && threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  Step<HALO> cur = first_step<HALO>(beg, end, g);
  if (tma && threadIdx.x < 2) prefetch_tensormap(a.tmap + threadIdx.x);
  // the first step's boxes into L2 while the previous kernel finishes
  if (tma && cur.n) prefetch_step_boxes<Step<HALO>, 2>(a.tmap, cur, static_cast<int>(g.H));
  grid_dependency_wait();
  grid_launch_dependents();
  // TMA staging of a step by warp 0: lane 0 posts the byte count, the lanes issue the boxes
  auto issue = [&](const Step<HALO>& st) {
    if (warp == 0) {
      if (lane == 0) mbar_arrive_expect_tx(&bar, tma_step_bytes<TIn, 2>(st.nh()));
      stage_tma_lanes<TIn, 2, SROWS>(stg, a.tmap, st, &bar, 0);
    }
  };
  if (cur.n) {
    if (!tma) {
      stage<TIn, 2, SROWS>(stg, src, g, cur, a.aligned16);
    } else {
      issue(cur);
    }
  }
  unsigned phase = 0;
  double run_sum = 0.0;
  double run_l1 = 0.0;
  const bool l1 = a.l1 != 0;
  bool failed = false;

  while (cur.n) {
    bool timed_out = false;
    if (tma) {
      timed_out = !mbar_wait_bounded(&bar, phase, a.wait_limit);
      phase ^= 1u;
    } else {
      cp_async_wait_all();
    }
    if (__syncthreads_or(timed_out)) {
      // staging did not complete: report it, give the copies in flight one more bounded
      // wait so none lands after the CTA has exited, and stop; the CTA still takes its
      // reduction ticket below, so the last CTA turns the outputs into NaN and leaves
      // the workspace zeroed for the next call
      if (threadIdx.x == 0) atomicOr(&g_device_error, kErrStagingTimeout);
      mbar_wait_bounded(&bar, phase ^ 1u, kWaitLimit);
      failed = true;
      break;
    }
    // The next step is staged into the other slot while this step's H-pass runs, unless
    // one of the two is the first step of a column run (which fills both slots); then it
    // is staged after the H-pass.
    Step<HALO> nxt = next_step<HALO>(cur, g);
    const bool early = tma && nxt.n && !cur.first && !nxt.first;
    nxt.slot = early ? (cur.slot ^ kRows) : 0;
    if (early) issue(nxt);
    float step_l1 = 0.f;
    {
      // L1 term: staged rows of the CTA's own output rows [segment start, t_end)
      const int l1_i0 = cur.first ? HALO : 0;
      const int l1_hi = cur.t_end - cur.h0();
      const int l1_i1 = l1_hi < cur.nh() ? l1_hi : cur.nh();
      const int l1_cols = static_cast<int>(g.W) - cur.strip * kStrip;
      fwd_hpass<HALO, TIn, SROWS, MERGED>(stg + cur.slot * SP, stg + (SROWS + cur.slot) * SP,
                                          ring, cur.nh(), cur.hdst(), T, l1, l1_i0, l1_i1,
                                          l1_cols, step_l1);
    }
    run_l1 += static_cast<double>(step_l1);
    __syncthreads();
    if (nxt.n && !early) {
      if (!tma) {
        stage<TIn, 2, SROWS>(stg, src, g, nxt, a.aligned16);
      } else {
        issue(nxt);
      }
    }

    // ---- V-pass + epilogue: rows r0..r0+kRPT-1 of the step, columns 2*lane, 2*lane+1 ----
    if (r0 < cur.n) {
      float2 res[NM][kRPT];
#pragma unroll
      for (int m = 0; m < NM; ++m) {
        float2 v[kRPT + 2 * HALO];
#pragma unroll
        for (int q = 0; q < kRPT + 2 * HALO; ++q)
          v[q] = *reinterpret_cast<const float2*>(ring + (r0 + q) * RP + m * kStrip + 2 * lane);
        vsumR<HALO, HW_>(v, res[m], T);
      }
      const int gx0 = cur.strip * kStrip + 2 * lane;
      const int W = static_cast<int>(g.W);
      const bool in0 = gx0 < W, in1 = gx0 + 1 < W;
      const bool pair = a.pair_ok && in1;
      // columns counted in the reduction / receiving gradient (valid crop)
      const bool col0 = in0 && (!a.valid || (gx0 >= HALO && gx0 < W - HALO));
      const bool col1 = in1 && (!a.valid || (gx0 + 1 >= HALO && gx0 + 1 < W - HALO));
      // step rows inside the valid crop: [rlo, rhi) in step-local row numbers
      int rlo = 0, rhi = cur.n;
      if (a.valid) {
        rlo = max(0, HALO - cur.t);
        rhi = min(cur.n, static_cast<int>(g.H) - HALO - cur.t);
      }
      // outputs addressed as plane base + 32-bit in-plane offset (planes < 2^31 elements)
      const int64_t plane_off = static_cast<int64_t>(cur.plane) * g.HW;
      const int off0 = (cur.t + r0) * W + gx0;
      float* mapp = a.map ? a.map + plane_off : nullptr;
      TP* q0 = TRAIN ? static_cast<TP*>(a.p0) + plane_off : nullptr;
      TP* q1 = TRAIN ? static_cast<TP*>(a.p1) + plane_off : nullptr;
      TP* q2 = TRAIN ? static_cast<TP*>(a.p2) + plane_off : nullptr;
      const float2 neg1 = splat(-1.f);
      // SSIM value and (TRAIN) its three partials for output row k of this thread
      auto pixel = [&](int k, float2& v, float2& pm, float2& ps, float2& pc) {
        const float2 mu1 = res[0][k], mu2 = res[2][k];
        const float2 mu1_sq = mul2(mu1, mu1), mu2_sq = mul2(mu2, mu2);
        const float2 msq = add2(mu1_sq, mu2_sq);
        const float2 mu12 = mul2(mu1, mu2);
        const float2 A = add2(msq, C1v);
        float2 B, sigma12;
        // differences as fma(b, -1, a): the same single rounding as a - b
        if constexpr (MERGED) {
          B = add2(fma2(msq, neg1, res[1][k]), C2v);
          sigma12 = fma2(mu12, neg1, res[3][k]);
        } else {
          const float2 sigma1_sq = fma2(mu1_sq, neg1, res[1][k]);
          const float2 sigma2_sq = fma2(mu2_sq, neg1, res[3][k]);
          B = add2(add2(sigma1_sq, sigma2_sq), C2v);
          sigma12 = fma2(mu12, neg1, res[NM - 1][k]);
        }
        const float2 Cc = fma2(two, mu12, C1v);
        const float2 D = fma2(two, sigma12, C2v);
        const float2 rA = make_float2(rcp_approx(A.x), rcp_approx(A.y));
        const float2 rB = make_float2(rcp_approx(B.x), rcp_approx(B.y));
        const float2 rAB = mul2(rA, rB);
        v = mul2(mul2(Cc, D), rAB);
        if (TRAIN) {
          // dm/dmu1 = 2 mu2 (D - C) / (AB) + 2 mu1 v (1/B - 1/A); dm/dsigma1^2 = -v / B;
          // dm/dsigma12 = 2 C / (AB)   (csrc/ssim.cu:323-330, with v = CD/(AB))
          pm = fma2(mul2(two, mu2), mul2(fma2(Cc, neg1, D), rAB),
                    mul2(mul2(two, mu1), mul2(v, fma2(rA, neg1, rB))));
          ps = mul2(mul2(v, neg1), rB);
          pc = mul2(mul2(two, Cc), rAB);
        }
      };
      // A full step of a strip that lies inside the image (and inside the valid crop),
      // without the clamp, needs no masks: every output is stored and summed as a pair.
      const int sx0 = cur.strip * kStrip;
      const bool fast =
          cur.n == kRows && a.pair_ok && !a.clamp && sx0 + kStrip <= W &&
          (!a.valid || (cur.t >= HALO && cur.t + kRows <= static_cast<int>(g.H) - HALO &&
                        sx0 >= HALO && sx0 + kStrip <= W - HALO));
      float step_sum = 0.f;
      if (fast) {
#pragma unroll
        for (int k = 0; k < kRPT; ++k) {
          float2 v, pm, ps, pc;
          pixel(k, v, pm, ps, pc);
          if (a.reduce) step_sum += v.x + v.y;
          const int off = off0 + k * W;
          if (mapp) store2(mapp, off, v, true, true, true);
          if (TRAIN) {
            store2(q0, off, pm, true, true, true);
            store2(q1, off, ps, true, true, true);
            store2(q2, off, pc, true, true, true);
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < kRPT; ++k) {
          const int row = r0 + k;
          if (row < cur.n) {
            const bool row_ok = row >= rlo && row < rhi;
            float2 v, pm, ps, pc;
            pixel(k, v, pm, ps, pc);
            const bool c0 = row_ok && col0, c1 = row_ok && col1;
            if (a.reduce) {
              const float v0 = (a.clamp && v.x < 0.f) ? 0.f : v.x;
              const float v1 = (a.clamp && v.y < 0.f) ? 0.f : v.y;
              step_sum += (c0 ? v0 : 0.f) + (c1 ? v1 : 0.f);
            }
            const int off = off0 + k * W;
            if (mapp) store2(mapp, off, v, pair, in0, in1);
            if (TRAIN) {
              const bool live0 = !a.mask_partials || (c0 && (!a.clamp || v.x >= 0.f));
              const bool live1 = !a.mask_partials || (c1 && (!a.clamp || v.y >= 0.f));
              if (!live0) pm.x = ps.x = pc.x = 0.f;
              if (!live1) pm.y = ps.y = pc.y = 0.f;
              store2(q0, off, pm, pair, in0, in1);
              store2(q1, off, ps, pair, in0, in1);
              store2(q2, off, pc, pair, in0, in1);
            }
          }
        }
      }
      run_sum += static_cast<double>(step_sum);
    }

    if (a.reduce && cur.last()) {
      // end of a column run: fold its sum into the image's fixed-point accumulator
      double s = run_sum, s1 = run_l1;
      if (l1) {
        block_sum2(s, s1, red);
      } else {
        s = block_sum(s, red);
      }
      run_sum = 0.0;
      run_l1 = 0.0;
      if (threadIdx.x == 0) {
        const long long q = __double2ll_rn(s * kFixScale);
        atomicAdd(a.acc + cur.img, static_cast<unsigned long long>(q));
        if (l1) {
          const long long q1 = __double2ll_rn(s1 * kFixScaleL1);
          atomicAdd(a.acc_l1 + cur.img, static_cast<unsigned long long>(q1));
        }
      }
    }
    __syncthreads();
    if (!cur.last()) ring_carry<HALO, RP>(ring);
    cur = nxt;
  }

  if (!a.reduce) return;
  __syncthreads();
  if (threadIdx.x == 0) {
    // One atomic per CTA on the ticket word: finished CTAs in its low 16 bits, CTAs that
    // gave up in its high 16 bits (grids stay below 2^16 CTAs, checked on the host). Its
    // release half orders this CTA's accumulator atomics before the count, its acquire
    // half (last CTA) every counted CTA's before what follows; the last CTA re-zeroes it.
    const unsigned add = failed ? 0x10001u : 1u;
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;\n"
                 : "=r"(prev)
                 : "l"(a.ticket), "r"(add)
                 : "memory");
    const bool last = (prev & 0xffffu) == gridDim.x - 1;
    if (last) *a.ticket = 0u;
    s_last = !last ? 0u : ((prev >> 16) != 0u || failed) ? 2u : 1u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // a CTA of this call gave up: every output of the call is NaN (the accumulators are
  // still zeroed for the next call)
  const double poison = s_last == 2u ? __longlong_as_double(0x7ff8000000000000ll) : 0.0;
  double local = 0.0, local_l1 = 0.0;
  for (int b = threadIdx.x; b < g.B; b += kThreads) {
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
    double total = local, total_l1 = local_l1;
    block_sum2(total, total_l1, red);
    if (threadIdx.x == 0) {
      a.out[0] = static_cast<float>(total * static_cast<double>(a.out_scale) +
                                    total_l1 * static_cast<double>(a.l1_weight) +
                                    static_cast<double>(a.out_offset));
      if (a.dp.world > 0) dp_publish(a.dp, total);
    }
  }
}

// ---------------------------------------------------------------------------------------
// Backward kernel
// ---------------------------------------------------------------------------------------
struct BwdParams {
  CUtensorMap tmap[4];    // p0, p1, p2 (TP) and dl (FP32) as (W, H, planes) (when use_tma)
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
  float l1_scale;         // fused L1 term: adds l1_scale * upstream * sign(x - y) (0: none)
  int grad_per_image, grad_dtype, aligned16, pair_ok, use_tma;
  int wait_limit;         // polls of a step's staging wait before the step fails
};

template <int HALO, typename TIn, typename TP, bool DLMAP>
struct BwdConfig {
  static constexpr bool kHalfW = HalfTaps<TIn>::value;
  static constexpr int kMaxR = MaxRows<HALO>::value;
  static constexpr int kSRows = StageRows<HALO>::value;
  // a first step's boxes fit the staging rows; a regular step's boxes fit one slot
  static_assert(kSRows >= (kMaxR + kBoxRows - 1) / kBoxRows * kBoxRows, "staging rows");
  static_assert(kRows % kBoxRows == 0 && kSRows >= 2 * kRows, "staging slots");
  static constexpr int kSP = StagePitch<TP>::value;
  static constexpr int kRP = RingPitch<3>::value;
  static constexpr size_t kStageBytes = 3ull * kSRows * kSP * sizeof(TP);
  static constexpr size_t kDlBytes =
      DLMAP ? static_cast<size_t>(kSRows) * StagePitch<float>::value * sizeof(float) : 0;
  static constexpr size_t kRingBytes = static_cast<size_t>(kMaxR) * kRP * sizeof(float);
  // + 128: the dynamic shared memory base is rounded up to 128 bytes for the TMA boxes
  static constexpr size_t kSmem = kStageBytes + kDlBytes + kRingBytes + 128;
  static constexpr int kFit = static_cast<int>((228 * 1024) / (kSmem + 1024));
  // compiled with the register budget of 3 CTAs/SM: ptxas then schedules the backward
  // better (1 us faster at 1080p) and still uses only ~110 registers, so 4 CTAs/SM fit
  static constexpr int kMinBlocks = kFit >= 3 ? 3 : 2;
};

// Horizontal pass of the backward over the three partial maps (times dL/dmap on the
// general path, as the reference multiplies at load, csrc/ssim.cu:408-411).
template <int HALO, typename TIn, typename TP, bool DLMAP, int MAXR>
__device__ __forceinline__ void bwd_hpass(const TP* sp, const float* sdl, float* ring, int nh,
                                          int hdst, const Taps2<HALO, HalfTaps<TIn>::value>& T) {
  constexpr int SP = StagePitch<TP>::value;
  constexpr int RP = RingPitch<3>::value;
  constexpr int HA = (sizeof(TP) == 2 || HALO > 4) ? 8 : 4;
  constexpr int NV = 8 + 2 * HA;
  // The general path only exists for FP32 partials, so dL and the partials share the
  // staged layout (same pitch, same aligned left extent HA).
  static_assert(!DLMAP || sizeof(TP) == 4, "per-pixel dL/dmap needs FP32 partials");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int rg = 0; rg < nh; rg += kRG) {
    const int i = rg + lane % kRG;
    if (i < nh) {
#pragma unroll 1
      for (int jj = 0; jj < kJJ; ++jj) {
        const int j = warp + 4 * (lane / kRG) + 4 * kLG * jj;
        float dl[NV];
        if (DLMAP) load_vec(sdl + i * StagePitch<float>::value + 8 * j + kLeft - HA, dl);
        float* dst = ring + (hdst + i) * RP + 8 * j;
#pragma unroll
        for (int m = 0; m < 3; ++m) {
          float v[NV];
          load_vec(sp + (m * MAXR + i) * SP + 8 * j + kLeft - HA, v);
          if (DLMAP) {
#pragma unroll
            for (int q = 0; q < NV; ++q) v[q] = v[q] * dl[q];
          }
          PairRow<NV> V;
          V.build(v);
          float2 s4[4];
#pragma unroll
          for (int p = 0; p < 4; ++p) s4[p] = make_float2(0.f, 0.f);
          // tap distance outermost: the 4 output pairs' chains advance together
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

template <int HALO, typename TIn, typename TP, bool DLMAP>
__global__ void __launch_bounds__(kThreads, (BwdConfig<HALO, TIn, TP, DLMAP>::kMinBlocks))
    ssim_bwd_kernel(const __grid_constant__ BwdParams a) {
  using Cfg = BwdConfig<HALO, TIn, TP, DLMAP>;
  constexpr int SROWS = Cfg::kSRows;
  constexpr int RP = Cfg::kRP;
  constexpr bool HW_ = Cfg::kHalfW;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u);
  TP* stg = reinterpret_cast<TP*>(smem);
  float* sdl = reinterpret_cast<float*>(smem + Cfg::kStageBytes);
  float* ring = reinterpret_cast<float*>(smem + Cfg::kStageBytes + Cfg::kDlBytes);
  __shared__ uint64_t bar;

  const Geometry& g = a.g;
  const int64_t beg = cta_range_start<HALO>(g, blockIdx.x, gridDim.x);
  const int64_t end = cta_range_start<HALO>(g, blockIdx.x + 1, gridDim.x);
  const TP* const src[3] = {static_cast<const TP*>(a.p0), static_cast<const TP*>(a.p1),
                            static_cast<const TP*>(a.p2)};
  const float* const dsrc[1] = {a.dl};
  const TIn* img1 = static_cast<const TIn*>(a.img1);
  const TIn* img2 = static_cast<const TIn*>(a.img2);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r0 = warp * kRPT;
  const float2 two = splat(2.f);
  Taps2<HALO, HW_> T;
  T.load();

  const bool tma = a.use_tma != 0;
  if (tma && threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  Step<HALO> cur = first_step<HALO>(beg, end, g);
  if (tma && threadIdx.x < (DLMAP ? 4 : 3)) prefetch_tensormap(a.tmap + threadIdx.x);
  // the first step's partial boxes into L2 while the previous kernel finishes
  if (tma && cur.n) prefetch_step_boxes<Step<HALO>, 3>(a.tmap, cur, static_cast<int>(g.H));
  grid_dependency_wait();
  grid_launch_dependents();
  // TMA staging of a step by warp 0: lane 0 posts the byte count, the lanes issue the boxes
  auto issue = [&](const Step<HALO>& st) {
    if (warp == 0) {
      if (lane == 0)
        mbar_arrive_expect_tx(&bar, tma_step_bytes<TP, 3>(st.nh()) +
                                        (DLMAP ? tma_step_bytes<float, 1>(st.nh()) : 0u));
      stage_tma_lanes<TP, 3, SROWS>(stg, a.tmap, st, &bar, 0);
      if (DLMAP) {
        const int nbox = (st.nh() + kBoxRows - 1) / kBoxRows;
        stage_tma_lanes<float, 1, SROWS>(sdl, a.tmap + 3, st, &bar, 3 * nbox);
      }
    }
  };
  if (cur.n) {
    if (!tma) {
      stage<TP, 3, SROWS>(stg, src, g, cur, a.aligned16);
      if (DLMAP) stage<float, 1, SROWS>(sdl, dsrc, g, cur, a.aligned16);
    } else {
      issue(cur);
    }
  }
  unsigned phase = 0;
  while (cur.n) {
    bool timed_out = false;
    if (tma) {
      timed_out = !mbar_wait_bounded(&bar, phase, a.wait_limit);
      phase ^= 1u;
    } else {
      cp_async_wait_all();
    }
    if (__syncthreads_or(timed_out)) {
      // staging did not complete: report it, give the copies in flight one more bounded
      // wait so none lands after the CTA has exited, and leave (the rest of the CTA's
      // gradient range is not written)
      if (threadIdx.x == 0) atomicOr(&g_device_error, kErrStagingTimeout);
      mbar_wait_bounded(&bar, phase ^ 1u, kWaitLimit);
      return;
    }
    // This step's epilogue operands: the image pairs of the thread's output pixels. The
    // loads are issued before the H-pass, so they are in flight while both passes run.
    const int W = static_cast<int>(g.W);
    const int gx0 = cur.strip * kStrip + 2 * lane;
    const bool in0 = gx0 < W, in1 = gx0 + 1 < W;
    const bool pair = a.pair_ok && in1;
    // a full step of a strip inside the image: no masks, pair loads and stores
    const bool fast = cur.n == kRows && a.pair_ok && cur.strip * kStrip + kStrip <= W;
    const int64_t plane_off = static_cast<int64_t>(cur.plane) * g.HW;
    // plane base + 32-bit in-plane offsets (planes < 2^31 elements)
    const int off0 = (cur.t + r0) * W + gx0;
    float2 xin[kRPT], yin[kRPT];
    {
      const TIn* x_pl = img1 + plane_off;
      const TIn* y_pl = img2 + plane_off;
      if (fast) {
#pragma unroll
        for (int k = 0; k < kRPT; ++k) {
          xin[k] = load2(x_pl, off0 + k * W, true, true, true);
          yin[k] = load2(y_pl, off0 + k * W, true, true, true);
        }
      } else {
#pragma unroll
        for (int k = 0; k < kRPT; ++k) {
          xin[k] = make_float2(0.f, 0.f);
          yin[k] = xin[k];
          if (r0 + k < cur.n) {
            xin[k] = load2(x_pl, off0 + k * W, pair, in0, in1);
            yin[k] = load2(y_pl, off0 + k * W, pair, in0, in1);
          }
        }
      }
    }
    // next step staged into the other slot during the H-pass (see the forward kernel)
    Step<HALO> nxt = next_step<HALO>(cur, g);
    const bool early = tma && nxt.n && !cur.first && !nxt.first;
    nxt.slot = early ? (cur.slot ^ kRows) : 0;
    if (early) issue(nxt);
    bwd_hpass<HALO, TIn, TP, DLMAP, SROWS>(stg + cur.slot * Cfg::kSP,
                                           sdl + cur.slot * StagePitch<float>::value, ring,
                                           cur.nh(), cur.hdst(), T);
    __syncthreads();
    if (nxt.n && !early) {
      if (!tma) {
        stage<TP, 3, SROWS>(stg, src, g, nxt, a.aligned16);
        if (DLMAP) stage<float, 1, SROWS>(sdl, dsrc, g, nxt, a.aligned16);
      } else {
        issue(nxt);
      }
    }

    if (r0 < cur.n) {
      float2 chain = splat(a.chain_scale);
      float2 l1c = splat(a.l1_scale);
      if (!DLMAP && a.grad_out) {
        const float2 up = splat(a.grad_out[a.grad_per_image ? cur.img : 0]);
        chain = mul2(chain, up);
        l1c = mul2(l1c, up);
      }
      float2 res[3][kRPT];
#pragma unroll
      for (int m = 0; m < 3; ++m) {
        float2 v[kRPT + 2 * HALO];
#pragma unroll
        for (int q = 0; q < kRPT + 2 * HALO; ++q)
          v[q] = *reinterpret_cast<const float2*>(ring + (r0 + q) * RP + m * kStrip + 2 * lane);
        vsumR<HALO, HW_>(v, res[m], T);
      }
      float2 gv[kRPT];
#pragma unroll
      for (int k = 0; k < kRPT; ++k) {
        gv[k] = fma2(yin[k], res[2][k], fma2(mul2(two, xin[k]), res[1][k], res[0][k]));
        if (!DLMAP) gv[k] = mul2(gv[k], chain);
      }
      if (!DLMAP && a.l1_scale != 0.f) {
        // d|x - y|/dx = sign(x - y), 0 where x == y (torch's abs backward)
#pragma unroll
        for (int k = 0; k < kRPT; ++k) {
          const float2 dv = sub2(xin[k], yin[k]);
          const float2 sg = make_float2(dv.x > 0.f ? 1.f : (dv.x < 0.f ? -1.f : 0.f),
                                        dv.y > 0.f ? 1.f : (dv.y < 0.f ? -1.f : 0.f));
          gv[k] = fma2(sg, l1c, gv[k]);
        }
      }
      auto store_grad = [&](auto* base) {
        auto* gp = base + plane_off;
        if (fast) {
#pragma unroll
          for (int k = 0; k < kRPT; ++k) store2(gp, off0 + k * W, gv[k], true, true, true);
        } else {
#pragma unroll
          for (int k = 0; k < kRPT; ++k)
            if (r0 + k < cur.n) store2(gp, off0 + k * W, gv[k], pair, in0, in1);
        }
      };
      if (a.grad_dtype == 0)
        store_grad(static_cast<float*>(a.grad));
      else if (a.grad_dtype == 1)
        store_grad(static_cast<__half*>(a.grad));
      else
        store_grad(static_cast<__nv_bfloat16*>(a.grad));
    }
    __syncthreads();
    if (!cur.last()) ring_carry<HALO, RP>(ring);
    cur = nxt;
  }
}

}  // namespace fssim
