// C ABI of the B200 SSIM engine: argument checks, launch configuration, dispatch over
// window size / element types, and the extern "C" entry points declared in
// include/fussim_b200.h. No torch, no Python: any host language can bind this library.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include <atomic>
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "fussim_b200.h"
#include "ssim_kernels.cuh"
#include "ssim_stream.cuh"

namespace {

thread_local std::string g_last_error;

// NVTX range over an entry point's host-side work (argument checks and launches), so a
// timeline tool shows the forward, backward and cross-GPU exchange by name. Without a tool
// attached a push/pop costs a few nanoseconds.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

std::string window_message(int ws) {
  // Same text as the reference's dispatch (csrc/ssim.cu:617).
  return "window_size must be 7, 9, or 11, got " + std::to_string(ws);
}

int check_window(int ws) {
  if (ws == 7 || ws == 9 || ws == 11) return FSSIM_OK;
  return fail(FSSIM_ERR_WINDOW, window_message(ws));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Shape checks shared by every entry point. Rows and columns are 32-bit inside the kernels.
int check_shape(int64_t B, int64_t C, int64_t H, int64_t W) {
  if (B < 0 || C < 0 || H < 0 || W < 0) return fail(FSSIM_ERR_SHAPE, "negative dimension");
  if (H > (INT_MAX / 2) || W > (INT_MAX / 2) || C > INT_MAX || B > INT_MAX)
    return fail(FSSIM_ERR_SHAPE, "dimension too large (H, W must be < 2^30)");
  if (H * W > static_cast<int64_t>(INT_MAX))
    return fail(FSSIM_ERR_SHAPE, "H*W must be < 2^31 elements per image plane");
  if (B * C > static_cast<int64_t>(INT_MAX))
    return fail(FSSIM_ERR_SHAPE, "B*C must be < 2^31 image planes");
  const double n = static_cast<double>(B) * C * H * W;
  if (n > 4.0e18) return fail(FSSIM_ERR_SHAPE, "B*C*H*W overflows int64");
  return FSSIM_OK;
}

fssim::Geometry make_geometry(int64_t B, int64_t C, int64_t H, int64_t W) {
  fssim::Geometry g;
  g.H = H;
  g.W = W;
  g.HW = H * W;
  g.S = static_cast<int>((W + fssim::kStrip - 1) / fssim::kStrip);
  g.C = static_cast<int>(C);
  g.B = static_cast<int>(B);
  g.LT = B * C * static_cast<int64_t>(g.S) * H;
  return g;
}

int device_sms(int* sms) {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(FSSIM_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    int v = 0;
    e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return fail(FSSIM_ERR_CUDA, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    cached[dev] = v;
  }
  *sms = cached[dev];
  return FSSIM_OK;
}

// Opt a kernel in to its dynamic shared memory size on the current device and return the
// number of resident CTAs per SM. `cache` is owned by one kernel instantiation (it lives in
// the launch_* template below), so every instantiation gets its own per-device entry.
template <typename Kernel>
int kernel_occupancy(Kernel k, size_t smem, int (&cache)[64], std::mutex& mu, int* occ,
                     int threads = fssim::kThreads) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(FSSIM_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (cache[dev] == 0) {
    e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess)
      return fail(FSSIM_ERR_CUDA, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    int v = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&v, k, threads, smem);
    if (e != cudaSuccess || v <= 0)
      return fail(FSSIM_ERR_CUDA, std::string("occupancy query failed: ") + cudaGetErrorString(e));
    cache[dev] = v;
  }
  *occ = cache[dev];
  return FSSIM_OK;
}

// Persistent grid: one CTA per resident slot, but no CTA with fewer than ~2 steps of rows.
// SMs the persistent grids leave free (fssim_set_reserved_sms), e.g. for a collective
// that runs concurrently with a kernel of this library.
std::atomic<int> g_reserved_sms{0};

// Bound of a staging step's wait (polls) and of the sharded gather's wait (ns).
constexpr long long kDefaultGatherTimeoutNs = 10ll * 1000 * 1000 * 1000;
std::atomic<int> g_wait_limit{fssim::kWaitLimit};
std::atomic<long long> g_gather_timeout_ns{kDefaultGatherTimeoutNs};

int grid_size(const fssim::Geometry& g, int occ, int sms) {
  int use = sms - g_reserved_sms.load(std::memory_order_relaxed);
  if (use < 1) use = 1;
  const int64_t slots = static_cast<int64_t>(occ) * use;
  const int64_t by_work = (g.LT + 2 * fssim::kRows - 1) / (2 * fssim::kRows);
  int64_t grid = slots < by_work ? slots : by_work;
  if (grid < 1) grid = 1;
  return static_cast<int>(grid);
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (the library
// does not link libcuda). nullptr if the driver does not provide it.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    (void)cudaGetLastError();
  });
  return fn;
}

// Tensor map for the kernels' TMA staging: the batch as a (planes, H, W) tensor of
// FP32 or FP16 elements, boxes of kBoxRows rows x one staged row pitch of columns,
// zero fill outside. False (the kernels then stage with cp.async) when the layout does not
// meet the copy unit's rules: 16-byte aligned base, row pitch a multiple of 16 bytes.
bool encode_rows(CUtensorMap* m, const void* base, size_t esize, const fssim::Geometry& g,
                 int box_rows) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = tensor_map_encoder();
  if (!fn || !base || !aligned(base, 16)) return false;
  if ((static_cast<size_t>(g.W) * esize) % 16 != 0) return false;
  const int64_t planes = static_cast<int64_t>(g.B) * g.C;
  if (planes < 1 || planes > INT_MAX || g.H < 1 || g.W < 1) return false;
  // 2-byte elements (half or bfloat16) use one map type: the copy is bitwise and its zero
  // fill is +0 in both formats
  const bool f32 = esize == 4;
  const int w = f32 ? fssim::StagePitch<float>::value : fssim::StagePitch<__half>::value;
  // A tensor map is a pure function of (base, shape, element size, box). The driver's
  // encoder costs microseconds of host time per map, so a small per-thread cache keeps it
  // off the per-call path of a training loop, which passes the same buffers every step.
  struct Entry {
    const void* base;
    int64_t W, H, planes;
    size_t esize;
    int box_w, box_h;
    bool valid;
    CUtensorMap map;
  };
  static thread_local Entry cache[32];
  const uintptr_t key = reinterpret_cast<uintptr_t>(base);
  Entry& e = cache[((key >> 8) ^ (key >> 20) ^ static_cast<uintptr_t>(g.W) ^
                    static_cast<uintptr_t>(w) * 7u ^ static_cast<uintptr_t>(box_rows) * 13u) % 32];
  if (e.valid && e.base == base && e.W == g.W && e.H == g.H && e.planes == planes &&
      e.esize == esize && e.box_w == w && e.box_h == box_rows) {
    *m = e.map;
    return true;
  }
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(g.W), static_cast<cuuint64_t>(g.H),
                        static_cast<cuuint64_t>(planes)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(g.W) * esize,
                           static_cast<cuuint64_t>(g.HW) * esize};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(w), static_cast<cuuint32_t>(box_rows), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r =
      fn(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
         const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  e.base = base;
  e.W = g.W;
  e.H = g.H;
  e.planes = planes;
  e.esize = esize;
  e.box_w = w;
  e.box_h = box_rows;
  e.map = *m;
  e.valid = true;
  return true;
}

// Sets p.use_tma when every staged tensor of the forward has a tensor map (boxes of
// box_rows rows: kBoxRows for the tile kernels, kSStep for the streaming kernels).
void set_fwd_tma(fssim::FwdParams& p, size_t esize, int box_rows = fssim::kBoxRows) {
  p.use_tma = encode_rows(&p.tmap[0], p.img1, esize, p.g, box_rows) &&
              encode_rows(&p.tmap[1], p.img2, esize, p.g, box_rows);
}
void set_bwd_tma(fssim::BwdParams& p, size_t pesize, int box_rows = fssim::kBoxRows) {
  bool ok = encode_rows(&p.tmap[0], p.p0, pesize, p.g, box_rows) &&
            encode_rows(&p.tmap[1], p.p1, pesize, p.g, box_rows) &&
            encode_rows(&p.tmap[2], p.p2, pesize, p.g, box_rows);
  if (ok && p.dl) ok = encode_rows(&p.tmap[3], p.dl, sizeof(float), p.g, box_rows);
  p.use_tma = ok;
}

// Launch with programmatic stream serialization allowed: the kernel may begin while the
// previous kernel on the stream finishes; it waits (griddepcontrol.wait) before touching
// global memory.
template <typename Kernel, typename Params>
cudaError_t launch_pdl(Kernel k, int grid, size_t smem, cudaStream_t stream, const Params& p,
                       int threads = fssim::kThreads) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, p);
}

int launch_error(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  return FSSIM_OK;
}

template <int HALO, typename TIn, typename TP, bool TRAIN, bool MERGED>
int launch_fwd(const fssim::FwdParams& p, cudaStream_t stream) {
  using Cfg = fssim::FwdConfig<HALO, TIn, TP, TRAIN, MERGED>;
  auto k = fssim::ssim_fwd_kernel<HALO, TIn, TP, TRAIN, MERGED>;
  static std::mutex mu;
  static int cache[64] = {0};
  int occ = 0, sms = 0;
  int st = kernel_occupancy(k, Cfg::kSmem, cache, mu, &occ);
  if (st) return st;
  st = device_sms(&sms);
  if (st) return st;
  const int grid = grid_size(p.g, occ, sms);
  if ((p.g.LT + grid - 1) / grid + 2 * p.g.H > INT_MAX) return fail(FSSIM_ERR_SHAPE, "batch too large");
  if (grid >= 65536) return fail(FSSIM_ERR_CUDA, "grid too large for the reduction ticket");
  fssim::FwdParams q = p;
  q.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  const cudaError_t e = launch_pdl(k, grid, Cfg::kSmem, stream, q);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(FSSIM_ERR_CUDA, std::string("ssim forward launch: ") + cudaGetErrorString(e));
  }
  return launch_error("ssim forward launch");
}

template <int HALO, typename TIn, typename TP, bool DLMAP>
int launch_bwd(const fssim::BwdParams& p, cudaStream_t stream) {
  using Cfg = fssim::BwdConfig<HALO, TIn, TP, DLMAP>;
  auto k = fssim::ssim_bwd_kernel<HALO, TIn, TP, DLMAP>;
  static std::mutex mu;
  static int cache[64] = {0};
  int occ = 0, sms = 0;
  int st = kernel_occupancy(k, Cfg::kSmem, cache, mu, &occ);
  if (st) return st;
  st = device_sms(&sms);
  if (st) return st;
  const int grid = grid_size(p.g, occ, sms);
  if ((p.g.LT + grid - 1) / grid + 2 * p.g.H > INT_MAX) return fail(FSSIM_ERR_SHAPE, "batch too large");
  fssim::BwdParams q = p;
  q.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  const cudaError_t e = launch_pdl(k, grid, Cfg::kSmem, stream, q);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(FSSIM_ERR_CUDA, std::string("ssim backward launch: ") + cudaGetErrorString(e));
  }
  return launch_error("ssim backward launch");
}

// The fused loss path's column-streaming kernels (ssim_stream.cuh).
template <int HALO, typename TIn, typename TP, bool TRAIN>
int launch_sfwd(const fssim::FwdParams& p, cudaStream_t stream) {
  using Cfg = fssim::SFwdConfig<HALO, TIn, TP, TRAIN>;
  auto k = fssim::loss_fwd_kernel<HALO, TIn, TP, TRAIN>;
  static std::mutex mu;
  static int cache[64] = {0};
  int occ = 0, sms = 0;
  int st = kernel_occupancy(k, Cfg::kSmem, cache, mu, &occ, fssim::kSThreads);
  if (st) return st;
  st = device_sms(&sms);
  if (st) return st;
  const int grid = grid_size(p.g, occ, sms);
  if ((p.g.LT + grid - 1) / grid + 2 * p.g.H > INT_MAX) return fail(FSSIM_ERR_SHAPE, "batch too large");
  if (grid >= 65536) return fail(FSSIM_ERR_CUDA, "grid too large for the reduction ticket");
  fssim::FwdParams q = p;
  q.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  const cudaError_t e = launch_pdl(k, grid, Cfg::kSmem, stream, q, fssim::kSThreads);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(FSSIM_ERR_CUDA, std::string("ssim loss forward launch: ") + cudaGetErrorString(e));
  }
  return launch_error("ssim loss forward launch");
}

template <int HALO, typename TIn, typename TP>
int launch_sbwd(const fssim::BwdParams& p, cudaStream_t stream) {
  using Cfg = fssim::SBwdConfig<HALO, TIn, TP>;
  auto k = fssim::loss_bwd_kernel<HALO, TIn, TP>;
  static std::mutex mu;
  static int cache[64] = {0};
  int occ = 0, sms = 0;
  int st = kernel_occupancy(k, Cfg::kSmem, cache, mu, &occ, fssim::kSThreads);
  if (st) return st;
  st = device_sms(&sms);
  if (st) return st;
  const int grid = grid_size(p.g, occ, sms);
  if ((p.g.LT + grid - 1) / grid + 2 * p.g.H > INT_MAX) return fail(FSSIM_ERR_SHAPE, "batch too large");
  fssim::BwdParams q = p;
  q.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  const cudaError_t e = launch_pdl(k, grid, Cfg::kSmem, stream, q, fssim::kSThreads);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return fail(FSSIM_ERR_CUDA, std::string("ssim loss backward launch: ") + cudaGetErrorString(e));
  }
  return launch_error("ssim loss backward launch");
}

// Kernel family of the fused loss path (fssim_set_loss_kernels): the column-streaming
// kernels, the 4-row tile kernels that the map entry points use, or (default) per launch
// the family that measured faster on a B200 for its size (CUDA events, FP32 and FP16,
// windows 7 and 11): the streaming kernels, except the tile kernels below 2^21
// channel-pixels (1x3x256^2: 8.4 + 5.1 us against 13.0 + 8.6 us; the streaming kernels'
// 8-row steps leave a short grid more latency-bound) and the tile backward from 2^27
// channel-pixels (16x3x2048^2: 1084 us against 1157 us).
std::atomic<int> g_loss_kernels{FSSIM_KERNELS_AUTO};
constexpr int64_t kStreamMinCpx = int64_t{1} << 21;
constexpr int64_t kStreamBwdMaxCpx = int64_t{1} << 27;
bool loss_streaming(bool forward, int64_t cpx) {
  const int f = g_loss_kernels.load(std::memory_order_relaxed);
  if (f == FSSIM_KERNELS_AUTO) return cpx >= kStreamMinCpx && (forward || cpx < kStreamBwdMaxCpx);
  return f == FSSIM_KERNELS_STREAM;
}

template <typename TIn, typename TP, bool TRAIN>
int dispatch_loss_fwd(int ws, const fssim::FwdParams& p, cudaStream_t s, bool streaming) {
  if (!streaming) {
    switch (ws) {
      case 7: return launch_fwd<3, TIn, TP, TRAIN, true>(p, s);
      case 9: return launch_fwd<4, TIn, TP, TRAIN, true>(p, s);
      case 11: return launch_fwd<5, TIn, TP, TRAIN, true>(p, s);
      default: return fail(FSSIM_ERR_WINDOW, window_message(ws));
    }
  }
  switch (ws) {
    case 7: return launch_sfwd<3, TIn, TP, TRAIN>(p, s);
    case 9: return launch_sfwd<4, TIn, TP, TRAIN>(p, s);
    case 11: return launch_sfwd<5, TIn, TP, TRAIN>(p, s);
    default: return fail(FSSIM_ERR_WINDOW, window_message(ws));
  }
}

template <typename TIn, typename TP>
int dispatch_loss_bwd(int ws, const fssim::BwdParams& p, cudaStream_t s, bool streaming) {
  if (!streaming) {
    switch (ws) {
      case 7: return launch_bwd<3, TIn, TP, false>(p, s);
      case 9: return launch_bwd<4, TIn, TP, false>(p, s);
      case 11: return launch_bwd<5, TIn, TP, false>(p, s);
      default: return fail(FSSIM_ERR_WINDOW, window_message(ws));
    }
  }
  switch (ws) {
    case 7: return launch_sbwd<3, TIn, TP>(p, s);
    case 9: return launch_sbwd<4, TIn, TP>(p, s);
    case 11: return launch_sbwd<5, TIn, TP>(p, s);
    default: return fail(FSSIM_ERR_WINDOW, window_message(ws));
  }
}

// MERGED selects the fused loss path's 4-map forward; the map-producing reference entry
// points use the reference's 5 maps.
template <typename TIn, typename TP, bool TRAIN, bool MERGED>
int dispatch_fwd(int ws, const fssim::FwdParams& p, cudaStream_t s) {
  switch (ws) {
    case 7: return launch_fwd<3, TIn, TP, TRAIN, MERGED>(p, s);
    case 9: return launch_fwd<4, TIn, TP, TRAIN, MERGED>(p, s);
    case 11: return launch_fwd<5, TIn, TP, TRAIN, MERGED>(p, s);
    default: return fail(FSSIM_ERR_WINDOW, window_message(ws));
  }
}

template <typename TIn, typename TP, bool DLMAP>
int dispatch_bwd(int ws, const fssim::BwdParams& p, cudaStream_t s) {
  switch (ws) {
    case 7: return launch_bwd<3, TIn, TP, DLMAP>(p, s);
    case 9: return launch_bwd<4, TIn, TP, DLMAP>(p, s);
    case 11: return launch_bwd<5, TIn, TP, DLMAP>(p, s);
    default: return fail(FSSIM_ERR_WINDOW, window_message(ws));
  }
}

size_t elem_size(int dt) { return dt == FSSIM_F32 ? 4 : 2; }

__global__ void fill_kernel(float* out, int64_t n, float v) {
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = v;
}

// Map-producing forward shared by the FP32 and FP16 reference entry points.
template <typename TIn>
int compat_forward(int ws, float C1, float C2, const TIn* img1, const TIn* img2, int64_t B,
                   int64_t C, int64_t H, int64_t W, bool train, float* map, float* p0, float* p1,
                   float* p2, cudaStream_t stream) {
  g_last_error.clear();
  int st = check_window(ws);
  if (st) return st;
  st = check_shape(B, C, H, W);
  if (st) return st;
  if (B * C * H * W == 0) return FSSIM_OK;
  if (!img1 || !img2 || !map) return fail(FSSIM_ERR_NULLPTR, "img1, img2 and ssim_map are required");
  if (train && (!p0 || !p1 || !p2))
    return fail(FSSIM_ERR_NULLPTR, "train requires dm_dmu1, dm_dsigma1_sq and dm_dsigma12");
  constexpr int64_t E = 16 / sizeof(TIn);
  fssim::FwdParams p{};
  p.img1 = img1;
  p.img2 = img2;
  p.map = map;
  p.p0 = p0;
  p.p1 = p1;
  p.p2 = p2;
  p.g = make_geometry(B, C, H, W);
  p.C1 = C1;
  p.C2 = C2;
  p.out_scale = 1.f;
  p.valid = 0;
  p.clamp = 0;
  p.reduce = FSSIM_REDUCE_NONE;
  p.mask_partials = 0;
  p.aligned16 = (W % E == 0) && aligned(img1, 16) && aligned(img2, 16);
  p.pair_ok = (W % 2 == 0) && aligned(map, 8) &&
              (!train || (aligned(p0, 8) && aligned(p1, 8) && aligned(p2, 8)));
  set_fwd_tma(p, sizeof(TIn));
  if (train) return dispatch_fwd<TIn, float, true, false>(ws, p, stream);
  return dispatch_fwd<TIn, float, false, false>(ws, p, stream);
}

template <typename TIn>
int compat_backward(int ws, const TIn* img1, const TIn* img2, const float* dl, const float* p0,
                    const float* p1, const float* p2, int64_t B, int64_t C, int64_t H, int64_t W,
                    float* grad, cudaStream_t stream) {
  g_last_error.clear();
  int st = check_window(ws);
  if (st) return st;
  st = check_shape(B, C, H, W);
  if (st) return st;
  if (B * C * H * W == 0) return FSSIM_OK;
  if (!img1 || !img2 || !dl || !p0 || !p1 || !p2 || !grad)
    return fail(FSSIM_ERR_NULLPTR, "all tensors of fusedssim_backward are required");
  fssim::BwdParams p{};
  p.img1 = img1;
  p.img2 = img2;
  p.p0 = p0;
  p.p1 = p1;
  p.p2 = p2;
  p.dl = dl;
  p.grad_out = nullptr;
  p.grad = grad;
  p.g = make_geometry(B, C, H, W);
  p.chain_scale = 1.f;
  p.grad_per_image = 0;
  p.grad_dtype = FSSIM_F32;
  p.aligned16 = (W % 4 == 0) && aligned(dl, 16) && aligned(p0, 16) && aligned(p1, 16) &&
                aligned(p2, 16);
  p.pair_ok = (W % 2 == 0) && aligned(img1, 2 * sizeof(TIn)) && aligned(img2, 2 * sizeof(TIn)) &&
              aligned(grad, 8);
  set_bwd_tma(p, sizeof(float));
  return dispatch_bwd<TIn, float, true>(ws, p, stream);
}

}  // namespace

extern "C" {

const char* fssim_status_string(int status) {
  switch (status) {
    case FSSIM_OK: return "success";
    case FSSIM_ERR_WINDOW: return "unsupported window size";
    case FSSIM_ERR_SHAPE: return "invalid shape";
    case FSSIM_ERR_DTYPE: return "unsupported element type";
    case FSSIM_ERR_NULLPTR: return "required pointer is NULL";
    case FSSIM_ERR_WORKSPACE: return "workspace missing or too small";
    case FSSIM_ERR_CUDA: return "CUDA error";
    case FSSIM_ERR_ARGUMENT: return "invalid argument";
    default: return "unknown status";
  }
}

const char* fssim_last_error(void) { return g_last_error.c_str(); }

const char* fssim_version(void) { return "0.1.0"; }

int fssim_set_reserved_sms(int n) {
  g_last_error.clear();
  if (n < 0) return fail(FSSIM_ERR_ARGUMENT, "reserved SM count must be >= 0");
  g_reserved_sms.store(n, std::memory_order_relaxed);
  return FSSIM_OK;
}

int fssim_set_loss_kernels(int family) {
  g_last_error.clear();
  if (family != FSSIM_KERNELS_STREAM && family != FSSIM_KERNELS_TILE &&
      family != FSSIM_KERNELS_AUTO)
    return fail(FSSIM_ERR_ARGUMENT,
                "family must be FSSIM_KERNELS_STREAM, FSSIM_KERNELS_TILE or FSSIM_KERNELS_AUTO");
  g_loss_kernels.store(family, std::memory_order_relaxed);
  return FSSIM_OK;
}

int fssim_set_staging_wait_limit(long long polls) {
  g_last_error.clear();
  const long long v = polls < 0 ? fssim::kWaitLimit : (polls > INT_MAX ? INT_MAX : polls);
  g_wait_limit.store(static_cast<int>(v), std::memory_order_relaxed);
  return FSSIM_OK;
}

int fssim_set_gather_timeout_us(long long us) {
  g_last_error.clear();
  const long long cap = LLONG_MAX / 1000;
  const long long ns = us <= 0 ? kDefaultGatherTimeoutNs : (us > cap ? cap : us) * 1000;
  g_gather_timeout_ns.store(ns, std::memory_order_relaxed);
  return FSSIM_OK;
}

int fssim_poll_device_error(unsigned* code, int clear) {
  g_last_error.clear();
  if (!code) return fail(FSSIM_ERR_NULLPTR, "code is NULL");
  unsigned v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, fssim::g_device_error, sizeof(v));
  if (e != cudaSuccess)
    return fail(FSSIM_ERR_CUDA, std::string("reading the device error flag: ") + cudaGetErrorString(e));
  if (clear && v) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(fssim::g_device_error, &zero, sizeof(zero));
    if (e != cudaSuccess)
      return fail(FSSIM_ERR_CUDA, std::string("clearing the device error flag: ") + cudaGetErrorString(e));
  }
  *code = v;
  return FSSIM_OK;
}

int fssim_fusedssim(int window_size, float C1, float C2, const float* img1, const float* img2,
                    int64_t B, int64_t C, int64_t H, int64_t W, int train, float* ssim_map,
                    float* dm_dmu1, float* dm_dsigma1_sq, float* dm_dsigma12,
                    fssim_stream_t stream) {
  NvtxRange range("fssim_fusedssim");
  return compat_forward<float>(window_size, C1, C2, img1, img2, B, C, H, W, train != 0, ssim_map,
                               dm_dmu1, dm_dsigma1_sq, dm_dsigma12, stream);
}

int fssim_fusedssim_backward(int window_size, float C1, float C2, const float* img1,
                             const float* img2, const float* dL_dmap, const float* dm_dmu1,
                             const float* dm_dsigma1_sq, const float* dm_dsigma12, int64_t B,
                             int64_t C, int64_t H, int64_t W, float* dL_dimg1,
                             fssim_stream_t stream) {
  (void)C1;
  (void)C2;  // the backward needs only the partials, as in the reference
  NvtxRange range("fssim_fusedssim_backward");
  return compat_backward<float>(window_size, img1, img2, dL_dmap, dm_dmu1, dm_dsigma1_sq,
                                dm_dsigma12, B, C, H, W, dL_dimg1, stream);
}

int fssim_fusedssim_fp16(int window_size, float C1, float C2, const uint16_t* img1,
                         const uint16_t* img2, int64_t B, int64_t C, int64_t H, int64_t W,
                         float* ssim_map, fssim_stream_t stream) {
  return compat_forward<__half>(window_size, C1, C2, reinterpret_cast<const __half*>(img1),
                                reinterpret_cast<const __half*>(img2), B, C, H, W, false,
                                ssim_map, nullptr, nullptr, nullptr, stream);
}

int fssim_fusedssim_fp16_train(int window_size, float C1, float C2, const uint16_t* img1,
                               const uint16_t* img2, int64_t B, int64_t C, int64_t H,
                               int64_t W, float* ssim_map, float* dm_dmu1,
                               float* dm_dsigma1_sq, float* dm_dsigma12,
                               fssim_stream_t stream) {
  return compat_forward<__half>(window_size, C1, C2, reinterpret_cast<const __half*>(img1),
                                reinterpret_cast<const __half*>(img2), B, C, H, W, true,
                                ssim_map, dm_dmu1, dm_dsigma1_sq, dm_dsigma12, stream);
}

int fssim_fusedssim_fp16_backward(int window_size, float C1, float C2, const uint16_t* img1,
                                  const uint16_t* img2, const float* dL_dmap,
                                  const float* dm_dmu1, const float* dm_dsigma1_sq,
                                  const float* dm_dsigma12, int64_t B, int64_t C, int64_t H,
                                  int64_t W, float* dL_dimg1, fssim_stream_t stream) {
  (void)C1;
  (void)C2;
  return compat_backward<__half>(window_size, reinterpret_cast<const __half*>(img1),
                                 reinterpret_cast<const __half*>(img2), dL_dmap, dm_dmu1,
                                 dm_dsigma1_sq, dm_dsigma12, B, C, H, W, dL_dimg1, stream);
}

size_t fssim_forward_workspace_bytes(int64_t B) {
  if (B <= 0) return 256;
  // ticket, then B SSIM and B L1 fixed-point accumulators
  return 256 + 2 * static_cast<size_t>(B) * sizeof(unsigned long long);
}

}  // extern "C"

namespace {

// fssim_forward, optionally publishing the batch sum to the ranks of a sharded loss.
int forward_impl(const fssim_forward_args* a, const fssim::DpParams* dp, cudaStream_t stream) {
  if (!a) return fail(FSSIM_ERR_NULLPTR, "args is NULL");
  int st = check_window(a->window_size);
  if (st) return st;
  st = check_shape(a->B, a->C, a->H, a->W);
  if (st) return st;
  if (a->dtype != FSSIM_F32 && a->dtype != FSSIM_F16 && a->dtype != FSSIM_BF16)
    return fail(FSSIM_ERR_DTYPE, "img dtype must be F32, F16 or BF16");
  if (a->train && !(a->partial_dtype == FSSIM_F32 ||
                    (a->partial_dtype == FSSIM_F16 && a->dtype == FSSIM_F16)))
    return fail(FSSIM_ERR_DTYPE, "partials must be F32 (or F16 with F16 images)");
  if (a->reduce < FSSIM_REDUCE_NONE || a->reduce > FSSIM_REDUCE_PER_IMAGE)
    return fail(FSSIM_ERR_ARGUMENT, "reduce must be 0, 1 or 2");
  const int64_t N = a->B * a->C * a->H * a->W;
  if (a->reduce != FSSIM_REDUCE_NONE) {
    if (!a->out) return fail(FSSIM_ERR_NULLPTR, "out is required when reducing");
    // an image's SSIM sum (|value| <= 1 per pixel) must fit the 2^28 fixed point in 63 bits
    if (a->C * a->H * a->W > (int64_t{1} << 34))
      return fail(FSSIM_ERR_SHAPE, "C*H*W must be <= 2^34 per image for the reductions");
    if (!a->workspace || a->workspace_bytes < fssim_forward_workspace_bytes(a->B))
      return fail(FSSIM_ERR_WORKSPACE, "workspace smaller than fssim_forward_workspace_bytes(B)");
    if (!aligned(a->workspace, 16)) return fail(FSSIM_ERR_WORKSPACE, "workspace must be 16-byte aligned");
  }
  if (N == 0) {
    // Nothing to reduce: sums are 0 and out = 0 * out_scale (NaN for a mean over no pixels,
    // out_scale = 1/0), which is what torch's mean of an empty tensor gives.
    if (a->reduce != FSSIM_REDUCE_NONE) {
      const int64_t n_out = a->reduce == FSSIM_REDUCE_SCALAR ? 1 : a->B;
      if (n_out > 0) {
        fill_kernel<<<1, 128, 0, stream>>>(a->out, n_out, 0.f * a->out_scale + a->out_offset);
        const int e = launch_error("fill launch");
        if (e) return e;
      }
      if (a->image_sums && a->B > 0) {
        const cudaError_t e = cudaMemsetAsync(a->image_sums, 0, sizeof(double) * a->B, stream);
        if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, cudaGetErrorString(e));
      }
    }
    return FSSIM_OK;
  }
  if (!a->img1 || !a->img2) return fail(FSSIM_ERR_NULLPTR, "img1 and img2 are required");
  if (a->train && !a->partials) return fail(FSSIM_ERR_NULLPTR, "train requires partials");

  const size_t E = elem_size(a->dtype);
  const size_t PE = elem_size(a->partial_dtype);
  fssim::FwdParams p{};
  p.img1 = a->img1;
  p.img2 = a->img2;
  p.map = a->ssim_map;
  if (a->train) {
    char* base = static_cast<char*>(a->partials);
    p.p0 = base;
    p.p1 = base + static_cast<size_t>(N) * PE;
    p.p2 = base + 2 * static_cast<size_t>(N) * PE;
  }
  p.out = a->out;
  p.image_sums = a->image_sums;
  if (a->reduce != FSSIM_REDUCE_NONE) {
    p.ticket = static_cast<unsigned*>(a->workspace);
    p.acc = reinterpret_cast<unsigned long long*>(static_cast<char*>(a->workspace) + 256);
    p.acc_l1 = p.acc + a->B;
  }
  p.g = make_geometry(a->B, a->C, a->H, a->W);
  p.C1 = a->C1;
  p.C2 = a->C2;
  p.out_scale = a->out_scale;
  p.l1_weight = a->l1_weight;
  p.out_offset = a->out_offset;
  p.l1 = (a->l1_weight != 0.f && a->reduce != FSSIM_REDUCE_NONE) ? 1 : 0;
  p.valid = a->valid ? 1 : 0;
  p.clamp = a->clamp ? 1 : 0;
  p.reduce = a->reduce;
  p.mask_partials = 1;
  p.aligned16 = (a->W % static_cast<int64_t>(16 / E) == 0) && aligned(a->img1, 16) &&
                aligned(a->img2, 16);
  bool pair = (a->W % 2 == 0) && (!a->ssim_map || aligned(a->ssim_map, 8));
  if (a->train) pair = pair && aligned(p.p0, 2 * PE) && aligned(p.p1, 2 * PE) && aligned(p.p2, 2 * PE);
  p.pair_ok = pair;
  // the family is read once: its tensor maps' box height must match the kernels launched
  const bool streaming = loss_streaming(true, N);
  set_fwd_tma(p, E, streaming ? fssim::kSStep : fssim::kBoxRows);
  if (dp) p.dp = *dp;

  const int ws = a->window_size;
  cudaStream_t s = stream;
  if (a->dtype == FSSIM_F32) {
    if (a->train) return dispatch_loss_fwd<float, float, true>(ws, p, s, streaming);
    return dispatch_loss_fwd<float, float, false>(ws, p, s, streaming);
  }
  if (a->dtype == FSSIM_BF16) {
    if (a->train) return dispatch_loss_fwd<__nv_bfloat16, float, true>(ws, p, s, streaming);
    return dispatch_loss_fwd<__nv_bfloat16, float, false>(ws, p, s, streaming);
  }
  if (!a->train) return dispatch_loss_fwd<__half, float, false>(ws, p, s, streaming);
  if (a->partial_dtype == FSSIM_F16) return dispatch_loss_fwd<__half, __half, true>(ws, p, s, streaming);
  return dispatch_loss_fwd<__half, float, true>(ws, p, s, streaming);
}

int check_dp(const fssim_dp_args* d, fssim::DpParams* out) {
  if (!d) return fail(FSSIM_ERR_NULLPTR, "dp args is NULL");
  if (d->world < 1 || d->world > FSSIM_DP_MAX_RANKS)
    return fail(FSSIM_ERR_ARGUMENT, "world must be in [1, " + std::to_string(FSSIM_DP_MAX_RANKS) + "]");
  if (d->rank < 0 || d->rank >= d->world) return fail(FSSIM_ERR_ARGUMENT, "rank out of range");
  fssim::DpParams p{};
  for (int r = 0; r < d->world; ++r) {
    if (!d->mailboxes[r]) return fail(FSSIM_ERR_NULLPTR, "mailbox pointer missing");
    if (!aligned(d->mailboxes[r], 16)) return fail(FSSIM_ERR_ARGUMENT, "mailbox not 16-byte aligned");
    p.mail[r] = static_cast<fssim::DpMailSlot*>(d->mailboxes[r]);
  }
  p.world = d->world;
  p.rank = d->rank;
  p.seq = d->seq;
  p.timeout_ns = static_cast<unsigned long long>(g_gather_timeout_ns.load(std::memory_order_relaxed));
  *out = p;
  return FSSIM_OK;
}

}  // namespace

extern "C" {

int fssim_forward(const fssim_forward_args* a, fssim_stream_t stream) {
  NvtxRange range("fssim_forward");
  g_last_error.clear();
  return forward_impl(a, nullptr, stream);
}

size_t fssim_dp_mailbox_bytes(int world) {
  if (world < 1) return 0;
  return 2 * static_cast<size_t>(world) * sizeof(fssim::DpMailSlot);
}

int fssim_dp_mailbox_alloc(int world, void** mailbox) {
  g_last_error.clear();
  if (!mailbox) return fail(FSSIM_ERR_NULLPTR, "mailbox is NULL");
  if (world < 1 || world > FSSIM_DP_MAX_RANKS) return fail(FSSIM_ERR_ARGUMENT, "world out of range");
  void* p = nullptr;
  // a whole allocation of its own, so its IPC handle maps exactly this buffer
  cudaError_t e = cudaMalloc(&p, fssim_dp_mailbox_bytes(world));
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaMalloc(mailbox): ") + cudaGetErrorString(e));
  // seq 0 is never used by a step, so zero-filled slots hold no message
  e = cudaMemset(p, 0, fssim_dp_mailbox_bytes(world));
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(FSSIM_ERR_CUDA, std::string("cudaMemset(mailbox): ") + cudaGetErrorString(e));
  }
  *mailbox = p;
  return FSSIM_OK;
}

int fssim_dp_mailbox_free(void* mailbox) {
  g_last_error.clear();
  if (!mailbox) return FSSIM_OK;
  const cudaError_t e = cudaFree(mailbox);
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaFree(mailbox): ") + cudaGetErrorString(e));
  return FSSIM_OK;
}

int fssim_ipc_get_handle(const void* mailbox, unsigned char handle[FSSIM_IPC_HANDLE_BYTES]) {
  g_last_error.clear();
  if (!mailbox || !handle) return fail(FSSIM_ERR_NULLPTR, "mailbox and handle are required");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(mailbox));
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == FSSIM_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return FSSIM_OK;
}

int fssim_ipc_open_handle(const unsigned char handle[FSSIM_IPC_HANDLE_BYTES], void** peer_mailbox) {
  g_last_error.clear();
  if (!handle || !peer_mailbox) return fail(FSSIM_ERR_NULLPTR, "handle and peer_mailbox are required");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  *peer_mailbox = p;
  return FSSIM_OK;
}

int fssim_ipc_close_handle(void* peer_mailbox) {
  g_last_error.clear();
  if (!peer_mailbox) return FSSIM_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_mailbox);
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaIpcCloseMemHandle: ") + cudaGetErrorString(e));
  return FSSIM_OK;
}

int fssim_forward_dp(const fssim_forward_args* a, const fssim_dp_args* dp, fssim_stream_t stream) {
  NvtxRange range("fssim_forward_dp");
  g_last_error.clear();
  if (!a) return fail(FSSIM_ERR_NULLPTR, "args is NULL");
  if (a->reduce != FSSIM_REDUCE_SCALAR) return fail(FSSIM_ERR_ARGUMENT, "fssim_forward_dp needs reduce = SCALAR");
  fssim::DpParams p{};
  int st = check_dp(dp, &p);
  if (st) return st;
  st = forward_impl(a, &p, stream);
  if (st || a->B * a->C * a->H * a->W != 0) return st;
  // an empty shard has no forward kernel to publish its (zero) sum
  fssim::dp_publish_kernel<<<1, 32, 0, stream>>>(p, 0.0);
  return launch_error("dp publish launch");
}

int fssim_dp_gather(const fssim_dp_args* dp, float scale, float* out, fssim_stream_t stream) {
  NvtxRange range("fssim_dp_gather");
  g_last_error.clear();
  if (!out) return fail(FSSIM_ERR_NULLPTR, "out is NULL");
  fssim::DpParams p{};
  const int st = check_dp(dp, &p);
  if (st) return st;
  fssim::dp_gather_kernel<<<1, 32, 0, stream>>>(p, scale, out);
  return launch_error("dp gather launch");
}

int fssim_backward(const fssim_backward_args* a, fssim_stream_t stream) {
  NvtxRange range("fssim_backward");
  g_last_error.clear();
  if (!a) return fail(FSSIM_ERR_NULLPTR, "args is NULL");
  int st = check_window(a->window_size);
  if (st) return st;
  st = check_shape(a->B, a->C, a->H, a->W);
  if (st) return st;
  if (a->dtype != FSSIM_F32 && a->dtype != FSSIM_F16 && a->dtype != FSSIM_BF16)
    return fail(FSSIM_ERR_DTYPE, "img dtype must be F32, F16 or BF16");
  if (!(a->partial_dtype == FSSIM_F32 || (a->partial_dtype == FSSIM_F16 && a->dtype == FSSIM_F16)))
    return fail(FSSIM_ERR_DTYPE, "partials must be F32 (or F16 with F16 images)");
  if (a->grad_dtype < FSSIM_F32 || a->grad_dtype > FSSIM_BF16)
    return fail(FSSIM_ERR_DTYPE, "grad dtype must be F32, F16 or BF16");
  const int64_t N = a->B * a->C * a->H * a->W;
  if (N == 0) return FSSIM_OK;
  if (!a->img1 || !a->img2 || !a->partials || !a->grad)
    return fail(FSSIM_ERR_NULLPTR, "img1, img2, partials and grad are required");
  const size_t E = elem_size(a->dtype);
  const size_t PE = elem_size(a->partial_dtype);
  const size_t GE = elem_size(a->grad_dtype);
  const char* base = static_cast<const char*>(a->partials);
  fssim::BwdParams p{};
  p.img1 = a->img1;
  p.img2 = a->img2;
  p.p0 = base;
  p.p1 = base + static_cast<size_t>(N) * PE;
  p.p2 = base + 2 * static_cast<size_t>(N) * PE;
  p.dl = nullptr;
  p.grad_out = a->grad_out;
  p.grad = a->grad;
  p.g = make_geometry(a->B, a->C, a->H, a->W);
  p.chain_scale = a->chain_scale;
  p.l1_scale = a->l1_scale;
  p.grad_per_image = a->grad_out_per_image ? 1 : 0;
  p.grad_dtype = a->grad_dtype;
  p.aligned16 = (a->W % static_cast<int64_t>(16 / PE) == 0) && aligned(p.p0, 16) &&
                aligned(p.p1, 16) && aligned(p.p2, 16);
  p.pair_ok = (a->W % 2 == 0) && aligned(a->img1, 2 * E) && aligned(a->img2, 2 * E) &&
              aligned(a->grad, 2 * GE);
  const bool streaming = loss_streaming(false, N);
  set_bwd_tma(p, PE, streaming ? fssim::kSStep : fssim::kBoxRows);
  const int ws = a->window_size;
  cudaStream_t s = stream;
  if (a->dtype == FSSIM_F32) return dispatch_loss_bwd<float, float>(ws, p, s, streaming);
  if (a->dtype == FSSIM_BF16) return dispatch_loss_bwd<__nv_bfloat16, float>(ws, p, s, streaming);
  if (a->partial_dtype == FSSIM_F16) return dispatch_loss_bwd<__half, __half>(ws, p, s, streaming);
  return dispatch_loss_bwd<__half, float>(ws, p, s, streaming);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// fssim_forward_noalloc: the fused forward for callers that cannot allocate GPU memory.
//
// fssim_forward needs a small reduction scratch buffer (a ticket word plus one 64-bit
// accumulator per image) that its caller allocates. Some callers cannot do that: a
// renderer or game-engine plugin whose host application owns every device allocation and
// hands the plugin only the buffers it reads and writes, a real-time loop with a fixed
// memory budget that forbids allocating after start-up, or a binding from a language
// runtime that has no device allocator at hand. This entry point serves them: its scratch
// is a fixed array in the library's own device memory, so nothing is allocated per call,
// by the library or by the caller, who still passes the inputs and outputs.
//
// What that costs:
//  * every GPU that loads this library holds the array (256 B + 16 B per image for
//    FSSIM_NOALLOC_MAX_IMAGES images, about 65 KiB) until the process exits;
//  * the array is shared by all calls: two calls whose kernels overlap on the GPU (on
//    different streams or from different host threads) race on it and return wrong
//    sums, so such calls must be serialised;
//  * at most FSSIM_NOALLOC_MAX_IMAGES images per call.
//
// The first call on each device looks the array's device address up with
// cudaGetSymbolAddress (one-time set-up per device); make that first call before any
// stream capture on that device.
// ---------------------------------------------------------------------------------------
namespace {

constexpr size_t kNoAllocScratchBytes =
    256 + 2 * sizeof(unsigned long long) * static_cast<size_t>(FSSIM_NOALLOC_MAX_IMAGES);

// In host code this name is only a stand-in for the symbol, never a device address: the
// address handed to the kernel comes from cudaGetSymbolAddress in noalloc_scratch().
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up once per device.
int noalloc_scratch(void** out) {
  static std::mutex mu;
  static void* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(FSSIM_ERR_CUDA, "device ordinal out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FSSIM_ERR_CUDA, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
    addr[dev] = p;
  }
  *out = addr[dev];
  return FSSIM_OK;
}

}  // namespace

extern "C" int fssim_forward_noalloc(const fssim_forward_args* args, fssim_stream_t stream) {
  g_last_error.clear();
  if (!args) return fail(FSSIM_ERR_NULLPTR, "args is NULL");
  if (args->B > FSSIM_NOALLOC_MAX_IMAGES)
    return fail(FSSIM_ERR_WORKSPACE,
                "fssim_forward_noalloc handles at most " + std::to_string(FSSIM_NOALLOC_MAX_IMAGES) +
                    " images per call, got " + std::to_string(args->B) +
                    "; use fssim_forward with a caller workspace for larger batches");
  void* scratch = nullptr;
  const int st = noalloc_scratch(&scratch);
  if (st) return st;
  fssim_forward_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocScratchBytes;
  if (a.reduce != FSSIM_REDUCE_NONE && a.B > 0) {
    // The array keeps what the previous call left; the ticket and this call's
    // accumulators must start at zero.
    const cudaError_t e =
        cudaMemsetAsync(scratch, 0, fssim_forward_workspace_bytes(a.B), stream);
    if (e != cudaSuccess) return fail(FSSIM_ERR_CUDA, std::string("clearing scratch: ") + cudaGetErrorString(e));
  }
  return fssim_forward(&a, stream);
}
