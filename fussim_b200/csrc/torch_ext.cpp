// Thin torch binding over the C ABI (include/fussim_b200.h).
//
// It exports the reference's five extension functions under their reference names
// (csrc/ext.cpp:11-17 of OpsiClear/fussim) with the same argument order, return values
// and error types, plus the fused loss entry points used by fussim_b200.fused_ssim.
// Everything launches on torch's current CUDA stream of the input's device.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>

#include "fussim_b200.h"

namespace {

void check_status(int st) {
  if (st == FSSIM_OK) return;
  const std::string msg = fssim_last_error();
  // The reference's dispatch throws std::invalid_argument for a bad window size, which
  // pybind11 turns into ValueError (csrc/ssim.cu:616-617).
  if (st == FSSIM_ERR_WINDOW) throw std::invalid_argument(msg);
  throw std::runtime_error(std::string("fussim_b200: ") + fssim_status_string(st) + ": " + msg);
}

void check_window(int ws) {
  if (ws != 7 && ws != 9 && ws != 11)
    throw std::invalid_argument("window_size must be 7, 9, or 11, got " + std::to_string(ws));
}

fssim_stream_t current_stream() {
  return reinterpret_cast<fssim_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

void check_cuda_4d(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 4, name, " must be 4-D (B, C, H, W), got ", t.dim(), "-D");
}

int dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kFloat: return FSSIM_F32;
    case at::kHalf: return FSSIM_F16;
    case at::kBFloat16: return FSSIM_BF16;
    default: throw std::invalid_argument("unsupported dtype for fussim_b200");
  }
}

// -------------------------------------------------------------------------------------
// Reference extension functions
// -------------------------------------------------------------------------------------
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor> fusedssim(
    int window_size, float C1, float C2, torch::Tensor& img1, torch::Tensor& img2, bool train) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  check_cuda_4d(img2, "img2");
  TORCH_CHECK(img1.sizes() == img2.sizes(), "img1 and img2 must have the same shape");
  TORCH_CHECK(img1.scalar_type() == at::kFloat && img2.scalar_type() == at::kFloat,
              "expected scalar type Float for img1 and img2");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = img1.contiguous();
  auto b = img2.contiguous();
  auto map = torch::empty_like(a);
  auto opts = a.options();
  auto p0 = train ? torch::empty_like(a) : torch::empty({0}, opts);
  auto p1 = train ? torch::empty_like(a) : torch::empty({0}, opts);
  auto p2 = train ? torch::empty_like(a) : torch::empty({0}, opts);
  check_status(fssim_fusedssim(window_size, C1, C2, a.data_ptr<float>(), b.data_ptr<float>(),
                               a.size(0), a.size(1), a.size(2), a.size(3), train ? 1 : 0,
                               map.data_ptr<float>(), train ? p0.data_ptr<float>() : nullptr,
                               train ? p1.data_ptr<float>() : nullptr,
                               train ? p2.data_ptr<float>() : nullptr, current_stream()));
  return {map, p0, p1, p2};
}

torch::Tensor fusedssim_backward(int window_size, float C1, float C2, torch::Tensor& img1,
                                 torch::Tensor& img2, torch::Tensor& dL_dmap,
                                 torch::Tensor& dm_dmu1, torch::Tensor& dm_dsigma1_sq,
                                 torch::Tensor& dm_dsigma12) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  TORCH_CHECK(img1.scalar_type() == at::kFloat, "expected scalar type Float for img1");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = img1.contiguous();
  auto b = img2.contiguous().to(at::kFloat);
  auto dl = dL_dmap.to(at::kFloat).contiguous();
  auto q0 = dm_dmu1.contiguous();
  auto q1 = dm_dsigma1_sq.contiguous();
  auto q2 = dm_dsigma12.contiguous();
  const int64_t n = a.numel();
  TORCH_CHECK(b.numel() == n && dl.numel() == n && q0.numel() == n && q1.numel() == n &&
                  q2.numel() == n,
              "fusedssim_backward: all tensors must have img1's number of elements");
  auto grad = torch::empty_like(a);
  check_status(fssim_fusedssim_backward(
      window_size, C1, C2, a.data_ptr<float>(), b.data_ptr<float>(), dl.data_ptr<float>(),
      q0.data_ptr<float>(), q1.data_ptr<float>(), q2.data_ptr<float>(), a.size(0), a.size(1),
      a.size(2), a.size(3), grad.data_ptr<float>(), current_stream()));
  return grad;
}

torch::Tensor as_half(const torch::Tensor& t) {
  auto c = t.contiguous();
  return c.scalar_type() == at::kHalf ? c : c.to(at::kHalf);
}

torch::Tensor fusedssim_fp16(int window_size, float C1, float C2, torch::Tensor& img1,
                             torch::Tensor& img2) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  check_cuda_4d(img2, "img2");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = as_half(img1);
  auto b = as_half(img2);
  auto map = torch::empty(a.sizes(), a.options().dtype(at::kFloat));
  check_status(fssim_fusedssim_fp16(
      window_size, C1, C2, reinterpret_cast<const uint16_t*>(a.data_ptr<at::Half>()),
      reinterpret_cast<const uint16_t*>(b.data_ptr<at::Half>()), a.size(0), a.size(1),
      a.size(2), a.size(3), map.data_ptr<float>(), current_stream()));
  return map;
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor> fusedssim_fp16_train(
    int window_size, float C1, float C2, torch::Tensor& img1, torch::Tensor& img2) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  check_cuda_4d(img2, "img2");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = as_half(img1);
  auto b = as_half(img2);
  auto fopts = a.options().dtype(at::kFloat);
  auto map = torch::empty(a.sizes(), fopts);
  auto p0 = torch::empty(a.sizes(), fopts);
  auto p1 = torch::empty(a.sizes(), fopts);
  auto p2 = torch::empty(a.sizes(), fopts);
  check_status(fssim_fusedssim_fp16_train(
      window_size, C1, C2, reinterpret_cast<const uint16_t*>(a.data_ptr<at::Half>()),
      reinterpret_cast<const uint16_t*>(b.data_ptr<at::Half>()), a.size(0), a.size(1),
      a.size(2), a.size(3), map.data_ptr<float>(), p0.data_ptr<float>(), p1.data_ptr<float>(),
      p2.data_ptr<float>(), current_stream()));
  return {map, p0, p1, p2};
}

torch::Tensor fusedssim_fp16_backward(int window_size, float C1, float C2, torch::Tensor& img1,
                                      torch::Tensor& img2, torch::Tensor& dL_dmap,
                                      torch::Tensor& dm_dmu1, torch::Tensor& dm_dsigma1_sq,
                                      torch::Tensor& dm_dsigma12) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = as_half(img1);
  auto b = as_half(img2);
  auto dl = dL_dmap.to(at::kFloat).contiguous();
  auto q0 = dm_dmu1.contiguous();
  auto q1 = dm_dsigma1_sq.contiguous();
  auto q2 = dm_dsigma12.contiguous();
  const int64_t n = a.numel();
  TORCH_CHECK(b.numel() == n && dl.numel() == n && q0.numel() == n && q1.numel() == n &&
                  q2.numel() == n,
              "fusedssim_fp16_backward: all tensors must have img1's number of elements");
  auto grad = torch::empty(a.sizes(), a.options().dtype(at::kFloat));
  check_status(fssim_fusedssim_fp16_backward(
      window_size, C1, C2, reinterpret_cast<const uint16_t*>(a.data_ptr<at::Half>()),
      reinterpret_cast<const uint16_t*>(b.data_ptr<at::Half>()), dl.data_ptr<float>(),
      q0.data_ptr<float>(), q1.data_ptr<float>(), q2.data_ptr<float>(), a.size(0), a.size(1),
      a.size(2), a.size(3), grad.data_ptr<float>(), current_stream()));
  return grad;
}

// -------------------------------------------------------------------------------------
// Fused loss path
// -------------------------------------------------------------------------------------

// One zero-filled reduction workspace per (device, stream). The kernels leave it zeroed,
// and launches on one stream are ordered, so reuse is safe; distinct streams get distinct
// workspaces. Entries live for the whole process (never freed, so no teardown ordering).
torch::Tensor workspace_for(const torch::Tensor& like, int64_t B) {
  static std::mutex mu;
  static auto* cache = new std::unordered_map<std::string, torch::Tensor>();
  const auto stream = at::cuda::getCurrentCUDAStream();
  const std::string key = std::to_string(like.get_device()) + ":" +
                          std::to_string(reinterpret_cast<uintptr_t>(stream.stream()));
  const int64_t bytes = static_cast<int64_t>(fssim_forward_workspace_bytes(B));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache->find(key);
  if (it == cache->end() || it->second.numel() * 8 < bytes) {
    const int64_t words = (bytes + 7) / 8 + 32;
    auto ws = torch::zeros({words}, like.options().dtype(at::kLong));
    (*cache)[key] = ws;
    return ws;
  }
  return it->second;
}

// Forward of the fused loss. Returns (out, partials, image_sums):
//   out        () for reduce == 1, (B,) for reduce == 2, FP32;
//   partials   (3, B, C, H, W) in FP32 or FP16, or an empty tensor when !train;
//   image_sums (B,) FP64 per-image sums of the (cropped, clamped) map.
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> loss_forward_impl(
    torch::Tensor img1, torch::Tensor img2, int window_size, double C1, double C2, bool valid,
    bool clamp, bool train, int reduce, bool half_partials, double out_scale,
    double l1_weight, double out_offset, const fssim_dp_args* dp, bool with_sums = true) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  check_cuda_4d(img2, "img2");
  TORCH_CHECK(img1.sizes() == img2.sizes(), "img1 and img2 must have the same shape");
  TORCH_CHECK(reduce == 1 || reduce == 2, "reduce must be 1 (scalar) or 2 (per image)");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = img1.contiguous();
  auto b = img2.contiguous();
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "img1 and img2 must have the same dtype");
  const int dt = dtype_code(a.scalar_type());
  TORCH_CHECK(dt == FSSIM_F32 || dt == FSSIM_F16 || dt == FSSIM_BF16,
              "images must be float32, float16 or bfloat16");
  TORCH_CHECK(!(half_partials && dt == FSSIM_BF16), "FP16 partials need float16 images");
  const int64_t B = a.size(0);
  const int pdt = (half_partials && dt == FSSIM_F16) ? FSSIM_F16 : FSSIM_F32;
  auto partials =
      train ? torch::empty({3, a.size(0), a.size(1), a.size(2), a.size(3)},
                           a.options().dtype(pdt == FSSIM_F16 ? at::kHalf : at::kFloat))
            : torch::empty({0}, a.options().dtype(at::kFloat));
  auto out = reduce == 1 ? torch::empty({}, a.options().dtype(at::kFloat))
                         : torch::empty({B}, a.options().dtype(at::kFloat));
  // the per-image FP64 sums are returned by the loss_forward binding; the autograd path
  // does not use them and skips the allocation
  auto sums = with_sums ? torch::empty({B}, a.options().dtype(at::kDouble))
                        : torch::Tensor();
  auto ws = workspace_for(a, B);
  fssim_forward_args args{};
  args.dtype = dt;
  args.partial_dtype = pdt;
  args.B = a.size(0);
  args.C = a.size(1);
  args.H = a.size(2);
  args.W = a.size(3);
  args.window_size = window_size;
  args.valid = valid ? 1 : 0;
  args.clamp = clamp ? 1 : 0;
  args.train = train ? 1 : 0;
  args.reduce = reduce;
  args.C1 = static_cast<float>(C1);
  args.C2 = static_cast<float>(C2);
  args.out_scale = static_cast<float>(out_scale);
  args.l1_weight = static_cast<float>(l1_weight);
  args.out_offset = static_cast<float>(out_offset);
  args.img1 = a.data_ptr();
  args.img2 = b.data_ptr();
  args.ssim_map = nullptr;
  args.partials = train ? partials.data_ptr() : nullptr;
  args.out = out.data_ptr<float>();
  args.image_sums = with_sums ? sums.data_ptr<double>() : nullptr;
  args.workspace = ws.data_ptr();
  args.workspace_bytes = static_cast<size_t>(ws.numel()) * 8;
  check_status(dp ? fssim_forward_dp(&args, dp, current_stream())
                  : fssim_forward(&args, current_stream()));
  return {out, partials, sums};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> loss_forward(
    torch::Tensor img1, torch::Tensor img2, int window_size, double C1, double C2, bool valid,
    bool clamp, bool train, int reduce, bool half_partials, double out_scale, double l1_weight,
    double out_offset) {
  return loss_forward_impl(img1, img2, window_size, C1, C2, valid, clamp, train, reduce,
                           half_partials, out_scale, l1_weight, out_offset, nullptr);
}

// ---- batch-sharded loss: peer mailboxes over CUDA IPC ----
fssim_dp_args make_dp(int64_t world, int64_t rank, int64_t seq,
                      const std::vector<int64_t>& mailboxes) {
  TORCH_CHECK(world >= 1 && world <= FSSIM_DP_MAX_RANKS, "world out of range");
  TORCH_CHECK(static_cast<int64_t>(mailboxes.size()) == world, "one mailbox per rank");
  fssim_dp_args d{};
  d.world = static_cast<int32_t>(world);
  d.rank = static_cast<int32_t>(rank);
  d.seq = static_cast<uint64_t>(seq);
  for (int64_t r = 0; r < world; ++r) d.mailboxes[r] = reinterpret_cast<void*>(mailboxes[r]);
  return d;
}

// Forward of this rank's shard (reduce = scalar) that also publishes its sum to every rank.
std::tuple<torch::Tensor, torch::Tensor> loss_forward_dp(
    torch::Tensor img1, torch::Tensor img2, int window_size, double C1, double C2, bool valid,
    bool train, double out_scale, int64_t world, int64_t rank, int64_t seq,
    std::vector<int64_t> mailboxes) {
  const fssim_dp_args d = make_dp(world, rank, seq, mailboxes);
  auto r = loss_forward_impl(img1, img2, window_size, C1, C2, valid, false, train, 1, false,
                             out_scale, 0.0, 0.0, &d);
  return {std::get<0>(r), std::get<1>(r)};
}

// out (a 0-d FP32 CUDA tensor) = scale * the sum over ranks of step seq.
void dp_gather(torch::Tensor out, double scale, int64_t world, int64_t rank, int64_t seq,
               std::vector<int64_t> mailboxes) {
  TORCH_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.numel() == 1,
              "out must be a one-element float32 CUDA tensor");
  const at::cuda::OptionalCUDAGuard guard(out.device());
  const fssim_dp_args d = make_dp(world, rank, seq, mailboxes);
  check_status(fssim_dp_gather(&d, static_cast<float>(scale), out.data_ptr<float>(),
                               current_stream()));
}

int64_t dp_mailbox_alloc(int64_t world) {
  void* p = nullptr;
  check_status(fssim_dp_mailbox_alloc(static_cast<int>(world), &p));
  return reinterpret_cast<int64_t>(p);
}

void dp_mailbox_free(int64_t ptr) { check_status(fssim_dp_mailbox_free(reinterpret_cast<void*>(ptr))); }

py::bytes ipc_get_handle(int64_t ptr) {
  unsigned char h[FSSIM_IPC_HANDLE_BYTES];
  check_status(fssim_ipc_get_handle(reinterpret_cast<void*>(ptr), h));
  return py::bytes(reinterpret_cast<const char*>(h), FSSIM_IPC_HANDLE_BYTES);
}

int64_t ipc_open_handle(py::bytes handle) {
  const std::string h = handle;
  TORCH_CHECK(h.size() == FSSIM_IPC_HANDLE_BYTES, "IPC handle must be 64 bytes");
  void* p = nullptr;
  check_status(fssim_ipc_open_handle(reinterpret_cast<const unsigned char*>(h.data()), &p));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close_handle(int64_t ptr) {
  check_status(fssim_ipc_close_handle(reinterpret_cast<void*>(ptr)));
}

torch::Tensor loss_backward_impl(torch::Tensor grad_out, torch::Tensor img1,
                                 torch::Tensor img2, torch::Tensor partials, int window_size,
                                 bool per_image, double chain_scale, int grad_dtype,
                                 double l1_scale) {
  check_window(window_size);
  check_cuda_4d(img1, "img1");
  const at::cuda::OptionalCUDAGuard guard(img1.device());
  auto a = img1.contiguous();
  auto b = img2.contiguous();
  auto p = partials.contiguous();
  auto go = grad_out.to(at::kFloat).contiguous();
  const int64_t B = a.size(0);
  TORCH_CHECK(go.numel() == (per_image ? B : 1), "grad_out has the wrong number of elements");
  TORCH_CHECK(grad_dtype >= FSSIM_F32 && grad_dtype <= FSSIM_BF16,
              "grad_dtype code must be 0, 1 or 2");
  const at::ScalarType gt = grad_dtype == FSSIM_F32   ? at::kFloat
                            : grad_dtype == FSSIM_F16 ? at::kHalf
                                                      : at::kBFloat16;
  auto grad = torch::empty(a.sizes(), a.options().dtype(gt));
  fssim_backward_args args{};
  args.dtype = dtype_code(a.scalar_type());
  args.partial_dtype = dtype_code(p.scalar_type());
  args.grad_dtype = grad_dtype;
  args.B = B;
  args.C = a.size(1);
  args.H = a.size(2);
  args.W = a.size(3);
  args.window_size = window_size;
  args.img1 = a.data_ptr();
  args.img2 = b.data_ptr();
  args.partials = p.data_ptr();
  args.grad_out = go.data_ptr<float>();
  args.grad_out_per_image = per_image ? 1 : 0;
  args.chain_scale = static_cast<float>(chain_scale);
  args.l1_scale = static_cast<float>(l1_scale);
  args.grad = grad.data_ptr();
  check_status(fssim_backward(&args, current_stream()));
  return grad;
}

torch::Tensor loss_backward(torch::Tensor grad_out, torch::Tensor img1, torch::Tensor img2,
                            torch::Tensor partials, int window_size, bool per_image,
                            double chain_scale, int grad_dtype) {
  return loss_backward_impl(grad_out, img1, img2, partials, window_size, per_image,
                            chain_scale, grad_dtype, 0.0);
}

std::string version() { return fssim_version(); }

// The fused loss as a C++ autograd function: the same forward and backward as the Python
// _FusedSSIMLoss, without the Python layer in either direction (the backward runs on the
// autograd engine thread without taking the GIL). Inputs are converted for the kernels
// inside the forward (not recorded), and the gradient is returned in img1's dtype.
struct FusedLossFn : public torch::autograd::Function<FusedLossFn> {
  static torch::Tensor forward(torch::autograd::AutogradContext* ctx, torch::Tensor img1,
                               torch::Tensor img2, double C1, double C2, int64_t window_size,
                               bool valid, bool clamp, int64_t reduce, bool half,
                               double scale, double chain_scale, double l1_weight,
                               double out_offset, double l1_scale, const fssim_dp_args* dp,
                               bool gather) {
    torch::Tensor a, b;
    if (half) {
      a = img1.scalar_type() == at::kHalf ? img1 : img1.to(at::kHalf);
      b = img2.scalar_type() == at::kHalf ? img2 : img2.to(at::kHalf);
    } else {
      a = img1;
      b = img2.scalar_type() == img1.scalar_type() ? img2 : img2.to(img1.scalar_type());
    }
    auto r = loss_forward_impl(a, b, static_cast<int>(window_size), C1, C2, valid, clamp, true,
                               static_cast<int>(reduce), false, scale, l1_weight, out_offset,
                               dp, /*with_sums=*/false);
    if (dp && gather) {
      // sharded loss: out = scale * (sum over every rank's shard), formed on this GPU
      check_status(fssim_dp_gather(dp, static_cast<float>(scale),
                                   std::get<0>(r).data_ptr<float>(), current_stream()));
    }
    ctx->save_for_backward({a, b, std::get<1>(r)});
    ctx->saved_data["ws"] = window_size;
    ctx->saved_data["per_image"] = reduce == 2;
    ctx->saved_data["chain"] = chain_scale;
    ctx->saved_data["l1"] = l1_scale;
    ctx->saved_data["gdt"] = static_cast<int64_t>(dtype_code(img1.scalar_type()));
    return std::get<0>(r);
  }

  static torch::autograd::variable_list backward(torch::autograd::AutogradContext* ctx,
                                                 torch::autograd::variable_list grads) {
    const auto saved = ctx->get_saved_variables();
    auto grad = loss_backward_impl(grads[0], saved[0], saved[1], saved[2],
                                   static_cast<int>(ctx->saved_data["ws"].toInt()),
                                   ctx->saved_data["per_image"].toBool(),
                                   ctx->saved_data["chain"].toDouble(),
                                   static_cast<int>(ctx->saved_data["gdt"].toInt()),
                                   ctx->saved_data["l1"].toDouble());
    torch::autograd::variable_list out(16);
    out[0] = grad;
    return out;
  }
};

// out = scale * sum(ssim) + l1_weight * sum|img1 - img2| + out_offset (per image when
// reduce == 2); d(out)/d(map) = chain_scale, and l1_scale * sign(img1 - img2) per pixel.
torch::Tensor fused_loss(torch::Tensor img1, torch::Tensor img2, double C1, double C2,
                         int64_t window_size, bool valid, bool clamp, int64_t reduce, bool half,
                         double scale, double chain_scale, double l1_weight, double out_offset,
                         double l1_scale) {
  return FusedLossFn::apply(img1, img2, C1, C2, window_size, valid, clamp, reduce, half, scale,
                            chain_scale, l1_weight, out_offset, l1_scale,
                            static_cast<const fssim_dp_args*>(nullptr), false);
}

// The fused loss of this rank's shard of a batch sharded over several GPUs: the value is
// the mean over every rank's shard (peer mailboxes, fssim_forward_dp + fssim_dp_gather),
// the gradient is local (d(out)/d(map) = scale = 1 / global count). With gather = false the
// forward only publishes this rank's sum; the caller runs dp_gather on `out` itself (on
// another stream, so that the backward does not wait for the other ranks).
torch::Tensor fused_loss_dp(torch::Tensor img1, torch::Tensor img2, int64_t window_size,
                            bool valid, bool half, double scale, double chain_scale,
                            int64_t world, int64_t rank, int64_t seq,
                            std::vector<int64_t> mailboxes, bool gather) {
  const fssim_dp_args d = make_dp(world, rank, seq, mailboxes);
  return FusedLossFn::apply(img1, img2, 0.01 * 0.01, 0.03 * 0.03, window_size, valid, false,
                            int64_t{1}, half, scale, chain_scale, 0.0, 0.0, 0.0, &d, gather);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("fusedssim", &fusedssim);
  m.def("fusedssim_backward", &fusedssim_backward);
  m.def("fusedssim_fp16", &fusedssim_fp16);
  m.def("fusedssim_fp16_train", &fusedssim_fp16_train);
  m.def("fusedssim_fp16_backward", &fusedssim_fp16_backward);
  m.def("loss_forward", &loss_forward, py::arg("img1"), py::arg("img2"),
        py::arg("window_size"), py::arg("C1"), py::arg("C2"), py::arg("valid"),
        py::arg("clamp"), py::arg("train"), py::arg("reduce"), py::arg("half_partials"),
        py::arg("out_scale"), py::arg("l1_weight") = 0.0, py::arg("out_offset") = 0.0);
  m.def("loss_backward", &loss_backward);
  m.def("fused_loss", &fused_loss);
  m.def("fused_loss_dp", &fused_loss_dp, py::arg("img1"), py::arg("img2"),
        py::arg("window_size"), py::arg("valid"), py::arg("half"), py::arg("scale"),
        py::arg("chain_scale"), py::arg("world"), py::arg("rank"), py::arg("seq"),
        py::arg("mailboxes"), py::arg("gather") = true);
  m.def("loss_forward_dp", &loss_forward_dp);
  m.def("dp_gather", &dp_gather);
  m.def("dp_mailbox_alloc", &dp_mailbox_alloc);
  m.def("dp_mailbox_free", &dp_mailbox_free);
  m.def("ipc_get_handle", &ipc_get_handle);
  m.def("ipc_open_handle", &ipc_open_handle);
  m.def("ipc_close_handle", &ipc_close_handle);
  m.def("version", &version);
  m.def("set_reserved_sms", [](int n) {
    const int st = fssim_set_reserved_sms(n);
    if (st != FSSIM_OK) throw std::invalid_argument(fssim_last_error());
  });
  // device error flag of the current CUDA device (synchronises with it)
  m.def("poll_device_error", [](bool clear) {
    unsigned code = 0;
    check_status(fssim_poll_device_error(&code, clear ? 1 : 0));
    return static_cast<int64_t>(code);
  });
  m.def("set_loss_kernels", [](int family) { check_status(fssim_set_loss_kernels(family)); });
  m.def("set_staging_wait_limit", [](int64_t polls) {
    check_status(fssim_set_staging_wait_limit(static_cast<long long>(polls)));
  });
  m.def("set_gather_timeout_us", [](int64_t us) {
    check_status(fssim_set_gather_timeout_us(static_cast<long long>(us)));
  });
}
