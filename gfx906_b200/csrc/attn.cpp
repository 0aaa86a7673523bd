// Torch operator `attn(q, k, v, scale) -> o` over the C-ABI launch shim.
//
// Same Python name, signature and checks as the reference binding
// (attn.cpp:6-21): q must be a CUDA fp16 tensor, k and v must have equal
// shapes, batch / heads / head_dim must match q, head_dim must be <= 64 and a
// multiple of 8, or 128, or 512; inputs are made contiguous, the output is a
// new contiguous [B,H,Sq,D] fp16 tensor, and the kernel is launched on the
// current stream of q's device. Two checks are added: k and v must also be
// CUDA fp16 tensors on q's device (the reference only checked q), and every
// tensor must be 4-D. Failures raise RuntimeError (TORCH_CHECK).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <map>
#include <mutex>
#include <utility>

#include "../../include/gfx906_b200_attn.h"

// One workspace per (device, stream), reused by every call on that stream and
// grown on demand. A workspace is never shared by two streams, so calls that
// overlap on the GPU never share one.
static std::mutex g_ws_mu;
static std::map<std::pair<int, cudaStream_t>, torch::Tensor> g_ws;

static torch::Tensor workspace_for(const torch::Tensor& like, cudaStream_t stream, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_ws_mu);
  auto key = std::make_pair(static_cast<int>(like.get_device()), stream);
  auto it = g_ws.find(key);
  if (it != g_ws.end() && static_cast<size_t>(it->second.numel()) >= bytes) return it->second;
  auto t = torch::empty({static_cast<int64_t>(bytes)}, like.options().dtype(torch::kUInt8));
  g_ws[key] = t;
  return t;
}

torch::Tensor attn(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale) {
  TORCH_CHECK(q.is_cuda() && q.dtype() == torch::kHalf, "kernel: q must be a CUDA float16 tensor");
  TORCH_CHECK(k.is_cuda() && v.is_cuda() && k.dtype() == torch::kHalf && v.dtype() == torch::kHalf,
              "kernel: k and v must be CUDA float16 tensors");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "kernel: q, k and v must be on the same device");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "kernel: q/k/v must be [B,H,S,D]");
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(1) == k.size(1) &&
                  q.size(3) == k.size(3),
              "kernel: q/k/v shape mismatch");
  const auto B = q.size(0), H = q.size(1), Sq = q.size(2), Skv = k.size(2), D = q.size(3);
  TORCH_CHECK((D <= 64 && D % 8 == 0) || D == 128 || D == 512,
              "kernel: head_dim<=64 multiple of 8, 128, or 512");
  TORCH_CHECK(B <= INT32_MAX && H <= INT32_MAX && Sq <= INT32_MAX && Skv <= INT32_MAX,
              "kernel: sizes must fit in int32");
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  auto o = torch::empty_like(qc);
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const size_t ws_bytes = gfx906_b200_attn_workspace_size(static_cast<int>(B), static_cast<int>(H),
                                                          static_cast<int>(Sq), static_cast<int>(Skv),
                                                          static_cast<int>(D));
  void* ws = nullptr;
  if (ws_bytes > 0) ws = workspace_for(q, stream, ws_bytes).data_ptr();
  const int rc = gfx906_b200_attn_launch_ws(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(),
                                            static_cast<int>(B), static_cast<int>(H), static_cast<int>(Sq),
                                            static_cast<int>(Skv), static_cast<int>(D),
                                            static_cast<float>(scale), ws, ws_bytes, stream);
  TORCH_CHECK(rc == GFX906_B200_OK, "kernel: ", gfx906_b200_attn_error_string(rc));
  return o;
}

// attn into a caller-provided output: o must be a contiguous CUDA fp16 tensor
// shaped like q on q's device (same checks on q, k, v as attn). Lets a caller
// that reuses device buffers (attn_host) run without allocating.
void attn_out(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale, torch::Tensor o) {
  TORCH_CHECK(q.is_cuda() && q.dtype() == torch::kHalf, "kernel: q must be a CUDA float16 tensor");
  TORCH_CHECK(k.is_cuda() && v.is_cuda() && k.dtype() == torch::kHalf && v.dtype() == torch::kHalf,
              "kernel: k and v must be CUDA float16 tensors");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "kernel: q, k and v must be on the same device");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "kernel: q/k/v must be [B,H,S,D]");
  TORCH_CHECK(o.is_cuda() && o.dtype() == torch::kHalf && o.device() == q.device() && o.is_contiguous() &&
                  o.sizes() == q.sizes(),
              "kernel: o must be a contiguous CUDA float16 tensor shaped like q on q's device");
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(1) == k.size(1) &&
                  q.size(3) == k.size(3),
              "kernel: q/k/v shape mismatch");
  const auto B = q.size(0), H = q.size(1), Sq = q.size(2), Skv = k.size(2), D = q.size(3);
  TORCH_CHECK((D <= 64 && D % 8 == 0) || D == 128 || D == 512,
              "kernel: head_dim<=64 multiple of 8, 128, or 512");
  TORCH_CHECK(B <= INT32_MAX && H <= INT32_MAX && Sq <= INT32_MAX && Skv <= INT32_MAX,
              "kernel: sizes must fit in int32");
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  const cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  const size_t ws_bytes = gfx906_b200_attn_workspace_size(static_cast<int>(B), static_cast<int>(H),
                                                          static_cast<int>(Sq), static_cast<int>(Skv),
                                                          static_cast<int>(D));
  void* ws = nullptr;
  if (ws_bytes > 0) ws = workspace_for(q, stream, ws_bytes).data_ptr();
  const int rc = gfx906_b200_attn_launch_ws(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(),
                                            static_cast<int>(B), static_cast<int>(H), static_cast<int>(Sq),
                                            static_cast<int>(Skv), static_cast<int>(D),
                                            static_cast<float>(scale), ws, ws_bytes, stream);
  TORCH_CHECK(rc == GFX906_B200_OK, "kernel: ", gfx906_b200_attn_error_string(rc));
}

// Attention on transposed ("d-major") tensors: q [B,H,D,Sq], k and v
// [B,H,D,Skv], D = 512, sequence innermost; returns o as [B,H,D,Sq]. A
// [b, c, h, w] feature map viewed as [b, 1, c, h*w] is this layout, so the VAE
// mid-block attention runs without transposing anything. Inputs are made
// contiguous in this layout (a no-op for feature maps). Sq and Skv must be
// multiples of 8.
torch::Tensor attn_dmajor(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda() && q.dtype() == torch::kHalf &&
                  k.dtype() == torch::kHalf && v.dtype() == torch::kHalf,
              "kernel: q, k and v must be CUDA float16 tensors");
  TORCH_CHECK(k.device() == q.device() && v.device() == q.device(),
              "kernel: q, k and v must be on the same device");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "kernel: q/k/v must be [B,H,D,S]");
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(1) == k.size(1) &&
                  q.size(2) == k.size(2),
              "kernel: q/k/v shape mismatch");
  const auto B = q.size(0), H = q.size(1), D = q.size(2), Sq = q.size(3), Skv = k.size(3);
  TORCH_CHECK(D == 512, "kernel: the transposed layout needs head_dim 512");
  TORCH_CHECK(Sq % 8 == 0 && Skv % 8 == 0, "kernel: the transposed layout needs sequence lengths % 8 == 0");
  TORCH_CHECK(B <= INT32_MAX && H <= INT32_MAX && Sq <= INT32_MAX && Skv <= INT32_MAX,
              "kernel: sizes must fit in int32");
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  auto o = torch::empty_like(qc);
  const int rc = gfx906_b200_attn_launch_dmajor(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(),
                                                static_cast<int>(B), static_cast<int>(H), static_cast<int>(Sq),
                                                static_cast<int>(Skv), static_cast<int>(D),
                                                static_cast<float>(scale), at::cuda::getCurrentCUDAStream());
  TORCH_CHECK(rc == GFX906_B200_OK, "kernel: ", gfx906_b200_attn_error_string(rc));
  return o;
}

// Device status word of the current device (see gfx906_b200_attn_device_status).
// Returns 0 when no kernel wait has timed out. Synchronises.
int64_t device_status(bool reset) { return gfx906_b200_attn_device_status(reset ? 1 : 0); }

// Process-wide cap on the SMs the persistent kernels use (0 = all); returns
// the previous cap (see gfx906_b200_attn_set_sm_limit).
int64_t set_sm_limit(int64_t sms) {
  TORCH_CHECK(sms >= 0 && sms <= INT32_MAX, "kernel: sm limit must be >= 0");
  return gfx906_b200_attn_set_sm_limit(static_cast<int>(sms));
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("attn", &attn, "flash-attention forward (fp16 [B,H,S,D], sm_100a)");
  m.def("attn_out", &attn_out, "flash-attention forward into a given contiguous fp16 output tensor");
  m.def("attn_dmajor", &attn_dmajor, "flash-attention forward on transposed [B,H,D,S] fp16, D = 512");
  m.def("device_status", &device_status, "device status word (0 = ok)", pybind11::arg("reset") = false);
  m.def("set_sm_limit", &set_sm_limit, "cap on the SMs the persistent kernels use (0 = all); returns the previous");
}
