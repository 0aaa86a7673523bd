// The reference's torch binding (dc740/gfx906 attn.cpp:1-21) restated for CUDA,
// used by tests/test_ref_binding_gpu.py to show that a binding written against
// the reference's C ABI links against libgfx906_b200_attn.so and runs on it.
//
// Only the HIP names change: hipStream_t -> cudaStream_t in the `launch`
// declaration (attn.cpp:4-5), ATen/hip/HIPContext.h -> ATen/cuda/CUDAContext.h,
// getCurrentHIPStream() -> getCurrentCUDAStream(). The checks, the
// .contiguous() copies, the empty_like output and the argument order of
// `launch` are the reference's (attn.cpp:7-18), because the point is that such
// a binding needs no other change.
#include <ATen/DeviceGuard.h>
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

extern "C" void launch(const void* q, const void* k, const void* v, void* o, int B, int H, int Sq, int Skv, int D,
                       float scale, cudaStream_t stream);

torch::Tensor attn(torch::Tensor q, torch::Tensor k, torch::Tensor v, double scale) {
  TORCH_CHECK(q.is_cuda() && q.dtype() == torch::kHalf);
  const at::DeviceGuard guard(q.device());
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(0) == k.size(0) && q.size(1) == k.size(1) && q.size(3) == k.size(3),
              "kernel: q/k/v shape mismatch");
  const auto B = q.size(0), H = q.size(1), Sq = q.size(2), Skv = k.size(2), D = q.size(3);
  TORCH_CHECK((D <= 64 && D % 8 == 0) || D == 128 || D == 512, "kernel: head_dim<=64 multiple of 8, 128, or 512");
  auto qc = q.contiguous();
  auto kc = k.contiguous();
  auto vc = v.contiguous();
  auto o = torch::empty_like(qc);
  launch(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), o.data_ptr(), static_cast<int>(B), static_cast<int>(H),
         static_cast<int>(Sq), static_cast<int>(Skv), static_cast<int>(D), static_cast<float>(scale),
         at::cuda::getCurrentCUDAStream());
  return o;
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) { m.def("attn", &attn); }
