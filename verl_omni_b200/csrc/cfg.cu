// Classifier-free guidance combine (+ optional "true CFG" norm renormalisation) in one pass.
//
//   comb = neg + g * (pos - neg)
//   renorm: comb *= ||pos|| / ||comb||, norms over the channel axis at each (sample, position)
//
// Tensors are [B, C, P] (channel-major latents, P = spatial positions) in fp32 or bf16; the output is
// fp32.  One thread owns one (b, position) column and walks the C channels (stride P), so reads are
// coalesced across threads.  Replaces the three-to-six elementwise/reduction passes of the eager form.
#include "common.cuh"

namespace vo {
namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  return static_cast<float>(*p);
}
template <>
__device__ __forceinline__ float ld<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}

template <typename T, bool RENORM>
__global__ void cfg_kernel(const T* __restrict__ pos, const T* __restrict__ neg, float* __restrict__ out, int64_t B,
                           int C, int64_t P, float g) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= B * P) return;
  const int64_t b = idx / P, s = idx % P;
  const int64_t base = b * C * P + s;
  float scale = 1.f;
  if (RENORM) {
    float sp = 0.f, sc = 0.f;
    for (int c = 0; c < C; ++c) {
      const float p = ld(pos + base + (int64_t)c * P), n = ld(neg + base + (int64_t)c * P);
      const float m = n + g * (p - n);
      sp += p * p;
      sc += m * m;
    }
    scale = sc > 0.f ? sqrtf(sp) / sqrtf(sc) : 1.f;
  }
  for (int c = 0; c < C; ++c) {
    const int64_t o = base + (int64_t)c * P;
    const float p = ld(pos + o), n = ld(neg + o);
    out[o] = (n + g * (p - n)) * scale;
  }
}

}  // namespace

// pos/neg [B, C, ...] -> fp32 combined prediction of the same shape
torch::Tensor cfg_combine(torch::Tensor pos, torch::Tensor neg, double g, bool renorm) {
  VO_CHECK_INPUT(pos);
  VO_CHECK_INPUT(neg);
  TORCH_CHECK(pos.sizes() == neg.sizes() && pos.scalar_type() == neg.scalar_type(), "pos/neg mismatch");
  TORCH_CHECK(pos.dim() >= 2, "expected [B, C, ...]");
  c10::cuda::CUDAGuard guard(pos.device());
  const int64_t B = pos.size(0);
  const int C = (int)pos.size(1);
  const int64_t P = pos.numel() / (B * C);
  auto out = torch::empty(pos.sizes(), pos.options().dtype(torch::kFloat32));
  const int64_t n = B * P;
  if (n == 0) return out;
  const unsigned grid = (unsigned)((n + 255) / 256);
  const float gf = (float)g;
  if (pos.scalar_type() == torch::kFloat32) {
    if (renorm)
      cfg_kernel<float, true><<<grid, 256, 0, stream()>>>(pos.data_ptr<float>(), neg.data_ptr<float>(),
                                                          out.data_ptr<float>(), B, C, P, gf);
    else
      cfg_kernel<float, false><<<grid, 256, 0, stream()>>>(pos.data_ptr<float>(), neg.data_ptr<float>(),
                                                           out.data_ptr<float>(), B, C, P, gf);
  } else {
    TORCH_CHECK(pos.scalar_type() == torch::kBFloat16, "fp32 or bf16 predictions");
    auto* pp = reinterpret_cast<const __nv_bfloat16*>(pos.data_ptr<at::BFloat16>());
    auto* np_ = reinterpret_cast<const __nv_bfloat16*>(neg.data_ptr<at::BFloat16>());
    if (renorm)
      cfg_kernel<__nv_bfloat16, true><<<grid, 256, 0, stream()>>>(pp, np_, out.data_ptr<float>(), B, C, P, gf);
    else
      cfg_kernel<__nv_bfloat16, false><<<grid, 256, 0, stream()>>>(pp, np_, out.data_ptr<float>(), B, C, P, gf);
  }
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return out;
}

}  // namespace vo
