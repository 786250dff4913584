// Torch-facing wrapper of the tcgen05 flash-attention forward.
#include "common.cuh"

extern "C" int vo_fmha_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Sq,
                           int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_error(int reset);

namespace vo {

// q [B, H, Sq, D], k/v [B, H, Skv, D] -> (o [B, Sq, H, D], lse [B, H, Sq] fp32)
std::vector<torch::Tensor> fmha_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, double scale) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k);
  VO_CHECK_INPUT(v);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "bf16 attention inputs");
  c10::cuda::CUDAGuard g(q.device());
  const int B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  auto o = torch::empty({B, Sq, H, D}, q.options());
  auto lse = torch::empty({B, H, Sq}, q.options().dtype(torch::kFloat32));
  int rc = vo_fmha_fwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), B, H, Sq, Skv,
                       D, (float)scale, causal ? 1 : 0, stream());
  TORCH_CHECK(rc == 0, "tcgen05 FMHA launch failed: code ", rc);
  count_launch();
  return {o, lse};
}

int64_t fmha_error(bool reset) { return vo_fmha_error(reset ? 1 : 0); }

}  // namespace vo
