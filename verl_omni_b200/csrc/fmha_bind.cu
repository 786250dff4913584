// Torch-facing wrapper of the tcgen05 flash-attention forward.
#include "common.cuh"

extern "C" int vo_fmha_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Sq,
                           int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_error(int reset);
extern "C" int vo_fmha_fwd2(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Sq,
                            int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_fwd2_error(int reset);
extern "C" int vo_fmha_fwd3(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Sq,
                            int Skv, int D, float scale, int causal, cudaStream_t stream);
extern "C" int vo_fmha_bwd(const void* q, const void* k, const void* v, const void* o, const void* dO,
                           const float* lse, void* dq, void* dk, void* dv, float* delta, float* dq_acc, int B, int H,
                           int Sq, int Skv, int D, float scale, int causal, cudaStream_t stream, int version);
extern "C" int vo_fmha_bwd_error(int reset);

namespace vo {

// q [B, H, Sq, D], k/v [B, H, Skv, D] -> (o [B, Sq, H, D], lse [B, H, Sq] fp32)
// version 1: one query tile per CTA, P staged in shared memory; version 2: two query tiles per CTA,
// P and O resident in tensor memory; version 3: as 2 with two softmax warpgroups per query tile.
std::vector<torch::Tensor> fmha_fwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, bool causal, double scale,
                                    int64_t version) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k);
  VO_CHECK_INPUT(v);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16, "bf16 attention inputs");
  c10::cuda::CUDAGuard g(q.device());
  const int B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  auto o = torch::empty({B, Sq, H, D}, q.options());
  auto lse = torch::empty({B, H, Sq}, q.options().dtype(torch::kFloat32));
  auto fn = version == 3 ? vo_fmha_fwd3 : version == 2 ? vo_fmha_fwd2 : vo_fmha_fwd;
  int rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr<float>(), B, H, Sq, Skv, D,
              (float)scale, causal ? 1 : 0, stream());
  TORCH_CHECK(rc == 0, "tcgen05 FMHA launch failed: code ", rc);
  count_launch();
  return {o, lse};
}

int64_t fmha_error(bool reset) {
  return vo_fmha_error(reset ? 1 : 0) | vo_fmha_fwd2_error(reset ? 1 : 0) | vo_fmha_bwd_error(reset ? 1 : 0);
}

// returns dq, dk, dv in the [B, H, S, D] layout of q, k, v
// version 1: one key tile per CTA, serial per query tile; version 2: pipelined (P^T / dS^T in
// tensor memory, concurrent dQ drain, next S^T overlapped for head_dim 64)
std::vector<torch::Tensor> fmha_bwd(torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor o,
                                    torch::Tensor lse, torch::Tensor dO, bool causal, double scale, int64_t version) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k);
  VO_CHECK_INPUT(v);
  VO_CHECK_INPUT(o);
  VO_CHECK_INPUT(dO);
  VO_CHECK_INPUT(lse);
  c10::cuda::CUDAGuard g(q.device());
  const int B = q.size(0), H = q.size(1), Sq = q.size(2), D = q.size(3), Skv = k.size(2);
  TORCH_CHECK(D == 64 || D == 128, "head_dim must be 64 or 128");
  auto dq = torch::empty_like(q);
  auto dk = torch::empty_like(k);
  auto dv = torch::empty_like(v);
  auto fo = q.options().dtype(torch::kFloat32);
  auto delta = torch::empty({B, H, Sq}, fo);
  auto dq_acc = torch::zeros({B, H, Sq, D}, fo);
  int rc = vo_fmha_bwd(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), dO.data_ptr(), lse.data_ptr<float>(),
                       dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), delta.data_ptr<float>(), dq_acc.data_ptr<float>(),
                       B, H, Sq, Skv, D, (float)scale, causal ? 1 : 0, stream(), (int)version);
  TORCH_CHECK(rc == 0, "tcgen05 FMHA backward launch failed: code ", rc);
  count_launch(3);
  return {dq, dk, dv};
}

}  // namespace vo
