// Fused clipped policy-gradient loss (FlowGRPO / DanceGRPO / MixGRPO per-step objective).
//   r = exp(logp - old); per = max(-A r, -A clip(r, 1-eps, 1+eps)) * w; loss = mean(per)
// plus ppo_kl, clip fractions and ratio mean/std, in one single-block kernel (B is one
// micro-batch of trajectories, so this is launch-bound: one launch instead of ~20 torch ops).
// Semantics: verl_omni/trainer/diffusion/diffusion_algos.py:307-342.
#include "common.cuh"

namespace vo {
namespace {

__global__ void ppo_clip_fwd_kernel(const float* __restrict__ logp, const float* __restrict__ old,
                                    const float* __restrict__ adv, const float* __restrict__ w, int B, float clip,
                                    float* __restrict__ loss, float* __restrict__ stats) {
  __shared__ float red[32];
  float s_per = 0, s_kl = 0, s_cf = 0, s_hi = 0, s_lo = 0, s_r = 0, s_r2 = 0;
  for (int i = threadIdx.x; i < B; i += blockDim.x) {
    float lr = logp[i] - old[i];
    float r = expf(lr);
    float a = adv[i];
    float unc = -a * r;
    float clp = -a * fminf(fmaxf(r, 1.f - clip), 1.f + clip);
    float per = fmaxf(unc, clp);
    if (w) per *= w[i];
    s_per += per;
    s_kl += -lr;
    s_cf += (fabsf(r - 1.f) > clip) ? 1.f : 0.f;
    s_hi += (r - 1.f > clip) ? 1.f : 0.f;
    s_lo += (1.f - r > clip) ? 1.f : 0.f;
    s_r += r;
  }
  s_per = block_sum(s_per, red);
  s_kl = block_sum(s_kl, red);
  s_cf = block_sum(s_cf, red);
  s_hi = block_sum(s_hi, red);
  s_lo = block_sum(s_lo, red);
  s_r = block_sum(s_r, red);
  const float mean_r = s_r / B;
  for (int i = threadIdx.x; i < B; i += blockDim.x) {
    float d = expf(logp[i] - old[i]) - mean_r;
    s_r2 += d * d;
  }
  s_r2 = block_sum(s_r2, red);
  if (threadIdx.x == 0) {
    loss[0] = s_per / B;
    stats[0] = s_kl / B;
    stats[1] = s_cf / B;
    stats[2] = s_hi / B;
    stats[3] = s_lo / B;
    stats[4] = mean_r;
    stats[5] = B > 1 ? sqrtf(s_r2 / (B - 1)) : 0.f;
  }
}

// d loss / d logp_i = (1/B) * w_i * d per_i / d r_i * r_i ; the max() picks the active branch
// (ties go to the unclipped branch, as torch.maximum's gradient splits evenly only on exact ties).
__global__ void ppo_clip_bwd_kernel(const float* __restrict__ logp, const float* __restrict__ old,
                                    const float* __restrict__ adv, const float* __restrict__ w, int B, float clip,
                                    const float* __restrict__ g_loss, float* __restrict__ g_logp) {
  const float g = g_loss[0] / B;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < B; i += gridDim.x * blockDim.x) {
    float r = expf(logp[i] - old[i]);
    float a = adv[i];
    float rc = fminf(fmaxf(r, 1.f - clip), 1.f + clip);
    float unc = -a * r, clp = -a * rc;
    float d;
    if (unc > clp)
      d = -a * r;
    else if (unc < clp)
      d = (r > 1.f - clip && r < 1.f + clip) ? -a * r : 0.f;
    else
      d = (r > 1.f - clip && r < 1.f + clip) ? -a * r : -0.5f * a * r;
    if (w) d *= w[i];
    g_logp[i] = g * d;
  }
}

}  // namespace

std::vector<torch::Tensor> ppo_clip_fwd(torch::Tensor logp, torch::Tensor old, torch::Tensor adv,
                                        c10::optional<torch::Tensor> w, double clip) {
  VO_CHECK_INPUT(logp);
  VO_CHECK_INPUT(old);
  VO_CHECK_INPUT(adv);
  c10::cuda::CUDAGuard g(logp.device());
  const int B = logp.numel();
  auto loss = torch::empty({}, logp.options());
  auto stats = torch::empty({6}, logp.options());
  const float* wp = (w.has_value() && w->defined()) ? w->data_ptr<float>() : nullptr;
  ppo_clip_fwd_kernel<<<1, 256, 0, stream()>>>(logp.data_ptr<float>(), old.data_ptr<float>(), adv.data_ptr<float>(),
                                               wp, B, (float)clip, loss.data_ptr<float>(), stats.data_ptr<float>()); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {loss, stats};
}

torch::Tensor ppo_clip_bwd(torch::Tensor logp, torch::Tensor old, torch::Tensor adv, c10::optional<torch::Tensor> w,
                           double clip, torch::Tensor g_loss) {
  c10::cuda::CUDAGuard g(logp.device());
  const int B = logp.numel();
  auto gl = torch::empty_like(logp);
  const float* wp = (w.has_value() && w->defined()) ? w->data_ptr<float>() : nullptr;
  ppo_clip_bwd_kernel<<<(B + 255) / 256, 256, 0, stream()>>>(logp.data_ptr<float>(), old.data_ptr<float>(),
                                                             adv.data_ptr<float>(), wp, B, (float)clip,
                                                             g_loss.data_ptr<float>(), gl.data_ptr<float>()); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return gl;
}

}  // namespace vo
