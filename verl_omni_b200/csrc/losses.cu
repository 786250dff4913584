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

// ------------------------------------------------------------------------------------------------
// Per-sample mean squared distance d_b = mean_i (a_bi - b_bi)^2 of two fp32 [B, n] tensors (the KL
// term of Flow-DPPO, GRPO-Guard, the reference KL and the distillation KL between reverse-SDE means):
// one pass, fp32 accumulation, block partial sums per (sample, chunk) then a chunk reduction.
namespace vo {
namespace {

__global__ void sq_dist_partial_kernel(const float4* __restrict__ a, const float4* __restrict__ b, int64_t n4,
                                       int chunks, float* __restrict__ part) {
  __shared__ float red[32];
  const int row = blockIdx.y, ch = blockIdx.x;
  const int64_t per = (n4 + chunks - 1) / chunks;
  const int64_t lo = (int64_t)ch * per, hi = min(n4, lo + per);
  const float4* ar = a + (int64_t)row * n4;
  const float4* br = b + (int64_t)row * n4;
  float s = 0.f;
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float4 x = ar[i], y = br[i];
    const float d0 = x.x - y.x, d1 = x.y - y.y, d2 = x.z - y.z, d3 = x.w - y.w;
    s += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) part[(int64_t)row * chunks + ch] = s;
}

__global__ void sq_dist_finalize_kernel(const float* __restrict__ part, int B, int chunks, float inv_n,
                                        float* __restrict__ out) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= B) return;
  float s = 0.f;
  for (int c = 0; c < chunks; ++c) s += part[(int64_t)row * chunks + c];
  out[row] = s * inv_n;
}

// ga = 2 (a - b) / n * g_row ; gb = -ga
__global__ void sq_dist_bwd_kernel(const float4* __restrict__ a, const float4* __restrict__ b,
                                   const float* __restrict__ g, int64_t n4, float inv_n, float4* __restrict__ ga,
                                   float4* __restrict__ gb, int64_t total4) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += (int64_t)gridDim.x * blockDim.x) {
    const float s = 2.f * inv_n * g[i / n4];
    const float4 x = a[i], y = b[i];
    const float4 r = make_float4(s * (x.x - y.x), s * (x.y - y.y), s * (x.z - y.z), s * (x.w - y.w));
    ga[i] = r;
    if (gb) gb[i] = make_float4(-r.x, -r.y, -r.z, -r.w);
  }
}

}  // namespace

// a, b: fp32 [B, ...] contiguous, per-sample element count a multiple of 4 -> [B] fp32
torch::Tensor sq_dist_fwd(torch::Tensor a, torch::Tensor b) {
  VO_CHECK_INPUT(a);
  VO_CHECK_INPUT(b);
  TORCH_CHECK(a.scalar_type() == torch::kFloat32 && b.scalar_type() == torch::kFloat32 && a.sizes() == b.sizes(),
              "fp32 tensors of one shape");
  const int B = (int)a.size(0);
  const int64_t n = a.numel() / std::max(B, 1);
  TORCH_CHECK(n % 4 == 0 && B >= 1 && B <= 65535, "per-sample size a multiple of 4, 1..65535 samples");
  c10::cuda::CUDAGuard g(a.device());
  const int64_t n4 = n / 4;
  const int chunks = (int)std::max<int64_t>(1, std::min<int64_t>((n4 + 2047) / 2048, (4 * num_sms() + B - 1) / B));
  auto part = torch::empty({B, chunks}, a.options());
  auto out = torch::empty({B}, a.options());
  sq_dist_partial_kernel<<<dim3(chunks, B), 256, 0, stream()>>>(reinterpret_cast<const float4*>(a.data_ptr<float>()),
                                                                reinterpret_cast<const float4*>(b.data_ptr<float>()),
                                                                n4, chunks, part.data_ptr<float>());
  sq_dist_finalize_kernel<<<(B + 127) / 128, 128, 0, stream()>>>(part.data_ptr<float>(), B, chunks, 1.f / (float)n,
                                                                 out.data_ptr<float>());
  count_launch(2);
  VO_CUDA_OK(cudaGetLastError());
  return out;
}

std::vector<torch::Tensor> sq_dist_bwd(torch::Tensor a, torch::Tensor b, torch::Tensor g, bool want_gb) {
  VO_CHECK_INPUT(a);
  VO_CHECK_INPUT(b);
  VO_CHECK_INPUT(g);
  const int B = (int)a.size(0);
  const int64_t n = a.numel() / B;
  c10::cuda::CUDAGuard gd(a.device());
  auto ga = torch::empty_like(a);
  torch::Tensor gb = want_gb ? torch::empty_like(b) : torch::Tensor();
  const int64_t total4 = a.numel() / 4;
  const int grid = (int)std::min<int64_t>((total4 + 255) / 256, 16LL * num_sms());
  sq_dist_bwd_kernel<<<grid, 256, 0, stream()>>>(reinterpret_cast<const float4*>(a.data_ptr<float>()),
                                                 reinterpret_cast<const float4*>(b.data_ptr<float>()),
                                                 g.data_ptr<float>(), n / 4, 1.f / (float)n,
                                                 reinterpret_cast<float4*>(ga.data_ptr<float>()),
                                                 want_gb ? reinterpret_cast<float4*>(gb.data_ptr<float>()) : nullptr,
                                                 total4);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  if (want_gb) return {ga, gb};
  return {ga};
}

}  // namespace vo
