// GroupNorm (+ optional SiLU) over channels-last (NHWC) bf16 activations, forward only.
//
// The VAE decoder of the reward path runs GroupNorm(32) -> SiLU -> conv at 512^2 resolution; on
// channels-last tensors the eager op converts layouts and reduces slowly.  Here:
//   1. stats:    grid (positions chunk, sample); each thread owns 8 consecutive channels (16-byte
//                loads) and accumulates per-group sum / sum of squares over its positions; block
//                partials are combined in shared memory and written per (sample, chunk, group);
//   2. finalize: mean / rstd per (sample, group) from the chunk partials (fp64 accumulation);
//   3. apply:    y = act((x - mean) * rstd * gamma[c] + beta[c]) in one read / one write pass.
#include "common.cuh"

namespace vo {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) gn_stats_kernel(const __nv_bfloat16* __restrict__ x, int64_t P, int C,
                                                            int G, int64_t pos_per_chunk, float* __restrict__ part) {
  // part: [N, chunks, G, 2]
  extern __shared__ float red[];  // [G][2]
  const int n = blockIdx.y;
  const int chunk = blockIdx.x, nchunks = gridDim.x;
  const int vpr = C / 8;  // 16-byte vectors per position
  const int cpg = C / G;  // channels per group
  for (int i = threadIdx.x; i < 2 * G; i += blockDim.x) red[i] = 0.f;
  __syncthreads();
  const int64_t p0 = (int64_t)chunk * pos_per_chunk;
  const int64_t p1 = min(P, p0 + pos_per_chunk);
  const bf16x8* base = reinterpret_cast<const bf16x8*>(x + (int64_t)n * P * C);
  // thread t handles vector column (t % vpr) of positions p0 + t / vpr, stepping by blockDim / vpr
  const int vc = threadIdx.x % vpr;
  const int pstep = blockDim.x / vpr;
  float s[8] = {0}, q[8] = {0};
  if (threadIdx.x < pstep * vpr) {
    for (int64_t p = p0 + threadIdx.x / vpr; p < p1; p += pstep) {
      float f[8];
      unpack8(base[p * vpr + vc], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j] += f[j];
        q[j] += f[j] * f[j];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int g = (vc * 8 + j) / cpg;
      atomicAdd(&red[2 * g], s[j]);
      atomicAdd(&red[2 * g + 1], q[j]);
    }
  }
  __syncthreads();
  float* out = part + ((int64_t)n * nchunks + chunk) * G * 2;
  for (int i = threadIdx.x; i < 2 * G; i += blockDim.x) out[i] = red[i];
}

__global__ void gn_finalize_kernel(const float* __restrict__ part, int nchunks, int G, double count, float eps,
                                   float* __restrict__ mean, float* __restrict__ rstd) {
  const int n = blockIdx.x;
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    double s = 0.0, q = 0.0;
    for (int c = 0; c < nchunks; ++c) {
      const float* p = part + (((int64_t)n * nchunks + c) * G + g) * 2;
      s += p[0];
      q += p[1];
    }
    const double mu = s / count;
    const double var = q / count - mu * mu;
    mean[n * G + g] = (float)mu;
    rstd[n * G + g] = (float)(1.0 / sqrt((var > 0.0 ? var : 0.0) + (double)eps));
  }
}

// grid (position chunks, sample): each thread owns one 8-channel vector column (fixed per thread, so the
// per-channel scale / shift are computed once) and walks positions with a stride; no integer division in
// the loop.
template <bool SILU>
__global__ void __launch_bounds__(kThreads) gn_apply_kernel(const __nv_bfloat16* __restrict__ x,
                                                            const __nv_bfloat16* __restrict__ gamma,
                                                            const __nv_bfloat16* __restrict__ beta,
                                                            const float* __restrict__ mean,
                                                            const float* __restrict__ rstd,
                                                            __nv_bfloat16* __restrict__ y, int64_t P, int C, int G,
                                                            int64_t pos_per_chunk) {
  const int n = blockIdx.y;
  const int vpr = C / 8;
  const int cpg = C / G;
  const int pstep = blockDim.x / vpr;
  if (threadIdx.x >= pstep * vpr) return;
  const int vc = threadIdx.x % vpr;
  float sc[8], sh[8];
  {
    float w[8], b[8];
    unpack8(reinterpret_cast<const bf16x8*>(gamma)[vc], w);
    unpack8(reinterpret_cast<const bf16x8*>(beta)[vc], b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int g = (vc * 8 + j) / cpg;
      const float r = rstd[n * G + g];
      sc[j] = r * w[j];
      sh[j] = b[j] - mean[n * G + g] * sc[j];
    }
  }
  const int64_t p0 = (int64_t)blockIdx.x * pos_per_chunk;
  const int64_t p1 = min(P, p0 + pos_per_chunk);
  const bf16x8* xin = reinterpret_cast<const bf16x8*>(x + (int64_t)n * P * C) + vc;
  bf16x8* yout = reinterpret_cast<bf16x8*>(y + (int64_t)n * P * C) + vc;
  for (int64_t p = p0 + threadIdx.x / vpr; p < p1; p += pstep) {
    float f[8], o[8];
    unpack8(xin[p * vpr], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float v = fmaf(f[j], sc[j], sh[j]);
      if (SILU) v = __fdividef(v, 1.f + __expf(-v));
      o[j] = v;
    }
    yout[p * vpr] = pack8(o);
  }
}

}  // namespace

// x: [N, C, H, W] bf16 in channels-last memory (NHWC); returns y in the same layout.
torch::Tensor group_norm_nhwc(torch::Tensor x, torch::Tensor gamma, torch::Tensor beta, int64_t groups, double eps,
                              bool silu) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.dim() == 4, "bf16 [N, C, H, W] input");
  TORCH_CHECK(x.is_contiguous(at::MemoryFormat::ChannelsLast), "input must be channels-last");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), C = x.size(1), P = x.size(2) * x.size(3);
  TORCH_CHECK(C % 8 == 0 && C % groups == 0 && (C / 8) <= kThreads, "C must be a multiple of 8 and of groups");
  TORCH_CHECK(gamma.numel() == C && beta.numel() == C && gamma.scalar_type() == torch::kBFloat16 &&
                  beta.scalar_type() == torch::kBFloat16,
              "bf16 affine parameters of length C");
  auto g = gamma.contiguous(), b = beta.contiguous();
  auto y = torch::empty_like(x, at::MemoryFormat::ChannelsLast);
  const int G = (int)groups;
  // ~4 blocks per SM over the batch for the statistics pass
  const int64_t want = std::max<int64_t>(1, 4LL * num_sms() / N);
  const int64_t per = std::max<int64_t>(64, (P + want - 1) / want);
  const int nchunks = (int)((P + per - 1) / per);
  auto fo = x.options().dtype(torch::kFloat32);
  auto part = torch::empty({N, nchunks, G, 2}, fo);
  auto mean = torch::empty({N, G}, fo), rstd = torch::empty({N, G}, fo);
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>());
  gn_stats_kernel<<<dim3(nchunks, (unsigned)N), kThreads, 2 * G * sizeof(float), stream()>>>(
      xp, P, (int)C, G, per, part.data_ptr<float>());
  gn_finalize_kernel<<<(unsigned)N, 64, 0, stream()>>>(part.data_ptr<float>(), nchunks, G, (double)P * (C / G),
                                                       (float)eps, mean.data_ptr<float>(), rstd.data_ptr<float>());
  // ~8 blocks per SM over the batch for the apply pass
  const int64_t want2 = std::max<int64_t>(1, 8LL * num_sms() / N);
  const int64_t per2 = std::max<int64_t>(32, (P + want2 - 1) / want2);
  const unsigned nch2 = (unsigned)((P + per2 - 1) / per2);
  auto* gp = reinterpret_cast<const __nv_bfloat16*>(g.data_ptr<at::BFloat16>());
  auto* bp = reinterpret_cast<const __nv_bfloat16*>(b.data_ptr<at::BFloat16>());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr<at::BFloat16>());
  if (silu)
    gn_apply_kernel<true><<<dim3(nch2, (unsigned)N), kThreads, 0, stream()>>>(
        xp, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), yp, P, (int)C, G, per2);
  else
    gn_apply_kernel<false><<<dim3(nch2, (unsigned)N), kThreads, 0, stream()>>>(
        xp, gp, bp, mean.data_ptr<float>(), rstd.data_ptr<float>(), yp, P, (int)C, G, per2);
  count_launch(3);
  VO_CUDA_OK(cudaGetLastError());
  return y;
}

}  // namespace vo
