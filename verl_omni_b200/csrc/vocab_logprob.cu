// Token log-probabilities over a large vocabulary without materialising [tokens, vocab] fp32 logits.
//
// The language-model head is processed in vocabulary chunks: the tcgen05 GEMM writes one bf16 logits
// chunk [N, Vc] at a time, and these row kernels fold it into per-row running statistics:
//   lse_update:  (m, s) <- online log-sum-exp of logits / T over the chunk; the target's logit / T is
//                picked up when the target id falls inside the chunk;
//   lse_grad:    in place over the recomputed chunk, dlogits = g / T * (onehot(target) - exp(z / T - lse))
//                in bf16, the operand of the dgrad and wgrad GEMMs of the chunk.
// One CTA per row, 16-byte vector loads, fp32 arithmetic.  Peak extra memory: one chunk of bf16 logits.
#include "common.cuh"

namespace vo {
namespace {

constexpr int kLseThreads = 256;

__device__ __forceinline__ void combine(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = (m == -INFINITY ? 0.f : s * __expf(m - mn)) + (m2 == -INFINITY ? 0.f : s2 * __expf(m2 - mn));
  m = mn;
}

__global__ void __launch_bounds__(kLseThreads) lse_update_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld,
                                                                 int Vc, int64_t lo, const int64_t* __restrict__ tgt,
                                                                 float inv_t, float* __restrict__ m_io,
                                                                 float* __restrict__ s_io, float* __restrict__ t_io) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const int nv = Vc / 8;
  for (int i = threadIdx.x; i < nv; i += kLseThreads) {
    float f[8];
    unpack8(reinterpret_cast<const bf16x8*>(x)[i], f);
    float mx = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) mx = fmaxf(mx, f[j]);
    mx *= inv_t;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += __expf(f[j] * inv_t - mx);
    combine(m, s, mx, acc);
  }
  for (int i = nv * 8 + threadIdx.x; i < Vc; i += kLseThreads) combine(m, s, bf2f(x[i]) * inv_t, 1.f);
  // block reduction of (m, s)
  __shared__ float sm_m[kLseThreads / 32], sm_s[kLseThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    combine(m, s, m2, s2);
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sm_m[w] = m;
    sm_s[w] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = m_io[row], S = s_io[row];
    for (int i = 0; i < kLseThreads / 32; ++i) combine(M, S, sm_m[i], sm_s[i]);
    m_io[row] = M;
    s_io[row] = S;
    const int64_t t = tgt[row] - lo;
    if (t >= 0 && t < Vc) t_io[row] = bf2f(x[t]) * inv_t;
  }
}

__global__ void __launch_bounds__(kLseThreads) lse_grad_kernel(__nv_bfloat16* __restrict__ logits, int64_t ld, int Vc,
                                                               int64_t lo, const int64_t* __restrict__ tgt,
                                                               float inv_t, const float* __restrict__ lse,
                                                               const float* __restrict__ g) {
  const int64_t row = blockIdx.x;
  bf16x8* x = reinterpret_cast<bf16x8*>(logits + row * ld);
  const float L = lse[row], gr = g[row] * inv_t;
  const int64_t t = tgt[row] - lo;
  const int nv = Vc / 8;
  for (int i = threadIdx.x; i < nv; i += kLseThreads) {
    float f[8];
    unpack8(x[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p = __expf(f[j] * inv_t - L);
      f[j] = gr * ((int64_t)(i * 8 + j) == t ? 1.f - p : -p);
    }
    x[i] = pack8(f);
  }
  __nv_bfloat16* xs = logits + row * ld;
  for (int i = nv * 8 + threadIdx.x; i < Vc; i += kLseThreads) {
    const float p = __expf(bf2f(xs[i]) * inv_t - L);
    xs[i] = f2bf(gr * ((int64_t)i == t ? 1.f - p : -p));
  }
}

}  // namespace

// logits [N, Vc] bf16 (row stride ld, 16-byte aligned rows); targets int64 [N]; m, s, tgt_logit fp32 [N]
// updated in place (start from -inf / 0 / anything).
void vocab_lse_update(torch::Tensor logits, int64_t lo, torch::Tensor targets, double inv_t, torch::Tensor m,
                      torch::Tensor s, torch::Tensor t) {
  VO_CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1 &&
                  logits.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0,
              "bf16 [N, Vc] logits with 16-byte aligned rows");
  VO_CHECK_INPUT(targets);
  VO_CHECK_INPUT(m);
  VO_CHECK_INPUT(s);
  VO_CHECK_INPUT(t);
  TORCH_CHECK(targets.scalar_type() == torch::kInt64 && m.scalar_type() == torch::kFloat32 &&
                  s.scalar_type() == torch::kFloat32 && t.scalar_type() == torch::kFloat32,
              "int64 targets, fp32 statistics");
  const int64_t N = logits.size(0);
  TORCH_CHECK(targets.numel() == N && m.numel() == N && s.numel() == N && t.numel() == N, "one row per token");
  if (N == 0) return;
  c10::cuda::CUDAGuard g(logits.device());
  lse_update_kernel<<<(unsigned)N, kLseThreads, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(logits.data_ptr<at::BFloat16>()), logits.stride(0), (int)logits.size(1),
      lo, targets.data_ptr<int64_t>(), (float)inv_t, m.data_ptr<float>(), s.data_ptr<float>(), t.data_ptr<float>());
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
}

// in place: logits [N, Vc] bf16 -> dlogits = g / T * (onehot - softmax); lse, g fp32 [N]
void vocab_lse_grad(torch::Tensor logits, int64_t lo, torch::Tensor targets, double inv_t, torch::Tensor lse,
                    torch::Tensor g) {
  VO_CHECK_CUDA(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kBFloat16 && logits.dim() == 2 && logits.stride(1) == 1 &&
                  logits.stride(0) % 8 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0,
              "bf16 [N, Vc] logits with 16-byte aligned rows");
  VO_CHECK_INPUT(targets);
  VO_CHECK_INPUT(lse);
  VO_CHECK_INPUT(g);
  const int64_t N = logits.size(0);
  TORCH_CHECK(targets.numel() == N && lse.numel() == N && g.numel() == N && lse.scalar_type() == torch::kFloat32 &&
                  g.scalar_type() == torch::kFloat32 && targets.scalar_type() == torch::kInt64,
              "one fp32 lse / grad and int64 target per row");
  if (N == 0) return;
  c10::cuda::CUDAGuard gd(logits.device());
  lse_grad_kernel<<<(unsigned)N, kLseThreads, 0, stream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr<at::BFloat16>()), logits.stride(0), (int)logits.size(1), lo,
      targets.data_ptr<int64_t>(), (float)inv_t, lse.data_ptr<float>(), g.data_ptr<float>());
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
}

}  // namespace vo
