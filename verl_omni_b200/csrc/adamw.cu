// Sharded AdamW over flat fp32 buffers with on-device global-norm clipping.
//
//   sq_norm_partial : per-block sum of squares of the (fp32) gradient shard; the host side
//                     sums the partials of every shard and (multi-GPU) all-reduces the scalar.
//   adamw_flat      : reads the global norm from device memory, skips the update when it is
//                     non-finite (the reference skips optimizer.step() on a non-finite grad norm),
//                     otherwise clip_coef = min(1, max_norm / (norm + 1e-6)) and the torch.optim.AdamW
//                     update (decoupled weight decay, bias-corrected moments); writes the fp32
//                     master and the bf16 compute copy in the same pass.  No host synchronisation.
#include "common.cuh"

namespace vo {
namespace {

__global__ void sq_norm_partial_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ partial) {
  __shared__ float red[32];
  float s = 0.f;
  const int64_t n4 = n / 4;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = g4[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    s += g[i] * g[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

__global__ void sum_partials_kernel(const float* __restrict__ p, int n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += p[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[0] = s;
}

__global__ void adamw_flat_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                                  float* __restrict__ v, __nv_bfloat16* __restrict__ p16, int64_t n, float lr, float b1,
                                  float b2, float eps, float wd, float bc1, float bc2_sqrt, float max_norm,
                                  const float* __restrict__ sq_norm, float grad_scale) {
  float coef = grad_scale;
  if (sq_norm) {
    const float norm = sqrtf(sq_norm[0]);
    if (!isfinite(norm)) return;
    if (max_norm > 0.f) coef *= fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const float step = lr / bc1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float gi = g[i] * coef;
    float pi = p[i] * (1.f - lr * wd);
    float mi = b1 * m[i] + (1.f - b1) * gi;
    float vi = b2 * v[i] + (1.f - b2) * gi * gi;
    pi -= step * mi / (sqrtf(vi) / bc2_sqrt + eps);
    p[i] = pi;
    m[i] = mi;
    v[i] = vi;
    if (p16) p16[i] = __float2bfloat16_rn(pi);
  }
}

// Same update on 4-element vectors (16-byte loads / stores of p, g, m, v; 8-byte bf16 stores): identical
// arithmetic per element, four times fewer memory instructions.  n4 = n / 4 vectors; the host runs the
// scalar kernel on the tail and whenever a pointer is not 16-byte aligned.
__global__ void __launch_bounds__(256) adamw_flat_vec_kernel(float4* __restrict__ p, const float4* __restrict__ g,
                                                             float4* __restrict__ m, float4* __restrict__ v,
                                                             uint2* __restrict__ p16, int64_t n4, float lr, float b1,
                                                             float b2, float eps, float wd, float bc1, float bc2_sqrt,
                                                             float max_norm, const float* __restrict__ sq_norm,
                                                             float grad_scale) {
  float coef = grad_scale;
  if (sq_norm) {
    const float norm = sqrtf(sq_norm[0]);
    if (!isfinite(norm)) return;
    if (max_norm > 0.f) coef *= fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const float step = lr / bc1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 g4 = g[i], p4 = p[i], m4 = m[i], v4 = v[i];
    float gi[4] = {g4.x, g4.y, g4.z, g4.w}, pi[4] = {p4.x, p4.y, p4.z, p4.w};
    float mi[4] = {m4.x, m4.y, m4.z, m4.w}, vi[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float gk = gi[k] * coef;
      float pk = pi[k] * (1.f - lr * wd);
      const float mk = b1 * mi[k] + (1.f - b1) * gk;
      const float vk = b2 * vi[k] + (1.f - b2) * gk * gk;
      pk -= step * mk / (sqrtf(vk) / bc2_sqrt + eps);
      pi[k] = pk;
      mi[k] = mk;
      vi[k] = vk;
    }
    p[i] = make_float4(pi[0], pi[1], pi[2], pi[3]);
    m[i] = make_float4(mi[0], mi[1], mi[2], mi[3]);
    v[i] = make_float4(vi[0], vi[1], vi[2], vi[3]);
    if (p16) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(pi[0], pi[1]), hi = __floats2bfloat162_rn(pi[2], pi[3]);
      p16[i] = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
    }
  }
}

}  // namespace

// returns the [1] fp32 sum of squares of g (deterministic two-stage reduction)
torch::Tensor sq_norm(torch::Tensor g) {
  VO_CHECK_INPUT(g);
  TORCH_CHECK(g.scalar_type() == torch::kFloat32, "fp32 grads required");
  c10::cuda::CUDAGuard gd(g.device());
  const int nb = 2 * num_sms();
  auto part = torch::empty({nb}, g.options());
  auto out = torch::empty({1}, g.options());
  sq_norm_partial_kernel<<<nb, 512, 0, stream()>>>(g.data_ptr<float>(), g.numel(), part.data_ptr<float>()); vo::count_launch();
  sum_partials_kernel<<<1, 512, 0, stream()>>>(part.data_ptr<float>(), nb, out.data_ptr<float>()); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return out;
}

void adamw_flat(torch::Tensor p, torch::Tensor g, torch::Tensor m, torch::Tensor v, c10::optional<torch::Tensor> p16,
                double lr, double b1, double b2, double eps, double wd, int64_t step, double max_norm,
                c10::optional<torch::Tensor> sq_norm_t, double grad_scale) {
  VO_CHECK_INPUT(p);
  VO_CHECK_INPUT(g);
  VO_CHECK_INPUT(m);
  VO_CHECK_INPUT(v);
  TORCH_CHECK(p.numel() == g.numel() && p.numel() == m.numel() && p.numel() == v.numel(), "size mismatch");
  c10::cuda::CUDAGuard gd(p.device());
  const double bc1 = 1.0 - std::pow(b1, (double)step);
  const double bc2 = 1.0 - std::pow(b2, (double)step);
  __nv_bfloat16* p16p = nullptr;
  if (p16.has_value() && p16->defined()) {
    TORCH_CHECK(p16->numel() == p.numel() && p16->scalar_type() == torch::kBFloat16, "bad bf16 copy");
    p16p = reinterpret_cast<__nv_bfloat16*>(p16->data_ptr<at::BFloat16>());
  }
  const float* sn = (sq_norm_t.has_value() && sq_norm_t->defined()) ? sq_norm_t->data_ptr<float>() : nullptr;
  const int64_t n = p.numel();
  auto a16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  const bool vec = a16(p.data_ptr()) && a16(g.data_ptr()) && a16(m.data_ptr()) && a16(v.data_ptr()) &&
                   (p16p == nullptr || reinterpret_cast<uintptr_t>(p16p) % 8 == 0);
  const int64_t n4 = vec ? n / 4 : 0, head = n4 * 4;
  if (n4 > 0) {
    const int nb = (int)std::min<int64_t>((n4 + 255) / 256, 8LL * num_sms());
    adamw_flat_vec_kernel<<<nb, 256, 0, stream()>>>(
        reinterpret_cast<float4*>(p.data_ptr<float>()), reinterpret_cast<const float4*>(g.data_ptr<float>()),
        reinterpret_cast<float4*>(m.data_ptr<float>()), reinterpret_cast<float4*>(v.data_ptr<float>()),
        reinterpret_cast<uint2*>(p16p), n4, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, (float)bc1,
        (float)std::sqrt(bc2), (float)max_norm, sn, (float)grad_scale);
    vo::count_launch();
  }
  if (n > head) {  // tail (or everything, when not 16-byte aligned)
    const int64_t rest = n - head;
    const int nb = (int)std::min<int64_t>((rest + 255) / 256, 8LL * num_sms());
    adamw_flat_kernel<<<nb, 256, 0, stream()>>>(p.data_ptr<float>() + head, g.data_ptr<float>() + head,
                                                m.data_ptr<float>() + head, v.data_ptr<float>() + head,
                                                p16p ? p16p + head : nullptr, rest, (float)lr, (float)b1, (float)b2,
                                                (float)eps, (float)wd, (float)bc1, (float)std::sqrt(bc2),
                                                (float)max_norm, sn, (float)grad_scale);
    vo::count_launch();
  }
  VO_CUDA_OK(cudaGetLastError());
}

}  // namespace vo
