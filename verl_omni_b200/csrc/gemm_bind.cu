// Torch-facing wrappers of the tcgen05 GEMM (forward / dgrad / wgrad of a linear layer) and the
// GELU(tanh) backward used with the fused GELU epilogue.
#include "common.cuh"

namespace vo_gemm {
struct EpiParams {
  int epi;
  __nv_bfloat16* out;
  __nv_bfloat16* out2;
  float* out_f32;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* gate;
  const __nv_bfloat16* res;
  int64_t gate_ld;
  int S;
  int ldc;
};
}  // namespace vo_gemm

extern "C" int vo_gemm_launch(const void* A, const void* B, int M, int N, int K, int64_t lda, int64_t ldb, int a_mn,
                              int b_mn, int splits, vo_gemm::EpiParams ep, cudaStream_t stream);
extern "C" int vo_gemm_error(int reset);
extern "C" int vo_gemm_launch_ext(const void* A, const void* B, const void* A2, const void* B2, int M, int N, int K,
                                  int K2, int64_t lda, int64_t ldb, int64_t lda2, int64_t ldb2, int a_mn, int b_mn,
                                  int splits, vo_gemm::EpiParams ep, cudaStream_t stream);

namespace vo {
namespace {

inline __nv_bfloat16* bf(const torch::Tensor& t) {
  return t.defined() ? reinterpret_cast<__nv_bfloat16*>(t.data_ptr<at::BFloat16>()) : nullptr;
}

void check_rc(int rc, const char* what) { TORCH_CHECK(rc == 0, "tcgen05 GEMM launch failed (", what, "): code ", rc); }

__global__ void gelu_tanh_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ pre,
                                     __nv_bfloat16* __restrict__ dx, int64_t n8) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float g[8], x[8], o[8];
    unpack8(reinterpret_cast<const bf16x8*>(dy)[i], g);
    unpack8(reinterpret_cast<const bf16x8*>(pre)[i], x);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float u = k0 * (x[j] + k1 * x[j] * x[j] * x[j]);
      float t = tanhf(u);
      float d = 0.5f * (1.f + t) + 0.5f * x[j] * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x[j] * x[j]);
      o[j] = g[j] * d;
    }
    reinterpret_cast<bf16x8*>(dx)[i] = pack8(o);
  }
}

}  // namespace

// y = x W^T (+ b) with epilogue; returns (out, saved) where saved is the GELU pre-activation or
// the GATE_RES linear output (undefined tensor otherwise).
// ext_a / ext_b (optional): extra reduction operands, out = x W^T + ext_a ext_b^T (+ epilogue) -- the
// fused low-rank path: ext_a = x A_lora^T [M, r], ext_b = scale * B_lora [N, r].
std::vector<torch::Tensor> gemm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, int64_t epi,
                                    c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> res, int64_t S,
                                    c10::optional<torch::Tensor> ext_a, c10::optional<torch::Tensor> ext_b) {
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(w);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16, "bf16 GEMM operands");
  c10::cuda::CUDAGuard g(x.device());
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "shape mismatch");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "GEMM dims must be multiples of 8 (16-byte rows)");
  auto out = torch::empty({M, N}, x.options());
  torch::Tensor saved;
  vo_gemm::EpiParams ep{};
  ep.epi = (int)epi;
  ep.out = bf(out);
  ep.ldc = (int)N;
  ep.S = (int)S;
  if (b.has_value() && b->defined()) ep.bias = bf(*b);
  if (epi == 2 || epi == 3) {
    saved = torch::empty({M, N}, x.options());
    ep.out2 = bf(saved);
  }
  torch::Tensor gate_c;
  if (epi == 3) {
    TORCH_CHECK(gate.has_value() && res.has_value(), "GATE_RES needs gate and res");
    // a strided per-sample row view (an AdaLN chunk of the modulation output) is read in place
    gate_c = (gate->dim() == 2 && gate->stride(1) == 1) ? *gate : gate->contiguous();
    ep.gate = bf(gate_c);
    ep.gate_ld = gate_c.stride(0);
    TORCH_CHECK(res->is_contiguous() && res->numel() == M * N, "res must be contiguous [M, N]");
    ep.res = bf(*res);
  }
  const void *a2 = nullptr, *b2 = nullptr;
  int64_t K2 = 0;
  if (ext_a.has_value() && ext_a->defined()) {
    TORCH_CHECK(ext_b.has_value() && ext_b->defined(), "ext_a needs ext_b");
    VO_CHECK_INPUT((*ext_a));
    VO_CHECK_INPUT((*ext_b));
    K2 = ext_a->size(1);
    TORCH_CHECK(ext_a->size(0) == M && ext_b->size(0) == N && ext_b->size(1) == K2 && K2 % 8 == 0,
                "extension operands must be [M, r] and [N, r] with r % 8 == 0");
    a2 = ext_a->data_ptr();
    b2 = ext_b->data_ptr();
  }
  check_rc(vo_gemm_launch_ext(x.data_ptr(), w.data_ptr(), a2, b2, (int)M, (int)N, (int)K, (int)K2, K, K, K2, K2, 0, 0,
                              1, ep, stream()),
           "fwd");
  count_launch();
  return {out, saved};
}

// dX[M, K] = dY[M, N] W[N, K] (+ ext_a[M, r] ext_b[r, K])   (B operands MN-major)
torch::Tensor gemm_dgrad(torch::Tensor dy, torch::Tensor w, c10::optional<torch::Tensor> ext_a,
                         c10::optional<torch::Tensor> ext_b) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(w);
  c10::cuda::CUDAGuard g(dy.device());
  const int64_t M = dy.size(0), N = dy.size(1), K = w.size(1);
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "GEMM dims must be multiples of 8 (16-byte rows)");
  auto dx = torch::empty({M, K}, dy.options());
  vo_gemm::EpiParams ep{};
  ep.epi = 0;
  ep.out = bf(dx);
  ep.ldc = (int)K;
  // GEMM: C[M, K] = sum_n dY(m, n) * W(n, k): GEMM-N = K, GEMM-K = N, B(col=k, red=n) = W[n, k] -> MN-major
  const void *a2 = nullptr, *b2 = nullptr;
  int64_t R = 0;
  if (ext_a.has_value() && ext_a->defined()) {
    TORCH_CHECK(ext_b.has_value() && ext_b->defined(), "ext_a needs ext_b");
    VO_CHECK_INPUT((*ext_a));
    VO_CHECK_INPUT((*ext_b));
    R = ext_a->size(1);
    TORCH_CHECK(ext_a->size(0) == M && ext_b->size(0) == R && ext_b->size(1) == K && R % 8 == 0,
                "extension operands must be [M, r] and [r, K] with r % 8 == 0");
    a2 = ext_a->data_ptr();
    b2 = ext_b->data_ptr();
  }
  check_rc(vo_gemm_launch_ext(dy.data_ptr(), w.data_ptr(), a2, b2, (int)M, (int)K, (int)N, (int)R, N, K, R, K, 0, 1, 1,
                              ep, stream()),
           "dgrad");
  count_launch();
  return dx;
}

// out[N, K] (+)= dY[M, N]^T X[M, K]   (both operands MN-major), fp32 output, split-K over M
void gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor out, bool accumulate) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(out);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32, "wgrad output must be fp32");
  c10::cuda::CUDAGuard g(dy.device());
  const int64_t M = dy.size(0), N = dy.size(1), K = x.size(1);
  TORCH_CHECK(out.numel() == N * K, "wgrad output shape");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "GEMM dims must be multiples of 8 (16-byte rows)");
  if (!accumulate) out.zero_();
  vo_gemm::EpiParams ep{};
  ep.epi = 4;
  ep.out_f32 = out.data_ptr<float>();
  ep.ldc = (int)K;
  const int tiles = (int)(((N + 127) / 128) * ((K + 255) / 256));
  const int kblocks = (int)((M + 63) / 64);
  int splits = std::max(1, std::min((2 * num_sms() + tiles - 1) / tiles, kblocks / 4));
  // GEMM-M = N (rows of dW), GEMM-N = K, GEMM-K = M tokens; A(m=n, k=t) = dY[t, n] (MN-major), B = X[t, k] (MN-major)
  check_rc(vo_gemm_launch(dy.data_ptr(), x.data_ptr(), (int)N, (int)K, (int)M, N, K, 1, 1, splits, ep, stream()),
           "wgrad");
  count_launch();
}

torch::Tensor gelu_tanh_bwd(torch::Tensor dy, torch::Tensor pre) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(pre);
  TORCH_CHECK(dy.numel() % 8 == 0, "numel must be a multiple of 8");
  c10::cuda::CUDAGuard g(dy.device());
  auto dx = torch::empty_like(dy);
  const int64_t n8 = dy.numel() / 8;
  const int nb = (int)std::min<int64_t>((n8 + 255) / 256, 8LL * num_sms());
  gelu_tanh_bwd_kernel<<<nb, 256, 0, stream()>>>(bf(dy), bf(pre), bf(dx), n8);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return dx;
}

int64_t gemm_error(bool reset) { return vo_gemm_error(reset ? 1 : 0); }

}  // namespace vo
