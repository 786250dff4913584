// Torch-facing wrappers of the tcgen05 GEMM (forward / dgrad / wgrad of a linear layer) and the
// GELU(tanh) backward used with the fused GELU epilogue.
#include "common.cuh"

#include "gemm_api.h"

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
struct FwdArgs {
  vo_gemm::GemmDesc d;
  torch::Tensor out, saved, gate_c;
};

FwdArgs prep_fwd(const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& b, int64_t epi,
                 const c10::optional<torch::Tensor>& gate, const c10::optional<torch::Tensor>& res, int64_t S,
                 const c10::optional<torch::Tensor>& ext_a, const c10::optional<torch::Tensor>& ext_b,
                 bool alloc_out = true) {
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(w);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16, "bf16 GEMM operands");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "shape mismatch");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "GEMM dims must be multiples of 8 (16-byte rows)");
  FwdArgs a;
  if (alloc_out) a.out = torch::empty({M, N}, x.options());
  vo_gemm::EpiParams& ep = a.d.ep;
  ep = vo_gemm::EpiParams{};
  ep.epi = (int)epi;
  ep.out = alloc_out ? bf(a.out) : nullptr;
  ep.ldc = (int)N;
  ep.S = (int)S;
  if (b.has_value() && b->defined()) ep.bias = bf(*b);
  if (epi == 2 || epi == 3) {
    a.saved = torch::empty({M, N}, x.options());
    ep.out2 = bf(a.saved);
  }
  if (epi == 3) {
    TORCH_CHECK(gate.has_value() && res.has_value(), "GATE_RES needs gate and res");
    // a strided per-sample row view (an AdaLN chunk of the modulation output) is read in place
    a.gate_c = (gate->dim() == 2 && gate->stride(1) == 1) ? *gate : gate->contiguous();
    ep.gate = bf(a.gate_c);
    ep.gate_ld = a.gate_c.stride(0);
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
  a.d.A = x.data_ptr();
  a.d.B = w.data_ptr();
  a.d.A2 = a2;
  a.d.B2 = b2;
  a.d.M = (int)M;
  a.d.N = (int)N;
  a.d.K = (int)K;
  a.d.K2 = (int)K2;
  a.d.lda = K;
  a.d.ldb = K;
  a.d.lda2 = K2;
  a.d.ldb2 = K2;
  a.d.a_mn = 0;
  a.d.b_mn = 0;
  a.d.splits = 1;
  return a;
}

std::vector<torch::Tensor> gemm_fwd(torch::Tensor x, torch::Tensor w, c10::optional<torch::Tensor> b, int64_t epi,
                                    c10::optional<torch::Tensor> gate, c10::optional<torch::Tensor> res, int64_t S,
                                    c10::optional<torch::Tensor> ext_a, c10::optional<torch::Tensor> ext_b) {
  c10::cuda::CUDAGuard g(x.device());
  FwdArgs a = prep_fwd(x, w, b, epi, gate, res, S, ext_a, ext_b);
  check_rc(vo_gemm_launch_group(&a.d, 1, stream()), "fwd");
  count_launch();
  return {a.out, a.saved};
}

// Two independent linear forwards (the image and text streams of a joint block) in one persistent
// launch; same epilogue kind for both.  Returns (out0, saved0, out1, saved1).
std::vector<torch::Tensor> gemm_fwd_pair(torch::Tensor x0, torch::Tensor w0, c10::optional<torch::Tensor> b0,
                                         c10::optional<torch::Tensor> gate0, c10::optional<torch::Tensor> res0,
                                         int64_t S0, torch::Tensor x1, torch::Tensor w1,
                                         c10::optional<torch::Tensor> b1, c10::optional<torch::Tensor> gate1,
                                         c10::optional<torch::Tensor> res1, int64_t S1, int64_t epi) {
  c10::cuda::CUDAGuard g(x0.device());
  const c10::optional<torch::Tensor> none;
  FwdArgs a0 = prep_fwd(x0, w0, b0, epi, gate0, res0, S0, none, none);
  FwdArgs a1 = prep_fwd(x1, w1, b1, epi, gate1, res1, S1, none, none);
  vo_gemm::GemmDesc d[2] = {a0.d, a1.d};
  check_rc(vo_gemm_launch_group(d, 2, stream()), "fwd pair");
  count_launch();
  return {a0.out, a0.saved, a1.out, a1.saved};
}

// Ulysses QKV projection with the head scatter fused into the epilogue: y = x W^T (+ b) for one or two
// token segments (image rows x0, text rows x1 of this rank), each output row and 32-column chunk stored
// straight into the buffer of the rank that owns its heads (`peers`: data pointers of the group's
// destination buffers, dst_rows rows of dst_ld elements).  Row t of sample b of segment i lands at
// destination row b * dst_seq_i + row_off_i + t.
void gemm_scatter(torch::Tensor x0, torch::Tensor w0, c10::optional<torch::Tensor> b0, int64_t seg_rows0,
                  int64_t dst_seq0, int64_t row_off0, c10::optional<torch::Tensor> x1, c10::optional<torch::Tensor> w1,
                  c10::optional<torch::Tensor> b1, int64_t seg_rows1, int64_t dst_seq1, int64_t row_off1,
                  std::vector<int64_t> peers, int64_t part_cols, int64_t dst_cols, int64_t dst_ld, int64_t dst_rows) {
  c10::cuda::CUDAGuard g(x0.device());
  TORCH_CHECK(!peers.empty() && (int64_t)peers.size() <= vo_gemm::kMaxPeers, "1..8 destination buffers");
  TORCH_CHECK(part_cols == dst_cols * (int64_t)peers.size(), "part_cols must be dst_cols x number of peers");
  const c10::optional<torch::Tensor> none;
  vo_gemm::GemmDesc d[2];
  int n = 0;
  auto add = [&](const torch::Tensor& x, const torch::Tensor& w, const c10::optional<torch::Tensor>& b,
                 int64_t seg_rows, int64_t dst_seq, int64_t row_off) {
    TORCH_CHECK(seg_rows > 0 && x.size(0) % seg_rows == 0, "rows must be whole samples of seg_rows tokens");
    const int64_t nb = x.size(0) / seg_rows;
    TORCH_CHECK(row_off >= 0 && seg_rows <= dst_seq && (nb - 1) * dst_seq + row_off + seg_rows <= dst_rows,
                "scatter rows fall outside the destination buffers");
    FwdArgs a = prep_fwd(x, w, b, 1, none, none, 1, none, none, false);
    a.d.ep.epi = vo_gemm::EPI_SCATTER;
    vo_gemm::ScatterParams& sc = a.d.ep.sc;
    for (size_t i = 0; i < peers.size(); ++i) sc.peers[i] = reinterpret_cast<__nv_bfloat16*>(peers[i]);
    sc.part_cols = (int)part_cols;
    sc.dst_cols = (int)dst_cols;
    sc.seg_rows = (int)seg_rows;
    sc.dst_seq = (int)dst_seq;
    sc.row_off = (int)row_off;
    sc.dst_ld = (int)dst_ld;
    d[n++] = a.d;
  };
  add(x0, w0, b0, seg_rows0, dst_seq0, row_off0);
  if (x1.has_value() && x1->defined()) add(*x1, *w1, b1, seg_rows1, dst_seq1, row_off1);
  check_rc(vo_gemm_launch_group(d, n, stream()), "scatter");
  count_launch();
}

// dX[M, K] = dY[M, N] W[N, K] (+ ext_a[M, r] ext_b[r, K])   (B operands MN-major)
vo_gemm::GemmDesc prep_dgrad(const torch::Tensor& dy, const torch::Tensor& w, const torch::Tensor& dx,
                             const c10::optional<torch::Tensor>& ext_a, const c10::optional<torch::Tensor>& ext_b) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(w);
  const int64_t M = dy.size(0), N = dy.size(1), K = w.size(1);
  TORCH_CHECK(w.size(0) == N, "shape mismatch");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "GEMM dims must be multiples of 8 (16-byte rows)");
  vo_gemm::GemmDesc d{};
  d.ep.epi = 0;
  d.ep.out = bf(dx);
  d.ep.ldc = (int)K;
  // GEMM: C[M, K] = sum_n dY(m, n) * W(n, k): GEMM-N = K, GEMM-K = N, B(col=k, red=n) = W[n, k] -> MN-major
  int64_t R = 0;
  if (ext_a.has_value() && ext_a->defined()) {
    TORCH_CHECK(ext_b.has_value() && ext_b->defined(), "ext_a needs ext_b");
    VO_CHECK_INPUT((*ext_a));
    VO_CHECK_INPUT((*ext_b));
    R = ext_a->size(1);
    TORCH_CHECK(ext_a->size(0) == M && ext_b->size(0) == R && ext_b->size(1) == K && R % 8 == 0,
                "extension operands must be [M, r] and [r, K] with r % 8 == 0");
    d.A2 = ext_a->data_ptr();
    d.B2 = ext_b->data_ptr();
  }
  d.A = dy.data_ptr();
  d.B = w.data_ptr();
  d.M = (int)M;
  d.N = (int)K;
  d.K = (int)N;
  d.K2 = (int)R;
  d.lda = N;
  d.ldb = K;
  d.lda2 = R;
  d.ldb2 = K;
  d.a_mn = 0;
  d.b_mn = 1;
  d.splits = 1;
  return d;
}

torch::Tensor gemm_dgrad(torch::Tensor dy, torch::Tensor w, c10::optional<torch::Tensor> ext_a,
                         c10::optional<torch::Tensor> ext_b) {
  c10::cuda::CUDAGuard g(dy.device());
  auto dx = torch::empty({dy.size(0), w.size(1)}, dy.options());
  vo_gemm::GemmDesc d = prep_dgrad(dy, w, dx, ext_a, ext_b);
  check_rc(vo_gemm_launch_group(&d, 1, stream()), "dgrad");
  count_launch();
  return dx;
}

std::vector<torch::Tensor> gemm_dgrad_pair(torch::Tensor dy0, torch::Tensor w0, torch::Tensor dy1, torch::Tensor w1) {
  c10::cuda::CUDAGuard g(dy0.device());
  const c10::optional<torch::Tensor> none;
  auto dx0 = torch::empty({dy0.size(0), w0.size(1)}, dy0.options());
  auto dx1 = torch::empty({dy1.size(0), w1.size(1)}, dy1.options());
  vo_gemm::GemmDesc d[2] = {prep_dgrad(dy0, w0, dx0, none, none), prep_dgrad(dy1, w1, dx1, none, none)};
  check_rc(vo_gemm_launch_group(d, 2, stream()), "dgrad pair");
  count_launch();
  return {dx0, dx1};
}

// out[N, K] (+)= dY[M, N]^T X[M, K]   (both operands MN-major), fp32 output, split-K over M
// `tiles_total`: output tiles of every problem in the launch (sizes the split so the launch fills the GPU).
vo_gemm::GemmDesc prep_wgrad(const torch::Tensor& dy, const torch::Tensor& x, torch::Tensor& out, bool accumulate,
                             int tiles_total) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(out);
  TORCH_CHECK(out.scalar_type() == torch::kFloat32, "wgrad output must be fp32");
  const int64_t M = dy.size(0), N = dy.size(1), K = x.size(1);
  TORCH_CHECK(x.size(0) == M, "shape mismatch");
  TORCH_CHECK(out.numel() == N * K, "wgrad output shape");
  TORCH_CHECK(N % 8 == 0 && K % 8 == 0, "GEMM dims must be multiples of 8 (16-byte rows)");
  if (!accumulate) out.zero_();
  vo_gemm::GemmDesc d{};
  d.ep.epi = 4;
  d.ep.out_f32 = out.data_ptr<float>();
  d.ep.ldc = (int)K;
  const int kblocks = (int)((M + 63) / 64);
  d.splits = std::max(1, std::min((2 * num_sms() + tiles_total - 1) / tiles_total, kblocks / 4));
  // GEMM-M = N (rows of dW), GEMM-N = K, GEMM-K = M tokens; A(m=n, k=t) = dY[t, n] (MN-major), B = X[t, k] (MN-major)
  d.A = dy.data_ptr();
  d.B = x.data_ptr();
  d.M = (int)N;
  d.N = (int)K;
  d.K = (int)M;
  d.lda = N;
  d.ldb = K;
  d.a_mn = 1;
  d.b_mn = 1;
  return d;
}

inline int wgrad_tiles(const torch::Tensor& dy, const torch::Tensor& x) {
  return (int)(((dy.size(1) + 127) / 128) * ((x.size(1) + 255) / 256));
}

void gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor out, bool accumulate) {
  c10::cuda::CUDAGuard g(dy.device());
  vo_gemm::GemmDesc d = prep_wgrad(dy, x, out, accumulate, wgrad_tiles(dy, x));
  check_rc(vo_gemm_launch_group(&d, 1, stream()), "wgrad");
  count_launch();
}

void gemm_wgrad_pair(torch::Tensor dy0, torch::Tensor x0, torch::Tensor out0, torch::Tensor dy1, torch::Tensor x1,
                     torch::Tensor out1, bool accumulate) {
  c10::cuda::CUDAGuard g(dy0.device());
  const int tiles = wgrad_tiles(dy0, x0) + wgrad_tiles(dy1, x1);
  vo_gemm::GemmDesc d[2] = {prep_wgrad(dy0, x0, out0, accumulate, tiles), prep_wgrad(dy1, x1, out1, accumulate, tiles)};
  check_rc(vo_gemm_launch_group(d, 2, stream()), "wgrad pair");
  count_launch();
}

// ---------------------------------------------------------------- tensor-parallel GEMMs over peer memory
// C[M, N] = A B^T with the operand conventions of vo_gemm_launch_ext (a_mn / b_mn), where one operand may
// be gathered from the ranks of a tensor-parallel group (gather 1: rows of a K-major A; 2: reduction rows
// of an MN-major A; 3: reduction rows of an MN-major B -- gather_rows rows per rank, read with plain TMA
// loads from the peers' buffers) and the output may be added into the owning ranks' fp32 buffers
// (red_ptrs, red_rows output rows per rank) instead of stored locally; with red_slot >= 0 the rows are
// stored in bf16 at slot red_slot ([red_rows, N] each) of the owners' buffers, for the owner to sum.
// out: bf16 [M, N] (ignored with red_ptrs); out_f32: fp32 [M, N] accumulated (weight gradients).
void gemm_tp(c10::optional<torch::Tensor> a, c10::optional<torch::Tensor> b, int64_t M, int64_t N, int64_t K,
             int64_t lda, int64_t ldb, int64_t a_mn, int64_t b_mn, c10::optional<torch::Tensor> out,
             c10::optional<torch::Tensor> out_f32, c10::optional<torch::Tensor> bias, int64_t gather,
             std::vector<int64_t> gather_ptrs, int64_t gather_rows, std::vector<int64_t> red_ptrs,
             int64_t red_rows, int64_t red_slot) {
  const torch::Tensor& dev_t = a.has_value() && a->defined() ? *a : *b;
  c10::cuda::CUDAGuard g(dev_t.device());
  vo_gemm::GemmDesc d{};
  d.A = a.has_value() && a->defined() ? a->data_ptr() : nullptr;
  d.B = b.has_value() && b->defined() ? b->data_ptr() : nullptr;
  d.M = (int)M;
  d.N = (int)N;
  d.K = (int)K;
  d.lda = lda;
  d.ldb = ldb;
  d.a_mn = (int)a_mn;
  d.b_mn = (int)b_mn;
  d.splits = 1;
  TORCH_CHECK(gather_ptrs.size() <= (size_t)vo_gemm::kMaxPeers && red_ptrs.size() <= (size_t)vo_gemm::kMaxPeers,
              "at most 8 ranks");
  d.gather = (int)gather;
  d.gather_rows = (int)gather_rows;
  d.gather_n = (int)gather_ptrs.size();
  for (size_t i = 0; i < gather_ptrs.size(); ++i) d.gather_ptrs[i] = reinterpret_cast<const void*>(gather_ptrs[i]);
  TORCH_CHECK((gather == 0) == gather_ptrs.empty(), "gather mode needs peer pointers");
  TORCH_CHECK(gather == 1 || gather == 2 || d.A, "A operand missing");
  TORCH_CHECK(gather == 3 || d.B, "B operand missing");
  if (!red_ptrs.empty()) {
    d.ep.epi = vo_gemm::EPI_PEER_RED;
    d.ep.red_rows = (int)red_rows;
    d.ep.red_store = red_slot >= 0;  // bf16 slot stores (slot red_slot) instead of fp32 atomics
    d.ep.red_slot_off = red_slot >= 0 ? (int)(red_slot * red_rows) : 0;
    d.ep.ldc = (int)N;
    for (size_t i = 0; i < red_ptrs.size(); ++i) d.ep.red_peers[i] = reinterpret_cast<float*>(red_ptrs[i]);
    TORCH_CHECK((int64_t)red_ptrs.size() * red_rows >= M, "owners must cover every output row");
  } else if (out_f32.has_value() && out_f32->defined()) {
    TORCH_CHECK(out_f32->scalar_type() == torch::kFloat32 && out_f32->numel() == M * N, "fp32 [M, N] output");
    d.ep.epi = vo_gemm::EPI_F32_ACC;
    d.ep.out_f32 = out_f32->data_ptr<float>();
    d.ep.ldc = (int)N;
  } else {
    TORCH_CHECK(out.has_value() && out->defined() && out->numel() == M * N, "bf16 [M, N] output");
    d.ep.epi = bias.has_value() && bias->defined() ? vo_gemm::EPI_BIAS : vo_gemm::EPI_NONE;
    d.ep.out = bf(*out);
    d.ep.ldc = (int)N;
    if (bias.has_value() && bias->defined()) d.ep.bias = bf(*bias);
  }
  check_rc(vo_gemm_launch_group(&d, 1, stream()), "tp");
  count_launch();
}

// ---------------------------------------------------------------- mixture-of-experts grouped GEMMs
// Rows are (token, expert) pairs sorted by expert, each expert's segment padded with zero rows to a
// multiple of 128 (so every 128-row tile belongs to one expert); `tile_expert[t]` = expert of tile t, -1
// for unused tiles.  Weights are stacked [E, N, K] (one tensor map over E*N rows).

// y[Mp, N] = x[Mp, K] W_e^T for the expert e of each row tile
torch::Tensor moe_gemm_fwd(torch::Tensor x, torch::Tensor w, torch::Tensor tile_expert) {
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(w);
  VO_CHECK_INPUT(tile_expert);
  TORCH_CHECK(w.dim() == 3 && x.size(1) == w.size(2) && tile_expert.scalar_type() == torch::kInt32, "moe shapes");
  const int64_t Mp = x.size(0), K = x.size(1), E = w.size(0), N = w.size(1);
  TORCH_CHECK(Mp % 128 == 0 && tile_expert.numel() == Mp / 128 && N % 8 == 0 && K % 8 == 0, "moe tiling");
  c10::cuda::CUDAGuard g(x.device());
  auto y = torch::empty({Mp, N}, x.options());
  vo_gemm::GemmDesc d{};
  d.A = x.data_ptr();
  d.B = w.data_ptr();
  d.M = (int)Mp;
  d.N = (int)N;
  d.K = (int)K;
  d.lda = K;
  d.ldb = K;
  d.splits = 1;
  d.ep.epi = vo_gemm::EPI_NONE;
  d.ep.out = bf(y);
  d.ep.ldc = (int)N;
  d.grp_mode = 1;
  d.grp_tab = tile_expert.data_ptr<int>();
  d.n_groups = (int)E;
  check_rc(vo_gemm_launch_group(&d, 1, stream()), "moe fwd");
  count_launch();
  return y;
}

// dx[Mp, K] = dy[Mp, N] W_e
torch::Tensor moe_gemm_dgrad(torch::Tensor dy, torch::Tensor w, torch::Tensor tile_expert) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(w);
  VO_CHECK_INPUT(tile_expert);
  const int64_t Mp = dy.size(0), N = dy.size(1), E = w.size(0), K = w.size(2);
  TORCH_CHECK(w.dim() == 3 && w.size(1) == N && Mp % 128 == 0 && tile_expert.numel() == Mp / 128 &&
                  tile_expert.scalar_type() == torch::kInt32,
              "moe shapes");
  c10::cuda::CUDAGuard g(dy.device());
  auto dx = torch::empty({Mp, K}, dy.options());
  vo_gemm::GemmDesc d{};
  d.A = dy.data_ptr();
  d.B = w.data_ptr();
  d.M = (int)Mp;
  d.N = (int)K;
  d.K = (int)N;
  d.lda = N;
  d.ldb = K;
  d.b_mn = 1;
  d.splits = 1;
  d.ep.epi = vo_gemm::EPI_NONE;
  d.ep.out = bf(dx);
  d.ep.ldc = (int)K;
  d.grp_mode = 1;
  d.grp_tab = tile_expert.data_ptr<int>();
  d.n_groups = (int)E;
  check_rc(vo_gemm_launch_group(&d, 1, stream()), "moe dgrad");
  count_launch();
  return dx;
}

// out[E, N, K] (+)= dy_e^T x_e over each expert's rows [seg[e], seg[e+1]) (fp32)
void moe_gemm_wgrad(torch::Tensor dy, torch::Tensor x, torch::Tensor seg, torch::Tensor out, bool accumulate) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(seg);
  VO_CHECK_INPUT(out);
  const int64_t Mp = dy.size(0), N = dy.size(1), K = x.size(1), E = out.size(0);
  TORCH_CHECK(out.dim() == 3 && out.size(1) == N && out.size(2) == K && out.scalar_type() == torch::kFloat32 &&
                  x.size(0) == Mp && seg.numel() == E + 1 && seg.scalar_type() == torch::kInt32 && N % 128 == 0,
              "moe wgrad shapes");
  c10::cuda::CUDAGuard g(dy.device());
  if (!accumulate) out.zero_();
  vo_gemm::GemmDesc d{};
  d.A = dy.data_ptr();
  d.B = x.data_ptr();
  d.M = (int)(E * N);
  d.N = (int)K;
  d.K = (int)Mp;
  d.lda = N;
  d.ldb = K;
  d.a_mn = 1;
  d.b_mn = 1;
  d.splits = 1;
  d.ep.epi = vo_gemm::EPI_F32_ACC;
  d.ep.out_f32 = out.data_ptr<float>();
  d.ep.ldc = (int)K;
  d.grp_mode = 2;
  d.grp_tab = seg.data_ptr<int>();
  d.n_groups = (int)E;
  d.grp_rows = (int)N;
  check_rc(vo_gemm_launch_group(&d, 1, stream()), "moe wgrad");
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
