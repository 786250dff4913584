// Fused elementwise prologue of a linear layer's backward, one pass over dY [M, N] (bf16):
//
//   mode 0 (plain)    : dY2 = dY                                   (not rewritten)
//   mode 1 (gelu)     : dY2 = dY * gelu_tanh'(pre)                 (pre = saved pre-activation)
//   mode 2 (gate_res) : dY2 = dY * gate[b, :];  dgate[b, n] = sum_{rows of sample b} dY * lin
//                                                                  (lin = saved linear output)
//   every mode        : db[n] = sum_rows dY2[:, n]                 (optional, fp32, may accumulate)
//
// Replaces the chain of fp32 casts, products and reductions that the same backward needs in eager
// torch.  Rows are cut into chunks of R rows that never straddle a sample (mode 2 needs per-sample
// sums); each thread owns 8 adjacent columns (16-byte loads) and keeps its sums in registers.  Per-
// chunk partial sums go to a small fp32 buffer and a second kernel reduces them in a fixed order,
// so results are deterministic run to run.
#include "common.cuh"

namespace vo {
namespace {

constexpr int kRows = 64;     // rows per chunk
constexpr int kThreads = 64;  // 64 threads x 8 columns = 512 columns per block

// d/dx of 0.5 x (1 + tanh(k0 (x + k1 x^3))); tanh via the hardware approximation, as in the
// forward GEMM epilogue that produced the activation
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(k0 * (x + k1 * x * x * x)));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

template <int MODE, bool DB>
__global__ void __launch_bounds__(kThreads) bwd_prep_kernel(const __nv_bfloat16* __restrict__ dy,
                                                            const __nv_bfloat16* __restrict__ saved,
                                                            const __nv_bfloat16* __restrict__ gate, int64_t gate_ld,
                                                            __nv_bfloat16* __restrict__ dy2, float* __restrict__ part_db,
                                                            float* __restrict__ part_dg, int N, int S, int cps) {
  const int col = (blockIdx.x * kThreads + threadIdx.x) * 8;
  if (col >= N) return;
  const int chunk = blockIdx.y;
  const int b = chunk / cps, j = chunk % cps;
  const int64_t r0 = (int64_t)b * S + (int64_t)j * kRows;
  const int64_t r1 = min((int64_t)b * S + (int64_t)(j + 1) * kRows, (int64_t)(b + 1) * S);
  float g8[8];
  if (MODE == 2) unpack8(*reinterpret_cast<const bf16x8*>(gate + (int64_t)b * gate_ld + col), g8);
  float db[8], dg[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) db[i] = dg[i] = 0.f;
  // unrolled so that several rows' loads are in flight per thread (the sums still run in row order)
#pragma unroll 4
  for (int64_t r = r0; r < r1; ++r) {
    const int64_t off = r * N + col;
    float d[8];
    unpack8(*reinterpret_cast<const bf16x8*>(dy + off), d);
    if (MODE == 1) {
      float x[8];
      unpack8(*reinterpret_cast<const bf16x8*>(saved + off), x);
#pragma unroll
      for (int i = 0; i < 8; ++i) d[i] *= gelu_tanh_grad(x[i]);
    } else if (MODE == 2) {
      float x[8];
      unpack8(*reinterpret_cast<const bf16x8*>(saved + off), x);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dg[i] += d[i] * x[i];
        d[i] *= g8[i];
      }
    }
    if (MODE != 0) {
      const bf16x8 o = pack8(d);
      *reinterpret_cast<bf16x8*>(dy2 + off) = o;
      if (DB) unpack8(o, d);  // the bias grad sums what the GEMMs consume (bf16-rounded)
    }
    if (DB) {
#pragma unroll
      for (int i = 0; i < 8; ++i) db[i] += d[i];
    }
  }
  const int64_t p = (int64_t)chunk * N + col;
  if (DB) {
    reinterpret_cast<float4*>(part_db + p)[0] = make_float4(db[0], db[1], db[2], db[3]);
    reinterpret_cast<float4*>(part_db + p)[1] = make_float4(db[4], db[5], db[6], db[7]);
  }
  if (MODE == 2) {
    reinterpret_cast<float4*>(part_dg + p)[0] = make_float4(dg[0], dg[1], dg[2], dg[3]);
    reinterpret_cast<float4*>(part_dg + p)[1] = make_float4(dg[4], dg[5], dg[6], dg[7]);
  }
}

// db[n] (+)= sum over all chunks; dgate[b, n] = sum over sample b's chunks (bf16 out).
// Block = 32 columns x 8 chunk lanes: lane rl sums chunks rl, rl + 8, ... of each sample, then the
// eight partial sums are added in a fixed order through shared memory (deterministic).
constexpr int kRedCols = 32, kRedLanes = 8;
__global__ void __launch_bounds__(kRedCols* kRedLanes)
    bwd_prep_reduce_kernel(const float* __restrict__ part_db, const float* __restrict__ part_dg, int N, int B,
                           int cps, float* __restrict__ db, int db_accumulate, __nv_bfloat16* __restrict__ dgate) {
  __shared__ float red[2][kRedLanes][kRedCols];
  const int cx = threadIdx.x % kRedCols, rl = threadIdx.x / kRedCols;
  const int n = blockIdx.x * kRedCols + cx;
  float tot = 0.f;
  for (int b = 0; b < B; ++b) {
    float s = 0.f, sg = 0.f;
    if (n < N) {
      for (int j = rl; j < cps; j += kRedLanes) {
        const int64_t p = (int64_t)(b * cps + j) * N + n;
        if (part_db) s += part_db[p];
        if (part_dg) sg += part_dg[p];
      }
    }
    red[0][rl][cx] = s;
    red[1][rl][cx] = sg;
    __syncthreads();
    if (rl == 0 && n < N) {
      float a = 0.f, c = 0.f;
#pragma unroll
      for (int i = 0; i < kRedLanes; ++i) {
        a += red[0][i][cx];
        c += red[1][i][cx];
      }
      tot += a;
      if (dgate) dgate[(int64_t)b * N + n] = __float2bfloat16_rn(c);
    }
    __syncthreads();
  }
  if (rl == 0 && n < N && db) db[n] = db_accumulate ? db[n] + tot : tot;
}

template <int MODE, bool DB>
void launch_prep(dim3 grid, const __nv_bfloat16* dy, const __nv_bfloat16* saved, const __nv_bfloat16* gate,
                 int64_t gate_ld, __nv_bfloat16* dy2, float* pdb, float* pdg, int N, int S, int cps) {
  bwd_prep_kernel<MODE, DB><<<grid, kThreads, 0, stream()>>>(dy, saved, gate, gate_ld, dy2, pdb, pdg, N, S, cps);
}

inline const __nv_bfloat16* cbf(const torch::Tensor& t) {
  return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr<at::BFloat16>());
}

}  // namespace

// Returns {dy2, dgate}.  dy2 is dy itself for mode 0; dgate is undefined unless mode 2.
// db (fp32 [N]) receives the bias gradient (added to its contents when db_accumulate).
std::vector<torch::Tensor> linear_bwd_prep(torch::Tensor dy, c10::optional<torch::Tensor> saved,
                                           c10::optional<torch::Tensor> gate, int64_t S, int64_t mode,
                                           c10::optional<torch::Tensor> db, bool db_accumulate) {
  VO_CHECK_INPUT(dy);
  TORCH_CHECK(dy.scalar_type() == at::kBFloat16 && dy.dim() == 2, "dy must be bf16 [M, N]");
  c10::cuda::CUDAGuard guard(dy.device());
  const int64_t M = dy.size(0), N = dy.size(1);
  TORCH_CHECK(N % 8 == 0, "N must be a multiple of 8");
  TORCH_CHECK(mode >= 0 && mode <= 2, "bad mode");
  const bool want_db = db.has_value() && db->defined();
  if (want_db) {
    TORCH_CHECK(db->scalar_type() == at::kFloat && db->is_contiguous() && db->numel() == N, "db must be fp32 [N]");
  }
  torch::Tensor sv, gt;
  if (mode >= 1) {
    TORCH_CHECK(saved.has_value(), "mode needs the saved activation");
    sv = saved->contiguous();
    TORCH_CHECK(sv.numel() == M * N && sv.scalar_type() == at::kBFloat16, "saved must be bf16 [M, N]");
  }
  int64_t Bs = 1, Ss = M;
  int64_t gate_ld = 0;
  if (mode == 2) {
    TORCH_CHECK(gate.has_value() && S > 0 && M % S == 0, "gate_res needs gate and S dividing M");
    gt = *gate;
    TORCH_CHECK(gt.scalar_type() == at::kBFloat16 && gt.dim() == 2 && gt.size(1) == N && gt.stride(1) == 1,
                "gate must be bf16 [B, N] with unit column stride");
    gate_ld = gt.stride(0);
    TORCH_CHECK(gate_ld % 8 == 0 && (reinterpret_cast<uintptr_t>(gt.data_ptr()) & 15) == 0, "gate not 16B aligned");
    Bs = M / S;
    Ss = S;
    TORCH_CHECK(gt.size(0) == Bs, "gate rows != samples");
  }
  TORCH_CHECK((reinterpret_cast<uintptr_t>(dy.data_ptr()) & 15) == 0 &&
                  (!sv.defined() || (reinterpret_cast<uintptr_t>(sv.data_ptr()) & 15) == 0),
              "dy / saved must be 16-byte aligned");
  if (M == 0) return {dy, torch::Tensor()};
  const int cps = (int)((Ss + kRows - 1) / kRows);
  const int chunks = (int)(Bs * cps);
  TORCH_CHECK(chunks <= 65535, "too many row chunks");
  auto f32 = dy.options().dtype(torch::kFloat32);
  torch::Tensor pdb = want_db ? torch::empty({chunks, N}, f32) : torch::Tensor();
  torch::Tensor pdg = mode == 2 ? torch::empty({chunks, N}, f32) : torch::Tensor();
  torch::Tensor dy2 = mode == 0 ? dy : torch::empty_like(dy);
  torch::Tensor dgate = mode == 2 ? torch::empty({Bs, N}, dy.options()) : torch::Tensor();
  if (mode == 0 && !want_db) return {dy2, dgate};
  dim3 grid((unsigned)((N / 8 + kThreads - 1) / kThreads), (unsigned)chunks);
  const __nv_bfloat16* sp = mode >= 1 ? cbf(sv) : nullptr;
  const __nv_bfloat16* gp = mode == 2 ? cbf(gt) : nullptr;
  auto* o = reinterpret_cast<__nv_bfloat16*>(dy2.data_ptr<at::BFloat16>());
  float* a = want_db ? pdb.data_ptr<float>() : nullptr;
  float* g = mode == 2 ? pdg.data_ptr<float>() : nullptr;
  const int iN = (int)N, iS = (int)Ss;
  if (mode == 0) launch_prep<0, true>(grid, cbf(dy), sp, gp, gate_ld, o, a, g, iN, iS, cps);
  else if (mode == 1 && want_db) launch_prep<1, true>(grid, cbf(dy), sp, gp, gate_ld, o, a, g, iN, iS, cps);
  else if (mode == 1) launch_prep<1, false>(grid, cbf(dy), sp, gp, gate_ld, o, a, g, iN, iS, cps);
  else if (want_db) launch_prep<2, true>(grid, cbf(dy), sp, gp, gate_ld, o, a, g, iN, iS, cps);
  else launch_prep<2, false>(grid, cbf(dy), sp, gp, gate_ld, o, a, g, iN, iS, cps);
  count_launch();
  if (want_db || mode == 2) {
    bwd_prep_reduce_kernel<<<(unsigned)((N + kRedCols - 1) / kRedCols), kRedCols * kRedLanes, 0, stream()>>>(
        a, g, iN, (int)Bs, cps, want_db ? db->data_ptr<float>() : nullptr, db_accumulate ? 1 : 0,
        mode == 2 ? reinterpret_cast<__nv_bfloat16*>(dgate.data_ptr<at::BFloat16>()) : nullptr);
    count_launch();
  }
  VO_CUDA_OK(cudaGetLastError());
  return {dy2, dgate};
}

}  // namespace vo
