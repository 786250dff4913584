// C interface of the tcgen05 GEMM (gemm_sm100.cu), shared by its torch bindings and other kernels' hosts.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vo_gemm {

enum Epi : int {
  EPI_NONE = 0,
  EPI_BIAS = 1,
  EPI_GELU = 2,
  EPI_GATE_RES = 3,
  EPI_F32_ACC = 4,
  EPI_SCATTER = 5,
  EPI_PEER_RED = 6  // fp32 tile added into the owning rank's buffer (tensor-parallel reduce-scatter)
};

constexpr int kMaxPeers = 8;

// EPI_SCATTER (Ulysses head scatter): the bf16 (+bias) output is stored straight into peer buffers.
// Output column c of part q = c / part_cols goes to destination d = (c % part_cols) / dst_cols, column
// q * dst_cols + c % dst_cols; output row m (sample m / seg_rows, token m % seg_rows) goes to row
// (m / seg_rows) * dst_seq + row_off + m % seg_rows of a destination with row stride dst_ld elements.
struct ScatterParams {
  __nv_bfloat16* peers[kMaxPeers];
  int part_cols, dst_cols, seg_rows, dst_seq, row_off, dst_ld;
};

struct EpiParams {
  int epi;
  __nv_bfloat16* out;          // [M, N] bf16 (primary output)
  __nv_bfloat16* out2;         // GELU: pre-activation; GATE_RES: linear output (saved for backward)
  float* out_f32;              // F32_ACC: [M, N] fp32, accumulated
  const __nv_bfloat16* bias;   // [N] or null
  const __nv_bfloat16* gate;   // [M/S, gate_ld] (GATE_RES)
  const __nv_bfloat16* res;    // [M, N] (GATE_RES)
  int64_t gate_ld;
  int S;  // rows per sample (GATE_RES)
  int ldc;
  ScatterParams sc;  // EPI_SCATTER
  // EPI_PEER_RED: output row m is owned by rank m / red_rows.  red_store 0: the row is added (fp32,
  // system-scope vector atomics over NVLink) at row m % red_rows of red_peers[owner] ([red_rows, ldc] fp32
  // each).  red_store 1: the row is stored in bf16 at row red_slot_off + m % red_rows of red_peers[owner]
  // (bf16 buffers holding one [red_rows, ldc] slot per source rank; the owner sums the slots afterwards).
  float* red_peers[kMaxPeers];
  int red_rows;
  int red_store;
  int red_slot_off;
};

// One GEMM of a grouped launch: C = A B^T (+ A2 B2^T), operand conventions as vo_gemm_launch_ext.
struct GemmDesc {
  const void* A = nullptr;
  const void* B = nullptr;
  const void* A2 = nullptr;
  const void* B2 = nullptr;
  int M = 0, N = 0, K = 0, K2 = 0;
  int64_t lda = 0, ldb = 0, lda2 = 0, ldb2 = 0;
  int a_mn = 0, b_mn = 0, splits = 1;
  EpiParams ep{};
  // Expert-grouped GEMM (mixture of experts; see Shape in gemm_sm100.cu): grp_mode 1 = forward / dgrad over
  // expert-sorted rows padded to 128 per expert, grp_tab[m-tile] = expert (-1 unused); B holds n_groups
  // stacked expert matrices.  grp_mode 2 = weight gradient: M = grp_rows per expert, output [n_groups *
  // grp_rows, N], reduction over rows [grp_tab[e], grp_tab[e+1]) of A and B.
  const int* grp_tab = nullptr;
  int grp_mode = 0, n_groups = 0, grp_rows = 0;
  // Operand gathered from the ranks of a tensor-parallel group (plain TMA loads of peer memory): gather 1 =
  // A rows (K-major A), 2 = A along the reduction (MN-major A), 3 = B along the reduction (MN-major B);
  // block r of gather_rows rows (of the gathered dimension) is read from gather_ptrs[r].
  const void* gather_ptrs[kMaxPeers] = {};
  int gather = 0, gather_rows = 0, gather_n = 0;
};

constexpr int kMaxGroup = 2;

}  // namespace vo_gemm

extern "C" int vo_gemm_launch(const void* A, const void* B, int M, int N, int K, int64_t lda, int64_t ldb, int a_mn,
                              int b_mn, int splits, vo_gemm::EpiParams ep, cudaStream_t stream);
extern "C" int vo_gemm_launch_ext(const void* A, const void* B, const void* A2, const void* B2, int M, int N, int K,
                                  int K2, int64_t lda, int64_t ldb, int64_t lda2, int64_t ldb2, int a_mn, int b_mn,
                                  int splits, vo_gemm::EpiParams ep, cudaStream_t stream);
// Up to kMaxGroup independent GEMMs in one persistent launch: their output tiles form one work list,
// so a small GEMM fills the last partial wave of a large one instead of running its own tail.
extern "C" int vo_gemm_launch_group(const vo_gemm::GemmDesc* d, int n, cudaStream_t stream);
extern "C" int vo_gemm_error(int reset);
