// Expert-parallel token exchange over peer memory: row copies into other GPUs' buffers.
//
// The dispatch of a mixture-of-experts layer sends every routed (token, slot) row to the rank that owns its
// expert, straight into that rank's expert-sorted, 128-row-padded input buffer (the layout of the
// expert-grouped GEMM); the combine sends every expert output row back to the slot of the rank that routed
// it.  Both are this one kernel: row i of `src` (row src_idx[i]) is stored at row dst_row[i] of the buffer
// of rank dst_rank[i] (a peer pointer of a symmetric allocation), one warp per row, 16-byte vectors over
// NVLink.  The grouped GEMMs run between the exchanges on each owner's own memory.
#include "common.cuh"

namespace vo {
namespace {

constexpr int kMaxRanks = 8;

struct PeerTable {
  __nv_bfloat16* ptr[kMaxRanks];
};

// A map entry whose source row, destination rank or destination row is out of range is skipped (never
// stored through) and counted in *err, which the host checks after the exchange.
__global__ void peer_row_copy_kernel(const __nv_bfloat16* __restrict__ src, const int64_t* __restrict__ src_idx,
                                     const int* __restrict__ dst_rank, const int64_t* __restrict__ dst_row,
                                     PeerTable peers, int npeers, int64_t src_rows, int64_t dst_rows, int64_t n,
                                     int vecs, int* __restrict__ err) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < n; i += warps) {
    const int64_t si = src_idx[i], di = dst_row[i];
    const int dr = dst_rank[i];
    if (!VO_DCHECK(si >= 0 && si < src_rows && dr >= 0 && dr < npeers && di >= 0 && di < dst_rows)) {
      if (lane == 0 && err) atomicAdd(err, 1);
      continue;
    }
    const bf16x8* s = reinterpret_cast<const bf16x8*>(src) + si * vecs;
    bf16x8* d = reinterpret_cast<bf16x8*>(peers.ptr[dr]) + di * vecs;
    for (int v = lane; v < vecs; v += 32) d[v] = s[v];
  }
}

// out[r, :] = sum over s < W of slots[s * R + r, :] (+ bias), fp32 accumulation, 8 columns per thread.
__global__ void slot_sum_kernel(const bf16x8* __restrict__ slots, const bf16x8* __restrict__ bias,
                                bf16x8* __restrict__ out, int64_t R, int vecs, int W) {
  const int64_t n = R * vecs;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8], f[8];
    if (bias) {
      unpack8(bias[i % vecs], acc);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    for (int s = 0; s < W; ++s) {
      unpack8(slots[(int64_t)s * n + i], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    out[i] = pack8(acc);
  }
}

}  // namespace

// slots: bf16 [W * R, N] (W partial-sum slots of R rows, this rank's own buffer) -> [R, N] bf16 sum (+ bias).
torch::Tensor slot_sum(torch::Tensor slots, int64_t W, c10::optional<torch::Tensor> bias) {
  VO_CHECK_INPUT(slots);
  TORCH_CHECK(slots.scalar_type() == torch::kBFloat16 && slots.dim() == 2 && slots.size(1) % 8 == 0 && W >= 1 &&
                  slots.size(0) % W == 0,
              "bf16 [W * R, N % 8] slots");
  const int64_t R = slots.size(0) / W, N = slots.size(1);
  const __nv_bfloat16* bp = nullptr;
  if (bias.has_value() && bias->defined()) {
    VO_CHECK_INPUT(*bias);
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->numel() == N, "bf16 [N] bias");
    bp = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr<at::BFloat16>());
  }
  auto out = torch::empty({R, N}, slots.options());
  if (R == 0) return out;
  c10::cuda::CUDAGuard g(slots.device());
  const int vecs = (int)(N / 8);
  const int64_t n = R * vecs;
  const int grid = (int)std::min<int64_t>((n + 255) / 256, 8LL * num_sms());
  slot_sum_kernel<<<grid, 256, 0, stream()>>>(reinterpret_cast<const bf16x8*>(slots.data_ptr<at::BFloat16>()),
                                              reinterpret_cast<const bf16x8*>(bp),
                                              reinterpret_cast<bf16x8*>(out.data_ptr<at::BFloat16>()), R, vecs, (int)W);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return out;
}

// dst (contiguous, this GPU) <- nbytes read from src_ptr (a peer's symmetric buffer) by the copy engine on
// the current stream: a remote operand crosses NVLink once before local GEMMs re-read it.
void peer_copy(torch::Tensor dst, int64_t src_ptr, int64_t nbytes) {
  VO_CHECK_INPUT(dst);
  TORCH_CHECK(nbytes >= 0 && nbytes <= (int64_t)(dst.numel() * dst.element_size()), "copy larger than dst");
  if (nbytes == 0) return;
  c10::cuda::CUDAGuard g(dst.device());
  VO_CUDA_OK(cudaMemcpyAsync(dst.data_ptr(), reinterpret_cast<const void*>(src_ptr), (size_t)nbytes,
                             cudaMemcpyDeviceToDevice, stream()));
}

// src [N, D] bf16; src_idx int64 [n]; dst_rank int32 [n] (< number of peers); dst_row int64 [n];
// peers: data pointers of each rank's [dst_rows, D] bf16 buffer (this rank's own included).  Entries out of
// range are skipped and counted into err (int32 [1] on the device) when it is given.
void peer_row_copy(torch::Tensor src, torch::Tensor src_idx, torch::Tensor dst_rank, torch::Tensor dst_row,
                   std::vector<int64_t> peers, int64_t dst_rows, c10::optional<torch::Tensor> err) {
  VO_CHECK_INPUT(src);
  VO_CHECK_INPUT(src_idx);
  VO_CHECK_INPUT(dst_rank);
  VO_CHECK_INPUT(dst_row);
  TORCH_CHECK(src.scalar_type() == torch::kBFloat16 && src.dim() == 2 && src.size(1) % 8 == 0, "bf16 [N, D % 8] rows");
  TORCH_CHECK(src_idx.scalar_type() == torch::kInt64 && dst_row.scalar_type() == torch::kInt64 &&
                  dst_rank.scalar_type() == torch::kInt32 && src_idx.numel() == dst_row.numel() &&
                  dst_rank.numel() == dst_row.numel(),
              "row maps: int64 source rows, int32 ranks, int64 destination rows of one length");
  TORCH_CHECK(!peers.empty() && peers.size() <= (size_t)kMaxRanks, "1..8 destination buffers");
  TORCH_CHECK(dst_rows >= 0, "destination capacity in rows");
  int* errp = nullptr;
  if (err.has_value() && err->defined()) {
    VO_CHECK_INPUT(*err);
    TORCH_CHECK(err->scalar_type() == torch::kInt32 && err->numel() >= 1, "int32 error counter");
    errp = err->data_ptr<int>();
  }
  const int64_t n = src_idx.numel();
  if (n == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  PeerTable t{};
  for (size_t i = 0; i < peers.size(); ++i) {
    TORCH_CHECK(peers[i] != 0 && peers[i] % 16 == 0, "destination buffers must be non-null and 16-byte aligned");
    t.ptr[i] = reinterpret_cast<__nv_bfloat16*>(peers[i]);
  }
  const int vecs = (int)(src.size(1) / 8);
  const int grid = (int)std::min<int64_t>((n + 7) / 8, 8LL * num_sms());
  peer_row_copy_kernel<<<grid, 256, 0, stream()>>>(reinterpret_cast<const __nv_bfloat16*>(src.data_ptr<at::BFloat16>()),
                                                  src_idx.data_ptr<int64_t>(), dst_rank.data_ptr<int>(),
                                                  dst_row.data_ptr<int64_t>(), t, (int)peers.size(), src.size(0),
                                                  dst_rows, n, vecs, errp);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
}

}  // namespace vo
