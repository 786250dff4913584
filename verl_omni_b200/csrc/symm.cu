// Symmetric-memory runtime and the fused optimizer collective over NVLink peer memory.
//
// Runtime: device buffers allocated with cudaMalloc and shared between the ranks of one node through
// CUDA IPC handles (exchanged by the Python side over the process group); every rank maps every
// peer's buffer, so kernels address peer memory with ordinary loads and stores over NVLink/NVSwitch.
//
// Fused optimizer step for the flat-parameter engine (replaces reduce-scatter -> AdamW -> all-gather):
//   pass 1  grad_shard[i] = scale * sum_r main_grad_r[lo + i]      (P2P loads from all W peers)
//           + per-block partial sums of grad_shard^2              (global-norm clipping)
//   pass 2  AdamW on the shard (fp32 master + moments, on-device clip / non-finite skip), then the
//           new bf16 value is stored into flat16_r[lo + i] of every peer r (P2P stores)
// Stream ordering plus a process-group barrier before pass 1 (all grads final) and after pass 2
// (all peers' weights written) make the exchange race-free; neither kernel waits on another GPU.
// Plain loads/stores only: no TMA and no multicast touch peer memory.
#include "common.cuh"

namespace vo {
namespace {

constexpr int kMaxPeers = 16;

struct PeerPtrs {
  const float* grad[kMaxPeers];
  __nv_bfloat16* flat16[kMaxPeers];
};

__global__ void peer_reduce_kernel(PeerPtrs pp, int W, int64_t lo, int64_t n, float scale, float* __restrict__ out,
                                   float* __restrict__ partial) {
  __shared__ float red[32];
  float s = 0.f;
  const int64_t n4 = n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < W; ++r) {
      const float4 g = reinterpret_cast<const float4*>(pp.grad[r] + lo)[i];
      acc.x += g.x;
      acc.y += g.y;
      acc.z += g.z;
      acc.w += g.w;
    }
    acc.x *= scale;
    acc.y *= scale;
    acc.z *= scale;
    acc.w *= scale;
    reinterpret_cast<float4*>(out)[i] = acc;
    s += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
  }
  for (int64_t i = n4 * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int r = 0; r < W; ++r) acc += pp.grad[r][lo + i];
    acc *= scale;
    out[i] = acc;
    s += acc * acc;
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

__global__ void adamw_bcast_kernel(PeerPtrs pp, int W, int64_t lo, int64_t n, float* __restrict__ p,
                                   const float* __restrict__ g, float* __restrict__ m, float* __restrict__ v, float lr,
                                   float b1, float b2, float eps, float wd, float bc1, float bc2_sqrt, float max_norm,
                                   const float* __restrict__ sq_norm) {
  float coef = 1.f;
  bool skip = false;
  if (sq_norm) {
    const float norm = sqrtf(sq_norm[0]);
    skip = !isfinite(norm);
    if (max_norm > 0.f) coef = fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const float step = lr / bc1;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float pi = p[i];
    if (!skip) {
      const float gi = g[i] * coef;
      pi *= (1.f - lr * wd);
      const float mi = b1 * m[i] + (1.f - b1) * gi;
      const float vi = b2 * v[i] + (1.f - b2) * gi * gi;
      pi -= step * mi / (sqrtf(vi) / bc2_sqrt + eps);
      p[i] = pi;
      m[i] = mi;
      v[i] = vi;
    }
    const __nv_bfloat16 b = __float2bfloat16_rn(pi);
    for (int r = 0; r < W; ++r) pp.flat16[r][lo + i] = b;
  }
}

__global__ void sum_partials(const float* __restrict__ p, int n, float* __restrict__ out) {
  __shared__ float red[32];
  float s = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s += p[i];
  s = block_sum(s, red);
  if (threadIdx.x == 0) out[0] = s;
}

// One kernel for every copy of a weight-sync plan: chunk c moves bytes [src_off, src_off + nbytes) of the
// local source buffer to dst_off of destination slot dst (a peer's mapped buffer).  16-byte vector
// stores over NVLink; each block walks the chunks with a grid-stride loop over 16-byte units.
struct PushChunk {
  int64_t src_off, dst_off, nbytes;
  int32_t dst, pad;
};
__global__ void peer_push_kernel(const uint8_t* __restrict__ src, const PushChunk* __restrict__ chunks, int nchunks,
                                 PeerPtrs dst) {
  for (int c = 0; c < nchunks; ++c) {
    const PushChunk ch = chunks[c];
    const uint4* s = reinterpret_cast<const uint4*>(src + ch.src_off);
    uint4* d = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(dst.flat16[ch.dst]) + ch.dst_off);
    const int64_t n16 = ch.nbytes >> 4;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
      d[i] = s[i];
    // tail (< 16 bytes)
    if (blockIdx.x == 0 && threadIdx.x < (ch.nbytes & 15)) {
      const int64_t o = (n16 << 4) + threadIdx.x;
      reinterpret_cast<uint8_t*>(dst.flat16[ch.dst])[ch.dst_off + o] = src[ch.src_off + o];
    }
  }
}

PeerPtrs make_ptrs(const std::vector<int64_t>& grads, const std::vector<int64_t>& flats) {
  TORCH_CHECK(grads.size() <= (size_t)kMaxPeers && flats.size() == grads.size(), "bad peer pointer lists");
  PeerPtrs pp{};
  for (size_t r = 0; r < grads.size(); ++r) {
    pp.grad[r] = reinterpret_cast<const float*>(grads[r]);
    pp.flat16[r] = reinterpret_cast<__nv_bfloat16*>(flats[r]);
  }
  return pp;
}

}  // namespace

// ---------------------------------------------------------------- runtime
int64_t symm_malloc(int64_t nbytes) {
  void* p = nullptr;
  VO_CUDA_OK(cudaMalloc(&p, (size_t)nbytes));
  VO_CUDA_OK(cudaMemset(p, 0, (size_t)nbytes));
  return reinterpret_cast<int64_t>(p);
}

void symm_free(int64_t ptr) { VO_CUDA_OK(cudaFree(reinterpret_cast<void*>(ptr))); }

torch::Tensor ipc_get_handle(int64_t ptr) {
  cudaIpcMemHandle_t h;
  VO_CUDA_OK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(ptr)));
  auto t = torch::empty({(int64_t)sizeof(h)}, torch::dtype(torch::kUInt8));
  std::memcpy(t.data_ptr(), &h, sizeof(h));
  return t;
}

int64_t ipc_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.cpu().data_ptr(), sizeof(h));
  void* p = nullptr;
  VO_CUDA_OK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { VO_CUDA_OK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

torch::Tensor tensor_from_ptr(int64_t ptr, int64_t numel, int64_t dtype_code, int64_t device) {
  auto dt = dtype_code == 0 ? torch::kFloat32 : torch::kBFloat16;
  return torch::from_blob(reinterpret_cast<void*>(ptr), {numel},
                          torch::TensorOptions().dtype(dt).device(torch::kCUDA, (int)device));
}

// ---------------------------------------------------------------- fused optimizer collective
// pass 1: returns the [1] squared norm of this rank's reduced grad shard (caller all-reduces it)
torch::Tensor peer_grad_reduce(std::vector<int64_t> grad_ptrs, int64_t lo, int64_t n, double scale,
                               torch::Tensor out) {
  VO_CHECK_INPUT(out);
  c10::cuda::CUDAGuard g(out.device());
  const int W = (int)grad_ptrs.size();
  PeerPtrs pp = make_ptrs(grad_ptrs, grad_ptrs);
  const int nb = 2 * num_sms();
  auto partial = torch::empty({nb}, out.options());
  auto sq = torch::empty({1}, out.options());
  peer_reduce_kernel<<<nb, 512, 0, stream()>>>(pp, W, lo, n, (float)scale, out.data_ptr<float>(),
                                               partial.data_ptr<float>());
  sum_partials<<<1, 512, 0, stream()>>>(partial.data_ptr<float>(), nb, sq.data_ptr<float>());
  count_launch(2);
  VO_CUDA_OK(cudaGetLastError());
  return sq;
}

// pass 2: AdamW on the shard, bf16 result stored into every peer's flat buffer at [lo, lo + n)
void peer_adamw_bcast(std::vector<int64_t> flat_ptrs, int64_t lo, int64_t n, torch::Tensor p, torch::Tensor grad,
                      torch::Tensor m, torch::Tensor v, double lr, double b1, double b2, double eps, double wd,
                      int64_t step, double max_norm, torch::Tensor sq_norm) {
  VO_CHECK_INPUT(p);
  c10::cuda::CUDAGuard g(p.device());
  const int W = (int)flat_ptrs.size();
  PeerPtrs pp = make_ptrs(flat_ptrs, flat_ptrs);
  const double bc1 = 1.0 - std::pow(b1, (double)step), bc2 = 1.0 - std::pow(b2, (double)step);
  const int nb = (int)std::min<int64_t>((n + 255) / 256, 8LL * num_sms());
  adamw_bcast_kernel<<<nb, 256, 0, stream()>>>(pp, W, lo, n, p.data_ptr<float>(), grad.data_ptr<float>(),
                                               m.data_ptr<float>(), v.data_ptr<float>(), (float)lr, (float)b1,
                                               (float)b2, (float)eps, (float)wd, (float)bc1, (float)std::sqrt(bc2),
                                               (float)max_norm, sq_norm.data_ptr<float>());
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
}

// Trainer -> rollout weight resharding: executes a copy plan (int64 [n, 5] rows: src_off, dst_off,
// nbytes, dst_slot, 0) from the local buffer at src_ptr into the mapped destination buffers.
void peer_push(int64_t src_ptr, torch::Tensor plan, std::vector<int64_t> dst_ptrs) {
  TORCH_CHECK(plan.dim() == 2 && plan.size(1) == 5 && plan.scalar_type() == torch::kInt64, "plan must be int64 [n, 5]");
  TORCH_CHECK(!dst_ptrs.empty() && dst_ptrs.size() <= (size_t)kMaxPeers, "1..16 destinations");
  auto pc = plan.contiguous().cpu();
  const int64_t* rows = pc.data_ptr<int64_t>();
  const int n = (int)pc.size(0);
  std::vector<PushChunk> chunks(n);
  for (int i = 0; i < n; ++i) {
    chunks[i] = PushChunk{rows[5 * i], rows[5 * i + 1], rows[5 * i + 2], (int32_t)rows[5 * i + 3], 0};
    TORCH_CHECK(chunks[i].dst >= 0 && chunks[i].dst < (int)dst_ptrs.size(), "bad destination slot");
    TORCH_CHECK(((chunks[i].src_off | chunks[i].dst_off) & 15) == 0, "chunk offsets must be 16-byte aligned");
  }
  if (n == 0) return;
  PeerPtrs pp{};
  for (size_t r = 0; r < dst_ptrs.size(); ++r) pp.flat16[r] = reinterpret_cast<__nv_bfloat16*>(dst_ptrs[r]);
  auto dev_chunks = torch::empty({(int64_t)(n * sizeof(PushChunk))}, torch::dtype(torch::kUInt8).device(torch::kCUDA));
  VO_CUDA_OK(cudaMemcpyAsync(dev_chunks.data_ptr(), chunks.data(), n * sizeof(PushChunk), cudaMemcpyHostToDevice,
                             stream()));
  peer_push_kernel<<<2 * num_sms(), 512, 0, stream()>>>(reinterpret_cast<const uint8_t*>(src_ptr),
                                                        reinterpret_cast<const PushChunk*>(dev_chunks.data_ptr()), n,
                                                        pp);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
}

}  // namespace vo
