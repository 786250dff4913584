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

// Peer counts known at compile time: every thread issues its 2 x W independent 16-byte peer loads before the
// first add (memory-level parallelism over NVLink; the runtime-W loop above serialises them).  The caller
// rotates the peer list by its own rank, so at any moment the W ranks read W different peers.
template <int W>
__global__ void peer_reduce_w_kernel(PeerPtrs pp, int64_t lo, int64_t n4, float scale, float4* __restrict__ out,
                                     float* __restrict__ partial) {
  __shared__ float red[32];
  const float4* src[W];
#pragma unroll
  for (int r = 0; r < W; ++r) src[r] = reinterpret_cast<const float4*>(pp.grad[r] + lo);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float s = 0.f;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += 2 * stride) {
    const int64_t j = i + stride;
    const bool two = j < n4;
    float4 a[W], b[W];
#pragma unroll
    for (int r = 0; r < W; ++r) {
      a[r] = src[r][i];
      b[r] = two ? src[r][j] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float4 x = a[0], y = b[0];
#pragma unroll
    for (int r = 1; r < W; ++r) {
      x.x += a[r].x; x.y += a[r].y; x.z += a[r].z; x.w += a[r].w;
      y.x += b[r].x; y.y += b[r].y; y.z += b[r].z; y.w += b[r].w;
    }
    x = make_float4(x.x * scale, x.y * scale, x.z * scale, x.w * scale);
    out[i] = x;
    s += x.x * x.x + x.y * x.y + x.z * x.z + x.w * x.w;
    if (two) {
      y = make_float4(y.x * scale, y.y * scale, y.z * scale, y.w * scale);
      out[j] = y;
      s += y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w;
    }
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) partial[blockIdx.x] = s;
}

// AdamW on 8 consecutive shard elements per thread (two float4 of master / grad / moments), the 8 bf16
// results packed into one 16-byte store per peer: full 16-byte NVLink writes instead of 2-byte ones.
template <int W>
__global__ void adamw_bcast8_kernel(PeerPtrs pp, int64_t lo, int64_t n8, float4* __restrict__ p,
                                    const float4* __restrict__ g, float4* __restrict__ m, float4* __restrict__ v,
                                    float lr, float b1, float b2, float eps, float wd, float bc1, float bc2_sqrt,
                                    float max_norm, const float* __restrict__ sq_norm) {
  float coef = 1.f;
  bool skip = false;
  if (sq_norm) {
    const float norm = sqrtf(sq_norm[0]);
    skip = !isfinite(norm);
    if (max_norm > 0.f) coef = fminf(1.f, max_norm / (norm + 1e-6f));
  }
  const float step = lr / bc1, decay = 1.f - lr * wd;
  uint4* dst[W];
#pragma unroll
  for (int r = 0; r < W; ++r) dst[r] = reinterpret_cast<uint4*>(pp.flat16[r] + lo);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float pv[8];
    *reinterpret_cast<float4*>(pv) = p[2 * i];
    *reinterpret_cast<float4*>(pv + 4) = p[2 * i + 1];
    if (!skip) {
      float gv[8], mv[8], vv[8];
      *reinterpret_cast<float4*>(gv) = g[2 * i];
      *reinterpret_cast<float4*>(gv + 4) = g[2 * i + 1];
      *reinterpret_cast<float4*>(mv) = m[2 * i];
      *reinterpret_cast<float4*>(mv + 4) = m[2 * i + 1];
      *reinterpret_cast<float4*>(vv) = v[2 * i];
      *reinterpret_cast<float4*>(vv + 4) = v[2 * i + 1];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float gi = gv[k] * coef;
        mv[k] = b1 * mv[k] + (1.f - b1) * gi;
        vv[k] = b2 * vv[k] + (1.f - b2) * gi * gi;
        pv[k] = pv[k] * decay - step * mv[k] / (sqrtf(vv[k]) / bc2_sqrt + eps);
      }
      p[2 * i] = *reinterpret_cast<float4*>(pv);
      p[2 * i + 1] = *reinterpret_cast<float4*>(pv + 4);
      m[2 * i] = *reinterpret_cast<float4*>(mv);
      m[2 * i + 1] = *reinterpret_cast<float4*>(mv + 4);
      v[2 * i] = *reinterpret_cast<float4*>(vv);
      v[2 * i + 1] = *reinterpret_cast<float4*>(vv + 4);
    }
    uint4 packed;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&packed);
#pragma unroll
    for (int k = 0; k < 4; ++k) h[k] = __floats2bfloat162_rn(pv[2 * k], pv[2 * k + 1]);
#pragma unroll
    for (int r = 0; r < W; ++r) dst[r][i] = packed;
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

// All-to-all with the layout change folded in (Ulysses sequence <-> head exchanges, forward and backward).
// A job moves n_i x n_j x n_k contiguous bf16 chunks of `len` elements: chunk (i, j, k) starts at
// src + i*si + j*sj + k*sk and lands on rank q = (rank_dim == 1 ? j : k) / rdiv, at
// dbase + i*di + j'*dj + k'*dk of q's receive buffer (j', k' = the index left after the rank is taken out).
// One warp per chunk, 16-byte loads and peer stores (four in flight per lane); no TMA, no multicast.
constexpr int kA2AJobs = 4;
struct A2AJob {
  const __nv_bfloat16* src;
  int64_t ni, nj, nk, si, sj, sk, di, dj, dk, dbase, len, chunk0;
  int32_t rank_dim, rdiv;
};
struct A2AParams {
  A2AJob job[kA2AJobs];
  __nv_bfloat16* dst[kMaxPeers];
  int njobs;
};

__global__ void peer_a2a_kernel(const __grid_constant__ A2AParams p, int64_t total_chunks) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; c < total_chunks; c += nwarps) {
    int jb = 0;
    while (jb + 1 < p.njobs && c >= p.job[jb + 1].chunk0) ++jb;
    const A2AJob& J = p.job[jb];
    int64_t t = c - J.chunk0;
    const int64_t k = t % J.nk;
    t /= J.nk;
    const int64_t j = t % J.nj, i = t / J.nj;
    int64_t jj = j, kk = k;
    int q;
    if (J.rank_dim == 1) {
      q = (int)(j / J.rdiv);
      jj = j % J.rdiv;
    } else {
      q = (int)(k / J.rdiv);
      kk = k % J.rdiv;
    }
    const uint4* s = reinterpret_cast<const uint4*>(J.src + i * J.si + j * J.sj + k * J.sk);
    uint4* d = reinterpret_cast<uint4*>(p.dst[q] + J.dbase + i * J.di + jj * J.dj + kk * J.dk);
    const int64_t nv = J.len >> 3;
    int64_t v = lane;
    for (; v + 96 < nv; v += 128) {
      const uint4 a = s[v], b = s[v + 32], e = s[v + 64], f = s[v + 96];
      d[v] = a;
      d[v + 32] = b;
      d[v + 64] = e;
      d[v + 96] = f;
    }
    for (; v < nv; v += 32) d[v] = s[v];
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
  bool vec = (lo % 4) == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr<float>()) & 15) == 0;
  for (int r = 0; r < W; ++r) vec = vec && (grad_ptrs[r] & 15) == 0;
  const int64_t n4 = n / 4;
  auto* o4 = reinterpret_cast<float4*>(out.data_ptr<float>());
  float* pt = partial.data_ptr<float>();
  if (vec && n % 4 == 0 && (W == 2 || W == 4 || W == 8)) {
    if (W == 2) peer_reduce_w_kernel<2><<<nb, 512, 0, stream()>>>(pp, lo, n4, (float)scale, o4, pt);
    if (W == 4) peer_reduce_w_kernel<4><<<nb, 512, 0, stream()>>>(pp, lo, n4, (float)scale, o4, pt);
    if (W == 8) peer_reduce_w_kernel<8><<<nb, 256, 0, stream()>>>(pp, lo, n4, (float)scale, o4, pt);
  } else {
    peer_reduce_kernel<<<nb, 512, 0, stream()>>>(pp, W, lo, n, (float)scale, out.data_ptr<float>(), pt);
  }
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
  const float bc2s = (float)std::sqrt(bc2);
  bool vec = (lo % 8) == 0;
  for (int r = 0; r < W; ++r) vec = vec && (flat_ptrs[r] & 15) == 0;
  for (const torch::Tensor* t : {&p, &grad, &m, &v})
    vec = vec && (reinterpret_cast<uintptr_t>(t->data_ptr<float>()) & 15) == 0;
  const int64_t n8 = (vec && (W == 1 || W == 2 || W == 4 || W == 8)) ? n / 8 : 0;
  if (n8 > 0) {
    const int nb8 = (int)std::min<int64_t>((n8 + 255) / 256, 8LL * num_sms());
    auto f4 = [](torch::Tensor& t) { return reinterpret_cast<float4*>(t.data_ptr<float>()); };
    const float4* g4 = reinterpret_cast<const float4*>(grad.data_ptr<float>());
#define VO_ADAMW8(WW)                                                                                         \
  adamw_bcast8_kernel<WW><<<nb8, 256, 0, stream()>>>(pp, lo, n8, f4(p), g4, f4(m), f4(v), (float)lr, (float)b1, \
                                                     (float)b2, (float)eps, (float)wd, (float)bc1, bc2s,          \
                                                     (float)max_norm, sq_norm.data_ptr<float>())
    if (W == 1) VO_ADAMW8(1);
    if (W == 2) VO_ADAMW8(2);
    if (W == 4) VO_ADAMW8(4);
    if (W == 8) VO_ADAMW8(8);
#undef VO_ADAMW8
    count_launch();
  }
  const int64_t done = n8 * 8, rest = n - done;
  if (rest > 0) {  // elements past the last full group of 8 (or every element when unaligned)
    const int nb = (int)std::min<int64_t>((rest + 255) / 256, 8LL * num_sms());
    adamw_bcast_kernel<<<nb, 256, 0, stream()>>>(pp, W, lo + done, rest, p.data_ptr<float>() + done,
                                                 grad.data_ptr<float>() + done, m.data_ptr<float>() + done,
                                                 v.data_ptr<float>() + done, (float)lr, (float)b1, (float)b2,
                                                 (float)eps, (float)wd, (float)bc1, bc2s, (float)max_norm,
                                                 sq_norm.data_ptr<float>());
    count_launch();
  }
  VO_CUDA_OK(cudaGetLastError());
}

// jobs: int64 [n, 14] rows (src_ptr, ni, nj, nk, si, sj, sk, di, dj, dk, dbase, len, rank_dim, rdiv), strides
// and offsets in elements; src_numel[n] bounds each source; dst_ptrs: every rank's receive buffer (this
// rank's own included) of dst_cap elements.  Every chunk is checked on the host against both bounds.
void peer_a2a(torch::Tensor jobs, std::vector<int64_t> src_numel, std::vector<int64_t> dst_ptrs, int64_t dst_cap) {
  TORCH_CHECK(jobs.dim() == 2 && jobs.size(1) == 14 && jobs.scalar_type() == torch::kInt64, "jobs must be int64 [n, 14]");
  const int n = (int)jobs.size(0);
  TORCH_CHECK(n >= 1 && n <= kA2AJobs && (int)src_numel.size() == n, "1..4 jobs with their source sizes");
  const int W = (int)dst_ptrs.size();
  TORCH_CHECK(W >= 1 && W <= kMaxPeers, "1..16 receive buffers");
  auto jc = jobs.contiguous().cpu();
  const int64_t* row = jc.data_ptr<int64_t>();
  A2AParams p{};
  p.njobs = n;
  int64_t total = 0;
  for (int t = 0; t < n; ++t, row += 14) {
    A2AJob& J = p.job[t];
    J.src = reinterpret_cast<const __nv_bfloat16*>(row[0]);
    J.ni = row[1]; J.nj = row[2]; J.nk = row[3];
    J.si = row[4]; J.sj = row[5]; J.sk = row[6];
    J.di = row[7]; J.dj = row[8]; J.dk = row[9]; J.dbase = row[10];
    J.len = row[11];
    J.rank_dim = (int32_t)row[12];
    J.rdiv = (int32_t)row[13];
    J.chunk0 = total;
    TORCH_CHECK(J.ni > 0 && J.nj > 0 && J.nk > 0 && J.len > 0 && J.len % 8 == 0, "chunks of a multiple of 8 elements");
    TORCH_CHECK((J.rank_dim == 1 || J.rank_dim == 2) && J.rdiv >= 1, "rank taken from dim 1 or 2");
    for (int64_t x : {J.si, J.sj, J.sk, J.di, J.dj, J.dk, J.dbase})
      TORCH_CHECK(x >= 0 && x % 8 == 0, "strides and offsets: non-negative multiples of 8 elements");
    TORCH_CHECK((reinterpret_cast<uintptr_t>(J.src) & 15) == 0, "16-byte aligned source");
    const int64_t rank_extent = J.rank_dim == 1 ? J.nj : J.nk;
    TORCH_CHECK((rank_extent - 1) / J.rdiv < W, "a chunk addresses a rank outside the group");
    const int64_t jmax = J.rank_dim == 1 ? std::min<int64_t>(J.nj, J.rdiv) - 1 : J.nj - 1;
    const int64_t kmax = J.rank_dim == 2 ? std::min<int64_t>(J.nk, J.rdiv) - 1 : J.nk - 1;
    TORCH_CHECK((J.ni - 1) * J.si + (J.nj - 1) * J.sj + (J.nk - 1) * J.sk + J.len <= src_numel[t], "source overrun");
    TORCH_CHECK(J.dbase + (J.ni - 1) * J.di + jmax * J.dj + kmax * J.dk + J.len <= dst_cap, "receive buffer overrun");
    total += J.ni * J.nj * J.nk;
  }
  for (int r = 0; r < W; ++r) {
    TORCH_CHECK((dst_ptrs[r] & 15) == 0, "16-byte aligned receive buffers");
    p.dst[r] = reinterpret_cast<__nv_bfloat16*>(dst_ptrs[r]);
  }
  const int64_t blocks = std::min<int64_t>((total + 7) / 8, 8LL * num_sms());
  peer_a2a_kernel<<<(int)std::max<int64_t>(blocks, 1), 256, 0, stream()>>>(p, total);
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
