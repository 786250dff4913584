// Fused flow-matching reverse-SDE step with per-sample log-probability.
//
// One pass over the latents computes, per element,
//   mean = ca[b]*x + cb[b]*v          (x = sample, v = model output; the three SDE variants
//                                      sde / cps / dance_sde are all affine in (x, v))
//   prev = mean + scale[b]*z          (z ~ N(0,1) from Philox4x32-10 keyed by seed, unless
//                                      prev or an explicit noise tensor is given)
//   d2  += (prev - mean)^2            (block partial sums, reduced in fixed order)
// and a second tiny kernel turns the per-row sums into the mean log-prob with the Gaussian
// normaliser.  The backward is elementwise: dL/dv = cb*(g_mean + g_logp*dlogp/dmean).
// Math restates verl_omni/pipelines/schedulers/flow_match_sde.py:214-313.
#include "common.cuh"
#include "sde_noalloc.h"

#include <atomic>
#include <mutex>

namespace vo {
namespace {

struct RowCoef {
  float ca, cb, scale, std, lp_coef, lp_const;  // logp = lp_coef*sum(d2)/N + lp_const
};

__device__ RowCoef row_coef(float sigma_f, float sigma_prev_f, float sigma_max, float eta, int type, bool norm) {
  // Per-row scalars in double, rounded once.
  double s = sigma_f, sp = sigma_prev_f, dt = sp - s;
  RowCoef c;
  if (type == 0) {  // FlowGRPO "sde"
    double den = 1.0 - (s == 1.0 ? (double)sigma_max : s);
    double std = sqrt(s / den) * eta;
    double ca = 1.0 + std * std / (2.0 * s) * dt;
    double cb = (1.0 + std * std * (1.0 - s) / (2.0 * s)) * dt;
    double scale = std * sqrt(-dt);
    c.ca = (float)ca;
    c.cb = (float)cb;
    c.scale = (float)scale;
    c.std = (float)std;
    c.lp_coef = (float)(-1.0 / (2.0 * scale * scale));
    c.lp_const = norm ? (float)(-log(scale) - 0.5 * log(2.0 * M_PI)) : 0.f;
  } else if (type == 1) {  // "cps"
    double std = sp * sin(eta * M_PI / 2.0);
    double sq = sqrt(fmax(sp * sp - std * std, 0.0));
    c.ca = (float)((1.0 - sp) + sq);
    c.cb = (float)(-s * (1.0 - sp) + (1.0 - s) * sq);
    c.scale = (float)std;
    c.std = (float)std;
    c.lp_coef = -1.f;
    c.lp_const = 0.f;
  } else {  // "dance_sde"
    double half = 0.5 * eta * eta;
    double std = eta * sqrt(s - sp);
    c.ca = (float)(1.0 + half * dt / s);
    c.cb = (float)(dt + half * (1.0 - s) * dt / s);
    c.scale = (float)std;
    c.std = (float)std;
    c.lp_coef = (float)(-1.0 / (2.0 * std * std));
    c.lp_const = norm ? (float)(-log(std) - 0.5 * log(2.0 * M_PI)) : 0.f;
  }
  return c;
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11).
__device__ __forceinline__ uint4 philox(uint4 c, uint2 k) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k.x += W0;
      k.y += W1;
    }
    uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  return c;
}

__device__ __forceinline__ float2 box_muller(uint32_t a, uint32_t b) {
  const double inv = 2.3283064365386963e-10;  // 2^-32
  float u1 = (float)(((double)a + 1.0) * inv);
  float u2 = (float)((double)b * inv);
  float r = sqrtf(-2.f * logf(u1));
  float ang = 6.2831855f * u2;
  return make_float2(r * cosf(ang), r * sinf(ang));
}

template <bool kHasPrev, bool kHasNoise>
__global__ void sde_fwd_kernel(const float* __restrict__ x, const float* __restrict__ v,
                               const float* __restrict__ sigma, const float* __restrict__ sigma_prev,
                               const float* __restrict__ prev_in, const float* __restrict__ noise,
                               float* __restrict__ prev_out, float* __restrict__ mean_out,
                               float* __restrict__ partial, int64_t n, int64_t chunk, int nchunks,
                               float sigma_max, float eta, int type, bool norm, uint64_t seed, uint32_t offset,
                               const int64_t* __restrict__ row_seeds) {
  __shared__ float red[32];
  const int b = blockIdx.y;
  const RowCoef c = row_coef(sigma[b], sigma_prev[b], sigma_max, eta, type, norm);
  const int64_t base = (int64_t)b * n;
  const int64_t lo = (int64_t)blockIdx.x * chunk;
  const int64_t hi = min(lo + chunk, n);
  // per-row seeds make a sample's noise independent of its position in the batch (request packing);
  // otherwise one seed keys the whole call and the row index enters the Philox counter
  const uint64_t s = row_seeds ? (uint64_t)row_seeds[b] : seed;
  const uint2 key = make_uint2((uint32_t)s, (uint32_t)(s >> 32));
  const uint32_t brow = row_seeds ? 0u : (uint32_t)b;
  float acc = 0.f;
  for (int64_t i = lo + 4 * (int64_t)threadIdx.x; i < hi; i += 4 * (int64_t)blockDim.x) {
    float xs[4], vs[4], ps[4], ms[4];
    const bool full = (i + 4 <= hi) && (((base + i) & 3) == 0);
    if (full) {
      float4 a = *reinterpret_cast<const float4*>(x + base + i);
      float4 bb = *reinterpret_cast<const float4*>(v + base + i);
      xs[0] = a.x; xs[1] = a.y; xs[2] = a.z; xs[3] = a.w;
      vs[0] = bb.x; vs[1] = bb.y; vs[2] = bb.z; vs[3] = bb.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        xs[j] = (i + j < hi) ? x[base + i + j] : 0.f;
        vs[j] = (i + j < hi) ? v[base + i + j] : 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) ms[j] = xs[j] * c.ca + vs[j] * c.cb;
    if (kHasPrev) {
#pragma unroll
      for (int j = 0; j < 4; ++j) ps[j] = (i + j < hi) ? prev_in[base + i + j] : ms[j];
    } else if (kHasNoise) {
#pragma unroll
      for (int j = 0; j < 4; ++j) ps[j] = (i + j < hi) ? ms[j] + c.scale * noise[base + i + j] : ms[j];
    } else {
      uint4 r = philox(make_uint4((uint32_t)(i >> 2), brow, offset, 0u), key);
      float2 z01 = box_muller(r.x, r.y), z23 = box_muller(r.z, r.w);
      ps[0] = ms[0] + c.scale * z01.x;
      ps[1] = ms[1] + c.scale * z01.y;
      ps[2] = ms[2] + c.scale * z23.x;
      ps[3] = ms[3] + c.scale * z23.y;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (i + j < hi) {
        float d = ps[j] - ms[j];
        acc += d * d;
      }
    }
    if (full) {
      *reinterpret_cast<float4*>(mean_out + base + i) = make_float4(ms[0], ms[1], ms[2], ms[3]);
      if (!kHasPrev) *reinterpret_cast<float4*>(prev_out + base + i) = make_float4(ps[0], ps[1], ps[2], ps[3]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (i + j < hi) {
          mean_out[base + i + j] = ms[j];
          if (!kHasPrev) prev_out[base + i + j] = ps[j];
        }
      }
    }
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) partial[(int64_t)b * nchunks + blockIdx.x] = acc;
}

// One warp per row: fixed-order reduction of the chunk partials, then the log-prob.
__global__ void sde_finalize_kernel(const float* __restrict__ partial, const float* __restrict__ sigma,
                                    const float* __restrict__ sigma_prev, float* __restrict__ logp,
                                    float* __restrict__ std_out, int B, int nchunks, int64_t n, float sigma_max,
                                    float eta, int type, bool norm) {
  const int b = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (b >= B) return;
  float s = 0.f;
  for (int i = lane; i < nchunks; i += 32) s += partial[(int64_t)b * nchunks + i];
  s = warp_sum(s);
  if (lane == 0) {
    RowCoef c = row_coef(sigma[b], sigma_prev[b], sigma_max, eta, type, norm);
    if (logp) logp[b] = c.lp_coef * (s / (float)n) + c.lp_const;
    std_out[b] = c.std;
  }
}

__global__ void sde_bwd_kernel(const float* __restrict__ prev, const float* __restrict__ mean,
                               const float* __restrict__ sigma, const float* __restrict__ sigma_prev,
                               const float* __restrict__ g_logp, const float* __restrict__ g_mean,
                               float* __restrict__ g_v, int64_t n, float sigma_max, float eta, int type) {
  const int b = blockIdx.y;
  const RowCoef c = row_coef(sigma[b], sigma_prev[b], sigma_max, eta, type, true);
  // d logp / d mean_i = -2*lp_coef*(prev_i - mean_i)/N   (lp_coef = -1/(2 var) or -1 for cps)
  const float k = g_logp[b] * (-2.f * c.lp_coef) / (float)n;
  const int64_t base = (int64_t)b * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float d = prev[base + i] - mean[base + i];
    g_v[base + i] = c.cb * (g_mean[base + i] + k * d);
  }
}

// z[b, i] ~ N(0, 1) from the same Philox4x32-10 / Box-Muller stream the SDE step draws, keyed by
// row_seeds[b] with counter (i / 4, 0, offset, 0): the initial latent noise of a rollout sample
// depends only on its own seed.
__global__ void normal_fill_kernel(float* __restrict__ out, const int64_t* __restrict__ row_seeds, int64_t n,
                                   uint32_t offset) {
  const int b = blockIdx.y;
  const uint64_t s = (uint64_t)row_seeds[b];
  const uint2 key = make_uint2((uint32_t)s, (uint32_t)(s >> 32));
  float* o = out + (int64_t)b * n;
  for (int64_t i = 4 * ((int64_t)blockIdx.x * blockDim.x + threadIdx.x); i < n; i += 4 * (int64_t)gridDim.x * blockDim.x) {
    uint4 r = philox(make_uint4((uint32_t)(i >> 2), 0u, offset, 0u), key);
    float2 z01 = box_muller(r.x, r.y), z23 = box_muller(r.z, r.w);
    const float z[4] = {z01.x, z01.y, z23.x, z23.y};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (i + j < n) o[i + j] = z[j];
  }
}

}  // namespace

torch::Tensor normal_fill(torch::Tensor row_seeds, int64_t n, int64_t offset) {
  VO_CHECK_INPUT(row_seeds);
  TORCH_CHECK(row_seeds.scalar_type() == torch::kInt64, "row_seeds must be int64");
  c10::cuda::CUDAGuard g(row_seeds.device());
  const int64_t B = row_seeds.numel();
  auto out = torch::empty({B, n}, row_seeds.options().dtype(torch::kFloat32));
  if (B == 0 || n == 0) return out;
  const int bx = (int)std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, 64));
  normal_fill_kernel<<<dim3(bx, (unsigned)B), 256, 0, stream()>>>(out.data_ptr<float>(), row_seeds.data_ptr<int64_t>(),
                                                                   n, (uint32_t)offset);
  vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return out;
}

std::vector<torch::Tensor> sde_step_fwd(torch::Tensor x, torch::Tensor v, torch::Tensor sigma,
                                        torch::Tensor sigma_prev, c10::optional<torch::Tensor> prev,
                                        c10::optional<torch::Tensor> noise, double sigma_max, double eta, int64_t type,
                                        int64_t seed, int64_t offset, bool want_logp, bool norm,
                                        c10::optional<torch::Tensor> row_seeds) {
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(v);
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && v.scalar_type() == torch::kFloat32, "fp32 inputs required");
  TORCH_CHECK(x.sizes() == v.sizes(), "sample/model_output shape mismatch");
  c10::cuda::CUDAGuard g(x.device());
  const int B = x.size(0);
  TORCH_CHECK(B >= 1 && B <= 65535, "sde_step_fwd: 1..65535 rows (one grid row per sample)");
  const int64_t n = x.numel() / B;
  auto mean = torch::empty_like(x);
  torch::Tensor prev_out;
  const bool has_prev = prev.has_value() && prev->defined();
  const bool has_noise = !has_prev && noise.has_value() && noise->defined();
  if (has_prev) {
    VO_CHECK_INPUT((*prev));
    prev_out = *prev;
  } else {
    prev_out = torch::empty_like(x);
  }
  if (has_noise) VO_CHECK_INPUT((*noise));
  // ~4 blocks per SM across the batch, chunks in multiples of 1024 elements
  int target = 4 * num_sms();
  int nchunks = std::max(1, std::min<int>((int)((n + 1023) / 1024), (target + B - 1) / B));
  int64_t chunk = ((n + nchunks - 1) / nchunks + 1023) / 1024 * 1024;
  nchunks = (int)((n + chunk - 1) / chunk);
  auto opts = x.options();
  auto partial = torch::empty({B, nchunks}, opts);
  auto logp = torch::empty({B}, opts);
  auto stdv = torch::empty({B}, opts);
  dim3 grid(nchunks, B);
  auto st = stream();
  const float* pp = has_prev ? prev->data_ptr<float>() : nullptr;
  const float* np_ = has_noise ? noise->data_ptr<float>() : nullptr;
  const int64_t* rsp = nullptr;
  if (row_seeds.has_value() && row_seeds->defined()) {
    VO_CHECK_INPUT((*row_seeds));
    TORCH_CHECK(row_seeds->scalar_type() == torch::kInt64 && row_seeds->numel() == B, "row_seeds must be int64 [B]");
    rsp = row_seeds->data_ptr<int64_t>();
  }
#define VO_SDE_LAUNCH(HP, HN)                                                                               \
  sde_fwd_kernel<HP, HN><<<grid, 256, 0, st>>>(x.data_ptr<float>(), v.data_ptr<float>(),                   \
                                               sigma.data_ptr<float>(), sigma_prev.data_ptr<float>(), pp, np_, \
                                               prev_out.data_ptr<float>(), mean.data_ptr<float>(),          \
                                               partial.data_ptr<float>(), n, chunk, nchunks, (float)sigma_max, \
                                               (float)eta, (int)type, norm, (uint64_t)seed, (uint32_t)offset, rsp)
  if (has_prev)
    VO_SDE_LAUNCH(true, false);
  else if (has_noise)
    VO_SDE_LAUNCH(false, true);
  else
    VO_SDE_LAUNCH(false, false);
  vo::count_launch();
#undef VO_SDE_LAUNCH
  sde_finalize_kernel<<<(B + 7) / 8, 256, 0, st>>>(partial.data_ptr<float>(), sigma.data_ptr<float>(),
                                                   sigma_prev.data_ptr<float>(),
                                                   want_logp ? logp.data_ptr<float>() : nullptr,
                                                   stdv.data_ptr<float>(), B, nchunks, n, (float)sigma_max,
                                                   (float)eta, (int)type, norm); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {prev_out, logp, mean, stdv};
}

torch::Tensor sde_step_bwd(torch::Tensor x, torch::Tensor prev, torch::Tensor mean, torch::Tensor sigma,
                           torch::Tensor sigma_prev, torch::Tensor g_logp, torch::Tensor g_mean, double sigma_max,
                           double eta, int64_t type) {
  VO_CHECK_INPUT(prev);
  VO_CHECK_INPUT(mean);
  VO_CHECK_INPUT(g_mean);
  c10::cuda::CUDAGuard g(x.device());
  const int B = x.size(0);
  const int64_t n = x.numel() / B;
  auto gv = torch::empty_like(x);
  int bx = std::max(1, std::min<int>((int)((n + 255) / 256), (4 * num_sms() + B - 1) / B));
  sde_bwd_kernel<<<dim3(bx, B), 256, 0, stream()>>>(prev.data_ptr<float>(), mean.data_ptr<float>(),
                                                     sigma.data_ptr<float>(), sigma_prev.data_ptr<float>(),
                                                     g_logp.data_ptr<float>(), g_mean.data_ptr<float>(),
                                                     gv.data_ptr<float>(), n, (float)sigma_max, (float)eta, (int)type); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return gv;
}

}  // namespace vo

// ------------------------------------------------------------------------------ allocation-free variant
// Scratch for the per-block partial sums of vo_sde_step_fwd_noalloc (see sde_noalloc.h).  In host code
// this name is only a stand-in for the symbol; the device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) float g_sde_noalloc_partials[VO_SDE_NOALLOC_MAX_PARTIALS];

namespace {
constexpr int kMaxDevices = 64;
// per-device scratch address and SM count; the set-up runs once per device under a mutex and publishes
// the pointer (release) only after the SM count is stored
std::atomic<float*> g_sde_noalloc_ptr[kMaxDevices];
int g_sde_noalloc_sms[kMaxDevices] = {0};
std::mutex g_sde_noalloc_mu;
}  // namespace

extern "C" __attribute__((visibility("default"))) int vo_sde_step_fwd_noalloc(
    const float* x, const float* v, const float* sigma, const float* sigma_prev, const float* prev_in,
    const float* noise, float* prev_out, float* mean_out, float* logp_out, float* std_out, int B, int64_t n,
    float sigma_max, float eta, int sde_type, uint64_t seed, uint32_t offset, int want_logp, int norm,
    cudaStream_t stream) {
  if (!x || !v || !sigma || !sigma_prev || !mean_out || !std_out || B <= 0 || n <= 0 || sde_type < 0 ||
      sde_type > 2 || (want_logp && !logp_out) || (!prev_in && !prev_out))
    return -1;
  if (B > 65535) return -2;  // one grid row per sample
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return -1;
  if (!g_sde_noalloc_ptr[dev].load(std::memory_order_acquire)) {  // one-time set-up, this device current
    std::lock_guard<std::mutex> lock(g_sde_noalloc_mu);
    if (!g_sde_noalloc_ptr[dev].load(std::memory_order_relaxed)) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_sde_noalloc_partials);
      if (e != cudaSuccess) return (int)e;
      int sms = 0;
      e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      if (e != cudaSuccess) return (int)e;
      g_sde_noalloc_sms[dev] = sms;
      g_sde_noalloc_ptr[dev].store(static_cast<float*>(ptr), std::memory_order_release);
    }
  }
  float* partial = g_sde_noalloc_ptr[dev].load(std::memory_order_acquire);
  // same chunking as the allocating entry point: ~4 blocks per SM, chunks of multiples of 1024
  const int target = 4 * g_sde_noalloc_sms[dev];
  int nchunks = (int)std::max<int64_t>(1, std::min<int64_t>((n + 1023) / 1024, (target + B - 1) / B));
  const int64_t chunk = ((n + nchunks - 1) / nchunks + 1023) / 1024 * 1024;
  nchunks = (int)((n + chunk - 1) / chunk);
  if ((int64_t)B * nchunks > VO_SDE_NOALLOC_MAX_PARTIALS) return -2;
  float* prev_dst = prev_in ? const_cast<float*>(prev_in) : prev_out;
  const dim3 grid(nchunks, B);
  if (prev_in)
    vo::sde_fwd_kernel<true, false><<<grid, 256, 0, stream>>>(x, v, sigma, sigma_prev, prev_in, nullptr, prev_dst,
                                                             mean_out, partial, n, chunk, nchunks, sigma_max, eta,
                                                             sde_type, norm != 0, seed, offset, nullptr);
  else if (noise)
    vo::sde_fwd_kernel<false, true><<<grid, 256, 0, stream>>>(x, v, sigma, sigma_prev, nullptr, noise, prev_dst,
                                                             mean_out, partial, n, chunk, nchunks, sigma_max, eta,
                                                             sde_type, norm != 0, seed, offset, nullptr);
  else
    vo::sde_fwd_kernel<false, false><<<grid, 256, 0, stream>>>(x, v, sigma, sigma_prev, nullptr, nullptr, prev_dst,
                                                              mean_out, partial, n, chunk, nchunks, sigma_max, eta,
                                                              sde_type, norm != 0, seed, offset, nullptr);
  vo::sde_finalize_kernel<<<(B + 7) / 8, 256, 0, stream>>>(partial, sigma, sigma_prev, want_logp ? logp_out : nullptr,
                                                           std_out, B, nchunks, n, sigma_max, eta, sde_type,
                                                           norm != 0);
  e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  // a caller-provided sample is also copied to a distinct prev_out (a device-to-device copy allocates nothing)
  if (prev_in && prev_out && prev_out != prev_in) {
    e = cudaMemcpyAsync(prev_out, prev_in, (size_t)B * (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}
