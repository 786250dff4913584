// Normalisation kernels for the DiT blocks.
//
//  * adaln_ln_fwd/bwd: LayerNorm without affine followed by AdaLN modulation
//      y = (x - mu) * rstd * (1 + scale[b]) + shift[b]
//    where (shift, scale) are per-sample rows of the block's modulation GEMM output
//    (accessed in place through a row stride, no chunk copies).  Optional plain affine mode
//    y = xhat * w + bias for the frozen ViT / text encoders.
//  * qk_rmsnorm_fwd/bwd: splits a fused QKV projection [rows, 3*H*Dh] into q, k, v in the
//    attention layout [B, H, S_total, Dh] at a sequence offset (joint text+image attention
//    writes both streams into one buffer), applying per-head RMSNorm with learned weights to
//    q and k (SD3.5 / FLUX / Wan qk-norm) and optionally rotary embeddings.
// One warp per row; rows are re-read from L1/L2 between passes so HBM sees one read and one
// write per tensor.
#include "common.cuh"

namespace vo {
namespace {

struct ModPtr {
  const __nv_bfloat16* shift;  // [B, stride] (element offset applied)
  const __nv_bfloat16* scale;
  int64_t stride;
};

// Register-resident variant: one warp per row, the row's D = 256 * NV bf16 values stay in registers
// (NV 16-byte vectors per lane, packed), so x is read from memory once; mean and variance are two passes
// over registers; at D = 1536 at most 64 registers, so four 256-thread CTAs fit on an SM.
template <int NV>
__global__ void __launch_bounds__(256, (NV <= 6 ? 4 : 1)) adaln_ln_fwd_reg_kernel(const __nv_bfloat16* __restrict__ x,
                                                               __nv_bfloat16* __restrict__ y,
                                                               float* __restrict__ mean_out,
                                                               float* __restrict__ rstd_out, ModPtr mod,
                                                               const __nv_bfloat16* __restrict__ aff_w,
                                                               const __nv_bfloat16* __restrict__ aff_b, int64_t rows,
                                                               int S, float eps) {
  constexpr int D = NV * 256;
  // the modulation (scale, shift) of the CTA's first row's sample -- or the affine weight and bias -- staged
  // once per CTA in shared memory while the rows' loads are in flight; rows of another sample (a CTA that
  // straddles a sample boundary) read theirs from global memory
  __shared__ bf16x8 sm_a[NV * 32], sm_c[NV * 32];
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const bool active = row < rows;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + (active ? row : 0) * D);
  // the row stays packed (4 registers per 8 values) and is unpacked in each pass: fewer registers, more
  // rows resident per SM, more loads in flight
  bf16x8 raw[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) raw[v] = xr[v * 32 + lane];
  const int64_t b0 = ((int64_t)blockIdx.x * (blockDim.x >> 5)) / S;
  {
    const bf16x8* sa = aff_w ? reinterpret_cast<const bf16x8*>(aff_w)
                             : reinterpret_cast<const bf16x8*>(mod.scale + b0 * mod.stride);
    const bf16x8* sc = aff_w ? reinterpret_cast<const bf16x8*>(aff_b)
                             : reinterpret_cast<const bf16x8*>(mod.shift + b0 * mod.stride);
    for (int i = threadIdx.x; i < NV * 32; i += blockDim.x) {
      sm_a[i] = sa[i];
      sm_c[i] = sc[i];
    }
  }
  __syncthreads();
  if (!active) return;
  float s = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float t[8];
    unpack8(raw[v], t);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += t[j];
  }
  const float mu = warp_sum(s) * (1.f / D);
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float t[8];
    unpack8(raw[v], t);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = t[j] - mu;
      ss += d * d;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) * (1.f / D) + eps);
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rstd;
  }
  const int64_t b = row / S;
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + row * D);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int i = v * 32 + lane;
    float a[8], c[8], o[8], fv[8];
    unpack8(raw[v], fv);
    if (aff_w || b == b0) {
      unpack8(sm_a[i], a);
      unpack8(sm_c[i], c);
    } else {
      unpack8(reinterpret_cast<const bf16x8*>(mod.scale + b * mod.stride)[i], a);
      unpack8(reinterpret_cast<const bf16x8*>(mod.shift + b * mod.stride)[i], c);
    }
    if (aff_w) {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (fv[j] - mu) * rstd * a[j] + c[j];
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (fv[j] - mu) * rstd * (1.f + a[j]) + c[j];
    }
    yr[i] = pack8(o);
  }
}

__global__ void adaln_ln_fwd_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ y,
                                    float* __restrict__ mean_out, float* __restrict__ rstd_out, ModPtr mod,
                                    const __nv_bfloat16* __restrict__ aff_w, const __nv_bfloat16* __restrict__ aff_b,
                                    int64_t rows, int D, int S, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + row * D);
  const int nv = D / 8;
  float s = 0.f;
  for (int i = lane; i < nv; i += 32) {
    float f[8];
    unpack8(xr[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += f[j];
  }
  const float mu = warp_sum(s) / D;
  float ss = 0.f;
  for (int i = lane; i < nv; i += 32) {
    float f[8];
    unpack8(xr[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float d = f[j] - mu;
      ss += d * d;
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / D + eps);
  if (lane == 0) {
    mean_out[row] = mu;
    rstd_out[row] = rstd;
  }
  const int64_t b = row / S;
  bf16x8* yr = reinterpret_cast<bf16x8*>(y + row * D);
  for (int i = lane; i < nv; i += 32) {
    float f[8], a[8], c[8], o[8];
    unpack8(xr[i], f);
    if (aff_w) {
      unpack8(reinterpret_cast<const bf16x8*>(aff_w)[i], a);
      unpack8(reinterpret_cast<const bf16x8*>(aff_b)[i], c);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (f[j] - mu) * rstd * a[j] + c[j];
    } else {
      unpack8(reinterpret_cast<const bf16x8*>(mod.scale + b * mod.stride)[i], a);
      unpack8(reinterpret_cast<const bf16x8*>(mod.shift + b * mod.stride)[i], c);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (f[j] - mu) * rstd * (1.f + a[j]) + c[j];
    }
    yr[i] = pack8(o);
  }
}

// dx for the modulated LayerNorm: dxhat = dy*(1+scale); dx = rstd*(dxhat - mean(dxhat) - xhat*mean(dxhat*xhat))
__global__ void adaln_ln_bwd_dx_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                       const float* __restrict__ mean, const float* __restrict__ rstd, ModPtr mod,
                                       __nv_bfloat16* __restrict__ dx, int64_t rows, int D, int S) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nv = D / 8;
  const int64_t b = row / S;
  const float mu = mean[row], rs = rstd[row];
  const bf16x8* xr = reinterpret_cast<const bf16x8*>(x + row * D);
  const bf16x8* gr = reinterpret_cast<const bf16x8*>(dy + row * D);
  const bf16x8* sc = reinterpret_cast<const bf16x8*>(mod.scale + b * mod.stride);
  float s1 = 0.f, s2 = 0.f;
  for (int i = lane; i < nv; i += 32) {
    float f[8], g[8], a[8];
    unpack8(xr[i], f);
    unpack8(gr[i], g);
    unpack8(sc[i], a);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float dxh = g[j] * (1.f + a[j]);
      s1 += dxh;
      s2 += dxh * (f[j] - mu) * rs;
    }
  }
  s1 = warp_sum(s1) / D;
  s2 = warp_sum(s2) / D;
  bf16x8* outr = reinterpret_cast<bf16x8*>(dx + row * D);
  for (int i = lane; i < nv; i += 32) {
    float f[8], g[8], a[8], o[8];
    unpack8(xr[i], f);
    unpack8(gr[i], g);
    unpack8(sc[i], a);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float xh = (f[j] - mu) * rs;
      o[j] = rs * (g[j] * (1.f + a[j]) - s1 - xh * s2);
    }
    outr[i] = pack8(o);
  }
}

// Column partial sums over a chunk of one sample's rows:
//   p_shift[b, c, :] = sum_rows dy ;  p_scale[b, c, :] = sum_rows dy * xhat
__global__ void adaln_ln_bwd_mod_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                        const float* __restrict__ mean, const float* __restrict__ rstd,
                                        float* __restrict__ p_shift, float* __restrict__ p_scale, int D, int S,
                                        int rows_per_chunk, int nchunk) {
  const int col8 = blockIdx.x * blockDim.x + threadIdx.x;  // index of an 8-column group
  const int b = blockIdx.z, c = blockIdx.y;
  if (col8 * 8 >= D) return;
  const int r0 = c * rows_per_chunk, r1 = min(S, r0 + rows_per_chunk);
  float a1[8] = {0}, a2[8] = {0};
  for (int r = r0; r < r1; ++r) {
    const int64_t row = (int64_t)b * S + r;
    float f[8], g[8];
    unpack8(reinterpret_cast<const bf16x8*>(x + row * D)[col8], f);
    unpack8(reinterpret_cast<const bf16x8*>(dy + row * D)[col8], g);
    const float mu = mean[row], rs = rstd[row];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      a1[j] += g[j];
      a2[j] += g[j] * (f[j] - mu) * rs;
    }
  }
  float* ps = p_shift + ((int64_t)b * nchunk + c) * D + col8 * 8;
  float* pc = p_scale + ((int64_t)b * nchunk + c) * D + col8 * 8;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ps[j] = a1[j];
    pc[j] = a2[j];
  }
}

__global__ void reduce_chunks_kernel(const float* __restrict__ p, float* __restrict__ out, int B, int nchunk, int D) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * D) return;
  const int b = i / D, d = i % D;
  float s = 0.f;
  for (int c = 0; c < nchunk; ++c) s += p[((int64_t)b * nchunk + c) * D + d];
  out[i] = s;
}

// ---------------------------------------------------------------- q/k RMSNorm + split
// Lane group of 8 lanes handles one (row, head): Dh = 64 -> 8 lanes x 8 elements.
template <int DH>
__global__ void qk_rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ wq,
                                      const __nv_bfloat16* __restrict__ wk, __nv_bfloat16* __restrict__ q,
                                      __nv_bfloat16* __restrict__ k, __nv_bfloat16* __restrict__ v,
                                      float* __restrict__ rstd_q, float* __restrict__ rstd_k,
                                      const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                                      int64_t rows, int H, int S_seg, int S_total, int seg_off, float eps,
                                      int64_t row_stride, int3 part_off) {
  constexpr int LPH = DH / 8;  // lanes per head
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t head_task = gid / LPH;
  const int sub = gid % LPH;
  const bool active = head_task < rows * H;
  const int64_t row = active ? head_task / H : 0;
  const int h = active ? (int)(head_task % H) : 0;
  const int64_t b = row / S_seg;
  const int s = (int)(row % S_seg) + seg_off;
  const int64_t out_off = (((int64_t)b * H + h) * S_total + s) * DH + sub * 8;
#pragma unroll
  for (int which = 0; which < 3; ++which) {
    const int poff = which == 0 ? part_off.x : which == 1 ? part_off.y : part_off.z;
    if (poff < 0) continue;
    float f[8] = {0};
    if (active) unpack8(*reinterpret_cast<const bf16x8*>(qkv + row * row_stride + poff + h * DH + sub * 8), f);
    if (which < 2) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
#pragma unroll
      for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rs = rsqrtf(ss / DH + eps);
      float w[8];
      unpack8(*reinterpret_cast<const bf16x8*>((which == 0 ? wq : wk) + sub * 8), w);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * rs * w[j];
      if (rope_cos) {
        // interleaved pairs (x0, x1) -> (x0 c - x1 s, x0 s + x1 c); table [S_total, DH/2]
        const float* cr = rope_cos + (int64_t)s * (DH / 2) + sub * 4;
        const float* sr = rope_sin + (int64_t)s * (DH / 2) + sub * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float x0 = f[2 * j], x1 = f[2 * j + 1];
          f[2 * j] = x0 * cr[j] - x1 * sr[j];
          f[2 * j + 1] = x0 * sr[j] + x1 * cr[j];
        }
      }
      if (active && sub == 0) (which == 0 ? rstd_q : rstd_k)[row * H + h] = rs;
    }
    if (active) *reinterpret_cast<bf16x8*>((which == 0 ? q : which == 1 ? k : v) + out_off) = pack8(f);
  }
}

template <int DH>
__global__ void qk_rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ wq,
                                      const __nv_bfloat16* __restrict__ wk, const __nv_bfloat16* __restrict__ dq,
                                      const __nv_bfloat16* __restrict__ dk, const __nv_bfloat16* __restrict__ dv,
                                      const float* __restrict__ rstd_q, const float* __restrict__ rstd_k,
                                      const float* __restrict__ rope_cos, const float* __restrict__ rope_sin,
                                      __nv_bfloat16* __restrict__ dqkv, float* __restrict__ dw_partial, int64_t rows,
                                      int H, int S_seg, int S_total, int seg_off, int64_t row_stride, int3 part_off) {
  // Thread (h, sub) owns 8 columns of head h for every row this block visits (rows strided by the
  // grid), so the weight-gradient partial sums stay in registers; one shared-memory pass at the end
  // folds the heads together.  blockDim.x = H * DH / 8 (rounded up to a warp multiple).
  constexpr int LPH = DH / 8;
  const int lanes = H * LPH;
  const bool active = threadIdx.x < lanes;
  const int h = active ? threadIdx.x / LPH : 0;
  const int sub = threadIdx.x % LPH;
  float wqv[8] = {0}, wkv[8] = {0};
  if (wq && part_off.x >= 0) unpack8(*reinterpret_cast<const bf16x8*>(wq + sub * 8), wqv);
  if (wk && part_off.y >= 0) unpack8(*reinterpret_cast<const bf16x8*>(wk + sub * 8), wkv);
  float dwacc[2][8] = {{0}};
  // every thread runs the same trip count (the row loop is block-uniform) so the width-LPH shuffles
  // below always see full warps; threads past H * LPH only skip their loads and stores
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
    const int64_t b = row / S_seg;
    const int s = (int)(row % S_seg) + seg_off;
    const int64_t in_off = (((int64_t)b * H + h) * S_total + s) * DH + sub * 8;
#pragma unroll
    for (int which = 0; which < 3; ++which) {
      const int poff = which == 0 ? part_off.x : which == 1 ? part_off.y : part_off.z;
      if (poff < 0) continue;
      float g[8] = {0};
      if (active) unpack8(*reinterpret_cast<const bf16x8*>((which == 0 ? dq : which == 1 ? dk : dv) + in_off), g);
      float o[8];
      if (which < 2) {
        if (rope_cos && active) {  // transpose of the rotation
          const float* cr = rope_cos + (int64_t)s * (DH / 2) + sub * 4;
          const float* sr = rope_sin + (int64_t)s * (DH / 2) + sub * 4;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float g0 = g[2 * j], g1 = g[2 * j + 1];
            g[2 * j] = g0 * cr[j] + g1 * sr[j];
            g[2 * j + 1] = -g0 * sr[j] + g1 * cr[j];
          }
        }
        float x[8] = {0};
        if (active) unpack8(*reinterpret_cast<const bf16x8*>(qkv + row * row_stride + poff + h * DH + sub * 8), x);
        const float* w = which == 0 ? wqv : wkv;
        const float rs = active ? (which == 0 ? rstd_q : rstd_k)[row * H + h] : 0.f;
        float dot = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = x[j] * rs;
          dot += g[j] * w[j] * xh;
          dwacc[which][j] += g[j] * xh;
        }
#pragma unroll
        for (int off = LPH / 2; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off, LPH);
        dot *= 1.f / DH;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rs * (g[j] * w[j] - x[j] * rs * dot);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = g[j];
      }
      if (active) *reinterpret_cast<bf16x8*>(dqkv + row * row_stride + poff + h * DH + sub * 8) = pack8(o);
    }
  }
  // fold the heads: red[lane][16] -> dw_partial[block][which][DH]
  extern __shared__ float red[];
  for (int i = 0; i < 16; ++i) red[threadIdx.x * 16 + i] = active ? dwacc[i >> 3][i & 7] : 0.f;
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * DH; i += blockDim.x) {
    const int which = i / DH, col = i % DH, sb = col / 8, j = col % 8;
    float s = 0.f;
    for (int hh = 0; hh < H; ++hh) s += red[(hh * LPH + sb) * 16 + which * 8 + j];
    dw_partial[(int64_t)blockIdx.x * 2 * DH + i] = s;
  }
}

}  // namespace

static ModPtr make_mod(torch::Tensor mod, int64_t shift_off, int64_t scale_off) {
  ModPtr m;
  auto* base = reinterpret_cast<const __nv_bfloat16*>(mod.data_ptr<at::BFloat16>());
  m.shift = base + shift_off;
  m.scale = base + scale_off;
  m.stride = mod.size(-1);
  return m;
}

std::vector<torch::Tensor> adaln_ln_fwd(torch::Tensor x, c10::optional<torch::Tensor> mod, int64_t shift_off,
                                        int64_t scale_off, c10::optional<torch::Tensor> w,
                                        c10::optional<torch::Tensor> bias, int64_t S, double eps) {
  VO_CHECK_INPUT(x);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16, "bf16 activations required");
  c10::cuda::CUDAGuard g(x.device());
  const int D = x.size(-1);
  TORCH_CHECK(D % 8 == 0, "hidden size must be a multiple of 8");
  const int64_t rows = x.numel() / D;
  auto y = torch::empty_like(x);
  auto fo = x.options().dtype(torch::kFloat32);
  auto mean = torch::empty({rows}, fo), rstd = torch::empty({rows}, fo);
  ModPtr m{nullptr, nullptr, 0};
  const __nv_bfloat16 *aw = nullptr, *ab = nullptr;
  if (mod.has_value() && mod->defined()) {
    VO_CHECK_INPUT((*mod));
    m = make_mod(*mod, shift_off, scale_off);
  } else {
    TORCH_CHECK(w.has_value() && bias.has_value(), "need either modulation or affine weights");
    aw = reinterpret_cast<const __nv_bfloat16*>(w->data_ptr<at::BFloat16>());
    ab = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr<at::BFloat16>());
  }
  const int wpb = 8;
  const unsigned grid = (unsigned)((rows + wpb - 1) / wpb);
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr<at::BFloat16>());
  switch (D) {  // register-resident rows for the hidden sizes of the model zoo (1536 / 3072 / 2048)
    case 1536:
      adaln_ln_fwd_reg_kernel<6><<<grid, wpb * 32, 0, stream()>>>(xp, yp, mean.data_ptr<float>(),
                                                                   rstd.data_ptr<float>(), m, aw, ab, rows, (int)S,
                                                                   (float)eps);
      break;
    case 2048:
      adaln_ln_fwd_reg_kernel<8><<<grid, wpb * 32, 0, stream()>>>(xp, yp, mean.data_ptr<float>(),
                                                                   rstd.data_ptr<float>(), m, aw, ab, rows, (int)S,
                                                                   (float)eps);
      break;
    case 3072:
      adaln_ln_fwd_reg_kernel<12><<<grid, wpb * 32, 0, stream()>>>(xp, yp, mean.data_ptr<float>(),
                                                                    rstd.data_ptr<float>(), m, aw, ab, rows, (int)S,
                                                                    (float)eps);
      break;
    default:
      adaln_ln_fwd_kernel<<<grid, wpb * 32, 0, stream()>>>(xp, yp, mean.data_ptr<float>(), rstd.data_ptr<float>(), m,
                                                           aw, ab, rows, D, (int)S, (float)eps);
  }
  vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {y, mean, rstd};
}

// returns dx, d_shift [B, D] (fp32), d_scale [B, D] (fp32)
std::vector<torch::Tensor> adaln_ln_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor mean, torch::Tensor rstd,
                                        torch::Tensor mod, int64_t shift_off, int64_t scale_off, int64_t S) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(x);
  c10::cuda::CUDAGuard g(x.device());
  const int D = x.size(-1);
  const int64_t rows = x.numel() / D;
  const int B = rows / S;
  auto dx = torch::empty_like(x);
  ModPtr m = make_mod(mod, shift_off, scale_off);
  const int wpb = 8;
  auto st = stream();
  adaln_ln_bwd_dx_kernel<<<(rows + wpb - 1) / wpb, wpb * 32, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()), mean.data_ptr<float>(),
      rstd.data_ptr<float>(), m, reinterpret_cast<__nv_bfloat16*>(dx.data_ptr<at::BFloat16>()), rows, D, (int)S); vo::count_launch();
  // column reductions
  const int cols8 = D / 8;
  const int tpb = std::min(128, cols8);
  const int gx = (cols8 + tpb - 1) / tpb;
  int nchunk = std::max(1, std::min<int>((int)((S + 31) / 32), (2 * num_sms() + B * gx - 1) / (B * gx)));
  int rpc = (int)((S + nchunk - 1) / nchunk);
  nchunk = (int)((S + rpc - 1) / rpc);
  auto fo = x.options().dtype(torch::kFloat32);
  auto ps = torch::empty({B, nchunk, D}, fo), pc = torch::empty({B, nchunk, D}, fo);
  adaln_ln_bwd_mod_kernel<<<dim3(gx, nchunk, B), tpb, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()), mean.data_ptr<float>(),
      rstd.data_ptr<float>(), ps.data_ptr<float>(), pc.data_ptr<float>(), D, (int)S, rpc, nchunk); vo::count_launch();
  auto dshift = torch::empty({B, D}, fo), dscale = torch::empty({B, D}, fo);
  const int64_t n = (int64_t)B * D;
  reduce_chunks_kernel<<<(n + 255) / 256, 256, 0, st>>>(ps.data_ptr<float>(), dshift.data_ptr<float>(), B, nchunk, D); vo::count_launch();
  reduce_chunks_kernel<<<(n + 255) / 256, 256, 0, st>>>(pc.data_ptr<float>(), dscale.data_ptr<float>(), B, nchunk, D); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {dx, dshift, dscale};
}

// qkv [rows, 3*H*Dh] -> writes q/k/v [B, H, S_total, Dh] at seq offset; returns rstd_q, rstd_k [rows, H]
static torch::Tensor first_defined(std::initializer_list<torch::Tensor> ts) {
  for (auto& t : ts)
    if (t.defined()) return t;
  TORCH_CHECK(false, "no output buffer given");
}

static __nv_bfloat16* bptr(const torch::Tensor& t) {
  return t.defined() ? reinterpret_cast<__nv_bfloat16*>(t.data_ptr<at::BFloat16>()) : nullptr;
}

// Parts: q at column part_off[0], k at part_off[1], v at part_off[2] of each qkv row (-1 = absent).
std::vector<torch::Tensor> qk_rmsnorm_fwd(torch::Tensor qkv, torch::Tensor wq, torch::Tensor wk,
                                          c10::optional<torch::Tensor> q_, c10::optional<torch::Tensor> k_,
                                          c10::optional<torch::Tensor> v_, int64_t S_seg, int64_t seg_off,
                                          c10::optional<torch::Tensor> rope_cos, c10::optional<torch::Tensor> rope_sin,
                                          double eps, std::vector<int64_t> part_off) {
  VO_CHECK_INPUT(qkv);
  c10::cuda::CUDAGuard g(qkv.device());
  // absent destinations (a q-only or k/v-only projection) are undefined tensors: the kernel skips them
  const torch::Tensor q = q_.value_or(torch::Tensor()), k = k_.value_or(torch::Tensor()),
                      v = v_.value_or(torch::Tensor());
  auto ref = first_defined({q, k, v});
  const int H = ref.size(1), S_total = ref.size(2), DH = ref.size(3);
  const int3 po = make_int3((int)part_off[0], (int)part_off[1], (int)part_off[2]);
  TORCH_CHECK(DH == 32 || DH == 64 || DH == 128, "head_dim must be 32, 64 or 128");
  const int64_t rows = qkv.size(0);
  auto fo = qkv.options().dtype(torch::kFloat32);
  auto rq = torch::empty({rows, H}, fo), rk = torch::empty({rows, H}, fo);
  const float* rc = (rope_cos.has_value() && rope_cos->defined()) ? rope_cos->data_ptr<float>() : nullptr;
  const float* rsn = (rope_sin.has_value() && rope_sin->defined()) ? rope_sin->data_ptr<float>() : nullptr;
  const int64_t threads = rows * H * (DH / 8);
  const int64_t rs_ = qkv.size(1);
  if (DH == 32)
    qk_rmsnorm_fwd_kernel<32><<<(threads + 255) / 256, 256, 0, stream()>>>(
        bptr(qkv), bptr(wq), bptr(wk), bptr(q), bptr(k), bptr(v), rq.data_ptr<float>(), rk.data_ptr<float>(), rc, rsn,
        rows, H, (int)S_seg, S_total, (int)seg_off, (float)eps, rs_, po);
  else if (DH == 64)
    qk_rmsnorm_fwd_kernel<64><<<(threads + 255) / 256, 256, 0, stream()>>>(
        bptr(qkv), bptr(wq), bptr(wk), bptr(q), bptr(k), bptr(v), rq.data_ptr<float>(), rk.data_ptr<float>(), rc, rsn,
        rows, H, (int)S_seg, S_total, (int)seg_off, (float)eps, rs_, po);
  else
    qk_rmsnorm_fwd_kernel<128><<<(threads + 255) / 256, 256, 0, stream()>>>(
        bptr(qkv), bptr(wq), bptr(wk), bptr(q), bptr(k), bptr(v), rq.data_ptr<float>(), rk.data_ptr<float>(), rc, rsn,
        rows, H, (int)S_seg, S_total, (int)seg_off, (float)eps, rs_, po); vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {rq, rk};
}

// returns dqkv [rows, 3D] (bf16), dwq [Dh] fp32, dwk [Dh] fp32
std::vector<torch::Tensor> qk_rmsnorm_bwd(torch::Tensor qkv, torch::Tensor wq, torch::Tensor wk,
                                          c10::optional<torch::Tensor> dq_, c10::optional<torch::Tensor> dk_,
                                          c10::optional<torch::Tensor> dv_, torch::Tensor rq, torch::Tensor rk,
                                          int64_t S_seg, int64_t seg_off, c10::optional<torch::Tensor> rope_cos,
                                          c10::optional<torch::Tensor> rope_sin, std::vector<int64_t> part_off) {
  c10::cuda::CUDAGuard g(qkv.device());
  const torch::Tensor dq = dq_.value_or(torch::Tensor()), dk = dk_.value_or(torch::Tensor()),
                      dv = dv_.value_or(torch::Tensor());
  auto ref = first_defined({dq, dk, dv});
  const int H = ref.size(1), S_total = ref.size(2), DH = ref.size(3);
  const int3 po = make_int3((int)part_off[0], (int)part_off[1], (int)part_off[2]);
  const int64_t rows = qkv.size(0);
  auto dqkv = torch::empty_like(qkv);
  const int lanes = H * (DH / 8);
  TORCH_CHECK(lanes <= 1024, "too many heads for the q/k-norm backward");
  const int threads = (lanes + 31) / 32 * 32;
  const int nblk = (int)std::max<int64_t>(1, std::min<int64_t>(rows, 8LL * num_sms()));
  const size_t smem = (size_t)threads * 16 * sizeof(float);
  auto part = torch::empty({nblk, 2, DH}, qkv.options().dtype(torch::kFloat32));
  const float* rc = (rope_cos.has_value() && rope_cos->defined()) ? rope_cos->data_ptr<float>() : nullptr;
  const float* rsn = (rope_sin.has_value() && rope_sin->defined()) ? rope_sin->data_ptr<float>() : nullptr;
  const int64_t rs_ = qkv.size(1);
#define VO_QKBWD(DHV)                                                                                              \
  qk_rmsnorm_bwd_kernel<DHV><<<nblk, threads, smem, stream()>>>(                                                   \
      bptr(qkv), bptr(wq), bptr(wk), bptr(dq), bptr(dk), bptr(dv), rq.data_ptr<float>(), rk.data_ptr<float>(), rc, \
      rsn, bptr(dqkv), part.data_ptr<float>(), rows, H, (int)S_seg, S_total, (int)seg_off, rs_, po)
  if (DH == 32)
    VO_QKBWD(32);
  else if (DH == 64)
    VO_QKBWD(64);
  else
    VO_QKBWD(128);
#undef VO_QKBWD
  vo::count_launch();
  VO_CUDA_OK(cudaGetLastError());
  auto dw = part.sum(0);  // [2, DH]
  return {dqkv, dw[0], dw[1]};
}

}  // namespace vo
