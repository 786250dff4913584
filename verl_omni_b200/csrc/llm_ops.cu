// Row kernels of the MoE language model (Qwen3-Omni-thinker-shaped): RMSNorm, SwiGLU, router top-k and
// per-head q/k RMSNorm + rotate-half RoPE.  All memory-bound: one pass over the data, fp32 math, bf16 I/O,
// 16-byte vectors.
#include "common.cuh"

namespace vo {
namespace {

// ------------------------------------------------------------------------------------------ RMSNorm
// y = x * rstd * w, rstd = 1 / sqrt(mean(x^2) + eps); one CTA per row, D / 8 vectors over 256 threads.
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const bf16x8* __restrict__ x, const bf16x8* __restrict__ w,
                                                          bf16x8* __restrict__ y, float* __restrict__ rstd, int vecs,
                                                          float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const bf16x8* xr = x + row * vecs;
  float ss = 0.f;
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) {
    float f[8];
    unpack8(xr[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
  ss = block_sum(ss, red);
  const float r = rsqrtf(ss / (vecs * 8) + eps);
  if (threadIdx.x == 0) rstd[row] = r;
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) {
    float f[8], g[8];
    unpack8(xr[i], f);
    unpack8(w[i], g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
    y[row * vecs + i] = pack8(f);
  }
}

// Warp-per-row variant for D = 256 * NV (NV in 4, 6, 8): the row stays in registers as packed bf16 vectors (NV per
// lane), read from memory once and unpacked per pass; eight rows per 256-thread CTA keep many rows' loads in
// flight (the CTA-per-row form above waits on a block-wide reduction between its two passes).
template <int NV>
__global__ void __launch_bounds__(256) rmsnorm_fwd_warp_kernel(const bf16x8* __restrict__ x,
                                                               const bf16x8* __restrict__ w, bf16x8* __restrict__ y,
                                                               float* __restrict__ rstd, int64_t rows, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bf16x8* xr = x + row * (NV * 32);
  bf16x8 raw[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) raw[v] = xr[v * 32 + lane];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float f[8];
    unpack8(raw[v], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
  const float r = rsqrtf(warp_sum(ss) * (1.f / (NV * 256)) + eps);
  if (lane == 0) rstd[row] = r;
  bf16x8* yr = y + row * (NV * 32);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float f[8], g[8];
    unpack8(raw[v], f);
    unpack8(w[v * 32 + lane], g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
    yr[v * 32 + lane] = pack8(f);
  }
}

// dx = rstd * (w dy - x rstd^2 mean(x w dy)); dw partials per CTA row-chunk: dw[c] = sum_rows dy x rstd
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const bf16x8* __restrict__ dy, const bf16x8* __restrict__ x,
                                                          const bf16x8* __restrict__ w, const float* __restrict__ rstd,
                                                          bf16x8* __restrict__ dx, float* __restrict__ dw_part,
                                                          int64_t rows, int vecs, int rows_per_cta) {
  __shared__ float red[32];
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r1 = min(rows, r0 + rows_per_cta);
  // this thread's dw accumulators: vectors i = threadIdx.x + k * blockDim.x (at most 4 for D <= 8192)
  float acc[4][8];
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[k][j] = 0.f;
  for (int64_t row = r0; row < r1; ++row) {
    const float r = rstd[row];
    float dot = 0.f;
    for (int i = threadIdx.x; i < vecs; i += blockDim.x) {
      float a[8], b[8], g[8];
      unpack8(dy[row * vecs + i], a);
      unpack8(x[row * vecs + i], b);
      unpack8(w[i], g);
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += a[j] * g[j] * b[j];
    }
    dot = block_sum(dot, red);
    const float c = dot * r * r / (vecs * 8);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = threadIdx.x + k * blockDim.x;
      if (i < vecs) {
        float a[8], b[8], g[8], o[8];
        unpack8(dy[row * vecs + i], a);
        unpack8(x[row * vecs + i], b);
        unpack8(w[i], g);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          o[j] = r * (a[j] * g[j] - b[j] * c);
          acc[k][j] += a[j] * b[j] * r;
        }
        dx[row * vecs + i] = pack8(o);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = threadIdx.x + k * blockDim.x;
    if (i < vecs)
#pragma unroll
      for (int j = 0; j < 8; ++j) dw_part[(int64_t)blockIdx.x * vecs * 8 + i * 8 + j] = acc[k][j];
  }
}

__global__ void sum_rows_kernel(const float* __restrict__ part, int n_parts, int D, float* __restrict__ out,
                                int accumulate) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  float s = 0.f;
  for (int p = 0; p < n_parts; ++p) s += part[(int64_t)p * D + c];
  out[c] = accumulate ? out[c] + s : s;
}

// ------------------------------------------------------------------------------------------ SwiGLU
__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

// gu [M, 2F] (gate | up) -> a [M, F] = silu(gate) * up
__global__ void swiglu_fwd_kernel(const bf16x8* __restrict__ gu, bf16x8* __restrict__ a, int64_t M, int fv) {
  const int64_t n = M * fv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / fv;
    const int c = (int)(i - m * fv);
    float g[8], u[8];
    unpack8(gu[m * 2 * fv + c], g);
    unpack8(gu[m * 2 * fv + fv + c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = silu_f(g[j]) * u[j];
    a[i] = pack8(g);
  }
}

// da [M, F], gu [M, 2F] -> dgu [M, 2F] = (da * up * silu'(gate) | da * silu(gate))
__global__ void swiglu_bwd_kernel(const bf16x8* __restrict__ da, const bf16x8* __restrict__ gu,
                                  bf16x8* __restrict__ dgu, int64_t M, int fv) {
  const int64_t n = M * fv;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t m = i / fv;
    const int c = (int)(i - m * fv);
    float d[8], g[8], u[8], dg[8], du[8];
    unpack8(da[i], d);
    unpack8(gu[m * 2 * fv + c], g);
    unpack8(gu[m * 2 * fv + fv + c], u);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float sg = 1.f / (1.f + __expf(-g[j]));
      dg[j] = d[j] * u[j] * sg * (1.f + g[j] * (1.f - sg));
      du[j] = d[j] * g[j] * sg;
    }
    dgu[m * 2 * fv + c] = pack8(dg);
    dgu[m * 2 * fv + fv + c] = pack8(du);
  }
}

// ------------------------------------------------------------------------------------------ router
// One warp per token: softmax over E <= 256 expert logits (fp32), then K rounds of warp arg-max; gates are
// the selected probabilities renormalised to sum 1 (ties go to the lower expert id).
template <int PER>
__global__ void router_topk_kernel(const float* __restrict__ logits, int64_t T, int E, int K,
                                   float* __restrict__ probs, float* __restrict__ gates, int64_t* __restrict__ idx) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  float v[PER];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    v[i] = e < E ? logits[t * E + e] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  mx = warp_max(mx);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    v[i] = (lane + 32 * i) < E ? __expf(v[i] - mx) : 0.f;
    s += v[i];
  }
  s = warp_sum(s);
  const float inv = 1.f / s;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    v[i] *= inv;
    if (lane + 32 * i < E) probs[t * E + lane + 32 * i] = v[i];
  }
  float tot = 0.f, sel_v = 0.f;
  int sel_e = 0;
  for (int k = 0; k < K; ++k) {
    float bv = -1.f;
    int be = 1 << 30;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (v[i] > bv) bv = v[i], be = lane + 32 * i;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) bv = ov, be = oe;
    }
    if (lane == k) sel_v = bv, sel_e = be;
    tot += bv;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) v[i] = -2.f;  // taken
  }
  if (lane < K) {
    gates[t * K + lane] = sel_v / tot;
    idx[t * K + lane] = sel_e;
  }
}

// ------------------------------------------------------------------------------------------ q/k norm + RoPE
// x [B, S, H, Dh] bf16 (a column slice of a projection output, row stride ld elements) -> y [B, H, S, Dh]
// = rotate_half_rope(rmsnorm(x) * w); cos/sin [S, Dh/2] fp32 tables for positions pos0 + s.  One warp per
// (token, head), Dh <= 256.
__global__ void head_rmsnorm_rope_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld, const __nv_bfloat16* __restrict__ w,
                                         const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                         __nv_bfloat16* __restrict__ y, int B, int S, int H, int Dh, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= (int64_t)B * S * H) return;
  const int h = (int)(item % H);
  const int64_t bs = item / H;
  const int s = (int)(bs % S);
  const int b = (int)(bs / S);
  const __nv_bfloat16* xr = x + bs * ld + (int64_t)h * Dh;
  const int half = Dh / 2;
  // lane holds pairs (d, d + half) for d = lane, lane + 32, ...
  float a[4], c[4];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    a[k] = d < half ? bf2f(xr[d]) : 0.f;
    c[k] = d < half ? bf2f(xr[d + half]) : 0.f;
    ss += a[k] * a[k] + c[k] * c[k];
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / Dh + eps);
  __nv_bfloat16* yr = y + (((int64_t)b * H + h) * S + s) * Dh;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    if (d < half) {
      const float x1 = a[k] * r * bf2f(w[d]), x2 = c[k] * r * bf2f(w[d + half]);
      const float co = cos_t[(int64_t)s * half + d], si = sin_t[(int64_t)s * half + d];
      yr[d] = f2bf(x1 * co - x2 * si);
      yr[d + half] = f2bf(x1 * si + x2 * co);
    }
  }
}

// Vectorised form for Dh in {64, 128, 256}: a head's Dh elements are Dh / 8 16-byte vectors held by LPH = Dh / 8
// consecutive lanes (32 / LPH heads per warp).  Lanes [0, LPH/2) of a head hold the first half (d < Dh/2), lanes
// [LPH/2, LPH) the second; the rotate-half partner of lane p is lane p ^ (LPH/2), one shuffle away.  Requires
// 16-byte aligned rows (ld, the column offset and the base a multiple of 8 elements).
template <int DH>
__global__ void __launch_bounds__(256) head_rmsnorm_rope_vec_kernel(const __nv_bfloat16* __restrict__ x, int64_t ld,
                                                                    const __nv_bfloat16* __restrict__ w,
                                                                    const float* __restrict__ cos_t,
                                                                    const float* __restrict__ sin_t,
                                                                    __nv_bfloat16* __restrict__ y, int B, int S, int H,
                                                                    float eps) {
  constexpr int LPH = DH / 8, HALF = DH / 2, PART = LPH / 2;
  const int lane = threadIdx.x & 31;
  const int p = lane % LPH;  // vector index within the head
  const int64_t item = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * (32 / LPH) + lane / LPH;
  const bool live = item < (int64_t)B * S * H;
  const uint32_t it = live ? (uint32_t)item : 0u;  // the host launches this form for B S H < 2^31 only
  const int h = (int)(it % (uint32_t)H);
  const uint32_t bs32 = it / (uint32_t)H;
  const int s = (int)(bs32 % (uint32_t)S);
  const int b = (int)(bs32 / (uint32_t)S);
  const int64_t bs = bs32;
  float f[8];
  unpack8(*reinterpret_cast<const bf16x8*>(x + bs * ld + (int64_t)h * DH + p * 8), f);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);  // within the head's lanes
  const float r = rsqrtf(ss * (1.f / DH) + eps);
  float g[8];
  unpack8(reinterpret_cast<const bf16x8*>(w)[p], g);
#pragma unroll
  for (int j = 0; j < 8; ++j) f[j] *= r * g[j];
  float o2[8];  // the partner's normalised values: x2 for a first-half lane, x1 for a second-half lane
#pragma unroll
  for (int j = 0; j < 8; ++j) o2[j] = __shfl_xor_sync(0xffffffffu, f[j], PART);
  const bool first = p < PART;
  const int d0 = (first ? p : p - PART) * 8;  // index into the half-width tables
  const float4* cp = reinterpret_cast<const float4*>(cos_t + (int64_t)s * HALF + d0);
  const float4* sp = reinterpret_cast<const float4*>(sin_t + (int64_t)s * HALF + d0);
  const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
  const float co[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
  const float si[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
  float out[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) out[j] = first ? f[j] * co[j] - o2[j] * si[j] : o2[j] * si[j] + f[j] * co[j];
  if (live) *reinterpret_cast<bf16x8*>(y + (((int64_t)b * H + h) * S + s) * DH + p * 8) = pack8(out);
}

// backward of the above: dy [B, H, S, Dh] -> dx [B, S, H, Dh] (contiguous), dw partial sums per item block
__global__ void head_rmsnorm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                                             int64_t ld, const __nv_bfloat16* __restrict__ w,
                                             const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                                             __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, int B, int S,
                                             int H, int Dh, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (item >= (int64_t)B * S * H) return;
  const int h = (int)(item % H);
  const int64_t bs = item / H;
  const int s = (int)(bs % S);
  const int b = (int)(bs / S);
  const __nv_bfloat16* xr = x + bs * ld + (int64_t)h * Dh;
  const __nv_bfloat16* dyr = dy + (((int64_t)b * H + h) * S + s) * Dh;
  const int half = Dh / 2;
  float a[4], c[4], g1[4], g2[4];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    a[k] = d < half ? bf2f(xr[d]) : 0.f;
    c[k] = d < half ? bf2f(xr[d + half]) : 0.f;
    ss += a[k] * a[k] + c[k] * c[k];
    if (d < half) {
      // un-rotate the gradient: d(x1), d(x2) of the normalised, scaled values
      const float co = cos_t[(int64_t)s * half + d], si = sin_t[(int64_t)s * half + d];
      const float d1 = bf2f(dyr[d]), d2 = bf2f(dyr[d + half]);
      g1[k] = d1 * co + d2 * si;
      g2[k] = -d1 * si + d2 * co;
    } else {
      g1[k] = g2[k] = 0.f;
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / Dh + eps);
  // n = x r; y' = n w; dn = g w; dx = r (dn - n mean(dn n))
  float dot = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    if (d < half) dot += g1[k] * bf2f(w[d]) * a[k] * r + g2[k] * bf2f(w[d + half]) * c[k] * r;
  }
  dot = warp_sum(dot) / Dh;
  __nv_bfloat16* dxr = dx + (bs * H + h) * Dh;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int d = lane + 32 * k;
    if (d < half) {
      const float n1 = a[k] * r, n2 = c[k] * r;
      dxr[d] = f2bf(r * (g1[k] * bf2f(w[d]) - n1 * dot));
      dxr[d + half] = f2bf(r * (g2[k] * bf2f(w[d + half]) - n2 * dot));
      atomicAdd(dw + d, g1[k] * n1);
      atomicAdd(dw + d + half, g2[k] * n2);
    }
  }
}

// Vectorised backward for Dh in {64, 128, 256} (same lane layout as the forward vector kernel): each warp walks
// groups of 32 / LPH heads with a grid stride, un-rotates the gradient with the partner lane's values, and keeps
// the weight-gradient partial sums of its 8 columns in registers; one atomic add per column per warp at the end
// (the per-element form above adds B S H Dh times into Dh addresses).
template <int DH>
__global__ void __launch_bounds__(256) head_rmsnorm_rope_bwd_vec_kernel(
    const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x, int64_t ld,
    const __nv_bfloat16* __restrict__ w, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
    __nv_bfloat16* __restrict__ dx, float* __restrict__ dw, int B, int S, int H, float eps) {
  constexpr int LPH = DH / 8, HALF = DH / 2, PART = LPH / 2, HPW = 32 / LPH;
  const int lane = threadIdx.x & 31;
  const int p = lane % LPH;
  const bool first = p < PART;
  const int d0 = (first ? p : p - PART) * 8;
  const uint32_t items = (uint32_t)B * S * H;
  const uint32_t groups = (items + HPW - 1) / HPW;
  const uint32_t warps = gridDim.x * (blockDim.x >> 5);
  float wv[8], acc[8];
  unpack8(reinterpret_cast<const bf16x8*>(w)[p], wv);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  // one group ahead: the next group's x / dy vectors are loaded before this group's math, so two groups'
  // loads are in flight per warp
  auto locate = [&](uint32_t grp, bool& live, int& h, uint32_t& bs, int& s, int& b) {
    const uint32_t item = grp * HPW + lane / LPH;
    live = item < items;  // uniform per head: its lanes skip together, shuffles stay in their head
    const uint32_t it = live ? item : 0u;
    h = (int)(it % (uint32_t)H);
    bs = it / (uint32_t)H;
    s = (int)(bs % (uint32_t)S);
    b = (int)(bs / (uint32_t)S);
  };
  uint32_t grp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  bool nlive;
  int nh, ns, nb;
  uint32_t nbs;
  bf16x8 xn, dn;
  if (grp < groups) {
    locate(grp, nlive, nh, nbs, ns, nb);
    xn = *reinterpret_cast<const bf16x8*>(x + (int64_t)nbs * ld + (int64_t)nh * DH + p * 8);
    dn = *reinterpret_cast<const bf16x8*>(dy + (((int64_t)nb * H + nh) * S + ns) * DH + p * 8);
  }
  for (; grp < groups; grp += warps) {
    const bool live = nlive;
    const int h = nh, s = ns;
    const uint32_t bs = nbs;
    float xv[8], gv[8], gp[8];
    unpack8(xn, xv);
    unpack8(dn, gv);
    if (grp + warps < groups) {
      locate(grp + warps, nlive, nh, nbs, ns, nb);
      xn = *reinterpret_cast<const bf16x8*>(x + (int64_t)nbs * ld + (int64_t)nh * DH + p * 8);
      dn = *reinterpret_cast<const bf16x8*>(dy + (((int64_t)nb * H + nh) * S + ns) * DH + p * 8);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) gp[j] = __shfl_xor_sync(0xffffffffu, gv[j], PART);
    const float4* cp = reinterpret_cast<const float4*>(cos_t + (int64_t)s * HALF + d0);
    const float4* sp = reinterpret_cast<const float4*>(sin_t + (int64_t)s * HALF + d0);
    const float4 c0 = cp[0], c1 = cp[1], s0 = sp[0], s1 = sp[1];
    const float co[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float si[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // gradient w.r.t. the normalised, scaled value of this lane's element (rotation undone):
      // first half  g1 = d1 cos + d2 sin;  second half g2 = -d1 sin + d2 cos
      gv[j] = first ? gv[j] * co[j] + gp[j] * si[j] : -gp[j] * si[j] + gv[j] * co[j];
      ss += xv[j] * xv[j];
    }
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss * (1.f / DH) + eps);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) dot += gv[j] * wv[j] * xv[j] * r;
#pragma unroll
    for (int o = LPH / 2; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    dot *= 1.f / DH;
    float out[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float n = xv[j] * r;
      out[j] = r * (gv[j] * wv[j] - n * dot);
      if (live) acc[j] += gv[j] * n;
    }
    if (live) *reinterpret_cast<bf16x8*>(dx + ((int64_t)bs * H + h) * DH + p * 8) = pack8(out);
  }
  // lanes holding the same columns (one per head of the warp) combine, then one lane adds them
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int o = LPH; o < 32; o <<= 1) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
  if (lane < LPH) {
#pragma unroll
    for (int j = 0; j < 8; ++j) atomicAdd(dw + p * 8 + j, acc[j]);
  }
}

inline int grid_for(int64_t n, int threads) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 16LL * num_sms()));
}

}  // namespace

std::vector<torch::Tensor> rms_norm_fwd(torch::Tensor x, torch::Tensor w, double eps) {
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(w);
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16, "bf16 RMSNorm");
  const int64_t D = x.size(-1), rows = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && w.numel() == D, "RMSNorm width a multiple of 8");
  c10::cuda::CUDAGuard g(x.device());
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  if (rows == 0) return {y, rstd};
  const auto* xp = reinterpret_cast<const bf16x8*>(x.data_ptr<at::BFloat16>());
  const auto* wp = reinterpret_cast<const bf16x8*>(w.data_ptr<at::BFloat16>());
  auto* yp = reinterpret_cast<bf16x8*>(y.data_ptr<at::BFloat16>());
  const unsigned wgrid = (unsigned)((rows + 7) / 8);
  switch (D) {  // warp per row for the model zoo's widths; a CTA per row otherwise
#define VO_RMS_WARP(NV) \
  case NV * 256:        \
    rmsnorm_fwd_warp_kernel<NV><<<wgrid, 256, 0, stream()>>>(xp, wp, yp, rstd.data_ptr<float>(), rows, (float)eps); \
    break;
    VO_RMS_WARP(4) VO_RMS_WARP(6) VO_RMS_WARP(8)
#undef VO_RMS_WARP
    default:
      rmsnorm_fwd_kernel<<<(unsigned)rows, 256, 0, stream()>>>(xp, wp, yp, rstd.data_ptr<float>(), (int)(D / 8),
                                                               (float)eps);
  }
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {y, rstd};
}

// returns dx; dw (fp32 [D]) is written, or added into when accumulate
torch::Tensor rms_norm_bwd(torch::Tensor dy, torch::Tensor x, torch::Tensor w, torch::Tensor rstd, torch::Tensor dw,
                           bool accumulate) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_INPUT(x);
  VO_CHECK_INPUT(w);
  VO_CHECK_INPUT(rstd);
  VO_CHECK_INPUT(dw);
  const int64_t D = x.size(-1), rows = x.numel() / D;
  TORCH_CHECK(D % 8 == 0 && D <= 8 * 4 * 256 && dw.scalar_type() == torch::kFloat32 && dw.numel() == D,
              "RMSNorm backward: width <= 8192, fp32 dw");
  c10::cuda::CUDAGuard g(x.device());
  auto dx = torch::empty_like(x);
  if (rows == 0) {
    if (!accumulate) dw.zero_();
    return dx;
  }
  const int rows_per_cta = (int)std::max<int64_t>(1, (rows + 4 * num_sms() - 1) / (4 * num_sms()));
  const int ctas = (int)((rows + rows_per_cta - 1) / rows_per_cta);
  auto part = torch::empty({ctas, D}, x.options().dtype(torch::kFloat32));
  rmsnorm_bwd_kernel<<<ctas, 256, 0, stream()>>>(
      reinterpret_cast<const bf16x8*>(dy.data_ptr<at::BFloat16>()), reinterpret_cast<const bf16x8*>(x.data_ptr<at::BFloat16>()),
      reinterpret_cast<const bf16x8*>(w.data_ptr<at::BFloat16>()), rstd.data_ptr<float>(),
      reinterpret_cast<bf16x8*>(dx.data_ptr<at::BFloat16>()), part.data_ptr<float>(), rows, (int)(D / 8), rows_per_cta);
  sum_rows_kernel<<<(int)((D + 255) / 256), 256, 0, stream()>>>(part.data_ptr<float>(), ctas, (int)D,
                                                                dw.data_ptr<float>(), accumulate ? 1 : 0);
  count_launch(2);
  VO_CUDA_OK(cudaGetLastError());
  return dx;
}

torch::Tensor swiglu_fwd(torch::Tensor gu) {
  VO_CHECK_INPUT(gu);
  TORCH_CHECK(gu.scalar_type() == torch::kBFloat16 && gu.size(-1) % 16 == 0, "bf16 [M, 2F], F % 8 == 0");
  const int64_t F2 = gu.size(-1), M = gu.numel() / F2;
  c10::cuda::CUDAGuard g(gu.device());
  auto sizes = gu.sizes().vec();
  sizes.back() = F2 / 2;
  auto a = torch::empty(sizes, gu.options());
  const int fv = (int)(F2 / 16);
  if (M == 0) return a;
  swiglu_fwd_kernel<<<grid_for(M * fv, 256), 256, 0, stream()>>>(
      reinterpret_cast<const bf16x8*>(gu.data_ptr<at::BFloat16>()), reinterpret_cast<bf16x8*>(a.data_ptr<at::BFloat16>()),
      M, fv);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return a;
}

torch::Tensor swiglu_bwd(torch::Tensor da, torch::Tensor gu) {
  VO_CHECK_INPUT(da);
  VO_CHECK_INPUT(gu);
  const int64_t F2 = gu.size(-1), M = gu.numel() / F2;
  TORCH_CHECK(da.numel() == M * F2 / 2 && da.scalar_type() == torch::kBFloat16, "bf16 da [M, F]");
  c10::cuda::CUDAGuard g(gu.device());
  auto dgu = torch::empty_like(gu);
  const int fv = (int)(F2 / 16);
  if (M == 0) return dgu;
  swiglu_bwd_kernel<<<grid_for(M * fv, 256), 256, 0, stream()>>>(
      reinterpret_cast<const bf16x8*>(da.data_ptr<at::BFloat16>()), reinterpret_cast<const bf16x8*>(gu.data_ptr<at::BFloat16>()),
      reinterpret_cast<bf16x8*>(dgu.data_ptr<at::BFloat16>()), M, fv);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return dgu;
}

// logits fp32 [T, E] (E <= 256) -> probs fp32 [T, E], gates fp32 [T, K] (renormalised), idx int64 [T, K]
std::vector<torch::Tensor> router_topk(torch::Tensor logits, int64_t K) {
  VO_CHECK_INPUT(logits);
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2, "fp32 [T, E] router logits");
  const int64_t T = logits.size(0), E = logits.size(1);
  TORCH_CHECK(E >= 1 && E <= 256 && K >= 1 && K <= 32 && K <= E, "E <= 256 experts, top-k <= 32");
  c10::cuda::CUDAGuard g(logits.device());
  auto probs = torch::empty_like(logits);
  auto gates = torch::empty({T, K}, logits.options());
  auto idx = torch::empty({T, K}, logits.options().dtype(torch::kInt64));
  if (T == 0) return {probs, gates, idx};
  const int warps = 8;
  const unsigned grid = (unsigned)((T + warps - 1) / warps);
#define VO_ROUTER(P) \
  router_topk_kernel<P><<<grid, 32 * warps, 0, stream()>>>(logits.data_ptr<float>(), T, (int)E, (int)K, \
                                                           probs.data_ptr<float>(), gates.data_ptr<float>(), \
                                                           idx.data_ptr<int64_t>())
  if (E <= 32) VO_ROUTER(1);
  else if (E <= 64) VO_ROUTER(2);
  else if (E <= 128) VO_ROUTER(4);
  else VO_ROUTER(8);
#undef VO_ROUTER
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return {probs, gates, idx};
}

// x: [B, S, *] bf16 whose columns [col0, col0 + H Dh) hold H heads (row stride x.stride(1)); returns
// [B, H, S, Dh] = rotate-half RoPE(RMSNorm_per_head(x) * w)
torch::Tensor head_rmsnorm_rope(torch::Tensor x, int64_t col0, int64_t H, torch::Tensor w, torch::Tensor cos_t,
                                torch::Tensor sin_t, double eps) {
  VO_CHECK_CUDA(x);
  VO_CHECK_INPUT(w);
  VO_CHECK_INPUT(cos_t);
  VO_CHECK_INPUT(sin_t);
  TORCH_CHECK(x.dim() == 3 && x.stride(2) == 1 && x.stride(0) == x.size(1) * x.stride(1), "x [B, S, *] rows");
  const int64_t B = x.size(0), S = x.size(1), Dh = w.numel();
  TORCH_CHECK(Dh % 2 == 0 && Dh <= 256 && col0 + H * Dh <= x.size(2), "head width <= 256");
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.numel() >= S * Dh / 2 && sin_t.numel() == cos_t.numel(),
              "fp32 [S, Dh/2] RoPE tables");
  c10::cuda::CUDAGuard g(x.device());
  auto y = torch::empty({B, H, S, Dh}, x.options());
  const int64_t items = B * S * H;
  if (items == 0) return y;
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()) + col0;
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr<at::BFloat16>());
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y.data_ptr<at::BFloat16>());
  const bool vec = (Dh == 64 || Dh == 128 || Dh == 256) && items < (int64_t(1) << 31) && x.stride(1) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(xp) % 16 == 0 && reinterpret_cast<uintptr_t>(wp) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(cos_t.data_ptr<float>()) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(sin_t.data_ptr<float>()) % 16 == 0;
  if (vec) {
    const int64_t heads_per_cta = 8 * (32 / (Dh / 8));
    const unsigned grid = (unsigned)((items + heads_per_cta - 1) / heads_per_cta);
#define VO_HNR(DH)                                                                                                  \
  if (Dh == DH)                                                                                                      \
    head_rmsnorm_rope_vec_kernel<DH><<<grid, 256, 0, stream()>>>(xp, x.stride(1), wp, cos_t.data_ptr<float>(),       \
                                                                 sin_t.data_ptr<float>(), yp, (int)B, (int)S, (int)H, \
                                                                 (float)eps);
    VO_HNR(64) VO_HNR(128) VO_HNR(256)
#undef VO_HNR
  } else {
    head_rmsnorm_rope_kernel<<<(unsigned)((items + 7) / 8), 256, 0, stream()>>>(
        xp, x.stride(1), wp, cos_t.data_ptr<float>(), sin_t.data_ptr<float>(), yp, (int)B, (int)S, (int)H, (int)Dh,
        (float)eps);
  }
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return y;
}

// returns dx [B, S, H, Dh] (contiguous); adds the weight gradient into dw (fp32 [Dh])
torch::Tensor head_rmsnorm_rope_bwd(torch::Tensor dy, torch::Tensor x, int64_t col0, int64_t H, torch::Tensor w,
                                    torch::Tensor cos_t, torch::Tensor sin_t, double eps, torch::Tensor dw) {
  VO_CHECK_INPUT(dy);
  VO_CHECK_CUDA(x);
  VO_CHECK_INPUT(dw);
  const int64_t B = x.size(0), S = x.size(1), Dh = w.numel();
  TORCH_CHECK(dy.numel() == B * H * S * Dh && dw.scalar_type() == torch::kFloat32 && dw.numel() == Dh,
              "dy [B, H, S, Dh], fp32 dw");
  c10::cuda::CUDAGuard g(x.device());
  auto dx = torch::empty({B, S, H, Dh}, x.options());
  const int64_t items = B * S * H;
  if (items == 0) return dx;
  {
    const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()) + col0;
    const bool vec = (Dh == 64 || Dh == 128 || Dh == 256) && items < (int64_t(1) << 31) && x.stride(1) % 8 == 0 &&
                     dy.is_contiguous() && reinterpret_cast<uintptr_t>(xp) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(dy.data_ptr()) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(cos_t.data_ptr<float>()) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(sin_t.data_ptr<float>()) % 16 == 0;
    if (vec) {
      const int64_t groups = (items + 32 / (Dh / 8) - 1) / (32 / (Dh / 8));
      const unsigned grid = (unsigned)std::min<int64_t>((groups + 7) / 8, 8LL * num_sms());
      const auto* dyp = reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr<at::BFloat16>());
      const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w.data_ptr<at::BFloat16>());
      auto* dxp = reinterpret_cast<__nv_bfloat16*>(dx.data_ptr<at::BFloat16>());
#define VO_HNRB(DH)                                                                                                  \
  if (Dh == DH)                                                                                                      \
    head_rmsnorm_rope_bwd_vec_kernel<DH><<<grid, 256, 0, stream()>>>(dyp, xp, x.stride(1), wp, cos_t.data_ptr<float>(), \
                                                                     sin_t.data_ptr<float>(), dxp, dw.data_ptr<float>(), \
                                                                     (int)B, (int)S, (int)H, (float)eps);
      VO_HNRB(64) VO_HNRB(128) VO_HNRB(256)
#undef VO_HNRB
      count_launch();
      VO_CUDA_OK(cudaGetLastError());
      return dx;
    }
  }
  head_rmsnorm_rope_bwd_kernel<<<(unsigned)((items + 7) / 8), 256, 0, stream()>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr<at::BFloat16>()),
      reinterpret_cast<const __nv_bfloat16*>(x.data_ptr<at::BFloat16>()) + col0, x.stride(1),
      reinterpret_cast<const __nv_bfloat16*>(w.data_ptr<at::BFloat16>()), cos_t.data_ptr<float>(),
      sin_t.data_ptr<float>(), reinterpret_cast<__nv_bfloat16*>(dx.data_ptr<at::BFloat16>()), dw.data_ptr<float>(),
      (int)B, (int)S, (int)H, (int)Dh, (float)eps);
  count_launch();
  VO_CUDA_OK(cudaGetLastError());
  return dx;
}

}  // namespace vo
