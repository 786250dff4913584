// Grouped-query decode attention over a preallocated KV cache (one new query token per sequence).
//
// Decode is bound by reading the cache, so each CTA owns one (sequence, KV head) pair and a slice of the
// keys, and serves every query head of that group from one read of each K / V tile:
//   * K and V tiles of 32 keys are staged in shared memory with 16-byte asynchronous copies, two tiles in
//     flight (rows padded by 16 bytes so the per-key row reads of the score phase do not collide in banks);
//   * scores: the REP x kTile scores of a tile are spread over the 128 threads (consecutive threads take
//     consecutive keys of one query head; REP <= 8 heads per group);
//   * online softmax per head over the CTA's keys; P V with each thread owning one head-dim column for
//     all heads of the group;
//   * key ranges split over `splits` CTAs (flash-decoding) write (max, sum, O) partials that a second
//     kernel merges; with one split the first kernel writes the output directly.
// Lengths differ per sequence (`lens[b]` valid cache rows).
//
// Paged mode (vLLM-style block tables): the cache is a pool of fixed-size blocks [blocks, Hk, block, HD] and
// row t of sequence b lives in block table[b][t / block] at offset t % block; the staging loads resolve
// every row through the table, the rest of the kernel is unchanged.
#include <cstdlib>

#include "common.cuh"

extern "C" int vo_decode_tc(const void* q, const void* kc, const void* vc, const int* lens, const int* table,
                            int stride, int block, int nblocks, int B, int Hk, int Lmax, int rep, int hd,
                            float scale_log2, int splits, void* out, float* part_o, float* part_ml,
                            cudaStream_t stream);
extern "C" int vo_decode_tc_error(int reset);

namespace vo {
namespace {

constexpr int kTile = 32;  // keys per tile; tiles are double-buffered
constexpr int kDecThreads = 128;

// 16-byte asynchronous global -> shared copy; valid == false fills the 16 bytes with zeros
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// N consecutive bf16 values (N in {1, 2, 4, 8}, N-element aligned) -> fp32
template <int N>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float* f) {
  if constexpr (N == 16) {
    unpack8(*reinterpret_cast<const bf16x8*>(p), f);
    unpack8(*reinterpret_cast<const bf16x8*>(p + 8), f + 8);
  } else if constexpr (N == 8) {
    unpack8(*reinterpret_cast<const bf16x8*>(p), f);
  } else if constexpr (N == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
    f[0] = a.x, f[1] = a.y, f[2] = b.x, f[3] = b.y;
  } else if constexpr (N == 2) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    f[0] = a.x, f[1] = a.y;
  } else {
    f[0] = bf2f(*p);
  }
}

struct PageTable {
  const int* table;  // [B, stride] block ids, null: contiguous [B, Hk, Lmax, HD] cache
  int stride;
  int block;    // rows per block
  int nblocks;  // blocks in the pool: a table entry outside [0, nblocks) reads as zeros
};

template <int HD, int REP>
__global__ void __launch_bounds__(kDecThreads) decode_attn_kernel(
    const __nv_bfloat16* __restrict__ q,      // [B, Hk * REP, HD]
    const __nv_bfloat16* __restrict__ kc,     // [B, Hk, Lmax, HD]
    const __nv_bfloat16* __restrict__ vc,     // [B, Hk, Lmax, HD]
    const int* __restrict__ lens, int Hk, int Lmax, float scale_log2, int splits, PageTable pt,
    __nv_bfloat16* __restrict__ out,          // [B, Hk * REP, HD] (splits == 1)
    float* __restrict__ part_o,               // [B, Hk, splits, REP, HD]
    float* __restrict__ part_ml) {            // [B, Hk, splits, REP, 2]
  constexpr int ROW = HD + 8;  // padded smem row (bf16 elements)
  __shared__ __align__(16) __nv_bfloat16 ks_buf[2][kTile * ROW];
  __shared__ __align__(16) __nv_bfloat16 vs_buf[2][kTile * HD];
  __shared__ __align__(16) float qs[REP * HD];
  __shared__ float ps[REP * kTile];
  __shared__ float mrow[REP], lrow[REP], alpha_s[REP];

  const int bk = blockIdx.x, split = blockIdx.y;
  const int b = bk / Hk, kh = bk % Hk;
  // lengths beyond the cache (or beyond the block table's reach) are clamped, so a bad length never reads
  // past the cache
  const int cap = pt.table ? pt.stride * pt.block : Lmax;
  VO_DCHECK(lens[b] >= 0 && lens[b] <= cap);  // checked builds record a clamped length
  const int L = max(0, min(lens[b], cap));
  const int per = (L + splits - 1) / splits;
  const int s0 = split * per, s1 = min(L, s0 + per);
  const int tid = threadIdx.x;
  const __nv_bfloat16* qb = q + ((int64_t)b * Hk * REP + (int64_t)kh * REP) * HD;
  for (int i = tid; i < REP * HD; i += kDecThreads) qs[i] = bf2f(qb[i]) * scale_log2;
  if (tid < REP) {
    mrow[tid] = -INFINITY;
    lrow[tid] = 0.f;
  }
  // this thread's outputs: OUT_PER consecutive head-dim columns [o0, o0 + OUT_PER) of the flattened
  // (head, dim) space, so each V row read is one vector load
  constexpr int OUT_PER = (REP * HD) / kDecThreads > 0 ? (REP * HD) / kDecThreads : 1;
  const int o0 = tid * OUT_PER;
  const bool o_ok = o0 < REP * HD;
  const int oh = o_ok ? o0 / HD : 0, od = o0 % HD;
  float acc[OUT_PER];
#pragma unroll
  for (int i = 0; i < OUT_PER; ++i) acc[i] = 0.f;
  const int64_t kvbase = ((int64_t)b * Hk + kh) * Lmax * HD;
  __syncthreads();

  // stage K (padded rows) and V of the tile at t0 into buffer buf: asynchronous copies, zero-filled past
  // the slice end, so the next tile's loads are in flight while the current tile is consumed
  auto stage = [&](int t0, int buf) {
    const int nk = min(kTile, s1 - t0);
    for (int i = tid; i < kTile * (HD / 8); i += kDecThreads) {
      const int r = i / (HD / 8), c = i % (HD / 8);
      int64_t off = 0;  // rows past the slice: zero fill, the source address is only a valid placeholder
      bool ok = r < nk;
      if (ok) {
        const int t = t0 + r;
        off = kvbase + (int64_t)t * HD;
        if (pt.table) {
          const int blk = __ldg(pt.table + (int64_t)b * pt.stride + t / pt.block);
          ok = VO_DCHECK(blk >= 0 && blk < pt.nblocks);  // out-of-pool block ids read as zeros
          off = ok ? (((int64_t)blk * Hk + kh) * pt.block + t % pt.block) * HD : 0;
        }
      }
      cp_async16(ks_buf[buf] + r * ROW + c * 8, kc + off + c * 8, ok);
      cp_async16(vs_buf[buf] + r * HD + c * 8, vc + off + c * 8, ok);
    }
  };
  if (s0 < s1) stage(s0, 0);
  cp_async_commit();

  for (int t0 = s0, it = 0; t0 < s1; t0 += kTile, ++it) {
    const int nk = min(kTile, s1 - t0);
    const __nv_bfloat16* ks = ks_buf[it & 1];
    const __nv_bfloat16* vs = vs_buf[it & 1];
    if (t0 + kTile < s1) stage(t0 + kTile, (it + 1) & 1);  // that buffer was released by the last barrier
    cp_async_commit();
    cp_async_wait1();  // this thread's copies of the current tile have landed
    __syncthreads();   // ... and every other thread's
    // scores (log2 domain): thread -> key k, heads h0, h0 + HSTEP, ...; each K chunk is read once for
    // all of the thread's heads
    {
      constexpr int HSTEP = kDecThreads / kTile;
      constexpr int HPT = (REP + HSTEP - 1) / HSTEP;
      const int k = tid % kTile, h0 = tid / kTile;
      float sc[HPT];
#pragma unroll
      for (int j = 0; j < HPT; ++j) sc[j] = 0.f;
      if (k < nk) {
#pragma unroll 2
        for (int c = 0; c < HD / 8; ++c) {
          float f[8];
          unpack8(*reinterpret_cast<const bf16x8*>(ks + k * ROW + c * 8), f);
#pragma unroll
          for (int j = 0; j < HPT; ++j) {
            const int h = h0 + j * HSTEP;
            if (h < REP) {
              const float4 qa = *reinterpret_cast<const float4*>(qs + h * HD + c * 8);
              const float4 qb = *reinterpret_cast<const float4*>(qs + h * HD + c * 8 + 4);
              float t = sc[j];
              t = fmaf(qa.x, f[0], t);
              t = fmaf(qa.y, f[1], t);
              t = fmaf(qa.z, f[2], t);
              t = fmaf(qa.w, f[3], t);
              t = fmaf(qb.x, f[4], t);
              t = fmaf(qb.y, f[5], t);
              t = fmaf(qb.z, f[6], t);
              t = fmaf(qb.w, f[7], t);
              sc[j] = t;
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < HPT; ++j) {
        const int h = h0 + j * HSTEP;
        if (h < REP) ps[h * kTile + k] = k < nk ? sc[j] : -INFINITY;
      }
    }
    __syncthreads();
    // per-head running max / sum (one warp per head, heads strided over the 4 warps)
    const int warp = tid >> 5, lane = tid & 31;
    for (int h = warp; h < REP; h += kDecThreads / 32) {
      const float a = ps[h * kTile + lane], c2 = kTile > 32 ? ps[h * kTile + 32 + lane] : -INFINITY;
      const float mx = warp_max(fmaxf(a, c2));
      const float m_old = mrow[h];
      const float m_new = fmaxf(m_old, mx);
      const float e0 = (a == -INFINITY) ? 0.f : exp2f(a - m_new);
      const float e1 = (c2 == -INFINITY) ? 0.f : exp2f(c2 - m_new);
      ps[h * kTile + lane] = e0;
      if (kTile > 32) ps[h * kTile + 32 + lane] = e1;
      const float sum = warp_sum(e0 + e1);
      if (lane == 0) {
        const float al = (m_old == -INFINITY) ? 0.f : exp2f(m_old - m_new);
        alpha_s[h] = al;
        lrow[h] = lrow[h] * al + sum;
        mrow[h] = m_new;
      }
    }
    __syncthreads();
    // O = O * alpha + P V (OUT_PER consecutive columns of one head per thread)
    if (o_ok) {
      const float al = alpha_s[oh];
#pragma unroll
      for (int i = 0; i < OUT_PER; ++i) acc[i] *= al;
      const float* ph = ps + oh * kTile;
      for (int k = 0; k < nk; ++k) {
        const float p = ph[k];
        float f[OUT_PER];
        load_row<OUT_PER>(vs + k * HD + od, f);
#pragma unroll
        for (int i = 0; i < OUT_PER; ++i) acc[i] = fmaf(p, f[i], acc[i]);
      }
    }
    __syncthreads();
  }
  if (splits == 1) {
    if (o_ok) {
      const float l = lrow[oh];
#pragma unroll
      for (int i = 0; i < OUT_PER; ++i)
        out[((int64_t)b * Hk * REP + (int64_t)kh * REP + oh) * HD + od + i] = f2bf(l > 0.f ? acc[i] / l : 0.f);
    }
    return;
  }
  const int64_t pbase = (((int64_t)b * Hk + kh) * splits + split) * REP;
  if (o_ok) {
#pragma unroll
    for (int i = 0; i < OUT_PER; ++i) part_o[pbase * HD + o0 + i] = acc[i];
  }
  if (tid < REP) {
    part_ml[(pbase + tid) * 2] = mrow[tid];
    part_ml[(pbase + tid) * 2 + 1] = lrow[tid];
  }
}

// merges the split partials: one thread per (sequence, head, dim)
template <int HD, int REP>
__global__ void decode_combine_kernel(const float* __restrict__ part_o, const float* __restrict__ part_ml, int Hk,
                                      int splits, int64_t total, __nv_bfloat16* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(i % HD);
    const int64_t bhq = i / HD;  // (b, kh, h)
    const int h = (int)(bhq % REP);
    const int64_t bk = bhq / REP;
    float m = -INFINITY;
    for (int s = 0; s < splits; ++s) m = fmaxf(m, part_ml[((bk * splits + s) * REP + h) * 2]);
    float l = 0.f, o = 0.f;
    if (m != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const int64_t pi = (bk * splits + s) * REP + h;
        const float ms = part_ml[pi * 2];
        if (ms == -INFINITY) continue;
        const float w = exp2f(ms - m);
        l += part_ml[pi * 2 + 1] * w;
        o += part_o[pi * HD + d] * w;
      }
    }
    out[bhq * HD + d] = f2bf(l > 0.f ? o / l : 0.f);
  }
}

template <int HD, int REP>
void launch_decode(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc, const torch::Tensor& lens,
                   float scale_log2, int splits, PageTable pt, torch::Tensor& out) {
  const int B = (int)q.size(0), Hk = (int)kc.size(1), Lmax = (int)kc.size(2);
  auto fo = q.options().dtype(torch::kFloat32);
  torch::Tensor po, pml;
  if (splits > 1) {
    po = torch::empty({B, Hk, splits, REP, HD}, fo);
    pml = torch::empty({B, Hk, splits, REP, 2}, fo);
  }
  auto bfp = [](const torch::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr<at::BFloat16>()); };
  decode_attn_kernel<HD, REP><<<dim3(B * Hk, splits), kDecThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      bfp(q), bfp(kc), bfp(vc), lens.data_ptr<int>(), Hk, Lmax, scale_log2, splits, pt,
      reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()), splits > 1 ? po.data_ptr<float>() : nullptr,
      splits > 1 ? pml.data_ptr<float>() : nullptr);
  count_launch();
  if (splits > 1) {
    const int64_t total = (int64_t)B * Hk * REP * HD;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 4096);
    decode_combine_kernel<HD, REP><<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        po.data_ptr<float>(), pml.data_ptr<float>(), Hk, splits, total,
        reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()));
    count_launch();
  }
  VO_CUDA_OK(cudaGetLastError());
}

// key splits: enough CTAs to cover the SMs `per_sm` times over, at least `min_keys` keys per split
int pick_splits(int64_t pairs, int64_t span, int per_sm, int64_t min_keys, int cap) {
  const int64_t want = (per_sm * (int64_t)num_sms() + pairs - 1) / std::max<int64_t>(pairs, 1);
  return (int)std::max<int64_t>(1, std::min<int64_t>({want, (int64_t)cap, std::max<int64_t>(1, span / min_keys)}));
}

}  // namespace

// q [B, Hk * rep, 128] against the cache on the tcgen05 kernel (csrc/decode_attn_sm100.cu); false when the
// shape is outside it (the CUDA-core kernel runs instead)
static bool decode_tc(const torch::Tensor& q, const torch::Tensor& kc, const torch::Tensor& vc, const torch::Tensor& lens,
                      float scale_log2, int64_t splits, const PageTable& pt, torch::Tensor& out) {
  const char* env = std::getenv("VO_DECODE_TC");
  if (env && env[0] == '0') return false;
  const int B = (int)q.size(0), Hk = (int)kc.size(1), HD = (int)q.size(2), rep = (int)(q.size(1) / Hk);
  if (HD != 128 || (rep != 1 && rep != 2 && rep != 4 && rep != 8 && rep != 16)) return false;
  if (pt.table && (pt.block % 8 || 128 % pt.block)) return false;
  const int Lmax = pt.table ? 0 : (int)kc.size(2);
  const int64_t span = pt.table ? (int64_t)pt.stride * pt.block : Lmax;
  // one CTA per SM (three 64 KB K / V stages): split the keys only while every CTA still gets an SM in the
  // first wave (a second partial wave costs more than the longer key range), >= four 128-key tiles each
  const int64_t pairs = (int64_t)B * Hk;
  const int sp = splits > 0 ? (int)splits
                            : (int)std::max<int64_t>(1, std::min<int64_t>({num_sms() / std::max<int64_t>(pairs, 1), 64,
                                                                           std::max<int64_t>(1, span / 512)}));
  auto fo = q.options().dtype(torch::kFloat32);
  torch::Tensor po, pml;
  if (sp > 1) {
    po = torch::empty({B, Hk, sp, rep, HD}, fo);
    pml = torch::empty({B, Hk, sp, rep, 2}, fo);
  }
  auto st = at::cuda::getCurrentCUDAStream();
  const int rc = vo_decode_tc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.data_ptr<int>(), pt.table, pt.stride,
                              pt.block, pt.nblocks, B, Hk, Lmax, rep, HD, scale_log2, sp, out.data_ptr(),
                              sp > 1 ? po.data_ptr<float>() : nullptr, sp > 1 ? pml.data_ptr<float>() : nullptr, st);
  if (rc == -1) return false;
  TORCH_CHECK(rc == 0, "tcgen05 decode attention launch failed: ", rc);
  count_launch();
  if (sp > 1) {
    const int64_t total = (int64_t)B * Hk * rep * HD;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 4096);
    auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>());
#define VO_COMB(R) \
  if (rep == R) decode_combine_kernel<128, R><<<grid, 256, 0, st>>>(po.data_ptr<float>(), pml.data_ptr<float>(), Hk, sp, total, o);
    VO_COMB(1) VO_COMB(2) VO_COMB(4) VO_COMB(8) VO_COMB(16)
#undef VO_COMB
    count_launch();
  }
  VO_CUDA_OK(cudaGetLastError());
  return true;
}

int64_t decode_tc_error(bool reset) { return vo_decode_tc_error(reset ? 1 : 0); }

// q [B, Hq, HD] bf16; k_cache / v_cache [B, Hk, Lmax, HD] bf16 -- or, with block_table [B, max_blocks]
// int32, block pools [blocks, Hk, block, HD]; lens [B] int32 (valid rows, >= 1; with a table at most
// max_blocks x block; longer lengths are clamped to the cache, table ids outside the pool read as zeros).
// Returns o [B, Hq, HD].  Hq = Hk x rep with rep in {1, 2, 4, 8} (16 as well at HD 128); HD in {64, 128}.
// splits <= 0 picks the key split count for the kernel that runs.  head_dim 128 runs the tcgen05 kernel
// (contiguous caches and paged blocks of 64 or 128 rows); the rest the CUDA-core kernel above.
torch::Tensor decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor lens,
                               double scale, int64_t splits, c10::optional<torch::Tensor> block_table) {
  VO_CHECK_INPUT(q);
  VO_CHECK_INPUT(k_cache);
  VO_CHECK_INPUT(v_cache);
  VO_CHECK_INPUT(lens);
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k_cache.scalar_type() == torch::kBFloat16 &&
                  v_cache.scalar_type() == torch::kBFloat16 && lens.scalar_type() == torch::kInt32,
              "bf16 q / cache, int32 lengths");
  const int64_t B = q.size(0), Hq = q.size(1), HD = q.size(2), Hk = k_cache.size(1);
  PageTable pt{nullptr, 0, 0, 0};
  if (block_table.has_value() && block_table->defined()) {
    VO_CHECK_INPUT(*block_table);
    TORCH_CHECK(block_table->scalar_type() == torch::kInt32 && block_table->dim() == 2 && block_table->size(0) == B,
                "int32 [B, max_blocks] block table");
    pt.table = block_table->data_ptr<int>();
    pt.stride = (int)block_table->size(1);
    pt.block = (int)k_cache.size(2);
    pt.nblocks = (int)k_cache.size(0);
    TORCH_CHECK(pt.block > 0, "empty blocks");
  } else {
    TORCH_CHECK(k_cache.size(0) == B, "one cache row per sequence");
  }
  TORCH_CHECK(k_cache.size(3) == HD && v_cache.sizes() == k_cache.sizes() && Hq % Hk == 0 && lens.numel() == B,
              "decode attention shapes");
  c10::cuda::CUDAGuard g(q.device());
  auto out = torch::empty_like(q);
  const int rep = (int)(Hq / Hk);
  const float sl2 = (float)scale * 1.4426950408889634f;
  if (decode_tc(q, k_cache, v_cache, lens, sl2, splits, pt, out)) return out;
  // CUDA-core kernel: about 16 CTAs per SM (5 resident at once) for memory parallelism, >= 256 keys each
  const int64_t span = pt.table ? (int64_t)pt.stride * pt.block : k_cache.size(2);
  const int sp = splits > 0 ? (int)splits : pick_splits(B * Hk, span, 16, 256, 16);
#define VO_DEC(HDV, REPV) \
  if (HD == HDV && rep == REPV) return launch_decode<HDV, REPV>(q, k_cache, v_cache, lens, sl2, sp, pt, out), out;
  VO_DEC(128, 16) VO_DEC(128, 8) VO_DEC(128, 4) VO_DEC(128, 2) VO_DEC(128, 1) VO_DEC(64, 8) VO_DEC(64, 4) VO_DEC(64, 2)
  VO_DEC(64, 1)
#undef VO_DEC
  TORCH_CHECK(false, "decode attention: head_dim 64 / 128 and 1, 2, 4 or 8 query heads per KV head (16 at 128)");
  return out;
}

}  // namespace vo
