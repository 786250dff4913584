// Flash attention forward for sm_100a on tcgen05 tensor cores.
//
//   O = softmax(Q K^T * scale) V,  LSE = log(sum exp(Q K^T * scale))
//   Q [BH, Sq, D], K/V [BH, Skv, D] (bf16, contiguous per head); O written token-major
//   [B, Sq, H, D]; D in {64, 128}; optional causal mask (query i sees keys <= i).
//
// One CTA per (128-query tile, head); head_dim 64 runs two CTAs per SM.  Roles (192 threads):
//   warp 0      TMA producer: Q once, then K_{j+1} (2-stage ring) ahead of V_j (3D tensor maps, OOB
//               rows zero-filled per head so ragged Sq/Skv need no padding);
//   warp 1      TMEM allocator + MMA issuer: S_j = Q K_j^T into TMEM, then O_j = P_j V_j into TMEM,
//               all tcgen05.mma kind::f16 (S/O/P double buffered for head_dim 128);
//   warps 2..5  softmax warpgroup, one query row per thread: row max and exp2 over S_j (two
//               passes of tcgen05.ld), P_j written as bf16 into 128B-swizzled SMEM (the A operand
//               of the PV MMA), online rescaling of the register-resident O accumulator with each
//               O_j read back from TMEM, final normalisation, O and LSE stores.
// While the softmax warps work on S_j the tensor core computes S_{j+1} and P_{j-1} V_{j-1}.
// Every mbarrier wait is bounded; a timeout records an error code and the CTA exits cleanly.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vo_fmha {

constexpr int BQ = 128, BKV = 128;
constexpr int NUM_THREADS = 192;
constexpr unsigned long long WAIT_BUDGET = 8ull * 1000 * 1000 * 1000;

__device__ int g_error = 0;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(c));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t par) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 200000;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(par)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t par, volatile int* abort_flag, int code) {
  if (mbar_try_wait(b, par)) return true;
  const unsigned long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(b, par)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > WAIT_BUDGET) {
      atomicCAS(&g_error, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(b))
               : "memory");
}
__device__ __forceinline__ void ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ uint64_t desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}
__host__ __device__ constexpr uint32_t idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Params {
  int Sq, Skv, H, nq_tiles;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* o;  // [B, Sq, H, D]
  float* lse;        // [B*H, Sq] natural log
};

// NB = number of S / O / P buffers.  NB == 1 (head_dim 64): 256 TMEM columns and 112 KB of SMEM per
// CTA so two CTAs share an SM and one CTA's softmax overlaps the other's MMAs.  NB == 2 (head_dim 128):
// one CTA per SM with double-buffered S/O/P inside the CTA.
// K always has a 2-stage ring (the next S MMA must not wait for a load); V has NB stages (V_j is
// consumed late, by the PV MMA after the softmax, so one stage hides its load behind that softmax).
template <int D, int NB>
struct Smem {
  static constexpr int TILE = 128 * D * 2;  // one 128-row tile of Q/K/V (D/64 chunks of 16 KB)
  static constexpr int P = 128 * 128 * 2;   // P tile (two 64-column chunks of 16 KB)
  static constexpr int VST = NB;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = TILE;
  static constexpr int V_OFF = 3 * TILE;
  static constexpr int P_OFF = (3 + VST) * TILE;
  static constexpr int BAR_OFF = P_OFF + NB * P;
  static constexpr int BYTES = BAR_OFF + 256;
  static constexpr int TMEM_COLS = NB == 1 ? 256 : 512;
  static constexpr int MIN_BLOCKS = NB == 1 ? 2 : 1;
};

template <int D, int NB>
__global__ void __launch_bounds__(NUM_THREADS, Smem<D, NB>::MIN_BLOCKS)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                    const __grid_constant__ CUtensorMap mv, Params p) {
  using L = Smem<D, NB>;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_free = bars + 7;    // [2]
  uint64_t* p_full = bars + 9;    // [2]
  uint64_t* p_free = bars + 11;   // [2]
  uint64_t* o_full = bars + 13;   // [2]
  uint64_t* o_free = bars + 15;   // [2]
  uint64_t* v_full = bars + 17;   // [2]
  uint64_t* v_empty = bars + 19;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x % p.nq_tiles;
  const int bh = blockIdx.x / p.nq_tiles;
  const int q0 = qt * BQ;
  int kv_end = p.Skv;
  if (p.causal) kv_end = min(p.Skv, q0 + BQ);
  const int nkv = (kv_end + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(L::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  // S buffers at columns [0, NB*128), O buffers after them
  const uint32_t S_COL[2] = {0u, 128u};
  const uint32_t O_COL[2] = {NB * 128u, NB * 128u + D};

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, L::TILE);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_3d(sm + L::Q_OFF + c * 16384, &mq, q_full, c * 64, q0, bh);
      // order: K_0, then for each j: K_{j+1} (2-slot ring), V_j (VST-slot ring)
      auto load_k = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(&k_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, 11)) return false;
        mbar_expect_tx(&k_full[s], L::TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + L::K_OFF + s * L::TILE + c * 16384, &mk, &k_full[s], c * 64, j * BKV, bh);
        return true;
      };
      bool ok = nkv > 0 ? load_k(0) : true;
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv && !(ok = load_k(j + 1))) break;
        const int s = j % L::VST;
        if (!mbar_wait(&v_empty[s], ((j / L::VST) & 1) ^ 1, abort_flag, 10)) break;
        mbar_expect_tx(&v_full[s], L::TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + L::V_OFF + s * L::TILE + c * 16384, &mv, &v_full[s], c * 64, j * BKV, bh);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc(128, 128, 0, 0);
      const uint32_t id_o = idesc(128, D, 0, 1);
      bool ok = mbar_wait(q_full, 0, abort_flag, 12);
      const uint32_t qa = smem_u32(sm + L::Q_OFF);
      for (int j = 0; ok && j <= nkv; ++j) {
        if (j < nkv) {
          const int st = j & 1, b = j % NB;
          if (!mbar_wait(&k_full[st], (j >> 1) & 1, abort_flag, 13)) break;
          if (!mbar_wait(&s_free[b], ((j / NB) & 1) ^ 1, abort_flag, 14)) break;
          fence_after();
          const uint32_t ka = smem_u32(sm + L::K_OFF + st * L::TILE);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            mma(tmem + S_COL[b], desc(qa + off, 16, 1024), desc(ka + off, 16, 1024), id_s, kk > 0);
          }
          commit(&s_full[b]);
          commit(&k_empty[st]);
        }
        if (j >= 1) {
          const int jj = j - 1, st = jj % L::VST, b = jj % NB;
          if (!mbar_wait(&v_full[st], (jj / L::VST) & 1, abort_flag, 20)) break;
          if (!mbar_wait(&p_full[b], (jj / NB) & 1, abort_flag, 15)) break;
          if (!mbar_wait(&o_free[b], ((jj / NB) & 1) ^ 1, abort_flag, 16)) break;
          fence_after();
          const uint32_t pa = smem_u32(sm + L::P_OFF + b * L::P);
          const uint32_t va = smem_u32(sm + L::V_OFF + st * L::TILE);
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
            mma(tmem + O_COL[b], desc(pa + aoff, 16, 1024), desc(va + kk * 2048, 16384, 1024), id_o, kk > 0);
          }
          commit(&o_full[b]);
          commit(&p_free[b]);
          commit(&v_empty[st]);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax warpgroup
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    const int q = q0 + row;
    const uint32_t trow = tmem + ((uint32_t)lane_base << 16);
    float o_acc[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o_acc[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_pending = 0.f;
    bool ok = true;
    for (int j = 0; j <= nkv && ok; ++j) {
      float alpha_j = 0.f;
      if (j < nkv) {
        const int s = j % NB;
        if (!mbar_wait(&s_full[s], (j / NB) & 1, abort_flag, 17)) {
          ok = false;
          break;
        }
        fence_after();
        const int kv0 = j * BKV;
        // blocks fully inside the key range and (causal) fully below the diagonal need no masks
        const bool full = kv0 + BKV <= p.Skv && (!p.causal || kv0 + BKV - 1 <= q0);
        float mx = -INFINITY;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          ld32(trow + S_COL[s] + c * 32, v);
          if (full) {
#pragma unroll
            for (int i = 0; i < 32; ++i) mx = fmaxf(mx, v[i]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int kv = kv0 + c * 32 + i;
              const bool valid = kv < p.Skv && (!p.causal || kv <= q);
              if (valid) mx = fmaxf(mx, v[i]);
            }
          }
        }
        const float m_new = fmaxf(m, mx * p.scale_log2);
        // P buffer s must be free (its previous PV MMA done)
        if (!mbar_wait(&p_free[s], ((j / NB) & 1) ^ 1, abort_flag, 18)) {
          ok = false;
          break;
        }
        uint8_t* pbuf = sm + L::P_OFF + s * L::P;
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float v[32];
          ld32(trow + S_COL[s] + c * 32, v);
#pragma unroll
          for (int g = 0; g < 4; ++g) {  // 4 x 16-byte units of 8 values
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              float e[2];
#pragma unroll
              for (int t = 0; t < 2; ++t) {
                const int i = g * 8 + h * 2 + t;
                const int kv = kv0 + c * 32 + i;
                const bool valid = full || (kv < p.Skv && (!p.causal || kv <= q));
                e[t] = valid ? ex2(fmaf(v[i], p.scale_log2, -m_new)) : 0.f;
                rs += e[t];
              }
              __nv_bfloat162 b2 = __floats2bfloat162_rn(e[0], e[1]);
              w[h] = *reinterpret_cast<uint32_t*>(&b2);
            }
            // column chunk (64 keys) and 16-byte unit within the 128-byte swizzled row
            const int col = c * 32 + g * 8;
            const int chunk = col >> 6;
            const int unit = (col & 63) >> 3;
            uint8_t* dst = pbuf + chunk * 16384 + row * 128 + ((unit ^ (row & 7)) << 4);
            *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[s]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[s]);
        alpha_j = ex2(m - m_new);
        l = l * alpha_j + rs;
        m = m_new;
      }
      if (j >= 1) {  // fold O_{j-1}
        const int jj = j - 1, s = jj % NB;
        if (!mbar_wait(&o_full[s], (jj / NB) & 1, abort_flag, 19)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          ld32(trow + O_COL[s] + c * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) o_acc[c * 32 + i] = o_acc[c * 32 + i] * alpha_pending + v[i];
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&o_free[s]);
      }
      alpha_pending = alpha_j;
    }
    if (ok && q < p.Sq) {
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int b = bh / p.H, h = bh % p.H;
      __nv_bfloat16* dst = p.o + (((int64_t)b * p.Sq + q) * p.H + h) * D;
#pragma unroll
      for (int i = 0; i < D; i += 8) {
        uint4 pk;
        __nv_bfloat162* h2 = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int t = 0; t < 4; ++t) h2[t] = __floats2bfloat162_rn(o_acc[i + 2 * t] * inv, o_acc[i + 2 * t + 1] * inv);
        *reinterpret_cast<uint4*>(dst + i) = pk;
      }
      p.lse[(int64_t)bh * p.Sq + q] = (m + __log2f(l)) * 0.69314718055994531f;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(L::TMEM_COLS));
  }
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeFn encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}

// 3D map over [BH, S, D] bf16 with box {64, 128, 1}, 128B swizzle.
static int map3(CUtensorMap* m, const void* ptr, int BH, int S, int D) {
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t str[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {64, 128, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return (int)encode()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

}  // namespace vo_fmha

extern "C" int vo_fmha_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Sq,
                           int Skv, int D, float scale, int causal, cudaStream_t stream) {
  using namespace vo_fmha;
  if (D != 64 && D != 128) return -1;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
    return -2;
  CUtensorMap mq, mk, mv;
  int r = map3(&mq, q, B * H, Sq, D);
  if (!r) r = map3(&mk, k, B * H, Skv, D);
  if (!r) r = map3(&mv, v, B * H, Skv, D);
  if (r) return r;
  Params p;
  p.Sq = Sq;
  p.Skv = Skv;
  p.H = H;
  p.nq_tiles = (Sq + BQ - 1) / BQ;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  const long long grid = (long long)p.nq_tiles * B * H;
  if (D == 64) {
    using L = Smem<64, 1>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(fmha_fwd_kernel<64, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES + 1024);
      set = true;
    }
    fmha_fwd_kernel<64, 1><<<(unsigned)grid, NUM_THREADS, L::BYTES + 1024, stream>>>(mq, mk, mv, p);
  } else {
    using L = Smem<128, 2>;
    static bool set = false;
    if (!set) {
      cudaFuncSetAttribute(fmha_fwd_kernel<128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES + 1024);
      set = true;
    }
    fmha_fwd_kernel<128, 2><<<(unsigned)grid, NUM_THREADS, L::BYTES + 1024, stream>>>(mq, mk, mv, p);
  }
  return (int)cudaGetLastError();
}

extern "C" int vo_fmha_error(int reset) {
  int e = 0;
  cudaMemcpyFromSymbol(&e, vo_fmha::g_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(vo_fmha::g_error, &z, sizeof(int));
  }
  return e;
}
