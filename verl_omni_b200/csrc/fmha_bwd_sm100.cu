// Flash attention backward for sm_100a on tcgen05 tensor cores.
//
// Given Q, K, V [BH, S, D] (bf16), O and dO token-major [B, Sq, H, D], LSE [BH, Sq] (natural log):
//   P = exp(Q K^T * scale - LSE),  dV = P^T dO,  dP = dO V^T,  dS = P * (dP - Delta),
//   Delta = rowsum(dO * O),  dQ = scale * dS K,  dK = scale * dS^T Q.
//
// Kernels:
//   delta_kernel     Delta[bh, q] in fp32 (one 8/16-lane group per row).
//   fmha_bwd_kernel  one CTA per (128-key tile, head); loops over 128-query tiles:
//     warp 0      TMA: K_j, V_j once; Q_i and dO_i per iteration (ring of STAGES);
//     warp 1      MMA issuer: S^T = K Q^T and dP^T = V dO^T into TMEM (lanes = keys), then
//                 dV += P^T dO, dK += dS^T Q (TMEM accumulators for the whole loop) and
//                 dQ_i = dS K (TMEM, reusing the S^T columns);
//     warps 2..5  one key row per thread: P^T and dS^T from the two TMEM rows, written bf16 into
//                 128B-swizzled SMEM -- read as K-major A operands by the dV/dK MMAs and as an
//                 MN-major A operand by the dQ MMA; then the dQ_i tile (one query row per thread)
//                 is added into an fp32 dQ accumulator with vector reductions; at the end dK/dV
//                 are scaled, rounded and stored.
//   dq_finalize      dQ = bf16(scale * dQ_acc).
// All operand majorness changes are expressed through smem descriptors (no transposes in memory).
// Every mbarrier wait is bounded; a timeout records an error code and the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace vo_fbwd {

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
// a waiting thread is suspended for up to this long (it wakes as soon as the phase completes), so warps
// that wait -- the drain, producer and issuer warps most of the time -- do not spin on issue slots and ALU
// cycles the gradient warps need
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t par) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(par), "r"(kSuspendNs)
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
__device__ __forceinline__ void tma3(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma4(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
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
__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

struct Params {
  int Sq, Skv, H, nkv_tiles, causal;
  const int* kv_len;  // optional per-sequence key count [B]: keys at or past it get no attention
  float scale, scale_log2;
  const float* lse;    // [BH, Sq]
  const float* delta;  // [BH, Sq]
  float* dq_acc;       // [BH, Sq, D] fp32 (pre-zeroed)
  __nv_bfloat16* dk;   // [BH, Skv, D]
  __nv_bfloat16* dv;   // [BH, Skv, D]
  int split;           // > 0: dO rows q >= split come from the second dO tensor map (split % 128 == 0)
  const float4* ls_rec = nullptr;  // version 4: [BH, ceil(Sq / 64), 32] {-lse q log2e, -lse q+1 log2e, Delta q, Delta q+1}
  long long* trace = nullptr;      // traced launches: SM clock stamps [32 CTAs][64 blocks][10 events]
};

template <int D>
struct Lay {
  static constexpr int STAGES = D == 64 ? 2 : 1;
  static constexpr int TILE = 128 * D * 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int Q_OFF = 2 * TILE;
  static constexpr int DO_OFF = Q_OFF + STAGES * TILE;
  static constexpr int PT_OFF = DO_OFF + STAGES * TILE;
  static constexpr int DS_OFF = PT_OFF + 32768;
  static constexpr int LSE_OFF = DS_OFF + 32768;  // 128 floats
  static constexpr int DEL_OFF = LSE_OFF + 512;   // 128 floats
  static constexpr int BAR_OFF = DEL_OFF + 512;
  static constexpr int BYTES = BAR_OFF + 256;
  static_assert(BYTES + 1024 <= 232448, "shared memory above the 227 KB per-block limit");
};

// write 32 bf16 values (one 32-column chunk of a 128-col row) into a 128B-swizzled [128 x 128] tile
__device__ __forceinline__ void store_row_chunk(uint8_t* tile, int row, int c, const float* v) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint32_t w[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      __nv_bfloat162 b2 = __floats2bfloat162_rn(v[g * 8 + 2 * h], v[g * 8 + 2 * h + 1]);
      w[h] = *reinterpret_cast<uint32_t*>(&b2);
    }
    const int col = c * 32 + g * 8;
    const int chunk = col >> 6, unit = (col & 63) >> 3;
    *reinterpret_cast<uint4*>(tile + chunk * 16384 + row * 128 + ((unit ^ (row & 7)) << 4)) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

template <int D>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fmha_bwd_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                    const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                    const __grid_constant__ CUtensorMap mdo2, Params p) {
  using L = Lay<D>;
  constexpr int ST = L::STAGES;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* sp_full = bars + 5;
  uint64_t* ds_full = bars + 6;
  uint64_t* mma2_done = bars + 7;
  uint64_t* dq_free = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* lse_s = reinterpret_cast<float*>(sm + L::LSE_OFF);
  float* del_s = reinterpret_cast<float*>(sm + L::DEL_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x % p.nkv_tiles;
  const int bh = blockIdx.x / p.nkv_tiles;
  const int b = bh / p.H, h = bh % p.H;
  const int kv0 = kt * 128;
  const int i0 = p.causal ? kv0 / 128 : 0;
  const int nq = (p.Sq + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(ds_full, 4);
    mbar_init(mma2_done, 1);
    mbar_init(dq_free, 4);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t C_ST = 0, C_DPT = 128, C_DV = 256, C_DK = 256 + D, C_DQ = 0;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(kv_full, 2 * L::TILE);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma3(sm + L::K_OFF + c * 16384, &mk, kv_full, c * 64, kv0, bh);
        tma3(sm + L::V_OFF + c * 16384, &mv, kv_full, c * 64, kv0, bh);
      }
      for (int i = i0, it = 0; i < nq; ++i, ++it) {
        const int st = it % ST;
        if (!mbar_wait(&qdo_empty[st], ((it / ST) & 1) ^ 1, abort_flag, 21)) break;
        mbar_expect_tx(&qdo_full[st], 2 * L::TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma3(sm + L::Q_OFF + st * L::TILE + c * 16384, &mq, &qdo_full[st], c * 64, i * 128, bh);
          if (p.split > 0 && i * 128 >= p.split)
            tma4(sm + L::DO_OFF + st * L::TILE + c * 16384, &mdo2, &qdo_full[st], c * 64, h, i * 128 - p.split, b);
          else
            tma4(sm + L::DO_OFF + st * L::TILE + c * 16384, &mdo, &qdo_full[st], c * 64, h, i * 128, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_kk = idesc(128, 128, 0, 0);  // S^T, dP^T: A, B K-major over d
      const uint32_t id_kn = idesc(128, D, 0, 1);    // dV, dK: A K-major over q, B MN-major (d contiguous)
      const uint32_t id_nn = idesc(128, D, 1, 1);    // dQ: A = dS^T read MN-major, B = K MN-major
      const uint32_t ka = smem_u32(sm + L::K_OFF), va = smem_u32(sm + L::V_OFF);
      const uint32_t pa = smem_u32(sm + L::PT_OFF), da = smem_u32(sm + L::DS_OFF);
      bool ok = mbar_wait(kv_full, 0, abort_flag, 22);
      for (int i = i0, it = 0; ok && i < nq; ++i, ++it) {
        const int st = it % ST;
        if (!mbar_wait(&qdo_full[st], (it / ST) & 1, abort_flag, 23)) break;
        if (it > 0 && !mbar_wait(dq_free, (it - 1) & 1, abort_flag, 24)) break;
        fence_after();
        const uint32_t qa = smem_u32(sm + L::Q_OFF + st * L::TILE);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + st * L::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma(tmem + C_ST, desc(ka + off, 16, 1024), desc(qa + off, 16, 1024), id_kk, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma(tmem + C_DPT, desc(va + off, 16, 1024), desc(oa + off, 16, 1024), id_kk, kk > 0);
        }
        commit(sp_full);
        if (!mbar_wait(ds_full, it & 1, abort_flag, 25)) break;
        fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // reduce over 128 queries
          const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma(tmem + C_DV, desc(pa + aoff, 16, 1024), desc(oa + kk * 2048, 16384, 1024), id_kn, (it > 0 || kk > 0));
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma(tmem + C_DK, desc(da + aoff, 16, 1024), desc(qa + kk * 2048, 16384, 1024), id_kn, (it > 0 || kk > 0));
        }
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // reduce over 128 keys
          mma(tmem + C_DQ, desc(da + kk * 2048, 16384, 1024), desc(ka + kk * 2048, 16384, 1024), id_nn, kk > 0);
        }
        commit(mma2_done);
        commit(&qdo_empty[st]);
      }
    }
  } else {
    const int tid = threadIdx.x - 64;  // 0..127 over the four softmax warps
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;  // TMEM lane = key row (S^T, dV, dK) or query row (dQ)
    const int kv = kv0 + r;
    const uint32_t trow = tmem + ((uint32_t)lane_base << 16);
    uint8_t* pt = sm + L::PT_OFF;
    uint8_t* ds = sm + L::DS_OFF;
    bool ok = true;
    int it = 0;
    for (int i = i0; i < nq && ok; ++i, ++it) {
      const int q0 = i * 128;
      named_bar(1, 128);
      {
        const int q = q0 + tid;
        lse_s[tid] = q < p.Sq ? p.lse[(int64_t)bh * p.Sq + q] * 1.4426950408889634f : INFINITY;
        del_s[tid] = q < p.Sq ? p.delta[(int64_t)bh * p.Sq + q] : 0.f;
      }
      named_bar(1, 128);
      if (!mbar_wait(sp_full, it & 1, abort_flag, 26)) {
        ok = false;
        break;
      }
      fence_after();
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float s[32], dp[32];
        ld32(trow + C_ST + c * 32, s);
        ld32(trow + C_DPT + c * 32, dp);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int qc = c * 32 + j;
          const int q = q0 + qc;
          const bool valid = kv < (p.kv_len ? min(p.Skv, __ldg(p.kv_len + bh / p.H)) : p.Skv) &&
                             (!p.causal || kv <= q);
          const float pv = valid ? ex2(s[j] * p.scale_log2 - lse_s[qc]) : 0.f;
          s[j] = pv;
          dp[j] = pv * (dp[j] - del_s[qc]);
        }
        store_row_chunk(pt, r, c, s);
        store_row_chunk(ds, r, c, dp);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
      if (!mbar_wait(mma2_done, it & 1, abort_flag, 27)) {
        ok = false;
        break;
      }
      fence_after();
      {  // dQ tile: TMEM lane r = query row q0 + r
        const int q = q0 + r;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          float v[32];
          ld32(trow + C_DQ + c * 32, v);
          if (q < p.Sq) {
            float* dst = p.dq_acc + ((int64_t)bh * p.Sq + q) * D + c * 32;
#pragma unroll
            for (int j = 0; j < 32; j += 4) red_add_v4(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
          }
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(dq_free);
    }
    if (ok && it > 0) {
      // all MMAs of the last iteration completed (mma2_done waited) -> dV, dK final
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float vv[32], kk[32];
        ld32(trow + C_DV + c * 32, vv);
        ld32(trow + C_DK + c * 32, kk);
        if (kv < p.Skv) {
          __nv_bfloat16* dvp = p.dv + ((int64_t)bh * p.Skv + kv) * D + c * 32;
          __nv_bfloat16* dkp = p.dk + ((int64_t)bh * p.Skv + kv) * D + c * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 a, bq;
            __nv_bfloat162* ha = reinterpret_cast<__nv_bfloat162*>(&a);
            __nv_bfloat162* hb = reinterpret_cast<__nv_bfloat162*>(&bq);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              ha[t] = __floats2bfloat162_rn(vv[j + 2 * t], vv[j + 2 * t + 1]);
              hb[t] = __floats2bfloat162_rn(kk[j + 2 * t] * p.scale, kk[j + 2 * t + 1] * p.scale);
            }
            *reinterpret_cast<uint4*>(dvp + j) = a;
            *reinterpret_cast<uint4*>(dkp + j) = bq;
          }
        }
      }
    } else if (ok && kv < p.Skv) {  // causal tile with no queries: zero gradients
      for (int j = 0; j < D; ++j) {
        p.dv[((int64_t)bh * p.Skv + kv) * D + j] = __float2bfloat16_rn(0.f);
        p.dk[((int64_t)bh * p.Skv + kv) * D + j] = __float2bfloat16_rn(0.f);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}

// ------------------------------------------------------------------------------------ version 2
// Same math, pipelined.  384 threads:
//   warp 0       TMA: K, V once; Q_i and dO_i per query tile (2-stage ring);
//   warp 1       MMA issuer;
//   warps 4..7   gradient warpgroup (one key row per thread): P^T = exp2(S^T*scale_log2 - lse) and
//                dS^T = P^T * (dP^T - Delta) computed chunk by chunk; P^T and dS^T go back into
//                tensor memory in place (bf16 pairs over the first 64 columns of their fp32 tiles)
//                where the dV / dK MMAs read them as A operands, and dS^T also into swizzled SMEM
//                for the dQ MMA (A = dS, MN-major);
//   warps 8..11  dQ drain: dQ_i tile (one query row per thread) from tensor memory into the fp32
//                dQ accumulator with vector reductions, concurrently with the next tile's math.
// Tensor memory (512 columns): S^T buffers (two for head_dim 64, one for 128), dP^T, dV, dK; dQ_i
// is written into the S^T buffer of tile i after the dV MMA has consumed P^T_i (the tensor pipe
// executes one thread's MMAs in order).  For head_dim 64 the next tile's S^T MMA runs while the
// gradient warpgroup works on the current tile.
namespace v2 {
__device__ __forceinline__ void ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
// (a0, a1) * s + (c0, c1) on the paired fp32 pipe
__device__ __forceinline__ void ffma2p(float a0, float a1, float s, float c0, float c1, float& r0, float& r1) {
  asm("{\n\t.reg .b64 x, y, z, r;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %4};\n\tmov.b64 z, {%5, %6};\n\t"
      "fma.rn.f32x2 r, x, y, z;\n\tmov.b64 {%0, %1}, r;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(s), "f"(c0), "f"(c1));
}
// (e0, e1) * ((p0, p1) - (d0, d1)) on the paired fp32 pipe
__device__ __forceinline__ void sub_mul2(float p0, float p1, float d0, float d1, float e0, float e1, float& r0,
                                         float& r1) {
  asm("{\n\t.reg .b64 x, y, e, t;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 e, {%6, %7};\n\t"
      "sub.rn.f32x2 t, x, y;\n\tmul.rn.f32x2 t, t, e;\n\tmov.b64 {%0, %1}, t;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(p0), "f"(p1), "f"(d0), "f"(d1), "f"(e0), "f"(e1));
}

// 16 query columns [c0, c0 + 16) of one key row (one thread): P^T = exp2(S^T scale_log2 - lse log2e) and
// dS^T = P^T (dP^T - Delta).  Written phase by phase over the 16 columns (all loads, all FMAs, all
// exponentials, all dS, all packs), so every phase is 8-16 independent instructions the scheduler can
// overlap instead of one dependent chain per column pair.  The packed bf16 P^T / dS^T go into tensor-memory
// columns [c0 / 2, c0 / 2 + 8) of the two score buffers: with the chunks of a row run in order c0 = 0, 16,
// 32, 48 by one thread, those columns have been read already.  dS^T also goes to the swizzled shared-memory
// row for the dQ MMA.  `ls` holds {-lse log2e, -lse log2e, Delta, Delta} per query pair.
__device__ __forceinline__ void grad_chunk16(uint32_t S_t, uint32_t DP_t, int c0, const float4* __restrict__ ls,
                                             float sl2, bool full, int qlo, int qhi, uint8_t* ds, int r) {
  uint32_t sa[16], pa[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(sa[0]), "=r"(sa[1]), "=r"(sa[2]), "=r"(sa[3]), "=r"(sa[4]), "=r"(sa[5]), "=r"(sa[6]), "=r"(sa[7]),
        "=r"(sa[8]), "=r"(sa[9]), "=r"(sa[10]), "=r"(sa[11]), "=r"(sa[12]), "=r"(sa[13]), "=r"(sa[14]), "=r"(sa[15])
      : "r"(S_t + c0));
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(pa[0]), "=r"(pa[1]), "=r"(pa[2]), "=r"(pa[3]), "=r"(pa[4]), "=r"(pa[5]), "=r"(pa[6]), "=r"(pa[7]),
        "=r"(pa[8]), "=r"(pa[9]), "=r"(pa[10]), "=r"(pa[11]), "=r"(pa[12]), "=r"(pa[13]), "=r"(pa[14]), "=r"(pa[15])
      : "r"(DP_t + c0));
  float4 l4[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) l4[u] = ls[(c0 >> 1) + u];  // broadcast reads, in flight with the tensor-memory loads
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  float x[16], d[16];
#pragma unroll
  for (int u = 0; u < 8; ++u)
    ffma2p(__uint_as_float(sa[2 * u]), __uint_as_float(sa[2 * u + 1]), sl2, l4[u].x, l4[u].y, x[2 * u], x[2 * u + 1]);
#pragma unroll
  for (int u = 0; u < 16; ++u) x[u] = ex2(x[u]);
  if (!full) {
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (c0 + u < qlo || c0 + u >= qhi) x[u] = 0.f;
  }
#pragma unroll
  for (int u = 0; u < 8; ++u)
    sub_mul2(__uint_as_float(pa[2 * u]), __uint_as_float(pa[2 * u + 1]), l4[u].z, l4[u].w, x[2 * u], x[2 * u + 1],
             d[2 * u], d[2 * u + 1]);
  uint32_t wp[8], wd[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    wp[u] = pack_bf16(x[2 * u], x[2 * u + 1]);
    wd[u] = pack_bf16(d[2 * u], d[2 * u + 1]);
  }
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(S_t + (c0 >> 1)),
               "r"(wp[0]), "r"(wp[1]), "r"(wp[2]), "r"(wp[3]), "r"(wp[4]), "r"(wp[5]), "r"(wp[6]), "r"(wp[7])
               : "memory");
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(DP_t + (c0 >> 1)),
               "r"(wd[0]), "r"(wd[1]), "r"(wd[2]), "r"(wd[3]), "r"(wd[4]), "r"(wd[5]), "r"(wd[6]), "r"(wd[7])
               : "memory");
  const int unit = c0 >> 3;  // 16-byte units of the 128-byte dS^T row
  *reinterpret_cast<uint4*>(ds + r * 128 + ((unit ^ (r & 7)) << 4)) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  *reinterpret_cast<uint4*>(ds + r * 128 + (((unit + 1) ^ (r & 7)) << 4)) = make_uint4(wd[4], wd[5], wd[6], wd[7]);
}

template <int D>
struct Lay2 {
  static constexpr int ST = 2;  // Q / dO stages
  static constexpr int TILE = 128 * D * 2;
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = TILE;
  static constexpr int Q_OFF = 2 * TILE;
  static constexpr int DO_OFF = Q_OFF + ST * TILE;
  static constexpr int DS_OFF = DO_OFF + ST * TILE;  // dS^T [128 keys x 128 queries] bf16, 2 x 16 KB
  // head_dim 64: the dQ drain stages 32 x 32 fp32 tiles for TMA bulk reduce-adds (2 x 4 KB per drain
  // warp); head_dim 128 has no room left and reduces with vector atomics
  static constexpr bool TMA_DQ = D == 64;
  static constexpr int DQST_OFF = DS_OFF + 32768;
  static constexpr int LSE_OFF = DQST_OFF + (TMA_DQ ? 32768 : 0);  // [2 warpgroups][32 pairs] float4
  static constexpr int BAR_OFF = LSE_OFF + 1024;
  static constexpr int BYTES = BAR_OFF + 256;  // head_dim 128: 224.25 KB, inside the 227 KB opt-in limit
  static_assert(BYTES + 1024 <= 232448, "shared memory above the 227 KB per-block limit");
  // tensor memory: S^T [0,128), dP^T [128,256), dV, dK, then (head_dim 64) two dQ buffers
  static constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 256 + D;
  static constexpr bool DQ_OWN = D == 64;  // head_dim 128: dQ reuses the S^T columns after the dV MMA
  __device__ static constexpr uint32_t dq_col(int i) { return DQ_OWN ? 384u + (uint32_t)(i & 1) * 64u : C_S; }
  // warpgroup w writes its 64 query columns as 32 packed columns at [64 w, 64 w + 32) of S^T / dP^T
  __device__ static constexpr uint32_t packed_col(int kk) { return kk < 4 ? kk * 8 : 64 + (kk - 4) * 8; }
};

template <int D>
__global__ void __launch_bounds__(512, 1)
    fmha_bwd2_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                     const __grid_constant__ CUtensorMap mdo2, const __grid_constant__ CUtensorMap mdq, Params p) {
  using L = Lay2<D>;
  constexpr int ST = L::ST;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* sp_full = bars + 5;
  uint64_t* ds_full = bars + 6;
  uint64_t* dq_full = bars + 7;
  uint64_t* dq_free = bars + 8;  // [2]: one per dQ buffer (a single barrier could run two phases ahead)
  uint64_t* kv_done = bars + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x % p.nkv_tiles;
  const int bh = blockIdx.x / p.nkv_tiles;
  const int b = bh / p.H, h = bh % p.H;
  const int kv0 = kt * 128;
  const int i0 = p.causal ? kv0 / 128 : 0;
  const int nq = (p.Sq + 127) / 128;
  const int ntile = nq - i0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(sp_full, 1);
    mbar_init(ds_full, 8);
    mbar_init(dq_full, 1);
    mbar_init(&dq_free[0], 4);
    mbar_init(&dq_free[1], 4);
    mbar_init(kv_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && ntile > 0) {
      mbar_expect_tx(kv_full, 2 * L::TILE);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma3(sm + L::K_OFF + c * 16384, &mk, kv_full, c * 64, kv0, bh);
        tma3(sm + L::V_OFF + c * 16384, &mv, kv_full, c * 64, kv0, bh);
      }
      for (int it = 0; it < ntile; ++it) {
        const int i = i0 + it, st = it % ST;
        if (!mbar_wait(&qdo_empty[st], ((it / ST) & 1) ^ 1, abort_flag, 61)) break;
        mbar_expect_tx(&qdo_full[st], 2 * L::TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          tma3(sm + L::Q_OFF + st * L::TILE + c * 16384, &mq, &qdo_full[st], c * 64, i * 128, bh);
          if (p.split > 0 && i * 128 >= p.split)
            tma4(sm + L::DO_OFF + st * L::TILE + c * 16384, &mdo2, &qdo_full[st], c * 64, h, i * 128 - p.split, b);
          else
            tma4(sm + L::DO_OFF + st * L::TILE + c * 16384, &mdo, &qdo_full[st], c * 64, h, i * 128, b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && ntile > 0) {
      const uint32_t id_kk = idesc(128, 128, 0, 0);  // S^T = K Q^T, dP^T = V dO^T
      const uint32_t id_kn = idesc(128, D, 0, 1);    // dV = P^T dO, dK = dS^T Q (A from tensor memory)
      const uint32_t id_nn = idesc(128, D, 1, 1);    // dQ = dS K (A = dS^T in SMEM read MN-major)
      const uint32_t ka = smem_u32(sm + L::K_OFF), va = smem_u32(sm + L::V_OFF);
      const uint32_t da = smem_u32(sm + L::DS_OFF);
      auto issue_sdp = [&](int it) {  // S^T_it and dP^T_it
        const uint32_t qa = smem_u32(sm + L::Q_OFF + (it % ST) * L::TILE);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + (it % ST) * L::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma(tmem + L::C_S, desc(ka + off, 16, 1024), desc(qa + off, 16, 1024), id_kk, kk > 0);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma(tmem + L::C_DP, desc(va + off, 16, 1024), desc(oa + off, 16, 1024), id_kk, kk > 0);
        }
        commit(sp_full);
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, 62) && mbar_wait(&qdo_full[0], 0, abort_flag, 63);
      if (ok) {
        fence_after();
        issue_sdp(0);
      }
      for (int it = 0; ok && it < ntile; ++it) {
        const int st = it % ST;
        if (!mbar_wait(ds_full, it & 1, abort_flag, 66)) break;
        fence_after();
        const uint32_t qa = smem_u32(sm + L::Q_OFF + st * L::TILE);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + st * L::TILE);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dV += P^T dO over 128 queries (8 packed columns per K=16 step)
          mma_ts(tmem + L::C_DV, tmem + L::C_S + L::packed_col(kk), desc(oa + kk * 2048, 16384, 1024), id_kn,
                 (it > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dK += dS^T Q
          mma_ts(tmem + L::C_DK, tmem + L::C_DP + L::packed_col(kk), desc(qa + kk * 2048, 16384, 1024), id_kn,
                 (it > 0 || kk > 0));
        // buffer it%2 was last used by tile it-2: wait for its drain (phase (it-2)/2 of that buffer's barrier)
        if (L::DQ_OWN && it >= 2 && !mbar_wait(&dq_free[it & 1], ((it >> 1) & 1) ^ 1, abort_flag, 64)) break;
        fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // dQ_it = dS K over 128 keys
          mma(tmem + L::dq_col(it), desc(da + kk * 2048, 16384, 1024), desc(ka + kk * 2048, 16384, 1024), id_nn,
              kk > 0);
        commit(dq_full);
        commit(&qdo_empty[st]);
        if (it + 1 < ntile) {
          if (!mbar_wait(&qdo_full[(it + 1) % ST], ((it + 1) / ST) & 1, abort_flag, 67)) break;
          if (!L::DQ_OWN && !mbar_wait(&dq_free[0], it & 1, abort_flag, 68)) break;  // dQ_it drained from S^T
          fence_after();
          issue_sdp(it + 1);
        } else {
          commit(kv_done);
        }
      }
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------------- gradient warpgroups
    // warpgroup g (0, 1) owns query columns [64 g, 64 g + 64) of every tile, one key row per thread
    const int g = (warp - 4) >> 2;
    const int tid = threadIdx.x - 128 - 128 * g;  // 0..127 within the warpgroup
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;
    const int kv = kv0 + r;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    uint8_t* ds = sm + L::DS_OFF;
    // per column pair (2i, 2i+1): {-lse_2i*log2e, -lse_2i+1*log2e, delta_2i, delta_2i+1}
    float* lsm = reinterpret_cast<float*>(sm + L::LSE_OFF) + g * 128;
    // one query column per thread (threads 0..63: -lse*log2e, 64..127: delta), fetched one tile ahead
    const int col = tid & 63;
    const int slot = (col >> 1) * 4 + (col & 1) + (tid < 64 ? 0 : 2);
    auto fetch = [&](int it) -> float {
      const int q = (i0 + it) * 128 + 64 * g + col;
      if (it >= ntile || q >= p.Sq) return tid < 64 ? -INFINITY : 0.f;
      return tid < 64 ? -p.lse[(int64_t)bh * p.Sq + q] * 1.4426950408889634f : p.delta[(int64_t)bh * p.Sq + q];
    };
    float pre = fetch(0);
    const float sl2 = p.scale_log2;
    bool ok = ntile > 0;
    for (int it = 0; ok && it < ntile; ++it) {
      named_bar(1 + g, 128);  // previous tile's readers of lsm are done
      lsm[slot] = pre;
      named_bar(1 + g, 128);  // this tile's values visible
      pre = fetch(it + 1);    // next tile's values load under this tile's math
      const int q0 = (i0 + it) * 128 + 64 * g;
      if (!mbar_wait(sp_full, it & 1, abort_flag, 69)) {
        ok = false;
        break;
      }
      fence_after();
      // visible query columns of this key row within the warpgroup's 64: [qlo, qhi)
      int qhi = kv < (p.kv_len ? min(p.Skv, __ldg(p.kv_len + bh / p.H)) : p.Skv) ? min(64, p.Sq - q0) : 0;
      int qlo = p.causal ? max(0, kv - q0) : 0;
      qhi = max(qhi, 0);
      if (qlo > qhi) qlo = qhi;
      const bool full = qlo == 0 && qhi == 64;
      const uint32_t S_t = tmem + L::C_S + lane_off + 64 * g;
      const uint32_t DP_t = tmem + L::C_DP + lane_off + 64 * g;
#pragma unroll 1
      for (int c0 = 0; c0 < 64; c0 += 16)  // 16 query columns at a time, phase by phase
        grad_chunk16(S_t, DP_t, c0, reinterpret_cast<const float4*>(lsm), sl2, full, qlo, qhi, ds + g * 16384, r);
      wait_st();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(ds_full);
    }
    if (g == 0 && ok && ntile > 0 && mbar_wait(kv_done, 0, abort_flag, 71)) {
      fence_after();
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float vv[32], kk[32];
        ld32(tmem + L::C_DV + lane_off + c * 32, vv);
        ld32(tmem + L::C_DK + lane_off + c * 32, kk);
        if (kv < p.Skv) {
          __nv_bfloat16* dvp = p.dv + ((int64_t)bh * p.Skv + kv) * D + c * 32;
          __nv_bfloat16* dkp = p.dk + ((int64_t)bh * p.Skv + kv) * D + c * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 8) {
            uint4 a, bq;
            a.x = pack_bf16(vv[j], vv[j + 1]);
            a.y = pack_bf16(vv[j + 2], vv[j + 3]);
            a.z = pack_bf16(vv[j + 4], vv[j + 5]);
            a.w = pack_bf16(vv[j + 6], vv[j + 7]);
            bq.x = pack_bf16(kk[j] * p.scale, kk[j + 1] * p.scale);
            bq.y = pack_bf16(kk[j + 2] * p.scale, kk[j + 3] * p.scale);
            bq.z = pack_bf16(kk[j + 4] * p.scale, kk[j + 5] * p.scale);
            bq.w = pack_bf16(kk[j + 6] * p.scale, kk[j + 7] * p.scale);
            *reinterpret_cast<uint4*>(dvp + j) = a;
            *reinterpret_cast<uint4*>(dkp + j) = bq;
          }
        }
      }
    } else if (g == 0 && ok && ntile == 0 && kv < p.Skv) {  // causal key tile past every query
      for (int j = 0; j < D; ++j) {
        p.dv[((int64_t)bh * p.Skv + kv) * D + j] = __float2bfloat16_rn(0.f);
        p.dk[((int64_t)bh * p.Skv + kv) * D + j] = __float2bfloat16_rn(0.f);
      }
    }
  } else if (warp >= 12) {
    // ---------------------------------------------------------------- dQ drain
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    uint8_t* stage = sm + L::DQST_OFF + (warp - 12) * 8192;
    int nchunk = 0;
    for (int it = 0; it < ntile; ++it) {
      if (!mbar_wait(dq_full, it & 1, abort_flag, 72)) break;
      fence_after();
      const int q = (i0 + it) * 128 + r;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        float v[32];
        ld32(tmem + L::dq_col(it) + lane_off + c * 32, v);
        if constexpr (L::TMA_DQ) {
          // 32 rows x 32 columns of this warp -> swizzled staging -> one bulk reduce-add into dQ_acc
          uint8_t* buf = stage + (nchunk & 1) * 4096;
          ++nchunk;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
          __syncwarp();
          uint8_t* rowp = buf + lane * 128;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(rowp + 16 * (u ^ (lane & 7))) =
                make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            asm volatile(
                "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                    &mdq),
                "r"(smem_u32(buf)), "r"(c * 32), "r"((i0 + it) * 128 + lane_base), "r"(bh)
                : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
        } else if (q < p.Sq) {
          float* dst = p.dq_acc + ((int64_t)bh * p.Sq + q) * D + c * 32;
#pragma unroll
          for (int j = 0; j < 32; j += 4) red_add_v4(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[L::DQ_OWN ? (it & 1) : 0]);
    }
    if (L::TMA_DQ && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}
}  // namespace v2


// ====================================================================================================
// Backward v3 (head_dim 64): 64-query blocks with double-buffered S^T / dP^T in tensor memory.
//
// One CTA per (128-key tile, head), 384 threads: warp 0 TMA (K, V once; Q_j, dO_j per 64-query block in a
// ring; lane-parallel staging of the block's -lse*log2e / Delta pairs), warp 1 TMEM allocator + MMA issuer,
// warps 4..7 gradient warps (one key row per thread, the block's 64 query columns), warps 8..11 dQ drain
// and the final dK / dV store.  Tensor memory (512 columns): S^T_b [64 b, 64 b + 64), dP^T_b
// [128 + 64 b, ...), dV [256, 320), dK [320, 384), dQ_c [384 + 64 c, ...) (c: pair parity).
// Per block j the MMA warp issues S^T_{j+2} / dP^T_{j+2} right behind dV_j / dK_j, into the buffers block j
// has just released, so the gradient warps' exponentials and products for block j+1 overlap the tensor
// core (v2 serialised them on one buffer).  dQ is computed for pairs of blocks (M = 128 queries) from the
// bf16 dS^T the gradient warps also write to shared memory (four 64-query slots, two pairs in flight), and
// drained with TMA bulk reduce-adds into the fp32 dQ accumulator.
// Barrier parities: ds_full[b] / sdp_full[b] carry block j at phase j >> 1 of buffer j & 1 (the producer of
// block j + 2 needs the consumer of block j first, so no barrier runs two phases ahead); dsfree / dq_full /
// dq_free carry pair q at phase q >> 1 of slot q & 1 under the same argument.
// version 4's per-block lse / Delta records: pair u of block j of row bh -> {-lse log2e, -lse log2e, Delta, Delta}
// for queries 64 j + 2u, + 1 (-inf / 0 past Sq)
__global__ void ls_record_kernel(const float* __restrict__ lse, const float* __restrict__ delta,
                                 float4* __restrict__ rec, int Sq, int nqb, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int u = (int)(i % 32);
  const int64_t bj = i / 32;
  const int j = (int)(bj % nqb);
  const int64_t bh = bj / nqb;
  const int q = j * 64 + 2 * u;
  const float* l = lse + bh * Sq;
  const float* d = delta + bh * Sq;
  float4 v;
  v.x = q < Sq ? -l[q] * 1.4426950408889634f : -INFINITY;
  v.y = q + 1 < Sq ? -l[q + 1] * 1.4426950408889634f : -INFINITY;
  v.z = q < Sq ? d[q] : 0.f;
  v.w = q + 1 < Sq ? d[q + 1] : 0.f;
  rec[i] = v;
}

namespace v3 {
using v2::ld32_nowait;
using v2::mma_ts;
using v2::pack_bf16;
using v2::st16;
using v2::wait_ld;
using v2::wait_st;

constexpr int BQ = 64;
constexpr int THREADS = 384;
constexpr int ST = 3;  // Q / dO stages
struct Lay3 {
  static constexpr int D = 64;
  static constexpr int KV_TILE = 128 * D * 2;        // K or V: 16 KB
  static constexpr int QB = BQ * D * 2;              // one Q or dO block: 8 KB
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = KV_TILE;
  static constexpr int Q_OFF = 2 * KV_TILE;
  static constexpr int DO_OFF = Q_OFF + ST * QB;
  static constexpr int DS_OFF = DO_OFF + ST * QB;    // 4 slots of dS^T [128 keys x 64 q] bf16 (16 KB each)
  static constexpr int DQST_OFF = DS_OFF + 4 * 16384;  // dQ drain staging: 4 warps x 2 x 4 KB
  static constexpr int LS_OFF = DQST_OFF + 32768;    // 2 x 32 float4 {-lse0 log2e, -lse1 log2e, d0, d1}
  static constexpr int BAR_OFF = LS_OFF + 2 * 32 * 16;
  static constexpr int BYTES = BAR_OFF + 256;
  static_assert(BYTES + 1024 <= 232448, "shared memory above the 227 KB per-block limit");
  static constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384;
};

__global__ void __launch_bounds__(THREADS, 1)
    fmha_bwd3_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                     const __grid_constant__ CUtensorMap mdo2, const __grid_constant__ CUtensorMap mdq, Params p) {
  using L = Lay3;
  constexpr int D = L::D;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;           // [ST]
  uint64_t* qdo_empty = qdo_full + ST;     // [ST]
  uint64_t* sdp_full = qdo_empty + ST;     // [2] S^T / dP^T of a block computed
  uint64_t* ds_full = sdp_full + 2;        // [2] P^T / dS^T of a block written (4 gradient warps)
  uint64_t* ls_full = ds_full + 2;         // [2] unused here: lse / Delta arrive with Q / dO
  uint64_t* dsfree = ls_full + 2;          // [2] the dQ MMA of a pair has read its dS^T slots
  uint64_t* dq_full = dsfree + 2;          // [2] dQ of a pair computed
  uint64_t* dq_free = dq_full + 2;         // [2] dQ of a pair drained (4 drain warps)
  uint64_t* kv_done = dq_free + 2;         // every MMA issued and complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float4* lsm = reinterpret_cast<float4*>(sm + L::LS_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x % p.nkv_tiles;
  const int bh = blockIdx.x / p.nkv_tiles;
  const int b = bh / p.H, h = bh % p.H;
  const int kv0 = kt * 128;
  const int j0 = p.causal ? kv0 / BQ : 0;  // even: kv0 is a multiple of 128
  const int nqb = (p.Sq + BQ - 1) / BQ;
  const int nblk = max(0, nqb - j0);
  const int npair = (nblk + 1) / 2;
  const int kvl = p.kv_len ? min(p.Skv, max(0, __ldg(p.kv_len + b))) : p.Skv;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < ST; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&ds_full[i], 4);
      mbar_init(&ls_full[i], 1);
      mbar_init(&dsfree[i], 1);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], 4);
    }
    mbar_init(kv_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer + lse / Delta staging
    if (nblk > 0) {
      if (lane == 0) {
        mbar_expect_tx(kv_full, 2 * L::KV_TILE);
        tma3(sm + L::K_OFF, &mk, kv_full, 0, kv0, bh);
        tma3(sm + L::V_OFF, &mv, kv_full, 0, kv0, bh);
      }
      for (int i = 0; i < nblk; ++i) {
        const int j = j0 + i, st = i % ST;
        const bool ok1 = mbar_wait(&qdo_empty[st], ((i / ST) & 1) ^ 1, abort_flag, 81);
        if (!ok1) break;
        if (lane == 0) {
          mbar_expect_tx(&qdo_full[st], 2 * L::QB);
          tma3(sm + L::Q_OFF + st * L::QB, &mq, &qdo_full[st], 0, j * BQ, bh);
          if (p.split > 0 && j * BQ >= p.split)
            tma4(sm + L::DO_OFF + st * L::QB, &mdo2, &qdo_full[st], 0, h, j * BQ - p.split, b);
          else
            tma4(sm + L::DO_OFF + st * L::QB, &mdo, &qdo_full[st], 0, h, j * BQ, b);
        }
        // slot i & 1 was last read by the gradient warps for block i - 2
        if (i >= 2 && !mbar_wait(&ds_full[i & 1], ((i >> 1) & 1) ^ 1, abort_flag, 82)) break;
        const int q = j * BQ + 2 * lane;
        float4 v;
        v.x = q < p.Sq ? -p.lse[(int64_t)bh * p.Sq + q] * 1.4426950408889634f : -INFINITY;
        v.y = q + 1 < p.Sq ? -p.lse[(int64_t)bh * p.Sq + q + 1] * 1.4426950408889634f : -INFINITY;
        v.z = q < p.Sq ? p.delta[(int64_t)bh * p.Sq + q] : 0.f;
        v.w = q + 1 < p.Sq ? p.delta[(int64_t)bh * p.Sq + q + 1] : 0.f;
        lsm[(i & 1) * 32 + lane] = v;
        __syncwarp();
        if (lane == 0) mbar_arrive(&ls_full[i & 1]);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && nblk > 0) {
      const uint32_t id_kq = idesc(128, BQ, 0, 0);  // S^T = K Q^T, dP^T = V dO^T  (M keys, N queries)
      const uint32_t id_kn = idesc(128, D, 0, 1);   // dV += P^T dO, dK += dS^T Q (A from tensor memory)
      const uint32_t id_nn = idesc(128, D, 1, 1);   // dQ = dS K (A = dS^T in SMEM read MN-major)
      const uint32_t ka = smem_u32(sm + L::K_OFF), va = smem_u32(sm + L::V_OFF);
      auto issue_sdp = [&](int i) {
        const uint32_t qa = smem_u32(sm + L::Q_OFF + (i % ST) * L::QB);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + (i % ST) * L::QB);
        const uint32_t cs = tmem + L::C_S + 64 * (i & 1), cdp = tmem + L::C_DP + 64 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma(cs, desc(ka + kk * 32, 16, 1024), desc(qa + kk * 32, 16, 1024), id_kq, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma(cdp, desc(va + kk * 32, 16, 1024), desc(oa + kk * 32, 16, 1024), id_kq, kk > 0);
        commit(&sdp_full[i & 1]);
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, 83);
      for (int i = 0; ok && i < 2 && i < nblk; ++i) {
        if (!(ok = mbar_wait(&qdo_full[i % ST], (i / ST) & 1, abort_flag, 84))) break;
        fence_after();
        issue_sdp(i);
      }
      for (int i = 0; ok && i < nblk; ++i) {
        const int st = i % ST;
        if (!mbar_wait(&ds_full[i & 1], (i >> 1) & 1, abort_flag, 85)) break;
        fence_after();
        const uint32_t qa = smem_u32(sm + L::Q_OFF + st * L::QB);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + st * L::QB);
        const uint32_t cs = tmem + L::C_S + 64 * (i & 1), cdp = tmem + L::C_DP + 64 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO over the block's 64 queries (8 packed columns / step)
          mma_ts(tmem + L::C_DV, cs + kk * 8, desc(oa + kk * 2048, 8192, 1024), id_kn, (i > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dK += dS^T Q
          mma_ts(tmem + L::C_DK, cdp + kk * 8, desc(qa + kk * 2048, 8192, 1024), id_kn, (i > 0 || kk > 0));
        commit(&qdo_empty[st]);
        if ((i & 1) || i + 1 == nblk) {  // dQ of the pair (blocks 2q, 2q + 1) over the 128 keys
          const int q = i >> 1, c = q & 1;
          if (q >= 2 && !mbar_wait(&dq_free[c], ((q >> 1) & 1) ^ 1, abort_flag, 86)) break;
          fence_after();
          const uint32_t da = smem_u32(sm + L::DS_OFF + c * 32768);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma(tmem + L::C_DQ + 64 * c, desc(da + kk * 2048, 16384, 1024), desc(ka + kk * 2048, 8192, 1024), id_nn,
                kk > 0);
          commit(&dq_full[c]);
          commit(&dsfree[c]);
        }
        if (i + 2 < nblk) {
          if (!mbar_wait(&qdo_full[(i + 2) % ST], ((i + 2) / ST) & 1, abort_flag, 87)) break;
          fence_after();
          issue_sdp(i + 2);
        }
      }
      if (ok) commit(kv_done);
    }
  } else if (warp >= 4 && warp < 8) {
    // ---------------------------------------------------------------- gradient warps: one key row per thread
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;
    const int kv = kv0 + r;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    const float sl2 = p.scale_log2;
    bool ok = nblk > 0;
    for (int i = 0; ok && i < nblk; ++i) {
      const int j = j0 + i;
      const int q0 = j * BQ;
      const int q = i >> 1, c = q & 1;
      // the pair's dS^T slots were last read by the dQ MMA of pair q - 2
      if (!(i & 1) && q >= 2 && !mbar_wait(&dsfree[c], ((q >> 1) & 1) ^ 1, abort_flag, 88)) {
        ok = false;
        break;
      }
      if (!mbar_wait(&ls_full[i & 1], (i >> 1) & 1, abort_flag, 89) ||
          !mbar_wait(&sdp_full[i & 1], (i >> 1) & 1, abort_flag, 90)) {
        ok = false;
        break;
      }
      fence_after();
      // visible query columns of this key row within the block: [qlo, qhi)
      int qhi = kv < kvl ? min(BQ, p.Sq - q0) : 0;
      int qlo = p.causal ? max(0, kv - q0) : 0;
      qhi = max(qhi, 0);
      if (qlo > qhi) qlo = qhi;
      const bool full = qlo == 0 && qhi == BQ;
      const uint32_t S_t = tmem + L::C_S + 64 * (i & 1) + lane_off;
      const uint32_t DP_t = tmem + L::C_DP + 64 * (i & 1) + lane_off;
      const float4* ls = lsm + (i & 1) * 32;
      uint8_t* ds = sm + L::DS_OFF + c * 32768 + (i & 1) * 16384;
#pragma unroll 1
      for (int c0 = 0; c0 < BQ; c0 += 16) v2::grad_chunk16(S_t, DP_t, c0, ls, sl2, full, qlo, qhi, ds, r);
      wait_st();
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[i & 1]);
    }
  } else if (warp >= 8) {
    // ---------------------------------------------------------------- dQ drain, then the dK / dV store
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    uint8_t* stage = sm + L::DQST_OFF + (warp - 8) * 8192;
    int nchunk = 0;
    bool ok = nblk > 0;
    for (int q = 0; ok && q < npair; ++q) {
      const int c = q & 1;
      if (!mbar_wait(&dq_full[c], (q >> 1) & 1, abort_flag, 91)) {
        ok = false;
        break;
      }
      fence_after();
      const int qrow0 = (j0 + 2 * q) * BQ;  // first query row of the pair
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t v[32];
        ld32_nowait(tmem + L::C_DQ + 64 * c + lane_off + cc * 32, v);
        wait_ld();
        uint8_t* buf = stage + (nchunk & 1) * 4096;
        ++nchunk;
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
        uint8_t* rowp = buf + lane * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(rowp + 16 * (u ^ (lane & 7))) =
              make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]), __uint_as_float(v[4 * u + 2]),
                          __uint_as_float(v[4 * u + 3]));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          // rows past Sq (the unused half of an odd last pair) are clipped by the tensor map
          asm volatile(
              "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(&mdq),
              "r"(smem_u32(buf)), "r"(cc * 32), "r"(qrow0 + lane_base), "r"(bh)
              : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[c]);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
    const int kv = kv0 + r;
    if (ok && nblk > 0 && mbar_wait(kv_done, 0, abort_flag, 92)) {
      fence_after();
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        float vv[32], kk[32];
        ld32(tmem + L::C_DV + lane_off + cc * 32, vv);
        ld32(tmem + L::C_DK + lane_off + cc * 32, kk);
        if (kv < p.Skv) {
          __nv_bfloat16* dvp = p.dv + ((int64_t)bh * p.Skv + kv) * D + cc * 32;
          __nv_bfloat16* dkp = p.dk + ((int64_t)bh * p.Skv + kv) * D + cc * 32;
#pragma unroll
          for (int jj = 0; jj < 32; jj += 8) {
            uint4 a, bq;
            a.x = pack_bf16(vv[jj], vv[jj + 1]);
            a.y = pack_bf16(vv[jj + 2], vv[jj + 3]);
            a.z = pack_bf16(vv[jj + 4], vv[jj + 5]);
            a.w = pack_bf16(vv[jj + 6], vv[jj + 7]);
            bq.x = pack_bf16(kk[jj] * p.scale, kk[jj + 1] * p.scale);
            bq.y = pack_bf16(kk[jj + 2] * p.scale, kk[jj + 3] * p.scale);
            bq.z = pack_bf16(kk[jj + 4] * p.scale, kk[jj + 5] * p.scale);
            bq.w = pack_bf16(kk[jj + 6] * p.scale, kk[jj + 7] * p.scale);
            *reinterpret_cast<uint4*>(dvp + jj) = a;
            *reinterpret_cast<uint4*>(dkp + jj) = bq;
          }
        }
      }
    } else if (nblk == 0 && kv < p.Skv) {  // causal key tile past every query: zero gradients
      for (int jj = 0; jj < D; ++jj) {
        p.dv[((int64_t)bh * p.Skv + kv) * D + jj] = __float2bfloat16_rn(0.f);
        p.dk[((int64_t)bh * p.Skv + kv) * D + jj] = __float2bfloat16_rn(0.f);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}
}  // namespace v3

// ------------------------------------------------------------------------------------ version 4
// Version 3 with the gradient math of a block split over two warpgroups (512 threads): warps 4-7 and 8-11
// each take 32 of the block's 64 query columns for the same 128 key rows (both warpgroups cover the four
// TMEM lane quadrants), so the exp2 / dS work per block runs on twice the warps; warps 12-15 drain dQ
// and store dK / dV.  Each warpgroup packs its bf16 P^T / dS^T into the first half of its own 32 fp32
// columns ([0, 16) and [32, 48)), never into columns the other warpgroup still reads; the dV / dK MMAs
// take their A operand from those two column ranges.  Shared-memory layout is version 3's.
namespace v4 {
using v3::Lay3;
// version 3's layout with ST Q / dO stages (three or five) and one 512-byte lse / Delta record per stage
template <int ST>
struct Lay4 {
  static constexpr int D = 64;
  static constexpr int KV_TILE = Lay3::KV_TILE, QB = Lay3::QB;
  static constexpr int K_OFF = 0, V_OFF = KV_TILE, Q_OFF = 2 * KV_TILE;
  static constexpr int DO_OFF = Q_OFF + ST * QB;
  static constexpr int DS_OFF = DO_OFF + ST * QB;      // 4 slots of dS^T [128 keys x 64 q] bf16
  static constexpr int DQST_OFF = DS_OFF + 4 * 16384;  // dQ drain staging: 4 warps x 2 x 4 KB
  static constexpr int LS_OFF = DQST_OFF + 32768;
  static constexpr int BAR_OFF = LS_OFF + ST * 512;
  static constexpr int BYTES = BAR_OFF + 256;
  static_assert(BYTES + 1024 <= 232448, "shared memory above the 227 KB per-block limit");
  static constexpr uint32_t C_S = Lay3::C_S, C_DP = Lay3::C_DP, C_DV = Lay3::C_DV, C_DK = Lay3::C_DK,
                            C_DQ = Lay3::C_DQ;
};
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
using v2::ld32_nowait;
using v2::mma_ts;
using v2::pack_bf16;
using v2::st16;
using v2::wait_ld;
using v2::wait_st;

constexpr int BQ = 64;
constexpr int THREADS = 512;


// event stamps of a traced launch (first 32 CTAs, first 64 query blocks, 16 event slots): SM clock per stamp
#define VO_TR(ev, blk)                                                                     \
  do {                                                                                      \
    if constexpr (TRACE) {                                                                  \
      if (blockIdx.x < 32 && (blk) < 64) p.trace[(blockIdx.x * 64 + (blk)) * 16 + (ev)] = clock64(); \
    }                                                                                       \
  } while (0)

// ALT: the two gradient warpgroups take alternate blocks (warps 4-7 even, 8-11 odd), all 64 columns each,
// so one warpgroup's exponential burst overlaps the other's wait for its next scores
template <int ST, bool TRACE = false, bool ALT = false>
__global__ void __launch_bounds__(THREADS, 1)
    fmha_bwd4_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mdo,
                     const __grid_constant__ CUtensorMap mdo2, const __grid_constant__ CUtensorMap mdq, Params p) {
  using L = Lay4<ST>;
  constexpr int D = L::D;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR_OFF);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;           // [ST]
  uint64_t* qdo_empty = qdo_full + ST;     // [ST]
  uint64_t* sdp_full = qdo_empty + ST;     // [2] S^T / dP^T of a block computed
  uint64_t* ds_full = sdp_full + 2;        // [2] P^T / dS^T of a block written (4 gradient warps)
  uint64_t* ls_full = ds_full + 2;         // [2] unused here: lse / Delta arrive with Q / dO
  uint64_t* dsfree = ls_full + 2;          // [2] the dQ MMA of a pair has read its dS^T slots
  uint64_t* dq_full = dsfree + 2;          // [2] dQ of a pair computed
  uint64_t* dq_free = dq_full + 2;         // [2] dQ of a pair drained (4 drain warps)
  uint64_t* kv_done = dq_free + 2;         // every MMA issued and complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(kv_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float4* lsm = reinterpret_cast<float4*>(sm + L::LS_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x % p.nkv_tiles;
  const int bh = blockIdx.x / p.nkv_tiles;
  const int b = bh / p.H, h = bh % p.H;
  const int kv0 = kt * 128;
  const int j0 = p.causal ? kv0 / BQ : 0;  // even: kv0 is a multiple of 128
  const int nqb = (p.Sq + BQ - 1) / BQ;
  const int nblk = max(0, nqb - j0);
  const int npair = (nblk + 1) / 2;
  const int kvl = p.kv_len ? min(p.Skv, max(0, __ldg(p.kv_len + b))) : p.Skv;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < ST; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sdp_full[i], 1);
      mbar_init(&ds_full[i], ALT ? 4 : 8);
      mbar_init(&ls_full[i], 1);
      mbar_init(&dsfree[i], 1);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_free[i], 4);
    }
    mbar_init(kv_done, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer + lse / Delta staging
    if (nblk > 0) {
      if (lane == 0) {
        mbar_expect_tx(kv_full, 2 * L::KV_TILE);
        tma3(sm + L::K_OFF, &mk, kv_full, 0, kv0, bh);
        tma3(sm + L::V_OFF, &mv, kv_full, 0, kv0, bh);
      }
      // Q, dO and the block's lse / Delta record arrive on one barrier per stage; the TMA warp never waits
      // on the gradient warps, so it runs up to three blocks ahead
      if (lane == 0) {
        const int nqb_all = (p.Sq + BQ - 1) / BQ;
        for (int i = 0; i < nblk; ++i) {
          const int j = j0 + i, st = i % ST;
          if (!mbar_wait(&qdo_empty[st], ((i / ST) & 1) ^ 1, abort_flag, 81)) break;
          VO_TR(0, i);
          mbar_expect_tx(&qdo_full[st], 2 * L::QB + 512);
          tma3(sm + L::Q_OFF + st * L::QB, &mq, &qdo_full[st], 0, j * BQ, bh);
          if (p.split > 0 && j * BQ >= p.split)
            tma4(sm + L::DO_OFF + st * L::QB, &mdo2, &qdo_full[st], 0, h, j * BQ - p.split, b);
          else
            tma4(sm + L::DO_OFF + st * L::QB, &mdo, &qdo_full[st], 0, h, j * BQ, b);
          bulk_load(sm + L::LS_OFF + st * 512, p.ls_rec + ((int64_t)bh * nqb_all + j) * 32, 512, &qdo_full[st]);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && nblk > 0) {
      const uint32_t id_kq = idesc(128, BQ, 0, 0);  // S^T = K Q^T, dP^T = V dO^T  (M keys, N queries)
      const uint32_t id_kn = idesc(128, D, 0, 1);   // dV += P^T dO, dK += dS^T Q (A from tensor memory)
      const uint32_t id_nn = idesc(128, D, 1, 1);   // dQ = dS K (A = dS^T in SMEM read MN-major)
      const uint32_t ka = smem_u32(sm + L::K_OFF), va = smem_u32(sm + L::V_OFF);
      auto issue_sdp = [&](int i) {
        const uint32_t qa = smem_u32(sm + L::Q_OFF + (i % ST) * L::QB);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + (i % ST) * L::QB);
        const uint32_t cs = tmem + L::C_S + 64 * (i & 1), cdp = tmem + L::C_DP + 64 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma(cs, desc(ka + kk * 32, 16, 1024), desc(qa + kk * 32, 16, 1024), id_kq, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma(cdp, desc(va + kk * 32, 16, 1024), desc(oa + kk * 32, 16, 1024), id_kq, kk > 0);
        commit(&sdp_full[i & 1]);
      };
      bool ok = mbar_wait(kv_full, 0, abort_flag, 83);
      for (int i = 0; ok && i < 2 && i < nblk; ++i) {
        if (!(ok = mbar_wait(&qdo_full[i % ST], (i / ST) & 1, abort_flag, 84))) break;
        fence_after();
        issue_sdp(i);
      }
      for (int i = 0; ok && i < nblk; ++i) {
        const int st = i % ST;
        if (!mbar_wait(&ds_full[i & 1], (i >> 1) & 1, abort_flag, 85)) break;
        VO_TR(1, i);
        fence_after();
        const uint32_t qa = smem_u32(sm + L::Q_OFF + st * L::QB);
        const uint32_t oa = smem_u32(sm + L::DO_OFF + st * L::QB);
        const uint32_t cs = tmem + L::C_S + 64 * (i & 1), cdp = tmem + L::C_DP + 64 * (i & 1);
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dV += P^T dO over the block's 64 queries (8 packed columns / step)
          mma_ts(tmem + L::C_DV, cs + kk * 8 + (ALT ? 0 : (kk >> 1) * 16), desc(oa + kk * 2048, 8192, 1024), id_kn,
                 (i > 0 || kk > 0));
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk)  // dK += dS^T Q
          mma_ts(tmem + L::C_DK, cdp + kk * 8 + (ALT ? 0 : (kk >> 1) * 16), desc(qa + kk * 2048, 8192, 1024), id_kn,
                 (i > 0 || kk > 0));
        commit(&qdo_empty[st]);
        VO_TR(2, i);
        if ((i & 1) || i + 1 == nblk) {  // dQ of the pair (blocks 2q, 2q + 1) over the 128 keys
          const int q = i >> 1, c = q & 1;
          if (q >= 2 && !mbar_wait(&dq_free[c], ((q >> 1) & 1) ^ 1, abort_flag, 86)) break;
          fence_after();
          const uint32_t da = smem_u32(sm + L::DS_OFF + c * 32768);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            mma(tmem + L::C_DQ + 64 * c, desc(da + kk * 2048, 16384, 1024), desc(ka + kk * 2048, 8192, 1024), id_nn,
                kk > 0);
          commit(&dq_full[c]);
          commit(&dsfree[c]);
        }
        if (i + 2 < nblk) {
          if (!mbar_wait(&qdo_full[(i + 2) % ST], ((i + 2) / ST) & 1, abort_flag, 87)) break;
          VO_TR(3, i);
          fence_after();
          issue_sdp(i + 2);
        }
      }
      if (ok) commit(kv_done);
    }
  } else if (warp >= 4 && warp < 12) {
    // ---------------------------------------------------------------- gradient warps: one key row per thread,
    // warps 4-7 take query columns [0, 32) of each block and warps 8-11 columns [32, 64)
    const int wg = (warp - 4) >> 2;
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;
    const int kv = kv0 + r;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    const float sl2 = p.scale_log2;
    bool ok = nblk > 0;
    for (int i = ALT ? wg : 0; ok && i < nblk; i += ALT ? 2 : 1) {
      const int j = j0 + i;
      const int q0 = j * BQ;
      const int q = i >> 1, c = q & 1;
      if (warp == 4 && lane == 0) VO_TR(4, i);
      // the pair's dS^T slots were last read by the dQ MMA of pair q - 2
      if ((ALT || !(i & 1)) && q >= 2 && !mbar_wait(&dsfree[c], ((q >> 1) & 1) ^ 1, abort_flag, 88)) {
        ok = false;
        break;
      }
      if (warp == 4 && lane == 0) VO_TR(5, i);
      if (!mbar_wait(&qdo_full[i % ST], (i / ST) & 1, abort_flag, 89) ||
          !mbar_wait(&sdp_full[i & 1], (i >> 1) & 1, abort_flag, 90)) {
        ok = false;
        break;
      }
      if (warp == 4 && lane == 0) VO_TR(6, i);
      fence_after();
      // visible query columns of this key row within the block: [qlo, qhi)
      int qhi = kv < kvl ? min(BQ, p.Sq - q0) : 0;
      int qlo = p.causal ? max(0, kv - q0) : 0;
      qhi = max(qhi, 0);
      if (qlo > qhi) qlo = qhi;
      const bool full = qlo == 0 && qhi == BQ;
      const uint32_t S_t = tmem + L::C_S + 64 * (i & 1) + lane_off;
      const uint32_t DP_t = tmem + L::C_DP + 64 * (i & 1) + lane_off;
      const float4* ls = lsm + (i % ST) * 32;
      uint8_t* ds = sm + L::DS_OFF + c * 32768 + (i & 1) * 16384;
if constexpr (ALT) {
#pragma unroll 1
        for (int c0 = 0; c0 < BQ; c0 += 16) v2::grad_chunk16(S_t, DP_t, c0, ls, sl2, full, qlo, qhi, ds, r);
      } else {  // this warpgroup's 32 query columns
        const int hf = wg;
        uint32_t sa[32], pa[32];
        ld32_nowait(S_t + hf * 32, sa);
        ld32_nowait(DP_t + hf * 32, pa);
        wait_ld();
        if (warp == 4 && lane == 0) VO_TR(10, i);
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int jj = 0; jj < 32; jj += 2) {
          const int qc = hf * 32 + jj;
          const float4 l4 = ls[qc >> 1];  // broadcast
          float x0, x1;
          v2::ffma2p(__uint_as_float(sa[jj]), __uint_as_float(sa[jj + 1]), sl2, l4.x, l4.y, x0, x1);
          float e0 = ex2(x0), e1 = ex2(x1);
          if (!full) {
            if (qc < qlo || qc >= qhi) e0 = 0.f;
            if (qc + 1 < qlo || qc + 1 >= qhi) e1 = 0.f;
          }
          float d0, d1;
          v2::sub_mul2(__uint_as_float(pa[jj]), __uint_as_float(pa[jj + 1]), l4.z, l4.w, e0, e1, d0, d1);
          wp[jj >> 1] = pack_bf16(e0, e1);
          wd[jj >> 1] = pack_bf16(d0, d1);
        }
        if (warp == 4 && lane == 0) VO_TR(11, i);
        // packed bf16 P^T / dS^T into the first half of this warpgroup's own 32 columns (already read)
        st16(S_t + hf * 32, wp);
        st16(DP_t + hf * 32, wd);
        // dS^T row r, query columns [32 hf, 32 hf + 32) of the block -> swizzled slot for the dQ MMA
#pragma unroll
        for (int u4 = 0; u4 < 4; ++u4) {
          const int unit = hf * 4 + u4;
          *reinterpret_cast<uint4*>(ds + r * 128 + ((unit ^ (r & 7)) << 4)) =
              make_uint4(wd[4 * u4], wd[4 * u4 + 1], wd[4 * u4 + 2], wd[4 * u4 + 3]);
        }
      }
      if (warp == 4 && lane == 0) VO_TR(12, i);
      wait_st();
      if (warp == 4 && lane == 0) VO_TR(13, i);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ds_full[i & 1]);
      if (warp == 4 && lane == 0) VO_TR(7, i);
    }
  } else if (warp >= 12) {
    // ---------------------------------------------------------------- dQ drain, then the dK / dV store
    const int lane_base = 32 * (warp & 3);
    const int r = lane_base + lane;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    uint8_t* stage = sm + L::DQST_OFF + (warp - 12) * 8192;
    int nchunk = 0;
    bool ok = nblk > 0;
    for (int q = 0; ok && q < npair; ++q) {
      const int c = q & 1;
      if (!mbar_wait(&dq_full[c], (q >> 1) & 1, abort_flag, 91)) {
        ok = false;
        break;
      }
      if (warp == 12 && lane == 0) VO_TR(8, 2 * q);
      fence_after();
      const int qrow0 = (j0 + 2 * q) * BQ;  // first query row of the pair
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t v[32];
        ld32_nowait(tmem + L::C_DQ + 64 * c + lane_off + cc * 32, v);
        wait_ld();
        uint8_t* buf = stage + (nchunk & 1) * 4096;
        ++nchunk;
        if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        __syncwarp();
        uint8_t* rowp = buf + lane * 128;
#pragma unroll
        for (int u = 0; u < 8; ++u)
          *reinterpret_cast<float4*>(rowp + 16 * (u ^ (lane & 7))) =
              make_float4(__uint_as_float(v[4 * u]), __uint_as_float(v[4 * u + 1]), __uint_as_float(v[4 * u + 2]),
                          __uint_as_float(v[4 * u + 3]));
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          // rows past Sq (the unused half of an odd last pair) are clipped by the tensor map
          asm volatile(
              "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(&mdq),
              "r"(smem_u32(buf)), "r"(cc * 32), "r"(qrow0 + lane_base), "r"(bh)
              : "memory");
          asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&dq_free[c]);
      if (warp == 12 && lane == 0) VO_TR(9, 2 * q);
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    __syncwarp();
    const int kv = kv0 + r;
    if (ok && nblk > 0 && mbar_wait(kv_done, 0, abort_flag, 92)) {
      fence_after();
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        float vv[32], kk[32];
        ld32(tmem + L::C_DV + lane_off + cc * 32, vv);
        ld32(tmem + L::C_DK + lane_off + cc * 32, kk);
        if (kv < p.Skv) {
          __nv_bfloat16* dvp = p.dv + ((int64_t)bh * p.Skv + kv) * D + cc * 32;
          __nv_bfloat16* dkp = p.dk + ((int64_t)bh * p.Skv + kv) * D + cc * 32;
#pragma unroll
          for (int jj = 0; jj < 32; jj += 8) {
            uint4 a, bq;
            a.x = pack_bf16(vv[jj], vv[jj + 1]);
            a.y = pack_bf16(vv[jj + 2], vv[jj + 3]);
            a.z = pack_bf16(vv[jj + 4], vv[jj + 5]);
            a.w = pack_bf16(vv[jj + 6], vv[jj + 7]);
            bq.x = pack_bf16(kk[jj] * p.scale, kk[jj + 1] * p.scale);
            bq.y = pack_bf16(kk[jj + 2] * p.scale, kk[jj + 3] * p.scale);
            bq.z = pack_bf16(kk[jj + 4] * p.scale, kk[jj + 5] * p.scale);
            bq.w = pack_bf16(kk[jj + 6] * p.scale, kk[jj + 7] * p.scale);
            *reinterpret_cast<uint4*>(dvp + jj) = a;
            *reinterpret_cast<uint4*>(dkp + jj) = bq;
          }
        }
      }
    } else if (nblk == 0 && kv < p.Skv) {  // causal key tile past every query: zero gradients
      for (int jj = 0; jj < D; ++jj) {
        p.dv[((int64_t)bh * p.Skv + kv) * D + jj] = __float2bfloat16_rn(0.f);
        p.dk[((int64_t)bh * p.Skv + kv) * D + jj] = __float2bfloat16_rn(0.f);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
  }
}
#undef VO_TR
}  // namespace v4

// Delta[bh, q] = sum_d dO[b, q, h, d] * O[b, q, h, d]
template <int D>
__global__ void delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dO,
                             const __nv_bfloat16* __restrict__ o2, const __nv_bfloat16* __restrict__ dO2, int split,
                             float* __restrict__ delta, int B, int Sq, int H) {
  constexpr int LPR = D / 8;  // lanes per row
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t row = gid / LPR;  // row over (b, q, h) token-major
  const int sub = gid % LPR;
  const int64_t rows = (int64_t)B * Sq * H;
  const int h = (int)(row % H);
  const int64_t bq = row / H;
  const int q = (int)(bq % Sq);
  const int b = (int)(bq / Sq);
  float s = 0.f;
  if (row < rows) {
    int64_t off;
    const __nv_bfloat16 *po = o, *pg = dO;
    if (split > 0 && q >= split) {
      off = (((int64_t)b * (Sq - split) + (q - split)) * H + h) * D;
      po = o2;
      pg = dO2;
    } else {
      off = (((int64_t)b * (split > 0 ? split : Sq) + q) * H + h) * D;
    }
    const uint4 a = *reinterpret_cast<const uint4*>(po + off + sub * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(pg + off + sub * 8);
    const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* hg = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float2 x = __bfloat1622float2(ha[t]), y = __bfloat1622float2(hg[t]);
      s += x.x * y.x + x.y * y.y;
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (row < rows && sub == 0) delta[((int64_t)b * H + h) * Sq + q] = s;
}

__global__ void dq_finalize_kernel(const float* __restrict__ acc, __nv_bfloat16* __restrict__ dq, int64_t n4,
                                   float scale) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 v = reinterpret_cast<const float4*>(acc)[i];
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x * scale, v.y * scale);
    __nv_bfloat162 b = __floats2bfloat162_rn(v.z * scale, v.w * scale);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    reinterpret_cast<uint2*>(dq)[i] = pk;
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
static int map3(CUtensorMap* m, const void* ptr, int BH, int S, int D, int rows = 128) {
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t str[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return (int)encode()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
// fp32 [BH, S, D] with box {32, 32, 1}, 128B swizzle (dQ accumulator, bulk reduce-add target)
static int map3_f32(CUtensorMap* m, const void* ptr, int BH, int S, int D) {
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t str[2] = {(cuuint64_t)D * 4, (cuuint64_t)S * D * 4};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return (int)encode()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(ptr), dims, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
// token-major [B, S, H, D] viewed as 4D {D, H, S, B}; box {64, 1, 128, 1}
static int map4_tok(CUtensorMap* m, const void* ptr, int B, int S, int H, int D, int rows = 128) {
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t str[3] = {(cuuint64_t)D * 2, (cuuint64_t)H * D * 2, (cuuint64_t)S * H * D * 2};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)rows, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return (int)encode()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(ptr), dims, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int D>
static int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                  const CUtensorMap& mdo2, Params p, int grid, cudaStream_t st) {
  static bool set = false;
  if (!set) {
    const cudaError_t e =
        cudaFuncSetAttribute(fmha_bwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay<D>::BYTES + 1024);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  fmha_bwd_kernel<D><<<grid, NUM_THREADS, Lay<D>::BYTES + 1024, st>>>(mq, mk, mv, mdo, mdo2, p);
  return (int)cudaGetLastError();
}

template <int D>
static int launch2(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                   const CUtensorMap& mdo2, const CUtensorMap& mdq, Params p, int grid, cudaStream_t st) {
  using L = v2::Lay2<D>;
  static bool set = false;
  if (!set) {
    const cudaError_t e =
        cudaFuncSetAttribute(v2::fmha_bwd2_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES + 1024);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  v2::fmha_bwd2_kernel<D><<<grid, 512, L::BYTES + 1024, st>>>(mq, mk, mv, mdo, mdo2, mdq, p);
  return (int)cudaGetLastError();
}

static int launch3(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                   const CUtensorMap& mdo2, const CUtensorMap& mdq, Params p, int grid, cudaStream_t st) {
  using L = v3::Lay3;
  static bool set = false;
  if (!set) {
    const cudaError_t e =
        cudaFuncSetAttribute(v3::fmha_bwd3_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES + 1024);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  v3::fmha_bwd3_kernel<<<grid, v3::THREADS, L::BYTES + 1024, st>>>(mq, mk, mv, mdo, mdo2, mdq, p);
  return (int)cudaGetLastError();
}

template <int ST, bool TRACE = false, bool ALT = false>
static int launch4(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mdo,
                   const CUtensorMap& mdo2, const CUtensorMap& mdq, Params p, int grid, cudaStream_t st) {
  using L = v4::Lay4<ST>;
  static bool set = false;
  if (!set) {
    const cudaError_t e = cudaFuncSetAttribute(v4::fmha_bwd4_kernel<ST, TRACE, ALT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES + 1024);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  v4::fmha_bwd4_kernel<ST, TRACE, ALT><<<grid, v4::THREADS, L::BYTES + 1024, st>>>(mq, mk, mv, mdo, mdo2, mdq, p);
  return (int)cudaGetLastError();
}

// traced launches (version 6) write their event stamps here
static long long* g_trace_buf = nullptr;
static constexpr size_t kTraceElems = 32 * 64 * 16;

}  // namespace vo_fbwd

// q [B,H,Sq,D], k/v [B,H,Skv,D], o/do [B,Sq,H,D], lse [B,H,Sq]; outputs dq [B,H,Sq,D], dk/dv [B,H,Skv,D].
// Scratch: delta [B*H*Sq] fp32 and dq_acc [B*H*Sq*D] fp32 (dq_acc must be zero on entry).
// o2 / dO2 / split: rows q >= split of O and dO live in separate [B, Sq - split, H, D] tensors
// (split % 128 == 0); split = 0: single O / dO.
extern "C" int vo_fmha_bwd(const void* q, const void* k, const void* v, const void* o, const void* dO,
                           const void* o2, const void* dO2, int split, const float* lse, void* dq, void* dk, void* dv,
                           float* delta, float* dq_acc, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                           cudaStream_t stream, int version, const int* kv_len) {
  using namespace vo_fbwd;
  if (D != 64 && D != 128) return -1;
  const int64_t rows = (int64_t)B * Sq * H;
  const int64_t threads = rows * (D / 8);
  if (D == 64)
    delta_kernel<64><<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)dO, (const __nv_bfloat16*)o2, (const __nv_bfloat16*)dO2, split,
        delta, B, Sq, H);
  else
    delta_kernel<128><<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
        (const __nv_bfloat16*)o, (const __nv_bfloat16*)dO, (const __nv_bfloat16*)o2, (const __nv_bfloat16*)dO2, split,
        delta, B, Sq, H);
  // versions 3-8 (head_dim 64): 64-query blocks (5 = 4 with a five-deep Q / dO ring; 6 = 4 traced: SM clock
  // stamps of the pipeline events, read back with vo_fmha_bwd_trace; 7 = gradient warpgroups on alternate
  // blocks; 8 = 7 traced); other widths run version 2
  if (version >= 3 && version <= 8 && D != 64) version = 2;
  const int qrows = (version >= 3 && version <= 8) ? 64 : 128;
  CUtensorMap mq, mk, mv, mdo;
  int r = map3(&mq, q, B * H, Sq, D, qrows);
  if (!r) r = map3(&mk, k, B * H, Skv, D);
  if (!r) r = map3(&mv, v, B * H, Skv, D);
  if (split < 0 || split >= Sq || split % 128 || (split > 0 && (!o2 || !dO2))) return -3;
  CUtensorMap mdo2;
  if (!r) r = map4_tok(&mdo, dO, B, split > 0 ? split : Sq, H, D, qrows);
  if (!r) r = split > 0 ? map4_tok(&mdo2, dO2, B, Sq - split, H, D, qrows) : map4_tok(&mdo2, dO, B, Sq, H, D, qrows);
  if (r) return r;
  Params p;
  p.kv_len = kv_len;
  p.Sq = Sq;
  p.Skv = Skv;
  p.H = H;
  p.nkv_tiles = (Skv + 127) / 128;
  p.causal = causal;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.dk = (__nv_bfloat16*)dk;
  p.dv = (__nv_bfloat16*)dv;
  p.split = split;
  const int grid = p.nkv_tiles * B * H;
  if (version >= 4 && version <= 8) {
    // records follow Delta in the caller's scratch, rounded up to 16 bytes
    float4* rec = reinterpret_cast<float4*>((reinterpret_cast<uintptr_t>(delta + (int64_t)B * H * Sq) + 15) &
                                            ~uintptr_t(15));
    const int nqb = (Sq + 63) / 64;
    const int64_t n = (int64_t)B * H * nqb * 32;
    ls_record_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(lse, delta, rec, Sq, nqb, n);
    p.ls_rec = rec;
  }
  if (version >= 3 && version <= 8) {
    CUtensorMap mdq;
    if ((r = map3_f32(&mdq, dq_acc, B * H, Sq, D))) return r;
    if (version == 6 || version == 8) {
      if (!g_trace_buf && cudaMalloc(&g_trace_buf, kTraceElems * sizeof(long long)) != cudaSuccess) return -4;
      cudaMemsetAsync(g_trace_buf, 0, kTraceElems * sizeof(long long), stream);
      p.trace = g_trace_buf;
    }
    r = version == 8   ? launch4<3, true, true>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream)
        : version == 7 ? launch4<3, false, true>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream)
        : version == 6 ? launch4<3, true>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream)
        : version == 5 ? launch4<5>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream)
        : version == 4 ? launch4<3>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream)
                       : launch3(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream);
  } else if (version == 2) {
    CUtensorMap mdq;
    if ((r = map3_f32(&mdq, dq_acc, B * H, Sq, D))) return r;
    r = D == 64 ? launch2<64>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream)
                : launch2<128>(mq, mk, mv, mdo, mdo2, mdq, p, grid, stream);
  }
  else {
    r = D == 64 ? launch<64>(mq, mk, mv, mdo, mdo2, p, grid, stream)
                : launch<128>(mq, mk, mv, mdo, mdo2, p, grid, stream);
  }
  if (r) return r;
  const int64_t n4 = (int64_t)B * H * Sq * D / 4;
  dq_finalize_kernel<<<(unsigned)((n4 + 255) / 256 < 4096 ? (n4 + 255) / 256 : 4096), 256, 0, stream>>>(
      dq_acc, (__nv_bfloat16*)dq, n4, scale);
  return (int)cudaGetLastError();
}

extern "C" int vo_fmha_bwd_error(int reset) {
  int e = 0;
  cudaMemcpyFromSymbol(&e, vo_fbwd::g_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(vo_fbwd::g_error, &z, sizeof(int));
  }
  return e;
}

// Copies the event stamps of the last traced backward launch ([32][64][16] SM clocks; 0 = not reached).
extern "C" int vo_fmha_bwd_trace(long long* host) {
  using namespace vo_fbwd;
  if (!g_trace_buf) return -1;
  return (int)cudaMemcpy(host, g_trace_buf, kTraceElems * sizeof(long long), cudaMemcpyDeviceToHost);
}
