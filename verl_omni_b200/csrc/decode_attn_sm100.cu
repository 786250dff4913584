// Grouped-query decode attention on the tcgen05 tensor cores (head_dim 128), one new query token per
// sequence against a contiguous or paged KV cache.
//
// Decode reads every cached K / V row once; the work per row is tiny, so the kernel is built to keep the
// copy engine (TMA) streaming and the issue slots free:
//   * one CTA per (sequence, KV head, key split); tiles of 128 keys, K and V staged by TMA (128B swizzle)
//     in a three-stage ring, paged caches resolved block by block through the block table (one warp reads
//     a tile's block ids in parallel, a tile ahead);
//   * S^T = K Q^T on the tensor core with the keys as M (128) and the query heads of the group as N (16,
//     zero-padded): 8 MMAs per tile, the 128 x 16 fp32 scores land in tensor memory, one key per lane;
//   * softmax warps (4 x 32 = 128 threads, thread = key) take per-head tile maxima with warp shuffles,
//     write the bf16 probabilities P^T [16 heads x 128 keys] to shared memory;
//   * O^T = V^T P^T on the tensor core (dims as M, V read MN-major from the same staged tile), one tile's
//     [128 dims x 16 heads] into tensor memory; the same warps (thread = dim) fold it into fp32 register
//     accumulators with the online-softmax rescale, so tensor memory never needs a read-modify-write;
//   * key splits write (max, sum, O) partials merged by the combine kernel of the CUDA-core path.
// Warp roles: 0-3 softmax / accumulate, 4 TMA producer, 5 TMEM allocator + MMA issuer.  The MMA issue
// order per tile is S(i+1) then PV(i), so the scores of the next tile are ready while softmax works.
// Every mbarrier wait is bounded; on timeout an error code is recorded and the CTA drains and exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dcheck.cuh"

namespace vo_dec {

constexpr int TK = 128;        // keys per tile (MMA M of S^T, K of O^T)
constexpr int HD = 128;        // head dim (MMA M of O^T)
constexpr int NH = 16;         // MMA N: query heads of one group, zero-padded
constexpr int NTHREADS = 192;  // warps 0-3 compute, 4 producer, 5 MMA
constexpr int STAGES = 3;     // K / V ring: three 64 KB tiles in flight per SM
constexpr int KV_BYTES = TK * HD * 2;  // K or V of one tile: 32 KB (two 16 KB swizzle atoms of 64 columns)
constexpr int STAGE_BYTES = 2 * KV_BYTES;
constexpr int Q_OFF = STAGES * STAGE_BYTES;      // Q: 16 rows x 128, K-major, two 2 KB atoms
constexpr int P_OFF = Q_OFF + 2 * 2048;          // P^T: two buffers of 16 rows x 128 keys (two 2 KB atoms)
constexpr int RED_OFF = P_OFF + 2 * 4096;        // per-warp head maxima, two tile parities: 2 x 4 x 16 floats
constexpr int MASK_OFF = RED_OFF + 2 * 4 * NH * 4;  // per stage: valid-row bitmask (4 words), zero-row bitmask (4)
constexpr int BAR_OFF = MASK_OFF + STAGES * 32;
constexpr int NBARS = 2 * STAGES + 10;
constexpr int SMEM_BYTES = BAR_OFF + NBARS * 8 + 16;
constexpr int S_COL = 0, O_COL = 32, TMEM_COLS = 64;
constexpr unsigned long long WAIT_BUDGET = 4ull * 1000 * 1000 * 1000;
constexpr uint32_t kSuspendNs = 100000;

__device__ int g_error = 0;

struct Params {
  const __nv_bfloat16* q;  // [B, Hk * rep, HD]
  const int* lens;         // [B]
  const int* table;        // [B, stride] block ids (paged) or null
  int stride, block, nblocks;
  int Hk, Lmax, splits;
  float scale_log2;
  __nv_bfloat16* out;  // [B, Hk * rep, HD] (splits == 1)
  float* part_o;       // [B, Hk, splits, rep, HD]
  float* part_ml;      // [B, Hk, splits, rep, 2]
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
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
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(par), "r"(kSuspendNs)
      : "memory");
  return ok != 0;
}
// bounded wait: false after the budget (error recorded, abort raised) or when another role aborted
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
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(b))
               : "memory");
}
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// K-major / MN-major shared-memory matrix descriptor, 128B swizzle (sm_100 descriptor version 1)
__device__ __forceinline__ uint64_t desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16 instruction descriptor: fp32 accumulate, bf16 A and B, A / B major-ness, N, M
__host__ __device__ constexpr uint32_t idesc(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// AND of `v` over the 128 compute threads (named barrier 1): a uniform continue / abort decision
__device__ __forceinline__ bool all_compute(bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v));
  return r != 0;
}
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }

template <int REP>
__global__ void __launch_bounds__(NTHREADS, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mv,
                     const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BAR_OFF);
  uint64_t* full = bars;                   // [STAGES] K / V of a tile landed (count 1 + tx)
  uint64_t* kv_empty = full + STAGES;      // [STAGES] PV of the stage's tile done (commit)
  uint64_t* s_full = kv_empty + STAGES;    // [2] scores in tensor memory (commit)
  uint64_t* s_empty = s_full + 2;          // [2] scores read (128 arrivals)
  uint64_t* p_full = s_empty + 2;          // [2] P^T written (128 arrivals)
  uint64_t* o_full = p_full + 2;           // [2] tile output in tensor memory (commit)
  uint64_t* o_empty = o_full + 2;          // [2] tile output read (128 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint32_t* mask = reinterpret_cast<uint32_t*>(sm + MASK_OFF);
  float* red = reinterpret_cast<float*>(sm + RED_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int bk = blockIdx.x, split = blockIdx.y;
  const int b = bk / p.Hk, kh = bk % p.Hk;
  const int cap = p.table ? p.stride * p.block : p.Lmax;
  VO_DCHECK(p.lens[b] >= 0 && p.lens[b] <= cap);  // checked builds record a clamped length
  const int L = max(0, min(p.lens[b], cap));
  // splits cover whole 128-key tiles: every tile starts on a block boundary of a paged cache
  const int per = ((L + p.splits - 1) / p.splits + TK - 1) / TK * TK;
  const int s0 = min(L, split * per), s1 = min(L, s0 + per);
  const int ntiles = (s1 - s0 + TK - 1) / TK;

  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 128);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mk) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mv) : "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (warp < 4) {
    // Q of the group as the B operand (16 rows x 128, K-major, 128B swizzle); padded rows are zero.  Both
    // P^T buffers start zeroed: rows of absent heads stay zero for the whole kernel.
    const __nv_bfloat16* qb = p.q + ((int64_t)b * p.Hk * REP + (int64_t)kh * REP) * HD;
    for (int u = tid; u < NH * (HD / 8); u += 128) {
      const int h = u / (HD / 8), c = u % (HD / 8);
      uint4 v = make_uint4(0, 0, 0, 0);
      if (h < REP) v = *reinterpret_cast<const uint4*>(qb + (int64_t)h * HD + c * 8);
      *reinterpret_cast<uint4*>(sm + Q_OFF + (c >> 3) * 2048 + h * 128 + (((c & 7) ^ (h & 7)) << 4)) = v;
    }
    for (int u = tid; u < 2 * 4096 / 16; u += 128) reinterpret_cast<uint4*>(sm + P_OFF)[u] = make_uint4(0, 0, 0, 0);
    fence_async_smem();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------------------ TMA producer (one warp)
    // Paged caches: lane j resolves block j of a tile (one table read per lane, all in flight at once) and,
    // once lane 0 has armed the stage's barrier, issues that block's copies; the next tile's ids are read
    // before the wait for its stage, so the table latency hides behind the ring.
    const int blk = p.table ? p.block : TK;
    const int nblk = TK / blk;
    auto read_id = [&](int i) {
      const int t = s0 + i * TK + lane * blk;
      if (i >= ntiles || lane >= nblk || t >= s1) return -2;  // no keys here
      return __ldg(p.table + (int64_t)b * p.stride + t / blk);
    };
    int id_next = p.table ? read_id(0) : -2;
    int issued = 0;
    for (int i = 0; i < ntiles; ++i) {
      const int kv = i % STAGES;
      const int id = id_next;
      bool ok = true;
      if (lane == 0) ok = mbar_wait(&kv_empty[kv], ((i / STAGES) & 1) ^ 1, abort_flag, 1);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      if (p.table) id_next = read_id(i + 1);
      const int t0 = s0 + i * TK;
      const int nvalid = min(TK, s1 - t0);
      uint8_t* sk = sm + kv * STAGE_BYTES;
      uint8_t* sv = sk + KV_BYTES;
      if (!p.table) {
        if (lane == 0) {
          for (int w = 0; w < 4; ++w) {
            const int lo = w * 32;
            mask[kv * 8 + w] = nvalid >= lo + 32 ? 0xffffffffu : nvalid <= lo ? 0u : (1u << (nvalid - lo)) - 1u;
            mask[kv * 8 + 4 + w] = 0u;
          }
          mbar_expect_tx(&full[kv], 2 * KV_BYTES);
          const int row = bk * p.Lmax + t0;
          for (int a = 0; a < HD / 64; ++a) {
            tma_load_2d(sk + a * (TK * 128), &mk, &full[kv], a * 64, row);
            tma_load_2d(sv + a * (TK * 128), &mv, &full[kv], a * 64, row);
          }
        }
      } else {
        const bool has = id != -2;                           // block holds keys of this split
        const bool in_pool = has && VO_DCHECK(id >= 0 && id < p.nblocks);  // out-of-pool ids read as zeros
        const unsigned load_mask = __ballot_sync(0xffffffffu, in_pool);
        const unsigned zero_mask = __ballot_sync(0xffffffffu, has && !in_pool);
        if (lane == 0) {
          // row bitmaps in closed form: valid = the first nvalid rows, zero = rows of out-of-pool blocks
          const uint32_t bmask = blk >= 32 ? 0xffffffffu : (1u << blk) - 1u;
          for (int w = 0; w < 4; ++w) {
            const int lo = w * 32;
            const uint32_t m = nvalid >= lo + 32 ? 0xffffffffu : nvalid <= lo ? 0u : (1u << (nvalid - lo)) - 1u;
            uint32_t z = 0u;
            for (int r = lo; r < lo + 32; r += blk < 32 ? blk : 32)
              if ((zero_mask >> (r / blk)) & 1u) z |= bmask << (r - lo);
            mask[kv * 8 + w] = m;
            mask[kv * 8 + 4 + w] = z & m;
          }
          mbar_expect_tx(&full[kv], (uint32_t)__popc(load_mask) * 2u * blk * HD * 2u);
        }
        __syncwarp();
        if (in_pool) {
          const int row = (id * p.Hk + kh) * blk;
          for (int a = 0; a < HD / 64; ++a) {
            tma_load_2d(sk + a * (TK * 128) + lane * blk * 128, &mk, &full[kv], a * 64, row);
            tma_load_2d(sv + a * (TK * 128) + lane * blk * 128, &mv, &full[kv], a * 64, row);
          }
        }
      }
      issued = i + 1;
    }
    // after an abort, let this producer's copies land before the CTA leaves (bounded)
    if (lane == 0 && *abort_flag) {
      for (int i = max(0, issued - STAGES); i < issued; ++i) {
        const unsigned long long t0 = clock64();
        while (!mbar_try_wait(&full[i % STAGES], (i / STAGES) & 1) && clock64() - t0 < WAIT_BUDGET) {
        }
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc(128, NH, 0, 0);  // S^T = K Q^T: A = K (K-major), B = Q (K-major)
      constexpr uint32_t id_o = idesc(128, NH, 1, 0);  // O^T = V^T P^T: A = V read MN-major, B = P^T (K-major)
      const uint32_t sbase = smem_u32(sm);
      bool ok = true;
      uint64_t* last_bar = nullptr;  // barrier of the latest commit: its completion covers every MMA issued
      uint32_t last_par = 0;
      auto issue_s = [&](int i) {
        const int kv = i % STAGES, sb = i & 1;
        const uint32_t sph = (i >> 1) & 1;
        if (!mbar_wait(&full[kv], (i / STAGES) & 1, abort_flag, 2) ||
            !mbar_wait(&s_empty[sb], sph ^ 1, abort_flag, 3))
          return false;
        fence_after();
        const uint32_t ka = sbase + kv * STAGE_BYTES, qa = sbase + Q_OFF;
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk)
          mma_ss(tmem + S_COL + sb * NH, desc(ka + (kk >> 2) * (TK * 128) + (kk & 3) * 32, 16, 1024),
                 desc(qa + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), id_s, kk > 0 ? 1u : 0u);
        commit(&s_full[sb]);
        last_bar = &s_full[sb];
        last_par = sph;
        return true;
      };
      auto issue_pv = [&](int i) {
        const int kv = i % STAGES, sb = i & 1;
        const uint32_t sph = (i >> 1) & 1;
        if (!mbar_wait(&p_full[sb], sph, abort_flag, 4) || !mbar_wait(&o_empty[sb], sph ^ 1, abort_flag, 5))
          return false;
        fence_after();
        const uint32_t va = sbase + kv * STAGE_BYTES + KV_BYTES, pa = sbase + P_OFF + sb * 4096;
#pragma unroll
        for (int kk = 0; kk < TK / 16; ++kk)
          mma_ss(tmem + O_COL + sb * NH, desc(va + kk * 2048, TK * 128, 1024),
                 desc(pa + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), id_o, kk > 0 ? 1u : 0u);
        commit(&o_full[sb]);
        commit(&kv_empty[kv]);
        last_bar = &kv_empty[kv];
        last_par = (i / STAGES) & 1;
        return true;
      };
      if (ntiles > 0) ok = issue_s(0);
      for (int i = 0; i < ntiles && ok; ++i) {
        if (i + 1 < ntiles) ok = issue_s(i + 1);
        if (ok) ok = issue_pv(i);
      }
      // every issued MMA must have completed before tensor memory is released (bounded)
      if (last_bar) {
        const unsigned long long t0 = clock64();
        while (!mbar_try_wait(last_bar, last_par) && clock64() - t0 < WAIT_BUDGET) {
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax / accumulate (warps 0-3)
    float m[REP], lpart[REP], acc[REP], alpha_pend[REP];
#pragma unroll
    for (int h = 0; h < REP; ++h) {
      m[h] = -INFINITY;
      lpart[h] = 0.f;
      acc[h] = 0.f;
      alpha_pend[h] = 1.f;
    }
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    auto fold_o = [&](int j) {  // thread = head-dim lane: acc = acc * alpha_j + O_j
      const int sj = j & 1;
      bool ok = mbar_wait(&o_full[sj], (j >> 1) & 1, abort_flag, 6);
      if (!all_compute(ok)) return false;
      fence_after();
      uint32_t r[16];
      ld16(trow + O_COL + sj * NH, r);
      fence_before();
      mbar_arrive(&o_empty[sj]);
#pragma unroll
      for (int h = 0; h < REP; ++h) acc[h] = fmaf(acc[h], alpha_pend[h], __uint_as_float(r[h]));
      return true;
    };
    bool ok = true;
    for (int i = 0; i < ntiles && ok; ++i) {
      const int kv = i % STAGES, sb = i & 1;
      ok = mbar_wait(&full[kv], (i / STAGES) & 1, abort_flag, 7) && mbar_wait(&s_full[sb], (i >> 1) & 1, abort_flag, 8);
      if (!all_compute(ok)) {
        ok = false;
        break;
      }
      fence_after();
      uint32_t r[16];
      ld16(trow + S_COL + sb * NH, r);
      fence_before();
      mbar_arrive(&s_empty[sb]);
      const bool valid = (mask[kv * 8 + (tid >> 5)] >> (tid & 31)) & 1u;
      const bool zero = (mask[kv * 8 + 4 + (tid >> 5)] >> (tid & 31)) & 1u;
      float s[REP];
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        s[h] = !valid ? -INFINITY : zero ? 0.f : __uint_as_float(r[h]) * p.scale_log2;
        float v = s[h];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (lane == 0) red[(sb * 4 + warp) * NH + h] = v;
      }
      compute_sync();
      __nv_bfloat16* pt = reinterpret_cast<__nv_bfloat16*>(sm + P_OFF + sb * 4096);
      const int kc = (tid & 63) >> 3, ke = tid & 7, katom = tid >> 6;
      float alpha_cur[REP];
#pragma unroll
      for (int h = 0; h < REP; ++h) {
        const float* rr = red + sb * 4 * NH + h;
        const float tmax = fmaxf(fmaxf(rr[0], rr[NH]), fmaxf(rr[2 * NH], rr[3 * NH]));
        const float mn = fmaxf(m[h], tmax);
        alpha_cur[h] = mn == -INFINITY ? 1.f : ex2(m[h] - mn);
        const float pv = s[h] == -INFINITY ? 0.f : ex2(s[h] - mn);
        lpart[h] = fmaf(lpart[h], alpha_cur[h], pv);
        m[h] = mn;
        pt[(katom * 2048 + h * 128 + ((kc ^ (h & 7)) << 4)) / 2 + ke] = __float2bfloat16_rn(pv);
      }
      if (!valid || zero) {  // rows past the range or of out-of-pool blocks: zero V (0 * garbage stays 0)
        uint4* vrow = reinterpret_cast<uint4*>(sm + kv * STAGE_BYTES + KV_BYTES + tid * 128);
#pragma unroll
        for (int a = 0; a < HD / 64; ++a)
#pragma unroll
          for (int c = 0; c < 8; ++c) vrow[a * (TK * 128 / 16) + c] = make_uint4(0, 0, 0, 0);
      }
      fence_async_smem();
      mbar_arrive(&p_full[sb]);
      if (i > 0 && !fold_o(i - 1)) {
        ok = false;
        break;
      }
#pragma unroll
      for (int h = 0; h < REP; ++h) alpha_pend[h] = alpha_cur[h];
    }
    if (ok && ntiles > 0) ok = fold_o(ntiles - 1);
    // row sums: per-thread partials over its keys -> per head
    compute_sync();
#pragma unroll
    for (int h = 0; h < REP; ++h) {
      float v = lpart[h];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane == 0) red[warp * NH + h] = v;
    }
    compute_sync();
    if (ok) {
      const int Hq = p.Hk * REP;
      if (p.splits == 1) {
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          const float l = red[h] + red[NH + h] + red[2 * NH + h] + red[3 * NH + h];
          p.out[((int64_t)b * Hq + (int64_t)kh * REP + h) * HD + tid] = __float2bfloat16_rn(l > 0.f ? acc[h] / l : 0.f);
        }
      } else {
        const int64_t pbase = (((int64_t)b * p.Hk + kh) * p.splits + split) * REP;
#pragma unroll
        for (int h = 0; h < REP; ++h) {
          p.part_o[(pbase + h) * HD + tid] = acc[h];
          if (tid == h) {
            p.part_ml[(pbase + h) * 2] = m[h];
            p.part_ml[(pbase + h) * 2 + 1] = red[h] + red[NH + h] + red[2 * NH + h] + red[3 * NH + h];
          }
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 5) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
static EncodeFn encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult qr;
    void* ptr = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &qr);
    fn = reinterpret_cast<EncodeFn>(ptr);
  }
  return fn;
}
// rows x 128 bf16 (row stride 256 B), box {64 columns, box_rows}, 128B swizzle, zero fill out of range
static int map_rows(CUtensorMap* m, const void* ptr, int64_t rows, int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)HD, (cuuint64_t)rows};
  cuuint64_t str[1] = {(cuuint64_t)HD * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return (int)encode()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int REP>
static int launch(const CUtensorMap& mk, const CUtensorMap& mv, const Params& p, int B, cudaStream_t stream) {
  static bool set = false;
  const int bytes = SMEM_BYTES + 1024;
  if (!set) {
    const cudaError_t e = cudaFuncSetAttribute(decode_tc_kernel<REP>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  decode_tc_kernel<REP><<<dim3(B * p.Hk, p.splits), NTHREADS, bytes, stream>>>(mk, mv, p);
  return (int)cudaGetLastError();
}

}  // namespace vo_dec

// Returns 0 on launch, -1 when the shape is outside the kernel (caller uses the CUDA-core path), or a CUDA /
// driver error code.  Caches: [B, Hk, Lmax, 128] (table == null) or block pools [nblocks, Hk, block, 128]
// with block a multiple of 8 dividing 128.  rep in {1, 2, 4, 8, 16}.
extern "C" int vo_decode_tc(const void* q, const void* kc, const void* vc, const int* lens, const int* table,
                            int stride, int block, int nblocks, int B, int Hk, int Lmax, int rep, int hd,
                            float scale_log2, int splits, void* out, float* part_o, float* part_ml,
                            cudaStream_t stream) {
  using namespace vo_dec;
  if (hd != HD || splits < 1 || B < 1 || Hk < 1) return -1;
  if (rep != 1 && rep != 2 && rep != 4 && rep != 8 && rep != 16) return -1;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15)
    return -1;
  CUtensorMap mk, mv;
  int64_t rows;
  int box;
  if (table) {
    if (block < 8 || block > TK || block % 8 || TK % block) return -1;
    rows = (int64_t)nblocks * Hk * block;
    box = block;
  } else {
    rows = (int64_t)B * Hk * Lmax;
    box = TK;
  }
  if (rows + TK >= (1ll << 31)) return -1;  // TMA row coordinates are 32-bit
  int e = map_rows(&mk, kc, rows, box);
  if (e) return e;
  e = map_rows(&mv, vc, rows, box);
  if (e) return e;
  Params p{reinterpret_cast<const __nv_bfloat16*>(q), lens, table, stride, block, nblocks, Hk, Lmax, splits,
           scale_log2, reinterpret_cast<__nv_bfloat16*>(out), part_o, part_ml};
  switch (rep) {
    case 1: return launch<1>(mk, mv, p, B, stream);
    case 2: return launch<2>(mk, mv, p, B, stream);
    case 4: return launch<4>(mk, mv, p, B, stream);
    case 8: return launch<8>(mk, mv, p, B, stream);
    default: return launch<16>(mk, mv, p, B, stream);
  }
}

// Reads (and with reset, clears) the first error code recorded by a bounded wait.
extern "C" int vo_decode_tc_error(int reset) {
  int h = 0;
  cudaMemcpyFromSymbol(&h, vo_dec::g_error, sizeof(int));
  if (reset && h) {
    const int z = 0;
    cudaMemcpyToSymbol(vo_dec::g_error, &z, sizeof(int));
  }
  return h;
}
