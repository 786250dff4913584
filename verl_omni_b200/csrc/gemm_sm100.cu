// Persistent warp-specialised bf16 GEMM for sm_100a: TMA -> SMEM (128B swizzle) -> tcgen05.mma
// (cta_group::1, M=128, N=256, K=16 per instruction) -> TMEM fp32 accumulators (double buffered,
// 2 x 256 columns) -> tcgen05.ld epilogue with fused ops -> global memory.
//
//   C[M,N] (+)= sum_k A(m,k) * B(n,k)
//
// A and B are each either K-major (row-major [rows, K]) or MN-major (row-major [K, rows]); the
// smem descriptors and the instruction descriptor's major bits tell the tensor core which, so
// all three GEMMs of a linear layer (forward NT, dgrad NN, wgrad TN) run without transposes.
//
// Roles (192 threads):  warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer (one lane),
// warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31, i.e. tile rows).
// Every mbarrier wait is bounded (clock budget); on expiry the kernel records an error code,
// stops issuing work, releases TMEM and exits instead of hanging.
//
// Epilogues: NONE/BIAS (bf16 out), GELU (bf16 pre-activation + gelu_tanh out), GATE_RES
// (bf16 linear out + res + gate[row/S, n] * lin), F32_ACC (fp32 C += acc via vector reductions,
// used by wgrad with split-K over the token dimension).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

namespace vo_gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // one 128-byte swizzle row of bf16
constexpr int STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr unsigned long long WAIT_BUDGET = 8ull * 1000 * 1000 * 1000;  // ~4 s of SM clock

enum Epi : int { EPI_NONE = 0, EPI_BIAS = 1, EPI_GELU = 2, EPI_GATE_RES = 3, EPI_F32_ACC = 4 };

struct EpiParams {
  int epi;
  __nv_bfloat16* out;          // [M, N] bf16 (primary output)
  __nv_bfloat16* out2;         // GELU: pre-activation; GATE_RES: linear output (saved for backward)
  float* out_f32;              // F32_ACC: [M, N] fp32, accumulated
  const __nv_bfloat16* bias;   // [N] or null
  const __nv_bfloat16* gate;   // [M/S, gate_ld] (GATE_RES)
  const __nv_bfloat16* res;    // [M, N] (GATE_RES)
  int64_t gate_ld;
  int S;  // rows per sample (GATE_RES)
  int ldc;
};

__device__ int g_error = 0;

// ------------------------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase does not complete in budget.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > WAIT_BUDGET) {
      atomicCAS(&g_error, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
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
}

// Shared-memory matrix descriptor, SWIZZLE_128B, sm_100 version bits.
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= 1ull << 46;  // descriptor version (Blackwell)
  d |= 2ull << 61;  // SWIZZLE_128B
  return d;
}

// kind::f16 instruction descriptor: fp32 accumulate, bf16 A/B, M=128, N=256.
__host__ __device__ constexpr uint32_t make_idesc(int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float u = k0 * (x + k1 * x * x * x);
  float t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.f + t);
}

__device__ __forceinline__ void red_add_v4(float* addr, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

struct Shape {
  int M, N, K;
  int tiles_m, tiles_n, splits, k_blocks_per_split, total_k_blocks;
  int a_mn, b_mn;
};

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float* v, int ncols) {
  if (ncols == 32) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      uint4 pk;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[j + 2 * q], v[j + 2 * q + 1]);
      *reinterpret_cast<uint4*>(dst + j) = pk;
    }
  } else {
    for (int j = 0; j < ncols; ++j) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

// ------------------------------------------------------------------------------------ kernel
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Shape sh,
                EpiParams ep) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_a = smem;
  uint8_t* stage_b = smem + STAGES * A_STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 4);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_a) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_b) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;

  const int units = sh.tiles_m * sh.tiles_n * sh.splits;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const int split = u % sh.splits;
        const int tile = u / sh.splits;
        const int tm = tile / sh.tiles_n, tn = tile % sh.tiles_n;
        const int kb0 = split * sh.k_blocks_per_split;
        const int kb1 = min(sh.total_k_blocks, kb0 + sh.k_blocks_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sa = stage_a + stage * A_STAGE_BYTES;
          uint8_t* sb = stage_b + stage * B_STAGE_BYTES;
          const int k0 = kb * BK;
          if (sh.a_mn) {  // [K, M] row-major: two 64x64 boxes (M chunks)
            tma_load_2d(sa, &map_a, &full[stage], tm * BM, k0);
            tma_load_2d(sa + 8192, &map_a, &full[stage], tm * BM + 64, k0);
          } else {
            tma_load_2d(sa, &map_a, &full[stage], k0, tm * BM);
          }
          if (sh.b_mn) {  // [K, N] row-major: four 64x64 boxes (N chunks)
#pragma unroll
            for (int c = 0; c < 4; ++c) tma_load_2d(sb + c * 8192, &map_b, &full[stage], tn * BN + 64 * c, k0);
          } else {
            tma_load_2d(sb, &map_b, &full[stage], k0, tn * BN);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = make_idesc(sh.a_mn, sh.b_mn);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x, ++it) {
        const int split = u % sh.splits;
        const int kb0 = split * sh.k_blocks_per_split;
        const int kb1 = min(sh.total_k_blocks, kb0 + sh.k_blocks_per_split);
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, 2)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stage_a + stage * A_STAGE_BYTES);
          const uint32_t sb = smem_u32(stage_b + stage * B_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // K-major: advance 32 B inside the 128 B swizzle row; MN-major: advance 16 K-rows (2 atoms)
            const uint64_t ad = sh.a_mn ? make_desc(sa + k * 2048, 8192, 1024) : make_desc(sa + k * 32, 16, 1024);
            const uint64_t bd = sh.b_mn ? make_desc(sb + k * 2048, 8192, 1024) : make_desc(sb + k * 32, 16, 1024);
            tc_mma(tmem_d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&tfull[acc]);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int lane_base = 32 * (warp & 3);
    int it = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
      const int tile = u / sh.splits;
      const int tm = tile / sh.tiles_n, tn = tile % sh.tiles_n;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, 4)) break;
      tc_fence_after();
      const int row = tm * BM + lane_base + lane;
      const bool row_ok = row < sh.M;
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tc_ld_32x32b_x32(tmem_base + ((uint32_t)lane_base << 16) + acc * BN + c * 32, r);
        const int col0 = tn * BN + c * 32;
        if (!row_ok || col0 >= sh.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        const int ncols = min(32, sh.N - col0);
        if (ep.epi == EPI_F32_ACC) {
          float* dst = ep.out_f32 + (int64_t)row * ep.ldc + col0;
          if (ncols == 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) red_add_v4(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
            for (int j = 0; j < ncols; ++j) atomicAdd(dst + j, v[j]);
          }
          continue;
        }
        if (ep.bias) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += (j < ncols) ? __bfloat162float(ep.bias[col0 + j]) : 0.f;
        }
        __nv_bfloat16* dst = ep.out + (int64_t)row * ep.ldc + col0;
        if (ep.epi == EPI_GELU || ep.epi == EPI_GATE_RES) {
          store_bf16x32(ep.out2 + (int64_t)row * ep.ldc + col0, v, ncols);
          if (ep.epi == EPI_GELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(__bfloat162float(__float2bfloat16_rn(v[j])));
          } else {
            const __nv_bfloat16* g = ep.gate + (int64_t)(row / ep.S) * ep.gate_ld + col0;
            const __nv_bfloat16* rs = ep.res + (int64_t)row * ep.ldc + col0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < ncols) {
                const float lin = __bfloat162float(__float2bfloat16_rn(v[j]));
                v[j] = __bfloat162float(rs[j]) + __bfloat162float(g[j]) * lin;
              }
            }
          }
        }
        store_bf16x32(dst, v, ncols);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ------------------------------------------------------------------------------------ 2-SM variant
// A cluster of two CTAs on two SMs computes a 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256):
// CTA r loads its own 128 rows of A and its own 128 columns of B (plain TMA, no multicast) into the
// same SMEM offsets; only CTA 0 issues the MMAs, which read both CTAs' SMEM and write each CTA's TMEM
// (its 128 rows x 256 columns).  Per SM this moves 32 KB per 64-deep k-block instead of 48 KB for the
// same tensor work.  Both CTAs' TMA completions land on CTA 0's "full" barrier; MMA completions are
// multicast to both CTAs' barriers; the epilogue warps of both CTAs release an accumulator by arriving
// on CTA 0's "tmem empty" barrier.
constexpr int STAGES2 = 6;
constexpr int STAGE2_BYTES = 2 * BM * BK * 2;  // A 128x64 + B 128x64 per CTA = 32 KB
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + 1024 + 256;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to_rank0(uint32_t saddr) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(saddr));
  return r;
}
// non-.aligned forms: the single-lane producer / MMA loops leave warps diverged at the final sync
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive;\n\tbarrier.cluster.wait;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_rank0, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(bar_rank0), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tc_mma2(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void tc_commit2_both(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__host__ __device__ constexpr uint32_t make_idesc2(int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, Shape sh,
                   EpiParams ep) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES2 * STAGE2_BYTES);
  uint64_t* empty = full + STAGES2;
  uint64_t* tfull = empty + STAGES2;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_base_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_base_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 8);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_a) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&map_b) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_base_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_base_slot;
  const int units = sh.tiles_m * sh.tiles_n * sh.splits;  // tiles_m counts 256-row tiles here

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        const int split = u % sh.splits;
        const int tile = u / sh.splits;
        const int tm = tile / sh.tiles_n, tn = tile % sh.tiles_n;
        const int kb0 = split * sh.k_blocks_per_split;
        const int kb1 = min(sh.total_k_blocks, kb0 + sh.k_blocks_per_split);
        const int m0 = tm * 256 + (int)rank * 128, n0 = tn * BN + (int)rank * 128;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, 31)) {
            ok = false;
            break;
          }
          const uint32_t bar0 = map_to_rank0(smem_u32(&full[stage]));
          if (rank == 0) mbar_expect_tx(&full[stage], 2 * STAGE2_BYTES);
          uint8_t* sa = smem + stage * STAGE2_BYTES;
          uint8_t* sb = sa + BM * BK * 2;
          const int k0 = kb * BK;
          if (sh.a_mn) {
            tma_load_2d_pair(sa, &map_a, bar0, m0, k0);
            tma_load_2d_pair(sa + 8192, &map_a, bar0, m0 + 64, k0);
          } else {
            tma_load_2d_pair(sa, &map_a, bar0, k0, m0);
          }
          if (sh.b_mn) {
            tma_load_2d_pair(sb, &map_b, bar0, n0, k0);
            tma_load_2d_pair(sb + 8192, &map_b, bar0, n0 + 64, k0);
          } else {
            tma_load_2d_pair(sb, &map_b, bar0, k0, n0);
          }
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = make_idesc2(sh.a_mn, sh.b_mn);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs, ++it) {
        const int split = u % sh.splits;
        const int kb0 = split * sh.k_blocks_per_split;
        const int kb1 = min(sh.total_k_blocks, kb0 + sh.k_blocks_per_split);
        const int acc = it & 1;
        if (!mbar_wait(&tempty[acc], ((it >> 1) & 1) ^ 1, abort_flag, 32)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, 33)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * STAGE2_BYTES);
          const uint32_t sb = sa + BM * BK * 2;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = sh.a_mn ? make_desc(sa + k * 2048, 8192, 1024) : make_desc(sa + k * 32, 16, 1024);
            const uint64_t bd = sh.b_mn ? make_desc(sb + k * 2048, 8192, 1024) : make_desc(sb + k * 32, 16, 1024);
            tc_mma2(tmem_d, ad, bd, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          tc_commit2_both(&empty[stage]);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit2_both(&tfull[acc]);
      }
    }
  } else {
    const int lane_base = 32 * (warp & 3);
    const uint32_t tempty0[2] = {map_to_rank0(smem_u32(&tempty[0])), map_to_rank0(smem_u32(&tempty[1]))};
    int it = 0;
    for (int u = pair; u < units; u += npairs, ++it) {
      const int tile = u / sh.splits;
      const int tm = tile / sh.tiles_n, tn = tile % sh.tiles_n;
      const int acc = it & 1;
      if (!mbar_wait(&tfull[acc], (it >> 1) & 1, abort_flag, 34)) break;
      tc_fence_after();
      const int row = tm * 256 + (int)rank * 128 + lane_base + lane;
      const bool row_ok = row < sh.M;
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tc_ld_32x32b_x32(tmem_base + ((uint32_t)lane_base << 16) + acc * BN + c * 32, r);
        const int col0 = tn * BN + c * 32;
        if (!row_ok || col0 >= sh.N) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        const int ncols = min(32, sh.N - col0);
        if (ep.epi == EPI_F32_ACC) {
          float* dst = ep.out_f32 + (int64_t)row * ep.ldc + col0;
          if (ncols == 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) red_add_v4(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
            for (int j = 0; j < ncols; ++j) atomicAdd(dst + j, v[j]);
          }
          continue;
        }
        if (ep.bias) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += (j < ncols) ? __bfloat162float(ep.bias[col0 + j]) : 0.f;
        }
        __nv_bfloat16* dst = ep.out + (int64_t)row * ep.ldc + col0;
        if (ep.epi == EPI_GELU || ep.epi == EPI_GATE_RES) {
          store_bf16x32(ep.out2 + (int64_t)row * ep.ldc + col0, v, ncols);
          if (ep.epi == EPI_GELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(__bfloat162float(__float2bfloat16_rn(v[j])));
          } else {
            const __nv_bfloat16* g = ep.gate + (int64_t)(row / ep.S) * ep.gate_ld + col0;
            const __nv_bfloat16* rs = ep.res + (int64_t)row * ep.ldc + col0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < ncols) {
                const float lin = __bfloat162float(__float2bfloat16_rn(v[j]));
                v[j] = __bfloat162float(rs[j]) + __bfloat162float(g[j]) * lin;
              }
            }
          }
        }
        store_bf16x32(dst, v, ncols);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0[acc]);
    }
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS));
  }
}

// ------------------------------------------------------------------------------------ host side
typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                             CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// 2D bf16 tensor map over a row-major [rows, cols] matrix with row stride `ld` elements.
static int make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_cols,
                    int box_rows) {
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

static int g_num_sms = 0;
static int g_use_2sm = -1;

}  // namespace vo_gemm

// C-style launcher (no torch dependency).  Operand conventions:
//   a_mn == 0: A is row-major [M, K] (lda >= K);  a_mn == 1: A is row-major [K, M] (lda >= M)
//   b_mn == 0: B is row-major [N, K] (ldb >= K);  b_mn == 1: B is row-major [K, N] (ldb >= N)
// splits > 1 is only valid with EPI_F32_ACC (partial sums are reduced in global memory).
// Returns 0 on success, otherwise a CUDA / driver error code.
extern "C" int vo_gemm_launch(const void* A, const void* B, int M, int N, int K, int64_t lda, int64_t ldb, int a_mn,
                              int b_mn, int splits, vo_gemm::EpiParams ep, cudaStream_t stream) {
  using namespace vo_gemm;
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if ((lda * 2) % 16 || (ldb * 2) % 16) return -1;  // TMA strides must be 16-byte multiples
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) return -2;
  if (splits > 1 && ep.epi != EPI_F32_ACC) return -3;
  if (g_use_2sm < 0) {
    const char* e = getenv("VO_GEMM_2SM");
    g_use_2sm = (e && e[0] == '0') ? 0 : 1;
  }
  const bool two_sm = g_use_2sm && M >= 256;
  CUtensorMap ma, mb;
  int r;
  // 2-SM tiles load 128 rows of A and 128 columns of B per CTA
  if (a_mn)
    r = make_map(&ma, A, K, M, lda, 64, 64);
  else
    r = make_map(&ma, A, M, K, lda, 64, BM);
  if (r) return r;
  if (b_mn)
    r = make_map(&mb, B, K, N, ldb, 64, 64);
  else
    r = make_map(&mb, B, N, K, ldb, 64, two_sm ? 128 : BN);
  if (r) return r;
  if (!g_num_sms) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         STAGES * STAGE_BYTES + 1024 + 256);
    cudaFuncSetAttribute(gemm2sm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES);
    cudaFuncSetAttribute(gemm2sm_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  }
  Shape sh;
  sh.M = M;
  sh.N = N;
  sh.K = K;
  sh.tiles_m = two_sm ? (M + 255) / 256 : (M + BM - 1) / BM;
  sh.tiles_n = (N + BN - 1) / BN;
  sh.total_k_blocks = (K + BK - 1) / BK;
  splits = splits < 1 ? 1 : splits;
  if (splits > sh.total_k_blocks) splits = sh.total_k_blocks;
  sh.k_blocks_per_split = (sh.total_k_blocks + splits - 1) / splits;
  sh.splits = (sh.total_k_blocks + sh.k_blocks_per_split - 1) / sh.k_blocks_per_split;
  sh.a_mn = a_mn;
  sh.b_mn = b_mn;
  const int units = sh.tiles_m * sh.tiles_n * sh.splits;
  if (two_sm) {
    const int pairs = units < g_num_sms / 2 ? units : g_num_sms / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM2_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm2sm_kernel, ma, mb, sh, ep);
    return (int)e;
  }
  const int grid = units < g_num_sms ? units : g_num_sms;
  gemm_kernel<<<grid, NUM_THREADS, STAGES * STAGE_BYTES + 1024 + 256, stream>>>(ma, mb, sh, ep);
  return (int)cudaGetLastError();
}

extern "C" int vo_gemm_error(int reset) {
  int e = 0;
  cudaMemcpyFromSymbol(&e, vo_gemm::g_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(vo_gemm::g_error, &z, sizeof(int));
  }
  return e;
}
