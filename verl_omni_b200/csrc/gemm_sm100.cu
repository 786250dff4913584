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
#include <string.h>

#include "gemm_api.h"

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

// waiting threads are suspended (up to this long, woken when the phase completes) instead of spinning: the
// epilogue warps wait for most of a tile's main loop and would otherwise take issue slots from the
// single-thread TMA producer and MMA issuer that share their SM sub-partitions
constexpr uint32_t kSuspendNs = 200000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendNs)
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


struct Shape {
  int M, N, K;
  int tiles_m, tiles_n, splits, k_blocks_per_split, total_k_blocks;
  int a_mn, b_mn;
  int kb_main;  // k-blocks [0, kb_main) come from (A, B), the rest from the extension operands (A2, B2)
  // Expert-grouped GEMMs (mixture-of-experts, 1-SM kernel only), tables in device memory:
  //   grp_mode 1 (forward / dgrad over expert-sorted rows padded to 128 per expert): grp_tab[m-tile] =
  //     expert of that 128-row tile (-1: unused tile, skipped); B rows are offset by expert * grp_stride;
  //   grp_mode 2 (weight gradient): units are (expert, output tile); the reduction runs over the expert's
  //     rows [grp_tab[e], grp_tab[e+1]) (multiples of 128) and output rows are offset by e * grp_stride.
  const int* grp_tab;
  int grp_mode, grp_stride, n_groups;
  int gather, gather_rows;  // operand gathered from tensor-parallel peers (GemmDesc::gather)
};

struct UnitInfo {
  int tm, tn, kb0, kb1, b_off, row_off;
  bool skip;
};

// Tensor-parallel gather: picks the peer's tensor map for the operand block that holds coordinate `x` of the
// gathered dimension and rebases `x` into that peer's buffer.
__device__ __forceinline__ const CUtensorMap* gather_map(const CUtensorMap* maps, int rows, int& x) {
  const int r = x / rows;
  x -= r * rows;
  return maps + r;
}

// Tile, k-block range and group offsets of one work unit (every role derives the same values).
__device__ __forceinline__ UnitInfo unit_info(const Shape& sh, int lu) {
  UnitInfo x;
  const int split = lu % sh.splits;
  int tile = lu / sh.splits;
  x.b_off = 0;
  x.row_off = 0;
  x.skip = false;
  if (sh.grp_mode == 2) {
    const int per = sh.tiles_m * sh.tiles_n;
    const int g = tile / per;
    tile -= g * per;
    x.kb0 = __ldg(sh.grp_tab + g) / BK;
    x.kb1 = __ldg(sh.grp_tab + g + 1) / BK;
    x.skip = x.kb1 <= x.kb0;
    x.row_off = g * sh.grp_stride;
  } else {
    x.kb0 = split * sh.k_blocks_per_split;
    x.kb1 = min(sh.total_k_blocks, x.kb0 + sh.k_blocks_per_split);
  }
  x.tm = tile / sh.tiles_n;
  x.tn = tile % sh.tiles_n;
  if (sh.grp_mode == 1) {
    const int g = __ldg(sh.grp_tab + x.tm);
    x.skip = g < 0;
    x.b_off = g * sh.grp_stride;
  }
  return x;
}

// Extension operands concatenated along the reduction: C = A B^T + A2 B2^T in one accumulation
// (the low-rank LoRA path: A2 = x A_lora^T, B2 = scale * B_lora), same majorness as A / B.
struct ExtMaps {
  CUtensorMap a2, b2;
};


// ------------------------------------------------------------------------------------ epilogue
// Each epilogue warp owns 32 accumulator rows and drains them 32 columns at a time: tcgen05.ld ->
// fused math in registers -> bf16 (or fp32) tile in a swizzled shared-memory staging buffer -> one
// TMA bulk store (or, for F32_ACC, a TMA bulk reduce-add) per 32 x 32 tile.  Two staging buffers per
// warp alternate so the next chunk is written while the previous store drains; bulk stores keep
// the L1/TEX pipe free for the TMA operand loads of the main loop.
constexpr int EPI_WARP_BYTES = 8192;              // 2 buffers x 4 KB per epilogue warp
constexpr int EPI_SMEM_BYTES = 4 * EPI_WARP_BYTES;  // 32 KB
constexpr int SMEM1_BYTES = STAGES * STAGE_BYTES + EPI_SMEM_BYTES + 1024 + 256;
static_assert(SMEM1_BYTES <= 232448, "shared memory above the 227 KB per-block limit");

struct EpiMaps {
  CUtensorMap out;   // bf16 [M, N], box {32, 32}, 64B swizzle
  CUtensorMap out2;  // bf16 [M, N] (GELU pre-activation / GATE_RES linear output)
  CUtensorMap acc;   // fp32 [M, N], box {32, 32}, 128B swizzle (F32_ACC)
};

// One GEMM of a launch.  A launch runs kMaxGroup problems at most; their work units are numbered
// consecutively (problem 0 first) and every role maps a unit to its problem with prob_of().
struct GatherMaps {
  CUtensorMap m[kMaxPeers];
};

struct Prob {
  CUtensorMap a, b;
  EpiMaps em;
  ExtMaps xm;
  GatherMaps gm;
  Shape sh;
  EpiParams ep;
  int unit_begin;
};
struct Launch {
  Prob p[kMaxGroup];
  int nprob;
  int units;
};

// Problem that owns work unit `u`; `local` = the unit's index inside that problem.  The launch lives
// in kernel-parameter space (__grid_constant__), so the reference is read in place, not copied.
// Problem index of work unit `u` (0 or 1) and the unit's index inside that problem.  Single-problem
// launches (GROUPED = false) fold to problem 0; grouped launches hold exactly two problems.  Fields are then
// read with PROB(field), a select between two compile-time parameter offsets, never a dynamic index into
// parameter space.
template <bool GROUPED>
__device__ __forceinline__ int prob_of(const Launch& L, int u, int& local) {
  if (!GROUPED) {
    local = u;
    return 0;
  }
  const int b1 = L.p[1].unit_begin;
  local = u >= b1 ? u - b1 : u;
  return u >= b1 ? 1 : 0;
}
#define PROB(field) (p ? L.p[1].field : L.p[0].field)
#define PROB_ADDR(field) (p ? &L.p[1].field : &L.p[0].field)

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map), "r"(src),
               "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(map),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// row `lane` of a 32 x 32 bf16 tile (64 B rows, 64B TMA swizzle: 16-byte unit u lands at u ^ ((row >> 1) & 3))
__device__ __forceinline__ void stage_bf16_row(uint8_t* buf, int lane, const float* v) {
  uint8_t* rowp = buf + lane * 64;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    uint4 pk;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
    for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[8 * u + 2 * q], v[8 * u + 2 * q + 1]);
    *reinterpret_cast<uint4*>(rowp + 16 * (u ^ ((lane >> 1) & 3))) = pk;
  }
}
// row `lane` of a 32 x 32 fp32 tile (128 B rows, 128B TMA swizzle: unit u lands at u ^ (row & 7))
__device__ __forceinline__ void stage_f32_row(uint8_t* buf, int lane, const float* v) {
  uint8_t* rowp = buf + lane * 128;
#pragma unroll
  for (int u = 0; u < 8; ++u)
    *reinterpret_cast<float4*>(rowp + 16 * (u ^ (lane & 7))) = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2],
                                                                           v[4 * u + 3]);
}

// Drains this warp's 32 rows x BN columns of one accumulator.  `tacc` = TMEM address of (row 0 of
// this warp, column 0 of the accumulator); rows [row0, row0 + 32), columns [col_base, col_base + BN).
// EPI_SCATTER: each lane stores its row's 32 columns (64 B) into the destination rank's buffer with plain
// 16-byte stores (peer memory over NVLink); `peers` points at the launch's parameter-space pointer table.
template <typename ShapeT>
__device__ __forceinline__ void epilogue_scatter(uint32_t tacc, int row0, int col_base, const ShapeT& sh,
                                                 const EpiParams& ep, __nv_bfloat16* const* peers, int lane) {
  const int row = row0 + lane;
  const bool row_ok = row < sh.M;
  const ScatterParams& sc = ep.sc;
  int64_t drow = 0;
  if (row_ok) {
    const int b = row / sc.seg_rows;
    drow = (int64_t)b * sc.dst_seq + sc.row_off + (row - b * sc.seg_rows);
  }
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    tc_ld_32x32b_x32(tacc + c * 32, r);
    const int col0 = col_base + c * 32;
    if (col0 >= sh.N || !row_ok) continue;  // col0 warp-uniform; a 32-column chunk never crosses a destination
    const int part = col0 / sc.part_cols, within = col0 - part * sc.part_cols;
    const int d = within / sc.dst_cols;
    const int dcol = part * sc.dst_cols + (within - d * sc.dst_cols);
    __nv_bfloat16* dst = peers[d] + drow * sc.dst_ld + dcol;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      uint4 pk;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a = __uint_as_float(r[8 * u + 2 * q]), b2 = __uint_as_float(r[8 * u + 2 * q + 1]);
        if (ep.bias) {
          a += __bfloat162float(ep.bias[col0 + 8 * u + 2 * q]);
          b2 += __bfloat162float(ep.bias[col0 + 8 * u + 2 * q + 1]);
        }
        h[q] = __floats2bfloat162_rn(a, b2);
      }
      *reinterpret_cast<uint4*>(dst + 8 * u) = pk;
    }
  }
}

// EPI_PEER_RED: each lane adds its row's 32 fp32 values into the owning rank's buffer (system-scope vector
// atomics over NVLink); `peers` points at the launch's parameter-space pointer table.
template <typename ShapeT>
__device__ __forceinline__ void epilogue_red(uint32_t tacc, int row0, int col_base, const ShapeT& sh,
                                             const EpiParams& ep, float* const* peers, int lane) {
  const int row = row0 + lane;
  const bool row_ok = row < sh.M;
  const int owner = row_ok ? row / ep.red_rows : 0;
  if (ep.red_store) {  // bf16 partial rows into this rank's slot of the owner's buffer: plain 16-byte stores
    __nv_bfloat16* dst =
        row_ok ? reinterpret_cast<__nv_bfloat16*>(peers[owner]) +
                     (int64_t)(ep.red_slot_off + row - owner * ep.red_rows) * ep.ldc
               : nullptr;
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tc_ld_32x32b_x32(tacc + c * 32, r);
      const int col0 = col_base + c * 32;
      if (col0 >= sh.N || !row_ok) continue;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        uint4 pk;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&pk);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          h[q] = __floats2bfloat162_rn(__uint_as_float(r[8 * u + 2 * q]), __uint_as_float(r[8 * u + 2 * q + 1]));
        *reinterpret_cast<uint4*>(dst + col0 + 8 * u) = pk;
      }
    }
    return;
  }
  float* base = row_ok ? peers[owner] + (int64_t)(row - owner * ep.red_rows) * ep.ldc : nullptr;
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    tc_ld_32x32b_x32(tacc + c * 32, r);
    const int col0 = col_base + c * 32;
    if (col0 >= sh.N || !row_ok) continue;  // N is a multiple of 32 (checked on the host)
#pragma unroll
    for (int j = 0; j < 8; ++j)
      atomicAdd_system(reinterpret_cast<float4*>(base + col0 + 4 * j),
                       make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
  }
}

template <typename ShapeT>
__device__ __forceinline__ void epilogue_rows(uint32_t tacc, int row0, int col_base, const ShapeT& sh,
                                              const EpiParams& ep, const EpiMaps& em, uint8_t* wbuf, int lane,
                                              int& nchunk) {
  const int row = row0 + lane;
  const bool row_ok = row < sh.M;
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t r[32];
    tc_ld_32x32b_x32(tacc + c * 32, r);
    const int col0 = col_base + c * 32;
    if (col0 >= sh.N) continue;  // warp-uniform
    const int ncols = min(32, sh.N - col0);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    uint8_t* buf = wbuf + (nchunk & 1) * 4096;
    ++nchunk;
    if (lane == 0) bulk_wait_read1();  // the store issued from this buffer two chunks ago has read it
    __syncwarp();
    if (ep.epi == EPI_F32_ACC) {
      stage_f32_row(buf, lane, v);
    } else {
      if (ep.bias) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] += (j < ncols) ? __bfloat162float(ep.bias[col0 + j]) : 0.f;
      }
      if (ep.epi == EPI_GELU || ep.epi == EPI_GATE_RES) {
        stage_bf16_row(buf + 2048, lane, v);
        if (ep.epi == EPI_GELU) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = gelu_tanh(__bfloat162float(__float2bfloat16_rn(v[j])));
        } else if (row_ok) {
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
      stage_bf16_row(buf, lane, v);
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (ep.epi == EPI_F32_ACC) {
        tma_reduce_add_2d(&em.acc, smem_u32(buf), col0, row0);
      } else {
        tma_store_2d(&em.out, smem_u32(buf), col0, row0);
        if (ep.epi == EPI_GELU || ep.epi == EPI_GATE_RES) tma_store_2d(&em.out2, smem_u32(buf + 2048), col0, row0);
      }
      bulk_commit();
    }
  }
}

// ------------------------------------------------------------------------------------ kernel
template <bool GROUPED>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_kernel(const __grid_constant__ Launch L) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_a = smem;
  uint8_t* stage_b = smem + STAGES * A_STAGE_BYTES;
  uint8_t* epi_stage = smem + STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_SMEM_BYTES);
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
    for (int q = 0; q < L.nprob; ++q) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&L.p[q].a) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&L.p[q].b) : "memory");
    }
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

  const int units = L.units;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int lu;
        const int p = prob_of<GROUPED>(L, u, lu);
        const Shape sh = PROB(sh);
        const UnitInfo ui = unit_info(sh, lu);
        if (ui.skip) continue;
        const int tm = ui.tm, tn = ui.tn;
        for (int kb = ui.kb0; kb < ui.kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sa = stage_a + stage * A_STAGE_BYTES;
          uint8_t* sb = stage_b + stage * B_STAGE_BYTES;
          const bool ext = kb >= sh.kb_main;
          const CUtensorMap* ma = ext ? PROB_ADDR(xm.a2) : PROB_ADDR(a);
          const CUtensorMap* mb = ext ? PROB_ADDR(xm.b2) : PROB_ADDR(b);
          const int k0 = (ext ? kb - sh.kb_main : kb) * BK;
          int am = tm * BM, ak = k0, bk = k0;
          if (sh.gather == 1) ma = gather_map(PROB(gm.m), sh.gather_rows, am);
          else if (sh.gather == 2) ma = gather_map(PROB(gm.m), sh.gather_rows, ak);
          else if (sh.gather == 3) mb = gather_map(PROB(gm.m), sh.gather_rows, bk);
          if (sh.a_mn) {  // [K, M] row-major: two 64x64 boxes (M chunks)
            tma_load_2d(sa, ma, &full[stage], am, ak);
            tma_load_2d(sa + 8192, ma, &full[stage], am + 64, ak);
          } else {
            tma_load_2d(sa, ma, &full[stage], ak, am);
          }
          if (sh.b_mn) {  // [K, N] row-major: four 64x64 boxes (N chunks)
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_2d(sb + c * 8192, mb, &full[stage], tn * BN + 64 * c, ui.b_off + bk);
          } else {
            tma_load_2d(sb, mb, &full[stage], bk, ui.b_off + tn * BN);
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
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int lu;
        const int p = prob_of<GROUPED>(L, u, lu);
        const Shape sh = PROB(sh);
        const UnitInfo ui = unit_info(sh, lu);
        if (ui.skip) continue;
        const int kb0 = ui.kb0, kb1 = ui.kb1;
        const uint32_t idesc = make_idesc(sh.a_mn, sh.b_mn);
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
        ++it;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int lane_base = 32 * (warp & 3);
    uint8_t* wbuf = epi_stage + (warp - 2) * EPI_WARP_BYTES;
    int it = 0, nchunk = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      int lu;
      const int p = prob_of<GROUPED>(L, u, lu);
      const Shape sh = PROB(sh);
      const UnitInfo ui = unit_info(sh, lu);
      if (ui.skip) continue;
      const int tm = ui.tm, tn = ui.tn;
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, 4)) break;
      tc_fence_after();
      const EpiParams ep = PROB(ep);
      if (ep.epi == EPI_SCATTER)
        epilogue_scatter(tmem_base + ((uint32_t)lane_base << 16) + acc * BN, tm * BM + lane_base, tn * BN, sh, ep,
                         PROB(ep.sc.peers), lane);
      else if (ep.epi == EPI_PEER_RED)
        epilogue_red(tmem_base + ((uint32_t)lane_base << 16) + acc * BN, tm * BM + lane_base, tn * BN, sh, ep,
                     PROB(ep.red_peers), lane);
      else
        epilogue_rows(tmem_base + ((uint32_t)lane_base << 16) + acc * BN, ui.row_off + tm * BM + lane_base, tn * BN,
                      sh, ep, *PROB_ADDR(em), wbuf, lane, nchunk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      ++it;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
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
constexpr int SMEM2_BYTES = STAGES2 * STAGE2_BYTES + EPI_SMEM_BYTES + 1024 + 256;
static_assert(SMEM2_BYTES <= 232448, "shared memory above the 227 KB per-block limit");

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

template <bool GROUPED>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm2sm_kernel(const __grid_constant__ Launch L) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* epi_stage = smem + STAGES2 * STAGE2_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi_stage + EPI_SMEM_BYTES);
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
    for (int q = 0; q < L.nprob; ++q) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&L.p[q].a) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&L.p[q].b) : "memory");
    }
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
  const int units = L.units;  // tiles_m counts 256-row tiles in the 2-SM kernel

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        int lu;
        const int p = prob_of<GROUPED>(L, u, lu);
        const Shape sh = PROB(sh);
        const int split = lu % sh.splits;
        const int tile = lu / sh.splits;
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
          const bool ext = kb >= sh.kb_main;
          const CUtensorMap* ma = ext ? PROB_ADDR(xm.a2) : PROB_ADDR(a);
          const CUtensorMap* mb = ext ? PROB_ADDR(xm.b2) : PROB_ADDR(b);
          const int k0 = (ext ? kb - sh.kb_main : kb) * BK;
          int am = m0, ak = k0, bk = k0;
          if (sh.gather == 1) ma = gather_map(PROB(gm.m), sh.gather_rows, am);
          else if (sh.gather == 2) ma = gather_map(PROB(gm.m), sh.gather_rows, ak);
          else if (sh.gather == 3) mb = gather_map(PROB(gm.m), sh.gather_rows, bk);
          if (sh.a_mn) {
            tma_load_2d_pair(sa, ma, bar0, am, ak);
            tma_load_2d_pair(sa + 8192, ma, bar0, am + 64, ak);
          } else {
            tma_load_2d_pair(sa, ma, bar0, ak, am);
          }
          if (sh.b_mn) {
            tma_load_2d_pair(sb, mb, bar0, n0, bk);
            tma_load_2d_pair(sb + 8192, mb, bar0, n0 + 64, bk);
          } else {
            tma_load_2d_pair(sb, mb, bar0, bk, n0);
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
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs, ++it) {
        int lu;
        const int p = prob_of<GROUPED>(L, u, lu);
        const Shape sh = PROB(sh);
        const int split = lu % sh.splits;
        const int kb0 = split * sh.k_blocks_per_split;
        const int kb1 = min(sh.total_k_blocks, kb0 + sh.k_blocks_per_split);
        const uint32_t idesc = make_idesc2(sh.a_mn, sh.b_mn);
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
    uint8_t* wbuf = epi_stage + (warp - 2) * EPI_WARP_BYTES;
    int it = 0, nchunk = 0;
    for (int u = pair; u < units; u += npairs, ++it) {
      int lu;
      const int p = prob_of<GROUPED>(L, u, lu);
      const Shape sh = PROB(sh);
      const int tile = lu / sh.splits;
      const int tm = tile / sh.tiles_n, tn = tile % sh.tiles_n;
      const int acc = it & 1;
      if (!mbar_wait(&tfull[acc], (it >> 1) & 1, abort_flag, 34)) break;
      tc_fence_after();
      const EpiParams ep = PROB(ep);
      if (ep.epi == EPI_SCATTER)
        epilogue_scatter(tmem_base + ((uint32_t)lane_base << 16) + acc * BN, tm * 256 + (int)rank * 128 + lane_base,
                         tn * BN, sh, ep, PROB(ep.sc.peers), lane);
      else if (ep.epi == EPI_PEER_RED)
        epilogue_red(tmem_base + ((uint32_t)lane_base << 16) + acc * BN, tm * 256 + (int)rank * 128 + lane_base,
                     tn * BN, sh, ep, PROB(ep.red_peers), lane);
      else
        epilogue_rows(tmem_base + ((uint32_t)lane_base << 16) + acc * BN, tm * 256 + (int)rank * 128 + lane_base,
                      tn * BN, sh, ep, *PROB_ADDR(em), wbuf, lane, nchunk);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(tempty0[acc]);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
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

// 2D tensor map for an epilogue output: [rows, cols] with row stride `ld` elements, 32 x 32 box.
static int make_out_map(CUtensorMap* m, const void* ptr, bool f32, int64_t rows, int64_t cols, int64_t ld) {
  const int esz = f32 ? 4 : 2;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * esz)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                            const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)r;
}

static int g_num_sms = 0;
static int g_use_2sm = -1;

// Fills one problem of a launch (tensor maps, tile shape, epilogue); 0 or an error code.
static int build_prob(const GemmDesc& d, bool two_sm, Prob* P) {
  memset(P, 0, sizeof(Prob));
  const bool has_ext = d.A2 != nullptr && d.B2 != nullptr && d.K2 > 0;
  const EpiParams& ep = d.ep;
  if ((d.lda * 2) % 16 || (d.ldb * 2) % 16) return -1;  // TMA strides must be 16-byte multiples
  if ((reinterpret_cast<uintptr_t>(d.A) | reinterpret_cast<uintptr_t>(d.B)) & 15) return -2;
  const bool a_gathered = d.gather == 1 || d.gather == 2, b_gathered = d.gather == 3;
  if (d.gather < 0 || d.gather > 3) return -9;
  if (d.gather) {
    // whole tiles per peer block: 128 rows of A (gather 1) or 64-row k-blocks (gather 2 / 3)
    const int unit = d.gather == 1 ? BM : BK;
    const int total = d.gather == 1 ? d.M : d.K;
    if (d.gather_n < 1 || d.gather_n > kMaxPeers || d.gather_rows <= 0 || d.gather_rows % unit ||
        d.gather_rows * d.gather_n != total || d.A2 || d.grp_mode || (d.gather == 1 && d.a_mn) ||
        (d.gather == 2 && !d.a_mn) || (d.gather == 3 && !d.b_mn))
      return -9;
    for (int i = 0; i < d.gather_n; ++i)
      if (!d.gather_ptrs[i] || (reinterpret_cast<uintptr_t>(d.gather_ptrs[i]) & 15)) return -9;
  }
  if (d.splits > 1 && ep.epi != EPI_F32_ACC) return -3;
  int r;
  // epilogue outputs go out through TMA: 16-byte aligned bases and row strides
  if (ep.epi == EPI_PEER_RED) {
    if (ep.red_rows <= 0 || d.N % 32 || (ep.ldc * (ep.red_store ? 2 : 4)) % 16 || ep.ldc < d.N ||
        ep.red_slot_off < 0)
      return -10;
    const int owners = (d.M + ep.red_rows - 1) / ep.red_rows;
    if (owners > kMaxPeers) return -10;
    for (int i = 0; i < owners; ++i)
      if (!ep.red_peers[i] || (reinterpret_cast<uintptr_t>(ep.red_peers[i]) & 15)) return -10;
  } else if (ep.epi == EPI_SCATTER) {
    const ScatterParams& sc = ep.sc;
    if (sc.part_cols <= 0 || sc.dst_cols <= 0 || sc.part_cols % 32 || sc.dst_cols % 32 || sc.part_cols % sc.dst_cols ||
        d.N % sc.part_cols || sc.seg_rows <= 0 || (sc.dst_ld * 2) % 16 || sc.part_cols / sc.dst_cols > kMaxPeers ||
        sc.dst_ld < (d.N / sc.part_cols) * sc.dst_cols || sc.row_off < 0 || sc.seg_rows > sc.dst_seq)
      return -7;
    for (int i = 0; i < sc.part_cols / sc.dst_cols; ++i)
      if (!sc.peers[i] || (reinterpret_cast<uintptr_t>(sc.peers[i]) & 15)) return -7;
  } else if (ep.epi == EPI_F32_ACC) {
    if ((reinterpret_cast<uintptr_t>(ep.out_f32) & 15) || (ep.ldc * 4) % 16) return -4;
    if ((r = make_out_map(&P->em.acc, ep.out_f32, true, d.M, d.N, ep.ldc))) return r;
  } else {
    if ((reinterpret_cast<uintptr_t>(ep.out) & 15) || (ep.ldc * 2) % 16) return -4;
    if ((r = make_out_map(&P->em.out, ep.out, false, d.M, d.N, ep.ldc))) return r;
    if (ep.epi == EPI_GELU || ep.epi == EPI_GATE_RES) {
      if (reinterpret_cast<uintptr_t>(ep.out2) & 15) return -4;
      if ((r = make_out_map(&P->em.out2, ep.out2, false, d.M, d.N, ep.ldc))) return r;
    }
  }
  if (d.grp_mode < 0 || d.grp_mode > 2) return -8;
  if (d.grp_mode) {
    if (two_sm || !d.grp_tab || d.n_groups < 1 || has_ext || d.splits > 1 || ep.epi == EPI_SCATTER) return -8;
    if (d.grp_mode == 2 && (d.grp_rows <= 0 || d.grp_rows % BM || ep.epi != EPI_F32_ACC || !d.a_mn || !d.b_mn))
      return -8;
    if (d.grp_mode == 1 && d.M % BM) return -8;
  }
  // grouped forward / dgrad: B stacks n_groups expert matrices along its rows
  const int64_t bscale = d.grp_mode == 1 ? d.n_groups : 1;
  // 2-SM tiles load 128 rows of A and 128 columns of B per CTA
  // (grouped weight gradient: A's columns are one expert's output rows; the output stacks n_groups of them)
  if (!a_gathered) {
    r = d.a_mn ? make_map(&P->a, d.A, d.K, d.grp_mode == 2 ? d.grp_rows : d.M, d.lda, 64, 64)
               : make_map(&P->a, d.A, d.M, d.K, d.lda, 64, BM);
    if (r) return r;
  }
  if (!b_gathered) {
    r = d.b_mn ? make_map(&P->b, d.B, d.K * bscale, d.N, d.ldb, 64, 64)
               : make_map(&P->b, d.B, d.N * bscale, d.K, d.ldb, 64, two_sm ? 128 : BN);
    if (r) return r;
  }
  for (int i = 0; i < d.gather_n && d.gather; ++i) {
    // each peer holds gather_rows rows of the gathered dimension, same row stride as the local operand
    if (d.gather == 1) r = make_map(&P->gm.m[i], d.gather_ptrs[i], d.gather_rows, d.K, d.lda, 64, BM);
    else if (d.gather == 2) r = make_map(&P->gm.m[i], d.gather_ptrs[i], d.gather_rows, d.M, d.lda, 64, 64);
    else r = make_map(&P->gm.m[i], d.gather_ptrs[i], d.gather_rows, d.N, d.ldb, 64, 64);
    if (r) return r;
  }
  if (has_ext) {
    if ((d.lda2 * 2) % 16 || (d.ldb2 * 2) % 16 ||
        ((reinterpret_cast<uintptr_t>(d.A2) | reinterpret_cast<uintptr_t>(d.B2)) & 15))
      return -5;
    r = d.a_mn ? make_map(&P->xm.a2, d.A2, d.K2, d.M, d.lda2, 64, 64)
               : make_map(&P->xm.a2, d.A2, d.M, d.K2, d.lda2, 64, BM);
    if (r) return r;
    r = d.b_mn ? make_map(&P->xm.b2, d.B2, d.K2, d.N, d.ldb2, 64, 64)
               : make_map(&P->xm.b2, d.B2, d.N, d.K2, d.ldb2, 64, two_sm ? 128 : BN);
    if (r) return r;
  }
  Shape& sh = P->sh;
  sh.M = d.M;
  sh.N = d.N;
  sh.K = d.K;
  sh.tiles_m = two_sm ? (d.M + 255) / 256 : (d.M + BM - 1) / BM;
  sh.tiles_n = (d.N + BN - 1) / BN;
  sh.kb_main = (d.K + BK - 1) / BK;
  sh.total_k_blocks = sh.kb_main + (has_ext ? (d.K2 + BK - 1) / BK : 0);
  int splits = d.splits < 1 ? 1 : d.splits;
  if (splits > sh.total_k_blocks) splits = sh.total_k_blocks;
  sh.k_blocks_per_split = (sh.total_k_blocks + splits - 1) / splits;
  sh.splits = (sh.total_k_blocks + sh.k_blocks_per_split - 1) / sh.k_blocks_per_split;
  sh.a_mn = d.a_mn;
  sh.b_mn = d.b_mn;
  sh.gather = d.gather;
  sh.gather_rows = d.gather_rows;
  sh.grp_tab = d.grp_tab;
  sh.grp_mode = d.grp_mode;
  sh.n_groups = d.n_groups;
  sh.grp_stride = 0;
  if (d.grp_mode == 1) {
    sh.grp_stride = d.b_mn ? d.K : d.N;  // rows of one expert's B matrix
  } else if (d.grp_mode == 2) {
    sh.grp_stride = d.grp_rows;
    sh.tiles_m = d.grp_rows / BM;  // per expert; units = n_groups x tiles_m x tiles_n
    sh.splits = 1;
    sh.k_blocks_per_split = sh.total_k_blocks;
  }
  P->ep = ep;
  return 0;
}

}  // namespace vo_gemm

// C-style launchers (no torch dependency).  Operand conventions:
//   a_mn == 0: A is row-major [M, K] (lda >= K);  a_mn == 1: A is row-major [K, M] (lda >= M)
//   b_mn == 0: B is row-major [N, K] (ldb >= K);  b_mn == 1: B is row-major [K, N] (ldb >= N)
// splits > 1 is only valid with EPI_F32_ACC (partial sums are reduced in global memory).
// Returns 0 on success, otherwise a CUDA / driver error code.
// General form: C = A B^T (+ A2 B2^T when A2 != null, K2 extra reduction columns, same majorness).
extern "C" int vo_gemm_launch_group(const vo_gemm::GemmDesc* d, int n, cudaStream_t stream) {
  using namespace vo_gemm;
  if (n < 1 || n > kMaxGroup) return -6;
  if (g_use_2sm < 0) {
    const char* e = getenv("VO_GEMM_2SM");
    g_use_2sm = (e && e[0] == '0') ? 0 : 1;
  }
  if (!g_num_sms) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t es[6] = {
        cudaFuncSetAttribute(gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM1_BYTES),
        cudaFuncSetAttribute(gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM1_BYTES),
        cudaFuncSetAttribute(gemm2sm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES),
        cudaFuncSetAttribute(gemm2sm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2_BYTES),
        cudaFuncSetAttribute(gemm2sm_kernel<false>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
        cudaFuncSetAttribute(gemm2sm_kernel<true>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1)};
    for (cudaError_t e : es)
      if (e != cudaSuccess) {
        g_num_sms = 0;
        return (int)e;
      }
  }
  // all problems of a launch share the kernel: the 2-SM form only when every one has >= 256 rows (expert-
  // grouped GEMMs run 128-row tiles on the 1-SM kernel)
  bool two_sm = g_use_2sm != 0;
  for (int i = 0; i < n; ++i) {
    if (d[i].M > 0 && d[i].N > 0 && d[i].K > 0 && d[i].M < 256) two_sm = false;
    if (d[i].grp_mode) {
      two_sm = false;
      if (n > 1) return -8;
    }
  }
  Launch L;
  memset(&L, 0, sizeof(L));
  int units = 0;
  for (int i = 0; i < n; ++i) {
    if (d[i].M <= 0 || d[i].N <= 0 || d[i].K <= 0) continue;
    Prob* P = &L.p[L.nprob];
    const int r = build_prob(d[i], two_sm, P);
    if (r) return r;
    P->unit_begin = units;
    units += P->sh.tiles_m * P->sh.tiles_n * P->sh.splits * (P->sh.grp_mode == 2 ? P->sh.n_groups : 1);
    ++L.nprob;
  }
  if (L.nprob == 0) return 0;
  L.units = units;
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
    return (int)(L.nprob > 1 ? cudaLaunchKernelEx(&cfg, gemm2sm_kernel<true>, L)
                             : cudaLaunchKernelEx(&cfg, gemm2sm_kernel<false>, L));
  }
  const int grid = units < g_num_sms ? units : g_num_sms;
  if (L.nprob > 1)
    gemm_kernel<true><<<grid, NUM_THREADS, SMEM1_BYTES, stream>>>(L);
  else
    gemm_kernel<false><<<grid, NUM_THREADS, SMEM1_BYTES, stream>>>(L);
  return (int)cudaGetLastError();
}

extern "C" int vo_gemm_launch_ext(const void* A, const void* B, const void* A2, const void* B2, int M, int N, int K,
                                  int K2, int64_t lda, int64_t ldb, int64_t lda2, int64_t ldb2, int a_mn, int b_mn,
                                  int splits, vo_gemm::EpiParams ep, cudaStream_t stream) {
  vo_gemm::GemmDesc d{A, B, A2, B2, M, N, K, K2, lda, ldb, lda2, ldb2, a_mn, b_mn, splits, ep};
  return vo_gemm_launch_group(&d, 1, stream);
}

extern "C" int vo_gemm_launch(const void* A, const void* B, int M, int N, int K, int64_t lda, int64_t ldb, int a_mn,
                              int b_mn, int splits, vo_gemm::EpiParams ep, cudaStream_t stream) {
  return vo_gemm_launch_ext(A, B, nullptr, nullptr, M, N, K, 0, lda, ldb, 0, 0, a_mn, b_mn, splits, ep, stream);
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
