// Flash attention forward for sm_100a: two query tiles per CTA, P and O resident in tensor memory.
//
//   O = softmax(Q K^T * scale) V,  LSE = log(sum exp(Q K^T * scale))
//   Q [BH, Sq, D], K/V [BH, Skv, D] (bf16, contiguous per head); O written token-major [B, Sq, H, D];
//   D in {64, 128}; optional causal mask (query i sees keys <= i).
//
// One CTA = 256 query rows (two 128-row tiles t = 0, 1) of one head, 384 threads:
//   warp 0        TMA producer: Q0, Q1 once; then K_0, and per key block j: K_{j+1}, V_j (rings);
//   warp 1        TMEM allocator + single-thread MMA issuer;
//   warps 4..7    softmax warpgroup of tile 0, one query row per thread;
//   warps 8..11   softmax warpgroup of tile 1.
// Tensor memory (512 columns): S_0 [0,128), S_1 [128,256), O_0 [256, 256+D), O_1 [256+D, 256+2D).
// The softmax of tile t reads S_t, and writes the bf16 probabilities P_t back into the first 64
// columns of S_t (tcgen05.st); the PV MMA then takes its A operand straight from tensor memory, so P
// never touches shared memory.  O_t accumulates in tensor memory across key blocks.
// MMA issue order per key block j:  PV_0(j), S_0(j+1), PV_1(j), S_1(j+1).  The tensor pipe executes
// one thread's MMAs in order, so S_t(j+1) may overwrite P_t(j) right after PV_t(j) is issued, and the
// commit that signals S_t(j) also proves PV_t(j-1) complete.  While softmax t works on S_t(j) the
// tensor core runs the other tile's MMAs: the two warpgroups ping-pong against the tensor pipe.
// Online softmax with a lazy rescale: the running max m only moves when a block's max exceeds it by
// more than 2^8 (exp2 domain); only then is O_t read, scaled and written back in tensor memory.  P
// values are bounded by 2^8, well inside bf16 / fp32 range, and l and O share the same reference m.
// Every mbarrier wait is bounded; on timeout an error code is recorded and the CTA exits cleanly.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

namespace vo_fmha2 {

constexpr int BQ = 128, BKV = 128;
constexpr int NUM_THREADS = 384;
constexpr unsigned long long WAIT_BUDGET = 8ull * 1000 * 1000 * 1000;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

__device__ int g_error = 0;
// mbarrier waits suspend the waiting thread for up to this long (it wakes early when the phase completes),
// so spinning producer / issuer / softmax warps do not take issue slots from the working ones
constexpr uint32_t kSuspendNs = 200000;

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
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D(tmem) (+)= A(smem) * B(smem)
__device__ __forceinline__ void mma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// D(tmem) (+)= A(tmem) * B(smem)
__device__ __forceinline__ void mma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void commit(uint64_t* b) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(b))
               : "memory");
}
// 32 lanes x 32 columns of 32-bit values; no wait (caller issues wait_ld)
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
// 32 lanes x 16 columns; no wait
__device__ __forceinline__ void ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
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
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
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
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// (a0, a1) * s + c on the paired fp32 pipe (one instruction for two lanes of work)
__device__ __forceinline__ void ffma2(float a0, float a1, float s, float c, float& r0, float& r1) {
  asm("{\n\t.reg .b64 x, y, z, r;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %4};\n\tmov.b64 z, {%5, %5};\n\t"
      "fma.rn.f32x2 r, x, y, z;\n\tmov.b64 {%0, %1}, r;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(s), "f"(c));
}
__device__ __forceinline__ void fadd2(float& s0, float& s1, float a0, float a1) {
  asm("{\n\t.reg .b64 x, y, r;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 r, x, y;\n\tmov.b64 {%0, %1}, r;\n\t}"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}
__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

struct Params {
  int Sq, Skv, H, npairs;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* o;   // [B, Sq, H, D], or [B, split, H, D] when split > 0
  __nv_bfloat16* o2;  // [B, Sq - split, H, D] (split > 0): rows q >= split
  int split;
  float* lse;         // [B*H, Sq] natural log
  // Ulysses output exchange (peer_sl > 0): the query rows are a sequence gathered from the ranks of a
  // sequence-parallel group (peer_sl rows per rank, image rows first); row q belongs to rank q / peer_sl
  // and is stored straight into that rank's buffers over NVLink -- image rows into peer_o[r], text rows
  // into peer_o2[r], both [B, rows, peer_htot, D] with this rank's heads at head offset peer_h0.
  __nv_bfloat16* peer_o[8];
  __nv_bfloat16* peer_o2[8];
  int peer_sl, peer_si, peer_htot, peer_h0;
  // optional per-sequence key count [B] (right-padded keys past it are masked: padded prompts)
  const int* kv_len;
};

__device__ __forceinline__ int kv_limit(const Params& p, int bh) {
  return p.kv_len ? min(p.Skv, max(0, __ldg(p.kv_len + bh / p.H))) : p.Skv;
}

// token-major output row of query q (head h, batch b): one buffer, or split at `split` into two
__device__ __forceinline__ __nv_bfloat16* out_row(const Params& p, int b, int q, int h, int D) {
  if (p.peer_sl > 0) {
    const int r = q / p.peer_sl, t = q - r * p.peer_sl;
    const bool img = t < p.peer_si;
    __nv_bfloat16* base = img ? p.peer_o[r] : p.peer_o2[r];
    const int rows = img ? p.peer_si : p.peer_sl - p.peer_si;
    const int row = img ? t : t - p.peer_si;
    return base + (((int64_t)b * rows + row) * p.peer_htot + p.peer_h0 + h) * D;
  }
  if (p.split > 0 && q >= p.split) return p.o2 + (((int64_t)b * (p.Sq - p.split) + (q - p.split)) * p.H + h) * D;
  const int rows = p.split > 0 ? p.split : p.Sq;
  return p.o + (((int64_t)b * rows + q) * p.H + h) * D;
}

template <int D>
struct Cfg {
  static constexpr int TILE = 128 * D * 2;  // one 128-row tile of Q/K/V (D/64 swizzled 16 KB chunks)
  static constexpr int KST = D == 64 ? 3 : 2;
  static constexpr int VST = 2;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = 2 * TILE;
  static constexpr int V_OFF = K_OFF + KST * TILE;
  static constexpr int BAR_OFF = V_OFF + VST * TILE;
  static constexpr int BYTES = BAR_OFF + 256 + 4096 + 1024;
  static_assert(BYTES + 1024 <= 232448, "shared memory above the 227 KB per-block limit");
  static constexpr uint32_t S_COL0 = 0, O_COL0 = 256;
};

__device__ __forceinline__ void named_bar(int id, int n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n)); }

// Softmax of one key half of one query tile (SPLIT == 2).  Warps 2..17 form groups g = 0..3 of four
// consecutive warps (covering the four 32-lane quarters of tensor memory); tile t = g / 2, key half
// h = g % 2.  Per key block: row max over the 64 own columns, exchange with the partner half through
// shared memory (double-buffered by block parity, one 256-thread named barrier), the shared lazy
// rescale of the own half of O_t, P for the own keys packed into the first 32 own columns.
// INDEP (head_dim 64): the two key halves keep separate running maxima, row sums and O accumulators
// (O_{t,h} = 64 columns each, 4 x 64 + 2 x 128 = 512 tensor-memory columns), so no exchange is needed
// per key block; the halves are combined once in the epilogue.
template <int D, bool INDEP>
__device__ __forceinline__ void softmax_split2(const Params& p, uint32_t tmem, int warp, int lane, int q0, int bh,
                                               int nkv, uint64_t* s_full, uint64_t* p_full, uint64_t* o_final,
                                               volatile int* abort_flag, float* xmax, float* xsum) {
  using C = Cfg<D>;
  static_assert(!INDEP || D == 64, "independent halves need 4 O tiles of 64 columns");
  const int g = (warp - 2) >> 2;
  const int t = g >> 1, hf = g & 1;
  const int quarter = warp & 3;
  const int row = 32 * quarter + lane;
  const int q = q0 + t * BQ + row;
  const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
  const uint32_t S_t = tmem + C::S_COL0 + t * 128 + lane_off + 64 * hf;
  // shared O_t: this half rescales / stores columns [hf D/2, (hf+1) D/2); INDEP: own O_{t,h}, all columns
  const uint32_t O_t = INDEP ? tmem + C::O_COL0 + t * 128 + hf * 64 + lane_off
                             : tmem + C::O_COL0 + t * D + lane_off + hf * (D / 2);
  const int bar_id = 1 + t;
  float* mx_mine = xmax + (t * 2 + hf) * 256;
  const float* mx_other = xmax + (t * 2 + (hf ^ 1)) * 256;
  const float sl2 = p.scale_log2;
  float m = -INFINITY, l = 0.f;
  bool ok = nkv > 0;
  for (int j = 0; ok && j < nkv; ++j) {
    if (!mbar_wait(&s_full[t], j & 1, abort_flag, 49)) {
      ok = false;
      break;
    }
    fence_after();
    const int kv0 = j * BKV + 64 * hf;
    int lim = kv_limit(p, bh) - kv0;
    if (p.causal) lim = min(lim, q - kv0 + 1);
    lim = max(0, min(64, lim));
    float mx = -INFINITY;
    {  // pass 1 (values are read again in pass 2: keeps the register budget of 576 threads)
    uint32_t a[32], b[32];
    ld32_nowait(S_t, a);
    ld32_nowait(S_t + 32, b);
    wait_ld();
    if (lim == 64) {
#pragma unroll
      for (int i = 0; i < 32; ++i) mx = max3(mx, __uint_as_float(a[i]), __uint_as_float(b[i]));
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        if (i < lim) mx = fmaxf(mx, __uint_as_float(a[i]));
        if (32 + i < lim) mx = fmaxf(mx, __uint_as_float(b[i]));
      }
    }
    }
    if (!INDEP) {
      const int par = (j & 1) * 128;
      mx_mine[par + row] = mx;
      named_bar(bar_id, 256);
      mx = fmaxf(mx, mx_other[par + row]);
    }
    const float m_blk = mx * sl2;
    float alpha = 1.f;
    const bool move = m_blk > m + RESCALE_THRESHOLD || (m == -INFINITY && m_blk != -INFINITY);
    if (move) {
      alpha = (m == -INFINITY) ? 0.f : ex2(m - m_blk);
      m = m_blk;
    }
    if (j > 0 && __any_sync(0xffffffffu, move)) {
      // shared O: both halves take the same decision and each rescales its half of O_t; INDEP: this
      // half's own O_{t,h} (all 64 columns).  O is quiescent here (see the MMA ordering above).
#pragma unroll
      for (int c = 0; c < (INDEP ? 2 : D / 64); ++c) {
        uint32_t o[32];
        ld32_nowait(O_t + c * 32, o);
        wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
        st32(O_t + c * 32, o);
      }
    }
    const float nmb = (m == -INFINITY) ? 0.f : -m;
    float rs = 0.f, rs0 = 0.f, rs1 = 0.f;
    auto emit = [&](const uint32_t (&v)[32], int c) {
      uint32_t w[16];
      if (lim == 64) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0, x1;
          ffma2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), sl2, nmb, x0, x1);
          const float e0 = ex2(x0), e1 = ex2(x1);
          fadd2(rs0, rs1, e0, e1);
          w[i] = pack_bf16(e0, e1);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k = c * 32 + 2 * i;
          const float e0 = k < lim ? ex2(fmaf(__uint_as_float(v[2 * i]), sl2, nmb)) : 0.f;
          const float e1 = k + 1 < lim ? ex2(fmaf(__uint_as_float(v[2 * i + 1]), sl2, nmb)) : 0.f;
          rs += e0 + e1;
          w[i] = pack_bf16(e0, e1);
        }
      }
      st16(S_t + c * 16, w);
    };
    {
      uint32_t v[32];
      ld32_nowait(S_t, v);
      wait_ld();
      emit(v, 0);
      ld32_nowait(S_t + 32, v);  // columns 32..63 are not touched by the chunk-0 stores (columns 0..15)
      wait_ld();
      emit(v, 1);
    }
    wait_st();
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&p_full[t]);
    l = l * alpha + (rs + (rs0 + rs1));
  }
  if (ok && mbar_wait(&o_final[t], 0, abort_flag, 50)) {
    fence_after();
    xsum[(t * 2 + hf) * 128 + row] = l;
    if (INDEP) mx_mine[row] = m;
    named_bar(bar_id, 256);
    const float l_o = xsum[(t * 2 + (hf ^ 1)) * 128 + row];
    float c_mine = 1.f, c_other = 1.f, lt, m_out = m;
    if (INDEP) {  // combine the halves against the larger reference max
      const float m_o = mx_other[row];
      m_out = fmaxf(m, m_o);
      c_mine = (m == -INFINITY) ? 0.f : ex2(m - m_out);
      c_other = (m_o == -INFINITY) ? 0.f : ex2(m_o - m_out);
      lt = l * c_mine + l_o * c_other;
    } else {
      lt = l + l_o;
    }
    const float inv = lt > 0.f ? 1.f / lt : 0.f;
    const int bb = bh / p.H, h = bh % p.H;
    const bool row_ok = q < p.Sq;
    __nv_bfloat16* dst = out_row(p, bb, q, h, D) + hf * (D / 2);
    // INDEP: both O_{t,0} and O_{t,1} are read for this half's output columns [hf D/2, +D/2)
    const uint32_t Oa = INDEP ? tmem + C::O_COL0 + t * 128 + hf * (D / 2) + lane_off : O_t;
    const uint32_t Ob = INDEP ? tmem + C::O_COL0 + t * 128 + 64 + hf * (D / 2) + lane_off : O_t;
    const float ca = INDEP ? (hf == 0 ? c_mine : c_other) : 1.f;  // O_{t,0} belongs to half 0
    const float cb = INDEP ? (hf == 0 ? c_other : c_mine) : 0.f;
#pragma unroll
    for (int c = 0; c < D / 64; ++c) {
      uint32_t o[32];
      ld32_nowait(Oa + c * 32, o);
      wait_ld();
      if (INDEP) {
        uint32_t o2[32];
        ld32_nowait(Ob + c * 32, o2);
        wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i)
          o[i] = __float_as_uint(__uint_as_float(o[i]) * ca + __uint_as_float(o2[i]) * cb);
      }
      if (row_ok) {
#pragma unroll
        for (int gg = 0; gg < 4; ++gg) {
          uint4 pk;
          pk.x = pack_bf16(__uint_as_float(o[gg * 8 + 0]) * inv, __uint_as_float(o[gg * 8 + 1]) * inv);
          pk.y = pack_bf16(__uint_as_float(o[gg * 8 + 2]) * inv, __uint_as_float(o[gg * 8 + 3]) * inv);
          pk.z = pack_bf16(__uint_as_float(o[gg * 8 + 4]) * inv, __uint_as_float(o[gg * 8 + 5]) * inv);
          pk.w = pack_bf16(__uint_as_float(o[gg * 8 + 6]) * inv, __uint_as_float(o[gg * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(dst + c * 32 + gg * 8) = pk;
        }
      }
    }
    if (row_ok && hf == 0) p.lse[(int64_t)bh * p.Sq + q] = (m_out + __log2f(lt)) * 0.69314718055994531f;
  }
}

// SPLIT = softmax warpgroups per query tile.  SPLIT == 2 (576 threads): warpgroup (t, h) owns key
// columns [64 h, 64 h + 64) of S_t; the two halves exchange row maxima and row sums through shared
// memory (one named barrier per key block), write P for their keys into their own 64-column half
// (packed into its first 32 columns) and rescale / store their half of O_t.  Twice the softmax
// warps per SMSP hide the tensor-memory and MUFU latencies that bound SPLIT == 1.
// SPLIT == 3: as 2 with independent key halves (head_dim 64 only), see softmax_split2.
template <int SPLIT>
__host__ __device__ constexpr int fwd_threads() { return SPLIT >= 2 ? 576 : NUM_THREADS; }

template <int D, int SPLIT>
__global__ void __launch_bounds__(fwd_threads<SPLIT>(), 1)
    fmha_fwd2_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv, const __grid_constant__ Params p) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;              // [KST]
  uint64_t* k_empty = k_full + C::KST;      // [KST]
  uint64_t* v_full = k_empty + C::KST;      // [VST]
  uint64_t* v_empty = v_full + C::VST;      // [VST]
  uint64_t* s_full = v_empty + C::VST;      // [2] per tile
  uint64_t* p_full = s_full + 2;            // [2]
  uint64_t* o_final = p_full + 2;           // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // SPLIT == 2 exchange buffers: [tile][half][parity][128 rows] maxima, [tile][half][128] row sums
  float* xmax = reinterpret_cast<float*>(sm + C::BAR_OFF + 256);
  float* xsum = xmax + 2 * 2 * 2 * 128;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heavier (later) query pairs first under a causal mask
  const int pr = p.npairs - 1 - (int)(blockIdx.x % p.npairs);
  const int bh = blockIdx.x / p.npairs;
  const int q0 = pr * 2 * BQ;
  int kv_end = kv_limit(p, bh);
  if (p.causal) kv_end = min(kv_end, q0 + 2 * BQ);
  const int nkv = (kv_end + BKV - 1) / BKV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::KST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < C::VST; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], SPLIT >= 2 ? 8 : 4);
      mbar_init(&o_final[t], 1);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0 && nkv > 0) {
      mbar_expect_tx(q_full, 2 * C::TILE);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + C::Q_OFF + t * C::TILE + c * 16384, &mq, q_full, c * 64, q0 + t * BQ, bh);
      auto load_k = [&](int j) -> bool {
        const int s = j % C::KST;
        if (!mbar_wait(&k_empty[s], ((j / C::KST) & 1) ^ 1, abort_flag, 41)) return false;
        mbar_expect_tx(&k_full[s], C::TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + C::K_OFF + s * C::TILE + c * 16384, &mk, &k_full[s], c * 64, j * BKV, bh);
        return true;
      };
      bool ok = load_k(0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (j + 1 < nkv && !(ok = load_k(j + 1))) break;
        const int s = j % C::VST;
        if (!mbar_wait(&v_empty[s], ((j / C::VST) & 1) ^ 1, abort_flag, 42)) break;
        mbar_expect_tx(&v_full[s], C::TILE);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + C::V_OFF + s * C::TILE + c * 16384, &mv, &v_full[s], c * 64, j * BKV, bh);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && nkv > 0) {
      const uint32_t id_s = idesc(128, 128, 0, 0);
      const uint32_t id_o = idesc(128, D, 0, 1);
      const uint32_t S_T[2] = {tmem + C::S_COL0, tmem + C::S_COL0 + 128};
      const uint32_t O_T[2] = {tmem + C::O_COL0, tmem + C::O_COL0 + D};
      auto issue_s = [&](int t, int j) {
        const uint32_t qa = smem_u32(sm + C::Q_OFF + t * C::TILE);
        const uint32_t ka = smem_u32(sm + C::K_OFF + (j % C::KST) * C::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_ss(S_T[t], desc(qa + off, 16, 1024), desc(ka + off, 16, 1024), id_s, kk > 0);
        }
        commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {
        const uint32_t va = smem_u32(sm + C::V_OFF + (j % C::VST) * C::TILE);
        if (SPLIT == 3) {  // keys [64 h, 64 h + 64) into O_{t,h}
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk) {
            const int hh = kk >> 2;
            mma_ts(tmem + C::O_COL0 + t * 128 + hh * 64, S_T[t] + hh * 64 + (kk & 3) * 8,
                   desc(va + kk * 2048, 16384, 1024), id_o, (j > 0 || (kk & 3) > 0) ? 1u : 0u);
          }
        } else {
#pragma unroll
          for (int kk = 0; kk < BKV / 16; ++kk)
            mma_ts(O_T[t], S_T[t] + (SPLIT == 2 && kk >= 4 ? 64 + (kk - 4) * 8 : kk * 8),
                   desc(va + kk * 2048, 16384, 1024), id_o, (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, 43) && mbar_wait(&k_full[0], 0, abort_flag, 44);
      if (ok) {
        fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        const bool more = j + 1 < nkv;
        if (!mbar_wait(&v_full[j % C::VST], (j / C::VST) & 1, abort_flag, 45)) break;
        if (!mbar_wait(&p_full[0], j & 1, abort_flag, 46)) break;
        fence_after();
        issue_pv(0, j);
        if (more) {
          if (!mbar_wait(&k_full[(j + 1) % C::KST], ((j + 1) / C::KST) & 1, abort_flag, 47)) break;
          fence_after();
          issue_s(0, j + 1);
        } else {
          commit(&o_final[0]);
        }
        if (!mbar_wait(&p_full[1], j & 1, abort_flag, 48)) break;
        fence_after();
        issue_pv(1, j);
        commit(&v_empty[j % C::VST]);
        if (more) {
          issue_s(1, j + 1);
          commit(&k_empty[(j + 1) % C::KST]);
        } else {
          commit(&o_final[1]);
        }
      }
    }
  } else if (SPLIT >= 2 && warp >= 2) {
    softmax_split2<D, SPLIT == 3>(p, tmem, warp, lane, q0, bh, nkv, s_full, p_full, o_final, abort_flag, xmax, xsum);
  } else if (SPLIT == 1 && warp >= 4) {
    // ---------------------------------------------------------------- softmax warpgroups
    const int t = (warp - 4) >> 2;
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    const int q = q0 + t * BQ + row;
    const uint32_t lane_off = (uint32_t)lane_base << 16;
    const uint32_t S_t = tmem + C::S_COL0 + t * 128 + lane_off;
    const uint32_t O_t = tmem + C::O_COL0 + t * D + lane_off;
    const float sl2 = p.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = nkv > 0;
    for (int j = 0; ok && j < nkv; ++j) {
      if (!mbar_wait(&s_full[t], j & 1, abort_flag, 49)) {
        ok = false;
        break;
      }
      fence_after();
      const int kv0 = j * BKV;
      // keys [kv0, kv0 + lim) of this block are visible to this row
      int lim = kv_limit(p, bh) - kv0;
      if (p.causal) lim = min(lim, q - kv0 + 1);
      lim = max(0, min(BKV, lim));
      // pass 1: row max.  Chunks 2,3 first so chunks 0,1 stay in registers for pass 2.
      uint32_t a[32], b[32];
      float mx = -INFINITY;
      ld32_nowait(S_t + 64, a);
      ld32_nowait(S_t + 96, b);
      wait_ld();
      if (lim == BKV) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = max3(mx, __uint_as_float(a[i]), __uint_as_float(b[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (64 + i < lim) mx = fmaxf(mx, __uint_as_float(a[i]));
          if (96 + i < lim) mx = fmaxf(mx, __uint_as_float(b[i]));
        }
      }
      uint32_t c0[32], c1[32];
      ld32_nowait(S_t + 0, c0);
      ld32_nowait(S_t + 32, c1);
      wait_ld();
      if (lim == BKV) {
#pragma unroll
        for (int i = 0; i < 32; ++i) mx = max3(mx, __uint_as_float(c0[i]), __uint_as_float(c1[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i < lim) mx = fmaxf(mx, __uint_as_float(c0[i]));
          if (32 + i < lim) mx = fmaxf(mx, __uint_as_float(c1[i]));
        }
      }
      // lazy rescale: move m only when the block max exceeds it by more than the threshold
      const float m_blk = mx * sl2;
      float alpha = 1.f;
      const bool move = m_blk > m + RESCALE_THRESHOLD || (m == -INFINITY && m_blk != -INFINITY);
      if (move) {
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_blk);
        m = m_blk;
      }
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        // O_t is quiescent: PV_t(j-1) completed before S_t(j) was signalled, PV_t(j) waits for us
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          ld32_nowait(O_t + c * 32, o);
          wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          st32(O_t + c * 32, o);
        }
      }
      const float mb = (m == -INFINITY) ? 0.f : m;
      float rs = 0.f, rs0 = 0.f, rs1 = 0.f;
      // pass 2: p = exp2(s*scale_log2 - m), packed bf16 pairs into columns [0, 64) of S_t
      auto emit = [&](const uint32_t (&v)[32], int c) {
        uint32_t w[16];
        const float nmb = -mb;
        if (lim == BKV) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float x0, x1;
            ffma2(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]), sl2, nmb, x0, x1);
            const float e0 = ex2(x0), e1 = ex2(x1);
            fadd2(rs0, rs1, e0, e1);
            w[i] = pack_bf16(e0, e1);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int k = c * 32 + 2 * i;
            const float e0 = k < lim ? ex2(fmaf(__uint_as_float(v[2 * i]), sl2, nmb)) : 0.f;
            const float e1 = k + 1 < lim ? ex2(fmaf(__uint_as_float(v[2 * i + 1]), sl2, nmb)) : 0.f;
            rs += e0 + e1;
            w[i] = pack_bf16(e0, e1);
          }
        }
        st16(S_t + c * 16, w);
      };
      ld32_nowait(S_t + 64, a);  // chunk 2 in flight while chunks 0, 1 are exponentiated
      emit(c0, 0);
      emit(c1, 1);
      wait_ld();
      ld32_nowait(S_t + 96, b);
      emit(a, 2);
      wait_ld();
      emit(b, 3);
      wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
      l = l * alpha + (rs + (rs0 + rs1));
    }
    if (ok && mbar_wait(&o_final[t], 0, abort_flag, 50)) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int bb = bh / p.H, h = bh % p.H;
      const bool row_ok = q < p.Sq;
      __nv_bfloat16* dst = out_row(p, bb, q, h, D);
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        ld32_nowait(O_t + c * 32, o);
        wait_ld();
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 pk;
            pk.x = pack_bf16(__uint_as_float(o[g * 8 + 0]) * inv, __uint_as_float(o[g * 8 + 1]) * inv);
            pk.y = pack_bf16(__uint_as_float(o[g * 8 + 2]) * inv, __uint_as_float(o[g * 8 + 3]) * inv);
            pk.z = pack_bf16(__uint_as_float(o[g * 8 + 4]) * inv, __uint_as_float(o[g * 8 + 5]) * inv);
            pk.w = pack_bf16(__uint_as_float(o[g * 8 + 6]) * inv, __uint_as_float(o[g * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + c * 32 + g * 8) = pk;
          }
        }
      }
      if (row_ok) p.lse[(int64_t)bh * p.Sq + q] = (m + __log2f(l)) * 0.69314718055994531f;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
  }
}


// ====================================================================================================
// Forward v4: one 128-row query tile per CTA, two CTAs per SM, 64-key blocks, double-buffered scores.
//
// 192 threads: warps 0..3 softmax (one query row per thread, TMEM lane quarter = warp), warp 4 TMA
// producer, warp 5 TMEM allocator + single-thread MMA issuer.  Tensor memory (256 columns per CTA, so
// two CTAs share an SM's 512): S buffers [0, 64) and [64, 128), O [128, 128 + D).  The QK^T of key
// block j + 2 goes into the buffer the softmax of block j has just turned into P, right behind the PV
// of block j, so the softmax of block j + 1 never waits for the tensor core: its scores were computed
// while block j was being exponentiated.  The other CTA on the SM supplies the second query tile that
// keeps the tensor pipe busy while this CTA's softmax runs, and overlaps this CTA's prologue/epilogue.
// Barriers: s_full[b] / p_full[b] per score buffer (a buffer's phase j >> 1 is block j), o_ready after
// every PV (the softmax waits on it only to rescale O: at block j, PV(j - 2) is known complete, so
// phases j - 1 and j are the only candidates and parity tells them apart), o_final after the last PV.
// A share (6 of 16 pairs) of the exponentials is evaluated on the FMA pipe: 2^x = 2^round(x) * p(f),
// f = x - round(x) in [-1/2, 1/2], with round() by the 1.5 * 2^23 magic-number addition and p the
// degree-3 polynomial minimising the relative error of 2^f on [-1/2, 1/2] (Lawson-weighted least
// squares, max relative error 8.4e-5, far below the bf16 rounding of P); 2^round(x) is an integer add
// into the exponent field.  The MUFU pipe alone is the bound of the score path at head_dim 64.
constexpr int FWD4_THREADS = 192;
constexpr int kFwd4Emu64 = 0;  // of every 8 exponential pairs, this many on the FMA pipe at head_dim 64 (0 measured fastest)
constexpr int BK4 = 64;

template <int D>
struct Cfg4 {
  static constexpr int Q_BYTES = 128 * D * 2;
  static constexpr int KV_BYTES = BK4 * D * 2;
  static constexpr int ST = D == 64 ? 4 : 2;  // K and V stages
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_BYTES;
  static constexpr int V_OFF = K_OFF + ST * KV_BYTES;
  static constexpr int BAR_OFF = V_OFF + ST * KV_BYTES;
  static constexpr int BYTES = BAR_OFF + 256;
  static_assert(2 * (BYTES + 1024) <= 232448, "two CTAs per SM must fit in shared memory");
  static constexpr uint32_t O_COL = 128;
};

__device__ __forceinline__ void fsub2(float a0, float a1, float b0, float b1, float& r0, float& r1) {
  asm("{\n\t.reg .b64 x, y, r;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\t"
      "sub.rn.f32x2 r, x, y;\n\tmov.b64 {%0, %1}, r;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ void ffma2v(float a0, float a1, float b0, float b1, float c0, float c1, float& r0,
                                       float& r1) {
  asm("{\n\t.reg .b64 x, y, z, r;\n\tmov.b64 x, {%2, %3};\n\tmov.b64 y, {%4, %5};\n\tmov.b64 z, {%6, %7};\n\t"
      "fma.rn.f32x2 r, x, y, z;\n\tmov.b64 {%0, %1}, r;\n\t}"
      : "=f"(r0), "=f"(r1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
// 2^x0, 2^x1 on the FMA pipe (x <= 2^22; inputs below -126 are clamped: the result is then ~1e-38)
__device__ __forceinline__ void ex2_fma2(float x0, float x1, float& y0, float& y1) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer in the low bits
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float t0 = x0, t1 = x1, r0, r1, f0, f1;
  fadd2(t0, t1, kMagic, kMagic);            // t = x + magic
  fsub2(t0, t1, kMagic, kMagic, r0, r1);    // r = round(x)
  fsub2(x0, x1, r0, r1, f0, f1);            // f in [-1/2, 1/2]
  float p0, p1;
  ffma2v(f0, f1, 0.05521300435066223f, 0.05521300435066223f, 0.24271394312381744f, 0.24271394312381744f, p0, p1);
  ffma2v(p0, p1, f0, f1, 0.6932621598243713f, 0.6932621598243713f, p0, p1);
  ffma2v(p0, p1, f0, f1, 0.999919593334198f, 0.999919593334198f, p0, p1);
  // the low 23 bits of t hold round(x) + 2^22 (the magic's mantissa); shifted into the exponent field the
  // 2^22 part leaves 32 bits, so the integer add scales p by 2^round(x)
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

template <int D, int EMU>
__global__ void __launch_bounds__(FWD4_THREADS, 2)
    fmha_fwd4_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv, const __grid_constant__ Params p) {
  using C = Cfg4<D>;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;           // [ST]
  uint64_t* k_empty = k_full + C::ST;    // [ST]
  uint64_t* v_full = k_empty + C::ST;    // [ST]
  uint64_t* v_empty = v_full + C::ST;    // [ST]
  uint64_t* s_full = v_empty + C::ST;    // [2] per score buffer
  uint64_t* p_full = s_full + 2;         // [2]
  uint64_t* o_ready = p_full + 2;        // [1] after every PV
  uint64_t* o_final = o_ready + 1;       // [1] after the last PV
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // heavier (later) query tiles first under a causal mask
  const int tile = p.npairs - 1 - (int)(blockIdx.x % p.npairs);
  const int bh = blockIdx.x / p.npairs;
  const int q0 = tile * BQ;
  int kv_end = kv_limit(p, bh);
  if (p.causal) kv_end = min(kv_end, q0 + BQ);
  const int nkv = (kv_end + BK4 - 1) / BK4;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::ST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
    }
    mbar_init(o_ready, 1);
    mbar_init(o_final, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0 && nkv > 0) {
      mbar_expect_tx(q_full, C::Q_BYTES);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) tma_load_3d(sm + C::Q_OFF + c * 16384, &mq, q_full, c * 64, q0, bh);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % C::ST, ph = ((j / C::ST) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], ph, abort_flag, 61)) break;
        mbar_expect_tx(&k_full[s], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + C::K_OFF + s * C::KV_BYTES + c * 8192, &mk, &k_full[s], c * 64, j * BK4, bh);
        if (!mbar_wait(&v_empty[s], ph, abort_flag, 62)) break;
        mbar_expect_tx(&v_full[s], C::KV_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(sm + C::V_OFF + s * C::KV_BYTES + c * 8192, &mv, &v_full[s], c * 64, j * BK4, bh);
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && nkv > 0) {
      const uint32_t id_s = idesc(128, BK4, 0, 0);
      const uint32_t id_o = idesc(128, D, 0, 1);
      const uint32_t O = tmem + C::O_COL;
      const uint32_t qa = smem_u32(sm + C::Q_OFF);
      auto issue_s = [&](int j) {
        const uint32_t ka = smem_u32(sm + C::K_OFF + (j % C::ST) * C::KV_BYTES);
        const uint32_t Sb = tmem + (j & 1) * BK4;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t in = (kk & 3) * 32;
          mma_ss(Sb, desc(qa + (kk >> 2) * 16384 + in, 16, 1024), desc(ka + (kk >> 2) * 8192 + in, 16, 1024), id_s,
                 kk > 0);
        }
        commit(&s_full[j & 1]);
        commit(&k_empty[j % C::ST]);
      };
      auto issue_pv = [&](int j) {
        const uint32_t va = smem_u32(sm + C::V_OFF + (j % C::ST) * C::KV_BYTES);
        const uint32_t Sb = tmem + (j & 1) * BK4;
#pragma unroll
        for (int kk = 0; kk < BK4 / 16; ++kk)
          mma_ts(O, Sb + kk * 8, desc(va + kk * 2048, 8192, 1024), id_o, (j > 0 || kk > 0) ? 1u : 0u);
        commit(o_ready);
        commit(&v_empty[j % C::ST]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, 63);
      for (int j = 0; ok && j < 2 && j < nkv; ++j) {
        if (!(ok = mbar_wait(&k_full[j % C::ST], (j / C::ST) & 1, abort_flag, 64))) break;
        fence_after();
        issue_s(j);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        if (!mbar_wait(&v_full[j % C::ST], (j / C::ST) & 1, abort_flag, 65)) break;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, abort_flag, 66)) break;
        fence_after();
        issue_pv(j);
        if (j + 1 == nkv) commit(o_final);
        if (j + 2 < nkv) {
          const int jn = j + 2;
          if (!mbar_wait(&k_full[jn % C::ST], (jn / C::ST) & 1, abort_flag, 67)) break;
          fence_after();
          issue_s(jn);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 0..3)
    const int row = 32 * warp + lane;
    const int q = q0 + row;
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    const uint32_t O_t = tmem + C::O_COL + lane_off;
    const float sl2 = p.scale_log2;
    const int kvl = kv_limit(p, bh);
    float m = -INFINITY, l = 0.f;
    bool ok = nkv > 0;
    for (int j = 0; ok && j < nkv; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort_flag, 68)) {
        ok = false;
        break;
      }
      fence_after();
      const uint32_t S_b = tmem + b * BK4 + lane_off;
      const int kv0 = j * BK4;
      int lim = kvl - kv0;
      if (p.causal) lim = min(lim, q - kv0 + 1);
      lim = max(0, min(BK4, lim));
      uint32_t a[32], c[32];
      ld32_nowait(S_b, a);
      ld32_nowait(S_b + 32, c);
      wait_ld();
      float mx = -INFINITY;
      if (lim == BK4) {
        // four independent max chains (short dependency chains), combined at the end
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 32; ++i) mq[i & 3] = max3(mq[i & 3], __uint_as_float(a[i]), __uint_as_float(c[i]));
        mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (i < lim) mx = fmaxf(mx, __uint_as_float(a[i]));
          if (32 + i < lim) mx = fmaxf(mx, __uint_as_float(c[i]));
        }
      }
      const float m_blk = mx * sl2;
      float alpha = 1.f;
      const bool move = m_blk > m + RESCALE_THRESHOLD || (m == -INFINITY && m_blk != -INFINITY);
      if (move) {
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_blk);
        m = m_blk;
      }
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        // O holds blocks < j once PV(j - 1) has completed; PV(j) waits for this block's P
        if (!mbar_wait(o_ready, (j - 1) & 1, abort_flag, 69)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int cc = 0; cc < D / 32; ++cc) {
          uint32_t o[32];
          ld32_nowait(O_t + cc * 32, o);
          wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          st32(O_t + cc * 32, o);
        }
      }
      const float nmb = (m == -INFINITY) ? 0.f : -m;
      uint32_t w[32];
      float rs0 = 0.f, rs1 = 0.f;
      if (lim == BK4 && EMU == 0) {
        // phase by phase over the 64 scores (all FMAs, all exponentials, all sums, all packs): each phase is
        // 32-64 independent instructions, so the scheduler overlaps their latencies instead of running one
        // dependent chain per pair
        float fa[32], fc[32];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          ffma2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]), sl2, nmb, fa[2 * i], fa[2 * i + 1]);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          ffma2(__uint_as_float(c[2 * i]), __uint_as_float(c[2 * i + 1]), sl2, nmb, fc[2 * i], fc[2 * i + 1]);
#pragma unroll
        for (int i = 0; i < 32; ++i) fa[i] = ex2(fa[i]);
#pragma unroll
        for (int i = 0; i < 32; ++i) fc[i] = ex2(fc[i]);
        float ra[4] = {0.f, 0.f, 0.f, 0.f}, rb[4] = {0.f, 0.f, 0.f, 0.f};  // four independent sum chains
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          fadd2(ra[i & 3], rb[i & 3], fa[2 * i], fa[2 * i + 1]);
          w[i] = pack_bf16(fa[2 * i], fa[2 * i + 1]);
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          fadd2(ra[i & 3], rb[i & 3], fc[2 * i], fc[2 * i + 1]);
          w[16 + i] = pack_bf16(fc[2 * i], fc[2 * i + 1]);
        }
        rs0 = (ra[0] + ra[1]) + (ra[2] + ra[3]);
        rs1 = (rb[0] + rb[1]) + (rb[2] + rb[3]);
      } else if (lim == BK4) {
        float ra[4] = {0.f, 0.f, 0.f, 0.f}, rb[4] = {0.f, 0.f, 0.f, 0.f};  // four independent sum chains
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t* v = i < 16 ? a : c;
          const int ii = i & 15;
          float x0, x1, e0, e1;
          ffma2(__uint_as_float(v[2 * ii]), __uint_as_float(v[2 * ii + 1]), sl2, nmb, x0, x1);
          if ((ii & 7) >= 8 - EMU) {  // EMU of every 8 pairs on the FMA pipe
            ex2_fma2(x0, x1, e0, e1);
          } else {
            e0 = ex2(x0);
            e1 = ex2(x1);
          }
          fadd2(ra[i & 3], rb[i & 3], e0, e1);
          w[i] = pack_bf16(e0, e1);
        }
        rs0 = (ra[0] + ra[1]) + (ra[2] + ra[3]);
        rs1 = (rb[0] + rb[1]) + (rb[2] + rb[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t* v = i < 16 ? a : c;
          const int ii = i & 15, k = 2 * i;
          const float e0 = k < lim ? ex2(fmaf(__uint_as_float(v[2 * ii]), sl2, nmb)) : 0.f;
          const float e1 = k + 1 < lim ? ex2(fmaf(__uint_as_float(v[2 * ii + 1]), sl2, nmb)) : 0.f;
          rs0 += e0;
          rs1 += e1;
          w[i] = pack_bf16(e0, e1);
        }
      }
      st32(S_b, w);  // P (bf16 pairs) over the first 32 columns of this score buffer
      wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      l = l * alpha + (rs0 + rs1);
    }
    // o_ready could not tell the last PV from the one two blocks earlier (equal parity): a barrier of its own
    if (ok && mbar_wait(o_final, 0, abort_flag, 70)) {
      fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int bb = bh / p.H, h = bh % p.H;
      const bool row_ok = q < p.Sq;
      __nv_bfloat16* dst = row_ok ? out_row(p, bb, q, h, D) : nullptr;
#pragma unroll
      for (int cc = 0; cc < D / 32; ++cc) {
        uint32_t o[32];
        ld32_nowait(O_t + cc * 32, o);
        wait_ld();
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint4 pk;
            pk.x = pack_bf16(__uint_as_float(o[g * 8 + 0]) * inv, __uint_as_float(o[g * 8 + 1]) * inv);
            pk.y = pack_bf16(__uint_as_float(o[g * 8 + 2]) * inv, __uint_as_float(o[g * 8 + 3]) * inv);
            pk.z = pack_bf16(__uint_as_float(o[g * 8 + 4]) * inv, __uint_as_float(o[g * 8 + 5]) * inv);
            pk.w = pack_bf16(__uint_as_float(o[g * 8 + 6]) * inv, __uint_as_float(o[g * 8 + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + cc * 32 + g * 8) = pk;
          }
        }
      }
      if (row_ok) p.lse[(int64_t)bh * p.Sq + q] = (m + __log2f(l)) * 0.69314718055994531f;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
}


// ====================================================================================================
// Forward v5 (head_dim 64): v4 with two softmax warpgroups per query tile.  Warpgroup h (warps 4h..4h+3)
// owns keys [32 h, 32 h + 32) of every 64-key block with its own running max, row sum and accumulator
// O_h (tensor-memory columns [128 + 64 h, 192 + 64 h)); the halves never synchronise inside the key loop
// and are combined once in the epilogue.  Twice the softmax warps per SM sub-partition hide the
// tensor-memory and MUFU latencies that bound v4 at this head width.  P of half h is packed into
// columns [32 h, 32 h + 16) of the score buffer (half 0's P lands on its own, already-read columns).
// 320 threads: warps 0..7 softmax, warp 8 TMA producer, warp 9 MMA issuer + TMEM allocator.
constexpr int FWD5_THREADS = 320;

__global__ void __launch_bounds__(FWD5_THREADS, 2)
    fmha_fwd5_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mk,
                     const __grid_constant__ CUtensorMap mv, const __grid_constant__ Params p) {
  constexpr int D = 64;
  using C = Cfg4<D>;
  extern __shared__ __align__(1024) uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;           // [ST]
  uint64_t* k_empty = k_full + C::ST;    // [ST]
  uint64_t* v_full = k_empty + C::ST;    // [ST]
  uint64_t* v_empty = v_full + C::ST;    // [ST]
  uint64_t* s_full = v_empty + C::ST;    // [2] per score buffer
  uint64_t* p_full = s_full + 2;         // [2]: 8 warps arrive
  uint64_t* o_ready = p_full + 2;        // [1] after every pair of PVs
  uint64_t* o_final = o_ready + 1;       // [1] after the last pair
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // epilogue exchange of the halves' (max, sum) per row: [half][2][128], then a per-half count of warps
  // that have written theirs (a bounded wait on it, never an unbounded barrier)
  float* xch = reinterpret_cast<float*>(sm + C::BAR_OFF + 256);
  int* xcnt = reinterpret_cast<int*>(xch + 512);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = p.npairs - 1 - (int)(blockIdx.x % p.npairs);
  const int bh = blockIdx.x / p.npairs;
  const int q0 = tile * BQ;
  int kv_end = kv_limit(p, bh);
  if (p.causal) kv_end = min(kv_end, q0 + BQ);
  const int nkv = (kv_end + BK4 - 1) / BK4;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < C::ST; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 8);
    }
    mbar_init(o_ready, 1);
    mbar_init(o_final, 1);
    *abort_flag = 0;
    xcnt[0] = xcnt[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    if (lane == 0 && nkv > 0) {
      mbar_expect_tx(q_full, C::Q_BYTES);
      tma_load_3d(sm + C::Q_OFF, &mq, q_full, 0, q0, bh);
      for (int j = 0; j < nkv; ++j) {
        const int s = j % C::ST, ph = ((j / C::ST) & 1) ^ 1;
        if (!mbar_wait(&k_empty[s], ph, abort_flag, 71)) break;
        mbar_expect_tx(&k_full[s], C::KV_BYTES);
        tma_load_3d(sm + C::K_OFF + s * C::KV_BYTES, &mk, &k_full[s], 0, j * BK4, bh);
        if (!mbar_wait(&v_empty[s], ph, abort_flag, 72)) break;
        mbar_expect_tx(&v_full[s], C::KV_BYTES);
        tma_load_3d(sm + C::V_OFF + s * C::KV_BYTES, &mv, &v_full[s], 0, j * BK4, bh);
      }
    }
  } else if (warp == 9) {
    if (lane == 0 && nkv > 0) {
      const uint32_t id_s = idesc(128, BK4, 0, 0);
      const uint32_t id_o = idesc(128, D, 0, 1);
      const uint32_t qa = smem_u32(sm + C::Q_OFF);
      auto issue_s = [&](int j) {
        const uint32_t ka = smem_u32(sm + C::K_OFF + (j % C::ST) * C::KV_BYTES);
        const uint32_t Sb = tmem + (j & 1) * BK4;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_ss(Sb, desc(qa + kk * 32, 16, 1024), desc(ka + kk * 32, 16, 1024), id_s, kk > 0);
        commit(&s_full[j & 1]);
        commit(&k_empty[j % C::ST]);
      };
      auto issue_pv = [&](int j) {
        const uint32_t va = smem_u32(sm + C::V_OFF + (j % C::ST) * C::KV_BYTES);
        const uint32_t Sb = tmem + (j & 1) * BK4;
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int kk = 0; kk < 2; ++kk)
            mma_ts(tmem + C::O_COL + 64 * h, Sb + 32 * h + kk * 8, desc(va + (2 * h + kk) * 2048, 8192, 1024), id_o,
                   (j > 0 || kk > 0) ? 1u : 0u);
        commit(o_ready);
        commit(&v_empty[j % C::ST]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, 73);
      for (int j = 0; ok && j < 2 && j < nkv; ++j) {
        if (!(ok = mbar_wait(&k_full[j % C::ST], (j / C::ST) & 1, abort_flag, 74))) break;
        fence_after();
        issue_s(j);
      }
      for (int j = 0; ok && j < nkv; ++j) {
        if (!mbar_wait(&v_full[j % C::ST], (j / C::ST) & 1, abort_flag, 75)) break;
        if (!mbar_wait(&p_full[j & 1], (j >> 1) & 1, abort_flag, 76)) break;
        fence_after();
        issue_pv(j);
        if (j + 1 == nkv) commit(o_final);
        if (j + 2 < nkv) {
          const int jn = j + 2;
          if (!mbar_wait(&k_full[jn % C::ST], (jn / C::ST) & 1, abort_flag, 77)) break;
          fence_after();
          issue_s(jn);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax halves (warps 0..7)
    const int hf = warp >> 2, quarter = warp & 3;
    const int row = 32 * quarter + lane;
    const int q = q0 + row;
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const uint32_t O_h = tmem + C::O_COL + 64 * hf + lane_off;
    const float sl2 = p.scale_log2;
    const int kvl = kv_limit(p, bh);
    float m = -INFINITY, l = 0.f;
    bool ok = nkv > 0;
    for (int j = 0; ok && j < nkv; ++j) {
      const int b = j & 1;
      if (!mbar_wait(&s_full[b], (j >> 1) & 1, abort_flag, 78)) {
        ok = false;
        break;
      }
      fence_after();
      const uint32_t S_h = tmem + b * BK4 + 32 * hf + lane_off;
      const int kv0 = j * BK4 + 32 * hf;
      int lim = kvl - kv0;
      if (p.causal) lim = min(lim, q - kv0 + 1);
      lim = max(0, min(32, lim));
      uint32_t a[32];
      ld32_nowait(S_h, a);
      wait_ld();
      float mx = -INFINITY;
      if (lim == 32) {
        float mq[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 16; ++i) mq[i & 3] = max3(mq[i & 3], __uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]));
        mx = fmaxf(fmaxf(mq[0], mq[1]), fmaxf(mq[2], mq[3]));
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (i < lim) mx = fmaxf(mx, __uint_as_float(a[i]));
      }
      const float m_blk = mx * sl2;
      float alpha = 1.f;
      const bool move = m_blk > m + RESCALE_THRESHOLD || (m == -INFINITY && m_blk != -INFINITY);
      if (move) {
        alpha = (m == -INFINITY) ? 0.f : ex2(m - m_blk);
        m = m_blk;
      }
      if (j > 0 && __any_sync(0xffffffffu, move)) {
        if (!mbar_wait(o_ready, (j - 1) & 1, abort_flag, 79)) {
          ok = false;
          break;
        }
        fence_after();
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {  // 16 columns at a time: the scores stay in registers
          uint32_t o[16];
          ld16_nowait(O_h + cc * 16, o);
          wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          st16(O_h + cc * 16, o);
        }
      }
      const float nmb = (m == -INFINITY) ? 0.f : -m;
      uint32_t w[16];
      float rs0 = 0.f, rs1 = 0.f;
      if (lim == 32) {
        float ra[4] = {0.f, 0.f, 0.f, 0.f}, rb[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float x0, x1, e0, e1;
          ffma2(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1]), sl2, nmb, x0, x1);
          if ((i & 7) >= 8 - kFwd4Emu64) {
            ex2_fma2(x0, x1, e0, e1);
          } else {
            e0 = ex2(x0);
            e1 = ex2(x1);
          }
          fadd2(ra[i & 3], rb[i & 3], e0, e1);
          w[i] = pack_bf16(e0, e1);
        }
        rs0 = (ra[0] + ra[1]) + (ra[2] + ra[3]);
        rs1 = (rb[0] + rb[1]) + (rb[2] + rb[3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int k = 2 * i;
          const float e0 = k < lim ? ex2(fmaf(__uint_as_float(a[k]), sl2, nmb)) : 0.f;
          const float e1 = k + 1 < lim ? ex2(fmaf(__uint_as_float(a[k + 1]), sl2, nmb)) : 0.f;
          rs0 += e0;
          rs1 += e1;
          w[i] = pack_bf16(e0, e1);
        }
      }
      st16(S_h, w);
      wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      l = l * alpha + (rs0 + rs1);
    }
    if (ok && mbar_wait(o_final, 0, abort_flag, 80)) {
      fence_after();
      xch[(hf * 2 + 0) * 128 + row] = m;
      xch[(hf * 2 + 1) * 128 + row] = l;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) atomicAdd(&xcnt[hf], 1);
      bool seen = false;
      const unsigned long long t0 = clock64();
      while (!(seen = (*reinterpret_cast<volatile int*>(&xcnt[hf ^ 1]) >= 4))) {
        if (*abort_flag) break;
        if (clock64() - t0 > WAIT_BUDGET) {
          atomicCAS(&g_error, 0, 81);
          *abort_flag = 1;
          break;
        }
      }
      __threadfence_block();
      if (seen) {
      const float m_o = xch[((hf ^ 1) * 2 + 0) * 128 + row], l_o = xch[((hf ^ 1) * 2 + 1) * 128 + row];
      const float m_out = fmaxf(m, m_o);
      const float c_me = (m == -INFINITY) ? 0.f : ex2(m - m_out);
      const float c_ot = (m_o == -INFINITY) ? 0.f : ex2(m_o - m_out);
      const float lt = l * c_me + l_o * c_ot;
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      // this half writes output columns [32 hf, 32 hf + 32): O_0 and O_1 combined with their weights
      const float c0 = (hf == 0 ? c_me : c_ot) * inv, c1 = (hf == 0 ? c_ot : c_me) * inv;
      const bool row_ok = q < p.Sq;
      __nv_bfloat16* dst = row_ok ? out_row(p, bh / p.H, q, bh % p.H, D) + 32 * hf : nullptr;
#pragma unroll
      for (int ch = 0; ch < 2; ++ch) {  // 16 output columns at a time
        uint32_t o0[16], o1[16];
        ld16_nowait(tmem + C::O_COL + 32 * hf + 16 * ch + lane_off, o0);
        ld16_nowait(tmem + C::O_COL + 64 + 32 * hf + 16 * ch + lane_off, o1);
        wait_ld();
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            float v[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              v[i] = __uint_as_float(o0[g * 8 + i]) * c0 + __uint_as_float(o1[g * 8 + i]) * c1;
            uint4 pk;
            pk.x = pack_bf16(v[0], v[1]);
            pk.y = pack_bf16(v[2], v[3]);
            pk.z = pack_bf16(v[4], v[5]);
            pk.w = pack_bf16(v[6], v[7]);
            *reinterpret_cast<uint4*>(dst + 16 * ch + g * 8) = pk;
          }
        }
      }
      if (row_ok) {
        if (hf == 0) p.lse[(int64_t)bh * p.Sq + q] = (m_out + __log2f(lt)) * 0.69314718055994531f;
      }
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
  }
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

// 3D map over [BH, S, D] bf16 with box {64, rows, 1}, 128B swizzle.
static int map3(CUtensorMap* m, const void* ptr, int BH, int S, int D, int rows = 128) {
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t str[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return (int)encode()(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, str, box, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int D, int SPLIT>
static int launch(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p,
                  unsigned grid, cudaStream_t stream) {
  static bool set = false;
  const int bytes = Cfg<D>::BYTES + 1024;
  if (!set) {
    const cudaError_t e =
        cudaFuncSetAttribute(fmha_fwd2_kernel<D, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  fmha_fwd2_kernel<D, SPLIT><<<grid, fwd_threads<SPLIT>(), bytes, stream>>>(mq, mk, mv, p);
  return (int)cudaGetLastError();
}

template <int D, int EMU>
static int launch4(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p,
                   unsigned grid, cudaStream_t stream) {
  static bool set = false;
  const int bytes = Cfg4<D>::BYTES + 1024;
  if (!set) {
    const cudaError_t e =
        cudaFuncSetAttribute(fmha_fwd4_kernel<D, EMU>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  fmha_fwd4_kernel<D, EMU><<<grid, FWD4_THREADS, bytes, stream>>>(mq, mk, mv, p);
  return (int)cudaGetLastError();
}

static int launch5(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const Params& p,
                   unsigned grid, cudaStream_t stream) {
  static bool set = false;
  const int bytes = Cfg4<64>::BYTES + 1024 + 3072;  // + the epilogue's (max, sum) exchange and counters
  if (!set) {
    const cudaError_t e = cudaFuncSetAttribute(fmha_fwd5_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return (int)e;
    set = true;
  }
  fmha_fwd5_kernel<<<grid, FWD5_THREADS, bytes, stream>>>(mq, mk, mv, p);
  return (int)cudaGetLastError();
}

struct PeerOut {
  void* const* o;   // per rank: image-row output [B, si, htot, D]
  void* const* o2;  // per rank: text-row output [B, sl - si, htot, D] (null entries when sl == si)
  int nranks, sl, si, htot, h0;
};

static int fwd2_impl(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse, int B,
                     int H, int Sq, int Skv, int D, float scale, int causal, cudaStream_t stream, int split,
                     const PeerOut* peer = nullptr, const int* kv_len = nullptr) {
  if (D != 64 && D != 128) return -1;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15)
    return -2;
  CUtensorMap mq, mk, mv;
  const int kv_rows = split >= 4 ? BK4 : 128;
  int r = map3(&mq, q, B * H, Sq, D);
  if (!r) r = map3(&mk, k, B * H, Skv, D, kv_rows);
  if (!r) r = map3(&mv, v, B * H, Skv, D, kv_rows);
  if (r) return r;
  Params p;
  memset(&p, 0, sizeof(p));
  if (peer) {
    if (peer->nranks < 1 || peer->nranks > 8 || peer->sl * peer->nranks != Sq || peer->si < 1 || peer->si > peer->sl ||
        peer->h0 + H > peer->htot)
      return -4;
    for (int r = 0; r < peer->nranks; ++r) {
      p.peer_o[r] = reinterpret_cast<__nv_bfloat16*>(peer->o[r]);
      p.peer_o2[r] = peer->sl > peer->si ? reinterpret_cast<__nv_bfloat16*>(peer->o2[r]) : nullptr;
      if (!p.peer_o[r] || (peer->sl > peer->si && !p.peer_o2[r])) return -4;
    }
    p.peer_sl = peer->sl;
    p.peer_si = peer->si;
    p.peer_htot = peer->htot;
    p.peer_h0 = peer->h0;
  }
  p.kv_len = kv_len;
  p.Sq = Sq;
  p.Skv = Skv;
  p.H = H;
  // v4: one query tile per CTA (npairs counts tiles); v1-v3: pairs of tiles
  p.npairs = split >= 4 ? (Sq + BQ - 1) / BQ : (Sq + 2 * BQ - 1) / (2 * BQ);  // 40..48 count as 4
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.o2 = reinterpret_cast<__nv_bfloat16*>(o2);
  p.split = out_split;
  if (out_split < 0 || out_split >= Sq || (out_split > 0 && !o2)) return -3;
  p.lse = lse;
  const long long grid = (long long)p.npairs * B * H;
  if (grid == 0) return 0;
  if (split == 5 && D == 64) return launch5(mq, mk, mv, p, (unsigned)grid, stream);
  // exponentials on the FMA pipe per 8 pairs: kFwd4Emu (head_dim 64, where MUFU bounds the score path),
  // none at head_dim 128 (tensor-bound); versions 40..48 select 0..8 of 8 for measurements
  if (split >= 40 && split <= 48) {
    const int emu = split - 40;
    if (D == 64) {
      switch (emu) {
        case 0: return launch4<64, 0>(mq, mk, mv, p, (unsigned)grid, stream);
        case 1: return launch4<64, 1>(mq, mk, mv, p, (unsigned)grid, stream);
        case 2: return launch4<64, 2>(mq, mk, mv, p, (unsigned)grid, stream);
        case 4: return launch4<64, 4>(mq, mk, mv, p, (unsigned)grid, stream);
        default: return launch4<64, 3>(mq, mk, mv, p, (unsigned)grid, stream);
      }
    }
    return emu == 0 ? launch4<128, 0>(mq, mk, mv, p, (unsigned)grid, stream)
                    : launch4<128, 2>(mq, mk, mv, p, (unsigned)grid, stream);
  }
  if (split >= 4)
    return D == 64 ? launch4<64, kFwd4Emu64>(mq, mk, mv, p, (unsigned)grid, stream)
                   : launch4<128, 0>(mq, mk, mv, p, (unsigned)grid, stream);
  if (D == 64)
    return split == 3 ? launch<64, 3>(mq, mk, mv, p, (unsigned)grid, stream)
           : split == 2 ? launch<64, 2>(mq, mk, mv, p, (unsigned)grid, stream)
                        : launch<64, 1>(mq, mk, mv, p, (unsigned)grid, stream);
  return split == 2 ? launch<128, 2>(mq, mk, mv, p, (unsigned)grid, stream)
                    : launch<128, 1>(mq, mk, mv, p, (unsigned)grid, stream);
}

}  // namespace vo_fmha2

// o2 / out_split: rows q >= out_split go to o2 ([B, Sq - out_split, H, D]); out_split = 0: one output
extern "C" int vo_fmha_fwd2(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            int B, int H, int Sq, int Skv, int D, float scale, int causal, cudaStream_t stream) {
  return vo_fmha2::fwd2_impl(q, k, v, o, o2, out_split, lse, B, H, Sq, Skv, D, scale, causal, stream, 1);
}

// two softmax warpgroups per query tile (576 threads); head_dim 64: independent key halves
extern "C" int vo_fmha_fwd3(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            int B, int H, int Sq, int Skv, int D, float scale, int causal, cudaStream_t stream) {
  return vo_fmha2::fwd2_impl(q, k, v, o, o2, out_split, lse, B, H, Sq, Skv, D, scale, causal, stream, D == 64 ? 3 : 2);
}

// Ulysses attention with the output exchange fused into the epilogue: q/k/v hold this rank's heads of the
// gathered sequence; every output row is written into the owning rank's image / text buffer (peer
// pointers of a sequence-parallel group, this rank's heads at head offset h0 of htot).
extern "C" int vo_fmha_fwd_peer(const void* q, const void* k, const void* v, void* const* peer_o,
                                void* const* peer_o2, int nranks, int sl, int si, int htot, int h0, float* lse, int B,
                                int H, int Sq, int Skv, int D, float scale, cudaStream_t stream) {
  vo_fmha2::PeerOut po{peer_o, peer_o2, nranks, sl, si, htot, h0};
  return vo_fmha2::fwd2_impl(q, k, v, nullptr, nullptr, 0, lse, B, H, Sq, Skv, D, scale, 0, stream, D == 64 ? 3 : 2,
                             &po);
}

// forward v3 with a per-sequence key count (int32 [B], device memory)
extern "C" int vo_fmha_fwd3_kvlen(const void* q, const void* k, const void* v, void* o, void* o2, int out_split,
                                  float* lse, const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale,
                                  cudaStream_t stream) {
  return vo_fmha2::fwd2_impl(q, k, v, o, o2, out_split, lse, B, H, Sq, Skv, D, scale, 0, stream, D == 64 ? 3 : 2,
                             nullptr, kv_len);
}

extern "C" int vo_fmha_fwd2_error(int reset) {
  int e = 0;
  cudaMemcpyFromSymbol(&e, vo_fmha2::g_error, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(vo_fmha2::g_error, &z, sizeof(int));
  }
  return e;
}

// forward v4 (one query tile per CTA, two CTAs per SM, double-buffered 64-key score blocks); optional
// per-sequence key count (int32 [B] in device memory, or null) and causal mask
extern "C" int vo_fmha_fwd4(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                            cudaStream_t stream) {
  return vo_fmha2::fwd2_impl(q, k, v, o, o2, out_split, lse, B, H, Sq, Skv, D, scale, causal, stream, 4, nullptr,
                             kv_len);
}

// Ulysses attention (peer output rows) on forward v4
extern "C" int vo_fmha_fwd4_peer(const void* q, const void* k, const void* v, void* const* peer_o,
                                 void* const* peer_o2, int nranks, int sl, int si, int htot, int h0, float* lse, int B,
                                 int H, int Sq, int Skv, int D, float scale, cudaStream_t stream) {
  vo_fmha2::PeerOut po{peer_o, peer_o2, nranks, sl, si, htot, h0};
  return vo_fmha2::fwd2_impl(q, k, v, nullptr, nullptr, 0, lse, B, H, Sq, Skv, D, scale, 0, stream, 4, &po);
}

// forward v5: head_dim 64 with two independent softmax halves per query tile (other widths run v4)
extern "C" int vo_fmha_fwd5(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                            const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                            cudaStream_t stream) {
  return vo_fmha2::fwd2_impl(q, k, v, o, o2, out_split, lse, B, H, Sq, Skv, D, scale, causal, stream, 5, nullptr,
                             kv_len);
}

extern "C" int vo_fmha_fwd5_peer(const void* q, const void* k, const void* v, void* const* peer_o,
                                 void* const* peer_o2, int nranks, int sl, int si, int htot, int h0, float* lse, int B,
                                 int H, int Sq, int Skv, int D, float scale, cudaStream_t stream) {
  vo_fmha2::PeerOut po{peer_o, peer_o2, nranks, sl, si, htot, h0};
  return vo_fmha2::fwd2_impl(q, k, v, nullptr, nullptr, 0, lse, B, H, Sq, Skv, D, scale, 0, stream, 5, &po);
}

// forward v4 with an explicit exponential split (variant 40..48: 0..8 of every 8 pairs on the FMA pipe)
extern "C" int vo_fmha_fwd4v(const void* q, const void* k, const void* v, void* o, void* o2, int out_split, float* lse,
                             const int* kv_len, int B, int H, int Sq, int Skv, int D, float scale, int causal,
                             cudaStream_t stream, int variant) {
  if (variant < 40 || variant > 48) return -1;
  return vo_fmha2::fwd2_impl(q, k, v, o, o2, out_split, lse, B, H, Sq, Skv, D, scale, causal, stream, variant,
                             nullptr, kv_len);
}
