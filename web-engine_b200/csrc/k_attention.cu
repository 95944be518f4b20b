// Attention: softmax(q k^T / sqrt(dim)) v with grouped-query heads, the reference's attention()
// (src/kernels/attention.ts:20-51: matmul -> softmax -> matmul per head and query chunk; GQA kv head
// = floor(h / (heads / kvHeads)); optional causal mask for the text encoder).
//
// Two kernels:
//  * attention_simt_kernel: CUDA cores, fp32, one warp per (query, head) with an online softmax over
//    the keys. The exact path for the reference's f32 buffers (its tests hold 1e-5) and for head
//    sizes / masks the tensor-core kernel does not take.
//  * flash_attn2_kernel: tcgen05 flash attention for bf16 q/k/v with 128-wide heads, no mask (the DiT
//    blocks). One CTA = one head x 256 queries (two 128-row tiles). Warp 0 TMA-loads both Q tiles once
//    and K / V key tiles of 128 into separate 2-stage rings (K runs two tiles ahead); warp 1 issues
//    S_i = Q_i K^T into TMEM and O_i += P_i V with P read from TMEM and V an MN-major operand straight from
//    its [tokens, kv_heads, dim] layout, interleaving the two tiles; warps 2-17 (two groups of eight, a
//    thread = one query row and one half of the keys, so two warps per scheduler work on each group) run the
//    online softmax (tcgen05.ld, packed f32x2 math, three quarters of the exponentials on the transcendental
//    unit and one quarter as a cubic on the FMA pipe), write P as bf16 over the first half of S_i
//    (tcgen05.st), and rescale O_i in TMEM only when a row's running maximum grows by more than 2^8 (the
//    probabilities stay <= 256 in between, which fp32 accumulation and bf16 P hold without loss of relative
//    precision).
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace we {

// ---------------- CUDA-core attention (fp32, exact reference semantics) ----------------
template <int DT, int OT, int VPL>
__global__ void __launch_bounds__(128) attention_simt_kernel(const void* __restrict__ q, const void* __restrict__ k,
                                                             const void* __restrict__ v, int64_t tokens, int64_t heads,
                                                             int64_t kv_heads, int64_t dim, int causal, float scale,
                                                             void* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = tokens * heads;
  const int64_t warps = (int64_t)gridDim.x * 4;
  const int64_t group = heads / kv_heads;
  for (int64_t row = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t i = row / heads, h = row % heads, g = h / group;
    float qv[VPL], acc[VPL];
#pragma unroll
    for (int e = 0; e < VPL; e++) {
      const int64_t d = lane + 32 * e;
      qv[e] = d < dim ? load_act<DT>(q, row * dim + d) * scale : 0.f;
      acc[e] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int64_t n = causal ? i + 1 : tokens;
    for (int64_t j = 0; j < n; j++) {
      const int64_t kb = (j * kv_heads + g) * dim;
      float dot = 0.f;
#pragma unroll
      for (int e = 0; e < VPL; e++) {
        const int64_t d = lane + 32 * e;
        if (d < dim) dot = fmaf(qv[e], load_act<DT>(k, kb + d), dot);
      }
      const float s = warp_sum(dot);
      const float mn = fmaxf(m, s);
      const float corr = expf(m - mn);  // m = -inf on the first key: corr = 0
      const float p = expf(s - mn);
      l = l * corr + p;
#pragma unroll
      for (int e = 0; e < VPL; e++) {
        const int64_t d = lane + 32 * e;
        acc[e] = acc[e] * corr + (d < dim ? p * load_act<DT>(v, kb + d) : 0.f);
      }
      m = mn;
    }
#pragma unroll
    for (int e = 0; e < VPL; e++) {
      const int64_t d = lane + 32 * e;
      if (d < dim) store_out<OT>(out, row * dim + d, acc[e] / l);
    }
  }
}

// ---------------- tcgen05 flash attention ----------------
// Blackwell packed-pair and 3-input forms (PTX ISA 8.6+ for sm_100a): one instruction per two values
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
  const float2 d = __ffma2_rn(make_float2(a0, a1), make_float2(b0, b1), make_float2(c0, c1));
  d0 = d.x;
  d1 = d.y;
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  const float2 d = __fadd2_rn(make_float2(a0, a1), make_float2(b0, b1));
  d0 = d.x;
  d1 = d.y;
}
// the hardware 2^x (MUFU.EX2, results below 2^-126 flush to 0: negligible weights)
__device__ __forceinline__ float exp2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// 2^x for two x <= 2^22 on the FMA pipe, leaving the transcendental unit to the other exponentials of the row:
// x = n + f with n = floor(x) (an add rounding toward -inf against 1.5 * 2^23 leaves n in the low mantissa bits),
// 2^f on [0, 1) by a cubic 1 + f (c1 + f (c2 + f c3)), and n added to the result's exponent field. The cubic is a
// relative-error minimax fit of 2^f on [0, 1) (Lawson's iteratively reweighted least squares): max relative
// error 9.5e-5, below bf16's 2^-9. x is clamped to -126 first, so a masked key (x = -inf) weighs 2^-126 ~ 1e-38.
__device__ __forceinline__ void exp2_poly2(float& y0, float& y1, float x0, float x1) {
  constexpr float C1 = 0.69507056f, C2 = 0.22765099f, C3 = 0.07714326f, MAGIC = 12582912.f;
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float n0, n1, f0, f1, p0, p1;
  const float2 t = __fadd2_rd(make_float2(x0, x1), make_float2(MAGIC, MAGIC));
  const float t0 = t.x, t1 = t.y;
  fadd2(n0, n1, t0, t1, -MAGIC, -MAGIC);  // floor(x), exact
  fadd2(f0, f1, x0, x1, -n0, -n1);        // f in [0, 1)
  ffma2(p0, p1, f0, f1, C3, C3, C2, C2);
  ffma2(p0, p1, p0, p1, f0, f1, C1, C1);
  ffma2(p0, p1, p0, p1, f0, f1, 1.f, 1.f);
  y0 = __uint_as_float(__float_as_uint(p0) + (__float_as_uint(t0) << 23));
  y1 = __uint_as_float(__float_as_uint(p1) + (__float_as_uint(t1) << 23));
}
// two non-negative f32 as bf16x2 (lo in the low half) with integer ops instead of the conversion unit: round to
// nearest by adding half a bf16 ulp to the bits (ties away from zero), then keep the high halves
__device__ __forceinline__ uint32_t pack_bf16x2_int(float lo, float hi) {
  return __byte_perm(__float_as_uint(lo) + 0x8000u, __float_as_uint(hi) + 0x8000u, 0x7632);
}

// which pair slots (e mod 8) of a row take the FMA-pipe exponential instead of MUFU.EX2. 0: none. Measured on
// config 3's attention (4608 tokens, 24 heads): none 258 us, a quarter 274 us, three eighths 280 us, a half
// 279 us. The softmax warps are bound by instruction issue, not by the transcendental unit.
#ifndef FA_POLY_MASK
#define FA_POLY_MASK 0x00
#endif
// 1: pack P to bf16 with cvt.rn.bf16x2.f32 (one instruction per pair); 0: with integer rounding (three)
#ifndef FA_PACK_CVT
#define FA_PACK_CVT 0
#endif

namespace fa {
struct Params {
  int64_t tokens, heads, kv_heads;
  float scale_log2;  // log2(e) / sqrt(dim)
  void* out;
  int out_dtype;
  uint32_t* err;
  // key splits (gridDim.z > 1): split z takes key tiles [z nt / splits, (z + 1) nt / splits) and writes its
  // unnormalised O rows (f32) to part_o[z][token][head][dim] and the rows' (max, sum) to part_ml[z][token][head]
  float* part_o;
  float* part_ml;
};
}  // namespace fa

// ---------------- two query tiles per CTA, P in TMEM ----------------
// One CTA = 256 queries (two 128-row tiles) of one head; K and V tiles of 128 keys are loaded once for both.
// TMEM (512 columns): S_i at 128 i, O_i at 256 + 128 i. Each softmax group (8 warps, thread = query row x half) turns
// S_i into bf16 P written back over the first 64 columns of S_i, and O_i += P_i V_j reads P straight from TMEM
// (no shared-memory round trip for P). The MMA warp interleaves the two tiles:
//     S0(0) S1(0) | PV0(0) S0(1) PV1(0) S1(1) | PV0(1) S0(2) PV1(1) S1(2) | ...
// so each softmax group works while the tensor core runs the other group's PV and S. The commit that signals
// S_i(j) also covers PV_i(j - 1) (issued before it), so the softmax may overwrite P_i and rescale O_i then.
namespace fa2 {
constexpr int BQ = 128, BK = 128, D = 128, QT = 2;
constexpr int ATOM = 128 * 128;  // one 128-row x 128-byte swizzle-128B box (64 bf16 per row)
constexpr int TILE = 2 * ATOM;   // 128 rows x 128 dims (or dims x keys for V^T)
constexpr int STAGES = 2;
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + QT * TILE;
constexpr int V_OFF = K_OFF + STAGES * TILE;
constexpr int BAR_OFF = V_OFF + STAGES * TILE;
// barriers: q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[QT], p_full[QT], pv_done[QT], drain
constexpr int NUM_BARS = 1 + 8 + 3 * QT + 1;
constexpr int RED_OFF = BAR_OFF + NUM_BARS * 8 + 16;              // row maxima (two tile parities) and row sums
constexpr int TOTAL = RED_OFF + (2 * QT * 2 * BQ + QT * 2 * BQ) * 4;
constexpr int ALLOC = TOTAL + 1024;
constexpr int SOFTMAX_WARPS = 8;                                   // per query tile: 4 row quarters x 2 key halves
constexpr int THREADS = 64 + QT * SOFTMAX_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t O_COL = 256;
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr uint32_t IDESC_V = IDESC | (1u << 16);  // B (V) MN-major
constexpr float RESCALE_LOG2 = 8.f;
}  // namespace fa2

__global__ void __launch_bounds__(fa2::THREADS, 1)
    flash_attn2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const fa::Params p) {
  using namespace tc;
  using namespace fa2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  pdl_launch_dependents();  // a kernel launched by launch_pdl after this one may place its CTAs as these finish
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + BAR_OFF;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + BAR_OFF + NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const uint32_t Q_FULL = bars;
#define K_FULL(s) (bars + 8u * (1 + (s)))
#define K_EMPTY(s) (bars + 8u * (3 + (s)))
#define V_FULL(s) (bars + 8u * (5 + (s)))
#define V_EMPTY(s) (bars + 8u * (7 + (s)))
#define S_FULL(i) (bars + 8u * (9 + (i)))
#define P_FULL(i) (bars + 8u * (9 + QT + (i)))
#define PV_DONE(i) (bars + 8u * (9 + 2 * QT + (i)))
#define DRAIN (bars + 8u * (9 + 3 * QT))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t q0 = (int64_t)blockIdx.x * (QT * BQ);
  const int64_t h = blockIdx.y;
  const int64_t g = h / (p.heads / p.kv_heads);
  const int nt_all = (int)((p.tokens + BK - 1) / BK);
  const int j0 = (int)((int64_t)blockIdx.z * nt_all / gridDim.z);  // this split's first key tile
  const int nt = (int)((int64_t)(blockIdx.z + 1) * nt_all / gridDim.z) - j0;

  if (threadIdx.x == 0) {
    mbar_init(Q_FULL, 1);
    for (int i = 0; i < 2; i++) {
      mbar_init(K_FULL(i), 1);
      mbar_init(K_EMPTY(i), 1);
      mbar_init(V_FULL(i), 1);
      mbar_init(V_EMPTY(i), 1);
    }
    for (int i = 0; i < QT; i++) {
      mbar_init(S_FULL(i), 1);
      mbar_init(P_FULL(i), SOFTMAX_WARPS);
      mbar_init(PV_DONE(i), 1);
    }
    mbar_init(DRAIN, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_holder), TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // launched by launch_pdl: q, k and v are complete before any global access

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      mbar_expect_tx(Q_FULL, QT * TILE);
      for (int i = 0; i < QT; i++) {
        tma_load_2d(sbase + Q_OFF + i * TILE, &tm_q, Q_FULL, (int32_t)(h * D), (int32_t)(q0 + i * BQ));
        tma_load_2d(sbase + Q_OFF + i * TILE + ATOM, &tm_q, Q_FULL, (int32_t)(h * D + 64), (int32_t)(q0 + i * BQ));
      }
      // K runs two tiles ahead of V: V_j, then K_{j+2} (its stage is freed once S0(j) and S1(j) are done)
      auto load_k = [&](int t) -> bool {
        const int st = t & 1;
        if (!wait_fast(K_EMPTY(st), ((t >> 1) & 1) ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER,
                          WAIT_LIMIT_NS, true))
          return false;
        const uint32_t dst = sbase + K_OFF + st * TILE;
        mbar_expect_tx(K_FULL(st), TILE);
        tma_load_2d(dst, &tm_k, K_FULL(st), (int32_t)(g * D), (j0 + t) * BK);
        tma_load_2d(dst + ATOM, &tm_k, K_FULL(st), (int32_t)(g * D + 64), (j0 + t) * BK);
        return true;
      };
      auto load_v = [&](int t) -> bool {
        const int st = t & 1;
        if (!wait_fast(V_EMPTY(st), ((t >> 1) & 1) ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER,
                          WAIT_LIMIT_NS, true))
          return false;
        const uint32_t dst = sbase + V_OFF + st * TILE;
        mbar_expect_tx(V_FULL(st), TILE);
        tma_load_2d(dst, &tm_v, V_FULL(st), (int32_t)(g * D), (j0 + t) * BK);  // V as stored: keys x 64 dims per box
        tma_load_2d(dst + ATOM, &tm_v, V_FULL(st), (int32_t)(g * D + 64), (j0 + t) * BK);
        return true;
      };
      int k_issued = 0, v_issued = 0;
      for (int t = 0; t < 2 && t < nt && ok; t++) {
        ok = load_k(t);
        if (ok) k_issued = t + 1;
      }
      for (int j = 0; j < nt && ok; j++) {
        ok = load_v(j);
        if (!ok) break;
        v_issued = j + 1;
        if (j + 2 < nt) {
          ok = load_k(j + 2);
          if (ok) k_issued = j + 3;
        }
      }
      if (!ok) {  // the copies already issued land before the CTA exits
        wait_fast(Q_FULL, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
        for (int t = k_issued - 2 < 0 ? 0 : k_issued - 2; t < k_issued; t++)
          wait_fast(K_FULL(t & 1), (t >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
        for (int t = v_issued - 2 < 0 ? 0 : v_issued - 2; t < v_issued; t++)
          wait_fast(V_FULL(t & 1), (t >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = wait_fast(Q_FULL, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true);
      tc_fence_after();
      // S_i(j) = Q_i K_j^T into TMEM columns [128 i, 128 i + 128)
      auto s_mma = [&](int i, int j) -> bool {
        if (!wait_fast(K_FULL(j & 1), (j >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true))
          return false;
        tc_fence_after();
        const uint64_t qdesc = sw128_desc(sbase + Q_OFF + i * TILE);
        const uint64_t kdesc = sw128_desc(sbase + K_OFF + (j & 1) * TILE);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {  // K = 128 dims: two 64-dim boxes, 4 MMAs of 16 each
          const uint64_t off = (uint64_t)((kk >> 2) * (ATOM >> 4) + (kk & 3) * 2);
          umma<true>(tmem + (uint32_t)(i * 128), qdesc + off, kdesc + off, IDESC, kk != 0);
        }
        umma_commit(S_FULL(i));
        return true;
      };
      // O_i += P_i(j) V_j: A = P_i from TMEM columns [128 i, 128 i + 64), B = V_j from shared memory, MN-major (dims
      // contiguous, as V is stored): two 64-dim boxes of 128 keys, the second one ATOM bytes after the first
      auto pv_mma = [&](int i, int j) -> bool {
        if (!wait_spin(P_FULL(i), j & 1, 4096, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true) ||
            !wait_fast(V_FULL(j & 1), (j >> 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true))
          return false;
        tc_fence_after();
        const uint64_t vdesc = mn_sw128_desc(sbase + V_OFF + (j & 1) * TILE, ATOM);
#pragma unroll
        for (int kk = 0; kk < 8; kk++) {  // K = 128 keys: 8 MMAs of 16 keys (16 rows of 128 bytes) = 8 TMEM columns of P
          umma_tmem_a(tmem + O_COL + (uint32_t)(i * 128), tmem + (uint32_t)(i * 128 + kk * 8),
                      vdesc + (uint64_t)(kk * (16 * 128 >> 4)), IDESC_V, (j | kk) != 0);
        }
        umma_commit(PV_DONE(i));
        return true;
      };
      if (ok && nt > 0) {
        ok = s_mma(0, 0) && s_mma(1, 0);
        if (ok) umma_commit(K_EMPTY(0));
      }
      for (int j = 0; j < nt && ok; j++) {
        const bool more = j + 1 < nt;
        ok = pv_mma(0, j) && (!more || s_mma(0, j + 1)) && pv_mma(1, j);
        if (!ok) break;
        umma_commit(V_EMPTY(j & 1));
        if (more) {
          ok = s_mma(1, j + 1);
          if (ok) umma_commit(K_EMPTY((j + 1) & 1));
        }
      }
      // every MMA this thread issued completes before TMEM is freed
      umma_commit(DRAIN);
      wait_fast(DRAIN, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
    }
    __syncwarp();
  } else {
    // softmax: group grp (query tile i = grp) of 8 warps; a thread holds query row r (TMEM lane r) and one half of
    // the 128 keys of a tile (and of the 128 output dims). The two warps of a row quarter exchange their halves'
    // maxima through shared memory behind a 64-thread named barrier, so both take the same rescaling decisions.
    const int sw = warp - 2;
    const int grp = sw >> 3;
    const int half = (sw >> 2) & 1;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = (uint32_t)(grp * 128), o_col = O_COL + (uint32_t)(grp * 128 + half * 64);
    const uint32_t pair_bar = 1u + (uint32_t)(grp * 4 + quarter);
    float* red_max = reinterpret_cast<float*>(smem + RED_OFF);         // [2 parities][QT][2 halves][128 rows]
    float* red_sum = red_max + 2 * QT * 2 * BQ;                       // [QT][2 halves][128 rows]
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; j++) {
      ok = wait_fast(S_FULL(grp), j & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE, WAIT_LIMIT_NS, true);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      uint32_t sc[64];
      tmem_ld32_async(tmem + lane_addr + s_col + (uint32_t)(half * 64), *reinterpret_cast<uint32_t(*)[32]>(sc));
      tmem_ld32_async(tmem + lane_addr + s_col + (uint32_t)(half * 64 + 32), *reinterpret_cast<uint32_t(*)[32]>(sc + 32));
      tmem_wait_ld(*reinterpret_cast<uint32_t(*)[32]>(sc));
      reg_fence(*reinterpret_cast<uint32_t(*)[32]>(sc + 32));
      const int64_t valid = p.tokens - (int64_t)(j0 + j) * BK - half * 64;  // keys of this half that exist (uniform)
      if (valid < 64) {
#pragma unroll
        for (int c = 0; c < 64; c++)
          if (c >= valid) sc[c] = __float_as_uint(-INFINITY);
      }
      float mx[4];
#pragma unroll
      for (int i = 0; i < 4; i++) mx[i] = fmaxf(__uint_as_float(sc[2 * i]), __uint_as_float(sc[2 * i + 1]));
#pragma unroll
      for (int c = 8; c < 64; c += 8)
#pragma unroll
        for (int i = 0; i < 4; i++) mx[i] = max3f(mx[i], __uint_as_float(sc[c + 2 * i]), __uint_as_float(sc[c + 2 * i + 1]));
      float* rm = red_max + ((j & 1) * QT + grp) * 2 * BQ;
      rm[half * BQ + r] = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      // the exchange barrier also ANDs the two warps' wait results, so a pair always leaves the loop together
      if (!named_bar_and(pair_bar, 64, ok)) {
        ok = false;
        break;
      }
      const float mt = fmaxf(rm[r], rm[BQ + r]) * p.scale_log2;
      float corr = 1.f;
      const bool grow = mt > m_used + RESCALE_LOG2;
      if (grow) {
        corr = exp2_approx(m_used - mt);  // 0 on the first tile
        l *= corr;
        m_used = mt;
      }
      const float nm = -m_used;
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // 4 packed pairs of running sums
      uint32_t pk[32];  // this half's 64 keys as 32 packed bf16 pairs: P columns [32 half, 32 half + 32) of S_i
#pragma unroll
      for (int e = 0; e < 32; e++) {
        const int c = 2 * e;
        float x0, x1, e0, e1;
        ffma2(x0, x1, __uint_as_float(sc[c]), __uint_as_float(sc[c + 1]), p.scale_log2, p.scale_log2, nm, nm);
        if ((FA_POLY_MASK >> (e & 7)) & 1) {  // a share of the row on the FMA pipe, the rest on the MUFU
          exp2_poly2(e0, e1, x0, x1);
        } else {
          e0 = exp2_approx(x0);
          e1 = exp2_approx(x1);
        }
        fadd2(acc[2 * (e & 3)], acc[2 * (e & 3) + 1], acc[2 * (e & 3)], acc[2 * (e & 3) + 1], e0, e1);
        pk[e] = FA_PACK_CVT ? pack_bf16x2(e0, e1) : pack_bf16x2_int(e0, e1);
      }
      tmem_st32(tmem + lane_addr + s_col + (uint32_t)(half * 32), pk);
      l += ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
      // O_i was scaled for the old maximum: bring this half of it to the new one before PV_i(j) adds to it
      // (PV_i(j-1) is done: its commit preceded S_i(j)'s)
      if (__any_sync(0xffffffffu, grow && j > 0)) {
        const float f = (grow && j > 0) ? corr : 1.f;
#pragma unroll
        for (int c = 0; c < 2; c++) {
          uint32_t u[32];
          tmem_ld32(tmem + lane_addr + o_col + (uint32_t)(c * 32), u);
#pragma unroll
          for (int e = 0; e < 32; e++) u[e] = __float_as_uint(__uint_as_float(u[e]) * f);
          tmem_st32(tmem + lane_addr + o_col + (uint32_t)(c * 32), u);
        }
      }
      tmem_st_wait();  // P (and O) stores land before the MMA reads them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(P_FULL(grp));
    }
    if (ok && nt > 0) {
      // the row's sum over both halves of the keys
      red_sum[(grp * 2 + half) * BQ + r] = l;
      named_bar_sync(pair_bar, 64);
      l += red_sum[(grp * 2 + (half ^ 1)) * BQ + r];
      ok = wait_fast(PV_DONE(grp), (nt - 1) & 1, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE, WAIT_LIMIT_NS, true);
      if (__all_sync(0xffffffffu, ok)) {
        tc_fence_after();
        const int64_t qi = q0 + grp * BQ + r;
        const float inv = 1.f / l;
        if (p.part_o) {  // a key split: the unnormalised rows and (max, sum), merged by flash_combine_kernel
          const int64_t row = ((int64_t)blockIdx.z * p.tokens + qi) * p.heads + h;
#pragma unroll
          for (int c = 0; c < 2; c++) {
            uint32_t u[32];
            tmem_ld32(tmem + lane_addr + o_col + (uint32_t)(c * 32), u);
            if (qi < p.tokens) {
              float4* dst = reinterpret_cast<float4*>(p.part_o + row * D + half * 64 + c * 32);
#pragma unroll
              for (int e = 0; e < 8; e++)
                dst[e] = make_float4(__uint_as_float(u[4 * e]), __uint_as_float(u[4 * e + 1]),
                                     __uint_as_float(u[4 * e + 2]), __uint_as_float(u[4 * e + 3]));
            }
          }
          if (qi < p.tokens && half == 0) {
            p.part_ml[2 * row] = m_used;
            p.part_ml[2 * row + 1] = l;
          }
        } else {
#pragma unroll
        for (int c = 0; c < 2; c++) {  // this half's 64 output dims
          uint32_t u[32];
          tmem_ld32(tmem + lane_addr + o_col + (uint32_t)(c * 32), u);
          if (qi < p.tokens) {
            const int64_t o = (qi * p.heads + h) * D + half * 64 + c * 32;
            if (p.out_dtype == WE_BF16) {
              uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(p.out) + o);
#pragma unroll
              for (int e = 0; e < 4; e++)
                dst[e] = make_uint4(pack_bf16x2(__uint_as_float(u[8 * e]) * inv, __uint_as_float(u[8 * e + 1]) * inv),
                                    pack_bf16x2(__uint_as_float(u[8 * e + 2]) * inv, __uint_as_float(u[8 * e + 3]) * inv),
                                    pack_bf16x2(__uint_as_float(u[8 * e + 4]) * inv, __uint_as_float(u[8 * e + 5]) * inv),
                                    pack_bf16x2(__uint_as_float(u[8 * e + 6]) * inv, __uint_as_float(u[8 * e + 7]) * inv));
            } else {
              float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + o);
#pragma unroll
              for (int e = 0; e < 8; e++)
                dst[e] = make_float4(__uint_as_float(u[4 * e]) * inv, __uint_as_float(u[4 * e + 1]) * inv,
                                     __uint_as_float(u[4 * e + 2]) * inv, __uint_as_float(u[4 * e + 3]) * inv);
            }
          }
        }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
#undef K_FULL
#undef K_EMPTY
#undef V_FULL
#undef V_EMPTY
#undef S_FULL
#undef P_FULL
#undef PV_DONE
#undef DRAIN
}


// Merges the key splits of flash_attn2_kernel: per (token, head) row, with M the largest split maximum,
// O = sum_z 2^(m_z - M) O_z / sum_z 2^(m_z - M) l_z (the maxima are in log2 units). One warp per row, 4 dims a lane.
template <int OT>
__global__ void __launch_bounds__(256) flash_combine_kernel(const float* __restrict__ part_o,
                                                            const float* __restrict__ part_ml, int splits,
                                                            int64_t rows, void* __restrict__ out) {
  pdl_wait();  // launched by launch_pdl: the splits' partial rows are complete (every CTA waits, even an idle one)
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int z = 0; z < splits; z++) mx = fmaxf(mx, part_ml[2 * ((int64_t)z * rows + row)]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float lsum = 0.f;
  for (int z = 0; z < splits; z++) {
    const int64_t zr = (int64_t)z * rows + row;
    const float w = exp2f(part_ml[2 * zr] - mx);
    lsum = fmaf(part_ml[2 * zr + 1], w, lsum);
    const float4 o = reinterpret_cast<const float4*>(part_o + zr * 128)[lane];
    acc.x = fmaf(o.x, w, acc.x);
    acc.y = fmaf(o.y, w, acc.y);
    acc.z = fmaf(o.z, w, acc.z);
    acc.w = fmaf(o.w, w, acc.w);
  }
  const float inv = 1.f / lsum;
  if (OT == WE_BF16) {
    uint2* dst = reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + row * 128) + lane;
    *dst = make_uint2(pack_bf16x2(acc.x * inv, acc.y * inv), pack_bf16x2(acc.z * inv, acc.w * inv));
  } else {
    reinterpret_cast<float4*>(static_cast<float*>(out) + row * 128)[lane] =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
}

// ---------------- host side ----------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_attn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// 2D bf16 map over [rows, cols] (row stride in bytes) with 64 x 128 boxes and 128-byte swizzle
static bool bf16_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows, int64_t stride_bytes) {
  auto fn = encode_fn_attn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride_bytes};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool flash_attention_supported(const AttnArgs& a) {
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  return a.dtype == WE_BF16 && a.dim == 128 && !a.causal && a.tokens >= 1 && al(a.q) && al(a.k) && al(a.v) &&
         al(a.out) && a.heads % a.kv_heads == 0 && a.tokens <= 0x7fffffffLL;
}

int flash_attention_splits(const AttnArgs& a, int sms) {
  const int64_t blocks = (a.tokens + fa2::QT * fa2::BQ - 1) / (fa2::QT * fa2::BQ);
  const int64_t nt = (a.tokens + fa2::BK - 1) / fa2::BK;
  const int64_t ctas = blocks * a.heads;
  // A CTA (one per SM) costs about 15 key tiles of fixed work plus its key tiles (measured at 4608 tokens: 25 us +
  // 1.7 us a tile), so splitting the keys pays only when it adds CTAs without adding a wave: pick the split count
  // with the least waves x (15 + tiles per split), the combine costing about 3 tiles.
  int splits = 1;
  int64_t best = -1;
  for (int s = 1; s <= 8 && s <= nt; s++) {
    const int64_t waves = (ctas * s + sms - 1) / sms;
    const int64_t cost = waves * (15 + (nt + s - 1) / s) + (s > 1 ? 3 : 0);
    if (best < 0 || cost < best) {
      best = cost;
      splits = s;
    }
  }
  if (const char* env = getenv("WE_FA_SPLITS")) {  // test / tuning override
    const int v = atoi(env);
    if (v >= 1 && v <= 8 && v <= nt) splits = v;
  }
  return splits;
}

int64_t flash_attention_scratch_bytes(const AttnArgs& a, int splits) {
  return splits > 1 ? (int64_t)splits * a.tokens * a.heads * (fa2::D + 2) * 4 : 0;
}

cudaError_t launch_flash_attention(const AttnArgs& a, int splits, void* scratch, uint32_t* err, cudaStream_t st) {
  CUtensorMap mq, mk, mv;
  if (!bf16_map(&mq, a.q, a.heads * a.dim, a.tokens, a.heads * a.dim * 2) ||
      !bf16_map(&mk, a.k, a.kv_heads * a.dim, a.tokens, a.kv_heads * a.dim * 2) ||
      !bf16_map(&mv, a.v, a.kv_heads * a.dim, a.tokens, a.kv_heads * a.dim * 2))
    return cudaErrorNotSupported;
  fa::Params p;
  p.tokens = a.tokens;
  p.heads = a.heads;
  p.kv_heads = a.kv_heads;
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)a.dim);
  p.out = a.out;
  p.out_dtype = a.out_dtype;
  p.err = err;
  p.part_o = splits > 1 ? static_cast<float*>(scratch) : nullptr;
  p.part_ml = splits > 1 ? static_cast<float*>(scratch) + (int64_t)splits * a.tokens * a.heads * fa2::D : nullptr;
  const unsigned blocks = (unsigned)((a.tokens + fa2::QT * fa2::BQ - 1) / (fa2::QT * fa2::BQ));
  cudaError_t e = cudaFuncSetAttribute(flash_attn2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, fa2::ALLOC);
  if (e != cudaSuccess) return e;
  dim3 grid(blocks, (unsigned)a.heads, (unsigned)splits);
  e = launch_pdl(flash_attn2_kernel, grid, fa2::THREADS, fa2::ALLOC, st, mq, mk, mv, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess || splits == 1) return e;
  const int64_t rows = a.tokens * a.heads;
  const unsigned cb = (unsigned)((rows + 7) / 8);
  e = a.out_dtype == WE_BF16
          ? launch_pdl(flash_combine_kernel<WE_BF16>, dim3(cb), 256, 0, st, p.part_o, p.part_ml, splits, rows, a.out)
          : launch_pdl(flash_combine_kernel<WE_F32>, dim3(cb), 256, 0, st, p.part_o, p.part_ml, splits, rows, a.out);
  return e == cudaSuccess ? cudaGetLastError() : e;
}

cudaError_t launch_attention_simt(const AttnArgs& a, int sms, cudaStream_t st) {
  const int64_t rows = a.tokens * a.heads;
  int64_t g = (rows + 3) / 4;
  if (g > (int64_t)sms * 16) g = (int64_t)sms * 16;
  const float scale = 1.f / sqrtf((float)a.dim);
  const int vpl = (int)((a.dim + 31) / 32);
#define ATT_CASE(V)                                                                                                 \
  if (vpl <= V) {                                                                                                   \
    if (a.dtype == WE_BF16 && a.out_dtype == WE_BF16)                                                               \
      attention_simt_kernel<WE_BF16, WE_BF16, V><<<(unsigned)g, 128, 0, st>>>(a.q, a.k, a.v, a.tokens, a.heads,     \
                                                                             a.kv_heads, a.dim, a.causal, scale, a.out); \
    else if (a.dtype == WE_BF16)                                                                                    \
      attention_simt_kernel<WE_BF16, WE_F32, V><<<(unsigned)g, 128, 0, st>>>(a.q, a.k, a.v, a.tokens, a.heads,      \
                                                                            a.kv_heads, a.dim, a.causal, scale, a.out); \
    else if (a.out_dtype == WE_BF16)                                                                                \
      attention_simt_kernel<WE_F32, WE_BF16, V><<<(unsigned)g, 128, 0, st>>>(a.q, a.k, a.v, a.tokens, a.heads,      \
                                                                            a.kv_heads, a.dim, a.causal, scale, a.out); \
    else                                                                                                            \
      attention_simt_kernel<WE_F32, WE_F32, V><<<(unsigned)g, 128, 0, st>>>(a.q, a.k, a.v, a.tokens, a.heads,       \
                                                                           a.kv_heads, a.dim, a.causal, scale, a.out); \
    return cudaGetLastError();                                                                                      \
  }
  ATT_CASE(1)
  ATT_CASE(2)
  ATT_CASE(4)
  ATT_CASE(8)
#undef ATT_CASE
  return cudaErrorInvalidValue;
}

}  // namespace we
