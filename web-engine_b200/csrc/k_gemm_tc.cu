// tcgen05 GEMM for the weight-quantized linear layers (sm_100a).
//
// Computes y[m, n] = (sum_t X_t[m, :] . W[n, :]) * row_scale[m] * (chan_scale[n] | scale) (+ bias) (+ y),
// the tensor-core form of matmulWgsl (src/kernels/matmul.ts:118-178) for bf16 activations:
//   * fp8 weights: kind::f8f6f4 with e4m3 W and e4m3 activation terms. The activation split
//     (k_quant.cu quant_act_kernel) writes X = 2^e (hi + lo) per row with hi, lo e4m3: for bf16 x the
//     two terms are exact, so the product equals the bf16 x fp8 dequant GEMM up to fp32 accumulation.
//     One term (hi only) is the fp8-peak mode.
//   * bf16 weights (and int4 weights decoded to bf16): kind::f16 with bf16 X, one term.
//
// Tile: 128 weight rows (UMMA M, TMEM lanes = output channels) x BT tokens (UMMA N, TMEM columns),
// K in 128-byte stages (one SWIZZLE_128B row: 128 e4m3 or 64 bf16). Warp-specialised, persistent:
//   warp 0     one thread issues TMA loads (no multicast) into a STAGES-deep shared-memory ring,
//   warp 1     allocates TMEM and one thread issues tcgen05.mma, committing to the ring's empty
//              barriers and, per tile, to a double-buffered TMEM accumulator's full barrier,
//   warps 2-5  epilogue: tcgen05.ld 32 lanes x 32 columns, scale, bias, store (consecutive lanes =
//              consecutive output channels, so each store instruction is coalesced).
// Every mbarrier wait is bounded (2 s of %globaltimer); on timeout the kernel records a code in the
// device error word, the other roles stop at their next wait, in-flight TMA loads and MMAs are
// drained with bounded waits, TMEM is freed and the kernel returns.
#include <cudaTypedefs.h>
#include <stdlib.h>

#include "common.cuh"
#include "kernels.h"
#include "tc_ptx.cuh"

namespace we {
namespace tc {

constexpr int BM = 128;           // weight rows per tile (UMMA M)
constexpr int KB_BYTES = 128;     // K bytes per stage
constexpr int THREADS = 192;
constexpr int EPI_LD = 36;  // floats per row of an epilogue warp's 32 x 32 staging tile (pad: no bank conflicts)
constexpr int EPI_BYTES = 4 * 32 * EPI_LD * 4;
constexpr int SMEM_BUDGET = 207 * 1024;  // for the stage ring; + epilogue staging + barriers <= 227 KB

struct Params {
  int64_t m, n;
  int num_kb;
  const float* row_scale;
  const float* chan_scale;
  float scale;
  const float* bias;
  void* y;
  int64_t y_stride;
  int y_dtype;
  int accumulate;
  int vec_ok;  // y rows allow 16-byte stores (aligned base, stride a multiple of 16 bytes)
  EpiOps epi;
  int epi_vec_ok;  // aux rows and the gate vector allow 16-byte loads
  uint32_t* err;
  void* ys[3];         // split output (ys[0] set): channels [seg_end[i-1], seg_end[i]) go to ys[i], rows as wide
  int64_t seg_end[3];  // as the part apart
  // second weight set: token rows in segments marked 1 use W2 (a second tensor map) with these scales, bias and
  // gate; segments [row_end[i-1], row_end[i]) with row_end multiples of the token tile
  const float* chan_scale2;
  float scale2;
  const float* bias2;
  const float* gate2;
  int nseg;
  int32_t row_end[WE_GEMM_MAX_SEGMENTS];
  uint8_t row_set[WE_GEMM_MAX_SEGMENTS];
  // int4 group-64 weights (gemm_tc_i4_kernel): packed [n, k / 2], f16 group scales [n, k / 64]
  const uint8_t* w4;
  const uint16_t* w4_scale;
  int64_t k;
  // peer output (peer_part >= 0): that part's heads go to the ranks that attend them (TcGemmArgs::peer)
  int peer_part;
  int64_t peer_row0, peer_hl;
  void* peer_dst[WE_PEER_MAX];
};

// The token tile of the i-th tile in schedule order. With two weight sets the tiles of set 0 come first, then those
// of set 1, so the CTAs sweep one set's weights at a time and keep them in L2 (alternating text and image rows of
// a batch would otherwise switch weights every few tiles). Inner segment ends are multiples of bt.
__device__ __forceinline__ int64_t tile_m(const Params& p, int64_t i, int bt) {
  if (p.nseg <= 0) return i;
  for (int set = 0; set < 2; set++) {
    int64_t start = 0;
    for (int k = 0; k < p.nseg; k++) {
      const int64_t n = (p.row_end[k] - start + bt - 1) / bt;
      if (p.row_set[k] == set) {
        if (i < n) return start / bt + i;
        i -= n;
      }
      start = p.row_end[k];
    }
  }
  return 0;  // not reached: i < the number of token tiles
}

// The weight set of the token tile starting at tok_base (0 without segments).
__device__ __forceinline__ int row_set(const Params& p, int64_t tok_base) {
  for (int i = 0; i < p.nseg; i++)
    if (tok_base < p.row_end[i]) return p.row_set[i];
  return 0;
}
// The epilogue's per-channel operands of one weight set.
struct SetOps {
  const float* chan_scale;
  float scale;
  const float* bias;
  const float* gate;
};
__device__ __forceinline__ SetOps set_ops(const Params& p, int set) {
  return set ? SetOps{p.chan_scale2, p.scale2, p.bias2, p.gate2} : SetOps{p.chan_scale, p.scale, p.bias, p.epi.gate};
}

// Where a tile's outputs go: the buffer, its first channel and its row stride (values).
struct YOut {
  void* y;
  int64_t cofs, stride;
};
// The peer part (peer_part) goes head by head (128 channels, one or more epilogue warps' channels) to rank
// o = h / hl's memory, rows [peer_row0, ...) of its [tokens of every rank, hl heads, 128] block.
__device__ __forceinline__ YOut y_out(const Params& p, int64_t ch_base) {
  const int s = p.ys[0] ? (ch_base >= p.seg_end[0]) + (ch_base >= p.seg_end[1]) : 0;
  const int64_t lo = s ? p.seg_end[s - 1] : 0;
  if (s == p.peer_part) {
    const int64_t h = (ch_base - lo) >> 7, o = h / p.peer_hl;
    return YOut{static_cast<uint16_t*>(p.peer_dst[o]) + (p.peer_row0 * p.peer_hl + h - o * p.peer_hl) * 128,
                lo + h * 128, p.peer_hl * 128};
  }
  if (!p.ys[0]) return YOut{p.y, 0, p.y_stride};
  return YOut{p.ys[s], lo, p.seg_end[s] - lo};
}

// TMEM columns for two accumulators of BT columns: tcgen05.alloc takes a power of two of at least 32
__host__ __device__ constexpr uint32_t tmem_cols(int bt) {
  uint32_t c = 32;
  while (c < 2u * (uint32_t)bt) c *= 2;
  return c;
}

template <int BT, int TERMS>
struct Layout {
  static constexpr int W_BYTES = BM * KB_BYTES;
  static constexpr int X_BYTES = BT * KB_BYTES;
  static constexpr int STAGE_BYTES = W_BYTES + TERMS * X_BYTES;
  static constexpr int STAGES = (SMEM_BUDGET / STAGE_BYTES) > 8 ? 8 : (SMEM_BUDGET / STAGE_BYTES);
  static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = EPI_OFFSET + EPI_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 5;  // full[S], empty[S], tfull[2], tempty[2], drain
  static constexpr int TOTAL = BAR_OFFSET + NUM_BARS * 8 + 16;
  static constexpr int ALLOC = TOTAL + 1024;      // slack to align the base to 1024 bytes
  static_assert(STAGES >= 2, "shared-memory ring needs at least 2 stages");
};

template <int BT, bool F16>
__host__ __device__ constexpr uint32_t make_idesc() {
  return (1u << 4) | ((F16 ? 1u : 0u) << 7) | ((F16 ? 1u : 0u) << 10) | ((uint32_t)(BT >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

// Epilogue of one 32-token chunk of a warp's 32 channels, in two layouts:
// - as read from TMEM (lane = channel, 32 tokens per thread): row scale (one coalesced load, broadcast by
//   shuffle), channel scale, bias and the activation, 32 independent values per thread;
// - after a transpose through shared memory (row stride EPI_LD, conflict-free): 8 consecutive channels of one
//   token per lane, where the aux operand, the channel gate and the accumulate read-modify-write run on
//   16-byte words, then one 16-byte bf16 store (or two f32); scalar accesses on ragged edges.
// The old y (accumulate) and the aux rows do not depend on the accumulator: EpiFetch holds them as raw
// 16-byte words, loaded one chunk ahead (each slot is refilled for the next chunk as soon as it is used), so
// their HBM latency hides behind the work of the chunk before.
struct EpiFetch {
  uint4 y[4][2];
  uint4 a[4][2];
};

// whether iteration `it` of the chunk at tok0 takes the 16-byte path (and so was fetched ahead)
__device__ __forceinline__ bool epi_fast(const Params& p, int64_t tok, int64_t c0) {
  return tok < p.m && c0 + 8 <= p.n && p.vec_ok && (!p.epi.aux_op || p.epi_vec_ok);
}

__device__ __forceinline__ void epi_fetch_iter(EpiFetch& f, int it, int lane, int64_t tok0, int64_t c0,
                                               const YOut& yo, const Params& p) {
  const int64_t tok = tok0 + it * 8 + (lane >> 2);
  if (!epi_fast(p, tok, c0)) return;
  const int64_t o = tok * yo.stride + c0 - yo.cofs;
  if (p.accumulate) {
    if (p.y_dtype == WE_BF16) {
      f.y[it][0] = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(yo.y) + o);
    } else {
      const uint4* q = reinterpret_cast<const uint4*>(static_cast<const float*>(yo.y) + o);
      f.y[it][0] = q[0];
      f.y[it][1] = q[1];
    }
  }
  if (p.epi.aux_op) {
    if (p.epi.aux_dtype == WE_BF16) {
      f.a[it][0] = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.epi.aux) + o));
    } else {
      const uint4* q = reinterpret_cast<const uint4*>(static_cast<const float*>(p.epi.aux) + o);
      f.a[it][0] = __ldg(q);
      f.a[it][1] = __ldg(q + 1);
    }
  }
}

__device__ __forceinline__ void unpack8(const uint4 (&w)[2], bool bf16, float (&v)[8]) {
  if (bf16) {
    const uint32_t u[4] = {w[0].x, w[0].y, w[0].z, w[0].w};
#pragma unroll
    for (int e = 0; e < 4; e++) {
      v[2 * e] = __uint_as_float(u[e] << 16);
      v[2 * e + 1] = __uint_as_float(u[e] & 0xffff0000u);
    }
  } else {
    v[0] = __uint_as_float(w[0].x); v[1] = __uint_as_float(w[0].y);
    v[2] = __uint_as_float(w[0].z); v[3] = __uint_as_float(w[0].w);
    v[4] = __uint_as_float(w[1].x); v[5] = __uint_as_float(w[1].y);
    v[6] = __uint_as_float(w[1].z); v[7] = __uint_as_float(w[1].w);
  }
}

// the per-tile channel gate of this lane's 8 post-transpose channels (zeros past n)
__device__ __forceinline__ void epi_gate(float (&gt)[8], int lane, int64_t ch_base, const float* gate,
                                         const Params& p) {
  const int64_t c0 = ch_base + (lane & 3) * 8;
  if (!gate) return;
  if (p.epi_vec_ok && c0 + 8 <= p.n) {
    load8f(gate, c0, gt);
  } else {
#pragma unroll
    for (int e = 0; e < 8; e++) gt[e] = (c0 + e < p.n) ? gate[c0 + e] : 0.f;
  }
}

// `more`: the warp goes on to the chunk at tok0 + 32, whose operands are fetched into f as slots free up
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], EpiFetch& f, const float (&gt)[8],
                                               bool more, float* stage, int lane, int64_t tok0, int64_t ch_base,
                                               float cs, float bias, const YOut& yo, const Params& p) {
  const int cg = (lane & 3) * 8;
  const float rs_lane = p.row_scale ? ((tok0 + lane < p.m) ? p.row_scale[tok0 + lane] : 0.f) : 1.f;
  const float2 cs2 = make_float2(cs, cs), b2 = make_float2(bias, bias);
  const int act = p.epi.act;
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    float2 v = __ffma2_rn(__fmul2_rn(make_float2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])),
                                     make_float2(__shfl_sync(0xffffffffu, rs_lane, j),
                                                 __shfl_sync(0xffffffffu, rs_lane, j + 1))),
                          cs2, b2);
    if (act == WE_ACT_GELU_TANH) v = gelu_tanh2(v);
    else if (act == WE_ACT_SILU) v = silu2(v);
    stage[j * EPI_LD + lane] = v.x;
    stage[(j + 1) * EPI_LD + lane] = v.y;
  }
  __syncwarp();
  const int64_t c0 = ch_base + cg;
  const bool ybf = p.y_dtype == WE_BF16, abf = p.epi.aux_dtype == WE_BF16;
#pragma unroll
  for (int it = 0; it < 4; it++) {
    const int tr = it * 8 + (lane >> 2);
    const int64_t tok = tok0 + tr;
    const float4 a = *reinterpret_cast<const float4*>(stage + tr * EPI_LD + cg);
    const float4 b = *reinterpret_cast<const float4*>(stage + tr * EPI_LD + cg + 4);
    float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    if (epi_fast(p, tok, c0)) {
      const int64_t o = tok * yo.stride + c0 - yo.cofs;
      if (p.epi.aux_op) {
        float ax[8];
        unpack8(f.a[it], abf, ax);
        if (p.epi.aux_op == WE_AUX_SIGMOID_GATE) {
#pragma unroll
          for (int e = 0; e < 8; e++) v[e] = ax[e] * sigmoid_fast(v[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; e++) v[e] = ax[e] * sigmoid_fast(ax[e]) * v[e];
        }
      }
      if (p.epi.gate) {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] *= gt[e];
      }
      if (p.accumulate) {
        float yo[8];
        unpack8(f.y[it], ybf, yo);
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] += yo[e];
      }
      if (ybf) {
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(yo.y) + o) =
            make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                       pack_bf16x2(v[6], v[7]));
      } else {
        float4* y = reinterpret_cast<float4*>(static_cast<float*>(yo.y) + o);
        y[0] = make_float4(v[0], v[1], v[2], v[3]);
        y[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
    } else if (tok < p.m && c0 < p.n) {
      // ragged or unaligned: per value, loads at use
#pragma unroll
      for (int e = 0; e < 8; e++) {
        if (c0 + e >= p.n) break;
        const int64_t o = tok * yo.stride + c0 + e - yo.cofs;
        float val = v[e];
        if (p.epi.aux_op) {
          const float ax = abf ? load_act<WE_BF16>(p.epi.aux, o) : load_act<WE_F32>(p.epi.aux, o);
          val = aux_apply(p.epi.aux_op, ax, val);
        }
        if (p.epi.gate) val *= gt[e];
        if (ybf) {
          uint16_t* y = static_cast<uint16_t*>(yo.y);
          y[o] = f32_to_bf16_bits(val + (p.accumulate ? bf16_bits_to_f32(y[o]) : 0.f));
        } else {
          float* y = static_cast<float*>(yo.y);
          y[o] = val + (p.accumulate ? y[o] : 0.f);
        }
      }
    }
    if (more && (p.accumulate || p.epi.aux_op)) epi_fetch_iter(f, it, lane, tok0 + 32, c0, yo, p);
  }
}

// Operands of a tile's first chunk, issued before the wait for its accumulator
__device__ __forceinline__ void epi_fetch_first(EpiFetch& f, int lane, int64_t tok0, int64_t ch_base,
                                                const YOut& yo, const Params& p) {
  if (!(p.accumulate || p.epi.aux_op)) return;
  const int64_t c0 = ch_base + (lane & 3) * 8;
#pragma unroll
  for (int it = 0; it < 4; it++) epi_fetch_iter(f, it, lane, tok0, c0, yo, p);
}

// ---------------- the kernel ----------------
template <int BT, int TERMS, bool F16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x0,
                   const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_w2,
                   const Params p) {
  using L = Layout<BT, TERMS>;
  constexpr int STAGES = L::STAGES;
  constexpr int KB_ELEMS = F16 ? KB_BYTES / 2 : KB_BYTES;
  constexpr uint32_t TMEM_COLS = tmem_cols(BT);
  constexpr uint32_t IDESC = make_idesc<BT, F16>();
  constexpr int MMAS_PER_KB = KB_BYTES / 32;  // 32 bytes of K per tcgen05.mma

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  pdl_launch_dependents();  // a kernel launched by launch_pdl after this one may place its CTAs as these finish
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::BAR_OFFSET;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::BAR_OFFSET + L::NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
#define FULL(s) (bars + 8u * (s))
#define EMPTY(s) (bars + 8u * (STAGES + (s)))
#define TFULL(b) (bars + 8u * (2 * STAGES + (b)))
#define TEMPTY(b) (bars + 8u * (2 * STAGES + 2 + (b)))
#define DRAIN (bars + 8u * (2 * STAGES + 4))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(FULL(s), 1);
      mbar_init(EMPTY(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(TFULL(b), 1);
      mbar_init(TEMPTY(b), 4);
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
  pdl_wait();  // launched by launch_pdl: the previous kernel's outputs are complete before any global access

  const int64_t tiles_n = (p.n + BM - 1) / BM;
  const int64_t tiles_m = (p.m + BT - 1) / BT;
  const int64_t tiles = tiles_n * tiles_m;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x0)) : "memory");
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[STAGES];
      int issued = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int32_t row_w = (int32_t)((t % tiles_n) * BM), row_x = (int32_t)(tile_m(p, t / tiles_n, BT) * BT);
        const CUtensorMap* mw = row_set(p, row_x) ? &tm_w2 : &tm_w;
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!wait_fast(EMPTY(s), ph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER, WAIT_LIMIT_NS, true)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + (uint32_t)(s * L::STAGE_BYTES);
          mbar_expect_tx(FULL(s), L::STAGE_BYTES);
          const int32_t kc = kb * KB_ELEMS;
          tma_load_2d(st, mw, FULL(s), kc, row_w);
          tma_load_2d(st + L::W_BYTES, &tm_x0, FULL(s), kc, row_x);
          if (TERMS > 1) tma_load_2d(st + L::W_BYTES + L::X_BYTES, &tm_x1, FULL(s), kc, row_x);
          issued_ph[s] = ph;
          issued++;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {  // let the loads already issued land before the CTA can exit
        for (int i = 0; i < STAGES && i < issued; i++)
          wait_fast(FULL(i), issued_ph[i], abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, aph = 0;
      int ab = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!wait_fast(TEMPTY(ab), aph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BT);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!wait_fast(FULL(s), ph, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + (uint32_t)(s * L::STAGE_BYTES);
          const uint64_t adesc = sw128_desc(st);
#pragma unroll
          for (int term = 0; term < TERMS; term++) {
            const uint64_t bdesc = sw128_desc(st + L::W_BYTES + term * L::X_BYTES);
#pragma unroll
            for (int kk = 0; kk < MMAS_PER_KB; kk++)
              umma<F16>(d, adesc + 2u * kk, bdesc + 2u * kk, IDESC, (kb | term | kk) != 0);
          }
          umma_commit(EMPTY(s));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(TFULL(ab));
        if (++ab == 2) {
          ab = 0;
          aph ^= 1u;
        }
      }
      // all MMAs issued by this thread complete before TMEM can be freed
      umma_commit(DRAIN);
      wait_fast(DRAIN, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    float* stage = reinterpret_cast<float*>(smem + L::EPI_OFFSET) + (warp - 2) * (32 * EPI_LD);
    int ab = 0;
    uint32_t aph = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      // everything that does not need the accumulator is loaded before waiting for it
      const int64_t ch_base = (t % tiles_n) * BM + q * 32;  // first output channel of this warp
      const int64_t ch = ch_base + lane;
      const int64_t tok_base = tile_m(p, t / tiles_n, BT) * BT;
      const bool ch_ok = ch < p.n;
      const SetOps so = set_ops(p, row_set(p, tok_base));
      const float cs = ch_ok ? (so.chan_scale ? so.chan_scale[ch] : so.scale) : 0.f;
      const float bias = (ch_ok && so.bias) ? so.bias[ch] : 0.f;
      EpiFetch f;
      float gt[8];
      const YOut yo = y_out(p, ch_base);
      epi_fetch_first(f, lane, tok_base, ch_base, yo, p);
      epi_gate(gt, lane, ch_base, so.gate, p);
      bool ok = wait_fast(TFULL(ab), aph, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE, WAIT_LIMIT_NS, true);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BT / 32; c++) {
        const int64_t tok0 = tok_base + c * 32;
        if (tok0 >= p.m) break;  // warp-uniform: the rest of the tile is padding
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BT + c * 32), r);
        const bool last = c == BT / 32 - 1 || tok0 + 32 >= p.m;
        if (last) {
          // last TMEM read of this tile: hand the accumulator back to the MMA warp before the stores
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(TEMPTY(ab));
        }
        epilogue_chunk(r, f, gt, !last, stage, lane, tok0, ch_base, cs, bias, yo, p);
        __syncwarp();
      }
      if (++ab == 2) {
        ab = 0;
        aph ^= 1u;
      }
    }
  }
  // peer output: this thread's stores to other GPUs are visible system-wide before the kernel ends
  if (p.peer_part >= 0) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
#undef DRAIN
}


// ---------------- the 2-SM kernel (cta_group::2) ----------------
// A CTA pair (cluster of 2, ranks 0 = leader and 1) computes 256 weight rows x BT tokens: each CTA
// TMA-loads its own 128 weight rows and its own BT/2 token rows (plain loads, no multicast; the bytes
// complete on the leader's barrier), the leader's MMA thread issues tcgen05.mma.cta_group::2 (M = 256,
// N = BT) and its commits arrive on both CTAs' barriers (tcgen05.commit multicast), and each CTA's
// epilogue drains its own 128-lane accumulator, releasing it on the leader's barrier (remote arrive).
// Per SM this halves the token bytes per FLOP of the 1-SM kernel, so the same shared memory holds
// twice the stages.
// ATOMS: 128-byte K atoms per stage and operand. bf16 (kind::f16) takes 2, so a stage holds 8 MMAs like a
// two-term e4m3 stage and the ring needs half the barrier round trips per FLOP.
template <int BT, int TERMS, int ATOMS = 1>
struct Layout2 {
  static constexpr int W_ATOM = BM * KB_BYTES;
  static constexpr int X_ATOM = (BT / 2) * KB_BYTES;
  static constexpr int W_BYTES = ATOMS * W_ATOM;
  static constexpr int X_BYTES = ATOMS * X_ATOM;
  static constexpr int STAGE_BYTES = W_BYTES + TERMS * X_BYTES;
  static constexpr int STAGES = (SMEM_BUDGET / STAGE_BYTES) > 8 ? 8 : (SMEM_BUDGET / STAGE_BYTES);
  static constexpr int EPI_OFFSET = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFFSET = EPI_OFFSET + EPI_BYTES;
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  static constexpr int TOTAL = BAR_OFFSET + NUM_BARS * 8 + 16;
  static constexpr int ALLOC = TOTAL + 1024;
  static_assert(STAGES >= 2, "shared-memory ring needs at least 2 stages");
};

template <int BT, bool F16>
__host__ __device__ constexpr uint32_t make_idesc_pair() {
  return (1u << 4) | ((F16 ? 1u : 0u) << 7) | ((F16 ? 1u : 0u) << 10) | ((uint32_t)(BT >> 3) << 17) |
         ((uint32_t)((2 * BM) >> 4) << 24);
}

template <int BT, int TERMS, bool F16>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x0,
                    const __grid_constant__ CUtensorMap tm_x1, const __grid_constant__ CUtensorMap tm_w2,
                    const Params p) {
  constexpr int ATOMS = F16 ? 2 : 1;
  using L = Layout2<BT, TERMS, ATOMS>;
  constexpr int STAGES = L::STAGES;
  constexpr int KB_ELEMS = F16 ? KB_BYTES / 2 : KB_BYTES;  // K elements per atom
  constexpr uint32_t TMEM_COLS = tmem_cols(BT);
  constexpr uint32_t IDESC = make_idesc_pair<BT, F16>();
  constexpr int MMAS_PER_KB = KB_BYTES / 32;
  const int num_stages = (p.num_kb + ATOMS - 1) / ATOMS;  // a K atom past the end loads as zeros

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  pdl_launch_dependents();  // a kernel launched by launch_pdl after this one may place its CTAs as these finish
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::BAR_OFFSET;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::BAR_OFFSET + L::NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
#define FULL(s) (bars + 8u * (s))
#define EMPTY(s) (bars + 8u * (STAGES + (s)))
#define TFULL(b) (bars + 8u * (2 * STAGES + (b)))
#define TEMPTY(b) (bars + 8u * (2 * STAGES + 2 + (b)))
#define DRAIN (bars + 8u * (2 * STAGES + 4))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(FULL(s), 1);   // leader: one arrive.expect_tx of the pair's bytes per use
      mbar_init(EMPTY(s), 1);  // both: the leader's multicast commit
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(TFULL(b), 1);   // both: the leader's multicast commit
      mbar_init(TEMPTY(b), 8);  // leader: 4 epilogue warps of each CTA
    }
    mbar_init(DRAIN, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) tmem_alloc_pair(smem_u32(tmem_holder), TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  pdl_wait();  // launched by launch_pdl: the previous kernel's outputs are complete before any global access

  const int64_t tiles_n = (p.n + 2 * BM - 1) / (2 * BM);  // pair tiles of 256 weight rows
  const int64_t tiles_m = (p.m + BT - 1) / BT;
  const int64_t tiles = tiles_n * tiles_m;
  const int64_t cid = cluster_id(), ncl = cluster_count();

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_w)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x0)) : "memory");
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[STAGES];
      int issued = 0;
      bool ok = true;
      for (int64_t t = cid; t < tiles && ok; t += ncl) {
        const int32_t row_w = (int32_t)((t % tiles_n) * 2 * BM + rank * BM);
        const int64_t tok_tile = tile_m(p, t / tiles_n, BT) * BT;
        const int32_t row_x = (int32_t)(tok_tile + rank * (BT / 2));
        const CUtensorMap* mw = row_set(p, tok_tile) ? &tm_w2 : &tm_w;
        for (int kb = 0; kb < num_stages; kb++) {
          if (!wait_fast(EMPTY(s), ph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER, WAIT_LIMIT_NS, true)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + (uint32_t)(s * L::STAGE_BYTES);
          if (leader) mbar_expect_tx(FULL(s), 2 * L::STAGE_BYTES);
          const uint32_t bar = map_rank(FULL(s), 0);
#pragma unroll
          for (int a = 0; a < ATOMS; a++) {
            const int32_t kc = (kb * ATOMS + a) * KB_ELEMS;
            tma_load_2d_pair(st + a * L::W_ATOM, mw, bar, kc, row_w);
            tma_load_2d_pair(st + L::W_BYTES + a * L::X_ATOM, &tm_x0, bar, kc, row_x);
            if (TERMS > 1) tma_load_2d_pair(st + L::W_BYTES + L::X_BYTES + a * L::X_ATOM, &tm_x1, bar, kc, row_x);
          }
          issued_ph[s] = ph;
          issued++;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok && leader) {  // the pair's loads already issued land before the CTAs can exit
        for (int i = 0; i < STAGES && i < issued; i++)
          wait_fast(FULL(i), issued_ph[i], abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int s = 0;
      uint32_t ph = 0, aph = 0;
      int ab = 0;
      bool ok = true;
      for (int64_t t = cid; t < tiles && ok; t += ncl) {
        if (!wait_fast(TEMPTY(ab), aph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BT);
        for (int kb = 0; kb < num_stages; kb++) {
          if (!wait_fast(FULL(s), ph, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + (uint32_t)(s * L::STAGE_BYTES);
#pragma unroll
          for (int a = 0; a < ATOMS; a++) {
            const uint64_t adesc = sw128_desc(st + a * L::W_ATOM);
#pragma unroll
            for (int term = 0; term < TERMS; term++) {
              const uint64_t bdesc = sw128_desc(st + L::W_BYTES + term * L::X_BYTES + a * L::X_ATOM);
#pragma unroll
              for (int kk = 0; kk < MMAS_PER_KB; kk++)
                umma_pair<F16>(d, adesc + 2u * kk, bdesc + 2u * kk, IDESC, (kb | a | term | kk) != 0);
            }
          }
          umma_commit_pair_both(EMPTY(s));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(TFULL(ab));
        if (++ab == 2) {
          ab = 0;
          aph ^= 1u;
        }
      }
      umma_commit_pair_local(DRAIN);
      wait_fast(DRAIN, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    float* stage = reinterpret_cast<float*>(smem + L::EPI_OFFSET) + (warp - 2) * (32 * EPI_LD);
    int ab = 0;
    uint32_t aph = 0;
    for (int64_t t = cid; t < tiles; t += ncl) {
      const int64_t ch_base = (t % tiles_n) * 2 * BM + rank * BM + q * 32;
      const int64_t ch = ch_base + lane;
      const int64_t tok_base = tile_m(p, t / tiles_n, BT) * BT;
      const bool ch_ok = ch < p.n;
      const SetOps so = set_ops(p, row_set(p, tok_base));
      const float cs = ch_ok ? (so.chan_scale ? so.chan_scale[ch] : so.scale) : 0.f;
      const float bias = (ch_ok && so.bias) ? so.bias[ch] : 0.f;
      EpiFetch f;
      float gt[8];
      const YOut yo = y_out(p, ch_base);
      epi_fetch_first(f, lane, tok_base, ch_base, yo, p);
      epi_gate(gt, lane, ch_base, so.gate, p);
      bool ok = wait_fast(TFULL(ab), aph, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE, WAIT_LIMIT_NS, true);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BT / 32; c++) {
        const int64_t tok0 = tok_base + c * 32;
        if (tok0 >= p.m) break;
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BT + c * 32), r);
        const bool last = c == BT / 32 - 1 || tok0 + 32 >= p.m;
        if (last) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(map_rank(TEMPTY(ab), 0));
        }
        epilogue_chunk(r, f, gt, !last, stage, lane, tok0, ch_base, cs, bias, yo, p);
        __syncwarp();
      }
      if (++ab == 2) {
        ab = 0;
        aph ^= 1u;
      }
    }
  }
  // peer output: this thread's stores to other GPUs are visible system-wide before the kernel ends
  if (p.peer_part >= 0) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA frees TMEM or exits while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, TMEM_COLS);
  }
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
#undef DRAIN
}

// 8 int4 values (one u32: value 2i in bits 8i..8i+3, value 2i+1 in bits 8i+4..8i+7) times the group scale s,
// rounded to bf16: the same bf16_rne(q * s) as int4_operand, on bf16x2 FMA-pipe math (a float -> bf16 convert per
// pair would saturate the conversion pipe). A byte permute and a mask build v = 128 + (nib ^ 8) as bf16 (exact),
// q = v - 136 = (nib ^ 8) - 8 exactly; with s = s_hi + s_lo split exactly into two bf16 values (s_lo has at most
// 3 significant bits), q * s_lo is exact and fma(q, s_hi, q * s_lo) rounds q * s once, to nearest even.
struct I4Scale {
  __nv_bfloat162 hi, lo;
};
__device__ __forceinline__ I4Scale i4_scale(float s) {
  const __nv_bfloat162 hi = __float2bfloat162_rn(s);
  return I4Scale{hi, __float2bfloat162_rn(s - __low2float(hi))};  // the remainder is exact in bf16
}
__device__ __forceinline__ uint4 int4x8_to_bf16x8(uint32_t w, const I4Scale& sc) {
  const uint32_t w4 = w >> 4;
  const __nv_bfloat162 m136 = __floats2bfloat162_rn(-136.f, -136.f);
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    // low half: byte j of w (value 2j in its low nibble), high half: byte j of w >> 4 (value 2j + 1); keeping the
    // low nibbles and flipping bit 3 under the 0x43 high byte gives bf16 128 + (nib ^ 8) in each half
    const uint32_t v = (__byte_perm(w, w4, (uint32_t)(j | (4 + j) << 8)) & 0x000F000Fu) ^ 0x43084308u;
    const __nv_bfloat162 q = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(&v), m136);
    const __nv_bfloat162 r = __hfma2(q, sc.hi, __hmul2(q, sc.lo));
    o[j] = *reinterpret_cast<const uint32_t*>(&r);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// ---------------- the 1-SM kernel with int4 group-64 weights unpacked in the kernel ----------------
// The 1-SM kernel's kind::f16 form (128 weight rows x BT tokens per CTA, one 64-value K atom per stage, which is
// exactly one int4 group), with W written by CW converter warps (warps 6 .. 6 + CW - 1) instead of TMA. All signals
// stay inside the CTA: the converters arrive on the stage's full barrier after fencing their stores into the async
// proxy. (A 2-SM form, where the peer CTA's converters must arrive on the leader's barrier every stage, measured
// slower than decoding W to bf16 first: the cross-SM release arrive cost 1-3 us per stage.) A converter thread takes
// 16 / CW items per stage: weight row (128 / CW) cw + 8 i + (lane & 7), values [16 part, 16 part + 16) with
// part = lane >> 3, i.e. 8 packed bytes (one 8-byte load; a warp reads 32 contiguous bytes of each of 8 rows) and
// two 16-byte stores (a quarter-warp covers 8 rows of one chunk: 8 different bank groups). The packed bytes and
// scales of a stage are loaded I4_AHEAD stages before it is written (a ring of register sets), since an L2 load
// under a running GEMM takes longer than a stage's MMAs.
constexpr int I4_AHEAD = 3;
template <int CW>
struct I4Stage1 {
  static constexpr int ITEMS = 16 / CW;
  uint2 w[ITEMS];
  float s[ITEMS];
};
template <int CW>
__device__ __forceinline__ void i4_load1(I4Stage1<CW>& st, const Params& p, int64_t row0, int kb, int cw, int lane) {
  const int part = lane >> 3;
  const int64_t groups = p.k / 64, row_bytes = p.k / 2;
#pragma unroll
  for (int i = 0; i < I4Stage1<CW>::ITEMS; i++) {
    const int64_t row = row0 + cw * (128 / CW) + i * 8 + (lane & 7);
    if (row < p.n && kb < groups) {
      st.w[i] = __ldg(reinterpret_cast<const uint2*>(p.w4 + row * row_bytes + (int64_t)kb * 32 + part * 8));
      st.s[i] = __half2float(__ushort_as_half(__ldg(p.w4_scale + row * groups + kb)));
    } else {  // past the weight's rows: zeros (the MMA must not see stale bytes)
      st.w[i] = make_uint2(0x88888888u, 0x88888888u);  // q = 0
      st.s[i] = 0.f;
    }
  }
}
template <int CW>
__device__ __forceinline__ void i4_store1(const I4Stage1<CW>& st, uint8_t* wst, int cw, int lane) {
  const int part = lane >> 3;
#pragma unroll
  for (int i = 0; i < I4Stage1<CW>::ITEMS; i++) {
    const int r = cw * (128 / CW) + i * 8 + (lane & 7);
    const I4Scale sc = i4_scale(st.s[i]);
    const uint32_t wd[2] = {st.w[i].x, st.w[i].y};
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int c = part * 2 + j;  // 16-byte chunk of the 128-byte row
      *reinterpret_cast<uint4*>(wst + r * 128 + ((c ^ (r & 7)) << 4)) = int4x8_to_bf16x8(wd[j], sc);
    }
  }
}

template <int BT, int CW>
__global__ void __launch_bounds__(192 + 32 * CW, 1)
    gemm_tc_i4_kernel(const __grid_constant__ CUtensorMap tm_x0, const Params p) {
  using L = Layout<BT, 1>;
  constexpr int STAGES = L::STAGES;
  constexpr int KB_ELEMS = KB_BYTES / 2;
  constexpr uint32_t TMEM_COLS = tmem_cols(BT);
  constexpr uint32_t IDESC = make_idesc<BT, true>();
  constexpr int MMAS_PER_KB = KB_BYTES / 32;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  pdl_launch_dependents();  // a kernel launched by launch_pdl after this one may place its CTAs as these finish
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + L::BAR_OFFSET;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + L::BAR_OFFSET + L::NUM_BARS * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
#define FULL(s) (bars + 8u * (s))
#define EMPTY(s) (bars + 8u * (STAGES + (s)))
#define TFULL(b) (bars + 8u * (2 * STAGES + (b)))
#define TEMPTY(b) (bars + 8u * (2 * STAGES + 2 + (b)))
#define DRAIN (bars + 8u * (2 * STAGES + 4))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(FULL(s), 1 + CW);  // the producer's arrive.expect_tx + the converter warps
      mbar_init(EMPTY(s), 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(TFULL(b), 1);
      mbar_init(TEMPTY(b), 4);
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
  pdl_wait();  // launched by launch_pdl: the previous kernel's outputs are complete before any global access

  const int64_t tiles_n = (p.n + BM - 1) / BM;
  const int64_t tiles_m = (p.m + BT - 1) / BT;
  const int64_t tiles = tiles_n * tiles_m;

  if (warp == 0) {
    if (lane == 0) {  // the token operand by TMA
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tm_x0)) : "memory");
      int s = 0;
      uint32_t ph = 0;
      uint32_t issued_ph[STAGES];
      int issued = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int32_t row_x = (int32_t)((t / tiles_n) * BT);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!wait_fast(EMPTY(s), ph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER, WAIT_LIMIT_NS, true)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + (uint32_t)(s * L::STAGE_BYTES);
          mbar_expect_tx(FULL(s), L::X_BYTES);
          tma_load_2d(st + L::W_BYTES, &tm_x0, FULL(s), kb * KB_ELEMS, row_x);
          issued_ph[s] = ph;
          issued++;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (!ok) {  // the loads already issued land before the CTA can exit
        for (int i = 0; i < STAGES && i < issued; i++)
          wait_fast(FULL(i), issued_ph[i], abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0, aph = 0;
      int ab = 0;
      bool ok = true;
      for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!wait_fast(TEMPTY(ab), aph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * BT);
        for (int kb = 0; kb < p.num_kb; kb++) {
          if (!wait_fast(FULL(s), ph, abort_flag, p.err, DEV_ERR_TIMEOUT_MMA, WAIT_LIMIT_NS, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = sbase + (uint32_t)(s * L::STAGE_BYTES);
          const uint64_t adesc = sw128_desc(st), bdesc = sw128_desc(st + L::W_BYTES);
#pragma unroll
          for (int kk = 0; kk < MMAS_PER_KB; kk++)
            umma<true>(d, adesc + 2u * kk, bdesc + 2u * kk, IDESC, (kb | kk) != 0);
          umma_commit(EMPTY(s));
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(TFULL(ab));
        if (++ab == 2) {
          ab = 0;
          aph ^= 1u;
        }
      }
      umma_commit(DRAIN);
      wait_fast(DRAIN, 0, abort_flag, p.err, DEV_ERR_TIMEOUT_DRAIN, DRAIN_LIMIT_NS, false);
    }
    __syncwarp();
  } else if (warp >= 6) {
    // converters: packed int4 + the stage's group scale -> bf16 W, loads I4_AHEAD stages ahead
    const int cw = warp - 6;
    int s = 0;
    uint32_t ph = 0;
    bool ok = true;
    auto put = [&](const I4Stage1<CW>& cur) -> bool {
      const bool got = wait_fast(EMPTY(s), ph ^ 1u, abort_flag, p.err, DEV_ERR_TIMEOUT_PRODUCER, WAIT_LIMIT_NS, true);
      if (!__all_sync(0xffffffffu, got)) return false;
      i4_store1<CW>(cur, smem + s * L::STAGE_BYTES, cw, lane);
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> the MMA's async reads
      __syncwarp();
      if (lane == 0) mbar_arrive(FULL(s));
      if (++s == STAGES) {
        s = 0;
        ph ^= 1u;
      }
      return true;
    };
    for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const int64_t row0 = (t % tiles_n) * BM;
      I4Stage1<CW> ring[I4_AHEAD + 1];
#pragma unroll
      for (int u = 0; u < I4_AHEAD; u++)
        if (u < p.num_kb) i4_load1<CW>(ring[u], p, row0, u, cw, lane);
      for (int kb = 0; kb < p.num_kb && ok; kb += I4_AHEAD + 1) {
#pragma unroll
        for (int u = 0; u <= I4_AHEAD; u++) {  // static ring slots: stage kb + u is in slot u
          if (!ok || kb + u >= p.num_kb) break;
          if (kb + u + I4_AHEAD < p.num_kb)
            i4_load1<CW>(ring[(u + I4_AHEAD) % (I4_AHEAD + 1)], p, row0, kb + u + I4_AHEAD, cw, lane);
          ok = put(ring[u]);
        }
      }
    }
  } else {
    const int q = warp & 3;
    float* stage = reinterpret_cast<float*>(smem + L::EPI_OFFSET) + (warp - 2) * (32 * EPI_LD);
    int ab = 0;
    uint32_t aph = 0;
    for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int64_t ch_base = (t % tiles_n) * BM + q * 32;
      const int64_t ch = ch_base + lane;
      const int64_t tok_base = (t / tiles_n) * BT;
      const bool ch_ok = ch < p.n;
      const float cs = ch_ok ? (p.chan_scale ? p.chan_scale[ch] : p.scale) : 0.f;
      const float bias = (ch_ok && p.bias) ? p.bias[ch] : 0.f;
      EpiFetch f;
      float gt[8];
      const YOut yo = y_out(p, ch_base);
      epi_fetch_first(f, lane, tok_base, ch_base, yo, p);
      epi_gate(gt, lane, ch_base, p.epi.gate, p);
      bool ok = wait_fast(TFULL(ab), aph, abort_flag, p.err, DEV_ERR_TIMEOUT_EPILOGUE, WAIT_LIMIT_NS, true);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BT / 32; c++) {
        const int64_t tok0 = tok_base + c * 32;
        if (tok0 >= p.m) break;
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * BT + c * 32), r);
        const bool last = c == BT / 32 - 1 || tok0 + 32 >= p.m;
        if (last) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(TEMPTY(ab));
        }
        epilogue_chunk(r, f, gt, !last, stage, lane, tok0, ch_base, cs, bias, yo, p);
        __syncwarp();
      }
      if (++ab == 2) {
        ab = 0;
        aph ^= 1u;
      }
    }
  }
  // peer output: this thread's stores to other GPUs are visible system-wide before the kernel ends
  if (p.peer_part >= 0) __threadfence_system();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
#undef FULL
#undef EMPTY
#undef TFULL
#undef TEMPTY
#undef DRAIN
}

// ---------------- host side ----------------
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// 2D map over [rows, k] with 128-byte-wide boxes of box_rows rows, 128-byte swizzle, zero fill.
static bool make_map(CUtensorMap* m, const void* base, bool f16, int64_t k, int64_t rows, int64_t stride_bytes,
                     int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)stride_bytes};
  cuuint32_t box[2] = {(cuuint32_t)(f16 ? KB_BYTES / 2 : KB_BYTES), (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool F16>
static Params make_params(const TcGemmArgs& a) {
  Params p;
  p.m = a.m;
  p.n = a.n;
  const int64_t kbytes = a.k * (F16 ? 2 : 1);
  p.num_kb = (int)((kbytes + KB_BYTES - 1) / KB_BYTES);
  p.row_scale = a.row_scale;
  p.chan_scale = a.chan_scale;
  p.scale = a.scale;
  p.bias = a.bias;
  p.y = a.y;
  p.y_stride = a.y_stride;
  p.y_dtype = a.y_dtype;
  p.accumulate = a.accumulate;
  const int esz = a.y_dtype == WE_BF16 ? 2 : 4;
  p.vec_ok = ((uintptr_t)a.y % 16 == 0) && ((a.y_stride * esz) % 16 == 0);
  for (int i = 0; i < 3; i++) {
    p.ys[i] = a.ys[i];
    p.seg_end[i] = a.seg_end[i];
    if (a.ys[0] && a.ys[i]) {
      const int64_t w = a.seg_end[i] - (i ? a.seg_end[i - 1] : 0);
      p.vec_ok = p.vec_ok && ((uintptr_t)a.ys[i] % 16 == 0) && ((w * esz) % 16 == 0);
    }
  }
  p.epi = a.epi;
  const int asz = a.epi.aux_dtype == WE_BF16 ? 2 : 4;
  p.epi_vec_ok = (!a.epi.aux || (((uintptr_t)a.epi.aux % 16 == 0) && ((a.y_stride * asz) % 16 == 0))) &&
                 (!a.epi.gate || (uintptr_t)a.epi.gate % 16 == 0) && (!a.gate2 || (uintptr_t)a.gate2 % 16 == 0);
  p.chan_scale2 = a.chan_scale2;
  p.scale2 = a.scale2;
  p.bias2 = a.bias2;
  p.gate2 = a.gate2;
  p.nseg = a.nseg;
  for (int i = 0; i < WE_GEMM_MAX_SEGMENTS; i++) {
    p.row_end[i] = i < a.nseg ? (int32_t)a.row_end[i] : 0;
    p.row_set[i] = i < a.nseg ? (uint8_t)a.row_set[i] : 0;
  }
  p.err = a.dev_err;
  p.peer_part = a.peer ? a.peer_part : -1;
  p.peer_row0 = a.peer_row0;
  p.peer_hl = 1;
  if (a.peer) {
    const int64_t lo = a.ys[0] && a.peer_part ? a.seg_end[a.peer_part - 1] : 0;
    const int64_t hi = a.ys[0] ? a.seg_end[a.peer_part] : a.n;
    p.peer_hl = (hi - lo) / (128 * a.peer_world);
    for (int r = 0; r < WE_PEER_MAX; r++) p.peer_dst[r] = r < a.peer_world ? a.peer_dst[r] : nullptr;
  }
  p.w4 = a.int4 ? static_cast<const uint8_t*>(a.w) : nullptr;
  p.w4_scale = a.int4 ? a.group_scale : nullptr;
  p.k = a.k;
  return p;
}

template <int BT, int TERMS, bool F16>
static cudaError_t run(const TcGemmArgs& a, int sms, cudaStream_t st) {
  using L = Layout<BT, TERMS>;
  CUtensorMap mw, mx0, mx1;
  if (!make_map(&mw, a.w, F16, a.k, a.n, a.w_stride_bytes, BM)) return cudaErrorNotSupported;
  if (!make_map(&mx0, a.x[0], F16, a.k, a.m, a.x_stride_bytes, BT)) return cudaErrorNotSupported;
  if (TERMS > 1) {
    if (!make_map(&mx1, a.x[1], F16, a.k, a.m, a.x_stride_bytes, BT)) return cudaErrorNotSupported;
  } else {
    mx1 = mx0;
  }
  CUtensorMap mw2 = mw;
  if (a.nseg > 0 && !make_map(&mw2, a.w2, F16, a.k, a.n, a.w_stride_bytes, BM)) return cudaErrorNotSupported;
  Params p = make_params<F16>(a);
  auto kern = gemm_tc_kernel<BT, TERMS, F16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((a.n + BM - 1) / BM) * ((a.m + BT - 1) / BT);
  const int grid = (int)(tiles < sms ? tiles : sms);
  e = launch_pdl(kern, dim3(grid), THREADS, L::ALLOC, st, mw, mx0, mx1, mw2, p);
  return e == cudaSuccess ? cudaGetLastError() : e;
}


template <int BT, int TERMS, bool F16>
static cudaError_t run_pair(const TcGemmArgs& a, int sms, cudaStream_t st) {
  using L = Layout2<BT, TERMS, F16 ? 2 : 1>;  // as the kernel lays out its stages
  CUtensorMap mw, mx0, mx1;
  if (!make_map(&mw, a.w, F16, a.k, a.n, a.w_stride_bytes, BM)) return cudaErrorNotSupported;
  if (!make_map(&mx0, a.x[0], F16, a.k, a.m, a.x_stride_bytes, BT / 2)) return cudaErrorNotSupported;
  if (TERMS > 1) {
    if (!make_map(&mx1, a.x[1], F16, a.k, a.m, a.x_stride_bytes, BT / 2)) return cudaErrorNotSupported;
  } else {
    mx1 = mx0;
  }
  CUtensorMap mw2 = mw;
  if (a.nseg > 0 && !make_map(&mw2, a.w2, F16, a.k, a.n, a.w_stride_bytes, BM)) return cudaErrorNotSupported;
  Params p = make_params<F16>(a);
  auto kern = gemm_tc2_kernel<BT, TERMS, F16>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  pdl_attribute(attr[1]);  // the kernel waits (griddepcontrol.wait) before its first global access
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = L::ALLOC;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the occupancy query below sees the cluster shape only
  const int64_t tiles = ((a.n + 2 * BM - 1) / (2 * BM)) * ((a.m + BT - 1) / BT);
  int clusters = sms / 2;
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  int max_clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&max_clusters, kern, &cfg) == cudaSuccess && max_clusters > 0 &&
      max_clusters < clusters)
    clusters = max_clusters;
  if (tiles < clusters) clusters = (int)tiles;
  cfg.gridDim = dim3((unsigned)(2 * clusters), 1, 1);
  cfg.numAttrs = 2;
  e = cudaLaunchKernelEx(&cfg, kern, mw, mx0, mx1, mw2, p);
  return e == cudaSuccess ? cudaGetLastError() : e;
}
// int4 group-64 weights: the W operand is made by the kernel's converter warps, so only the tokens have a tensor map
template <int BT, int CW>
static cudaError_t run_i4(const TcGemmArgs& a, int sms, cudaStream_t st) {
  using L = Layout<BT, 1>;
  CUtensorMap mx0;
  if (!make_map(&mx0, a.x[0], true, a.k, a.m, a.x_stride_bytes, BT)) return cudaErrorNotSupported;
  Params p = make_params<true>(a);
  auto kern = gemm_tc_i4_kernel<BT, CW>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::ALLOC);
  if (e != cudaSuccess) return e;
  const int64_t tiles = ((a.n + BM - 1) / BM) * ((a.m + BT - 1) / BT);
  const int grid = (int)(tiles < sms ? tiles : sms);
  e = launch_pdl(kern, dim3(grid), 192 + 32 * CW, L::ALLOC, st, mx0, p);
  return e == cudaSuccess ? cudaGetLastError() : e;
}
}  // namespace tc

bool gemm_tc_supported(const TcGemmArgs& a) {
  if (a.int4) {  // packed weights read by the converter warps (16-byte loads), bf16 tokens by TMA
    auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
    return a.kind_f16 && a.terms == 1 && a.nseg == 0 && a.group_scale && ((uintptr_t)a.group_scale & 1) == 0 &&
           a.m >= 1 && a.n >= 1 && a.k >= 64 &&
           a.k % 64 == 0 && al(a.w) && al(a.x[0]) && a.x_stride_bytes % 16 == 0 && a.x_stride_bytes >= a.k * 2 &&
           a.m <= 0x7fffffffLL && a.n <= 0x7fffffffLL && a.k <= 0x7fffffffLL;
  }
  const int es = a.kind_f16 ? 2 : 1;
  auto al = [](const void* p) { return ((uintptr_t)p & 15) == 0; };
  if (a.m < 1 || a.n < 1 || a.k < 1) return false;
  if ((a.k * es) % 16 != 0) return false;
  if (a.w_stride_bytes % 16 != 0 || a.x_stride_bytes % 16 != 0) return false;
  if (a.w_stride_bytes < a.k * es || a.x_stride_bytes < a.k * es) return false;
  if (!al(a.w) || !al(a.x[0]) || (a.terms > 1 && !al(a.x[1]))) return false;
  if (a.m > 0x7fffffffLL || a.n > 0x7fffffffLL || a.k > 0x7fffffffLL) return false;
  if (a.nseg < 0 || a.nseg > WE_GEMM_MAX_SEGMENTS || (a.nseg > 0 && (!a.w2 || !al(a.w2)))) return false;
  if (a.nseg > 0 && (!a.epi.gate) != (!a.gate2)) return false;
  return true;
}

// Whether every inner segment boundary of a two-weight-set GEMM is a multiple of a token tile of c rows (token tiles
// may not straddle two weight sets).
static bool segments_fit(const TcGemmArgs& a, int c) {
  for (int i = 0; i + 1 < a.nseg; i++)
    if (a.row_end[i] % c) return false;
  return true;
}

template <int TERMS, bool F16>
static cudaError_t run_1sm(const TcGemmArgs& a, int bt, int sms, cudaStream_t st) {
  switch (bt) {
    case 256: return tc::run<256, TERMS, F16>(a, sms, st);
    case 128: return tc::run<128, TERMS, F16>(a, sms, st);
    case 96: return tc::run<96, TERMS, F16>(a, sms, st);
    default: return tc::run<64, TERMS, F16>(a, sms, st);
  }
}
template <int TERMS, bool F16>
static cudaError_t run_2sm(const TcGemmArgs& a, int bt, int sms, cudaStream_t st) {
  switch (bt) {
    case 128: return tc::run_pair<128, TERMS, F16>(a, sms, st);
    case 192: return tc::run_pair<192, TERMS, F16>(a, sms, st);
    default: return tc::run_pair<256, TERMS, F16>(a, sms, st);
  }
}

// Kernel and token tile by a cost model of waves x per-SM tile cost: a 1-SM tile (128 channels x c tokens) costs
// 1.2 c + 96 token-units, a pair tile (256 channels x c tokens on two SMs, half the shared-memory bytes per FLOP)
// c + 96. Fitted on 576 to 4608 tokens x N 3072 / 9216 / 12288 with c of 64 / 128 / 256; the 96- and 192-token
// tiles serve token counts that are multiples of 96 (a sequence-parallel rank's 576 rows: 6 x 96 or 3 x 192, where
// 64 / 128 / 256 leave a ragged last tile or a ragged last wave).
cudaError_t launch_gemm_tc(const TcGemmArgs& a, int sms, cudaStream_t st) {
  if (!gemm_tc_supported(a)) return cudaErrorNotSupported;
  if (a.int4) {
    if (const char* env = getenv("WE_TC_I4_WARPS"))  // tuning override: 4 converter warps instead of 8
      if (atoi(env) == 4) return tc::run_i4<256, 4>(a, sms, st);
    return tc::run_i4<256, 8>(a, sms, st);
  }
  const int64_t tn = (a.n + tc::BM - 1) / tc::BM;
  auto waves = [&](int64_t tiles, int64_t slots) { return (tiles + slots - 1) / slots; };
  double best_cost = -1.0;
  bool pair = false;
  int bt = 0;
  for (int c : {256, 192}) {
    if (!segments_fit(a, c)) continue;
    const double cost = (double)waves(((a.n + 255) / 256) * ((a.m + c - 1) / c), sms / 2) * (c + 96.0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      pair = true;
      bt = c;
    }
  }
  for (int c : {256, 128, 96, 64}) {
    if (!segments_fit(a, c)) continue;
    const double cost = (double)waves(tn * ((a.m + c - 1) / c), sms) * (1.2 * c + 96.0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      pair = false;
      bt = c;
    }
  }
  if (bt == 0) return cudaErrorNotSupported;  // no token tile fits the segments
  if (const char* env = getenv("WE_TC_2SM")) {  // tuning / test override: 0 never, 2 always (where tiles allow)
    const int v = atoi(env);
    if (v == 2 && segments_fit(a, 256)) {
      pair = true;
      bt = 256;
    } else if (v == 0 && pair) {
      pair = false;
      bt = 64;
      for (int c : {256, 128, 96})
        if (segments_fit(a, c) && c <= a.m) {
          bt = c;
          break;
        }
    }
  }
  if (pair) {
    // A 128-token pair tile fills the last wave better on some shapes (2304 tokens x 3072 channels: 2.92 waves of
    // 74 pairs against 1.46) but halves each tile's reuse of W from L2 and measured slower on every shape tried
    // (2304 x 3072 x 3072: 61.4 against 58.1 us; 4608 x 3072 x 3072: 100.7 against 73.4 us), so it is left to the
    // override.
    if (const char* env = getenv("WE_TC_PAIR_BT")) {  // tuning / test override: 128, 192 or 256 tokens per pair tile
      const int v = atoi(env);
      if ((v == 128 || v == 192 || v == 256) && segments_fit(a, v)) bt = v;
    }
    if (a.kind_f16) return run_2sm<1, true>(a, bt, sms, st);
    if (a.terms > 1) return run_2sm<2, false>(a, bt, sms, st);
    return run_2sm<1, false>(a, bt, sms, st);
  }
  if (const char* env = getenv("WE_TC_BT")) {  // tuning / test override: 64, 96, 128 or 256 tokens per tile
    const int v = atoi(env);
    if ((v == 64 || v == 96 || v == 128 || v == 256) && segments_fit(a, v)) bt = v;
  }
  if (a.kind_f16) return run_1sm<1, true>(a, bt, sms, st);
  if (a.terms > 1) return run_1sm<2, false>(a, bt, sms, st);
  return run_1sm<1, false>(a, bt, sms, st);
}

}  // namespace we
