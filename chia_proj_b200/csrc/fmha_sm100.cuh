// fmha_sm100.cuh -- forward attention with fused score modification, mask and
// normaliser for B200 (sm_100a).
//
// One CTA owns NQ = 2 query tiles of BM = 128 rows of one (batch, head) and
// streams key/value tiles of BN = 128 keys through shared memory:
//
//   warp 0-3   softmax warpgroup 0  (query tile 0; thread = one query row)
//   warp 4-7   softmax warpgroup 1  (query tile 1)
//   warp 8     MMA warp: one thread issues every tcgen05.mma
//   warp 9     load warp: one thread issues every TMA load
//
// Tensor memory (512 columns x 128 lanes, fp32 cells):
//   cols [  0,128)  S0 = Q0 K^T,  cols [128,256)  S1 = Q1 K^T
//   cols [256,256+D) O0,          cols [384,384+D) O1   (output accumulators)
// Shared memory: Q0 Q1 | P0 P1 (16-bit softmax output) | K/V tile ring.
//
// Pipeline per key tile j: as soon as softmax warpgroup w has copied S_w(j)
// out of TMEM it releases the S_w columns, and the MMA warp computes
// S_w(j+1) = Q_w K(j+1)^T into them while the warpgroup is still turning
// S_w(j) into P_w(j); once P_w(j) is in shared memory the MMA warp issues
// O_w += P_w(j) V(j). All UMMAs are SS (operands in 128-byte-swizzled smem:
// Q, K and P K-major, V MN-major). The softmax warpgroup waits for
// O_w += P_w(j-1) V(j-1) to retire before it overwrites P_w or rescales O_w.
//
// Normalisers: online softmax in the log2 domain with lazy rescaling (the
// running max only moves when it grows by more than 8, i.e. a factor 256, so
// O is rarely touched), or sigmoid / ReLU which need no row statistics.
// Masks never materialise: each query tile visits only the key tiles of its
// mask hull (mask_geom.cuh) and tiles entirely inside the mask skip the
// element-wise test.
//
// Every mbarrier wait is bounded; on expiry the kernel ORs
// CHIA_ERR_DEVICE_TIMEOUT into *status, drains its own copies and MMAs,
// frees its TMEM and returns.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "mask_geom.cuh"
#include "ptx.cuh"

namespace chia {

enum Kind : int {
  KIND_SOFTMAX = 0,  // plain / per-head temperature (folded into the scale)
  KIND_SOFTCAP = 1,
  KIND_ALIBI = 2,
  KIND_SIGMOID = 3,
  KIND_RELU = 4,
};

struct KernelArgs {
  MaskGeom mask;        // geometry in (virtual) row / key index space
  int32_t heads;        // H
  int32_t group;        // q heads per K/V head (grouped-query attention; 1 = none)
  int32_t vdil;         // rows of one virtual head are i' * vdil + r (1 = plain)
  int32_t n_qblocks;    // ceil(sq / (NQ * BM))
  int32_t n_vheads;     // B * H * vdil
  int32_t n_units;      // n_qblocks * n_vheads work units
  int32_t *sched;       // [next unit, finished CTAs] or null (static round robin)
  float score_scale;    // multiplies q.k before the mod (1/sqrt(D) by default)
  float softcap;        // KIND_SOFTCAP
  float sig_bias;       // KIND_SIGMOID
  float out_scale;      // KIND_RELU
  const float *head_param;  // ALiBi slope or TEMP multiplier per head, may be null
  void *o;
  int64_t o_sb, o_sh, o_ss;  // output strides (elements)
  int32_t *status;
  uint64_t timeout_ns;  // limit of every pipeline wait
  uint64_t drain_ns;    // limit of the waits for this CTA's own copies / MMAs at exit
  float *lse;           // softmax kinds: natural log-sum-exp per row [B, H, S_q], or null
};

template <int D>
struct FmhaConfig {
  static constexpr int BM = 128;
  static constexpr int BN = 128;
  static constexpr int NQ = 2;
  static constexpr int NCHUNK = D / 64;  // 128-byte column chunks per row
  static constexpr int Q_TILE_BYTES = BM * D * 2;
  static constexpr int KV_TILE_BYTES = BN * D * 2;
  static constexpr int CHUNK_Q_BYTES = BM * 128;
  static constexpr int CHUNK_KV_BYTES = BN * 128;
  // P tiles (softmax output, 16-bit, 128 rows x BN keys) live in shared
  // memory in the same 128-byte-swizzled K-major layout as Q, one per query
  // tile, so the next S = Q K^T can be computed in TMEM while the softmax
  // warpgroup still works on the current one.
  static constexpr int P_TILE_BYTES = BM * BN * 2;
  static constexpr int CHUNK_P_BYTES = BM * 128;
  // One ring of NKV tile slots shared by K and V (slot = item % NKV). Items
  // are loaded in the order the MMA warp consumes them: K of the first tile of
  // a unit, then for each tile K of the next tile before V of this one.
  static constexpr int NKV = (D == 128) ? 3 : 8;
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_P = OFF_Q + NQ * Q_TILE_BYTES;
  static constexpr int OFF_KV = OFF_P + NQ * P_TILE_BYTES;
  static constexpr int OFF_BAR = OFF_KV + NKV * KV_TILE_BYTES;
  // barriers: q q_empty | kv_full[NKV] kv_empty[NKV] |
  //           s_full[2] s_free[2] p_full[2] p_free[2] o_full[2] o_empty[2] |
  //           unit_full[2] unit_empty[2] | drain
  static constexpr int BAR_Q = 0;
  static constexpr int BAR_QEMPTY = 1;
  static constexpr int BAR_KVFULL = 2;
  static constexpr int BAR_KVEMPTY = BAR_KVFULL + NKV;
  static constexpr int BAR_SFULL = BAR_KVEMPTY + NKV;
  static constexpr int BAR_SFREE = BAR_SFULL + NQ;
  static constexpr int BAR_PFULL = BAR_SFREE + NQ;
  static constexpr int BAR_PFREE = BAR_PFULL + NQ;
  static constexpr int BAR_OFULL = BAR_PFREE + NQ;
  static constexpr int BAR_OEMPTY = BAR_OFULL + NQ;
  static constexpr int BAR_UFULL = BAR_OEMPTY + NQ;
  static constexpr int BAR_UEMPTY = BAR_UFULL + 2;
  static constexpr int BAR_DRAIN = BAR_UEMPTY + 2;
  static constexpr int NUM_BARS = BAR_DRAIN + 1;
  // misc: [0] TMEM base, [1] abort flag, [2..3] unit ring
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  // the ring's two units as decoded by the load thread (UnitSlot2 each)
  static constexpr int OFF_US = OFF_MISC + 16;
  static constexpr int SMEM_BYTES = OFF_US + 2 * 96;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack for 1024-byte alignment
  // 12 warps: warpgroups 0 and 1 = softmax (one query tile each), warpgroup 2
  // = MMA warp, load warp and two idle warps. setmaxnreg moves registers from
  // warpgroup 2 to the softmax warpgroups: 2*128*REG_SOFTMAX + 128*REG_OTHER
  // must equal 384 * 168 (the launch allocation under __launch_bounds__(384,1)).
  // 192 / 120 is the split at which neither side spills (208 / 88 left the
  // MMA and load warps spilling; 3% slower at config 2).
  static constexpr int THREADS = 384;
  static constexpr int MMA_WARP = 8;
  static constexpr int LOAD_WARP = 9;
  static constexpr int REG_SOFTMAX = 192;
  static constexpr int REG_OTHER = 120;
  static_assert(2 * 128 * REG_SOFTMAX + 128 * REG_OTHER == THREADS * 168, "register split");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t TMEM_S = 0;    // + w * 128 (fp32 S tile)
  static constexpr uint32_t TMEM_O = 256;  // + w * 128
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct WaitCtx {
  volatile int *abort;
  int32_t *status;
  uint64_t timeout_ns;  // pipeline waits
  uint64_t drain_ns;    // waits that ignore the abort flag (copies and MMAs in flight)
};

// ------------------------------------------------------------------------
// Optional timeline tracing (compile with -DCHIA_TRACE; nothing is emitted
// otherwise). CTA 0 records (tag, clock64) pairs per role into a static
// device buffer that chia_attn_trace_read() copies out. Roles: 0/1 softmax
// warpgroups (warp 0 / warp 4, lane 0), 2 MMA thread, 3 load thread.
// ------------------------------------------------------------------------
#ifdef CHIA_TRACE
#ifndef CHIA_TRACE_BLOCK
#define CHIA_TRACE_BLOCK 0
#endif
constexpr int kTraceEvents = 4096;
__device__ unsigned long long g_chia_trace[4][kTraceEvents][2];
struct Tracer {
  int role, n;
  __device__ __forceinline__ Tracer(int r) : role(r), n(0) {}
  __device__ __forceinline__ void operator()(int tag) {
    if (blockIdx.x == CHIA_TRACE_BLOCK && n < kTraceEvents) {
      g_chia_trace[role][n][0] = static_cast<unsigned long long>(tag);
      g_chia_trace[role][n][1] = clock64();
      ++n;
    }
  }
};
#else
struct Tracer {
  __device__ __forceinline__ Tracer(int) {}
  __device__ __forceinline__ void operator()(int) {}
};
#endif

// Bounded wait on an mbarrier phase. Returns false (and raises the CTA abort
// flag and the device status) when the wait expires or another warp aborted.
// A wait that ignores the abort flag waits for this CTA's own copies or MMAs
// before it exits; it keeps its own (long) limit, so that a short pipeline
// limit never lets a CTA leave with a copy in flight.
__device__ __forceinline__ bool bounded_wait(const WaitCtx &c, uint32_t bar, uint32_t parity,
                                             bool honour_abort = true) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  const uint64_t limit = honour_abort ? c.timeout_ns : c.drain_ns;
  // Each try may suspend for up to `hint` ns. With the default limit the
  // clock is read every 64 tries; a short limit (tests) shortens the
  // suspension and reads the clock after every try.
  const bool short_limit = limit < (64ull << 20);
  const uint32_t hint = short_limit ? static_cast<uint32_t>(limit >> 6) + 32u : (1u << 20);
  const uint32_t check_mask = short_limit ? 0u : 63u;
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity, hint)) return true;
    if ((it & check_mask) == 0) {
      if (honour_abort && *c.abort) return false;
      if (ptx::globaltimer_ns() - t0 > limit) {
        *c.abort = 1;
        if (c.status) atomicOr(c.status, 5 /* CHIA_ERR_DEVICE_TIMEOUT */);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------------
// softmax-warpgroup helpers: one thread owns one query row of a 128-key tile
// ------------------------------------------------------------------------
struct EpiConsts {
  float k_mul;   // multiplies the raw score
  float k_cap;   // softcap output scale (log2 domain)
  float k_bias;  // ALiBi slope * log2e * vdil, or sigmoid bias * -log2e
  float rel0;    // (j - i) of column 0 of the current tile
};

// Visibility of column c of the current tile for this thread's row.
struct RowMask {
  int c_lo;       // first band column relative to the tile (may be out of range)
  uint32_t span;  // band width - 1
  int c_pre;      // columns below this are in the always-visible prefix
  int i_rel;      // i - kv0, for the dilation test
  int dil;
};

// Visibility of column col for this thread's row (MODE 1: band + prefix,
// MODE 2: also the dilation test).
template <int MODE>
__device__ __forceinline__ bool col_visible(const RowMask &rm, int col) {
  bool vis = static_cast<uint32_t>(col - rm.c_lo) <= rm.span;
  if (MODE == 2) vis = vis && ((rm.i_rel - col) % rm.dil) == 0;
  return vis || (col < rm.c_pre);
}

// Softmax kinds, pass 1: score -> log2-domain logit x (modified and masked)
// in place; returns the row maximum. Work is done on packed pairs of columns.
// MODE 0: tile fully visible (no mask code); 1: band + prefix; 2: + dilation.
// NC chunks of 32 columns; EpiConsts::rel0 and RowMask refer to column 0 of
// sr, so a thread may own any 32-column-aligned part of the tile.
template <int KIND, int MODE, int NC = 4>
__device__ __forceinline__ float softmax_pass1(uint32_t (&sr)[NC][32], const EpiConsts &k,
                                               const RowMask &rm) {
  const uint64_t K2 = ptx::f2(k.k_mul, k.k_mul);
  const uint64_t CAP2 = ptx::f2(k.k_cap, k.k_cap);
  const uint64_t KB2 = ptx::f2(k.k_bias, k.k_bias);
  const uint64_t REL2 = ptx::f2(k.rel0, k.rel0 + 1.0f);
  float m[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    float mc = -INFINITY;
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const int col = c * 32 + e;
      uint64_t x2 = ptx::mul2(ptx::f2(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])), K2);
      if (KIND == KIND_SOFTCAP) {
        float a, b;
        ptx::f2_split(x2, a, b);
        x2 = ptx::mul2(ptx::f2(ptx::tanh_fast(a), ptx::tanh_fast(b)), CAP2);
      } else if (KIND == KIND_ALIBI) {
        // bias = slope * (j - i): (j - i) is formed exactly before scaling
        const uint64_t rel = ptx::add2(REL2, ptx::f2(static_cast<float>(col), static_cast<float>(col)));
        x2 = ptx::fma2(KB2, rel, x2);
      }
      float a, b;
      ptx::f2_split(x2, a, b);
      if (MODE != 0) {
        if (!col_visible<MODE>(rm, col)) a = -INFINITY;
        if (!col_visible<MODE>(rm, col + 1)) b = -INFINITY;
      }
      mc = ptx::max3(mc, a, b);
      sr[c][e] = __float_as_uint(a);
      sr[c][e + 1] = __float_as_uint(b);
    }
    m[c] = mc;
  }
  static_assert(NC == 2 || NC == 4, "64 or 128 columns");
  if constexpr (NC == 4)
    return fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
  else
    return fmaxf(m[0], m[1]);
}

// Write 64 keys (32 packed pairs) of this thread's P row into the
// 128-byte-swizzled K-major P tile: 16-byte unit u of row r goes to unit
// u ^ (r % 8), so the eight rows of a quarter-warp hit eight distinct bank
// groups. prow = address of row r in chunk 0; chunk h2 holds keys 64*h2..+63.
__device__ __forceinline__ void store_p_chunk(uint32_t prow, int h2, int rsw,
                                              const uint32_t (&pk)[32]) {
#pragma unroll
  for (int u = 0; u < 8; ++u)
    ptx::st_shared_v4(prow + h2 * (128 * 128) + ((u ^ rsw) << 4), pk[4 * u], pk[4 * u + 1],
                      pk[4 * u + 2], pk[4 * u + 3]);
}

// Destinations of a P row: 64 keys (32 packed pairs) at a time.
struct PSinkSmem {  // shared-memory P tile (single-CTA kernel)
  uint32_t prow;
  int rsw;
  __device__ __forceinline__ void operator()(int h2, const uint32_t (&pk)[32]) const {
    store_p_chunk(prow, h2, rsw, pk);
  }
};
struct PSinkTmem {  // TMEM columns of the S tile, read back by a TS-UMMA (2-SM kernel)
  uint32_t tP;
  __device__ __forceinline__ void operator()(int h2, const uint32_t (&pk)[32]) const {
    ptx::tmem_st32(tP + h2 * 32, pk);
  }
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? ptx::pack_bf16(lo, hi) : ptx::pack_f16(lo, hi);
}

// Softmax pass 2: p = 2^(x - m), packed to 16-bit pairs and handed to the
// P sink 64 keys at a time; returns the row sum of p.
template <bool BF16, class Sink, int NC = 4>
__device__ __forceinline__ float softmax_pass2(uint32_t (&sr)[NC][32], float m, const Sink &sink) {
  static_assert(NC == 2 || NC == 4, "64 or 128 columns");
  const uint64_t NM2 = ptx::f2(-m, -m);
  uint64_t acc[2] = {ptx::f2(0.f, 0.f), ptx::f2(0.f, 0.f)};
#pragma unroll
  for (int h2 = 0; h2 < NC / 2; ++h2) {
    uint32_t pk[32];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * h2 + cc;
#pragma unroll
      for (int e = 0; e < 32; e += 2) {
        float a, b;
        ptx::f2_split(ptx::add2(ptx::f2(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])), NM2),
                      a, b);
        const float p0 = ptx::ex2(a), p1 = ptx::ex2(b);
        acc[cc] = ptx::add2(acc[cc], ptx::f2(p0, p1));
        pk[cc * 16 + e / 2] = pack2<BF16>(p0, p1);
      }
    }
    sink(h2, pk);
  }
  float s0, s1, s2, s3;
  ptx::f2_split(acc[0], s0, s1);
  ptx::f2_split(acc[1], s2, s3);
  return (s0 + s1) + (s2 + s3);
}

// Non-softmax kinds: P = relu(s * scale) or sigmoid(s * scale + bias),
// masked, packed and handed to the P sink.
// Sigmoid is 1 / (1 + 2^t): 2^t on the MUFU, the reciprocal on the FMA pipe:
// an initial guess r0 = as_float(0x7EF311C2 - bits(y)) and Newton steps
// r <- r (2 - y r). The constant minimises the largest relative error of r0
// over all y (0.0505; the search is recip_seed.py beside this file). One step
// leaves a one-sided error 1 - y r in [0, 0.0505^2 = 2.55e-3]; the epilogue
// multiplies O by kSigmoidCentre = 1 / (1 - 2.55e-3 / 2), which centres it to
// +-1.28e-3, below the rounding of a bf16 P (2^-9 .. 2^-8 relative). fp16 P
// rounds to 2^-11, so fp16 takes a second step (error 0.0505^4 = 6.5e-6).
// y is negated and quartered here, y = -(1 + 2^t) / 4 (hence 0xFEF311C2 -
// bits), so r and P are 4 sigmoid and the epilogue's output scale takes the
// 4 back. The quarter keeps bits(y) below the seed constant for every finite
// 2^t, so no clamp of t is needed: 2^t = inf (t >= 128) gives r = -inf,
// which the ReLU form of the conversion packs as 0, the limit of sigmoid.
// One 32-column chunk (src, columns col0..col0+31 of the tile) of the
// pointwise kinds, as 16 packed pairs into pk[off .. off+15].
// Output scale that centres the one-sided error of the single Newton step
// of a bf16 sigmoid P (see pointwise_chunk): 1 / (1 - 0.0505^2 / 2).
constexpr float kSigmoidCentre = 1.001277273908313f;
template <bool BF16>
__device__ __forceinline__ constexpr float pointwise_out_scale(int kind) {
  return kind == KIND_SIGMOID ? (BF16 ? 0.25f * kSigmoidCentre : 0.25f) : 1.0f;
}

template <int KIND, int MODE, bool BF16>
__device__ __forceinline__ void pointwise_chunk(const uint32_t (&src)[32], int col0,
                                                const EpiConsts &k, const RowMask &rm,
                                                uint32_t (&pk)[32], int off) {
  const uint64_t K2 = ptx::f2(k.k_mul, k.k_mul);
  const uint64_t KB2 = ptx::f2(k.k_bias, k.k_bias);
  const uint64_t NEGQ = ptx::f2(-0.25f, -0.25f);
  const uint64_t TWO2 = ptx::f2(2.0f, 2.0f);
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const int col = col0 + e;
    const uint64_t s2 = ptx::f2(__uint_as_float(src[e]), __uint_as_float(src[e + 1]));
    float a, b;
    if (KIND == KIND_RELU) {
      ptx::f2_split(ptx::mul2(s2, K2), a, b);
      if (MODE != 0) {
        if (!col_visible<MODE>(rm, col)) a = 0.f;
        if (!col_visible<MODE>(rm, col + 1)) b = 0.f;
      }
      pk[off + e / 2] = BF16 ? ptx::pack_bf16_relu(a, b) : ptx::pack_f16_relu(a, b);
    } else {
      // t = -(s*scale + bias) * log2(e)
      float t0, t1;
      ptx::f2_split(ptx::fma2(s2, K2, KB2), t0, t1);
      const uint64_t e2 = ptx::f2(ptx::ex2(t0), ptx::ex2(t1));
      const uint64_t ny = ptx::fma2(e2, NEGQ, NEGQ);  // -(1 + 2^t) / 4
      float y0, y1;
      ptx::f2_split(ny, y0, y1);
      uint64_t r = ptx::f2(__uint_as_float(0xFEF311C2u - __float_as_uint(y0)),
                           __uint_as_float(0xFEF311C2u - __float_as_uint(y1)));
      r = ptx::mul2(r, ptx::fma2(ny, r, TWO2));
      if (!BF16) r = ptx::mul2(r, ptx::fma2(ny, r, TWO2));
      ptx::f2_split(r, a, b);
      if (MODE != 0) {
        if (!col_visible<MODE>(rm, col)) a = 0.f;
        if (!col_visible<MODE>(rm, col + 1)) b = 0.f;
      }
      pk[off + e / 2] = BF16 ? ptx::pack_bf16_relu(a, b) : ptx::pack_f16_relu(a, b);
    }
  }
}

template <int KIND, int MODE, bool BF16, class Sink, int NC = 4>
__device__ __forceinline__ void pointwise_tile(uint32_t (&sr)[NC][32], const EpiConsts &k,
                                               const RowMask &rm, const Sink &sink) {
  static_assert(NC == 2 || NC == 4, "64 or 128 columns");
#pragma unroll
  for (int h2 = 0; h2 < NC / 2; ++h2) {
    uint32_t pk[32];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc)
      pointwise_chunk<KIND, MODE, BF16>(sr[2 * h2 + cc], (2 * h2 + cc) * 32, k, rm, pk, cc * 16);
    sink(h2, pk);
  }
}

// Pointwise kinds on this thread's 64 columns of a TMEM S tile (2-SM
// kernel): chunk 0 is transformed while chunk 1 is still being read from
// tensor memory; P (64 keys) goes back over chunk 0's columns.
template <int KIND, int MODE, bool BF16>
__device__ __forceinline__ void pointwise_tmem64(uint32_t tS, const EpiConsts &k,
                                                 const RowMask &rm) {
  uint32_t s0[32], s1[32], pk[32];
  ptx::tmem_ld32(tS, s0);
  ptx::tmem_wait_ld();
  ptx::reg_fence(s0);
  ptx::tmem_ld32(tS + 32, s1);
  pointwise_chunk<KIND, MODE, BF16>(s0, 0, k, rm, pk, 0);
  ptx::tmem_wait_ld();
  ptx::reg_fence(s1);
  pointwise_chunk<KIND, MODE, BF16>(s1, 32, k, rm, pk, 16);
  ptx::tmem_st32(tS, pk);
}

// D columns of O (from tO) of this thread's row *= alpha (lazy softmax
// rescale; rare).
template <int D>
__device__ __noinline__ void rescale_rows(uint32_t tO, float alpha) {
#pragma unroll 1
  for (int dc = 0; dc < D / 32; ++dc) {
    uint32_t o[32];
    ptx::tmem_ld32(tO + dc * 32, o);
    ptx::tmem_wait_ld();
    ptx::reg_fence(o);
#pragma unroll
    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
    ptx::tmem_st32(tO + dc * 32, o);
  }
}

// Epilogue: D columns of O row (from tO) * inv -> 16-bit -> global at orow
// (one thread per row).
template <int D, bool BF16>
__device__ __forceinline__ void store_rows(uint32_t tO, float inv, bool row_ok, uint8_t *orow) {
#pragma unroll 1
  for (int dc = 0; dc < D / 32; ++dc) {
    uint32_t o[32];
    ptx::tmem_ld32(tO + dc * 32, o);
    ptx::tmem_wait_ld();
    ptx::reg_fence(o);
    uint32_t pkd[16];
#pragma unroll
    for (int e = 0; e < 16; ++e)
      pkd[e] = pack2<BF16>(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
    if (row_ok) {
#pragma unroll
      for (int v4 = 0; v4 < 4; ++v4)
        ptx::st_global_v4(orow + dc * 64 + v4 * 16, pkd[4 * v4], pkd[4 * v4 + 1], pkd[4 * v4 + 2],
                          pkd[4 * v4 + 3]);
    }
  }
}

// Natural log-sum-exp of one row, ln(sum_j e^{s_j}) = (m + log2 l) ln 2, from
// the running maximum m (log2 domain) and the row sum l = sum 2^(x - m); -inf
// for a row that sees no key. Layout [B, H, S_q] (real rows), fp32.
__device__ __forceinline__ void store_lse(const KernelArgs &a, int b, int h, int64_t real_row,
                                          float m, float l) {
  constexpr float LN2 = 0.6931471805599453f;
  const int64_t sq_real = a.mask.sq * a.vdil;
  const float v = (l > 0.f) ? (m + __log2f(l)) * LN2 : -INFINITY;
  a.lse[(static_cast<int64_t>(b) * a.heads + h) * sq_real + real_row] = v;
}

// One work unit: two query tiles (NQ * BM rows) of one (virtual) head.
struct UnitInfo {
  int r_res, h, b;
  int64_t m0;
  int64_t tlo[2], thi[2];  // key-tile range per query tile (empty: lo == hi)
  int64_t jlo, jhi;        // union of both ranges
  __device__ __forceinline__ bool active(int w, int64_t j) const {
    return j >= tlo[w] && j < thi[w];
  }
  __device__ __forceinline__ bool any_active(int64_t j) const { return active(0, j) || active(1, j); }
  __device__ __forceinline__ bool wg_on(int w) const { return tlo[w] < thi[w]; }
};

// Units are ordered head-major with the heaviest query block of a head first,
// so the units in flight at any time share K/V in L2 and the light blocks
// finish the schedule.
template <int BM, int BN, bool SEG = false>
__device__ __forceinline__ void decode_unit(int u, const KernelArgs &a, UnitInfo &U) {
  const int vh = u / a.n_qblocks;
  const int qb = a.n_qblocks - 1 - (u % a.n_qblocks);
  U.r_res = vh % a.vdil;
  U.h = (vh / a.vdil) % a.heads;
  U.b = vh / (a.vdil * a.heads);
  U.m0 = static_cast<int64_t>(qb) * (2 * BM);
  U.jlo = INT64_MAX;
  U.jhi = 0;
#pragma unroll
  for (int w = 0; w < 2; ++w) {
    tile_range<SEG>(a.mask, U.m0 + w * BM, U.m0 + w * BM + BM - 1, BN, U.tlo[w], U.thi[w]);
    if (U.tlo[w] < U.thi[w]) {
      U.jlo = imin64(U.jlo, U.tlo[w]);
      U.jhi = imax64(U.jhi, U.thi[w]);
    }
  }
  if (U.jlo > U.jhi) U.jlo = U.jhi = 0;  // no row of the unit sees a key
}

// A work unit of the head_dim-64 kernel as its load thread hands it to the
// MMA warp and the softmax warpgroups through the unit ring, decoded once
// (decoding costs each reader a few thousand cycles of dependent integer work
// at every unit boundary).
struct UnitSlot2 {
  int32_t jlo, jhi;        // key tiles of the unit
  int32_t m0;              // first query row
  int32_t r_res, h, b;     // residue class (dilation), query head, batch
  int32_t tlo[2], thi[2];  // key tiles of each query tile (empty: lo == hi)
  FullTiles ft[2];         // key tiles each query tile's rows all see completely
  float hp;                // per-head parameter
  int32_t pad[5];
};
static_assert(sizeof(UnitSlot2) == 96, "unit slot layout");

// Persistent kernel: each CTA loops over work units. With a scheduler
// workspace the load warp takes the next unit from a global counter (dynamic
// balance; the last CTA to finish puts the counter back to zero), otherwise
// CTA c runs units c, c + grid, c + 2 grid, ... . The unit index travels to the
// other roles through a two-slot ring in shared memory.
template <int D, bool BF16, int KIND, bool SEG>
__global__ void __launch_bounds__(FmhaConfig<D>::THREADS, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const KernelArgs args) {
  using C = FmhaConfig<D>;
  constexpr int BM = C::BM, BN = C::BN, NQ = C::NQ, NKV = C::NKV;
  constexpr bool SOFTMAX = (KIND == KIND_SOFTMAX || KIND == KIND_SOFTCAP || KIND == KIND_ALIBI);
  constexpr float LOG2E = 1.4426950408889634f;

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  auto bar = [&](int idx) -> uint32_t { return sbase + C::OFF_BAR + idx * 8; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 4);
  volatile int *unit_ring = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 8);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const MaskGeom &g = args.mask;

  // ---- setup: barriers, TMEM ----
  if (threadIdx.x == 0) {
    ptx::mbar_init(bar(C::BAR_Q), 1);
    ptx::mbar_init(bar(C::BAR_QEMPTY), 1);
    for (int s = 0; s < NKV; ++s) {
      ptx::mbar_init(bar(C::BAR_KVFULL + s), 1);
      ptx::mbar_init(bar(C::BAR_KVEMPTY + s), 1);
    }
    for (int w = 0; w < NQ; ++w) {
      ptx::mbar_init(bar(C::BAR_SFULL + w), 1);
      ptx::mbar_init(bar(C::BAR_SFREE + w), 4);   // one arrive per softmax warp
      ptx::mbar_init(bar(C::BAR_PFULL + w), 4);   // one arrive per softmax warp
      ptx::mbar_init(bar(C::BAR_PFREE + w), 1);
      ptx::mbar_init(bar(C::BAR_OFULL + w), 1);
      ptx::mbar_init(bar(C::BAR_OEMPTY + w), 4);  // one arrive per softmax warp
    }
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(bar(C::BAR_UFULL + s), 1);
      ptx::mbar_init(bar(C::BAR_UEMPTY + s), 1 + 8);  // MMA thread + 8 softmax warps
    }
    ptx::mbar_init(bar(C::BAR_DRAIN), 1);
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == C::LOAD_WARP && lane == 0) {
    ptx::tma_prefetch_desc(&tm_q);
    ptx::tma_prefetch_desc(&tm_k);
    ptx::tma_prefetch_desc(&tm_v);
  }
  if (warp == C::MMA_WARP) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_slot), C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, args.status, args.timeout_ns, args.drain_ns};

  if (warp >= 8) {
    ptx::setmaxnreg_dec<C::REG_OTHER>();
    if (warp == C::LOAD_WARP && lane == 0) {
      // ==================== scheduler + TMA producer ====================
      Tracer tr(3);
      uint32_t n = 0;  // ring items issued (K and V of every tile)
      int last_q = -1;  // unit whose Q copies were issued last
      int64_t last_item[NKV];
      for (int s = 0; s < NKV; ++s) last_item[s] = -1;
      auto load_item = [&](const CUtensorMap *map, int64_t j, const UnitInfo &U) -> bool {
        const int s = n % NKV;
        if (!bounded_wait(wc, bar(C::BAR_KVEMPTY + s), ((n / NKV) & 1) ^ 1)) return false;
        tr(30);  // ring slot free, issuing a K or V tile
        ptx::mbar_arrive_expect_tx(bar(C::BAR_KVFULL + s), C::KV_TILE_BYTES);
#pragma unroll
        for (int c = 0; c < C::NCHUNK; ++c)
          ptx::tma_load_5d(sbase + C::OFF_KV + s * C::KV_TILE_BYTES + c * C::CHUNK_KV_BYTES, map,
                           bar(C::BAR_KVFULL + s), c * 64, static_cast<int>(j * BN), U.r_res,
                           U.h / args.group, U.b);
        last_item[s] = n;
        ++n;
        return true;
      };
      for (int k = 0;; ++k) {
        const int slot = k & 1;
        if (!bounded_wait(wc, bar(C::BAR_UEMPTY + slot), ((k >> 1) & 1) ^ 1)) break;
        int u = args.sched ? atomicAdd(args.sched, 1) : static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
        if (u >= args.n_units || u < 0) u = -1;
        unit_ring[slot] = u;
        UnitInfo U;
        if (u >= 0) {
          decode_unit<BM, BN, SEG>(u, args, U);
          UnitSlot2 *e = reinterpret_cast<UnitSlot2 *>(smem + C::OFF_US) + slot;
          e->jlo = static_cast<int32_t>(U.jlo);
          e->jhi = static_cast<int32_t>(U.jhi);
          e->m0 = static_cast<int32_t>(U.m0);
          e->r_res = U.r_res;
          e->h = U.h;
          e->b = U.b;
#pragma unroll
          for (int w = 0; w < NQ; ++w) {
            e->tlo[w] = static_cast<int32_t>(U.tlo[w]);
            e->thi[w] = static_cast<int32_t>(U.thi[w]);
            e->ft[w] = full_tiles<SEG>(g, U.m0 + w * BM, U.m0 + w * BM + BM - 1, BN);
          }
          e->hp = args.head_param != nullptr ? args.head_param[U.h] : 1.0f;
        }
        ptx::mbar_arrive(bar(C::BAR_UFULL + slot));
        if (u < 0) break;
        // Q tiles: the previous unit's S MMAs must be done with the buffer
        if (k > 0 && !bounded_wait(wc, bar(C::BAR_QEMPTY), (k - 1) & 1)) break;
        uint32_t qbytes = 0;
#pragma unroll
        for (int w = 0; w < NQ; ++w)
          if (U.wg_on(w)) qbytes += C::Q_TILE_BYTES;
        ptx::mbar_arrive_expect_tx(bar(C::BAR_Q), qbytes);
        last_q = k;
#pragma unroll
        for (int w = 0; w < NQ; ++w)
          if (U.wg_on(w))
#pragma unroll
            for (int c = 0; c < C::NCHUNK; ++c)
              ptx::tma_load_5d(sbase + C::OFF_Q + w * C::Q_TILE_BYTES + c * C::CHUNK_Q_BYTES,
                               &tm_q, bar(C::BAR_Q), c * 64, static_cast<int>(U.m0 + w * BM),
                               U.r_res, U.h, U.b);
        // K(jlo), then K(j+1) before V(j): ring position of K_i is 2i-1
        // (K_0 at 0), of V_i 2i+2, of the last V 2T-1 (T tiles in the unit)
        bool ok = U.jlo == U.jhi || load_item(&tm_k, U.jlo, U);  // no items for a keyless unit
        for (int64_t j = U.jlo; ok && j < U.jhi; ++j) {
          if (j + 1 < U.jhi) ok = load_item(&tm_k, j + 1, U);
          ok = ok && load_item(&tm_v, j, U);
        }
        if (!ok) break;
      }
      // Drain: every copy this thread issued lands before the CTA exits. The
      // Q copies of a unit are issued only after the previous unit's have
      // been consumed, so the last unit's phase is the only one to wait for.
      for (int s = 0; s < NKV; ++s)
        if (last_item[s] >= 0)
          bounded_wait(wc, bar(C::BAR_KVFULL + s), (last_item[s] / NKV) & 1, false);
      if (last_q >= 0) bounded_wait(wc, bar(C::BAR_Q), last_q & 1, false);
    } else if (warp == C::MMA_WARP) {
      // =========================== UMMA issuer ===========================
      // The whole warp runs this loop in lockstep: readiness is tested by
      // lane 0 and broadcast, so control flow stays uniform, the descriptors
      // stay in uniform registers, and elect.sync picks the issuing lane.
      auto uni = [&](bool x) { return __shfl_sync(0xffffffffu, x ? 1 : 0, 0) != 0; };
      constexpr uint32_t IDESC_QK = ptx::make_idesc_f16(BM, BN, BF16, false, false);
      constexpr uint32_t IDESC_PV = ptx::make_idesc_f16(BM, D, BF16, false, true);
      const uint32_t q_s = sbase + C::OFF_Q, p_s = sbase + C::OFF_P, kv_s = sbase + C::OFF_KV;

      // Descriptor of each operand at k-step 0; the start-address field (bits
      // 0-13, address >> 4) is then advanced by plain adds: shared memory
      // addresses stay below 256 KB, so the field never carries.
      const uint64_t dq = ptx::make_sdesc_sw128(q_s, 16, 1024);
      const uint64_t dp = ptx::make_sdesc_sw128(p_s, 16, 1024);
      const uint64_t dk = ptx::make_sdesc_sw128(kv_s, 16, 1024);
      const uint64_t dv = ptx::make_sdesc_sw128(kv_s, C::CHUNK_KV_BYTES, 1024);
      auto issue_s = [&](int w, int stage) {
        const uint32_t d_tmem = tmem_base + C::TMEM_S + w * 128;
        const uint64_t a0 = dq + ((w * C::Q_TILE_BYTES) >> 4);
        const uint64_t b0 = dk + ((stage * C::KV_TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = ((kk >> 2) * C::CHUNK_Q_BYTES + (kk & 3) * 32) >> 4;
          const uint32_t offk = ((kk >> 2) * C::CHUNK_KV_BYTES + (kk & 3) * 32) >> 4;
          ptx::umma_ss_warp(d_tmem, a0 + off, b0 + offk, IDESC_QK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int w, int stage, bool first) {
        const uint32_t d_tmem = tmem_base + C::TMEM_O + w * 128;
        const uint64_t a0 = dp + ((w * C::P_TILE_BYTES) >> 4);
        const uint64_t b0 = dv + ((stage * C::KV_TILE_BYTES) >> 4);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t offp = ((kk >> 2) * C::CHUNK_P_BYTES + (kk & 3) * 32) >> 4;
          ptx::umma_ss_warp(d_tmem, a0 + offp, b0 + ((kk * 2048) >> 4), IDESC_PV,
                       (first && kk == 0) ? 0u : 1u);
        }
      };

      Tracer trc(2);
      auto tr = [&](int tag) { if (lane == 0) trc(tag); };
      // Event-driven issue: the thread polls every pending step of both query
      // tiles and issues whichever is ready, so neither softmax warpgroup
      // waits behind the other.
      //   S_w(t)  needs K(t) resident and S_w(t-1) copied out of TMEM (s_free)
      //   PV_w(t) needs P_w(t) written (p_full), V(t) resident, and for the
      //           first tile of a unit the previous epilogue done (o_empty)
      // A K / V ring slot is released once every query tile that uses it has
      // issued its MMA (and the copy into it has landed).
      uint32_t base = 0;  // ring position of the current unit's first item
      uint32_t scnt[NQ] = {0, 0}, pcnt[NQ] = {0, 0}, units_w[NQ] = {0, 0};
      auto test_item = [&](uint32_t item) {
        return uni(ptx::mbar_test_wait(bar(C::BAR_KVFULL + item % NKV), (item / NKV) & 1));
      };
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k & 1;
        if (!__all_sync(0xffffffffu, bounded_wait(wc, bar(C::BAR_UFULL + slot), (k >> 1) & 1)))
          break;
        const int u = __shfl_sync(0xffffffffu, unit_ring[slot], 0);
        const UnitSlot2 U = reinterpret_cast<const UnitSlot2 *>(smem + C::OFF_US)[slot];
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(C::BAR_UEMPTY + slot));
        if (u < 0) break;
        if (!__all_sync(0xffffffffu, bounded_wait(wc, bar(C::BAR_Q), k & 1))) break;
        const int jlo = U.jlo, T = U.jhi - U.jlo;
        auto kpos = [&](int i) { return base + static_cast<uint32_t>(i == 0 ? 0 : 2 * i - 1); };
        auto vpos = [&](int i) {
          return base + static_cast<uint32_t>(i < T - 1 ? 2 * i + 2 : 2 * T - 1);
        };
        int sn[NQ], pn[NQ], lo[NQ], hi[NQ];
#pragma unroll
        for (int w = 0; w < NQ; ++w) {
          lo[w] = U.tlo[w];
          hi[w] = U.thi[w];
          sn[w] = pn[w] = lo[w];
        }
        auto user = [&](int w, int t) { return t >= lo[w] && t < hi[w]; };
        int krel = 0, vrel = 0;  // next K / V item (tile offset) to release
        bool q_released = false;
        uint64_t idle_since = 0;
        while (true) {
          bool progress = false;
#pragma unroll
          for (int w = 0; w < NQ; ++w) {
            if (sn[w] < hi[w]) {
              const uint32_t it = kpos(sn[w] - jlo);
              if (test_item(it) &&
                  (scnt[w] == 0 ||
                   uni(ptx::mbar_test_wait(bar(C::BAR_SFREE + w), (scnt[w] - 1) & 1)))) {
                ptx::tc_fence_after();
                issue_s(w, it % NKV);
                ptx::umma_commit_warp(bar(C::BAR_SFULL + w));
                ++scnt[w];
                ++sn[w];
                progress = true;
                tr(20 + w);  // S_w issued
              }
            }
            if (pn[w] < hi[w]) {
              const uint32_t it = vpos(pn[w] - jlo);
              const bool first = pn[w] == lo[w];
              if (uni(ptx::mbar_test_wait(bar(C::BAR_PFULL + w), pcnt[w] & 1)) && test_item(it) &&
                  (!first || units_w[w] == 0 ||
                   uni(ptx::mbar_test_wait(bar(C::BAR_OEMPTY + w), (units_w[w] - 1) & 1)))) {
                ptx::tc_fence_after();
                issue_pv(w, it % NKV, first);
                ptx::umma_commit_warp(bar(C::BAR_PFREE + w));
                ++pcnt[w];
                if (pn[w] == hi[w] - 1) {
                  ptx::umma_commit_warp(bar(C::BAR_OFULL + w));
                  ++units_w[w];
                }
                ++pn[w];
                progress = true;
                tr(22 + w);  // PV_w issued
              }
            }
          }
          // release ring items, in order, once all their users have issued
          while (krel < T) {
            const int t = jlo + krel;
            if ((user(0, t) && sn[0] <= t) || (user(1, t) && sn[1] <= t)) break;
            const uint32_t it = kpos(krel);
            if (!test_item(it)) break;  // an unused item must still have landed
            ptx::umma_commit_warp(bar(C::BAR_KVEMPTY + it % NKV));
            ++krel;
          }
          while (vrel < T) {
            const int t = jlo + vrel;
            if ((user(0, t) && pn[0] <= t) || (user(1, t) && pn[1] <= t)) break;
            const uint32_t it = vpos(vrel);
            if (!test_item(it)) break;
            ptx::umma_commit_warp(bar(C::BAR_KVEMPTY + it % NKV));
            ++vrel;
          }
          if (!q_released && sn[0] >= hi[0] && sn[1] >= hi[1]) {
            ptx::umma_commit_warp(bar(C::BAR_QEMPTY));  // every S of this unit issued
            q_released = true;
          }
          if (krel >= T && vrel >= T && pn[0] >= hi[0] && pn[1] >= hi[1]) break;
          if (progress) {
            idle_since = 0;
          } else {
            // nothing ready: back off briefly, bounded like every other wait
            const uint64_t now = __shfl_sync(0xffffffffu, ptx::globaltimer_ns(), 0);
            if (idle_since == 0) idle_since = now;
            if (uni(*abort_flag != 0)) { ok = false; break; }
            if (now - idle_since > args.timeout_ns) {
              *abort_flag = 1;
              if (args.status && lane == 0) atomicOr(args.status, 5 /* CHIA_ERR_DEVICE_TIMEOUT */);
              ok = false;
              break;
            }
            __nanosleep(20);
          }
        }
        base += 2 * static_cast<uint32_t>(T);
      }
      // Drain: all UMMAs issued by this thread complete before TMEM is freed.
      ptx::umma_commit_warp(bar(C::BAR_DRAIN));
      bounded_wait(wc, bar(C::BAR_DRAIN), 0, false);
    }
    __syncwarp();
  } else {
    ptx::setmaxnreg_inc<C::REG_SOFTMAX>();
    // ======================= softmax / epilogue =======================
    const int w = warp >> 2;           // query tile of this warpgroup
    const int quad = warp & 3;         // TMEM lane quadrant of this warp
    const int row = quad * 32 + lane;  // row inside the query tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + C::TMEM_S + w * 128;
    const uint32_t tO = tmem_base + lane_off + C::TMEM_O + w * 128;
    const uint32_t prow = sbase + C::OFF_P + w * C::P_TILE_BYTES + row * 128;  // this row of P_w
    const int rsw = row & 7;
    const int prefix = static_cast<int>(g.prefix);
    const int dil = static_cast<int>(g.dil);
    const float score_scale = args.score_scale;

    Tracer tr(warp == 0 ? 0 : 1);
    const bool tracing = (warp & 3) == 0 && lane == 0;
    auto trs = [&](int tag) { if (tracing) tr(tag); };
    uint32_t cnt = 0, units_w = 0;
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      if (!bounded_wait(wc, bar(C::BAR_UFULL + slot), (k >> 1) & 1)) break;
      const int u = unit_ring[slot];
      const UnitSlot2 U = reinterpret_cast<const UnitSlot2 *>(smem + C::OFF_US)[slot];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_UEMPTY + slot));
      if (u < 0) break;
      const int i = U.m0 + w * BM + row;
      if (U.tlo[w] >= U.thi[w]) {
        // no row of this query tile sees a key: its output is zero
        if (i < g.sq) {
          const int64_t real_row = static_cast<int64_t>(i) * args.vdil + U.r_res;
          if (SOFTMAX && args.lse != nullptr) store_lse(args, U.b, U.h, real_row, -INFINITY, 0.f);
          uint8_t *orow = reinterpret_cast<uint8_t *>(args.o) +
                          2 * (U.b * args.o_sb + static_cast<int64_t>(U.h) * args.o_sh +
                               real_row * args.o_ss);
#pragma unroll
          for (int v4 = 0; v4 < D / 8; ++v4) ptx::st_global_v4(orow + v4 * 16, 0u, 0u, 0u, 0u);
        }
        continue;
      }

      const FullTiles ft = U.ft[w];
      int64_t blo64, bhi64;
      row_band<SEG>(g, i, blo64, bhi64);
      const bool band_empty = bhi64 < blo64;
      const int blo = band_empty ? (1 << 30) : static_cast<int>(blo64);
      const uint32_t span = band_empty ? 0u : static_cast<uint32_t>(bhi64 - blo64);
      // per-kind constants (log2 domain for the softmax kinds)
      const float hp = U.hp;
      EpiConsts kc;
      kc.k_mul = score_scale * LOG2E;
      kc.k_cap = 0.f;
      kc.k_bias = 0.f;
      if (KIND == KIND_SOFTMAX) kc.k_mul *= hp;
      if (KIND == KIND_SOFTCAP) {
        kc.k_mul = score_scale / args.softcap;
        kc.k_cap = args.softcap * LOG2E;
      }
      if (KIND == KIND_ALIBI) kc.k_bias = hp * LOG2E * static_cast<float>(args.vdil);
      if (KIND == KIND_SIGMOID) {
        kc.k_mul = -score_scale * LOG2E;
        kc.k_bias = -args.sig_bias * LOG2E;
      }
      if (KIND == KIND_RELU) kc.k_mul = score_scale;

      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int t = U.tlo[w]; t < U.thi[w]; ++t, ++cnt) {
        if (!bounded_wait(wc, bar(C::BAR_SFULL + w), cnt & 1)) { ok = false; break; }
        trs(10);  // S ready
        ptx::tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) ptx::tmem_ld32(tS + c * 32, sr[c]);
        ptx::tmem_wait_ld();
        trs(11);  // S in registers
#pragma unroll
        for (int c = 0; c < 4; ++c) ptx::reg_fence(sr[c]);
        // S_w is in registers: its TMEM columns may take the next tile
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(C::BAR_SFREE + w));

        const int kv0 = static_cast<int>(t) * BN;
        RowMask rm;
        rm.c_lo = blo - kv0;
        rm.span = span;
        rm.c_pre = prefix - kv0;
        rm.i_rel = i - kv0;
        rm.dil = dil;
        kc.rel0 = static_cast<float>(kv0 - i);  // (j - i) of column 0, exact in fp32
        const int mode = ft.full(t) ? 0 : (dil == 1 ? 1 : 2);
        if (SOFTMAX) {
          float mx;
          if (mode == 0)
            mx = softmax_pass1<KIND, 0>(sr, kc, rm);
          else if (mode == 1)
            mx = softmax_pass1<KIND, 1>(sr, kc, rm);
          else
            mx = softmax_pass1<KIND, 2>(sr, kc, rm);
          trs(12);  // mod + mask done
          // P_w and O_w may only change once O_w += P_w V of the previous tile retired
          if (cnt > 0 && !bounded_wait(wc, bar(C::BAR_PFREE + w), (cnt - 1) & 1)) { ok = false; break; }
          ptx::tc_fence_after();
          const float m_new = fmaxf(m_run, mx);
          const bool need = m_new > m_run + 8.0f;
          // a row that has seen no key yet has a zero O row: no rescale
          const bool need_o = need && m_run != -INFINITY;
          float alpha = 1.0f;
          if (need) {
            alpha = ptx::ex2(m_run - m_new);
            l_run *= alpha;
            m_run = m_new;
          }
          if (t > U.tlo[w] && __any_sync(0xffffffffu, need_o)) rescale_rows<D>(tO, alpha);
          const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
          l_run += softmax_pass2<BF16>(sr, m_use, PSinkSmem{prow, rsw});
        } else {
          if (cnt > 0 && !bounded_wait(wc, bar(C::BAR_PFREE + w), (cnt - 1) & 1)) { ok = false; break; }
          const PSinkSmem sink{prow, rsw};
          if (mode == 0)
            pointwise_tile<KIND, 0, BF16>(sr, kc, rm, sink);
          else if (mode == 1)
            pointwise_tile<KIND, 1, BF16>(sr, kc, rm, sink);
          else
            pointwise_tile<KIND, 2, BF16>(sr, kc, rm, sink);
          trs(12);
        }
        ptx::tmem_wait_st();  // O rescale stores (rare)
        // generic-proxy P writes must be visible to the UMMA (async proxy)
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(C::BAR_PFULL + w));
        trs(13);  // P stored and signalled
      }
      if (!ok) break;

      // ---------------- epilogue: O * inv -> global ----------------
      if (!bounded_wait(wc, bar(C::BAR_OFULL + w), units_w & 1)) break;
      ptx::tc_fence_after();
      float inv;
      if (SOFTMAX)
        inv = (l_run > 0.f) ? 1.0f / l_run : 0.f;
      else if (KIND == KIND_RELU)
        inv = args.out_scale;
      else
        inv = pointwise_out_scale<BF16>(KIND);
      const bool row_ok = i < g.sq;
      const int64_t real_row = static_cast<int64_t>(i) * args.vdil + U.r_res;
      uint8_t *orow = reinterpret_cast<uint8_t *>(args.o) +
                      2 * (U.b * args.o_sb + static_cast<int64_t>(U.h) * args.o_sh +
                           real_row * args.o_ss);
      trs(14);  // O ready
      if (SOFTMAX && args.lse != nullptr && row_ok)
        store_lse(args, U.b, U.h, real_row, m_run, l_run);
      store_rows<D, BF16>(tO, inv, row_ok, orow);
      trs(15);  // O stored
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_OEMPTY + w));
      ++units_w;
    }
  }

  // ---- teardown ----
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == C::MMA_WARP) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && args.sched != nullptr) {
    // The last CTA to finish returns the scheduler to zero for the next launch;
    // every CTA has made its final fetch before it counts itself finished.
    __threadfence();
    if (atomicAdd(args.sched + 1, 1) == static_cast<int>(gridDim.x) - 1) {
      atomicExch(args.sched, 0);
      atomicExch(args.sched + 1, 0);
    }
  }
}

}  // namespace chia
