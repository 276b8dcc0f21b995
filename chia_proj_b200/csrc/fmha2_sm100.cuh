// fmha2_sm100.cuh -- head_dim 128 forward attention on CTA pairs (2-SM UMMA).
//
// A cluster of two CTAs on two SMs computes one work unit of 256 query rows:
// CTA rank r owns query tile r (128 rows). Every UMMA is a cta_group::2 MMA
// with M = 256 issued by the even CTA:
//   S = Q K^T   A = Q (each CTA its own 128 rows, smem), B = K tile of 128
//               keys split by keys: CTA r holds keys [64r, 64r+64)
//   O += P V    A = P (each CTA's TMEM), B = V tile split by feature columns:
//               CTA r holds columns [64r, 64r+64)
// so each SM reads a full A and half a B per MMA: 96 bytes/clock of shared
// memory at the tensor core's full rate (a single-SM 128x128 MMA needs 128),
// and each SM loads only half of every K/V tile.
//
// Per CTA, tensor memory (512 columns x 128 lanes):
//   cols [0,384)  three S/P buffers of 128 columns,  cols [384,512) O
// Tile t uses buffer t % 3. Its softmax output P (16-bit pairs) of the COLS
// keys of column part p overwrites columns [p COLS, p COLS + COLS/2) of that
// buffer, inside the S columns of the warpgroup that wrote it, and is read
// back by the TS-UMMA. With three buffers the MMA warp keeps S up to three
// tiles ahead of the softmax warpgroups:
//   per tile i:  once P(t_i) is ready, O += P(t_i) V(t_i), then S(t_{i+3})
// into the buffer P(t_i) just left (UMMAs of one thread run in order).
// K and V halves of a tile share one ring stage (one wait, one release).
// Q is double-buffered by unit, so the next unit's Q arrives while the
// current one runs. Once a unit's MMAs have retired, its Q buffer stages
// the unit's output: the softmax warps write O (16-bit, 128-byte swizzle)
// there, and the load thread stores it with TMA before it loads the Q of
// the unit two ahead into the same buffer.
//
// Warps per CTA: 4 NP softmax warps in NP warpgroups (NP = 2 for the softmax
// kinds, 4 for sigmoid and ReLU); warp w owns TMEM lanes (query rows)
// 32 (w % 4) .. +31 and key columns COLS (w / 4) .. +COLS-1 of every tile
// (COLS = 128 / NP), so each thread transforms 1/NP of a row. Softmax kinds
// combine the parts' row maxima through shared memory once per tile and the
// row sums once per unit; each warpgroup rescales and stores its own COLS
// columns of O. Warp 4 NP issues MMAs (the even CTA's lane 0; both CTAs'
// warp 4 NP allocate TMEM), warp 4 NP + 1 loads.
// Barriers that collect both CTAs live in the even CTA; the even CTA's
// commits are multicast to both. The (dynamic) unit index and its key-tile
// count are broadcast by the even CTA's load thread into both CTAs' unit
// rings; each CTA's load thread also hands the decoded unit to its softmax
// warps through a four-slot queue, so only the load thread decodes units.
#pragma once
#include "fmha_sm100.cuh"

namespace chia {

// Column parts per row (softmax warpgroups): four for sigmoid, whose
// per-score work (exponential, reciprocal seed, two Newton steps) is long
// enough that four warps per SM sub-partition hide its latencies better (3%
// in an A/B run on one GPU); two for ReLU (1.5% slower with four) and for the
// softmax kinds, which exchange row maxima between the parts every tile.
__host__ __device__ constexpr int fmha2_parts(int kind) {
  return kind == KIND_SIGMOID ? 4 : 2;
}

template <int D, int NP_ = 2>
struct Fmha2Config {
  static_assert(D == 128, "the 2-SM kernel is specialised for head_dim 128");
  static constexpr int BM = 128;  // query rows per CTA
  static constexpr int BN = 128;  // keys per tile
  // softmax warpgroups = column parts of a row: each thread owns COLS keys
  // (CH chunks of 32) of its row in every tile
  static constexpr int NP = NP_;
  static constexpr int COLS = BN / NP;
  static constexpr int CH = COLS / 32;
  static_assert(NP == 2 || NP == 4, "two or four column parts");
  // the row-maximum / row-sum exchange is written for two parts
  static constexpr bool EXCHANGE = NP == 2;
  static constexpr int Q_BYTES = BM * D * 2;          // 32 KB, two 128-byte chunks
  static constexpr int Q_CHUNK = BM * 128;            // 16 KB
  static constexpr int KH_ROWS = BN / 2;              // keys per CTA per K tile
  static constexpr int KH_CHUNK = KH_ROWS * 128;      // 8 KB
  static constexpr int HALF_BYTES = 16384;            // half a K or V tile
  static constexpr int STAGE_BYTES = 2 * HALF_BYTES;  // [K half | V half] of one tile
  static constexpr int NKV = 5;                       // ring stages (160 KB)
  static constexpr int NSBUF = 3;                     // S/P buffers in TMEM
  static constexpr int OFF_Q = 0;                  // two Q buffers, alternating by unit
  static constexpr int OFF_KV = OFF_Q + 2 * Q_BYTES;
  static constexpr int OFF_BAR = OFF_KV + NKV * STAGE_BYTES;
  // barriers (same offsets in both CTAs)
  // even CTA only: q_full[2], kv_full[NKV], p_full, o_empty, unit_empty[2], drain
  // both CTAs:     o_staged[2], kv_empty[NKV], s_full[NSBUF], o_full, unit_full[2]
  static constexpr int BAR_QFULL = 0;     // [2] Q of the unit using buffer b landed
  static constexpr int BAR_OSTAGED = 2;   // [2] O of the unit using buffer b is in it
  static constexpr int BAR_KVFULL = 4;
  static constexpr int BAR_KVEMPTY = BAR_KVFULL + NKV;
  static constexpr int BAR_SFULL = BAR_KVEMPTY + NKV;  // [NSBUF]
  // P ready, per S/P buffer: one CTA's softmax may run up to two tiles ahead
  // of the other's, so one barrier per buffer keeps the 8 arrivals of a phase
  // from mixing tiles.
  static constexpr int BAR_PFULL = BAR_SFULL + NSBUF;  // [NSBUF]
  // "PV(t) retired" is kv_empty[t % NKV] (the commit that frees tile t's
  // stage). A rescale at tile t waits for PV(t-1) while PV(t-3) is known to
  // have retired, so the wanted phase of that stage barrier is at most one
  // behind and its parity is unambiguous.
  static constexpr int BAR_OFULL = BAR_PFULL + NSBUF;
  static constexpr int BAR_OEMPTY = BAR_OFULL + 1;
  static constexpr int BAR_UFULL = BAR_OEMPTY + 1;     // [2]
  static constexpr int BAR_UEMPTY = BAR_UFULL + 2;     // [2]
  static constexpr int BAR_DRAIN = BAR_UEMPTY + 2;
  // exchange between the two softmax warps of one lane quadrant: [4 quad][2 slot]
  static constexpr int BAR_XCH = BAR_DRAIN + 1;
  // per-CTA unit queue from the load thread to the softmax warps: [4] full / free
  static constexpr int BAR_UQFULL = BAR_XCH + 8;
  static constexpr int BAR_UQFREE = BAR_UQFULL + 4;
  static constexpr int NUM_BARS = BAR_UQFREE + 4;
  // tmem base, abort flag, unit ring [2], key tiles of the ring's units [2]
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  // row-max / row-sum exchange between the two softmax warpgroups:
  // float [2 parity][2 column part][128 rows]
  static constexpr int OFF_XCH = OFF_MISC + 32;
  // unit queue: 4 UnitSlot entries
  static constexpr int OFF_UQ = OFF_XCH + 2 * 2 * 128 * 4;
  static constexpr int SMEM_BYTES = OFF_UQ + 4 * 64;
  // No slack for aligning the base: the dynamic shared memory of a kernel
  // without static shared memory starts 1024-byte aligned (checked at run
  // time), and the second Q buffer needs the room.
  static constexpr int SMEM_ALLOC = SMEM_BYTES;
  static constexpr int SOFTMAX_WARPS = 4 * NP;
  static constexpr int MMA_WARP = SOFTMAX_WARPS;
  static constexpr int LOAD_WARP = SOFTMAX_WARPS + 1;
  static constexpr int THREADS = 32 * (SOFTMAX_WARPS + 2);
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t TMEM_O = 384;
  static constexpr int UNIT_CONSUMERS = 2;  // of the ring: the MMA warp, the odd CTA's loader
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// One work unit as the load thread hands it to its CTA's softmax warps,
// decoded once (the unit index alone costs the warps a few thousand cycles
// of dependent integer arithmetic at every unit boundary).
struct UnitSlot {
  int32_t u;              // unit index (< 0: no more units)
  int32_t tiles;          // key tiles of the unit (0: no row of it sees a key)
  int32_t jlo;            // first key tile of the unit
  int32_t rev;            // tiles visited last to first
  int32_t r_res, h, b;    // residue class (dilation), query head, batch
  int32_t pad;
  int32_t m0;             // first query row of the unit
  int32_t tlo, thi;       // key tiles [tlo, thi) of this CTA's query tile
  FullTiles ft;           // key tiles this CTA's rows all see completely
  float hp;               // per-head parameter (ALiBi slope, temperature)
};
static_assert(sizeof(UnitSlot) == 64, "unit slot layout");

// Per-kind constants of the softmax / pointwise epilogue.
template <int KIND>
__device__ __forceinline__ EpiConsts make_epi_consts(const KernelArgs &a, float hp) {
  constexpr float LOG2E = 1.4426950408889634f;
  EpiConsts kc;
  kc.k_mul = a.score_scale * LOG2E;
  kc.k_cap = 0.f;
  kc.k_bias = 0.f;
  kc.rel0 = 0.f;
  if (KIND == KIND_SOFTMAX) kc.k_mul *= hp;
  if (KIND == KIND_SOFTCAP) {
    kc.k_mul = a.score_scale / a.softcap;
    kc.k_cap = a.softcap * LOG2E;
  }
  if (KIND == KIND_ALIBI) kc.k_bias = hp * LOG2E * static_cast<float>(a.vdil);
  if (KIND == KIND_SIGMOID) {
    kc.k_mul = -a.score_scale * LOG2E;
    kc.k_bias = -a.sig_bias * LOG2E;
  }
  if (KIND == KIND_RELU) kc.k_mul = a.score_scale;
  return kc;
}

// Key tiles of a unit are visited from the last to the first for ALiBi with a
// positive slope: the bias slope * (j - i) then starts at its largest, the
// running row maximum is set by the first tile, and later tiles never force
// an O rescale (visited forwards, it would grow by slope * 128 per tile).
// Every role of the kernel visits tiles in the same order.
template <int KIND>
__device__ __forceinline__ bool reverse_tiles(const KernelArgs &a, const UnitInfo &U) {
  return KIND == KIND_ALIBI && a.head_param[U.h] > 0.f;
}

// ---- masked tiles of the softmax kinds (64 columns per thread) ----
// A tile that is not wholly visible is classified per 32-column chunk,
// uniformly over the warp: a chunk every row of the warp sees completely
// takes the unmasked code, a chunk no row sees is skipped (P = 0, no
// exponentials), only the rest applies a per-column visibility bit. The
// warp's 32 rows are 32 consecutive queries, so on a causal or banded
// diagonal tile most chunks are one or the other.

// Visibility of columns col0 .. col0+31 (relative to RowMask's column 0)
// for this thread's row, one bit per column: the band [c_lo, c_lo + span]
// thinned to the row's dilation residue, or'ed with the always-visible
// prefix. dil_pat has a bit at every multiple of the dilation below 32.
__device__ __forceinline__ uint32_t visible_bits(const RowMask &rm, int col0, uint32_t dil_pat) {
  uint32_t w = 0u;
  const int64_t lo = static_cast<int64_t>(rm.c_lo) - col0;
  const int64_t hi = lo + rm.span;
  if (lo <= 31 && hi >= 0) {
    const int l = lo < 0 ? 0 : static_cast<int>(lo);
    const int h = hi > 31 ? 31 : static_cast<int>(hi);
    w = (0xFFFFFFFFu >> (31 - h)) & (0xFFFFFFFFu << l);
  }
  if (rm.dil > 1) {
    // visible: columns col0 + p, p = (i - key of column col0) mod dil (+ k dil)
    int p0 = (rm.i_rel - col0) % rm.dil;
    if (p0 < 0) p0 += rm.dil;
    w &= p0 < 32 ? dil_pat << p0 : 0u;
  }
  const int n = rm.c_pre - col0;
  const uint32_t pre = n <= 0 ? 0u : (n >= 32 ? 0xFFFFFFFFu : (1u << n) - 1u);
  return w | pre;
}

// Pass 1 of one chunk, in place: score -> log2-domain logit (columns whose
// bit in vis is clear -> -inf when MASK); returns the chunk maximum.
template <int KIND, bool MASK>
__device__ __forceinline__ float logit_chunk(uint32_t (&x)[32], int col0, const EpiConsts &k,
                                             uint32_t vis) {
  const uint64_t K2 = ptx::f2(k.k_mul, k.k_mul);
  const uint64_t CAP2 = ptx::f2(k.k_cap, k.k_cap);
  const uint64_t KB2 = ptx::f2(k.k_bias, k.k_bias);
  const uint64_t REL2 = ptx::f2(k.rel0 + static_cast<float>(col0), k.rel0 + static_cast<float>(col0 + 1));
  float mc = -INFINITY;
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    uint64_t x2 = ptx::mul2(ptx::f2(__uint_as_float(x[e]), __uint_as_float(x[e + 1])), K2);
    if (KIND == KIND_SOFTCAP) {
      float a, b;
      ptx::f2_split(x2, a, b);
      x2 = ptx::mul2(ptx::f2(ptx::tanh_fast(a), ptx::tanh_fast(b)), CAP2);
    } else if (KIND == KIND_ALIBI) {
      // bias = slope * (j - i): (j - i) is formed exactly before scaling
      const uint64_t rel = ptx::add2(REL2, ptx::f2(static_cast<float>(e), static_cast<float>(e)));
      x2 = ptx::fma2(KB2, rel, x2);
    }
    float a, b;
    ptx::f2_split(x2, a, b);
    if (MASK) {
      if (!((vis >> e) & 1u)) a = -INFINITY;
      if (!((vis >> (e + 1)) & 1u)) b = -INFINITY;
    }
    mc = ptx::max3(mc, a, b);
    x[e] = __float_as_uint(a);
    x[e + 1] = __float_as_uint(b);
  }
  return mc;
}

// Pass 1 on this thread's CH chunks: scores -> logits in place; returns the
// maximum. MASK_TILE: the tile is not wholly visible, so each chunk is
// classified first; bit c of `skip` is set for a chunk no row of the warp
// sees (its logits are left unwritten).
template <int KIND, int CH, bool MASK_TILE>
__device__ __forceinline__ float softmax_pass1_cols(uint32_t (&sr)[CH][32], const EpiConsts &k,
                                                    const RowMask &rm, uint32_t dil_pat,
                                                    uint32_t &skip) {
  float m = -INFINITY;
  skip = 0u;
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    if (MASK_TILE) {
      const uint32_t vis = visible_bits(rm, c * 32, dil_pat);
      if (__all_sync(0xffffffffu, vis == 0u)) {
        skip |= 1u << c;
        continue;
      }
      if (!__all_sync(0xffffffffu, vis == 0xFFFFFFFFu)) {
        m = fmaxf(m, logit_chunk<KIND, true>(sr[c], c * 32, k, vis));
        continue;
      }
    }
    m = fmaxf(m, logit_chunk<KIND, false>(sr[c], c * 32, k, 0u));
  }
  return m;
}

// Pass 2: P = 2^(x - m) of the chunks not in `skip`, 0 for the others,
// packed over the first CH * 16 of these columns; returns the row sum.
template <bool BF16, int CH>
__device__ __forceinline__ float softmax_pass2_cols(const uint32_t (&sr)[CH][32], float m,
                                                    uint32_t skip, uint32_t tP) {
  const uint64_t NM2 = ptx::f2(-m, -m);
  uint64_t acc[2] = {ptx::f2(0.f, 0.f), ptx::f2(0.f, 0.f)};
  uint32_t pk[CH * 16];
#pragma unroll
  for (int c = 0; c < CH; ++c) {
    if ((skip >> c) & 1u) {
#pragma unroll
      for (int e = 0; e < 16; ++e) pk[c * 16 + e] = 0u;
      continue;
    }
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      float a, b;
      ptx::f2_split(ptx::add2(ptx::f2(__uint_as_float(sr[c][e]), __uint_as_float(sr[c][e + 1])), NM2),
                    a, b);
      const float p0 = ptx::ex2(a), p1 = ptx::ex2(b);
      // one accumulator per chunk; a single chunk alternates two
      const int ai = CH == 2 ? c : (e >> 1) & 1;
      acc[ai] = ptx::add2(acc[ai], ptx::f2(p0, p1));
      pk[c * 16 + e / 2] = pack2<BF16>(p0, p1);
    }
  }
  if constexpr (CH == 2)
    ptx::tmem_st32(tP, pk);
  else
    ptx::tmem_st16(tP, pk);
  float s0, s1, s2, s3;
  ptx::f2_split(acc[0], s0, s1);
  ptx::f2_split(acc[1], s2, s3);
  return (s0 + s1) + (s2 + s3);
}

// Pointwise kinds on this thread's CH chunks of a TMEM S tile: P (CH * 32
// keys) goes back over the first CH * 16 columns.
template <int KIND, int MODE, bool BF16, int CH>
__device__ __forceinline__ void pointwise_tmem_cols(uint32_t tS, const EpiConsts &k,
                                                    const RowMask &rm) {
  if constexpr (CH == 2) {
    pointwise_tmem64<KIND, MODE, BF16>(tS, k, rm);
  } else {
    uint32_t s0[32], pk[32];
    ptx::tmem_ld32(tS, s0);
    ptx::tmem_wait_ld();
    ptx::reg_fence(s0);
    pointwise_chunk<KIND, MODE, BF16>(s0, 0, k, rm, pk, 0);
    uint32_t p16[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) p16[e] = pk[e];
    ptx::tmem_st16(tS, p16);
  }
}

// P = 0 over the first CH * 16 columns at tS.
template <int CH>
__device__ __forceinline__ void tmem_zero_cols(uint32_t tS) {
  uint32_t z[CH * 16];
#pragma unroll
  for (int e = 0; e < CH * 16; ++e) z[e] = 0u;
  if constexpr (CH == 2)
    ptx::tmem_st32(tS, z);
  else
    ptx::tmem_st16(tS, z);
}

// Bounded wait on a local barrier that may receive arrivals from the other CTA.
__device__ __forceinline__ bool bounded_wait_cl(const WaitCtx &c, uint32_t bar, uint32_t parity,
                                                bool honour_abort = true) {
  if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  const uint64_t limit = honour_abort ? c.timeout_ns : c.drain_ns;
  // Each try may suspend for up to `hint` ns. With the default limit the
  // clock is read every 64 tries; a short limit (tests) shortens the
  // suspension and reads the clock after every try.
  const bool short_limit = limit < (64ull << 20);
  const uint32_t hint = short_limit ? static_cast<uint32_t>(limit >> 6) + 32u : (1u << 20);
  const uint32_t check_mask = short_limit ? 0u : 63u;
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait_cluster(bar, parity, hint)) return true;
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

// MASKED = false: every key tile of every unit is fully visible (the host
// checks: no window, block or dilation and S_kv a multiple of 128), so the
// element-wise mask code is left out of the kernel. SEG: packed sequences.
template <int D, bool BF16, int KIND, bool MASKED, bool SEG>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Fmha2Config<D, fmha2_parts(KIND)>::THREADS, 1)
    fmha2_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                     const __grid_constant__ CUtensorMap tm_kh,
                     const __grid_constant__ CUtensorMap tm_vh,
                     const __grid_constant__ CUtensorMap tm_o, const KernelArgs args) {
  using C = Fmha2Config<D, fmha2_parts(KIND)>;
  constexpr int BM = C::BM, BN = C::BN, NKV = C::NKV;
  constexpr bool SOFTMAX = (KIND == KIND_SOFTMAX || KIND == KIND_SOFTCAP || KIND == KIND_ALIBI);

  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t sbase = ptx::smem_u32(smem);
  // The 128-byte-swizzled tiles need a 1024-byte aligned base. Both CTAs of a
  // pair share the layout, so both leave here together, before any cluster
  // barrier; the status word reports it.
  if (sbase & 1023u) {
    if (threadIdx.x == 0 && args.status) atomicOr(args.status, 4 /* CHIA_ERR_LAUNCH */);
    return;
  }
  auto bar = [&](int idx) -> uint32_t { return sbase + C::OFF_BAR + idx * 8; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 4);
  volatile int *unit_ring = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 8);
  volatile int *unit_tiles = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 16);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const uint32_t pair = ptx::cluster_id_x(), npairs = ptx::cluster_count_x();
  const MaskGeom &g = args.mask;
  // address of barrier idx in the even CTA (shared::cluster window)
  auto lbar = [&](int idx) -> uint32_t { return ptx::mapa(bar(idx), 0); };

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(C::BAR_QFULL + b), 2);                   // both CTAs' Q loads
      ptx::mbar_init(bar(C::BAR_OSTAGED + b), C::SOFTMAX_WARPS);  // this CTA's softmax warps
    }
    for (int s = 0; s < NKV; ++s) {
      ptx::mbar_init(bar(C::BAR_KVFULL + s), 2);
      ptx::mbar_init(bar(C::BAR_KVEMPTY + s), 1);
    }
    for (int b = 0; b < C::NSBUF; ++b) {
      ptx::mbar_init(bar(C::BAR_SFULL + b), 1);
      ptx::mbar_init(bar(C::BAR_PFULL + b), 2 * C::SOFTMAX_WARPS);  // both CTAs
    }
    ptx::mbar_init(bar(C::BAR_OFULL), 1);
    ptx::mbar_init(bar(C::BAR_OEMPTY), 2 * C::SOFTMAX_WARPS);  // both CTAs
    for (int s = 0; s < 2; ++s) {
      ptx::mbar_init(bar(C::BAR_UFULL + s), 1);
      ptx::mbar_init(bar(C::BAR_UEMPTY + s), C::UNIT_CONSUMERS);
    }
    ptx::mbar_init(bar(C::BAR_DRAIN), 1);
    for (int x = 0; x < 4; ++x) {
      ptx::mbar_init(bar(C::BAR_UQFULL + x), 1);
      ptx::mbar_init(bar(C::BAR_UQFREE + x), C::SOFTMAX_WARPS);
    }
    for (int x = 0; x < 8; ++x) ptx::mbar_init(bar(C::BAR_XCH + x), 2);  // one arrive per warp
    *abort_flag = 0;
    *reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 24) = -1;
    ptx::fence_barrier_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == C::LOAD_WARP && lane == 0) {
    ptx::tma_prefetch_desc(&tm_q);
    ptx::tma_prefetch_desc(&tm_kh);
    ptx::tma_prefetch_desc(&tm_vh);
    ptx::tma_prefetch_desc(&tm_o);
  }
  if (warp == C::MMA_WARP) {
    ptx::tmem_alloc_2sm(ptx::smem_u32(tmem_slot), C::TMEM_COLS);
    ptx::tmem_relinquish_2sm();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // barriers of both CTAs initialised before any remote access
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const WaitCtx wc{abort_flag, args.status, args.timeout_ns, args.drain_ns};
  // unit k of this CTA's last Q-barrier contribution (its Q copy, or the bare
  // arrival of a keyless unit); -1 = none. The odd CTA hands its value to the
  // even CTA, which waits for those phases before either CTA exits.
  int last_q = -1;
  volatile int *peer_last_q = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 24);

  if (warp == C::LOAD_WARP && lane == 0) {
    // ========== unit scheduler (even CTA) + loads of this CTA's halves ==========
    Tracer tr(3);
    uint32_t n = 0;  // ring stages filled (one per tile)
    int64_t last_item[NKV];
    for (int s = 0; s < NKV; ++s) last_item[s] = -1;
    // one tile: this CTA's K half (keys [64 rank, 64 rank + 64), two 64-column
    // chunks) and V half (columns [64 rank, 64 rank + 64) of all 128 keys)
    auto load_tile = [&](int64_t t, const UnitInfo &U) -> bool {
      const int s = n % NKV;
      if (!bounded_wait(wc, bar(C::BAR_KVEMPTY + s), ((n / NKV) & 1) ^ 1)) return false;
      const uint32_t full = lbar(C::BAR_KVFULL + s);
      ptx::mbar_arrive_expect_tx_remote(full, C::STAGE_BYTES);
      const uint32_t dst = sbase + C::OFF_KV + s * C::STAGE_BYTES;
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        ptx::tma_load_5d_2sm(dst + c * C::KH_CHUNK, &tm_kh, full, c * 64,
                             static_cast<int>(t * BN) + C::KH_ROWS * static_cast<int>(rank),
                             U.r_res, U.h / args.group, U.b);
      ptx::tma_load_5d_2sm(dst + C::HALF_BYTES, &tm_vh, full, 64 * static_cast<int>(rank),
                           static_cast<int>(t * BN), U.r_res, U.h / args.group, U.b);
      tr(30);
      last_item[s] = n;
      ++n;
      return true;
    };
    // O of the unit that used Q buffer b: once this CTA's softmax warps have
    // staged it there, store this CTA's 128 rows with TMA (rows past the
    // sequence end are not written) and wait until the store has read the
    // buffer. A unit whose rows see no key has its zeros written by the
    // softmax warps directly and stages nothing, so the staging barrier's
    // phases count the other units only (oph).
    UnitInfo uq[2];
    uint32_t oph[2] = {0, 0};
    auto store_o = [&](int b) -> bool {
      const UnitInfo &V = uq[b];
      if (V.jhi == V.jlo) return true;
      if (!bounded_wait(wc, bar(C::BAR_OSTAGED + b), oph[b])) return false;
      oph[b] ^= 1u;
#pragma unroll
      for (int c = 0; c < D / 64; ++c)
        ptx::tma_store_5d(&tm_o, sbase + C::OFF_Q + b * C::Q_BYTES + c * C::Q_CHUNK, c * 64,
                          static_cast<int>(V.m0) + BM * static_cast<int>(rank), V.r_res, V.h, V.b);
      ptx::bulk_commit_group();
      ptx::bulk_wait_read_all();
      return true;
    };
    int k_end = 0;  // units taken
    bool clean = false;
    for (int k = 0;; ++k) {
      k_end = k;
      const int slot = k & 1;
      int u;
      if (leader) {
        if (!bounded_wait_cl(wc, bar(C::BAR_UEMPTY + slot), ((k >> 1) & 1) ^ 1)) break;
        u = args.sched ? atomicAdd(args.sched, 1)
                       : static_cast<int>(pair) + k * static_cast<int>(npairs);
        if (u >= args.n_units || u < 0) u = -1;
      } else {
        if (!bounded_wait_cl(wc, bar(C::BAR_UFULL + slot), (k >> 1) & 1)) break;
        u = unit_ring[slot];
        ptx::mbar_arrive_cluster(lbar(C::BAR_UEMPTY + slot));
      }
      UnitInfo U;
      int T = 0;
      bool rev = false;
      if (u >= 0) {
        decode_unit<BM, BN, SEG>(u, args, U);
        T = static_cast<int>(U.jhi - U.jlo);
        rev = reverse_tiles<KIND>(args, U);
      }
      if (leader) {  // publish the unit and its key-tile count to both CTAs
        unit_ring[slot] = u;
        unit_tiles[slot] = T;
        const uint32_t peer_misc = ptx::mapa(sbase + C::OFF_MISC, 1);
        ptx::st_shared_cluster_u32(peer_misc + 8 + 4 * slot, static_cast<uint32_t>(u));
        ptx::st_shared_cluster_u32(peer_misc + 16 + 4 * slot, static_cast<uint32_t>(T));
        ptx::mbar_arrive(bar(C::BAR_UFULL + slot));
        ptx::mbar_arrive_cluster(ptx::mapa(bar(C::BAR_UFULL + slot), 1));
      }
      // hand the unit, decoded, to this CTA's softmax warps
      const int qs = k & 3;
      if (k >= 4 && !bounded_wait(wc, bar(C::BAR_UQFREE + qs), ((k >> 2) & 1) ^ 1)) break;
      {
        UnitSlot *e = reinterpret_cast<UnitSlot *>(smem + C::OFF_UQ) + qs;
        e->u = u;
        e->tiles = T;
        if (u >= 0) {
          const int64_t r0 = U.m0 + BM * static_cast<int64_t>(rank);
          e->jlo = static_cast<int32_t>(U.jlo);
          e->rev = rev ? 1 : 0;
          e->r_res = U.r_res;
          e->h = U.h;
          e->b = U.b;
          e->m0 = static_cast<int32_t>(U.m0);
          e->tlo = static_cast<int32_t>(U.tlo[rank]);
          e->thi = static_cast<int32_t>(U.thi[rank]);
          e->ft = full_tiles<SEG>(g, r0, r0 + BM - 1, BN);
          e->hp = args.head_param != nullptr ? args.head_param[U.h] : 1.0f;
        }
      }
      ptx::mbar_arrive(bar(C::BAR_UQFULL + qs));
      if (u < 0) {
        clean = true;
        break;
      }
      // Q buffer qb held unit k-2, whose output is staged there: store it first
      const int qb = k & 1;
      if (k >= 2 && !store_o(qb)) break;
      uq[qb] = U;
      // this CTA's query tile (zero-filled by TMA when past the sequence end);
      // a unit without key tiles only completes the barrier phase
      const uint32_t qfull = lbar(C::BAR_QFULL + qb);
      last_q = k;
      if (U.jhi > U.jlo) {
        ptx::mbar_arrive_expect_tx_remote(qfull, C::Q_BYTES);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          ptx::tma_load_5d_2sm(sbase + C::OFF_Q + qb * C::Q_BYTES + c * C::Q_CHUNK, &tm_q, qfull,
                               c * 64, static_cast<int>(U.m0) + BM * static_cast<int>(rank),
                               U.r_res, U.h, U.b);
      } else {
        ptx::mbar_arrive_remote(qfull);
      }
      bool ok = true;
      for (int64_t k2 = 0; ok && k2 < T; ++k2)
        ok = load_tile(rev ? U.jhi - 1 - k2 : U.jlo + k2, U);
      if (!ok) break;
    }
    // outputs of the last two units
    if (clean)
      for (int j = k_end >= 2 ? k_end - 2 : 0; j < k_end; ++j)
        if (!store_o(j & 1)) break;
    ptx::bulk_wait_all();
    // Drain: this CTA's copies have landed once the even CTA released their
    // slots; on an abort the bounded waits below outlast any copy in flight.
    for (int s = 0; s < NKV; ++s)
      if (last_item[s] >= 0)
        bounded_wait(wc, bar(C::BAR_KVEMPTY + s), ((last_item[s] / NKV) & 1), false);
    if (!leader) ptx::st_shared_cluster_u32(ptx::mapa(sbase + C::OFF_MISC + 24, 0),
                                            static_cast<uint32_t>(last_q));
  } else if (warp == C::MMA_WARP && leader) {
    // =========================== 2-SM UMMA issuer ===========================
    // The whole warp runs this loop in lockstep; elect.sync inside the
    // tcgen05 wrappers picks the issuing lane.
    constexpr uint32_t IDESC_QK = ptx::make_idesc_f16(2 * BM, BN, BF16, false, false);
    constexpr uint32_t IDESC_PV = ptx::make_idesc_f16(2 * BM, D, BF16, false, true);
    const uint32_t q_s = sbase + C::OFF_Q, kv_s = sbase + C::OFF_KV;
    const uint64_t dq0 = ptx::make_sdesc_sw128(q_s, 16, 1024);
    uint64_t dq = dq0;  // Q buffer of the current unit
    const uint64_t dk = ptx::make_sdesc_sw128(kv_s, 16, 1024);
    const uint64_t dv = ptx::make_sdesc_sw128(kv_s + C::HALF_BYTES, C::HALF_BYTES, 1024);
    constexpr uint16_t BOTH = 0x3;
    auto issue_s = [&](uint32_t buf, int stage) {
      const uint32_t d_tmem = tmem_base + buf * 128;
      const uint64_t b0 = dk + ((stage * C::STAGE_BYTES) >> 4);
      static_assert(D / 16 == 8, "eight K-steps per S tile");
      uint64_t ad[8], bd[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        ad[kk] = dq + (((kk >> 2) * C::Q_CHUNK + (kk & 3) * 32) >> 4);
        bd[kk] = b0 + (((kk >> 2) * C::KH_CHUNK + (kk & 3) * 32) >> 4);
      }
      ptx::umma_ss_2sm_x8_warp(d_tmem, ad, bd, IDESC_QK, 0u);
    };
    auto issue_pv = [&](uint32_t buf, int stage, bool first) {
      const uint32_t d_tmem = tmem_base + C::TMEM_O;
      const uint32_t p_tmem = tmem_base + buf * 128;
      const uint64_t b0 = dv + ((stage * C::STAGE_BYTES) >> 4);
      static_assert(BN / 16 == 8, "eight K-steps per PV tile");
      uint32_t at[8];
      uint64_t bd[8];
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {  // P of keys 16kk.. inside their part's S columns
        at[kk] = p_tmem + (kk * 16 / C::COLS) * C::COLS + (kk * 16 % C::COLS) / 2;
        bd[kk] = b0 + ((kk * 2048) >> 4);
      }
      ptx::umma_ts_2sm_x8_warp(d_tmem, at, bd, IDESC_PV, first ? 0u : 1u);
    };
    Tracer trc(2);
    auto tr = [&](int tag) { if (lane == 0) trc(tag); };
    uint32_t tcnt = 0;     // tiles issued = ring stage index = S/P buffer sequence
    uint32_t units = 0;
    bool ok = true;
    // every lane waits; the warp proceeds only if all of them saw the phase
    auto wait = [&](uint32_t b, uint32_t parity) {
      return __all_sync(0xffffffffu, bounded_wait(wc, b, parity));
    };
    auto stage_wait = [&](uint32_t t) { return wait(bar(C::BAR_KVFULL + t % NKV), (t / NKV) & 1); };
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      if (!__all_sync(0xffffffffu, bounded_wait_cl(wc, bar(C::BAR_UFULL + slot), (k >> 1) & 1)))
        break;
      const int u = __shfl_sync(0xffffffffu, unit_ring[slot], 0);
      const int T = __shfl_sync(0xffffffffu, unit_tiles[slot], 0);  // decoded by the loader
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_UEMPTY + slot));
      if (u < 0) break;
      if (T == 0) continue;  // no key tiles: the softmax warps write zeros
      if (!wait(bar(C::BAR_QFULL + (k & 1)), (k >> 1) & 1)) break;
      dq = dq0 + (((k & 1) * C::Q_BYTES) >> 4);
      // S of up to NSBUF tiles ahead
      const int pre = T < C::NSBUF ? T : C::NSBUF;
      for (int i = 0; i < pre; ++i) {
        const uint32_t t = tcnt + i;
        if (!stage_wait(t)) { ok = false; break; }
        ptx::tc_fence_after();
        issue_s(t % C::NSBUF, t % NKV);
        ptx::umma_commit_2sm_warp(bar(C::BAR_SFULL + t % C::NSBUF), BOTH);
        tr(20);
      }
      if (!ok) break;
      for (int i = 0; i < T; ++i) {
        const uint32_t t = tcnt + i, b = t % C::NSBUF;
        if (!wait(bar(C::BAR_PFULL + b), (t / C::NSBUF) & 1)) { ok = false; break; }
        tr(21);
        if (i == 0 && units > 0 && !wait(bar(C::BAR_OEMPTY), (units - 1) & 1)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        issue_pv(b, t % NKV, i == 0);
        // K and V halves of tile t are free, and O holds PV(t)
        ptx::umma_commit_2sm_warp(bar(C::BAR_KVEMPTY + t % NKV), BOTH);
        if (i == T - 1) ptx::umma_commit_2sm_warp(bar(C::BAR_OFULL), BOTH);
        tr(22);
        if (i + C::NSBUF < T) {  // S three tiles ahead, into the buffer P(t) just left
          const uint32_t t3 = t + C::NSBUF;
          if (!stage_wait(t3)) { ok = false; break; }
          ptx::tc_fence_after();
          issue_s(b, t3 % NKV);
          ptx::umma_commit_2sm_warp(bar(C::BAR_SFULL + b), BOTH);
          tr(20);
        }
      }
      if (!ok) break;
      tcnt += T;
      ++units;
    }
    ptx::umma_commit_2sm_warp(bar(C::BAR_DRAIN), 0x1);  // every 2-SM UMMA of this warp retired
    bounded_wait(wc, bar(C::BAR_DRAIN), 0, false);
    __syncwarp();
  } else if (warp < C::SOFTMAX_WARPS) {
    // ======================= softmax / epilogue =======================
    constexpr int COLS = C::COLS, CH = C::CH;
    const int quad = warp & 3, part = warp >> 2;
    const int row = quad * 32 + lane;  // TMEM lane = query row in this CTA's tile
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tO = tmem_base + lane_off + C::TMEM_O + part * COLS;
    const int prefix = static_cast<int>(g.prefix);
    const int dil = static_cast<int>(g.dil);
    uint32_t dil_pat = 0u;  // a bit at every multiple of the dilation below 32
    for (int p = 0; p < 32; p += dil) dil_pat |= 1u << p;
    const uint32_t pfull0 = lbar(C::BAR_PFULL), oempty = lbar(C::BAR_OEMPTY);
    float *xch = reinterpret_cast<float *>(smem + C::OFF_XCH);
    uint32_t xcnt = 0;
    // Exchange of one float per row with the warp that owns the other column
    // part of these rows (softmax kinds, two parts): publish() hands v over
    // without waiting, collect() returns the other warp's value of the same
    // exchange. Both warps publish and collect in the same order. Two slots
    // per quadrant keep a fast warp from overwriting a value the other has
    // not read: a warp publishes exchange n+2 only after collecting n+1,
    // which the other publishes only after collecting n. collect() waits
    // with a bound: false means the kernel is aborting.
    static_assert(!SOFTMAX || C::EXCHANGE, "softmax kinds run with two column parts");
    auto publish = [&](float v) {
      const uint32_t slot = xcnt & 1;
      xch[slot * 256 + (part & 1) * 128 + row] = v;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_XCH + quad * 2 + slot));
    };
    auto collect = [&](float &other) -> bool {
      const uint32_t slot = xcnt & 1, phase = (xcnt >> 1) & 1;
      ++xcnt;
      if (!bounded_wait(wc, bar(C::BAR_XCH + quad * 2 + slot), phase)) return false;
      other = xch[slot * 256 + ((part & 1) ^ 1) * 128 + row];
      return true;
    };
    Tracer tr(warp == 0 ? 0 : 1);
    const bool tracing = (warp == 0 || warp == 4) && lane == 0;
    auto trs = [&](int tag) { if (tracing) tr(tag); };
    uint32_t cnt = 0;  // tiles seen (all tiles of every unit)
    uint32_t units = 0;
    const int w = static_cast<int>(rank);  // this CTA's query tile in every unit
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      // the unit, as decoded by this CTA's load thread
      const int qs = k & 3;
      if (!bounded_wait(wc, bar(C::BAR_UQFULL + qs), (k >> 2) & 1)) break;
      const UnitSlot U = reinterpret_cast<const UnitSlot *>(smem + C::OFF_UQ)[qs];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_UQFREE + qs));
      if (U.u < 0) break;
      const int i = U.m0 + w * BM + row;
      if (U.tiles == 0) {
        // No row of the unit sees a key: its output is zero, written here
        // (nothing is staged for the load thread to store).
        if (i < g.sq) {
          const int64_t real_row = static_cast<int64_t>(i) * args.vdil + U.r_res;
          if (SOFTMAX && args.lse != nullptr && part == 0)
            store_lse(args, U.b, U.h, real_row, -INFINITY, 0.f);
          uint8_t *orow = reinterpret_cast<uint8_t *>(args.o) +
                          2 * (U.b * args.o_sb + static_cast<int64_t>(U.h) * args.o_sh +
                               real_row * args.o_ss + part * COLS);
#pragma unroll
          for (int v4 = 0; v4 < COLS / 8; ++v4) ptx::st_global_v4(orow + v4 * 16, 0u, 0u, 0u, 0u);
        }
        continue;
      }
      int64_t blo64, bhi64;
      row_band<SEG>(g, i, blo64, bhi64);
      const bool band_empty = bhi64 < blo64;
      const int blo = band_empty ? (1 << 30) : static_cast<int>(blo64);
      const uint32_t span = band_empty ? 0u : static_cast<uint32_t>(bhi64 - blo64);
      EpiConsts kc = make_epi_consts<KIND>(args, U.hp);
      const FullTiles ft = U.ft;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true, first_mine = true;
      for (int k2 = 0; k2 < U.tiles; ++k2, ++cnt) {
        const int t = U.rev ? U.jlo + U.tiles - 1 - k2 : U.jlo + k2;
        const uint32_t buf = cnt % C::NSBUF;
        const uint32_t tS = tmem_base + lane_off + buf * 128 + part * COLS;
        if (!bounded_wait(wc, bar(C::BAR_SFULL + buf), (cnt / C::NSBUF) & 1)) {
          ok = false;
          break;
        }
        trs(10);
        ptx::tc_fence_after();
        if (t >= U.tlo && t < U.thi) {  // this CTA's query tile sees key tile t
          uint32_t sr[CH][32];
          if (SOFTMAX) {
#pragma unroll
            for (int c = 0; c < CH; ++c) ptx::tmem_ld32(tS + 32 * c, sr[c]);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < CH; ++c) ptx::reg_fence(sr[c]);
          }
          trs(11);
          const int kv0 = static_cast<int>(t) * BN + part * COLS;  // key of column 0 of sr
          RowMask rm;
          rm.c_lo = blo - kv0;
          rm.span = span;
          rm.c_pre = prefix - kv0;
          rm.i_rel = i - kv0;
          rm.dil = dil;
          kc.rel0 = static_cast<float>(kv0 - i);
          const int mode = (!MASKED || ft.full(t)) ? 0 : (dil == 1 ? 1 : 2);
          if (SOFTMAX) {
            uint32_t skip = 0u;  // chunks of a masked tile no row of this warp sees
            const float mx = mode == 0 ? softmax_pass1_cols<KIND, CH, false>(sr, kc, rm, dil_pat, skip)
                                       : softmax_pass1_cols<KIND, CH, true>(sr, kc, rm, dil_pat, skip);
            // The row maximum of the whole tile needs the other parts'. After
            // the first tile, P is computed optimistically against the running
            // maximum, which stays exact unless the maximum grew by more than
            // 2^8 (lazy rescale); the other parts' values are collected only
            // afterwards, when they have long been published.
            publish(mx);
            float lsum = 0.f;
            if (!first_mine)
              lsum = softmax_pass2_cols<BF16, CH>(sr, m_run == -INFINITY ? 0.f : m_run, skip, tS);
            float mx_other;
            if (!collect(mx_other)) { ok = false; break; }
            const float m_new = fmaxf(m_run, fmaxf(mx, mx_other));  // row maximum, whole tile
            const bool need = m_new > m_run + 8.0f;
            if (first_mine || __any_sync(0xffffffffu, need)) {
              // A row that has seen no key yet (m_run = -inf) has a zero O row
              // and l_run = 0: it takes the new maximum without a rescale of O.
              const bool need_o = need && m_run != -INFINITY;
              float alpha = 1.0f;
              if (need) {
                alpha = ptx::ex2(m_run - m_new);
                l_run *= alpha;
                m_run = m_new;
              }
              if (!first_mine) {
                ptx::tmem_wait_st();  // the optimistic P is written before it is replaced
                if (__any_sync(0xffffffffu, need_o)) {
                  // O holds every earlier PV once PV(t-1) retired (it frees that stage)
                  const uint32_t prev = cnt - 1;
                  if (!bounded_wait(wc, bar(C::BAR_KVEMPTY + prev % NKV), (prev / NKV) & 1)) {
                    ok = false;
                    break;
                  }
                  ptx::tc_fence_after();
                  rescale_rows<COLS>(tO, alpha);
                }
              }
              // (re)compute P against the new maximum; P is not yet signalled
              lsum = softmax_pass2_cols<BF16, CH>(sr, m_run == -INFINITY ? 0.f : m_run, skip, tS);
            }
            l_run += lsum;
          } else {
            if (mode == 0)
              pointwise_tmem_cols<KIND, 0, BF16, CH>(tS, kc, rm);
            else if (mode == 1)
              pointwise_tmem_cols<KIND, 1, BF16, CH>(tS, kc, rm);
            else
              pointwise_tmem_cols<KIND, 2, BF16, CH>(tS, kc, rm);
          }
          first_mine = false;
          trs(12);
        } else {
          // the pair computes this tile for the other query tile only: P = 0 here
          tmem_zero_cols<CH>(tS);
        }
        ptx::tmem_wait_st();
        trs(16);  // P stores retired
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader)
            ptx::mbar_arrive(bar(C::BAR_PFULL + buf));
          else
            ptx::mbar_arrive_remote(pfull0 + 8 * buf);
        }
        trs(13);
      }
      if (!ok) break;
      // ---------------- epilogue: O * inv -> global ----------------
      float inv;
      if (SOFTMAX) {
        float l_other;
        publish(l_run);
        if (!collect(l_other)) break;
        // in part order, so both parts hold the same bits
        const float l_tot = part == 0 ? l_run + l_other : l_other + l_run;
        inv = (l_tot > 0.f) ? 1.0f / l_tot : 0.f;
        // every part holds the same running maximum (they agree on every tile's)
        if (args.lse != nullptr && part == 0 && i < g.sq)
          store_lse(args, U.b, U.h, static_cast<int64_t>(i) * args.vdil + U.r_res, m_run, l_tot);
      } else if (KIND == KIND_RELU) {
        inv = args.out_scale;
      } else {
        inv = pointwise_out_scale<BF16>(KIND);
      }
      if (!bounded_wait(wc, bar(C::BAR_OFULL), units & 1)) break;  // units with key tiles
      ptx::tc_fence_after();
      trs(14);
      uint32_t o[CH][32];
#pragma unroll
      for (int c = 0; c < CH; ++c) ptx::tmem_ld32(tO + 32 * c, o[c]);
      ptx::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < CH; ++c) ptx::reg_fence(o[c]);
      // O is in registers: the MMA may start the next unit's PV
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_remote(oempty);
      // stage this row's COLS columns (16-bit) in the unit's Q buffer (column
      // chunk part * COLS / 64, 16-byte units from (part * COLS % 64) / 8), in
      // the 128-byte swizzle of the output tensor map
      uint32_t pk[CH * 16];
#pragma unroll
      for (int c = 0; c < CH; ++c)
#pragma unroll
        for (int e = 0; e < 16; ++e)
          pk[c * 16 + e] = pack2<BF16>(__uint_as_float(o[c][2 * e]) * inv,
                                       __uint_as_float(o[c][2 * e + 1]) * inv);
      const uint32_t qrow = sbase + C::OFF_Q + slot * C::Q_BYTES +
                            (part * COLS / 64) * C::Q_CHUNK + row * 128;
      const int u0 = (part * COLS % 64) / 8;
#pragma unroll
      for (int u = 0; u < COLS / 8; ++u)
        ptx::st_shared_v4(qrow + (((u0 + u) ^ (row & 7)) << 4), pk[4 * u], pk[4 * u + 1],
                          pk[4 * u + 2], pk[4 * u + 3]);
      ptx::fence_proxy_async_smem();  // visible to the TMA store
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_OSTAGED + slot));
      trs(15);
      ++units;
    }
  }

  // ---- teardown: both CTAs finish before TMEM is freed and before either exits ----
  __syncwarp();
  ptx::tc_fence_before();
  ptx::cluster_sync();
  // The Q copies of both CTAs complete on the even CTA's q_full barriers.
  // Unless a wait was abandoned (abort), the MMA warp has already waited for
  // every phase and the waits below return at once. After an abort they
  // make sure that no Q copy is still landing when the CTAs exit: the last
  // phase of each Q buffer either CTA contributed to. A phase whose other
  // half never came (one CTA stopped first) runs into the drain limit, long
  // after the one copy of it landed.
  if (leader && warp == C::LOAD_WARP && lane == 0) {
    const int kq = last_q > *peer_last_q ? last_q : *peer_last_q;
    for (int j = kq - 1; j <= kq; ++j)
      if (j >= 0) bounded_wait(wc, bar(C::BAR_QFULL + (j & 1)), (j >> 1) & 1, false);
  }
  __syncwarp();
  ptx::cluster_sync();
  if (warp == C::MMA_WARP) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_2sm(tmem_base, C::TMEM_COLS);
  }
  if (threadIdx.x == 0 && leader && args.sched != nullptr) {
    __threadfence();
    if (atomicAdd(args.sched + 1, 1) == static_cast<int>(npairs) - 1) {
      atomicExch(args.sched, 0);
      atomicExch(args.sched + 1, 0);
    }
  }
}

}  // namespace chia
