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
//   cols [  0,128)  S0 = Q0 K^T   (P0 is written back over its first BN/2 columns)
//   cols [128,256)  S1 = Q1 K^T   (P1 likewise)
//   cols [256,256+D) O0,  cols [384,384+D) O1   (fp32 output accumulators)
//
// Per key tile j the MMA warp issues S0(j), S1(j) (SS-UMMA, Q and K both
// K-major in 128-byte-swizzled smem), and once softmax warpgroup w has written
// P_w(j) into TMEM, O_w += P_w(j) V(j) (TS-UMMA: A = P from TMEM, B = V
// MN-major in smem) followed immediately by S_w(j+1). UMMAs of one thread
// execute in issue order, so the commit that signals "S_w(j+1) ready" also
// proves that O_w has absorbed P_w(j): the softmax warpgroup may then rescale
// O_w in TMEM without another barrier.
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
  uint64_t timeout_ns;
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
  static constexpr int NS = (D == 128) ? 2 : 4;  // K ring and V ring depth
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + NQ * Q_TILE_BYTES;
  static constexpr int OFF_V = OFF_K + NS * KV_TILE_BYTES;
  static constexpr int OFF_BAR = OFF_V + NS * KV_TILE_BYTES;
  // barriers: q q_empty | k_full[NS] k_empty[NS] v_full[NS] v_empty[NS] |
  //           s_full[2] p_full[2] o_full[2] o_empty[2] | unit_full[2] unit_empty[2] | drain
  static constexpr int BAR_Q = 0;
  static constexpr int BAR_QEMPTY = 1;
  static constexpr int BAR_KFULL = 2;
  static constexpr int BAR_KEMPTY = BAR_KFULL + NS;
  static constexpr int BAR_VFULL = BAR_KEMPTY + NS;
  static constexpr int BAR_VEMPTY = BAR_VFULL + NS;
  static constexpr int BAR_SFULL = BAR_VEMPTY + NS;
  static constexpr int BAR_PFULL = BAR_SFULL + NQ;
  static constexpr int BAR_OFULL = BAR_PFULL + NQ;
  static constexpr int BAR_OEMPTY = BAR_OFULL + NQ;
  static constexpr int BAR_UFULL = BAR_OEMPTY + NQ;
  static constexpr int BAR_UEMPTY = BAR_UFULL + 2;
  static constexpr int BAR_DRAIN = BAR_UEMPTY + 2;
  static constexpr int NUM_BARS = BAR_DRAIN + 1;
  // misc: [0] TMEM base, [1] abort flag, [2..3] unit ring
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  static constexpr int SMEM_ALLOC = SMEM_BYTES + 1024;  // slack for 1024-byte alignment
  // 12 warps: warpgroups 0 and 1 = softmax (one query tile each), warpgroup 2
  // = MMA warp, load warp and two idle warps. setmaxnreg moves registers from
  // warpgroup 2 to the softmax warpgroups: 2*128*REG_SOFTMAX + 128*REG_OTHER
  // must equal 384 * 168 (the launch allocation under __launch_bounds__(384,1)).
  static constexpr int THREADS = 384;
  static constexpr int MMA_WARP = 8;
  static constexpr int LOAD_WARP = 9;
  static constexpr int REG_SOFTMAX = 216;
  static constexpr int REG_OTHER = 72;
  static_assert(2 * 128 * REG_SOFTMAX + 128 * REG_OTHER == THREADS * 168, "register split");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t TMEM_S = 0;    // + w * 128
  static constexpr uint32_t TMEM_O = 256;  // + w * 128
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

struct WaitCtx {
  volatile int *abort;
  int32_t *status;
  uint64_t timeout_ns;
};

// Bounded wait on an mbarrier phase. Returns false (and raises the CTA abort
// flag and the device status) when the wait expires or another warp aborted.
__device__ __forceinline__ bool bounded_wait(const WaitCtx &c, uint32_t bar, uint32_t parity,
                                             bool honour_abort = true) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (honour_abort && *c.abort) return false;
      if (ptx::globaltimer_ns() - t0 > c.timeout_ns) {
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

// Score -> modified, masked value, in place. MODE 0: tile fully visible (no
// mask code at all); 1: band + prefix test; 2: band + prefix + dilation.
// mx[c] receives the maximum of chunk c (softmax kinds only).
template <int KIND, int MODE>
__device__ __forceinline__ void transform_tile(uint32_t (&sr)[4][32], const EpiConsts &k,
                                               const RowMask &rm, float (&mx)[4]) {
  constexpr bool SOFTMAX = (KIND == KIND_SOFTMAX || KIND == KIND_SOFTCAP || KIND == KIND_ALIBI);
  constexpr float MASKED = SOFTMAX ? -INFINITY : 0.0f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float m = -INFINITY;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int col = c * 32 + e;
      const float s = __uint_as_float(sr[c][e]);
      float x;
      if (KIND == KIND_SOFTMAX) {
        x = s * k.k_mul;
      } else if (KIND == KIND_SOFTCAP) {
        x = ptx::tanh_fast(s * k.k_mul) * k.k_cap;
      } else if (KIND == KIND_ALIBI) {
        x = fmaf(k.k_bias, k.rel0 + static_cast<float>(col), s * k.k_mul);
      } else if (KIND == KIND_SIGMOID) {
        x = ptx::rcp_fast(1.0f + ptx::ex2(fmaf(s, k.k_mul, k.k_bias)));
      } else {
        x = fmaxf(s * k.k_mul, 0.0f);
      }
      if (MODE != 0) {
        bool vis = static_cast<uint32_t>(col - rm.c_lo) <= rm.span;
        if (MODE == 2) vis = vis && ((rm.i_rel - col) % rm.dil) == 0;
        vis = vis || (col < rm.c_pre);
        x = vis ? x : MASKED;
      }
      if (SOFTMAX) m = fmaxf(m, x);
      sr[c][e] = __float_as_uint(x);
    }
    mx[c] = m;
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return BF16 ? ptx::pack_bf16(lo, hi) : ptx::pack_f16(lo, hi);
}

// p = 2^(x - m), packed to 16-bit pairs and stored over the first 64 TMEM
// columns of the S tile (32 columns at a time); returns the row sum of p.
template <bool BF16>
__device__ __forceinline__ float exp_pack_store(uint32_t (&sr)[4][32], float m, uint32_t tS) {
  float ls[4];
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    uint32_t pk[32];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = 2 * h2 + cc;
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float p0 = ptx::ex2(__uint_as_float(sr[c][2 * e]) - m);
        const float p1 = ptx::ex2(__uint_as_float(sr[c][2 * e + 1]) - m);
        acc += p0 + p1;
        pk[cc * 16 + e] = pack2<BF16>(p0, p1);
      }
      ls[c] = acc;
    }
    ptx::tmem_st32(tS + h2 * 32, pk);
  }
  return (ls[0] + ls[1]) + (ls[2] + ls[3]);
}

template <bool BF16>
__device__ __forceinline__ void pack_store(uint32_t (&sr)[4][32], uint32_t tS) {
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2) {
    uint32_t pk[32];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc)
#pragma unroll
      for (int e = 0; e < 16; ++e)
        pk[cc * 16 + e] = pack2<BF16>(__uint_as_float(sr[2 * h2 + cc][2 * e]),
                                      __uint_as_float(sr[2 * h2 + cc][2 * e + 1]));
    ptx::tmem_st32(tS + h2 * 32, pk);
  }
}

// O_w rows of this warp *= alpha (lazy softmax rescale; rare).
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

// Epilogue: O row * inv -> 16-bit -> global (one thread per row).
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
template <int BM, int BN>
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
    tile_range(a.mask, U.m0 + w * BM, U.m0 + w * BM + BM - 1, BN, U.tlo[w], U.thi[w]);
    if (U.tlo[w] < U.thi[w]) {
      U.jlo = imin64(U.jlo, U.tlo[w]);
      U.jhi = imax64(U.jhi, U.thi[w]);
    }
  }
}

// Persistent kernel: each CTA loops over work units. With a scheduler
// workspace the load warp takes the next unit from a global counter (dynamic
// balance; the last CTA to finish puts the counter back to zero), otherwise
// CTA c runs units c, c + grid, c + 2 grid, ... . The unit index travels to the
// other roles through a two-slot ring in shared memory.
template <int D, bool BF16, int KIND>
__global__ void __launch_bounds__(FmhaConfig<D>::THREADS, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const KernelArgs args) {
  using C = FmhaConfig<D>;
  constexpr int BM = C::BM, BN = C::BN, NQ = C::NQ, NS = C::NS;
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
    for (int s = 0; s < NS; ++s) {
      ptx::mbar_init(bar(C::BAR_KFULL + s), 1);
      ptx::mbar_init(bar(C::BAR_KEMPTY + s), 1);
      ptx::mbar_init(bar(C::BAR_VFULL + s), 1);
      ptx::mbar_init(bar(C::BAR_VEMPTY + s), 1);
    }
    for (int w = 0; w < NQ; ++w) {
      ptx::mbar_init(bar(C::BAR_SFULL + w), 1);
      ptx::mbar_init(bar(C::BAR_PFULL + w), 4);   // one arrive per softmax warp
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
  const WaitCtx wc{abort_flag, args.status, args.timeout_ns};

  if (warp >= 8) {
    ptx::setmaxnreg_dec<C::REG_OTHER>();
    if (warp == C::LOAD_WARP && lane == 0) {
      // ==================== scheduler + TMA producer ====================
      uint32_t it = 0;
      int64_t last_use[2 * NS];
      for (int s = 0; s < 2 * NS; ++s) last_use[s] = -1;
      for (int k = 0;; ++k) {
        const int slot = k & 1;
        if (!bounded_wait(wc, bar(C::BAR_UEMPTY + slot), ((k >> 1) & 1) ^ 1)) break;
        int u = args.sched ? atomicAdd(args.sched, 1) : static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x);
        if (u >= args.n_units || u < 0) u = -1;
        unit_ring[slot] = u;
        ptx::mbar_arrive(bar(C::BAR_UFULL + slot));
        if (u < 0) break;
        UnitInfo U;
        decode_unit<BM, BN>(u, args, U);
        // Q tiles: the previous unit's S MMAs must be done with the buffer
        if (k > 0 && !bounded_wait(wc, bar(C::BAR_QEMPTY), (k - 1) & 1)) break;
        uint32_t qbytes = 0;
#pragma unroll
        for (int w = 0; w < NQ; ++w)
          if (U.wg_on(w)) qbytes += C::Q_TILE_BYTES;
        ptx::mbar_arrive_expect_tx(bar(C::BAR_Q), qbytes);
#pragma unroll
        for (int w = 0; w < NQ; ++w)
          if (U.wg_on(w))
#pragma unroll
            for (int c = 0; c < C::NCHUNK; ++c)
              ptx::tma_load_5d(sbase + C::OFF_Q + w * C::Q_TILE_BYTES + c * C::CHUNK_Q_BYTES,
                               &tm_q, bar(C::BAR_Q), c * 64, static_cast<int>(U.m0 + w * BM),
                               U.r_res, U.h, U.b);
        bool ok = true;
        for (int64_t j = U.jlo; j < U.jhi; ++j) {
          if (!U.any_active(j)) continue;
          const int s = it % NS;
          const uint32_t ph = (it / NS) & 1;
          if (!bounded_wait(wc, bar(C::BAR_KEMPTY + s), ph ^ 1)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(bar(C::BAR_KFULL + s), C::KV_TILE_BYTES);
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c)
            ptx::tma_load_5d(sbase + C::OFF_K + s * C::KV_TILE_BYTES + c * C::CHUNK_KV_BYTES,
                             &tm_k, bar(C::BAR_KFULL + s), c * 64, static_cast<int>(j * BN),
                             U.r_res, U.h, U.b);
          last_use[s] = it;
          if (!bounded_wait(wc, bar(C::BAR_VEMPTY + s), ph ^ 1)) { ok = false; break; }
          ptx::mbar_arrive_expect_tx(bar(C::BAR_VFULL + s), C::KV_TILE_BYTES);
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c)
            ptx::tma_load_5d(sbase + C::OFF_V + s * C::KV_TILE_BYTES + c * C::CHUNK_KV_BYTES,
                             &tm_v, bar(C::BAR_VFULL + s), c * 64, static_cast<int>(j * BN),
                             U.r_res, U.h, U.b);
          last_use[NS + s] = it;
          ++it;
        }
        if (!ok) break;
      }
      // Drain: every copy this thread issued lands before the CTA exits (the
      // Q copies complete before the MMA thread can finish its last unit).
      for (int s = 0; s < NS; ++s) {
        if (last_use[s] >= 0)
          bounded_wait(wc, bar(C::BAR_KFULL + s), (last_use[s] / NS) & 1, false);
        if (last_use[NS + s] >= 0)
          bounded_wait(wc, bar(C::BAR_VFULL + s), (last_use[NS + s] / NS) & 1, false);
      }
    } else if (warp == C::MMA_WARP && lane == 0) {
      // =========================== UMMA issuer ===========================
      constexpr uint32_t IDESC_QK = ptx::make_idesc_f16(BM, BN, BF16, false, false);
      constexpr uint32_t IDESC_PV = ptx::make_idesc_f16(BM, D, BF16, false, true);
      const uint32_t q_s = sbase + C::OFF_Q, k_s = sbase + C::OFF_K, v_s = sbase + C::OFF_V;

      auto issue_s = [&](int w, int stage) {
        const uint32_t d_tmem = tmem_base + C::TMEM_S + w * 128;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk & 3) * 32;
          const uint32_t qa = q_s + w * C::Q_TILE_BYTES + (kk >> 2) * C::CHUNK_Q_BYTES + off;
          const uint32_t ka = k_s + stage * C::KV_TILE_BYTES + (kk >> 2) * C::CHUNK_KV_BYTES + off;
          ptx::umma_ss(d_tmem, ptx::make_sdesc_sw128(qa, 16, 1024),
                       ptx::make_sdesc_sw128(ka, 16, 1024), IDESC_QK, kk > 0 ? 1u : 0u);
        }
      };
      auto issue_pv = [&](int w, int stage, bool first) {
        const uint32_t d_tmem = tmem_base + C::TMEM_O + w * 128;
        const uint32_t p_tmem = tmem_base + C::TMEM_S + w * 128;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t va = v_s + stage * C::KV_TILE_BYTES + kk * 2048;
          ptx::umma_ts(d_tmem, p_tmem + kk * 8, ptx::make_sdesc_sw128(va, C::CHUNK_KV_BYTES, 1024),
                       IDESC_PV, (first && kk == 0) ? 0u : 1u);
        }
      };

      uint32_t kit = 0, vit = 0, pcnt[NQ] = {0, 0}, units_w[NQ] = {0, 0};
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k & 1;
        if (!bounded_wait(wc, bar(C::BAR_UFULL + slot), (k >> 1) & 1)) break;
        const int u = unit_ring[slot];
        ptx::mbar_arrive(bar(C::BAR_UEMPTY + slot));
        if (u < 0) break;
        UnitInfo U;
        decode_unit<BM, BN>(u, args, U);
        if (!bounded_wait(wc, bar(C::BAR_Q), k & 1)) break;
        if (!bounded_wait(wc, bar(C::BAR_KFULL + kit % NS), (kit / NS) & 1)) break;
        ptx::tc_fence_after();
#pragma unroll
        for (int w = 0; w < NQ; ++w)
          if (U.active(w, U.jlo)) {
            issue_s(w, kit % NS);
            ptx::umma_commit(bar(C::BAR_SFULL + w));
          }
        ptx::umma_commit(bar(C::BAR_KEMPTY + kit % NS));
        ++kit;
        bool first[NQ] = {true, true};
        for (int64_t j = U.jlo; j < U.jhi;) {
          int64_t jn = j + 1;
          while (jn < U.jhi && !U.any_active(jn)) ++jn;
          const bool has_next = jn < U.jhi;
          if (!has_next) ptx::umma_commit(bar(C::BAR_QEMPTY));  // every S of this unit issued
          const int vs = vit % NS;
          const int ks = kit % NS;
          if (!bounded_wait(wc, bar(C::BAR_VFULL + vs), (vit / NS) & 1)) { ok = false; break; }
          if (has_next && !bounded_wait(wc, bar(C::BAR_KFULL + ks), (kit / NS) & 1)) { ok = false; break; }
          ptx::tc_fence_after();
#pragma unroll
          for (int w = 0; w < NQ; ++w) {
            if (U.active(w, j)) {
              if (!bounded_wait(wc, bar(C::BAR_PFULL + w), pcnt[w] & 1)) { ok = false; break; }
              ++pcnt[w];
              // the previous unit's epilogue must have read O_w before it is overwritten
              if (first[w] && units_w[w] > 0 &&
                  !bounded_wait(wc, bar(C::BAR_OEMPTY + w), (units_w[w] - 1) & 1)) { ok = false; break; }
              ptx::tc_fence_after();
              issue_pv(w, vs, first[w]);
              first[w] = false;
              if (j == U.thi[w] - 1) {
                ptx::umma_commit(bar(C::BAR_OFULL + w));
                ++units_w[w];
              }
            }
            if (has_next && U.active(w, jn)) {
              issue_s(w, ks);
              ptx::umma_commit(bar(C::BAR_SFULL + w));
            }
          }
          if (!ok) break;
          ptx::umma_commit(bar(C::BAR_VEMPTY + vs));
          ++vit;
          if (has_next) {
            ptx::umma_commit(bar(C::BAR_KEMPTY + ks));
            ++kit;
          }
          j = jn;
        }
      }
      // Drain: all UMMAs issued by this thread complete before TMEM is freed.
      ptx::umma_commit(bar(C::BAR_DRAIN));
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
    const int prefix = static_cast<int>(g.prefix);
    const int dil = static_cast<int>(g.dil);
    const float score_scale = args.score_scale;

    uint32_t cnt = 0, units_w = 0;
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      if (!bounded_wait(wc, bar(C::BAR_UFULL + slot), (k >> 1) & 1)) break;
      const int u = unit_ring[slot];
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_UEMPTY + slot));
      if (u < 0) break;
      UnitInfo U;
      decode_unit<BM, BN>(u, args, U);
      if (!U.wg_on(w)) continue;

      const int i = static_cast<int>(U.m0) + w * BM + row;
      const int64_t r0 = U.m0 + w * BM, r1 = r0 + BM - 1;
      int64_t blo64, bhi64;
      row_band(g, i, blo64, bhi64);
      const bool band_empty = bhi64 < blo64;
      const int blo = band_empty ? (1 << 30) : static_cast<int>(blo64);
      const uint32_t span = band_empty ? 0u : static_cast<uint32_t>(bhi64 - blo64);
      // per-kind constants (log2 domain for the softmax kinds)
      float hp = 1.0f;
      if (args.head_param != nullptr) hp = args.head_param[U.h];
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
      for (int64_t t = U.tlo[w]; t < U.thi[w]; ++t, ++cnt) {
        if (!bounded_wait(wc, bar(C::BAR_SFULL + w), cnt & 1)) { ok = false; break; }
        ptx::tc_fence_after();
        uint32_t sr[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) ptx::tmem_ld32(tS + c * 32, sr[c]);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) ptx::reg_fence(sr[c]);

        const int kv0 = static_cast<int>(t) * BN;
        RowMask rm;
        rm.c_lo = blo - kv0;
        rm.span = span;
        rm.c_pre = prefix - kv0;
        rm.i_rel = i - kv0;
        rm.dil = dil;
        kc.rel0 = static_cast<float>(kv0 - i);  // (j - i) of column 0, exact in fp32
        float mx[4];
        if (tile_full(g, r0, r1, BN, t))
          transform_tile<KIND, 0>(sr, kc, rm, mx);
        else if (dil == 1)
          transform_tile<KIND, 1>(sr, kc, rm, mx);
        else
          transform_tile<KIND, 2>(sr, kc, rm, mx);

        if (SOFTMAX) {
          const float m_new = fmaxf(m_run, fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])));
          const bool need = m_new > m_run + 8.0f;
          float alpha = 1.0f;
          if (need) {
            alpha = ptx::ex2(m_run - m_new);
            l_run *= alpha;
            m_run = m_new;
          }
          if (t > U.tlo[w] && __any_sync(0xffffffffu, need)) rescale_rows<D>(tO, alpha);
          const float m_use = (m_run == -INFINITY) ? 0.0f : m_run;
          l_run += exp_pack_store<BF16>(sr, m_use, tS);
        } else {
          pack_store<BF16>(sr, tS);
        }
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(C::BAR_PFULL + w));
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
        inv = 1.0f;
      const bool row_ok = i < g.sq;
      const int64_t real_row = static_cast<int64_t>(i) * args.vdil + U.r_res;
      uint8_t *orow = reinterpret_cast<uint8_t *>(args.o) +
                      2 * (U.b * args.o_sb + static_cast<int64_t>(U.h) * args.o_sh +
                           real_row * args.o_ss);
      store_rows<D, BF16>(tO, inv, row_ok, orow);
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
