// bwd_sm100.cuh -- backward pass (dQ, dK, dV) of the attention variants on
// sm_100a: 5th-generation tensor cores (tcgen05) with operands staged by TMA
// and accumulators in tensor memory.
//
// One persistent CTA per SM walks work units; a unit is one tile of 128 keys
// of one (batch, K/V head) -- the keys of a dilated mask's residue class on
// the same "virtual head" path as the forward. K and V of the unit stay in
// shared memory while every query tile that sees the keys streams through
// (for grouped K/V heads, the query tiles of every query head of the group):
//
//   S^T  = K Q^T                (SS)  -> TMEM cols [0,128)    keys x queries
//   dP^T = V dO^T               (SS)  -> TMEM cols [128,256)
//   compute warps (thread = key): P^T, dS^T from S^T, dP^T, the forward's
//         log-sum-exp and delta = rowsum(dO * O); P^T (16-bit) back into TMEM
//         cols [0,32) and [64,96), dS^T (16-bit) into shared memory
//   dV  += P^T dO               (TS, A from TMEM)  -> cols [256,256+D)
//   dK  += dS^T Q               (SS, A K-major)    -> cols [384,384+D)
//   dQ_t = dS K                 (SS, A = the same dS^T tile read MN-major)
//                                                  -> cols [128,128+D)
//   the same warps (thread = query): dQ_t staged in the tile's spent Q and dO
//         buffers and added to an fp32 dQ buffer by TMA tensor reductions
//
// The gradient of the score modification is folded into dS (with respect to
// the raw q.k): softmax kinds dS = P (dP - delta) dz/ds, dz/ds = scale * tau
// (temperature), scale (ALiBi, plain) or scale (1 - tanh^2) (softcap);
// sigmoid dS = dP sigma (1 - sigma) scale; ReLU dS = dP out_scale [z > 0]
// scale. So dQ = dS K and dK = dS^T Q need no further scaling; dV carries
// the ReLU output scale. Masked pairs contribute nothing.
//
// Warps: 0-7 compute (two column halves of each lane quadrant), 8 MMA issuer,
// 9 TMA loads.
// Every wait is bounded like the forward's.
#pragma once
#include "fmha_sm100.cuh"

namespace chia {

struct BwdArgs {
  MaskGeom mask;        // virtual index space (as in the forward)
  int32_t heads;        // H
  int32_t heads_kv;     // K/V heads
  int32_t group;        // H / heads_kv
  int32_t vdil;         // 1, or the dilation of the residue-class path
  int32_t n_qt;         // query tiles of 128 (virtual rows)
  int32_t n_kt;         // key tiles of 128
  int32_t n_units;      // n_kt * batch * heads_kv * vdil
  float score_scale, softcap, sig_bias, out_scale;
  const float *head_param;  // ALiBi slope / temperature per query head, or null
  const float *lse;         // natural log-sum-exp [B, H, S_q] (softmax kinds)
  const float *delta;       // rowsum(dO * O) [B, H, S_q] (softmax kinds)
  float *dq_acc;            // fp32 [B, H, S_q, D] (real rows), zero on entry
  void *dk, *dv;
  int64_t dk_sb, dk_sh, dk_ss, dv_sb, dv_sh, dv_ss;
  int64_t sq_real;          // S_q
  int32_t *status;
  uint64_t timeout_ns, drain_ns;
};

template <int D>
struct BwdConfig {
  static constexpr int BM = 128;                  // queries per tile
  static constexpr int BN = 128;                  // keys per unit
  static constexpr int NCH = D / 64;              // 128-byte column chunks of a row
  static constexpr int CHUNK = 128 * 128;         // 128 rows x 64 elements (16 KB)
  static constexpr int TILE = NCH * CHUNK;        // a Q, dO, K or V tile
  static constexpr int DS_BYTES = 2 * CHUNK;      // dS^T: 128 keys x 128 queries
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TILE;
  static constexpr int OFF_Q = OFF_V + TILE;      // two buffers
  static constexpr int OFF_DO = OFF_Q + 2 * TILE;  // two buffers
  static constexpr int OFF_DS = OFF_DO + 2 * TILE;
  // per query column of the tile, two buffers: lse2, delta (fp32)
  static constexpr int OFF_VEC = OFF_DS + DS_BYTES;
  static constexpr int VEC_BYTES = 2 * 2 * 128 * 4;
  static constexpr int OFF_BAR = OFF_VEC + VEC_BYTES;
  static constexpr int BAR_KVFULL = 0, BAR_KVEMPTY = 1, BAR_QFULL = 2 /* [2] */,
                       BAR_QEMPTY = 4 /* [2] */, BAR_DOFULL = 6 /* [2] */,
                       BAR_DOEMPTY = 8 /* [2] */, BAR_SFULL = 10, BAR_PREADY = 11,
                       BAR_DQFULL = 12, BAR_DQEMPTY = 13, BAR_ACCFULL = 14, BAR_ACCEMPTY = 15,
                       BAR_DRAIN = 16, BAR_VEC = 17 /* [2] */,
                       BAR_STAGED = 19 /* [2]: dQ_t half staged for its reduction */,
                       NUM_BARS = 21;
  static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;  // tmem base, abort flag
  static constexpr int SMEM_BYTES = OFF_MISC + 16;
  // No slack for aligning the base at head_dim 128 (the double-buffered dO
  // needs the room): the dynamic shared memory of a kernel without static
  // shared memory starts 1024-byte aligned, which the kernel checks.
  static constexpr int SMEM_ALLOC = D == 128 ? SMEM_BYTES : SMEM_BYTES + 1024;
  static constexpr int THREADS = 320;
  static constexpr int MMA_WARP = 8, LOAD_WARP = 9;
  static constexpr uint32_t TMEM_S = 0, TMEM_DP = 128, TMEM_DQ = 128, TMEM_DV = 256,
                            TMEM_DK = 384, TMEM_COLS = 512;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(SMEM_ALLOC <= 232448, "shared memory budget");
};

// One unit: key tile jt of one virtual (batch, K/V head, residue) and the
// interval of query tiles that see it (lo() and hi() of the mask never
// decrease, so those tiles are contiguous).
struct BwdUnit {
  int jt, r_res, hk, b;
  int ilo, ihi;
};

__device__ __forceinline__ void decode_bwd_unit(int u, const BwdArgs &a, BwdUnit &U) {
  U.jt = u % a.n_kt;
  const int vh = u / a.n_kt;
  U.r_res = vh % a.vdil;
  U.hk = (vh / a.vdil) % a.heads_kv;
  U.b = vh / (a.vdil * a.heads_kv);
  U.ilo = a.n_qt;
  U.ihi = 0;
  for (int qt = 0; qt < a.n_qt; ++qt) {
    int64_t lo, hi;
    tile_range(a.mask, static_cast<int64_t>(qt) * 128, static_cast<int64_t>(qt) * 128 + 127, 128,
               lo, hi);
    if (lo <= U.jt && U.jt < hi) {
      if (qt < U.ilo) U.ilo = qt;
      U.ihi = qt + 1;
    }
  }
  if (U.ilo >= U.ihi) U.ilo = U.ihi = 0;
}

// Gradient of one (key, query) pair for kind KIND. s: raw q.k; dp: dO.v;
// returns P (what P V used) in p and dL/ds in ds.
template <int KIND>
__device__ __forceinline__ void bwd_pair(float s, float dp, bool vis, float lse2, float delta,
                                         float kmul, float kaux, float rel, const BwdArgs &a,
                                         float &p, float &ds) {
  constexpr float LOG2E = 1.4426950408889634f;
  if (KIND == KIND_SIGMOID) {
    // kmul = -scale log2e, kaux = -bias log2e: sigma = 1 / (1 + 2^(s kmul + kaux))
    const float e = ptx::ex2(fminf(fmaf(s, kmul, kaux), 126.f));
    const float sg = __fdividef(1.f, 1.f + e);
    p = vis ? sg : 0.f;
    ds = dp * p * (1.f - p) * a.score_scale;
  } else if (KIND == KIND_RELU) {
    const float z = s * a.score_scale;
    const bool on = vis && z > 0.f;
    p = on ? z : 0.f;
    ds = on ? dp * a.out_scale * a.score_scale : 0.f;
  } else {
    float x, dzds;
    if (KIND == KIND_SOFTCAP) {
      const float t = ptx::tanh_fast(s * kmul);  // kmul = scale / cap
      x = kaux * t;                              // kaux = cap log2e
      dzds = a.score_scale * (1.f - t * t);
    } else {
      x = s * kmul;                              // scale log2e (times tau)
      dzds = kmul * (1.0f / LOG2E);
      if (KIND == KIND_ALIBI) x = fmaf(kaux, rel, x);  // kaux = slope log2e vdil, rel = j - i
    }
    p = vis ? ptx::ex2(x - lse2) : 0.f;
    ds = p * (dp - delta) * dzds;
  }
}

template <int D, bool BF16, int KIND>
__global__ void __launch_bounds__(BwdConfig<D>::THREADS, 1)
    fmha_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                    const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v,
                    const __grid_constant__ CUtensorMap tm_do,
                    const __grid_constant__ CUtensorMap tm_dq, const BwdArgs args) {
  using C = BwdConfig<D>;
  constexpr int NCH = C::NCH;
  constexpr bool SOFTMAX = (KIND == KIND_SOFTMAX || KIND == KIND_SOFTCAP || KIND == KIND_ALIBI);
  constexpr float LOG2E = 1.4426950408889634f;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  // 128-byte swizzled tiles need a 1024-byte aligned base; without slack the
  // base itself must be aligned (reported through the status word otherwise)
  if (C::SMEM_ALLOC == C::SMEM_BYTES && (ptx::smem_u32(smem_raw) & 1023u)) {
    if (threadIdx.x == 0 && args.status) atomicOr(args.status, 4 /* CHIA_ERR_LAUNCH */);
    return;
  }
  auto bar = [&](int idx) -> uint32_t { return sbase + C::OFF_BAR + idx * 8; };
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::OFF_MISC);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::OFF_MISC + 4);
  // per query column: log-sum-exp (log2) [2][128], then delta [2][128]
  const uint32_t s_lse = sbase + C::OFF_VEC, s_delta = s_lse + 2 * 128 * 4;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const MaskGeom &g = args.mask;

  if (threadIdx.x == 0) {
    ptx::mbar_init(bar(C::BAR_KVFULL), 1);
    ptx::mbar_init(bar(C::BAR_KVEMPTY), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(C::BAR_QFULL + b), 1);
      ptx::mbar_init(bar(C::BAR_QEMPTY + b), 1);
      ptx::mbar_init(bar(C::BAR_DOFULL + b), 1);
      ptx::mbar_init(bar(C::BAR_DOEMPTY + b), 1);
    }
    ptx::mbar_init(bar(C::BAR_SFULL), 1);
    ptx::mbar_init(bar(C::BAR_PREADY), 8);    // the eight compute warps
    ptx::mbar_init(bar(C::BAR_DQFULL), 1);
    ptx::mbar_init(bar(C::BAR_DQEMPTY), 8);
    ptx::mbar_init(bar(C::BAR_ACCFULL), 1);
    ptx::mbar_init(bar(C::BAR_ACCEMPTY), 8);
    ptx::mbar_init(bar(C::BAR_DRAIN), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(C::BAR_VEC + b), 4);     // first-half warps
      ptx::mbar_init(bar(C::BAR_STAGED + b), 4);  // the warps of one column half
    }
    *abort_flag = 0;
    ptx::fence_barrier_init();
    ptx::fence_proxy_async_smem();
  }
  if (warp == C::LOAD_WARP && lane == 0) {
    ptx::tma_prefetch_desc(&tm_q);
    ptx::tma_prefetch_desc(&tm_k);
    ptx::tma_prefetch_desc(&tm_v);
    ptx::tma_prefetch_desc(&tm_do);
    ptx::tma_prefetch_desc(&tm_dq);
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

  if (warp == C::LOAD_WARP) {
    if (lane == 0) {
      // ============================ TMA loads ============================
      Tracer tr(3);
      uint32_t n = 0, un = 0;
      int last_q[2] = {-1, -1}, last_do[2] = {-1, -1};
      int last_kv = -1;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < args.n_units; u += gridDim.x) {
        BwdUnit U;
        decode_bwd_unit(u, args, U);
        if (U.ihi == U.ilo) continue;
        if (un > 0 && !bounded_wait(wc, bar(C::BAR_KVEMPTY), (un - 1) & 1)) break;
        ptx::mbar_arrive_expect_tx(bar(C::BAR_KVFULL), 2 * C::TILE);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          ptx::tma_load_5d(sbase + C::OFF_K + c * C::CHUNK, &tm_k, bar(C::BAR_KVFULL), c * 64,
                           U.jt * 128, U.r_res, U.hk, U.b);
          ptx::tma_load_5d(sbase + C::OFF_V + c * C::CHUNK, &tm_v, bar(C::BAR_KVFULL), c * 64,
                           U.jt * 128, U.r_res, U.hk, U.b);
        }
        last_kv = static_cast<int>(un);
        for (int gi = 0; ok && gi < args.group; ++gi) {
          const int h = U.hk * args.group + gi;
          for (int qt = U.ilo; qt < U.ihi; ++qt, ++n) {
            const int qb = n & 1;
            if (!bounded_wait(wc, bar(C::BAR_QEMPTY + qb), ((n >> 1) & 1) ^ 1)) { ok = false; break; }
            ptx::mbar_arrive_expect_tx(bar(C::BAR_QFULL + qb), C::TILE);
#pragma unroll
            for (int c = 0; c < NCH; ++c)
              ptx::tma_load_5d(sbase + C::OFF_Q + qb * C::TILE + c * C::CHUNK, &tm_q,
                               bar(C::BAR_QFULL + qb), c * 64, qt * 128, U.r_res, h, U.b);
            last_q[qb] = static_cast<int>(n);
            tr(40);  // Q of tile n issued
            if (!bounded_wait(wc, bar(C::BAR_DOEMPTY + qb), ((n >> 1) & 1) ^ 1)) { ok = false; break; }
            ptx::mbar_arrive_expect_tx(bar(C::BAR_DOFULL + qb), C::TILE);
#pragma unroll
            for (int c = 0; c < NCH; ++c)
              ptx::tma_load_5d(sbase + C::OFF_DO + qb * C::TILE + c * C::CHUNK, &tm_do,
                               bar(C::BAR_DOFULL + qb), c * 64, qt * 128, U.r_res, h, U.b);
            last_do[qb] = static_cast<int>(n);
            tr(41);  // dO of tile n issued
          }
        }
        ++un;
      }
      // Drain: every copy this thread issued has landed before the CTA exits.
      if (last_kv >= 0) bounded_wait(wc, bar(C::BAR_KVFULL), last_kv & 1, false);
      for (int b = 0; b < 2; ++b) {
        if (last_q[b] >= 0) bounded_wait(wc, bar(C::BAR_QFULL + b), (last_q[b] >> 1) & 1, false);
        if (last_do[b] >= 0)
          bounded_wait(wc, bar(C::BAR_DOFULL + b), (last_do[b] >> 1) & 1, false);
      }
    }
    __syncwarp();
  } else if (warp == C::MMA_WARP) {
    // ======================= UMMA issuer (whole warp) =======================
    constexpr uint32_t IDESC_SS = ptx::make_idesc_f16(128, 128, BF16, false, false);  // S^T, dP^T
    constexpr uint32_t IDESC_DV = ptx::make_idesc_f16(128, D, BF16, false, true);     // TS, B MN
    constexpr uint32_t IDESC_DK = ptx::make_idesc_f16(128, D, BF16, false, true);     // A K, B MN
    constexpr uint32_t IDESC_DQ = ptx::make_idesc_f16(128, D, BF16, true, true);      // A MN, B MN
    const uint64_t dk_k = ptx::make_sdesc_sw128(sbase + C::OFF_K, 16, 1024);    // K, K-major
    const uint64_t dv_k = ptx::make_sdesc_sw128(sbase + C::OFF_V, 16, 1024);    // V, K-major
    const uint64_t dq_k = ptx::make_sdesc_sw128(sbase + C::OFF_Q, 16, 1024);    // Q, K-major
    const uint64_t ddo_k = ptx::make_sdesc_sw128(sbase + C::OFF_DO, 16, 1024);  // dO, K-major
    const uint64_t dq_mn = ptx::make_sdesc_sw128(sbase + C::OFF_Q, C::CHUNK, 1024);   // Q, MN
    const uint64_t ddo_mn = ptx::make_sdesc_sw128(sbase + C::OFF_DO, C::CHUNK, 1024); // dO, MN
    const uint64_t dk_mn = ptx::make_sdesc_sw128(sbase + C::OFF_K, C::CHUNK, 1024);   // K, MN
    const uint64_t dds_k = ptx::make_sdesc_sw128(sbase + C::OFF_DS, 16, 1024);        // dS^T
    const uint64_t dds_mn = ptx::make_sdesc_sw128(sbase + C::OFF_DS, C::CHUNK, 1024); // dS
    // K-major operand, k-step kk of 16 elements: chunk kk / 4, 32 bytes per step inside it
    auto kstep = [](int kk) -> uint32_t {
      return static_cast<uint32_t>(((kk >> 2) * C::CHUNK + (kk & 3) * 32) >> 4);
    };
    // MN-major operand, k-step kk: 16 rows of 128 bytes
    auto mnstep = [](int kk) -> uint32_t { return static_cast<uint32_t>((kk * 2048) >> 4); };
    auto wait = [&](uint32_t b, uint32_t parity) {
      return __all_sync(0xffffffffu, bounded_wait(wc, b, parity));
    };
    Tracer trc(2);
    auto tr = [&](int tag) { if (lane == 0) trc(tag); };
    uint32_t n = 0, un = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < args.n_units; u += gridDim.x) {
      BwdUnit U;
      decode_bwd_unit(u, args, U);
      if (U.ihi == U.ilo) continue;
      if (!wait(bar(C::BAR_KVFULL), un & 1)) break;
      tr(29);  // K, V of the unit landed
      const int T = (U.ihi - U.ilo) * args.group;
      for (int t = 0; t < T; ++t, ++n) {
        const int qb = n & 1;
        const uint32_t qoff = static_cast<uint32_t>((qb * C::TILE) >> 4);
        if (!wait(bar(C::BAR_QFULL + qb), (n >> 1) & 1)) { ok = false; break; }
        ptx::tc_fence_after();
        // k-steps in groups of four under one elect.sync
        auto ss4 = [&](uint32_t d, uint64_t a0, uint64_t b0, bool a_mn, bool b_mn, int k0,
                       uint32_t idesc, uint32_t acc0) {
          uint64_t a[4], b[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            a[x] = a0 + (a_mn ? mnstep(k0 + x) : kstep(k0 + x));
            b[x] = b0 + (b_mn ? mnstep(k0 + x) : kstep(k0 + x));
          }
          ptx::umma_ss_x4_warp(d, a, b, idesc, acc0);
        };
#pragma unroll
        for (int k4 = 0; k4 < D / 16; k4 += 4)  // S^T = K Q^T
          ss4(tmem_base + C::TMEM_S, dk_k, dq_k + qoff, false, false, k4, IDESC_SS,
              k4 > 0 ? 1u : 0u);
        tr(30);  // S^T issued
        if (!wait(bar(C::BAR_DOFULL + qb), (n >> 1) & 1)) { ok = false; break; }
        tr(31);  // dO landed
        if (n > 0 && !wait(bar(C::BAR_DQEMPTY), (n - 1) & 1)) { ok = false; break; }
        tr(32);  // previous dQ drained
        ptx::tc_fence_after();
#pragma unroll
        for (int k4 = 0; k4 < D / 16; k4 += 4)  // dP^T = V dO^T
          ss4(tmem_base + C::TMEM_DP, dv_k, ddo_k + qoff, false, false, k4, IDESC_SS,
              k4 > 0 ? 1u : 0u);
        ptx::umma_commit_warp(bar(C::BAR_SFULL));
        if (!wait(bar(C::BAR_PREADY), n & 1)) { ok = false; break; }
        tr(33);  // P^T, dS^T ready
        if (t == 0 && un > 0 && !wait(bar(C::BAR_ACCEMPTY), (un - 1) & 1)) { ok = false; break; }
        ptx::tc_fence_after();
#pragma unroll
        for (int k4 = 0; k4 < 128 / 16; k4 += 4) {  // over the 128 queries of the tile
          const uint32_t acc = (t > 0 || k4 > 0) ? 1u : 0u;
          // dV += P^T dO    (P^T: 16-bit pairs in TMEM columns [0, 32) and [64, 96))
          uint32_t pa[4];
          uint64_t pb[4];
#pragma unroll
          for (int x = 0; x < 4; ++x) {
            // queries 16 kk..+15 at column 8 kk, the second 64 queries from column 64
            const int kk = k4 + x;
            pa[x] = tmem_base + C::TMEM_S + kk * 8 + (kk >= 4 ? 32 : 0);
            pb[x] = ddo_mn + qoff + mnstep(kk);
          }
          ptx::umma_ts_x4_warp(tmem_base + C::TMEM_DV, pa, pb, IDESC_DV, acc);
          // dK += dS^T Q
          ss4(tmem_base + C::TMEM_DK, dds_k, dq_mn + qoff, false, true, k4, IDESC_DK, acc);
        }
#pragma unroll
        for (int k4 = 0; k4 < 128 / 16; k4 += 4)  // dQ_t = dS K, over the 128 keys
          ss4(tmem_base + C::TMEM_DQ, dds_mn, dk_mn, true, true, k4, IDESC_DQ, k4 > 0 ? 1u : 0u);
        // Q_n and dO_n are then reused to stage dQ_t for its reduction; their
        // "empty" barriers are arrived on by the staging threads once the
        // reductions have read them
        ptx::umma_commit_warp(bar(C::BAR_DQFULL));
        tr(34);  // dV, dK, dQ issued
        if (t == T - 1) {
          ptx::umma_commit_warp(bar(C::BAR_ACCFULL));
          ptx::umma_commit_warp(bar(C::BAR_KVEMPTY));
        }
      }
      ++un;
    }
    ptx::umma_commit_warp(bar(C::BAR_DRAIN));  // every UMMA of this warp retired
    bounded_wait(wc, bar(C::BAR_DRAIN), 0, false);
    __syncwarp();
  } else {
    // ============ compute warps 0-7: P^T, dS^T; dQ_t drain; dK, dV out ============
    // Warp w works on TMEM lane quadrant w % 4 and column half w / 4: queries
    // [64 half, 64 half + 64) of each tile for P^T and dS^T, and feature
    // columns [half D / 2, half D / 2 + D / 2) of dQ_t, dV and dK.
    const int quad = warp & 3, half = warp >> 2;
    const int row = quad * 32 + lane;  // key of the unit's tile (query of dQ_t)
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + C::TMEM_S;
    const uint32_t tDP = tmem_base + lane_off + C::TMEM_DP;
    const uint32_t dsrow = sbase + C::OFF_DS + row * 128;  // this key's row of dS^T, chunk 0
    const int rsw = row & 7;
    constexpr int HD = D / 2;  // feature columns per half
    Tracer trc(half);
    auto tr = [&](int tag) { if (quad == 0 && lane == 0) trc(tag); };
    uint32_t n = 0, un = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < args.n_units; u += gridDim.x) {
      BwdUnit U;
      decode_bwd_unit(u, args, U);
      const int j = U.jt * 128 + row;  // virtual key index
      const int64_t real_j = static_cast<int64_t>(j) * args.vdil + U.r_res;
      uint8_t *dkrow = reinterpret_cast<uint8_t *>(args.dk) +
                       2 * (U.b * args.dk_sb + static_cast<int64_t>(U.hk) * args.dk_sh +
                            real_j * args.dk_ss + half * HD);
      uint8_t *dvrow = reinterpret_cast<uint8_t *>(args.dv) +
                       2 * (U.b * args.dv_sb + static_cast<int64_t>(U.hk) * args.dv_sh +
                            real_j * args.dv_ss + half * HD);
      const bool key_ok = j < g.skv;
      if (U.ihi == U.ilo) {  // no query sees these keys: zero gradients
        if (key_ok)
#pragma unroll
          for (int v4 = 0; v4 < HD / 8; ++v4) {
            ptx::st_global_v4(dkrow + v4 * 16, 0u, 0u, 0u, 0u);
            ptx::st_global_v4(dvrow + v4 * 16, 0u, 0u, 0u, 0u);
          }
        continue;
      }
      for (int gi = 0; ok && gi < args.group; ++gi) {
        const int h = U.hk * args.group + gi;
        const float hp = args.head_param != nullptr ? args.head_param[h] : 1.0f;
        float kmul, kaux = 0.f;
        if (KIND == KIND_SOFTCAP) {
          kmul = args.score_scale / args.softcap;
          kaux = args.softcap * LOG2E;
        } else if (KIND == KIND_SIGMOID) {
          kmul = -args.score_scale * LOG2E;
          kaux = -args.sig_bias * LOG2E;
        } else {
          kmul = args.score_scale * LOG2E * (KIND == KIND_SOFTMAX ? hp : 1.0f);
          if (KIND == KIND_ALIBI) kaux = hp * LOG2E * static_cast<float>(args.vdil);
        }
        for (int qt = U.ilo; qt < U.ihi; ++qt, ++n) {
          const int vb = n & 1;
          // per query column of the tile: log-sum-exp (log2 units) and delta,
          // written by the first column half's warps
          if (half == 0) {
            const int i = qt * 128 + row;
            const int64_t real_i = static_cast<int64_t>(i) * args.vdil + U.r_res;
            const int64_t vi = (static_cast<int64_t>(U.b) * args.heads + h) * args.sq_real + real_i;
            float l2 = INFINITY, dl = 0.f;
            if (SOFTMAX && i < g.sq) {
              l2 = args.lse[vi] * LOG2E;
              dl = args.delta[vi];
            }
            ptx::st_shared_f32(s_lse + (vb * 128 + row) * 4, l2);
            ptx::st_shared_f32(s_delta + (vb * 128 + row) * 4, dl);
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar(C::BAR_VEC + vb));
          }
          // Bounded, unlike a named barrier, so that a warp leaving on an abort
          // cannot strand the others. The buffer of tile n is rewritten for tile
          // n + 2 only after its writers passed this point for tile n + 1, which
          // every warp reaches only after finishing tile n (it waits for
          // DQ_FULL(n), which needs all eight P_READY arrivals of tile n).
          if (!bounded_wait(wc, bar(C::BAR_VEC + vb), (n >> 1) & 1)) { ok = false; break; }
          const FullTiles ft = full_tiles(g, static_cast<int64_t>(qt) * 128,
                                          static_cast<int64_t>(qt) * 128 + 127, 128);
          const bool full = ft.full(U.jt) && qt * 128 + 127 < g.sq;
          tr(9);  // per-column vectors exchanged
          if (!bounded_wait(wc, bar(C::BAR_SFULL), n & 1)) { ok = false; break; }
          ptx::tc_fence_after();
          tr(10);  // S^T, dP^T in TMEM
          const uint32_t vl = s_lse + vb * 128 * 4, vd = s_delta + vb * 128 * 4;
#pragma unroll 1
          for (int c = 2 * half; c < 2 * half + 2; ++c) {  // 32 queries at a time
            uint32_t sr[32], dr[32];
            ptx::tmem_ld32(tS + c * 32, sr);
            ptx::tmem_ld32(tDP + c * 32, dr);
            ptx::tmem_wait_ld();
            ptx::reg_fence(sr);
            ptx::reg_fence(dr);
            float pv[32], dsv[32];
            if (full) {
#pragma unroll
              for (int e4 = 0; e4 < 8; ++e4) {
                const float4 L = ptx::ld_shared_v4f(vl + (c * 32 + e4 * 4) * 4);
                const float4 Dl = ptx::ld_shared_v4f(vd + (c * 32 + e4 * 4) * 4);
                const float la[4] = {L.x, L.y, L.z, L.w}, da[4] = {Dl.x, Dl.y, Dl.z, Dl.w};
#pragma unroll
                for (int u4 = 0; u4 < 4; ++u4) {
                  const int e = e4 * 4 + u4;
                  const int i = qt * 128 + c * 32 + e;
                  bwd_pair<KIND>(__uint_as_float(sr[e]), __uint_as_float(dr[e]), true, la[u4],
                                 da[u4], kmul, kaux, static_cast<float>(j - i), args, pv[e],
                                 dsv[e]);
                }
              }
            } else {
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                const int i = qt * 128 + c * 32 + e;
                bool vis = false;
                if (i < g.sq) {
                  int64_t lo, hi;
                  row_band(g, i, lo, hi);
                  vis = j < g.prefix ||
                        (j >= lo && j <= hi && (g.dil == 1 || ((i - j) % g.dil) == 0));
                }
                float la, da;
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(la) : "r"(vl + (c * 32 + e) * 4));
                asm volatile("ld.shared.f32 %0, [%1];" : "=f"(da) : "r"(vd + (c * 32 + e) * 4));
                bwd_pair<KIND>(__uint_as_float(sr[e]), __uint_as_float(dr[e]), vis, la, da, kmul,
                               kaux, static_cast<float>(j - i), args, pv[e], dsv[e]);
              }
            }
            uint32_t pk[16], dk2[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              pk[e] = pack2<BF16>(pv[2 * e], pv[2 * e + 1]);
              dk2[e] = pack2<BF16>(dsv[2 * e], dsv[2 * e + 1]);
            }
            // P^T (queries 32c..+31) -> TMEM columns 64 (c / 2) + 16 (c % 2)..+15, inside
            // this half's own S^T columns [64 half, 64 half + 64), of which 32c..+31
            // (and everything below in the half) has been read already; the other
            // half's warps never touch these columns
            ptx::tmem_st16(tS + (c >> 1) * 64 + (c & 1) * 16, pk);
            // dS^T row: queries 32c..+31 = 16-byte units 4 (c & 1) .. +3 of chunk c / 2
#pragma unroll
            for (int uu = 0; uu < 4; ++uu)
              ptx::st_shared_v4(dsrow + (c >> 1) * C::CHUNK + ((((c & 1) * 4 + uu) ^ rsw) << 4),
                                dk2[4 * uu], dk2[4 * uu + 1], dk2[4 * uu + 2], dk2[4 * uu + 3]);
          }
          ptx::tmem_wait_st();
          ptx::fence_proxy_async_smem();  // dS^T visible to the tensor core
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar(C::BAR_PREADY));
          tr(11);  // P^T, dS^T written
          // ---- dQ_t of this tile: TMEM -> registers, columns released, then added ----
          if (!bounded_wait(wc, bar(C::BAR_DQFULL), n & 1)) { ok = false; break; }
          ptx::tc_fence_after();
          tr(20);  // dQ_t in TMEM
          {
            uint32_t r[HD / 32][32];
#pragma unroll
            for (int c = 0; c < HD / 32; ++c)
              ptx::tmem_ld32(tmem_base + lane_off + C::TMEM_DQ + half * HD + c * 32, r[c]);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) ptx::reg_fence(r[c]);
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar(C::BAR_DQEMPTY));
            // The additions go to the fp32 buffer as TMA tensor reductions of
            // 128-row x 32-column boxes (16 KB, one L2 line per row): per-thread
            // vector atomics (8 KB per tile per warp) throttle the SM's memory
            // pipe, and thousands of small bulk copies the TMA engine. The boxes
            // are staged, 128-byte swizzled, in this tile's Q buffer (first column
            // half) or dO buffer (second half): every UMMA of the tile has read
            // them (DQ_FULL), and the loader refills them only after this half's
            // reductions have read the staging (the arrival on Q_EMPTY / DO_EMPTY).
            const int qb = n & 1;
            const uint32_t stage = sbase + (half == 0 ? C::OFF_Q : C::OFF_DO) + qb * C::TILE;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c)
#pragma unroll
              for (int u = 0; u < 8; ++u)
                ptx::st_shared_v4(stage + c * C::CHUNK + row * 128 + ((u ^ rsw) << 4),
                                  r[c][4 * u], r[c][4 * u + 1], r[c][4 * u + 2], r[c][4 * u + 3]);
            ptx::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(bar(C::BAR_STAGED + half));
            if (quad == 0 && lane == 0) {  // one thread per half issues and releases
              if (!bounded_wait(wc, bar(C::BAR_STAGED + half), n & 1)) ok = false;
              if (ok) {
#pragma unroll
                for (int c = 0; c < HD / 32; ++c)
                  ptx::tma_reduce_add_5d(&tm_dq, stage + c * C::CHUNK, half * HD + c * 32,
                                         qt * 128, U.r_res, h, U.b);
                ptx::bulk_commit_group();
                ptx::bulk_wait_read_all();
              }
              ptx::mbar_arrive(bar(half == 0 ? C::BAR_QEMPTY + qb : C::BAR_DOEMPTY + qb));
            }
          }
          tr(21);  // dQ_t read and added
        }
      }
      if (!ok) break;
      // ---------------- unit epilogue: dK, dV of these keys ----------------
      if (!bounded_wait(wc, bar(C::BAR_ACCFULL), un & 1)) break;
      ptx::tc_fence_after();
      const float vsc = KIND == KIND_RELU ? args.out_scale : 1.0f;
#pragma unroll 1
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t rv[32], rk[32];
        ptx::tmem_ld32(tmem_base + lane_off + C::TMEM_DV + half * HD + c * 32, rv);
        ptx::tmem_ld32(tmem_base + lane_off + C::TMEM_DK + half * HD + c * 32, rk);
        ptx::tmem_wait_ld();
        ptx::reg_fence(rv);
        ptx::reg_fence(rk);
        if (key_ok) {
#pragma unroll
          for (int v4 = 0; v4 < 4; ++v4) {
            uint32_t a4[4], b4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int x = v4 * 8 + 2 * e;
              a4[e] = pack2<BF16>(__uint_as_float(rv[x]) * vsc, __uint_as_float(rv[x + 1]) * vsc);
              b4[e] = pack2<BF16>(__uint_as_float(rk[x]), __uint_as_float(rk[x + 1]));
            }
            ptx::st_global_v4(dvrow + c * 64 + v4 * 16, a4[0], a4[1], a4[2], a4[3]);
            ptx::st_global_v4(dkrow + c * 64 + v4 * 16, b4[0], b4[1], b4[2], b4[3]);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(C::BAR_ACCEMPTY));
      ++un;
    }
    ptx::bulk_wait_all();  // every reduction of dQ this thread issued has completed
  }

  // ---- teardown ----
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == C::MMA_WARP) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// delta = rowsum(dO * O) per row (softmax kinds); one warp per row. Also
// zeroes the fp32 dQ buffer row.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) bwd_prep_kernel(const void *o, const void *dout,
                                                       int64_t o_sb, int64_t o_sh, int64_t o_ss,
                                                       int64_t d_sb, int64_t d_sh, int64_t d_ss,
                                                       int32_t heads, int64_t sq, float *delta,
                                                       float *dq_acc, int64_t rows, bool want_delta) {
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t b = r / (heads * sq), h = (r / sq) % heads, i = r % sq;
  constexpr int PER = D / 32;  // elements per lane
  float acc = 0.f;
  if (want_delta) {
    const uint16_t *orow = reinterpret_cast<const uint16_t *>(o) + b * o_sb + h * o_sh + i * o_ss;
    const uint16_t *drow =
        reinterpret_cast<const uint16_t *>(dout) + b * d_sb + h * d_sh + i * d_ss;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int d = lane * PER + e;
      float ov, dv;
      if (BF16) {
        ov = __uint_as_float(static_cast<uint32_t>(orow[d]) << 16);
        dv = __uint_as_float(static_cast<uint32_t>(drow[d]) << 16);
      } else {
        ov = __half2float(__ushort_as_half(orow[d]));
        dv = __half2float(__ushort_as_half(drow[d]));
      }
      acc = fmaf(ov, dv, acc);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) delta[r] = acc;
  }
  float *q = dq_acc + r * D;
#pragma unroll
  for (int e = 0; e < PER; ++e) q[lane * PER + e] = 0.f;
}

// dq = dq_acc (fp32) rounded to the 16-bit type, any strides.
template <int D, bool BF16>
__global__ void __launch_bounds__(256) bwd_dq_kernel(const float *dq_acc, void *dq, int64_t sb,
                                                     int64_t sh, int64_t ss, int32_t heads,
                                                     int64_t sq, int64_t rows) {
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int64_t b = r / (heads * sq), h = (r / sq) % heads, i = r % sq;
  constexpr int PER = D / 32;
  const float *src = dq_acc + r * D + lane * PER;
  uint16_t *dst = reinterpret_cast<uint16_t *>(dq) + b * sb + h * sh + i * ss + lane * PER;
#pragma unroll
  for (int e = 0; e < PER; e += 2) {
    const uint32_t pk = pack2<BF16>(src[e], src[e + 1]);
    *reinterpret_cast<uint32_t *>(dst + e) = pk;
  }
}

}  // namespace chia
