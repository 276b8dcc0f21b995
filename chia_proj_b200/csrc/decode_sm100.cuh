// decode_sm100.cuh -- split-KV forward attention for decode-shaped calls:
// few query rows per K/V head (grouped heads x queries <= 32) over a long
// key sequence.
//
// Such a call is a matrix-vector product per K/V head: every key and value
// is read once and used by at most 32 rows, so the work is bound by HBM. A
// 5th-generation (tcgen05) MMA needs M >= 64 rows, which a decode step does
// not have, so the two small products run as warp-level m16n8k16 MMAs with
// fp32 accumulation, rows padded to 16 (32): their cost stays far below the
// time the keys and values take to arrive.
//
// One CTA (4 warps) takes one (batch, K/V head) and one contiguous key range
// ("split"); splits spread a head over the SMs. Tiles of 64 keys stream
// through a three-stage cp.async ring (K and V rows padded to a 16-byte
// multiple that keeps ldmatrix free of bank conflicts); warp w owns keys
// [16 w, 16 w + 16) of every tile and keeps its own running maximum, sum and
// output for the CTA's rows (online softmax in the log2 domain, in
// registers, rows in the fragment layout of the MMA). After the last tile the
// warps' results are merged in shared memory into the split's partial
// result; the last CTA of a head to finish (a per-head ticket) merges the
// splits into the output and the log-sum-exp and returns the ticket to zero.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "fmha_sm100.cuh"

namespace chia {

struct DecodeArgs {
  const void *q, *k, *v;
  void *o;
  int64_t q_sb, q_sh, q_ss;  // element strides (batch, head, row)
  int64_t k_sb, k_sh, k_ss;
  int64_t v_sb, v_sh, v_ss;
  int64_t o_sb, o_sh, o_ss;
  int32_t heads;     // query heads H
  int32_t heads_kv;  // K/V heads
  int32_t group;     // H / heads_kv
  int32_t sq;        // query rows per head
  int32_t rows;      // group * sq rows per K/V head
  int32_t kind;      // KIND_* (uniform per launch)
  MaskGeom mask;     // real index space (no packed sequences)
  int64_t key_lo;    // first key of the range the splits share
  int32_t keys_per_split;  // multiple of the tile width
  int32_t splits;
  float score_scale, softcap, sig_bias, out_scale;
  const float *head_param;  // ALiBi slope / temperature per query head, or null
  int32_t *tickets;         // [B * heads_kv], zero between launches
  float *part_o;            // [B * heads_kv][splits][RP][D] fp32
  float *part_ml;           // [B * heads_kv][splits][RP][2] (max log2, sum)
  float *lse;               // [B, H, sq] or null (softmax kinds)
};

template <int D>
struct DecodeConfig {
  static constexpr int TK = 64;                  // keys per tile (16 per warp)
  static constexpr int NST = 3;                  // ring stages
  static constexpr int THREADS = 128;
  static constexpr int PITCH = D * 2 + 16;       // bytes per padded K / V / Q row
  static constexpr int TILE_BYTES = TK * PITCH;  // one K or V tile
  static constexpr int STAGE_BYTES = 2 * TILE_BYTES;
};

struct RowC {  // per row of the CTA's head group
  int32_t lo, hi;  // mask band of the row's query position (keys < 2^30)
  float k_mul;     // multiplies the raw score
  float k_bias;    // ALiBi slope * log2(e) (times (j - i)), or the sigmoid offset
  int32_t i;       // query position
  int32_t valid;   // row < rows
  int32_t pad[2];
};

// RP: rows per K/V head padded to 16 or 32 (MMA row tiles of 16).
template <int D, int RP>
constexpr int decode_smem_bytes() {
  using C = DecodeConfig<D>;
  constexpr int ring = C::NST * C::STAGE_BYTES;
  constexpr int merge = 4 * RP * (D + 2) * 4;  // per warp: O rows, max, sum (after the ring)
  return (ring > merge ? ring : merge) + RP * C::PITCH + RP * static_cast<int>(sizeof(RowC));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                          uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D (16x8, fp32) += A (16x16, row) * B (16x8, col), 16-bit inputs
template <bool BF16>
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  if (BF16)
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
        "{%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <bool BF16>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  return BF16 ? ptx::pack_bf16(lo, hi) : ptx::pack_f16(lo, hi);
}

// Grid: (splits, batch * heads_kv); 128 threads. KIND: the score
// modification and normaliser (compile time, so that the element loop has
// no branches on it).
template <int D, int RP, bool BF16, int KIND>
__global__ void __launch_bounds__(128) decode_kernel(const DecodeArgs a) {
  using C = DecodeConfig<D>;
  constexpr int TK = C::TK, NST = C::NST, PITCH = C::PITCH;
  constexpr int MT = RP / 16;  // row tiles of 16
  constexpr int NT = D / 8;    // output column tiles of 8
  static_assert(RP == 16 || RP == 32, "rows padded to 16 or 32");
  constexpr float LOG2E = 1.4426950408889634f;
  extern __shared__ __align__(16) uint8_t sm[];
  constexpr int RING = NST * C::STAGE_BYTES;
  constexpr int MERGE = 4 * RP * (D + 2) * 4;
  constexpr int BODY = RING > MERGE ? RING : MERGE;
  uint8_t *qsm = sm + BODY;                                       // [RP][PITCH] bf16 / f16
  RowC *rc = reinterpret_cast<RowC *>(sm + BODY + RP * PITCH);    // [RP]
  __shared__ int last_cta;
  __shared__ int32_t band_lo_max, band_hi_min;  // over the valid rows

  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  const int split = blockIdx.x;
  const int kvh = blockIdx.y;  // b * heads_kv + head_kv
  const int b = kvh / a.heads_kv, hk = kvh % a.heads_kv;
  const MaskGeom &g = a.mask;
  constexpr int kind = KIND;
  constexpr bool softmax = KIND == 0 || KIND == 1 || KIND == 2;

  // ---- per-row constants, Q rows (16-bit, padded rows zero) ----
  if (t < RP) {
    RowC r{};
    r.valid = t < a.rows;
    const int gi = r.valid ? t / a.sq : 0, qi = r.valid ? t % a.sq : 0;
    const int h = hk * a.group + gi;
    r.i = qi;
    int64_t lo64, hi64;
    row_band(g, qi, lo64, hi64);
    r.lo = static_cast<int32_t>(lo64);
    r.hi = static_cast<int32_t>(hi64 < 0 ? -1 : hi64);
    const float hp = a.head_param != nullptr ? a.head_param[h] : 1.0f;
    r.k_mul = a.score_scale * LOG2E;
    r.k_bias = 0.f;
    if (kind == 0) r.k_mul *= hp;                        // plain / temperature
    if (kind == 1) r.k_mul = a.score_scale / a.softcap;  // softcap: tanh argument
    if (kind == 2) r.k_bias = hp * LOG2E;                // ALiBi
    if (kind == 3) {                                     // sigmoid: 2^-((s*scale + bias) log2e)
      r.k_mul = -a.score_scale * LOG2E;
      r.k_bias = -a.sig_bias * LOG2E;
    }
    if (kind == 4) r.k_mul = a.score_scale;              // ReLU
    rc[t] = r;
  }
  if (t == 0) {
    band_lo_max = 0;
    band_hi_min = 0x7fffffff;
  }
  __syncthreads();
  if (t < a.rows) {  // the key range every valid row sees completely (dilation 1, no prefix)
    atomicMax(&band_lo_max, rc[t].lo);
    atomicMin(&band_hi_min, rc[t].hi);
  }
  for (int e = t; e < RP * (D / 8); e += C::THREADS) {  // 16-byte pieces of Q rows
    const int r = e / (D / 8), c = e % (D / 8);
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < a.rows) {
      const int h = hk * a.group + r / a.sq, qi = r % a.sq;
      val = *reinterpret_cast<const uint4 *>(reinterpret_cast<const uint16_t *>(a.q) + b * a.q_sb +
                                             h * a.q_sh + qi * a.q_ss + c * 8);
    }
    *reinterpret_cast<uint4 *>(qsm + r * PITCH + c * 16) = val;
  }

  // ---- key tiles of this split ----
  const int64_t k0 = a.key_lo + static_cast<int64_t>(split) * a.keys_per_split;
  int64_t k1 = k0 + a.keys_per_split;
  if (k1 > g.skv) k1 = g.skv;
  const int ntiles = k1 > k0 ? static_cast<int>((k1 - k0 + TK - 1) / TK) : 0;
  const uint8_t *kbase = reinterpret_cast<const uint8_t *>(a.k) + 2 * (b * a.k_sb + hk * a.k_sh);
  const uint8_t *vbase = reinterpret_cast<const uint8_t *>(a.v) + 2 * (b * a.v_sb + hk * a.v_sh);
  const uint32_t ring = ptx::smem_u32(sm);
  constexpr int CHUNKS = TK * D / 8;  // 16-byte copies per K (V) tile
  auto load_tile = [&](int tile) {
    if (tile < ntiles) {
      const int64_t j0 = k0 + static_cast<int64_t>(tile) * TK;
      const uint32_t kd = ring + (tile % NST) * C::STAGE_BYTES;
      const uint32_t vd = kd + C::TILE_BYTES;
#pragma unroll 4
      for (int c = t; c < CHUNKS; c += C::THREADS) {
        const int row = c / (D / 8), col = c % (D / 8);
        const int64_t j = j0 + row;
        const bool ok = j < k1;
        const int64_t jj = ok ? j : k0;  // a valid address; nothing is read when !ok
        cp_async16(kd + row * PITCH + col * 16, kbase + 2 * (jj * a.k_ss) + col * 16, ok);
        cp_async16(vd + row * PITCH + col * 16, vbase + 2 * (jj * a.v_ss) + col * 16, ok);
      }
    }
    cp_async_commit();  // (an empty group past the last tile keeps the counting uniform)
  };
#pragma unroll
  for (int s = 0; s < NST - 1; ++s) load_tile(s);
  __syncthreads();  // Q and the row constants

  // Per thread: rows gid + 8 h2 + 16 m (h2 = 0, 1; m < MT) in the MMA layout.
  float o[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int n = 0; n < NT; ++n) o[m][n][0] = o[m][n][1] = o[m][n][2] = o[m][n][3] = 0.f;
  float m_run[MT][2], l_run[MT][2];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    m_run[m][0] = m_run[m][1] = -INFINITY;
    l_run[m][0] = l_run[m][1] = 0.f;
  }
  const uint32_t qaddr = ptx::smem_u32(qsm);

  Tracer trc(warp == 0 ? 0 : 1);
  auto tr = [&](int tag) { if (lane == 0 && (warp == 0 || warp == 1)) trc(tag); };
  tr(1);  // prologue issued
  for (int tile = 0; tile < ntiles; ++tile) {
    load_tile(tile + NST - 1);
    cp_async_wait<NST - 1>();  // tile `tile` has landed (this thread's copies)
    tr(2);
    __syncthreads();           // ... and every thread's
    tr(3);
    const uint32_t kst = ring + (tile % NST) * C::STAGE_BYTES + warp * 16 * PITCH;
    const uint32_t vst = kst + C::TILE_BYTES;
    // ---------------- S = Q K^T for this warp's 16 keys ----------------
    float s[MT][2][4];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int n = 0; n < 2; ++n) s[m][n][0] = s[m][n][1] = s[m][n][2] = s[m][n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      // B fragments: keys 0-7 / 8-15 x features 16kk..+15 (key rows, non-transposed)
      uint32_t b0, b1, b2, b3;
      ldsm_x4(kst + ((lane & 7) + ((lane >> 4) << 3)) * PITCH + (kk * 16 + ((lane >> 3) & 1) * 8) * 2,
              b0, b1, b2, b3);
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        uint32_t qa[4];
        ldsm_x4(qaddr + (m * 16 + (lane & 15)) * PITCH + (kk * 16 + (lane >> 4) * 8) * 2, qa[0],
                qa[1], qa[2], qa[3]);
        mma16816<BF16>(s[m][0], qa, b0, b1);
        mma16816<BF16>(s[m][1], qa, b2, b3);
      }
    }
    // ---------------- mod, mask, normaliser ----------------
    const int jw = static_cast<int>(k0) + tile * TK + warp * 16;
    // every valid row sees these 16 keys: no element test (padded rows of the
    // MMA are never stored, whatever their scores)
    const bool full = g.dil == 1 && jw >= band_lo_max && jw + 15 <= band_hi_min &&
                      jw + 16 <= k1;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const RowC R = rc[m * 16 + h2 * 8 + gid];
        float mx = -INFINITY;
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = jw + n * 8 + 2 * tig + e;
            const float sv = s[m][n][2 * h2 + e];
            const bool vis =
                full || (R.valid && j < k1 &&
                         (j < g.prefix ||
                          (j >= R.lo && j <= R.hi && (g.dil == 1 || (R.i - j) % g.dil == 0))));
            float x;
            if (kind == 3) {  // sigmoid(s * scale + bias)
              const float ex = ptx::ex2(fminf(fmaf(sv, R.k_mul, R.k_bias), 126.f));
              x = vis ? __fdividef(1.f, 1.f + ex) : 0.f;
            } else if (kind == 4) {  // ReLU(s * scale)
              x = vis ? fmaxf(sv * R.k_mul, 0.f) : 0.f;
            } else {
              if (kind == 1)
                x = a.softcap * LOG2E * ptx::tanh_fast(sv * R.k_mul);
              else
                x = sv * R.k_mul;
              if (kind == 2) x = fmaf(R.k_bias, static_cast<float>(j - R.i), x);
              if (!vis) x = -INFINITY;
              mx = fmaxf(mx, x);
            }
            s[m][n][2 * h2 + e] = x;
          }
        if (softmax) {
          // the quad of lanes holding this row: max over its 16 keys
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
          mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
          const float m_new = fmaxf(m_run[m][h2], mx);
          const float mu = m_new == -INFINITY ? 0.f : m_new;
          const float alpha = ptx::ex2(m_run[m][h2] - mu);  // 0 while nothing was seen
          float sum = 0.f;
#pragma unroll
          for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const float p = ptx::ex2(s[m][n][2 * h2 + e] - mu);
              s[m][n][2 * h2 + e] = p;
              sum += p;
            }
          l_run[m][h2] = l_run[m][h2] * alpha + sum;  // this lane's keys only
          m_run[m][h2] = m_new;
          if (__any_sync(0xffffffffu, alpha != 1.0f)) {  // the maximum grew somewhere
#pragma unroll
            for (int n = 0; n < NT; ++n) {
              o[m][n][2 * h2] *= alpha;
              o[m][n][2 * h2 + 1] *= alpha;
            }
          }
        }
      }
    }
    tr(4);  // scores and softmax done
    // ---------------- O += P V ----------------
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      // P as the A operand: the score fragments of keys 0-7 and 8-15 are its two halves
      const uint32_t pa[4] = {pack16<BF16>(s[m][0][0], s[m][0][1]),
                              pack16<BF16>(s[m][0][2], s[m][0][3]),
                              pack16<BF16>(s[m][1][0], s[m][1][1]),
                              pack16<BF16>(s[m][1][2], s[m][1][3])};
#pragma unroll
      for (int n2 = 0; n2 < NT / 2; ++n2) {
        // V (keys x features) transposed: B fragments of feature tiles 2 n2, 2 n2 + 1
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vst + ((lane & 7) + ((lane >> 3) & 1) * 8) * PITCH + (n2 * 16 + (lane >> 4) * 8) * 2,
                  b0, b1, b2, b3);
        mma16816<BF16>(o[m][2 * n2], pa, b0, b1);
        mma16816<BF16>(o[m][2 * n2 + 1], pa, b2, b3);
      }
    }
    tr(5);  // P V done
    __syncthreads();  // the stage is refilled by the next iteration's load
  }
  cp_async_wait<0>();
  __syncthreads();
  tr(6);  // main loop done

  // ---------------- merge the four warps (shared memory) ----------------
  float *mo = reinterpret_cast<float *>(sm);            // [4][RP][D]
  float *mml = mo + 4 * RP * D;                         // [4][RP][2]
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int r = m * 16 + h2 * 8 + gid;
      float l = l_run[m][h2];
      l += __shfl_xor_sync(0xffffffffu, l, 1);
      l += __shfl_xor_sync(0xffffffffu, l, 2);
#pragma unroll
      for (int n = 0; n < NT; ++n)
        *reinterpret_cast<float2 *>(mo + (warp * RP + r) * D + n * 8 + 2 * tig) =
            make_float2(o[m][n][2 * h2], o[m][n][2 * h2 + 1]);
      if (tig == 0) {
        mml[(warp * RP + r) * 2] = m_run[m][h2];
        mml[(warp * RP + r) * 2 + 1] = l;
      }
    }
  __syncthreads();
  const int64_t slot = static_cast<int64_t>(kvh) * a.splits + split;
  for (int e = t; e < RP * D; e += C::THREADS) {  // the split's partial result
    const int r = e / D;
    float M = -INFINITY;
    if (softmax)
      for (int w = 0; w < 4; ++w) M = fmaxf(M, mml[(w * RP + r) * 2]);
    float acc = 0.f, L = 0.f;
    for (int w = 0; w < 4; ++w) {
      float wt = 1.f;
      if (softmax) {
        const float mw = mml[(w * RP + r) * 2];
        wt = mw == -INFINITY ? 0.f : ptx::ex2(mw - M);
        L += wt * mml[(w * RP + r) * 2 + 1];
      }
      acc = fmaf(wt, mo[(w * RP + r) * D + (e % D)], acc);
    }
    a.part_o[slot * RP * D + e] = acc;
    if (e % D == 0) {
      a.part_ml[(slot * RP + r) * 2] = M;
      a.part_ml[(slot * RP + r) * 2 + 1] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) last_cta = atomicAdd(a.tickets + kvh, 1) == a.splits - 1;
  __syncthreads();
  tr(7);  // partial result written
  if (!last_cta) return;
  __threadfence();

  // ---------------- the last split of the head merges all of them ----------------
  // Every split's row maxima and sums go to shared memory in one round of
  // loads; the weights 2^(m_s - M) follow per row; then each thread sums the
  // splits' partial outputs for four columns of a row, loads issued together.
  const float *pml = a.part_ml + static_cast<int64_t>(kvh) * a.splits * RP * 2;
  const float *pob = a.part_o + static_cast<int64_t>(kvh) * a.splits * RP * D;
  float *wsm = reinterpret_cast<float *>(sm);  // [splits][RP] weights, then [RP] 1/L, [RP] M, [RP] L
  const int nsw = a.splits * RP;
  for (int e = t; e < nsw; e += C::THREADS) wsm[e] = __ldcg(pml + 2 * e);  // maxima
  __syncthreads();
  float *inv_s = wsm + nsw, *m_sm = inv_s + RP, *l_sm = m_sm + RP;
  if (t < RP) {
    float M = -INFINITY;
    if (softmax)
      for (int s2 = 0; s2 < a.splits; ++s2) M = fmaxf(M, wsm[s2 * RP + t]);
    float L = 0.f;
    for (int s2 = 0; s2 < a.splits; ++s2) {
      float wt = 1.f;
      if (softmax) {
        const float ms = wsm[s2 * RP + t];
        wt = ms == -INFINITY ? 0.f : ptx::ex2(ms - M);
        L += wt * __ldcg(pml + (s2 * RP + t) * 2 + 1);
      }
      wsm[s2 * RP + t] = wt;
    }
    float inv = 1.f;
    if (softmax) inv = L > 0.f ? 1.f / L : 0.f;
    if (kind == 4) inv = a.out_scale;
    inv_s[t] = inv;
    m_sm[t] = M;
    l_sm[t] = L;
  }
  __syncthreads();
  for (int e = t; e < a.rows * (D / 4); e += C::THREADS) {  // four columns per step
    const int r = e / (D / 4), c4 = e % (D / 4);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 *src = reinterpret_cast<const float4 *>(pob + r * D) + c4;
    constexpr int U4 = 4;
    int s2 = 0;
    for (; s2 + U4 <= a.splits; s2 += U4) {
      float4 ov[U4];
#pragma unroll
      for (int uu = 0; uu < U4; ++uu) ov[uu] = __ldcg(src + (s2 + uu) * (RP * D / 4));
#pragma unroll
      for (int uu = 0; uu < U4; ++uu) {
        const float wt = wsm[(s2 + uu) * RP + r];
        acc.x = fmaf(wt, ov[uu].x, acc.x);
        acc.y = fmaf(wt, ov[uu].y, acc.y);
        acc.z = fmaf(wt, ov[uu].z, acc.z);
        acc.w = fmaf(wt, ov[uu].w, acc.w);
      }
    }
    for (; s2 < a.splits; ++s2) {
      const float4 ov = __ldcg(src + s2 * (RP * D / 4));
      const float wt = wsm[s2 * RP + r];
      acc.x = fmaf(wt, ov.x, acc.x);
      acc.y = fmaf(wt, ov.y, acc.y);
      acc.z = fmaf(wt, ov.z, acc.z);
      acc.w = fmaf(wt, ov.w, acc.w);
    }
    const float inv = inv_s[r];
    const int h = hk * a.group + r / a.sq, qi = r % a.sq;
    uint8_t *orow = reinterpret_cast<uint8_t *>(a.o) + 2 * (b * a.o_sb + h * a.o_sh + qi * a.o_ss);
    *reinterpret_cast<uint2 *>(orow + 8 * c4) =
        make_uint2(pack16<BF16>(acc.x * inv, acc.y * inv), pack16<BF16>(acc.z * inv, acc.w * inv));
    if (softmax && a.lse != nullptr && c4 == 0) {
      constexpr float LN2 = 0.6931471805599453f;
      const float L = l_sm[r];
      a.lse[(static_cast<int64_t>(b) * a.heads + h) * a.sq + qi] =
          L > 0.f ? (m_sm[r] + __log2f(L)) * LN2 : -INFINITY;
    }
  }
  tr(8);  // merged
  if (t == 0) a.tickets[kvh] = 0;  // ready for the next launch
}

}  // namespace chia
