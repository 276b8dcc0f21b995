// attn_api.cu -- extern "C" entry points of libchia_attn.so (include/chia_attn.h).
//
// Host responsibilities: validate arguments (errors are returned before any
// launch), turn the mask fields into MaskGeom, pick the kernel
// instantiation (head_dim x dtype x kind), encode the three TMA tensor maps
// and launch on the caller's stream. No allocation, no synchronisation.
//
// Dilated masks take a residue-class fast path when it is exact: with
// dilation d, query i only sees keys j == i (mod d), so the problem splits
// into d independent problems over rows r, r+d, r+2d, ... . Each becomes a
// "virtual head" whose rows are read by TMA with a row stride of d rows, and
// whose mask is the same band divided by d. None of its tiles is then 3/4
// masked, unlike the plain causal path with an element-wise (i-j)%d test.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/chia_attn.h"
#include "bwd_sm100.cuh"
#include "decode_sm100.cuh"
#include "fmha2_sm100.cuh"

namespace {

using chia::MaskGeom;

constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s per barrier wait
// Waits for a CTA's own copies and MMAs before it exits keep this limit
// whatever params->wait_limit_ns says: a copy lands within microseconds, so
// the limit only matters when the consumer of a stage aborted first.
constexpr uint64_t kDrainNs = 2000000000ull;

struct Derived {
  MaskGeom geom;  // in virtual index space
  int vdil;       // 1, or d for the dilated fast path
};

int derive(const chia_attn_params_t *p, Derived &out) {
  if (p->win_left < -1 || p->win_right < -1 || p->block < 0 || p->prefix < 0 ||
      p->dilation < 1)
    return CHIA_ERR_INVALID_ARGUMENT;
  MaskGeom g{};
  g.sq = p->seqlen_q;
  g.skv = p->seqlen_kv;
  g.left = p->win_left;
  g.right = p->win_right;
  g.block = p->block;
  g.prefix = p->prefix < p->seqlen_kv ? p->prefix : p->seqlen_kv;
  g.dil = p->dilation;
  g.seg = p->seq_offsets;
  g.nseg = p->num_seqs;
  out.vdil = 1;
  const int64_t d = p->dilation;
  if (d > 1 && g.block == 0 && g.prefix == 0 && g.seg == nullptr && g.sq % d == 0 &&
      g.skv % d == 0) {
    // i = i' d + r, j = j' d + r  =>  i - j = (i' - j') d
    g.sq /= d;
    g.skv /= d;
    if (g.left >= 0) g.left /= d;
    if (g.right >= 0) g.right /= d;
    g.dil = 1;
    out.vdil = static_cast<int>(d);
  }
  out.geom = g;
  return CHIA_OK;
}

// Host-side mask geometry in REAL index space (for counting and planning).
MaskGeom real_geom(const chia_attn_params_t *p) {
  MaskGeom g{};
  g.sq = p->seqlen_q;
  g.skv = p->seqlen_kv;
  g.left = p->win_left;
  g.right = p->win_right;
  g.block = p->block;
  g.prefix = p->prefix < p->seqlen_kv ? p->prefix : p->seqlen_kv;
  g.dil = p->dilation;
  return g;
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int validate(const chia_attn_params_t *p) {
  if (p == nullptr) return CHIA_ERR_INVALID_ARGUMENT;
  if (p->abi_version != CHIA_ATTN_ABI_VERSION) return CHIA_ERR_INVALID_ARGUMENT;
  if (p->dtype != CHIA_DTYPE_BF16 && p->dtype != CHIA_DTYPE_F16) return CHIA_ERR_UNSUPPORTED;
  if (p->head_dim != 64 && p->head_dim != 128) return CHIA_ERR_UNSUPPORTED;
  if (p->norm < CHIA_NORM_SOFTMAX || p->norm > CHIA_NORM_RELU) return CHIA_ERR_INVALID_ARGUMENT;
  if (p->mod < CHIA_MOD_NONE || p->mod > CHIA_MOD_TEMP) return CHIA_ERR_INVALID_ARGUMENT;
  if (p->norm != CHIA_NORM_SOFTMAX && p->mod != CHIA_MOD_NONE) return CHIA_ERR_UNSUPPORTED;
  if (p->batch < 1 || p->heads < 1 || p->seqlen_q < 1 || p->seqlen_kv < 1)
    return CHIA_ERR_INVALID_ARGUMENT;
  if (p->heads_kv < 0 || (p->heads_kv > 0 && p->heads % p->heads_kv != 0))
    return CHIA_ERR_INVALID_ARGUMENT;
  if (p->seq_offsets != nullptr) {  // packed sequences
    if (p->num_seqs < 1 || p->num_seqs > (int64_t(1) << 30) || p->batch != 1 ||
        p->seqlen_q != p->seqlen_kv || p->seqlen_q > 0x7fffffffLL)
      return CHIA_ERR_INVALID_ARGUMENT;
    if (p->block != 0 || p->prefix != 0 || p->dilation != 1) return CHIA_ERR_UNSUPPORTED;
    if ((reinterpret_cast<uintptr_t>(p->seq_offsets) & 3u) != 0) return CHIA_ERR_MISALIGNED;
  }
  // S_q may exceed S_kv: a query row that sees no key (a window past the
  // last key) gets a zero output row, and so do whole work units of them.
  if (p->seqlen_q > (int64_t(1) << 30) || p->seqlen_kv > (int64_t(1) << 30) ||
      p->heads > (int64_t(1) << 24) || p->batch > (int64_t(1) << 24))
    return CHIA_ERR_UNSUPPORTED;
  if (!p->q || !p->k || !p->v || !p->o) return CHIA_ERR_INVALID_ARGUMENT;
  if ((p->mod == CHIA_MOD_ALIBI || p->mod == CHIA_MOD_TEMP) && p->head_param == nullptr)
    return CHIA_ERR_INVALID_ARGUMENT;
  if (p->mod == CHIA_MOD_SOFTCAP && !(p->softcap > 0.f)) return CHIA_ERR_INVALID_ARGUMENT;
  if (!std::isfinite(p->scale) || !std::isfinite(p->sig_bias) || !std::isfinite(p->out_scale))
    return CHIA_ERR_INVALID_ARGUMENT;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v) || !aligned16(p->o))
    return CHIA_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(p->workspace) & 15u) != 0) return CHIA_ERR_MISALIGNED;
  if ((reinterpret_cast<uintptr_t>(p->lse) & 3u) != 0) return CHIA_ERR_MISALIGNED;
  const int64_t *strides[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (auto *s : strides)
    for (int d = 0; d < 3; ++d) {
      if (s[d] < 0) return CHIA_ERR_INVALID_ARGUMENT;
      if (s[d] % 8 != 0) return CHIA_ERR_MISALIGNED;  // 16-byte TMA stride rule
    }
  Derived dv;
  return derive(p, dv);
}

// ----------------------------------------------------------------- TMA maps
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 5-D view (D, S', vdil, H, B) of a [B, H, S, D] tensor; box (64, box_rows,
// 1, 1, 1), 128-byte swizzle, zero fill out of bounds.
bool encode_map(CUtensorMap *map, const void *base, int dtype, int64_t D, int64_t s_virtual,
                int vdil, int64_t H, int64_t B, const int64_t *stride_el, uint32_t box_rows = 128) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[5] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(s_virtual),
                              static_cast<cuuint64_t>(vdil), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[4] = {static_cast<cuuint64_t>(stride_el[2] * vdil * 2),
                                 static_cast<cuuint64_t>(stride_el[2] * 2),
                                 static_cast<cuuint64_t>(stride_el[1] * 2),
                                 static_cast<cuuint64_t>(stride_el[0] * 2)};
  const cuuint32_t box[5] = {64, box_rows, 1, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == CHIA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // strides of size-1 dims must still be valid multiples of 16; a zero stride
  // (broadcast) is replaced by the next one, which it never affects.
  cuuint64_t st[4];
  for (int d = 0; d < 4; ++d) st[d] = strides[d] ? strides[d] : 16;
  const CUresult r = fn(map, dt, 5, const_cast<void *>(base), dims, st, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// fp32 [B, H, S, D] buffer (contiguous, real rows) viewed like encode_map
// (D, S', vdil, H, B), box (32, 128, 1, 1, 1): 128 bytes per box row, 128-byte
// swizzle. The backward pass adds its dQ tiles into it with TMA reductions.
bool encode_map_f32(CUtensorMap *map, float *base, int64_t D, int64_t s_real, int64_t s_virtual,
                    int vdil, int64_t H, int64_t B) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[5] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(s_virtual),
                              static_cast<cuuint64_t>(vdil), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t row = static_cast<cuuint64_t>(D) * 4;
  const cuuint64_t st[4] = {row * vdil, row, row * s_real, row * s_real * H};
  const cuuint32_t box[5] = {32, 128, 1, 1, 1};
  const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, base, dims, st, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ----------------------------------------------------------------- dispatch
template <int D, bool BF16, int KIND, bool SEG>
int launch_one(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
               const chia::KernelArgs &a, int64_t nblocks, cudaStream_t stream) {
  using Cfg = chia::FmhaConfig<D>;
  auto kern = chia::fmha_fwd_kernel<D, BF16, KIND, SEG>;
  static std::atomic<uint32_t> configured{0};  // bit per device ordinal (< 32)
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  const uint32_t bit = 1u << (dev & 31);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC) !=
        cudaSuccess)
      return CHIA_ERR_LAUNCH;
    // setmaxnreg.inc can only hand out registers the launch allocated: refuse
    // to run a build whose register count cannot cover the warpgroup split.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return CHIA_ERR_LAUNCH;
    if (fa.numRegs * Cfg::THREADS < 2 * 128 * Cfg::REG_SOFTMAX + 128 * Cfg::REG_OTHER)
      return CHIA_ERR_UNSUPPORTED;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  kern<<<static_cast<unsigned>(nblocks), Cfg::THREADS, Cfg::SMEM_ALLOC, stream>>>(mq, mk, mv, a);
  return cudaGetLastError() == cudaSuccess ? CHIA_OK : CHIA_ERR_LAUNCH;
}

// head_dim 128: CTA pairs with 2-SM UMMAs (fmha2_sm100.cuh)
template <bool BF16, int KIND, bool MASKED, bool SEG>
int launch_pair(const CUtensorMap &mq, const CUtensorMap &mkh, const CUtensorMap &mvh,
                const CUtensorMap &mo, const chia::KernelArgs &a, int64_t nunits,
                cudaStream_t stream) {
  using Cfg = chia::Fmha2Config<128, chia::fmha2_parts(KIND)>;
  auto kern = chia::fmha2_fwd_kernel<128, BF16, KIND, MASKED, SEG>;
  static std::atomic<uint32_t> configured{0};
  static std::atomic<int> max_pairs[32];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  const uint32_t bit = 1u << (dev & 31);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC) !=
        cudaSuccess)
      return CHIA_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
    cfg.dynamicSmemBytes = Cfg::SMEM_ALLOC;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess || clusters < 1)
      return CHIA_ERR_LAUNCH;
    max_pairs[dev & 31].store(clusters, std::memory_order_relaxed);
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int64_t pairs_max = max_pairs[dev & 31].load(std::memory_order_relaxed);
  const int64_t pairs = nunits < pairs_max ? nunits : pairs_max;
  kern<<<static_cast<unsigned>(2 * pairs), Cfg::THREADS, Cfg::SMEM_ALLOC, stream>>>(mq, mkh, mvh,
                                                                                   mo, a);
  return cudaGetLastError() == cudaSuccess ? CHIA_OK : CHIA_ERR_LAUNCH;
}

template <bool BF16, bool MASKED, bool SEG>
int launch_pair_kind(int kind, const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                     const CUtensorMap &mo, const chia::KernelArgs &a, int64_t nunits,
                     cudaStream_t s) {
  switch (kind) {
    case chia::KIND_SOFTMAX:
      return launch_pair<BF16, chia::KIND_SOFTMAX, MASKED, SEG>(mq, mk, mv, mo, a, nunits, s);
    case chia::KIND_SOFTCAP:
      return launch_pair<BF16, chia::KIND_SOFTCAP, MASKED, SEG>(mq, mk, mv, mo, a, nunits, s);
    case chia::KIND_ALIBI:
      return launch_pair<BF16, chia::KIND_ALIBI, MASKED, SEG>(mq, mk, mv, mo, a, nunits, s);
    case chia::KIND_SIGMOID:
      return launch_pair<BF16, chia::KIND_SIGMOID, MASKED, SEG>(mq, mk, mv, mo, a, nunits, s);
    case chia::KIND_RELU:
      return launch_pair<BF16, chia::KIND_RELU, MASKED, SEG>(mq, mk, mv, mo, a, nunits, s);
  }
  return CHIA_ERR_INVALID_ARGUMENT;
}

template <int D, bool BF16, bool SEG>
int launch_kind(int kind, const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                const chia::KernelArgs &a, int64_t nblocks, cudaStream_t s) {
  switch (kind) {
    case chia::KIND_SOFTMAX: return launch_one<D, BF16, chia::KIND_SOFTMAX, SEG>(mq, mk, mv, a, nblocks, s);
    case chia::KIND_SOFTCAP: return launch_one<D, BF16, chia::KIND_SOFTCAP, SEG>(mq, mk, mv, a, nblocks, s);
    case chia::KIND_ALIBI: return launch_one<D, BF16, chia::KIND_ALIBI, SEG>(mq, mk, mv, a, nblocks, s);
    case chia::KIND_SIGMOID: return launch_one<D, BF16, chia::KIND_SIGMOID, SEG>(mq, mk, mv, a, nblocks, s);
    case chia::KIND_RELU: return launch_one<D, BF16, chia::KIND_RELU, SEG>(mq, mk, mv, a, nblocks, s);
  }
  return CHIA_ERR_INVALID_ARGUMENT;
}

int kind_of(const chia_attn_params_t *p) {
  if (p->norm == CHIA_NORM_SIGMOID) return chia::KIND_SIGMOID;
  if (p->norm == CHIA_NORM_RELU) return chia::KIND_RELU;
  switch (p->mod) {
    case CHIA_MOD_SOFTCAP: return chia::KIND_SOFTCAP;
    case CHIA_MOD_ALIBI: return chia::KIND_ALIBI;
    default: return chia::KIND_SOFTMAX;  // NONE and TEMP (TEMP folds into the scale)
  }
}

// ------------------------------------------------- library-owned scratch
// Scheduler counters of chia_attn_fwd_noalloc: a file-scope device array, so
// the entry point needs no allocation. In host code `g_noalloc_scratch` is a
// stand-in for the device object, not an address; the device address is
// looked up with cudaGetSymbolAddress once per device, with it current.
static_assert(CHIA_ATTN_NOALLOC_SCRATCH_BYTES >= CHIA_ATTN_WORKSPACE_BYTES,
              "scratch must hold the scheduler workspace");
static __device__ __align__(256) int32_t g_noalloc_scratch[CHIA_ATTN_NOALLOC_SCRATCH_BYTES / 4];

constexpr int kMaxDevices = 64;
std::atomic<void *> g_noalloc_addr[kMaxDevices];
std::mutex g_noalloc_mutex;

int noalloc_scratch_addr(int dev, void **out) {
  if (dev < 0 || dev >= kMaxDevices) return CHIA_ERR_UNSUPPORTED;
  void *ptr = g_noalloc_addr[dev].load(std::memory_order_acquire);
  if (ptr == nullptr) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    ptr = g_noalloc_addr[dev].load(std::memory_order_acquire);
    if (ptr == nullptr) {
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr)
        return CHIA_ERR_LAUNCH;
      g_noalloc_addr[dev].store(ptr, std::memory_order_release);
    }
  }
  *out = ptr;
  return CHIA_OK;
}

// ------------------------------------------------------- split-KV decode
// Plan of a decode-shaped call: rows per K/V head, their padding, the key
// range all rows can see, and how it is split over CTAs.
struct DecodePlan {
  int rows, rp;
  int64_t nkvh;
  int64_t key_lo, nkeys;
  int32_t kps, splits;
  int64_t off_tickets, off_o, off_ml, bytes;  // workspace layout
};

constexpr int kDecodeMaxRows = 32;
constexpr int64_t kDecodeMaxHeads = 65535;  // batch * K/V heads (grid y)
constexpr int64_t kDecodeMaxSplits = 256;

int decode_plan(const chia_attn_params_t *p, int sms, DecodePlan &pl) {
  if (p->seq_offsets != nullptr) return CHIA_ERR_UNSUPPORTED;
  const int64_t hkv = p->heads_kv > 0 ? p->heads_kv : p->heads;
  const int64_t group = p->heads / hkv;
  if (group * p->seqlen_q > kDecodeMaxRows) return CHIA_ERR_UNSUPPORTED;
  pl.rows = static_cast<int>(group * p->seqlen_q);
  pl.rp = pl.rows <= 16 ? 16 : 32;  // MMA row tiles of 16
  pl.nkvh = p->batch * hkv;
  // key hull of rows [0, S_q): lo() and hi() do not decrease with the row
  const MaskGeom g = real_geom(p);
  int64_t lo0, hi0, lo1, hi1;
  chia::row_band(g, 0, lo0, hi0);
  chia::row_band(g, p->seqlen_q - 1, lo1, hi1);
  int64_t klo = lo0, khi = hi1;
  if (g.prefix > 0) {
    klo = 0;
    khi = khi > g.prefix - 1 ? khi : g.prefix - 1;
  }
  pl.key_lo = klo;
  pl.nkeys = khi >= klo ? khi - klo + 1 : 0;
  constexpr int TK = 64;
  const int64_t min_keys = 4 * TK;  // per split: amortises the Q load and the merge
  // at most one wave of CTAs (two per SM fit): a second, partial wave would
  // double the time; few partial results for the merge
  int64_t splits = 2 * static_cast<int64_t>(sms) / pl.nkvh;
  const int64_t by_keys = (pl.nkeys + min_keys - 1) / min_keys;
  if (splits > by_keys) splits = by_keys;
  if (splits > kDecodeMaxSplits) splits = kDecodeMaxSplits;  // the merge's weights fit in smem
  if (splits < 1) splits = 1;
  int64_t kps = (pl.nkeys + splits - 1) / splits;
  kps = (kps + TK - 1) / TK * TK;
  if (kps < TK) kps = TK;
  splits = pl.nkeys > 0 ? (pl.nkeys + kps - 1) / kps : 1;
  if (kps > 0x7fffffff || splits > kDecodeMaxSplits) return CHIA_ERR_UNSUPPORTED;
  pl.kps = static_cast<int32_t>(kps);
  pl.splits = static_cast<int32_t>(splits);
  // Workspace: the tickets first, at a fixed place and size (one per possible
  // (batch, K/V head) -- the grid's y limit), so that they stay zero whatever
  // the plans of earlier calls were; then the splits' partial results, which
  // every call overwrites.
  if (pl.nkvh > kDecodeMaxHeads) return CHIA_ERR_UNSUPPORTED;
  auto up256 = [](int64_t x) { return (x + 255) / 256 * 256; };
  const int64_t n_part = pl.nkvh * splits * pl.rp;
  pl.off_tickets = 0;
  pl.off_o = up256(kDecodeMaxHeads * 4);  // 256-byte aligned, like every region
  pl.off_ml = pl.off_o + up256(n_part * p->head_dim * 4);
  pl.bytes = pl.off_ml + up256(n_part * 2 * 4);
  // the merge reads the partial outputs as 8-byte pairs
  if ((pl.off_o | pl.off_ml) & 255) return CHIA_ERR_LAUNCH;
  return CHIA_OK;
}

template <int D, int RP, bool BF16, int KIND>
int launch_decode(const chia::DecodeArgs &a, dim3 grid, cudaStream_t s) {
  auto kern = chia::decode_kernel<D, RP, BF16, KIND>;
  constexpr int smem = chia::decode_smem_bytes<D, RP>();
  static std::atomic<uint32_t> configured{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  const uint32_t bit = 1u << (dev & 31);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return CHIA_ERR_LAUNCH;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  kern<<<grid, 128, smem, s>>>(a);
  return cudaGetLastError() == cudaSuccess ? CHIA_OK : CHIA_ERR_LAUNCH;
}

template <int D, int RP, bool BF16>
int launch_decode_kind(const chia::DecodeArgs &a, dim3 grid, cudaStream_t s) {
  switch (a.kind) {
    case chia::KIND_SOFTMAX: return launch_decode<D, RP, BF16, chia::KIND_SOFTMAX>(a, grid, s);
    case chia::KIND_SOFTCAP: return launch_decode<D, RP, BF16, chia::KIND_SOFTCAP>(a, grid, s);
    case chia::KIND_ALIBI: return launch_decode<D, RP, BF16, chia::KIND_ALIBI>(a, grid, s);
    case chia::KIND_SIGMOID: return launch_decode<D, RP, BF16, chia::KIND_SIGMOID>(a, grid, s);
    case chia::KIND_RELU: return launch_decode<D, RP, BF16, chia::KIND_RELU>(a, grid, s);
  }
  return CHIA_ERR_INVALID_ARGUMENT;
}

template <int D, bool BF16>
int launch_decode_rp(int rp, const chia::DecodeArgs &a, dim3 grid, cudaStream_t s) {
  return rp == 16 ? launch_decode_kind<D, 16, BF16>(a, grid, s)
                  : launch_decode_kind<D, 32, BF16>(a, grid, s);
}

// ------------------------------------------------------------- backward
template <int D, bool BF16, int KIND>
int launch_bwd(const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
               const CUtensorMap &mdo, const CUtensorMap &mdq, const chia::BwdArgs &a, int grid,
               cudaStream_t s) {
  using Cfg = chia::BwdConfig<D>;
  auto kern = chia::fmha_bwd_kernel<D, BF16, KIND>;
  static std::atomic<uint32_t> configured{0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  const uint32_t bit = 1u << (dev & 31);
  if (!(configured.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_ALLOC) !=
        cudaSuccess)
      return CHIA_ERR_LAUNCH;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  kern<<<grid, Cfg::THREADS, Cfg::SMEM_ALLOC, s>>>(mq, mk, mv, mdo, mdq, a);
  return cudaGetLastError() == cudaSuccess ? CHIA_OK : CHIA_ERR_LAUNCH;
}

template <int D, bool BF16>
int launch_bwd_kind(int kind, const CUtensorMap &mq, const CUtensorMap &mk, const CUtensorMap &mv,
                    const CUtensorMap &mdo, const CUtensorMap &mdq, const chia::BwdArgs &a,
                    int grid, cudaStream_t s) {
  switch (kind) {
    case chia::KIND_SOFTMAX:
      return launch_bwd<D, BF16, chia::KIND_SOFTMAX>(mq, mk, mv, mdo, mdq, a, grid, s);
    case chia::KIND_SOFTCAP:
      return launch_bwd<D, BF16, chia::KIND_SOFTCAP>(mq, mk, mv, mdo, mdq, a, grid, s);
    case chia::KIND_ALIBI:
      return launch_bwd<D, BF16, chia::KIND_ALIBI>(mq, mk, mv, mdo, mdq, a, grid, s);
    case chia::KIND_SIGMOID:
      return launch_bwd<D, BF16, chia::KIND_SIGMOID>(mq, mk, mv, mdo, mdq, a, grid, s);
    case chia::KIND_RELU:
      return launch_bwd<D, BF16, chia::KIND_RELU>(mq, mk, mv, mdo, mdq, a, grid, s);
  }
  return CHIA_ERR_INVALID_ARGUMENT;
}

struct BwdLayout {
  int64_t rows, off_dq, bytes;
};

BwdLayout bwd_layout(const chia_attn_params_t *p) {
  BwdLayout l;
  l.rows = p->batch * p->heads * p->seqlen_q;
  auto up256 = [](int64_t x) { return (x + 255) / 256 * 256; };
  l.off_dq = up256(l.rows * 4);                       // delta
  l.bytes = l.off_dq + up256(l.rows * p->head_dim * 4);  // fp32 dq accumulator
  return l;
}

bool strides_ok(const int64_t *st) {
  for (int d = 0; d < 3; ++d)
    if (st[d] < 0 || st[d] % 8 != 0) return false;
  return true;
}

}  // namespace

extern "C" {

int64_t chia_attn_bwd_workspace_bytes(const chia_attn_params_t *p) {
  if (validate(p) != CHIA_OK) return -1;
  return bwd_layout(p).bytes;
}

int chia_attn_bwd(const chia_attn_params_t *p, const chia_attn_grads_t *gr, void *workspace,
                  int64_t workspace_bytes, void *stream) {
  const int v = validate(p);
  if (v != CHIA_OK) return v;
  if (gr == nullptr || !gr->dout || !gr->dq || !gr->dk || !gr->dv) return CHIA_ERR_INVALID_ARGUMENT;
  if (p->seq_offsets != nullptr) return CHIA_ERR_UNSUPPORTED;
  if (p->norm == CHIA_NORM_SOFTMAX && p->lse == nullptr) return CHIA_ERR_INVALID_ARGUMENT;
  if (!aligned16(gr->dout) || !aligned16(gr->dq) || !aligned16(gr->dk) || !aligned16(gr->dv))
    return CHIA_ERR_MISALIGNED;
  if (!strides_ok(gr->dout_stride) || !strides_ok(gr->dq_stride) || !strides_ok(gr->dk_stride) ||
      !strides_ok(gr->dv_stride))
    return CHIA_ERR_MISALIGNED;
  const BwdLayout lay = bwd_layout(p);
  if (workspace == nullptr || workspace_bytes < lay.bytes) return CHIA_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return CHIA_ERR_MISALIGNED;
  int dev = 0, major = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return CHIA_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return CHIA_ERR_NO_DEVICE;

  Derived dv;
  derive(p, dv);
  const MaskGeom &g = dv.geom;
  const int D = p->head_dim;
  const int64_t hkv = p->heads_kv > 0 ? p->heads_kv : p->heads;
  const bool bf16 = p->dtype == CHIA_DTYPE_BF16;
  const int kind = kind_of(p);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  float *delta = reinterpret_cast<float *>(ws);
  float *dq_acc = reinterpret_cast<float *>(ws + lay.off_dq);

  // 1. delta = rowsum(dout * o) (softmax kinds) and a zeroed dq accumulator
  {
    const int64_t blocks = (lay.rows * 32 + 255) / 256;
    if (blocks > 0x7fffffffLL) return CHIA_ERR_UNSUPPORTED;
    const bool want = p->norm == CHIA_NORM_SOFTMAX;
#define CHIA_PREP(DD, BB)                                                                        \
  chia::bwd_prep_kernel<DD, BB><<<static_cast<unsigned>(blocks), 256, 0, s>>>(                    \
      p->o, gr->dout, p->o_stride[0], p->o_stride[1], p->o_stride[2], gr->dout_stride[0],        \
      gr->dout_stride[1], gr->dout_stride[2], static_cast<int32_t>(p->heads), p->seqlen_q, delta, \
      dq_acc, lay.rows, want)
    if (D == 128) {
      if (bf16) CHIA_PREP(128, true); else CHIA_PREP(128, false);
    } else {
      if (bf16) CHIA_PREP(64, true); else CHIA_PREP(64, false);
    }
#undef CHIA_PREP
    if (cudaGetLastError() != cudaSuccess) return CHIA_ERR_LAUNCH;
  }
  // 2. the tensor-core kernel
  CUtensorMap mq, mk, mv, mdo, mdq;
  if (!encode_map(&mq, p->q, p->dtype, D, g.sq, dv.vdil, p->heads, p->batch, p->q_stride) ||
      !encode_map(&mk, p->k, p->dtype, D, g.skv, dv.vdil, hkv, p->batch, p->k_stride) ||
      !encode_map(&mv, p->v, p->dtype, D, g.skv, dv.vdil, hkv, p->batch, p->v_stride) ||
      !encode_map(&mdo, gr->dout, p->dtype, D, g.sq, dv.vdil, p->heads, p->batch,
                  gr->dout_stride) ||
      !encode_map_f32(&mdq, dq_acc, D, p->seqlen_q, g.sq, dv.vdil, p->heads, p->batch))
    return CHIA_ERR_LAUNCH;
  chia::BwdArgs a{};
  a.mask = g;
  a.heads = static_cast<int32_t>(p->heads);
  a.heads_kv = static_cast<int32_t>(hkv);
  a.group = static_cast<int32_t>(p->heads / hkv);
  a.vdil = dv.vdil;
  const int64_t n_qt = (g.sq + 127) / 128, n_kt = (g.skv + 127) / 128;
  const int64_t n_units = n_kt * p->batch * hkv * dv.vdil;
  if (n_units > 0x7fffffffLL || n_qt > 0x7fffffffLL) return CHIA_ERR_UNSUPPORTED;
  a.n_qt = static_cast<int32_t>(n_qt);
  a.n_kt = static_cast<int32_t>(n_kt);
  a.n_units = static_cast<int32_t>(n_units);
  a.score_scale = p->scale;
  a.softcap = p->softcap;
  a.sig_bias = p->sig_bias;
  a.out_scale = p->out_scale;
  a.head_param = (p->mod == CHIA_MOD_ALIBI || p->mod == CHIA_MOD_TEMP) ? p->head_param : nullptr;
  a.lse = p->lse;
  a.delta = delta;
  a.dq_acc = dq_acc;
  a.dk = gr->dk;
  a.dv = gr->dv;
  a.dk_sb = gr->dk_stride[0]; a.dk_sh = gr->dk_stride[1]; a.dk_ss = gr->dk_stride[2];
  a.dv_sb = gr->dv_stride[0]; a.dv_sh = gr->dv_stride[1]; a.dv_ss = gr->dv_stride[2];
  a.sq_real = p->seqlen_q;
  a.status = p->status;
  a.timeout_ns = p->wait_limit_ns > 0 ? p->wait_limit_ns : kDefaultTimeoutNs;
  a.drain_ns = kDrainNs;
  const int grid = static_cast<int>(n_units < sms ? n_units : sms);
  int r;
  if (D == 128)
    r = bf16 ? launch_bwd_kind<128, true>(kind, mq, mk, mv, mdo, mdq, a, grid, s)
             : launch_bwd_kind<128, false>(kind, mq, mk, mv, mdo, mdq, a, grid, s);
  else
    r = bf16 ? launch_bwd_kind<64, true>(kind, mq, mk, mv, mdo, mdq, a, grid, s)
             : launch_bwd_kind<64, false>(kind, mq, mk, mv, mdo, mdq, a, grid, s);
  if (r != CHIA_OK) return r;
  // 3. dq = the fp32 accumulator rounded to the input type
  {
    const int64_t blocks = (lay.rows * 32 + 255) / 256;
#define CHIA_DQ(DD, BB)                                                                   \
  chia::bwd_dq_kernel<DD, BB><<<static_cast<unsigned>(blocks), 256, 0, s>>>(               \
      dq_acc, gr->dq, gr->dq_stride[0], gr->dq_stride[1], gr->dq_stride[2],                \
      static_cast<int32_t>(p->heads), p->seqlen_q, lay.rows)
    if (D == 128) {
      if (bf16) CHIA_DQ(128, true); else CHIA_DQ(128, false);
    } else {
      if (bf16) CHIA_DQ(64, true); else CHIA_DQ(64, false);
    }
#undef CHIA_DQ
    if (cudaGetLastError() != cudaSuccess) return CHIA_ERR_LAUNCH;
  }
  return CHIA_OK;
}

int64_t chia_attn_decode_workspace_bytes(const chia_attn_params_t *p) {
  if (validate(p) != CHIA_OK) return -1;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    sms = 148;  // host-only callers (no GPU): size for a B200
  DecodePlan pl;
  if (decode_plan(p, sms, pl) != CHIA_OK) return -1;
  return pl.bytes;
}

int chia_attn_decode(const chia_attn_params_t *p, void *workspace, int64_t workspace_bytes,
                     void *stream) {
  const int v = validate(p);
  if (v != CHIA_OK) return v;
  int dev = 0, major = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return CHIA_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return CHIA_ERR_NO_DEVICE;
  DecodePlan pl;
  const int r = decode_plan(p, sms, pl);
  if (r != CHIA_OK) return r;
  if (workspace == nullptr || workspace_bytes < pl.bytes) return CHIA_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return CHIA_ERR_MISALIGNED;
  chia::DecodeArgs a{};
  a.q = p->q;
  a.k = p->k;
  a.v = p->v;
  a.o = p->o;
  a.q_sb = p->q_stride[0]; a.q_sh = p->q_stride[1]; a.q_ss = p->q_stride[2];
  a.k_sb = p->k_stride[0]; a.k_sh = p->k_stride[1]; a.k_ss = p->k_stride[2];
  a.v_sb = p->v_stride[0]; a.v_sh = p->v_stride[1]; a.v_ss = p->v_stride[2];
  a.o_sb = p->o_stride[0]; a.o_sh = p->o_stride[1]; a.o_ss = p->o_stride[2];
  const int64_t hkv = p->heads_kv > 0 ? p->heads_kv : p->heads;
  a.heads = static_cast<int32_t>(p->heads);
  a.heads_kv = static_cast<int32_t>(hkv);
  a.group = static_cast<int32_t>(p->heads / hkv);
  a.sq = static_cast<int32_t>(p->seqlen_q);
  a.rows = pl.rows;
  a.kind = kind_of(p);
  a.mask = real_geom(p);
  a.key_lo = pl.key_lo;
  a.keys_per_split = pl.kps;
  a.splits = pl.splits;
  a.score_scale = p->scale;
  a.softcap = p->softcap;
  a.sig_bias = p->sig_bias;
  a.out_scale = p->out_scale;
  a.head_param = (p->mod == CHIA_MOD_ALIBI || p->mod == CHIA_MOD_TEMP) ? p->head_param : nullptr;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  a.tickets = reinterpret_cast<int32_t *>(ws + pl.off_tickets);
  a.part_o = reinterpret_cast<float *>(ws + pl.off_o);
  a.part_ml = reinterpret_cast<float *>(ws + pl.off_ml);
  a.lse = p->norm == CHIA_NORM_SOFTMAX ? p->lse : nullptr;
  const dim3 grid(static_cast<unsigned>(pl.splits), static_cast<unsigned>(pl.nkvh));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool bf16 = p->dtype == CHIA_DTYPE_BF16;
  if (p->head_dim == 128)
    return bf16 ? launch_decode_rp<128, true>(pl.rp, a, grid, s)
                : launch_decode_rp<128, false>(pl.rp, a, grid, s);
  return bf16 ? launch_decode_rp<64, true>(pl.rp, a, grid, s)
              : launch_decode_rp<64, false>(pl.rp, a, grid, s);
}


int chia_attn_abi_version(void) { return CHIA_ATTN_ABI_VERSION; }

#ifdef CHIA_TRACE
// Trace builds only (not part of the public ABI): copy the timeline buffer
// of the last traced launch to host memory and clear it; returns bytes copied.
__attribute__((visibility("default"))) long chia_attn_trace_read(void *dst, long bytes) {
  const long n = bytes < static_cast<long>(sizeof(chia::g_chia_trace))
                     ? bytes : static_cast<long>(sizeof(chia::g_chia_trace));
  if (cudaMemcpyFromSymbol(dst, chia::g_chia_trace, n) != cudaSuccess) return -1;
  void *sym = nullptr;
  if (cudaGetSymbolAddress(&sym, chia::g_chia_trace) != cudaSuccess ||
      cudaMemset(sym, 0, sizeof(chia::g_chia_trace)) != cudaSuccess)
    return -1;
  return n;
}
#endif

const char *chia_attn_status_string(int status) {
  switch (status) {
    case CHIA_OK: return "ok";
    case CHIA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CHIA_ERR_UNSUPPORTED: return "unsupported configuration";
    case CHIA_ERR_MISALIGNED: return "pointer or stride not 16-byte aligned";
    case CHIA_ERR_LAUNCH: return "kernel launch or tensor-map encoding failed";
    case CHIA_ERR_DEVICE_TIMEOUT: return "bounded device wait expired";
    case CHIA_ERR_NO_DEVICE: return "no usable sm_100 device";
  }
  return "unknown status";
}

int64_t chia_attn_visible_pairs(const chia_attn_params_t *p) {
  if (p == nullptr || p->seq_offsets != nullptr || p->seqlen_q < 0 || p->seqlen_kv < 0 ||
      p->win_left < -1 ||
      p->win_right < -1 || p->block < 0 || p->prefix < 0 || p->dilation < 1)
    return -1;
  return chia::visible_pairs(real_geom(p));
}

int chia_attn_tile_plan(const chia_attn_params_t *p, int64_t row0, int32_t tile_m,
                        int32_t tile_n, int64_t *tile_lo, int64_t *tile_hi,
                        uint64_t *full_mask) {
  if (p == nullptr || tile_m < 1 || tile_n < 1 || !tile_lo || !tile_hi || !full_mask || row0 < 0)
    return CHIA_ERR_INVALID_ARGUMENT;
  if (p->seq_offsets != nullptr) return CHIA_ERR_UNSUPPORTED;  // device memory
  if (p->seqlen_q < 1 || p->seqlen_kv < 1 || p->win_left < -1 || p->win_right < -1 ||
      p->block < 0 || p->prefix < 0 || p->dilation < 1)
    return CHIA_ERR_INVALID_ARGUMENT;
  const MaskGeom g = real_geom(p);
  int64_t lo, hi;
  chia::tile_range(g, row0, row0 + tile_m - 1, tile_n, lo, hi);
  uint64_t m = 0;
  const chia::FullTiles ft = chia::full_tiles(g, row0, row0 + tile_m - 1, tile_n);
  for (int64_t t = lo; t < hi && t - lo < 64; ++t)
    if (ft.full(t)) m |= 1ull << (t - lo);
  *tile_lo = lo;
  *tile_hi = hi;
  *full_mask = m;
  return CHIA_OK;
}

int chia_attn_fwd(const chia_attn_params_t *p, void *stream) {
  const int v = validate(p);
  if (v != CHIA_OK) return v;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return CHIA_ERR_NO_DEVICE;

  Derived dv;
  derive(p, dv);
  const MaskGeom &g = dv.geom;
  const int D = p->head_dim;
  CUtensorMap mq, mk, mv;
  const int64_t hkv = p->heads_kv > 0 ? p->heads_kv : p->heads;  // K/V heads
  if (!encode_map(&mq, p->q, p->dtype, D, g.sq, dv.vdil, p->heads, p->batch, p->q_stride) ||
      !encode_map(&mk, p->k, p->dtype, D, g.skv, dv.vdil, hkv, p->batch, p->k_stride) ||
      !encode_map(&mv, p->v, p->dtype, D, g.skv, dv.vdil, hkv, p->batch, p->v_stride))
    return CHIA_ERR_LAUNCH;

  chia::KernelArgs a{};
  a.mask = g;
  a.heads = static_cast<int32_t>(p->heads);
  a.group = static_cast<int32_t>(p->heads / hkv);
  a.vdil = dv.vdil;
  const int64_t rows_per_unit = 2 * 128;
  const int64_t nqb = (g.sq + rows_per_unit - 1) / rows_per_unit;
  const int64_t nvh = p->batch * p->heads * dv.vdil;
  const int64_t nunits = nqb * nvh;
  if (nunits > 0x7fffffffLL) return CHIA_ERR_UNSUPPORTED;
  a.n_qblocks = static_cast<int32_t>(nqb);
  a.n_vheads = static_cast<int32_t>(nvh);
  a.n_units = static_cast<int32_t>(nunits);
  a.sched = static_cast<int32_t *>(p->workspace);
  // persistent grid: one CTA per SM (shared memory admits no more)
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
    return CHIA_ERR_NO_DEVICE;
  const int64_t nblocks = nunits < sms ? nunits : sms;
  a.score_scale = p->scale;
  a.softcap = p->softcap;
  a.sig_bias = p->sig_bias;
  a.out_scale = p->out_scale;
  a.head_param = (p->mod == CHIA_MOD_ALIBI || p->mod == CHIA_MOD_TEMP) ? p->head_param : nullptr;
  a.o = p->o;
  a.o_sb = p->o_stride[0];
  a.o_sh = p->o_stride[1];
  a.o_ss = p->o_stride[2];
  a.status = p->status;
  a.timeout_ns = p->wait_limit_ns > 0 ? p->wait_limit_ns : kDefaultTimeoutNs;
  a.drain_ns = kDrainNs;
  a.lse = p->norm == CHIA_NORM_SOFTMAX ? p->lse : nullptr;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int kind = kind_of(p);
  const bool bf16 = p->dtype == CHIA_DTYPE_BF16;
  if (D == 128) {
    // K in half tiles of 64 keys (one per CTA of the pair); V as loaded above
    // (box of 128 keys x 64 columns; each CTA takes one column chunk)
    CUtensorMap mkh, mo;
    if (!encode_map(&mkh, p->k, p->dtype, D, g.skv, dv.vdil, hkv, p->batch, p->k_stride, 64))
      return CHIA_ERR_LAUNCH;
    // output through TMA stores, in the same 5-D view as Q
    if (!encode_map(&mo, p->o, p->dtype, D, g.sq, dv.vdil, p->heads, p->batch, p->o_stride))
      return CHIA_ERR_LAUNCH;
    // every tile of every unit fully visible: the kernel without mask code
    const bool all_full = g.left < 0 && g.right < 0 && g.block == 0 && g.dil == 1 &&
                          g.seg == nullptr && g.skv % 128 == 0;
    if (all_full)
      return bf16 ? launch_pair_kind<true, false, false>(kind, mq, mkh, mv, mo, a, nunits, s)
                  : launch_pair_kind<false, false, false>(kind, mq, mkh, mv, mo, a, nunits, s);
    if (g.seg != nullptr)  // packed sequences: the instantiation with the sequence lookup
      return bf16 ? launch_pair_kind<true, true, true>(kind, mq, mkh, mv, mo, a, nunits, s)
                  : launch_pair_kind<false, true, true>(kind, mq, mkh, mv, mo, a, nunits, s);
    return bf16 ? launch_pair_kind<true, true, false>(kind, mq, mkh, mv, mo, a, nunits, s)
                : launch_pair_kind<false, true, false>(kind, mq, mkh, mv, mo, a, nunits, s);
  }
  if (g.seg != nullptr)
    return bf16 ? launch_kind<64, true, true>(kind, mq, mk, mv, a, nblocks, s)
                : launch_kind<64, false, true>(kind, mq, mk, mv, a, nblocks, s);
  return bf16 ? launch_kind<64, true, false>(kind, mq, mk, mv, a, nblocks, s)
              : launch_kind<64, false, false>(kind, mq, mk, mv, a, nblocks, s);
}

int chia_attn_fwd_noalloc(const chia_attn_params_t *p, void *stream) {
  const int v = validate(p);
  if (v != CHIA_OK) return v;
  if (p->workspace != nullptr) return CHIA_ERR_INVALID_ARGUMENT;
  Derived dv;
  derive(p, dv);
  const int64_t units = (dv.geom.sq + 255) / 256 * p->batch * p->heads * dv.vdil;
  if (units > CHIA_ATTN_NOALLOC_MAX_UNITS) return CHIA_ERR_UNSUPPORTED;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHIA_ERR_NO_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return CHIA_ERR_NO_DEVICE;
  void *scratch = nullptr;
  const int r = noalloc_scratch_addr(dev, &scratch);
  if (r != CHIA_OK) return r;
  // The counters must start at zero; a call that ended early (device timeout)
  // may have left them set, so clear them on the stream before every launch.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, CHIA_ATTN_WORKSPACE_BYTES, s) != cudaSuccess)
    return CHIA_ERR_LAUNCH;
  chia_attn_params_t q = *p;
  q.workspace = scratch;
  return chia_attn_fwd(&q, stream);
}

}  // extern "C"
