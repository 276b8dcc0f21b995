/*
 * chia_attn.h -- C ABI of the B200 (sm_100a) attention-variant library.
 *
 * One entry point, chia_attn_fwd(), runs the forward pass of any of the ten
 * attention operators that JoshiP-commits/CHIA_proj ("GraphSynth") defines as
 * eager PyTorch functions and benchmarks as Triton plugins. In the reference
 * every operator is a Python module exposing
 *
 *     launch_kernel(q, k, v) -> out                (extra_bench.py:24-27, :119)
 *
 * whose semantics are fixed by the eager closures of build_refs()
 * (extra_bench.py:32-62; corrected sigmoid in sigmoid_fix.py:34-40). The
 * reference has no compiled FFI of its own; this header is the binding a
 * ctypes / cffi / C++ caller uses in place of those Python plugins. It takes
 * plain device pointers, sizes and strides -- no framework types.
 *
 * Operator = score modification + mask + normaliser, all expressed as fields
 * of chia_attn_params_t:
 *
 *   op (reference)        norm     mod      mask fields                 ref file:line
 *   softcap_gemma2        SOFTMAX  SOFTCAP  causal (win_left=-1,right=0) extra_bench.py:60
 *   bias_sliding_window   SOFTMAX  NONE     left=W-1, right=0            extra_bench.py:61
 *   bias_local            SOFTMAX  NONE     left=W-1, right=W-1          extra_bench.py:57
 *   bias_alibi            SOFTMAX  ALIBI    causal; head_param = slopes  extra_bench.py:47-50
 *   bias_block_diagonal   SOFTMAX  NONE     causal, block=512            extra_bench.py:58
 *   bias_dilated          SOFTMAX  NONE     causal, dilation=4           extra_bench.py:56
 *   bias_prefix_lm        SOFTMAX  NONE     causal, prefix=256           extra_bench.py:59
 *   temp_perhead          SOFTMAX  TEMP     causal; head_param = temps   extra_bench.py:35,54
 *   sigmoid_attn          SIGMOID  NONE     causal; sig_bias             sigmoid_fix.py:34-40
 *   relu_attn             RELU     NONE     causal; out_scale            extra_bench.py:44
 *
 * Visibility of key j for query i (all integer arithmetic):
 *   vis = (j < prefix) ||
 *         ( (win_left  < 0 || i - j <= win_left)  &&
 *           (win_right < 0 || j - i <= win_right) &&
 *           (block == 0 || i / block == j / block) &&
 *           ((i - j) % dilation == 0) )
 *   and always j < seqlen_kv.
 *
 * Threading: chia_attn_fwd() is asynchronous on `stream` (a cudaStream_t),
 * never synchronises, keeps no mutable global state, and is safe to call
 * from several host threads.
 */
#ifndef CHIA_ATTN_H
#define CHIA_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CHIA_API __attribute__((visibility("default")))
#else
#define CHIA_API
#endif

#define CHIA_ATTN_ABI_VERSION 4

/* Size of the optional scheduler workspace (bytes). */
#define CHIA_ATTN_WORKSPACE_BYTES 256

/* element types of q, k, v, o (all four share one type) */
enum chia_dtype { CHIA_DTYPE_BF16 = 0, CHIA_DTYPE_F16 = 1 };

/* row normaliser applied to the (modified, masked) scores */
enum chia_norm {
  CHIA_NORM_SOFTMAX = 0, /* softmax over visible keys                    */
  CHIA_NORM_SIGMOID = 1, /* sigmoid(s + sig_bias) * vis                  */
  CHIA_NORM_RELU = 2     /* relu(s) * vis, output multiplied by out_scale */
};

/* score modification applied to s = (q.k) * scale before masking */
enum chia_mod {
  CHIA_MOD_NONE = 0,
  CHIA_MOD_SOFTCAP = 1, /* s -> softcap * tanh(s / softcap)             */
  CHIA_MOD_ALIBI = 2,   /* s -> s + head_param[h] * (j - i)             */
  CHIA_MOD_TEMP = 3     /* s -> s * head_param[h]                       */
};

/* status codes returned by chia_attn_fwd and written to *status */
enum chia_status {
  CHIA_OK = 0,
  CHIA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, bad enum        */
  CHIA_ERR_UNSUPPORTED = 2,      /* head_dim / dtype / layout not supported */
  CHIA_ERR_MISALIGNED = 3,       /* pointer or stride not 16-byte aligned   */
  CHIA_ERR_LAUNCH = 4,           /* CUDA launch / tensor-map encode failed  */
  CHIA_ERR_DEVICE_TIMEOUT = 5,   /* a bounded in-kernel wait expired        */
  CHIA_ERR_NO_DEVICE = 6         /* no sm_100 device / driver entry point   */
};

typedef struct chia_attn_params {
  int32_t abi_version; /* must be CHIA_ATTN_ABI_VERSION                     */
  int32_t dtype;       /* enum chia_dtype                                   */
  int32_t head_dim;    /* D: 64 or 128                                      */
  int32_t norm;        /* enum chia_norm                                    */
  int32_t mod;         /* enum chia_mod                                     */
  int32_t heads_kv;    /* K/V heads (grouped-query attention): q head h
                          reads K/V head h / (heads / heads_kv); must divide
                          heads; 0 = heads. No counterpart in the reference,
                          whose operators take K/V with all H heads.        */

  int64_t batch;     /* B                                                  */
  int64_t heads;     /* H                                                  */
  int64_t seqlen_q;  /* S_q  (the reference operators use S_q == S_kv; a
                        row that sees no key gets a zero output row)    */
  int64_t seqlen_kv; /* S_kv                                               */

  /* device pointers, layout [B, H, S, D] with unit stride on D; strides in
   * ELEMENTS for (batch, head, seq); all must be multiples of 8 elements and
   * the pointers 16-byte aligned */
  const void *q;
  const void *k;
  const void *v;
  void *o;
  int64_t q_stride[3];
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];

  float scale;     /* multiplies q.k; reference: 1/sqrt(D)             */
  float softcap;   /* CHIA_MOD_SOFTCAP cap (reference 30)               */
  float sig_bias;  /* CHIA_NORM_SIGMOID additive bias (reference 0)     */
  float out_scale; /* CHIA_NORM_RELU output multiplier (reference 1)    */
  const float *head_param; /* device fp32 [heads]: ALiBi slopes or TEMP  */

  /* mask (see visibility rule above); -1 = unbounded */
  int64_t win_left;
  int64_t win_right;
  int64_t block;    /* 0 = no block structure                          */
  int64_t prefix;   /* keys j < prefix always visible; 0 = none        */
  int64_t dilation; /* >= 1                                            */

  int32_t *status; /* optional device int32; in-kernel errors are OR-ed in
                      (CHIA_ERR_DEVICE_TIMEOUT); caller zeroes it       */

  /* optional device buffer of CHIA_ATTN_WORKSPACE_BYTES, zero-filled before
   * its first use. It holds the counters of the load-balancing work
   * scheduler; every call leaves it zeroed again. Calls that share one
   * workspace must not run concurrently on the GPU. NULL selects a static
   * round-robin schedule (no scratch memory at all). */
  void *workspace;

  /* Variable-length packed sequences: NULL, or a device int32 array of
   * num_seqs + 1 cumulative offsets (0 = offsets[0] <= ... <=
   * offsets[num_seqs] = seqlen_q; the array is read on the device only). Sequence s occupies rows and keys [offsets[s], offsets[s+1])
   * of a batch of 1 with seqlen_q == seqlen_kv, and query i sees only keys of
   * its own sequence (then the window rules above, with the same i - j).
   * Requires block == 0, prefix == 0, dilation == 1. No counterpart in the
   * reference, whose operators take one fixed length per batch. */
  const int32_t *seq_offsets;
  int64_t num_seqs;

  /* Optional device fp32 [batch, heads, seqlen_q] (contiguous, 4-byte
   * aligned): for CHIA_NORM_SOFTMAX the natural log-sum-exp of each row's
   * modified, masked scores, ln sum_j exp(s_ij) (-inf for a row that sees no
   * key); the backward pass reads it. Ignored for the sigmoid and ReLU
   * normalisers. NULL = not written. The reference's eager functions do not
   * return it. */
  float *lse;

  /* Limit of each in-kernel wait, in nanoseconds; 0 = the default (2 s). A
   * wait that runs out ORs CHIA_ERR_DEVICE_TIMEOUT into *status and the
   * kernel returns early, with its outputs unspecified; waits for the
   * kernel's own copies and MMAs before it exits keep the default limit.
   * Small values exist so that a test can make a wait run out. */
  uint64_t wait_limit_ns;
} chia_attn_params_t;

/* Forward attention on `stream` (cudaStream_t; NULL = legacy default
 * stream). Replaces the reference's launch_kernel(q, k, v)
 * (extra_bench.py:24-27 loads it; e.g. kernels_gemini31propre_0018/
 * softcap_gemma2_BEST.py:93-122 defines it) and its eager specification
 * build_refs() (extra_bench.py:32-62). Returns enum chia_status; argument
 * errors are reported before anything is launched. */
CHIA_API int chia_attn_fwd(const chia_attn_params_t *params, void *stream);

/* Size of the library-owned scratch used by chia_attn_fwd_noalloc, and the
 * largest problem it accepts, counted in work units of 256 query rows of one
 * (batch, head) pair: ceil(seqlen_q / 256) * batch * heads (times dilation
 * when seqlen_q and seqlen_kv are multiples of it and block == prefix == 0). */
#define CHIA_ATTN_NOALLOC_SCRATCH_BYTES 256
#define CHIA_ATTN_NOALLOC_MAX_UNITS (1 << 30)

/* chia_attn_fwd for callers that cannot allocate device memory. No
 * counterpart in the reference: its launch_kernel(q, k, v) allocates its own
 * output with torch. A plugin host or FFI caller that owns all device memory
 * and keeps no per-device state between calls has nowhere to keep the
 * scheduler workspace, and cudaMalloc on every call would synchronise the
 * device. This entry point takes params->workspace == NULL (anything else is
 * CHIA_ERR_INVALID_ARGUMENT) and schedules with a file-scope device array of
 * CHIA_ATTN_NOALLOC_SCRATCH_BYTES instead, which every GPU that loads the
 * library holds until the process exits. It calls no cudaMalloc, cudaFree or
 * other allocating routine; it zeroes the array on `stream` before the
 * launch. Problems of more than CHIA_ATTN_NOALLOC_MAX_UNITS work units return
 * CHIA_ERR_UNSUPPORTED before anything is enqueued. The first call on a
 * device looks up the array's device address (with that device current), so
 * make that first call before any stream capture. All calls on one device
 * share the array: calls that overlap on the GPU (different streams, no
 * ordering between them) race on it and may compute wrong outputs. Inputs,
 * output, status and all other fields are as for chia_attn_fwd. */
CHIA_API int chia_attn_fwd_noalloc(const chia_attn_params_t *params, void *stream);

/* Split-KV forward for decode-shaped calls: few query rows per K/V head
 * (heads / heads_kv * seqlen_q <= 32, e.g. one new token of a grouped-query
 * model) over a long key sequence. Same fields, same visibility rule and
 * score modifications as chia_attn_fwd, and the same output (plus lse when
 * given); seq_offsets must be NULL and params->workspace is ignored. The key
 * range is split over many CTAs, each reading its keys and values once; the
 * last CTA of each K/V head merges the splits' partial results. The
 * reference has no counterpart: its operators take S_q == S_kv; this is the
 * decode step of the same operators (Gemma-2 style softcap + sliding window
 * included).
 *
 * workspace: device memory of at least chia_attn_decode_workspace_bytes()
 * bytes, 256-byte aligned, zero-filled before its first use. Its first
 * 256 KiB hold the merge counters, which every call leaves zeroed again, so
 * one workspace serves calls of any shape that fit in it. Calls that share a
 * workspace must not overlap on the GPU. Returns CHIA_ERR_UNSUPPORTED for
 * calls outside the decode shape (the caller then uses chia_attn_fwd) and
 * for more than 65535 (batch, K/V head) pairs. */
CHIA_API int chia_attn_decode(const chia_attn_params_t *params, void *workspace,
                              int64_t workspace_bytes, void *stream);

/* Workspace bytes chia_attn_decode needs for params on the current device
 * (host-only arithmetic); -1 when params are invalid or not decode-shaped. */
CHIA_API int64_t chia_attn_decode_workspace_bytes(const chia_attn_params_t *params);

/* Gradient tensors of chia_attn_bwd: [B, H, S, D] like q, k, v, o (K/V
 * gradients with heads_kv heads), 16-bit of params->dtype, unit stride on D,
 * strides in elements, multiples of 8; pointers 16-byte aligned. */
typedef struct chia_attn_grads {
  const void *dout;     /* upstream gradient of the output o           */
  int64_t dout_stride[3];
  void *dq;             /* written: gradient of q                      */
  void *dk;             /* written: gradient of k                      */
  void *dv;             /* written: gradient of v                      */
  int64_t dq_stride[3];
  int64_t dk_stride[3];
  int64_t dv_stride[3];
} chia_attn_grads_t;

/* Backward pass of chia_attn_fwd: dq, dk, dv for the same params (q, k, v,
 * the forward's output in params->o and, for CHIA_NORM_SOFTMAX, the
 * forward's log-sum-exp in params->lse). Every score modification, mask and
 * normaliser of chia_attn_fwd, grouped K/V heads (dk, dv summed over the
 * query heads of a group) and the dilated residue-class path; packed
 * sequences (seq_offsets) return CHIA_ERR_UNSUPPORTED. The reference is
 * forward only (README.md); the gradients are those of its eager functions
 * (extra_bench.py:32-62, sigmoid_fix.py:34-40) differentiated exactly, with
 * P and dS rounded to the input type for the tensor cores.
 *
 * workspace: device memory of chia_attn_bwd_workspace_bytes() bytes,
 * 256-byte aligned, no initial contents needed (fp32 dq accumulator and
 * the row sums of dout * o). Calls that share a workspace must not overlap
 * on the GPU. */
CHIA_API int chia_attn_bwd(const chia_attn_params_t *params, const chia_attn_grads_t *grads,
                           void *workspace, int64_t workspace_bytes, void *stream);

/* Workspace bytes of chia_attn_bwd (host-only); -1 for invalid params. */
CHIA_API int64_t chia_attn_bwd_workspace_bytes(const chia_attn_params_t *params);

/* Number of visible (i, j) pairs of the mask described by params for one
 * (batch, head) pair -- the mask-aware FLOP count is 4 * D * pairs * B * H.
 * Host-only integer arithmetic; needs no GPU. Returns -1 on bad params and
 * for packed sequences (seq_offsets is device memory). */
CHIA_API int64_t chia_attn_visible_pairs(const chia_attn_params_t *params);

/* Key-tile plan of one query tile, the schedule the kernel runs. For query
 * rows [row0, row0 + tile_m) writes the first and one-past-last key tile of
 * width tile_n it visits and, into full_mask (bit t set = tile t needs no
 * element-wise masking; up to 64 tiles), which of them are unmasked.
 * Host-only; lets tests check the schedule without a GPU. Returns status
 * (CHIA_ERR_UNSUPPORTED for packed sequences). */
CHIA_API int chia_attn_tile_plan(const chia_attn_params_t *params, int64_t row0,
                        int32_t tile_m, int32_t tile_n, int64_t *tile_lo,
                        int64_t *tile_hi, uint64_t *full_mask);

/* Human-readable name of a status code (static string). */
CHIA_API const char *chia_attn_status_string(int status);

/* CHIA_ATTN_ABI_VERSION the library was built with. */
CHIA_API int chia_attn_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CHIA_ATTN_H */
