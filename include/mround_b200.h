/*
 * mround_b200.h -- C ABI of libmround_b200.so, the sm_100a kernels of the
 * SignRound v2 block-tuning path.
 *
 * The library fills the slot MRound leaves empty (reference
 * mround/kernels/__init__.py:1-10, "empty by design"): every entry point below
 * replaces one reference call site, named in its comment as file:line of the
 * fbaldassarri/mround tree (version 0.1.0a6).
 *
 * Conventions, for every entry point:
 *  - All pointers are DEVICE pointers, contiguous row-major, 16-byte aligned
 *    unless stated.  bf16 tensors are passed as uint16_t bit patterns.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Every call is asynchronous and stream-ordered; nothing synchronizes
 *    except where stated.
 *  - Nothing allocates, frees, or keeps a pointer past the call.  Scratch
 *    ("workspace") is passed in by the caller, sized by the matching *_bytes
 *    query.
 *  - The return value is a status: 0 = MR_OK, negative on error (see
 *    mr_status_string).  No exception or abort crosses the ABI.
 *
 * Weight layout: a layer's weight is (rows = out_features, cols = in_features);
 * a quantization group is `group` consecutive elements of a row, so the
 * grouped view (rows, cols/group, group) of the reference is the same bytes.
 * V has the weight's shape; alpha and beta are (rows, cols/group).
 * Supported on the device: asymmetric observed-range schemes, bits 2..8,
 * group in {8, 16, 32, 64, 128, 256} dividing cols.
 */
#ifndef MROUND_B200_H_
#define MROUND_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MR_OK = 0,
  MR_ERR_ARGUMENT = -1,   /* bad shape, bits, group or size */
  MR_ERR_ALIGNMENT = -2,  /* a pointer or leading dimension is misaligned */
  MR_ERR_LAUNCH = -3,     /* a CUDA launch or runtime call failed */
  MR_ERR_DEVICE = -4,     /* no sm_100 device, or the device is unusable */
  MR_ERR_TIMEOUT = -5,    /* a bounded device-side wait gave up */
  MR_ERR_WORKSPACE = -6   /* workspace pointer missing or too small */
};

/* Library version (major*10000 + minor*100 + patch). */
int mr_version(void);

/* Static description of a status code. */
const char* mr_status_string(int status);

/* 0 when the current device is an sm_100 part the library was built for. */
int mr_device_check(void);

/* Last CUDA error string seen by the library on this host thread. */
const char* mr_last_cuda_error(void);

/*
 * Scheme arguments shared by K1, K2 and K5 (reference QuantScheme.symmetry and
 * .scale_init, mround/schemes.py:74-200):
 *   symmetric = 0, init_scale = NULL   asymmetric observed range: codes in
 *       [0, 2^bits-1], scale and zero point from the clipped extremes;
 *   symmetric = 1, init_scale = NULL   symmetric observed range: codes in
 *       [-2^(bits-1), 2^(bits-1)-1], scale = s / 2^(bits-1) with s the
 *       dominant clipped extreme negated (positive side: -max(gmax,0)*alpha,
 *       else -min(gmin,0)*beta), then sign(s)*max(|s|, eps);
 *   symmetric = 1, init_scale != NULL  searched (v2): scale =
 *       sign*max(|init_scale*beta|, eps), alpha inert; init_scale is float32
 *       (rows, cols/group), e.g. from mr_scale_search.
 * symmetric = 0 with init_scale != NULL is refused (MR_ERR_ARGUMENT).
 */

/*
 * K1 -- fused fake-quant forward.
 * Replaces fake_quantize (mround/core/quantizer.py:287-347) as called by
 * _TunableLinear.__call__ (mround/pipeline/runner.py:364-366).
 *   asymmetric: scale = max((max(gmax,0)*alpha - min(gmin,0)*beta) / (2^bits-1), eps)
 *               zp = rint(-w_min / scale); q = clamp(rint(w/scale + v) + zp, 0, 2^bits-1)
 *               wq = scale * (q - zp)
 *   symmetric:  q = clamp(rint(w/scale + v), -2^(bits-1), 2^(bits-1)-1); wq = scale * q
 * Outputs (any may be NULL): wq_hi = bf16(wq), wq_lo = bf16(wq - wq_hi) (the
 * split that lets two bf16 GEMM operands carry a float32 weight), wq_f32,
 * wq_t32 = wq rounded to tf32 (the operand of mr_gemm_tf32), scale and zp per
 * group (float32, (rows, cols/group); zp is 0 under the symmetric schemes).
 * IEEE division and ties-to-even rounding: codes are bit-exact.
 */
int mr_fq_forward(const uint16_t* w_bf16, const float* v, const float* alpha,
                  const float* beta, int64_t rows, int64_t cols, int group, int bits,
                  int symmetric, const float* init_scale, float eps, uint16_t* wq_hi,
                  uint16_t* wq_lo, float* wq_f32, float* wq_t32, float* scale, float* zp,
                  void* stream);

/*
 * K2 -- straight-through backward fused with signSGD and projection.
 * Replaces the autodiff of fake_quantize (mround/core/quantizer.py:110-149,
 * 228-266, 319-345; hand form mround/reference/quantize.py:370-397, 465-520)
 * and SignSGD.apply + project_params (mround/core/signsgd.py:125-145,
 * mround/core/quantizer.py:430-446; called at mround/pipeline/runner.py:926-931).
 * gq = dL/dwq, float32 (rows, cols).  With update != 0, V, alpha and beta are
 * updated in place:  p <- clip(p - lr*sign(g_p), lo, hi)  (V bounded by 0.5,
 * alpha and beta by [coef_lo, coef_hi]).  Under the symmetric schemes only the
 * dominant side's coefficient receives gradient; under the searched scheme
 * alpha receives none.
 * Optional outputs (NULL to skip): the gradients gv (rows, cols), galpha and
 * gbeta (rows, cols/group); and, when update != 0, the NEXT step's operands
 * wq_hi/wq_lo/wq_t32 recomputed from the updated parameters (fusing K1).
 */
int mr_ste_signsgd(const float* gq, const uint16_t* w_bf16, float* v, float* alpha,
                   float* beta, int64_t rows, int64_t cols, int group, int bits,
                   int symmetric, const float* init_scale, float eps, float lr,
                   float coef_lo, float coef_hi, int update, float* gv, float* galpha,
                   float* gbeta, uint16_t* wq_hi, uint16_t* wq_lo, float* wq_t32,
                   void* stream);

/*
 * K2 over several matrices in one launch (the members of a block, or this
 * rank's rows of them): the signed step of mr_ste_signsgd with update = 1 on
 * every segment, each writing its next operands (wq_hi / wq_lo / wq_t32, any
 * may be NULL) or its next codes (codes, qscale, qzp as in
 * mr_ste_signsgd_codes).  All segments share the group size, the scheme
 * (symmetric; init_scale NULL on all or on none) and eps; bits, the rate and
 * the coefficient bounds are per segment.  1 <= count <= 8.  Results are bit
 * for bit those of one mr_ste_signsgd / mr_ste_signsgd_codes call per
 * segment; the launch's warp tiles run over all segments, so small matrices
 * share one ramp and tail.  Same reference call sites as mr_ste_signsgd.
 */
typedef struct mr_k2_segment {
  const float* gq;
  const uint16_t* w_bf16;
  float* v;
  float* alpha;
  float* beta;
  const float* init_scale;
  int64_t rows;
  int64_t cols;
  int bits;
  float lr;
  float coef_lo;
  float coef_hi;
  uint16_t* wq_hi;
  uint16_t* wq_lo;
  float* wq_t32;
  uint8_t* codes;
  float* qscale;
  float* qzp;
} mr_k2_segment;

int mr_ste_signsgd_segments(const mr_k2_segment* segs, int count, int group, int symmetric,
                            float eps, void* stream);

/*
 * K2 for the row-sharded data-parallel update: the same straight-through
 * step as mr_ste_signsgd with update = 1, writing the NEXT step's integer
 * codes (one byte each: unsigned under the asymmetric scheme, two's
 * complement under the symmetric ones) and per-group float32 scale and zero
 * point (qzp only under the asymmetric scheme; may be NULL otherwise)
 * instead of the operands.  These are what the ranks exchange (about 1.1
 * bytes per weight instead of 8); mr_dequant_split rebuilds the operands
 * from them, bit for bit as mr_ste_signsgd writes them.  Same reference call
 * sites as mr_ste_signsgd (mround/pipeline/runner.py:926-931).  codes 8-byte
 * aligned.
 */
int mr_ste_signsgd_codes(const float* gq, const uint16_t* w_bf16, float* v, float* alpha,
                         float* beta, int64_t rows, int64_t cols, int group, int bits,
                         int symmetric, const float* init_scale, float eps, float lr,
                         float coef_lo, float coef_hi, uint8_t* codes, float* qscale,
                         float* qzp, void* stream);

/*
 * Operands from codes (the receiving side of the exchange above):
 *   wq = qscale * (code - qzp)  (symmetric = 0)   or   qscale * code  (symmetric = 1)
 * in float32 -- the fake-quant reconstruction of mround/core/quantizer.py:
 * 341-347 given its codes -- written as bf16 hi/lo and the tf32 copy (any may
 * be NULL).
 */
int mr_dequant_split(const uint8_t* codes, const float* qscale, const float* qzp, int64_t rows,
                     int64_t cols, int group, int symmetric, uint16_t* wq_hi, uint16_t* wq_lo,
                     float* wq_t32, void* stream);

/*
 * K5 -- commit and MLX packing in one pass.
 * Replaces quantize_codes (mround/core/quantizer.py:350-398), narrow_codes
 * (mround/formats/mlx_export.py:109-125), the symmetric offset and pack_codes
 * (mlx_export.py:215-222, mround/formats/packing.py:119-163) and to_affine
 * (mround/formats/mlx_export.py:159-195):
 *   packed (rows, cols*bits/32) uint32 of the unsigned codes (the code, or
 *   code + 2^(bits-1) under the symmetric schemes), element 0 in the least
 *   significant bits; 2/4/8 bits tile words, 3/5/6/7 form a little-endian
 *   bitstream; scales = bf16(scale), biases = bf16(-scales * zp) with zp the
 *   bf16 zero point or the fixed 2^(bits-1), (rows, cols/group).
 * codes (rows x cols, one byte each: uint8, or int8 under the symmetric
 * schemes) is optional.  Bit-exact.
 * cols must be a multiple of 32 for 3/5/6/7 bits and of 32/bits otherwise.
 */
int mr_pack_mlx(const uint16_t* w_bf16, const float* v, const float* alpha,
                const float* beta, int64_t rows, int64_t cols, int group, int bits,
                int symmetric, const float* init_scale, float eps, uint32_t* packed,
                uint16_t* scales_bf16, uint16_t* biases_bf16, uint8_t* codes, void* stream);

/*
 * K4 -- block-output loss, the exact global outlier threshold and dL/dpred.
 * Replaces reconstruction_loss / outlier_suppressed_loss / outlier_threshold /
 * piece_loss (mround/core/losses.py:42-56, 59-93, 96-107, 110-130; called at
 * mround/pipeline/runner.py:866).
 *   r = pred - target (float32), n elements.
 *   suppress: thr = k-th largest |r| (radix select, exact), keep = |r| < thr.
 *   loss = sum((r*keep)^2) / denom   (float64, written to *loss)
 *   grad = 2 * r * keep / denom      (float32, may be NULL)
 * `denom` is the element count of the whole batch (a piece passes the whole
 * batch's count).  thr_in >= 0 skips the selection and uses that threshold
 * (micro-batch pieces); otherwise the selected threshold is written to
 * *thr_out (device float, may be NULL).  `workspace` must hold
 * mr_loss_workspace_bytes() bytes.  n of 2^32 elements or more is refused
 * with MR_ERR_ARGUMENT (the selection's histogram counters are 32-bit).
 */
size_t mr_loss_workspace_bytes(void);
int mr_loss_outlier(const float* pred, const float* target, int64_t n, int64_t k,
                    int suppress, double denom, float thr_in, float* grad,
                    double* loss, float* thr_out, void* workspace, void* stream);

/*
 * K4 without a workspace argument.  No counterpart in the reference: MRound
 * has no native code and no caller that must avoid allocation.  It exists
 * for callers of this library that cannot allocate device memory themselves
 * -- a host binding the C ABI through an FFI with no device allocator, or an
 * asynchronous pipeline that must not call cudaMalloc because cudaMalloc can
 * synchronize the device.  Same arguments and results as mr_loss_outlier,
 * but the scratch lives in a fixed 16 KiB array compiled into the library
 * (mr_loss_noalloc_scratch_bytes), held by every GPU that loads the library
 * until the process exits.  n above 2^32 - 1 elements is refused with
 * MR_ERR_ARGUMENT (the selection counters are 32-bit).  The first call on
 * each device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  All calls share the one
 * array: calls that overlap on the GPU (two streams, or two host threads on
 * one device) race and must be serialized by the caller.  The stream must
 * belong to the current device (the array's address is the current
 * device's); a stream of another device is refused with MR_ERR_DEVICE.
 * Nothing is allocated or freed.
 */
size_t mr_loss_noalloc_scratch_bytes(void);
int mr_loss_outlier_noalloc(const float* pred, const float* target, int64_t n, int64_t k,
                            int suppress, double denom, float thr_in, float* grad,
                            double* loss, float* thr_out, void* stream);

/*
 * K4, distributed form: one radix pass of the global threshold selection.
 * pass = 0, 1, 2 over key bits [21,31), [10,21), [0,10) of |r|.  Each pass
 * writes this rank's histogram of the candidates to hist (2048 uint32); the
 * caller sums hist across ranks (an all-reduce) and then calls
 * mr_loss_select_digit, which narrows the device-side selection state.
 * `state` is the workspace of mr_loss_workspace_bytes() (its selection
 * state comes first).
 * mr_loss_outlier uses the same passes with no exchange.  n of 2^32 elements
 * or more is refused with MR_ERR_ARGUMENT.
 */
int mr_loss_hist_pass(const float* pred, const float* target, int64_t n, int pass,
                      const void* state, uint32_t* hist, void* stream);
int mr_loss_select_digit(const uint32_t* hist, int64_t k, int pass, void* state,
                         float* thr_out, void* stream);
int mr_loss_apply(const float* pred, const float* target, int64_t n, double denom,
                  const float* thr_dev, int suppress, float* grad, double* loss,
                  void* workspace, void* stream);

/*
 * K6 -- DeltaLoss reduction for the mixed-precision planner.
 * Replaces the per-layer term of _accumulate (mround/pipeline/scoring.py:262,
 * definition mround/planner/sensitivity.py:190-229):
 *   out[j] += sum |g * (RTN_{bits[j]}(w) - w)|   for j < n_bits,
 * RTN being the quantizer with v = 0 and unit coefficients (scoring.py:213-221)
 * under the scheme given by symmetric / grids: grids NULL is the observed
 * range; otherwise grids[j] is the searched scale of width bits[j] (float32,
 * rows x cols/group, scoring.py:195-210) and symmetric must be 1.  grids is a
 * host array of n_bits device pointers.  Float64 accumulation.  out is device
 * memory (n_bits doubles), accumulated into.
 */
int mr_deltaloss(const float* g, const uint16_t* w_bf16, int64_t rows, int64_t cols,
                 int group, const int* bits, int n_bits, int symmetric,
                 const float* const* grids, float eps, double* out, void* stream);

/*
 * K8 -- the v2 candidate scale grid search (symmetric schemes).
 * Replaces search_scales (mround/core/scale_search.py:73-187; NumPy oracle
 * mround/reference/scale_search.py:130-211), called by
 * QuantizationRunner._search_scales (mround/pipeline/runner.py:712-760) and
 * scoring's _grids (mround/pipeline/scoring.py:195-210).
 * Per group of w_bf16 (rows, cols): anchor = the signed largest-magnitude
 * element (first on ties); for each candidate c in order, eff = cands[c],
 *   inverse = -eff * (1/anchor)  (0 when anchor is 0)
 *   codes   = clamp(rint(inverse * w), -2^(bits-1), 2^(bits-1)-1)
 *   scale   = 1/inverse          (0 when inverse is 0)
 *   loss    = sum (scale*codes - w)^2 [* importance[col]]
 * keeping the first candidate with the strictly smallest loss.  Float32, the
 * sum of each group formed by 8-element runs combined pairwise.
 * cands: host array of n_cands (1..256) float32 effective ranges, the anchor
 * 2^(bits-1) first.  importance: float32 (cols) or NULL.
 * out: float32 (rows, cols/group), a zero scale for an all-zero group.
 */
int mr_scale_search(const uint16_t* w_bf16, int64_t rows, int64_t cols, int group, int bits,
                    const float* cands, int n_cands, const float* importance, float* out,
                    void* stream);

/*
 * Importance statistics for the searched scale: out[c] += sum_r x[r, c]^2
 * over rows of a float32 activation given as its bf16 parts (x = hi + lo;
 * lo may be NULL).  Replaces the collection mode of _TunableLinear.__call__
 * (mround/pipeline/runner.py:359-363).  Float32 accumulation in a fixed order
 * (no atomics: the result is reproducible); cols a multiple
 * of 8, pointers 16-byte aligned.
 */
int mr_colsumsq_split(const uint16_t* hi, const uint16_t* lo, int64_t rows, int64_t cols,
                      float* out, void* stream);

/*
 * Self-test of the kernels' arithmetic (no reference counterpart): counts, into
 * *mismatches (device, accumulated), the elements where the quantizer's
 * division -- a correctly rounded reciprocal per group and one Markstein
 * correction per element -- differs in any bit from IEEE division of a[i] by
 * b[i].
 */
int mr_selftest_division(const float* a, const float* b, int64_t n, unsigned int* mismatches,
                         void* stream);

/*
 * Operand preparation for the split-precision GEMMs: x (float32, n elements)
 * -> hi = bf16(x), lo = bf16(x - hi) (lo may be NULL).
 */
int mr_split_bf16(const float* x, int64_t n, uint16_t* hi, uint16_t* lo, void* stream);

/*
 * Gradient of the mean shifted cross-entropy in the DeltaLoss scoring
 * backward (mround/pipeline/scoring.py:183-192, _causal_loss): for each of
 * `rows` rows of `vocab` float32 logits and its int64 label,
 *   g = (softmax(logits) - onehot(label)) * scale     (scale = 1 / rows)
 * written as bf16 hi/lo, the operand of the LM-head input-gradient GEMM.
 * vocab % 4 == 0; labels in [0, vocab).
 */
int mr_ce_grad_split(const float* logits, const int64_t* labels, int64_t rows, int vocab,
                     float scale, uint16_t* hi, uint16_t* lo, void* stream);

/*
 * Operand preparation for the tf32 GEMM: out = x rounded to tf32 (round to
 * nearest, ties away from zero; the low 13 bits cleared), n elements of
 * float32; out may equal x.
 */
int mr_round_tf32(const float* x, int64_t n, float* out, void* stream);

/*
 * Fused element-wise operators of the decoder block (the mlx-lm layer the
 * reference runs inside block_output, mround/pipeline/blocks.py:578-606).
 * Each reads float32 activations and writes the next GEMM operand directly as
 * a bf16 hi/lo pair, and, where a `t32` pointer is given, as float32 rounded
 * to tf32 (the operand of mr_gemm_tf32).  In the backward kernels hi/lo may be
 * NULL (together) when only t32 is wanted.  Token t = b*S + s; attention
 * operands are (B, H, S, D).
 *   mr_rmsnorm_split:     y = x * rsqrt(mean(x^2) + eps) * w; rstd per row
 *   mr_rmsnorm_bwd_split: dx = resid + rstd * (g - xhat * mean(g * xhat)), g = dy * w;
 *                         resid may be NULL; written as hi/lo and/or float32 (out)
 *   mr_rope_split:        qkv (T, (Hq+2Hkv)*D) -> rope(q), rope(k), v as (B,H,S,D)
 *   mr_rope_bwd_split:    dq, dk, dv (B,H,S,D) -> dqkv (T, (Hq+2Hkv)*D)
 *   mr_heads_split:       merge=1: (B,H,S,D) -> (T, H*D); merge=0: the reverse
 *   mr_swiglu_split:      act = silu(g) * u, gu = [g | u] per row
 *   mr_swiglu_bwd_split:  dgu = [dact * u * silu'(g) | dact * silu(g)]
 *   mr_softmax_causal_split: rows of length S, row r at position r % S:
 *                         P = softmax(scale * scores) over columns <= position,
 *                         written as hi/lo (scores unchanged); S % 4 == 0,
 *                         S <= 8192
 *   mr_softmax_bwd_split: dS = scale * P * (dP - sum(dP * P)), P given as hi/lo
 *   band != 0 (softmax kernels): columns from (pos/128 + 2)*128 on are not
 *   written -- the causal modes of mr_gemm_batched never read them.
 */
int mr_rmsnorm_split(const float* x, const uint16_t* w, int64_t rows, int h, float eps,
                     uint16_t* hi, uint16_t* lo, float* t32, float* rstd, void* stream);
int mr_rmsnorm_bwd_split(const float* dy, const float* x, const uint16_t* w, const float* rstd,
                         const float* resid, int64_t rows, int h, uint16_t* hi, uint16_t* lo,
                         float* t32, float* out, void* stream);
int mr_rope_split(const float* qkv, const float* cosv, const float* sinv, int b, int s, int hq,
                  int hkv, int d, uint16_t* q_hi, uint16_t* q_lo, uint16_t* k_hi, uint16_t* k_lo,
                  uint16_t* v_hi, uint16_t* v_lo, void* stream);
int mr_rope_bwd_split(const float* dq, const float* dk, const float* dv, const float* cosv,
                      const float* sinv, int b, int s, int hq, int hkv, int d, uint16_t* hi,
                      uint16_t* lo, float* t32, void* stream);
int mr_heads_split(const float* src, int b, int s, int h, int d, int merge, uint16_t* hi,
                   uint16_t* lo, float* t32, void* stream);
int mr_swiglu_split(const float* gu, int64_t t, int i, uint16_t* hi, uint16_t* lo, float* t32,
                    void* stream);
int mr_swiglu_bwd_split(const float* dact, const float* gu, int64_t t, int i, uint16_t* hi,
                        uint16_t* lo, float* t32, void* stream);
int mr_softmax_causal_split(const float* scores, int64_t rows, int s, float scale, int band,
                            uint16_t* hi, uint16_t* lo, void* stream);
int mr_softmax_bwd_split(const float* dp, const uint16_t* p_hi, const uint16_t* p_lo,
                         int64_t rows, int s, float scale, int band, uint16_t* hi, uint16_t* lo,
                         void* stream);

/*
 * K3 -- tcgen05/TMEM GEMM, bf16 operands, float32 accumulate in tensor memory.
 * The contraction of every decoder-block linear in the tuning step
 * (mround/pipeline/runner.py:367, y = x @ Wq.T, and the two products its
 * backward needs, which MLX autodiff forms at runner.py:920).
 *   C[m, n] (+)= sum_k A[m, k] * B[n, k]   (+ bias[n])
 * A is K-major (a_kmajor = 1: element (m,k) at a[m*lda + k]) or M-major
 * (a_kmajor = 0: at a[k*lda + m]); B likewise with N.
 * precision = 1: a_hi*b_hi.  precision = 2: a_hi*b_hi + a_lo*b_hi (B exact in
 * bf16).  precision = 3: a_hi*b_hi + a_hi*b_lo + a_lo*b_hi, the split that
 * carries float32 operands (x = hi + lo) through bf16 tensor cores.
 * accumulate != 0 adds into C.  Any m, n, k >= 1 (edges are zero-filled by
 * TMA); leading dimensions multiples of 8 elements; bf16 pointers 16-byte
 * aligned.  Device-side waits are bounded: a wait that gives up sets a status
 * word read (synchronously) by mr_gemm_status.
 */
int mr_gemm(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda, int a_kmajor,
            const uint16_t* b_hi, const uint16_t* b_lo, int64_t ldb, int b_kmajor,
            float* c, int64_t ldc, const float* bias, int accumulate, int64_t m,
            int64_t n, int64_t k, int precision, void* stream);

/*
 * K3, batched: `batch` independent GEMMs of the same shape, operand i at
 * a + i*stride_a, b + i*stride_b, c + i*stride_c (elements; strides multiples
 * of 8 for bf16 operands).  One launch (grid.y = batch).  Serves the
 * attention products of the decoder block (scores, probabilities times
 * values, and their gradients), which the reference runs inside the mlx-lm
 * layer (mround/pipeline/blocks.py:578-606).
 * causal (seq = positions per head, a multiple of 128; rows of a problem stack
 * heads of seq positions): 0 none; 1 C = Q K^T-shaped (n = seq), tiles above
 * the diagonal are not computed or written; 2 C = P V-shaped (k = seq), the
 * K loop stops after each row tile's last position; 3 C = dS^T Q-shaped
 * (m = seq, k = heads*seq), K tiles whose rows precede the tile's first key
 * are skipped.  Modes 2 and 3 read only what mr_softmax_*_split writes with
 * band != 0.
 */
int mr_gemm_batched(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda, int64_t stride_a,
                    int a_kmajor, const uint16_t* b_hi, const uint16_t* b_lo, int64_t ldb,
                    int64_t stride_b, int b_kmajor, float* c, int64_t ldc, int64_t stride_c,
                    const float* bias, int accumulate, int64_t m, int64_t n, int64_t k,
                    int64_t batch, int precision, int causal, int64_t seq, void* stream);

/*
 * The output tile K3 uses for this shape on the current device (a query;
 * launches nothing; negative status on bad arguments): mr_gemm_tile_n its
 * width (128, 224 or 256 columns), mr_gemm_tile_m its height (128 or 256
 * rows).  128 x 128 for n <= 128; 128 x 256 for the bf16 products; for one
 * tf32 product (precision 4, no batch, no causal mode) the shape of 128 or
 * 256 rows by 224 or 256 columns with the shortest persistent schedule (whole
 * waves of tiles over the SMs, each tile's time the larger of its staged
 * operand bytes and its flops at one SM's rates).
 */
int mr_gemm_tile_n(int64_t m, int64_t n, int64_t k, int64_t batch, int precision, int a_kmajor,
                   int b_kmajor, int causal);
int mr_gemm_tile_m(int64_t m, int64_t n, int64_t k, int64_t batch, int precision, int a_kmajor,
                   int b_kmajor, int causal);

/* Device status word of K3: 0, or MR_ERR_TIMEOUT.  Synchronizes the device;
 * reset != 0 clears it. */
int mr_gemm_status(int reset);

/*
 * K3 fused with the data-parallel reduce-scatter of a weight gradient.
 * Replaces the gradient all-reduce of the data-parallel step (the reference's
 * micro-batch sum, mround/pipeline/runner.py:984-1044, across GPUs): the same
 * GEMM as mr_gemm (no bias, no accumulate, batch 1), but row r of the
 * (m, n) result is stored over NVLink into its owner's slot,
 *   dst[r / rows_per_rank] + (r % rows_per_rank) * ldd,
 * where dst[o] is rank o's slot buffer for this source rank (a peer pointer
 * from mr_ipc_import, or local memory for this rank's own rows);
 * m == rows_per_rank * world.  After every tile is stored, the kernel
 * releases ``epoch`` (> 0, increasing) into flags[o] on every rank o, each a
 * peer pointer to rank o's flag for this source.  ``done`` is a zeroed device
 * counter owned by this rank (left zero on return).  Plain peer stores only: no
 * multicast, no loads from peer memory.
 */
int mr_gemm_rs(const uint16_t* a_hi, const uint16_t* a_lo, int64_t lda, int a_kmajor,
               const uint16_t* b_hi, const uint16_t* b_lo, int64_t ldb, int b_kmajor, int64_t m,
               int64_t n, int64_t k, int precision, float* const* dst, int64_t ldd,
               int64_t rows_per_rank, unsigned long long* const* flags, int world,
               unsigned int* done, unsigned long long epoch, void* stream);

/*
 * K3 with one tf32 product: float32 operands, float32 accumulate in tensor
 * memory.  The backward products of the decoder-block linears
 * (mround/pipeline/runner.py:920, the input and weight gradients MLX autodiff
 * forms for y = x @ Wq.T at runner.py:367): same contraction, majorness,
 * bias and accumulate semantics as mr_gemm, through tcgen05.mma kind::tf32.
 * The tensor core reads the upper 19 bits of each float32 (10 explicit
 * mantissa bits): operands must already be rounded to tf32 (round to nearest,
 * as mr_round_tf32 and the *_split kernels' t32 outputs do) for the product
 * to use exactly those values.  A tf32 product takes the tensor time of two
 * bf16 products and keeps 11 significant bits per operand.  Leading
 * dimensions multiples of 4 elements; pointers 16-byte aligned.
 */
int mr_gemm_tf32(const float* a, int64_t lda, int a_kmajor, const float* b, int64_t ldb,
                 int b_kmajor, float* c, int64_t ldc, const float* bias, int accumulate,
                 int64_t m, int64_t n, int64_t k, void* stream);

/* mr_gemm_rs with tf32 operands (the fused weight-gradient GEMM ->
 * reduce-scatter of the data-parallel step, one tf32 product). */
int mr_gemm_rs_tf32(const float* a, int64_t lda, int a_kmajor, const float* b, int64_t ldb,
                    int b_kmajor, int64_t m, int64_t n, int64_t k, float* const* dst,
                    int64_t ldd, int64_t rows_per_rank, unsigned long long* const* flags,
                    int world, unsigned int* done, unsigned long long epoch, void* stream);

/*
 * Peer memory of the exchange.  mr_ipc_export writes the CUDA IPC handle
 * (mr_ipc_handle_bytes() bytes) of the allocation holding ``ptr`` and the
 * offset of ``ptr`` in it; mr_ipc_import maps a peer's handle into this
 * device's address space (base, and base + offset in ``ptr``); mr_ipc_close
 * releases a mapping by its base.
 */
size_t mr_ipc_handle_bytes(void);
int mr_ipc_export(const void* ptr, void* handle, int64_t* offset);
int mr_ipc_import(const void* handle, int64_t offset, void** base, void** ptr);
int mr_ipc_close(void* base);

/*
 * The owner's side of mr_gemm_rs: wait (bounded: 2 s, then the status word
 * below) until flags[r] >= epoch for every source rank r, then
 * out[i] = sum over r in rank order of slots[r * slot_stride + i], i < n.
 * Float32, 16-byte aligned, n and slot_stride multiples of 4.
 */
int mr_reduce_slots(const float* slots, int64_t slot_stride, int64_t n, int world,
                    const unsigned long long* flags, unsigned long long epoch, float* out,
                    void* stream);

/*
 * Copy-engine form of the source side of the exchange (the GEMM writes the
 * full weight gradient locally): copy ``bytes`` from ``src`` (this rank's rows
 * for one owner) to ``dst`` (the owner's slot for this source; peer memory
 * from mr_ipc_import, or this rank's own slot) with one cudaMemcpyAsync on
 * ``stream``, then release ``epoch`` into ``flag`` (the owner's flag for this
 * source) from a one-thread kernel ordered after the copy.  No SM moves data.
 * Replaces, like mr_gemm_rs, the gradient sum across data-parallel ranks
 * (mround/pipeline/runner.py:984-1044).
 */
int mr_peer_send(void* dst, const void* src, int64_t bytes, unsigned long long* flag,
                 unsigned long long epoch, void* stream);

/* Device status word of the exchange (0 ok, MR_ERR_TIMEOUT); synchronizes. */
int mr_peer_status(int reset);

#ifdef __cplusplus
}
#endif

#endif /* MROUND_B200_H_ */
