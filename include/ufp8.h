/*
 * ufp8 — C ABI of the B200 (sm_100a) FP8 dense-contraction library.
 *
 * This is the drop-in boundary for the FP8 mode of macrogpt-jax's `Einsum` layer and the
 * layers built on it.  The reference computes that path with XLA; each entry point below
 * replaces one piece of it (file:line relative to the reference repository):
 *
 *   ufp8_amax / ufp8_quantize / ufp8_amax_quant
 *       replace the forward/backward fp8 casts of `custom_astype`
 *       (ueaj/utils/gradutils.py:15-54, `lax.convert_element_type` at :34,:41,:49),
 *       composed with per-tensor current scaling: amax = max|x|, s = FMAX/amax
 *       (amax == 0 -> s = 1), q = RNE(f32(x) * s) with ml_dtypes 0.5.4 cast semantics,
 *       inv_scale = 1/s (both divisions IEEE round-to-nearest).
 *   ufp8_gemm (UFP8_EPI_STORE)
 *       replaces the contraction `jnp.einsum(self.einsum_expr, x, self.w.value)`
 *       (ueaj/model/einsum.py:243) and the two dot_generals JAX derives for its
 *       backward pass; fp32 accumulation, output multiplied by inv_scale_a * inv_scale_b.
 *   ufp8_gemm (UFP8_EPI_SWIGLU)
 *       replaces GMLP's fused gate/up Einsum "bnd,idh->ibnh" plus its gating
 *       `up * swish(gate)` (ueaj/model/mlp.py:78-86, 102-107).
 *   ufp8_gemm (UFP8_EPI_DSWIGLU)
 *       replaces the backward of the down-projection input together with the gating's
 *       backward (JAX autodiff of ueaj/model/mlp.py:102-114).
 *
 * Conventions.  All pointers are device pointers owned by the caller; nothing here
 * allocates device memory.  Every call is stream-ordered and asynchronous; nothing
 * synchronises the device except ufp8_device_status.  Shapes and alignment are checked
 * on the host before any launch: a call returns UFP8_OK (0) or a negative UFP8_ERR_*
 * code, and ufp8_last_error() (per host thread) describes the last failure.  Device code
 * never traps: every pipeline wait is bounded, and a wait that runs out sets a bit in
 * the library's device status word, which ufp8_device_status reads.
 */
#ifndef UFP8_H_
#define UFP8_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ufp8_stream_t; /* same handle as cudaStream_t */

#define UFP8_ABI_VERSION 5

/* return codes */
#define UFP8_OK 0
#define UFP8_ERR_INVALID (-1)     /* bad shape, null pointer, bad enum */
#define UFP8_ERR_ALIGN (-2)       /* pointer / leading dimension breaks a 16-byte rule */
#define UFP8_ERR_UNSUPPORTED (-3) /* valid request this build does not implement */
#define UFP8_ERR_CUDA (-4)        /* a CUDA runtime / driver call failed */
#define UFP8_ERR_DEVICE (-5)      /* device older than sm_100 */

/* bits of the device status word */
#define UFP8_STATUS_WAIT_TIMEOUT 1 /* a GEMM pipeline wait ran out */
#define UFP8_STATUS_PEER_TIMEOUT 2 /* a tensor-parallel peer never signalled */

/* fp8 formats (values match the MMA instruction-descriptor encoding) */
#define UFP8_E4M3 0 /* float8_e4m3fn: forward operands, max 448   */
#define UFP8_E5M2 1 /* float8_e5m2:   gradients,        max 57344 */
#define UFP8_BF16 2 /* bf16: the operand format of the 16-bit GEMM (both operands of a ufp8_gemm), and the
                     unquantised gradient output of ufp8_xent_backward */

/* operand storage order */
#define UFP8_K_MAJOR 0  /* stored [rows = M or N][K], K contiguous   */
#define UFP8_MN_MAJOR 1 /* stored [K][cols = M or N], M/N contiguous */

/* output element type */
#define UFP8_OUT_BF16 0
#define UFP8_OUT_F32 1

/* GEMM epilogues */
#define UFP8_EPI_STORE 0   /* D = acc * sa * sb                                          */
#define UFP8_EPI_SWIGLU 1  /* D[0]=U, D[1]=G, H = U * silu(G), amax_out = max|H|          */
#define UFP8_EPI_DSWIGLU 2 /* dH = acc*sa*sb; D[0]=dU, D[1]=dG from saved U,G; amax |dUG| */
#define UFP8_EPI_RS_PUSH 3 /* D rows stored into their owner rank's reduce-scatter staging slot */
#define UFP8_EPI_XENT 4    /* D = logits (bf16, optionally soft-capped) + per-row softmax partials  */
#define UFP8_EPI_AXPBY 5   /* D = alpha * acc * sa * sb + beta * C (bf16 operands only)            */
/* Attention products with the default positions (bf16 operands; see the attn_* fields): */
#define UFP8_EPI_ATTN_STATS 6 /* scores: per-row softmax partials of scale * acc, nothing stored  */
#define UFP8_EPI_ATTN_P 7     /* scores: D = bf16(exp(scale * acc - lse[row])), masked -> 0       */
#define UFP8_EPI_ATTN_DS 8    /* dP: D = bf16(scale * P (acc - attn_row[row])), P read from `c`  */

/* tile masks of a bf16 GEMM (ufp8_gemm_desc.tile_mask; tiles are 256 x 256): causal attention's
 * products skip what its mask zeroes */
#define UFP8_TILES_ALL 0
#define UFP8_TILES_LOWER 1       /* only tiles whose N tile index <= M tile index; D elsewhere not written */
#define UFP8_TILES_K_TO_DIAG 2   /* M tile m contracts K in [0, 256 (m + 1)) of each K slice           */
#define UFP8_TILES_K_FROM_DIAG 3 /* M tile m contracts K in [256 m, K) of each K slice                  */
/* (tile masks: an M tile whose K range is empty is not written either)                              */

const char* ufp8_last_error(void);
int ufp8_abi_version(void);

/* amax = max |x| over n bf16 elements (NaN-propagating), written to *amax (device f32).
 * Replaces the amax half of the per-tensor recipe feeding custom_astype
 * (ueaj/utils/gradutils.py:15-54). */
int ufp8_amax(const void* x_bf16, int64_t n, float* amax, ufp8_stream_t stream);

/* q = fp8(x * s) with s = FMAX(fmt) / *amax, *inv_scale = 1/s.  `amax` is a device
 * pointer produced by ufp8_amax or by a GEMM epilogue.  Replaces the forward cast
 * `lax.convert_element_type(x, float8)` (ueaj/utils/gradutils.py:34,41) and, with
 * fmt = UFP8_E5M2, the backward cast of the gradient (ueaj/utils/gradutils.py:49). */
int ufp8_quantize(const void* x_bf16, int64_t n, int fmt, const float* amax, void* q, float* inv_scale,
                  ufp8_stream_t stream);

/* ufp8_amax followed by ufp8_quantize on the same stream. */
int ufp8_amax_quant(const void* x_bf16, int64_t n, int fmt, void* q, float* amax, float* inv_scale,
                    ufp8_stream_t stream);

/* ufp8_amax_quant without the caller's amax buffer and without any allocation: the amax
 * scratch (one partial max per 65 536 elements, plus the reduced amax) lives in static
 * device arrays of the library (16 KiB per device), so n is limited to 268 435 456 elements
 * (larger n returns UFP8_ERR_UNSUPPORTED and launches nothing).  q and *inv_scale are
 * bit-identical to ufp8_amax_quant's.  No scratch word has to start at zero.  For callers that
 * may not allocate device memory nor hold a spare device word, e.g. an XLA FFI handler whose
 * buffers all come from XLA.  This entry point has no counterpart in the reference (XLA's cast
 * needs no scratch).  Overlapping calls on one device race on the shared scratch: calls must be
 * ordered (one stream, or synchronised).  The first call in a device's CUDA context looks up the
 * scratch address (cudaGetSymbolAddress, with that device current; again after the context
 * changes, e.g. after cudaDeviceReset); make that first call outside any stream capture. */
int ufp8_amax_quant_noalloc(const void* x_bf16, int64_t n, int fmt, void* q, float* inv_scale,
                            ufp8_stream_t stream);

/* q = fp8(x) with a unit scale: the plain element-type conversion of custom_astype
 * (ueaj/utils/gradutils.py:34,41,49 `lax.convert_element_type`) to float8_e4m3fn /
 * float8_e5m2, round to nearest even with the ml_dtypes overflow rules. */
int ufp8_cast(const void* x_bf16, int64_t n, int fmt, void* q, ufp8_stream_t stream);

/* ---- RMSNorm fused with the fp8 quantisation of its output -------------------------------
 * Replaces RMSNorm.__call__ (ueaj/model/rmsnorm.py:68-84) followed by the per-tensor cast of its
 * output that the next FP8 Einsum makes (ueaj/model/layer.py:54,56: attn(attn_norm(x)),
 * mlp(mlp_norm(x))).  x: [rows, d] bf16 with row pitch ldx.  scale: bf16, scale_len 1 or d
 * (NULL: scale_mode 'none'); centered != 0 multiplies by 1 + scale ('centered' modes).
 * Per row: r = 1 / sqrt(mean(x^2) + eps) in f32 (fixed summation order, see csrc/norm.cu),
 * y = bf16((x * r) * w); rstd[row] = r (f32, kept for the backward).  If y_bf16 is not NULL, y
 * is stored (pitch ldy).  If inv_scale is not NULL, amax = max|y| and q = fp8(y * FMAX/amax)
 * ([rows, d] contiguous; q may be NULL only when rows == 0) with *inv_scale as ufp8_quantize
 * writes it; amax alone may be asked for with inv_scale = NULL.  Two passes over x: 5 bytes of
 * HBM traffic per element with the fp8 output. */
int ufp8_rmsnorm_quant(const void* x_bf16, int64_t rows, int64_t d, int64_t ldx, const void* scale_bf16,
                       int64_t scale_len, int centered, float eps, int fmt, void* q, float* amax, float* inv_scale,
                       float* rstd, void* y_bf16, int64_t ldy, ufp8_stream_t stream);

/* Backward of the RMSNorm above (the derivative JAX takes of ueaj/model/rmsnorm.py:68-84):
 * dx = bf16(r * w * dy - x * r^3 * sum(dy * w * x) / d) per row, from the forward's rstd, and,
 * when dscale (f32, scale_len entries) is not NULL, dscale = sum over rows of dy * x * r (summed
 * over the row too for a one-element scale), deterministic: per-CTA partials in `workspace`
 * (ufp8_rmsnorm_backward_workspace bytes), summed in CTA order.  d <= 8192. */
int ufp8_rmsnorm_backward_workspace(int64_t rows, int64_t d, int64_t* bytes);
int ufp8_rmsnorm_backward(const void* x_bf16, int64_t rows, int64_t d, int64_t ldx, const void* scale_bf16,
                          int64_t scale_len, int centered, const float* rstd, const void* dy_bf16, int64_t lddy,
                          void* dx_bf16, int64_t lddx, float* dscale, float* workspace, int64_t workspace_bytes,
                          ufp8_stream_t stream);

/* One fp8 operand of a GEMM.  Logical shape [rows, K] for A (rows = M) and for B
 * (rows = N); `major` says which index is contiguous in memory.  `ld` is the pitch in
 * elements between consecutive stored rows (K-major: >= K; MN-major: >= rows) and
 * `batch_stride` the pitch between batch slices (elements). */
typedef struct ufp8_operand {
  const void* ptr;
  int32_t fmt;   /* UFP8_E4M3 / UFP8_E5M2 */
  int32_t major; /* UFP8_K_MAJOR / UFP8_MN_MAJOR */
  int64_t ld;
  int64_t batch_stride;
  int32_t batch_count;    /* slices present in memory (1 = broadcast over the GEMM batch) */
  int32_t batch_group;    /* > 1: GEMM batch g reads slice g / batch_group (a slice shared by
                             batch_group consecutive products, e.g. one key head for its group of
                             query heads); 0 or 1: slice g.  Needs k_batches == 1, not SWIGLU. */
  const float* inv_scale; /* device f32: 1/s of this operand */
} ufp8_operand;

/* D[g] = sum_{kb < k_batches} A[g * k_batches + kb] * B[g * k_batches + kb]^T for g < batch (with
 * k_batches == 1: A[g] B[g]^T, a one-slice operand broadcast over the batch).
 * k_batches > 1 concatenates K over operand slices (e.g. dx = sum_i dUG[i] W[i]^T).
 * UFP8_EPI_SWIGLU reads B slice 0 as `up` and slice 1 as `gate` for the same N range;
 * D then holds U (slice 0) and G (slice 1) and `h` receives U * silu(G).
 * UFP8_EPI_DSWIGLU reads the saved U / G from `ug` (slice pitch ug_batch_stride) and
 * writes dU / dG to D slices 0 / 1.  `amax_out` (device f32, may be null for STORE) is
 * overwritten with max |H| (SWIGLU) or max |dU, dG| (DSWIGLU). */
typedef struct ufp8_gemm_desc {
  int64_t M, N, K;
  int32_t batch;
  int32_t k_batches;
  ufp8_operand a;
  ufp8_operand b;
  void* d;
  int32_t d_dtype; /* UFP8_OUT_BF16 / UFP8_OUT_F32 (F32 only with UFP8_EPI_STORE) */
  int32_t epilogue;
  int64_t ldd;
  int64_t d_batch_stride;
  void* h; /* SWIGLU: bf16 H [M, N] */
  int64_t ldh;
  const void* ug; /* DSWIGLU: bf16 U at ug, G at ug + ug_batch_stride */
  int64_t ldug;
  int64_t ug_batch_stride;
  float* amax_out;
  /* RS_PUSH: rows [o*R, (o+1)*R) belong to rank o (R = rs_rows_per_rank); row m is stored at
   * rs_slots[o] + ((rs_rank * R + m - o*R) * ldd + n) elements, i.e. this rank's slot in the
   * owner's staging buffer (rs_slots comes from ufp8_tp_begin; `d` is ignored). */
  void* const* rs_slots;
  int32_t rs_rank;
  int32_t rs_reserved;
  int64_t rs_rows_per_rank;
  /* All-gathered A (CTA-pair kernel only): rows [s*R, (s+1)*R) of A (R = ag_rows_per_rank, a
   * multiple of 256) arrive from rank s through ufp8_tp_ag_push; before the first load of a
   * block s != ag_rank the producer waits (bounded; UFP8_STATUS_PEER_TIMEOUT) until
   * ag_flags[s] == ag_epoch (ag_flags from ufp8_tp_local).  The tile order starts at this
   * rank's own block.  ag_flags == NULL: no waits.  Not combinable with RS_PUSH. */
  const uint32_t* ag_flags;
  uint32_t ag_epoch;
  int32_t ag_rank;
  int64_t ag_rows_per_rank;
  /* XENT (CTA-pair kernel, bf16 D, batch 1): D receives the logits l = bf16(acc * sa * sb), or,
   * with xent_cap > 0, c = bf16(cap * bf16(tanh(bf16(l / cap)))) (the soft cap of
   * ueaj/model/model.py:162-163 with bf16 rounding after each operation).  For every row and
   * every group of 128 columns [128 j, 128 j + 128) that holds a column < N, the pair
   * (m, s) = (max c, sum exp(c - m)) over the group's columns < N is written as two f32 at
   * xent_stats + 2 * (row * xent_ld_stats + j); xent_ld_stats >= ceil(N / 128). */
  float* xent_stats;
  int64_t xent_ld_stats;
  float xent_cap;
  int32_t xent_reserved;
  /* AXPBY: D = alpha * (acc * sa * sb) + beta * C, with C bf16 [batch][M, N] (pitch ldc elements,
   * slice pitch c_batch_stride); each product and the sum rounded once in f32, then D's type.
   * With bf16 operands (fmt UFP8_BF16 for both A and B) inv_scale may be NULL (factor 1); only
   * the STORE and AXPBY epilogues take bf16 operands, on the CTA-pair kernel. */
  const void* c;
  int64_t ldc;
  int64_t c_batch_stride;
  float alpha;
  float beta;
  int32_t tile_mask; /* UFP8_TILES_* (bf16 operands only) */
  int32_t reserved2;
  /* UFP8_EPI_ATTN_*: batch entry g, row r (query), column c (key) of the score matrix
   * scale * (A_g B_g^T)[r, c] is visible iff c <= r and both carry the same non-negative segment
   * id (attn_q_segment_ids[r], attn_kv_segment_ids[c]; NULL: all 0).
   *   STATS: in base 2, y = x * log2(e): (m, s) = (max y, sum 2^(y - m)) of the visible y of each
   *          group j of 128 columns as two f32 at attn_stats + 2 * ((g * M + r) * attn_ld_stats + j)
   *          (m = -inf, s = 0 when none is visible); D is not written (may be NULL).
   *   P:     D = bf16(2^(x * log2(e) - attn_row[g * M + r] * log2(e))) where visible, else 0
   *          (attn_row = lse, natural log).
   *   DS:    D = bf16(scale * (P * (acc - attn_row[g * M + r]))), each step rounded in f32, with
   *          P the bf16 matrix `c` (pitch ldc, slice pitch c_batch_stride; attn_row = rowsum(dO O)).
   * With UFP8_TILES_LOWER the tiles past the diagonal are not computed (not written). */
  const int32_t* attn_q_segment_ids;
  const int32_t* attn_kv_segment_ids;
  float* attn_stats;
  int64_t attn_ld_stats;
  const float* attn_row;
  float attn_scale;
  int32_t attn_reserved;
} ufp8_gemm_desc;

int ufp8_gemm(const ufp8_gemm_desc* desc, ufp8_stream_t stream);

/* ---- next-token cross-entropy on the lm_head logits ---------------------------------------
 * Replaces the loss of chunked_softmax_cross_entropy (ueaj/opt/next_token_loss.py:99-174):
 * optax.softmax_cross_entropy_with_integer_labels on each chunk's logits, times the loss mask.
 * Logits: [rows, V] bf16 with row pitch ldl (the capped values when the model soft-caps them).
 * labels: int32 [rows]; a negative label counts from the end (as jnp.take_along_axis normalises
 * it) and a label outside [-V, V) has no column.  mask: uint8 [rows] multiplied into the loss
 * (NULL = all ones).  Per row, in f32: M = max_j c_j, lse = M + log(sum_j exp(c_j - M)),
 * loss = (lse - c[label]) * mask (NaN for a label without a column, as the reference's fill-mode
 * gather gives), qrow = 1 - exp(c[label] - lse) (1 without a column): the largest
 * |softmax_j - onehot_j| of the row, which the backward's fp8 scale uses. */
int ufp8_xent_forward(const void* logits_bf16, int64_t rows, int64_t V, int64_t ldl, const int32_t* labels,
                      const uint8_t* mask, float* lse, float* loss, float* qrow, ufp8_stream_t stream);

/* The same per-row results from the partials of a UFP8_EPI_XENT GEMM (stats, pitch ld_stats in
 * pairs, ceil(V / 128) groups per row): the logits are read only at the labels. */
int ufp8_xent_combine(const float* stats, int64_t ld_stats, const void* logits_bf16, int64_t rows, int64_t V,
                      int64_t ldl, const int32_t* labels, const uint8_t* mask, float* lse, float* loss, float* qrow,
                      ufp8_stream_t stream);

/* Backward of the loss above (JAX's derivative of the per-token loss, with the soft cap's):
 * g_r = dloss[r] * mask[r] (dloss NULL = all ones), dl_rj = g_r * (exp(c_rj - lse_r) - [j == label_r]),
 * times (1 - (c_rj * (1 / cap))^2) when cap > 0 (tanh' from the stored capped value).
 * fmt UFP8_BF16: dl stored as bf16 [rows, V] (pitch ldo); amax / inv_scale unused.
 * fmt UFP8_E4M3 / UFP8_E5M2: amax = max_r |g_r| * qrow_r, which equals max |dl| when cap == 0 (the
 * label column holds each row's largest |softmax - onehot|, computed with the same operations) and
 * bounds it otherwise; then s = FMAX / amax as ufp8_quantize derives it, q = fp8(dl * s), and
 * *amax, *inv_scale as ufp8_quantize writes them.  Two launches, 3 bytes of HBM traffic per
 * element with the fp8 output. */
int ufp8_xent_backward(const void* logits_bf16, int64_t rows, int64_t V, int64_t ldl, const int32_t* labels,
                       const uint8_t* mask, const float* lse, const float* qrow, const float* dloss, float cap,
                       int fmt, void* dlogits, int64_t ldo, float* amax, float* inv_scale, ufp8_stream_t stream);

/* ---- Newton-Schulz orthogonalisation (Muon) ------------------------------------------------
 * Replaces orthogonalize (ueaj/opt/multiscale.py:110-141): optax.contrib's
 * orthogonalize_via_newton_schulz (optax 0.2.6) mapped over `batch` slices g[b] of shape [m, n]
 * (f32 or bf16, contiguous).  Per slice: work on X^T when m > n; X = X / (||X||_F + eps); then for
 * each of `steps` coefficient triples (a, b, c) (host array coeffs[steps][3]):
 *   A = X X^T, B = b A + c A A, X = a X + B X,
 * each product a bf16 tcgen05 GEMM (fp32 accumulation) and each update its AXPBY epilogue; X, A
 * and B are rounded to bf16 between the GEMMs (optax runs the iteration in the input's dtype, f32
 * under the reference's Muon), and the last step is written to `out` (f32 or bf16, [batch][m][n]).
 * m and n must be multiples of 8; batch <= 65535.  workspace: ufp8_newton_schulz_workspace bytes,
 * 256-byte aligned.  Stream-ordered; 2 + 3 * steps launches. */
int ufp8_newton_schulz_workspace(int64_t batch, int64_t m, int64_t n, int64_t* bytes);
int ufp8_newton_schulz(const void* g, int g_dtype, int64_t batch, int64_t m, int64_t n, int steps,
                       const float* coeffs, float eps, void* out, int out_dtype, void* workspace,
                       int64_t workspace_bytes, ufp8_stream_t stream);

/* ---- RoPE and softmax attention ----------------------------------------------------------
 * RoPE (ueaj/model/rope.py:10-104): ufp8_rope_table writes, for `count` positions (f32) and
 * `half` = rope_d / 2 frequencies inv_freq (f32, the caller's 1 / theta^(j / half)), the bf16
 * tables sin / cos [count][half] of angle = position * inv_freq.  ufp8_rope rotates x (bf16
 * [tokens][heads][d], contiguous) in place or into `out`: with x1 = x[..., :d/2], x2 = x[..., d/2:],
 * (x1 c - x2 s, x2 c + x1 s), each product and sum rounded to bf16 as the reference's bf16
 * expression is; token t uses table row t % period; inverse != 0 applies the transpose (the
 * backward). */
int ufp8_rope_table(const float* positions, int64_t count, int64_t half, const float* inv_freq, void* sin_bf16,
                    void* cos_bf16, ufp8_stream_t stream);
int ufp8_rope(const void* x_bf16, int64_t tokens, int64_t heads, int64_t d, const void* sin_bf16,
              const void* cos_bf16, int64_t period, int inverse, void* out_bf16, ufp8_stream_t stream);

/* Softmax attention: the flash_attention call of SoftmaxAttention.__call__ (ueaj/model/soft_attn.py:
 * 186-196; kvax 0.1.2).  q [batch][seq][kv_heads * group][head_dim], k and v [batch][seq][kv_heads]
 * [head_dim], out like q, all bf16; query head (h, i) attends with key/value head h.  Query p sees key
 * p' of the same batch element iff positions[p'] <= positions[p] and both segment ids are equal and
 * non-negative (a negative id is padding); a row that sees nothing outputs 0.  P = softmax(scale *
 * Q K^T) over the visible keys.  Products are bf16 tcgen05 GEMMs with fp32 accumulation; the scores
 * (f32) of one batch element live in `workspace`, the probabilities (bf16) of all of them in `saved`
 * for the backward (sizes from ufp8_attention_workspace, 256-byte aligned).  Segment ids and
 * positions: int32 [batch][seq], NULL = all 0 / 0..seq-1.  seq and head_dim multiples of 8. */
typedef struct ufp8_attn_desc {
  int64_t batch, seq, kv_heads, group, head_dim;
  const int32_t* q_segment_ids;
  const int32_t* kv_segment_ids;
  const int32_t* q_positions;
  const int32_t* kv_positions;
  float scale;
  int32_t reserved;
} ufp8_attn_desc;
int ufp8_attention_workspace(const ufp8_attn_desc* desc, int64_t* fwd_bytes, int64_t* saved_bytes,
                             int64_t* bwd_bytes);
int ufp8_attention_forward(const ufp8_attn_desc* desc, const void* q, const void* k, const void* v, void* out,
                           void* saved, void* workspace, ufp8_stream_t stream);
/* dq, dk, dv (bf16, shaped like q, k, v) of a loss with gradient dout at out. */
int ufp8_attention_backward(const ufp8_attn_desc* desc, const void* q, const void* k, const void* v, const void* out,
                            const void* dout, const void* saved, void* dq, void* dk, void* dv, void* workspace,
                            ufp8_stream_t stream);

/* ---- tensor-parallel reduce-scatter over NVLink peer memory ------------------------------
 * Replaces the reduce-scatter XLA/GSPMD would insert after the row-split down projection of
 * a tensor-parallel GMLP (implied by ueaj/model/mlp.py:96 'tensor' on the hidden axis and
 * ueaj/model/layer.py:57 token sharding).  A context owns two staging buffers (CUDA IPC,
 * plain peer mappings, no multicast objects), each holding one slot per source rank.
 * Per reduce-scatter: ufp8_tp_begin -> GEMM with UFP8_EPI_RS_PUSH -> ufp8_tp_finish, which
 * signals the peers, waits (bounded by the context timeout) for all of them, and sums the
 * slots in fp32 in rank order into `out`.  The context allocates its buffers with cudaMalloc
 * (the one exception to caller-owned memory). */
#define UFP8_IPC_HANDLE_BYTES 64
typedef struct ufp8_tp_ctx ufp8_tp_ctx;
int ufp8_tp_create(int rank, int world, int64_t slot_bytes, ufp8_tp_ctx** ctx, uint8_t* ipc_handle_out);
int ufp8_tp_connect(ufp8_tp_ctx* ctx, const uint8_t* ipc_handles /* world x UFP8_IPC_HANDLE_BYTES */);
/* Connects contexts that live in one process (one process driving several GPUs with peer
 * access, or one GPU for tests): peers[r] is the context of rank r. */
int ufp8_tp_connect_local(ufp8_tp_ctx* ctx, ufp8_tp_ctx* const* peers);
int ufp8_tp_destroy(ufp8_tp_ctx* ctx);
int ufp8_tp_set_timeout_ms(ufp8_tp_ctx* ctx, int ms);
int ufp8_tp_slot_bytes(const ufp8_tp_ctx* ctx, int64_t* slot_bytes);
int ufp8_tp_begin(ufp8_tp_ctx* ctx, void* const** slot_table, uint64_t* epoch);
int ufp8_tp_finish(ufp8_tp_ctx* ctx, uint64_t epoch, int64_t rows, int64_t cols, int64_t ld_slot, void* out,
                   int64_t ld_out, ufp8_stream_t stream);

/* This rank's buffer of `epoch`: *data = its slot region (slot s at *data + s * slot_bytes),
 * *flags = its k arrival flags.  Used by the all-gather below. */
int ufp8_tp_local(ufp8_tp_ctx* ctx, uint64_t epoch, void** data, uint32_t** flags);

/* All-gather over the same staging layout (replaces the all-gather GSPMD would insert before
 * the column-split gate/up projection and the down projection's input gradient, implied by
 * ueaj/model/layer.py:57 token sharding and ueaj/model/mlp.py:85 'tensor' on hidden): the
 * caller has written this rank's block (`bytes` <= slot_bytes, a multiple of 16) into its own
 * slot [rank] of the buffer of `epoch`; this call copies it into slot [rank] of the peers
 * rank-1, rank-2, ..., rank-(k-1) (mod k), in that order, and sets each peer's flag[rank] to
 * `epoch` once its copy is complete.  `stream` can run beside a GEMM that consumes the blocks
 * as they arrive (ufp8_gemm_desc.ag_*).  Engines:
 *   UFP8_AG_COPY_ENGINE  one cudaMemcpyAsync per peer, each followed by a stream write of the
 *                        flag (with a memory fence before it);
 *   UFP8_AG_SM           one small kernel (256-thread CTAs, no shared memory, so its CTAs fit
 *                        beside a persistent GEMM): 16-byte coalesced stores into the peers,
 *                        the last CTA of each destination sets its flag with a system-scope
 *                        release. */
#define UFP8_AG_COPY_ENGINE 0
#define UFP8_AG_SM 1
int ufp8_tp_ag_push(ufp8_tp_ctx* ctx, uint64_t epoch, int64_t bytes, int engine, ufp8_stream_t stream);

/* Copy lanes of a context (1..8, default 1): the copy-engine pushes (UFP8_AG_COPY_ENGINE and
 * ufp8_tp_rs_push_copy) spread their per-peer copies round-robin over this many streams,
 * forked from the caller's stream and joined back into it, so that several copy engines move
 * blocks at once; the flag of each all-gather block still follows its own copy. */
int ufp8_tp_set_copy_lanes(ufp8_tp_ctx* ctx, int lanes);

/* Reduce-scatter push by copy engines (the alternative to the UFP8_EPI_RS_PUSH epilogue when
 * independent work can run while the blocks travel): src holds this rank's partial sums,
 * k * rows rows of `cols` bf16 at pitch ld_src; block p (rows p*rows .. ) goes into slot
 * [rank] of rank p's buffer of `epoch` (from ufp8_tp_begin) at pitch cols, this rank's own
 * block included.  The copies are ordered before later work on `stream`; ufp8_tp_finish on
 * that stream (ld_slot = cols) then signals the peers and sums as after the epilogue push. */
int ufp8_tp_rs_push_copy(ufp8_tp_ctx* ctx, uint64_t epoch, const void* src, int64_t ld_src, int64_t rows,
                         int64_t cols, ufp8_stream_t stream);

/* MAX all-reduce of n (1..8) non-negative f32 values (per-tensor amax values) over the group
 * of a connected context: every rank's `out` receives the elementwise maximum of all ranks'
 * `in` (NaN propagates).  One single-warp kernel: P2P stores with a system-scope release into
 * each peer's exchange slot, then a bounded wait for all of them (UFP8_STATUS_PEER_TIMEOUT on
 * expiry, `out` then unchanged).  Replaces the MAX all-reduces of the local amax values that
 * global per-tensor scales need under tensor parallelism (the all-reduce GSPMD would insert
 * for a max over a sharded tensor).  Every rank must make the same sequence of calls. */
int ufp8_tp_allreduce_max(ufp8_tp_ctx* ctx, const float* in, float* out, int n, ufp8_stream_t stream);

/* Synchronises the current device, returns its status word in *status (0 = clean,
 * UFP8_STATUS_* bits otherwise) and clears it when `clear` is non-zero. */
int ufp8_device_status(int* status, int clear);

/* Number of CTAs the persistent GEMM launches (0 = one per SM, the default). */
int ufp8_set_gemm_ctas(int ctas);

/* GEMM kernel variant for this process: UFP8_GEMM_AUTO (default: the CTA-pair kernel, with
 * the ring stages of UFP8_GEMM_CTA_PAIR_WIDE for the epilogues that store directly),
 * UFP8_GEMM_SINGLE_CTA (128 x 256 tiles, one CTA each), UFP8_GEMM_CTA_PAIR (256 x 256
 * tiles on a cluster of two CTAs with tcgen05.mma.cta_group::2, ring stages of one 128-byte K
 * chunk, 7 deep; RS_PUSH rows leave through shared memory as bulk async stores and DSWIGLU
 * reads the saved U / G through TMA), UFP8_GEMM_CTA_PAIR_DIRECT (the same tiles with plain
 * 16-byte loads and stores in every epilogue) or UFP8_GEMM_CTA_PAIR_WIDE (UFP8_GEMM_CTA_PAIR
 * with ring stages of two 128-byte K chunks, 3 deep, for the epilogues that store directly) or
 * UFP8_GEMM_CTA_PAIR_N512 (256 x 512 tiles on a CTA pair, for bf16 STORE and SWIGLU outputs;
 * the others as UFP8_GEMM_CTA_PAIR). */
#define UFP8_GEMM_AUTO 0
#define UFP8_GEMM_SINGLE_CTA 1
#define UFP8_GEMM_CTA_PAIR 2
#define UFP8_GEMM_CTA_PAIR_DIRECT 3
#define UFP8_GEMM_CTA_PAIR_WIDE 4
#define UFP8_GEMM_CTA_PAIR_N512 5
int ufp8_set_gemm_variant(int variant);

/* Tile raster of the persistent GEMM: how many M tiles form a group that is swept along N
 * before the next group starts (0 = default 16).  Tuning knob for L2 reuse. */
int ufp8_set_gemm_raster(int group_m);

#ifdef __cplusplus
}
#endif

#endif /* UFP8_H_ */
