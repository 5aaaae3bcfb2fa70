/*
 * unblend_b200 — C ABI of the B200 (sm_100a) segmented separation forward.
 *
 * Every entry point is stream-ordered on the `stream` argument (a
 * cudaStream_t passed as void*), never synchronises, allocates nothing, and
 * returns 0 on success or a positive code (a cudaError_t value, or
 * UNBLEND_ERR_INVALID for bad arguments). The caller owns all memory: inputs,
 * outputs and workspaces are plain device pointers. Activations are
 * channels-last float32 unless a field says otherwise.
 *
 * The reference (Python/PyTorch) has no FFI for this path; each entry point
 * replaces the torch operator sequence named beside it, with the reference
 * file:line it restates.
 */
#ifndef UNBLEND_B200_H
#define UNBLEND_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define UNBLEND_ERR_INVALID 1000
#define UNBLEND_ERR_TOO_LARGE 1001 /* request exceeds a fixed built-in capacity */

/* Activation applied in a convolution epilogue. */
enum UnblendAct {
  UNBLEND_ACT_NONE = 0,
  UNBLEND_ACT_GELU = 1, /* exact erf GELU, F.gelu */
  UNBLEND_ACT_GLU = 2,  /* F.glu over interleaved (value, gate) column pairs */
  UNBLEND_ACT_TANH = 3, /* torch.tanh (BS-RoFormer mask estimator hidden layers) */
  UNBLEND_ACT_SWISH = 4 /* x * sigmoid(x) (SCNet ConvolutionModule, unblend/scnet.py:37-47) */
};

/* Transform applied to each input element as it is loaded. */
enum UnblendPrologue {
  UNBLEND_PRO_NONE = 0,
  UNBLEND_PRO_GN_GELU = 1, /* gelu((x - mean[g]) * rstd[g] * gamma[c] + beta[c]) */
  UNBLEND_PRO_ADD = 2      /* x + x2 (decoder skip connection) */
};

/*
 * Implicit-GEMM 2-D convolution over a channels-last tensor:
 *   y[b,ho,wo,n] = bias[n] + sum_{kh,kw,c} A(b, ho*sh+kh*dh-ph, wo*sw+kw*dw-pw, c) * w[n,kh,kw,c]
 * with zero padding outside [0,h_in) x [0,w_in). Covers every Conv1d/Conv2d
 * and Linear of the path (1-D convs use h=1; linears use h=1, kernel 1x1).
 * Weights are [n_out, kh, kw, c_in] row-major (K contiguous).
 * Output element (b,ho,wo,n') with n' = n (or n/2 after GLU) is written to
 *   out + b*out_sb + ho*out_sh + wo*out_sw + (n'/n_group)*out_sg + n'%n_group.
 * Epilogue order: bias, activation, then `out = res + scale[n'] * y` when
 * `res` is set (res may alias out), then optional GroupNorm statistics
 * (sum, sum of squares in double) per group (b) or (b, ho).
 */
typedef struct {
  int batch, h_in, w_in, c_in;
  long long in_sb, in_sh, in_sw;
  int h_out, w_out, n_out;
  int kh, kw, sh, sw, dh, dw, ph, pw;
  long long out_sb, out_sh, out_sw, out_sg;
  int n_group;
  int act;            /* UnblendAct */
  int prologue;       /* UnblendPrologue */
  /* prologue GN: float (mean, rstd) per group g = pro_group_per_h ? b*h_in + hi : b */
  const float* pro_stats;
  const float* pro_gamma;
  const float* pro_beta;
  int pro_group_per_h;
  const float* pro_x2; /* UNBLEND_PRO_ADD: second input, same strides as the input */
  /* residual epilogue */
  const float* res;
  const float* res_scale; /* [n'] or NULL for scale 1 */
  /* statistics epilogue: double[2*groups], group = b*(stats_per_h ? h_out : 1) + ... */
  double* stats;
  int stats_per_h;
  /* post-activation add (tensor-core kernel only; NULL elsewhere): output channel n'
   * of output row h gains post[h * post_sh + n'] after the activation / GLU (a
   * per-(row, channel) table such as HTDemucs' frequency embedding). */
  const float* post;
  long long post_sh;
  /* 1: y is bf16 (round to nearest even), tensor-core kernel only, for outputs that
   * feed bf16 consumers directly: no GLU, residual or output groups, n_out a multiple
   * of 32, whole 16-row tiles (the TMA bulk-store epilogue). */
  int y_bf16;
  /* 1: x is bf16 (tensor-core mode 3 only): activations a producing kernel wrote as
   * bf16 for a consumer that multiplies in bf16; unit stride along w, row strides
   * multiples of 8 elements. */
  int x_bf16;
} UnblendConvParams;

/* Conv1d / Conv2d / Linear (unblend/blocks.py:461,467,695,297,300; torch nn.Linear in
 * unblend/transformer.py:290-301,402-412) as an implicit GEMM, fp32 SIMT path. */
int unblend_conv2d_f32(const float* x, const float* w, const float* bias, float* y,
                       const UnblendConvParams* p, void* stream);

/* The same convolution on the tcgen05 tensor cores (TMA-fed implicit GEMM,
 * TMEM accumulator). mode 0: fp32 accuracy by the 3-pass TF32 split, weights
 * given as w_hi = w with the low 13 mantissa bits cleared and w_lo = w - w_hi
 * (fp32, [n_out, K]); mode 1: bf16 operands, w_hi is bf16 [n_out, K], w_lo
 * unused; mode 2: fp32 accuracy by the 3-pass bf16 split, w_hi = bf16(w) and
 * w_lo = bf16(w - w_hi) (bf16, [n_out, K]); mode 3: as mode 1 with bf16 x
 * (p->x_bf16 = 1; x is fp32 in the other modes); mode 4: as mode 2, with the
 * taps of each kernel row (up to three, shifts within 8 positions) sharing one
 * input load and split, block_n <= 128 (K summed in another order than mode 2).
 * block_n: 64, 96, 128, 192 or 256 output channels per tile. Requirements:
 * no prologue, c_in % 8 == 0 and >= 16, unit stride along w (or the stride-4
 * kernel-8 pad-2 time convolution, whose input rows up to a multiple of 4
 * past w_in must be zero), n_group and all output strides multiples of 4.
 * Replaces the same reference operators as unblend_conv2d_f32. */
int unblend_conv2d_tc(const void* x, const void* w_hi, const void* w_lo, const float* bias, float* y,
                      const UnblendConvParams* p, int mode, int block_n, void* stream);

/* Read the device flag that the tensor-core kernels set when a bounded
 * barrier wait gives up (0 = none); clear it when `clear` is non-zero.
 * Synchronous host call. */
int unblend_error_flag(int* out_host, int clear);

/* Per-group mean / rstd from the double (sum, sumsq) statistics:
 * mean = s/n, var = (sq - s*mean)/(n - unbiased), rstd = 1/sqrt(var + eps) when
 * `std_mode` is 0 (GroupNorm / LayerNorm); when 1, writes std = sqrt(var) and
 * the normaliser 1/(1e-5 + std) (HTDemucs input normalisation,
 * unblend/htdemucs.py:671-678). out: float[2*groups] = (mean, rstd_or_inv). */
int unblend_stats_finalize(const double* stats, float* out, int groups, double count,
                           float eps, int unbiased, int std_mode, void* stream);

/* Zero a double buffer (statistics accumulators). */
int unblend_zero_f64(double* p, long long n, void* stream);

/* Zero `count` blocks of n floats starting `stride` floats apart (count 1: one
 * contiguous run, e.g. overlap-add accumulators; count > 1: padding rows of a
 * batch of activations, stride >= n). p 4-byte aligned. */
int unblend_zero_f32(float* p, long long n, int count, long long stride, void* stream);

/* Sum / sum of squares per group of a contiguous [groups, n] fp32 array (double). */
int unblend_group_sums(const float* x, double* stats, int groups, long long n, void* stream);

/*
 * Normalise + optionally apply affine + activation elementwise:
 *   y[r, c] = act((x[r,c] - mean[g]) * rstd[g] * gamma[c] + beta[c])
 * for rows r of a [rows, c] tensor with group g = r / rows_per_group.
 * gamma/beta may be NULL (1 and 0). act: UnblendAct (GLU not allowed).
 */
int unblend_group_norm_apply(const float* x, float* y, const float* stats2, const float* gamma,
                             const float* beta, long long rows, int c, long long rows_per_group,
                             int act, void* stream);

/* DConv tail (unblend/blocks.py:293-317): x += scale * glu(gn(z)) per element.
 * z is contiguous [groups, rows_per_group, 2c] with interleaved (value, gate)
 * columns and GroupNorm(1) stats2 = (mean, rstd) per group; x element
 * (g, r, ch) lives at x + g*x_group_stride + r*c + ch. gamma/beta are in the
 * interleaved column order of z. */
int unblend_dconv_tail(float* x, const float* z, const float* stats2, const float* gamma,
                       const float* beta, const float* scale, long long groups,
                       long long rows_per_group, int c, long long x_group_stride, void* stream);

/* Fused DConv layer (unblend/blocks.py:238-317) in streaming passes: conv1,
 * then the GN2 statistics from moments (dconv_moments / dconv_moment_sums,
 * below), then apply.
 * x element (g, r, c) is at x + g*x_gs + r*c_in + c for groups g (GroupNorm
 * groups: (batch, frequency) rows or batch items) and rows r along time.
 * The hidden width hid is padded to hs = round_up(hid, 4): h rows, W1 rows,
 * the GN1 affine and W2 rows hold hs values, those past hid zero (so the
 * padded hidden channels stay exactly 0 and meet zero weights).
 * conv1: h[g, r, :] = b1 + sum_t W1[:, t, :] x[g, r + (t-1)*dil, :] (zero
 *   padded), W1 [hs, 3, c]; accumulates (sum, sumsq) of h per group into
 *   stats (double, zeroed by the caller). Shared memory must hold
 *   (128 + 2*dil)*(c+4) + 3*hs*c floats (<= 220 KiB).
 * apply: x += scale * glu(gn2(z)) with z = W2 gelu(gn1(h)) + b2 recomputed,
 *   st1 = (mean, rstd) of h, W2 [2c, hs] rows interleaved (value, gate),
 *   st2 = (mean, rstd) of z,
 *   GN2 affine interleaved like W2. z is never stored. With h_is_act != 0, h
 *   already holds a = gelu(gn1(h)) rows (written by dconv_moments' a_out;
 *   st1, g1w, g1b unused and may be null; hid <= 16). */
int unblend_dconv_conv1(const float* x, long long x_gs, int groups, int rows, int c, const float* w1,
                        const float* b1, int hid, int dil, float* h, double* stats, void* stream);
int unblend_dconv_apply(float* x, long long x_gs, const float* h, int groups, int rows, int hid, int c,
                        const float* st1, const float* g1w, const float* g1b, const float* w2,
                        const float* b2, const float* st2, const float* g2w, const float* g2b,
                        const float* scale, int h_is_act, void* stream);

/* GN2 statistics of the DConv 1x1 output z = W2 a + b2 (a = GELU(GN1(h))) from
 * the moments of a, for the thin levels (hid <= 16):
 * dconv_moments adds, per group g, S1[j] = sum_r a[r, j] and
 * S2[j, k] = sum_r a[r, j] a[r, k] (j <= k, upper triangle row by row) into
 * moments[g * K ...], K = hw + hw (hw + 1) / 2, hw the computed hidden width
 * (hid when even, else hid rounded up to a multiple of 4); moments are double
 * and zeroed by the caller.
 * dconv_moment_sums turns them into (sum z, sum z^2) per group for
 * unblend_stats_finalize, from coef = [W2^T 1 (hw), W2^T b2 (hw), W2^T W2 as
 * the same packed triangle with off-diagonal entries doubled, sum b2,
 * sum b2^2] (double, over all 2c rows of W2): hw + hw(hw+1)/2 operations per
 * row instead of the 2 c hw of evaluating z. a_out (nullable,
 * 16-byte aligned, may be h itself) receives the rows of a (hs floats each,
 * zero past hw) for dconv_apply with h_is_act. */
int unblend_dconv_moments(const float* h, int groups, int rows, int hid, const float* st1, const float* g1w,
                          const float* g1b, double* moments, float* a_out, void* stream);
int unblend_dconv_moment_sums(const double* moments, const double* coef, int groups, int rows, int hid,
                              double* sums, void* stream);

/* Device flag set when a bounded wait of the DConv apply kernel gives up (0 = none). Synchronous host call. */
int unblend_dconv_error_flag(int* out_host, int clear);

/* LayerNorm over the last dim (eps 1e-5) with optional additive table:
 * y[r,:] = ln(x[r,:]) * gamma + beta + (pos ? pos_scale * pos[r % pos_rows, :] : 0). */
int unblend_layer_norm(const float* x, float* y, const float* gamma, const float* beta,
                       const float* pos, float pos_scale, long long pos_rows, long long rows,
                       int c, void* stream);

/* The same LayerNorm written as bf16 (round to nearest even), for rows that only feed
 * bf16 tensor-core GEMMs (the transformer projections and FeedForward input in bf16
 * precision): replaces the same torch nn.LayerNorm (unblend/transformer.py:328-359). */
int unblend_layer_norm_bf16(const float* x, void* y, const float* gamma, const float* beta,
                            const float* pos, float pos_scale, long long pos_rows, long long rows,
                            int c, void* stream);

/* Multi-head attention core softmax(Q K^T * scale) V for all heads
 * (torch nn.MultiheadAttention, unblend/transformer.py:290-301, 402-412).
 * Q rows are [b, lq, q_stride] with head h at columns h*hd; K, V likewise.
 * Output [b, lq, heads*hd]. */
int unblend_attention_f32(const float* q, const float* k, const float* v, float* out, int batch,
                          int heads, int lq, int lk, int hd, long long q_sb, long long q_sr,
                          long long kv_sb, long long kv_sr, long long o_sb, long long o_sr,
                          float scale, void* stream);

/* The same attention on the tcgen05 tensor cores (flash attention: S and O in
 * TMEM, P written back to TMEM as the A operand of the PV product, V
 * transposed in shared memory). mode 0: 3-pass TF32 split for fp32 accuracy;
 * mode 1: single-pass TF32 with round-to-nearest operands; mode 2: 3-pass bf16
 * split (hi = bf16(x), lo = bf16(x - hi)) for fp32 accuracy. Requires hd <= 64,
 * hd % 4 == 0, strides that are multiples of 4 elements and 16-byte aligned
 * base pointers. */
int unblend_attention_tc(const float* q, const float* k, const float* v, float* out, int batch,
                         int heads, int lq, int lk, int hd, long long q_sb, long long q_sr,
                         long long kv_sb, long long kv_sr, long long o_sb, long long o_sr,
                         float scale, int mode, void* stream);

/* Device flag set when a bounded wait of the attention kernel gives up
 * (0 = none); cleared when `clear` is non-zero. Synchronous host call. */
int unblend_attention_error_flag(int* out_host, int clear);

/*
 * Attention with a two-level batch and BS-RoFormer's fusions (gated rotary
 * Attention, unblend/roformer.py:478-511; axial sequences of
 * _run_transformers, unblend/roformer.py:1135-1159). Sequence (o, i) of Q has
 * row r, head h, dim d at q + o*q_so + i*q_si + r*q_sr + h*hd + d (K and V
 * share the kv_* strides; the output likewise with o_*). Optional:
 *   rope  float[rope_len, hd/2, 2] (cos, sin) of position r * freq: Q and K
 *         rows are rotated (interleaved pairs) before QK^T;
 *   gate  float, the output row of head h is multiplied by
 *         gate[o*g_so + i*g_si + r*g_sr + h];
 *   out_bf16  write the output as bf16 instead of fp32.
 * mode as in unblend_attention_tc; same alignment rules.
 */
typedef struct {
  int outer, inner, heads, lq, lk, hd;
  long long q_so, q_si, q_sr;
  long long kv_so, kv_si, kv_sr;
  void* out;
  long long o_so, o_si, o_sr;
  int out_bf16;
  const float* gate;
  long long g_so, g_si, g_sr;
  const float* rope;
  int rope_len;
  float scale;
} UnblendAttnParams;

int unblend_attention_tc2(const float* q, const float* k, const float* v, const UnblendAttnParams* p, int mode,
                          void* stream);

/* The same attention with bf16 Q, K, V (head dim 64) on kind::f16 tensor cores:
 * a persistent flash-attention kernel over (sequence, head, 128-query) units,
 * fp32 softmax and accumulation, P rounded to bf16. Strides as in
 * unblend_attention_tc2 (elements of the bf16 tensors, multiples of 8); rope
 * must be NULL (apply the rotation when producing Q and K, e.g. in
 * unblend_gemm_tc); gate and out_bf16 as there. */
int unblend_attention_bf16(const void* q, const void* k, const void* v, const UnblendAttnParams* p,
                           void* stream);

/* Device flag of unblend_attention_bf16's bounded waits (0 = none). Synchronous host call. */
int unblend_attention_bf16_error_flag(int* out_host, int clear);

/*
 * Grouped linear layers on the tcgen05 tensor cores (nn.Linear of
 * BS-RoFormer's Attention / FeedForward, unblend/roformer.py:274-308, 478-511,
 * and the per-band linears of BandSplit / MaskEstimator, 673-800).
 * A is [rows, a_cols] with leading dimension lda (elements); W is
 * [w_rows, w_cols] row-major. Each group g computes, for every row r,
 *   y[j] = act(sum_{k < K_g} A[r, a_col0 + k] * W[w_row0 + j, k] + bias[w_row0 + j]), j < n,
 * where K_g is k rounded up to the K chunk (32 fp32 / 64 bf16 elements): the
 * weights must be zero in columns k..K_g-1 (A columns past a_cols read as 0).
 * With act = UNBLEND_ACT_GLU weight rows are interleaved (value, gate) pairs
 * and y has n/2 columns. With rope set, each (even, odd) column pair j < rope_cols
 * is rotated by rope[pos, (j % rope_hd) / 2] = (cos, sin), pos = (r / rope_div) %
 * rope_mod (the rotary embedding of Q and K, unblend/roformer.py:251-271; rope is
 * float[rope_mod, rope_hd/2, 2]). The result (plus res[r, c] when res is set; res
 * may alias out) goes to out[r * ldo + out_col0 + c] as fp32 or bf16.
 * mode 0: A and W fp32 (W as TF32 hi/lo split like unblend_conv2d_tc), 3-pass
 * TF32; mode 1: A and W bf16. block_n: 64, 128 or 256.
 * Alignment: A, W 16-byte aligned, lda, w_cols and every a_col0 multiples of
 * 16 bytes' worth of elements.
 */
#define UNBLEND_GEMM_MAX_GROUPS 64
typedef struct {
  int a_col0, w_row0, n, k, out_col0;
} UnblendGemmGroup;

typedef struct {
  int groups;
  const UnblendGemmGroup* group; /* host array of `groups` entries */
  const float* bias;             /* [w_rows] or NULL */
  int act;                       /* UnblendAct */
  const float* res;              /* fp32 residual or NULL */
  long long ldr;
  void* out;
  long long ldo;
  int out_bf16;
  const float* rope; /* optional rotary table (act must be NONE) */
  int rope_cols, rope_hd, rope_div, rope_mod;
} UnblendGemmParams;

int unblend_gemm_tc(const void* a, long long lda, int rows, int a_cols, const void* w_hi, const void* w_lo,
                    long long w_rows, int w_cols, const UnblendGemmParams* p, int mode, int block_n,
                    void* stream);

/* Device flag of the grouped GEMM's bounded waits (0 = none). Synchronous host call. */
int unblend_gemm_error_flag(int* out_host, int clear);

/* RMSNorm over the last dim (F.rms_norm, eps 1e-12; unblend/roformer.py:60-91) of
 * contiguous fp32 rows [rows, dim] into y (fp32 or bf16, leading dim ldy); dim
 * % 4 == 0, dim <= 1024. With gates > 0 (<= 16) also writes the attention gates
 * gate_out[r, h] = sigmoid(y[r] . gate_w[h] + gate_b[h]) (unblend/roformer.py:478-511)
 * computed from the fp32 normalised row; gate_w is [gates, dim]. */
int unblend_rms_norm(const float* x, long long rows, int dim, const float* gamma, void* y, long long ldy,
                     int y_bf16, const float* gate_w, const float* gate_b, int gates, float* gate_out,
                     void* stream);

/* Per-band RMSNorm of BandSplit (unblend/roformer.py:673-705): band b is columns
 * [band_start[b], band_start[b+1]) of each fp32 row of x (leading dim ldx);
 * band_start is a device int array of bands+1 multiples of 4; gamma holds the
 * bands' weights back to back in column order. Band b is written from column
 * y_start[b] of y (device array of multiples of 4), or band_start[b] when
 * y_start is NULL. */
int unblend_band_rms_norm(const float* x, long long rows, long long ldx, const int* band_start, int bands,
                          const float* gamma, void* y, long long ldy, int y_bf16, const int* y_start,
                          void* stream);

/* Mel-Band RoFormer band gather (unblend/roformer.py:1541-1544, index_select):
 * dst[r, 2j + k] = src[r, 2 idx[j] + k] for k in {0, 1}, j < n; idx is a device
 * int array of pair indices into the channel-interleaved (bin, channel) axis.
 * src/dst 8-byte aligned, even leading dims (floats). */
int unblend_gather_pairs(const float* src, long long src_ld, long long rows, const int* idx, int n, float* dst,
                         long long dst_ld, void* stream);

/* Mel-Band RoFormer mask scatter-average (unblend/roformer.py:1561-1575,
 * scatter_add_ then divide by the covering band count):
 * dst[r, 2c + k] = sum_{q in [offsets[c], offsets[c+1])} src[r, 2 pos[q] + k] / count_c,
 * summed in ascending q; offsets (n_dst + 1 ints) and pos are device arrays. */
int unblend_scatter_mean_pairs(const float* src, long long src_ld, long long rows, const int* offsets,
                               const int* pos, int n_dst, float* dst, long long dst_ld, void* stream);

/* y[i] = bf16(x[i]) (round to nearest even); n a multiple of 4, x 16-byte and
 * y 8-byte aligned. Feeds fp32 projections to the bf16 attention kernel. */
int unblend_cast_bf16(const float* x, void* y, long long n, void* stream);

/* Audio I/O edges (unblend/api.py:1080-1112, unblend/audio.py:14-90), fp32 planar [channels, frames]:
 * pcm16_to_f32: interleaved int16 [frames, cin] -> dst[cout, frames] = x / 32768 with the channel
 *   conversion of convert_audio_channels (same count: copy; cout 1: mean; cin 1: replicate;
 *   cin > cout: the first cout); cin, cout <= 8.
 * convert_channels: the same conversion on fp32 planar input.
 * resample: y[c, k*lout + p] = sum_{m < taps} x[c, k*lin + m - width] * kern[p, m] (x zero outside
 *   [0, length)), out_length outputs per channel; kern [lout, taps] is the polyphase filter bank.
 * max_abs: atomically maxes max|x| (as float bits) into *out_bits (zeroed by the caller).
 * prevent_clip: mode 1 y = x / max(1.01 max|x|, 1) reading *maxabs_bits; 2 clamp to [-0.99, 0.99];
 *   3 tanh. */
int unblend_pcm16_to_f32(const void* src, int cin, long long frames, float* dst, int cout, void* stream);
int unblend_convert_channels(const float* x, int cin, long long frames, float* y, int cout, void* stream);
int unblend_resample(const float* x, int channels, long long length, const float* kern, int taps, int lin,
                     int lout, int width, float* y, long long out_length, void* stream);
int unblend_max_abs(const float* x, long long n, unsigned* out_bits, void* stream);
int unblend_prevent_clip(const float* x, float* y, long long n, int mode, const unsigned* maxabs_bits,
                         void* stream);

/* 16-bit PCM export of one stem (unblend/api.py:94-148 export_stem -> prevent_clip, then the
 * encoder's float -> s16 conversion): x planar fp32 [channels, frames] -> dst interleaved int16
 * [frames, channels]; the clipping guard of prevent_clip applied first (mode 0 none, 1-3 as above),
 * then q = saturate_s16(round_half_even(v * 32768)); NaN -> 0. channels <= 8. */
int unblend_encode_pcm16(const float* x, int channels, long long frames, int mode, const unsigned* maxabs_bits,
                         void* dst, void* stream);

/* Elementwise y[i] = a[i] + alpha * b[i % b_period] (skip adds, embeddings). */
int unblend_add(const float* a, const float* b, float* y, long long n, long long b_period,
                float alpha, void* stream);

/*
 * HTDemucs STFT front end (unblend/htdemucs.py:370-395, unblend/blocks.py:60-88):
 * mix [batch, 2, length] (channel-first, as given to forward) ->
 * spec [batch, nfft/2, frames, 4] channels-last CaC (c0.re, c0.im, c1.re, c1.im),
 * frames = ceil(length / hop), hop = nfft/4, Hann window (periodic), normalized.
 * window: float[nfft]. Only nfft = 4096 is supported.
 */
int unblend_stft_cac(const float* mix, float* spec, const float* window, int batch, int length,
                     int nfft, void* stream);

/* y = (x - mean[b]) / (1e-5 + std[b]) over a contiguous [batch, n] array with
 * stats2 = (mean, std) per batch (unblend/htdemucs.py:671-673). */
int unblend_standardize(const float* x, float* y, const float* stats2, long long n_per_batch,
                        int batch, void* stream);

/* Transpose + normalise the time branch input: mix [b, 2, L] -> xt [b, L_pad, 2]
 * with (x - mean[b]) / (1e-5 + std[b]); rows L..L_pad-1 are zero. stats2 = (mean, std) per b. */
int unblend_time_input(const float* mix, float* xt, const float* stats2, int batch, int length,
                       int length_pad, void* stream);

/*
 * HTDemucs output stage (unblend/htdemucs.py:692-704, _ispec :397-412,
 * ispectro unblend/blocks.py:165-204):
 *   out[b,s,c,n] = istft(spec*std+mean)[b,s,c,n] + xt[b, n, s*2+c] * stdt + meant
 * spec: [batch, nfft/2, frames, S*4] channels-last CaC; xt: [batch, >=length, S*2];
 * fstats/tstats: float (mean, std) per batch; frames_buf: workspace of
 * batch*S*2*frames*nfft floats. out: [batch, S, 2, length].
 */
int unblend_istft_output(const float* spec, const float* xt, long long xt_sb, const float* fstats,
                         const float* tstats, const float* window, float* frames_buf, float* out,
                         int batch, int sources, int length, int nfft, void* stream);

/*
 * BS-RoFormer STFT (unblend/roformer.py:1320-1345): torch.stft with center=True
 * (reflect padding of nfft/2), Hann window (periodic, length nfft), not
 * normalised, any hop, of both channels of mix [batch, 2, length] into the
 * frame-major feature layout out[batch, frames, nfft/2+1, 2 (channel), 2 (re, im)],
 * frames = 1 + length / hop. nfft: 2048 or 4096; length > nfft/2.
 */
int unblend_stft_frames(const float* mix, float* out, const float* window, int batch, int length, int nfft,
                        int hop, void* stream);

/*
 * BS-RoFormer output (unblend/roformer.py:1346-1379, 1176-1189): for each stem s,
 * X = stft * mask_s as complex numbers (both [batch, frames, nfft/2+1, 2, 2];
 * mask_s at mask + s*mask_ss), DC bin zeroed when zero_dc, then torch.istft
 * (center, Hann, not normalised, window-square envelope) trimmed to `length`:
 * out[batch, stems (+1), 2, length]. With `complement` (stems must be 1) a second
 * stem mix - stem 0 is appended. frames_buf: batch*stems*2*frames*nfft floats.
 * A null stft stands for a unit spectrum: the masks themselves are inverted
 * (SCNet's decoder output, unblend/scnet.py:775-782).
 */
int unblend_istft_masked(const float* stft, const float* mask, long long mask_ss, const float* window,
                         const float* mix, float* frames_buf, float* out, int batch, int stems, int complement,
                         int length, int nfft, int hop, int zero_dc, void* stream);

/* Per-batch (mean, std) with torch.var_mean semantics (unbiased) of a contiguous
 * [batch, n] array; out float[2*batch] = (mean, std). Uses `work` double[2*batch]. */
int unblend_mean_std(const float* x, double* work, float* out, int batch, long long n,
                     void* stream);

/* Largest batch unblend_mean_std_noalloc takes (its static accumulator holds
 * 2 doubles per batch item: 64 KiB). */
#define UNBLEND_NOALLOC_MAX_BATCH 4096

/* unblend_mean_std without the caller-provided `work` buffer. This entry point
 * has no counterpart in the reference; it exists for callers that cannot
 * allocate device memory at call time (a real-time audio thread, where
 * cudaMalloc may stall on a device-wide synchronisation, or a host whose own
 * memory manager owns all device allocations). Its accumulator is a static
 * device array of UNBLEND_NOALLOC_MAX_BATCH batch items (64 KiB, held by every
 * GPU that loads the library until process exit); larger batches return
 * UNBLEND_ERR_TOO_LARGE. It calls no allocator. The first call on each device
 * looks up the array's device address (cudaGetSymbolAddress) with that device
 * current, so make that first call before any stream capture; the address is
 * looked up again when the device's current CUDA context changes (after
 * cudaDeviceReset, or under a context the host created itself). All calls
 * share the one array: each call clears the part it uses, and calls that
 * overlap on the GPU (e.g. on two streams at once) race with each other. */
int unblend_mean_std_noalloc(const float* x, float* out, int batch, long long n, void* stream);

/* Segment engine (unblend/apply.py:278-311, 406-432, 1219-1238, 1329). */
/* Gather centred, zero-padded chunks: batch[i, c, :] = track[c, start_i ...] for
 * i < n, where start_i = offsets[i] - (segment - min(L - offsets[i], segment)) / 2.
 * offsets is a device array of n int64 values. */
int unblend_gather_chunks(const float* track, int channels, long long length, const long long* offsets,
                          int n, int segment, float* batch, void* stream);

/* Weighted overlap-add of model outputs y[i, rows, segment] (rows = S*C) into
 * acc[rows, L] and sum_w[L] with the triangular weight raised to `power` (the
 * reference's transition_power, > 0), after the centre trim of short chunks.
 * Positions [lo, hi) are visited; they must cover every position the n chunks
 * touch. offsets ascend (as the segment plan produces them). */
int unblend_overlap_add(const float* y, int n, int rows, int segment, const long long* offsets,
                        long long length, long long lo, long long hi, float power, float* acc, float* sum_w,
                        void* stream);

/* In place: y[i, r, trim_i + j] *= weight(j)^power for j < len_i, where len_i =
 * min(L - offsets[i], segment) and trim_i = (segment - len_i) / 2 (the centre
 * trim). The weighted contributions of a batch for accumulation on the host
 * when the track's accumulators do not fit the device
 * (unblend/apply.py:1058-1085, 1211-1238). */
int unblend_weight_chunks(float* y, int n, int rows, int segment, const long long* offsets, long long length,
                          float power, void* stream);

/* out = acc / sum_w (broadcast over [S*C, L]). */
int unblend_divide(const float* acc, const float* sum_w, float* out, int rows, long long length,
                   void* stream);

/* SCNet (unblend/scnet.py). Activations are channels-last [B, F, T, C]. */

/* y[r, i] = i < n_in ? x[r, i] : 0 for i < n_out: the segment's trailing zeros
 * before the STFT (stft_padding, unblend/scnet.py:543-572). */
int unblend_pad_tail(const float* x, float* y, int rows, long long n_in, long long n_out, void* stream);

/* x [batch, n1, n2, groups*4] -> y [groups, batch, n2, n1, 4] (elements of 4
 * floats; 16-byte aligned buffers), plus add[c * n2 + j] on channel c of
 * element (., j) when `add` is given (groups must then be 1). Turns the
 * frame-major STFT [B, T, F, 4] into [B, F, T, 4] (with SCNetMasked's
 * frequency embedding, unblend/scnet.py:868-874) and the decoder output
 * [B, F, T, 4S] into per-stem iSTFT input [S, B, T, F, 4]. */
int unblend_swap_axes(const float* x, float* y, const float* add, int batch, int n1, int n2, int groups,
                      void* stream);

/* ConvolutionModule depthwise Conv1d (kernel 3, padding 1, groups = channels;
 * unblend/scnet.py:78-86) along T of z [rows, T, c]: u = b + sum_k w[c, k]
 * z[t + k - 1]; stats[2r], stats[2r + 1] = sum and sum of squares of row r of u
 * (double, written, not accumulated) for the GroupNorm(1) that follows. */
int unblend_depthwise3(const float* z, const float* w, const float* bias, float* u, double* stats, int rows,
                       int t_len, int c, void* stream);

/* y[k * y_stride + j] = act(x[k * x_stride + j]) for k < count, j < n; act one
 * of NONE, GELU, TANH, SWISH; in place when x == y with equal strides. */
int unblend_act_copy(const float* x, long long x_stride, float* y, long long y_stride, int count, long long n,
                     int act, void* stream);

/* FeatureConversion (unblend/scnet.py:333-437): orthonormal real DFT along T
 * of x [rows, T, c] (T even) into y [rows, T/2 + 1, 2c] (real parts on the first
 * c channels, imaginary parts on the next c), and its inverse from
 * [rows, K, 2c] to [rows, 2 (K - 1), c] (imaginary parts of the first and last
 * bins ignored, as torch.fft.irfft). */
int unblend_rfft_time(const float* x, float* y, int rows, int t_len, int c, void* stream);
int unblend_irfft_time(const float* y, float* x, int rows, int n_bins, int c, void* stream);

/* Bidirectional single-layer LSTM recurrence (torch.nn.LSTM; DualPathRNN,
 * unblend/scnet.py:440-500). xp rows hold the gate pre-activations
 * W_ih x + b_ih + b_hh as [forward (i, f, g, o) x hid | reverse ...] (8 hid
 * floats); whh_t is [2][hid][4 hid] (W_hh transposed, forward then reverse);
 * h_out rows receive [forward h | reverse h] (2 hid floats). Sequence s step t
 * is row (s / inner) * outer_stride + (s % inner) * inner_stride +
 * t * step_stride of both; the reverse direction runs t from steps - 1 down.
 * hid: 32, 64, 128, 256 or 512. */
int unblend_lstm_recurrence(const float* xp, const float* whh_t, float* h_out, int n_seq, int steps, int hid,
                            int inner, long long outer_stride, long long inner_stride, long long step_stride,
                            void* stream);

/* The same recurrence for the bf16 precision setting on the tensor cores: W_hh and h
 * rounded to bf16 for the W_hh h product (fp32 accumulation, cell state and input
 * projections); xp 16-byte aligned; hid 128 or 256 (other sizes: unblend_lstm_recurrence). */
int unblend_lstm_recurrence_bf16(const float* xp, const float* whh_t, float* h_out, int n_seq, int steps, int hid,
                                 int inner, long long outer_stride, long long inner_stride, long long step_stride,
                                 void* stream);

/* Device flag set when a bounded wait of unblend_lstm_recurrence_bf16 gives up (0 = none). Synchronous. */
int unblend_lstm_error_flag(int* out_host, int clear);

#ifdef __cplusplus
}
#endif

#endif /* UNBLEND_B200_H */
