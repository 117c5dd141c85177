/*
 * d1kernels.h — the C ABI of libd1kernels, the sm_100a (B200) kernel library of the d1rs forward pass.
 *
 * This is a drop-in for the static library that the reference's build.rs:11-40 archives from
 * cuda/kernels.cu + cuda/gemm.cu. Every symbol below keeps the name, argument order, argument meaning and
 * return-code convention of the declaration the Rust host binds in src/cuda.rs:102-175, so src/model.rs,
 * src/vision.rs, src/audio.rs and src/engine.rs call it unchanged.
 *
 * Conventions (same as the reference):
 *   - Every pointer argument is a device pointer unless noted; rows are row-major.
 *   - Launchers are asynchronous on `stream` and return 0 on success, a cudaError_t value on a launch error,
 *     or -1 for an unsupported argument (the reference returns -1 for an unsupported hidden size,
 *     cuda/kernels.cu:654). n = 0 is a no-op that returns 0.
 *   - fp16 arguments are IEEE binary16 (`d1_half`, ABI-identical to `__half` and to the Rust `u16`).
 *
 * Symbols added beyond the reference surface are grouped at the end, each marked "extension".
 */
#ifndef D1KERNELS_H
#define D1KERNELS_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __CUDACC__
#include <cuda_fp16.h>
typedef __half d1_half;
#else
typedef uint16_t d1_half; /* IEEE binary16 bit pattern */
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Per-sequence metadata of a packed batch. Layout of `SeqInfo` in cuda/kernels.cu:15-24 and src/cuda.rs:59-70
 * (48 bytes, repr(C)). */
typedef struct SeqInfo {
    int start;              /* first row in the packed buffer */
    int len;                /* number of rows */
    int pos_off;            /* RoPE position of the first row (media prefix length for text after a prefix) */
    int qtype;              /* decision-head question type (row of the type embedding) */
    const d1_half* ext_bx;  /* [n_conv][D] conv state of the prefix's last position, or NULL */
    d1_half* save_bx;       /* prefix pass: store this sequence's last-position conv state [n_conv][D] */
    d1_half* save_k;        /* prefix pass: [n_attn][len][kv_dim] */
    d1_half* save_v;
} SeqInfo;

/* Attention metadata per sequence. Layout of `AttnSeq` in cuda/kernels.cu:26-32 and src/cuda.rs:88-99
 * (40 bytes, repr(C)). Keys are [ext prefix keys | local keys]. */
typedef struct AttnSeq {
    int q_start, q_len;     /* query rows */
    int kv_start, kv_len;   /* local key/value rows */
    int ext_len, _pad;      /* external (cached prefix) keys, placed before the local ones */
    const d1_half* ext_k;   /* [ext_len][ext_ld], already offset to this layer and kv head 0 */
    const d1_half* ext_v;
} AttnSeq;

#ifdef __cplusplus
static_assert(sizeof(SeqInfo) == 48, "SeqInfo must match src/cuda.rs:59-70");
static_assert(offsetof(SeqInfo, ext_bx) == 16 && offsetof(SeqInfo, save_v) == 40, "SeqInfo layout");
static_assert(sizeof(AttnSeq) == 40, "AttnSeq must match src/cuda.rs:88-99");
static_assert(offsetof(AttnSeq, ext_k) == 24 && offsetof(AttnSeq, ext_v) == 32, "AttnSeq layout");
#endif

/* ------------------------------------------------------------------------------------------------ norms */

/* y16 = x * rsqrt(mean(x^2) + eps) * w, per row of D in {512, 768, 1024}.
 * Replaces d1_rmsnorm, cuda/kernels.cu:648-657 (decl. src/cuda.rs:105). */
int d1_rmsnorm(const float* x, const float* w, d1_half* y, int rows, int D, float eps, cudaStream_t stream);

/* x += pend_scale * pend_bias (written back when pend_bias != NULL), then LayerNorm(x)*w + b into y (fp16,
 * optional) and/or yf (fp32, optional, may alias x). D in {512, 768, 1024}.
 * Replaces d1_layernorm, cuda/kernels.cu:659-669 (decl. src/cuda.rs:106-109). */
int d1_layernorm(float* x, const float* pend_bias, float pend_scale, const float* w, const float* b, d1_half* y,
                 float* yf, int rows, int D, float eps, cudaStream_t stream);

/* out = RMSNorm(h) * w + type_emb[seqs[tok_seq[row]].qtype], D = 1024, fp32 -> fp32 (out may alias h).
 * Replaces d1_head_init, cuda/kernels.cu:671-675 (decl. src/cuda.rs:110-113). */
int d1_head_init(const float* h, const float* w, const float* type_emb, const int* tok_seq, const SeqInfo* seqs,
                 float* out, int rows, float eps, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------------ elementwise */

/* h[row] = (float)table[ids[row]], D even. Replaces d1_embed, cuda/kernels.cu:677-681 (src/cuda.rs:114). */
int d1_embed(const d1_half* table, const int* ids, float* h, int rows, int D, cudaStream_t stream);

/* out[t][i] = silu(gu[t][i]) * gu[t][F+i]. Replaces d1_swiglu, cuda/kernels.cu:683-686 (src/cuda.rs:115). */
int d1_swiglu(const d1_half* gu, d1_half* out, int rows, int F, cudaStream_t stream);

/* x = act(x + bias) in place, fp16; act 0 none, 1 ReLU, 2 GELU-erf, 3 GELU-tanh, 4 SiLU (cuda/kernels.cu:46-54).
 * Replaces d1_bias_act_h, cuda/kernels.cu:688-691 (src/cuda.rs:116). */
int d1_bias_act_h(d1_half* x, const float* bias, int rows, int N, int act, cudaStream_t stream);

/* x = act(x + bias) in place, fp32. Replaces d1_bias_act_f, cuda/kernels.cu:693-696 (src/cuda.rs:117). */
int d1_bias_act_f(float* x, const float* bias, int rows, int N, int act, cudaStream_t stream);

/* out[t][i] = bias[i] (+ add[t][i]). Replaces d1_fill_rows, cuda/kernels.cu:698-701 (src/cuda.rs:118). */
int d1_fill_rows(float* out, const float* bias, const float* add, int rows, int N, cudaStream_t stream);

/* y = (half)x, n elements. Replaces d1_f32_to_f16, cuda/kernels.cu:703-706 (src/cuda.rs:119). */
int d1_f32_to_f16(const float* x, d1_half* y, size_t n, cudaStream_t stream);

/* dst[i] = src[idx[i]] for rows of row_bytes bytes (a multiple of 16).
 * Replaces d1_gather_rows, cuda/kernels.cu:708-712 (src/cuda.rs:120-122). */
int d1_gather_rows(const void* src, void* dst, const int* idx, int n, int row_bytes, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------------ trunk mixers */

/* Double-gated centred 3-tap short conv over bcu [rows][3D] = [b | c | u]:
 * out[t] = c[t] * (w0*bx[t-1] + w1*bx[t] + w2*bx[t+1]), bx = b*u, zero outside each sequence; the left neighbour
 * of a sequence's first row is seqs[].ext_bx (prefix state) when given; a sequence's last bx is stored to
 * seqs[].save_bx when given. convw is f32 [D][3].
 * Replaces d1_shortconv, cuda/kernels.cu:714-718 (src/cuda.rs:123-126). */
int d1_shortconv(const d1_half* bcu, const float* convw, const int* tok_seq, const SeqInfo* seqs, d1_half* out,
                 int rows, int D, int conv_idx, cudaStream_t stream);

/* Per-head RMSNorm (head dim 64) of the q and k heads of each qkv row (in place), then RoPE rotate-half on the
 * pairs (l, l+32) with pos = row-in-sequence + pos_off; rope is float2 (cos, sin) [pos][32]. When seqs[].save_k
 * / save_v are set, the normed+rotated K and the raw V are stored to the prefix cache at layer attn_idx.
 * Replaces d1_qk_norm_rope, cuda/kernels.cu:720-724 (src/cuda.rs:127-130). */
int d1_qk_norm_rope(d1_half* qkv, int ld, int H, int KVH, const float* qn, const float* kn, const float* rope,
                    const int* tok_seq, const SeqInfo* seqs, int attn_idx, int rows, float eps, cudaStream_t stream);

/* Bidirectional varlen attention, head dim 64, fp32 softmax: for every work item (seq, q0) and head h,
 * O[q] = softmax(scale * Q[q] K^T) V over keys [ext prefix | local], kv head g = h / group; optional fp32 q/k/v
 * biases are added on load. work is int2 (seq index, first query row of a 64-row tile).
 * Replaces d1_flash_attn, cuda/kernels.cu:726-734 (src/cuda.rs:131-135). */
int d1_flash_attn(const d1_half* Q, int ldq, const d1_half* K, const d1_half* V, int ldkv, int ext_ld,
                  const float* bq, const float* bk, const float* bv, d1_half* O, int ldo, const AttnSeq* seqs,
                  const int* work, int n_work, int heads, int group, float scale, cudaStream_t stream);

/* logits[r] = sum_i gelu_erf(x[r][i] + b1[i]) * w2[i] + b2.
 * Replaces d1_scorer_out, cuda/kernels.cu:736-741 (src/cuda.rs:136-138). */
int d1_scorer_out(const d1_half* x, const float* b1, const d1_half* w2, float b2, float* logits, int rows, int D,
                  cudaStream_t stream);

/* ------------------------------------------------------------------------------------------------ vision, audio */

/* 2x2 pixel unshuffle [ph*pw][C] -> [(ph/2)*(pw/2)][4C]. Replaces d1_unshuffle, cuda/kernels.cu:743-746. */
int d1_unshuffle(const d1_half* x, d1_half* out, int ph, int pw, int C, cudaStream_t stream);

/* 3x3 stride-2 conv 1->256 + ReLU over mel [Tin][F]. Replaces d1_sub_conv0, cuda/kernels.cu:748-753. */
int d1_sub_conv0(const float* mel, int tin_valid, int F, const float* w, const float* b, float* out, int Tout,
                 int Fout, cudaStream_t stream);

/* Depthwise 3x3 stride-2 conv on [Tin][Fin][256]. Replaces d1_sub_dwconv, cuda/kernels.cu:755-760. */
int d1_sub_dwconv(const float* x, int tin_valid, int Fin, const float* w, const float* b, float* out, int Tout,
                  int Fout, cudaStream_t stream);

/* qkv [T][3Dm] -> q+bq+u, q+bq+v, k+bk, v+bv (fp16). Replaces d1_relpos_prep, cuda/kernels.cu:762-766. */
int d1_relpos_prep(const d1_half* qkv, const float* bq, const float* bk, const float* bv, const float* pu,
                   const float* pv, d1_half* qu, d1_half* qv, d1_half* k, d1_half* v, int T, int Dm,
                   cudaStream_t stream);

/* p[h][i][:] = softmax_j((ac[h][i][j] + bd[h][i][j+T-1-i]) * scale). Replaces d1_relpos_softmax,
 * cuda/kernels.cu:768-772. */
int d1_relpos_softmax(const float* ac, const float* bd, d1_half* p, int T, int H, float scale, cudaStream_t stream);

/* Conformer conv-module middle: GLU -> depthwise k (zero pad) + bias -> BN affine -> SiLU.
 * Replaces d1_conformer_dw, cuda/kernels.cu:774-778. */
int d1_conformer_dw(const d1_half* a, const float* b1, const float* dw, const float* dwb, const float* bn_s,
                    const float* bn_b, d1_half* out, int T, int C, int ksize, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------------ GEMM */

/* Per-device GEMM context (tile plans + error word). Replaces d1_lt_init, cuda/gemm.cu:119-125
 * (src/cuda.rs:162). Call after cudaSetDevice; one context per device. ws_bytes is accepted for ABI
 * compatibility; the tcgen05 GEMMs need no workspace. Returns NULL on failure. */
void* d1_lt_init(size_t ws_bytes);

/* Row-major Y[M,N] = alpha * X[M,K] . W^T + beta * Y, W = nn.Linear [N,K] (w_kn = 0) or [K,N] (w_kn = 1);
 * Y fp16 (y_f32 = 0) or fp32 (y_f32 = 1); fp32 accumulation always (f16acc is accepted and ignored: fp16
 * accumulation has no throughput advantage on tcgen05). Returns 0 on success, -1 on bad arguments or a launch
 * error; it never returns -2 ("no plan"), so the caller's cuBLAS fallback (src/cuda.rs:448-489) never runs.
 * Replaces d1_lt_gemm, cuda/gemm.cu:128-137 (src/cuda.rs:163-166). */
int d1_lt_gemm(void* ctx, int M, int N, int K, const void* X, int ldx, const void* W, int ldw, int w_kn, void* Y,
               int ldy, int y_f32, int f16acc, float alpha, float beta, cudaStream_t stream);

/* Times the tile configurations of this library for the shape at M's bucket and stores the winner in the
 * context. Returns microseconds (> 0), or a negative value on failure.
 * Replaces d1_lt_tune, cuda/gemm.cu:141-266 (src/cuda.rs:167-170). */
float d1_lt_tune(void* ctx, int M, int N, int K, int ldx, int ldw, int w_kn, int ldy, int y_f32, int f16acc,
                 int effort, cudaStream_t stream);

/* Save / load the tile plans as text (keyed by this library's build id). load returns the number of plans read,
 * -1 if the file cannot be opened, -2 on a version mismatch. Replace d1_lt_save / d1_lt_load,
 * cuda/gemm.cu:268-314 (src/cuda.rs:171-172). */
int d1_lt_save(void* ctx, const char* path);
int d1_lt_load(void* ctx, const char* path);

/* M bucket (16 .. 16384). Replaces d1_lt_bucket, cuda/gemm.cu:316 (src/cuda.rs:173). */
int d1_lt_bucket(int m);

/* Releases tuning scratch. Replaces d1_lt_free_scratch, cuda/gemm.cu:319-327 (src/cuda.rs:174). */
void d1_lt_free_scratch(void* ctx);

/* ------------------------------------------------------------------------------------------------ extensions */

/* extension — fused SwiGLU GEMM: out[M,F] = silu(X.Wg^T) * (X.Wu^T) with W = [Wg; Wu] the reference's
 * concatenated gate_up weight [2F, K] (src/model.rs:184). Equal to d1_lt_gemm(..., N = 2F, fp16 out) followed by
 * d1_swiglu (src/model.rs:394-395, cuda/kernels.cu:159-168), with g and u rounded to fp16 before the gate as the
 * reference does, without writing the [M, 2F] intermediate. */
int d1_gemm_swiglu(void* ctx, int M, int F, int K, const d1_half* X, int ldx, const d1_half* W, int ldw,
                   d1_half* out, int ldo, cudaStream_t stream);

/* extension — fused bias + activation GEMM with fp16 output: Y = act(half(X.W^T) + bias). Equal to
 * d1_lt_gemm(fp16 out, alpha 1, beta 0) followed by d1_bias_act_h (src/model.rs:568-569, src/vision.rs:364-365). */
int d1_gemm_bias_act(void* ctx, int M, int N, int K, const d1_half* X, int ldx, const d1_half* W, int ldw,
                     const float* bias, int act, d1_half* Y, int ldy, cudaStream_t stream);

/* extension — the attention layers' QKV projection with QK-norm + RoPE in the epilogue: Y = [q | k | v] (fp16,
 * H + 2 KVH heads of 64 columns) = X . W^T, then q and k heads as d1_qk_norm_rope gives them (same arithmetic on the
 * fp16-rounded GEMM output). Equal to d1_lt_gemm (fp16 out) followed by d1_qk_norm_rope (src/model.rs:376-381),
 * except that seqs[].save_k / save_v are not written: prefix passes use the two calls. rope, qn and kn 16-byte
 * aligned. */
int d1_gemm_qk_norm_rope(void* ctx, int M, int K, const d1_half* X, int ldx, const d1_half* W, int ldw, d1_half* Y,
                         int ldy, int H, int KVH, const float* qn, const float* kn, const float* rope,
                         const int* tok_seq, const SeqInfo* seqs, float eps, cudaStream_t stream);

/* extension — reads and clears the context's device error word: nonzero when a kernel of this library gave up
 * on a bounded wait (the kernel returns early instead of hanging; its output is then undefined). */
int d1_lt_error(void* ctx);

/* extension — d1_flash_attn without biases on tcgen05 tensor cores (S and O in TMEM); same arguments and result
 * as d1_flash_attn with bq = bk = bv = NULL. The kernel works in 256-row blocks, each starting at a work item whose
 * q0 is a multiple of 256 (other items are ignored): the work list must hold such an item for every 256-row block
 * of every sequence — a list of every 64-row tile (as src/model.rs builds it) does, and a list of only the
 * 256-row block starts is the cheaper form. Pointers 16-byte aligned, leading dimensions multiples of 8.
 * q_rows / kv_rows: rows of Q and O / of K and V (every sequence's q_start + q_len <= q_rows, kv_start + kv_len <=
 * kv_rows), the row counts of the kernel's TMA tensor maps. Its bulk copies move only whole 128-row tiles that lie
 * inside a sequence; a tile a sequence ends in is copied (Q, K, V) or stored (O) row by row, so no row outside the
 * sequences is read or written. */
int d1_flash_attn_tc(const d1_half* Q, int ldq, const d1_half* K, const d1_half* V, int ldkv, int ext_ld, d1_half* O,
                     int ldo, const AttnSeq* seqs, const int* work, int n_work, int heads, int group, float scale,
                     int q_rows, int kv_rows, cudaStream_t stream);

/* extension — reads and clears the attention kernels' device error word (nonzero: a kernel gave up on a bounded
 * wait and returned early; its output is undefined). */
int d1_flash_attn_error(void);

/* extension — fp32 GEMM with the bias / activation folded in: row-major
 * Y[M,N] = act(X[M,K] . W[N,K]^T + beta * Y + bias) (bias fp32 [N] or NULL; act as d1_bias_act_f).
 * Replaces Blas::sgemm (src/cuda.rs:493-505, a cublasGemmEx call made from Rust) and the d1_fill_rows /
 * d1_bias_act_f around it in the audio subsampling (src/audio.rs:517-525). fp32 FFMA, no TF32; results do not
 * depend on the launch (split-K partials are summed in a fixed order). */
int d1_sgemm(int M, int N, int K, const float* X, int ldx, const float* W, int ldw, float* Y, int ldy, float beta,
             const float* bias, int act, cudaStream_t stream);

/* extension — the FastConformer rel-pos self-attention of packed clips in one kernel. Replaces the three
 * Blas::gemm_batched calls (src/cuda.rs:507-527, cuBLAS from Rust) and d1_relpos_softmax of src/audio.rs:559-562.
 * Clip c holds rows offs[c] .. offs[c+1]-1 (offs: device int [n_clips + 1], every clip <= max_len <= 384 rows);
 * for head h (64 columns at h*64 of each operand), query i and key j of the clip:
 *   P[i][j] = fp16(softmax_j((qu_i . k_j + qv_i . pp[pp_center + j - i]) * scale)),  O_i = fp16(sum_j P[i][j] v_j)
 * where pp row pp_center + j - i (of pp_rows rows; rows outside read as zero) is the projected sinusoid of
 * relative position i - j: the reference's per-clip pp has pp_center = T - 1. qu/qv/k/v share row pitch ld. */
int d1_relpos_attn(const d1_half* qu, const d1_half* qv, const d1_half* k, const d1_half* v, int ld,
                   const d1_half* pp, int ldp, int pp_rows, int pp_center, d1_half* o, int ldo, const int* offs,
                   int n_clips, int max_len, int heads, float scale, cudaStream_t stream);

/* extension — resized position embeddings of one vision crop, written as the crop's initial residual rows:
 * out[y*pw + x][c] = sum_j wy_j * (sum_i wx_i * grid[(sy+j)*16 + sx+i][c]) + patch_b[c], with the separable
 * antialiased-bilinear taps of src/vision.rs:173-196 given per output row y (entries 0..ph-1) and column x (entries
 * ph..ph+pw-1): spans int2 (first input index, tap count), w [ph+pw][taps] weights. grid fp32 [256][C]. Replaces
 * VisionModel::pos_for (src/vision.rs:263-302, computed on the host and cached per grid shape in the reference),
 * with the same fp32 operation order. */
int d1_vision_pos(const float* grid, const float* patch_b, const int* spans, const float* w, int taps, int ph, int pw,
                  int C, float* out, cudaStream_t stream);

/* extension — d1_layernorm (pending bias folded into x as there) with only the fp16 output, whose row r goes to
 * row y_rows[r] of y (device int [rows]). With y_rows the 2x2 unshuffle permutation of a crop (row p = y*pw + x of
 * the crop to row 4*((y/2)*(pw/2) + x/2) + 2*(y%2) + x%2 of y viewed as [rows][D]), the vision tower's
 * post-LayerNorm writes the projector's input directly: src/vision.rs:369-377 (post_layernorm, then d1_unshuffle
 * per crop) in one pass. */
int d1_layernorm_rows(float* x, const float* pend_bias, float pend_scale, const float* w, const float* b, d1_half* y,
                      const int* y_rows, int rows, int D, float eps, cudaStream_t stream);

/* extension — the first two subsampling convs of the audio encoder in one kernel: d1_sub_conv0 (F mel bins ->
 * F1 = (F-1)/2+1 bins x 256 channels, l1 rows) followed by d1_sub_dwconv (-> F2 = (F1-1)/2+1 bins, l2 rows), the
 * intermediate kept in shared memory (src/audio.rs:514-515). out fp32 [l2][F2][256], bit-identical to the two calls.
 * F <= 128. */
int d1_sub_conv01(const float* mel, int tin_valid, int F, const float* w0, const float* b0, const float* w1,
                  const float* b1, float* out, int l1, int l2, cudaStream_t stream);

/* extension — d1_conformer_dw over the packed rows of several clips in one call: clip c holds rows offs[c] ..
 * offs[c+1]-1 (offs: device int [n_clips + 1], offs[0] = 0, offs[n_clips] = rows), each zero-padded at its own
 * edges, as src/audio.rs:567 does with one call per clip (the reference encodes one clip at a time). ksize <= 31. */
int d1_conformer_dw_clips(const d1_half* a, const float* b1, const float* dw, const float* dwb, const float* bn_s,
                          const float* bn_b, d1_half* out, const int* offs, int n_clips, int rows, int C, int ksize,
                          cudaStream_t stream);

/* extension — the audio front end on the GPU: normalised log-mel features of n (>= 1) samples at 16 kHz, device x
 * -> device mel fp32 [1 + n/160][128], of which the first n/160 frames are valid (the rest zero). Replaces
 * audio::mel (src/audio.rs:238-299, host code in the reference), with the caller doing its truncation to 30 s and
 * zero-padding to 0.5 s: pre-emphasis 0.97, 512-point frames every 160 samples under a centred 400-point Hann
 * window, f64 radix-2 FFT, power, 128 Slaney mel filters, ln(x + 2^-24), per-channel normalisation over the valid
 * frames (f64 mean, unbiased std + 1e-5). The reference's precision and per-frame operation order; the channel
 * statistics are f64 sums in 8 interleaved parts (the reference sums sequentially). */
int d1_log_mel(const float* x, int n, float* mel, cudaStream_t stream);

/* extension — the number of 16 kHz samples d1_resample writes for n input samples at `from` Hz (to = 16000 in the
 * reference): n * up / down with up / down = to / from reduced (src/audio.rs:108-113); -1 for a rate <= 0. */
int d1_resample_len(int n, int from, int to);

/* extension — sample-rate conversion of n samples (device x) to `to` Hz (device y, d1_resample_len(n, from, to)
 * samples): the reference's polyphase Kaiser-windowed sinc resampler (src/audio.rs:108-148, host code in the
 * reference, run after WAV decoding) with the same fp32 filter table (evaluated in f64 on the host, once per rate
 * pair and device, then kept on the device) and the same fp32 accumulation order: bit-identical results. from == to
 * copies. Returns 0, or -1 for bad arguments or a rate pair whose filter table would exceed 64 Mi taps. */
int d1_resample(const float* x, int n, int from, int to, float* y, cudaStream_t stream);

/* extension — reads and clears d1_relpos_attn's device error word (nonzero: a clip longer than max_len was
 * skipped). */
int d1_relpos_attn_error(void);

/* extension, no reference counterpart — fp16-output GEMM that allocates nothing: Y[M,N] = fp16(X[M,K] . W[N,K]^T)
 * (W nn.Linear, fp32 accumulation), the K range of every 128x128 output tile split across up to `split` CTAs
 * (1 .. 64). Needs no context: its scratch — the fp32 partial sums and the kernels' error word — is a file-scope
 * static device buffer of 2^20 floats (4 MiB), cleared at the start of every call; M*N above 2^20 is rejected
 * (-1), as are null pointers, N not a multiple of 4 and X/W rows that are not 16-byte aligned. Calls that overlap
 * on one device (other streams or threads) race on that buffer and must not be issued. Returns 0 when both
 * launches were issued, -1 otherwise (bad argument, set-up failure or launch error); a kernel that gave up on a
 * bounded wait shows only in d1_gemm_noalloc_error(). */
int d1_gemm_noalloc(int M, int N, int K, const d1_half* X, int ldx, const d1_half* W, int ldw, d1_half* Y, int ldy,
                    int split, cudaStream_t stream);

/* extension, no reference counterpart — reads and clears the error word of d1_gemm_noalloc on the current device
 * (0: the last call's GEMM completed; nonzero: one of its bounded waits ran out and Y is not the product; -1: the
 * word could not be read). Waits for the device's outstanding work. */
int d1_gemm_noalloc_error(void);

/* extension — releases a context made by d1_lt_init (the reference never frees it). */
void d1_lt_destroy(void* ctx);

/* extension — build identifier of this library (the key of saved tile plans). */
const char* d1_build_id(void);

#ifdef __cplusplus
}
#endif

#endif /* D1KERNELS_H */
