/*
 * d1h.h — host runner of the d1rs text forward pass over a d1kernels library.
 *
 * A C++ restatement of the reference's Rust host for this path, kept call-for-call:
 *   - TextModel / TrunkLayer / HeadLayer weights            src/model.rs:19-68
 *   - PrefixCache (media prefix K/V + conv state)            src/model.rs:70-104
 *   - Workspace, MetaWriter, work_items                      src/model.rs:250-339
 *   - Runner::trunk, launch_prefix, launch_text, finish      src/model.rs:355-607
 *   - Blas::gemm over d1_lt_gemm                             src/cuda.rs:433-490
 * There is no Rust toolchain on this machine, so the Rust host cannot be linked here; this runner is what the
 * tests and the benchmark drive, and the Rust crate links libd1kernels unchanged (the d1_* ABI in d1kernels.h).
 *
 * The runner reaches every kernel through a function table. By default the table holds this library's own
 * sm_100a kernels; d1h_model_create can instead load any library that exports the d1kernels.h ABI (used by the
 * tests to run the reference's own kernels through the same host code).
 *
 * Weights are device pointers owned by the caller (they must outlive the model). All launches are asynchronous
 * on the stream given to each call. Functions return 0 on success, a nonzero kernel/CUDA status otherwise.
 */
#ifndef D1H_H
#define D1H_H

#include "d1kernels.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One trunk layer (src/model.rs:19-31). is_attn selects the mixer; fields of the other mixer are ignored. */
typedef struct D1TrunkLayer {
    int is_attn;
    const d1_half* in_proj;   /* conv: shortconv.in_proj [3D, D] */
    const d1_half* out_proj;  /* conv: shortconv.out_proj [D, D] */
    const float* convw;       /* conv: shortconv.conv [D][3] */
    const d1_half* qkv;       /* attn: [q; k; v] rows [D + 2*512, D] (src/model.rs:160) */
    const d1_half* out;       /* attn: attn_output [D, D] */
    const float* qn;          /* attn: attn_q_norm [64] */
    const float* kn;          /* attn: attn_k_norm [64] */
    const float* op_norm;     /* attn_norm [D] */
    const float* ffn_norm;    /* ffn_norm [D] */
    const d1_half* gate_up;   /* [gate; up] rows [2F, D] (src/model.rs:184) */
    const d1_half* down;      /* ffn_down [D, F] */
    int ffn;                  /* F */
} D1TrunkLayer;

/* One decision-head layer (src/model.rs:33-47). */
typedef struct D1HeadLayer {
    const float* n1_w;
    const float* n1_b;
    const d1_half* qkv;       /* [3D, D] */
    const float* qkv_b;       /* [3D] */
    const d1_half* out;       /* [D, D] */
    const float* out_b;
    const float* n2_w;
    const float* n2_b;
    const d1_half* up;        /* [F, D] */
    const float* up_b;
    const d1_half* down;      /* [D, F] */
    const float* down_b;
    int ffn;
} D1HeadLayer;

/* The text model (src/model.rs:49-68). D = 1024, 16 heads, 8 kv heads, head dim 64 (src/model.rs:12-17). */
typedef struct D1TextWeights {
    int n_layers;
    const D1TrunkLayer* layers;
    int n_head;
    const D1HeadLayer* head;
    int vocab;
    const d1_half* embed;     /* token_embd [vocab, D] */
    const float* final_norm;  /* token_embd_norm [D] */
    const float* type_emb;    /* token_types [n_types, D] */
    const float* cls_norm_w;
    const float* cls_norm_b;
    const d1_half* cls_w;     /* [D, D] */
    const float* cls_b;
    const d1_half* out_w;     /* [D] */
    float out_b;
    float eps;                /* RMSNorm eps (1e-5) */
    float rope_theta;         /* 1e6 */
} D1TextWeights;

typedef struct D1Model D1Model;
typedef struct D1Workspace D1Workspace;

/* A media prefix that went through the trunk (src/model.rs:70-104): per attention layer K/V and the last
 * position's conv state, allocated in stream order. */
typedef struct D1PrefixCache {
    int len;
    d1_half* k;   /* [n_attn][len][512] */
    d1_half* v;   /* [n_attn][len][512] */
    d1_half* bx;  /* [n_conv][D] */
} D1PrefixCache;

/* One question sequence of a text batch (src/model.rs:236-242). markers are row offsets within the sequence. */
typedef struct D1TextSeq {
    const int* ids;
    int n_ids;
    const int* markers;
    int n_markers;
    int qtype;
    const D1PrefixCache* prefix; /* NULL for text without media */
} D1TextSeq;

/* One prefix to run through the trunk: fp32 embeddings [len, D] on the device -> cache (src/model.rs:244-248). */
typedef struct D1PrefixSeq {
    const float* emb;
    const D1PrefixCache* cache;
} D1PrefixSeq;

/* Creates a model over caller-owned device weights on the current device. kernel_lib: NULL for this library's
 * kernels, else the path of a library exporting the d1kernels.h ABI. fused: 1 uses the fused GEMM epilogues
 * (d1_gemm_swiglu, d1_gemm_bias_act) when the library exports them. Returns NULL on failure. */
D1Model* d1h_model_create(const D1TextWeights* w, const char* kernel_lib, int fused);
void d1h_model_destroy(D1Model* m);
/* Last error text of the calling thread (static storage). */
const char* d1h_last_error(void);

/* Scratch for batches of up to cap_tokens tokens (src/model.rs:277-299); 2 in-flight slots. */
D1Workspace* d1h_workspace_create(D1Model* m, int cap_tokens);
void d1h_workspace_destroy(D1Workspace* ws);

/* Enqueue a text batch (src/model.rs:470-599). The slot's logits (one per option marker, in sequence then
 * marker order) are ready after d1h_finish. Returns 0 or an error status. */
int d1h_launch_text(D1Model* m, D1Workspace* ws, int slot, const D1TextSeq* seqs, int n_seqs, cudaStream_t stream);
/* Blocks until the slot's batch is done; copies its logits to out (up to cap floats). Returns the number of
 * logits, or a negative status. */
int d1h_finish(D1Model* m, D1Workspace* ws, int slot, float* out, int cap);

/* Prefix caches (src/model.rs:85-103) and prefix passes (src/model.rs:402-459). */
int d1h_prefix_alloc(D1Model* m, int len, D1PrefixCache* out, cudaStream_t stream);
void d1h_prefix_free(D1PrefixCache* c, cudaStream_t stream);
int d1h_launch_prefix(D1Model* m, D1Workspace* ws, int slot, const D1PrefixSeq* items, int n_items, cudaStream_t stream);

/* Tunes the GEMM plans of every trunk/head shape for every M bucket up to max_tokens (src/engine.rs:528-616).
 * Returns the number of shapes tuned or a negative status. */
int d1h_tune(D1Model* m, D1Workspace* ws, int max_tokens, cudaStream_t stream);

/* ------------------------------------------------------------------------------------------------ vision
 * SigLIP2-NaFlex tower + 2x2 pixel-unshuffle projector (src/vision.rs:128-164, 198-385): hidden 768, 12 heads,
 * GELU-tanh MLP 3072, LayerNorm (eps from GGUF, 1e-6), projector 3072 -> 2048 (GELU-erf) -> 1024. */
typedef struct D1VisionLayer {
    const float* ln1_w;
    const float* ln1_b;
    const d1_half* qkv;      /* [q; k; v] rows [2304, 768] (src/vision.rs:217-219) */
    const float* qkv_b;      /* [2304] */
    const d1_half* out;      /* [768, 768] */
    const float* out_b;
    const float* ln2_w;
    const float* ln2_b;
    const d1_half* fc1;      /* [3072, 768] */
    const float* fc1_b;
    const d1_half* fc2;      /* [768, 3072] */
    const float* fc2_b;
} D1VisionLayer;

typedef struct D1VisionWeights {
    int n_layers;
    const D1VisionLayer* layers;
    const d1_half* patch_w;  /* [768, 768] with inputs in (y, x, c) patch order (src/vision.rs:202-213) */
    const float* patch_b;    /* host [768] (folded into the position embeddings, src/vision.rs:293-295) */
    const float* pos;        /* host [16*16][768] position embedding grid */
    const float* post_w;
    const float* post_b;
    const d1_half* proj1;    /* [2048, 3072] */
    const float* proj1_b;
    const d1_half* proj2;    /* [1024, 2048] */
    const float* proj2_b;
    float eps;
} D1VisionWeights;

typedef struct D1Vision D1Vision;

/* Creates the encoder over caller-owned device weights (host pointers for patch_b and pos, which are copied);
 * max_patches bounds one call. kernel_lib / fused as d1h_model_create. NULL on failure. */
D1Vision* d1h_vision_create(const D1VisionWeights* w, const char* kernel_lib, int fused, int max_patches);
void d1h_vision_destroy(D1Vision* v);

/* Runs crops through the tower and projector (src/vision.rs:305-385). ph, pw: each crop's patch grid (even);
 * pixels: host fp16 [sum ph*pw][768] patch rows in (y, x, c) order; out: device fp32 [sum ph*pw/4][1024] in crop
 * order. Asynchronous on `stream` (the host staging buffers are reused by the next call after it waits for
 * this one). Returns 0 or an error status. */
int d1h_vision_encode(D1Vision* v, int n_crops, const int* ph, const int* pw, const d1_half* pixels, float* out,
                      cudaStream_t stream);

/* ------------------------------------------------------------------------------------------------ audio
 * FastConformer encoder + adapter (src/audio.rs:302-594): 8x conv subsampling of 128-bin log-mel frames
 * (fp32, 256 channels), 17 layers of hidden 512 with 8-head rel-pos attention, depthwise conv kernel 9 and
 * half-step SiLU FFNs of width 2048, adapter LN -> 1024 GELU -> 1024 plus LN -> 512 GELU -> 1024 residual.
 * Matrices fp16 [out, in] (fused QKV rows [q; k; v]); vectors and subsampling weights fp32. */
typedef struct D1AudioLayer {
    const float* ff1_n_w;
    const float* ff1_n_b;
    const d1_half* ff1_up;     /* [2048, 512] */
    const float* ff1_up_b;
    const d1_half* ff1_down;   /* [512, 2048] */
    const float* ff1_down_b;
    const float* att_n_w;
    const float* att_n_b;
    const d1_half* qkv;        /* [1536, 512] */
    const float* bq;
    const float* bk;
    const float* bv;
    const float* pu;           /* pos_bias_u [8*64] */
    const float* pv;           /* pos_bias_v [8*64] */
    const d1_half* pos;        /* linear_pos [512, 512] */
    const d1_half* out;        /* [512, 512] */
    const float* out_b;
    const float* conv_n_w;
    const float* conv_n_b;
    const d1_half* pw1;        /* [1024, 512] */
    const float* pw1_b;
    const float* dw;           /* [512][9] */
    const float* dw_b;
    const float* bn_s;         /* batch-norm folded scale / shift */
    const float* bn_b;
    const d1_half* pw2;        /* [512, 512] */
    const float* pw2_b;
    const float* ff2_n_w;
    const float* ff2_n_b;
    const d1_half* ff2_up;
    const float* ff2_up_b;
    const d1_half* ff2_down;
    const float* ff2_down_b;
    const float* out_n_w;
    const float* out_n_b;
} D1AudioLayer;

typedef struct D1AudioWeights {
    int n_layers;
    const D1AudioLayer* layers;
    const float* c0_w;         /* conv 1 -> 256, 3x3 stride 2: [256][9] */
    const float* c0_b;
    const float* c2_w;         /* depthwise 3x3 stride 2: [256][9] */
    const float* c2_b;
    const float* c3_w;         /* pointwise [256, 256] */
    const float* c3_b;
    const float* c5_w;
    const float* c5_b;
    const float* c6_w;
    const float* c6_b;
    const float* pre_out;      /* [512, 16*256] with columns in (f, c) order (src/audio.rs:434-442) */
    const float* pre_out_b;
    const float* ad_n_w;
    const float* ad_n_b;
    const d1_half* ad1;        /* [1024, 512] */
    const float* ad1_b;
    const d1_half* ad2;        /* [1024, 1024] */
    const float* ad2_b;
    const float* res_n_w;
    const float* res_n_b;
    const d1_half* res_down;   /* [512, 1024] */
    const float* res_down_b;
    const d1_half* res_up;     /* [1024, 512] */
    const float* res_up_b;
    float eps;
} D1AudioWeights;

typedef struct D1Audio D1Audio;

/* Creates the encoder over caller-owned device weights, with this library's kernels; max_rows bounds the encoder
 * output rows (sum over clips of ceil(valid / 8)) of one call. fused: fold biases / activations into the GEMM
 * epilogues (0: the reference's separate d1_fill_rows / d1_bias_act_* calls). NULL on failure. */
D1Audio* d1h_audio_create(const D1AudioWeights* w, int fused, int max_rows);
void d1h_audio_destroy(D1Audio* a);

/* Encodes clips (src/audio.rs:505-594) packed into one pass: clip c contributes valid[c] (1 .. 3000) normalised
 * log-mel frames, mel is host fp32 [sum valid][128] in clip order; out: device fp32 [sum T_c][1024] in clip
 * order, T_c = ceil(valid[c] / 8) <= 375. Asynchronous on `stream` (the host staging is reused by the next call
 * after it waits for this one). Returns the number of output rows or a negative status. */
int d1h_audio_encode(D1Audio* a, int n_clips, const int* valid, const float* mel, float* out, cudaStream_t stream);

/* As d1h_audio_encode from 16 kHz waveforms: clip c has n_samples[c] host fp32 samples (pcm holds the clips back to
 * back); each clip is cut to 30 s and zero-padded to 0.5 s (src/audio.rs:238-247) and its log-mel features are
 * computed on the device (d1_log_mel). valid_out (optional, [n_clips]) receives each clip's mel frame count. */
int d1h_audio_encode_pcm(D1Audio* a, int n_clips, const int* n_samples, const float* pcm, float* out, int* valid_out,
                         cudaStream_t stream);
/* d1h_audio_encode_pcm with a sample rate per clip (rates NULL, or an entry 0 or 16000: 16 kHz). A clip at another
 * rate is what the reference's WAV decoder hands on (src/audio.rs:24-80: mono fp32, at most 30 s + 1 s of input):
 * it is converted to 16 kHz on the device by d1_resample (src/audio.rs:108-148) before the front end. n_samples
 * counts samples at the clip's own rate. */
int d1h_audio_encode_pcm_rates(D1Audio* a, int n_clips, const int* n_samples, const int* rates, const float* pcm,
                               float* out, int* valid_out, cudaStream_t stream);

/* Vision batch capacity in patches (max_patches of d1h_vision_create). */
int d1h_vision_capacity(const D1Vision* v);
/* Number of attention (is_attn = 1) or conv (is_attn = 0) trunk layers of the model. */
int d1h_model_layers(const D1Model* m, int is_attn);
/* The model's GEMM context (the ctx of d1_lt_*): d1_lt_save / d1_lt_load keep its tuned plans across runs, as the
 * reference's engine keeps its cuBLASLt plans (src/engine.rs:528-616). */
void* d1h_gemm_ctx(D1Model* m);
/* Effort (the d1_lt_tune argument: 0 heuristics, 1 pruned search, 2 exhaustive) of the plans the model tunes on
 * the first use of a GEMM shape and M bucket that has none (default 0). The reference's engine tunes its startup
 * plans at effort 1 (src/engine.rs:593); with effort 1 here, the buckets a workload touches get the same plans
 * without tuning the ones it never uses. Returns 0, or -1 for a null model or an effort outside 0..2. */
int d1h_set_tune_effort(D1Model* m, int effort);

/* ------------------------------------------------------------------------------------------------ engine
 * Continuous batching over one device's runners (src/engine.rs:149-525): requests (jobs) of question rows and
 * optional media; every d1e_step packs question rows FIFO across requests into one varlen batch under the token
 * budget and launches it, encodes at most one media group and runs its prefixes through the trunk once, keeps up
 * to two batches in flight, and moves finished requests to a completion queue (d1e_take). One engine per
 * device, driven from one host thread; engines of different devices are independent. */
enum { D1_MEDIA_NONE = 0, D1_MEDIA_IMAGES = 1, D1_MEDIA_AUDIO = 2 };

typedef struct D1EngineConfig {
    int max_batch_tokens;        /* token budget per text batch (src/main.rs:153, default 8192) */
    int cap_tokens;              /* workspace capacity in tokens (>= max_batch_tokens, >= the longest question) */
    long long media_cache_bytes; /* budget for live prefix caches (src/main.rs:155, default 1536 MiB) */
} D1EngineConfig;

typedef struct D1Row {           /* one question (src/engine.rs:21-25) */
    const int* ids;
    int n_ids;
    const int* markers;          /* option-marker rows within the question */
    int n_markers;
    int qtype;
} D1Row;

typedef struct D1Media {         /* src/engine.rs:27-31 */
    int kind;                    /* D1_MEDIA_* */
    int n_crops;                 /* images: crops of all the request's images, in order */
    const int* ph;
    const int* pw;
    const d1_half* patches;      /* host fp16 [sum ph*pw][768] */
    const float* mel;            /* audio: host fp32 [valid][128] normalised log-mel frames, or NULL with pcm */
    int valid;                   /* 1 .. 3000 */
    const float* pcm;            /* audio as a waveform (features computed on the device), or NULL */
    int n_samples;               /* at sample_rate */
    int sample_rate;             /* of pcm in Hz; 0 means 16000 (other rates are resampled on the device) */
} D1Media;

typedef struct D1Job {           /* src/engine.rs:49-53 */
    const D1Row* rows;
    int n_rows;
    D1Media media;
} D1Job;

typedef struct D1EngineStats {
    long long tokens;            /* question tokens launched */
    long long media_tokens;      /* prefix positions run through the trunk */
    long long batches;
    long long media_jobs;          /* requests whose media were encoded */
    long long rows;
} D1EngineStats;

typedef struct D1Engine D1Engine;

/* Creates an engine on the current device over a text model and optional encoders (NULL: requests with that
 * media fail), with its own workspace; all work goes to `stream`. NULL on failure (d1e_last_error). */
D1Engine* d1e_create(D1Model* m, D1Vision* vision, D1Audio* audio, const D1EngineConfig* cfg, cudaStream_t stream);
void d1e_destroy(D1Engine* e);
/* Copies a request into the engine; returns its id (>= 0) or a negative status. */
long long d1e_submit(D1Engine* e, const D1Job* job);
/* One engine iteration (src/engine.rs:182-221). Returns the number of requests that finished in it, or a
 * negative status. */
int d1e_step(D1Engine* e);
/* Requests submitted and not finished. */
int d1e_pending(const D1Engine* e);
/* Question tokens (plus unencoded media positions) still queued: the dispatcher's load measure. */
long long d1e_queued_tokens(const D1Engine* e);
/* Logit count of the next finished request, or -1 if none. */
int d1e_next_logits(const D1Engine* e);
/* Pops the next finished request: its id, its logits (rows in order, one per option marker) and its error text
 * (empty on success). Returns the number of logits, -1 if none finished, -2 if cap is too small. */
int d1e_take(D1Engine* e, long long* id, float* logits, int cap, char* err, int err_cap);
void d1e_stats(const D1Engine* e, D1EngineStats* out);
const char* d1e_last_error(void);

/* Number of kernel launches the runner made since the model was created (a counter for benchmarks). */
long long d1h_launch_count(const D1Model* m);
/* Bytes the last launch on `slot` copied host->device (its batch metadata, token ids included) and
 * device->host (its logits). */
long long d1h_h2d_bytes(const D1Workspace* ws, int slot);
long long d1h_d2h_bytes(const D1Workspace* ws, int slot);

#ifdef __cplusplus
}
#endif

#endif /* D1H_H */
