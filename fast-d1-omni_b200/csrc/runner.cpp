// Host runner of the d1rs text forward pass: a C++ restatement of src/model.rs (TextModel, PrefixCache, Workspace,
// MetaWriter, work_items, Runner::trunk / launch_prefix / launch_text / finish) and of Blas::gemm
// (src/cuda.rs:433-490), driving any library that exports the d1kernels.h ABI through a function table.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <map>
#include <string>
#include <vector>

#include "d1h.h"

namespace {

constexpr int D = 1024;         // src/model.rs:12
constexpr int HEADS = 16;       // :13
constexpr int KV_HEADS = 8;     // :14
constexpr int HD = 64;          // :15
constexpr int KV_DIM = KV_HEADS * HD;
constexpr int MAX_POS = 16384 + 64;  // :17
constexpr size_t META_BYTES = 8 << 20;  // :250
constexpr int SLOTS = 2;        // :251

thread_local std::string g_err;

int fail(const std::string& msg, int code = -1) {
    g_err = msg;
    return code;
}

// ------------------------------------------------------------------------------------------------ kernel table

struct Kt {
    void* dl = nullptr;
    int (*rmsnorm)(const float*, const float*, d1_half*, int, int, float, cudaStream_t) = nullptr;
    int (*layernorm)(float*, const float*, float, const float*, const float*, d1_half*, float*, int, int, float,
                     cudaStream_t) = nullptr;
    int (*head_init)(const float*, const float*, const float*, const int*, const SeqInfo*, float*, int, float,
                     cudaStream_t) = nullptr;
    int (*embed)(const d1_half*, const int*, float*, int, int, cudaStream_t) = nullptr;
    int (*swiglu)(const d1_half*, d1_half*, int, int, cudaStream_t) = nullptr;
    int (*bias_act_h)(d1_half*, const float*, int, int, int, cudaStream_t) = nullptr;
    int (*gather_rows)(const void*, void*, const int*, int, int, cudaStream_t) = nullptr;
    int (*shortconv)(const d1_half*, const float*, const int*, const SeqInfo*, d1_half*, int, int, int,
                     cudaStream_t) = nullptr;
    int (*qk_norm_rope)(d1_half*, int, int, int, const float*, const float*, const float*, const int*,
                        const SeqInfo*, int, int, float, cudaStream_t) = nullptr;
    int (*flash_attn)(const d1_half*, int, const d1_half*, const d1_half*, int, int, const float*, const float*,
                      const float*, d1_half*, int, const AttnSeq*, const int*, int, int, int, float,
                      cudaStream_t) = nullptr;
    int (*scorer_out)(const d1_half*, const float*, const d1_half*, float, float*, int, int, cudaStream_t) = nullptr;
    int (*unshuffle)(const d1_half*, d1_half*, int, int, int, cudaStream_t) = nullptr;
    int (*fill_rows)(float*, const float*, const float*, int, int, cudaStream_t) = nullptr;
    void* (*lt_init)(size_t) = nullptr;
    int (*lt_gemm)(void*, int, int, int, const void*, int, const void*, int, int, void*, int, int, int, float, float,
                   cudaStream_t) = nullptr;
    float (*lt_tune)(void*, int, int, int, int, int, int, int, int, int, int, cudaStream_t) = nullptr;
    int (*lt_bucket)(int) = nullptr;
    void (*lt_free_scratch)(void*) = nullptr;
    // optional (this library's fused epilogues)
    int (*gemm_swiglu)(void*, int, int, int, const d1_half*, int, const d1_half*, int, d1_half*, int,
                       cudaStream_t) = nullptr;
    int (*gemm_bias_act)(void*, int, int, int, const d1_half*, int, const d1_half*, int, const float*, int, d1_half*,
                         int, cudaStream_t) = nullptr;
    int (*flash_attn_tc)(const d1_half*, int, const d1_half*, const d1_half*, int, int, d1_half*, int, const AttnSeq*,
                         const int*, int, int, int, float, int, int, cudaStream_t) = nullptr;
    int (*gemm_qk_rope)(void*, int, int, const d1_half*, int, const d1_half*, int, d1_half*, int, int, int,
                        const float*, const float*, const float*, const int*, const SeqInfo*, float,
                        cudaStream_t) = nullptr;
    void (*lt_destroy)(void*) = nullptr;

    // Bidirectional attention over a complete work list (every 64-row tile of every sequence, as the runners
    // build it): the tcgen05 kernel when the library has it, fused forms are on and there are no biases to add
    // on load; d1_flash_attn otherwise. q_rows / kv_rows bound the rows of Q and of K/V. The work list is the
    // one work_items(spans, attn_step(fused)) builds.
    int attn_step(bool fused) const { return fused && flash_attn_tc ? 256 : 64; }
    int attention(bool fused, const d1_half* Q, int ldq, const d1_half* K, const d1_half* V, int ldkv, int ext_ld,
                  const float* bq, const float* bk, const float* bv, d1_half* O, int ldo, const AttnSeq* seqs,
                  const int* work, int n_work, int heads, int group, float scale, int q_rows, int kv_rows,
                  cudaStream_t st) const {
        if (attn_step(fused) == 256) {
            if (bq || bk || bv) return -1;  // fused runs fold the q/k/v biases into the QKV GEMM
            return flash_attn_tc(Q, ldq, K, V, ldkv, ext_ld, O, ldo, seqs, work, n_work, heads, group, scale, q_rows,
                                 kv_rows, st);
        }
        return flash_attn(Q, ldq, K, V, ldkv, ext_ld, bq, bk, bv, O, ldo, seqs, work, n_work, heads, group, scale, st);
    }

    bool load_builtin() {
        rmsnorm = d1_rmsnorm;
        layernorm = d1_layernorm;
        head_init = d1_head_init;
        embed = d1_embed;
        swiglu = d1_swiglu;
        bias_act_h = d1_bias_act_h;
        gather_rows = d1_gather_rows;
        shortconv = d1_shortconv;
        qk_norm_rope = d1_qk_norm_rope;
        flash_attn = d1_flash_attn;
        scorer_out = d1_scorer_out;
        unshuffle = d1_unshuffle;
        fill_rows = d1_fill_rows;
        lt_init = d1_lt_init;
        lt_gemm = d1_lt_gemm;
        lt_tune = d1_lt_tune;
        lt_bucket = d1_lt_bucket;
        lt_free_scratch = d1_lt_free_scratch;
        gemm_swiglu = d1_gemm_swiglu;
        gemm_bias_act = d1_gemm_bias_act;
        flash_attn_tc = d1_flash_attn_tc;
        gemm_qk_rope = d1_gemm_qk_norm_rope;
        lt_destroy = d1_lt_destroy;
        return true;
    }

    template <class F>
    bool sym(F& f, const char* name, bool required = true) {
        f = reinterpret_cast<F>(dlsym(dl, name));
        if (!f && required) {
            g_err = std::string("kernel library lacks ") + name;
            return false;
        }
        return true;
    }

    bool load_lib(const char* path) {
        dl = dlopen(path, RTLD_NOW | RTLD_LOCAL);
        if (!dl) {
            g_err = std::string("dlopen failed: ") + dlerror();
            return false;
        }
        return sym(rmsnorm, "d1_rmsnorm") && sym(layernorm, "d1_layernorm") && sym(head_init, "d1_head_init") &&
               sym(embed, "d1_embed") && sym(swiglu, "d1_swiglu") && sym(bias_act_h, "d1_bias_act_h") &&
               sym(gather_rows, "d1_gather_rows") && sym(shortconv, "d1_shortconv") &&
               sym(qk_norm_rope, "d1_qk_norm_rope") && sym(flash_attn, "d1_flash_attn") &&
               sym(scorer_out, "d1_scorer_out") && sym(unshuffle, "d1_unshuffle") && sym(fill_rows, "d1_fill_rows") &&
               sym(lt_init, "d1_lt_init") && sym(lt_gemm, "d1_lt_gemm") &&
               sym(lt_tune, "d1_lt_tune") && sym(lt_bucket, "d1_lt_bucket") &&
               sym(lt_free_scratch, "d1_lt_free_scratch") && sym(gemm_swiglu, "d1_gemm_swiglu", false) &&
               sym(gemm_bias_act, "d1_gemm_bias_act", false) && sym(flash_attn_tc, "d1_flash_attn_tc", false) &&
               sym(gemm_qk_rope, "d1_gemm_qk_norm_rope", false) &&
               sym(lt_destroy, "d1_lt_destroy", false);
    }
};

// IEEE binary32 -> binary16 bits, round to nearest even (overflow to infinity, gradual underflow).
uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    x &= 0x7fffffffu;
    if (x >= 0x7f800000u) return sign | (x > 0x7f800000u ? 0x7e00 : 0x7c00);
    if (x >= 0x477ff000u) return sign | 0x7c00;  // >= 65520 rounds past the largest half
    if (x < 0x38800000u) {                      // half subnormal range (|f| < 2^-14)
        if (x < 0x33000000u) return sign;        // below half of the smallest subnormal
        const int shift = 126 - (int)(x >> 23);
        const uint32_t m = (x & 0x7fffffu) | 0x800000u;
        uint32_t r = m >> shift;
        const uint32_t rem = m & ((1u << shift) - 1), half = 1u << (shift - 1);
        if (rem > half || (rem == half && (r & 1))) r++;
        return sign | (uint16_t)r;
    }
    uint32_t r = (x >> 13) - (112u << 10);      // rebias the exponent (127 -> 15)
    const uint32_t rem = x & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (r & 1))) r++;
    return sign | (uint16_t)r;
}

// RoPE table [pos][32] of (cos, sin), computed as src/model.rs:121-136 does: fp32 inverse frequency, fp32 angle
// p * f, then cos/sin in double precision rounded to float.
std::vector<float> rope_table(float theta) {
    float inv[32];
    for (int i = 0; i < 32; i++) {
        const float e = (float)(2 * i) / (float)HD;
        inv[i] = 1.0f / powf(theta, e);
    }
    std::vector<float> t;
    t.reserve((size_t)MAX_POS * 64);
    for (int p = 0; p < MAX_POS; p++)
        for (int i = 0; i < 32; i++) {
            const double a = (double)((float)p * inv[i]);
            t.push_back((float)cos(a));
            t.push_back((float)sin(a));
        }
    return t;
}

}  // namespace

// ------------------------------------------------------------------------------------------------ model

struct D1Model {
    Kt k;
    void* lt = nullptr;       // GEMM context (d1_lt_init)
    D1TextWeights w{};
    std::vector<D1TrunkLayer> layers;
    std::vector<D1HeadLayer> head;
    std::vector<int> mixer_idx;  // per trunk layer: index among its kind (conv_idx / attn_idx)
    int n_attn = 0, n_conv = 0, max_ffn = 0;
    float* rope = nullptr;
    bool fused = false;
    std::atomic<long long> launches{0};  // engines of one device may share the model
    int dev = 0;
    int tune_effort = 0;  // d1_lt_tune effort of the plans tuned on first use

    // Blas::gemm (src/cuda.rs:433-490): Y = alpha X W^T + beta Y. A library without a plan for the shape
    // (d1_lt_gemm == -2) gets a heuristic plan tuned on the spot instead of a cuBLAS fallback.
    int gemm(int m, int n, int kk, const d1_half* x, int ldx, const d1_half* wt, int ldw, void* y, int ldy, int y_f32,
             float alpha, float beta, cudaStream_t st) {
        if (m == 0 || n == 0) return 0;
        launches++;
        int e = k.lt_gemm(lt, m, n, kk, x, ldx, wt, ldw, 0, y, ldy, y_f32, 0, alpha, beta, st);
        if (e == -2) {
            if (k.lt_tune(lt, m, n, kk, ldx, ldw, 0, ldy, y_f32, 0, tune_effort, st) < 0.f)
                return fail("GEMM tuning failed for m=" + std::to_string(m) + " n=" + std::to_string(n));
            e = k.lt_gemm(lt, m, n, kk, x, ldx, wt, ldw, 0, y, ldy, y_f32, 0, alpha, beta, st);
        }
        if (e) return fail("d1_lt_gemm failed (" + std::to_string(e) + ") m=" + std::to_string(m) + " n=" +
                           std::to_string(n) + " k=" + std::to_string(kk), e);
        return 0;
    }
};

// Blas::gemm over any kernel table and context (shared by the text model and the encoders).
int kt_gemm(Kt& k, void* lt, long long& launches, int m, int n, int kk, const d1_half* x, int ldx, const d1_half* wt,
            int ldw, void* y, int ldy, int y_f32, float alpha, float beta, cudaStream_t st) {
    if (m == 0 || n == 0) return 0;
    launches++;
    int e = k.lt_gemm(lt, m, n, kk, x, ldx, wt, ldw, 0, y, ldy, y_f32, 0, alpha, beta, st);
    if (e == -2) {
        if (k.lt_tune(lt, m, n, kk, ldx, ldw, 0, ldy, y_f32, 0, 0, st) < 0.f)
            return fail("GEMM tuning failed for m=" + std::to_string(m) + " n=" + std::to_string(n));
        e = k.lt_gemm(lt, m, n, kk, x, ldx, wt, ldw, 0, y, ldy, y_f32, 0, alpha, beta, st);
    }
    if (e) return fail("d1_lt_gemm failed (" + std::to_string(e) + ") m=" + std::to_string(m) + " n=" +
                       std::to_string(n) + " k=" + std::to_string(kk), e);
    return 0;
}

struct D1Workspace {
    int cap_tokens = 0, cap_markers = 0;
    float* h = nullptr;
    d1_half* xn = nullptr;
    d1_half* big = nullptr;
    d1_half* act = nullptr;
    d1_half* mq = nullptr;
    d1_half* mo = nullptr;
    float* mh = nullptr;
    d1_half* mx = nullptr;
    d1_half* mbig = nullptr;
    float* logits = nullptr;
    uint8_t* meta = nullptr;
    uint8_t* host_meta[SLOTS] = {};
    float* host_logits[SLOTS] = {};
    cudaEvent_t events[SLOTS] = {};
    bool busy[SLOTS] = {};
    int n_logits[SLOTS] = {};
    long long h2d[SLOTS] = {};
};

namespace {

// Bump writer over a pinned host buffer returning the device address of each section (src/model.rs:309-326).
struct MetaWriter {
    uint8_t* host;
    uint8_t* dev;
    size_t off = 0;
    bool overflow = false;
    template <class T>
    const T* put(const T* items, size_t n) {
        off = (off + 15) / 16 * 16;
        const size_t bytes = n * sizeof(T);
        if (off + bytes > META_BYTES) {
            overflow = true;
            return nullptr;
        }
        if (bytes) memcpy(host + off, items, bytes);
        const T* d = reinterpret_cast<const T*>(dev + off);
        off += bytes;
        return d;
    }
    template <class T>
    const T* put(const std::vector<T>& v) {
        return put(v.data(), v.size());
    }
};

// (seq index, query-tile start) for every 64-row query tile (src/model.rs:328-339), longest sequences first so
// the long tiles start in the first wave. step 256: one item per 256-row block, the list the tcgen05 attention
// takes without scanning past the items it skips.
std::vector<int> work_items(const std::vector<std::pair<int, int>>& spans, int step = 64) {
    std::vector<int> order(spans.size());
    for (size_t i = 0; i < order.size(); i++) order[i] = (int)i;
    std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return spans[a].second > spans[b].second; });
    std::vector<int> w;
    for (int i : order)
        for (int q = 0; q < spans[i].second; q += step) {
            w.push_back(i);
            w.push_back(q);
        }
    return w;
}

#define CK(expr)                                                                               \
    do {                                                                                       \
        int _e = (expr);                                                                       \
        if (_e) return fail(std::string("kernel failed (") + std::to_string(_e) + "): " #expr, _e); \
    } while (0)

template <class T>
int dmalloc(T** p, size_t bytes) {
    if (cudaMalloc((void**)p, bytes < 16 ? 16 : bytes) != cudaSuccess) return fail("cudaMalloc failed");
    return 0;
}

int wait_slot(D1Workspace* ws, int slot) {
    if (ws->busy[slot]) {
        if (cudaEventSynchronize(ws->events[slot]) != cudaSuccess) return fail("event sync failed");
        ws->busy[slot] = false;
    }
    return 0;
}

// Runner::trunk (src/model.rs:355-399).
int trunk(D1Model* m, D1Workspace* ws, int t, const int* tok_seq, const SeqInfo* seqs,
          const std::vector<const AttnSeq*>& attn, const int* work, int n_work, bool prefix_pass, cudaStream_t st) {
    Kt& k = m->k;
    float* h = ws->h;
    d1_half *xn = ws->xn, *big = ws->big, *act = ws->act;
    const int nl = (int)m->layers.size();
    for (int li = 0; li < nl; li++) {
        const D1TrunkLayer& l = m->layers[li];
        const bool last = li + 1 == nl;
        const int idx = m->mixer_idx[li];
        m->launches++;
        CK(k.rmsnorm(h, l.op_norm, xn, t, D, m->w.eps, st));
        if (!l.is_attn) {
            CK(m->gemm(t, 3 * D, D, xn, D, l.in_proj, D, big, 3 * D, 0, 1.f, 0.f, st));
            m->launches++;
            CK(k.shortconv(big, l.convw, tok_seq, seqs, act, t, D, idx, st));
            if (prefix_pass && last) return 0;  // only the conv state of the last layer is needed
            CK(m->gemm(t, D, D, act, D, l.out_proj, D, h, D, 1, 1.f, 1.f, st));
        } else {
            const int ld = D + 2 * KV_DIM;
            if (m->fused && k.gemm_qk_rope && !prefix_pass) {  // prefix passes also store K/V to the cache
                m->launches += 2;
                CK(k.gemm_qk_rope(m->lt, t, D, xn, D, l.qkv, D, big, ld, HEADS, KV_HEADS, l.qn, l.kn, m->rope, tok_seq,
                                  seqs, m->w.eps, st));
            } else {
                CK(m->gemm(t, ld, D, xn, D, l.qkv, D, big, ld, 0, 1.f, 0.f, st));
                m->launches += 2;
                CK(k.qk_norm_rope(big, ld, HEADS, KV_HEADS, l.qn, l.kn, m->rope, tok_seq, seqs, idx, t, m->w.eps, st));
            }
            CK(k.attention(m->fused, big, ld, big + D, big + D + KV_DIM, ld, KV_DIM, nullptr, nullptr, nullptr, act, D,
                           attn[idx], work, n_work, HEADS, HEADS / KV_HEADS, 0.125f, t, t, st));
            if (prefix_pass && last) return 0;
            CK(m->gemm(t, D, D, act, D, l.out, D, h, D, 1, 1.f, 1.f, st));
        }
        m->launches++;
        CK(k.rmsnorm(h, l.ffn_norm, xn, t, D, m->w.eps, st));
        if (m->fused && k.gemm_swiglu) {
            m->launches++;
            CK(k.gemm_swiglu(m->lt, t, l.ffn, D, xn, D, l.gate_up, D, act, l.ffn, st));
        } else {
            CK(m->gemm(t, 2 * l.ffn, D, xn, D, l.gate_up, D, big, 2 * l.ffn, 0, 1.f, 0.f, st));
            m->launches++;
            CK(k.swiglu(big, act, t, l.ffn, st));
        }
        CK(m->gemm(t, D, l.ffn, act, l.ffn, l.down, l.ffn, h, D, 1, 1.f, 1.f, st));
    }
    return 0;
}

// up GEMM + ReLU(+b) of a head FFN: fused epilogue when available, else GEMM then d1_bias_act_h (src/model.rs:568-569).
int head_up(D1Model* m, int rows, int F, const d1_half* x, const d1_half* w, const float* b, d1_half* y,
            cudaStream_t st) {
    if (m->fused && m->k.gemm_bias_act) {
        m->launches++;
        CK(m->k.gemm_bias_act(m->lt, rows, F, D, x, D, w, D, b, 1, y, F, st));
        return 0;
    }
    CK(m->gemm(rows, F, D, x, D, w, D, y, F, 0, 1.f, 0.f, st));
    m->launches++;
    CK(m->k.bias_act_h(y, b, rows, F, 1, st));
    return 0;
}

}  // namespace

extern "C" {

const char* d1h_last_error(void) { return g_err.c_str(); }

D1Model* d1h_model_create(const D1TextWeights* w, const char* kernel_lib, int fused) {
    if (!w || w->n_layers <= 0 || !w->layers) {
        fail("invalid weights");
        return nullptr;
    }
    D1Model* m = new D1Model();
    bool ok = kernel_lib ? m->k.load_lib(kernel_lib) : m->k.load_builtin();
    if (!ok) {
        delete m;
        return nullptr;
    }
    cudaGetDevice(&m->dev);
    m->w = *w;
    m->layers.assign(w->layers, w->layers + w->n_layers);
    if (w->n_head > 0) m->head.assign(w->head, w->head + w->n_head);
    m->w.layers = nullptr;
    m->w.head = nullptr;
    for (const auto& l : m->layers) {
        m->mixer_idx.push_back(l.is_attn ? m->n_attn++ : m->n_conv++);
        m->max_ffn = std::max(m->max_ffn, l.ffn);
    }
    for (const auto& l : m->head) m->max_ffn = std::max(m->max_ffn, l.ffn);
    m->fused = fused != 0;
    m->lt = m->k.lt_init(32 << 20);  // src/cuda.rs:406
    if (!m->lt) {
        fail("d1_lt_init failed (needs an sm_100 GPU)");
        delete m;
        return nullptr;
    }
    std::vector<float> rt = rope_table(w->rope_theta);
    if (cudaMalloc(&m->rope, rt.size() * sizeof(float)) != cudaSuccess ||
        cudaMemcpy(m->rope, rt.data(), rt.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        fail("rope table upload failed");
        d1h_model_destroy(m);
        return nullptr;
    }
    return m;
}

void d1h_model_destroy(D1Model* m) {
    if (!m) return;
    if (m->rope) cudaFree(m->rope);
    if (m->lt && m->k.lt_destroy) m->k.lt_destroy(m->lt);
    if (m->k.dl) dlclose(m->k.dl);
    delete m;
}

long long d1h_launch_count(const D1Model* m) { return m ? m->launches.load() : 0LL; }

long long d1h_h2d_bytes(const D1Workspace* ws, int slot) {
    return ws && slot >= 0 && slot < SLOTS ? ws->h2d[slot] : -1;
}

long long d1h_d2h_bytes(const D1Workspace* ws, int slot) {
    return ws && slot >= 0 && slot < SLOTS ? 4LL * ws->n_logits[slot] : -1;
}

D1Workspace* d1h_workspace_create(D1Model* m, int cap_tokens) {
    if (!m || cap_tokens <= 0) return nullptr;
    D1Workspace* ws = new D1Workspace();
    ws->cap_tokens = cap_tokens;
    ws->cap_markers = cap_tokens / 2 + 64;
    const size_t ct = cap_tokens, cm = ws->cap_markers;
    const size_t big_w = std::max<size_t>(2 * (size_t)m->max_ffn, 3 * D);
    int e = 0;
    e |= dmalloc(&ws->h, ct * D * 4);
    e |= dmalloc(&ws->xn, ct * D * 2);
    e |= dmalloc(&ws->big, ct * big_w * 2);
    e |= dmalloc(&ws->act, ct * std::max(m->max_ffn, D) * 2);
    e |= dmalloc(&ws->mq, cm * 3 * D * 2);
    e |= dmalloc(&ws->mo, cm * D * 2);
    e |= dmalloc(&ws->mh, cm * D * 4);
    e |= dmalloc(&ws->mx, cm * D * 2);
    e |= dmalloc(&ws->mbig, cm * std::max(m->max_ffn, 1) * 2);
    e |= dmalloc(&ws->logits, cm * 4);
    e |= dmalloc(&ws->meta, META_BYTES);
    for (int s = 0; s < SLOTS && !e; s++) {
        if (cudaMallocHost((void**)&ws->host_meta[s], META_BYTES) != cudaSuccess ||
            cudaMallocHost((void**)&ws->host_logits[s], cm * 4) != cudaSuccess ||
            cudaEventCreateWithFlags(&ws->events[s], cudaEventDisableTiming) != cudaSuccess)
            e = fail("workspace host allocation failed");
    }
    if (e) {
        d1h_workspace_destroy(ws);
        return nullptr;
    }
    return ws;
}

void d1h_workspace_destroy(D1Workspace* ws) {
    if (!ws) return;
    for (void* p : {(void*)ws->h, (void*)ws->xn, (void*)ws->big, (void*)ws->act, (void*)ws->mq, (void*)ws->mo,
                    (void*)ws->mh, (void*)ws->mx, (void*)ws->mbig, (void*)ws->logits, (void*)ws->meta})
        if (p) cudaFree(p);
    for (int s = 0; s < SLOTS; s++) {
        if (ws->busy[s]) cudaEventSynchronize(ws->events[s]);
        if (ws->host_meta[s]) cudaFreeHost(ws->host_meta[s]);
        if (ws->host_logits[s]) cudaFreeHost(ws->host_logits[s]);
        if (ws->events[s]) cudaEventDestroy(ws->events[s]);
    }
    delete ws;
}

int d1h_prefix_alloc(D1Model* m, int len, D1PrefixCache* out, cudaStream_t st) {
    if (!m || !out || len <= 0) return fail("bad prefix size");
    const size_t kv = (size_t)m->n_attn * len * KV_DIM * 2;
    out->len = len;
    out->k = out->v = out->bx = nullptr;
    if (cudaMallocAsync((void**)&out->k, std::max<size_t>(kv, 256), st) != cudaSuccess ||
        cudaMallocAsync((void**)&out->v, std::max<size_t>(kv, 256), st) != cudaSuccess ||
        cudaMallocAsync((void**)&out->bx, std::max<size_t>((size_t)m->n_conv * D * 2, 256), st) != cudaSuccess)
        return fail("cudaMallocAsync failed for a prefix cache");
    return 0;
}

void d1h_prefix_free(D1PrefixCache* c, cudaStream_t st) {
    if (!c) return;
    for (d1_half** p : {&c->k, &c->v, &c->bx})
        if (*p) {
            cudaFreeAsync(*p, st);
            *p = nullptr;
        }
}

// Runner::launch_prefix (src/model.rs:402-459).
int d1h_launch_prefix(D1Model* m, D1Workspace* ws, int slot, const D1PrefixSeq* items, int n_items, cudaStream_t st) {
    if (!m || !ws || slot < 0 || slot >= SLOTS || n_items <= 0) return fail("bad arguments");
    int t = 0;
    for (int i = 0; i < n_items; i++) t += items[i].cache->len;
    if (t > ws->cap_tokens) return fail("prefix batch exceeds workspace capacity");
    if (wait_slot(ws, slot)) return -1;
    MetaWriter w{ws->host_meta[slot], ws->meta};
    std::vector<int> tok_seq;
    tok_seq.reserve(t);
    std::vector<SeqInfo> seqs;
    std::vector<std::pair<int, int>> spans;
    int start = 0;
    for (int i = 0; i < n_items; i++) {
        const int n = items[i].cache->len;
        tok_seq.insert(tok_seq.end(), n, i);
        SeqInfo s{};
        s.start = start;
        s.len = n;
        s.save_bx = items[i].cache->bx;
        s.save_k = items[i].cache->k;
        s.save_v = items[i].cache->v;
        seqs.push_back(s);
        spans.push_back({start, n});
        start += n;
    }
    const int* d_tok = w.put(tok_seq);
    const SeqInfo* d_seqs = w.put(seqs);
    std::vector<const AttnSeq*> attn;
    for (int l = 0; l < m->n_attn; l++) {
        std::vector<AttnSeq> a;
        for (auto& sp : spans) a.push_back(AttnSeq{sp.first, sp.second, sp.first, sp.second, 0, 0, nullptr, nullptr});
        attn.push_back(w.put(a));
    }
    std::vector<int> work = work_items(spans, m->k.attn_step(m->fused));
    const int* d_work = w.put(work);
    if (w.overflow) return fail("batch metadata exceeds 8 MB");
    if (cudaMemcpyAsync(ws->meta, ws->host_meta[slot], w.off, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail("metadata upload failed");
    for (int i = 0; i < n_items; i++)
        if (cudaMemcpyAsync(ws->h + (size_t)spans[i].first * D, items[i].emb, (size_t)spans[i].second * D * 4,
                            cudaMemcpyDeviceToDevice, st) != cudaSuccess)
            return fail("prefix embedding copy failed");
    int e = trunk(m, ws, t, d_tok, d_seqs, attn, d_work, (int)work.size() / 2, true, st);
    if (e) return e;
    ws->h2d[slot] = (long long)w.off;
    cudaEventRecord(ws->events[slot], st);
    ws->busy[slot] = true;
    ws->n_logits[slot] = 0;
    return 0;
}

// Runner::launch_text (src/model.rs:470-599).
int d1h_launch_text(D1Model* m, D1Workspace* ws, int slot, const D1TextSeq* seqs_in, int n_seqs, cudaStream_t st) {
    if (!m || !ws || slot < 0 || slot >= SLOTS || n_seqs <= 0) return fail("bad arguments");
    if (m->head.empty()) return fail("the model has no decision head");
    Kt& k = m->k;
    int t = 0, n_mark = 0;
    for (int i = 0; i < n_seqs; i++) {
        if (seqs_in[i].n_ids <= 0) return fail("empty sequence");
        t += seqs_in[i].n_ids;
        n_mark += seqs_in[i].n_markers;
        for (int j = 0; j < seqs_in[i].n_markers; j++)
            if (seqs_in[i].markers[j] < 0 || seqs_in[i].markers[j] >= seqs_in[i].n_ids) return fail("marker out of range");
    }
    if (t > ws->cap_tokens) return fail("text batch exceeds workspace capacity");
    if (n_mark > ws->cap_markers) return fail("too many markers for the workspace");
    if (wait_slot(ws, slot)) return -1;
    MetaWriter w{ws->host_meta[slot], ws->meta};

    std::vector<int> ids, tok_seq, marker_rows;
    ids.reserve(t);
    tok_seq.reserve(t);
    std::vector<SeqInfo> seqs;
    std::vector<std::pair<int, int>> spans, mspans;
    int start = 0;
    for (int i = 0; i < n_seqs; i++) {
        const D1TextSeq& s = seqs_in[i];
        ids.insert(ids.end(), s.ids, s.ids + s.n_ids);
        tok_seq.insert(tok_seq.end(), s.n_ids, i);
        SeqInfo si{};
        si.start = start;
        si.len = s.n_ids;
        si.pos_off = s.prefix ? s.prefix->len : 0;
        si.qtype = s.qtype;
        si.ext_bx = s.prefix ? s.prefix->bx : nullptr;
        seqs.push_back(si);
        mspans.push_back({(int)marker_rows.size(), s.n_markers});
        for (int j = 0; j < s.n_markers; j++) marker_rows.push_back(start + s.markers[j]);
        spans.push_back({start, s.n_ids});
        start += s.n_ids;
    }
    const int* d_ids = w.put(ids);
    const int* d_tok = w.put(tok_seq);
    const SeqInfo* d_seqs = w.put(seqs);
    std::vector<const AttnSeq*> attn;
    for (int l = 0; l < m->n_attn; l++) {
        std::vector<AttnSeq> a;
        for (int i = 0; i < n_seqs; i++) {
            const D1PrefixCache* p = seqs_in[i].prefix;
            AttnSeq as{spans[i].first, spans[i].second, spans[i].first, spans[i].second, 0, 0, nullptr, nullptr};
            if (p) {
                as.ext_len = p->len;
                as.ext_k = p->k + (size_t)l * p->len * KV_DIM;
                as.ext_v = p->v + (size_t)l * p->len * KV_DIM;
            }
            a.push_back(as);
        }
        attn.push_back(w.put(a));
    }
    std::vector<AttnSeq> head_attn, last_attn;
    for (int i = 0; i < n_seqs; i++) {
        head_attn.push_back(AttnSeq{spans[i].first, spans[i].second, spans[i].first, spans[i].second, 0, 0, nullptr, nullptr});
        last_attn.push_back(AttnSeq{mspans[i].first, mspans[i].second, spans[i].first, spans[i].second, 0, 0, nullptr, nullptr});
    }
    const AttnSeq* d_head_attn = w.put(head_attn);
    const AttnSeq* d_last_attn = w.put(last_attn);
    const int step = m->k.attn_step(m->fused);
    std::vector<int> work = work_items(spans, step), mwork = work_items(mspans, step);
    const int* d_work = w.put(work);
    const int* d_mwork = w.put(mwork);
    const int* d_mrows = w.put(marker_rows);
    if (w.overflow) return fail("batch metadata exceeds 8 MB");
    const int n_work = (int)work.size() / 2, n_mwork = (int)mwork.size() / 2;

    float* h = ws->h;
    d1_half *xn = ws->xn, *big = ws->big, *act = ws->act;
    if (cudaMemcpyAsync(ws->meta, ws->host_meta[slot], w.off, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail("metadata upload failed");
    m->launches++;
    CK(k.embed(m->w.embed, d_ids, h, t, D, st));
    int e = trunk(m, ws, t, d_tok, d_seqs, attn, d_work, n_work, false, st);
    if (e) return e;

    m->launches++;
    CK(k.head_init(h, m->w.final_norm, m->w.type_emb, d_tok, d_seqs, h, t, m->w.eps, st));
    const float* pend = nullptr;
    const int nh = (int)m->head.size();
    const int qkv_ld = 3 * D;
    for (int li = 0; li < nh; li++) {
        const D1HeadLayer& l = m->head[li];
        m->launches++;
        CK(k.layernorm(h, pend, 1.f, l.n1_w, l.n1_b, xn, nullptr, t, D, 1e-5f, st));
        // q/k/v biases: the reference adds them as flash attention loads q/k/v (fp32 add, rounded to fp16); with
        // the fused epilogue the QKV GEMM adds them to its fp16-rounded output instead — the same values — and the
        // attention runs its bias-free path.
        const bool fold = m->fused && k.gemm_bias_act;
        if (fold) {
            m->launches++;
            CK(k.gemm_bias_act(m->lt, t, qkv_ld, D, xn, D, l.qkv, D, l.qkv_b, 0, big, qkv_ld, st));
        } else {
            CK(m->gemm(t, qkv_ld, D, xn, D, l.qkv, D, big, qkv_ld, 0, 1.f, 0.f, st));
        }
        const float* bq = fold ? nullptr : l.qkv_b;
        const float* bk = fold ? nullptr : l.qkv_b + D;
        const float* bv = fold ? nullptr : l.qkv_b + 2 * D;
        if (li + 1 < nh) {
            m->launches++;
            CK(k.attention(m->fused, big, qkv_ld, big + D, big + 2 * D, qkv_ld, 0, bq, bk, bv, act, D, d_head_attn,
                           d_work, n_work, HEADS, 1, 0.125f, t, t, st));
            CK(m->gemm(t, D, D, act, D, l.out, D, h, D, 1, 1.f, 1.f, st));
            m->launches++;
            CK(k.layernorm(h, l.out_b, 1.f, l.n2_w, l.n2_b, xn, nullptr, t, D, 1e-5f, st));
            if (head_up(m, t, l.ffn, xn, l.up, l.up_b, big, st)) return -1;
            CK(m->gemm(t, D, l.ffn, big, l.ffn, l.down, l.ffn, h, D, 1, 1.f, 1.f, st));
            pend = l.down_b;
        } else {
            // Last head layer: queries, the output projection and the FFN run on marker rows only; keys/values
            // still cover every text position (src/model.rs:572-592).
            const int nm = n_mark;
            if (nm > 0) {
                m->launches += 3;
                CK(k.gather_rows(big, ws->mq, d_mrows, nm, qkv_ld * 2, st));
                CK(k.gather_rows(h, ws->mh, d_mrows, nm, D * 4, st));
                CK(k.attention(m->fused, ws->mq, qkv_ld, big + D, big + 2 * D, qkv_ld, 0, bq, bk, bv, ws->mo, D,
                               d_last_attn, d_mwork, n_mwork, HEADS, 1, 0.125f, nm, t, st));
                CK(m->gemm(nm, D, D, ws->mo, D, l.out, D, ws->mh, D, 1, 1.f, 1.f, st));
                m->launches++;
                CK(k.layernorm(ws->mh, l.out_b, 1.f, l.n2_w, l.n2_b, ws->mx, nullptr, nm, D, 1e-5f, st));
                if (head_up(m, nm, l.ffn, ws->mx, l.up, l.up_b, ws->mbig, st)) return -1;
                CK(m->gemm(nm, D, l.ffn, ws->mbig, l.ffn, l.down, l.ffn, ws->mh, D, 1, 1.f, 1.f, st));
                // scorer: LN -> Linear -> GELU -> Linear(1)
                m->launches++;
                CK(k.layernorm(ws->mh, l.down_b, 1.f, m->w.cls_norm_w, m->w.cls_norm_b, ws->mx, nullptr, nm, D, 1e-5f,
                               st));
                CK(m->gemm(nm, D, D, ws->mx, D, m->w.cls_w, D, ws->mo, D, 0, 1.f, 0.f, st));
                m->launches++;
                CK(k.scorer_out(ws->mo, m->w.cls_b, m->w.out_w, m->w.out_b, ws->logits, nm, D, st));
            }
        }
    }
    if (n_mark > 0 &&
        cudaMemcpyAsync(ws->host_logits[slot], ws->logits, (size_t)n_mark * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        return fail("logits download failed");
    ws->h2d[slot] = (long long)w.off;
    cudaEventRecord(ws->events[slot], st);
    ws->busy[slot] = true;
    ws->n_logits[slot] = n_mark;
    return 0;
}

// Runner::finish (src/model.rs:602-607).
int d1h_finish(D1Model* m, D1Workspace* ws, int slot, float* out, int cap) {
    if (!m || !ws || slot < 0 || slot >= SLOTS) return fail("bad arguments");
    if (!ws->busy[slot]) return fail("slot not launched");
    if (cudaEventSynchronize(ws->events[slot]) != cudaSuccess) return fail("event sync failed");
    ws->busy[slot] = false;
    const int n = ws->n_logits[slot];
    if (out) memcpy(out, ws->host_logits[slot], (size_t)std::min(n, cap) * 4);
    return n;
}

// GEMM tuning over every trunk/head shape and M bucket (src/engine.rs:528-616, text shapes only).
int d1h_tune(D1Model* m, D1Workspace* ws, int max_tokens, cudaStream_t st) {
    if (!m || !ws) return fail("bad arguments");
    struct Shape {
        int n, k, ldx, ldw, ldy, y_f32, cap;
    };
    std::vector<Shape> shapes;
    auto add = [&](Shape s) {
        for (auto& x : shapes)
            if (x.n == s.n && x.k == s.k && x.ldx == s.ldx && x.ldw == s.ldw && x.ldy == s.ldy && x.y_f32 == s.y_f32) {
                x.cap = std::max(x.cap, s.cap);
                return;
            }
        shapes.push_back(s);
    };
    const int mk = std::min(max_tokens, ws->cap_tokens), mm = std::min(max_tokens / 2 + 64, ws->cap_markers);
    for (const auto& l : m->layers) {
        if (l.is_attn) {
            add({D + 2 * KV_DIM, D, D, D, D + 2 * KV_DIM, 0, mk});
        } else {
            add({3 * D, D, D, D, 3 * D, 0, mk});
        }
        add({D, D, D, D, D, 1, mk});
        if (!(m->fused && m->k.gemm_swiglu)) add({2 * l.ffn, D, D, D, 2 * l.ffn, 0, mk});
        add({D, l.ffn, l.ffn, l.ffn, D, 1, mk});
    }
    for (const auto& l : m->head) {
        add({3 * D, D, D, D, 3 * D, 0, mk});
        if (!(m->fused && m->k.gemm_bias_act)) add({l.ffn, D, D, D, l.ffn, 0, mk});
        add({D, l.ffn, l.ffn, l.ffn, D, 1, mk});
        add({D, D, D, D, D, 0, mm});
    }
    int n = 0;
    for (const auto& s : shapes) {
        int b = 1;
        while (true) {
            const int nb = m->k.lt_bucket(b);
            if (m->k.lt_tune(m->lt, nb, s.n, s.k, s.ldx, s.ldw, 0, s.ldy, s.y_f32, 0, 1, st) < 0.f)
                return fail("tuning failed for n=" + std::to_string(s.n) + " k=" + std::to_string(s.k));
            n++;
            if (nb >= s.cap || nb >= 16384) break;
            b = nb + 1;
        }
    }
    cudaStreamSynchronize(st);
    m->k.lt_free_scratch(m->lt);
    return n;
}

}  // extern "C"

// ================================================================================================ vision encoder
// VisionModel (src/vision.rs:143-164) and VisionModel::encode (:305-385).

namespace {
constexpr int VD = 768;       // src/vision.rs:13
constexpr int VHEADS = 12;    // :14
constexpr int VFF = 3072;     // :15
constexpr int VOUT = 1024;    // :16
constexpr int VHID = 2048;    // projector hidden (src/vision.rs:379)
constexpr size_t VMETA = 1 << 20;

// Separable antialiased bilinear weights, as F.interpolate(antialias=True, align_corners=False) computes them
// (src/vision.rs:173-196): for every output index, the first input index and the normalised weights.
std::vector<std::pair<int, std::vector<float>>> aa_weights(int inp, int out) {
    const double scale = (double)inp / (double)out;
    const double support = scale >= 1.0 ? scale : 1.0;
    const double invscale = scale >= 1.0 ? 1.0 / scale : 1.0;
    std::vector<std::pair<int, std::vector<float>>> res;
    for (int i = 0; i < out; i++) {
        const double center = scale * (i + 0.5);
        long long xmin = (long long)(center - support + 0.5);
        long long xmax = (long long)(center + support + 0.5);
        if (xmin < 0) xmin = 0;
        if (xmax > inp) xmax = inp;
        std::vector<double> w;
        double t = 0.0;
        for (long long j = xmin; j < xmax; j++) {
            const double x = ((double)j - center + 0.5) * invscale;
            const double v = fabs(x) < 1.0 ? 1.0 - fabs(x) : 0.0;
            w.push_back(v);
            t += v;
        }
        std::vector<float> wf;
        for (double v : w) wf.push_back((float)(t != 0.0 ? v / t : v));
        res.push_back({(int)xmin, wf});
    }
    return res;
}
}  // namespace

struct D1Vision {
    Kt k;
    void* lt = nullptr;
    D1VisionWeights w{};
    std::vector<D1VisionLayer> layers;
    std::vector<float> patch_b, pos;
    bool builtin = true;               // this library's kernels: position embeddings resized on the GPU
    float* d_grid = nullptr;           // device [256][768] position grid
    float* d_patch_b = nullptr;        // device [768]
    // another kernel library (the reference's): the reference's host resize, cached per grid shape
    std::map<std::pair<int, int>, float*> pos_cache;  // (ph, pw) -> device [ph*pw][768] pos + bias
    bool fused = false;
    long long launches = 0;
    int max_patches = 0;
    float* h = nullptr;
    d1_half *xn = nullptr, *big = nullptr, *act = nullptr, *pix = nullptr;
    uint8_t* meta = nullptr;
    uint8_t* host_meta = nullptr;
    uint8_t* host_pix = nullptr;       // pinned staging of the patch rows
    cudaEvent_t done = nullptr;        // the previous call's last kernel
    cudaEvent_t staged = nullptr;      // the previous call's host->device copies
    bool busy = false;

    // With another kernel library (the reference's): resized position embeddings + patch bias for a (ph, pw) grid,
    // computed on the host and cached on the
    // device (src/vision.rs:263-302).
    float* pos_for(int ph, int pw) {
        auto it = pos_cache.find({ph, pw});
        if (it != pos_cache.end()) return it->second;
        auto wy = aa_weights(16, ph), wx = aa_weights(16, pw);
        std::vector<float> tmp((size_t)16 * pw * VD, 0.f), out((size_t)ph * pw * VD, 0.f);
        for (int y = 0; y < 16; y++)
            for (int x = 0; x < pw; x++) {
                const int s0 = wx[x].first;
                const auto& ws = wx[x].second;
                float* dst = &tmp[((size_t)y * pw + x) * VD];
                for (size_t j = 0; j < ws.size(); j++) {
                    const float* src = &pos[((size_t)y * 16 + s0 + j) * VD];
                    for (int c = 0; c < VD; c++) dst[c] += ws[j] * src[c];
                }
            }
        for (int y = 0; y < ph; y++) {
            const int s0 = wy[y].first;
            const auto& ws = wy[y].second;
            for (int x = 0; x < pw; x++) {
                float* dst = &out[((size_t)y * pw + x) * VD];
                for (size_t j = 0; j < ws.size(); j++) {
                    const float* src = &tmp[(((size_t)s0 + j) * pw + x) * VD];
                    for (int c = 0; c < VD; c++) dst[c] += ws[j] * src[c];
                }
                for (int c = 0; c < VD; c++) dst[c] += patch_b[c];
            }
        }
        float* d = nullptr;
        if (cudaMalloc(&d, out.size() * 4) != cudaSuccess ||
            cudaMemcpy(d, out.data(), out.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            fail("position embedding upload failed");
            return nullptr;
        }
        pos_cache[{ph, pw}] = d;
        return d;
    }
};

extern "C" {

D1Vision* d1h_vision_create(const D1VisionWeights* w, const char* kernel_lib, int fused, int max_patches) {
    if (!w || w->n_layers <= 0 || !w->layers || !w->patch_b || !w->pos || max_patches <= 0) {
        fail("invalid vision weights");
        return nullptr;
    }
    D1Vision* v = new D1Vision();
    if (!(kernel_lib ? v->k.load_lib(kernel_lib) : v->k.load_builtin())) {
        delete v;
        return nullptr;
    }
    v->w = *w;
    v->layers.assign(w->layers, w->layers + w->n_layers);
    v->w.layers = nullptr;
    v->patch_b.assign(w->patch_b, w->patch_b + VD);
    v->pos.assign(w->pos, w->pos + 256 * VD);
    v->w.patch_b = v->w.pos = nullptr;
    v->builtin = kernel_lib == nullptr;
    v->fused = fused != 0;
    v->max_patches = max_patches;
    v->lt = v->k.lt_init(32 << 20);
    const size_t cap = max_patches;
    int e = 0;
    if (!v->lt) e = fail("d1_lt_init failed");
    if (!e) e |= dmalloc(&v->h, cap * VD * 4);
    if (!e) e |= dmalloc(&v->xn, cap * VD * 2);
    if (!e) e |= dmalloc(&v->big, cap * VFF * 2);
    if (!e) e |= dmalloc(&v->act, cap * VD * 2);
    if (!e) e |= dmalloc(&v->pix, cap * VD * 2);
    if (!e) e |= dmalloc(&v->meta, VMETA);
    if (!e && v->builtin) {
        e |= dmalloc(&v->d_grid, v->pos.size() * 4);
        if (!e) e |= dmalloc(&v->d_patch_b, VD * 4);
        if (!e && (cudaMemcpy(v->d_grid, v->pos.data(), v->pos.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                   cudaMemcpy(v->d_patch_b, v->patch_b.data(), VD * 4, cudaMemcpyHostToDevice) != cudaSuccess))
            e = fail("position grid upload failed");
    }
    if (!e && (cudaMallocHost((void**)&v->host_meta, VMETA) != cudaSuccess ||
               cudaMallocHost((void**)&v->host_pix, cap * VD * 2) != cudaSuccess ||
               cudaEventCreateWithFlags(&v->done, cudaEventDisableTiming) != cudaSuccess ||
               cudaEventCreateWithFlags(&v->staged, cudaEventDisableTiming) != cudaSuccess))
        e = fail("vision host allocation failed");
    if (e) {
        d1h_vision_destroy(v);
        return nullptr;
    }
    return v;
}

void d1h_vision_destroy(D1Vision* v) {
    if (!v) return;
    if (v->busy) cudaEventSynchronize(v->done);
    for (void* p : {(void*)v->h, (void*)v->xn, (void*)v->big, (void*)v->act, (void*)v->pix, (void*)v->meta,
                    (void*)v->d_grid, (void*)v->d_patch_b})
        if (p) cudaFree(p);
    for (auto& kv : v->pos_cache) cudaFree(kv.second);
    if (v->host_meta) cudaFreeHost(v->host_meta);
    if (v->host_pix) cudaFreeHost(v->host_pix);
    if (v->done) cudaEventDestroy(v->done);
    if (v->staged) cudaEventDestroy(v->staged);
    if (v->lt && v->k.lt_destroy) v->k.lt_destroy(v->lt);
    if (v->k.dl) dlclose(v->k.dl);
    delete v;
}

int d1h_vision_encode(D1Vision* v, int n_crops, const int* ph, const int* pw, const d1_half* pixels, float* out,
                      cudaStream_t st) {
    if (!v || n_crops <= 0 || !ph || !pw || !pixels || !out) return fail("bad arguments");
    Kt& k = v->k;
    long long t = 0;
    for (int i = 0; i < n_crops; i++) {
        if (ph[i] <= 0 || pw[i] <= 0 || (ph[i] & 1) || (pw[i] & 1) || ph[i] > 1024 || pw[i] > 1024)
            return fail("crop grids must be positive and even");
        t += (long long)ph[i] * pw[i];
    }
    if (t > v->max_patches) return fail("patches exceed the vision batch capacity");
    if (v->busy) {
        // the host staging may be refilled once the previous call's copies are done; its device buffers are
        // reused in stream order after its last kernel
        if (cudaEventSynchronize(v->staged) != cudaSuccess || cudaStreamWaitEvent(st, v->done, 0) != cudaSuccess)
            return fail("event sync failed");
        v->busy = false;
    }
    // metadata: one AttnSeq per crop and its 64-row query tiles (src/vision.rs:310-326)
    std::vector<AttnSeq> seqs;
    std::vector<std::pair<int, int>> spans;
    int off = 0;
    for (int i = 0; i < n_crops; i++) {
        const int n = ph[i] * pw[i];
        seqs.push_back(AttnSeq{off, n, off, n, 0, 0, nullptr, nullptr});
        spans.push_back({off, n});
        off += n;
    }
    std::vector<int> work = work_items(spans, v->k.attn_step(v->fused));
    MetaWriter mw{v->host_meta, v->meta};
    const AttnSeq* d_seqs = mw.put(seqs);
    const int* d_work = mw.put(work);
    // per crop: the separable resize taps of its position embeddings (src/vision.rs:173-196), for d1_vision_pos
    std::vector<const int*> pos_spans(n_crops);
    std::vector<const float*> pos_w(n_crops);
    std::vector<int> pos_taps(n_crops);
    if (v->builtin) {
        for (int i = 0; i < n_crops; i++) {
            auto wy = aa_weights(16, ph[i]), wx = aa_weights(16, pw[i]);
            size_t taps = 1;
            for (auto& e : wy) taps = std::max(taps, e.second.size());
            for (auto& e : wx) taps = std::max(taps, e.second.size());
            std::vector<int> sp;
            std::vector<float> wt((size_t)(ph[i] + pw[i]) * taps, 0.f);
            size_t r = 0;
            for (auto* tab : {&wy, &wx})
                for (auto& e : *tab) {
                    sp.push_back(e.first);
                    sp.push_back((int)e.second.size());
                    std::copy(e.second.begin(), e.second.end(), wt.begin() + r * taps);
                    r++;
                }
            pos_spans[i] = mw.put(sp);
            pos_w[i] = mw.put(wt);
            pos_taps[i] = (int)taps;
        }
    }
    // fused: the unshuffle (src/vision.rs:372-376) as the output rows of the post-LayerNorm, which then writes the
    // projector input directly (row y*pw + x of a crop -> row 4*((y/2)*(pw/2) + x/2) + 2*(y%2) + x%2 of big)
    const int* d_unshuffle = nullptr;
    if (v->fused && v->builtin) {
        std::vector<int> yr((size_t)t);
        size_t src = 0, dst = 0;
        for (int i = 0; i < n_crops; i++) {
            const int hw = pw[i] / 2;
            for (int y = 0; y < ph[i]; y++)
                for (int x = 0; x < pw[i]; x++)
                    yr[src++] = (int)(4 * (dst + (size_t)(y / 2) * hw + x / 2) + 2 * (y % 2) + x % 2);
            dst += (size_t)ph[i] * pw[i] / 4;
        }
        d_unshuffle = mw.put(yr);
    }
    if (mw.overflow || mw.off > VMETA) return fail("vision metadata too large");
    memcpy(v->host_pix, pixels, (size_t)t * VD * 2);
    if (cudaMemcpyAsync(v->meta, v->host_meta, mw.off, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(v->pix, v->host_pix, (size_t)t * VD * 2, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaEventRecord(v->staged, st) != cudaSuccess)
        return fail("vision upload failed");
    const int ti = (int)t, n_work = (int)work.size() / 2;
    // embeddings: h = pos + bias per crop, then += pixels . W^T
    off = 0;
    for (int i = 0; i < n_crops; i++) {
        if (v->builtin) {
            v->launches++;
            CK(d1_vision_pos(v->d_grid, v->d_patch_b, pos_spans[i], pos_w[i], pos_taps[i], ph[i], pw[i], VD,
                             v->h + (size_t)off * VD, st));
        } else {
            float* p = v->pos_for(ph[i], pw[i]);
            if (!p) return -1;
            if (cudaMemcpyAsync(v->h + (size_t)off * VD, p, (size_t)ph[i] * pw[i] * VD * 4, cudaMemcpyDeviceToDevice,
                                st) != cudaSuccess)
                return fail("position copy failed");
        }
        off += ph[i] * pw[i];
    }
    float* h = v->h;
    d1_half *xn = v->xn, *big = v->big, *act = v->act;
    long long& L = v->launches;
    CK(kt_gemm(k, v->lt, L, ti, VD, VD, v->pix, VD, v->w.patch_w, VD, h, VD, 1, 1.f, 1.f, st));
    const float* pend = nullptr;
    const float eps = v->w.eps;
    for (const auto& l : v->layers) {
        L++;
        CK(k.layernorm(h, pend, 1.f, l.ln1_w, l.ln1_b, xn, nullptr, ti, VD, eps, st));
        // q/k/v biases folded into the QKV GEMM epilogue when fused (same fp16 values as adding them on load)
        const bool fold = v->fused && k.gemm_bias_act;
        if (fold) {
            L++;
            CK(k.gemm_bias_act(v->lt, ti, 3 * VD, VD, xn, VD, l.qkv, VD, l.qkv_b, 0, big, 3 * VD, st));
        } else {
            CK(kt_gemm(k, v->lt, L, ti, 3 * VD, VD, xn, VD, l.qkv, VD, big, 3 * VD, 0, 1.f, 0.f, st));
        }
        L++;
        CK(k.attention(v->fused, big, 3 * VD, big + VD, big + 2 * VD, 3 * VD, 0, fold ? nullptr : l.qkv_b,
                       fold ? nullptr : l.qkv_b + VD, fold ? nullptr : l.qkv_b + 2 * VD, act, VD, d_seqs, d_work,
                       n_work, VHEADS, 1, 0.125f, ti, ti, st));
        CK(kt_gemm(k, v->lt, L, ti, VD, VD, act, VD, l.out, VD, h, VD, 1, 1.f, 1.f, st));
        L++;
        CK(k.layernorm(h, l.out_b, 1.f, l.ln2_w, l.ln2_b, xn, nullptr, ti, VD, eps, st));
        if (v->fused && k.gemm_bias_act) {
            L++;
            CK(k.gemm_bias_act(v->lt, ti, VFF, VD, xn, VD, l.fc1, VD, l.fc1_b, 3, big, VFF, st));
        } else {
            CK(kt_gemm(k, v->lt, L, ti, VFF, VD, xn, VD, l.fc1, VD, big, VFF, 0, 1.f, 0.f, st));
            L++;
            CK(k.bias_act_h(big, l.fc1_b, ti, VFF, 3, st));
        }
        CK(kt_gemm(k, v->lt, L, ti, VD, VFF, big, VFF, l.fc2, VFF, h, VD, 1, 1.f, 1.f, st));
        pend = l.fc2_b;
    }
    L++;
    int src = 0, dst = 0;
    if (d_unshuffle) {
        CK(d1_layernorm_rows(h, pend, 1.f, v->w.post_w, v->w.post_b, big, d_unshuffle, ti, VD, eps, st));
        dst = ti / 4;
    } else {
        CK(k.layernorm(h, pend, 1.f, v->w.post_w, v->w.post_b, xn, nullptr, ti, VD, eps, st));
        // projector: unshuffle each crop -> big [P, 3072] -> linear_1 + GELU -> linear_2 (+bias) -> out
        for (int i = 0; i < n_crops; i++) {
            L++;
            CK(k.unshuffle(xn + (size_t)src * VD, big + (size_t)dst * 4 * VD, ph[i], pw[i], VD, st));
            src += ph[i] * pw[i];
            dst += ph[i] * pw[i] / 4;
        }
    }
    const int p = dst;
    if (v->fused && k.gemm_bias_act) {
        L++;
        CK(k.gemm_bias_act(v->lt, p, VHID, 4 * VD, big, 4 * VD, v->w.proj1, 4 * VD, v->w.proj1_b, 2, act, VHID, st));
    } else {
        CK(kt_gemm(k, v->lt, L, p, VHID, 4 * VD, big, 4 * VD, v->w.proj1, 4 * VD, act, VHID, 0, 1.f, 0.f, st));
        L++;
        CK(k.bias_act_h(act, v->w.proj1_b, p, VHID, 2, st));
    }
    L++;
    CK(k.fill_rows(out, v->w.proj2_b, nullptr, p, VOUT, st));
    CK(kt_gemm(k, v->lt, L, p, VOUT, VHID, act, VHID, v->w.proj2, VHID, out, VOUT, 1, 1.f, 1.f, st));
    cudaEventRecord(v->done, st);
    v->busy = true;
    return 0;
}

}  // extern "C"

// ================================================================================================ audio encoder
// AudioModel (src/audio.rs:302-455) and AudioModel::encode (:505-594), with several clips per call: each clip's
// subsampling runs on its own rows, then the conformer layers and the adapter run once over all clips' rows
// (every op is row-wise except the depthwise conv, launched per clip, and the rel-pos attention, which takes the
// clip offsets). The relative-position projections pp = pe . linear_pos^T depend only on the weights and the
// relative position, so they are computed once at create for positions -(MAX_T-1) .. MAX_T-1 (one table per
// layer) instead of per clip and layer (src/audio.rs:546-558, 568).

namespace {
constexpr int AD = 512;          // src/audio.rs:16
constexpr int AHEADS = 8;        // :17
constexpr int SUB_C = 256;       // :18
constexpr int AOUT = 1024;       // :19
constexpr int N_MELS = 128;      // :15
constexpr int A_MAX_T = 384;     // :401
constexpr int A_MAX_VALID = 3000;  // 30 s at hop 160 (src/audio.rs:11-14, 241-247)
constexpr int A_MAX_SAMPLES = 30 * 16000;  // src/audio.rs:10-11
constexpr int A_MIN_SAMPLES = 8000;
constexpr int PP_ROWS = 2 * A_MAX_T - 1;
constexpr int PP_CENTER = A_MAX_T - 1;

// pe rows for relative positions PP_CENTER - m, m = 0 .. PP_ROWS-1, as src/audio.rs:546-558 computes each row:
// fp32 frequency exp(2i * -(ln 10000 / 512)), fp32 angle p * f, sin / cos in double, rounded to fp16.
std::vector<uint16_t> audio_pe_table() {
    std::vector<uint16_t> pe((size_t)PP_ROWS * AD);
    const float c = (float)(-(log(10000.0) / (double)AD));
    for (int m = 0; m < PP_ROWS; m++) {
        const float p = (float)(PP_CENTER - m);
        for (int i = 0; i < AD / 2; i++) {
            const float div = expf((float)(2 * i) * c);
            const double a = (double)(p * div);
            pe[(size_t)m * AD + 2 * i] = f32_to_f16_bits((float)sin(a));
            pe[(size_t)m * AD + 2 * i + 1] = f32_to_f16_bits((float)cos(a));
        }
    }
    return pe;
}

int audio_out_len(int valid) {
    const int l1 = (valid - 1) / 2 + 1, l2 = (l1 - 1) / 2 + 1;
    return (l2 - 1) / 2 + 1;
}
}  // namespace

struct D1Audio {
    void* lt = nullptr;
    D1AudioWeights w{};
    std::vector<D1AudioLayer> layers;
    bool fused = true;
    int max_rows = 0;
    long long launches = 0;
    d1_half* pp = nullptr;          // [n_layers][PP_ROWS][512]
    float *mel = nullptr, *s1 = nullptr, *s2 = nullptr, *s3 = nullptr, *x = nullptr, *pcm = nullptr;
    long long mel_rows = 0;  // capacity of mel in frames
    size_t pcm_cap = 0;      // capacity of pcm in samples
    d1_half *xn = nullptr, *big = nullptr, *qu = nullptr, *qv = nullptr, *kk = nullptr, *vv = nullptr, *o = nullptr;
    int* offs = nullptr;
    int* host_offs = nullptr;          // pinned: clip offsets
    float* host_mel = nullptr;         // pinned staging of log-mel frames [mel_rows][128]
    float* host_pcm = nullptr;         // pinned staging of waveforms [pcm_cap]
    float* src = nullptr;              // waveforms at other sample rates, before d1_resample [src_cap]
    float* host_src = nullptr;         // their pinned staging
    float* rs = nullptr;               // one clip resampled to 16 kHz [rs_cap]
    size_t src_cap = 0, rs_cap = 0;    // grown on demand
    cudaEvent_t done = nullptr;        // the previous call's last kernel
    cudaEvent_t staged = nullptr;      // the previous call's host->device copies
    bool busy = false;
};

extern "C" {

D1Audio* d1h_audio_create(const D1AudioWeights* w, int fused, int max_rows) {
    if (!w || w->n_layers <= 0 || !w->layers || max_rows <= 0 || max_rows > (1 << 20)) {
        fail("invalid audio weights or capacity");
        return nullptr;
    }
    D1Audio* a = new D1Audio();
    a->w = *w;
    a->layers.assign(w->layers, w->layers + w->n_layers);
    a->w.layers = nullptr;
    a->fused = fused != 0;
    a->max_rows = max_rows;
    const size_t R = max_rows, L1 = (A_MAX_VALID - 1) / 2 + 1, L2 = (L1 - 1) / 2 + 1;
    int e = 0;
    a->lt = d1_lt_init(0);
    if (!a->lt) e = fail("d1_lt_init failed");
    if (!e) e |= dmalloc(&a->pp, (size_t)w->n_layers * PP_ROWS * AD * 2);
    a->mel_rows = (long long)R * 8 + 4096;  // sum of valid <= 8 * rows, plus one spare frame per clip
    if (!e) e |= dmalloc(&a->mel, (size_t)a->mel_rows * N_MELS * 4);
    // waveform staging for d1h_audio_encode_pcm: a clip of T rows has valid <= 8T frames and fewer than
    // 160 (valid + 1) samples, and a call has at most R / 7 clips (0.5 s minimum -> 7 rows): < 1303 R samples
    a->pcm_cap = std::min<size_t>(R * 1304 + 2 * (size_t)A_MIN_SAMPLES, (size_t)64 * A_MAX_SAMPLES);
    if (!e) e |= dmalloc(&a->pcm, a->pcm_cap * 4);
    if (!e) e |= dmalloc(&a->s1, L1 * 64 * SUB_C * 4);
    if (!e) e |= dmalloc(&a->s2, L2 * 32 * SUB_C * 4);
    if (!e) e |= dmalloc(&a->s3, L2 * 32 * SUB_C * 4);
    if (!e) e |= dmalloc(&a->x, R * AD * 4);
    if (!e) e |= dmalloc(&a->xn, R * AOUT * 2);
    if (!e) e |= dmalloc(&a->big, R * 4 * AD * 2);
    for (d1_half** p : {&a->qu, &a->qv, &a->kk, &a->vv, &a->o})
        if (!e) e |= dmalloc(p, R * AD * 2);
    if (!e) e |= dmalloc(&a->offs, 4096 * 4);
    if (!e && (cudaMallocHost((void**)&a->host_offs, 4096 * 4) != cudaSuccess ||
               cudaMallocHost((void**)&a->host_mel, (size_t)a->mel_rows * N_MELS * 4) != cudaSuccess ||
               cudaMallocHost((void**)&a->host_pcm, a->pcm_cap * 4) != cudaSuccess ||
               cudaEventCreateWithFlags(&a->done, cudaEventDisableTiming) != cudaSuccess ||
               cudaEventCreateWithFlags(&a->staged, cudaEventDisableTiming) != cudaSuccess))
        e = fail("audio host allocation failed");
    if (!e) {  // per-layer relative-position projections
        std::vector<uint16_t> pe = audio_pe_table();
        d1_half* dpe = nullptr;
        e |= dmalloc(&dpe, pe.size() * 2);
        if (!e && cudaMemcpy(dpe, pe.data(), pe.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess)
            e = fail("pe upload failed");
        for (int l = 0; l < w->n_layers && !e; l++) {
            a->launches++;
            if (d1_lt_gemm(a->lt, PP_ROWS, AD, AD, dpe, AD, a->layers[l].pos, AD, 0, a->pp + (size_t)l * PP_ROWS * AD,
                           AD, 0, 0, 1.f, 0.f, 0))
                e = fail("pp projection failed");
        }
        if (!e && cudaDeviceSynchronize() != cudaSuccess) e = fail("pp projection failed");
        if (dpe) cudaFree(dpe);
    }
    if (e) {
        d1h_audio_destroy(a);
        return nullptr;
    }
    return a;
}

void d1h_audio_destroy(D1Audio* a) {
    if (!a) return;
    if (a->busy) cudaEventSynchronize(a->done);
    for (void* p : {(void*)a->pp, (void*)a->mel, (void*)a->pcm, (void*)a->s1, (void*)a->s2, (void*)a->s3, (void*)a->x, (void*)a->xn,
                    (void*)a->big, (void*)a->qu, (void*)a->qv, (void*)a->kk, (void*)a->vv, (void*)a->o,
                    (void*)a->offs})
        if (p) cudaFree(p);
    for (void* p : {(void*)a->src, (void*)a->rs})
        if (p) cudaFree(p);
    for (void* p : {(void*)a->host_offs, (void*)a->host_mel, (void*)a->host_pcm, (void*)a->host_src})
        if (p) cudaFreeHost(p);
    if (a->done) cudaEventDestroy(a->done);
    if (a->staged) cudaEventDestroy(a->staged);
    if (a->lt) d1_lt_destroy(a->lt);
    delete a;
}

}  // extern "C"

namespace {

// Checks the clips, waits for the previous call, uploads the clip offsets; returns the output rows (or < 0).
int audio_prepare(D1Audio* a, int n_clips, const int* valid, int& max_t, cudaStream_t st) {
    int rows = 0;
    max_t = 0;
    for (int c = 0; c < n_clips; c++) {
        if (valid[c] < 1 || valid[c] > A_MAX_VALID) return fail("clip frames must be 1 .. 3000");
        const int t = audio_out_len(valid[c]);
        rows += t;
        max_t = std::max(max_t, t);
    }
    if (rows > a->max_rows) return fail("clips exceed the audio batch capacity");
    if (a->busy) {
        // host staging refilled once the previous call's copies are done; device buffers reused in stream order
        if (cudaEventSynchronize(a->staged) != cudaSuccess || cudaStreamWaitEvent(st, a->done, 0) != cudaSuccess)
            return fail("event sync failed");
        a->busy = false;
    }
    a->host_offs[0] = 0;
    for (int c = 0; c < n_clips; c++) a->host_offs[c + 1] = a->host_offs[c] + audio_out_len(valid[c]);
    if (cudaMemcpyAsync(a->offs, a->host_offs, (size_t)(n_clips + 1) * 4, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return fail("audio upload failed");
    return rows;
}

int audio_encode_core(D1Audio* a, int n_clips, const int* valid, const float* const* melc_dev, int rows, int max_t,
                      float* out, cudaStream_t st);

}  // namespace

extern "C" {

int d1h_audio_encode(D1Audio* a, int n_clips, const int* valid, const float* mel, float* out, cudaStream_t st) {
    if (!a || n_clips <= 0 || n_clips > 4095 || !valid || !mel || !out) return fail("bad arguments");
    int max_t = 0;
    const int rows = audio_prepare(a, n_clips, valid, max_t, st);
    if (rows < 0) return rows;
    long long frames = 0;
    for (int c = 0; c < n_clips; c++) frames += valid[c];
    if (frames > a->mel_rows) return fail("clips exceed the audio batch capacity");
    memcpy(a->host_mel, mel, (size_t)frames * N_MELS * 4);
    if (cudaMemcpyAsync(a->mel, a->host_mel, (size_t)frames * N_MELS * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaEventRecord(a->staged, st) != cudaSuccess)
        return fail("audio upload failed");
    std::vector<const float*> mp(n_clips);
    const float* p = a->mel;
    for (int c = 0; c < n_clips; c++) {
        mp[c] = p;
        p += (size_t)valid[c] * N_MELS;
    }
    return audio_encode_core(a, n_clips, valid, mp.data(), rows, max_t, out, st);
}

int d1h_audio_encode_pcm(D1Audio* a, int n_clips, const int* n_samples, const float* pcm, float* out, int* valid_out,
                         cudaStream_t st) {
    return d1h_audio_encode_pcm_rates(a, n_clips, n_samples, nullptr, pcm, out, valid_out, st);
}

int d1h_audio_encode_pcm_rates(D1Audio* a, int n_clips, const int* n_samples, const int* rates, const float* pcm,
                               float* out, int* valid_out, cudaStream_t st) {
    if (!a || n_clips <= 0 || n_clips > 4095 || !n_samples || !pcm || !out) return fail("bad arguments");
    // a clip at another rate: the WAV decoder keeps at most 30 s + 1 s of it (src/audio.rs:59), resample() takes it
    // to 16 kHz (:108-148); then, as for 16 kHz input, src/audio.rs:238-247: at most 30 s, zero-padded to at least
    // 0.5 s; valid = n / 160 frames
    std::vector<int> valid(n_clips), used(n_clips), rate(n_clips), src_n(n_clips, 0);
    size_t total = 0, frames = 0, src_total = 0, rs_max = 0;
    for (int c = 0; c < n_clips; c++) {
        if (n_samples[c] < 0) return fail("negative sample count");
        rate[c] = rates && rates[c] ? rates[c] : 16000;
        if (rate[c] <= 0) return fail("sample rate must be positive");
        int len16 = n_samples[c];
        if (rate[c] != 16000) {
            src_n[c] = (int)std::min<long long>(n_samples[c], 31ll * rate[c]);
            len16 = d1_resample_len(src_n[c], rate[c], 16000);
            if (len16 < 0) return fail("unsupported sample rate");
            src_total += (size_t)src_n[c];
            rs_max = std::max(rs_max, (size_t)len16);
        }
        used[c] = std::min(len16, A_MAX_SAMPLES);
        const int n = std::max(used[c], A_MIN_SAMPLES);
        valid[c] = n / 160;
        total += (size_t)n;
        frames += (size_t)valid[c] + 1;
    }
    if ((long long)frames > a->mel_rows) return fail("clips exceed the audio batch capacity");
    int max_t = 0;
    const int rows = audio_prepare(a, n_clips, valid.data(), max_t, st);
    if (rows < 0) return rows;
    if (total > a->pcm_cap) return fail("clips exceed the audio waveform staging capacity");
    if (src_total > a->src_cap || rs_max > a->rs_cap) {  // grow the resampling buffers (rare): nothing may use them
        if (cudaStreamSynchronize(st) != cudaSuccess) return fail("stream sync failed");
        if (src_total > a->src_cap) {
            if (a->src) cudaFree(a->src);
            if (a->host_src) cudaFreeHost(a->host_src);
            a->src = nullptr;
            a->host_src = nullptr;
            a->src_cap = 0;
            if (dmalloc(&a->src, src_total * 4) ||
                cudaMallocHost((void**)&a->host_src, src_total * 4) != cudaSuccess)
                return fail("resampler staging allocation failed");
            a->src_cap = src_total;
        }
        if (rs_max > a->rs_cap) {
            if (a->rs) cudaFree(a->rs);
            a->rs = nullptr;
            a->rs_cap = 0;
            if (dmalloc(&a->rs, rs_max * 4)) return fail("resampler buffer allocation failed");
            a->rs_cap = rs_max;
        }
    }
    // stage every 16 kHz clip (cut, zero-padded) in pinned memory, and the other clips at their own rates; one
    // copy each, then per clip the resampler (other rates) and the front end
    const float* sp = pcm;
    size_t off = 0, soff = 0;
    for (int c = 0; c < n_clips; c++) {
        const int n = std::max(used[c], A_MIN_SAMPLES);
        if (rate[c] == 16000) {
            memcpy(a->host_pcm + off, sp, (size_t)used[c] * 4);
            if (n > used[c]) memset(a->host_pcm + off + used[c], 0, (size_t)(n - used[c]) * 4);
        } else {
            memcpy(a->host_src + soff, sp, (size_t)src_n[c] * 4);
            soff += (size_t)src_n[c];
        }
        sp += n_samples[c];
        off += (size_t)n;
    }
    if (cudaMemcpyAsync(a->pcm, a->host_pcm, total * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        (src_total && cudaMemcpyAsync(a->src, a->host_src, src_total * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) ||
        cudaEventRecord(a->staged, st) != cudaSuccess)
        return fail("audio upload failed");
    std::vector<const float*> mp(n_clips);
    off = 0;
    soff = 0;
    size_t moff = 0;
    for (int c = 0; c < n_clips; c++) {
        const int n = std::max(used[c], A_MIN_SAMPLES);
        if (rate[c] != 16000) {
            a->launches++;
            if (d1_resample(a->src + soff, src_n[c], rate[c], 16000, a->rs, st) ||
                (used[c] && cudaMemcpyAsync(a->pcm + off, a->rs, (size_t)used[c] * 4, cudaMemcpyDeviceToDevice, st)) ||
                (n > used[c] && cudaMemsetAsync(a->pcm + off + used[c], 0, (size_t)(n - used[c]) * 4, st)))
                return fail("resampling failed");
            soff += (size_t)src_n[c];
        }
        a->launches += 2;
        if (d1_log_mel(a->pcm + off, n, a->mel + moff * N_MELS, st)) return fail("log-mel front end failed");
        mp[c] = a->mel + moff * N_MELS;
        off += (size_t)n;
        moff += (size_t)valid[c] + 1;
        if (valid_out) valid_out[c] = valid[c];
    }
    return audio_encode_core(a, n_clips, valid.data(), mp.data(), rows, max_t, out, st);
}

}  // extern "C"

namespace {

int audio_encode_core(D1Audio* a, int n_clips, const int* valid, const float* const* melc_dev, int rows, int max_t,
                      float* out, cudaStream_t st) {
    long long& L = a->launches;
    const D1AudioWeights& w = a->w;
    const bool fz = a->fused;
    // fp32 pointwise GEMM of the subsampling with bias (+ReLU), fused or in the reference's three calls
    auto sgemm_ba = [&](int m, int n, int k, const float* x, const float* wt, float* y, const float* b, int act) -> int {
        if (fz) {
            L++;
            return d1_sgemm(m, n, k, x, k, wt, k, y, n, 0.f, b, act, st);
        }
        L += 3;
        int r = d1_fill_rows(y, b, nullptr, m, n, st);
        if (!r) r = d1_sgemm(m, n, k, x, k, wt, k, y, n, 1.f, nullptr, 0, st);
        if (!r && act) r = d1_bias_act_f(y, nullptr, m, n, act, st);
        return r;
    };
    // ---- subsampling per clip (src/audio.rs:511-525) into rows offs[c] .. of x
    for (int c = 0; c < n_clips; c++) {
        const int v = valid[c], l1 = (v - 1) / 2 + 1, l2 = (l1 - 1) / 2 + 1, t = audio_out_len(v);
        if (fz) {  // conv0 + the first depthwise conv in one kernel, the conv0 rows kept on chip
            L += 2;
            CK(d1_sub_conv01(melc_dev[c], v, N_MELS, w.c0_w, w.c0_b, w.c2_w, w.c2_b, a->s2, l1, l2, st));
        } else {
            L += 3;
            CK(d1_sub_conv0(melc_dev[c], v, N_MELS, w.c0_w, w.c0_b, a->s1, l1, 64, st));
            CK(d1_sub_dwconv(a->s1, l1, 64, w.c2_w, w.c2_b, a->s2, l2, 32, st));
        }
        CK(sgemm_ba(l2 * 32, SUB_C, SUB_C, a->s2, w.c3_w, a->s3, w.c3_b, 1));
        CK(d1_sub_dwconv(a->s3, l2, 32, w.c5_w, w.c5_b, a->s2, t, 16, st));
        CK(sgemm_ba(t * 16, SUB_C, SUB_C, a->s2, w.c6_w, a->s1, w.c6_b, 1));
        CK(sgemm_ba(t, AD, 16 * SUB_C, a->s1, w.pre_out, a->x + (size_t)a->host_offs[c] * AD, w.pre_out_b, 0));
    }
    // ---- conformer layers over all rows (src/audio.rs:561-588)
    const int R = rows;
    float* x = a->x;
    d1_half *xn = a->xn, *big = a->big, *o = a->o;
    auto ln = [&](float* xx, const float* pb, float ps, const float* g, const float* b, d1_half* y, float* yf,
                  int d) -> int {
        L++;
        return d1_layernorm(xx, pb, ps, g, b, y, yf, R, d, w.eps, st);
    };
    auto gemm_h = [&](int n, int k, const d1_half* in, const d1_half* wt, d1_half* y, const float* b, int act) -> int {
        if (fz && b) {
            L++;
            return d1_gemm_bias_act(a->lt, R, n, k, in, k, wt, k, b, act, y, n, st);
        }
        L++;
        int r = d1_lt_gemm(a->lt, R, n, k, in, k, wt, k, 0, y, n, 0, 0, 1.f, 0.f, st);
        if (!r && b) {
            L++;
            r = d1_bias_act_h(y, b, R, n, act, st);
        }
        return r;
    };
    auto gemm_add = [&](int n, int k, const d1_half* in, const d1_half* wt, float* y, float alpha) -> int {
        L++;
        return d1_lt_gemm(a->lt, R, n, k, in, k, wt, k, 0, y, n, 1, 0, alpha, 1.f, st);
    };
    const int ff = 4 * AD;
    for (size_t li = 0; li < a->layers.size(); li++) {
        const D1AudioLayer& l = a->layers[li];
        // FF1 half step (pending bias of the previous layer's norm_out is none: it replaced x)
        CK(ln(x, nullptr, 1.f, l.ff1_n_w, l.ff1_n_b, xn, nullptr, AD));
        CK(gemm_h(ff, AD, xn, l.ff1_up, big, l.ff1_up_b, 4));
        CK(gemm_add(AD, ff, big, l.ff1_down, x, 0.5f));
        // rel-pos self-attention
        CK(ln(x, l.ff1_down_b, 0.5f, l.att_n_w, l.att_n_b, xn, nullptr, AD));
        CK(gemm_h(3 * AD, AD, xn, l.qkv, big, nullptr, 0));
        L += 2;
        CK(d1_relpos_prep(big, l.bq, l.bk, l.bv, l.pu, l.pv, a->qu, a->qv, a->kk, a->vv, R, AD, st));
        CK(d1_relpos_attn(a->qu, a->qv, a->kk, a->vv, AD, a->pp + li * PP_ROWS * AD, AD, PP_ROWS, PP_CENTER, o, AD,
                          a->offs, n_clips, max_t, AHEADS, 0.125f, st));
        CK(gemm_add(AD, AD, o, l.out, x, 1.f));
        // conv module: pw1 -> GLU / depthwise 9 / BN / SiLU (per clip: zero padding at the clip's edges) -> pw2
        CK(ln(x, l.out_b, 1.f, l.conv_n_w, l.conv_n_b, xn, nullptr, AD));
        CK(gemm_h(2 * AD, AD, xn, l.pw1, big, nullptr, 0));
        if (fz) {  // every clip in one launch, each zero-padded at its own edges
            L++;
            CK(d1_conformer_dw_clips(big, l.pw1_b, l.dw, l.dw_b, l.bn_s, l.bn_b, o, a->offs, n_clips, R, AD, 9, st));
        } else {
            for (int c = 0; c < n_clips; c++) {
                const int s = a->host_offs[c], t = a->host_offs[c + 1] - s;
                L++;
                CK(d1_conformer_dw(big + (size_t)s * 2 * AD, l.pw1_b, l.dw, l.dw_b, l.bn_s, l.bn_b,
                                   o + (size_t)s * AD, t, AD, 9, st));
            }
        }
        CK(gemm_add(AD, AD, o, l.pw2, x, 1.f));
        // FF2 half step
        CK(ln(x, l.pw2_b, 1.f, l.ff2_n_w, l.ff2_n_b, xn, nullptr, AD));
        CK(gemm_h(ff, AD, xn, l.ff2_up, big, l.ff2_up_b, 4));
        CK(gemm_add(AD, ff, big, l.ff2_down, x, 0.5f));
        // norm_out replaces the residual stream
        CK(ln(x, l.ff2_down_b, 0.5f, l.out_n_w, l.out_n_b, nullptr, x, AD));
    }
    // ---- adapter (src/audio.rs:589-593): LN -> Linear -> GELU -> Linear, then a + up(GELU(down(LN(a))))
    CK(ln(x, nullptr, 1.f, w.ad_n_w, w.ad_n_b, xn, nullptr, AD));
    CK(gemm_h(AOUT, AD, xn, w.ad1, big, w.ad1_b, 2));
    L++;
    CK(d1_fill_rows(out, w.ad2_b, nullptr, R, AOUT, st));
    CK(gemm_add(AOUT, AOUT, big, w.ad2, out, 1.f));
    CK(ln(out, nullptr, 1.f, w.res_n_w, w.res_n_b, xn, nullptr, AOUT));
    CK(gemm_h(AD, AOUT, xn, w.res_down, big, w.res_down_b, 2));
    CK(gemm_add(AOUT, AD, big, w.res_up, out, 1.f));
    L++;
    CK(d1_bias_act_f(out, w.res_up_b, R, AOUT, 0, st));
    cudaEventRecord(a->done, st);
    a->busy = true;
    return R;
}

}  // namespace

extern "C" {

int d1h_vision_capacity(const D1Vision* v) { return v ? v->max_patches : 0; }

int d1h_model_layers(const D1Model* m, int is_attn) {
    if (!m) return 0;
    int n = 0;
    for (const auto& l : m->layers) n += (l.is_attn != 0) == (is_attn != 0);
    return n;
}

void* d1h_gemm_ctx(D1Model* m) { return m ? m->lt : nullptr; }

int d1h_set_tune_effort(D1Model* m, int effort) {
    if (!m || effort < 0 || effort > 2) return -1;
    m->tune_effort = effort;
    return 0;
}

}  // extern "C"
