// HBM-bound kernels of the d1rs forward pass for sm_100a: norms, the double-gated short convolution, QK-norm +
// RoPE, the elementwise glue and the vision/audio pieces. Each replaces the launcher of the same name in the
// reference's cuda/kernels.cu (cited per function) with the same arguments and arithmetic; the data movement is
// re-planned for B200 (16-byte vector accesses, a warp or a rolling register window per row, grids sized to the
// work and capped at a whole number of waves).
#include "common.cuh"

using namespace d1;

namespace {

inline int nblk(size_t n, int t) { return (int)((n + t - 1) / t); }

// Grid for grid-stride elementwise loops: enough CTAs to fill every SM several times over, never more than the
// work needs.
inline int egrid(size_t n_items, int threads) {
    size_t b = (n_items + threads - 1) / threads;
    const size_t cap = 148 * 16;
    return (int)(b > cap ? cap : (b < 1 ? 1 : b));
}

__device__ __forceinline__ void h8_to_f(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

__device__ __forceinline__ uint32_t h2u(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint4 f_to_h8(const float* f) {
    return make_uint4(h2u(f[0], f[1]), h2u(f[2], f[3]), h2u(f[4], f[5]), h2u(f[6], f[7]));
}

// ------------------------------------------------------------------------------------------------ norms
// One warp per row; lane l holds the float4 groups l, l+32, ... (NV = D / 128 of them).

template <int NV>
__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w,
                                                 __half* __restrict__ y, int rows, float eps) {
    pdl_entry();
    constexpr int D = NV * 128;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * D);
    float4 v[NV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        v[i] = __ldg(xr + lane + 32 * i);  // h stays in L2 for the next residual GEMM
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    const float r = rsqrtf(warp_sum(ss) / D + eps);
    const float4* w4 = reinterpret_cast<const float4*>(w);
    uint2* yr = reinterpret_cast<uint2*>(y + (size_t)row * D);
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float4 g = __ldg(w4 + lane + 32 * i);
        yr[lane + 32 * i] = make_uint2(h2u(v[i].x * r * g.x, v[i].y * r * g.y), h2u(v[i].z * r * g.z, v[i].w * r * g.w));
    }
}

// x += s * pend (written back), then LayerNorm to fp16 y and/or fp32 yf (yf may alias x).
template <int NV>
__global__ void __launch_bounds__(256) k_layernorm(float* x, const float* __restrict__ pend, float pend_scale,
                                                   const float* __restrict__ w, const float* __restrict__ b,
                                                   __half* __restrict__ y, float* yf,
                                                   const int* __restrict__ y_rows, int rows, float eps) {
    pdl_entry();
    constexpr int D = NV * 128;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float4* xr = reinterpret_cast<float4*>(x + (size_t)row * D);
    float4 v[NV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        v[i] = xr[lane + 32 * i];
        if (pend) {
            const float4 p = __ldg(reinterpret_cast<const float4*>(pend) + lane + 32 * i);
            v[i].x += pend_scale * p.x;
            v[i].y += pend_scale * p.y;
            v[i].z += pend_scale * p.z;
            v[i].w += pend_scale * p.w;
            xr[lane + 32 * i] = v[i];
        }
        s += v[i].x + v[i].y + v[i].z + v[i].w;
    }
    const float mean = warp_sum(s) / D;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
        ss += a * a + bb * bb + c * c + d * d;
    }
    const float r = rsqrtf(warp_sum(ss) / D + eps);
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(w) + lane + 32 * i);
        const float4 bb = __ldg(reinterpret_cast<const float4*>(b) + lane + 32 * i);
        float4 o;
        o.x = (v[i].x - mean) * r * g.x + bb.x;
        o.y = (v[i].y - mean) * r * g.y + bb.y;
        o.z = (v[i].z - mean) * r * g.z + bb.z;
        o.w = (v[i].w - mean) * r * g.w + bb.w;
        if (y) {
            const size_t yr = y_rows ? (size_t)__ldg(y_rows + row) : (size_t)row;
            reinterpret_cast<uint2*>(y + yr * D)[lane + 32 * i] = make_uint2(h2u(o.x, o.y), h2u(o.z, o.w));
        }
        if (yf) reinterpret_cast<float4*>(yf + (size_t)row * D)[lane + 32 * i] = o;
    }
}

// out = RMSNorm(h) * w + type_emb[qtype of the row's sequence], D = 1024 (out may alias h).
__global__ void __launch_bounds__(256) k_head_init(const float* h, const float* __restrict__ w,
                                                   const float* __restrict__ type_emb, const int* __restrict__ tok_seq,
                                                   const SeqInfo* __restrict__ seqs, float* out, int rows, float eps) {
    pdl_entry();
    constexpr int NV = 8, D = 1024;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float4* xr = reinterpret_cast<const float4*>(h + (size_t)row * D);
    const float4* te = reinterpret_cast<const float4*>(type_emb + (size_t)seqs[tok_seq[row]].qtype * D);
    float4 v[NV];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; i++) {
        v[i] = xr[lane + 32 * i];
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    const float r = rsqrtf(warp_sum(ss) / D + eps);
    float4* o = reinterpret_cast<float4*>(out + (size_t)row * D);
#pragma unroll
    for (int i = 0; i < NV; i++) {
        const float4 g = __ldg(reinterpret_cast<const float4*>(w) + lane + 32 * i), t = __ldg(te + lane + 32 * i);
        o[lane + 32 * i] = make_float4(v[i].x * r * g.x + t.x, v[i].y * r * g.y + t.y, v[i].z * r * g.z + t.z,
                                       v[i].w * r * g.w + t.w);
    }
}

// ------------------------------------------------------------------------------------------------ elementwise

// h[row] = table[ids[row]] (fp16 -> fp32); a warp per row, 8 halves per access.
__global__ void __launch_bounds__(256) k_embed(const __half* __restrict__ table, const int* __restrict__ ids,
                                               float* __restrict__ h, int rows, int D) {
    pdl_entry();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const uint4* src = reinterpret_cast<const uint4*>(table + (size_t)ids[row] * D);
    float4* dst = reinterpret_cast<float4*>(h + (size_t)row * D);
    for (int c = lane; c < D / 8; c += 32) {
        float f[8];
        h8_to_f(__ldg(src + c), f);
        dst[2 * c] = make_float4(f[0], f[1], f[2], f[3]);
        dst[2 * c + 1] = make_float4(f[4], f[5], f[6], f[7]);
    }
}

__global__ void k_embed_scalar(const __half* __restrict__ table, const int* __restrict__ ids, float* __restrict__ h,
                               int rows, int D) {
    pdl_entry();
    const int row = blockIdx.x;
    for (int c = threadIdx.x; c < D; c += blockDim.x) h[(size_t)row * D + c] = __half2float(table[(size_t)ids[row] * D + c]);
}

// out[t][i] = silu(gu[t][i]) * gu[t][F + i], 8 columns per step (F % 8 == 0).
__global__ void k_swiglu8(const __half* __restrict__ gu, __half* __restrict__ out, int rows, int F) {
    pdl_entry();
    const int f8 = F / 8;
    const size_t n = (size_t)rows * f8;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t r = idx / f8;
        const int c = (int)(idx % f8) * 8;
        float g[8], u[8], o[8];
        h8_to_f(__ldcs(reinterpret_cast<const uint4*>(gu + r * 2 * F + c)), g);
        h8_to_f(__ldcs(reinterpret_cast<const uint4*>(gu + r * 2 * F + F + c)), u);
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = silu(g[i]) * u[i];
        *reinterpret_cast<uint4*>(out + r * F + c) = f_to_h8(o);
    }
}

__global__ void k_swiglu_scalar(const __half* __restrict__ gu, __half* __restrict__ out, int rows, int F) {
    pdl_entry();
    const size_t n = (size_t)rows * F;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const size_t r = idx / F;
        const int c = (int)(idx % F);
        out[idx] = __float2half_rn(silu(__half2float(gu[r * 2 * F + c])) * __half2float(gu[r * 2 * F + F + c]));
    }
}

// x = act(x + bias), fp16 in place, 8 columns per step (N % 8 == 0).
__global__ void k_bias_act_h8(__half* __restrict__ x, const float* __restrict__ bias, int rows, int N, int act) {
    pdl_entry();
    const int n8 = N / 8;
    const size_t n = (size_t)rows * n8;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % n8) * 8;
        uint4* p = reinterpret_cast<uint4*>(x) + idx;
        float f[8];
        h8_to_f(*p, f);
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = apply_act(f[i] + (bias ? __ldg(bias + c + i) : 0.f), act);
        *p = f_to_h8(f);
    }
}

__global__ void k_bias_act_h_scalar(__half* __restrict__ x, const float* __restrict__ bias, int rows, int N, int act) {
    pdl_entry();
    const size_t n = (size_t)rows * N;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % N);
        x[idx] = __float2half_rn(apply_act(__half2float(x[idx]) + (bias ? bias[c] : 0.f), act));
    }
}

// x = act(x + bias), fp32 in place.
__global__ void k_bias_act_f(float* __restrict__ x, const float* __restrict__ bias, int rows, int N, int act) {
    pdl_entry();
    const size_t n = (size_t)rows * N;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % N);
        x[idx] = apply_act(x[idx] + (bias ? bias[c] : 0.f), act);
    }
}

// out[t][i] = bias[i] (+ add[t][i]).
__global__ void k_fill_rows(float* __restrict__ out, const float* __restrict__ bias, const float* __restrict__ add,
                            int rows, int N) {
    pdl_entry();
    const size_t n = (size_t)rows * N;
    for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < n; idx += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % N);
        float v = bias ? bias[c] : 0.f;
        if (add) v += add[idx];
        out[idx] = v;
    }
}

__global__ void k_f32_to_f16(const float* __restrict__ x, __half* __restrict__ y, size_t n) {
    pdl_entry();
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        y[i] = __float2half(x[i]);
}

// dst[i] = src[idx[i]]: a warp per row of width16 x 16 bytes.
__global__ void __launch_bounds__(256) k_gather_rows(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                                     const int* __restrict__ idx, int n, int width16) {
    pdl_entry();
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= n) return;
    const uint4* s = src + (size_t)idx[r] * width16;
    uint4* d = dst + (size_t)r * width16;
    for (int c = lane; c < width16; c += 32) d[c] = s[c];
}

// ------------------------------------------------------------------------------------------------ short conv
// bcu [T][3D] = [b | c | u]. Each CTA covers kConvRows consecutive rows; a thread owns 8 channels. All of the
// thread's loads (b and u of rows t0-1 .. t0+kConvRows, c of its rows: 10 independent 16-byte loads) are issued
// before any arithmetic. Two rows per CTA keep the thread's registers few (many CTAs resident per SM) and the CTAs
// short, so the last partial wave of CTAs costs little; the one-row halo each side is an L2 hit (the neighbouring
// CTAs read those rows at the same time), so DRAM sees each row once. Sequence boundaries, the prefix's left state
// (ext_bx) and the saved last state (save_bx) follow cuda/kernels.cu:224-259.
constexpr int kConvRows = 2;

__device__ __forceinline__ void mul8(const uint4& b, const uint4& u, float* bx) {
    float fb[8], fu[8];
    h8_to_f(b, fb);
    h8_to_f(u, fu);
#pragma unroll
    for (int i = 0; i < 8; i++) bx[i] = fb[i] * fu[i];
}

__global__ void __launch_bounds__(128) k_shortconv(const __half* __restrict__ bcu, const float* __restrict__ convw,
                                                   const int* __restrict__ tok_seq, const SeqInfo* __restrict__ seqs,
                                                   __half* __restrict__ out, int rows, int D, int conv_idx) {
    pdl_entry();
    const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
    if (c >= D) return;
    const int t0 = blockIdx.x * kConvRows;
    const size_t ld = (size_t)3 * D;
    uint4 rb[kConvRows + 2], ru[kConvRows + 2], rc[kConvRows];
    int sq[kConvRows];
#pragma unroll
    for (int j = 0; j < kConvRows + 2; j++) {
        const int t = min(max(t0 - 1 + j, 0), rows - 1);
        rb[j] = __ldg(reinterpret_cast<const uint4*>(bcu + t * ld + c));
        ru[j] = __ldg(reinterpret_cast<const uint4*>(bcu + t * ld + 2 * D + c));
    }
#pragma unroll
    for (int j = 0; j < kConvRows; j++) {
        const int t = min(t0 + j, rows - 1);
        rc[j] = __ldg(reinterpret_cast<const uint4*>(bcu + t * ld + D + c));
        sq[j] = __ldg(tok_seq + t);
    }
    float w0[8], w1[8], w2[8];
    {
        const float4* w4 = reinterpret_cast<const float4*>(convw + (size_t)c * 3);  // 24 consecutive floats
        float wf[24];
#pragma unroll
        for (int i = 0; i < 6; i++) {
            const float4 q = __ldg(w4 + i);
            wf[4 * i] = q.x;
            wf[4 * i + 1] = q.y;
            wf[4 * i + 2] = q.z;
            wf[4 * i + 3] = q.w;
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            w0[i] = wf[3 * i];
            w1[i] = wf[3 * i + 1];
            w2[i] = wf[3 * i + 2];
        }
    }
#pragma unroll
    for (int j = 0; j < kConvRows; j++) {
        const int t = t0 + j;
        if (t >= rows) break;
        const SeqInfo& s = seqs[sq[j]];
        const int local = t - s.start;
        const bool has_left = local > 0, has_right = local + 1 < s.len;
        float cur[8], l[8], r[8], cc[8], y[8];
        mul8(rb[j + 1], ru[j + 1], cur);
        if (has_left) {
            mul8(rb[j], ru[j], l);
        } else if (s.ext_bx) {
            h8_to_f(*reinterpret_cast<const uint4*>(s.ext_bx + (size_t)conv_idx * D + c), l);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) l[i] = 0.f;
        }
        if (has_right) {
            mul8(rb[j + 2], ru[j + 2], r);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) r[i] = 0.f;
            if (s.save_bx) *reinterpret_cast<uint4*>(s.save_bx + (size_t)conv_idx * D + c) = f_to_h8(cur);
        }
        h8_to_f(rc[j], cc);
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = cc[i] * (w0[i] * l[i] + w1[i] * cur[i] + w2[i] * r[i]);
        *reinterpret_cast<uint4*>(out + (size_t)t * D + c) = f_to_h8(y);
    }
}

// ------------------------------------------------------------------------------------------------ QK norm + RoPE
// qkv row = [q (H*64) | k (KVH*64) | v (KVH*64)], in place. Half a warp per 64-wide head vector: lane j of the
// half holds dims (2j, 2j+1) and (2j+32, 2j+33), i.e. both halves of the rotate-half pairs (l, l+32), l = 2j, 2j+1
// (cuda/kernels.cu:263-303).
// QK-norm + RoPE with 16-byte accesses, one warp per row: 8 lanes per 64-element head vector (lane k of a group holds
// elements 8k .. 8k+7, so the rotate-half partner of element e, e ^ 32, sits in lane k ^ 4 of the same group); the
// warp's 4 groups walk the row's H query and KVH key heads with every head load issued up front, and share the
// row's sequence lookup and RoPE (cos, sin) values. The KVH value heads are copied to the prefix cache when the
// sequence saves one. Needs 16-byte aligned rows and H + KVH <= 32; d1_qk_norm_rope falls back to k_qk_norm_rope
// otherwise.
constexpr int kQkMaxPerGroup = 8;  // (H + KVH) / 4 heads per group at most

__global__ void __launch_bounds__(256) k_qk_norm_rope8(__half* __restrict__ qkv, int ld, int H, int KVH,
                                                       const float* __restrict__ qn, const float* __restrict__ kn,
                                                       const float* __restrict__ rope,
                                                       const int* __restrict__ tok_seq,
                                                       const SeqInfo* __restrict__ seqs, int attn_idx, int rows,
                                                       float eps) {
    pdl_entry();
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= rows) return;  // whole warps leave together
    const int lane = threadIdx.x & 31, grp = lane >> 3, k = lane & 7;
    const int nh = H + KVH;
    uint4* row = reinterpret_cast<uint4*>(qkv + (size_t)t * ld);
    uint4 raw[kQkMaxPerGroup];
#pragma unroll
    for (int j = 0; j < kQkMaxPerGroup; j++) {
        const int u = grp + 4 * j;
        raw[j] = u < nh ? row[u * 8 + k] : make_uint4(0, 0, 0, 0);
    }
    const SeqInfo s = seqs[__ldg(tok_seq + t)];
    const int local = t - s.start, pos = local + s.pos_off;
    float cs[16];  // (cos, sin) of pairs 8(k & 3) .. +7 at this position
    const float4* cs4 = reinterpret_cast<const float4*>(rope + ((size_t)pos * 32 + 8 * (k & 3)) * 2);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 c = __ldg(cs4 + i);
        cs[4 * i] = c.x;
        cs[4 * i + 1] = c.y;
        cs[4 * i + 2] = c.z;
        cs[4 * i + 3] = c.w;
    }
#pragma unroll
    for (int j = 0; j < kQkMaxPerGroup; j++) {
        const int u = grp + 4 * j;
        if (4 * j >= nh) break;  // uniform across the warp
        const bool active = u < nh, isq = u < H;
        const __half2* h2 = reinterpret_cast<const __half2*>(&raw[j]);
        float x[8];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 f = __half22float2(h2[i]);
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
        }
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) ss += x[i] * x[i];
        ss += __shfl_xor_sync(D1_FULL_MASK, ss, 1);
        ss += __shfl_xor_sync(D1_FULL_MASK, ss, 2);
        ss += __shfl_xor_sync(D1_FULL_MASK, ss, 4);
        const float r = rsqrtf(ss / 64.f + eps);
        const float* w = (isq ? qn : kn) + 8 * k;
        float y[8], q[8];
#pragma unroll
        for (int i = 0; i < 8; i++) y[i] = active ? x[i] * r * __ldg(w + i) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) q[i] = __shfl_xor_sync(D1_FULL_MASK, y[i], 4);
        if (!active) continue;
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            if (k < 4) {  // first half: a = own value, b = partner
                o[i] = y[i] * cs[2 * i] - q[i] * cs[2 * i + 1];
                o[i + 1] = y[i + 1] * cs[2 * i + 2] - q[i + 1] * cs[2 * i + 3];
            } else {      // second half: b = own value, a = partner
                o[i] = y[i] * cs[2 * i] + q[i] * cs[2 * i + 1];
                o[i + 1] = y[i + 1] * cs[2 * i + 2] + q[i + 1] * cs[2 * i + 3];
            }
        }
        uint4 out;
        __half2* oh = reinterpret_cast<__half2*>(&out);
#pragma unroll
        for (int i = 0; i < 4; i++) oh[i] = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
        row[u * 8 + k] = out;
        if (!isq && s.save_k)
            reinterpret_cast<uint4*>(s.save_k + ((size_t)attn_idx * s.len + local) * (KVH * 64) + (u - H) * 64)[k] = out;
    }
    if (s.save_v)  // raw V heads into the prefix cache
        for (int g = grp; g < KVH; g += 4)
            reinterpret_cast<uint4*>(s.save_v + ((size_t)attn_idx * s.len + local) * (KVH * 64) + g * 64)[k] =
                row[(nh + g) * 8 + k];
}

__global__ void __launch_bounds__(256) k_qk_norm_rope(__half* __restrict__ qkv, int ld, int H, int KVH,
                                                      const float* __restrict__ qn, const float* __restrict__ kn,
                                                      const float* __restrict__ rope, const int* __restrict__ tok_seq,
                                                      const SeqInfo* __restrict__ seqs, int attn_idx, int rows,
                                                      float eps) {
    pdl_entry();
    const int t = blockIdx.x;
    const int half_id = threadIdx.x >> 4, j = threadIdx.x & 15;
    const SeqInfo s = seqs[tok_seq[t]];
    const int local = t - s.start;
    const int pos = local + s.pos_off;
    const float4 cs = __ldg(reinterpret_cast<const float4*>(rope + ((size_t)pos * 32 + 2 * j) * 2));  // (c0,s0,c1,s1)
    __half* row = qkv + (size_t)t * ld;
    const int units = H + KVH + (s.save_v ? KVH : 0);
    for (int u = half_id; u < (units + 1) / 2 * 2; u += blockDim.x / 16) {
        const bool active = u < units;
        if (active && u >= H + KVH) {  // raw V into the prefix cache
            const int g = u - H - KVH;
            const __half2* src = reinterpret_cast<const __half2*>(row + (H + KVH) * 64 + g * 64);
            __half2* dst = reinterpret_cast<__half2*>(s.save_v + ((size_t)attn_idx * s.len + local) * (KVH * 64) + g * 64);
            dst[j] = src[j];
            dst[j + 16] = src[j + 16];
        }
        const bool norm = active && u < H + KVH;
        float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
        __half2* p = reinterpret_cast<__half2*>(row + (norm ? u : 0) * 64);
        if (norm) {
            a = __half22float2(p[j]);
            b = __half22float2(p[j + 16]);
        }
        float ss = a.x * a.x + b.x * b.x + a.y * a.y + b.y * b.y;
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(D1_FULL_MASK, ss, o);
        if (!norm) continue;
        const bool isq = u < H;
        const float* w = isq ? qn : kn;
        const float r = rsqrtf(ss / 64.f + eps);
        const float a0 = a.x * r * __ldg(w + 2 * j), a1 = a.y * r * __ldg(w + 2 * j + 1);
        const float b0 = b.x * r * __ldg(w + 2 * j + 32), b1 = b.y * r * __ldg(w + 2 * j + 33);
        const __half2 oa = __floats2half2_rn(a0 * cs.x - b0 * cs.y, a1 * cs.z - b1 * cs.w);
        const __half2 ob = __floats2half2_rn(b0 * cs.x + a0 * cs.y, b1 * cs.z + a1 * cs.w);
        p[j] = oa;
        p[j + 16] = ob;
        if (!isq && s.save_k) {
            const int g = u - H;
            __half2* dst = reinterpret_cast<__half2*>(s.save_k + ((size_t)attn_idx * s.len + local) * (KVH * 64) + g * 64);
            dst[j] = oa;
            dst[j + 16] = ob;
        }
    }
}

// ------------------------------------------------------------------------------------------------ decision scorer
// logit[r] = sum_i gelu_erf(x[r][i] + b1[i]) * w2[i] + b2; a warp per row, 8 columns per access (D % 256 == 0).
__global__ void __launch_bounds__(256) k_scorer_out(const __half* __restrict__ x, const float* __restrict__ b1,
                                                    const __half* __restrict__ w2, float b2, float* __restrict__ logits,
                                                    int rows, int D) {
    pdl_entry();
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    float s = 0.f;
    if (D % 256 == 0) {
        for (int c = lane * 8; c < D; c += 256) {
            float xv[8], wv[8];
            h8_to_f(*reinterpret_cast<const uint4*>(x + (size_t)row * D + c), xv);
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(w2 + c)), wv);
#pragma unroll
            for (int i = 0; i < 8; i++) s += gelu_erf(xv[i] + __ldg(b1 + c + i)) * wv[i];
        }
    } else {
        for (int c = lane; c < D; c += 32) s += gelu_erf(__half2float(x[(size_t)row * D + c]) + b1[c]) * __half2float(w2[c]);
    }
    s = warp_sum(s);
    if (lane == 0) logits[row] = s + b2;
}

// ------------------------------------------------------------------------------------------------ vision
// 2x2 pixel unshuffle x [ph*pw][C] -> out [(ph/2)*(pw/2)][4C] (cuda/kernels.cu:517-525), uint4 copies.
// Resized position embeddings of one crop (src/vision.rs:263-302, host code in the reference): the 16x16 grid of
// position vectors resampled to (ph, pw) by separable antialiased-bilinear taps — horizontal pass, then vertical
// pass, each a sum from zero of weight * value in tap order (fp32, multiply then add, as the reference's host
// loops) — plus the patch bias. spans: (first input index, taps) for the ph output rows then the pw output
// columns; w: their weights, `taps` per entry. One CTA per output patch row, threads over channels.
__global__ void __launch_bounds__(256) k_vision_pos(const float* __restrict__ grid, const float* __restrict__ bias,
                                                    const int2* __restrict__ spans, const float* __restrict__ w,
                                                    int taps, int ph, int pw, int C, float* __restrict__ out) {
    pdl_entry();
    const int p = blockIdx.x, y = p / pw, x = p % pw;
    const int2 sy = spans[y], sx = spans[ph + x];
    const float* wy = w + (size_t)y * taps;
    const float* wx = w + (size_t)(ph + x) * taps;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < sy.y; j++) {
            const float* row = grid + ((size_t)(sy.x + j) * 16 + sx.x) * C + c;
            float t = 0.f;
            for (int i = 0; i < sx.y; i++) t = __fadd_rn(t, __fmul_rn(__ldg(wx + i), __ldg(row + (size_t)i * C)));
            acc = __fadd_rn(acc, __fmul_rn(__ldg(wy + j), t));
        }
        out[(size_t)p * C + c] = __fadd_rn(acc, __ldg(bias + c));
    }
}

// 2x2 pixel unshuffle (cuda/kernels.cu:517-525) as a row permutation: viewed as [ph*pw][C], row 4*o + q of
// out [(ph/2)*(pw/2)][4C] is input row (2*(o / (pw/2)) + (q >> 1)) * pw + 2*(o % (pw/2)) + (q & 1). A flat grid
// over the 16-byte vectors of out, each thread computing its source vector: every load and store is a whole
// 16-byte vector and consecutive threads touch consecutive output bytes. (The runners fold the permutation into
// the post-LayerNorm's stores instead: d1_layernorm_rows.)
__global__ void __launch_bounds__(256) k_unshuffle16(const uint4* __restrict__ x, uint4* __restrict__ out, int pw,
                                                     int vpr, long long total) {
    pdl_entry();
    const int hw = pw >> 1;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / vpr;
        const int v = (int)(i - r * vpr), o = (int)(r >> 2), q = (int)(r & 3);
        const long long src = (long long)(2 * (o / hw) + (q >> 1)) * pw + 2 * (o % hw) + (q & 1);
        out[i] = __ldg(x + src * vpr + v);
    }
}

// ------------------------------------------------------------------------------------------------ audio
// The FastConformer subsampling (src/audio.rs:514-525): conv0 = 3x3 stride-2 conv 1 -> 256 channels + ReLU over the
// mel frames (cuda/kernels.cu:529-545), then 3x3 stride-2 depthwise convs (:548-564). Per output element both sum
// bias + w.x over the taps in (dt, df) order as fused multiply-adds, skipping taps outside the valid input — the
// reference's arithmetic, so the results are bit-identical. The data movement is this file's own:
//   k_sub_conv0_rows   one CTA per output time row, a thread per channel keeping its 9 weights in registers; the
//                      three mel rows it reads are staged once in shared memory and broadcast to all channels.
//   k_sub_conv01       conv0 and the first depthwise conv fused: a CTA per (output row of the depthwise conv,
//                      32-channel group) computes the three conv0 rows it needs into shared memory (never written
//                      to HBM) and convolves them there.
//   k_dw3s2_v4         the depthwise conv alone: a thread per (output position, 4 channels), 16-byte loads and
//                      stores, the 36 weights of its channels in registers.
constexpr int kSubC = 256;

__global__ void __launch_bounds__(256) k_sub_conv0_rows(const float* __restrict__ mel, int tin_valid, int F,
                                                        const float* __restrict__ w, const float* __restrict__ b,
                                                        float* __restrict__ out, int Fout) {
    extern __shared__ float rows3[];  // [3][F]
    pdl_entry();
    const int t = blockIdx.x, c = threadIdx.x;
    for (int i = threadIdx.x; i < 3 * F; i += blockDim.x) {
        const int ti = 2 * t - 1 + i / F;
        rows3[i] = (ti >= 0 && ti < tin_valid) ? mel[(size_t)ti * F + i % F] : 0.f;
    }
    float wc[9];
#pragma unroll
    for (int k = 0; k < 9; k++) wc[k] = __ldg(w + c * 9 + k);
    const float bc = __ldg(b + c);
    bool rv[3];
#pragma unroll
    for (int dt = 0; dt < 3; dt++) rv[dt] = 2 * t - 1 + dt >= 0 && 2 * t - 1 + dt < tin_valid;
    __syncthreads();
    for (int f = 0; f < Fout; f++) {
        float acc = bc;
#pragma unroll
        for (int dt = 0; dt < 3; dt++) {
            if (!rv[dt]) continue;
#pragma unroll
            for (int df = 0; df < 3; df++) {
                const int fi = 2 * f - 1 + df;
                if (fi >= 0 && fi < F) acc = __fmaf_rn(wc[dt * 3 + df], rows3[dt * F + fi], acc);
            }
        }
        out[((size_t)t * Fout + f) * kSubC + c] = fmaxf(acc, 0.f);
    }
}

constexpr int kSubGroup = 32;   // channels per CTA of the fused kernel
constexpr int kSubMaxF = 128;   // mel bins the fused kernel stages (the encoder's 128)
constexpr int kSubMaxF1 = 64;   // conv0 output bins: (kSubMaxF - 1) / 2 + 1

__global__ void __launch_bounds__(256) k_sub_conv01(const float* __restrict__ mel, int tin_valid, int F,
                                                    const float* __restrict__ w0, const float* __restrict__ b0,
                                                    const float* __restrict__ w1, const float* __restrict__ b1,
                                                    float* __restrict__ out, int l1, int F1, int F2) {
    __shared__ float m7[7][kSubMaxF];                  // mel rows 4*t2-3 .. 4*t2+3
    __shared__ float s1[3][kSubMaxF1][kSubGroup];      // conv0 rows 2*t2-1 .. 2*t2+1, this CTA's channels
    pdl_entry();
    const int t2 = blockIdx.x, c0 = blockIdx.y * kSubGroup;
    const int c = threadIdx.x & (kSubGroup - 1), g = threadIdx.x / kSubGroup, ng = blockDim.x / kSubGroup;
    for (int i = threadIdx.x; i < 7 * F; i += blockDim.x) {
        const int ti = 4 * t2 - 3 + i / F;
        m7[i / F][i % F] = (ti >= 0 && ti < tin_valid) ? mel[(size_t)ti * F + i % F] : 0.f;
    }
    float wa[9], wb[9];
#pragma unroll
    for (int k = 0; k < 9; k++) {
        wa[k] = __ldg(w0 + (c0 + c) * 9 + k);
        wb[k] = __ldg(w1 + (c0 + c) * 9 + k);
    }
    const float ba = __ldg(b0 + c0 + c), bb = __ldg(b1 + c0 + c);
    __syncthreads();
    // conv0 rows r = 2*t2 - 1 + j (those inside [0, l1)), mel row of tap dt: 2r - 1 + dt = 4*t2 - 3 + 2j + dt
    for (int j = 0; j < 3; j++) {
        const int r = 2 * t2 - 1 + j;
        if (r < 0 || r >= l1) continue;
        bool rv[3];
#pragma unroll
        for (int dt = 0; dt < 3; dt++) rv[dt] = 2 * r - 1 + dt >= 0 && 2 * r - 1 + dt < tin_valid;
        for (int f = g; f < F1; f += ng) {
            float acc = ba;
#pragma unroll
            for (int dt = 0; dt < 3; dt++) {
                if (!rv[dt]) continue;
#pragma unroll
                for (int df = 0; df < 3; df++) {
                    const int fi = 2 * f - 1 + df;
                    if (fi >= 0 && fi < F) acc = __fmaf_rn(wa[dt * 3 + df], m7[2 * j + dt][fi], acc);
                }
            }
            s1[j][f][c] = fmaxf(acc, 0.f);
        }
    }
    __syncthreads();
    bool rv[3];
#pragma unroll
    for (int dt = 0; dt < 3; dt++) rv[dt] = 2 * t2 - 1 + dt >= 0 && 2 * t2 - 1 + dt < l1;
    for (int f2 = g; f2 < F2; f2 += ng) {
        float acc = bb;
#pragma unroll
        for (int dt = 0; dt < 3; dt++) {
            if (!rv[dt]) continue;
#pragma unroll
            for (int df = 0; df < 3; df++) {
                const int fi = 2 * f2 - 1 + df;
                if (fi >= 0 && fi < F1) acc = __fmaf_rn(wb[dt * 3 + df], s1[dt][fi][c], acc);
            }
        }
        out[((size_t)t2 * F2 + f2) * kSubC + c0 + c] = acc;
    }
}

__global__ void __launch_bounds__(256) k_dw3s2_v4(const float4* __restrict__ x, int tin_valid, int Fin,
                                                  const float* __restrict__ w, const float* __restrict__ b,
                                                  float4* __restrict__ out, int Tout, int Fout) {
    pdl_entry();
    constexpr int V = kSubC / 4;  // float4 vectors per position
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)Tout * Fout * V) return;
    const int v = (int)(i % V);
    const long long pos = i / V;
    const int f = (int)(pos % Fout), t = (int)(pos / Fout);
    // weights of channels 4v .. 4v+3: 36 consecutive floats, tap-major per channel
    float wr[36];
    const float4* w4 = reinterpret_cast<const float4*>(w + (size_t)v * 36);
#pragma unroll
    for (int k = 0; k < 9; k++) {
        const float4 q = __ldg(w4 + k);
        wr[4 * k] = q.x;
        wr[4 * k + 1] = q.y;
        wr[4 * k + 2] = q.z;
        wr[4 * k + 3] = q.w;
    }
    float4 acc = __ldg(reinterpret_cast<const float4*>(b) + v);
#pragma unroll
    for (int dt = 0; dt < 3; dt++) {
        const int ti = 2 * t - 1 + dt;
        if (ti < 0 || ti >= tin_valid) continue;
#pragma unroll
        for (int df = 0; df < 3; df++) {
            const int fi = 2 * f - 1 + df;
            if (fi < 0 || fi >= Fin) continue;
            const float4 xv = __ldg(x + ((size_t)ti * Fin + fi) * V + v);
            const int k = dt * 3 + df;
            acc.x = __fmaf_rn(wr[k], xv.x, acc.x);
            acc.y = __fmaf_rn(wr[9 + k], xv.y, acc.y);
            acc.z = __fmaf_rn(wr[18 + k], xv.z, acc.z);
            acc.w = __fmaf_rn(wr[27 + k], xv.w, acc.w);
        }
    }
    out[i] = acc;
}

// Rel-pos attention inputs (cuda/kernels.cu:566-580): qu = half(q + bq + u), qv = half(q + bq + v),
// k = half(k + bk), v = half(v + bv) from qkv [T][3Dm] (fp32 sums in that order). A flat grid over 8-column groups
// of all rows: one 16-byte load of each of q, k, v and four 16-byte stores per thread (VEC 8), or one column per
// thread when Dm or the pointers do not allow 16-byte vectors (VEC 1).
template <int VEC>
__global__ void __launch_bounds__(256) k_relpos_prep_v(const __half* __restrict__ qkv, const float* __restrict__ bq,
                                                       const float* __restrict__ bk, const float* __restrict__ bv,
                                                       const float* __restrict__ pu, const float* __restrict__ pv,
                                                       __half* __restrict__ qu, __half* __restrict__ qvv,
                                                       __half* __restrict__ ko, __half* __restrict__ vo, int T,
                                                       int Dm) {
    pdl_entry();
    const int gpr = Dm / VEC;
    const long long n = (long long)T * gpr;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / gpr), c = (int)(i - (long long)t * gpr) * VEC;
        const __half* r = qkv + (size_t)t * 3 * Dm;
        float q[VEC], k[VEC], v[VEC];
        if constexpr (VEC == 8) {
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(r + c)), q);
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(r + Dm + c)), k);
            h8_to_f(__ldg(reinterpret_cast<const uint4*>(r + 2 * Dm + c)), v);
        } else {
            q[0] = __half2float(r[c]);
            k[0] = __half2float(r[Dm + c]);
            v[0] = __half2float(r[2 * Dm + c]);
        }
        float a[VEC], bq2[VEC], kk[VEC], vv[VEC];
#pragma unroll
        for (int e = 0; e < VEC; e++) {
            const float qb = q[e] + __ldg(bq + c + e);
            a[e] = qb + __ldg(pu + c + e);
            bq2[e] = qb + __ldg(pv + c + e);
            kk[e] = k[e] + __ldg(bk + c + e);
            vv[e] = v[e] + __ldg(bv + c + e);
        }
        const size_t o = (size_t)t * Dm + c;
        if constexpr (VEC == 8) {
            *reinterpret_cast<uint4*>(qu + o) = f_to_h8(a);
            *reinterpret_cast<uint4*>(qvv + o) = f_to_h8(bq2);
            *reinterpret_cast<uint4*>(ko + o) = f_to_h8(kk);
            *reinterpret_cast<uint4*>(vo + o) = f_to_h8(vv);
        } else {
            qu[o] = __float2half(a[0]);
            qvv[o] = __float2half(bq2[0]);
            ko[o] = __float2half(kk[0]);
            vo[o] = __float2half(vv[0]);
        }
    }
}

// p[h][i][j] = softmax_j((ac[h][i][j] + bd[h][i][j + T-1-i]) * scale) (cuda/kernels.cu:582-616: the same formulas
// — row max, sum of expf(z - max), expf(z - max) * (1 / sum)). One warp per row; each lane keeps its K scores of
// the row in registers (rows of up to 32*K columns), so ac and bd are read once instead of once per pass.
// K == 0: longer rows, re-read per pass.
template <int K>
__global__ void __launch_bounds__(256) k_relpos_softmax_warp(const float* __restrict__ ac, const float* __restrict__ bd,
                                                             __half* __restrict__ p, int T, int H, float scale) {
    pdl_entry();
    const int lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= (long long)H * T) return;
    const int i = (int)(row % T);
    const float* a = ac + row * T;
    const float* b = bd + row * (2 * T - 1) + (T - 1 - i);
    __half* pr = p + row * T;
    float mx = -INFINITY;
    if constexpr (K > 0) {
        float z[K];
#pragma unroll
        for (int k = 0; k < K; k++) {
            const int j = lane + 32 * k;
            z[k] = j < T ? (__ldg(a + j) + __ldg(b + j)) * scale : -INFINITY;
            mx = fmaxf(mx, z[k]);
        }
        mx = warp_max(mx);
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < K; k++) {
            z[k] = expf(z[k] - mx);  // exp(-inf) = 0 for the padding lanes
            s += z[k];
        }
        const float inv = 1.f / warp_sum(s);
#pragma unroll
        for (int k = 0; k < K; k++)
            if (lane + 32 * k < T) pr[lane + 32 * k] = __float2half(z[k] * inv);
    } else {
        for (int j = lane; j < T; j += 32) mx = fmaxf(mx, (__ldg(a + j) + __ldg(b + j)) * scale);
        mx = warp_max(mx);
        float s = 0.f;
        for (int j = lane; j < T; j += 32) s += expf((__ldg(a + j) + __ldg(b + j)) * scale - mx);
        const float inv = 1.f / warp_sum(s);
        for (int j = lane; j < T; j += 32) pr[j] = __float2half(expf((__ldg(a + j) + __ldg(b + j)) * scale - mx) * inv);
    }
}

// Conformer conv module middle (cuda/kernels.cu:618-637): GLU (x + b1) * sigmoid(gate + b1'), depthwise conv of
// `ksize` taps zero-padded at each clip's edges + bias, BN affine, SiLU, fp16 out; the reference's arithmetic per
// element (GLU values, then fused multiply-adds over the taps in order, then the affine). Data movement: a CTA per
// (32-row time window, 64-channel group) over the packed rows of all clips. The GLU of every input row the window
// reads (window + halo) is computed once into shared memory — not once per tap — and the taps are summed from
// there; each output row finds its clip's bounds in `offs` (null: one clip of all rows).
constexpr int kCdwRows = 32, kCdwCh = 64, kCdwMaxK = 31;

__global__ void __launch_bounds__(256) k_conformer_glu_dw(const __half* __restrict__ a, const float* __restrict__ b1,
                                                          const float* __restrict__ dw, const float* __restrict__ dwb,
                                                          const float* __restrict__ bn_s,
                                                          const float* __restrict__ bn_b, __half* __restrict__ out,
                                                          const int* __restrict__ offs, int n_clips, int R, int C,
                                                          int ksize) {
    __shared__ float glu[kCdwRows + kCdwMaxK - 1][kCdwCh];
    __shared__ int clip_lo[kCdwRows], clip_hi[kCdwRows];
    pdl_entry();
    const int r0 = blockIdx.x * kCdwRows, c0 = blockIdx.y * kCdwCh;
    const int pad = (ksize - 1) / 2, span = kCdwRows + ksize - 1;
    const int cl = threadIdx.x % kCdwCh, rg = threadIdx.x / kCdwCh, nrg = blockDim.x / kCdwCh;
    const int c = c0 + cl;
    if (threadIdx.x < kCdwRows) {
        const int r = r0 + threadIdx.x;
        int lo = 0, hi = R;
        if (offs && r < R) {  // the clip holding row r: offs[k] <= r < offs[k + 1]
            int l = 0, h = n_clips;
            while (h - l > 1) {
                const int m = (l + h) >> 1;
                if (__ldg(offs + m) <= r) l = m; else h = m;
            }
            lo = __ldg(offs + l);
            hi = __ldg(offs + l + 1);
        }
        clip_lo[threadIdx.x] = lo;
        clip_hi[threadIdx.x] = hi;
    }
    if (c < C) {
        const float bx = __ldg(b1 + c), bg = __ldg(b1 + C + c);
        for (int j = rg; j < span; j += nrg) {
            const int ti = r0 - pad + j;
            float gv = 0.f;
            if (ti >= 0 && ti < R) {
                const float x = __half2float(a[(size_t)ti * 2 * C + c]) + bx;
                const float gt = __half2float(a[(size_t)ti * 2 * C + C + c]) + bg;
                gv = x / (1.f + expf(-gt));
            }
            glu[j][cl] = gv;
        }
    }
    __syncthreads();
    if (c >= C) return;
    const float bias = __ldg(dwb + c), s = __ldg(bn_s + c), sh = __ldg(bn_b + c);
    for (int i = rg; i < kCdwRows; i += nrg) {
        const int r = r0 + i;
        if (r >= R) break;
        const int lo = clip_lo[i], hi = clip_hi[i];
        float acc = bias;
        for (int kk = 0; kk < ksize; kk++) {
            const int ti = r + kk - pad;
            if (ti >= lo && ti < hi) acc = __fmaf_rn(__ldg(dw + (size_t)c * ksize + kk), glu[i + kk][cl], acc);
        }
        acc = __fmaf_rn(acc, s, sh);
        out[(size_t)r * C + c] = __float2half(silu(acc));
    }
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

// ================================================================================================ C ABI
extern "C" {

int d1_rmsnorm(const float* x, const float* w, d1_half* y, int rows, int D, float eps, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (!al16(x) || !al16(w) || ((uintptr_t)y & 7)) return -1;
    const int grid = nblk(rows, 8);
    switch (D) {
        case 1024: launch_pdl(k_rmsnorm<8>, grid, 256, 0, st, x, w, y, rows, eps); break;
        case 768: launch_pdl(k_rmsnorm<6>, grid, 256, 0, st, x, w, y, rows, eps); break;
        case 512: launch_pdl(k_rmsnorm<4>, grid, 256, 0, st, x, w, y, rows, eps); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

int d1_layernorm(float* x, const float* pend_bias, float pend_scale, const float* w, const float* b, d1_half* y,
                 float* yf, int rows, int D, float eps, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (!al16(x) || !al16(w) || !al16(b) || (pend_bias && !al16(pend_bias)) || ((uintptr_t)y & 7) || !al16(yf))
        return -1;
    const int grid = nblk(rows, 8);
    switch (D) {
        case 1024: launch_pdl(k_layernorm<8>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, yf, nullptr, rows, eps); break;
        case 768: launch_pdl(k_layernorm<6>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, yf, nullptr, rows, eps); break;
        case 512: launch_pdl(k_layernorm<4>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, yf, nullptr, rows, eps); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

int d1_head_init(const float* h, const float* w, const float* type_emb, const int* tok_seq, const SeqInfo* seqs,
                 float* out, int rows, float eps, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (!al16(h) || !al16(w) || !al16(type_emb) || !al16(out)) return -1;
    launch_pdl(k_head_init, nblk(rows, 8), 256, 0, st, h, w, type_emb, tok_seq, seqs, out, rows, eps);
    return (int)cudaGetLastError();
}

int d1_embed(const d1_half* table, const int* ids, float* h, int rows, int D, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (D % 8 == 0 && al16(table) && al16(h))
        launch_pdl(k_embed, nblk(rows, 8), 256, 0, st, table, ids, h, rows, D);
    else
        launch_pdl(k_embed_scalar, rows, 256, 0, st, table, ids, h, rows, D);
    return (int)cudaGetLastError();
}

int d1_swiglu(const d1_half* gu, d1_half* out, int rows, int F, cudaStream_t st) {
    if (rows <= 0 || F <= 0) return rows == 0 || F == 0 ? 0 : -1;
    if (F % 8 == 0 && al16(gu) && al16(out))
        launch_pdl(k_swiglu8, egrid((size_t)rows * F / 8, 256), 256, 0, st, gu, out, rows, F);
    else
        launch_pdl(k_swiglu_scalar, egrid((size_t)rows * F, 256), 256, 0, st, gu, out, rows, F);
    return (int)cudaGetLastError();
}

int d1_bias_act_h(d1_half* x, const float* bias, int rows, int N, int act, cudaStream_t st) {
    if (rows <= 0 || N <= 0) return rows == 0 || N == 0 ? 0 : -1;
    if (N % 8 == 0 && al16(x))
        launch_pdl(k_bias_act_h8, egrid((size_t)rows * N / 8, 256), 256, 0, st, x, bias, rows, N, act);
    else
        launch_pdl(k_bias_act_h_scalar, egrid((size_t)rows * N, 256), 256, 0, st, x, bias, rows, N, act);
    return (int)cudaGetLastError();
}

int d1_bias_act_f(float* x, const float* bias, int rows, int N, int act, cudaStream_t st) {
    if (rows <= 0 || N <= 0) return rows == 0 || N == 0 ? 0 : -1;
    launch_pdl(k_bias_act_f, egrid((size_t)rows * N, 256), 256, 0, st, x, bias, rows, N, act);
    return (int)cudaGetLastError();
}

int d1_fill_rows(float* out, const float* bias, const float* add, int rows, int N, cudaStream_t st) {
    if (rows <= 0 || N <= 0) return rows == 0 || N == 0 ? 0 : -1;
    launch_pdl(k_fill_rows, egrid((size_t)rows * N, 256), 256, 0, st, out, bias, add, rows, N);
    return (int)cudaGetLastError();
}

int d1_f32_to_f16(const float* x, d1_half* y, size_t n, cudaStream_t st) {
    if (n == 0) return 0;
    launch_pdl(k_f32_to_f16, egrid(n, 256), 256, 0, st, x, y, n);
    return (int)cudaGetLastError();
}

int d1_gather_rows(const void* src, void* dst, const int* idx, int n, int row_bytes, cudaStream_t st) {
    if (n <= 0) return n == 0 ? 0 : -1;
    if (row_bytes % 16 || !al16(src) || !al16(dst)) return -1;
    launch_pdl(k_gather_rows, nblk(n, 8), 256, 0, st, (const uint4*)src, (uint4*)dst, idx, n, row_bytes / 16);
    return (int)cudaGetLastError();
}

int d1_shortconv(const d1_half* bcu, const float* convw, const int* tok_seq, const SeqInfo* seqs, d1_half* out,
                 int rows, int D, int conv_idx, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (D % 8 || !al16(bcu) || !al16(out) || !al16(convw)) return -1;
    const int threads = D / 8 < 128 ? D / 8 : 128;
    dim3 grid(nblk(rows, kConvRows), nblk(D / 8, threads));
    launch_pdl(k_shortconv, grid, threads, 0, st, bcu, convw, tok_seq, seqs, out, rows, D, conv_idx);
    return (int)cudaGetLastError();
}

int d1_qk_norm_rope(d1_half* qkv, int ld, int H, int KVH, const float* qn, const float* kn, const float* rope,
                    const int* tok_seq, const SeqInfo* seqs, int attn_idx, int rows, float eps, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (((uintptr_t)qkv & 3) || (ld & 1) || !al16(rope)) return -1;
    if (al16(qkv) && ld % 8 == 0 && H + KVH <= 4 * kQkMaxPerGroup) {
        launch_pdl(k_qk_norm_rope8, nblk(rows, 8), 256, 0, st, qkv, ld, H, KVH, qn, kn, rope, tok_seq, seqs, attn_idx, rows,
                                                       eps);
        return (int)cudaGetLastError();
    }
    launch_pdl(k_qk_norm_rope, rows, 256, 0, st, qkv, ld, H, KVH, qn, kn, rope, tok_seq, seqs, attn_idx, rows, eps);
    return (int)cudaGetLastError();
}

int d1_scorer_out(const d1_half* x, const float* b1, const d1_half* w2, float b2, float* logits, int rows, int D,
                  cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    launch_pdl(k_scorer_out, nblk(rows, 8), 256, 0, st, x, b1, w2, b2, logits, rows, D);
    return (int)cudaGetLastError();
}

int d1_vision_pos(const float* grid, const float* patch_b, const int* spans, const float* w, int taps, int ph,
                  int pw, int C, float* out, cudaStream_t st) {
    if (ph <= 0 || pw <= 0) return 0;
    if (!grid || !patch_b || !spans || !w || !out || taps < 1 || C < 1 || ((uintptr_t)spans & 7)) return -1;
    launch_pdl(k_vision_pos, ph * pw, 256, 0, st, grid, patch_b, reinterpret_cast<const int2*>(spans), w, taps, ph, pw, C,
                                           out);
    return (int)cudaGetLastError();
}

int d1_unshuffle(const d1_half* x, d1_half* out, int ph, int pw, int C, cudaStream_t st) {
    if (ph <= 0 || pw <= 0) return 0;
    if ((ph & 1) || (pw & 1) || C % 8 || !al16(x) || !al16(out)) return -1;
    const long long total = (long long)ph * pw * (C / 8);
    launch_pdl(k_unshuffle16, egrid((size_t)total, 256), 256, 0, st, reinterpret_cast<const uint4*>(x),
               reinterpret_cast<uint4*>(out), pw, C / 8, total);
    return (int)cudaGetLastError();
}

int d1_sub_conv0(const float* mel, int tin_valid, int F, const float* w, const float* b, float* out, int Tout, int Fout,
                 cudaStream_t st) {
    if (Tout <= 0 || Fout <= 0) return 0;
    if (!mel || !w || !b || !out || F <= 0 || F > 4096 || tin_valid < 0) return -1;
    launch_pdl(k_sub_conv0_rows, Tout, kSubC, (size_t)3 * F * sizeof(float), st, mel, tin_valid, F, w, b, out, Fout);
    return (int)cudaGetLastError();
}

int d1_sub_dwconv(const float* x, int tin_valid, int Fin, const float* w, const float* b, float* out, int Tout,
                  int Fout, cudaStream_t st) {
    if (Tout <= 0 || Fout <= 0) return 0;
    if (!al16(x) || !al16(w) || !al16(b) || !al16(out) || Fin <= 0 || tin_valid < 0) return -1;
    const long long n = (long long)Tout * Fout * (kSubC / 4);
    launch_pdl(k_dw3s2_v4, nblk((size_t)n, 256), 256, 0, st, reinterpret_cast<const float4*>(x), tin_valid, Fin, w, b,
               reinterpret_cast<float4*>(out), Tout, Fout);
    return (int)cudaGetLastError();
}

int d1_relpos_prep(const d1_half* qkv, const float* bq, const float* bk, const float* bv, const float* pu,
                   const float* pv, d1_half* qu, d1_half* qv, d1_half* k, d1_half* v, int T, int Dm, cudaStream_t st) {
    if (T <= 0 || Dm <= 0) return T == 0 ? 0 : -1;
    if (Dm % 8 == 0 && al16(qkv) && al16(qu) && al16(qv) && al16(k) && al16(v))
        launch_pdl(k_relpos_prep_v<8>, egrid((size_t)T * Dm / 8, 256), 256, 0, st, qkv, bq, bk, bv, pu, pv, qu, qv, k, v,
                   T, Dm);
    else
        launch_pdl(k_relpos_prep_v<1>, egrid((size_t)T * Dm, 256), 256, 0, st, qkv, bq, bk, bv, pu, pv, qu, qv, k, v,
                   T, Dm);
    return (int)cudaGetLastError();
}

int d1_relpos_softmax(const float* ac, const float* bd, d1_half* p, int T, int H, float scale, cudaStream_t st) {
    if (T <= 0 || H <= 0) return 0;
    const int grid = nblk((size_t)T * H, 8);  // a warp per row, 8 rows per CTA
    if (T <= 128)
        launch_pdl(k_relpos_softmax_warp<4>, grid, 256, 0, st, ac, bd, p, T, H, scale);
    else if (T <= 256)
        launch_pdl(k_relpos_softmax_warp<8>, grid, 256, 0, st, ac, bd, p, T, H, scale);
    else if (T <= 512)
        launch_pdl(k_relpos_softmax_warp<16>, grid, 256, 0, st, ac, bd, p, T, H, scale);
    else
        launch_pdl(k_relpos_softmax_warp<0>, grid, 256, 0, st, ac, bd, p, T, H, scale);
    return (int)cudaGetLastError();
}

int d1_conformer_dw(const d1_half* a, const float* b1, const float* dw, const float* dwb, const float* bn_s,
                    const float* bn_b, d1_half* out, int T, int C, int ksize, cudaStream_t st) {
    return d1_conformer_dw_clips(a, b1, dw, dwb, bn_s, bn_b, out, nullptr, 1, T, C, ksize, st);
}

int d1_conformer_dw_clips(const d1_half* a, const float* b1, const float* dw, const float* dwb, const float* bn_s,
                          const float* bn_b, d1_half* out, const int* offs, int n_clips, int rows, int C, int ksize,
                          cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (C <= 0 || ksize < 1 || ksize > kCdwMaxK || n_clips < 1 || !a || !b1 || !dw || !dwb || !bn_s || !bn_b || !out)
        return -1;
    dim3 grid(nblk(rows, kCdwRows), nblk(C, kCdwCh));
    launch_pdl(k_conformer_glu_dw, grid, 256, 0, st, a, b1, dw, dwb, bn_s, bn_b, out, offs, n_clips, rows, C, ksize);
    return (int)cudaGetLastError();
}

int d1_sub_conv01(const float* mel, int tin_valid, int F, const float* w0, const float* b0, const float* w1,
                  const float* b1, float* out, int l1, int l2, cudaStream_t st) {
    if (l2 <= 0) return l2 == 0 ? 0 : -1;
    const int F1 = (F - 1) / 2 + 1, F2 = (F1 - 1) / 2 + 1;
    if (!mel || !w0 || !b0 || !w1 || !b1 || !out || F <= 0 || F > kSubMaxF || l1 <= 0 || tin_valid < 0) return -1;
    dim3 grid(l2, kSubC / kSubGroup);
    launch_pdl(k_sub_conv01, grid, 256, 0, st, mel, tin_valid, F, w0, b0, w1, b1, out, l1, F1, F2);
    return (int)cudaGetLastError();
}

int d1_layernorm_rows(float* x, const float* pend_bias, float pend_scale, const float* w, const float* b, d1_half* y,
                      const int* y_rows, int rows, int D, float eps, cudaStream_t st) {
    if (rows <= 0) return rows == 0 ? 0 : -1;
    if (!y || !y_rows || !al16(x) || !al16(w) || !al16(b) || (pend_bias && !al16(pend_bias)) || ((uintptr_t)y & 7))
        return -1;
    const int grid = nblk(rows, 8);
    switch (D) {
        case 1024: launch_pdl(k_layernorm<8>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, nullptr, y_rows, rows, eps); break;
        case 768: launch_pdl(k_layernorm<6>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, nullptr, y_rows, rows, eps); break;
        case 512: launch_pdl(k_layernorm<4>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, nullptr, y_rows, rows, eps); break;
        default: return -1;
    }
    return (int)cudaGetLastError();
}

}  // extern "C"
