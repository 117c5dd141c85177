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
                                                   __half* __restrict__ y, float* yf, int rows, float eps) {
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
        if (y) reinterpret_cast<uint2*>(y + (size_t)row * D)[lane + 32 * i] = make_uint2(h2u(o.x, o.y), h2u(o.z, o.w));
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
// thread's loads (b and u of rows t0-1 .. t0+kConvRows, c of its rows: 28 independent 16-byte loads) are issued
// before any arithmetic, so the kernel runs at HBM bandwidth instead of one dependent row at a time; each row is
// read once per CTA plus a one-row halo on each side (an L2 hit). Sequence boundaries, the prefix's left state
// (ext_bx) and the saved last state (save_bx) follow cuda/kernels.cu:224-259.
constexpr int kConvRows = 8;

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
#pragma unroll
    for (int i = 0; i < 8; i++) {
        w0[i] = __ldg(convw + (c + i) * 3);
        w1[i] = __ldg(convw + (c + i) * 3 + 1);
        w2[i] = __ldg(convw + (c + i) * 3 + 2);
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

__global__ void k_unshuffle(const __half* __restrict__ x, __half* __restrict__ out, int ph, int pw, int C) {
    pdl_entry();
    const int o = blockIdx.x;
    const int i = o / (pw / 2), jj = o % (pw / 2);
    for (int k = threadIdx.x * 8; k < 4 * C; k += blockDim.x * 8) {
        const int q = k / C, c = k % C;
        const int yy = 2 * i + (q >> 1), xx = 2 * jj + (q & 1);
        *reinterpret_cast<uint4*>(out + (size_t)o * 4 * C + k) =
            __ldg(reinterpret_cast<const uint4*>(x + ((size_t)yy * pw + xx) * C + c));
    }
}

// ------------------------------------------------------------------------------------------------ audio
// First subsampling conv: mel [Tin][F] -> [Tout][Fout][256], 3x3 stride 2, pad 1, ReLU (cuda/kernels.cu:529-545).
__global__ void __launch_bounds__(256) k_sub_conv0(const float* __restrict__ mel, int tin_valid, int F,
                                                   const float* __restrict__ w, const float* __restrict__ b,
                                                   float* __restrict__ out, int Tout, int Fout) {
    pdl_entry();
    const int t = blockIdx.x, f = blockIdx.y, c = threadIdx.x;
    __shared__ float patch[9];
    if (threadIdx.x < 9) {
        const int ti = 2 * t - 1 + threadIdx.x / 3, fi = 2 * f - 1 + threadIdx.x % 3;
        patch[threadIdx.x] = (ti >= 0 && ti < tin_valid && fi >= 0 && fi < F) ? mel[(size_t)ti * F + fi] : 0.f;
    }
    __syncthreads();
    float acc = b[c];
#pragma unroll
    for (int dt = 0; dt < 3; dt++) {
        const int ti = 2 * t - 1 + dt;
        if (ti < 0 || ti >= tin_valid) continue;
#pragma unroll
        for (int df = 0; df < 3; df++) {
            const int fi = 2 * f - 1 + df;
            if (fi < 0 || fi >= F) continue;
            acc += w[c * 9 + dt * 3 + df] * patch[dt * 3 + df];
        }
    }
    out[((size_t)t * Fout + f) * 256 + c] = fmaxf(acc, 0.f);
}

// Depthwise 3x3 stride-2 conv on [Tin][Fin][256] (cuda/kernels.cu:548-564).
__global__ void __launch_bounds__(256) k_sub_dwconv(const float* __restrict__ x, int tin_valid, int Fin,
                                                    const float* __restrict__ w, const float* __restrict__ b,
                                                    float* __restrict__ out, int Fout) {
    pdl_entry();
    const int t = blockIdx.x, f = blockIdx.y, c = threadIdx.x;
    float acc = b[c];
#pragma unroll
    for (int dt = 0; dt < 3; dt++) {
        const int ti = 2 * t - 1 + dt;
        if (ti < 0 || ti >= tin_valid) continue;
#pragma unroll
        for (int df = 0; df < 3; df++) {
            const int fi = 2 * f - 1 + df;
            if (fi < 0 || fi >= Fin) continue;
            acc += w[c * 9 + dt * 3 + df] * x[((size_t)ti * Fin + fi) * 256 + c];
        }
    }
    out[((size_t)t * Fout + f) * 256 + c] = acc;
}

// qkv [T][3Dm] -> qu = q+bq+u, qv = q+bq+v, k+bk, v+bv (cuda/kernels.cu:566-580).
__global__ void k_relpos_prep(const __half* __restrict__ qkv, const float* __restrict__ bq,
                              const float* __restrict__ bk, const float* __restrict__ bv, const float* __restrict__ pu,
                              const float* __restrict__ pv, __half* __restrict__ qu, __half* __restrict__ qvv,
                              __half* __restrict__ k, __half* __restrict__ v, int T, int Dm) {
    pdl_entry();
    const int t = blockIdx.x;
    const __half* r = qkv + (size_t)t * 3 * Dm;
    for (int c = threadIdx.x; c < Dm; c += blockDim.x) {
        const float q = __half2float(r[c]) + bq[c];
        qu[(size_t)t * Dm + c] = __float2half(q + pu[c]);
        qvv[(size_t)t * Dm + c] = __float2half(q + pv[c]);
        k[(size_t)t * Dm + c] = __float2half(__half2float(r[Dm + c]) + bk[c]);
        v[(size_t)t * Dm + c] = __float2half(__half2float(r[2 * Dm + c]) + bv[c]);
    }
}

// p[h][i][j] = softmax_j((ac[h][i][j] + bd[h][i][j + T-1-i]) * scale) (cuda/kernels.cu:582-616).
__global__ void __launch_bounds__(256) k_relpos_softmax(const float* __restrict__ ac, const float* __restrict__ bd,
                                                        __half* __restrict__ p, int T, float scale) {
    pdl_entry();
    const int h = blockIdx.y, i = blockIdx.x;
    const float* a = ac + ((size_t)h * T + i) * T;
    const float* b = bd + ((size_t)h * T + i) * (2 * T - 1) + (T - 1 - i);
    __shared__ float red[32];
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < T; j += blockDim.x) mx = fmaxf(mx, (a[j] + b[j]) * scale);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : -INFINITY;
        v = warp_max(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    mx = red[0];
    __syncthreads();
    float sum = 0.f;
    for (int j = threadIdx.x; j < T; j += blockDim.x) sum += expf((a[j] + b[j]) * scale - mx);
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
        v = warp_sum(v);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float inv = 1.f / red[0];
    __half* pr = p + ((size_t)h * T + i) * T;
    for (int j = threadIdx.x; j < T; j += blockDim.x) pr[j] = __float2half(expf((a[j] + b[j]) * scale - mx) * inv);
}

// Conformer conv module middle: GLU -> depthwise k (zero pad) + bias -> BN affine -> SiLU (cuda/kernels.cu:618-637).
__global__ void k_conformer_dw(const __half* __restrict__ a, const float* __restrict__ b1, const float* __restrict__ dw,
                               const float* __restrict__ dwb, const float* __restrict__ bn_s,
                               const float* __restrict__ bn_b, __half* __restrict__ out, int T, int C, int ksize) {
    pdl_entry();
    const int t = blockIdx.x;
    const int pad = (ksize - 1) / 2;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float acc = dwb[c];
        for (int kk = 0; kk < ksize; kk++) {
            const int ti = t + kk - pad;
            if (ti < 0 || ti >= T) continue;
            const float x = __half2float(a[(size_t)ti * 2 * C + c]) + b1[c];
            const float gt = __half2float(a[(size_t)ti * 2 * C + C + c]) + b1[C + c];
            acc += dw[c * ksize + kk] * (x / (1.f + expf(-gt)));
        }
        acc = acc * bn_s[c] + bn_b[c];
        out[(size_t)t * C + c] = __float2half(silu(acc));
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
        case 1024: launch_pdl(k_layernorm<8>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, yf, rows, eps); break;
        case 768: launch_pdl(k_layernorm<6>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, yf, rows, eps); break;
        case 512: launch_pdl(k_layernorm<4>, grid, 256, 0, st, x, pend_bias, pend_scale, w, b, y, yf, rows, eps); break;
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
    if (D % 8 || !al16(bcu) || !al16(out)) return -1;
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
    if (C % 8 || !al16(x) || !al16(out)) return -1;
    launch_pdl(k_unshuffle, (ph / 2) * (pw / 2), 128, 0, st, x, out, ph, pw, C);
    return (int)cudaGetLastError();
}

int d1_sub_conv0(const float* mel, int tin_valid, int F, const float* w, const float* b, float* out, int Tout, int Fout,
                 cudaStream_t st) {
    if (Tout <= 0 || Fout <= 0) return 0;
    dim3 grid(Tout, Fout);
    launch_pdl(k_sub_conv0, grid, 256, 0, st, mel, tin_valid, F, w, b, out, Tout, Fout);
    return (int)cudaGetLastError();
}

int d1_sub_dwconv(const float* x, int tin_valid, int Fin, const float* w, const float* b, float* out, int Tout,
                  int Fout, cudaStream_t st) {
    if (Tout <= 0 || Fout <= 0) return 0;
    dim3 grid(Tout, Fout);
    launch_pdl(k_sub_dwconv, grid, 256, 0, st, x, tin_valid, Fin, w, b, out, Fout);
    return (int)cudaGetLastError();
}

int d1_relpos_prep(const d1_half* qkv, const float* bq, const float* bk, const float* bv, const float* pu,
                   const float* pv, d1_half* qu, d1_half* qv, d1_half* k, d1_half* v, int T, int Dm, cudaStream_t st) {
    if (T <= 0) return 0;
    launch_pdl(k_relpos_prep, T, 256, 0, st, qkv, bq, bk, bv, pu, pv, qu, qv, k, v, T, Dm);
    return (int)cudaGetLastError();
}

int d1_relpos_softmax(const float* ac, const float* bd, d1_half* p, int T, int H, float scale, cudaStream_t st) {
    if (T <= 0 || H <= 0) return 0;
    dim3 grid(T, H);
    launch_pdl(k_relpos_softmax, grid, 256, 0, st, ac, bd, p, T, scale);
    return (int)cudaGetLastError();
}

int d1_conformer_dw(const d1_half* a, const float* b1, const float* dw, const float* dwb, const float* bn_s,
                    const float* bn_b, d1_half* out, int T, int C, int ksize, cudaStream_t st) {
    if (T <= 0) return 0;
    launch_pdl(k_conformer_dw, T, 256, 0, st, a, b1, dw, dwb, bn_s, bn_b, out, T, C, ksize);
    return (int)cudaGetLastError();
}

}  // extern "C"
