// FastConformer audio-encoder kernels that the reference runs through cuBLAS from Rust (src/cuda.rs:493-527,
// called from src/audio.rs:514-571), rebuilt for B200:
//
// d1_sgemm — fp32 row-major Y[M,N] = act(X[M,K] . W[N,K]^T + beta * Y + bias): Blas::sgemm (src/cuda.rs:493-505)
//   with the d1_fill_rows / d1_bias_act_f calls around it (src/audio.rs:517-525) folded into the epilogue.
//   fp32 FFMA (the reference asks cuBLAS for CUDA_R_32F with COMPUTE_32F, i.e. no TF32). 256 threads per CTA;
//   128 x 128 tiles (8 x 8 outputs per thread) when they fill the GPU, else 64 x 64 tiles with the K range split
//   across a thread-block cluster of up to 8 CTAs whose partial tiles are summed in rank order through
//   distributed shared memory — deterministic, no global workspace, no atomics.
//
// d1_relpos_attn — the encoder's relative-position self-attention (src/audio.rs:565-571: three strided-batched
//   GEMMs around d1_relpos_softmax, cuda/kernels.cu:583-616) as one kernel over packed clips. For clip c, head h
//   and query i, key j < T:
//       score(i, j) = (qu_i . k_j + qv_i . pp[center + j - i]) * scale,  P = softmax_j(score) rounded to fp16,
//       O_i = P . V (fp32 accumulation, fp16 out)
//   where row `center + j - i` of pp holds the projected sinusoid of relative position i - j (the reference's
//   per-clip pp has center = T - 1; the runner passes a per-layer table for all positions of the longest clip).
//   One CTA per (64-query tile, clip, head): the 64 x T score block lives in shared memory (fp32), the qu.k^T
//   tiles are written into it, the qv.pp^T tiles of the 64-row pp chunks that the tile's band touches are added
//   at their shifted columns, an exact row softmax (expf, like the reference) writes P in place as fp16, and P.V
//   accumulates in registers. K tiles, pp chunks and V tiles stream through one double-buffered cp.async ring;
//   the MMAs are m16n8k16 fp16 with fp32 accumulation. Clips up to 384 frames after subsampling
//   (src/audio.rs:401 MAX_T) — the reference's limit.
#include <cooperative_groups.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "warp_mma.cuh"

using namespace d1;
namespace cg = cooperative_groups;

namespace {

// ================================================================================================ fp32 GEMM

struct SgArgs {
    const float* X;
    const float* W;
    float* Y;
    const float* bias;
    int M, N, K, ldx, ldw, ldy, act, kchunk;
    float beta;
};

constexpr int SG_BK = 16;

template <int BM, int BN>
struct SgSmem {
    static constexpr int A = 2 * SG_BK * (BM + 4);
    static constexpr int B = 2 * SG_BK * (BN + 4);
    static constexpr int TOTAL = A + B;
};

template <int BM, int BN, bool VEC, bool SPLIT>
__global__ void __launch_bounds__(256) k_sgemm(const SgArgs a) {
    constexpr int TM = BM / 16, TN = BN / 16;
    constexpr int LX = BM / 64, LW = BN / 64;
    __shared__ __align__(16) float sm[SgSmem<BM, BN>::TOTAL];
    float(*As)[SG_BK][BM + 4] = reinterpret_cast<float(*)[SG_BK][BM + 4]>(sm);
    float(*Bs)[SG_BK][BN + 4] = reinterpret_cast<float(*)[SG_BK][BN + 4]>(sm + SgSmem<BM, BN>::A);

    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int kb = SPLIT ? blockIdx.z * a.kchunk : 0;
    const int ke = SPLIT ? min(a.K, kb + a.kchunk) : a.K;
    const int nkt = ke > kb ? (ke - kb + SG_BK - 1) / SG_BK : 0;

    float4 rx[LX], rw[LW];
    auto ld4 = [&](const float* base, int ld, int r, int rmax, int k) {
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < rmax && k < ke) {
            const float* p = base + (size_t)r * ld + k;
            if (VEC) {
                v = __ldg(reinterpret_cast<const float4*>(p));
            } else {
                v.x = __ldg(p);
                if (k + 1 < ke) v.y = __ldg(p + 1);
                if (k + 2 < ke) v.z = __ldg(p + 2);
                if (k + 3 < ke) v.w = __ldg(p + 3);
            }
        }
        return v;
    };
    auto gload = [&](int k0) {
#pragma unroll
        for (int i = 0; i < LX; i++) {
            const int f = tid + 256 * i;
            rx[i] = ld4(a.X, a.ldx, m0 + (f >> 2), a.M, k0 + (f & 3) * 4);
        }
#pragma unroll
        for (int i = 0; i < LW; i++) {
            const int f = tid + 256 * i;
            rw[i] = ld4(a.W, a.ldw, n0 + (f >> 2), a.N, k0 + (f & 3) * 4);
        }
    };
    auto sstore = [&](int buf) {
#pragma unroll
        for (int i = 0; i < LX; i++) {
            const int f = tid + 256 * i, r = f >> 2, k = (f & 3) * 4;
            As[buf][k][r] = rx[i].x;
            As[buf][k + 1][r] = rx[i].y;
            As[buf][k + 2][r] = rx[i].z;
            As[buf][k + 3][r] = rx[i].w;
        }
#pragma unroll
        for (int i = 0; i < LW; i++) {
            const int f = tid + 256 * i, r = f >> 2, k = (f & 3) * 4;
            Bs[buf][k][r] = rw[i].x;
            Bs[buf][k + 1][r] = rw[i].y;
            Bs[buf][k + 2][r] = rw[i].z;
            Bs[buf][k + 3][r] = rw[i].w;
        }
    };

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = 0.f;

    if (nkt > 0) {
        gload(kb);
        sstore(0);
    }
    __syncthreads();
    for (int kt = 0; kt < nkt; kt++) {
        const int cur = kt & 1;
        if (kt + 1 < nkt) gload(kb + (kt + 1) * SG_BK);
#pragma unroll
        for (int k = 0; k < SG_BK; k++) {
            float av[TM], bv[TN];
#pragma unroll
            for (int g = 0; g < TM / 4; g++) {
                const float4 t = *reinterpret_cast<const float4*>(&As[cur][k][g * 64 + ty * 4]);
                av[g * 4] = t.x;
                av[g * 4 + 1] = t.y;
                av[g * 4 + 2] = t.z;
                av[g * 4 + 3] = t.w;
            }
#pragma unroll
            for (int g = 0; g < TN / 4; g++) {
                const float4 t = *reinterpret_cast<const float4*>(&Bs[cur][k][g * 64 + tx * 4]);
                bv[g * 4] = t.x;
                bv[g * 4 + 1] = t.y;
                bv[g * 4 + 2] = t.z;
                bv[g * 4 + 3] = t.w;
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (kt + 1 < nkt) sstore(cur ^ 1);
        __syncthreads();
    }

    auto epilogue = [&](int m, int n, float v) {
        if (m < a.M && n < a.N) {
            float* y = a.Y + (size_t)m * a.ldy + n;
            if (a.beta != 0.f) v += a.beta * *y;
            if (a.bias) v += __ldg(a.bias + n);
            *y = apply_act(v, a.act);
        }
    };

    if constexpr (!SPLIT) {
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++)
                epilogue(m0 + (i / 4) * 64 + ty * 4 + (i & 3), n0 + (j / 4) * 64 + tx * 4 + (j & 3), acc[i][j]);
    } else {
        // partial tile -> own shared memory; rank r then sums rows [r*BM/S, (r+1)*BM/S) over all ranks in rank
        // order (deterministic) and runs the epilogue for them
        static_assert(BM * BN <= SgSmem<BM, BN>::TOTAL, "partial tile must fit the operand buffers");
        cg::cluster_group cl = cg::this_cluster();
        float* red = sm;
#pragma unroll
        for (int i = 0; i < TM; i++)
#pragma unroll
            for (int j = 0; j < TN; j++)
                red[((i / 4) * 64 + ty * 4 + (i & 3)) * BN + (j / 4) * 64 + tx * 4 + (j & 3)] = acc[i][j];
        cl.sync();
        const int S = (int)cl.num_blocks(), r = (int)cl.block_rank();
        const int rows = BM / S;
        for (int e = tid; e < rows * BN; e += 256) {
            const int row = r * rows + e / BN, col = e % BN;
            float v = 0.f;
            for (int q = 0; q < S; q++) v += cl.map_shared_rank(red, q)[row * BN + col];
            epilogue(m0 + row, n0 + col, v);
        }
        cl.sync();  // keep this CTA's partial alive until every rank has read it
    }
}

// ================================================================================================ rel-pos attention

constexpr int RP_B = 64;     // query rows per CTA, keys / pp rows per tile
constexpr int RP_LD = 72;    // padded shared row (halves): conflict-free ldmatrix
constexpr int RP_MAXT = 384; // src/audio.rs:401

struct RpArgs {
    const __half* qu;
    const __half* qv;
    const __half* k;
    const __half* v;
    const __half* pp;
    __half* o;
    const int* offs;
    int ld, ldp, pp_rows, pp_center, ldo, max_len, srow;
    float scale;
};

__device__ int g_rp_err = 0;

__global__ void __launch_bounds__(256) k_relpos_attn(const RpArgs a) {
    extern __shared__ __align__(16) uint8_t rp_smem[];
    __half* sQu = reinterpret_cast<__half*>(rp_smem);   // [64][RP_LD]
    __half* sQv = sQu + RP_B * RP_LD;                    // [64][RP_LD]
    __half* sT = sQv + RP_B * RP_LD;                     // [2][64][RP_LD] tile ring
    float* sS = reinterpret_cast<float*>(sT + 2 * RP_B * RP_LD);  // [64][srow] scores; P aliases each row

    const int clip = blockIdx.y, h = blockIdx.z;
    const int start = a.offs[clip], len = a.offs[clip + 1] - start;
    const int i0 = blockIdx.x * RP_B;
    if (len > a.max_len || len < 0) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(&g_rp_err, 1);
        return;
    }
    if (i0 >= len) return;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gid = lane >> 2, tig = lane & 3;
    const int nk = (len + RP_B - 1) / RP_B;
    const int np = (len + 2 * RP_B - 2) / RP_B;        // pp rows center-(i0+63) .. center+len-1-i0
    const int mbase = a.pp_center - i0 - (RP_B - 1);
    const int ntiles = nk + np + nk;
    const int hc = h * 64;

    // Q tiles (qu, qv) of this head; committed together with tile 0
    for (int i = tid; i < 2 * RP_B * 8; i += 256) {
        const int which = i / (RP_B * 8), r = (i / 8) % RP_B, c = (i % 8) * 8;
        const bool ok = i0 + r < len;
        const __half* base = which ? a.qv : a.qu;
        const __half* src = ok ? base + (size_t)(start + i0 + r) * a.ld + hc + c : base;
        cp_async16(smem_u32((which ? sQv : sQu) + r * RP_LD + c), src, ok);
    }
    auto load_tile = [&](int q, int buf) {
        __half* dst = sT + buf * RP_B * RP_LD;
        for (int i = tid; i < RP_B * 8; i += 256) {
            const int r = i / 8, c = (i % 8) * 8;
            const __half* src = a.k;
            bool ok;
            if (q < nk) {
                const int j = q * RP_B + r;
                ok = j < len;
                if (ok) src = a.k + (size_t)(start + j) * a.ld + hc + c;
            } else if (q < nk + np) {
                const int m = mbase + (q - nk) * RP_B + r;
                ok = m >= 0 && m < a.pp_rows;
                if (ok) src = a.pp + (size_t)m * a.ldp + hc + c;
            } else {
                const int j = (q - nk - np) * RP_B + r;
                ok = j < len;
                if (ok) src = a.v + (size_t)(start + j) * a.ld + hc + c;
            }
            cp_async16(smem_u32(dst + r * RP_LD + c), src, ok);
        }
        cp_async_commit();
    };

    const int wr = (warp & 3) * 16, wc = (warp >> 2) * 32;  // warp's 16 rows x 32 columns of a 64 x 64 tile
    const int lr = (lane & 7) + ((lane >> 3) & 1) * 8, lc = (lane >> 4) * 8;
    uint32_t qa[4][4];
    float o[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    __half* sP = reinterpret_cast<__half*>(sS);
    const int prow = a.srow * 2;  // P row pitch in halves (P row r overlays S row r)

    load_tile(0, 0);
    for (int q = 0; q < ntiles; q++) {
        const int buf = q & 1;
        if (q + 1 < ntiles) {
            load_tile(q + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const __half* T = sT + buf * RP_B * RP_LD;

        if (q == 0 || q == nk) {  // A fragments: qu for the qu.k^T tiles, qv for the qv.pp^T tiles
            const __half* Qs = q == 0 ? sQu : sQv;
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], smem_u32(Qs + (wr + lr) * RP_LD + kk * 16 + lc));
        }
        if (q < nk + np) {
            float acc[4][4];
#pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
#pragma unroll
                for (int kk = 0; kk < 4; kk += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(b0, b1, b2, b3, smem_u32(T + (wc + nt * 8 + (lane & 7)) * RP_LD + kk * 16 + (lane >> 3) * 8));
                    mma16816(acc[nt], qa[kk], b0, b1);
                    mma16816(acc[nt], qa[kk + 1], b2, b3);
                }
            }
            if (q < nk) {  // ac tile -> S[:, q*64 + col]
#pragma unroll
                for (int nt = 0; nt < 4; nt++) {
                    const int col = q * RP_B + wc + nt * 8 + 2 * tig;
                    *reinterpret_cast<float2*>(sS + (wr + gid) * a.srow + col) = make_float2(acc[nt][0], acc[nt][1]);
                    *reinterpret_cast<float2*>(sS + (wr + gid + 8) * a.srow + col) = make_float2(acc[nt][2], acc[nt][3]);
                }
            } else {  // bd tile: pp row m = mbase + 64(q-nk) + col pairs with key j = m - center + i
                const int jb = (q - nk) * RP_B - (RP_B - 1);
#pragma unroll
                for (int nt = 0; nt < 4; nt++)
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int r = wr + gid + (e >> 1) * 8;
                        const int j = jb + wc + nt * 8 + 2 * tig + (e & 1) + r;
                        if (j >= 0 && j < len) sS[r * a.srow + j] += acc[nt][e];
                    }
            }
        }
        if (q == nk + np - 1) {
            __syncthreads();  // the score block is complete
            // exact row softmax (cuda/kernels.cu:583-616): max, sum of expf, P = fp16(expf(s - max) / sum)
            for (int rr = 0; rr < 8; rr++) {
                const int r = warp * 8 + rr;
                const bool valid = i0 + r < len;
                float* Srow = sS + r * a.srow;
                float vals[RP_MAXT / 32];
                float mx = -INFINITY;
#pragma unroll
                for (int u = 0; u < RP_MAXT / 32; u++) {
                    const int j = lane + 32 * u;
                    vals[u] = valid && j < len ? Srow[j] * a.scale : -INFINITY;
                    mx = fmaxf(mx, vals[u]);
                }
                mx = warp_max(mx);
                float sum = 0.f;
#pragma unroll
                for (int u = 0; u < RP_MAXT / 32; u++)
                    if (lane + 32 * u < len) sum += expf(vals[u] - mx);
                sum = warp_sum(sum);
                const float inv = 1.f / sum;
                __syncwarp();  // every lane has read the row before P overwrites it
                __half* Prow = sP + r * prow;
#pragma unroll
                for (int u = 0; u < RP_MAXT / 32; u++) {
                    const int j = lane + 32 * u;
                    if (j < nk * RP_B) Prow[j] = __float2half(valid && j < len ? expf(vals[u] - mx) * inv : 0.f);
                }
            }
            __syncthreads();
        }
        if (q >= nk + np) {  // O += P[:, 64kt .. 64kt+63] . V tile
            const int kt = q - nk - np;
#pragma unroll
            for (int kk = 0; kk < 4; kk++) {
                uint32_t pa[4];
                ldsm_x4(pa[0], pa[1], pa[2], pa[3], smem_u32(sP + (wr + lr) * prow + kt * RP_B + kk * 16 + lc));
#pragma unroll
                for (int dt = 0; dt < 4; dt += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(b0, b1, b2, b3, smem_u32(T + (kk * 16 + lr) * RP_LD + wc + dt * 8 + lc));
                    mma16816(o[dt], pa, b0, b1);
                    mma16816(o[dt + 1], pa, b2, b3);
                }
            }
        }
        __syncthreads();  // tile buffer `buf` is free for the load issued next iteration
    }

    // fp16 output rows of this head
#pragma unroll
    for (int dt = 0; dt < 4; dt++) {
        const int c = hc + wc + dt * 8 + 2 * tig;
        const int r0 = i0 + wr + gid, r1 = r0 + 8;
        if (r0 < len) *reinterpret_cast<uint32_t*>(a.o + (size_t)(start + r0) * a.ldo + c) = pack_h2(o[dt][0], o[dt][1]);
        if (r1 < len) *reinterpret_cast<uint32_t*>(a.o + (size_t)(start + r1) * a.ldo + c) = pack_h2(o[dt][2], o[dt][3]);
    }
}

int rp_smem_bytes(int max_len) {
    const int srow = (max_len + RP_B - 1) / RP_B * RP_B + 4;
    return 4 * RP_B * RP_LD * 2 + RP_B * srow * 4;
}

template <int BM, int BN, bool VEC, bool SPLIT>
int launch_sgemm(const SgArgs& a, int split, cudaStream_t st) {
    dim3 grid((a.N + BN - 1) / BN, (a.M + BM - 1) / BM, split);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (SPLIT) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = split;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaLaunchKernelEx(&cfg, k_sgemm<BM, BN, VEC, SPLIT>, a);
    return (int)cudaGetLastError();
}

}  // namespace

extern "C" {

int d1_sgemm(int M, int N, int K, const float* X, int ldx, const float* W, int ldw, float* Y, int ldy, float beta,
             const float* bias, int act, cudaStream_t st) {
    if (M < 0 || N < 0 || K < 0 || act < 0 || act > 4) return -1;
    if (M == 0 || N == 0) return 0;
    if (!X || !W || !Y || ldx < K || ldw < K || ldy < N) return -1;
    SgArgs a{X, W, Y, bias, M, N, K, ldx, ldw, ldy, act, K, beta};
    const bool vec = K % 4 == 0 && ldx % 4 == 0 && ldw % 4 == 0 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0;
    const long tiles128 = (long)((M + 127) / 128) * ((N + 127) / 128);
    if (tiles128 >= 148) {
        return vec ? launch_sgemm<128, 128, true, false>(a, 1, st) : launch_sgemm<128, 128, false, false>(a, 1, st);
    }
    const long tiles64 = (long)((M + 63) / 64) * ((N + 63) / 64);
    int split = 1;
    while (split < 8 && tiles64 * split < 2 * 148 && K / (2 * split) >= 128) split *= 2;
    if (split == 1)
        return vec ? launch_sgemm<64, 64, true, false>(a, 1, st) : launch_sgemm<64, 64, false, false>(a, 1, st);
    a.kchunk = ((K + split - 1) / split + SG_BK - 1) / SG_BK * SG_BK;
    return vec ? launch_sgemm<64, 64, true, true>(a, split, st) : launch_sgemm<64, 64, false, true>(a, split, st);
}

int d1_relpos_attn(const d1_half* qu, const d1_half* qv, const d1_half* k, const d1_half* v, int ld,
                   const d1_half* pp, int ldp, int pp_rows, int pp_center, d1_half* o, int ldo, const int* offs,
                   int n_clips, int max_len, int heads, float scale, cudaStream_t st) {
    if (n_clips < 0 || max_len < 0 || max_len > RP_MAXT || heads < 1) return -1;
    if (n_clips == 0 || max_len == 0) return 0;
    if (!qu || !qv || !k || !v || !pp || !o || !offs) return -1;
    if (ld % 8 || ldp % 8 || ldo % 2 || ld < heads * 64 || ldp < heads * 64 || ldo < heads * 64 || pp_rows < 1)
        return -1;
    for (const void* p : {(const void*)qu, (const void*)qv, (const void*)k, (const void*)v, (const void*)pp})
        if ((uintptr_t)p & 15) return -1;
    if ((uintptr_t)o & 3) return -1;
    const int smem = rp_smem_bytes(max_len);
    static unsigned long long attr_done = 0;  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(__atomic_load_n(&attr_done, __ATOMIC_ACQUIRE) & bit)) {
        if (cudaFuncSetAttribute(k_relpos_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, rp_smem_bytes(RP_MAXT)) !=
            cudaSuccess)
            return -1;
        __atomic_fetch_or(&attr_done, bit, __ATOMIC_RELEASE);
    }
    RpArgs a{reinterpret_cast<const __half*>(qu), reinterpret_cast<const __half*>(qv),
             reinterpret_cast<const __half*>(k),  reinterpret_cast<const __half*>(v),
             reinterpret_cast<const __half*>(pp), reinterpret_cast<__half*>(o),
             offs, ld, ldp, pp_rows, pp_center, ldo, max_len, (max_len + RP_B - 1) / RP_B * RP_B + 4, scale};
    dim3 grid((max_len + RP_B - 1) / RP_B, n_clips, heads);
    k_relpos_attn<<<grid, 256, smem, st>>>(a);
    return (int)cudaGetLastError();
}

int d1_relpos_attn_error(void) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_rp_err, sizeof(int)) != cudaSuccess) return -1;
    if (v) {
        const int z = 0;
        cudaMemcpyToSymbol(g_rp_err, &z, sizeof(int));
    }
    return v;
}

}  // extern "C"

// ================================================================================================ log-mel front end
// src/audio.rs:238-299 (the reference computes it on the host) on the GPU, in the reference's precision and
// operation order: fp32 pre-emphasis y[i] = x[i] - 0.97 x[i-1]; 512-sample frames centred every 160 samples (zero
// outside the clip) times a 400-point Hann window centred in the frame (f64); an iterative radix-2 FFT in f64 with
// the same bit-reversal, twiddle table (e^{-2 pi i k / 512}) and butterfly expressions; power spectrum rounded to
// fp32; 128 Slaney mel filters summed in fp32 over each filter's nonzero bins in order; ln(s + 2^-24); then each mel
// channel normalised over the valid frames with f64 mean and unbiased std (std + 1e-5), frames past `valid` zero.
// Explicit _rn intrinsics keep the compiler from contracting multiply-adds the reference evaluates separately.
// Everything per frame follows the reference's order; the channel statistics are f64 sums taken in 8 interleaved
// parts (the reference sums the frames in sequence), a difference at f64 rounding level.

namespace {

constexpr int MEL_NFFT = 512, MEL_HOP = 160, MEL_WIN = 400, MEL_N = 128, MEL_NB = MEL_NFFT / 2 + 1;

__device__ double g_mel_tw[MEL_NFFT];      // (cos, sin) pairs of -2 pi k / 512, k < 256
__device__ double g_mel_win[MEL_NFFT];
__device__ float g_mel_fb[MEL_N * MEL_NB];
__device__ int g_mel_rng[MEL_N * 2];        // nonzero bin range [lo, hi) per filter

__global__ void __launch_bounds__(256) k_mel_frames(const float* __restrict__ x, int n, float* __restrict__ out) {
    __shared__ double re[MEL_NFFT], im[MEL_NFFT];
    __shared__ float pw[MEL_NB];
    const int f = blockIdx.x, tid = threadIdx.x;
    for (int i = tid; i < MEL_NFFT; i += 256) {
        const long si = (long)f * MEL_HOP + i - MEL_NFFT / 2;
        float y = 0.f;
        if (si >= 0 && si < n) y = si == 0 ? x[0] : __fsub_rn(x[si], __fmul_rn(0.97f, x[si - 1]));
        const int r = (int)(__brev((unsigned)i) >> (32 - 9));
        re[r] = __dmul_rn((double)y, g_mel_win[i]);
        im[r] = 0.0;
    }
    __syncthreads();
    for (int len = 2; len <= MEL_NFFT; len <<= 1) {
        const int half = len >> 1, step = MEL_NFFT / len;
        const int b = tid;  // 256 butterflies per stage, one per thread
        const int a = (b / half) * len + (b % half), c = a + half, k = b % half;
        const double wr = g_mel_tw[2 * (k * step)], wi = g_mel_tw[2 * (k * step) + 1];
        const double xr = __dsub_rn(__dmul_rn(re[c], wr), __dmul_rn(im[c], wi));
        const double xi = __dadd_rn(__dmul_rn(re[c], wi), __dmul_rn(im[c], wr));
        const double ar = re[a], ai = im[a];
        re[c] = __dsub_rn(ar, xr);
        im[c] = __dsub_rn(ai, xi);
        re[a] = __dadd_rn(ar, xr);
        im[a] = __dadd_rn(ai, xi);
        __syncthreads();
    }
    for (int kk = tid; kk < MEL_NB; kk += 256)
        pw[kk] = __double2float_rn(__dadd_rn(__dmul_rn(re[kk], re[kk]), __dmul_rn(im[kk], im[kk])));
    __syncthreads();
    if (tid < MEL_N) {
        float s = 0.f;
        const int lo = g_mel_rng[2 * tid], hi = g_mel_rng[2 * tid + 1];
        for (int kk = lo; kk < hi; kk++) s = __fadd_rn(s, __fmul_rn(g_mel_fb[tid * MEL_NB + kk], pw[kk]));
        out[(size_t)f * MEL_N + tid] = logf(__fadd_rn(s, 5.9604644775390625e-8f));  // 2^-24
    }
}

// Per-channel normalisation over the valid frames. CTA g owns channels [8g, 8g + 8): thread (part, channel) of its
// first 64 sums the frames f = part (mod 8) in f64 and the 8 partial sums are combined in part order (the reference
// sums frames sequentially in f64; the orders differ by f64 rounding only, ~1e-16 relative), then all 256 threads
// normalise the CTA's channels over every frame. 16 CTAs instead of one: the f64 divides and the 3 passes over the
// features spread over 16 SMs.
constexpr int MEL_PARTS = 8;
constexpr int MEL_CH = 8;  // channels per CTA

__global__ void __launch_bounds__(256) k_mel_norm(float* __restrict__ mel, int frames, int valid) {
    __shared__ double part_sum[MEL_PARTS][MEL_CH];
    __shared__ double stat[2][MEL_CH];  // mean, std + 1e-5
    const int c0 = blockIdx.x * MEL_CH;
    const int lc = threadIdx.x % MEL_CH, part = threadIdx.x / MEL_CH;  // stats: threads 0 .. 63
    const bool stats = threadIdx.x < MEL_CH * MEL_PARTS;
    double acc = 0.0;
    if (stats) {
#pragma unroll 4
        for (int f = part; f < valid; f += MEL_PARTS) acc = __dadd_rn(acc, (double)mel[(size_t)f * MEL_N + c0 + lc]);
        part_sum[part][lc] = acc;
    }
    __syncthreads();
    if (threadIdx.x < MEL_CH) {
        double t = 0.0;
        for (int q = 0; q < MEL_PARTS; q++) t = __dadd_rn(t, part_sum[q][lc]);
        stat[0][lc] = __ddiv_rn(t, (double)valid);
    }
    __syncthreads();
    if (stats) {
        const double mean = stat[0][lc];
        acc = 0.0;
#pragma unroll 4
        for (int f = part; f < valid; f += MEL_PARTS) {
            const double d = __dsub_rn((double)mel[(size_t)f * MEL_N + c0 + lc], mean);
            acc = __dadd_rn(acc, __dmul_rn(d, d));
        }
    }
    __syncthreads();
    if (stats) part_sum[part][lc] = acc;
    __syncthreads();
    if (threadIdx.x < MEL_CH) {
        double t = 0.0;
        for (int q = 0; q < MEL_PARTS; q++) t = __dadd_rn(t, part_sum[q][lc]);
        double sd = sqrt(__ddiv_rn(t, __dsub_rn((double)valid, 1.0)));
        if (isnan(sd)) sd = 0.0;
        stat[1][lc] = __dadd_rn(sd, 1e-5);
    }
    __syncthreads();
    for (size_t i = threadIdx.x; i < (size_t)frames * MEL_CH; i += blockDim.x) {
        const int c = (int)(i % MEL_CH);
        const int f = (int)(i / MEL_CH);
        float* p = mel + (size_t)f * MEL_N + c0 + c;
        *p = f < valid ? __double2float_rn(__ddiv_rn(__dsub_rn((double)*p, stat[0][c]), stat[1][c])) : 0.f;
    }
}

// Host tables, as src/audio.rs:151-205 builds them (f64 math, Slaney scale, area normalisation).
struct MelTables {
    double tw[MEL_NFFT], win[MEL_NFFT];
    float fb[MEL_N * MEL_NB];
    int rng[MEL_N * 2];
    MelTables() {
        const double PI = 3.14159265358979323846;
        for (int k = 0; k < MEL_NFFT / 2; k++) {
            const double a = -2.0 * PI * (double)k / (double)MEL_NFFT;
            tw[2 * k] = cos(a);
            tw[2 * k + 1] = sin(a);
        }
        for (int i = 0; i < MEL_NFFT; i++) win[i] = 0.0;
        const int off = (MEL_NFFT - MEL_WIN) / 2;
        for (int i = 0; i < MEL_WIN; i++) win[off + i] = 0.5 - 0.5 * cos(2.0 * PI * (double)i / (double)(MEL_WIN - 1));
        const double f_sp = 200.0 / 3.0, min_log_hz = 1000.0, logstep = log(6.4) / 27.0;
        const double min_log_mel = min_log_hz / f_sp;
        auto hz_to_mel = [&](double f) { return f >= min_log_hz ? min_log_mel + log(f / min_log_hz) / logstep : f / f_sp; };
        auto mel_to_hz = [&](double m) { return m >= min_log_mel ? min_log_hz * exp(logstep * (m - min_log_mel)) : f_sp * m; };
        const double m0 = hz_to_mel(0.0), m1 = hz_to_mel(16000.0 / 2.0);
        double mel_f[MEL_N + 2];
        for (int i = 0; i < MEL_N + 2; i++) mel_f[i] = mel_to_hz(m0 + (m1 - m0) * (double)i / (double)(MEL_N + 1));
        for (int i = 0; i < MEL_N; i++) {
            const double fd0 = mel_f[i + 1] - mel_f[i], fd1 = mel_f[i + 2] - mel_f[i + 1];
            const double enorm = 2.0 / (mel_f[i + 2] - mel_f[i]);
            int lo = -1, hi = 0;
            for (int j = 0; j < MEL_NB; j++) {
                const double f = (double)j * 16000.0 / (double)MEL_NFFT;
                const double lower = -(mel_f[i] - f) / fd0, upper = (mel_f[i + 2] - f) / fd1;
                const float v = (float)std::max(std::min(lower, upper), 0.0);
                fb[i * MEL_NB + j] = v * (float)enorm;
                if (fb[i * MEL_NB + j] != 0.f) {
                    if (lo < 0) lo = j;
                    hi = j + 1;
                }
            }
            if (lo < 0) lo = 0;
            rng[2 * i] = lo;
            rng[2 * i + 1] = std::max(hi, lo);
        }
    }
};

int mel_tables_ready() {
    static unsigned long long done = 0;  // one bit per device
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (__atomic_load_n(&done, __ATOMIC_ACQUIRE) & bit) return 0;
    static const MelTables t;
    if (cudaMemcpyToSymbol(g_mel_tw, t.tw, sizeof(t.tw)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_mel_win, t.win, sizeof(t.win)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_mel_fb, t.fb, sizeof(t.fb)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_mel_rng, t.rng, sizeof(t.rng)) != cudaSuccess)
        return -1;
    __atomic_fetch_or(&done, bit, __ATOMIC_RELEASE);
    return 0;
}

}  // namespace

extern "C" int d1_log_mel(const float* x, int n, float* mel, cudaStream_t st) {
    if (!x || !mel || n < 1) return -1;
    if (mel_tables_ready()) return -1;
    const int frames = 1 + n / MEL_HOP, valid = n / MEL_HOP;
    k_mel_frames<<<frames, 256, 0, st>>>(x, n, mel);
    k_mel_norm<<<MEL_N / MEL_CH, 256, 0, st>>>(mel, frames, valid);
    return (int)cudaGetLastError();
}

// ================================================================================================ resampler
// d1_resample — the WAV front end's sample-rate conversion to 16 kHz (src/audio.rs:108-148, host code in the
// reference) on the GPU. A polyphase Kaiser-windowed sinc filter: output n reads input position n * down / up
// (up / down = dst / src reduced by their gcd), phase p = (n * down) % up, taps at inputs base - half .. base + half
// with base = n * down / up; cutoff = min(up / down, 1) * 0.97, half = ceil(32 / cutoff), Kaiser beta 8.6.
// The filter table [up][2*half+1] is evaluated on the host in f64 exactly as the reference's tap() does (its
// zeroth-order Bessel series, its operation order) and rounded to fp32, once per (device, rate pair), then kept on
// the device. The sum per output runs over the taps in order, skipping inputs outside the clip, as fp32 products
// added to an fp32 accumulator (the reference's Rust does not fuse them), so the result is bit-identical.
// A CTA computes 256 consecutive outputs from the input window they share, staged in shared memory.
namespace {

struct RsTable {
    int up = 0, down = 0, half = 0;
    float* d_table = nullptr;
};

bool rs_plan(int from, int to, int& up, int& down, int& half, double& cutoff) {
    if (from <= 0 || to <= 0) return false;
    int a = from, b = to;
    while (b) {
        const int t = a % b;
        a = b;
        b = t;
    }
    up = to / a;
    down = from / a;
    cutoff = std::min((double)up / (double)down, 1.0) * 0.97;
    half = (int)std::ceil(32.0 / cutoff);
    return true;
}

double rs_bessel_i0(double x) {  // src/audio.rs:97-104
    double s = 1.0, t = 1.0;
    for (int k = 1; k < 50; k++) {
        const double y = x / (2.0 * (double)k);
        t *= y * y;
        s += t;
    }
    return s;
}

// The device table for (from, to) on the current device, built on first use (host f64 evaluation + one upload).
const RsTable* rs_table(int from, int to) {
    static std::mutex mu;
    static std::map<std::tuple<int, int, int>, RsTable> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_tuple(dev, from, to);
    auto it = cache.find(key);
    if (it != cache.end()) return &it->second;
    RsTable t;
    double cutoff = 0.0;
    if (!rs_plan(from, to, t.up, t.down, t.half, cutoff)) return nullptr;
    const int taps = 2 * t.half + 1;
    if ((long long)t.up * taps > (64ll << 20)) return nullptr;  // rates with no small common divisor
    const double beta = 8.6, i0b = rs_bessel_i0(beta), pi = 3.14159265358979323846;
    std::vector<float> h((size_t)t.up * taps);
    for (int p = 0; p < t.up; p++) {
        const double frac = (double)p / (double)t.up;
        for (int j = 0; j < taps; j++) {
            const double tt = (double)(j - t.half) - frac;
            const double r = tt / (double)t.half;
            double v = 0.0;
            if (std::fabs(r) < 1.0) {
                const double sinc = tt == 0.0 ? 1.0 : std::sin(pi * tt * cutoff) / (pi * tt * cutoff);
                v = cutoff * sinc * rs_bessel_i0(beta * std::sqrt(1.0 - r * r)) / i0b;
            }
            h[(size_t)p * taps + j] = (float)v;
        }
    }
    if (cudaMalloc(&t.d_table, h.size() * sizeof(float)) != cudaSuccess) return nullptr;
    if (cudaMemcpy(t.d_table, h.data(), h.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(t.d_table);
        return nullptr;
    }
    return &(cache[key] = t);
}

constexpr int kRsOut = 256;  // outputs per CTA

__global__ void __launch_bounds__(kRsOut) k_resample(const float* __restrict__ x, int n,
                                                     const float* __restrict__ table, int up, int down, int half,
                                                     float* __restrict__ y, int n_out, int win_cap) {
    extern __shared__ float win[];
    const int o0 = blockIdx.x * kRsOut;
    const long long first = (long long)o0 * down / up - half;  // first input the CTA's outputs read
    const int o_last = min(o0 + kRsOut, n_out) - 1;
    const long long last = (long long)o_last * down / up + half;
    const int len = (int)(last - first + 1);
    for (int i = threadIdx.x; i < len && i < win_cap; i += blockDim.x) {
        const long long g = first + i;
        win[i] = (g >= 0 && g < n) ? x[g] : 0.f;
    }
    __syncthreads();
    const int o = o0 + threadIdx.x;
    if (o >= n_out) return;
    const long long pos = (long long)o * down;
    const long long base = pos / up;
    const int ph = (int)(pos - base * up), taps = 2 * half + 1;
    const float* w = table + (size_t)ph * taps;
    // inputs base - half + j inside [0, n): the taps the reference does not skip
    const int j0 = (int)max(0ll, (long long)half - base), j1 = (int)min((long long)taps, (long long)n - base + half);
    const int off = (int)(base - half - first);
    float acc = 0.f;
    for (int j = j0; j < j1; j++) acc = __fadd_rn(acc, __fmul_rn(__ldg(w + j), win[off + j]));
    y[o] = acc;
}

}  // namespace

extern "C" int d1_resample_len(int n, int from, int to) {
    int up, down, half;
    double cutoff;
    if (n < 0 || !rs_plan(from, to, up, down, half, cutoff)) return -1;
    if (from == to) return n;
    return (int)((long long)n * up / down);
}

extern "C" int d1_resample(const float* x, int n, int from, int to, float* y, cudaStream_t st) {
    const int n_out = d1_resample_len(n, from, to);
    if (n_out < 0 || (n > 0 && (!x || !y))) return -1;
    if (n_out == 0) return 0;
    if (from == to) return cudaMemcpyAsync(y, x, (size_t)n * sizeof(float), cudaMemcpyDeviceToDevice, st) ? -1 : 0;
    const RsTable* t = rs_table(from, to);
    if (!t) return -1;
    // shared-memory window: the inputs of 256 consecutive outputs plus the taps on both sides
    const int win_cap = (int)((long long)kRsOut * t->down / t->up + 2 * t->half + 2);
    if ((size_t)win_cap * sizeof(float) > 48 * 1024) return -1;
    const int grid = (n_out + kRsOut - 1) / kRsOut;
    k_resample<<<grid, kRsOut, (size_t)win_cap * sizeof(float), st>>>(x, n, t->d_table, t->up, t->down, t->half, y,
                                                                       n_out, win_cap);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
