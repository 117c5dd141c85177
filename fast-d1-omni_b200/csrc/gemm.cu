// Projection GEMMs of the d1rs forward pass on 5th-generation tensor cores (tcgen05, sm_100a).
//
// Replaces the cuBLASLt autotuner of the reference (cuda/gemm.cu) behind the same C ABI (d1_lt_*), plus two
// fused forms (SwiGLU and bias+activation epilogues) that remove the separate elementwise launches the
// reference makes after its GEMMs (src/model.rs:394-395, :568-569; src/vision.rs:364-365).
//
// Semantics (cuda/gemm.cu:8): row-major Y[M,N] = alpha * X[M,K] . W^T + beta * Y, W = nn.Linear weight [N,K].
//
// Kernel design: a persistent, warp-specialised kernel with one CTA per SM.
//   warp 0      TMA producer: 128x64 A tiles and BNx64 B tiles (fp16, 128-byte swizzle) into a STAGES-deep
//               shared-memory ring, completion tracked by mbarrier transaction counts.
//   warp 1      allocates TMEM (2 x BN fp32 columns: a double-buffered 128 x BN accumulator); one thread
//               issues tcgen05.mma (M=128, N=BN, K=16) and releases ring slots with tcgen05.commit.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (each warp owns the 32 TMEM lanes = rows it may
//               access), the fused epilogue in registers, and stores to global memory. The double-buffered
//               accumulator lets the epilogue of one tile overlap the main loop of the next.
// Every mbarrier wait is bounded in time: on expiry the kernel records an error code in the context's device
// error word and returns instead of hanging.
#include <stdio.h>
#include <string.h>

#include <map>
#include <mutex>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "common.cuh"

using namespace d1;

namespace {

constexpr int BM = 128;           // rows of A per tile (tcgen05 M)
constexpr int BK = 64;            // K per ring stage: 64 fp16 = one 128-byte swizzle row
constexpr int kThreads = 192;     // 6 warps
constexpr int A_BYTES = BM * BK * 2;

enum Epi : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_BIAS_ACT = 2 };

struct GemmArgs {
    int M, N, K;          // N: accumulator columns in total (2F for SwiGLU)
    int num_m, num_n;     // tile grid
    int num_tiles, num_kb;
    void* Y;
    int ldy;
    int y_f32;
    int vec;              // 16-byte aligned rows of Y: vector stores allowed
    float alpha, beta;
    const float* bias;
    int act;
    int F;                // SwiGLU: output columns (rows [0,F) of W are gate, [F,2F) up)
    int* err;
};

template <int BN, int STAGES>
struct Smem {
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RING = STAGES * STAGE_BYTES;
    static constexpr int NBARS = 2 * STAGES + 5;
    static constexpr size_t BYTES = 1024 /* alignment slack */ + RING + NBARS * 8 + 16;
};

__device__ __forceinline__ void record_error(int* err, volatile int* abort_flag, int code) {
    *abort_flag = 1;
    if (err) atomicExch(err, code);
}

// Wait bounded by time only (used when draining on the way out).
__device__ __forceinline__ bool mbar_wait_timed(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    return true;
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// ---------------------------------------------------------------------------------------------- epilogues

// Y = alpha * acc + beta * Y (beta == 0: Y is not read), fp16 or fp32 Y.
template <int BN>
__device__ __forceinline__ void epi_store(const GemmArgs& a, uint32_t tbase, int row, int n0) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tbase + c0, r);
        tc_wait_ld();
        const int col = n0 + c0;
        if (row >= a.M || col >= a.N) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = a.alpha * __uint_as_float(r[i]);
        const bool full = a.vec && col + 32 <= a.N;
        if (a.y_f32) {
            float* y = reinterpret_cast<float*>(a.Y) + (size_t)row * a.ldy + col;
            if (full) {
                float4* y4 = reinterpret_cast<float4*>(y);
                if (a.beta != 0.f) {
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        float4 o = y4[i];
                        v[4 * i] += a.beta * o.x;
                        v[4 * i + 1] += a.beta * o.y;
                        v[4 * i + 2] += a.beta * o.z;
                        v[4 * i + 3] += a.beta * o.w;
                    }
                }
#pragma unroll
                for (int i = 0; i < 8; i++) y4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            } else {
                for (int i = 0; i < 32 && col + i < a.N; i++) y[i] = v[i] + (a.beta != 0.f ? a.beta * y[i] : 0.f);
            }
        } else {
            __half* y = reinterpret_cast<__half*>(a.Y) + (size_t)row * a.ldy + col;
            if (full) {
                uint4* y4 = reinterpret_cast<uint4*>(y);
                if (a.beta != 0.f) {
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        uint4 o = y4[i];
                        const __half2* h = reinterpret_cast<const __half2*>(&o);
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            float2 f = __half22float2(h[j]);
                            v[8 * i + 2 * j] += a.beta * f.x;
                            v[8 * i + 2 * j + 1] += a.beta * f.y;
                        }
                    }
                }
#pragma unroll
                for (int i = 0; i < 4; i++)
                    y4[i] = make_uint4(pack_h2(v[8 * i], v[8 * i + 1]), pack_h2(v[8 * i + 2], v[8 * i + 3]),
                                       pack_h2(v[8 * i + 4], v[8 * i + 5]), pack_h2(v[8 * i + 6], v[8 * i + 7]));
            } else {
                for (int i = 0; i < 32 && col + i < a.N; i++)
                    y[i] = __float2half_rn(v[i] + (a.beta != 0.f ? a.beta * __half2float(y[i]) : 0.f));
            }
        }
    }
}

// out[row][c] = silu(g) * u with g, u the fp16-rounded gate and up accumulators (as the reference's GEMM writes
// fp16 and k_swiglu, cuda/kernels.cu:159-168, reads it back). Accumulator columns [0, BN/2) hold gate rows
// [n0, n0+BN/2) of W and [BN/2, BN) the matching up rows [F+n0, ...).
template <int BN>
__device__ __forceinline__ void epi_swiglu(const GemmArgs& a, uint32_t tbase, int row, int n0) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN / 2; c0 += 32) {
        uint32_t g[32], u[32];
        tmem_ld32(tbase + c0, g);
        tmem_ld32(tbase + BN / 2 + c0, u);
        tc_wait_ld();
        const int col = n0 + c0;
        if (row >= a.M || col >= a.F) continue;
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) v[i] = silu(round_h(__uint_as_float(g[i]))) * round_h(__uint_as_float(u[i]));
        __half* y = reinterpret_cast<__half*>(a.Y) + (size_t)row * a.ldy + col;
        if (a.vec && col + 32 <= a.F) {
            uint4* y4 = reinterpret_cast<uint4*>(y);
#pragma unroll
            for (int i = 0; i < 4; i++)
                y4[i] = make_uint4(pack_h2(v[8 * i], v[8 * i + 1]), pack_h2(v[8 * i + 2], v[8 * i + 3]),
                                   pack_h2(v[8 * i + 4], v[8 * i + 5]), pack_h2(v[8 * i + 6], v[8 * i + 7]));
        } else {
            for (int i = 0; i < 32 && col + i < a.F; i++) y[i] = __float2half_rn(v[i]);
        }
    }
}

// Y = act(half(acc) + bias), fp16 (the reference's fp16 GEMM output followed by k_bias_act_h,
// cuda/kernels.cu:171-184).
template <int BN>
__device__ __forceinline__ void epi_bias_act(const GemmArgs& a, uint32_t tbase, int row, int n0) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tbase + c0, r);
        tc_wait_ld();
        const int col = n0 + c0;
        if (row >= a.M || col >= a.N) continue;
        float v[32];
        const bool full = a.vec && col + 32 <= a.N;
        if (full) {
            const float4* b4 = reinterpret_cast<const float4*>(a.bias + col);
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float4 b = a.bias ? __ldg(b4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
                v[4 * i] = apply_act(round_h(__uint_as_float(r[4 * i])) + b.x, a.act);
                v[4 * i + 1] = apply_act(round_h(__uint_as_float(r[4 * i + 1])) + b.y, a.act);
                v[4 * i + 2] = apply_act(round_h(__uint_as_float(r[4 * i + 2])) + b.z, a.act);
                v[4 * i + 3] = apply_act(round_h(__uint_as_float(r[4 * i + 3])) + b.w, a.act);
            }
            uint4* y4 = reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.Y) + (size_t)row * a.ldy + col);
#pragma unroll
            for (int i = 0; i < 4; i++)
                y4[i] = make_uint4(pack_h2(v[8 * i], v[8 * i + 1]), pack_h2(v[8 * i + 2], v[8 * i + 3]),
                                   pack_h2(v[8 * i + 4], v[8 * i + 5]), pack_h2(v[8 * i + 6], v[8 * i + 7]));
        } else {
            __half* y = reinterpret_cast<__half*>(a.Y) + (size_t)row * a.ldy + col;
            for (int i = 0; i < 32 && col + i < a.N; i++)
                y[i] = __float2half_rn(apply_act(round_h(__uint_as_float(r[i])) + (a.bias ? a.bias[col + i] : 0.f), a.act));
        }
    }
}

// ---------------------------------------------------------------------------------------------- the kernel

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmArgs a) {
    using S = Smem<BN, STAGES>;
    constexpr uint32_t TMEM_COLS = 2 * BN;
    constexpr uint32_t IDESC = idesc_f16_f32(BM, BN);
    static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "tcgen05 M=128 needs N % 16 == 0, 16..256");
    static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocations are powers of 2");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::RING);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + S::NBARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    auto sA = [&](int s) { return smem_u32(smem + s * S::STAGE_BYTES); };
    auto sB = [&](int s) { return smem_u32(smem + s * S::STAGE_BYTES + A_BYTES); };
    auto full_bar = [&](int s) { return smem_u32(bars + s); };
    auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
    auto accf_bar = [&](int i) { return smem_u32(bars + 2 * STAGES + i); };
    auto acce_bar = [&](int i) { return smem_u32(bars + 2 * STAGES + 2 + i); };
    const uint32_t drain_bar = smem_u32(bars + 2 * STAGES + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(accf_bar(0), 1);
        mbar_init(accf_bar(1), 1);
        mbar_init(acce_bar(0), 4);
        mbar_init(acce_bar(1), 4);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued = 0, issued_par = 0;
            bool aborted = false;
            for (int tile = blockIdx.x; tile < a.num_tiles && !aborted; tile += gridDim.x) {
                const int m_blk = tile % a.num_m, n_blk = tile / a.num_m;
                for (int kb = 0; kb < a.num_kb; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag)) {
                        record_error(a.err, abort_flag, kErrWaitEmpty);
                        aborted = true;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), S::STAGE_BYTES);
                    tma_load_2d(sA(stage), &tmA, kb * BK, m_blk * BM, full_bar(stage));
                    if (EPI == EPI_SWIGLU) {
                        tma_load_2d(sB(stage), &tmB, kb * BK, n_blk * (BN / 2), full_bar(stage));
                        tma_load_2d(sB(stage) + (BN / 2) * BK * 2, &tmB, kb * BK, a.F + n_blk * (BN / 2),
                                    full_bar(stage));
                    } else {
                        tma_load_2d(sB(stage), &tmB, kb * BK, n_blk * BN, full_bar(stage));
                    }
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Leave no copy in flight: each stage's last load has landed before the CTA may exit.
            for (int s = 0; s < STAGES; s++)
                if ((issued >> s) & 1)
                    if (!mbar_wait_timed(full_bar(s), (issued_par >> s) & 1)) record_error(a.err, abort_flag, kErrDrain);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int stage = 0, it = 0;
            uint32_t phase = 0;
            bool aborted = false;
            for (int tile = blockIdx.x; tile < a.num_tiles && !aborted; tile += gridDim.x, it++) {
                const int acc = it & 1;
                const uint32_t acc_par = (it >> 1) & 1;
                if (!mbar_wait(acce_bar(acc), acc_par ^ 1, abort_flag)) {
                    record_error(a.err, abort_flag, kErrWaitAccEmpty);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < a.num_kb; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
                        record_error(a.err, abort_flag, kErrWaitFull);
                        aborted = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sA(stage), b0 = sB(stage);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        tc_mma_f16(d_tmem, smem_desc_k128(a0 + k * 32), smem_desc_k128(b0 + k * 32), IDESC,
                                   (kb | k) != 0);
                    tc_commit(empty_bar(stage));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (aborted) break;
                tc_commit(accf_bar(acc));
            }
            // Every MMA this thread issued has completed before TMEM is released.
            tc_commit(drain_bar);
            if (!mbar_wait_timed(drain_bar, 0)) record_error(a.err, abort_flag, kErrDrain);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue (warps 2..5)
        const int sub = warp & 3;  // TMEM lane quarter this warp may access
        int it = 0;
        for (int tile = blockIdx.x; tile < a.num_tiles; tile += gridDim.x, it++) {
            const int acc = it & 1;
            const uint32_t acc_par = (it >> 1) & 1;
            const bool ok = __all_sync(D1_FULL_MASK, mbar_wait(accf_bar(acc), acc_par, abort_flag));
            if (!ok) {
                if (lane == 0) record_error(a.err, abort_flag, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            const int m_blk = tile % a.num_m, n_blk = tile / a.num_m;
            const int row = m_blk * BM + sub * 32 + lane;
            const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * BN);
            if (EPI == EPI_SWIGLU)
                epi_swiglu<BN>(a, tbase, row, n_blk * (BN / 2));
            else if (EPI == EPI_BIAS_ACT)
                epi_bias_act<BN>(a, tbase, row, n_blk * BN);
            else
                epi_store<BN>(a, tbase, row, n_blk * BN);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce_bar(acc));
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------------------- SIMT path
// General layouts the TMA path cannot take (W given as [K,N], strides that are not 16-byte multiples):
// a plain tiled CUDA-core GEMM, 64x64 tile, 4x4 outputs per thread. Not used by any shape of the forward pass.
__global__ void __launch_bounds__(256) k_gemm_simt(int M, int N, int K, const __half* __restrict__ X, int ldx,
                                                   const __half* __restrict__ W, int ldw, int w_kn, void* Y,
                                                   int ldy, int y_f32, float alpha, float beta) {
    __shared__ float sx[16][65];
    __shared__ float sw[16][65];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int r = i / 16, k = i % 16;
            const int m = m0 + r, n = n0 + r, kk = k0 + k;
            sx[k][r] = (m < M && kk < K) ? __half2float(X[(size_t)m * ldx + kk]) : 0.f;
            float wv = 0.f;
            if (n < N && kk < K) wv = __half2float(w_kn ? W[(size_t)kk * ldw + n] : W[(size_t)n * ldw + kk]);
            sw[k][r] = wv;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++)
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] += sx[k][ty * 4 + i] * sw[k][tx * 4 + j];
        __syncthreads();
    }
    for (int i = 0; i < 4; i++)
        for (int j = 0; j < 4; j++) {
            const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
            if (m >= M || n >= N) continue;
            float v = alpha * acc[i][j];
            if (y_f32) {
                float* y = reinterpret_cast<float*>(Y) + (size_t)m * ldy + n;
                *y = v + (beta != 0.f ? beta * *y : 0.f);
            } else {
                __half* y = reinterpret_cast<__half*>(Y) + (size_t)m * ldy + n;
                *y = __float2half_rn(v + (beta != 0.f ? beta * __half2float(*y) : 0.f));
            }
        }
}

__global__ void k_fill_pattern(__half* p, size_t n, uint32_t seed) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        uint32_t s = (uint32_t)i * 2654435761u + seed;
        s ^= s >> 13;
        s *= 0x5bd1e995u;
        s ^= s >> 15;
        p[i] = __float2half(((int)(s % 2000u) - 1000) * 1e-3f);
    }
}

// ---------------------------------------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

struct TmapKey {
    uintptr_t ptr;
    uint64_t inner, outer, stride;
    uint32_t box_inner, box_outer;
    bool operator==(const TmapKey& o) const {
        return ptr == o.ptr && inner == o.inner && outer == o.outer && stride == o.stride &&
               box_inner == o.box_inner && box_outer == o.box_outer;
    }
};
struct TmapHash {
    size_t operator()(const TmapKey& k) const {
        size_t h = k.ptr * 0x9E3779B97F4A7C15ull;
        h ^= k.inner + 0x9E3779B9 + (h << 6) + (h >> 2);
        h ^= k.outer + 0x9E3779B9 + (h << 6) + (h >> 2);
        h ^= k.stride + 0x9E3779B9 + (h << 6) + (h >> 2);
        h ^= ((uint64_t)k.box_inner << 32 | k.box_outer) + 0x9E3779B9 + (h << 6) + (h >> 2);
        return h;
    }
};

// Tile plan: which kernel configuration runs a shape (the analogue of the reference's cuBLASLt algo choice).
typedef std::tuple<int, int, int, int, int, int, int, int, int> PlanKey;  // N K ldx ldw ldy w_kn y_f32 epi bucket
struct Plan {
    int bn;
    float us;
};

struct Ctx {
    int dev = 0;
    int num_sms = 148;
    int* d_err = nullptr;
    std::unordered_map<TmapKey, CUtensorMap, TmapHash> tmaps;
    std::map<PlanKey, Plan> plans;
    uint32_t attr_done = 0;  // per kernel instance: max dynamic smem attribute set
    void* sx = nullptr;
    void* sw = nullptr;
    void* sy = nullptr;
    size_t sx_b = 0, sw_b = 0, sy_b = 0;
};

const int BUCKETS[] = {16,  32,  48,  64,   96,   128,  160,  192,  256,  320,  384,   512,
                       640, 768, 1024, 1280, 1536, 2048, 3072, 4096, 6144, 8192, 12288, 16384};
const int NBUCKETS = sizeof(BUCKETS) / sizeof(int);

int bucket_of(int m) {
    for (int i = 0; i < NBUCKETS; i++)
        if (m <= BUCKETS[i]) return BUCKETS[i];
    return BUCKETS[NBUCKETS - 1];
}

const CUtensorMap* get_tmap(Ctx* c, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
                            uint32_t box_inner, uint32_t box_outer) {
    TmapKey key{(uintptr_t)base, inner, outer, ld_elems * 2, box_inner, box_outer};
    auto it = c->tmaps.find(key);
    if (it != c->tmaps.end()) return &it->second;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return nullptr;
    CUtensorMap m;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld_elems * 2};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return nullptr;
    if (c->tmaps.size() > 4096) c->tmaps.clear();
    return &c->tmaps.emplace(key, m).first->second;
}

bool tc_ok(const void* X, int ldx, const void* W, int ldw, int w_kn, int K) {
    return !w_kn && K >= 1 && ldx % 8 == 0 && ldw % 8 == 0 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0;
}

template <int BN, int STAGES, int EPI>
int launch_tc(Ctx* c, int bit, const void* X, int ldx, const void* W, int ldw, int w_rows, GemmArgs& a,
              cudaStream_t st) {
    using S = Smem<BN, STAGES>;
    auto kern = k_gemm_tc<BN, STAGES, EPI>;
    if (!(c->attr_done & (1u << bit))) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::BYTES) != cudaSuccess)
            return -1;
        c->attr_done |= 1u << bit;
    }
    const uint32_t b_rows = EPI == EPI_SWIGLU ? BN / 2 : BN;
    const CUtensorMap* ta = get_tmap(c, X, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)ldx, BK, BM);
    const CUtensorMap* tb = get_tmap(c, W, (uint64_t)a.K, (uint64_t)w_rows, (uint64_t)ldw, BK, b_rows);
    if (!ta || !tb) return -1;
    a.num_m = (a.M + BM - 1) / BM;
    a.num_n = EPI == EPI_SWIGLU ? (a.F + BN / 2 - 1) / (BN / 2) : (a.N + BN - 1) / BN;
    a.num_tiles = a.num_m * a.num_n;
    a.num_kb = (a.K + BK - 1) / BK;
    a.err = c->d_err;
    const int grid = a.num_tiles < c->num_sms ? a.num_tiles : c->num_sms;
    kern<<<grid, kThreads, S::BYTES, st>>>(*ta, *tb, a);
    return (int)cudaGetLastError();
}

// Wave efficiency of a tile count over the SMs.
double wave_eff(long tiles, int sms) {
    long waves = (tiles + sms - 1) / sms;
    return (double)tiles / (double)(waves * sms);
}

int default_bn(Ctx* c, int M, int N) {
    const long mt = (M + BM - 1) / BM;
    const double e256 = wave_eff(mt * ((N + 255) / 256), c->num_sms) * (double)N / (double)(((N + 255) / 256) * 256);
    const double e128 = wave_eff(mt * ((N + 127) / 128), c->num_sms) * (double)N / (double)(((N + 127) / 128) * 128);
    return e128 > e256 + 0.08 ? 128 : 256;
}

int run_store(Ctx* c, int bn, int M, int N, int K, const void* X, int ldx, const void* W, int ldw, void* Y, int ldy,
              int y_f32, float alpha, float beta, cudaStream_t st) {
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.y_f32 = y_f32;
    a.vec = ((uintptr_t)Y % 16 == 0) && ((size_t)ldy * (y_f32 ? 4 : 2)) % 16 == 0;
    a.alpha = alpha;
    a.beta = beta;
    if (bn == 128) return launch_tc<128, 6, EPI_STORE>(c, 0, X, ldx, W, ldw, N, a, st);
    return launch_tc<256, 4, EPI_STORE>(c, 1, X, ldx, W, ldw, N, a, st);
}

int run_simt(int M, int N, int K, const void* X, int ldx, const void* W, int ldw, int w_kn, void* Y, int ldy,
             int y_f32, float alpha, float beta, cudaStream_t st) {
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    k_gemm_simt<<<grid, 256, 0, st>>>(M, N, K, (const __half*)X, ldx, (const __half*)W, ldw, w_kn, Y, ldy, y_f32,
                                      alpha, beta);
    return (int)cudaGetLastError();
}

void ensure(void** p, size_t* have, size_t need, uint32_t seed) {
    if (*have >= need) return;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    if (cudaMalloc(p, need) != cudaSuccess) {
        *p = nullptr;
        return;
    }
    *have = need;
    k_fill_pattern<<<1024, 256>>>((__half*)*p, need / 2, seed);
    cudaDeviceSynchronize();
}

}  // namespace

// ================================================================================================ C ABI
extern "C" {

const char* d1_build_id(void) { return "d1b200-tc-gemm-v1"; }

void* d1_lt_init(size_t ws_bytes) {
    (void)ws_bytes;
    Ctx* c = new Ctx();
    if (cudaGetDevice(&c->dev) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->dev);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, c->dev);
    if (major != 10 || !encode_fn()) {  // sm_100a code only
        delete c;
        return nullptr;
    }
    if (cudaMalloc(&c->d_err, 16) != cudaSuccess || cudaMemset(c->d_err, 0, 16) != cudaSuccess) {
        delete c;
        return nullptr;
    }
    return c;
}

void d1_lt_destroy(void* ctx) {
    Ctx* c = (Ctx*)ctx;
    if (!c) return;
    d1_lt_free_scratch(ctx);
    if (c->d_err) cudaFree(c->d_err);
    delete c;
}

int d1_lt_error(void* ctx) {
    Ctx* c = (Ctx*)ctx;
    if (!c) return -1;
    int e = 0;
    if (cudaMemcpy(&e, c->d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (e) cudaMemset(c->d_err, 0, sizeof(int));
    return e;
}

int d1_lt_gemm(void* ctx, int M, int N, int K, const void* X, int ldx, const void* W, int ldw, int w_kn, void* Y,
               int ldy, int y_f32, int f16acc, float alpha, float beta, cudaStream_t st) {
    (void)f16acc;
    Ctx* c = (Ctx*)ctx;
    if (!c || M < 0 || N < 0 || K < 0) return -1;
    if (M == 0 || N == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, w_kn, K))
        return run_simt(M, N, K, X, ldx, W, ldw, w_kn, Y, ldy, y_f32, alpha, beta, st) ? -1 : 0;
    int bn;
    auto it = c->plans.find(PlanKey(N, K, ldx, ldw, ldy, w_kn, y_f32, EPI_STORE, bucket_of(M)));
    bn = it != c->plans.end() ? it->second.bn : default_bn(c, M, N);
    return run_store(c, bn, M, N, K, X, ldx, W, ldw, Y, ldy, y_f32, alpha, beta, st) ? -1 : 0;
}

int d1_gemm_swiglu(void* ctx, int M, int F, int K, const d1_half* X, int ldx, const d1_half* W, int ldw,
                   d1_half* out, int ldo, cudaStream_t st) {
    Ctx* c = (Ctx*)ctx;
    if (!c || M < 0 || F <= 0 || K <= 0) return M == 0 ? 0 : -1;
    if (M == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, 0, K)) return -1;
    GemmArgs a{};
    a.M = M;
    a.N = 2 * F;
    a.K = K;
    a.F = F;
    a.Y = out;
    a.ldy = ldo;
    a.vec = ((uintptr_t)out % 16 == 0) && (ldo % 8 == 0);
    a.alpha = 1.f;
    return launch_tc<256, 4, EPI_SWIGLU>(c, 2, X, ldx, W, ldw, 2 * F, a, st) ? -1 : 0;
}

int d1_gemm_bias_act(void* ctx, int M, int N, int K, const d1_half* X, int ldx, const d1_half* W, int ldw,
                     const float* bias, int act, d1_half* Y, int ldy, cudaStream_t st) {
    Ctx* c = (Ctx*)ctx;
    if (!c || M < 0 || N < 0 || K <= 0 || act < 0 || act > 4) return -1;
    if (M == 0 || N == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, 0, K)) return -1;
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.vec = ((uintptr_t)Y % 16 == 0) && (ldy % 8 == 0) && ((uintptr_t)bias % 16 == 0);
    a.alpha = 1.f;
    a.bias = bias;
    a.act = act;
    if (default_bn(c, M, N) == 128) return launch_tc<128, 6, EPI_BIAS_ACT>(c, 3, X, ldx, W, ldw, N, a, st) ? -1 : 0;
    return launch_tc<256, 4, EPI_BIAS_ACT>(c, 4, X, ldx, W, ldw, N, a, st) ? -1 : 0;
}

float d1_lt_tune(void* ctx, int M, int N, int K, int ldx, int ldw, int w_kn, int ldy, int y_f32, int f16acc,
                 int effort, cudaStream_t st) {
    (void)f16acc;
    (void)effort;
    Ctx* c = (Ctx*)ctx;
    if (!c || M <= 0 || N <= 0 || K <= 0) return -1.f;
    const int bm = bucket_of(M);
    PlanKey key(N, K, ldx, ldw, ldy, w_kn, y_f32, EPI_STORE, bm);
    auto it = c->plans.find(key);
    if (it != c->plans.end()) return it->second.us;
    M = bm;
    ensure(&c->sx, &c->sx_b, (size_t)M * ldx * 2 + 256, 1);
    ensure(&c->sw, &c->sw_b, (size_t)(w_kn ? K : N) * ldw * 2 + 256, 2);
    ensure(&c->sy, &c->sy_b, (size_t)M * ldy * 4 + 256, 3);
    if (!c->sx || !c->sw || !c->sy) return -1.f;
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const int reps = M >= 4096 ? 5 : M >= 1024 ? 10 : 20;
    float best = 1e30f;
    int best_bn = 256;
    const bool tc = tc_ok(c->sx, ldx, c->sw, ldw, w_kn, K);
    for (int bn : {128, 256}) {
        auto run = [&]() {
            return tc ? run_store(c, bn, M, N, K, c->sx, ldx, c->sw, ldw, c->sy, ldy, y_f32, 1.f, 0.f, st)
                      : run_simt(M, N, K, c->sx, ldx, c->sw, ldw, w_kn, c->sy, ldy, y_f32, 1.f, 0.f, st);
        };
        if (run() || run()) continue;
        cudaEventRecord(e0, st);
        for (int i = 0; i < reps; i++) run();
        cudaEventRecord(e1, st);
        cudaEventSynchronize(e1);
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        const float us = ms * 1000.f / reps;
        if (cudaGetLastError() == cudaSuccess && us < best) {
            best = us;
            best_bn = bn;
        }
        if (!tc) break;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (best >= 1e29f) return -1.f;
    c->plans[key] = Plan{best_bn, best};
    return best;
}

int d1_lt_save(void* ctx, const char* path) {
    Ctx* c = (Ctx*)ctx;
    FILE* f = fopen(path, "w");
    if (!f) return -1;
    fprintf(f, "d1b200-gemm-plans v1 %s\n", d1_build_id());
    for (auto& kv : c->plans) {
        int N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b;
        std::tie(N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b) = kv.first;
        fprintf(f, "%d %d %d %d %d %d %d %d %d %d %.2f\n", N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b, kv.second.bn,
                kv.second.us);
    }
    fclose(f);
    return 0;
}

int d1_lt_load(void* ctx, const char* path) {
    Ctx* c = (Ctx*)ctx;
    FILE* f = fopen(path, "r");
    if (!f) return -1;
    char tag[64], ver[16], id[128];
    if (fscanf(f, "%63s %15s %127s\n", tag, ver, id) != 3 || strcmp(id, d1_build_id()) != 0) {
        fclose(f);
        return -2;
    }
    int n = 0;
    while (true) {
        int N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b, bn;
        float us;
        if (fscanf(f, "%d %d %d %d %d %d %d %d %d %d %f", &N, &K, &ldx, &ldw, &ldy, &w_kn, &y_f32, &epi, &b, &bn,
                   &us) != 11)
            break;
        if (bn != 128 && bn != 256) continue;
        c->plans[PlanKey(N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b)] = Plan{bn, us};
        n++;
    }
    fclose(f);
    return n;
}

int d1_lt_bucket(int m) { return bucket_of(m); }

void d1_lt_free_scratch(void* ctx) {
    Ctx* c = (Ctx*)ctx;
    if (!c) return;
    for (void** p : {&c->sx, &c->sw, &c->sy})
        if (*p) {
            cudaFree(*p);
            *p = nullptr;
        }
    c->sx_b = c->sw_b = c->sy_b = 0;
}

}  // extern "C"
