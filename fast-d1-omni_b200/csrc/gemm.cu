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
//               access), the fused epilogue in registers, then each 32x32 output block goes through a swizzled
//               shared-memory staging tile to one TMA bulk store (or TMA reduce-add for the fp32 residual
//               Y += X.W^T). The double-buffered accumulator lets the epilogue of one tile overlap the main loop
//               of the next; the accumulator is handed back as soon as its last column is read.
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
constexpr int EPI_BUF = 4096;     // one staging tile: 32 rows x 128 bytes
constexpr int EPI_SMEM = 4 * 2 * EPI_BUF;  // 4 epilogue warps, double-buffered

// Epilogue forms. The TMA forms stage each 32x32 output block through swizzled shared memory and write it with
// one bulk tensor store (or reduce-add) per warp; rows/columns past M/N are clipped by the tensor map.
enum Epi : int {
    EPI_STORE = 0,     // Y = alpha * acc (fp16 or fp32 Y), beta == 0
    EPI_ADD = 1,       // Y += alpha * acc (fp32 Y, beta == 1): TMA reduce-add, Y is never read by the SM
    EPI_SWIGLU = 2,    // out = silu(half(g)) * half(u), fp16
    EPI_BIAS_ACT = 3,  // Y = act(half(acc) + bias), fp16
    EPI_DIRECT = 4,    // any alpha/beta, direct stores (strides or alignment the tensor maps cannot take)
    EPI_QKROPE = 5,    // fp16 Y = [q | k | v] heads, q and k heads RMS-normed and rotated (d1_qk_norm_rope)
};

struct GemmArgs {
    int M, N, K;          // N: accumulator columns in total (2F for SwiGLU)
    int num_m, num_n;     // tile grid
    int num_tiles, num_kb;
    int num_units, kb_per; // split-K: work unit u = (tile u % num_tiles, K blocks [(u / num_tiles) * kb_per, +kb_per))
    void* Y;
    int ldy;
    int y_f32;
    float alpha, beta;
    const float* bias;
    int act;
    int F;                // SwiGLU: output columns (rows [0,F) of W are gate, [F,2F) up)
    int n_fast;           // tile order: 1 walks N fastest (A, the larger operand, is read from DRAM once)
    int* err;
    // EPI_QKROPE: columns [0, q_cols) are query heads, [q_cols, qk_cols) key heads, the rest value heads
    int q_cols, qk_cols;
    float eps;
    const float* qn;
    const float* kn;
    const float* rope;     // (cos, sin) [pos][32]
    const int* tok_seq;
    const SeqInfo* seqs;
};

// The i-th work unit of worker p of P (a CTA, or a CTA pair): units p, p + P, ... of the split grid, each an output
// tile and its K-block range [kb0, kb1). Every role of a worker walks the same sequence. (A stream-K schedule,
// whole tiles plus equal shares of the last wave's K blocks meeting in Y through the reduce-add, measured 2% slower
// on the forward than this one: its extra reduce-add traffic costs more than the idle part of the last wave.)
__device__ __forceinline__ bool unit_of(const GemmArgs& a, int p, int P, int i, int& tile, int& kb0, int& kb1) {
    const int u = p + i * P;
    if (u >= a.num_units) return false;
    tile = u % a.num_tiles;
    kb0 = (u / a.num_tiles) * a.kb_per;
    kb1 = min(a.num_kb, kb0 + a.kb_per);
    return true;
}

// Tile index -> (row block, column block). The CTAs running at the same time share the operand that the order
// repeats, so the larger operand is walked slowest: it streams from DRAM once while the smaller stays in L2.
__device__ __forceinline__ void tile_coords(const GemmArgs& a, int tile, int& m_blk, int& n_blk) {
    if (a.n_fast) {
        n_blk = tile % a.num_n;
        m_blk = tile / a.num_n;
    } else {
        m_blk = tile % a.num_m;
        n_blk = tile / a.num_m;
    }
}

template <int BN, int STAGES>
struct Smem {
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RING = STAGES * STAGE_BYTES;
    static constexpr int NBARS = 2 * STAGES + 5;
    static constexpr size_t BYTES = 1024 /* alignment slack */ + RING + EPI_SMEM + NBARS * 8 + 16;
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

// ---------------------------------------------------------------------------------------------- bulk stores

// Output tiles are written with an L2 evict-last hint: the next kernel of the forward reads them straight away.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
            (uint64_t)map),
        "r"(src), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
// Reduce-add into the fp32 residual with an L2 evict-last hint: the residual stream is read again by the next
// RMSNorm right after this GEMM, so its lines are kept in L2 ahead of the operand tiles streaming through.
__device__ __forceinline__ void tma_add_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
    uint64_t policy;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(policy));
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
            (uint64_t)map),
        "r"(src), "r"(x), "r"(y), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Thread t of the warp owns row t of a 32-row staging tile. fp16: 64-byte rows in the 64-byte swizzle pattern
// (16-byte chunk j of row t at chunk j ^ ((t >> 1) & 3)); fp32: 128-byte rows in the 128-byte pattern (chunk
// j ^ (t & 7)). These are the layouts the tensor maps' SWIZZLE_64B / SWIZZLE_128B expect, and each quarter-warp
// of 16-byte stores hits 8 distinct bank groups.
__device__ __forceinline__ void stage_h(uint8_t* buf, int t, const float* v) {
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint4 q = make_uint4(pack_h2(v[8 * j], v[8 * j + 1]), pack_h2(v[8 * j + 2], v[8 * j + 3]),
                                   pack_h2(v[8 * j + 4], v[8 * j + 5]), pack_h2(v[8 * j + 6], v[8 * j + 7]));
        *reinterpret_cast<uint4*>(buf + t * 64 + ((j ^ ((t >> 1) & 3)) << 4)) = q;
    }
}
__device__ __forceinline__ void stage_f(uint8_t* buf, int t, const float* v) {
#pragma unroll
    for (int j = 0; j < 8; j++)
        *reinterpret_cast<float4*>(buf + t * 128 + ((j ^ (t & 7)) << 4)) =
            make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}

// RoPE position of output row `row` (EPI_QKROPE): its place in its sequence plus the sequence's position offset.
__device__ __forceinline__ int qkrope_pos(const GemmArgs& a, int row) {
    if (row >= a.M) return 0;
    const SeqInfo& s = a.seqs[__ldg(a.tok_seq + row)];
    return row - s.start + s.pos_off;
}

// One 64-column head of the row this thread owns (TMEM lane), from the fp32 accumulator: the GEMM output rounded to
// fp16, as the unfused path stores it, then for query and key heads the arithmetic of k_qk_norm_rope8 term for term
// (cuda/kernels.cu:263-303): RMS over the head's 64 values (eight 8-value chains, then a pairwise tree), the q/k
// norm weight, rotate-half RoPE at `pos` (pairs l, l + 32). Value heads are only rounded.
__device__ __forceinline__ void qkrope_head(const GemmArgs& a, uint32_t taddr, int col, int pos, float (&o)[64]) {
    {
        uint32_t r0[32], r1[32];
        tmem_ld32(taddr, r0);
        tmem_ld32(taddr + 32, r1);
        tc_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; i++) {
            o[i] = round_h(__uint_as_float(r0[i]));
            o[32 + i] = round_h(__uint_as_float(r1[i]));
        }
    }
    if (col >= a.qk_cols) return;
    float c[8];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++) s += o[8 * k + i] * o[8 * k + i];
        c[k] = s;
    }
    const float ss = ((c[0] + c[1]) + (c[2] + c[3])) + ((c[4] + c[5]) + (c[6] + c[7]));
    const float r = rsqrtf(ss / 64.f + a.eps);
    // weights and (cos, sin) are loaded four float4 at a time (the empty asm statements keep the compiler from
    // hoisting all 32 loads at once, which would not fit the pair kernel's registers)
    const float4* w4 = reinterpret_cast<const float4*>(col < a.q_cols ? a.qn : a.kn);
#pragma unroll
    for (int i = 0; i < 16; i++) {
        if ((i & 3) == 0) asm volatile("" ::: "memory");
        const float4 w = __ldg(w4 + i);
        o[4 * i] = o[4 * i] * r * w.x;
        o[4 * i + 1] = o[4 * i + 1] * r * w.y;
        o[4 * i + 2] = o[4 * i + 2] * r * w.z;
        o[4 * i + 3] = o[4 * i + 3] * r * w.w;
    }
    const float4* cs4 = reinterpret_cast<const float4*>(a.rope + (size_t)pos * 64);
#pragma unroll
    for (int p2 = 0; p2 < 16; p2++) {
        if ((p2 & 3) == 0) asm volatile("" ::: "memory");
        const float4 t = __ldg(cs4 + p2);  // (cos, sin) of pairs 2 p2 and 2 p2 + 1
        float y0 = o[2 * p2], y1 = o[2 * p2 + 32];
        o[2 * p2] = y0 * t.x - y1 * t.y;
        o[2 * p2 + 32] = y1 * t.x + y0 * t.y;
        y0 = o[2 * p2 + 1];
        y1 = o[2 * p2 + 33];
        o[2 * p2 + 1] = y0 * t.z - y1 * t.w;
        o[2 * p2 + 33] = y1 * t.z + y0 * t.w;
    }
}

// v = act(half(acc) + bias) for one 32-column chunk: bias read as float4 when aligned, the activation chosen once
// per chunk (cuda/kernels.cu:171-184 applied to the fp16-rounded GEMM output).
__device__ __forceinline__ void bias_act32(const GemmArgs& a, int col, const uint32_t (&r)[32], float (&v)[32]) {
    float bb[32];
    if (a.bias && col + 32 <= a.N && ((reinterpret_cast<uintptr_t>(a.bias + col) & 15) == 0)) {
        const float4* b4 = reinterpret_cast<const float4*>(a.bias + col);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 t = __ldg(b4 + i);
            bb[4 * i] = t.x;
            bb[4 * i + 1] = t.y;
            bb[4 * i + 2] = t.z;
            bb[4 * i + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; i++) bb[i] = (a.bias && col + i < a.N) ? __ldg(a.bias + col + i) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = round_h(__uint_as_float(r[i])) + bb[i];
    switch (a.act) {
        case 1:
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = fmaxf(v[i], 0.0f);
            break;
        case 2:
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = gelu_erf(v[i]);
            break;
        case 3:
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = gelu_tanh(v[i]);
            break;
        case 4:
#pragma unroll
            for (int i = 0; i < 32; i++) v[i] = silu(v[i]);
            break;
        default: break;
    }
}

// Direct stores for EPI_DIRECT (fully unrolled so v[] stays in registers).
__device__ __forceinline__ void direct_store(const GemmArgs& a, int row, int col, float* v) {
    if (row >= a.M) return;
    if (a.y_f32) {
        float* y = reinterpret_cast<float*>(a.Y) + (size_t)row * a.ldy + col;
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (col + i < a.N) y[i] = v[i] + (a.beta != 0.f ? a.beta * y[i] : 0.f);
    } else {
        __half* y = reinterpret_cast<__half*>(a.Y) + (size_t)row * a.ldy + col;
#pragma unroll
        for (int i = 0; i < 32; i++)
            if (col + i < a.N) y[i] = __float2half_rn(v[i] + (a.beta != 0.f ? a.beta * __half2float(y[i]) : 0.f));
    }
}

// ---------------------------------------------------------------------------------------------- the kernel

template <int BN, int STAGES, int EPI, bool OUT32>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmY, const GemmArgs a) {
    using S = Smem<BN, STAGES>;
    constexpr uint32_t TMEM_COLS = 2 * BN;
    constexpr uint32_t IDESC = idesc_f16_f32(BM, BN);
    constexpr int OUT_COLS = EPI == EPI_SWIGLU ? BN / 2 : BN;  // output columns per tile
    static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "tcgen05 M=128 needs N % 16 == 0, 16..256");
    static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocations are powers of 2");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* epi_smem = smem + S::RING;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::RING + EPI_SMEM);
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
        if (EPI != EPI_DIRECT) prefetch_tmap(&tmY);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_entry();  // barriers, TMEM and tensor maps are set up; global memory is touched only after this

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued = 0, issued_par = 0;
            bool aborted = false;
            int tile, kb0, kb1;
            for (int i = 0; !aborted && unit_of(a, blockIdx.x, gridDim.x, i, tile, kb0, kb1); i++) {
                int m_blk, n_blk;
                tile_coords(a, tile, m_blk, n_blk);
                for (int kb = kb0; kb < kb1; kb++) {
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
            int tile, kb0, kb1;
            for (; !aborted && unit_of(a, blockIdx.x, gridDim.x, it, tile, kb0, kb1); it++) {
                const int acc = it & 1;
                const uint32_t acc_par = (it >> 1) & 1;
                if (!mbar_wait(acce_bar(acc), acc_par ^ 1, abort_flag)) {
                    record_error(a.err, abort_flag, kErrWaitAccEmpty);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = kb0; kb < kb1; kb++) {
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
                                   ((kb - kb0) | k) != 0);
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
        const int sub = warp & 3;  // TMEM lane quarter (rows sub*32 .. +31) this warp may access
        uint8_t* stage0 = epi_smem + sub * 2 * EPI_BUF;
        int buf = 0, it = 0;
        int tile, kb0, kb1;
        for (; unit_of(a, blockIdx.x, gridDim.x, it, tile, kb0, kb1); it++) {
            const int acc = it & 1;
            const uint32_t acc_par = (it >> 1) & 1;
            const bool ok = __all_sync(D1_FULL_MASK, mbar_wait(accf_bar(acc), acc_par, abort_flag));
            if (!ok) {
                if (lane == 0) record_error(a.err, abort_flag, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            int m_blk, n_blk;
                tile_coords(a, tile, m_blk, n_blk);
            const int row0 = m_blk * BM + sub * 32;
            const int col_base = n_blk * OUT_COLS;
            const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * BN);
            if constexpr (EPI == EPI_QKROPE) {  // one 64-column head at a time: two 32x32 fp16 blocks per buffer
                const int pos = qkrope_pos(a, row0 + lane);
#pragma unroll 1
                for (int h0 = 0; h0 < OUT_COLS; h0 += 64) {
                    float o[64];
                    qkrope_head(a, tbase + h0, col_base + h0, pos, o);
                    if (h0 + 64 >= OUT_COLS) {
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(acce_bar(acc));
                    }
                    uint8_t* sbuf = stage0 + buf * EPI_BUF;
                    if (lane == 0) bulk_wait_read<1>();
                    __syncwarp();
                    stage_h(sbuf, lane, o);
                    stage_h(sbuf + EPI_BUF / 2, lane, o + 32);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&tmY, smem_u32(sbuf), col_base + h0, row0);
                        tma_store_2d(&tmY, smem_u32(sbuf) + EPI_BUF / 2, col_base + h0 + 32, row0);
                        bulk_commit();
                    }
                    buf ^= 1;
                }
            } else {
    #pragma unroll 1
                for (int c0 = 0; c0 < OUT_COLS; c0 += 32) {
                    float v[32];
                    {
                        uint32_t r[32];
                        tmem_ld32(tbase + c0, r);
                        if (EPI == EPI_SWIGLU) {
                            uint32_t u[32];
                            tmem_ld32(tbase + BN / 2 + c0, u);
                            tc_wait_ld();
    #pragma unroll
                            for (int i = 0; i < 32; i++)
                                v[i] = silu(round_h(__uint_as_float(r[i]))) * round_h(__uint_as_float(u[i]));
                        } else {
                            tc_wait_ld();
                            if (EPI == EPI_BIAS_ACT) {
                                bias_act32(a, col_base + c0, r, v);
                            } else {
    #pragma unroll
                                for (int i = 0; i < 32; i++) v[i] = a.alpha * __uint_as_float(r[i]);
                            }
                        }
                    }
                    if (c0 + 32 >= OUT_COLS) {  // last TMEM read of this tile: hand the accumulator back to the MMA
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(acce_bar(acc));
                    }
                    if (EPI == EPI_DIRECT) {
                        direct_store(a, row0 + lane, col_base + c0, v);
                        continue;
                    }
                    uint8_t* sbuf = stage0 + buf * EPI_BUF;
                    if (lane == 0) bulk_wait_read<1>();  // the store that last read this buffer is done with it
                    __syncwarp();
                    if (OUT32)
                        stage_f(sbuf, lane, v);
                    else
                        stage_h(sbuf, lane, v);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (EPI == EPI_ADD)
                            tma_add_2d(&tmY, smem_u32(sbuf), col_base + c0, row0);
                        else
                            tma_store_2d(&tmY, smem_u32(sbuf), col_base + c0, row0);
                        bulk_commit();
                    }
                    buf ^= 1;
                }
            }
        }
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------------------------- CTA-pair kernel
// The same pipeline on a cluster of 2 CTAs (2 SMs) sharing one tcgen05 cta_group::2 MMA of 256 x BN x 16:
// each CTA holds 128 rows of A and BN/2 rows of B per stage (its own TMA loads, both completing on the pair
// leader's `full` barrier), and 128 rows x BN columns of the accumulator in its own TMEM. Per SM this halves the
// shared-memory operand bytes the tensor core reads per MMA and the L2->SM operand traffic per FLOP drops by
// a third, relative to the single-SM 128 x BN tile. The leader's thread issues the MMAs; its commits arrive on both CTAs'
// `empty` and `accf` barriers. 8 epilogue warps per CTA (2 per TMEM lane quarter, alternating 32-column chunks)
// arrive on the leader's `acce` barrier when their part of an accumulator has been read.
constexpr int kPairEpiWarps = 8;
constexpr int kPairThreads = 64 + 32 * kPairEpiWarps;
constexpr int PAIR_EPI_SMEM = kPairEpiWarps * EPI_BUF;

template <int BN, int STAGES>
struct PairSmem {
    static constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's half of the B tile
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int RING = STAGES * STAGE_BYTES;
    static constexpr int NBARS = 2 * STAGES + 5;
    static constexpr size_t BYTES = 1024 + RING + PAIR_EPI_SMEM + NBARS * 8 + 16;
};

template <int BN, int STAGES, int EPI, bool OUT32>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    k_gemm_tc2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmY, const GemmArgs a) {
    using S = PairSmem<BN, STAGES>;
    constexpr uint32_t TMEM_COLS = BN <= 128 ? 256 : 512;  // 2 accumulators of BN fp32 columns
    constexpr uint32_t IDESC = idesc_f16_f32(2 * BM, BN);
    constexpr int OUT_COLS = EPI == EPI_SWIGLU ? BN / 2 : BN;
    constexpr int SUBTILES = OUT32 ? 1 : 2;  // 32x32 output blocks per 4 KB staging buffer
    constexpr int SUB_BYTES = EPI_BUF / SUBTILES;
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "pair MMA: M=256 needs N % 16 == 0, 16..256");
    static_assert(S::BYTES <= 232448, "shared memory of the pair GEMM");
    static_assert(EPI != EPI_DIRECT && EPI != EPI_QKROPE, "the pair kernel takes the TMA epilogues but QK-rope");

    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* epi_smem = smem + S::RING;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::RING + PAIR_EPI_SMEM);
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
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        mbar_init(accf_bar(0), 1);
        mbar_init(accf_bar(1), 1);
        mbar_init(acce_bar(0), 2 * kPairEpiWarps);
        mbar_init(acce_bar(1), 2 * kPairEpiWarps);
        mbar_init(drain_bar, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        prefetch_tmap(&tmY);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_slot), TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();  // both CTAs' barriers are initialised before either signals the other
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    pdl_entry();

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, issued = 0, issued_par = 0;
            bool aborted = false;
            int tile, kb0, kb1;
            for (int i = 0; !aborted && unit_of(a, pair, npairs, i, tile, kb0, kb1); i++) {
                int m_blk, n_blk;
                tile_coords(a, tile, m_blk, n_blk);
                const int arow = m_blk * 2 * BM + (int)rank * BM;
                const int brow = EPI == EPI_SWIGLU ? (int)rank * a.F + n_blk * (BN / 2) : n_blk * BN + (int)rank * (BN / 2);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag)) {
                        record_error(a.err, abort_flag, kErrWaitEmpty);
                        aborted = true;
                        break;
                    }
                    const uint32_t fb = mapa_shared(full_bar(stage), 0);
                    if (leader) mbar_arrive_expect_tx(full_bar(stage), 2 * S::STAGE_BYTES);
                    tma_load_2d_pair(sA(stage), &tmA, kb * BK, arow, fb);
                    tma_load_2d_pair(sB(stage), &tmB, kb * BK, brow, fb);
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // The leader's full barriers see both CTAs' bytes; wait there for every stage last issued.
            if (leader)
                for (int s = 0; s < STAGES; s++)
                    if ((issued >> s) & 1)
                        if (!mbar_wait_timed(full_bar(s), (issued_par >> s) & 1))
                            record_error(a.err, abort_flag, kErrDrain);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issuer (leader CTA)
        if (leader && lane == 0) {
            int stage = 0, it = 0;
            uint32_t phase = 0;
            bool aborted = false;
            int tile, kb0, kb1;
            for (; !aborted && unit_of(a, pair, npairs, it, tile, kb0, kb1); it++) {
                const int acc = it & 1;
                const uint32_t acc_par = (it >> 1) & 1;
                if (!mbar_wait_cluster(acce_bar(acc), acc_par ^ 1, abort_flag)) {
                    record_error(a.err, abort_flag, kErrWaitAccEmpty);
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * (TMEM_COLS / 2);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!mbar_wait(full_bar(stage), phase, abort_flag)) {
                        record_error(a.err, abort_flag, kErrWaitFull);
                        aborted = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = sA(stage), b0 = sB(stage);
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        tc_mma_f16_pair(d_tmem, smem_desc_k128(a0 + k * 32), smem_desc_k128(b0 + k * 32), IDESC,
                                        ((kb - kb0) | k) != 0);
                    tc_commit_pair_both(empty_bar(stage));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (aborted) break;
                tc_commit_pair_both(accf_bar(acc));
            }
            tc_commit_pair(drain_bar);
            if (!mbar_wait_timed(drain_bar, 0)) record_error(a.err, abort_flag, kErrDrain);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue (warps 2..9, both CTAs)
        const int ew = warp - 2;
        const int sub = warp & 3;          // TMEM lane quarter this warp may access
        const int half = ew >> 2;          // which alternating 32-column chunks
        uint8_t* sbuf0 = epi_smem + ew * EPI_BUF;
        const uint32_t acce_leader0 = mapa_shared(acce_bar(0), 0), acce_leader1 = mapa_shared(acce_bar(1), 0);
        int sb = 0, it = 0;
        int tile, kb0, kb1;
        for (; unit_of(a, pair, npairs, it, tile, kb0, kb1); it++) {
            const int acc = it & 1;
            const uint32_t acc_par = (it >> 1) & 1;
            const bool ok = __all_sync(D1_FULL_MASK, mbar_wait(accf_bar(acc), acc_par, abort_flag));
            if (!ok) {
                if (lane == 0) record_error(a.err, abort_flag, kErrWaitAccFull);
                break;
            }
            tc_fence_after();
            int m_blk, n_blk;
                tile_coords(a, tile, m_blk, n_blk);
            const int row0 = m_blk * 2 * BM + (int)rank * BM + sub * 32;
            const int col_base = n_blk * OUT_COLS;
            const uint32_t tbase = tmem_base + ((uint32_t)(sub * 32) << 16) + (uint32_t)(acc * (TMEM_COLS / 2));
#pragma unroll 1
            for (int c0 = half * 32; c0 < OUT_COLS; c0 += 64) {
                float v[32];
                {
                    uint32_t r[32];
                    tmem_ld32(tbase + c0, r);
                    if (EPI == EPI_SWIGLU) {
                        uint32_t u[32];
                        tmem_ld32(tbase + BN / 2 + c0, u);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) {
                            const float g = round_h(__uint_as_float(r[i]));
                            v[i] = __fdividef(g, 1.0f + __expf(-g)) * round_h(__uint_as_float(u[i]));
                        }
                    } else {
                        tc_wait_ld();
                        if (EPI == EPI_BIAS_ACT) {
                            bias_act32(a, col_base + c0, r, v);
                        } else {
#pragma unroll
                            for (int i = 0; i < 32; i++) v[i] = a.alpha * __uint_as_float(r[i]);
                        }
                    }
                }
                if (c0 + 64 >= OUT_COLS) {  // this warp's last read of the accumulator
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(acc ? acce_leader1 : acce_leader0);
                }
                uint8_t* sbuf = sbuf0 + sb * SUB_BYTES;
                if (lane == 0) {
                    if (SUBTILES == 2)
                        bulk_wait_read<1>();
                    else
                        bulk_wait_read<0>();
                }
                __syncwarp();
                if (OUT32)
                    stage_f(sbuf, lane, v);
                else
                    stage_h(sbuf, lane, v);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (EPI == EPI_ADD)
                        tma_add_2d(&tmY, smem_u32(sbuf), col_base + c0, row0);
                    else
                        tma_store_2d(&tmY, smem_u32(sbuf), col_base + c0, row0);
                    bulk_commit();
                }
                sb = (sb + 1) % SUBTILES;
            }
        }
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
    }

    tc_fence_before();
    cluster_sync();  // no CTA leaves while its peer may still signal its barriers or read its shared memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, TMEM_COLS);
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

struct TmapKey {
    uintptr_t ptr;
    uint64_t inner, outer, stride;
    uint32_t box_inner, box_outer, kind;
    bool operator==(const TmapKey& o) const {
        return ptr == o.ptr && inner == o.inner && outer == o.outer && stride == o.stride &&
               box_inner == o.box_inner && box_outer == o.box_outer && kind == o.kind;
    }
};
struct TmapHash {
    size_t operator()(const TmapKey& k) const {
        size_t h = k.ptr * 0x9E3779B97F4A7C15ull;
        h ^= k.inner + 0x9E3779B9 + (h << 6) + (h >> 2);
        h ^= k.outer + 0x9E3779B9 + (h << 6) + (h >> 2);
        h ^= k.stride + 0x9E3779B9 + (h << 6) + (h >> 2);
        h ^= ((uint64_t)k.box_inner << 40 | (uint64_t)k.box_outer << 8 | k.kind) + 0x9E3779B9 + (h << 6) + (h >> 2);
        return h;
    }
};

// Tile plan: which kernel configuration runs a shape (the analogue of the reference's cuBLASLt algo choice).
typedef std::tuple<int, int, int, int, int, int, int, int, int> PlanKey;  // N K ldx ldw ldy w_kn y_f32 epi bucket
struct Plan {
    int cfg;    // Cfg
    int split;  // split-K factor (reduce-add epilogue only)
    float us;
};

// One per device. Several host threads may share a context (engines of one device over one model): `mu` guards the
// plan table, the tensor-map cache and the lazily set kernel attributes during each call's host work.
struct Ctx {
    std::mutex mu;
    int dev = 0;
    int num_sms = 148;
    int* d_err = nullptr;
    std::unordered_map<TmapKey, CUtensorMap, TmapHash> tmaps;
    std::map<PlanKey, Plan> plans;
    uint64_t attr_done = 0;  // per kernel instance: max dynamic smem attribute set
    int pair_slots = 74;     // co-resident CTA pairs (clusters of 2) for the pair kernels
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

// Tensor map kinds: operand loads (fp16, 128B swizzle) and output stores (fp16 64B / fp32 128B swizzle).
enum TmapKind : uint32_t { TM_LOAD16 = 0, TM_STORE16 = 1, TM_STORE32 = 2 };

bool get_tmap(Ctx* c, CUtensorMap* out, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
              uint32_t box_inner, uint32_t box_outer, TmapKind kind) {
    const uint64_t esize = kind == TM_STORE32 ? 4 : 2;
    TmapKey key{(uintptr_t)base, inner, outer, ld_elems * esize, box_inner, box_outer, (uint32_t)kind};
    auto it = c->tmaps.find(key);
    if (it != c->tmaps.end()) {
        *out = it->second;
        return true;
    }
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    CUtensorMap m;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld_elems * esize};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = kind == TM_STORE32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUtensorMapSwizzle sw = kind == TM_STORE16 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    CUresult r = enc(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    if (c->tmaps.size() > 4096) c->tmaps.clear();
    c->tmaps.emplace(key, m);
    *out = m;
    return true;
}

// Split-K: a.kb_per holds the requested split on entry; every split gets a non-empty K range.
void set_split(GemmArgs& a) {
    int ks = a.kb_per < 1 ? 1 : a.kb_per;
    if (ks > a.num_kb) ks = a.num_kb;
    a.kb_per = (a.num_kb + ks - 1) / ks;
    a.num_units = a.num_tiles * ((a.num_kb + a.kb_per - 1) / a.kb_per);
}

bool tc_ok(const void* X, int ldx, const void* W, int ldw, int w_kn, int K) {
    return !w_kn && K >= 1 && ldx % 8 == 0 && ldw % 8 == 0 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)W & 15) == 0;
}

// Output through a TMA tensor map: base 16-byte aligned and a row pitch that is a multiple of 16 bytes.
bool tma_out_ok(const void* Y, int ldy, int y_f32) {
    return ((uintptr_t)Y & 15) == 0 && ((size_t)ldy * (y_f32 ? 4 : 2)) % 16 == 0;
}

template <int BN, int STAGES, int EPI, bool OUT32>
int launch_tc(Ctx* c, int bit, const void* X, int ldx, const void* W, int ldw, int w_rows, GemmArgs& a,
              cudaStream_t st) {
    using S = Smem<BN, STAGES>;
    auto kern = k_gemm_tc<BN, STAGES, EPI, OUT32>;
    if (!(c->attr_done & (1ull << bit))) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::BYTES) != cudaSuccess)
            return -1;
        c->attr_done |= 1ull << bit;
    }
    const uint32_t b_rows = EPI == EPI_SWIGLU ? BN / 2 : BN;
    CUtensorMap ta, tb, ty;
    if (!get_tmap(c, &ta, X, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)ldx, BK, BM, TM_LOAD16) ||
        !get_tmap(c, &tb, W, (uint64_t)a.K, (uint64_t)w_rows, (uint64_t)ldw, BK, b_rows, TM_LOAD16))
        return -1;
    const int out_cols = EPI == EPI_SWIGLU ? a.F : a.N;
    if (EPI == EPI_DIRECT)
        ty = ta;  // unused
    else if (!get_tmap(c, &ty, a.Y, (uint64_t)out_cols, (uint64_t)a.M, (uint64_t)a.ldy, 32, 32,
                       OUT32 ? TM_STORE32 : TM_STORE16))
        return -1;
    a.num_m = (a.M + BM - 1) / BM;
    a.num_n = EPI == EPI_SWIGLU ? (a.F + BN / 2 - 1) / (BN / 2) : (a.N + BN - 1) / BN;
    a.num_tiles = a.num_m * a.num_n;
    a.num_kb = (a.K + BK - 1) / BK;
    set_split(a);
    a.n_fast = a.M > w_rows;
    a.err = c->d_err;
    const int grid = a.num_units < c->num_sms ? a.num_units : c->num_sms;
    launch_pdl(kern, grid, kThreads, S::BYTES, st, ta, tb, ty, a);
    return (int)cudaGetLastError();
}

template <int BN, int STAGES, int EPI, bool OUT32>
int launch_tc2(Ctx* c, int bit, const void* X, int ldx, const void* W, int ldw, int w_rows, GemmArgs& a,
               cudaStream_t st) {
    using S = PairSmem<BN, STAGES>;
    auto kern = k_gemm_tc2<BN, STAGES, EPI, OUT32>;
    if (!(c->attr_done & (1ull << bit))) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)S::BYTES) != cudaSuccess)
            return -1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2 * (c->num_sms / 2));
        cfg.blockDim = dim3(kPairThreads);
        cfg.dynamicSmemBytes = S::BYTES;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            n = c->num_sms / 2;
        }
        c->pair_slots = n;
        c->attr_done |= 1ull << bit;
    }
    const uint32_t b_rows = BN / 2;
    CUtensorMap ta, tb, ty;
    const int out_cols = EPI == EPI_SWIGLU ? a.F : a.N;
    if (!get_tmap(c, &ta, X, (uint64_t)a.K, (uint64_t)a.M, (uint64_t)ldx, BK, BM, TM_LOAD16) ||
        !get_tmap(c, &tb, W, (uint64_t)a.K, (uint64_t)w_rows, (uint64_t)ldw, BK, b_rows, TM_LOAD16) ||
        !get_tmap(c, &ty, a.Y, (uint64_t)out_cols, (uint64_t)a.M, (uint64_t)a.ldy, 32, 32,
                  OUT32 ? TM_STORE32 : TM_STORE16))
        return -1;
    a.num_m = (a.M + 2 * BM - 1) / (2 * BM);
    a.num_n = EPI == EPI_SWIGLU ? (a.F + BN / 2 - 1) / (BN / 2) : (a.N + BN - 1) / BN;
    a.num_tiles = a.num_m * a.num_n;
    a.num_kb = (a.K + BK - 1) / BK;
    set_split(a);
    a.n_fast = a.M > w_rows;
    a.err = c->d_err;
    const int pairs = a.num_units < c->pair_slots ? a.num_units : c->pair_slots;
    launch_pdl(kern, 2 * pairs, kPairThreads, S::BYTES, st, ta, tb, ty, a);
    return (int)cudaGetLastError();
}

// Wave efficiency of a tile count over the SMs.
double wave_eff(long tiles, int sms) {
    long waves = (tiles + sms - 1) / sms;
    return (double)tiles / (double)(waves * sms);
}

// Kernel configurations a plan can name: the single-SM kernel with 128- or 256-column tiles, or the CTA-pair
// kernel with 256 x 256 or 256 x 128 tiles.
// (A 256 x 192 pair tile, which turns the 5.19 waves of 256-column tiles for N = 3072 into 6.92 fuller ones, was
// slower than 256 x 256 on every trunk shape at M = 8192: in_proj 44.3 against 40.9 us, QKV 32.0 against 28.3 us.
// Narrower tiles cost more per FLOP here, so the last wave is not what limits these GEMMs.)
enum Cfg : int { CFG_1SM_128 = 0, CFG_1SM_256 = 1, CFG_PAIR_256 = 2, CFG_PAIR_128 = 3, CFG_1SM_64 = 4 };
constexpr int CFG_LAST = CFG_1SM_64;

inline bool cfg_pair(int cfg) { return cfg == CFG_PAIR_256 || cfg == CFG_PAIR_128; }
inline int cfg_bn(int cfg) { return cfg == CFG_1SM_64 ? 64 : (cfg == CFG_1SM_128 || cfg == CFG_PAIR_128) ? 128 : 256; }

// Fraction of the SM-time the tiles keep busy (wave quantisation x column padding), per configuration.
double cfg_eff(Ctx* c, int cfg, int M, int N) {
    const bool pair = cfg_pair(cfg);
    const int bm = pair ? 2 * BM : BM;
    const int bn = cfg_bn(cfg);
    const long tiles = (long)((M + bm - 1) / bm) * ((N + bn - 1) / bn);
    const int slots = pair ? c->pair_slots : c->num_sms;
    const double pad = (double)M * N / ((double)((M + bm - 1) / bm) * bm * ((N + bn - 1) / bn) * bn);
    return wave_eff(tiles, slots) * pad;
}

// Heuristic plan when none was tuned: the pair kernel for large problems (it needs half the shared-memory and
// L2 operand bandwidth per FLOP), preferring the tile width that quantises better.
int default_cfg(Ctx* c, int M, int N) {
    if (M >= 512) {
        // 256x256 tiles read the fewest operand bytes per FLOP; 256x128 only for much better quantisation
        const double e256 = cfg_eff(c, CFG_PAIR_256, M, N), e128 = cfg_eff(c, CFG_PAIR_128, M, N);
        return e128 > e256 + 0.15 ? CFG_PAIR_128 : CFG_PAIR_256;
    }
    // small M is bound by reading W: narrow tiles put more SMs on it
    const long mt = (M + BM - 1) / BM;
    if (mt * ((N + 127) / 128) < c->num_sms / 2) return CFG_1SM_64;
    if (mt * ((N + 255) / 256) < c->num_sms / 2) return CFG_1SM_128;
    const double e256 = cfg_eff(c, CFG_1SM_256, M, N), e128 = cfg_eff(c, CFG_1SM_128, M, N);
    return e128 > e256 + 0.08 ? CFG_1SM_128 : CFG_1SM_256;
}

// Split-K for the reduce-add epilogue (partial sums land in Y through TMA reduce-add): enough work units to
// cover the SMs when the tiles alone leave most of them idle, keeping >= 4 K blocks per unit.
int default_split(Ctx* c, int cfg, int M, int N, int K) {
    const bool pair = cfg_pair(cfg);
    const int bm = pair ? 2 * BM : BM;
    const int bn = cfg_bn(cfg);
    const long tiles = (long)((M + bm - 1) / bm) * ((N + bn - 1) / bn);
    const int slots = pair ? c->pair_slots : c->num_sms;
    const int kb = (K + BK - 1) / BK;
    int split = 1;
    while (tiles * split * 2 <= slots && kb / (split * 2) >= 4) split *= 2;
    return split;
}

// Y = alpha X W^T + beta Y: TMA store (beta 0), TMA reduce-add (fp32 Y, beta 1), else direct stores.
int run_store(Ctx* c, int cfg, int split, int M, int N, int K, const void* X, int ldx, const void* W, int ldw,
              void* Y, int ldy, int y_f32, float alpha, float beta, cudaStream_t st) {
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.y_f32 = y_f32;
    a.alpha = alpha;
    a.beta = beta;
    const bool tma = tma_out_ok(Y, ldy, y_f32);
    const bool store = tma && beta == 0.f, add = tma && beta == 1.f && y_f32;
    a.kb_per = add ? split : 1;  // split request (set_split turns it into K blocks per unit)
    if (cfg == CFG_1SM_64 && (store || add)) {
        if (add) return launch_tc<64, 8, EPI_ADD, true>(c, 20, X, ldx, W, ldw, N, a, st);
        if (y_f32) return launch_tc<64, 8, EPI_STORE, true>(c, 21, X, ldx, W, ldw, N, a, st);
        return launch_tc<64, 8, EPI_STORE, false>(c, 22, X, ldx, W, ldw, N, a, st);
    }
    if (cfg == CFG_PAIR_256 && (store || add)) {
        if (add) return launch_tc2<256, 6, EPI_ADD, true>(c, 11, X, ldx, W, ldw, N, a, st);
        if (y_f32) return launch_tc2<256, 6, EPI_STORE, true>(c, 12, X, ldx, W, ldw, N, a, st);
        return launch_tc2<256, 6, EPI_STORE, false>(c, 13, X, ldx, W, ldw, N, a, st);
    }
    if (cfg == CFG_PAIR_128 && (store || add)) {
        if (add) return launch_tc2<128, 8, EPI_ADD, true>(c, 14, X, ldx, W, ldw, N, a, st);
        if (y_f32) return launch_tc2<128, 8, EPI_STORE, true>(c, 15, X, ldx, W, ldw, N, a, st);
        return launch_tc2<128, 8, EPI_STORE, false>(c, 16, X, ldx, W, ldw, N, a, st);
    }
    const bool b128 = cfg == CFG_1SM_128 || cfg == CFG_1SM_64;
    if (store) {
        if (y_f32)
            return b128 ? launch_tc<128, 6, EPI_STORE, true>(c, 0, X, ldx, W, ldw, N, a, st)
                        : launch_tc<256, 4, EPI_STORE, true>(c, 1, X, ldx, W, ldw, N, a, st);
        return b128 ? launch_tc<128, 6, EPI_STORE, false>(c, 2, X, ldx, W, ldw, N, a, st)
                    : launch_tc<256, 4, EPI_STORE, false>(c, 3, X, ldx, W, ldw, N, a, st);
    }
    if (add)
        return b128 ? launch_tc<128, 6, EPI_ADD, true>(c, 4, X, ldx, W, ldw, N, a, st)
                    : launch_tc<256, 4, EPI_ADD, true>(c, 5, X, ldx, W, ldw, N, a, st);
    return b128 ? launch_tc<128, 6, EPI_DIRECT, false>(c, 6, X, ldx, W, ldw, N, a, st)
                : launch_tc<256, 4, EPI_DIRECT, false>(c, 7, X, ldx, W, ldw, N, a, st);
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

const char* d1_build_id(void) { return "d1b200-tc-gemm-v4"; }

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
    std::lock_guard<std::mutex> lock(c->mu);
    if (M == 0 || N == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, w_kn, K))
        return run_simt(M, N, K, X, ldx, W, ldw, w_kn, Y, ldy, y_f32, alpha, beta, st) ? -1 : 0;
    auto it = c->plans.find(PlanKey(N, K, ldx, ldw, ldy, w_kn, y_f32, EPI_STORE, bucket_of(M)));
    int cfg, split;
    if (it != c->plans.end()) {
        cfg = it->second.cfg;
        split = it->second.split;
    } else {
        cfg = default_cfg(c, M, N);
        split = default_split(c, cfg, M, N, K);
    }
    return run_store(c, cfg, split, M, N, K, X, ldx, W, ldw, Y, ldy, y_f32, alpha, beta, st) ? -1 : 0;
}

int d1_gemm_swiglu(void* ctx, int M, int F, int K, const d1_half* X, int ldx, const d1_half* W, int ldw,
                   d1_half* out, int ldo, cudaStream_t st) {
    Ctx* c = (Ctx*)ctx;
    if (!c || M < 0 || F <= 0 || K <= 0) return M == 0 ? 0 : -1;
    std::lock_guard<std::mutex> lock(c->mu);
    if (M == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, 0, K)) return -1;
    GemmArgs a{};
    a.M = M;
    a.N = 2 * F;
    a.K = K;
    a.F = F;
    a.Y = out;
    a.ldy = ldo;
    a.alpha = 1.f;
    if (!tma_out_ok(out, ldo, 0)) return -1;
    if (M >= 512) return launch_tc2<256, 6, EPI_SWIGLU, false>(c, 17, X, ldx, W, ldw, 2 * F, a, st) ? -1 : 0;
    return launch_tc<256, 4, EPI_SWIGLU, false>(c, 8, X, ldx, W, ldw, 2 * F, a, st) ? -1 : 0;
}

int d1_gemm_bias_act(void* ctx, int M, int N, int K, const d1_half* X, int ldx, const d1_half* W, int ldw,
                     const float* bias, int act, d1_half* Y, int ldy, cudaStream_t st) {
    Ctx* c = (Ctx*)ctx;
    if (!c || M < 0 || N < 0 || K <= 0 || act < 0 || act > 4) return -1;
    std::lock_guard<std::mutex> lock(c->mu);
    if (M == 0 || N == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, 0, K)) return -1;
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.alpha = 1.f;
    a.bias = bias;
    a.act = act;
    if (!tma_out_ok(Y, ldy, 0)) return -1;
    switch (default_cfg(c, M, N)) {
        case CFG_PAIR_256: return launch_tc2<256, 6, EPI_BIAS_ACT, false>(c, 18, X, ldx, W, ldw, N, a, st) ? -1 : 0;
        case CFG_PAIR_128: return launch_tc2<128, 8, EPI_BIAS_ACT, false>(c, 19, X, ldx, W, ldw, N, a, st) ? -1 : 0;
        case CFG_1SM_128: return launch_tc<128, 6, EPI_BIAS_ACT, false>(c, 9, X, ldx, W, ldw, N, a, st) ? -1 : 0;
        case CFG_1SM_64: return launch_tc<64, 8, EPI_BIAS_ACT, false>(c, 23, X, ldx, W, ldw, N, a, st) ? -1 : 0;
        default: return launch_tc<256, 4, EPI_BIAS_ACT, false>(c, 10, X, ldx, W, ldw, N, a, st) ? -1 : 0;
    }
}

int d1_gemm_qk_norm_rope(void* ctx, int M, int K, const d1_half* X, int ldx, const d1_half* W, int ldw, d1_half* Y,
                         int ldy, int H, int KVH, const float* qn, const float* kn, const float* rope,
                         const int* tok_seq, const SeqInfo* seqs, float eps, cudaStream_t st) {
    Ctx* c = (Ctx*)ctx;
    if (!c || M < 0 || K <= 0 || H <= 0 || KVH <= 0 || !qn || !kn || !rope || !tok_seq || !seqs) return -1;
    if ((reinterpret_cast<uintptr_t>(rope) | reinterpret_cast<uintptr_t>(qn) | reinterpret_cast<uintptr_t>(kn)) & 15)
        return -1;  // read as float4
    std::lock_guard<std::mutex> lock(c->mu);
    const int N = (H + 2 * KVH) * 64;
    if (M == 0) return 0;
    if (!tc_ok(X, ldx, W, ldw, 0, K) || !tma_out_ok(Y, ldy, 0) || ldy < N) return -1;
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.Y = Y;
    a.ldy = ldy;
    a.alpha = 1.f;
    a.q_cols = H * 64;
    a.qk_cols = (H + KVH) * 64;
    a.eps = eps;
    a.qn = qn;
    a.kn = kn;
    a.rope = rope;
    a.tok_seq = tok_seq;
    a.seqs = seqs;
    // single-SM tiles only: the epilogue's 64-value heads fit the 1-SM kernel's registers (on par with the CTA pair
    // for this shape on B200)
    int cfg = default_cfg(c, M, N);
    if (cfg == CFG_PAIR_256) cfg = CFG_1SM_256;
    if (cfg == CFG_PAIR_128) cfg = CFG_1SM_128;
    switch (cfg) {
        case CFG_1SM_128: return launch_tc<128, 6, EPI_QKROPE, false>(c, 24, X, ldx, W, ldw, N, a, st) ? -1 : 0;
        case CFG_1SM_64: return launch_tc<64, 8, EPI_QKROPE, false>(c, 25, X, ldx, W, ldw, N, a, st) ? -1 : 0;
        default: return launch_tc<256, 4, EPI_QKROPE, false>(c, 26, X, ldx, W, ldw, N, a, st) ? -1 : 0;
    }
}

float d1_lt_tune(void* ctx, int M, int N, int K, int ldx, int ldw, int w_kn, int ldy, int y_f32, int f16acc,
                 int effort, cudaStream_t st) {
    (void)f16acc;
    (void)effort;
    Ctx* c = (Ctx*)ctx;
    if (!c || M <= 0 || N <= 0 || K <= 0) return -1.f;
    std::lock_guard<std::mutex> lock(c->mu);
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
    int best_cfg = CFG_1SM_256, best_split = 1;
    const bool tc = tc_ok(c->sx, ldx, c->sw, ldw, w_kn, K);
    for (int cfg : {CFG_1SM_64, CFG_1SM_128, CFG_1SM_256, CFG_PAIR_256, CFG_PAIR_128}) {
        for (int split : {1, 2, 4}) {
            if (split > 1 && !y_f32) break;  // split-K only through the reduce-add epilogue
            if ((K + BK - 1) / BK < 4 * split) break;
            auto run = [&]() {
                return tc ? run_store(c, cfg, split, M, N, K, c->sx, ldx, c->sw, ldw, c->sy, ldy, y_f32, 1.f,
                                      y_f32 ? 1.f : 0.f, st)
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
                best_cfg = cfg;
                best_split = split;
            }
            if (!tc) break;
        }
        if (!tc) break;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (best >= 1e29f) return -1.f;
    c->plans[key] = Plan{best_cfg, best_split, best};
    return best;
}

int d1_lt_save(void* ctx, const char* path) {
    Ctx* c = (Ctx*)ctx;
    if (!c) return -1;
    std::lock_guard<std::mutex> lock(c->mu);
    FILE* f = fopen(path, "w");
    if (!f) return -1;
    fprintf(f, "d1b200-gemm-plans v1 %s\n", d1_build_id());
    for (auto& kv : c->plans) {
        int N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b;
        std::tie(N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b) = kv.first;
        fprintf(f, "%d %d %d %d %d %d %d %d %d %d %d %.2f\n", N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b, kv.second.cfg,
                kv.second.split, kv.second.us);
    }
    fclose(f);
    return 0;
}

int d1_lt_load(void* ctx, const char* path) {
    Ctx* c = (Ctx*)ctx;
    if (!c) return -1;
    std::lock_guard<std::mutex> lock(c->mu);
    FILE* f = fopen(path, "r");
    if (!f) return -1;
    char tag[64], ver[16], id[128];
    if (fscanf(f, "%63s %15s %127s\n", tag, ver, id) != 3 || strcmp(id, d1_build_id()) != 0) {
        fclose(f);
        return -2;
    }
    int n = 0;
    while (true) {
        int N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b, cfg, split;
        float us;
        if (fscanf(f, "%d %d %d %d %d %d %d %d %d %d %d %f", &N, &K, &ldx, &ldw, &ldy, &w_kn, &y_f32, &epi, &b, &cfg,
                   &split, &us) != 12)
            break;
        if (cfg < CFG_1SM_128 || cfg > CFG_LAST || split < 1 || split > 64) continue;
        c->plans[PlanKey(N, K, ldx, ldw, ldy, w_kn, y_f32, epi, b)] = Plan{cfg, split, us};
        n++;
    }
    fclose(f);
    return n;
}

int d1_lt_bucket(int m) { return bucket_of(m); }

void d1_lt_free_scratch(void* ctx) {
    Ctx* c = (Ctx*)ctx;
    if (!c) return;
    std::lock_guard<std::mutex> lock(c->mu);
    for (void** p : {&c->sx, &c->sw, &c->sy})
        if (*p) {
            cudaFree(*p);
            *p = nullptr;
        }
    c->sx_b = c->sw_b = c->sy_b = 0;
}

}  // extern "C"

// ================================================================================================ allocation-free form
// d1_gemm_noalloc: an fp16-output GEMM whose only scratch — the fp32 split-K accumulator and the kernels' error word
// — lives in a file-scope static device buffer, so the call allocates nothing (no context, no cudaMalloc, no
// cached tensor maps). The K range of every output tile is split across CTAs; each CTA reduce-adds its partial
// tile into the buffer through the same tcgen05 kernel the residual GEMMs use, then one pass rounds the sums to
// fp16 into Y. The buffer is cleared (cudaMemsetAsync) before every call. Overlapping calls on one device race on
// the buffer.

namespace {

constexpr size_t kNoallocMaxElems = (size_t)1 << 20;  // fp32 partial sums: 4 MiB
constexpr size_t kNoallocErrOff = kNoallocMaxElems;   // error word right after the accumulator

static __device__ __align__(256) float g_noalloc_scratch[kNoallocMaxElems + 64];

__global__ void __launch_bounds__(256) k_noalloc_to_f16(const float* __restrict__ acc, int M, int N,
                                                        __half* __restrict__ Y, int ldy) {
    const size_t total = (size_t)M * N;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t m = i / N, n = i % N;
        Y[m * ldy + n] = __float2half_rn(acc[i]);
    }
}

struct NoallocDev {
    float* scratch = nullptr;
    int num_sms = 0;
};

// Per-device set-up, once: the buffer's device address (cudaGetSymbolAddress, checked), the SM count and the
// kernel's shared-memory attribute.
bool noalloc_setup(NoallocDev& d) {
    static NoallocDev devs[64];
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lock(mu);
    NoallocDev& s = devs[dev];
    if (!s.scratch) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return false;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return false;
        using S = Smem<128, 6>;
        if (cudaFuncSetAttribute(k_gemm_tc<128, 6, EPI_ADD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)S::BYTES) != cudaSuccess)
            return false;
        s.num_sms = sms;
        s.scratch = static_cast<float*>(p);
    }
    d = s;
    return true;
}

bool encode_nocache(CUtensorMap* m, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_bytes,
                    uint32_t box_inner, uint32_t box_outer, bool f32) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {ld_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base),
               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

extern "C" int d1_gemm_noalloc(int M, int N, int K, const d1_half* X, int ldx, const d1_half* W, int ldw, d1_half* Y,
                               int ldy, int split, cudaStream_t st) {
    if (M < 0 || N < 0 || K < 0 || split < 1 || split > 64) return -1;
    if (M == 0 || N == 0) return 0;
    if ((size_t)M * (size_t)N > kNoallocMaxElems) return -1;  // beyond the static accumulator
    if (!X || !W || !Y || ldy < N || N % 4 || !tc_ok(X, ldx, W, ldw, 0, K)) return -1;
    NoallocDev d;
    if (!noalloc_setup(d)) return -1;
    float* acc = d.scratch;
    int* err = reinterpret_cast<int*>(d.scratch + kNoallocErrOff);
    // what must start at zero: the reduce-add accumulator and the error word
    if (cudaMemsetAsync(acc, 0, (size_t)M * N * sizeof(float), st) != cudaSuccess ||
        cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess)
        return -1;
    CUtensorMap ta, tb, ty;
    if (!encode_nocache(&ta, X, (uint64_t)K, (uint64_t)M, (uint64_t)ldx * 2, BK, BM, false) ||
        !encode_nocache(&tb, W, (uint64_t)K, (uint64_t)N, (uint64_t)ldw * 2, BK, 128, false) ||
        !encode_nocache(&ty, acc, (uint64_t)N, (uint64_t)M, (uint64_t)N * 4, 32, 32, true))
        return -1;
    GemmArgs a{};
    a.M = M;
    a.N = N;
    a.K = K;
    a.Y = acc;
    a.ldy = N;
    a.y_f32 = 1;
    a.alpha = 1.f;
    a.beta = 1.f;
    a.kb_per = split;
    a.num_m = (M + BM - 1) / BM;
    a.num_n = (N + 127) / 128;
    a.num_tiles = a.num_m * a.num_n;
    a.num_kb = (K + BK - 1) / BK;
    set_split(a);
    a.n_fast = M > N;
    a.err = err;
    const int grid = a.num_units < d.num_sms ? a.num_units : d.num_sms;
    k_gemm_tc<128, 6, EPI_ADD, true><<<grid, kThreads, Smem<128, 6>::BYTES, st>>>(ta, tb, ty, a);
    if (cudaGetLastError() != cudaSuccess) return -1;
    const size_t total = (size_t)M * N;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, (size_t)d.num_sms * 8);
    k_noalloc_to_f16<<<blocks, 256, 0, st>>>(acc, M, N, reinterpret_cast<__half*>(Y), ldy);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Reads and clears the error word the last d1_gemm_noalloc call on the current device left in the static buffer
// (a bounded wait of the GEMM kernel that ran out; Y is then not the product). Synchronous: it waits for the
// device's work, so the word is the one the last issued call wrote.
extern "C" int d1_gemm_noalloc_error(void) {
    NoallocDev d;
    if (!noalloc_setup(d)) return -1;
    int* err = reinterpret_cast<int*>(d.scratch + kNoallocErrOff);
    int e = 0;
    if (cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    if (e && cudaMemset(err, 0, sizeof(int)) != cudaSuccess) return -1;
    return e;
}
