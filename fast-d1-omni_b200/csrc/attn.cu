// Packed variable-length bidirectional flash attention, head dim 64, for the d1rs trunk (GQA), the decision head
// (MHA + q/k/v bias), and the SigLIP2 tower. Replaces d1_flash_attn of the reference (cuda/kernels.cu:351-500,
// launcher :726-734) with the same arguments and semantics:
//   for every work item (seq, q0) and head h: O[q] = softmax(scale * Q[q] . K^T) . V over the keys
//   [ext prefix keys | local keys] of that sequence, kv head g = h / group, fp32 softmax, optional fp32 biases
//   added to q/k/v as they are loaded.
//
// d1_flash_attn runs an mma.sync kernel: one CTA per (64-query tile, kv head) runs all the query heads that share
// that kv head (GQA group 2:
// 8 warps, two heads), so each K/V tile is fetched once for the group. Each warp owns 16 query rows of one head.
// K/V tiles of 64 keys are double-buffered in shared memory with cp.async (bias-free case) so the next tile's
// loads overlap this tile's math; QK^T and PV run on m16n8k16 fp16 tensor-core MMAs with fp32 accumulation,
// S stays in registers and is re-packed as the A operand of PV; the online softmax works in the exp2 domain.
// The output tile is staged through shared memory for 16-byte coalesced stores; 2 CTAs per SM.
//
// d1_flash_attn_tc (extension) is the same computation for the bias-free forms on tcgen05 (S and O in TMEM;
// k_flash_attn_tc below). Measured on B200 it is on par with the mma.sync kernel at 256-token sequences
// (68.6 vs ~70 us for 32 x 256 tokens x 16 heads) and up to 2x slower on long ones: with 128 x 64 tiles its
// per-tile S -> softmax -> P -> P.V handoffs are latency-bound (tensor pipe 5%, MUFU 10% busy). The remaining
// steps to make it the default: 128-key tiles with two query tiles per CTA in ping-pong, lazy O rescaling.
#include "common.cuh"
#include "warp_mma.cuh"

using namespace d1;

namespace {

constexpr int FA_B = 64;    // query rows per tile and keys per K/V tile
constexpr int FA_LD = 72;   // padded shared-memory row (halves): conflict-free ldmatrix

__device__ __forceinline__ uint4 add_bias8(uint4 v, const float* bias) {
    __half2* h = reinterpret_cast<__half2*>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        float2 f = __half22float2(h[i]);
        h[i] = __floats2half2_rn(f.x + __ldg(bias + 2 * i), f.y + __ldg(bias + 2 * i + 1));
    }
    return v;
}

struct FaArgs {
    const __half* Q;
    const __half* K;
    const __half* V;
    const float* bq;
    const float* bk;
    const float* bv;
    __half* O;
    const AttnSeq* seqs;
    const int2* work;
    int ldq, ldkv, ext_ld, ldo, group;
    float scale_log2;
};

// HPC query heads per CTA (all of them sharing one kv head), 4 warps per head.
template <int HPC, bool BIAS>
__global__ void __launch_bounds__(128 * HPC, 2) k_flash_attn(const FaArgs p) {
    extern __shared__ __align__(16) uint8_t fa_smem[];
    __half* sQ = reinterpret_cast<__half*>(fa_smem);                 // [HPC][64][FA_LD]
    __half* sK = sQ + HPC * FA_B * FA_LD;                           // [2][64][FA_LD]
    __half* sV = sK + 2 * FA_B * FA_LD;                             // [2][64][FA_LD]

    const int2 wi = p.work[blockIdx.x];
    const AttnSeq s = p.seqs[wi.x];
    const int q0 = wi.y;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int hl = warp >> 2;                          // head of this warp within the CTA
    const int g = blockIdx.y;                          // kv head
    const int h0 = HPC > 1 ? g * p.group : blockIdx.y;  // first query head of the CTA
    const int kvh = HPC > 1 ? g : blockIdx.y / p.group;
    const int total = s.ext_len + s.kv_len;
    constexpr int NT = 128 * HPC;

    // ---- Q tiles (all heads of the CTA)
    for (int i = tid; i < HPC * FA_B * 8; i += NT) {
        const int hh = i / (FA_B * 8), r = (i / 8) % FA_B, c = (i % 8) * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (q0 + r < s.q_len) {
            v = *reinterpret_cast<const uint4*>(p.Q + (size_t)(s.q_start + q0 + r) * p.ldq + (h0 + hh) * 64 + c);
            if (BIAS && p.bq) v = add_bias8(v, p.bq + (h0 + hh) * 64 + c);
        }
        *reinterpret_cast<uint4*>(sQ + (hh * FA_B + r) * FA_LD + c) = v;
    }

    // ---- K/V tile loader (64 keys x 64 dims each)
    auto load_kv = [&](int j0, int buf) {
        __half* dK = sK + buf * FA_B * FA_LD;
        __half* dV = sV + buf * FA_B * FA_LD;
        for (int i = tid; i < FA_B * 8; i += NT) {
            const int r = i / 8, c = (i % 8) * 8;
            const int j = j0 + r;
            const __half* srck;
            const __half* srcv;
            bool valid = j < total;
            bool ext = j < s.ext_len;
            if (ext) {
                srck = s.ext_k + (size_t)j * p.ext_ld + kvh * 64 + c;
                srcv = s.ext_v + (size_t)j * p.ext_ld + kvh * 64 + c;
            } else {
                const size_t row = (size_t)(s.kv_start + (valid ? j - s.ext_len : 0)) * p.ldkv + kvh * 64 + c;
                srck = p.K + row;
                srcv = p.V + row;
            }
            if (BIAS) {
                uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
                if (valid) {
                    kv = *reinterpret_cast<const uint4*>(srck);
                    vv = *reinterpret_cast<const uint4*>(srcv);
                    if (!ext && p.bk) kv = add_bias8(kv, p.bk + kvh * 64 + c);
                    if (!ext && p.bv) vv = add_bias8(vv, p.bv + kvh * 64 + c);
                }
                *reinterpret_cast<uint4*>(dK + r * FA_LD + c) = kv;
                *reinterpret_cast<uint4*>(dV + r * FA_LD + c) = vv;
            } else {
                cp_async16(smem_u32(dK + r * FA_LD + c), valid ? srck : p.K, valid);
                cp_async16(smem_u32(dV + r * FA_LD + c), valid ? srcv : p.V, valid);
            }
        }
        if (!BIAS) cp_async_commit();
    };

    const int n_tiles = (total + FA_B - 1) / FA_B;
    if (n_tiles > 0) load_kv(0, 0);
    __syncthreads();

    // ---- Q fragments of this warp's 16 rows (4 k-steps of 16 dims)
    uint32_t qa[4][4];
    {
        const __half* base = sQ + (hl * FA_B + (warp & 3) * 16) * FA_LD;
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8, c = (lane >> 4) * 8;
#pragma unroll
        for (int kk = 0; kk < 4; kk++)
            ldsm_x4(qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], smem_u32(base + r * FA_LD + kk * 16 + c));
    }

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    const int gid = lane >> 2, tig = lane & 3;

    for (int t = 0; t < n_tiles; t++) {
        const int buf = t & 1;
        if (t + 1 < n_tiles) {
            __syncthreads();  // everyone is done reading buffer buf^1 (tile t-1)
            load_kv((t + 1) * FA_B, buf ^ 1);
            if (!BIAS) cp_async_wait<1>();
        } else if (!BIAS) {
            cp_async_wait<0>();
        }
        __syncthreads();
        const __half* cK = sK + buf * FA_B * FA_LD;
        const __half* cV = sV + buf * FA_B * FA_LD;

        // S = Q K^T: 16 rows x 64 keys per warp
        float sc[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < 4; kk += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, smem_u32(cK + (nt * 8 + (lane & 7)) * FA_LD + kk * 16 + (lane >> 3) * 8));
                mma16816(sc[nt], qa[kk], b0, b1);
                mma16816(sc[nt], qa[kk + 1], b2, b3);
            }
        }
        // mask keys beyond the sequence, scale into the exp2 domain, running max
        const int j0 = t * FA_B;
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const int key = j0 + nt * 8 + 2 * tig;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const bool ok = key + e < total;
                sc[nt][e] = ok ? sc[nt][e] * p.scale_log2 : -INFINITY;
                sc[nt][2 + e] = ok ? sc[nt][2 + e] * p.scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, sc[nt][e]);
                mx1 = fmaxf(mx1, sc[nt][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(D1_FULL_MASK, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(D1_FULL_MASK, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(D1_FULL_MASK, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(D1_FULL_MASK, mx1, 2));
        const float nm0 = fmaxf(m0, mx0), nm1 = fmaxf(m1, mx1);
        const float a0 = exp2f(m0 - nm0), a1 = exp2f(m1 - nm1);
        m0 = nm0;
        m1 = nm1;
        float rs0 = 0.f, rs1 = 0.f;
        uint32_t pa[4][4];  // P as A fragments: k-step kk covers key n-tiles 2kk, 2kk+1
#pragma unroll
        for (int nt = 0; nt < 8; nt++) {
            const float p0 = exp2f(sc[nt][0] - nm0), p1 = exp2f(sc[nt][1] - nm0);
            const float p2 = exp2f(sc[nt][2] - nm1), p3 = exp2f(sc[nt][3] - nm1);
            rs0 += p0 + p1;
            rs1 += p2 + p3;
            pa[nt >> 1][(nt & 1) * 2] = pack_h2(p0, p1);
            pa[nt >> 1][(nt & 1) * 2 + 1] = pack_h2(p2, p3);
        }
        l0 = l0 * a0 + rs0;
        l1 = l1 * a1 + rs1;
#pragma unroll
        for (int dt = 0; dt < 8; dt++) {
            o[dt][0] *= a0;
            o[dt][1] *= a0;
            o[dt][2] *= a1;
            o[dt][3] *= a1;
        }
        // O += P V
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
#pragma unroll
            for (int dt = 0; dt < 8; dt += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3,
                          smem_u32(cV + (kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * FA_LD + dt * 8 + (lane >> 4) * 8));
                mma16816(o[dt], pa[kk], b0, b1);
                mma16816(o[dt + 1], pa[kk], b2, b3);
            }
        }
    }

    // ---- normalise, stage through this warp's Q rows in shared memory, 16-byte coalesced stores
    l0 += __shfl_xor_sync(D1_FULL_MASK, l0, 1);
    l0 += __shfl_xor_sync(D1_FULL_MASK, l0, 2);
    l1 += __shfl_xor_sync(D1_FULL_MASK, l1, 1);
    l1 += __shfl_xor_sync(D1_FULL_MASK, l1, 2);
    const float il0 = l0 > 0.f ? 1.f / l0 : 0.f, il1 = l1 > 0.f ? 1.f / l1 : 0.f;
    __half* stage = sQ + (hl * FA_B + (warp & 3) * 16) * FA_LD;
#pragma unroll
    for (int dt = 0; dt < 8; dt++) {
        *reinterpret_cast<uint32_t*>(stage + gid * FA_LD + dt * 8 + 2 * tig) = pack_h2(o[dt][0] * il0, o[dt][1] * il0);
        *reinterpret_cast<uint32_t*>(stage + (gid + 8) * FA_LD + dt * 8 + 2 * tig) =
            pack_h2(o[dt][2] * il1, o[dt][3] * il1);
    }
    __syncwarp();
    const int h = h0 + hl;
#pragma unroll
    for (int i = lane; i < 16 * 8; i += 32) {
        const int r = i / 8, c = (i % 8) * 8;
        const int q = q0 + (warp & 3) * 16 + r;
        if (q < s.q_len)
            *reinterpret_cast<uint4*>(p.O + (size_t)(s.q_start + q) * p.ldo + h * 64 + c) =
                *reinterpret_cast<const uint4*>(stage + r * FA_LD + c);
    }
}

// ---------------------------------------------------------------------------------------------- tcgen05 form
// Persistent CTAs (2 per SM) loop over units = (128-query tile, head); the reference's work list holds 64-row
// tiles, so a unit starts at every item whose first row is a multiple of 128 and the other items are skipped.
// TMEM per CTA: S = Q.K^T (128 x 64 fp32, columns [0,64)) and the output accumulator O (128 x 64 fp32, [64,128)).
// Warps:
//   0-3  softmax: thread t owns query row t (TMEM lane t): reads its S row, online softmax in the exp2 domain,
//        writes P (fp16) into shared memory as the A operand of P.V, rescales its O row in TMEM when its running
//        max rises, and at the end of a unit writes O / l to global memory.
//   4    loader: Q of each unit into a 2-slot ring, K/V tiles of 64 keys ([ext prefix keys | local keys]) into a
//        3-stage ring, with cp.async into the 128-byte-swizzled K-major layout (V is the MN-major B operand of
//        P.V: same bytes). Several copy groups stay in flight; each is signalled when it lands.
//   5    TMEM allocation and the MMA issuer: S_j = Q.K_j^T (M=128, N=64, K=64), then O += P_j.V_j (M=128, N=64,
//        K=64); S_{j+1} is issued as soon as the softmax has read S_j, so the tensor core works while it exps.
// Loads for the next unit are issued while the current one is computed, which hides the copy latency that a
// one-unit-per-CTA kernel exposes on short sequences.
constexpr int TQ = 128;                  // query rows per unit
constexpr int TKV = 64;                  // keys per K/V tile
constexpr int T_QSLOTS = 2, T_KVSTAGES = 3;
constexpr int T_Q_BYTES = TQ * 128;      // 128 rows x 64 dims fp16
constexpr int T_KV_BYTES = TKV * 128;
constexpr int T_P_BYTES = TQ * TKV * 2;
constexpr uint32_t T_TMEM_COLS = 128;
constexpr int T_NBARS = 2 * T_QSLOTS + 2 * T_KVSTAGES + 6;
constexpr int T_SMEM = T_QSLOTS * T_Q_BYTES + T_KVSTAGES * 2 * T_KV_BYTES + T_P_BYTES + T_NBARS * 8 + 16;

// Error word of the attention kernels (a wait that gave up); read and cleared by d1_flash_attn_error().
__device__ int g_fa_err = 0;

struct FaTcArgs {
    const __half* Q;
    const __half* K;
    const __half* V;
    __half* O;
    const AttnSeq* seqs;
    const int2* work;
    int n_units;  // work items x heads
    int heads;
    int ldq, ldkv, ext_ld, ldo, group;
    float scale_log2;
    int* err;
};

__device__ __forceinline__ void fence_async_smem_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void record_err(int* err, volatile int* abort_flag, int code) {
    *abort_flag = 1;
    if (err) atomicExch(err, code);
}

__device__ __forceinline__ bool mbar_wait_timed2(uint32_t bar, uint32_t parity) {
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity))
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    return true;
}

__device__ __forceinline__ void cp_async16z(uint32_t dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}

// 2^x with the hardware approximation (relative error ~2^-22, far below the fp16 rounding of P).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// A unit: work item w (its 64-row query tile must start at a multiple of 128) and head h.
struct Unit {
    AttnSeq s;
    int q0, h, nt;
};
__device__ __forceinline__ bool unit_at(const FaTcArgs& a, int u, Unit& out) {
    const int2 wi = a.work[u / a.heads];
    if (wi.y % TQ) return false;
    out.s = a.seqs[wi.x];
    out.q0 = wi.y;
    out.h = u % a.heads;
    out.nt = (out.s.ext_len + out.s.kv_len + TKV - 1) / TKV;
    return out.nt > 0 && out.s.q_len > out.q0;  // units with no keys or no queries are skipped by every role
}

__global__ void __launch_bounds__(192, 2) k_flash_attn_tc(const FaTcArgs a) {
    constexpr uint32_t IDESC_S = idesc_f16_f32(TQ, TKV);
    constexpr uint32_t IDESC_O = idesc_f16_f32(TQ, 64) | (1u << 16);  // B (= V) MN-major
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sQ = smem_raw;  // the 128-byte swizzle needs 1024-byte aligned tiles: checked below
    uint8_t* sKV = sQ + T_QSLOTS * T_Q_BYTES;  // stage s: K at s * 2 * T_KV_BYTES, V right after
    uint8_t* sP = sKV + T_KVSTAGES * 2 * T_KV_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + T_P_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + T_NBARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    auto q_full = [&](int i) { return smem_u32(bars + i); };
    auto q_empty = [&](int i) { return smem_u32(bars + T_QSLOTS + i); };
    auto kv_full = [&](int i) { return smem_u32(bars + 2 * T_QSLOTS + i); };
    auto kv_empty = [&](int i) { return smem_u32(bars + 2 * T_QSLOTS + T_KVSTAGES + i); };
    const uint32_t s_full = smem_u32(bars + 2 * T_QSLOTS + 2 * T_KVSTAGES);
    const uint32_t s_free = s_full + 8, p_full = s_full + 16, o_done = s_full + 24, o_free = s_full + 32;
    const uint32_t drain = s_full + 40;

    if (smem_u32(smem_raw) & 1023) {  // never expected: dynamic shared memory starts at the window base
        if (threadIdx.x == 0 && a.err) atomicExch(a.err, kErrDrain);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < T_QSLOTS; i++) {
            mbar_init(q_full(i), 32);
            mbar_init(q_empty(i), 1);
        }
        for (int i = 0; i < T_KVSTAGES; i++) {
            mbar_init(kv_full(i), 32);
            mbar_init(kv_empty(i), 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 4);
        mbar_init(p_full, 4);
        mbar_init(o_done, 1);
        mbar_init(o_free, 4);
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(smem_u32(tmem_slot), T_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        // ------------------------------------------------------------------ loader
        // Copy groups in flight, oldest first: the barrier each one signals when it lands (at most 4).
        uint32_t pend[4];
        int npend = 0;
        auto land_oldest = [&](bool all) {
            if (all)
                asm volatile("cp.async.wait_group 0;" ::: "memory");
            else
                asm volatile("cp.async.wait_group 1;" ::: "memory");
            fence_async_smem_cta();
            const int n = all ? npend : npend - 1;
            for (int i = 0; i < n; i++) mbar_arrive(pend[i]);
            for (int i = n; i < npend; i++) pend[i - n] = pend[i];
            npend -= n;
        };
        // wait for a free slot; never block while a landed copy is still unsignalled
        auto acquire = [&](uint32_t bar, uint32_t parity) -> bool {
            if (!__all_sync(D1_FULL_MASK, mbar_try_wait(bar, parity))) {
                if (npend) land_oldest(true);
                return __all_sync(D1_FULL_MASK, mbar_wait(bar, parity, abort_flag)) != 0;
            }
            return true;
        };
        int qi = 0, ki = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < a.n_units && ok; u += gridDim.x) {
            Unit un;
            if (!unit_at(a, u, un)) continue;
            const int g = un.h / a.group, total = un.s.ext_len + un.s.kv_len;
            const int qs = qi % T_QSLOTS;
            if (!(ok = acquire(q_empty(qs), ((qi / T_QSLOTS) & 1) ^ 1))) break;
            uint8_t* dq = sQ + qs * T_Q_BYTES;
            for (int c = lane; c < TQ * 8; c += 32) {
                const int r = c >> 3, ch = c & 7;
                const bool v = un.q0 + r < un.s.q_len;
                const __half* src = v ? a.Q + (size_t)(un.s.q_start + un.q0 + r) * a.ldq + un.h * 64 + ch * 8 : a.Q;
                cp_async16z(smem_u32(dq + r * 128 + ((ch ^ (r & 7)) << 4)), src, v ? 16 : 0);
            }
            asm volatile("cp.async.commit_group;" ::: "memory");
            pend[npend++] = q_full(qs);
            if (npend > 2) land_oldest(false);
            qi++;
            for (int j = 0; j < un.nt; j++) {
                const int s = ki % T_KVSTAGES;
                if (!(ok = acquire(kv_empty(s), ((ki / T_KVSTAGES) & 1) ^ 1))) break;
                uint8_t* dK = sKV + s * 2 * T_KV_BYTES;
                uint8_t* dV = dK + T_KV_BYTES;
                for (int c = lane; c < TKV * 8; c += 32) {
                    const int r = c >> 3, ch = c & 7;
                    const int key = j * TKV + r;
                    const __half *srck = a.K, *srcv = a.V;
                    int bytes = 0;
                    if (key < un.s.ext_len) {
                        srck = un.s.ext_k + (size_t)key * a.ext_ld + g * 64 + ch * 8;
                        srcv = un.s.ext_v + (size_t)key * a.ext_ld + g * 64 + ch * 8;
                        bytes = 16;
                    } else if (key < total) {
                        const size_t row = (size_t)(un.s.kv_start + key - un.s.ext_len) * a.ldkv + g * 64 + ch * 8;
                        srck = a.K + row;
                        srcv = a.V + row;
                        bytes = 16;
                    }
                    const uint32_t off = r * 128 + ((ch ^ (r & 7)) << 4);
                    cp_async16z(smem_u32(dK + off), srck, bytes);
                    cp_async16z(smem_u32(dV + off), srcv, bytes);
                }
                asm volatile("cp.async.commit_group;" ::: "memory");
                pend[npend++] = kv_full(s);
                if (npend > 2) land_oldest(false);
                ki++;
            }
        }
        if (npend) land_oldest(true);
        if (!ok && lane == 0) record_err(a.err, abort_flag, kErrWaitEmpty);
    } else if (warp == 5) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t tS = tmem, tO = tmem + TKV;
            const uint32_t p_addr = smem_u32(sP);
            int qi = 0, ki = 0, ui = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < a.n_units && ok; u += gridDim.x) {
                Unit un;
                if (!unit_at(a, u, un)) continue;
                const int qs = qi % T_QSLOTS;
                if (!(ok = mbar_wait(q_full(qs), (qi / T_QSLOTS) & 1, abort_flag))) break;
                const uint32_t q_addr = smem_u32(sQ + qs * T_Q_BYTES);
                auto issue_s = [&](int kidx) {  // S = Q . K^T for the tile in ring slot kidx
                    const uint32_t k_addr = smem_u32(sKV + (kidx % T_KVSTAGES) * 2 * T_KV_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        tc_mma_f16(tS, smem_desc_k128(q_addr + k * 32), smem_desc_k128(k_addr + k * 32), IDESC_S,
                                   k != 0);
                    tc_commit(s_full);
                };
                // S_0 of this unit: its K tile has landed and the softmax has read the previous S
                ok = mbar_wait(kv_full(ki % T_KVSTAGES), (ki / T_KVSTAGES) & 1, abort_flag) &&
                     (ki == 0 || mbar_wait(s_free, (ki - 1) & 1, abort_flag));
                if (!ok) break;
                tc_fence_after();
                issue_s(ki);
                for (int j = 0; j < un.nt && ok; j++) {
                    const int kj = ki + j;
                    if (j + 1 < un.nt) {
                        ok = mbar_wait(kv_full((kj + 1) % T_KVSTAGES), ((kj + 1) / T_KVSTAGES) & 1, abort_flag) &&
                             mbar_wait(s_free, kj & 1, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        issue_s(kj + 1);
                    }
                    ok = mbar_wait(p_full, kj & 1, abort_flag) &&
                         (j > 0 || ui == 0 || mbar_wait(o_free, (ui - 1) & 1, abort_flag));
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t v_addr = smem_u32(sKV + (kj % T_KVSTAGES) * 2 * T_KV_BYTES + T_KV_BYTES);
#pragma unroll
                    for (int k = 0; k < TKV / 16; k++)
                        tc_mma_f16(tO, smem_desc_k128(p_addr + k * 32), smem_desc_k128(v_addr + k * 2048), IDESC_O,
                                   (j | k) != 0);
                    tc_commit(kv_empty(kj % T_KVSTAGES));
                    tc_commit(o_done);
                }
                if (!ok) break;
                tc_commit(q_empty(qs));
                ki += un.nt;
                qi++;
                ui++;
            }
            if (!ok) record_err(a.err, abort_flag, kErrWaitFull);
            tc_commit(drain);  // every issued MMA has completed before TMEM is released
            if (!mbar_wait_timed2(drain, 0)) record_err(a.err, abort_flag, kErrDrain);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ softmax (warps 0-3, row = thread)
        const int row = warp * 32 + lane;
        const uint32_t tS = tmem + ((uint32_t)(warp * 32) << 16), tO = tS + TKV;
        int ki = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < a.n_units && ok; u += gridDim.x) {
            Unit un;
            if (!unit_at(a, u, un)) continue;
            const int total = un.s.ext_len + un.s.kv_len;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < un.nt; j++) {
                const int kj = ki + j;
                if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(s_full, kj & 1, abort_flag)))) break;
                tc_fence_after();
                uint32_t sr[TKV];
#pragma unroll
                for (int c = 0; c < TKV / 32; c++)
                    tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c * 32));
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(s_free);
                const int kbase = j * TKV;
                float mx = -INFINITY;
#pragma unroll
                for (int c = 0; c < TKV; c++) {
                    const float v = kbase + c < total ? __uint_as_float(sr[c]) * a.scale_log2 : -INFINITY;
                    sr[c] = __float_as_uint(v);
                    mx = fmaxf(mx, v);
                }
                const float m_new = fmaxf(m, mx);
                const float alpha = ex2(m - m_new);
                // P.V of the previous tile (possibly the previous unit's last) has consumed P and updated O
                if (kj > 0 && !(ok = __all_sync(D1_FULL_MASK, mbar_wait(o_done, (kj - 1) & 1, abort_flag)))) break;
                tc_fence_after();
                if (j > 0 && __any_sync(D1_FULL_MASK, alpha < 1.f)) {
                    uint32_t o[32];
#pragma unroll
                    for (int c = 0; c < 2; c++) {
                        tmem_ld32(tO + c * 32, o);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st32(tO + c * 32, o);
                    }
                    tc_wait_st();
                }
                float rs = 0.f;
                uint8_t* prow = sP + row * 128;
#pragma unroll
                for (int ch = 0; ch < 8; ch++) {
                    float p[8];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        p[e] = ex2(__uint_as_float(sr[ch * 8 + e]) - m_new);
                        rs += p[e];
                    }
                    *reinterpret_cast<uint4*>(prow + ((ch ^ (row & 7)) << 4)) =
                        make_uint4(pack_h2(p[0], p[1]), pack_h2(p[2], p[3]), pack_h2(p[4], p[5]), pack_h2(p[6], p[7]));
                }
                fence_async_smem_cta();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full);
                l = l * alpha + rs;
                m = m_new;
            }
            if (!ok) break;
            ki += un.nt;
            if (un.nt == 0) continue;
            if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(o_done, (ki - 1) & 1, abort_flag)))) break;
            tc_fence_after();
            const float il = l > 0.f ? 1.f / l : 0.f;
            const bool store = un.q0 + row < un.s.q_len;
            __half* orow = a.O + (size_t)(un.s.q_start + un.q0 + row) * a.ldo + un.h * 64;
            uint32_t o[2][32];
            tmem_ld32(tO, o[0]);
            tmem_ld32(tO + 32, o[1]);
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);  // the next unit's first P.V may overwrite O
            if (store) {
#pragma unroll
                for (int c = 0; c < 2; c++)
#pragma unroll
                    for (int q = 0; q < 4; q++)
                        *reinterpret_cast<uint4*>(orow + c * 32 + q * 8) = make_uint4(
                            pack_h2(__uint_as_float(o[c][8 * q]) * il, __uint_as_float(o[c][8 * q + 1]) * il),
                            pack_h2(__uint_as_float(o[c][8 * q + 2]) * il, __uint_as_float(o[c][8 * q + 3]) * il),
                            pack_h2(__uint_as_float(o[c][8 * q + 4]) * il, __uint_as_float(o[c][8 * q + 5]) * il),
                            pack_h2(__uint_as_float(o[c][8 * q + 6]) * il, __uint_as_float(o[c][8 * q + 7]) * il));
            }
        }
        if (!ok && lane == 0) record_err(a.err, abort_flag, kErrWaitAccFull);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, T_TMEM_COLS);
    }
}

int launch_fa_tc(FaTcArgs& a, int n_work, int heads, cudaStream_t st) {
    static unsigned long long attr_done = 0;
    static int sms[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(__atomic_load_n(&attr_done, __ATOMIC_ACQUIRE) & bit)) {
        if (cudaFuncSetAttribute(k_flash_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, T_SMEM) != cudaSuccess)
            return -1;
        cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev);
        __atomic_fetch_or(&attr_done, bit, __ATOMIC_RELEASE);
    }
    a.n_units = n_work * heads;
    a.heads = heads;
    const int grid = a.n_units < 2 * sms[dev & 63] ? a.n_units : 2 * sms[dev & 63];
    k_flash_attn_tc<<<grid, 192, T_SMEM, st>>>(a);
    return (int)cudaGetLastError();
}

template <int HPC, bool BIAS>
int launch_fa(const FaArgs& a, int n_work, int gy, cudaStream_t st) {
    constexpr size_t smem = (size_t)(HPC * FA_B * FA_LD + 4 * FA_B * FA_LD) * sizeof(__half);
    // The shared-memory opt-in is per function and device: set it on the first launch on each device.
    static unsigned long long attr_done = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const unsigned long long bit = 1ull << (dev & 63);
    if (!(__atomic_load_n(&attr_done, __ATOMIC_ACQUIRE) & bit)) {
        if (cudaFuncSetAttribute(k_flash_attn<HPC, BIAS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return -1;
        __atomic_fetch_or(&attr_done, bit, __ATOMIC_RELEASE);
    }
    dim3 grid(n_work, gy);
    k_flash_attn<HPC, BIAS><<<grid, 128 * HPC, smem, st>>>(a);
    return (int)cudaGetLastError();
}

}  // namespace

extern "C" int d1_flash_attn_tc(const d1_half* Q, int ldq, const d1_half* K, const d1_half* V, int ldkv, int ext_ld,
                                d1_half* O, int ldo, const AttnSeq* seqs, const int* work, int n_work, int heads,
                                int group, float scale, cudaStream_t st) {
    if (n_work <= 0) return n_work == 0 ? 0 : -1;
    if (heads <= 0 || group <= 0 || heads % group) return -1;
    if ((((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)O) & 15) || (ldq | ldkv | ldo | ext_ld) % 8) return -1;
    FaTcArgs t;
    t.Q = Q;
    t.K = K;
    t.V = V;
    t.O = O;
    t.seqs = seqs;
    t.work = reinterpret_cast<const int2*>(work);
    t.ldq = ldq;
    t.ldkv = ldkv;
    t.ext_ld = ext_ld;
    t.ldo = ldo;
    t.group = group;
    t.scale_log2 = scale * 1.4426950408889634f;
    static int* err_addr[64] = {};  // device address of g_fa_err, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!err_addr[dev & 63] && cudaGetSymbolAddress(reinterpret_cast<void**>(&err_addr[dev & 63]), g_fa_err) != cudaSuccess)
        return -1;
    t.err = err_addr[dev & 63];
    return launch_fa_tc(t, n_work, heads, st);
}

extern "C" int d1_flash_attn_error(void) {
    int e = 0;
    if (cudaMemcpyFromSymbol(&e, g_fa_err, sizeof(int)) != cudaSuccess) return -1;
    if (e) {
        const int z = 0;
        cudaMemcpyToSymbol(g_fa_err, &z, sizeof(int));
    }
    return e;
}

extern "C" int d1_flash_attn(const d1_half* Q, int ldq, const d1_half* K, const d1_half* V, int ldkv, int ext_ld,
                             const float* bq, const float* bk, const float* bv, d1_half* O, int ldo,
                             const AttnSeq* seqs, const int* work, int n_work, int heads, int group, float scale,
                             cudaStream_t st) {
    if (n_work <= 0) return n_work == 0 ? 0 : -1;
    if (heads <= 0 || group <= 0 || heads % group) return -1;
    if ((((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)O) & 15) || (ldq | ldkv | ldo | ext_ld) % 8) return -1;
    FaArgs a;
    a.Q = Q;
    a.K = K;
    a.V = V;
    a.bq = bq;
    a.bk = bk;
    a.bv = bv;
    a.O = O;
    a.seqs = seqs;
    a.work = reinterpret_cast<const int2*>(work);
    a.ldq = ldq;
    a.ldkv = ldkv;
    a.ext_ld = ext_ld;
    a.ldo = ldo;
    a.group = group;
    a.scale_log2 = scale * 1.4426950408889634f;
    const bool bias = bq || bk || bv;
    if (group == 2) {
        const int gy = heads / 2;
        return bias ? launch_fa<2, true>(a, n_work, gy, st) : launch_fa<2, false>(a, n_work, gy, st);
    }
    return bias ? launch_fa<1, true>(a, n_work, heads, st) : launch_fa<1, false>(a, n_work, heads, st);
}
