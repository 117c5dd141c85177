// Packed variable-length bidirectional flash attention, head dim 64, for the d1rs trunk (GQA), the decision head
// (MHA + q/k/v bias), and the SigLIP2 tower. Replaces d1_flash_attn of the reference (cuda/kernels.cu:351-500,
// launcher :726-734) with the same arguments and semantics:
//   for every work item (seq, q0) and head h: O[q] = softmax(scale * Q[q] . K^T) . V over the keys
//   [ext prefix keys | local keys] of that sequence, kv head g = h / group, fp32 softmax, optional fp32 biases
//   added to q/k/v as they are loaded.
//
// Design: one CTA per (64-query tile, kv head) runs all the query heads that share that kv head (GQA group 2:
// 8 warps, two heads), so each K/V tile is fetched once for the group. Each warp owns 16 query rows of one head.
// K/V tiles of 64 keys are double-buffered in shared memory with cp.async (bias-free case) so the next tile's
// loads overlap this tile's math; QK^T and PV run on m16n8k16 fp16 tensor-core MMAs with fp32 accumulation,
// S stays in registers and is re-packed as the A operand of PV; the online softmax works in the exp2 domain.
// The output tile is staged through shared memory for 16-byte coalesced stores.
#include "common.cuh"

using namespace d1;

namespace {

constexpr int FA_B = 64;    // query rows per tile and keys per K/V tile
constexpr int FA_LD = 72;   // padded shared-memory row (halves): conflict-free ldmatrix

__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    const int n = valid ? 16 : 0;  // src-size 0: zero-fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

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
__global__ void __launch_bounds__(128 * HPC) k_flash_attn(const FaArgs p) {
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
