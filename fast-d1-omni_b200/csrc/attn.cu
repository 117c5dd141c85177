// Packed variable-length bidirectional flash attention, head dim 64, for the d1rs trunk (GQA), the decision head
// (MHA + q/k/v bias), and the SigLIP2 tower. Replaces d1_flash_attn of the reference (cuda/kernels.cu:351-500,
// launcher :726-734) with the same arguments and semantics:
//   for every work item (seq, q0) and head h: O[q] = softmax(scale * Q[q] . K^T) . V over the keys
//   [ext prefix keys | local keys] of that sequence, kv head g = h / group, fp32 softmax, optional fp32 biases
//   added to q/k/v as they are loaded.
//
// d1_flash_attn takes any work list, as the reference's kernel does. Without biases it runs the tcgen05 kernel below
// on the 256-row blocks the list names whole (all of the reference's own lists) and an mma.sync kernel on any other
// item (see "reference ABI" below); with biases, the mma.sync kernel alone. The mma.sync kernel: one CTA per
// (64-query tile, kv head) runs all the query heads that share that kv head (GQA group 2: 8 warps, two heads), so
// each K/V tile is fetched once for the group. Each warp owns 16 query rows of one head. K/V tiles of 64 keys are
// double-buffered in shared memory with cp.async (bias-free case) so the next tile's loads overlap this tile's math;
// QK^T and PV run on m16n8k16 fp16 tensor-core MMAs with fp32 accumulation, S stays in registers and is re-packed as
// the A operand of PV; the online softmax works in the exp2 domain. The output tile is staged through shared memory
// for 16-byte coalesced stores; 2 CTAs per SM. It adds biases on load.
//
// d1_flash_attn_tc (extension) is the same computation for the bias-free forms on tcgen05 (k_flash_attn_tc below:
// S, P and O in TMEM, 128-key tiles, the next score tile computed while two softmax warpgroups run the exponentials,
// TMA loads and stores). Measured on B200 (CUDA events, 16 heads, GQA 2): ~24.3 us at 32 x 256 tokens (44 us for the
// mma.sync kernel) and ~117 us at 4 x 2048 tokens (587 TF/s; 263 us). The runners use it whenever the attention has
// no biases to add on load (their work lists cover every 256-row block).
#include <map>
#include <mutex>

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
    const int* n_items;  // when set: a pool of *n_items work items that the CTAs of each kv head (blockIdx.y) take
    int* next_item;      // in turn through next_item[blockIdx.y]
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

    pdl_entry();
    // one item per CTA, or (the leftovers of the ABI split) items taken from a pool in turn until it is empty
    __shared__ int s_item;
    const int n_items = p.n_items ? *p.n_items : 0;
    for (int iter = 0;; iter++) {
        int item = blockIdx.x;
        if (p.n_items) {
            __syncthreads();  // the previous item's shared-memory reads are done, and s_item is free
            if (threadIdx.x == 0) s_item = atomicAdd(p.next_item + blockIdx.y, 1);
            __syncthreads();
            item = s_item;
            if (item >= n_items) break;
        } else if (iter > 0) {
            break;
        }
        const int2 wi = p.work[item];
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
}

// ---------------------------------------------------------------------------------------------- tcgen05 form
// Persistent CTAs (one per SM) loop over units = (256-query block, head). A unit starts at every work item whose
// first row is a multiple of 256; other items are skipped, so the reference's list of 64-row tiles works as it is
// (it must cover every tile) and the runners pass one item per 256-row block. A unit is two 128-row query tiles
// that share each K/V tile, one per softmax warpgroup.
//
// Each softmax warpgroup has its own S, P and O columns in TMEM. The softmax copies S(j) into registers and releases
// it at once (SFREE), so the MMA issuer computes S(j+1) = Q.K_{j+1}^T while the exponentials of tile j run; P(j) goes
// to the P columns as fp16 pairs once P(j-1).V_{j-1} has read them (ODONE), and P(j).V_j reads its A operand from
// there (tcgen05.mma with A in tensor memory). The softmax therefore almost never waits for its scores: the
// critical resource is the SFU (ex2), shared by the two warpgroups.
// TMEM (512 columns): warpgroup w at 256w: S in 128 columns, P in 64, O in 64.
// Warps:
//   0-3, 4-7  softmax warpgroups 0 and 1: thread t owns query row t of its tile (TMEM lane t). Per 128-key tile it
//        reads its S row (one TMEM round trip), takes the row max in the exp2 domain (3-input max), writes
//        P = 2^(s - m) as fp16 to TMEM and accumulates the row sum. O is rescaled in TMEM only when the row max
//        grows by more than 8 (log2 units); otherwise P is taken against the old max (P <= 2^8, well inside fp16)
//        and the final O / l is unchanged. At the end of a unit it writes O / l to global memory: a whole 128-row
//        tile through its own shared-memory staging buffer and one bulk tensor store.
//   8, 10, 11  loaders: the unit's two Q tiles into a 2-slot ring and K/V tiles of 128 keys ([ext prefix keys |
//        local keys]) into a 4-stage ring, in the swizzled layouts (V is the MN-major B operand of P.V: same
//        bytes): Q and whole local K/V tiles by TMA from one thread, prefix and partial tiles by cp.async from all
//        three warps (each lane's copies complete the slot's barrier when they land); the next unit's loads overlap
//        the current unit's math.
//   9    TMEM allocation and the MMA issuer (one thread): S_w(j) = Q_w.K_j^T (M=128, N=128, K=64, both operands in
//        shared memory) and O_w += P_w(j).V_j (M=128, N=64, K=128, A in TMEM).
// Measured on B200 (per-tile clock64 stamps and a tcgen05 microbenchmark): an exponential phase of 128 keys takes
// ~1500 clocks for one warp alone and ~2400 when both warpgroups run it at once (the SFU does 16 lanes per clock
// per SM); loads, max and the P store add ~1100 per tile. One in eight exponential pairs is therefore computed on
// the FMA pipe (ex2_poly2). The A-in-TMEM P.V runs at ~67 clocks per N=64 instruction (half the dense rate) but
// overlaps the shared-memory S MMAs. (Tried and slower or equal: 64-key tiles with S two tiles ahead, 145 us at
// 4 x 2048 against 117; 96-key tiles with two S buffers, 123 us; the two warpgroups taking turns on the
// exponentials, 128 us; four softmax warpgroups, two per query tile each taking 64 of the 128 keys and exchanging
// the row max through shared memory, 127 us; a fourth warpgroup that reads, normalises and stores O so the softmax
// warpgroups go straight on to the next unit (512 threads, registers split 184 / 72 by setmaxnreg), 126 against 121 us
// and 28.3 against 25.7 us at 32 x 256; units taken from a device counter through a shared-memory ring instead of
// round robin, 6-7% faster on ragged batches of 8192-16384 tokens but 10-14% slower at 32 x 256; a quarter of the
// exponentials on the FMA pipe, 122 us; the row sums
// by one more MMA per tile, P times a shared-memory tile whose first column is ones, 144 -> 189 us with P through
// shared memory.)
constexpr int TQ = 128;                   // query rows per tile (TMEM lanes)
constexpr int TQU = 2 * TQ;               // query rows per unit
constexpr int TKV = 128;                  // keys per K/V tile
constexpr int T_QSLOTS = 2, T_KVSTAGES = 4;
constexpr int T_QT_BYTES = TQ * 128;      // one 128-row x 64-dim fp16 tile
constexpr int T_KV_BYTES = TKV * 128;     // K or V of one tile
constexpr int T_O_BYTES = TQ * 128;       // one warpgroup's O staging tile
constexpr uint32_t T_TMEM_COLS = 512;
constexpr uint32_t T_WG_COLS = 256;       // TMEM columns per warpgroup: S, P, O
constexpr uint32_t T_P_COL = TKV;         // P: TKV fp16 keys, two per column
constexpr uint32_t T_O_COL = TKV + TKV / 2;
constexpr float kLazyRescale = 8.f;
enum : int {
    B_QFULL = 0,
    B_QEMPTY = B_QFULL + T_QSLOTS,
    B_KVFULL = B_QEMPTY + T_QSLOTS,
    B_KVEMPTY = B_KVFULL + T_KVSTAGES,
    B_SFULL = B_KVEMPTY + T_KVSTAGES,  // [w]: S of the warpgroup's next tile is in TMEM
    B_PFULL = B_SFULL + 2,             // [w]: its P is in TMEM (4 warp arrivals)
    B_ODONE = B_PFULL + 2,             // [w]: P.V of its last P has completed
    B_OFREE = B_ODONE + 2,             // [w]: its O has been read (4 warp arrivals)
    B_DRAIN = B_OFREE + 2,
    B_OSTAGED = B_DRAIN + 1,           // [w]: the warpgroup's O tile is in shared memory (4 warp arrivals)
    B_OREAD = B_OSTAGED + 2,           // [w]: its previous bulk store has read the staging buffer
    B_SFREE = B_OREAD + 2,             // [w]: the warpgroup has read its S tile (4 warp arrivals)
    T_NBARS = B_SFREE + 2
};
constexpr int T_SMEM = T_QSLOTS * 2 * T_QT_BYTES + T_KVSTAGES * 2 * T_KV_BYTES + 2 * T_O_BYTES + T_NBARS * 8 + 16;
static_assert(T_SMEM <= 232448, "shared memory of the tcgen05 attention");
static_assert(T_O_COL + 64 <= T_WG_COLS && 2 * T_WG_COLS <= T_TMEM_COLS, "TMEM of the tcgen05 attention");

// Error word of the attention kernels (a wait that gave up); read and cleared by d1_flash_attn_error().
__device__ int g_fa_err = 0;

struct FaTcArgs {
    const __half* Q;
    const __half* K;
    const __half* V;
    __half* O;
    const AttnSeq* seqs;
    const int2* work;
    const int* n_blocks;  // when set, the number of work items is read from here (device count)
    int n_units;  // work items x heads
    int heads;
    int ldq, ldkv, ext_ld, ldo, group;
    float scale_log2;
    int* err;
};

__device__ __forceinline__ void fence_async_smem_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bulk tensor store of a staged O tile and its completion waits (issued and awaited by one thread).
__device__ __forceinline__ void o_tile_store(const CUtensorMap* map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)map),
                 "r"(src), "r"(x), "r"(y)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void o_store_read_done() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void o_store_done() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

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

// Two fp32 lanes in one 64-bit register for the packed sm_100 instructions: d = a * b + c and d = a + b, per lane.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 2^x of two lanes on the FMA pipe (Cody-Waite style): n = round(x) by the 1.5 * 2^23 shifter, f = x - n in
// [-0.5, 0.5], 2^f by a cubic fitted for relative error on that interval (7.5e-5 max, below the fp16 rounding of
// P), 2^n added into the exponent field. x is clamped to -126 first (masked keys give ~1e-38, zero in fp16).
__device__ __forceinline__ void ex2_poly2(float x0, float x1, float& p0, float& p1) {
    const uint64_t x = f2_pack(fmaxf(x0, -126.f), fmaxf(x1, -126.f));
    const uint64_t t = f2_add(x, f2_pack(12582912.f, 12582912.f));
    const uint64_t n = f2_add(t, f2_pack(-12582912.f, -12582912.f));
    const uint64_t f = f2_fma(n, f2_pack(-1.f, -1.f), x);
    uint64_t q = f2_fma(f2_pack(0.0551716685f, 0.0551716685f), f, f2_pack(0.24261114f, 0.24261114f));
    q = f2_fma(q, f, f2_pack(0.69326097f, 0.69326097f));
    q = f2_fma(q, f, f2_pack(0.99992806f, 0.99992806f));
    float q0, q1, t0, t1;
    f2_unpack(q, q0, q1);
    f2_unpack(t, t0, t1);
    p0 = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(t0) << 23));
    p1 = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(t1) << 23));
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// D[tmem] (+)= A[tmem] . B[smem]: A (M=128 rows = TMEM lanes, K fp16 values packed two per 32-bit column) in
// tensor memory, B through a shared-memory descriptor, fp32 accumulate; shape from the instruction descriptor.
__device__ __forceinline__ void tc_mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
        : "memory");
}

// A unit: work item w (its 64-row query tile must start at a multiple of 256) and head h.
struct Unit {
    AttnSeq s;
    int q0, h, nt;
    bool two;  // the second 128-row tile has queries
};
// This CTA's next unit at or after candidate u (its candidates are u, u + gridDim.x, ...); false when none is left.
// Every role walks the same sequence.
__device__ __forceinline__ bool next_unit(const FaTcArgs& a, int n_units, int& u, Unit& out) {
    for (; u < n_units; u += gridDim.x) {
        const int2 wi = a.work[u / a.heads];
        if (wi.y % TQU) continue;
        out.s = a.seqs[wi.x];
        out.q0 = wi.y;
        out.h = u % a.heads;
        out.nt = (out.s.ext_len + out.s.kv_len + TKV - 1) / TKV;
        out.two = out.s.q_len > out.q0 + TQ;
        if (out.nt > 0 && out.s.q_len > out.q0) return true;  // units with no keys or no queries are skipped
    }
    return false;
}

constexpr int T_LOADERS = 3;             // loader warps (8, 10, 11): K/V copy issue is instruction-bound
constexpr int T_THREADS = 384;

__global__ void __launch_bounds__(T_THREADS, 1)
    k_flash_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const FaTcArgs a) {
    constexpr uint32_t IDESC_S = idesc_f16_f32(TQ, TKV);
    constexpr uint32_t IDESC_O = idesc_f16_f32(TQ, 64) | (1u << 16);  // B (= V) MN-major
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sQ = smem_raw;                                    // slot q: Q0 at q * 2 * T_QT_BYTES, Q1 after it
    uint8_t* sKV = sQ + T_QSLOTS * 2 * T_QT_BYTES;             // stage s: K at s * 2 * T_KV_BYTES, V after it
    uint8_t* sO = sKV + T_KVSTAGES * 2 * T_KV_BYTES;           // O staging of warpgroup w at w * T_O_BYTES
    uint64_t* bars = reinterpret_cast<uint64_t*>(sO + 2 * T_O_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + T_NBARS);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    auto bar = [&](int i) { return smem_u32(bars + i); };

    if (smem_u32(smem_raw) & 1023) {  // never expected: dynamic shared memory starts at the window base
        pdl_wait();
        if (threadIdx.x == 0 && a.err) atomicExch(a.err, kErrDrain);
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int i = 0; i < T_QSLOTS; i++) {
            mbar_init(bar(B_QFULL + i), 1);
            mbar_init(bar(B_QEMPTY + i), 1);
        }
        for (int i = 0; i < T_KVSTAGES; i++) {
            mbar_init(bar(B_KVFULL + i), 32 * T_LOADERS);
            mbar_init(bar(B_KVEMPTY + i), 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(B_SFULL + i), 1);
            mbar_init(bar(B_PFULL + i), 4);
            mbar_init(bar(B_ODONE + i), 1);
        }
        mbar_init(bar(B_OFREE + 0), 4);
        mbar_init(bar(B_OFREE + 1), 4);
        mbar_init(bar(B_DRAIN), 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(bar(B_OSTAGED + i), 4);
            mbar_init(bar(B_OREAD + i), 1);
            mbar_init(bar(B_SFREE + i), 4);
        }
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 8 && lane == 0) {
        prefetch_tmap(&tmQ);
        prefetch_tmap(&tmK);
        prefetch_tmap(&tmV);
        prefetch_tmap(&tmO);
    }
    if (warp == 9) {
        tmem_alloc(smem_u32(tmem_slot), T_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_entry();  // barriers and TMEM are set up; global memory is touched only after this
    const int n_units = a.n_blocks ? *a.n_blocks * a.heads : a.n_units;

    if (warp == 8 || warp >= 10) {
        // ------------------------------------------------------------------ loaders (warps 8, 10, 11)
        // Q tiles and K/V tiles of local keys come in by TMA, issued by one thread (warp 8, lane 0) into the
        // 128-byte-swizzled layouts the MMAs read. A K/V tile with prefix keys (their rows live in a per-sequence
        // buffer) or with keys past the sequence end (they must read as zeros) is copied by all three loader warps
        // with cp.async instead; each lane's copies complete the stage's barrier by themselves
        // (cp.async.mbarrier.arrive.noinc counts the lane once its earlier copies have landed). A TMA stage
        // completes on its byte count plus the other 95 lanes' plain arrivals, so both kinds use one barrier count.
        const int lt = (warp == 8 ? 0 : warp - 9) * 32 + lane;  // loader thread 0 .. 32 * T_LOADERS - 1
        const bool issuer = warp == 8 && lane == 0;
        auto landed_arrive = [&](uint32_t b) {
            asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(b) : "memory");
        };
        int qi = 0, ki = 0;
        bool ok = true;
        Unit un;
        for (int u = blockIdx.x; ok && next_unit(a, n_units, u, un); u += gridDim.x) {
            const int g = un.h / a.group, total = un.s.ext_len + un.s.kv_len;
            const int qs = qi % T_QSLOTS;
            if (warp == 8) {
                if (!(ok = __all_sync(D1_FULL_MASK,
                                      mbar_wait(bar(B_QEMPTY + qs), ((qi / T_QSLOTS) & 1) ^ 1, abort_flag))))
                    break;
                // A Q tile inside the sequence comes by TMA; one that the sequence ends in is copied row by row with
                // the rows past its end as zeros, so no load reads a row outside a sequence. The copies are complete
                // and visible to the tensor core before the slot's one arrival.
                const uint32_t dq = smem_u32(sQ + qs * 2 * T_QT_BYTES);
                const int nq = un.two ? 2 : 1;
                bool partial = false;
                for (int t = 0; t < nq; t++) {
                    const int rows = un.s.q_len - (un.q0 + t * TQ);
                    if (rows >= TQ) continue;
                    partial = true;
                    for (int c = lane; c < TQ * 8; c += 32) {
                        const int r = c >> 3, ch = c & 7;
                        const __half* src =
                            r < rows ? a.Q + (size_t)(un.s.q_start + un.q0 + t * TQ + r) * a.ldq + un.h * 64 + ch * 8 : a.Q;
                        cp_async16z(dq + t * T_QT_BYTES + r * 128 + ((ch ^ (r & 7)) << 4), src, r < rows ? 16 : 0);
                    }
                }
                if (partial) {
                    asm volatile("cp.async.wait_all;" ::: "memory");
                    fence_async_smem_cta();
                    __syncwarp();
                }
                if (issuer) {
                    uint32_t bytes = 0;
                    for (int t = 0; t < nq; t++)
                        if (un.s.q_len - (un.q0 + t * TQ) >= TQ) bytes += T_QT_BYTES;
                    mbar_arrive_expect_tx(bar(B_QFULL + qs), bytes);
                    for (int t = 0; t < nq; t++)
                        if (un.s.q_len - (un.q0 + t * TQ) >= TQ)
                            tma_load_2d(dq + t * T_QT_BYTES, &tmQ, un.h * 64, un.s.q_start + un.q0 + t * TQ,
                                        bar(B_QFULL + qs));
                }
            }
            qi++;
            for (int j = 0; j < un.nt; j++) {
                const int st = ki % T_KVSTAGES;
                if (!(ok = __all_sync(D1_FULL_MASK,
                                      mbar_wait(bar(B_KVEMPTY + st), ((ki / T_KVSTAGES) & 1) ^ 1, abort_flag))))
                    break;
                uint8_t* dK = sKV + st * 2 * T_KV_BYTES;
                uint8_t* dV = dK + T_KV_BYTES;
                const int key0 = j * TKV;
                if (key0 >= un.s.ext_len && key0 + TKV <= total) {
                    if (issuer) {
                        const int row = un.s.kv_start + key0 - un.s.ext_len;
                        mbar_arrive_expect_tx(bar(B_KVFULL + st), 2 * T_KV_BYTES);
                        tma_load_2d(smem_u32(dK), &tmK, g * 64, row, bar(B_KVFULL + st));
                        tma_load_2d(smem_u32(dV), &tmV, g * 64, row, bar(B_KVFULL + st));
                    } else {
                        mbar_arrive(bar(B_KVFULL + st));
                    }
                } else {
                    for (int c = lt; c < TKV * 8; c += 32 * T_LOADERS) {
                        const int r = c >> 3, ch = c & 7;
                        const int key = key0 + r;
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
                    landed_arrive(bar(B_KVFULL + st));
                }
                ki++;
            }
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // nothing in flight when the CTA exits
        if (!ok && lane == 0) record_err(a.err, abort_flag, kErrWaitEmpty);
        if (issuer) {
            // TMA copies still in flight (only after an abort) land before the CTA exits: wait (bounded) for the
            // last use of every stage and Q slot
            for (int i = ki > T_KVSTAGES ? ki - T_KVSTAGES : 0; i < ki; i++)
                if (!mbar_wait_timed2(bar(B_KVFULL + i % T_KVSTAGES), (i / T_KVSTAGES) & 1)) break;
            for (int i = qi > T_QSLOTS ? qi - T_QSLOTS : 0; i < qi; i++)
                if (!mbar_wait_timed2(bar(B_QFULL + i % T_QSLOTS), (i / T_QSLOTS) & 1)) break;
        }
    } else if (warp == 9) {
        // ------------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            int cnt[2] = {0, 0}, units[2] = {0, 0};  // tiles and units given to each warpgroup so far
            int qi = 0, ki = 0;
            bool ok = true;
            Unit un;
            for (int u = blockIdx.x; ok && next_unit(a, n_units, u, un); u += gridDim.x) {
                const int nw = un.two ? 2 : 1;
                const int qs = qi % T_QSLOTS;
                if (!(ok = mbar_wait(bar(B_QFULL + qs), (qi / T_QSLOTS) & 1, abort_flag))) break;
                const uint32_t q_addr = smem_u32(sQ + qs * 2 * T_QT_BYTES);
                auto k_addr = [&](int j) { return smem_u32(sKV + ((ki + j) % T_KVSTAGES) * 2 * T_KV_BYTES); };
                auto kv_ready = [&](int j) {
                    return mbar_wait(bar(B_KVFULL + (ki + j) % T_KVSTAGES), ((ki + j) / T_KVSTAGES) & 1, abort_flag);
                };
                // S_w(j) into the warpgroup's S columns once its softmax has read S_w(j - 1) (its tile cnt[w] + j - 1)
                auto issue_s = [&](int w, int j) -> bool {
                    const int c = cnt[w] + j;
                    if (c > 0 && !mbar_wait(bar(B_SFREE + w), (c - 1) & 1, abort_flag)) return false;
                    tc_fence_after();
                    const uint32_t ka = k_addr(j);
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        tc_mma_f16(tmem + w * T_WG_COLS, smem_desc_k128(q_addr + w * T_QT_BYTES + k * 32),
                                   smem_desc_k128(ka + k * 32), IDESC_S, k != 0);
                    tc_commit(bar(B_SFULL + w));
                    return true;
                };
                if (!(ok = kv_ready(0))) break;
                for (int w = 0; w < nw && ok; w++) ok = issue_s(w, 0);
                for (int j = 0; j < un.nt && ok; j++) {
                    if (j + 1 < un.nt) {  // S(j+1) computes while the softmax works on tile j
                        if (!(ok = kv_ready(j + 1))) break;
                        for (int w = 0; w < nw && ok; w++) ok = issue_s(w, j + 1);
                        if (!ok) break;
                    }
                    const uint32_t v_addr = k_addr(j) + T_KV_BYTES;
                    for (int w = 0; w < nw && ok; w++) {
                        const int c = cnt[w] + j;
                        ok = mbar_wait(bar(B_PFULL + w), c & 1, abort_flag);
                        // the first P.V of a unit overwrites O_w: its previous unit's O must have been read
                        if (ok && j == 0 && units[w] > 0) ok = mbar_wait(bar(B_OFREE + w), (units[w] - 1) & 1, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
#pragma unroll
                        for (int k = 0; k < TKV / 16; k++)
                            tc_mma_f16_ts(tmem + w * T_WG_COLS + T_O_COL, tmem + w * T_WG_COLS + T_P_COL + k * 8,
                                          smem_desc_k128(v_addr + k * 2048), IDESC_O, (j | k) != 0);
                        tc_commit(bar(B_ODONE + w));
                    }
                    if (!ok) break;
                    tc_commit(bar(B_KVEMPTY + (ki + j) % T_KVSTAGES));
                }
                if (!ok) break;
                tc_commit(bar(B_QEMPTY + qs));
                ki += un.nt;
                qi++;
                for (int w = 0; w < nw; w++) {
                    cnt[w] += un.nt;
                    units[w]++;
                }
            }
            if (!ok) record_err(a.err, abort_flag, kErrWaitFull);
            tc_commit(bar(B_DRAIN));  // every issued MMA has completed before TMEM is released
            if (!mbar_wait_timed2(bar(B_DRAIN), 0)) record_err(a.err, abort_flag, kErrDrain);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ softmax (warpgroups 0 and 1)
        const int w = warp >> 2, row = (warp & 3) * 32 + lane;
        const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tO = tmem + w * T_WG_COLS + T_O_COL + lane_off;
        const uint32_t tP = tmem + w * T_WG_COLS + T_P_COL + lane_off;
        uint8_t* stile = sO + w * T_O_BYTES;
        int cnt = 0;
        int nst = 0;  // O tiles this warpgroup has staged
        bool ok = true;
        Unit un;
        for (int u = blockIdx.x; ok && next_unit(a, n_units, u, un); u += gridDim.x) {
            if (w == 1 && !un.two) continue;
            const int total = un.s.ext_len + un.s.kv_len;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < un.nt; j++) {
                const int c = cnt + j;
                if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(bar(B_SFULL + w), c & 1, abort_flag)))) break;
                tc_fence_after();
                uint32_t sr[TKV];
                const uint32_t tS = tmem + w * T_WG_COLS + lane_off;
#pragma unroll
                for (int c32 = 0; c32 < TKV / 32; c32++)
                    tmem_ld32(tS + c32 * 32, *reinterpret_cast<uint32_t(*)[32]>(sr + c32 * 32));
                tc_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_SFREE + w));  // S is in registers: S(j+1) may overwrite it
                const int kbase = j * TKV;
                if (kbase + TKV > total) {  // keys past the sequence: only in its last tile
#pragma unroll
                    for (int i = 0; i < TKV; i++)
                        if (kbase + i >= total) sr[i] = __float_as_uint(-INFINITY);
                }
                // the max of the raw scores (the scale is positive) in eight independent 3-input chains, scaled
                // once; the exponent below folds the scale in: P = 2^(s * scale - m)
                float mx8[8];
#pragma unroll
                for (int e = 0; e < 8; e++) mx8[e] = fmaxf(__uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1]));
#pragma unroll
                for (int i = 16; i < TKV; i += 16) {
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        mx8[e] = fmax3(mx8[e], __uint_as_float(sr[i + 2 * e]), __uint_as_float(sr[i + 2 * e + 1]));
                }
                const float mx = fmaxf(fmax3(mx8[0], mx8[1], mx8[2]), fmax3(mx8[3], mx8[4], fmax3(mx8[5], mx8[6], mx8[7]))) *
                                 a.scale_log2;
                float m_use = m, alpha = 1.f;
                if (j == 0) {
                    m_use = mx;
                } else if (mx > m + kLazyRescale) {
                    m_use = mx;
                    alpha = ex2(m - mx);
                }
                if (j > 0 && __any_sync(D1_FULL_MASK, alpha < 1.f)) {  // rare: O must hold P.V up to tile c - 1
                    const int cp = c - 1;
                    if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(bar(B_ODONE + w), cp & 1, abort_flag)))) break;
                    tc_fence_after();
#pragma unroll 1
                    for (int q = 0; q < 8; q++) {
                        uint32_t o[8];
                        tmem_ld8(tO + q * 8, o);
                        tc_wait_ld();
#pragma unroll
                        for (int i = 0; i < 8; i++) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
                        tmem_st8(tO + q * 8, o);
                    }
                }
                // x = s * scale - m two scores at a time; P = 2^x; the row sum in four packed pairs of partial sums
                const uint64_t sc2 = f2_pack(a.scale_log2, a.scale_log2), nm2 = f2_pack(-m_use, -m_use);
                uint64_t rs2[4];
#pragma unroll
                for (int e = 0; e < 4; e++) rs2[e] = f2_pack(0.f, 0.f);
                uint32_t pr[TKV / 2];
#pragma unroll
                for (int i = 0; i < TKV / 2; i++) {
                    float x0, x1;
                    f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nm2),
                              x0, x1);
                    float p0, p1;
                    if (i % 8 == 7) {
                        ex2_poly2(x0, x1, p0, p1);
                    } else {
                        p0 = ex2(x0);
                        p1 = ex2(x1);
                    }
                    rs2[i & 3] = f2_add(rs2[i & 3], f2_pack(p0, p1));
                    pr[i] = pack_h2(p0, p1);
                }
                float rs8[8];
#pragma unroll
                for (int e = 0; e < 4; e++) f2_unpack(rs2[e], rs8[2 * e], rs8[2 * e + 1]);
                // P(j) into the P columns (two fp16 keys per column), the A operand of P.V, once P.V(j-1) has read
                // them
                if (c > 0) {
                    if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(bar(B_ODONE + w), (c - 1) & 1, abort_flag)))) break;
                    tc_fence_after();
                }
#pragma unroll
                for (int c32 = 0; c32 < TKV / 64; c32++)
                    tmem_st32(tP + c32 * 32, *reinterpret_cast<uint32_t(*)[32]>(pr + c32 * 32));
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_PFULL + w));
                const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
                l = l * alpha + rs;
                m = m_use;
            }
            if (!ok) break;
            cnt += un.nt;
            // the unit's last P.V (the earlier ones completed before it)
            const int cl = cnt - 1;
            if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(bar(B_ODONE + w), cl & 1, abort_flag)))) break;
            tc_fence_after();
            const float il = l > 0.f ? 1.f / l : 0.f;
            uint32_t o[64];
            tmem_ld32(tO, *reinterpret_cast<uint32_t(*)[32]>(o));
            tmem_ld32(tO + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
            tc_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(bar(B_OFREE + w));  // O is read: the next unit's first P.V may overwrite it
            const int q0w = un.q0 + w * TQ, q = q0w + row;
            if (q0w + TQ <= un.s.q_len) {
                // a whole 128-row tile: staged in this warpgroup's buffer, then one bulk tensor store of 16 KB. The
                // previous store from the buffer must have read it first (long done by now: a unit ago).
                if (nst > 0) {
                    if (row == 0) {
                        o_store_read_done();
                        mbar_arrive(bar(B_OREAD + w));
                    }
                    if (!(ok = __all_sync(D1_FULL_MASK, mbar_wait(bar(B_OREAD + w), (nst - 1) & 1, abort_flag))))
                        break;
                }
#pragma unroll
                for (int ch = 0; ch < 8; ch++)
                    *reinterpret_cast<uint4*>(stile + row * 128 + ((ch ^ (row & 7)) << 4)) = make_uint4(
                        pack_h2(__uint_as_float(o[8 * ch]) * il, __uint_as_float(o[8 * ch + 1]) * il),
                        pack_h2(__uint_as_float(o[8 * ch + 2]) * il, __uint_as_float(o[8 * ch + 3]) * il),
                        pack_h2(__uint_as_float(o[8 * ch + 4]) * il, __uint_as_float(o[8 * ch + 5]) * il),
                        pack_h2(__uint_as_float(o[8 * ch + 6]) * il, __uint_as_float(o[8 * ch + 7]) * il));
                fence_async_smem_cta();
                __syncwarp();
                if (lane == 0) mbar_arrive(bar(B_OSTAGED + w));
                bool staged_ok = true;
                if (row == 0) {
                    staged_ok = mbar_wait(bar(B_OSTAGED + w), nst & 1, abort_flag);
                    if (staged_ok) o_tile_store(&tmO, smem_u32(stile), un.h * 64, un.s.q_start + q0w);
                }
                nst++;
                if (!(ok = __all_sync(D1_FULL_MASK, staged_ok))) break;
            } else if (q < un.s.q_len) {  // a partial tile: this row's 128 bytes directly
                __half* orow = a.O + (size_t)(un.s.q_start + q) * a.ldo + un.h * 64;
#pragma unroll
                for (int k8 = 0; k8 < 8; k8++)
                    *reinterpret_cast<uint4*>(orow + k8 * 8) = make_uint4(
                        pack_h2(__uint_as_float(o[8 * k8]) * il, __uint_as_float(o[8 * k8 + 1]) * il),
                        pack_h2(__uint_as_float(o[8 * k8 + 2]) * il, __uint_as_float(o[8 * k8 + 3]) * il),
                        pack_h2(__uint_as_float(o[8 * k8 + 4]) * il, __uint_as_float(o[8 * k8 + 5]) * il),
                        pack_h2(__uint_as_float(o[8 * k8 + 6]) * il, __uint_as_float(o[8 * k8 + 7]) * il));
            }
        }
        if (row == 0) o_store_done();  // no O store still reads this CTA's shared memory when it exits
        if (!ok && lane == 0) record_err(a.err, abort_flag, kErrWaitAccFull);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, T_TMEM_COLS);
    }
}

// A 2-D fp16 tensor map over rows x cols (row pitch ld elements) with 64-column x box_rows boxes in the 128-byte
// swizzle; rows past `rows` read as zeros.
bool attn_tmap(CUtensorMap* m, const void* base, int cols, int rows, int ld, uint32_t box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_fa_tc(FaTcArgs& a, int n_work, int heads, int q_rows, int kv_rows, int o_rows, cudaStream_t st) {
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
    CUtensorMap tq, tk, tv, to;
    const int kv_cols = heads / a.group * 64;
    if (!attn_tmap(&tq, a.Q, heads * 64, q_rows, a.ldq, TQ) || !attn_tmap(&tk, a.K, kv_cols, kv_rows, a.ldkv, TKV) ||
        !attn_tmap(&tv, a.V, kv_cols, kv_rows, a.ldkv, TKV) || !attn_tmap(&to, a.O, heads * 64, o_rows, a.ldo, TQ))
        return -1;
    const int grid = a.n_units < sms[dev & 63] ? a.n_units : sms[dev & 63];
    launch_pdl(k_flash_attn_tc, grid, T_THREADS, T_SMEM, st, tq, tk, tv, to, a);
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
    launch_pdl(k_flash_attn<HPC, BIAS>, grid, 128 * HPC, smem, st, a);
    return (int)cudaGetLastError();
}


// ---------------------------------------------------------------------------------------------- reference ABI
// d1_flash_attn takes any list of 64-row work items and no buffer bounds. Its bias-free calls run on the tcgen05
// kernel as far as the list allows: a one-CTA pass splits the list into the 256-row blocks whose tiles (those
// inside the sequence) are listed consecutively from a multiple of 256 (the reference's own lists,
// src/model.rs:328-339, consist of such blocks only) and every other item, which the mma.sync kernel computes
// after it. Each row is computed as often as the list names it, as before. The caller gives no buffer sizes, and
// the tcgen05 kernel needs none: its TMA loads and stores move only whole tiles inside a sequence (partial Q and K/V
// tiles are copied row by row with zero fill, partial O tiles stored row by row), so its tensor maps carry a
// nominal row count (kAbiRows) that no access reaches.
constexpr int kAbiMaxItems = 1 << 16;
constexpr int kAbiRows = 1 << 30;
constexpr int kAbiMaxGy = 128;  // leftover pool counters, one per grid row of the mma.sync kernel

// Is work[j] part of a 256-row block the list names whole (its tiles inside the sequence listed consecutively from a
// multiple of 256)? head: work[j] is the block's first tile.
__device__ __forceinline__ bool whole_block(const int2* __restrict__ work, int n_work, const AttnSeq* __restrict__ seqs,
                                            int j, int2 it, bool& head) {
    const int q_len = seqs[it.x].q_len;
    const int r = (it.y & (TQU - 1)) / 64;  // the item's tile within its 256-row block
    const int base = it.y - 64 * r;
    head = r == 0;
    if (it.y < 0 || it.y % 64 != 0 || it.y >= q_len || j < r) return false;
    const int n = min(TQU / 64, (q_len - base + 63) / 64);  // the block's tiles inside the sequence
    if (j - r + n > n_work) return false;
    for (int k = 0; k < n; k++) {
        const int2 o = work[j - r + k];
        if (o.x != it.x || o.y != base + 64 * k) return false;
    }
    return true;
}

constexpr int kSplitBins = 1024;  // block cost classes: key tiles of 128 (ext + local keys), capped

// The split, one CTA. Whole blocks are written longest sequence first (a counting sort on their key tiles), so the
// tcgen05 kernel's round-robin assignment of units to CTAs starts the long ones in its first wave; leftovers in any
// order (the mma.sync kernel takes them from a pool).
__global__ void __launch_bounds__(1024) k_split_work(const int2* __restrict__ work, int n_work,
                                                     const AttnSeq* __restrict__ seqs, int2* blocks, int2* left,
                                                     int* counts) {
    __shared__ int start[kSplitBins];  // blocks per cost class, then each class's next output slot
    __shared__ int warp_sum[32];
    __shared__ int nl;
    pdl_entry();
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    start[tid] = 0;
    if (tid == 0) nl = 0;
    if (tid < kAbiMaxGy) counts[4 + tid] = 0;  // the leftover pools' next items
    __syncthreads();
    auto cost = [&](int2 it) {
        const AttnSeq& q = seqs[it.x];
        return min((q.ext_len + q.kv_len + TKV - 1) / TKV, kSplitBins - 1);
    };
    for (int j = tid; j < n_work; j += blockDim.x) {
        const int2 it = work[j];
        bool head;
        if (!whole_block(work, n_work, seqs, j, it, head))
            left[atomicAdd(&nl, 1)] = it;
        else if (head)
            atomicAdd(&start[cost(it)], 1);
    }
    __syncthreads();
    // exclusive scan from the costliest class down: thread t holds class kSplitBins - 1 - t
    const int c = start[kSplitBins - 1 - tid];
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(D1_FULL_MASK, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) warp_sum[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        int w = warp_sum[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(D1_FULL_MASK, w, o);
            if (lane >= o) w += v;
        }
        warp_sum[lane] = w - warp_sum[lane];  // exclusive over warps
    }
    __syncthreads();
    start[kSplitBins - 1 - tid] = warp_sum[wid] + incl - c;
    if (tid == blockDim.x - 1) counts[0] = warp_sum[wid] + incl;  // whole blocks in all
    __syncthreads();
    for (int j = tid; j < n_work; j += blockDim.x) {
        const int2 it = work[j];
        bool head;
        if (whole_block(work, n_work, seqs, j, it, head) && head)
            blocks[atomicAdd(&start[cost(it)], 1)] = make_int2(it.x, it.y);
    }
    __syncthreads();
    if (tid == 0) counts[1] = nl;
}

// Device lists of the split and the leftover pools' counters, one set per (device, stream) so that calls on
// different streams do not share them; 1 MB each, allocated on a stream's first call (not while it is being
// captured) and kept until exit.
struct AbiScratch {
    int2* blocks;
    int2* left;
    int* counts;
};
std::mutex g_abi_mu;
std::map<std::pair<int, cudaStream_t>, AbiScratch> g_abi_scratch;

AbiScratch* abi_scratch(int dev, cudaStream_t st) {
    std::lock_guard<std::mutex> lock(g_abi_mu);
    auto it = g_abi_scratch.find({dev, st});
    if (it != g_abi_scratch.end()) return &it->second;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return nullptr;
    }
    void* mem = nullptr;
    if (cudaMalloc(&mem, (size_t)2 * kAbiMaxItems * sizeof(int2) + (4 + kAbiMaxGy) * sizeof(int)) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    AbiScratch s;
    s.blocks = static_cast<int2*>(mem);
    s.left = s.blocks + kAbiMaxItems;
    s.counts = reinterpret_cast<int*>(s.left + kAbiMaxItems);
    return &(g_abi_scratch[{dev, st}] = s);
}

int* fa_err_addr() {
    static int* addr[64] = {};  // device address of g_fa_err, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!addr[dev & 63] && cudaGetSymbolAddress(reinterpret_cast<void**>(&addr[dev & 63]), g_fa_err) != cudaSuccess)
        return nullptr;
    return addr[dev & 63];
}

// The bias-free d1_flash_attn call on the tcgen05 kernel plus the mma.sync kernel for the rest of the list:
// 0 when launched, 1 when this path cannot take the call (the caller runs the mma.sync kernel alone), or a launch
// error.
int abi_flash_attn_tc(const FaArgs& fa, int n_work, int heads, cudaStream_t st) {
    if (n_work > kAbiMaxItems || heads > kAbiMaxGy || fa.ldq < heads * 64 || fa.ldo < heads * 64 ||
        fa.ldkv < heads / fa.group * 64)
        return 1;
    int dev = 0, major = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major != 10) return 1;
    int* err = fa_err_addr();
    AbiScratch* sc = abi_scratch(dev, st);
    if (!err || !sc) return 1;
    launch_pdl(k_split_work, 1, 1024, 0, st, fa.work, n_work, fa.seqs, sc->blocks, sc->left, sc->counts);
    if (cudaError_t e = cudaGetLastError()) return (int)e;
    FaTcArgs t;
    t.Q = fa.Q;
    t.K = fa.K;
    t.V = fa.V;
    t.O = fa.O;
    t.seqs = fa.seqs;
    t.work = sc->blocks;
    t.n_blocks = sc->counts;
    t.ldq = fa.ldq;
    t.ldkv = fa.ldkv;
    t.ext_ld = fa.ext_ld;
    t.ldo = fa.ldo;
    t.group = fa.group;
    t.scale_log2 = fa.scale_log2;
    t.err = err;
    if (int r = launch_fa_tc(t, n_work, heads, kAbiRows, kAbiRows, kAbiRows, st)) return r;
    // the leftover items (none for the reference's own lists) on one resident wave of CTAs taking them in turn
    FaArgs rest = fa;
    rest.work = sc->left;
    rest.n_items = sc->counts + 1;
    rest.next_item = sc->counts + 4;
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int gy = fa.group == 2 ? heads / 2 : heads;
    int gx = 2 * sms / gy;
    gx = gx < 1 ? 1 : gx > n_work ? n_work : gx;
    return fa.group == 2 ? launch_fa<2, false>(rest, gx, gy, st) : launch_fa<1, false>(rest, gx, gy, st);
}

}  // namespace

extern "C" int d1_flash_attn_tc(const d1_half* Q, int ldq, const d1_half* K, const d1_half* V, int ldkv, int ext_ld,
                                d1_half* O, int ldo, const AttnSeq* seqs, const int* work, int n_work, int heads,
                                int group, float scale, int q_rows, int kv_rows, cudaStream_t st) {
    if (n_work <= 0) return n_work == 0 ? 0 : -1;
    if (heads <= 0 || group <= 0 || heads % group || q_rows <= 0 || kv_rows <= 0) return -1;
    if (ldq < heads * 64 || ldo < heads * 64 || ldkv < heads / group * 64) return -1;
    if ((((uintptr_t)Q | (uintptr_t)K | (uintptr_t)V | (uintptr_t)O) & 15) || (ldq | ldkv | ldo | ext_ld) % 8) return -1;
    FaTcArgs t;
    t.Q = Q;
    t.K = K;
    t.V = V;
    t.O = O;
    t.seqs = seqs;
    t.work = reinterpret_cast<const int2*>(work);
    t.n_blocks = nullptr;
    t.ldq = ldq;
    t.ldkv = ldkv;
    t.ext_ld = ext_ld;
    t.ldo = ldo;
    t.group = group;
    t.scale_log2 = scale * 1.4426950408889634f;
    t.err = fa_err_addr();
    if (!t.err) return -1;
    return launch_fa_tc(t, n_work, heads, q_rows, kv_rows, q_rows, st);
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
    a.n_items = nullptr;
    a.next_item = nullptr;
    a.ldq = ldq;
    a.ldkv = ldkv;
    a.ext_ld = ext_ld;
    a.ldo = ldo;
    a.group = group;
    a.scale_log2 = scale * 1.4426950408889634f;
    const bool bias = bq || bk || bv;
    if (!bias) {  // the tcgen05 kernel for the list's whole 256-row blocks, the mma.sync kernel for the rest
        const int r = abi_flash_attn_tc(a, n_work, heads, st);
        if (r != 1) return r;
    }
    if (group == 2) {
        const int gy = heads / 2;
        return bias ? launch_fa<2, true>(a, n_work, gy, st) : launch_fa<2, false>(a, n_work, gy, st);
    }
    return bias ? launch_fa<1, true>(a, n_work, heads, st) : launch_fa<1, false>(a, n_work, heads, st);
}
