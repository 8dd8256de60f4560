// prefill_kernels.cuh — the batched prefill (ref src/model.c:283-360): every
// layer runs once over all n prompt tokens, each weight row streamed once per
// token tile instead of once per token.
//
// The arithmetic per token is the single-token step's, so the cache and the
// last token's logits equal n sequential ember_forward calls bit for bit:
//
//   GEMM      ember_matmul_batch (ref src/kernels.c:227-264): per output
//             (row r, token t) the int32 dot of each 32-element block, exact,
//             then sum = 0; sum += ((float)acc_b * d_w[r][b]) * d_x[t][b] for
//             b = 0, 1, ... in order. The int32 block dots come from the 5th
//             generation tensor cores (tcgen05.mma kind::i8, one MMA of K = 32
//             per quant block into its own TMEM accumulator); the epilogue
//             warps read each block's int32 tile from TMEM and run the fp32
//             chain in registers, two columns per packed f32x2 instruction.
//   norms     RMSNorm sum of squares as one sequential chain per token.
//   attention per (kv head, token tile): scores in index order, softmax with
//             the sequential denominator, outputs as sequential chains over
//             positions — one chain per (query row, dimension).
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "attn_decode.cuh"

namespace emb {

// ------------------------------------------------------------ tcgen05 / TMA ----

EMB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
EMB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// whole warp: allocate `ncols` TMEM columns (power of two >= 32), address -> *slot
EMB_DEV void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
EMB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}


EMB_DEV unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait of the GEMM's roles: gives up after PF_WAIT_NS (recording
// ERR_PF_WAIT) or as soon as another role of the CTA has given up (*abort), so
// a lost copy or MMA ends the whole CTA within about a second.
constexpr unsigned long long PF_WAIT_NS = 1000000000ull;

// drain wait: copies or MMAs already in flight must land before the CTA exits,
// whatever other roles did; bounded by the same time limit
EMB_DEV bool mbar_wait_ns(uint64_t *bar, uint32_t parity, int *err) {
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > PF_WAIT_NS) {
            if (err) atomicExch(err, ERR_PF_WAIT);
            return false;
        }
    }
    return true;
}
EMB_DEV bool pf_wait(uint64_t *bar, uint32_t parity, int *err, volatile int *abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (global_ns() - t0 > PF_WAIT_NS) {
            *abort = 1;
            if (err) atomicExch(err, ERR_PF_WAIT);
            return false;
        }
    }
    return true;
}

// 2-D tiled TMA load into this CTA only: box at (x = inner element, y = row)
EMB_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// Shared-memory matrix descriptor of a K-major operand written by a TMA load
// with 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
// The K offset inside the 128-byte row is added to the start address.
EMB_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);      // start address, 16-byte units
    d |= (uint64_t)1 << 16;                        // leading byte offset (unused when swizzled)
    d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                        // 128-byte swizzle
    return d;
}

// D[tmem] = A * B^T for one K = 32 step of int8 operands (no accumulation)
EMB_DEV void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(0u)
        : "memory");
}

// arrive on `bar` when every tcgen05.mma this thread issued so far has completed
EMB_DEV void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 16 consecutive 32-bit TMEM columns of this thread's lane at two addresses
// (r[0..15] from ta, r[16..31] from tb); the wait is in the same statement so
// no use of r[] is scheduled before the data arrives
EMB_DEV void tmem_ld16x2(uint32_t ta, uint32_t tb, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(ta), "r"(tb)
        : "memory");
}

// packed pairs of IEEE fp32 operations, each lane rounded to nearest even
// (the same results as two scalar __fadd_rn / __fmul_rn). Unlike the scalar
// .rn forms, ptxas may contract a mul.rn.f32x2 whose result feeds an add into a
// fused multiply-add, so a packed multiply must never feed an addition.
EMB_DEV float2 add_f32x2(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
EMB_DEV float2 sub_f32x2(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
EMB_DEV float2 mul_f32x2(float2 a, float2 b) {
    float2 r;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}

// ------------------------------------------------------------------- GEMM ------

// profiling build only (-DEMBER_PROBES): CTA (0,0) of the last GEMM launch
// records when the producer issued each stage, the MMA warp each block, and
// epilogue warp 0 the phases of each block pair. Timestamps only.
#ifdef EMBER_PROBES
__device__ unsigned long long g_pf_trace[1024];
__device__ unsigned long long g_pf_cta[1024][3];   // per CTA: SM id, start, end
EMB_DEV unsigned pf_smid() {
    unsigned r;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
    return r;
}
#define PF_CTA_MARK(k)                                                                   \
    do {                                                                                 \
        const unsigned c_ = blockIdx.y * gridDim.x + blockIdx.x;                         \
        if (threadIdx.x == 0 && c_ < 1024) {                                             \
            if ((k) == 1) g_pf_cta[c_][0] = pf_smid();                                   \
            g_pf_cta[c_][k] = probe_now();                                               \
        }                                                                                \
    } while (0)
#else
#define PF_CTA_MARK(k) do {} while (0)
#endif
#ifdef EMBER_PROBES
#define PF_TRACE(idx)                                                                    \
    do {                                                                                 \
        if (blockIdx.x == 0 && blockIdx.y == 0 && (idx) < 1024) g_pf_trace[idx] = probe_now(); \
    } while (0)
#else
#define PF_TRACE(idx) do {} while (0)
#endif

constexpr int PF_BM = 128;      // weight rows per tile (the MMA's M)
constexpr int PF_SW_BN = 32;    // swapped GEMM: weight rows per tile (the MMA's N)
constexpr int PF_BK = 128;      // K bytes per pipeline stage: four quant blocks
constexpr int PF_STAGES = 4;
// |acc| <= 32*127*127 < 2^22: acc + 1.5*2^23 read as a float is exact, and
// subtracting 1.5*2^23 gives (float)acc exactly
constexpr int PF_MAGIC_I = 0x4B400000;
constexpr float PF_MAGIC_F = 12582912.0f;

enum { PF_EPI_STORE = 0, PF_EPI_RESID = 1 };

struct PfGemmArgs {
    const float *ws;   // weight block scales, fp32 [rows_pad][nbp]
    const float *ws_t; // the same transposed, [nbp][rows_pad] (SWAP)
    int rows_pad;
    const float *xs;   // activation block scales, fp32 [nb][n_pad]
    float *out;        // STORE: out[t*ld + r] = y; RESID: out[t*ld + r] += y
    int *err;
    int rows;          // valid weight rows
    int nb;            // quant blocks per row (K / 32)
    int nbp;           // ws row stride (nb rounded up to 4)
    int n;             // valid tokens
    int n_pad;         // xs row stride (tokens, multiple of 128)
    int ld;            // out row stride
};

template <int BN>
struct PfLayout {
    // columns per epilogue warp: 16 for BN = 32 (eight epilogue warps share the
    // tile's chains), else 32
    static constexpr int CW = BN <= 32 ? 16 : 32;
    static constexpr int EW = 4 * BN / CW;            // epilogue warps: 4 lane quarters x BN/CW column groups
    static constexpr int THREADS = (EW + 2) * 32;     // + TMA producer warp + MMA warp
    static constexpr int A_BYTES = PF_BM * PF_BK;
    static constexpr int B_BYTES = BN * PF_BK;
    static constexpr int XS_BYTES = 4 * BN * 4;
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + PF_STAGES * A_BYTES;
    static constexpr int OFF_XS = OFF_B + PF_STAGES * B_BYTES;
    static constexpr int OFF_BAR = OFF_XS + PF_STAGES * XS_BYTES;
    // CTAs per SM: three for BN = 16 (74 KB of shared memory), two for BN = 32 /
    // 64 (83 / 101 KB), one for BN = 128 (137 KB); the TMEM rings of block-pair
    // accumulators share the SM's 512 columns
    static constexpr int MIN_CTAS = BN == 128 ? 1 : (BN == 16 ? 3 : 2);
    static constexpr int NPAIR = (512 / MIN_CTAS) / (2 * BN) > 4 ? 4 : (512 / MIN_CTAS) / (2 * BN);
    static constexpr int N_BARS = 2 * PF_STAGES + 2 * NPAIR + 1;
    static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;  // + slack to align the base to 1024
    static constexpr uint32_t TMEM_COLS = 2 * NPAIR * BN;
};

// One CTA computes a 128-row x BN-token output tile over all K blocks, the
// blocks taken in pairs (one handshake per pair between the MMA warp and the
// epilogue: each tcgen05 / mbarrier operation costs tens of cycles to issue).
//   warp EW      (lane 0) TMA producer: per stage, a 128 x 128-byte weight box,
//                a BN x 128-byte activation box (both 128-byte swizzled) and the
//                activation scales of the stage's four blocks (bulk copies).
//   warp EW + 1  TMEM allocator; (lane 0) MMA issuer: per block pair, two
//                kind::i8 MMAs (K = 32 each) into the pair's two accumulators,
//                one commit to acc_full[pair slot].
//   warps < EW   epilogue: warp w owns TMEM lanes 32*(w%4).. (tile rows) and
//                columns CW*(w/4).. (tokens); per pair it reads the two blocks'
//                int32 sums 16 columns at a time, frees the pair slot, and adds
//                the terms of block 2p then 2p+1 to each column's chain.
// Every wait is bounded; a wait that gives up records ERR_PF_WAIT and the CTA
// drains its copies and MMAs, frees its TMEM and exits.
//
// SWAP (few token rows): the operands trade places -- A is 128 token rows of
// the activations, B is BN weight rows -- so a matrix of R rows spreads over
// R / BN CTAs instead of R / 128. Accumulator lanes are then tokens and columns
// weight rows: the producer stages the weight scales of the stage's blocks
// (from the transposed copy), each lane reads its token's activation scales,
// and every term is still ((float)acc * d_w) * d_x, added in block order.
template <int BN, int EPI, bool SWAP = false>
__global__ void __launch_bounds__(PfLayout<BN>::THREADS, PfLayout<BN>::MIN_CTAS)
    pf_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const PfGemmArgs a) {
    using Lay = PfLayout<BN>;
    constexpr int NP = Lay::NPAIR;
    extern __shared__ unsigned char pf_smem_raw[];
    __shared__ int abort_flag;
    const uint32_t raw = smem_u32(pf_smem_raw);
    unsigned char *sm = pf_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Lay::OFF_BAR);
    uint64_t *empty = full + PF_STAGES;
    uint64_t *accf = empty + PF_STAGES;
    uint64_t *acce = accf + NP;
    uint64_t *fin = acce + NP;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + Lay::OFF_TMEM);
    volatile int *abort_v = &abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * PF_BM, n0 = blockIdx.y * BN;
    const int nb = a.nb, n_st = (nb + 3) / 4, n_pairs = (nb + 1) / 2;
    PF_CTA_MARK(1);

    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1 + Lay::EW);
        }
        for (int i = 0; i < NP; i++) {
            mbar_init(&accf[i], 1);
            mbar_init(&acce[i], Lay::EW);
        }
        mbar_init(fin, 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == Lay::EW + 1) tmem_alloc(tmem_slot, Lay::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == Lay::EW) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            int issued = 0;
            for (int st = 0; st < n_st; st++) {
                const int slot = st % PF_STAGES;
                if (!pf_wait(&empty[slot], (uint32_t)(((st / PF_STAGES) & 1) ^ 1), a.err, abort_v)) {
                    *abort_v = 1;
                    break;
                }
                const int nblk = min(4, nb - 4 * st);
                if (st < 128) PF_TRACE(st);
                mbar_expect_tx(&full[slot], (uint32_t)(Lay::A_BYTES + Lay::B_BYTES + nblk * BN * 4));
                tma_load_2d(sm + Lay::OFF_A + slot * Lay::A_BYTES, &tmA, st * PF_BK, m0, &full[slot]);
                tma_load_2d(sm + Lay::OFF_B + slot * Lay::B_BYTES, &tmB, st * PF_BK, n0, &full[slot]);
                float *xsd = reinterpret_cast<float *>(sm + Lay::OFF_XS + slot * Lay::XS_BYTES);
                for (int j = 0; j < nblk; j++) {
                    if (SWAP)   // this CTA's BN weight rows' scales of block 4st+j
                        bulk_g2s(xsd + j * BN, a.ws_t + (size_t)(4 * st + j) * a.rows_pad + n0, (uint32_t)(BN * 4),
                                 &full[slot]);
                    else
                        bulk_g2s(xsd + j * BN, a.xs + (size_t)(4 * st + j) * a.n_pad + n0, (uint32_t)(BN * 4),
                                 &full[slot]);
                }
                issued = st + 1;
            }
            // drain: every stage this thread issued has landed before the CTA exits
            for (int st = issued - PF_STAGES < 0 ? 0 : issued - PF_STAGES; st < issued; st++)
                mbar_wait_ns(&full[st % PF_STAGES], (uint32_t)((st / PF_STAGES) & 1), a.err);
        }
    } else if (warp == Lay::EW + 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = (2u << 4)                        // D: s32
                                   | (1u << 7) | (1u << 10)         // A, B: signed int8
                                   | ((uint32_t)(BN >> 3) << 17)    // N
                                   | ((uint32_t)(PF_BM >> 4) << 24);  // M
            for (int p = 0; p < n_pairs; p++) {
                const int st = p >> 1, slot = st % PF_STAGES, ps = p % NP;
                if ((p & 1) == 0 && !pf_wait(&full[slot], (uint32_t)((st / PF_STAGES) & 1), a.err, abort_v)) {
                    *abort_v = 1;
                    break;
                }
                if (!pf_wait(&acce[ps], (uint32_t)(((p / NP) & 1) ^ 1), a.err, abort_v)) {
                    *abort_v = 1;
                    break;
                }
                tc_fence_after();
                if (p < 64) PF_TRACE(128 + p);
                const uint32_t sa = smem_u32(sm + Lay::OFF_A + slot * Lay::A_BYTES) + 64u * (p & 1);
                const uint32_t sb = smem_u32(sm + Lay::OFF_B + slot * Lay::B_BYTES) + 64u * (p & 1);
                mma_i8(tmem + (uint32_t)(2 * ps * BN), umma_desc_sw128(sa), umma_desc_sw128(sb), idesc);
                if (2 * p + 1 < nb)
                    mma_i8(tmem + (uint32_t)((2 * ps + 1) * BN), umma_desc_sw128(sa + 32u), umma_desc_sw128(sb + 32u),
                           idesc);
                mma_commit(&accf[ps]);
                if ((p & 1) == 1 || p == n_pairs - 1) mma_commit(&empty[slot]);
            }
            // every MMA issued above has completed before TMEM is released
            mma_commit(fin);
            mbar_wait_ns(fin, 0, a.err);
        }
    } else {
        // ---------------- epilogue ----------------
        constexpr int CW = Lay::CW, NH = CW / 16;   // columns of this warp, in 16-column halves
        const int quarter = warp & 3, cg = warp >> 2;
        // this lane's accumulator row: a weight row, or (SWAP) a token
        const int row = m0 + 32 * quarter + lane;
        const bool row_ok = SWAP ? row < a.n : row < a.rows;
        const float *wsr = a.ws + (size_t)(SWAP ? 0 : row) * a.nbp;   // rows are padded: always in bounds
        const float *xsl = a.xs + row;                                // SWAP: [block][n_pad], row < n_pad
        float2 s2[CW / 2];
#pragma unroll
        for (int j = 0; j < CW / 2; j++) s2[j] = make_float2(0.0f, 0.0f);
        const float2 magic = make_float2(PF_MAGIC_F, PF_MAGIC_F);
        // this row's weight scales (SWAP: this token's activation scales), four
        // blocks at a time, fetched one stage ahead
        auto lane_scales = [&](int b) {
            if (SWAP) {
                float4 v;
                v.x = xsl[(size_t)(b + 0) * a.n_pad];
                v.y = b + 1 < a.nb ? xsl[(size_t)(b + 1) * a.n_pad] : 0.0f;
                v.z = b + 2 < a.nb ? xsl[(size_t)(b + 2) * a.n_pad] : 0.0f;
                v.w = b + 3 < a.nb ? xsl[(size_t)(b + 3) * a.n_pad] : 0.0f;
                return v;
            }
            return *reinterpret_cast<const float4 *>(wsr + b);
        };
        float4 dw4 = lane_scales(0);
        float4 dw4n = a.nbp > 4 ? lane_scales(4) : dw4;
        const uint32_t tl = tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(cg * CW);
        for (int p = 0; p < n_pairs; p++) {
            const int st = p >> 1, slot = st % PF_STAGES, ps = p % NP;
            const int b = 2 * p, two = b + 1 < nb;
            const int tr = warp == 0 && lane == 0 && p < 160 ? 384 + 4 * p : 1024;
            PF_TRACE(tr);
            // lane 0 waits, the warp follows it (tcgen05.ld needs the whole warp)
            int ok = 1;
            if ((p & 1) == 0) {
                if (p > 0) {
                    dw4 = dw4n;
                    if (b + 4 < a.nbp) dw4n = lane_scales(b + 4);
                }
                // the stage's scale copies: observed by this warp too
                if (lane == 0) ok = pf_wait(&full[slot], (uint32_t)((st / PF_STAGES) & 1), a.err, abort_v);
            }
            if (lane == 0 && ok) ok = pf_wait(&accf[ps], (uint32_t)((p / NP) & 1), a.err, abort_v);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            PF_TRACE(tr + 1);
            tc_fence_after();
            const float dwa = (p & 1) ? dw4.z : dw4.x, dwb = (p & 1) ? dw4.w : dw4.y;
            const float4 *xsa = reinterpret_cast<const float4 *>(sm + Lay::OFF_XS + slot * Lay::XS_BYTES) +
                                ((b & 3) * BN + cg * CW) / 4;
            const float4 *xsb = xsa + BN / 4;
#pragma unroll
            for (int h = 0; h < NH; h++) {
                uint32_t r[32];
                tmem_ld16x2(tl + (uint32_t)(2 * ps * BN + 16 * h), tl + (uint32_t)((2 * ps + 1) * BN + 16 * h), r);
                if (h == NH - 1) {
                    // both halves read: the pair slot is free for the MMA warp
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&acce[ps]);
                }
#pragma unroll
                for (int blk = 0; blk < 2; blk++) {
                    if (blk == 1 && !two) break;
                    const float2 dw2 = blk ? make_float2(dwb, dwb) : make_float2(dwa, dwa);
                    const float4 *xsv = (blk ? xsb : xsa) + 4 * h;
#pragma unroll
                    for (int q4 = 0; q4 < 4; q4++) {
                        const float4 xv = xsv[q4];
                        const uint32_t *rr = r + 16 * blk + 4 * q4;
                        float2 f0 = make_float2(__int_as_float((int)rr[0] + PF_MAGIC_I), __int_as_float((int)rr[1] + PF_MAGIC_I));
                        float2 f1 = make_float2(__int_as_float((int)rr[2] + PF_MAGIC_I), __int_as_float((int)rr[3] + PF_MAGIC_I));
                        if (SWAP) {
                            // columns are weight rows: d_w from the staged scales,
                            // then this lane's token scale
                            f0 = mul_f32x2(sub_f32x2(f0, magic), make_float2(xv.x, xv.y));
                            f1 = mul_f32x2(sub_f32x2(f1, magic), make_float2(xv.z, xv.w));
                            f0 = make_float2(fmul(f0.x, dw2.x), fmul(f0.y, dw2.x));
                            f1 = make_float2(fmul(f1.x, dw2.x), fmul(f1.y, dw2.x));
                        } else {
                            f0 = mul_f32x2(sub_f32x2(f0, magic), dw2);
                            f1 = mul_f32x2(sub_f32x2(f1, magic), dw2);
                            // the multiply whose result is added is scalar: ptxas may contract a
                            // packed mul.f32x2 feeding an add into an fma, a scalar mul.rn never
                            f0 = make_float2(fmul(f0.x, xv.x), fmul(f0.y, xv.y));
                            f1 = make_float2(fmul(f1.x, xv.z), fmul(f1.y, xv.w));
                        }
                        s2[8 * h + 2 * q4] = add_f32x2(s2[8 * h + 2 * q4], f0);
                        s2[8 * h + 2 * q4 + 1] = add_f32x2(s2[8 * h + 2 * q4 + 1], f1);
                    }
                }
            }
            PF_TRACE(tr + 3);
            if ((p & 1) == 1 || p == n_pairs - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
        }
        if (row_ok && !*abort_v) {
#pragma unroll
            for (int j = 0; j < CW; j++) {
                const int c = n0 + cg * CW + j;   // the column: a token, or (SWAP) a weight row
                const float v = (j & 1) ? s2[j >> 1].y : s2[j >> 1].x;
                if (SWAP ? c < a.rows : c < a.n) {
                    float *o = SWAP ? a.out + (size_t)row * a.ld + c : a.out + (size_t)c * a.ld + row;
                    *o = EPI == PF_EPI_RESID ? fadd(*o, v) : v;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == Lay::EW + 1) {
        tc_fence_after();
        tmem_dealloc(tmem, Lay::TMEM_COLS);
    }
    PF_CTA_MARK(2);
}

// --------------------------------------------------- few tokens: dp4a GEMV -------
// A multi-token GEMV for batches of at most a few dozen tokens (batched decode
// of streams, short prefills), where the tensor-core tiles leave a CTA walking
// a long serial chain of block MMAs. One CTA per (16 weight rows, 16 tokens):
// bulk copies bring the rows (int8, the pack's layout), their fp32 scales and
// the tokens' int8 activations (rows padded by 16 bytes, so the eight threads
// of a shared-memory phase read eight bank groups); thread (row, token) runs
// that output's chain: per block the int32 dot (exact), the term
// ((float)acc * d_w) * d_x, added in block order (ref src/kernels.c:152-164).
constexpr int MTV_R = 16, MTV_T = 16;

struct PfMtvArgs {
    const int8_t *wq;    // pack rows [rows_pad][k_pad]
    const float *ws;     // pack scales [rows_pad][nbp]
    const int8_t *xq;    // activations [n_pad][k_pad]
    const float *xs;     // activation scales [nb][n_pad]
    float *out;          // STORE: out[t*ld + r] = y; RESID: += y
    int *err;
    int rows, nb, nbp, k_pad, n, n_pad, ld;
};

__host__ __device__ inline size_t mtv_smem_bytes(int k_pad, int nbp) {
    return (size_t)MTV_R * k_pad + (size_t)MTV_T * (k_pad + 16) + (size_t)MTV_R * nbp * 4 + (size_t)nbp * MTV_T * 4;
}

template <int EPI>
__global__ void __launch_bounds__(MTV_R * MTV_T) pf_mtv_kernel(const PfMtvArgs a) {
    extern __shared__ __align__(128) unsigned char mtv_sm[];
    __shared__ __align__(8) uint64_t bar;
    const int tid = threadIdx.x, r0 = blockIdx.x * MTV_R, t0 = blockIdx.y * MTV_T;
    const int nt = min(MTV_T, a.n - t0), kp = a.k_pad, xstride = kp + 16;
    int8_t *wq_s = reinterpret_cast<int8_t *>(mtv_sm);                    // [MTV_R][kp]
    int8_t *xq_s = wq_s + (size_t)MTV_R * kp;                              // [MTV_T][kp + 16]
    float *ws_s = reinterpret_cast<float *>(xq_s + (size_t)MTV_T * xstride);   // [MTV_R][nbp]
    float *xs_s = ws_s + (size_t)MTV_R * a.nbp;                           // [nbp][MTV_T]
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
        mbar_expect_tx(&bar, (uint32_t)(MTV_R * kp + MTV_R * a.nbp * 4 + nt * kp));
        bulk_g2s(wq_s, a.wq + (size_t)r0 * kp, (uint32_t)(MTV_R * kp), &bar);
        bulk_g2s(ws_s, a.ws + (size_t)r0 * a.nbp, (uint32_t)(MTV_R * a.nbp * 4), &bar);
        for (int t = 0; t < nt; t++)
            bulk_g2s(xq_s + (size_t)t * xstride, a.xq + (size_t)(t0 + t) * kp, (uint32_t)kp, &bar);
    }
    // the activation scales of these tokens (n_pad >= t0 + MTV_T: in bounds)
    for (int idx = tid; idx < a.nb * MTV_T; idx += MTV_R * MTV_T) {
        const int b = idx / MTV_T, t = idx - b * MTV_T;
        xs_s[idx] = a.xs[(size_t)b * a.n_pad + t0 + t];
    }
    __syncthreads();
    mbar_wait_cta(&bar, 0, a.err, ERR_PF_WAIT);
    const int r = tid / MTV_T, t = tid - r * MTV_T, row = r0 + r;
    if (t < nt && row < a.rows) {
        const int8_t *wr = wq_s + (size_t)r * kp, *xr = xq_s + (size_t)t * xstride;
        const float *wsr = ws_s + (size_t)r * a.nbp, *xsr = xs_s + t;
        float s = 0.0f;
#pragma unroll 4
        for (int b = 0; b < a.nb; b++) {
            const int4 *wv = reinterpret_cast<const int4 *>(wr + b * 32);
            const int4 *xv = reinterpret_cast<const int4 *>(xr + b * 32);
            const int acc = dp8(wv[0], wv[1], xv[0], xv[1]);
            s = fadd(s, fmul(fmul(__int2float_rn(acc), wsr[b]), xsr[b * MTV_T]));
        }
        float *o = a.out + (size_t)(t0 + t) * a.ld + row;
        *o = EPI == PF_EPI_RESID ? fadd(*o, s) : s;
    }
}

// --------------------------------------------------------------- packing -------

// dst[b][r] = src[r][b] for a [rows][cols] fp32 matrix (the weight scales'
// transposed copy for the swapped GEMM)
__global__ void __launch_bounds__(256) pf_transpose_kernel(const float *src, float *dst, int rows, int cols) {
    const long long total = (long long)rows * cols;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / rows), r = (int)(i - (long long)b * rows);
        dst[i] = src[(size_t)r * cols + b];
    }
}

// One row group of a prefill weight pack: int8 rows [rows_pad][k_pad] (Q4_0
// nibbles expanded to q - 8, zero padding) and fp32 block scales [rows_pad][nbp].
struct PfPackArgs {
    const uint8_t *q;      // source quant rows (device layout of DevMat)
    const __half *s;       // source scales [rows][nb]
    int dtype, rows, nb;
    int8_t *dq;            // destination rows, starting at this matrix's first row
    float *ds;
    int k_pad, nbp;
};

__global__ void __launch_bounds__(256) pf_pack_kernel(const PfPackArgs a) {
    const long long total = (long long)a.rows * a.nb;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / a.nb), b = (int)(i - (long long)r * a.nb);
        int8_t *dst = a.dq + (size_t)r * a.k_pad + (size_t)b * 32;
        if (a.dtype == EMBER_DT_Q8_0) {
            const uint4 *src = reinterpret_cast<const uint4 *>(a.q + ((size_t)r * a.nb + b) * 32);
            reinterpret_cast<uint4 *>(dst)[0] = src[0];
            reinterpret_cast<uint4 *>(dst)[1] = src[1];
        } else {
            // Q4_0: byte j holds element j (low nibble) and element j+16 (high), value nib - 8
            const uint8_t *src = a.q + ((size_t)r * a.nb + b) * 16;
            for (int j = 0; j < 16; j++) {
                const int v = src[j];
                dst[j] = (int8_t)((v & 15) - 8);
                dst[j + 16] = (int8_t)((v >> 4) - 8);
            }
        }
        a.ds[(size_t)r * a.nbp + b] = __half2float(a.s[(size_t)r * a.nb + b]);
    }
}

// ----------------------------------------------------- per-token elementwise ---

struct PfTokArgs {
    const float *x;        // input rows [n][ld_x] (norm: residual stream; swiglu: [g | u])
    int ld_x;
    const float *norm_w;   // RMSNorm weights (norm kernel)
    float eps;
    int cols;              // K of the next GEMM
    int hidden;            // swiglu: offset of u in a row
    int8_t *xq;            // [n_pad][k_pad] int8
    int k_pad;
    float *xs;             // [nb][n_pad] block scales
    int n_pad;
    ExpfDev ex;
};

// Quantize the smem row v[0..cols) into row t of xq / column t of xs, eight
// threads per 32-block (ref src/kernels.c:73-92).
EMB_DEV void pf_quant_row(const float *v, const PfTokArgs &a, int t) {
    const int nb = a.cols / 32;
    for (int base = 0; base < nb * 8; base += blockDim.x) {
        const int q8 = base + threadIdx.x;
        const bool act = q8 < nb * 8;
        const unsigned mask = __ballot_sync(0xffffffffu, act);
        if (act) {
            const int b = q8 >> 3, sub = q8 & 7;
            float dq;
            const uint32_t packed = quant_quad(reinterpret_cast<const float4 *>(v + b * 32)[sub], mask, &dq);
            reinterpret_cast<uint32_t *>(a.xq + (size_t)t * a.k_pad + b * 32)[sub] = packed;
            if (sub == 0) a.xs[(size_t)b * a.n_pad + t] = dq;
        }
    }
}

// RMSNorm of token t's residual row (ref src/model.c:50-55), then quantize.
// dynamic shared memory: the row, then its squares (2 * cols floats). The sum of
// squares is the sequential loop's, evaluated by split_chain_sum (common.cuh).
__global__ void __launch_bounds__(256) pf_norm_quant_kernel(const PfTokArgs a) {
    extern __shared__ __align__(16) float pf_row[];
    float *sq = pf_row + a.cols;
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) {
        const float v = a.x[(size_t)t * a.ld_x + i];
        pf_row[i] = v;
        sq[i] = fmul(v, v);
    }
    __syncthreads();
    const float sc = rms_scale(split_chain_sum<256>(sq, a.cols), a.cols, a.eps);
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) pf_row[i] = fmul(fmul(pf_row[i], sc), a.norm_w[i]);
    __syncthreads();
    pf_quant_row(pf_row, a, t);
}

// h = g / (1 + expf(-g)) * u (ref src/model.c:403-406), then quantize.
__global__ void __launch_bounds__(256) pf_swiglu_quant_kernel(const PfTokArgs a) {
    extern __shared__ __align__(16) float pf_row[];
    __shared__ double tab_s[64];
    const int t = blockIdx.x;
    expf_table_load(tab_s, a.ex);
    __syncthreads();
    const float *xr = a.x + (size_t)t * a.ld_x;
    // the loads of four elements go out before their arithmetic
    for (int i0 = threadIdx.x; i0 < a.cols; i0 += 4 * blockDim.x) {
        float g[4], u[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int i = i0 + k * blockDim.x;
            g[k] = i < a.cols ? __ldg(xr + i) : 0.0f;
            u[k] = i < a.cols ? __ldg(xr + a.hidden + i) : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int i = i0 + k * blockDim.x;
            if (i < a.cols) pf_row[i] = fmul(fdiv(g[k], fadd(1.0f, expf_exact(a.ex, tab_s, -g[k]))), u[k]);
        }
    }
    __syncthreads();
    pf_quant_row(pf_row, a, t);
}

// The token's embedding row (ref src/model.c:83-100).
struct PfEmbedArgs {
    const uint8_t *q;
    const __half *s;
    int dtype, dim, vocab;
    const int *ids;
    float *x;
    int *err;
};

__global__ void __launch_bounds__(256) pf_embed_kernel(const PfEmbedArgs a) {
    const int t = blockIdx.x;
    const int tok = a.ids[t];
    if (tok < 0 || tok >= a.vocab) {   // the host checked the ids; never read out of bounds
        if (threadIdx.x == 0) atomicExch(a.err, ERR_PF_WAIT);
        return;
    }
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x) {
        if (a.dtype == EMBER_DT_F32) {
            a.x[(size_t)t * a.dim + i] = reinterpret_cast<const float *>(a.q)[(size_t)tok * a.dim + i];
        } else {
            const int8_t q = reinterpret_cast<const int8_t *>(a.q)[(size_t)tok * a.dim + i];
            const float d = __half2float(a.s[(size_t)tok * (a.dim / 32) + i / 32]);
            a.x[(size_t)t * a.dim + i] = fmul((float)q, d);
        }
    }
}

// ---------------------------------------------------- q/k/v post-processing ----

struct PfQkvArgs {
    const float *qkv;      // [n][ld]: q | k | v of each token (GEMM output)
    int ld;
    const float *bq, *bk, *bv;
    const float *q_norm, *k_norm;
    const float2 *rope;    // [ctx][hd/2]
    float *qr;             // [n][qd] roped queries
    void *kc, *vc;         // this layer's cache: keys [n_kv][hd][kstride], values [n_kv][ctx][hd]
    int nh, nkv, hd, ctx, kstride, neox, start;
    int n;                 // tokens
    const int *pos;        // batched decode: token t's position pos[t] (device) and
    size_t cache_stride;   //   its own cache at kc/vc + t * cache_stride elements
    float eps;
};

// One warp per (token, head) for the nh query heads and nkv key heads, eight
// pairs per CTA; the key warps also store the values. Bias (ref :319-321),
// QK-norm (:326-329, the sum of squares in index order on lane 0), RoPE
// (:66-80), KV store (:39-48) -- the single-token step's arithmetic.
constexpr int PF_QKV_WARPS = 8;
template <typename T>
__global__ void __launch_bounds__(32 * PF_QKV_WARPS) pf_qkv_post_kernel(const PfQkvArgs a) {
    __shared__ float vals_s[PF_QKV_WARPS][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, hd = a.hd;
    const int nhh = a.nh + a.nkv;
    const int pair = blockIdx.x * PF_QKV_WARPS + warp;
    if (pair >= a.n * nhh) return;   // whole warps only; no CTA barrier follows
    const int t = pair / nhh, hh = pair - t * nhh;
    float *vals = vals_s[warp];
    const int pos = a.pos ? a.pos[t] : a.start + t;
    const size_t coff = a.pos ? (size_t)t * a.cache_stride : 0;
    const int qd = a.nh * hd, kvd = a.nkv * hd;
    const bool is_q = hh < a.nh;
    const int head = is_q ? hh : hh - a.nh;
    const int off = is_q ? head * hd : qd + head * hd;
    const float *bias = is_q ? a.bq : a.bk;
    const float *nw = is_q ? a.q_norm : a.k_norm;
    const float *row = a.qkv + (size_t)t * a.ld;
    for (int i = lane; i < hd; i += 32) {
        float v = row[off + i];
        if (bias) v = fadd(v, bias[head * hd + i]);
        vals[i] = v;
    }
    __syncwarp();
    if (nw) {
        float sc = 0.0f;
        if (lane == 0) sc = rms_scale(chain_sumsq(vals, hd), hd, a.eps);
        sc = __shfl_sync(0xffffffffu, sc, 0);
        for (int i = lane; i < hd; i += 32) vals[i] = fmul(fmul(vals[i], sc), nw[i]);
        __syncwarp();
    }
    for (int i = lane; i < hd / 2; i += 32) {
        const int ia = a.neox ? i : 2 * i, ib = a.neox ? i + hd / 2 : 2 * i + 1;
        const float2 cs = a.rope[(size_t)pos * (hd / 2) + i];
        const float v0 = vals[ia], v1 = vals[ib];
        vals[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        vals[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
    }
    __syncwarp();
    for (int i = lane; i < hd; i += 32) {
        if (is_q) {
            a.qr[(size_t)t * qd + head * hd + i] = vals[i];
        } else {
            T *kt = reinterpret_cast<T *>(a.kc) + coff + (size_t)head * hd * a.kstride;
            T *vt = reinterpret_cast<T *>(a.vc) + coff + (size_t)head * a.ctx * hd;
            T kq, vq;
            kv_round(vals[i], &kq);
            float v = row[qd + kvd + head * hd + i];
            if (a.bv) v = fadd(v, a.bv[head * hd + i]);
            kv_round(v, &vq);
            kt[(size_t)i * a.kstride + pos] = kq;
            vt[(size_t)pos * hd + i] = vq;
        }
    }
}

// ------------------------------------------------------------------ attention --

constexpr int PF_ATT_THREADS = 256;
constexpr int PF_ATT_MAX_ROWS = 16;

struct PfAttnArgs {
    const float *qr;       // [n][qd] roped queries
    const void *kc, *vc;   // this layer's cache
    int8_t *xq;            // outputs quantized: [n_pad][k_pad] ...
    int k_pad;
    float *xs;             //   ... scales [qd/32][n_pad]
    int n_pad;
    int nh, nkv, hd, ctx, kstride, start, n;
    int tq;                // tokens per CTA; rows = tq * (nh / nkv) <= PF_ATT_MAX_ROWS
    int rs;                // weight row stride: rows rounded up to 4
    const int *pos;        // batched decode (tq = 1): token t's position pos[t] and its
    size_t cache_stride;   //   own cache at kc/vc + t * cache_stride elements
    int p_cap;             // positions held in shared memory (>= start + n)
    ExpfDev ex;
};

// positions per staged chunk of keys or values
constexpr int PF_ATT_CH = 64;

// shared memory of one attention CTA: the queries [hd][16] (RS <= 16 rows), the
// weights [p_cap][rs], then two chunk buffers of PF_ATT_CH positions x hd cache
// elements (keys or values)
__host__ __device__ inline size_t pf_attn_w_bytes(int p_cap, int rs) {
    return ((size_t)p_cap * rs * 4 + 15) / 16 * 16;
}
__host__ __device__ inline size_t pf_attn_smem(int p_cap, int rs, int hd, int es) {
    return (size_t)hd * PF_ATT_MAX_ROWS * 4 + pf_attn_w_bytes(p_cap, rs) + 2 * (size_t)PF_ATT_CH * hd * es;
}

// keys of positions [c0, c0+n) -> buf[hd][PF_ATT_CH] (the cache keeps keys
// transposed, [hd][kstride]); values -> buf[PF_ATT_CH][hd]. 16-byte cp.async by
// every thread, committed as one group. Rows are padded to kstride (a multiple
// of 8 positions) and c0 is a multiple of 8, so whole vectors stay in bounds.
template <typename T>
EMB_DEV void pf_stage_k(T *buf, const T *kt, int kstride, int c0, int n, int hd) {
    constexpr int E = 16 / (int)sizeof(T);
    const int nv = (n + E - 1) / E, total = hd * nv;
    for (int idx = threadIdx.x; idx < total; idx += PF_ATT_THREADS) {
        const int i = idx / nv, v = idx - i * nv;
        cp_async16(buf + (size_t)i * PF_ATT_CH + v * E, kt + (size_t)i * kstride + c0 + v * E);
    }
    cp_async_commit();
}
template <typename T>
EMB_DEV void pf_stage_v(T *buf, const T *vt, int c0, int n, int hd) {
    constexpr int E = 16 / (int)sizeof(T);
    const int total = n * hd / E;
    for (int idx = threadIdx.x; idx < total; idx += PF_ATT_THREADS)
        cp_async16(buf + (size_t)idx * E, vt + (size_t)c0 * hd + (size_t)idx * E);
    cp_async_commit();
}

// One CTA per (kv head, tile of tq consecutive tokens); its query rows are the
// tile's tokens x the kv head's query heads (row r = token r / kv_mul, head
// kvh * kv_mul + r % kv_mul). Token j attends to positions 0..start+b0+j. For
// every row, as in the single-token step (ref src/model.c:221-259):
//   scores   sc_t = sum_i q_i*k_t,i in index order, * (1/sqrt(hd)) -- per
//            chunk of 64 cached positions staged in shared memory, one thread
//            per (position, four rows): each key element loaded once serves
//            four rows' chains, each query quad is a broadcast;
//   softmax  max, e_t = expf(sc_t - max), den = sequential sum over t,
//            w_t = e_t * (1/den);
//   output   o_i = sum_t w_t*v_t,i in position order -- one thread per
//            (dimension, row group) over staged value chunks, then quantized
//            per (token, head).
// Chunks are double-buffered: the copies of chunk c+1 run while chunk c is
// used. Products are rounded by scalar multiplies and added in pairs
// (add.f32x2): the same two roundings per step as the reference.
// RS: the register rows (4, 8 or 16, >= rs): a prefill tile takes 16 rows, a
// batched decode row (one token of one stream) only its kv head's query heads.
// RG: the rows of one output thread's chains (pf_attn_rows_per_group), fixed at
// compile time so the unrolled output loop issues no dead rows.
__host__ __device__ inline int pf_attn_groups(int hd) { return hd >= PF_ATT_THREADS ? 1 : PF_ATT_THREADS / hd; }
__host__ inline int pf_attn_rows_per_group(int rs, int hd) {
    const int g = pf_attn_groups(hd), need = (rs + g - 1) / g;
    return need <= 4 ? 4 : (need <= 8 ? 8 : 16);
}
template <typename T, int RS, int RG>
__global__ void __launch_bounds__(PF_ATT_THREADS) pf_attn_kernel(const PfAttnArgs a) {
    static_assert(RS == 4 || RS == 8 || RS == 16, "pf_attn_kernel: RS is 4, 8 or 16");
    static_assert(RG == 4 || RG == 8 || RG == 16, "pf_attn_kernel: RG is 4, 8 or 16");
    extern __shared__ __align__(16) float pf_dyn[];              // q_s [hd][RS], weights, chunk buffers
    float *q_s = pf_dyn;                                          // [hd][RS]
    float *pf_att = pf_dyn + (size_t)a.hd * PF_ATT_MAX_ROWS;      // [p_cap][rs]
    __shared__ float red[RS][PF_ATT_THREADS / 32];
    __shared__ float s_max[RS], s_inv[RS];
    __shared__ double tab_s[64];
    const int rs = a.rs;                  // weight stride in shared memory (<= RS)
    // the heaviest tiles (the prompt's end, the longest causal rows) start first
    const int kvh = blockIdx.x, b0 = (gridDim.y - 1 - blockIdx.y) * a.tq, tid = threadIdx.x, hd = a.hd;
    const int kv_mul = a.nh / a.nkv;
    const int ntok = min(a.tq, a.n - b0);
    const int rows = ntok * kv_mul;
    const int qd = a.nh * hd;
    // position of the tile's first token (rows of token j sit at pos0 + j)
    const int pos0 = a.pos ? a.pos[b0] : a.start + b0;
    const size_t coff = a.pos ? (size_t)b0 * a.cache_stride : 0;
    const int p_first = pos0;                        // every row sees positions 0..p_first
    const int p_last = pos0 + ntok - 1;              // the tile's last position
    const T *kt = reinterpret_cast<const T *>(a.kc) + coff + (size_t)kvh * hd * a.kstride;
    const T *vt = reinterpret_cast<const T *>(a.vc) + coff + (size_t)kvh * a.ctx * hd;
    // the two chunk buffers: kvb0 + (c & 1) * cbuf
    T *kvb0 = reinterpret_cast<T *>(reinterpret_cast<unsigned char *>(pf_att) + pf_attn_w_bytes(a.p_cap, rs));
    const size_t cbuf = (size_t)PF_ATT_CH * hd;
    const int npos = p_last + 1, nch = (npos + PF_ATT_CH - 1) / PF_ATT_CH;
    pf_stage_k(kvb0, kt, a.kstride, 0, min(PF_ATT_CH, npos), hd);
    expf_table_load(tab_s, a.ex);
    for (int idx = tid; idx < RS * hd; idx += PF_ATT_THREADS) {
        const int r = idx / hd, i = idx - r * hd;
        const int j = r / kv_mul, hm = r - j * kv_mul;
        q_s[i * RS + r] = r < rows ? a.qr[(size_t)(b0 + j) * qd + (kvh * kv_mul + hm) * hd + i] : 0.0f;
    }

    // ---- scores: thread = (position in the chunk, row quad) ----
    constexpr int QUADS = RS / 4, PP = PF_ATT_THREADS / QUADS;   // positions a pass covers
    const int tl = tid % PP, rq = tid / PP;
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    for (int c = 0; c < nch; c++) {
        const int c0 = c * PF_ATT_CH, n = min(PF_ATT_CH, npos - c0);
        if (c + 1 < nch) {
            pf_stage_k(kvb0 + ((c + 1) & 1) * cbuf, kt, a.kstride, c0 + PF_ATT_CH,
                       min(PF_ATT_CH, npos - c0 - PF_ATT_CH), hd);
            cp_async_wait_1();
        } else {
            cp_async_wait_all();
        }
        __syncthreads();
        const T *kb = kvb0 + (c & 1) * cbuf;
        if (tl < n) {
            float2 s0 = make_float2(0.0f, 0.0f), s1 = s0;
            const float4 *qv = reinterpret_cast<const float4 *>(q_s) + rq;
            for (int i = 0; i < hd; i += 8) {
                float kk[8];
#pragma unroll
                for (int j = 0; j < 8; j++) kk[j] = widen(kb[(size_t)(i + j) * PF_ATT_CH + tl]);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    const float4 q4 = qv[(i + j) * QUADS];
                    s0 = add_f32x2(s0, make_float2(fmul(q4.x, kk[j]), fmul(q4.y, kk[j])));
                    s1 = add_f32x2(s1, make_float2(fmul(q4.z, kk[j]), fmul(q4.w, kk[j])));
                }
            }
            if (4 * rq < rs)
                *reinterpret_cast<float4 *>(pf_att + (size_t)(c0 + tl) * rs + 4 * rq) =
                    make_float4(fmul(s0.x, inv_sqrt), fmul(s0.y, inv_sqrt), fmul(s1.x, inv_sqrt), fmul(s1.y, inv_sqrt));
        }
        __syncthreads();   // the buffer is free for chunk c + 2
    }
    // the first value chunk streams in during the softmax
    pf_stage_v(kvb0, vt, 0, min(PF_ATT_CH, npos), hd);

    // ---- softmax ----
    const int warp = tid >> 5, lane = tid & 31;
    for (int r = 0; r < rows; r++) {
        const int pr = pos0 + r / kv_mul;   // this row's position
        float m = -INFINITY;
        for (int t = tid; t <= pr; t += PF_ATT_THREADS) m = fmaxf(m, pf_att[(size_t)t * rs + r]);
        m = warp_max(m);
        if (lane == 0) red[r][warp] = m;
    }
    __syncthreads();
    if (tid < rows) {
        float m = red[tid][0];
        for (int w = 1; w < PF_ATT_THREADS / 32; w++) m = fmaxf(m, red[tid][w]);
        s_max[tid] = m;
    }
    __syncthreads();
    // every row's last position (rows of token j sit at pos0 + j)
    int rlast[RS];
#pragma unroll
    for (int r = 0; r < RS; r++) rlast[r] = r < rows ? pos0 + r / kv_mul : -1;
    for (int t = tid; t < npos; t += PF_ATT_THREADS) {
        float *w = pf_att + (size_t)t * rs;
#pragma unroll
        for (int r = 0; r < RS; r++)
            if (t <= rlast[r]) w[r] = expf_exact(a.ex, tab_s, fsub(w[r], s_max[r]));
    }
    __syncthreads();
    // denominators: the sequential sum over t, one chain per row (rows in parallel)
    if (tid < rows) {
        const int pr = pos0 + tid / kv_mul;
        float sum = 0.0f;
        int t = 0;
        for (; t + 8 <= pr + 1; t += 8) {
            float e[8];
#pragma unroll
            for (int j = 0; j < 8; j++) e[j] = pf_att[(size_t)(t + j) * rs + tid];
#pragma unroll
            for (int j = 0; j < 8; j++) sum = fadd(sum, e[j]);
        }
        for (; t <= pr; t++) sum = fadd(sum, pf_att[(size_t)t * rs + tid]);
        s_inv[tid] = fdiv(1.0f, sum);
    }
    __syncthreads();
    for (int t = tid; t < npos; t += PF_ATT_THREADS) {
        float *w = pf_att + (size_t)t * rs;
#pragma unroll
        for (int r = 0; r < RS; r++)
            if (t <= rlast[r]) w[r] = fmul(w[r], s_inv[r]);
    }

    // ---- outputs: thread = (dimension, row group), over staged value chunks ----
    const int groups = pf_attn_groups(hd);   // 1, 2, 4 or 8
    constexpr int rg = RG;                   // rows per group (groups * RG >= rs)
    for (int i0 = 0; i0 < hd; i0 += PF_ATT_THREADS) {
        const int g = groups > 1 ? tid / hd : 0;
        const int i = groups > 1 ? tid - g * hd : i0 + tid;
        const int r0 = g * rg;
        const bool live = i < hd && r0 < rows;
        float2 o[RG / 2];
#pragma unroll
        for (int r = 0; r < RG / 2; r++) o[r] = make_float2(0.0f, 0.0f);
        if (i0 > 0) {   // a second pass over the dimensions stages the values again
            __syncthreads();
            pf_stage_v(kvb0, vt, 0, min(PF_ATT_CH, npos), hd);
        }
        for (int c = 0; c < nch; c++) {
            const int c0 = c * PF_ATT_CH, n = min(PF_ATT_CH, npos - c0);
            if (c + 1 < nch) {
                pf_stage_v(kvb0 + ((c + 1) & 1) * cbuf, vt, c0 + PF_ATT_CH, min(PF_ATT_CH, npos - c0 - PF_ATT_CH), hd);
                cp_async_wait_1();
            } else {
                cp_async_wait_all();
            }
            __syncthreads();   // the chunk (and, for c = 0, the weights) are visible
            const T *vb = kvb0 + (c & 1) * cbuf;
            if (live) {
                // positions every row takes, then each row up to its own position
                const int t_all = min(n, p_first + 1 - c0);
                int t = 0;
                for (; t + 8 <= t_all; t += 8) {
                    float vv[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) vv[j] = widen(vb[(size_t)(t + j) * hd + i]);
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        const float4 *wv = reinterpret_cast<const float4 *>(pf_att + (size_t)(c0 + t + j) * rs + r0);
#pragma unroll
                        for (int r4 = 0; r4 < RG / 4; r4++) {
                            if (r0 + 4 * r4 < rs) {   // stay inside this position's row
                                const float4 w4 = wv[r4];
                                o[2 * r4] = add_f32x2(o[2 * r4], make_float2(fmul(w4.x, vv[j]), fmul(w4.y, vv[j])));
                                o[2 * r4 + 1] = add_f32x2(o[2 * r4 + 1], make_float2(fmul(w4.z, vv[j]), fmul(w4.w, vv[j])));
                            }
                        }
                    }
                }
                for (; t < n; t++) {
                    const int tp = c0 + t;
                    const float v = widen(vb[(size_t)t * hd + i]);
#pragma unroll
                    for (int r = 0; r < RG; r++) {
                        const int rr = r0 + r;
                        if (rr < rows && tp <= pos0 + rr / kv_mul) {
                            const float w = pf_att[(size_t)tp * rs + rr];
                            if (r & 1) o[r >> 1].y = fadd(o[r >> 1].y, fmul(w, v));
                            else o[r >> 1].x = fadd(o[r >> 1].x, fmul(w, v));
                        }
                    }
                }
            }
            __syncthreads();   // the buffer is free for chunk c + 2
        }
        // quantize per (token, head): a warp holds 32 consecutive dimensions of
        // its group's rows
        const bool warp_live = (groups > 1 ? (warp * 32) / hd < groups : i0 + warp * 32 < hd);
        if (warp_live) {
#pragma unroll
            for (int r = 0; r < RG; r++) {
                const int rr = r0 + r;
                if (rr < rows) {
                    const float orr = (r & 1) ? o[r >> 1].y : o[r >> 1].x;
                    float dq;
                    const int8_t q = quant_lane(orr, &dq);
                    const int j = rr / kv_mul, hm = rr - j * kv_mul;
                    const int gi = (kvh * kv_mul + hm) * hd + i;
                    a.xq[(size_t)(b0 + j) * a.k_pad + gi] = q;
                    if (lane == 0) a.xs[(size_t)(gi / 32) * a.n_pad + b0 + j] = dq;
                }
            }
        }
    }
}

}  // namespace emb
