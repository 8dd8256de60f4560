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
#include "exact_sum.cuh"

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

EMB_DEV void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// 2-D tiled TMA load (no multicast): box at (x = inner element, y = row)
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

// 32 consecutive 32-bit TMEM columns of this thread's lane; the wait is in the
// same statement so no use of r[] can be scheduled before the data arrives
EMB_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
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

constexpr int PF_BM = 128;      // weight rows per tile (the MMA's M)
constexpr int PF_BK = 128;      // K bytes per pipeline stage: four quant blocks
constexpr int PF_STAGES = 4;
// |acc| <= 32*127*127 < 2^22: acc + 1.5*2^23 read as a float is exact, and
// subtracting 1.5*2^23 gives (float)acc exactly
constexpr int PF_MAGIC_I = 0x4B400000;
constexpr float PF_MAGIC_F = 12582912.0f;

enum { PF_EPI_STORE = 0, PF_EPI_RESID = 1 };

struct PfGemmArgs {
    const float *ws;   // weight block scales, fp32 [rows_pad][nbp]
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
    static constexpr int EW = BN / 8;                 // epilogue warps: 4 lane quarters x BN/32 column groups
    static constexpr int THREADS = (EW + 2) * 32;     // + TMA producer warp + MMA warp
    static constexpr int A_BYTES = PF_BM * PF_BK;
    static constexpr int B_BYTES = BN * PF_BK;
    static constexpr int XS_BYTES = 4 * BN * 4;
    static constexpr int OFF_A = 0;
    static constexpr int OFF_B = OFF_A + PF_STAGES * A_BYTES;
    static constexpr int OFF_XS = OFF_B + PF_STAGES * B_BYTES;
    static constexpr int OFF_BAR = OFF_XS + PF_STAGES * XS_BYTES;
    static constexpr int N_BARS = 2 * PF_STAGES + 5;
    static constexpr int OFF_TMEM = OFF_BAR + N_BARS * 8;
    static constexpr int SMEM = OFF_TMEM + 16 + 1024;  // + slack to align the base to 1024
    static constexpr uint32_t TMEM_COLS = 2 * BN;     // two accumulators
};

// One CTA computes a 128-row x BN-token output tile over all K blocks.
//   warp EW      (lane 0) TMA producer: per stage, a 128 x 128-byte weight box,
//                a BN x 128-byte activation box (both 128-byte swizzled) and the
//                activation scales of the stage's four blocks (bulk copies).
//   warp EW + 1  TMEM allocator; (lane 0) MMA issuer: one kind::i8 MMA per quant
//                block into accumulator b & 1, committed to acc_full.
//   warps < EW   epilogue: warp w owns TMEM lanes 32*(w%4).. (tile rows) and
//                columns 32*(w/4).. (tokens); per block it reads its 32 int32
//                sums, frees the accumulator, and adds the block's terms.
// Every wait is bounded; a wait that gives up records ERR_PF_WAIT and the CTA
// drains its copies and MMAs, frees its TMEM and exits.
template <int BN, int EPI>
__global__ void __launch_bounds__(PfLayout<BN>::THREADS) pf_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                                                                       const __grid_constant__ CUtensorMap tmB,
                                                                       const PfGemmArgs a) {
    using Lay = PfLayout<BN>;
    extern __shared__ unsigned char pf_smem_raw[];
    __shared__ int abort_flag;
    const uint32_t raw = smem_u32(pf_smem_raw);
    unsigned char *sm = pf_smem_raw + ((1024u - (raw & 1023u)) & 1023u);
    uint64_t *full = reinterpret_cast<uint64_t *>(sm + Lay::OFF_BAR);
    uint64_t *empty = full + PF_STAGES;
    uint64_t *accf = empty + PF_STAGES;
    uint64_t *acce = accf + 2;
    uint64_t *fin = acce + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sm + Lay::OFF_TMEM);
    volatile int *abort_v = &abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * PF_BM, n0 = blockIdx.y * BN;
    const int nb = a.nb, n_st = (nb + 3) / 4;

    if (threadIdx.x == 0) {
        for (int i = 0; i < PF_STAGES; i++) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1 + Lay::EW);
        }
        for (int i = 0; i < 2; i++) {
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
                mbar_expect_tx(&full[slot], (uint32_t)(Lay::A_BYTES + Lay::B_BYTES + nblk * BN * 4));
                tma_load_2d(sm + Lay::OFF_A + slot * Lay::A_BYTES, &tmA, st * PF_BK, m0, &full[slot]);
                tma_load_2d(sm + Lay::OFF_B + slot * Lay::B_BYTES, &tmB, st * PF_BK, n0, &full[slot]);
                float *xsd = reinterpret_cast<float *>(sm + Lay::OFF_XS + slot * Lay::XS_BYTES);
                for (int j = 0; j < nblk; j++)
                    bulk_g2s(xsd + j * BN, a.xs + (size_t)(4 * st + j) * a.n_pad + n0, (uint32_t)(BN * 4), &full[slot]);
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
            for (int b = 0; b < nb; b++) {
                const int st = b >> 2, j = b & 3, slot = st % PF_STAGES, buf = b & 1;
                if (j == 0 && !pf_wait(&full[slot], (uint32_t)((st / PF_STAGES) & 1), a.err, abort_v)) {
                    *abort_v = 1;
                    break;
                }
                if (!pf_wait(&acce[buf], (uint32_t)(((b >> 1) & 1) ^ 1), a.err, abort_v)) {
                    *abort_v = 1;
                    break;
                }
                tc_fence_after();
                const uint64_t ad = umma_desc_sw128(smem_u32(sm + Lay::OFF_A + slot * Lay::A_BYTES) + 32u * j);
                const uint64_t bd = umma_desc_sw128(smem_u32(sm + Lay::OFF_B + slot * Lay::B_BYTES) + 32u * j);
                mma_i8(tmem + (uint32_t)(buf * BN), ad, bd, idesc);
                mma_commit(&accf[buf]);
                if (j == 3 || b == nb - 1) mma_commit(&empty[slot]);
            }
            // every MMA issued above has completed before TMEM is released
            mma_commit(fin);
            mbar_wait_ns(fin, 0, a.err);
        }
    } else {
        // ---------------- epilogue ----------------
        const int quarter = warp & 3, cg = warp >> 2;
        const int row = m0 + 32 * quarter + lane;
        const bool row_ok = row < a.rows;
        const float *wsr = a.ws + (size_t)row * a.nbp;   // rows are padded: always in bounds
        float2 s2[16];
#pragma unroll
        for (int j = 0; j < 16; j++) s2[j] = make_float2(0.0f, 0.0f);
        const float2 magic = make_float2(PF_MAGIC_F, PF_MAGIC_F);
        float4 dw4 = *reinterpret_cast<const float4 *>(wsr);
        for (int b = 0; b < nb; b++) {
            const int buf = b & 1, st = b >> 2, slot = st % PF_STAGES;
            // lane 0 waits, the warp follows it (tcgen05.ld needs the whole warp)
            int ok = 1;
            if ((b & 3) == 0) {
                if (b > 0) dw4 = *reinterpret_cast<const float4 *>(wsr + b);
                // the stage's scale copies: observed by this warp too
                if (lane == 0) ok = pf_wait(&full[slot], (uint32_t)((st / PF_STAGES) & 1), a.err, abort_v);
            }
            if (lane == 0 && ok) ok = pf_wait(&accf[buf], (uint32_t)((b >> 1) & 1), a.err, abort_v);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(32 * quarter) << 16) + (uint32_t)(buf * BN + cg * 32), r);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[buf]);
            const float dw = (b & 3) == 0 ? dw4.x : (b & 3) == 1 ? dw4.y : (b & 3) == 2 ? dw4.z : dw4.w;
            const float2 dw2 = make_float2(dw, dw);
            const float4 *xsv = reinterpret_cast<const float4 *>(sm + Lay::OFF_XS + slot * Lay::XS_BYTES) +
                                ((b & 3) * BN + cg * 32) / 4;
#pragma unroll
            for (int q4 = 0; q4 < 8; q4++) {
                const float4 xv = xsv[q4];
                float2 f0 = make_float2(__int_as_float((int)r[4 * q4 + 0] + PF_MAGIC_I),
                                        __int_as_float((int)r[4 * q4 + 1] + PF_MAGIC_I));
                float2 f1 = make_float2(__int_as_float((int)r[4 * q4 + 2] + PF_MAGIC_I),
                                        __int_as_float((int)r[4 * q4 + 3] + PF_MAGIC_I));
                f0 = mul_f32x2(sub_f32x2(f0, magic), dw2);
                f1 = mul_f32x2(sub_f32x2(f1, magic), dw2);
                // the multiply whose result is added is scalar: ptxas may contract a
                // packed mul.f32x2 feeding an add into an fma, a scalar mul.rn never
                f0 = make_float2(fmul(f0.x, xv.x), fmul(f0.y, xv.y));
                f1 = make_float2(fmul(f1.x, xv.z), fmul(f1.y, xv.w));
                s2[2 * q4] = add_f32x2(s2[2 * q4], f0);
                s2[2 * q4 + 1] = add_f32x2(s2[2 * q4 + 1], f1);
            }
            if ((b & 3) == 3 || b == nb - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[slot]);
            }
        }
        if (row_ok && !*abort_v) {
#pragma unroll
            for (int j = 0; j < 32; j++) {
                const int t = n0 + cg * 32 + j;
                const float v = (j & 1) ? s2[j >> 1].y : s2[j >> 1].x;
                if (t < a.n) {
                    float *o = a.out + (size_t)t * a.ld + row;
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
}

// --------------------------------------------------------------- packing -------

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
__global__ void __launch_bounds__(256) pf_norm_quant_kernel(const PfTokArgs a) {
    extern __shared__ __align__(16) float pf_row[];
    __shared__ float s_scale;
    const int t = blockIdx.x;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) pf_row[i] = a.x[(size_t)t * a.ld_x + i];
    __syncthreads();
    if (threadIdx.x == 0) s_scale = rms_scale(chain_sumsq(pf_row, a.cols), a.cols, a.eps);
    __syncthreads();
    const float sc = s_scale;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) pf_row[i] = fmul(fmul(pf_row[i], sc), a.norm_w[i]);
    __syncthreads();
    pf_quant_row(pf_row, a, t);
}

// h = g / (1 + expf(-g)) * u (ref src/model.c:403-406), then quantize.
__global__ void __launch_bounds__(256) pf_swiglu_quant_kernel(const PfTokArgs a) {
    extern __shared__ __align__(16) float pf_row[];
    const int t = blockIdx.x;
    const float *xr = a.x + (size_t)t * a.ld_x;
    for (int i = threadIdx.x; i < a.cols; i += blockDim.x) {
        const float g = xr[i], u = xr[a.hidden + i];
        pf_row[i] = fmul(fdiv(g, fadd(1.0f, expf_exact(a.ex, -g))), u);
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
    float eps;
};

// One CTA per (token, head) for the nh query heads and nkv key heads; the key
// CTAs also store the values. Bias (ref :319-321), QK-norm (:326-329), RoPE
// (:66-80), KV store (:39-48) -- the single-token step's arithmetic.
template <typename T>
__global__ void __launch_bounds__(256) pf_qkv_post_kernel(const PfQkvArgs a) {
    __shared__ float vals[256];
    __shared__ float s_scale;
    const int t = blockIdx.x, hh = blockIdx.y, tid = threadIdx.x, hd = a.hd;
    const int pos = a.start + t;
    const int qd = a.nh * hd, kvd = a.nkv * hd;
    const bool is_q = hh < a.nh;
    const int head = is_q ? hh : hh - a.nh;
    const int off = is_q ? head * hd : qd + head * hd;
    const float *bias = is_q ? a.bq : a.bk;
    const float *nw = is_q ? a.q_norm : a.k_norm;
    const float *row = a.qkv + (size_t)t * a.ld;
    if (tid < hd) {
        float v = row[off + tid];
        if (bias) v = fadd(v, bias[head * hd + tid]);
        vals[tid] = v;
    }
    __syncthreads();
    if (nw) {
        if (tid == 0) s_scale = rms_scale(chain_sumsq(vals, hd), hd, a.eps);
        __syncthreads();
        if (tid < hd) vals[tid] = fmul(fmul(vals[tid], s_scale), nw[tid]);
        __syncthreads();
    }
    if (tid < hd / 2) {
        const int ia = a.neox ? tid : 2 * tid, ib = a.neox ? tid + hd / 2 : 2 * tid + 1;
        const float2 cs = a.rope[(size_t)pos * (hd / 2) + tid];
        const float v0 = vals[ia], v1 = vals[ib];
        vals[ia] = fsub(fmul(v0, cs.x), fmul(v1, cs.y));
        vals[ib] = fadd(fmul(v0, cs.y), fmul(v1, cs.x));
    }
    __syncthreads();
    if (tid < hd) {
        if (is_q) {
            a.qr[(size_t)t * qd + head * hd + tid] = vals[tid];
        } else {
            T *kt = reinterpret_cast<T *>(a.kc) + (size_t)head * hd * a.kstride;
            T *vt = reinterpret_cast<T *>(a.vc) + (size_t)head * a.ctx * hd;
            T kq, vq;
            kv_round(vals[tid], &kq);
            float v = row[qd + kvd + head * hd + tid];
            if (a.bv) v = fadd(v, a.bv[head * hd + tid]);
            kv_round(v, &vq);
            kt[(size_t)tid * a.kstride + pos] = kq;
            vt[(size_t)pos * hd + tid] = vq;
        }
    }
}

// ------------------------------------------------------------------ attention --

constexpr int PF_ATT_THREADS = 128;
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
    int p_cap;             // score columns per row in shared memory
    ExpfDev ex;
};

// One CTA per (kv head, tile of tq consecutive tokens); its query rows are the
// tile's tokens x the kv head's query heads. Token j of the tile attends to
// positions 0..start+b0+j. For every row, as in the single-token step (ref
// src/model.c:221-259):
//   scores   sc_t = sum_i q_i*k_t,i in index order, * (1/sqrt(hd));
//   softmax  max, e_t = expf(sc_t - max), den = sequential sum over t (CTA-
//            parallel exact evaluation above 2048 terms), w_t = e_t * (1/den);
//   output   o_i = sum_t w_t*v_t,i in position order, then quantized.
// Each thread carries the chains of all rows at once, so every key and value
// element it loads serves `rows` chains.
template <typename T>
__global__ void __launch_bounds__(PF_ATT_THREADS) pf_attn_kernel(const PfAttnArgs a) {
    extern __shared__ __align__(16) float pf_att[];        // [rows][p_cap] scores / weights
    __shared__ __align__(16) float q_s[256 * PF_ATT_MAX_ROWS];   // [hd][rows]
    __shared__ float red[PF_ATT_MAX_ROWS][PF_ATT_THREADS / 32];
    __shared__ float s_max[PF_ATT_MAX_ROWS], s_inv[PF_ATT_MAX_ROWS];
    __shared__ XsScratch xs;
    const int kvh = blockIdx.x, b0 = blockIdx.y * a.tq, tid = threadIdx.x, hd = a.hd;
    const int kv_mul = a.nh / a.nkv;
    const int ntok = min(a.tq, a.n - b0);
    const int rows = ntok * kv_mul;
    const int qd = a.nh * hd;
    const int p_last = a.start + b0 + ntok - 1;     // the tile's last position
    const T *kt = reinterpret_cast<const T *>(a.kc) + (size_t)kvh * hd * a.kstride;
    const T *vt = reinterpret_cast<const T *>(a.vc) + (size_t)kvh * a.ctx * hd;
    // row r = token j * kv_mul + head hm  (query head kvh * kv_mul + hm)
    for (int idx = tid; idx < PF_ATT_MAX_ROWS * hd; idx += PF_ATT_THREADS) {
        const int r = idx / hd, i = idx - r * hd;
        const int j = r / kv_mul, hm = r - j * kv_mul;
        q_s[i * PF_ATT_MAX_ROWS + r] = r < rows ? a.qr[(size_t)(b0 + j) * qd + (kvh * kv_mul + hm) * hd + i] : 0.0f;
    }
    __syncthreads();

    // ---- scores ----
    const float inv_sqrt = fdiv(1.0f, fsqrt((float)hd));
    for (int t = tid; t <= p_last; t += PF_ATT_THREADS) {
        float sc[PF_ATT_MAX_ROWS];
#pragma unroll
        for (int r = 0; r < PF_ATT_MAX_ROWS; r++) sc[r] = 0.0f;
        for (int i = 0; i < hd; i++) {
            const float k = widen(kt[(size_t)i * a.kstride + t]);
            const float4 *qv = reinterpret_cast<const float4 *>(q_s + i * PF_ATT_MAX_ROWS);
#pragma unroll
            for (int r4 = 0; r4 < PF_ATT_MAX_ROWS / 4; r4++) {
                const float4 q4 = qv[r4];
                sc[4 * r4 + 0] = fadd(sc[4 * r4 + 0], fmul(q4.x, k));
                sc[4 * r4 + 1] = fadd(sc[4 * r4 + 1], fmul(q4.y, k));
                sc[4 * r4 + 2] = fadd(sc[4 * r4 + 2], fmul(q4.z, k));
                sc[4 * r4 + 3] = fadd(sc[4 * r4 + 3], fmul(q4.w, k));
            }
        }
#pragma unroll
        for (int r = 0; r < PF_ATT_MAX_ROWS; r++)
            if (r < rows) pf_att[(size_t)r * a.p_cap + t] = fmul(sc[r], inv_sqrt);
    }
    __syncthreads();

    // ---- softmax, row by row for the reductions ----
    const int warp = tid >> 5, lane = tid & 31;
    for (int r = 0; r < rows; r++) {
        const int pr = a.start + b0 + r / kv_mul;   // this row's position
        float m = -INFINITY;
        for (int t = tid; t <= pr; t += PF_ATT_THREADS) m = fmaxf(m, pf_att[(size_t)r * a.p_cap + t]);
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
    for (int r = 0; r < rows; r++) {
        const int pr = a.start + b0 + r / kv_mul;
        const float mx = s_max[r];
        float *ar = pf_att + (size_t)r * a.p_cap;
        for (int t = tid; t <= pr; t += PF_ATT_THREADS) ar[t] = expf_exact(a.ex, fsub(ar[t], mx));
    }
    __syncthreads();
    // denominators: short sums as one chain per row (rows in parallel), long
    // ones by the CTA-parallel exact evaluation, one row at a time
    if (tid < rows) {
        const int pr = a.start + b0 + tid / kv_mul;
        if (pr + 1 <= 2048) s_inv[tid] = fdiv(1.0f, chain_sum(0.0f, pf_att + (size_t)tid * a.p_cap, pr + 1));
    }
    for (int r = 0; r < rows; r++) {
        const int pr = a.start + b0 + r / kv_mul;
        if (pr + 1 > 2048) {
            const float den = exact_pos_sum<PF_ATT_THREADS>(pf_att + (size_t)r * a.p_cap, pr + 1, &xs);
            if (tid == 0) s_inv[r] = fdiv(1.0f, den);
        }
    }
    __syncthreads();
    for (int r = 0; r < rows; r++) {
        const int pr = a.start + b0 + r / kv_mul;
        const float inv = s_inv[r];
        float *ar = pf_att + (size_t)r * a.p_cap;
        for (int t = tid; t <= pr; t += PF_ATT_THREADS) ar[t] = fmul(ar[t], inv);
    }
    __syncthreads();

    // ---- outputs: one thread per dimension (and per further 128 dimensions) ----
    for (int i0 = 0; i0 < hd; i0 += PF_ATT_THREADS) {
        const int i = i0 + tid;
        float o[PF_ATT_MAX_ROWS];
#pragma unroll
        for (int r = 0; r < PF_ATT_MAX_ROWS; r++) o[r] = 0.0f;
        if (i < hd) {
            int pr[PF_ATT_MAX_ROWS];   // each row's last position (-1: no such row)
#pragma unroll
            for (int r = 0; r < PF_ATT_MAX_ROWS; r++) pr[r] = r < rows ? a.start + b0 + r / kv_mul : -1;
            for (int t = 0; t <= p_last; t++) {
                const float v = widen(vt[(size_t)t * hd + i]);
#pragma unroll
                for (int r = 0; r < PF_ATT_MAX_ROWS; r++)
                    if (t <= pr[r]) o[r] = fadd(o[r], fmul(pf_att[(size_t)r * a.p_cap + t], v));
            }
        }
        // quantize per (token, head): 32 consecutive dimensions per warp
        for (int r = 0; r < rows; r++) {
            const int j = r / kv_mul, hm = r - j * kv_mul;
            float orr = 0.0f;
#pragma unroll
            for (int rr = 0; rr < PF_ATT_MAX_ROWS; rr++)
                if (rr == r) orr = o[rr];
            if (i0 + warp * 32 < hd) {
                float dq;
                const int8_t q = quant_lane(orr, &dq);
                const int gi = (kvh * kv_mul + hm) * hd + i;
                a.xq[(size_t)(b0 + j) * a.k_pad + gi] = q;
                if (lane == 0) a.xs[(size_t)(gi / 32) * a.n_pad + b0 + j] = dq;
            }
        }
    }
}

}  // namespace emb
