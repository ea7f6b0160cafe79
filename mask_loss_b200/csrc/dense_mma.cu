// dense_mma.cu -- dense per-GT mask costs on the 5th-generation tensor cores.
//
// With dense (B, GT_total, H_t, W_t) masks (overlap allowed; no reference
// counterpart, the reference API takes a label map) the contractions of the
// pairwise costs (src/cuda/pw_mask.cu:52-308)
//     D[q,g] = sum_j x_qj k_gj          (sigmoid-CE, before the sign)
//     I[q,g] = sum_j sigmoid(x_qj) k_gj (dice intersection)
// are real GEMMs: k_gj is the pixel count of GT g in cell j, and a cell may
// be covered by several GTs.  Two kernels run them on tcgen05 UMMA with the
// fp32 accumulators in tensor memory (TMEM): dense_mma_tf32_kernel (fp32
// logits, kind::tf32, below) and dense_mma_kernel (16-bit logits, and fp32
// logits when the tf32 one is switched off; kind::f16), described here:
//   * per CTA: one image, one query tile (M = 128 rows, rows >= qrows unused)
//     and half a cell chunk, all GT columns (N = GT_total rounded up to 16,
//     <= 64; the background column is computed and dropped on output);
//   * K blocks of 32 cells.  A TMA box brings the block's logits into shared
//     memory (the cost kernel's tensor map: fp32 rows with the 128-byte
//     swizzle, bf16/fp16 rows with the 64-byte one, widened exactly);
//   * eight producer warps (warp w: rows 32*(w%4).., cells 16*(w/4)..) compute
//     sigmoid and the row sums on CUDA cores and write the A operands to TMEM
//     as bf16 hi/lo pairs (x = xh + xl and p = ph + pl, each part rounded to
//     nearest, so |x - xh - xl| <= 2^-18 |x|): four K-major 128 x 32 bf16
//     operands, 16 TMEM columns each;
//   * the B operand -- the block's pixel counts, kept as bf16 by the count
//     kernel (exact for counts <= 256) -- arrives by TMA with the logits:
//     N rows of 64 bytes in the 64-byte swizzled K-major layout the MMA reads;
//   * one thread of the control warp issues the TMA loads and the MMAs
//     (kind::f16, A from TMEM, B from shared memory, 128 x N x 16 each):
//     D += xh k + xl k, I += ph k + pl k, and signals completion with
//     tcgen05.commit on an mbarrier;
//   * two rings: four shared-memory stages of logits + counts, refilled as
//     soon as the MMAs that read a stage's counts completed (loads run up to
//     three blocks ahead), and two TMEM stages of A operands: while the
//     tensor core works on block kb the producers write block kb+1;
//   * epilogue: the producer warps read D and I from TMEM (tcgen05.ld) and
//     write the label path's chunk-partial slot, so cost_rows / cost_pairs,
//     the solver and the matched loss run unchanged.
// TMEM: 2N accumulator columns + 2 stages x 4 operands x 16 columns <= 256,
// so two CTAs share an SM.  With bf16 logits x is already an exact bf16
// operand: the MMA reads it from the TMA'd tile and only p is split (two
// TMEM operands a stage).  With unscaled masks (and bf16 logits, N <= 32)
// the B tile is built by the producers from the mask bytes themselves, and
// the mask areas are summed on the way, so no count pass runs.  Every wait
// is bounded (2 s) and reports through the status word instead of hanging;
// TMEM is released on every path.
#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

namespace {

constexpr int kMmaK = 32;          // cells per K block
constexpr int kMmaStages = 2;     // A operand stages in TMEM
constexpr int kTmaStages = 4;     // logits + counts stages in shared memory
constexpr int kMmaProducers = 8;   // warps
constexpr int kMmaThreads = (kMmaProducers + 1) * 32;
constexpr int kMmaTmemCols = 256;

// --- tcgen05 / TMEM wrappers (PTX ISA 8.7, sm_100a) -------------------------
ML_INLINE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
}
ML_INLINE void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
ML_INLINE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
ML_INLINE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ML_INLINE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
ML_INLINE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// eight 32-bit columns of this warp's 32 lanes
ML_INLINE void tmem_st8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
                   "r"(v[6]), "r"(v[7]) : "memory");
}
ML_INLINE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
ML_INLINE void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, "
                 "%10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
                   "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
                   "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                 : "r"(taddr) : "memory");
}
ML_INLINE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] x B[smem]^T, kind::f16 (bf16 in, fp32 accumulate).
ML_INLINE void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                       bool accumulate) {
    const uint32_t acc = accumulate ? 1u : 0u;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc) : "memory");
}
// D[tmem] (+)= A[smem] x B[smem]^T, kind::f16 (bf16 in, fp32 accumulate).
ML_INLINE void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                       bool accumulate) {
    const uint32_t acc = accumulate ? 1u : 0u;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc) : "memory");
}
// Arrive once on `bar` when every MMA this thread issued before has completed.
ML_INLINE void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// Shared-memory matrix descriptor, K-major with the 64-byte swizzle (rows of
// 32 bf16; 8-row atoms of 512 bytes, so SBO = 512; LBO unused, 1): the layout
// a TMA box with CU_TENSOR_MAP_SWIZZLE_64B writes.  Layout type 4 [61,64).
ML_INLINE uint64_t smem_desc_sw64(const void* p) {
    const uint64_t a = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
    return a | (1ull << 16) | ((uint64_t)(512u >> 4) << 32) | (1ull << 46) | (4ull << 61);
}

// Instruction descriptor of kind::f16: bf16 A and B (K-major), fp32 D,
// M = 128, N = n (multiple of 16, <= 256).
ML_INLINE uint32_t idesc_bf16_f32(int n) {
    return (1u << 4)             // D format: f32
           | (1u << 7)           // A format: bf16
           | (1u << 10)          // B format: bf16
           | ((uint32_t)(n >> 3) << 17)
           | ((uint32_t)(128 >> 4) << 24);
}

ML_INLINE uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
ML_INLINE float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
ML_INLINE float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// The kind::tf32 forms (fp32 logits): D[tmem] (+)= A x B^T with A from TMEM
// (ts) or shared memory (ss), B from shared memory, 32-bit operands of
// which the tensor core uses the tf32 part.
ML_INLINE void umma_ts_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                            bool accumulate) {
    const uint32_t acc = accumulate ? 1u : 0u;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc) : "memory");
}
ML_INLINE void umma_ss_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                            bool accumulate) {
    const uint32_t acc = accumulate ? 1u : 0u;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc) : "memory");
}
// K-major, 128-byte swizzle (rows of 32 fp32; 8-row atoms of 1024 bytes, so
// SBO = 1024; LBO unused, 1): the layout a TMA box with
// CU_TENSOR_MAP_SWIZZLE_128B writes.  Layout type 2 [61,64).
ML_INLINE uint64_t smem_desc_sw128(const void* p) {
    const uint64_t a = (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu);
    return a | (1ull << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// kind::tf32 instruction descriptor: tf32 A and B (K-major), fp32 D, M = 128.
ML_INLINE uint32_t idesc_tf32_f32(int n) {
    return (1u << 4)             // D format: f32
           | (2u << 7)           // A format: tf32
           | (2u << 10)          // B format: tf32
           | ((uint32_t)(n >> 3) << 17)
           | ((uint32_t)(128 >> 4) << 24);
}
// sixteen 32-bit columns of this warp's 32 lanes
ML_INLINE void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, "
                 "%9, %10, %11, %12, %13, %14, %15, %16};"
                 ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
                   "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]),
                   "r"(v[13]), "r"(v[14]), "r"(v[15]) : "memory");
}
// the tf32 part of x (the low 13 mantissa bits cleared) and its remainder
ML_INLINE float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

struct MmaShared {
    uint64_t full[kTmaStages];    // logits and counts of the stage landed (TMA)
    uint64_t aready[kMmaStages];  // A operands of the TMEM stage written
    uint64_t mdone[kTmaStages];   // the MMAs of the block held in the stage completed
    uint64_t accf;                // all MMAs completed
    uint32_t tmem_base;
    int32_t err;
    float rows[4][32][3];         // row sums of the second cell half (warps 4..7)
};

}  // namespace

// Four logits [4*u, 4*u + 4) of cells 16*kh.. of row r from the swizzled TMA
// tile: fp32 rows of 128 bytes (16-byte granule g at g ^ (r & 7)), 16-bit
// rows of 64 bytes (granule g at g ^ ((r >> 1) & 3)), widened exactly.
template <typename T>
ML_INLINE float4 tile_quad(const T* row, int r, int kh, int u) {
    if constexpr (sizeof(T) == 4) {
        const int g = 4 * kh + u;
        return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(row) + ((g ^ (r & 7)) << 2));
    } else {
        const int k = 16 * kh + 4 * u;           // first of the four cells
        const int g = k >> 3;                     // 8 cells per granule
        const uint2 w = *reinterpret_cast<const uint2*>(row + ((g ^ ((r >> 1) & 3)) << 3) + (k & 7));
        float4 v;
        widen2(w.x, v.x, v.y, row);
        widen2(w.y, v.z, v.w, row);
        return v;
    }
}

// grid = (nchunk * 2, nqt, L*B); block = kMmaThreads.
// Dynamic shared memory: per stage the logits tile [qrows_smem][32] of T
// (1024-aligned), then per stage the B tile [4][N][8] bf16, then MmaShared.
// MASKB (bf16 logits, s = 1, N <= 32): kmap covers the uint8 masks; the
// producers build the bf16 B tile from the mask bytes (one thread per GT row
// and 4 cells) and sum the mask areas, as in dense_mma_tf32_kernel.
template <typename T, bool MASKB>
__global__ void __launch_bounds__(kMmaThreads, 2)
dense_mma_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap kmap,
                 CostArgs a, int N) {
    extern __shared__ __align__(1024) unsigned char dsm_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
    // bf16 logits are exact bf16 A operands: the MMA reads x straight from the
    // TMA'd tile (128 rows per stage, so the M = 128 read stays in the stage)
    // and only p is split; fp32 and fp16 logits are split into bf16 hi/lo
    constexpr bool AX = std::is_same<T, __nv_bfloat16>::value;
    constexpr int NOP = AX ? 2 : 4;  // TMEM operands per stage
    const int QS = AX ? 128 : (a.qrows + 7) / 8 * 8;
    // per stage: counts [N][32] bf16 (64-byte rows, 1024-aligned), logits [QS][32] of T
    const int bstage = (N * 64 + 1023) / 1024 * 1024;
    __nv_bfloat16* bs = reinterpret_cast<__nv_bfloat16*>(base);                 // [stage][N][32]
    T* xs = reinterpret_cast<T*>(base + kTmaStages * bstage);                    // [stage][QS][32]
    unsigned char* ms = reinterpret_cast<unsigned char*>(xs + kTmaStages * QS * kMmaK);  // MASKB bytes
    const uint32_t mstage = MASKB ? ((uint32_t)N * 32u + 127u) / 128u * 128u : 0u;
    MmaShared* sh = reinterpret_cast<MmaShared*>(ms + kTmaStages * mstage);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slot = blockIdx.x, chunk = slot >> 1, half = slot & 1;
    const int qt = blockIdx.y, lb = blockIdx.z, b = lb % a.B;
    const int HW = a.H * a.W, G = a.gout, NG = a.gt_total;
    const int half_cells = a.chunk_cells / 2;
    const int cb = min(HW, chunk * a.chunk_cells + half * half_cells);
    const int ce = min(HW, cb + half_cells);
    const int nkb = (ce - cb + kMmaK - 1) / kMmaK;
    const int row0 = lb * a.Q + qt * a.qrows;
    const uint32_t cols_acc = 2u * N;

    if (tid == 0) {
        for (int i = 0; i < kTmaStages; ++i) {
            mbar_init(&sh->full[i], 1);
            mbar_init(&sh->mdone[i], 1);
        }
        for (int i = 0; i < kMmaStages; ++i) mbar_init(&sh->aready[i], kMmaProducers);
        mbar_init(&sh->accf, 1);
        sh->err = 0;
        fence_mbar_init();
    }
    if (warp == kMmaProducers) {  // the control warp owns the TMEM allocation
        tmem_alloc(&sh->tmem_base, kMmaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = sh->tmem_base;
    // TMEM columns: D [0, N), I [N, 2N), then stage s operand o at 2N + (NOP s + o) * 16
    auto a_col = [&](int s, int o) { return tbase + cols_acc + (uint32_t)((NOP * s + o) * 16); };

    if (warp == kMmaProducers) {
        // ------------------------------ control warp ------------------------------
        if (lane == 0) {
            bool ok = true;
            const uint32_t idesc = idesc_bf16_f32(N);
            auto issue_tma = [&](int kb) {
                const int s = kb % kTmaStages;
                mbar_arrive_expect_tx(&sh->full[s], (uint32_t)a.qrows * kMmaK * (uint32_t)sizeof(T) +
                                                        (uint32_t)N * kMmaK * (MASKB ? 1u : 2u));
                const int c0 = cb + kb * kMmaK;
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                    " [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(xs + s * QS * kMmaK)), "l"(&tmap), "r"(c0), "r"(row0),
                      "r"(smem_u32(&sh->full[s])) : "memory");
                // counts of GT rows [b*NG, b*NG + N) (rows past the image's own
                // are other images' or zeros: their accumulators are never read)
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                    " [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(MASKB ? ms + s * mstage
                                         : reinterpret_cast<unsigned char*>(bs) + s * bstage)),
                      "l"(&kmap), "r"(c0), "r"(b * NG), "r"(smem_u32(&sh->full[s])) : "memory");
            };
            for (int kb = 0; kb < min(nkb, kTmaStages); ++kb) issue_tma(kb);
            for (int kb = 0; kb < nkb && ok; ++kb) {
                const int s = kb % kTmaStages;   // shared-memory stage (counts)
                const int ts = kb % kMmaStages;  // TMEM stage (A operands)
                if (!mbar_wait(&sh->aready[ts], (uint32_t)((kb / kMmaStages) & 1))) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 2; ++kk) {  // K = 16 cells (32 bytes of a row) per MMA
                    const uint64_t bd =
                        smem_desc_sw64(reinterpret_cast<unsigned char*>(bs) + s * bstage + 32 * kk);
                    const bool acc = kb > 0 || kk > 0;
                    if constexpr (AX) {
                        const uint64_t ad = smem_desc_sw64(
                            reinterpret_cast<const unsigned char*>(xs + s * QS * kMmaK) + 32 * kk);
                        umma_ss(tbase, ad, bd, idesc, acc);                             // D += x k
                        umma_ts(tbase + N, a_col(ts, 0) + 8 * kk, bd, idesc, acc);      // I += ph k
                        umma_ts(tbase + N, a_col(ts, 1) + 8 * kk, bd, idesc, true);     // I += pl k
                    } else {
                        umma_ts(tbase, a_col(ts, 0) + 8 * kk, bd, idesc, acc);          // D += xh k
                        umma_ts(tbase, a_col(ts, 1) + 8 * kk, bd, idesc, true);         // D += xl k
                        umma_ts(tbase + N, a_col(ts, 2) + 8 * kk, bd, idesc, acc);      // I += ph k
                        umma_ts(tbase + N, a_col(ts, 3) + 8 * kk, bd, idesc, true);     // I += pl k
                    }
                }
                umma_commit(&sh->mdone[s]);
                // refill the stage of the previous block (its MMAs, issued one
                // block ago, read its counts) with the block kTmaStages later,
                // so loads run up to three blocks ahead of the producers
                const int kp = kb - 1;
                if (kp >= 0 && kp + kTmaStages < nkb) {
                    if (!mbar_wait(&sh->mdone[kp % kTmaStages], (uint32_t)((kp / kTmaStages) & 1))) {
                        ok = false;
                        break;
                    }
                    issue_tma(kp + kTmaStages);
                }
            }
            if (ok && nkb > 0) umma_commit(&sh->accf);
            if (!ok) {
                sh->err = 1;
                if (a.status) atomicOr(a.status, 2);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------ producer warps ------------------------------
        const int r = 32 * (warp & 3) + lane;      // query row of the tile (TMEM lane)
        const int kh = warp >> 2;                  // cells [16 kh, 16 kh + 16) of each block
        const bool rvalid = r < a.qrows && qt * a.qrows + r < a.Q;
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        float rsum[3] = {0.0f, 0.0f, 0.0f};        // sum max(x,0), sum p, sum log2(1+e)
        int area = 0;  // MASKB: non-zero mask bytes this thread converted (its GT row)
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % kTmaStages;   // shared-memory stage
            const int ts = kb % kMmaStages;  // TMEM stage
            const int c0 = cb + kb * kMmaK;
            const int nv = min(kMmaK, ce - c0);
            // the TMEM stage is free once the MMAs of block kb - kMmaStages completed
            if (kb >= kMmaStages) {
                const int kq = kb - kMmaStages;
                if (!mbar_wait(&sh->mdone[kq % kTmaStages], (uint32_t)((kq / kTmaStages) & 1))) {
                    ok = false;
                    break;
                }
            }
            if (!mbar_wait(&sh->full[s], (uint32_t)((kb / kTmaStages) & 1))) { ok = false; break; }
            // A: this thread's 16 cells of row r
            const T* xr = xs + (s * QS + r) * kMmaK;
            uint32_t xh[8], xl[8], ph[8], pl[8];
            const bool full = nv == kMmaK && rvalid;
            float prod = 1.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {  // four 16-byte granules = 16 cells
                const float4 v = rvalid ? tile_quad<T>(xr, r, kh, u) : make_float4(0.f, 0.f, 0.f, 0.f);
                float xv[4] = {v.x, v.y, v.z, v.w};
                float pv[4];
                if (full) {
#pragma unroll
                    for (int e4 = 0; e4 < 4; ++e4) {
                        const Fast f = fast_elem(xv[e4]);
                        pv[e4] = f.p;
                        rsum[0] += fmaxf(xv[e4], 0.0f);
                        rsum[1] += f.p;
                        prod *= f.d;
                    }
                } else {
#pragma unroll
                    for (int e4 = 0; e4 < 4; ++e4) {
                        const bool in = rvalid && 16 * kh + 4 * u + e4 < nv;
                        xv[e4] = in ? xv[e4] : 0.0f;
                        const Fast f = fast_elem(xv[e4]);
                        pv[e4] = in ? f.p : 0.0f;
                        if (in) {
                            rsum[0] += fmaxf(xv[e4], 0.0f);
                            rsum[1] += f.p;
                            prod *= f.d;
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    if constexpr (!AX) {
                        const uint32_t hx = pack_bf16(xv[2 * j], xv[2 * j + 1]);
                        xh[2 * u + j] = hx;
                        xl[2 * u + j] = pack_bf16(xv[2 * j] - bf16_lo(hx), xv[2 * j + 1] - bf16_hi(hx));
                    }
                    const uint32_t hp = pack_bf16(pv[2 * j], pv[2 * j + 1]);
                    ph[2 * u + j] = hp;
                    pl[2 * u + j] = pack_bf16(pv[2 * j] - bf16_lo(hp), pv[2 * j + 1] - bf16_hi(hp));
                }
            }
            rsum[2] += lg2_approx(prod);  // 16 factors in [1, 2]
            if constexpr (MASKB) {  // mask bytes -> the bf16 B tile (64-byte swizzle), 4 cells a thread
                const int pt = warp * 32 + lane;
                if (pt < N * 8) {
                    const int n = pt >> 3, q = pt & 7;
                    const uint32_t m = *reinterpret_cast<const uint32_t*>(ms + s * mstage + n * 32 + q * 4);
                    const uint32_t one = 0x3F80u;  // bf16 1.0
                    const uint2 w = make_uint2(((m & 0xFFu) ? one : 0u) | ((m & 0xFF00u) ? one << 16 : 0u),
                                               ((m & 0xFF0000u) ? one : 0u) | ((m & 0xFF000000u) ? one << 16 : 0u));
                    *reinterpret_cast<uint2*>(reinterpret_cast<unsigned char*>(bs) + s * bstage + n * 64 +
                                              ((((q >> 1) ^ ((n >> 1) & 3))) << 4) + (q & 1) * 8) = w;
                    area += __popc(__vcmpne4(m, 0u)) >> 3;  // cells past H*W read as zeros
                }
                fence_proxy_async_smem();  // the B tile is read by the tensor core
            }
            const uint32_t colk = (uint32_t)(8 * kh);  // 16 bf16 cells = 8 columns
            if constexpr (AX) {
                tmem_st8(a_col(ts, 0) + lane_off + colk, ph);
                tmem_st8(a_col(ts, 1) + lane_off + colk, pl);
            } else {
                tmem_st8(a_col(ts, 0) + lane_off + colk, xh);
                tmem_st8(a_col(ts, 1) + lane_off + colk, xl);
                tmem_st8(a_col(ts, 2) + lane_off + colk, ph);
                tmem_st8(a_col(ts, 3) + lane_off + colk, pl);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->aready[ts]);
        }
        if (!ok) {
            sh->err = 1;
            if (lane == 0 && a.status) atomicOr(a.status, 2);
        }
        if (MASKB && qt == 0 && lb < a.B) {  // mask areas: first query tile of the first layer
#pragma unroll
            for (int o = 4; o > 0; o >>= 1) area += __shfl_down_sync(0xffffffffu, area, o);
            const int n = (warp * 32 + lane) >> 3;
            if ((lane & 7) == 0 && n < NG && area > 0)
                atomicAdd(const_cast<int32_t*>(a.totals) + (int64_t)b * NG + n, area);
        }
        // ---- epilogue: row sums of the two cell halves, then D and I from TMEM ----
        if (kh == 1) {
#pragma unroll
            for (int i = 0; i < 3; ++i) sh->rows[warp & 3][lane][i] = rsum[i];
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kMmaProducers * 32) : "memory");
        const bool have_acc = ok && nkb > 0 && mbar_wait(&sh->accf, 0u);
        tc_fence_after();
        float* part = a.part + ((((int64_t)lb * a.nqt + qt) * a.nchunk + chunk) * 2 + half) *
                                   (int64_t)a.part_stride;
        const int QP = a.qrows_pad;
        // warps 0-3 write D (as -D: the partial holds sum(-x k)) and the row
        // sums, warps 4-7 write I
        const uint32_t acc_base = tbase + lane_off + (kh ? (uint32_t)N : 0u);
        for (int c0a = 0; c0a < N; c0a += 16) {  // accumulator columns = GT ids
            uint32_t v[16];
            if (have_acc) {
                tmem_ld16(acc_base + (uint32_t)c0a, v);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0u;
            }
            if (rvalid) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int ga = c0a + j;
                    if (ga < NG && ga != a.bg) {
                        const int g = ga - (ga > a.bg ? 1 : 0);  // output column
                        const float val = __uint_as_float(v[j]);
                        part[((int64_t)kh * G + g) * QP + r] = kh ? val : -val;
                    }
                }
            }
        }
        if (kh == 0 && rvalid) {
#pragma unroll
            for (int i = 0; i < 3; ++i)
                part[(int64_t)2 * G * QP + (int64_t)i * QP + r] = rsum[i] + sh->rows[warp & 3][lane][i];
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == kMmaProducers) {
        tc_fence_after();
        tmem_dealloc(tbase, kMmaTmemCols);
    }
}

// fp32 logits on kind::tf32.  The same tiling, rings and epilogue as
// dense_mma_kernel, with the operands split the tf32 way:
//   * D += x_hi k + x_lo k: x_hi is the logits tile itself -- the producers
//     clear the low 13 mantissa bits of each value in place (so the tensor
//     core's tf32 read is exact whatever its rounding) and the MMA takes it
//     straight from shared memory; x_lo = x - x_hi goes to TMEM;
//   * I += p_hi k + p_lo k, both from TMEM (p_hi with the low bits cleared);
//   * B: the counts as fp32 (exact), N rows of 128 bytes, 128-byte swizzle.
// Per logit the producers thus do a sigmoid, two splits and the row sums;
// the bf16 kernel's four operand conversions become one in-place mask.
// |x - x_hi - tf32(x_lo)| <= 2^-21 |x|, likewise for p.
// TMEM: 2N accumulator columns + TS stages x 3 operands x 32 columns <= 256
// (TS = 2 for N <= 32, 1 for N <= 64), so two CTAs share an SM.
// MASKB (s = 1): kmap covers the uint8 masks themselves ([B*GT_total][H*W],
// boxes of 32 cells x N rows, no swizzle); the producers turn each block's
// mask bytes into the fp32 B tile (1.0 where non-zero), so no count planes
// are written or read.
template <bool MASKB, int TS>
__global__ void __launch_bounds__(kMmaThreads, 2)
dense_mma_tf32_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap kmap,
                      CostArgs a, int N) {
    extern __shared__ __align__(1024) unsigned char dsm_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
    constexpr uint32_t kXStage = 128u * kMmaK * 4u;   // logits [128][32] fp32 per stage
    const uint32_t bstage = ((uint32_t)N * 128u + 1023u) / 1024u * 1024u;
    float* xs = reinterpret_cast<float*>(base);                               // [stage][128][32]
    unsigned char* bs = base + kTmaStages * kXStage;                          // [stage][N][32] fp32
    // MASKB: the TMA'd mask bytes, [stage][N][32] uint8
    unsigned char* ms = bs + kTmaStages * bstage;
    const uint32_t mstage = MASKB ? ((uint32_t)N * 32u + 127u) / 128u * 128u : 0u;
    MmaShared* sh = reinterpret_cast<MmaShared*>(ms + kTmaStages * mstage);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slot = blockIdx.x, chunk = slot >> 1, half = slot & 1;
    const int qt = blockIdx.y, lb = blockIdx.z, b = lb % a.B;
    const int HW = a.H * a.W, G = a.gout, NG = a.gt_total;
    const int half_cells = a.chunk_cells / 2;
    const int cb = min(HW, chunk * a.chunk_cells + half * half_cells);
    const int ce = min(HW, cb + half_cells);
    const int nkb = (ce - cb + kMmaK - 1) / kMmaK;
    const int row0 = lb * a.Q + qt * a.qrows;
    const uint32_t cols_acc = 2u * N;

    if (tid == 0) {
        for (int i = 0; i < kTmaStages; ++i) {
            mbar_init(&sh->full[i], 1);
            mbar_init(&sh->mdone[i], 1);
        }
        for (int i = 0; i < TS; ++i) mbar_init(&sh->aready[i], kMmaProducers);
        mbar_init(&sh->accf, 1);
        sh->err = 0;
        fence_mbar_init();
    }
    if (warp == kMmaProducers) {
        tmem_alloc(&sh->tmem_base, kMmaTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = sh->tmem_base;
    // TMEM columns: D [0, N), I [N, 2N), then stage s operand o at 2N + (3s + o) * 32
    auto a_col = [&](int s, int o) { return tbase + cols_acc + (uint32_t)((3 * s + o) * 32); };

    if (warp == kMmaProducers) {
        // ------------------------------ control warp ------------------------------
        if (lane == 0) {
            bool ok = true;
            const uint32_t idesc = idesc_tf32_f32(N);
            auto issue_tma = [&](int kb) {
                const int s = kb % kTmaStages;
                mbar_arrive_expect_tx(&sh->full[s], (uint32_t)a.qrows * kMmaK * 4u +
                                                        (uint32_t)N * kMmaK * (MASKB ? 1u : 4u));
                const int c0 = cb + kb * kMmaK;
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                    " [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(reinterpret_cast<unsigned char*>(xs) + s * kXStage)), "l"(&tmap),
                      "r"(c0), "r"(row0), "r"(smem_u32(&sh->full[s])) : "memory");
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                    " [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(MASKB ? ms + s * mstage : bs + s * bstage)), "l"(&kmap), "r"(c0),
                      "r"(b * NG), "r"(smem_u32(&sh->full[s])) : "memory");
            };
            for (int kb = 0; kb < min(nkb, kTmaStages); ++kb) issue_tma(kb);
            for (int kb = 0; kb < nkb && ok; ++kb) {
                const int s = kb % kTmaStages;
                const int ts = kb % TS;
                if (!mbar_wait(&sh->aready[ts], (uint32_t)((kb / TS) & 1))) { ok = false; break; }
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {  // K = 8 cells (32 bytes of a row) per MMA
                    const uint64_t ad =
                        smem_desc_sw128(reinterpret_cast<unsigned char*>(xs) + s * kXStage + 32 * kk);
                    const uint64_t bd = smem_desc_sw128(bs + s * bstage + 32 * kk);
                    const bool acc = kb > 0 || kk > 0;
                    umma_ss_tf32(tbase, ad, bd, idesc, acc);                      // D += x_hi k
                    umma_ts_tf32(tbase, a_col(ts, 0) + 8 * kk, bd, idesc, true);  // D += x_lo k
                    umma_ts_tf32(tbase + N, a_col(ts, 1) + 8 * kk, bd, idesc, acc);  // I += p_hi k
                    umma_ts_tf32(tbase + N, a_col(ts, 2) + 8 * kk, bd, idesc, true); // I += p_lo k
                }
                umma_commit(&sh->mdone[s]);
                const int kp = kb - 1;
                if (kp >= 0 && kp + kTmaStages < nkb) {
                    if (!mbar_wait(&sh->mdone[kp % kTmaStages], (uint32_t)((kp / kTmaStages) & 1))) {
                        ok = false;
                        break;
                    }
                    issue_tma(kp + kTmaStages);
                }
            }
            if (ok && nkb > 0) umma_commit(&sh->accf);
            if (!ok) {
                sh->err = 1;
                if (a.status) atomicOr(a.status, 2);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------ producer warps ------------------------------
        const int r = 32 * (warp & 3) + lane;      // query row of the tile (TMEM lane)
        const int kh = warp >> 2;                  // cells [16 kh, 16 kh + 16) of each block
        const bool rvalid = r < a.qrows && qt * a.qrows + r < a.Q;
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        float rsum[3] = {0.0f, 0.0f, 0.0f};        // sum max(x,0), sum p, sum log2(1+e)
        int area[2] = {0, 0};  // MASKB: non-zero mask bytes converted, GT rows n and n + 32
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % kTmaStages;
            const int ts = kb % TS;
            const int c0 = cb + kb * kMmaK;
            const int nv = min(kMmaK, ce - c0);
            if (kb >= TS) {
                const int kq = kb - TS;
                if (!mbar_wait(&sh->mdone[kq % kTmaStages], (uint32_t)((kq / kTmaStages) & 1))) {
                    ok = false;
                    break;
                }
            }
            if (!mbar_wait(&sh->full[s], (uint32_t)((kb / kTmaStages) & 1))) { ok = false; break; }
            float* xr = xs + (size_t)s * (kXStage / 4) + r * kMmaK;   // row r: 128 swizzled bytes
            uint32_t xl[16], ph[16], pl[16];
            float prod = 1.0f;
#pragma unroll
            for (int u = 0; u < 4; ++u) {  // four 16-byte granules = 16 cells
                float4* gp = reinterpret_cast<float4*>(xr + (((4 * kh + u) ^ (r & 7)) << 2));
                const float4 v = *gp;
                const float xv[4] = {v.x, v.y, v.z, v.w};
                float xt[4];
#pragma unroll
                for (int e4 = 0; e4 < 4; ++e4) {
                    const float x = xv[e4];
                    xt[e4] = tf32_hi(x);
                    const Fast f = fast_elem(x);
                    const float pt = tf32_hi(f.p);
                    xl[4 * u + e4] = __float_as_uint(x - xt[e4]);
                    ph[4 * u + e4] = __float_as_uint(pt);
                    pl[4 * u + e4] = __float_as_uint(f.p - pt);
                    if (rvalid && 16 * kh + 4 * u + e4 < nv) {
                        rsum[0] += fmaxf(x, 0.0f);
                        rsum[1] += f.p;
                        prod *= f.d;
                    }
                }
                *gp = make_float4(xt[0], xt[1], xt[2], xt[3]);  // the MMA reads x_hi here
            }
            if (MASKB) {  // mask bytes -> the fp32 B tile, 4 cells per thread
                const int pt = warp * 32 + lane;
#pragma unroll
                for (int h2 = 0; h2 < 2; ++h2) {  // rows n and n + 32 (N <= 64)
                    const int t2 = pt + 256 * h2;
                    if (t2 >= N * 8) break;
                    const int n = t2 >> 3, g = t2 & 7;
                    const uint32_t m = *reinterpret_cast<const uint32_t*>(ms + s * mstage + n * 32 + g * 4);
                    *reinterpret_cast<float4*>(bs + s * bstage + n * 128 + ((g ^ (n & 7)) << 4)) =
                        make_float4((m & 0xFFu) ? 1.0f : 0.0f, (m & 0xFF00u) ? 1.0f : 0.0f,
                                    (m & 0xFF0000u) ? 1.0f : 0.0f, (m & 0xFF000000u) ? 1.0f : 0.0f);
                    area[h2] += __popc(__vcmpne4(m, 0u)) >> 3;  // cells past H*W read as zeros
                }
            }
            rsum[2] += lg2_approx(prod);  // 16 factors in [1, 2]
            const uint32_t colk = (uint32_t)(16 * kh);  // 16 fp32 cells = 16 columns
            tmem_st16(a_col(ts, 0) + lane_off + colk, xl);
            tmem_st16(a_col(ts, 1) + lane_off + colk, ph);
            tmem_st16(a_col(ts, 2) + lane_off + colk, pl);
            tmem_wait_st();
            fence_proxy_async_smem();  // the in-place x_hi (and B tile) are read by the tensor core
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sh->aready[ts]);
        }
        if (!ok) {
            sh->err = 1;
            if (lane == 0 && a.status) atomicOr(a.status, 2);
        }
        if (MASKB && qt == 0 && lb < a.B) {  // first query tile of the first layer
            // mask areas (the count pass's other output): the eight lanes of a
            // GT row sum their bytes, one atomic per row, the image's own rows
            // only (the box's rows past GT_total are the next image's)
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {
                int v = area[h2];
#pragma unroll
                for (int o = 4; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
                const int n = ((warp * 32 + lane) >> 3) + 32 * h2;
                if ((lane & 7) == 0 && n < NG && v > 0)
                    atomicAdd(const_cast<int32_t*>(a.totals) + (int64_t)b * NG + n, v);
            }
        }
        // ---- epilogue (as dense_mma_kernel): row sums, then D and I from TMEM ----
        if (kh == 1) {
#pragma unroll
            for (int i = 0; i < 3; ++i) sh->rows[warp & 3][lane][i] = rsum[i];
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kMmaProducers * 32) : "memory");
        const bool have_acc = ok && nkb > 0 && mbar_wait(&sh->accf, 0u);
        tc_fence_after();
        float* part = a.part + ((((int64_t)lb * a.nqt + qt) * a.nchunk + chunk) * 2 + half) *
                                   (int64_t)a.part_stride;
        const int QP = a.qrows_pad;
        const uint32_t acc_base = tbase + lane_off + (kh ? (uint32_t)N : 0u);
        for (int c0a = 0; c0a < N; c0a += 16) {
            uint32_t v[16];
            if (have_acc) {
                tmem_ld16(acc_base + (uint32_t)c0a, v);
                tmem_wait_ld();
            } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) v[j] = 0u;
            }
            if (rvalid) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int ga = c0a + j;
                    if (ga < NG && ga != a.bg) {
                        const int g = ga - (ga > a.bg ? 1 : 0);
                        const float val = __uint_as_float(v[j]);
                        part[((int64_t)kh * G + g) * QP + r] = kh ? val : -val;
                    }
                }
            }
        }
        if (kh == 0 && rvalid) {
#pragma unroll
            for (int i = 0; i < 3; ++i)
                part[(int64_t)2 * G * QP + (int64_t)i * QP + r] = rsum[i] + sh->rows[warp & 3][lane][i];
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == kMmaProducers) {
        tc_fence_after();
        tmem_dealloc(tbase, kMmaTmemCols);
    }
}

int dense_mma_n(int gt_total) { return (gt_total + 15) / 16 * 16; }

bool dense_mma_usable(const CostArgs& a, int ldt, bool unc, bool foc, bool tma) {
    (void)ldt;
    const int HW = a.H * a.W;
    return !unc && !foc && tma && a.gout > 0 && dense_mma_n(a.gt_total) <= 64 && a.qrows <= 128 &&
           a.chunk_cells % (2 * kMmaK) == 0 && HW % 8 == 0;  // counts rows: 16-byte pitch
}

size_t dense_mma_smem(const CostArgs& a, int esize, bool ax, bool masks_b) {
    const int N = dense_mma_n(a.gt_total);
    const int QS = ax ? 128 : (a.qrows + 7) / 8 * 8;
    const size_t bstage = ((size_t)N * 64 + 1023) / 1024 * 1024;
    const size_t mstage = masks_b ? ((size_t)N * 32 + 127) / 128 * 128 : 0;
    return 1024 + kTmaStages * bstage + (size_t)kTmaStages * QS * kMmaK * esize + kTmaStages * mstage +
           sizeof(MmaShared);
}

template <typename T, bool MASKB>
cudaError_t launch_dense_mma_t(const CUtensorMap& tm, const CUtensorMap& km, const CostArgs& a,
                               cudaStream_t st) {
    const int N = dense_mma_n(a.gt_total);
    const size_t smem = dense_mma_smem(a, (int)sizeof(T), std::is_same<T, __nv_bfloat16>::value, MASKB);
    cudaError_t e = cudaFuncSetAttribute(dense_mma_kernel<T, MASKB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 g(a.nchunk * 2, a.nqt, a.L * a.B);
    dense_mma_kernel<T, MASKB><<<g, kMmaThreads, smem, st>>>(tm, km, a, N);
    return cudaGetLastError();
}

bool dense_mma_tf32_usable(const CostArgs& a, int ldt) {
    return ldt == 0 && dense_mma_n(a.gt_total) <= 64;
}

cudaError_t launch_dense_mma_tf32(const CUtensorMap& tm, const CUtensorMap& km, const CostArgs& a,
                                  cudaStream_t st, bool masks_b) {
    const int N = dense_mma_n(a.gt_total);
    const size_t bstage = ((size_t)N * 128 + 1023) / 1024 * 1024;
    const size_t mstage = masks_b ? ((size_t)N * 32 + 127) / 128 * 128 : 0;
    const size_t smem = 1024 + kTmaStages * ((size_t)128 * kMmaK * 4 + bstage + mstage) + sizeof(MmaShared);
    // two TMEM operand stages while 2N + 2 x 96 columns fit in 256 (N <= 32),
    // else one (the producers then wait for the previous block's MMAs)
    auto k = N <= 32 ? (masks_b ? dense_mma_tf32_kernel<true, 2> : dense_mma_tf32_kernel<false, 2>)
                     : (masks_b ? dense_mma_tf32_kernel<true, 1> : dense_mma_tf32_kernel<false, 1>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    dim3 g(a.nchunk * 2, a.nqt, a.L * a.B);
    k<<<g, kMmaThreads, smem, st>>>(tm, km, a, N);
    return cudaGetLastError();
}

cudaError_t launch_dense_mma(const CUtensorMap& tm, const CUtensorMap& km, const CostArgs& a,
                             cudaStream_t st, int ldt, bool masks_b) {
    if (ldt == 1)
        return masks_b ? launch_dense_mma_t<__nv_bfloat16, true>(tm, km, a, st)
                       : launch_dense_mma_t<__nv_bfloat16, false>(tm, km, a, st);
    if (masks_b) return cudaErrorInvalidValue;  // bf16 logits only
    if (ldt == 2) return launch_dense_mma_t<__half, false>(tm, km, a, st);
    return launch_dense_mma_t<float, false>(tm, km, a, st);
}

}  // namespace mlb
