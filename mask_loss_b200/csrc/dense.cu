// dense.cu -- matching costs against dense per-GT masks (overlap allowed).
//
// The reference takes a label map only (src/bindings.cpp:66), so every pixel
// belongs to one GT.  Here the targets may also be (B, GT_total, H_t, W_t)
// uint8 masks aligned with cls_targets' columns, possibly overlapping.  The
// costs keep the reference's formulas (src/cuda/pw_mask.cu:290-304) with the
// one-hot count of a cell replaced by each GT's pixel count in the cell; on
// non-overlapping masks the result equals the label-map path.
//
// Two kernels feed the label path's finalize (cost_rows / cost_pairs), the
// solver and the matched loss unchanged:
//   dense_count_kernel  per (image, cell) the pixel count of every GT
//                       (uint16, [b][cell][GT_total]) and per (image, GT) the
//                       mask area (the histogram the label path builds);
//   dense_cost_kernel   per (layer*image, query tile, cell chunk, GT chunk)
//                       the chunk partials in the label path's layout: row
//                       sums, and per GT sum(val * count) accumulated in shared
//                       memory from a per-tile list of the non-zero
//                       (GT, count) pairs of each cell.  Deterministic: every
//                       accumulator has one owner thread.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

namespace {
constexpr int kDenseTile = 32;   // cells per staged tile
constexpr int kDenseGC = 64;     // GT columns per block (grid chunk)
}  // namespace

// grid = (ceil(HW / 256), B), block 256: thread per cell.
__global__ void __launch_bounds__(256)
dense_count_kernel(const uint8_t* __restrict__ masks, int H, int W, int Ht, int Wt, int s,
                   int gt_total, uint16_t* __restrict__ cnt, int32_t* __restrict__ totals) {
    extern __shared__ int32_t area[];  // [gt_total]
    const int b = blockIdx.y;
    const int HW = H * W;
    for (int g = threadIdx.x; g < gt_total; g += blockDim.x) area[g] = 0;
    __syncthreads();
    const int cell = blockIdx.x * blockDim.x + threadIdx.x;
    if (cell < HW) {
        const int ci = cell / W, cj = cell - ci * W;
        uint16_t* out = cnt + ((int64_t)b * HW + cell) * gt_total;
        for (int g = 0; g < gt_total; ++g) {
            const uint8_t* mg = masks + ((int64_t)b * gt_total + g) * Ht * Wt +
                                (int64_t)(ci * s) * Wt + (int64_t)cj * s;
            int n = 0;
            for (int dy = 0; dy < s; ++dy)
                for (int dx = 0; dx < s; ++dx) n += mg[(int64_t)dy * Wt + dx] != 0;
            out[g] = (uint16_t)n;
            if (n) atomicAdd(&area[g], n);
        }
    }
    __syncthreads();
    for (int g = threadIdx.x; g < gt_total; g += blockDim.x)
        if (area[g]) atomicAdd(&totals[(int64_t)b * gt_total + g], area[g]);
}

// grid = (nchunk * ngc, nqt, L*B), block = QP threads (query row t of the tile).
// Dynamic shared memory: see dense_cost_smem.
template <bool UNC, bool FOC>
__device__ __forceinline__ void dense_cost_body(const CostArgs& a, const uint16_t* cnt) {
    constexpr int NACC = UNC ? 3 : 2;
    constexpr int NROW = UNC ? 5 : 3;
    constexpr bool FAST = !UNC && !FOC;
    extern __shared__ __align__(16) float dsh[];
    const int QP = a.qrows_pad, G = a.gout;
    const int ngc = (G + kDenseGC - 1) / kDenseGC;
    const int chunk = blockIdx.x / ngc, gc = blockIdx.x - chunk * ngc;
    const int g0 = gc * kDenseGC, g1 = min(G, g0 + kDenseGC), gn = g1 - g0;
    const int qt = blockIdx.y, lb = blockIdx.z, b = lb % a.B;
    const int t = threadIdx.x;
    const int q = qt * a.qrows + t;
    const bool qvalid = t < a.qrows && q < a.Q;
    const int HW = a.H * a.W;
    const int cell_begin = chunk * a.chunk_cells;
    const int cell_end = min(HW, cell_begin + a.chunk_cells);
    float* xs = dsh;                                         // [QP][kDenseTile + 1]
    float* acc = xs + QP * (kDenseTile + 1);                 // [NACC][kDenseGC][QP]
    int* lcnt = reinterpret_cast<int*>(acc + NACC * kDenseGC * QP);  // [kDenseTile]
    int* lg = lcnt + kDenseTile;                             // [kDenseTile][kDenseGC]
    float* ln = reinterpret_cast<float*>(lg + kDenseTile * kDenseGC);  // [kDenseTile][kDenseGC]
    for (int i = t; i < NACC * kDenseGC * QP; i += blockDim.x) acc[i] = 0.0f;
    const int row0 = lb * a.Q + qt * a.qrows;
    const Focal foc = make_focal(a.mask_gamma, a.mask_alpha);
    float rows[NROW];
#pragma unroll
    for (int i = 0; i < NROW; ++i) rows[i] = 0.0f;
    const int nwarps = blockDim.x >> 5, warp = t >> 5, lane = t & 31;
    for (int c0 = cell_begin; c0 < cell_end; c0 += kDenseTile) {
        const int nv = min(kDenseTile, cell_end - c0);
        __syncthreads();  // previous tile consumed
        // logits tile: warp w loads rows w, w+nwarps, ... (coalesced per row)
        for (int r = warp; r < a.qrows; r += nwarps) {
            const int qq = qt * a.qrows + r;
            float v = 0.0f;
            if (lane < nv && qq < a.Q) v = a.logits[(int64_t)(row0 + r) * HW + c0 + lane];
            xs[r * (kDenseTile + 1) + lane] = v;
        }
        // non-zero (GT, count) list of every cell of the tile
        for (int k = warp; k < nv; k += nwarps) {
            const uint16_t* cc = cnt + ((int64_t)b * HW + c0 + k) * a.gt_total;
            int base = 0;
            for (int j0 = 0; j0 < gn; j0 += 32) {
                const int j = j0 + lane;
                int n = 0;
                if (j < gn) {
                    const int g = g0 + j;
                    n = cc[g + (g >= a.bg ? 1 : 0)];
                }
                const unsigned bal = __ballot_sync(0xffffffffu, n != 0);
                if (n) {
                    const int pos = base + __popc(bal & ((1u << lane) - 1u));
                    lg[k * kDenseGC + pos] = j;
                    ln[k * kDenseGC + pos] = (float)n;
                }
                base += __popc(bal);
            }
            if (lane == 0) lcnt[k] = base;
        }
        __syncthreads();
        if (t < a.qrows) {
            for (int k = 0; k < nv; ++k) {
                const float x = xs[t * (kDenseTile + 1) + k];
                float v[NACC];
                if (FAST) {
                    const float e = ex2_approx(-fabsf(x) * 1.4426950408889634f);
                    const float d = 1.0f + e;
                    const float r = rcp_approx(d);
                    const float p = x >= 0.0f ? r : e * r;
                    rows[0] += fmaxf(x, 0.0f);
                    rows[1] += p;
                    rows[2] += lg2_approx(d);
                    v[0] = -x;
                    v[1] = p;
                } else {
                    const Elem e = elem(x);
                    const float w = UNC ? unc_weight(e.p, a.ug, a.ugmin) : 1.0f;
                    const float nt = FOC ? focal_neg(foc, e) : e.neg;
                    const float dl = FOC ? w * (focal_pos(foc, e) - nt) : -w * x;
                    if (UNC) {
                        rows[0] += w * nt; rows[1] += w * e.p; rows[2] += w;
                        rows[3] += nt; rows[4] += e.p;
                    } else {
                        rows[0] += nt; rows[1] += e.p;
                    }
                    v[0] = dl;
                    v[1] = w * e.p;
                    if (UNC) v[NACC - 1] = w;
                }
                const int m = lcnt[k];
                for (int i = 0; i < m; ++i) {
                    const int j = lg[k * kDenseGC + i];
                    const float n = ln[k * kDenseGC + i];
#pragma unroll
                    for (int z = 0; z < NACC; ++z) acc[(z * kDenseGC + j) * QP + t] += v[z] * n;
                }
            }
        }
    }
    __syncthreads();
    if (!qvalid) return;
    // slot h = 0 carries the chunk, slot h = 1 is cleared (the finalize sums both)
    float* part0 = a.part + (((int64_t)lb * a.nqt + qt) * a.nchunk + chunk) * 2 * (int64_t)a.part_stride;
    float* part1 = part0 + a.part_stride;
    for (int z = 0; z < NACC; ++z)
        for (int j = 0; j < gn; ++j) {
            const int64_t o = ((int64_t)z * G + g0 + j) * QP + t;
            part0[o] = acc[(z * kDenseGC + j) * QP + t];
            part1[o] = 0.0f;
        }
    if (gc == 0) {
#pragma unroll
        for (int i = 0; i < NROW; ++i) {
            const int64_t o = (int64_t)NACC * G * QP + (int64_t)i * QP + t;
            part0[o] = (FAST && i == 2) ? rows[2] : rows[i];
            part1[o] = 0.0f;
        }
    }
}

__global__ void __launch_bounds__(128) dense_cost_kernel(CostArgs a, const uint16_t* cnt) {
    dense_cost_body<false, false>(a, cnt);
}
__global__ void __launch_bounds__(128) dense_cost_unc_kernel(CostArgs a, const uint16_t* cnt) {
    dense_cost_body<true, false>(a, cnt);
}
__global__ void __launch_bounds__(128) dense_cost_foc_kernel(CostArgs a, const uint16_t* cnt) {
    dense_cost_body<false, true>(a, cnt);
}
__global__ void __launch_bounds__(128) dense_cost_unc_foc_kernel(CostArgs a, const uint16_t* cnt) {
    dense_cost_body<true, true>(a, cnt);
}

size_t dense_cost_smem(int qrows_pad, bool unc) {
    const int nacc = unc ? 3 : 2;
    return sizeof(float) * ((size_t)qrows_pad * (kDenseTile + 1) + (size_t)nacc * kDenseGC * qrows_pad) +
           sizeof(int) * (kDenseTile + (size_t)kDenseTile * kDenseGC) +
           sizeof(float) * (size_t)kDenseTile * kDenseGC;
}

cudaError_t launch_dense_count(const uint8_t* masks, int B, int H, int W, int Ht, int Wt, int s,
                               int gt_total, uint16_t* cnt, int32_t* totals, cudaStream_t st) {
    const int HW = H * W;
    dim3 g((HW + 255) / 256, B);
    dense_count_kernel<<<g, 256, sizeof(int32_t) * (size_t)std::max(gt_total, 1), st>>>(
        masks, H, W, Ht, Wt, s, gt_total, cnt, totals);
    return cudaGetLastError();
}

cudaError_t launch_dense_cost(const CostArgs& a, bool unc, bool foc, const uint16_t* cnt,
                              cudaStream_t st) {
    const size_t smem = dense_cost_smem(a.qrows_pad, unc);
    const int ngc = (a.gout + kDenseGC - 1) / kDenseGC;
    dim3 g(a.nchunk * ngc, a.nqt, a.L * a.B);
    auto k = unc ? (foc ? dense_cost_unc_foc_kernel : dense_cost_unc_kernel)
                 : (foc ? dense_cost_foc_kernel : dense_cost_kernel);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<g, a.qrows_pad, smem, st>>>(a, cnt);
    return cudaGetLastError();
}

}  // namespace mlb
