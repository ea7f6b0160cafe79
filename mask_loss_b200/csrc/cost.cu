// cost.cu -- pairwise matching costs (sigmoid-CE, dice, label) for one batch.
//
// Replaces pairwise_mask_loss_forward (src/cuda/pw_mask.cu:314-501) and the
// label-cost kernels (src/cuda/pw_softmax_label_loss.cu:12-103,
// src/cuda/pw_sigmoid_label_loss.cu:16-106).
//
// Shape of the work.  For image b and query q the costs need, per GT column
// g, the contractions  D[q,g] = sum_j dlt(x_qj) k_jg,  I[q,g] = sum_j w p k_jg,
// T[q,g] = sum_j w k_jg  over the low-res cells j, where k_jg counts the
// high-res pixels of cell j that carry label g (src/cuda/utils.cuh:6-36), plus
// per-query row sums.  With s = H_t/H = 1 (and for every "pure" cell when
// s > 1) k is one-hot, so the contraction is a segmented sum over the cell
// stream: every query of a CTA walks the SAME label sequence, so label runs
// are uniform across the CTA and each thread (one query) accumulates a run in
// registers and flushes it to a per-thread column of shared-memory bins only
// when the label changes.  Mixed cells (s > 1 on a label boundary) add their
// per-pixel counts directly.  Logits stream through a 4-stage TMA pipeline
// (cp.async.bulk.tensor, 128-byte swizzle, conflict-free LDS.128), each read
// from HBM exactly once.
//
// The HW axis is split into chunks across CTAs (grid.x) to fill the 148 SMs;
// chunk partials are reduced in fixed order by cost_finalize_kernel, so the
// costs are deterministic run to run.
#include <cuda.h>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

// ---------------------------------------------------------------------------
// Per-image label histogram: totals[b, lab] for lab in [0, GT_total).
// Same counts as counts.sum({2,3}) in src/cuda/pw_mask.cu:391.
// ---------------------------------------------------------------------------
__global__ void label_hist_kernel(const int64_t* __restrict__ targets, int64_t npix,
                                  int gt_total, int32_t* __restrict__ totals) {
    extern __shared__ int32_t sh[];
    const int b = blockIdx.y;
    const bool use_sh = gt_total <= kHistSmemMax;
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x) sh[i] = 0;
    __syncthreads();
    const int64_t* t = targets + (int64_t)b * npix;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < npix;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t lab = t[i];
        if (lab >= 0 && lab < gt_total) {
            if (use_sh) atomicAdd(&sh[lab], 1);
            else atomicAdd(&totals[(int64_t)b * gt_total + lab], 1);
        }
    }
    __syncthreads();
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x)
            if (sh[i]) atomicAdd(&totals[(int64_t)b * gt_total + i], sh[i]);
}

// ---------------------------------------------------------------------------
// Cell codes for one tile of KC cells: pure column (>= 0, local to the
// column range [g0, g0+gp)), kNone, or kMixed with the s*s per-pixel local
// columns in `mix` (s > 1 only).
// ---------------------------------------------------------------------------
ML_INLINE void tile_codes(const int64_t* __restrict__ tb, int cell0, int nvalid, int W, int Wt,
                          int s, int gt_total, int bg, int g0, int gp, int* code, int16_t* mix,
                          int tid, int nthreads) {
    const int s2 = s * s;
    for (int k = tid; k < KC; k += nthreads) {
        int c = kNone;
        if (k < nvalid) {
            const int cell = cell0 + k;
            const int ci = cell / W, cj = cell - ci * W;
            if (s == 1) {
                int col = label_to_col(tb[cell], gt_total, bg) - g0;
                c = (col >= 0 && col < gp) ? col : kNone;
            } else {
                const int64_t* row0 = tb + (int64_t)(ci * s) * Wt + (int64_t)cj * s;
                int first = -3;
                bool pure = true;
                for (int dy = 0; dy < s; ++dy)
                    for (int dx = 0; dx < s; ++dx) {
                        int col = label_to_col(row0[(int64_t)dy * Wt + dx], gt_total, bg) - g0;
                        col = (col >= 0 && col < gp) ? col : kNone;
                        mix[k * s2 + dy * s + dx] = (int16_t)col;
                        if (first == -3) first = col;
                        else if (col != first) pure = false;
                    }
                c = pure ? first : kMixed;
            }
        }
        code[k] = c;
    }
}

// ---------------------------------------------------------------------------
// The streaming cost kernel.  grid = (nchunk, nqt * ngr, L*B); block = QT
// threads, thread t <-> query row q = qt*qrows + t.  Template flags:
//   UNC   entropy weights on (uncertainty_gamma != 0)
//   FOC   focal gamma/alpha on the mask BCE
//   TMA   logits rows are 16-byte strided so the tensor-map path is legal
// ---------------------------------------------------------------------------
template <bool UNC, bool FOC, bool TMA>
__global__ void __launch_bounds__(256)
cost_partial_kernel(const __grid_constant__ CUtensorMap tmap, CostArgs a) {
    constexpr int NACC = UNC ? 3 : 2;
    constexpr int NROW = UNC ? 5 : 2;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // layout: [stages][qrows_pad][32 floats] swizzled | bins | codes | mix | bars
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int QT = blockDim.x;
    float* stage = reinterpret_cast<float*>(base);
    const int stage_floats = a.qrows_pad * KC;
    float* bins = stage + kStages * stage_floats;           // [NACC][gp][QT]
    int* codes = reinterpret_cast<int*>(bins + NACC * a.gp * QT);  // [2][KC]
    int16_t* mix = reinterpret_cast<int16_t*>(codes + 2 * KC);     // [2][KC*s2]
    const int s2 = a.s * a.s;
    uint64_t* bars = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(mix + 2 * KC * s2) + 7) & ~uintptr_t(7));

    const int t = threadIdx.x;
    const int lb = blockIdx.z;
    const int b = lb % a.B;
    const int qt = blockIdx.y % a.nqt;
    const int gr = blockIdx.y / a.nqt;
    const int g0 = gr * a.gp;
    const int q = qt * a.qrows + t;
    const bool qvalid = (t < a.qrows) && (q < a.Q);
    const int HW = a.H * a.W;
    const int cell_begin = blockIdx.x * a.chunk_cells;
    const int cell_end = min(HW, cell_begin + a.chunk_cells);
    const int ntiles = (cell_end - cell_begin + KC - 1) / KC;
    const int64_t row0 = ((int64_t)lb * a.Q) + qt * a.qrows;  // first global logits row
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;

    for (int i = 0; i < NACC * a.gp; ++i) bins[i * QT + t] = 0.0f;

    const uint32_t stage_bytes = (uint32_t)a.qrows * KC * 4u;
    if (TMA) {
        if (t == 0) {
            for (int i = 0; i < kStages; ++i) mbar_init(&bars[i], 1);
            fence_mbar_init();
        }
        __syncthreads();
        if (t == 0) {
            for (int i = 0; i < kStages - 1 && i < ntiles; ++i) {
                mbar_arrive_expect_tx(&bars[i], stage_bytes);
                const int cx = cell_begin + i * KC;
                asm volatile(
                    "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                    " [%0], [%1, {%2, %3}], [%4];"
                    ::"r"(smem_u32(stage + i * stage_floats)), "l"(&tmap), "r"(cx),
                      "r"((int)row0), "r"(smem_u32(&bars[i])) : "memory");
            }
        }
    }

    float racc[NACC];
#pragma unroll
    for (int i = 0; i < NACC; ++i) racc[i] = 0.0f;
    float rows[NROW];
#pragma unroll
    for (int i = 0; i < NROW; ++i) rows[i] = 0.0f;
    int cur = kNone;
    const float N2 = (float)s2;
    const Focal foc = make_focal(a.mask_gamma, a.mask_alpha);
    bool ok = true;

    auto flush = [&](int col) {
        if (col >= 0) {
#pragma unroll
            for (int i = 0; i < NACC; ++i) {
                bins[(i * a.gp + col) * QT + t] += racc[i] * N2;
                racc[i] = 0.0f;
            }
        }
    };

    for (int it = 0; it < ntiles; ++it) {
        const int st = it % kStages;
        const int cell0 = cell_begin + it * KC;
        const int nvalid = min(KC, cell_end - cell0);
        float* sx = stage + st * stage_floats;
        if (TMA) {
            if (!mbar_wait(&bars[st], (uint32_t)((it / kStages) & 1))) ok = false;
        } else {
            // plain loads into the same swizzled layout
            if (qvalid) {
                const float* src = a.logits + (row0 + t) * (int64_t)HW + cell0;
                for (int c = 0; c < KC / 4; ++c) {
                    float4 v;
                    float* vv = reinterpret_cast<float*>(&v);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const int k = c * 4 + u;
                        vv[u] = (k < nvalid) ? src[k] : 0.0f;
                    }
                    *reinterpret_cast<float4*>(sx + t * KC + ((c ^ (t & 7)) << 2)) = v;
                }
            }
        }
        int* code = codes + (it & 1) * KC;
        int16_t* mx = mix + (it & 1) * KC * s2;
        tile_codes(tb, cell0, nvalid, a.W, a.Wt, a.s, a.gt_total, a.bg, g0, a.gp, code, mx, t, QT);
        __syncthreads();
        if (TMA && t == 0 && it + kStages - 1 < ntiles) {
            const int nit = it + kStages - 1;
            const int nst = nit % kStages;
            mbar_arrive_expect_tx(&bars[nst], stage_bytes);
            asm volatile(
                "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                " [%0], [%1, {%2, %3}], [%4];"
                ::"r"(smem_u32(stage + nst * stage_floats)), "l"(&tmap),
                  "r"(cell_begin + nit * KC), "r"((int)row0), "r"(smem_u32(&bars[nst]))
                : "memory");
        }
        if (t < a.qrows) {
            float trow[NROW];
#pragma unroll
            for (int i = 0; i < NROW; ++i) trow[i] = 0.0f;
            const float* rowp = sx + t * KC;
#pragma unroll 2
            for (int c = 0; c < KC / 4; ++c) {
                const float4 v = *reinterpret_cast<const float4*>(rowp + ((c ^ (t & 7)) << 2));
                const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int k = c * 4 + u;
                    if (k >= nvalid) break;
                    const float x = xs[u];
                    const Elem e = elem(x);
                    const float w = UNC ? unc_weight(e.p, a.ug, a.ugmin) : 1.0f;
                    const float nt = FOC ? focal_neg(foc, e) : e.neg;
                    float dlt;
                    if (FOC) dlt = w * (focal_pos(foc, e) - nt);
                    else if (UNC) dlt = -w * x;
                    else dlt = -x;  // softplus(-x) - softplus(x) == -x exactly
                    if (UNC) {
                        trow[0] += w * nt; trow[1] += w * e.p; trow[2] += w;
                        trow[3] += nt; trow[4] += e.p;
                    } else {
                        trow[0] += nt; trow[1] += e.p;
                    }
                    const int cc = code[k];
                    if (cc >= kNone) {
                        if (cc != cur) { flush(cur); cur = cc; }
                        if (cc >= 0) {
                            racc[0] += dlt;
                            racc[1] += w * e.p;
                            if (UNC) racc[2] += w;
                        }
                    } else {  // mixed cell: one count per pixel
                        const int16_t* mc = mx + k * s2;
                        for (int pp = 0; pp < s2; ++pp) {
                            const int col = mc[pp];
                            if (col >= 0) {
                                bins[(0 * a.gp + col) * QT + t] += dlt;
                                bins[(1 * a.gp + col) * QT + t] += w * e.p;
                                if (UNC) bins[(2 * a.gp + col) * QT + t] += w;
                            }
                        }
                    }
                }
            }
            flush(cur);  // two-level summation: runs never span tiles
#pragma unroll
            for (int i = 0; i < NROW; ++i) rows[i] += trow[i];
        }
    }

    if (!ok && t == 0) atomicOr(a.status, 2);
    if (!qvalid) return;
    float* out = a.part + ((((int64_t)lb * a.nqt + qt) * a.ngr + gr) * a.nchunk + blockIdx.x) *
                              (int64_t)a.part_stride;
    for (int i = 0; i < NACC * a.gp; ++i) out[i * a.qrows_pad + t] = bins[i * QT + t];
#pragma unroll
    for (int i = 0; i < NROW; ++i) out[(NACC * a.gp + i) * a.qrows_pad + t] = rows[i];
}

// ---------------------------------------------------------------------------
// Finalize: fixed-order reduction of the chunk partials, cost formulas,
// label cost, total cost, and the per-query terms the loss needs.
// grid = (nqt, L*B); block = 256.
// ---------------------------------------------------------------------------
template <bool UNC>
__global__ void __launch_bounds__(256) cost_finalize_kernel(CostArgs a) {
    constexpr int NACC = UNC ? 3 : 2;
    constexpr int NROW = UNC ? 5 : 2;
    extern __shared__ float fsh[];
    const int qt = blockIdx.x;
    const int lb = blockIdx.y;
    const int l = lb / a.B, b = lb % a.B;
    const int nq = min(a.qrows, a.Q - qt * a.qrows);
    if (nq <= 0) return;
    float* rP = fsh;              // P = N2 * sum w p
    float* rWt = rP + a.qrows;    // weight total (normalised)
    float* rBase = rWt + a.qrows; // N2 * sum w neg
    float* rLse = rBase + a.qrows;  // class: lse (softmax) or sum focal-neg (sigmoid)
    const int HW = a.H * a.W;
    const float N2 = (float)(a.s * a.s);
    const int tid = threadIdx.x;

    // rows
    for (int t = tid; t < nq; t += blockDim.x) {
        float r[NROW];
#pragma unroll
        for (int i = 0; i < NROW; ++i) r[i] = 0.0f;
        for (int ch = 0; ch < a.nchunk; ++ch) {
            const float* p = a.part + ((((int64_t)lb * a.nqt + qt) * a.ngr + 0) * a.nchunk + ch) *
                                          (int64_t)a.part_stride;
#pragma unroll
            for (int i = 0; i < NROW; ++i) r[i] += p[(NACC * a.gp + i) * a.qrows_pad + t];
        }
        float base = r[0] * N2, P = r[1] * N2;
        float wt = UNC ? r[2] * N2 : (float)a.Ht * (float)a.Wt;
        if (!a.normalize_uncertainty) wt = (float)a.Ht * (float)a.Wt;
        wt = fmaxf(wt, 1e-12f);
        rP[t] = P; rWt[t] = wt; rBase[t] = base;
        // unmatched-mask terms (src/cuda/mask_matching_forward.cu:122-143,224-235):
        // unweighted BCE mean over HW and empty-mask dice.
        const float su = UNC ? r[3] : r[0];
        const float pu = UNC ? r[4] : r[1];
        const int64_t qi = (int64_t)lb * a.Q + qt * a.qrows + t;
        const float ps = pu * a.area_scale;
        a.qstat[qi * kQStat + 2] = a.sigmoid_scale * (su / (float)HW);
        a.qstat[qi * kQStat + 3] = a.dice_scale * (ps / (ps + a.smooth));
        a.qstat[qi * kQStat + 0] = P;
        a.qstat[qi * kQStat + 1] = wt;
    }

    // class rows: one warp per query
    const int warp = tid >> 5, lane = tid & 31, nw = blockDim.x >> 5;
    const Focal cf = make_focal(a.cls_gamma, a.cls_alpha);
    const bool fwd_sig_focal = !a.use_softmax;  // forward kernel uses focal only for sigmoid
    const Focal uf = make_focal(fwd_sig_focal ? a.cls_gamma : 0.0f, fwd_sig_focal ? a.cls_alpha : -1.0f);
    for (int t = warp; t < nq; t += nw) {
        const int64_t qi = (int64_t)lb * a.Q + qt * a.qrows + t;
        const float* z = a.cls_logits + qi * a.C;
        float m = -INFINITY;
        for (int c = lane; c < a.C; c += 32) m = fmaxf(m, z[c]);
        m = warp_max(m);
        float se = 0.0f, sn = 0.0f, snu = 0.0f;
        for (int c = lane; c < a.C; c += 32) {
            const float zc = z[c];
            se += __expf(zc - m);
            const Elem e = elem(zc);
            sn += focal_neg(cf, e);
            snu += focal_neg(uf, e);
        }
        se = warp_sum(se); sn = warp_sum(sn); snu = warp_sum(snu);
        const float lse = __logf(fmaxf(se, 1e-20f)) + m;
        if (lane == 0) {
            rLse[t] = a.use_softmax ? lse : sn;
            // unmatched class loss (src/cuda/mask_matching_forward.cu:150-276)
            float um = 0.0f;
            if (a.has_void) {
                const float zv = z[a.void_index];
                if (a.use_softmax && a.force_cls) {
                    um = lse - zv;
                } else {
                    const Elem ev = elem(zv);
                    const float vp = focal_pos(uf, ev), vn = focal_neg(uf, ev);
                    um = a.force_cls ? (snu / (float)a.C + (vp - vn) / (float)a.C) : vp;
                }
            } else if (a.force_cls) {
                um = snu / (float)a.C;
            }
            a.qstat[qi * kQStat + 4] = um * a.cls_scale;
        }
    }
    __syncthreads();

    // pairs (q, g)
    const int G = a.gout;
    const int64_t slice = (int64_t)a.L * a.B * a.Q * G;
    for (int i = tid; i < nq * G; i += blockDim.x) {
        const int g = i / nq, t = i - g * nq;
        const int gr = g / a.gp, gl = g - gr * a.gp;
        float acc[NACC];
#pragma unroll
        for (int k = 0; k < NACC; ++k) acc[k] = 0.0f;
        for (int ch = 0; ch < a.nchunk; ++ch) {
            const float* p = a.part + ((((int64_t)lb * a.nqt + qt) * a.ngr + gr) * a.nchunk + ch) *
                                          (int64_t)a.part_stride;
#pragma unroll
            for (int k = 0; k < NACC; ++k) acc[k] += p[(k * a.gp + gl) * a.qrows_pad + t];
        }
        const int ga = g + (g >= a.bg ? 1 : 0);
        const int64_t qi = (int64_t)lb * a.Q + qt * a.qrows + t;
        const int64_t o = qi * G + g;
        const int32_t tc = a.totals[(int64_t)b * a.gt_total + ga];
        const float T = UNC ? acc[2] : (float)tc;
        float bce, dice;
        if (tc == 0) {
            bce = INFINITY; dice = INFINITY;
        } else {
            bce = (rBase[t] + acc[0]) / rWt[t] * a.sigmoid_scale;
            dice = (1.0f - (2.0f * acc[1] + a.smooth) / (rP[t] + T + a.smooth)) * a.dice_scale;
        }
        // label cost
        const int64_t y = a.cls_targets[(int64_t)b * a.gt_total + ga];
        float cls;
        if (y < 0 || y >= a.C) {
            cls = INFINITY;
        } else {
            const float zy = a.cls_logits[qi * a.C + y];
            if (a.use_softmax) {
                cls = (rLse[t] - zy) * a.cls_scale;
            } else {
                const Elem e = elem(zy);
                cls = (rLse[t] + focal_pos(cf, e) - focal_neg(cf, e)) / (float)a.C * a.cls_scale;
            }
        }
        if (a.sep) {
            a.sep[o] = bce;
            a.sep[slice + o] = dice;
            a.sep[2 * slice + o] = cls;
        }
        if (a.total) a.total[o] = (bce + dice) + cls;
        if (a.rawI) { a.rawI[o] = acc[1]; a.rawT[o] = T; }
    }
}

template __global__ void cost_partial_kernel<false, false, true>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, false>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_finalize_kernel<false>(CostArgs);
template __global__ void cost_finalize_kernel<true>(CostArgs);

}  // namespace mlb

namespace mlb {

// Standalone pairwise label cost, one warp per (l,b,q) row
// (src/cuda/pw_softmax_label_loss.cu:12-103, src/cuda/pw_sigmoid_label_loss.cu:16-106).
__global__ void __launch_bounds__(256)
label_cost_kernel(const float* __restrict__ z_all, const int64_t* __restrict__ y_all,
                  float* __restrict__ out, int L, int B, int Q, int C, int gt_total, int bg,
                  int gout, float scale, float gamma, float alpha, int use_softmax) {
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= (int64_t)L * B * Q) return;
    const int b = (int)((row / Q) % B);
    const float* z = z_all + row * C;
    const Focal f = make_focal(gamma, alpha);
    float m = -INFINITY;
    for (int c = lane; c < C; c += 32) m = fmaxf(m, z[c]);
    m = warp_max(m);
    float se = 0.0f, sn = 0.0f;
    for (int c = lane; c < C; c += 32) {
        se += __expf(z[c] - m);
        sn += focal_neg(f, elem(z[c]));
    }
    se = warp_sum(se);
    sn = warp_sum(sn);
    const float lse = __logf(fmaxf(se, 1e-20f)) + m;
    for (int g = lane; g < gout; g += 32) {
        const int ga = g + (g >= bg ? 1 : 0);
        const int64_t y = y_all[(int64_t)b * gt_total + ga];
        float v;
        if (y < 0 || y >= C) {
            v = INFINITY;
        } else if (use_softmax) {
            v = (lse - z[y]) * scale;
        } else {
            const Elem e = elem(z[y]);
            v = (sn + focal_pos(f, e) - focal_neg(f, e)) / (float)C * scale;
        }
        out[row * gout + g] = v;
    }
}

}  // namespace mlb
