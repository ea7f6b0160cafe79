// loss.cu -- matched-loss forward and the backward of the matching loss.
//
// Forward: replaces mask_matching_forward (src/cuda/mask_matching_forward.cu:
// 21-586).  The matched terms are gathered from the cost slices (the
// reference does the same with float atomics, :63-71); the unmatched terms
// were already reduced per query by cost_finalize_kernel, so this kernel
// touches only O(L*B*Q) numbers.  Sums use a fixed-order block reduction, so
// the layer means are deterministic.
//
// Backward: replaces mask_matching_backward (src/cuda/mask_matching_backward.cu:
// 21-621).  With the forward's saved per-query statistics the mask gradient is
// a single streaming pass: read the matched rows' logits once (four values
// per access), write the gradient once (rows the loss does not reach are
// pure streaming stores of zeros).  The matched label's pixel count per cell
// comes from the label map directly for s = 1 (16-byte label loads) and from
// the per-cell codes plus the mixed-cell table for s > 1.  Without the
// statistics (the standalone binding call) a statistics pass re-reads the
// logits first, like the reference.  Logits and gradient are fp32, bf16 or
// fp16 (template T / LT); arithmetic is fp32.
#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

// ---------------------------------------------------------------------------
// Block-wide fixed-order sum of NV values per thread (blockDim.x <= 1024).
// ---------------------------------------------------------------------------
template <int NV>
ML_INLINE void block_sum(float (&v)[NV], float* sh /* [32*NV] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = warp_sum(v[i]);
    __syncthreads();
    if (lane == 0)
#pragma unroll
        for (int i = 0; i < NV; ++i) sh[warp * NV + i] = v[i];
    __syncthreads();
    if (warp == 0) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            float x = lane < nw ? sh[lane * NV + i] : 0.0f;
            v[i] = warp_sum(x);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0)
#pragma unroll
        for (int i = 0; i < NV; ++i) sh[i] = v[i];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = sh[i];
    __syncthreads();
}

// Denominators (src/cuda/mask_matching_forward.cu:549-578 and
// src/cuda/mask_matching_backward.cu:483-508).
ML_INLINE void denominators(const LossArgs& a, float matched, float* md, float* cd) {
    const float tot = (float)a.B * (float)a.Q;
    float nm = a.num_masks_dev ? *a.num_masks_dev : a.num_masks;
    const bool has_nm = nm > 0.0f;
    float m = a.force_masks ? tot : (has_nm ? nm : matched);
    float c = (a.force_cls || a.has_void) ? tot : (has_nm ? nm : matched);
    *md = fmaxf(m, 1.0f);
    *cd = fmaxf(c, 1.0f);
}

// ---------------------------------------------------------------------------
// Forward: grid = L, block = 1024.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) loss_fwd_kernel(LossArgs a) {
    pdl_enter();
    __shared__ float sh[32 * 4];
    const int l = blockIdx.x;
    if (a.void_status && l == 0) {  // functions/mask/matching.py:180-181
        bool hit = false;
        for (int i = threadIdx.x; i < a.B * a.gt_total; i += blockDim.x)
            hit |= a.cls_targets[i] == (int64_t)a.void_index;
        if (__any_sync(0xffffffffu, hit) && (threadIdx.x & 31) == 0) atomicOr(a.void_status, 4);
    }
    if (a.auto_num_masks) {
        // num_masks = present non-background GT ids of this batch, clamped >= 1;
        // block 0 publishes it for the backward
        float c[1] = {0.0f};
        for (int i = threadIdx.x; i < a.B * a.gt_total; i += blockDim.x)
            if (i % a.gt_total != a.bg && a.totals[i] > 0) c[0] += 1.0f;
        block_sum<1>(c, sh);
        a.num_masks = fmaxf(c[0], 1.0f);
        if (l == 0 && threadIdx.x == 0 && a.num_masks_out) *a.num_masks_out = a.num_masks;
        a.num_masks_dev = nullptr;
    }
    const int n = a.B * a.Q;
    const int64_t G = a.G;
    const int64_t slice = (int64_t)a.L * a.B * a.Q * G;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};  // mask, dice, cls, matched
    const bool need_cls = a.force_cls || a.has_void;
    // rows in pairs: both assignments load before either row's gathers, so
    // each thread has two dependent load chains in flight
    auto row = [&](int64_t qi, int64_t g) {
        const float* qs = a.qstat + qi * kQStat;
        float sv[kSaved] = {qs[0], 0.0f, 0.0f, qs[1]};
        if (g >= 0) {
            const int64_t o = qi * G + g;
            acc[0] += a.sep[o];
            acc[1] += a.sep[slice + o];
            acc[2] += a.sep[2 * slice + o];
            acc[3] += 1.0f;
            sv[1] = a.rawT[o];
            sv[2] = a.rawI[o];
        } else {
            if (a.force_masks) { acc[0] += qs[2]; acc[1] += qs[3]; }
            if (need_cls) acc[2] += qs[4];
        }
        if (a.saved)
#pragma unroll
            for (int k = 0; k < kSaved; ++k) a.saved[qi * kSaved + k] = sv[k];
    };
    for (int i = threadIdx.x; i < n; i += 2 * blockDim.x) {
        const int i2 = i + blockDim.x;
        const int64_t q1 = (int64_t)l * n + i, q2 = (int64_t)l * n + i2;
        const int64_t g1 = a.pred_to_gt[q1];
        const int64_t g2 = i2 < n ? a.pred_to_gt[q2] : -1;
        row(q1, g1);
        if (i2 < n) row(q2, g2);
    }
    block_sum<4>(acc, sh);
    if (threadIdx.x == 0) {
        float md, cd;
        denominators(a, acc[3], &md, &cd);
        a.layer_means[l] = acc[0] / md;
        a.layer_means[a.L + l] = acc[1] / md;
        a.layer_means[2 * a.L + l] = acc[2] / cd;
    }
}

// Sum of present, non-background GT columns over the batch (num_masks).
__global__ void count_masks_kernel(const int32_t* totals, int B, int gt_total, int bg, float* out) {
    __shared__ float sh[32];
    float v[1] = {0.0f};
    for (int i = threadIdx.x; i < B * gt_total; i += blockDim.x) {
        const int g = i % gt_total;
        if (g != bg && totals[i] > 0) v[0] += 1.0f;
    }
    block_sum<1>(v, sh);
    if (threadIdx.x == 0) *out = v[0];
}

// Count of pixels labelled `ga` in low-res cell `cell` (s x s block).
ML_INLINE float cell_count(const int64_t* tb, int cell, int W, int Wt, int s, int64_t ga) {
    const int ci = cell / W, cj = cell - ci * W;
    const int64_t* r0 = tb + (int64_t)(ci * s) * Wt + (int64_t)cj * s;
    int c = 0;
    for (int dy = 0; dy < s; ++dy)
        for (int dx = 0; dx < s; ++dx) c += r0[(int64_t)dy * Wt + dx] == ga;
    return (float)c;
}

// The same count from the per-cell codes of the image (codes_b) and its
// mixed-cell table (mix_b): a pure cell is all or nothing, a mixed cell reads
// its table entry, and a wide cell falls back to the label map.  `gcol` is the
// output column of label `ga`.
ML_INLINE float cell_count_coded(const int32_t* codes_b, const uint4* mix_b, const int64_t* tb,
                                 int cell, int W, int Wt, int s, int64_t ga, int gcol, float N2) {
    const int code = codes_b[cell];
    if (code != kMixed) return code == gcol ? N2 : 0.0f;
    const uint4 e = mix_b[cell];
    if (e.x != kMixWide) return mix_count(e, gcol);
    return cell_count(tb, cell, W, Wt, s, ga);
}

// ---------------------------------------------------------------------------
// Statistics pass for the standalone backward (no saved statistics):
// grid = (Q, L*B), block = 256.  Mirrors the first loop of
// src/cuda/mask_matching_backward.cu:110-138 with a fixed-order reduction.
// ---------------------------------------------------------------------------
template <bool UNC, typename T>
__global__ void __launch_bounds__(256) bwd_stats_kernel(LossArgs a) {
    __shared__ float sh[32 * 4];
    const int q = blockIdx.x, lb = blockIdx.y, b = lb % a.B;
    const int64_t qi = (int64_t)lb * a.Q + q;
    const int64_t og = a.pred_to_gt[qi];
    const int64_t ga = og + (og >= a.bg ? 1 : 0);
    const bool matched = og >= 0 && ga < a.gt_total;
    if (!matched && !a.force_masks) return;
    const int HW = a.H * a.W;
    const float N2 = (float)(a.s * a.s);
    const T* x = reinterpret_cast<const T*>(a.mask_logits) + qi * HW;
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;
    const int32_t* codes_b = a.codes ? a.codes + (int64_t)b * HW : nullptr;
    const uint4* mix_b = a.codes ? a.mixtab + (int64_t)b * HW : nullptr;
    const int gcol = matched ? label_to_col(ga, a.gt_total, a.bg) : kNone;
    float v[4] = {0.f, 0.f, 0.f, 0.f};  // sum w p, sum w t, sum w p t, sum w
    for (int j = threadIdx.x; j < HW; j += blockDim.x) {
        const Elem e = elem(to_f(x[j]));
        const float w = UNC ? unc_weight(e.p, a.ug, a.ugmin) : 1.0f;
        const float t = !matched ? 0.0f
                        : codes_b ? cell_count_coded(codes_b, mix_b, tb, j, a.W, a.Wt, a.s, ga, gcol, N2)
                                  : cell_count(tb, j, a.W, a.Wt, a.s, ga);
        v[0] += w * e.p; v[1] += w * t; v[2] += w * e.p * t; v[3] += w;
    }
    block_sum<4>(v, sh);
    if (threadIdx.x == 0) {
        float wt = a.normalize_uncertainty ? v[3] * N2 : N2 * (float)HW;
        wt = fmaxf(wt, 1e-12f);
        float* o = a.stats_out + qi * kSaved;
        o[0] = v[0] * N2; o[1] = v[1]; o[2] = v[2]; o[3] = wt;
    }
}

// ---------------------------------------------------------------------------
// Mask-logit gradient: grid = (L*B*Q, nchunk), block = 256; a block owns one
// query row and a contiguous range of chunk_cells cells.  Rows the loss does
// not reach are pure 128-bit streaming stores of zeros (memset speed); the
// matched (or forced) rows read logits and labels and write the gradient of
// src/cuda/mask_matching_backward.cu:169-215.
// ---------------------------------------------------------------------------
template <bool UNC, bool FOC, bool VEC, typename LT>
__global__ void __launch_bounds__(256) mask_grad_kernel(LossArgs a) {
    pdl_enter();
    const int64_t qi = blockIdx.x;
    const int lb = (int)(qi / a.Q), l = lb / a.B, b = lb % a.B;
    const int HW = a.H * a.W;
    const int c0 = blockIdx.y * a.chunk_cells;
    const int nc = min(a.chunk_cells, HW - c0);
    LT* gout = reinterpret_cast<LT*>(a.grad_mask_logits) + qi * HW + c0;
    const float mcoef = a.coef[l * 3 + 0], dcoef = a.coef[l * 3 + 1];
    const int64_t og = a.pred_to_gt[qi];
    const int64_t ga = og + (og >= a.bg ? 1 : 0);
    const bool matched = og >= 0 && ga < a.gt_total;
    const bool active = (matched || a.force_masks) && !(mcoef == 0.0f && dcoef == 0.0f);
    if (!active) {
        if (a.rows_zeroed) return;  // the caller zeroed the gradient beforehand
        if (VEC) {
            const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k = threadIdx.x * 4; k < nc; k += blockDim.x * 4) st4cs(gout + k, z);
        } else {
            for (int k = threadIdx.x; k < nc; k += blockDim.x) gout[k] = from_f<LT>(0.0f);
        }
        return;
    }
    const LT* xin = reinterpret_cast<const LT*>(a.mask_logits) + qi * HW + c0;
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;
    const int s = a.s;
    const float N2 = (float)(s * s);
    const Focal f = make_focal(a.mask_gamma, a.mask_alpha);
    const float* sv = a.stats_in + qi * kSaved;
    const float P = sv[0], T = matched ? sv[1] : 0.0f, I = matched ? sv[2] : 0.0f, Wt = sv[3];
    const float sf = a.sigmoid_scale / Wt;
    const float den = P + T + a.smooth;
    const float num = 2.0f * I + a.smooth;
    const float inv_d2 = 1.0f / fmaxf(den * den, 1e-20f);
    const float two_den = 2.0f * den;
    // dense targets: the matched GT's own mask
    const uint8_t* mb = (a.masks && matched) ? a.masks + ((int64_t)b * a.gt_total + ga) * a.Ht * a.Wt
                                             : nullptr;
    const int32_t* codes_b = a.codes ? a.codes + (int64_t)b * HW : nullptr;
    const uint4* mix_b = a.codes ? a.mixtab + (int64_t)b * HW : nullptr;
    const int gcol = matched ? label_to_col(ga, a.gt_total, a.bg) : kNone;
    auto count = [&](int k) -> float {  // pixels of the matched label in cell c0 + k
        if (!matched) return 0.0f;
        if (mb) {
            if (s == 1) return mb[c0 + k] != 0 ? 1.0f : 0.0f;
            const int cell = c0 + k, ci = cell / a.W, cj = cell - ci * a.W;
            const uint8_t* r0 = mb + (int64_t)(ci * s) * a.Wt + (int64_t)cj * s;
            int n = 0;
            for (int dy = 0; dy < s; ++dy)
                for (int dx = 0; dx < s; ++dx) n += r0[(int64_t)dy * a.Wt + dx] != 0;
            return (float)n;
        }
        if (s == 1) return tb[c0 + k] == ga ? 1.0f : 0.0f;
        if (codes_b) return cell_count_coded(codes_b, mix_b, tb, c0 + k, a.W, a.Wt, s, ga, gcol, N2);
        return cell_count(tb, c0 + k, a.W, a.Wt, s, ga);
    };
    auto g1 = [&](float x, float t) -> float {
        const Elem e = elem(x);
        const float om = 1.0f - e.p, pp = e.p * om;
        const float w = UNC ? unc_weight(e.p, a.ug, a.ugmin) : 1.0f;
        const float ncnt = fmaxf(N2 - t, 0.0f);
        float gs;
        if (FOC) {
            const float mp = f.use_gamma ? __powf(om, f.gamma) : 1.0f;
            const float mn = f.use_gamma ? __powf(e.p, f.gamma) : 1.0f;
            const float gpos = -w * f.alpha_pos * t * mp * (f.gamma * e.p * e.pos + om);
            const float gneg = w * f.alpha_neg * ncnt * mn * (f.gamma * om * e.neg + e.p);
            gs = (gpos + gneg) * sf;
        } else {
            gs = (w * (ncnt * e.p - t * om)) * sf;
        }
        const float gd = (num * (w * pp * N2) - two_den * (w * pp * t)) * inv_d2 * a.dice_scale;
        return mcoef * gs + dcoef * gd;
    };
    if (VEC) {
        // one pixel per cell and 16-byte aligned labels: the four labels of a
        // float4 are two 16-byte loads, issued with the logits
        const bool lab2 = s == 1 && matched && !a.masks && ((reinterpret_cast<uintptr_t>(tb + c0) & 15) == 0);
        if (lab2) {
            const LT* __restrict__ xr = xin;
            const longlong2* __restrict__ lr = reinterpret_cast<const longlong2*>(tb + c0);
            LT* __restrict__ gr = gout;
#pragma unroll 4
            for (int k = threadIdx.x * 4; k < nc; k += blockDim.x * 4) {
                const float4 xv = ld4cs(xr + k);
                const longlong2 l01 = lr[k >> 1], l23 = lr[(k >> 1) + 1];
                float4 r;
                r.x = g1(xv.x, l01.x == ga ? 1.0f : 0.0f);
                r.y = g1(xv.y, l01.y == ga ? 1.0f : 0.0f);
                r.z = g1(xv.z, l23.x == ga ? 1.0f : 0.0f);
                r.w = g1(xv.w, l23.y == ga ? 1.0f : 0.0f);
                st4cs(gr + k, r);
            }
            return;
        }
        for (int k = threadIdx.x * 4; k < nc; k += blockDim.x * 4) {
            const float4 xv = ld4cs(xin + k);
            float4 r;
            r.x = g1(xv.x, count(k));
            r.y = g1(xv.y, count(k + 1));
            r.z = g1(xv.z, count(k + 2));
            r.w = g1(xv.w, count(k + 3));
            st4cs(gout + k, r);
        }
    } else {
        for (int k = threadIdx.x; k < nc; k += blockDim.x) gout[k] = from_f<LT>(g1(to_f(xin[k]), count(k)));
    }
}

// ---------------------------------------------------------------------------
// Class-logit gradient of one (l,b,q) row by one warp; `base` = the layer's
// class coefficient.  src/cuda/mask_matching_backward.cu:218-376.  Every
// element is written.
// ---------------------------------------------------------------------------
ML_INLINE void cls_grad_row(const LossArgs& a, int64_t qi, int lane, float base) {
    const int b = (int)((qi / a.Q) % a.B);
    const int C = a.C;
    const float* z = a.cls_logits + qi * C;
    float* gz = a.grad_cls_logits + qi * C;
    const int64_t og = a.pred_to_gt[qi];
    const int64_t ga = og + (og >= a.bg ? 1 : 0);
    const bool matched = og >= 0 && ga < a.gt_total;
    const bool need = a.force_cls || a.has_void;
    int y = -1;
    bool zero = !(matched || need) || base == 0.0f;
    if (!zero && matched) {
        const int64_t y64 = a.cls_targets[(int64_t)b * a.gt_total + ga];
        if (y64 < 0 || y64 >= C) zero = true;
        else y = (int)y64;
    }
    if (zero) {
        for (int c = lane; c < C; c += 32) gz[c] = 0.0f;
        return;
    }
    const float invC = 1.0f / (float)C;
    if (a.use_softmax) {
        if (matched || (a.force_cls && a.has_void)) {
            const int ti = matched ? y : a.void_index;
            float m = -INFINITY;
            for (int c = lane; c < C; c += 32) m = fmaxf(m, z[c]);
            m = warp_max(m);
            float se = 0.0f;
            for (int c = lane; c < C; c += 32) se += __expf(z[c] - m);
            se = warp_sum(se);
            const float inv = se > 0.0f ? 1.0f / se : 0.0f;
            for (int c = lane; c < C; c += 32) {
                float g = __expf(z[c] - m) * inv;
                if (c == ti) g -= 1.0f;
                gz[c] = base * g;
            }
        } else {  // void present, not forced: sigmoid pull on the void logit
            for (int c = lane; c < C; c += 32) {
                float g = 0.0f;
                if (c == a.void_index) g = base * (elem(z[c]).p - 1.0f);
                gz[c] = g;
            }
        }
        return;
    }
    const Focal f = make_focal(a.cls_gamma, a.cls_alpha);
    for (int c = lane; c < C; c += 32) {
        const Elem e = elem(z[c]);
        const float om = 1.0f - e.p;
        const float mp = f.use_gamma ? __powf(om, f.gamma) : 1.0f;
        const float mn = f.use_gamma ? __powf(e.p, f.gamma) : 1.0f;
        const float gpos = -f.alpha_pos * mp * (f.gamma * e.p * e.pos + om);
        const float gneg = f.alpha_neg * mn * (f.gamma * om * e.neg + e.p);
        const bool is_void = a.has_void && c == a.void_index;
        float g;
        if (matched) g = base * invC * (c == y ? gpos : gneg);
        else if (a.force_cls) g = base * invC * (is_void ? gpos : gneg);
        else if (is_void) g = base * gpos;
        else g = 0.0f;
        gz[c] = g;
    }
}

// ---------------------------------------------------------------------------
// Backward coefficients + class-logit gradient: grid = ceil(L*B*Q / 8),
// block = 256, one warp per (l,b,q) row.  Each block counts the matched rows
// of its layer(s) with the same fixed-order reduction (so every block gets
// the same coefficients), and the block holding a layer's first row publishes
// coef[l] for mask_grad_kernel, which runs after it.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) bwd_cls_kernel(LossArgs a) {
    pdl_enter();
    __shared__ float sh[32];
    __shared__ float scoef[8][3];
    const int64_t rows = (int64_t)a.L * a.B * a.Q;
    const int64_t n = (int64_t)a.B * a.Q;
    const int64_t r0 = (int64_t)blockIdx.x * 8;
    const int64_t r1 = min(rows, r0 + 8) - 1;
    const int l0 = (int)(r0 / n), l1 = (int)(r1 / n);
    for (int l = l0; l <= l1; ++l) {
        float v[1] = {0.0f};
        for (int64_t i = threadIdx.x; i < n; i += blockDim.x) v[0] += a.pred_to_gt[(int64_t)l * n + i] >= 0;
        block_sum<1>(v, sh);
        if (threadIdx.x == 0) {
            float md, cd;
            denominators(a, v[0], &md, &cd);
            const float im = 1.0f / md, ic = 1.0f / cd;
            const float c[3] = {a.grad_mask[l] * im, a.grad_dice[l] * im, a.grad_cls[l] * (ic * a.cls_scale)};
            const bool first = (int64_t)l * n >= r0 && (int64_t)l * n <= r1;
            for (int k = 0; k < 3; ++k) {
                scoef[l - l0][k] = c[k];
                if (first) a.coef[l * 3 + k] = c[k];
            }
        }
    }
    __syncthreads();
    const int64_t qi = r0 + (threadIdx.x >> 5);
    if (qi > r1 || a.C <= 0) return;
    cls_grad_row(a, qi, threadIdx.x & 31, scoef[(int)(qi / n) - l0][2]);
}

template __global__ void bwd_stats_kernel<false, float>(LossArgs);
template __global__ void bwd_stats_kernel<true, float>(LossArgs);
template __global__ void mask_grad_kernel<false, false, false, float>(LossArgs);
template __global__ void mask_grad_kernel<false, false, true, float>(LossArgs);
template __global__ void mask_grad_kernel<false, true, false, float>(LossArgs);
template __global__ void mask_grad_kernel<false, true, true, float>(LossArgs);
template __global__ void mask_grad_kernel<true, false, false, float>(LossArgs);
template __global__ void mask_grad_kernel<true, false, true, float>(LossArgs);
template __global__ void mask_grad_kernel<true, true, false, float>(LossArgs);
template __global__ void mask_grad_kernel<true, true, true, float>(LossArgs);
template __global__ void bwd_stats_kernel<false, __nv_bfloat16>(LossArgs);
template __global__ void bwd_stats_kernel<true, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<false, false, false, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<false, false, true, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<false, true, false, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<false, true, true, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<true, false, false, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<true, false, true, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<true, true, false, __nv_bfloat16>(LossArgs);
template __global__ void mask_grad_kernel<true, true, true, __nv_bfloat16>(LossArgs);
template __global__ void bwd_stats_kernel<false, __half>(LossArgs);
template __global__ void bwd_stats_kernel<true, __half>(LossArgs);
template __global__ void mask_grad_kernel<false, false, false, __half>(LossArgs);
template __global__ void mask_grad_kernel<false, false, true, __half>(LossArgs);
template __global__ void mask_grad_kernel<false, true, false, __half>(LossArgs);
template __global__ void mask_grad_kernel<false, true, true, __half>(LossArgs);
template __global__ void mask_grad_kernel<true, false, false, __half>(LossArgs);
template __global__ void mask_grad_kernel<true, false, true, __half>(LossArgs);
template __global__ void mask_grad_kernel<true, true, false, __half>(LossArgs);
template __global__ void mask_grad_kernel<true, true, true, __half>(LossArgs);

}  // namespace mlb
