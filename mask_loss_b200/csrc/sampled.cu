// sampled.cu -- point-sampled matching costs and gradients (config 3).
//
// Replaces pairwise_sigmoid_cross_entropy_loss_sampling_py
// (functions/sigmoid/pw_sigmoid_ce.py:407-549) and pairwise_dice_loss_sampling_py
// (functions/dice/pw_dice_loss.py:174-268): per image one shared set of P
// points; logits are sampled bilinearly (grid_sample, zero padding), labels
// with the floor-nearest rule ix = floor(x * (W_t - 1)).
//
// Layout trick: the P points of an image are sorted by the output column of
// their label (a deterministic counting sort, one block per image), and the
// sampled logits are written in that order.  Label runs are then contiguous
// and the streaming cost kernel of cost.cu runs unchanged on the (L,B,Q,P)
// sampled values with points as cells.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

// Floor-nearest label of point p (fp32 arithmetic as in the reference:
// (x * (W_t - 1)).long(), clamped).
ML_INLINE int64_t point_label(const int64_t* tb, int Ht, int Wt, float x, float y) {
    int ix = (int)(x * (float)(Wt - 1));
    int iy = (int)(y * (float)(Ht - 1));
    ix = min(max(ix, 0), Wt - 1);
    iy = min(max(iy, 0), Ht - 1);
    return tb[(int64_t)iy * Wt + ix];
}

// ---------------------------------------------------------------------------
// One block per image: stable counting sort of the points by output column
// (bucket 0 = no column).  Writes perm[b][pos] = point, scodes[b][pos] =
// column (or kNone), and ptotals[b][label] = points per label id.
// Dynamic shared memory: (gout + 2) ints.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
point_sort_kernel(const int64_t* __restrict__ targets, const float* __restrict__ coords, int Ht,
                  int Wt, int P, int gt_total, int bg, int gout, int32_t* __restrict__ perm,
                  int32_t* __restrict__ scodes, int32_t* __restrict__ ptotals) {
    extern __shared__ int32_t bucket[];  // [gout + 1] counts, then running offsets
    const int b = blockIdx.x;
    const int64_t* tb = targets + (int64_t)b * Ht * Wt;
    const float* cb = coords + (int64_t)b * P * 2;
    int32_t* pt = ptotals + (int64_t)b * gt_total;
    for (int i = threadIdx.x; i <= gout; i += blockDim.x) bucket[i] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const int64_t lab = point_label(tb, Ht, Wt, cb[2 * p], cb[2 * p + 1]);
        if (lab >= 0 && lab < gt_total) atomicAdd(&pt[lab], 1);
        atomicAdd(&bucket[label_to_col(lab, gt_total, bg) + 1], 1);
    }
    __syncthreads();
    if (threadIdx.x == 0) {  // exclusive prefix (gout is small)
        int run = 0;
        for (int i = 0; i <= gout; ++i) {
            const int c = bucket[i];
            bucket[i] = run;
            run += c;
        }
    }
    __syncthreads();
    if (threadIdx.x >= 32) return;
    // stable scatter: warp 0 walks the points in order, 32 at a time
    const int lane = threadIdx.x;
    for (int base = 0; base < P; base += 32) {
        const int p = base + lane;
        int key = -1;
        if (p < P) key = label_to_col(point_label(tb, Ht, Wt, cb[2 * p], cb[2 * p + 1]), gt_total, bg) + 1;
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int pos = 0;
        if (p < P) pos = bucket[key] + rank;
        __syncwarp();
        if (p < P && rank == 0) bucket[key] += __popc(peers);
        __syncwarp();
        if (p < P) {
            perm[(int64_t)b * P + pos] = p;
            scodes[(int64_t)b * P + pos] = key - 1;
        }
    }
}

// Bilinear taps of a point (grid_sample semantics, zero padding).
struct Taps {
    int idx[4];
    float w[4];
};

ML_INLINE Taps bilinear_taps(float x, float y, int H, int W, bool align) {
    const float ix = align ? x * (float)(W - 1) : x * (float)W - 0.5f;
    const float iy = align ? y * (float)(H - 1) : y * (float)H - 0.5f;
    const float fx0 = floorf(ix), fy0 = floorf(iy);
    const int x0 = (int)fx0, y0 = (int)fy0;
    const float fx = ix - fx0, fy = iy - fy0;
    Taps t;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int xx = x0 + (k & 1), yy = y0 + (k >> 1);
        const float wx = (k & 1) ? fx : 1.0f - fx;
        const float wy = (k >> 1) ? fy : 1.0f - fy;
        const bool in = xx >= 0 && xx < W && yy >= 0 && yy < H;
        t.idx[k] = in ? yy * W + xx : 0;
        t.w[k] = in ? wx * wy : 0.0f;
    }
    return t;
}

template <typename T>
ML_INLINE float ld_logit(const T* p);
template <>
ML_INLINE float ld_logit<float>(const float* p) { return __ldg(p); }
template <>
ML_INLINE float ld_logit<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// ---------------------------------------------------------------------------
// Sampled logits in sorted point order: zs[lbq][pos] for every query.
// grid = (ceil(P/256), L*B, ceil(Q/kSampleQ)); a thread computes its point's
// taps once and reuses them for kSampleQ queries.
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ void point_sample_body(const T* __restrict__ logits,
                                                  const float* __restrict__ coords,
                                                  const int32_t* __restrict__ perm, int B, int Q,
                                                  int H, int W, int P, int align,
                                                  float* __restrict__ zs) {
    const int pos = blockIdx.x * blockDim.x + threadIdx.x;
    const int lb = blockIdx.y, b = lb % B;
    if (pos >= P) return;
    const int p = perm[(int64_t)b * P + pos];
    const float* cb = coords + ((int64_t)b * P + p) * 2;
    const Taps tp = bilinear_taps(cb[0], cb[1], H, W, align != 0);
    const int q0 = blockIdx.z * kSampleQ;
    const int q1 = min(Q, q0 + kSampleQ);
    const int64_t HW = (int64_t)H * W;
    for (int q = q0; q < q1; ++q) {
        const int64_t row = (int64_t)lb * Q + q;
        const T* m = logits + row * HW;
        float z = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) z += tp.w[k] * ld_logit(m + tp.idx[k]);
        zs[row * P + pos] = z;
    }
}

__global__ void __launch_bounds__(256)
point_sample_f32_kernel(const float* logits, const float* coords, const int32_t* perm, int B, int Q,
                        int H, int W, int P, int align, float* zs) {
    point_sample_body<float>(logits, coords, perm, B, Q, H, W, P, align, zs);
}

__global__ void __launch_bounds__(256)
point_sample_bf16_kernel(const __nv_bfloat16* logits, const float* coords, const int32_t* perm,
                         int B, int Q, int H, int W, int P, int align, float* zs) {
    point_sample_body<__nv_bfloat16>(logits, coords, perm, B, Q, H, W, P, align, zs);
}

// ---------------------------------------------------------------------------
// Backward of the sampled mask costs: per (query, sorted point) the point
// gradient of the matched (or forced-empty) sigmoid-CE + dice terms, scattered
// to the 4 bilinear taps with atomicAdd into the fp32 gradient map.
// grid = (ceil(P/256), L*B*Q).  zs holds the forward's sampled values.
// ---------------------------------------------------------------------------
template <bool FOC>
__device__ __forceinline__ void point_grad_body(const LossArgs& a, const float* __restrict__ zs,
                                                const float* __restrict__ coords,
                                                const int32_t* __restrict__ perm,
                                                const int32_t* __restrict__ scodes, int P,
                                                int align, float* __restrict__ gacc) {
    const int pos = blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t qi = blockIdx.y;
    if (pos >= P) return;
    const int lb = (int)(qi / a.Q), l = lb / a.B, b = lb % a.B;
    const int64_t og = a.pred_to_gt[qi];
    const int64_t ga = og + (og >= a.bg ? 1 : 0);
    const bool matched = og >= 0 && ga < a.gt_total;
    const float mcoef = a.coef[l * 3 + 0], dcoef = a.coef[l * 3 + 1];
    if (!(matched || a.force_masks) || (mcoef == 0.0f && dcoef == 0.0f)) return;
    const float* sv = a.stats_in + qi * kSaved;
    const float Ps = sv[0], T = matched ? sv[1] : 0.0f, I = matched ? sv[2] : 0.0f, Wt = sv[3];
    const float sf = a.sigmoid_scale / Wt;
    const float den = Ps + T + a.smooth;
    const float num = 2.0f * I + a.smooth;
    const float inv_d2 = 1.0f / fmaxf(den * den, 1e-20f);
    const float x = zs[qi * P + pos];
    const Elem e = elem(x);
    const float om = 1.0f - e.p, pp = e.p * om;
    const float t = (matched && scodes[(int64_t)b * P + pos] == (int)og) ? 1.0f : 0.0f;
    const float ncnt = 1.0f - t;
    float gs;
    if (FOC) {
        const Focal f = make_focal(a.mask_gamma, a.mask_alpha);
        const float mp = f.use_gamma ? __powf(om, f.gamma) : 1.0f;
        const float mn = f.use_gamma ? __powf(e.p, f.gamma) : 1.0f;
        gs = (-f.alpha_pos * t * mp * (f.gamma * e.p * e.pos + om) +
              f.alpha_neg * ncnt * mn * (f.gamma * om * e.neg + e.p)) * sf;
    } else {
        gs = (ncnt * e.p - t * om) * sf;
    }
    const float gd = (num * pp - 2.0f * den * pp * t) * inv_d2 * a.dice_scale;
    const float g = mcoef * gs + dcoef * gd;
    const int p = perm[(int64_t)b * P + pos];
    const float* cb = coords + ((int64_t)b * P + p) * 2;
    const Taps tp = bilinear_taps(cb[0], cb[1], a.H, a.W, align != 0);
    float* gm = gacc + qi * (int64_t)a.H * a.W;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        if (tp.w[k] != 0.0f) atomicAdd(gm + tp.idx[k], g * tp.w[k]);
}

__global__ void __launch_bounds__(256)
point_grad_kernel(LossArgs a, const float* zs, const float* coords, const int32_t* perm,
                  const int32_t* scodes, int P, int align, float* gacc) {
    point_grad_body<false>(a, zs, coords, perm, scodes, P, align, gacc);
}

__global__ void __launch_bounds__(256)
point_grad_focal_kernel(LossArgs a, const float* zs, const float* coords, const int32_t* perm,
                        const int32_t* scodes, int P, int align, float* gacc) {
    point_grad_body<true>(a, zs, coords, perm, scodes, P, align, gacc);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                   int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

// Host-side launchers (kernels and launches live in this file).
cudaError_t launch_point_sample(int dtype, const void* logits, const float* coords,
                                const int32_t* perm, int B, int L, int Q, int H, int W, int P,
                                int align, float* zs, cudaStream_t st) {
    dim3 g((P + 255) / 256, (unsigned)(L * B), (Q + kSampleQ - 1) / kSampleQ);
    if (dtype == 1)
        point_sample_bf16_kernel<<<g, 256, 0, st>>>(
            static_cast<const __nv_bfloat16*>(logits), coords, perm, B, Q, H, W, P, align, zs);
    else
        point_sample_f32_kernel<<<g, 256, 0, st>>>(static_cast<const float*>(logits), coords,
                                                      perm, B, Q, H, W, P, align, zs);
    return cudaGetLastError();
}

cudaError_t launch_point_grad(bool foc, const LossArgs& la, const float* zs, const float* coords,
                              const int32_t* perm, const int32_t* scodes, int P, int align,
                              float* gacc, int64_t rows, cudaStream_t st) {
    dim3 g((P + 255) / 256, (unsigned)rows);
    if (foc) point_grad_focal_kernel<<<g, 256, 0, st>>>(la, zs, coords, perm, scodes, P, align, gacc);
    else point_grad_kernel<<<g, 256, 0, st>>>(la, zs, coords, perm, scodes, P, align, gacc);
    return cudaGetLastError();
}

cudaError_t launch_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t st) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 65535);
    f32_to_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(src, static_cast<__nv_bfloat16*>(dst), n);
    return cudaGetLastError();
}


}  // namespace mlb
