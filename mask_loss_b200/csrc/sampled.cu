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
// (bucket 0 = no column).  Keys are computed in parallel into shared memory;
// each warp histograms its contiguous segment, the segment offsets come from
// a fixed-order prefix, and each warp scatters its segment in order, so the
// result is deterministic.  Writes perm[b][pos] = point, scodes[b][pos] =
// column (or kNone), scoords[b][pos] = the point's (x, y), and
// ptotals[b][label] = points per label id.
// Dynamic shared memory: P + (kSortWarps + 1) * (gout + 1) ints.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSortWarps * 32)
point_sort_kernel(const int64_t* __restrict__ targets, const float* __restrict__ coords, int Ht,
                  int Wt, int P, int gt_total, int bg, int gout, int32_t* __restrict__ perm,
                  int32_t* __restrict__ scodes, float* __restrict__ scoords,
                  int32_t* __restrict__ ptotals) {
    extern __shared__ int32_t sm[];
    const int NB = gout + 1;
    int32_t* keys = sm;                    // [P]
    int32_t* wcnt = keys + P;              // [kSortWarps][NB] counts, then offsets
    int32_t* total = wcnt + kSortWarps * NB;  // [NB]
    const int b = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int64_t* tb = targets + (int64_t)b * Ht * Wt;
    const float* cb = coords + (int64_t)b * P * 2;
    int32_t* pt = ptotals + (int64_t)b * gt_total;
    for (int i = tid; i < kSortWarps * NB; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    const int seg = (P + kSortWarps - 1) / kSortWarps;
    const int s0 = min(P, warp * seg), s1 = min(P, s0 + seg);
    // four points per lane in flight: coordinates, then the label gathers,
    // then the counts (the atomics would otherwise serialise the loads)
    for (int p0 = s0; p0 < s1; p0 += 4 * 32) {
        float x[4], y[4];
        int64_t lab[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int p = p0 + 32 * u + lane;
            x[u] = p < s1 ? cb[2 * p] : 0.0f;
            y[u] = p < s1 ? cb[2 * p + 1] : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
            lab[u] = p0 + 32 * u + lane < s1 ? point_label(tb, Ht, Wt, x[u], y[u]) : -1;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int p = p0 + 32 * u + lane;
            if (p >= s1) continue;
            if (lab[u] >= 0 && lab[u] < gt_total) atomicAdd(&pt[lab[u]], 1);
            const int key = label_to_col(lab[u], gt_total, bg) + 1;
            keys[p] = key;
            atomicAdd(&wcnt[warp * NB + key], 1);
        }
    }
    __syncthreads();
    // offsets: bucket-major, then warp order (fixed order -> stable, deterministic)
    for (int k = tid; k < NB; k += blockDim.x) {
        int run = 0;
        for (int w = 0; w < kSortWarps; ++w) run += wcnt[w * NB + k];
        total[k] = run;
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int k = 0; k < NB; ++k) {
            const int c = total[k];
            total[k] = run;
            run += c;
        }
    }
    __syncthreads();
    for (int k = tid; k < NB; k += blockDim.x) {
        int run = total[k];
        for (int w = 0; w < kSortWarps; ++w) {
            const int c = wcnt[w * NB + k];
            wcnt[w * NB + k] = run;
            run += c;
        }
    }
    __syncthreads();
    int32_t* off = wcnt + warp * NB;
    for (int base = s0; base < s1; base += 32) {
        const int p = base + lane;
        const int key = p < s1 ? keys[p] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const int pos = p < s1 ? off[key] + rank : 0;
        __syncwarp();
        if (p < s1 && rank == 0) off[key] += __popc(peers);
        __syncwarp();
        if (p < s1) {
            const int64_t o = (int64_t)b * P + pos;
            perm[o] = p;
            scodes[o] = key - 1;
            scoords[2 * o] = cb[2 * p];
            scoords[2 * o + 1] = cb[2 * p + 1];
        }
    }
}

// ---------------------------------------------------------------------------
// The same stable counting sort spread over kSortBlockPts-point blocks of
// every image (the single-block form leaves most SMs idle: one CTA per image).
//   point_keys_kernel     grid (nblk, B): each point's key (column + 1, 0 =
//                         no column) and the block's bucket counts; the
//                         per-label point totals.
//   point_scatter_kernel  grid (nblk, B): the block's bucket offsets (all
//                         buckets before, then earlier blocks of the same
//                         bucket -- a fixed order), then the single-block
//                         kernel's warp-ordered scatter within the block.
// Same result as point_sort_kernel, bit for bit.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
point_keys_kernel(const int64_t* __restrict__ targets, const float* __restrict__ coords, int Ht,
                  int Wt, int P, int gt_total, int bg, int gout, int32_t* __restrict__ keys,
                  int32_t* __restrict__ bhist, int32_t* __restrict__ ptotals) {
    extern __shared__ int32_t hsm[];  // [NB] bucket counts, then [gt_total] label counts
    const int NB = gout + 1;
    int32_t* hl = hsm + NB;
    const int b = blockIdx.y, j = blockIdx.x, nblk = gridDim.x;
    for (int k = threadIdx.x; k < NB + gt_total; k += blockDim.x) hsm[k] = 0;
    __syncthreads();
    const int64_t* tb = targets + (int64_t)b * Ht * Wt;
    const float2* cb = reinterpret_cast<const float2*>(coords + (int64_t)b * P * 2);
    int32_t* pt = ptotals + (int64_t)b * gt_total;
    const int p0 = j * kSortBlockPts, p1 = min(P, p0 + kSortBlockPts);
    constexpr int U = kSortBlockPts / 256;
    float2 c[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int p = p0 + u * 256 + (int)threadIdx.x;
        c[u] = p < p1 ? cb[p] : make_float2(0.0f, 0.0f);
    }
    int64_t lab[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
        lab[u] = p0 + u * 256 + (int)threadIdx.x < p1 ? point_label(tb, Ht, Wt, c[u].x, c[u].y) : -1;
#pragma unroll
    for (int u = 0; u < U; ++u) {
        const int p = p0 + u * 256 + (int)threadIdx.x;
        if (p >= p1) continue;
        if (lab[u] >= 0 && lab[u] < gt_total) atomicAdd(&hl[lab[u]], 1);
        const int key = label_to_col(lab[u], gt_total, bg) + 1;
        keys[(int64_t)b * P + p] = key;
        atomicAdd(&hsm[key], 1);
    }
    __syncthreads();
    for (int k = threadIdx.x; k < NB; k += blockDim.x) bhist[((int64_t)b * nblk + j) * NB + k] = hsm[k];
    // one global atomic per label present in the block (integer: order-free)
    for (int k = threadIdx.x; k < gt_total; k += blockDim.x)
        if (hl[k]) atomicAdd(&pt[k], hl[k]);
}

__global__ void __launch_bounds__(256)
point_scatter_kernel(const int32_t* __restrict__ keys, const int32_t* __restrict__ bhist,
                     const float* __restrict__ coords, int P, int gout, int32_t* __restrict__ perm,
                     int32_t* __restrict__ scodes, float* __restrict__ scoords) {
    extern __shared__ int32_t ssm[];
    constexpr int NW = 8;
    const int NB = gout + 1;
    int32_t* base = ssm;             // [NB] this block's first position per bucket
    int32_t* wcnt = base + NB;       // [NW][NB]
    const int b = blockIdx.y, j = blockIdx.x, nblk = gridDim.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int32_t* bh = bhist + (int64_t)b * nblk * NB;
    for (int k = tid; k < NB; k += blockDim.x) {
        int all = 0, before = 0;
        for (int jj = 0; jj < nblk; ++jj) {
            const int c = bh[(int64_t)jj * NB + k];
            all += c;
            if (jj < j) before += c;
        }
        base[k] = all;      // bucket total for now
        wcnt[k] = before;   // scratch: earlier blocks' share of bucket k
    }
    __syncthreads();
    if (tid == 0) {
        int run = 0;
        for (int k = 0; k < NB; ++k) {
            const int c = base[k];
            base[k] = run + wcnt[k];
            run += c;
        }
    }
    __syncthreads();
    for (int i = tid; i < NW * NB; i += blockDim.x) wcnt[i] = 0;
    __syncthreads();
    const int p0 = j * kSortBlockPts, p1 = min(P, p0 + kSortBlockPts);
    const int seg = kSortBlockPts / NW;
    const int s0 = min(p1, p0 + warp * seg), s1 = min(p1, s0 + seg);
    const int32_t* kb = keys + (int64_t)b * P;
    for (int p = s0 + lane; p < s1; p += 32) atomicAdd(&wcnt[warp * NB + kb[p]], 1);
    __syncthreads();
    for (int k = tid; k < NB; k += blockDim.x) {
        int run = base[k];
        for (int w = 0; w < NW; ++w) {
            const int c = wcnt[w * NB + k];
            wcnt[w * NB + k] = run;
            run += c;
        }
    }
    __syncthreads();
    int32_t* off = wcnt + warp * NB;
    const float* cb = coords + (int64_t)b * P * 2;
    for (int q0 = s0; q0 < s1; q0 += 32) {
        const int p = q0 + lane;
        const int key = p < s1 ? kb[p] : -1;
        const unsigned peers = __match_any_sync(0xffffffffu, key);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        const int pos = p < s1 ? off[key] + rank : 0;
        __syncwarp();
        if (p < s1 && rank == 0) off[key] += __popc(peers);
        __syncwarp();
        if (p < s1) {
            const int64_t o = (int64_t)b * P + pos;
            perm[o] = p;
            scodes[o] = key - 1;
            scoords[2 * o] = cb[2 * p];
            scoords[2 * o + 1] = cb[2 * p + 1];
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

ML_INLINE float to_f32(float v) { return v; }
template <typename T> ML_INLINE T from_f32(float v);
template <> ML_INLINE float from_f32<float>(float v) { return v; }
template <> ML_INLINE __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
ML_INLINE float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

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
                                                  const float* __restrict__ scoords, int B, int Q,
                                                  int H, int W, int P, int align,
                                                  float* __restrict__ zs) {
    const int pos = blockIdx.x * blockDim.x + threadIdx.x;
    const int lb = blockIdx.y, b = lb % B;
    if (pos >= P) return;
    const float* cb = scoords + ((int64_t)b * P + pos) * 2;
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
point_sample_f32_kernel(const float* logits, const float* scoords, int B, int Q, int H, int W, int P,
                        int align, float* zs) {
    point_sample_body<float>(logits, scoords, B, Q, H, W, P, align, zs);
}

__global__ void __launch_bounds__(256)
point_sample_bf16_kernel(const __nv_bfloat16* logits, const float* scoords, int B, int Q, int H,
                         int W, int P, int align, float* zs) {
    point_sample_body<__nv_bfloat16>(logits, scoords, B, Q, H, W, P, align, zs);
}

// Block per (l,b,q) row: the row's logit map is staged in shared memory, so
// the 4 taps of every point are shared-memory reads and the sampled row is
// written contiguously.
template <typename T>
__device__ __forceinline__ void point_sample_row_body(const T* __restrict__ logits,
                                                      const float* __restrict__ scoords, int B,
                                                      int Q, int H, int W, int P, int align,
                                                      float* __restrict__ zs) {
    extern __shared__ __align__(16) unsigned char smap_raw[];
    T* map = reinterpret_cast<T*>(smap_raw);
    const int64_t row = blockIdx.x;
    const int b = (int)((row / Q) % B);
    const int HW = H * W;
    const T* src = logits + row * (int64_t)HW;
    const int nvec = (HW * (int)sizeof(T)) / 16;  // 16-byte chunks
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        for (int i = threadIdx.x; i < nvec; i += blockDim.x)
            reinterpret_cast<uint4*>(map)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
        for (int i = nvec * 16 / (int)sizeof(T) + threadIdx.x; i < HW; i += blockDim.x) map[i] = src[i];
    } else {
        for (int i = threadIdx.x; i < HW; i += blockDim.x) map[i] = src[i];
    }
    __syncthreads();
    const float* cb = scoords + (int64_t)b * P * 2;
    float* out = zs + row * P;
#pragma unroll 4
    for (int pos = threadIdx.x; pos < P; pos += blockDim.x) {
        const float2 c = reinterpret_cast<const float2*>(cb)[pos];
        const Taps tp = bilinear_taps(c.x, c.y, H, W, align != 0);
        float z = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) z += tp.w[k] * to_f32(map[tp.idx[k]]);
        out[pos] = z;
    }
}

__global__ void __launch_bounds__(kPointRowThreads)
point_sample_row_f32_kernel(const float* logits, const float* scoords, int B, int Q, int H, int W,
                            int P, int align, float* zs) {
    point_sample_row_body<float>(logits, scoords, B, Q, H, W, P, align, zs);
}

__global__ void __launch_bounds__(kPointRowThreads)
point_sample_row_bf16_kernel(const __nv_bfloat16* logits, const float* scoords, int B, int Q, int H,
                             int W, int P, int align, float* zs) {
    point_sample_row_body<__nv_bfloat16>(logits, scoords, B, Q, H, W, P, align, zs);
}

// ---------------------------------------------------------------------------
// Backward of the sampled mask costs: per (query, sorted point) the point
// gradient of the matched (or forced-empty) sigmoid-CE + dice terms, spread
// to the 4 bilinear taps.
// ---------------------------------------------------------------------------
struct RowGrad {
    bool active, matched;
    int gcol;
    float mcoef, dcoef, sf, den, num, inv_d2;
};

ML_INLINE RowGrad row_grad_setup(const LossArgs& a, int64_t qi) {
    RowGrad r;
    const int lb = (int)(qi / a.Q), l = lb / a.B;
    const int64_t og = a.pred_to_gt[qi];
    const int64_t ga = og + (og >= a.bg ? 1 : 0);
    r.matched = og >= 0 && ga < a.gt_total;
    r.gcol = r.matched ? (int)og : -100;
    r.mcoef = a.coef[l * 3 + 0];
    r.dcoef = a.coef[l * 3 + 1];
    r.active = (r.matched || a.force_masks) && !(r.mcoef == 0.0f && r.dcoef == 0.0f);
    const float* sv = a.stats_in + qi * kSaved;
    const float Ps = sv[0], T = r.matched ? sv[1] : 0.0f, I = r.matched ? sv[2] : 0.0f;
    r.sf = a.sigmoid_scale / sv[3];
    r.den = Ps + T + a.smooth;
    r.num = 2.0f * I + a.smooth;
    r.inv_d2 = 1.0f / fmaxf(r.den * r.den, 1e-20f);
    return r;
}

template <bool FOC>
ML_INLINE float point_grad_value(const LossArgs& a, const RowGrad& r, float x, int code) {
    const Elem e = elem(x);
    const float om = 1.0f - e.p, pp = e.p * om;
    const float t = (code == r.gcol) ? 1.0f : 0.0f;
    const float ncnt = 1.0f - t;
    float gs;
    if (FOC) {
        const Focal f = make_focal(a.mask_gamma, a.mask_alpha);
        const float mp = f.use_gamma ? __powf(om, f.gamma) : 1.0f;
        const float mn = f.use_gamma ? __powf(e.p, f.gamma) : 1.0f;
        gs = (-f.alpha_pos * t * mp * (f.gamma * e.p * e.pos + om) +
              f.alpha_neg * ncnt * mn * (f.gamma * om * e.neg + e.p)) * r.sf;
    } else {
        gs = (ncnt * e.p - t * om) * r.sf;
    }
    const float gd = (r.num * pp - 2.0f * r.den * pp * t) * r.inv_d2 * a.dice_scale;
    return r.mcoef * gs + r.dcoef * gd;
}

// Large maps: global fp32 accumulation (caller zeroes gacc).
// grid = (ceil(P/256), L*B*Q).
template <bool FOC>
__device__ __forceinline__ void point_grad_global_body(const LossArgs& a, const float* zs,
                                                       const float* scoords, const int32_t* scodes,
                                                       int P, int align, float* gacc) {
    const int pos = blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t qi = blockIdx.y;
    if (pos >= P) return;
    const RowGrad r = row_grad_setup(a, qi);
    if (!r.active) return;
    const int b = (int)((qi / a.Q) % a.B);
    const float g = point_grad_value<FOC>(a, r, zs[qi * P + pos], scodes[(int64_t)b * P + pos]);
    const float* cb = scoords + ((int64_t)b * P + pos) * 2;
    const Taps tp = bilinear_taps(cb[0], cb[1], a.H, a.W, align != 0);
    float* gm = gacc + qi * (int64_t)a.H * a.W;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        if (tp.w[k] != 0.0f) atomicAdd(gm + tp.idx[k], g * tp.w[k]);
}

__global__ void __launch_bounds__(256)
point_grad_global_kernel(LossArgs a, const float* zs, const float* scoords, const int32_t* scodes,
                         int P, int align, float* gacc) {
    point_grad_global_body<false>(a, zs, scoords, scodes, P, align, gacc);
}

__global__ void __launch_bounds__(256)
point_grad_global_focal_kernel(LossArgs a, const float* zs, const float* scoords,
                               const int32_t* scodes, int P, int align, float* gacc) {
    point_grad_global_body<true>(a, zs, scoords, scodes, P, align, gacc);
}

// One row of HW values in the logits' dtype, from a shared-memory fp32 map
// (or zeros when map is null): 16-byte stores where the row allows them.
template <typename TO>
ML_INLINE void write_grad_row(TO* out, const float* map, int HW) {
    constexpr int V = 16 / (int)sizeof(TO);
    if (HW % V == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0) {
        uint4* o = reinterpret_cast<uint4*>(out);
        for (int i = threadIdx.x; i < HW / V; i += blockDim.x) {
            float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            if (map) {
                const float4* m = reinterpret_cast<const float4*>(map + i * V);
                const float4 a = m[0];
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                if (V == 8) {
                    const float4 b = m[1];
                    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
                }
            }
            uint4 w;
            if constexpr (sizeof(TO) == 4) {
                w = make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]),
                               __float_as_uint(v[3]));
            } else {
                w = make_uint4(narrow2(v[0], v[1], out), narrow2(v[2], v[3], out),
                               narrow2(v[4], v[5], out), narrow2(v[6], v[7], out));
            }
            o[i] = w;
        }
    } else {
        for (int i = threadIdx.x; i < HW; i += blockDim.x) out[i] = from_f32<TO>(map ? map[i] : 0.0f);
    }
}

// Block per (l,b,q) row: the gradient map is accumulated in shared memory
// and written once in the logits' dtype (zeros for rows the loss does not
// reach), so no memset, no global atomics and no conversion pass.
template <bool FOC, typename TO>
__device__ __forceinline__ void point_grad_row_body(const LossArgs& a, const float* zs,
                                                    const float* scoords, const int32_t* scodes,
                                                    int P, int align, TO* grad) {
    extern __shared__ __align__(16) float gmap[];
    const int64_t qi = blockIdx.x;
    const int HW = a.H * a.W;
    TO* out = grad + qi * (int64_t)HW;
    const RowGrad r = row_grad_setup(a, qi);
    if (!r.active) {
        write_grad_row<TO>(out, nullptr, HW);
        return;
    }
    for (int i = threadIdx.x; i < HW / 4; i += blockDim.x)
        reinterpret_cast<float4*>(gmap)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = (HW / 4) * 4 + threadIdx.x; i < HW; i += blockDim.x) gmap[i] = 0.0f;
    __syncthreads();
    const int b = (int)((qi / a.Q) % a.B);
    const float* cb = scoords + (int64_t)b * P * 2;
    const int32_t* cd = scodes + (int64_t)b * P;
    const float* z = zs + qi * P;
#pragma unroll 4
    for (int pos = threadIdx.x; pos < P; pos += blockDim.x) {
        const float g = point_grad_value<FOC>(a, r, z[pos], cd[pos]);
        const float2 c = reinterpret_cast<const float2*>(cb)[pos];
        const Taps tp = bilinear_taps(c.x, c.y, a.H, a.W, align != 0);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (tp.w[k] != 0.0f) atomicAdd(&gmap[tp.idx[k]], g * tp.w[k]);
    }
    __syncthreads();
    write_grad_row<TO>(out, gmap, HW);
}

__global__ void __launch_bounds__(kPointRowThreads)
point_grad_row_f32_kernel(LossArgs a, const float* zs, const float* scoords, const int32_t* scodes,
                          int P, int align, float* grad) {
    point_grad_row_body<false, float>(a, zs, scoords, scodes, P, align, grad);
}
__global__ void __launch_bounds__(kPointRowThreads)
point_grad_row_focal_f32_kernel(LossArgs a, const float* zs, const float* scoords,
                                const int32_t* scodes, int P, int align, float* grad) {
    point_grad_row_body<true, float>(a, zs, scoords, scodes, P, align, grad);
}
__global__ void __launch_bounds__(kPointRowThreads)
point_grad_row_bf16_kernel(LossArgs a, const float* zs, const float* scoords, const int32_t* scodes,
                           int P, int align, __nv_bfloat16* grad) {
    point_grad_row_body<false, __nv_bfloat16>(a, zs, scoords, scodes, P, align, grad);
}
__global__ void __launch_bounds__(kPointRowThreads)
point_grad_row_focal_bf16_kernel(LossArgs a, const float* zs, const float* scoords,
                                 const int32_t* scodes, int P, int align, __nv_bfloat16* grad) {
    point_grad_row_body<true, __nv_bfloat16>(a, zs, scoords, scodes, P, align, grad);
}

__global__ void f32_to_bf16_kernel(const float* __restrict__ src, __nv_bfloat16* __restrict__ dst,
                                   int64_t n) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(src[i]);
}

// ---------------------------------------------------------------------------
// Host-side launchers (kernels and their launches live in this file).
// ---------------------------------------------------------------------------
size_t point_sort_smem(int P, int gout) {
    return sizeof(int32_t) * ((size_t)P + (size_t)(kSortWarps + 1) * (gout + 1));
}

size_t point_sort_scratch_bytes(int B, int P, int gout) {
    const int nblk = (P + kSortBlockPts - 1) / kSortBlockPts;
    return sizeof(int32_t) * ((size_t)B * P + (size_t)B * nblk * (gout + 1));
}

cudaError_t launch_point_sort(const int64_t* targets, const float* coords, int B, int Ht, int Wt,
                              int P, int gt_total, int bg, int gout, int32_t* perm, int32_t* scodes,
                              float* scoords, int32_t* ptotals, cudaStream_t st, int32_t* scratch) {
    if (scratch) {  // blocks of kSortBlockPts points: keys + block histograms, then the scatter
        const int nblk = (P + kSortBlockPts - 1) / kSortBlockPts;
        const int NB = gout + 1;
        int32_t* keys = scratch;
        int32_t* bhist = scratch + (size_t)B * P;
        const size_t ks = sizeof(int32_t) * ((size_t)NB + (size_t)gt_total);
        const size_t ss = sizeof(int32_t) * (size_t)NB * 9;
        cudaError_t e = cudaFuncSetAttribute(point_keys_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ks);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(point_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)ss);
        if (e != cudaSuccess) return e;
        point_keys_kernel<<<dim3(nblk, B), 256, ks, st>>>(targets, coords, Ht, Wt, P, gt_total, bg,
                                                          gout, keys, bhist, ptotals);
        point_scatter_kernel<<<dim3(nblk, B), 256, ss, st>>>(keys, bhist, coords, P, gout, perm,
                                                             scodes, scoords);
        return cudaGetLastError();
    }
    const size_t smem = point_sort_smem(P, gout);
    cudaError_t e = cudaFuncSetAttribute(point_sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    point_sort_kernel<<<B, kSortWarps * 32, smem, st>>>(targets, coords, Ht, Wt, P, gt_total, bg, gout,
                                                         perm, scodes, scoords, ptotals);
    return cudaGetLastError();
}

cudaError_t launch_point_sample(int dtype, const void* logits, const float* scoords, int B, int L,
                                int Q, int H, int W, int P, int align, float* zs, cudaStream_t st) {
    const size_t map = (size_t)H * W * (dtype == 1 ? 2 : 4);
    const int64_t rows = (int64_t)L * B * Q;
    if (map <= kRowMapMaxBytes) {
        const int smem = (int)((map + 15) & ~size_t(15));
        if (dtype == 1) {
            cudaError_t e = cudaFuncSetAttribute(point_sample_row_bf16_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            point_sample_row_bf16_kernel<<<(unsigned)rows, kPointRowThreads, smem, st>>>(
                static_cast<const __nv_bfloat16*>(logits), scoords, B, Q, H, W, P, align, zs);
        } else {
            cudaError_t e = cudaFuncSetAttribute(point_sample_row_f32_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (e != cudaSuccess) return e;
            point_sample_row_f32_kernel<<<(unsigned)rows, kPointRowThreads, smem, st>>>(
                static_cast<const float*>(logits), scoords, B, Q, H, W, P, align, zs);
        }
        return cudaGetLastError();
    }
    dim3 g((P + 255) / 256, (unsigned)(L * B), (Q + kSampleQ - 1) / kSampleQ);
    if (dtype == 1)
        point_sample_bf16_kernel<<<g, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), scoords,
                                                    B, Q, H, W, P, align, zs);
    else
        point_sample_f32_kernel<<<g, 256, 0, st>>>(static_cast<const float*>(logits), scoords, B, Q, H,
                                                   W, P, align, zs);
    return cudaGetLastError();
}

// Returns true in *used_rows when the row kernel wrote grad_out directly;
// otherwise the caller zeroed `gacc` (fp32) and must convert when needed.
cudaError_t launch_point_grad(bool foc, int dtype, const LossArgs& la, const float* zs,
                              const float* scoords, const int32_t* scodes, int P, int align,
                              void* grad_out, float* gacc, int64_t rows, bool* used_rows,
                              cudaStream_t st) {
    const size_t map = (size_t)la.H * la.W * 4;
    if (map <= kRowMapMaxBytes) {
        *used_rows = true;
        const int smem = (int)map;
#define ML_PG(K, T)                                                                             \
    do {                                                                                         \
        cudaError_t e = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, smem); \
        if (e != cudaSuccess) return e;                                                          \
        K<<<(unsigned)rows, kPointRowThreads, smem, st>>>(la, zs, scoords, scodes, P, align, static_cast<T*>(grad_out)); \
    } while (0)
        if (dtype == 1) {
            if (foc) ML_PG(point_grad_row_focal_bf16_kernel, __nv_bfloat16);
            else ML_PG(point_grad_row_bf16_kernel, __nv_bfloat16);
        } else {
            if (foc) ML_PG(point_grad_row_focal_f32_kernel, float);
            else ML_PG(point_grad_row_f32_kernel, float);
        }
#undef ML_PG
        return cudaGetLastError();
    }
    *used_rows = false;
    dim3 g((P + 255) / 256, (unsigned)rows);
    if (foc) point_grad_global_focal_kernel<<<g, 256, 0, st>>>(la, zs, scoords, scodes, P, align, gacc);
    else point_grad_global_kernel<<<g, 256, 0, st>>>(la, zs, scoords, scodes, P, align, gacc);
    return cudaGetLastError();
}

cudaError_t launch_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t st) {
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, 65535);
    f32_to_bf16_kernel<<<(unsigned)blocks, 256, 0, st>>>(src, static_cast<__nv_bfloat16*>(dst), n);
    return cudaGetLastError();
}

}  // namespace mlb
