// semantic.cu -- standalone semantic losses over C class channels.
//
// Replaces forward/backward_sigmoid_ce_loss (src/cuda/sigmoid_ce.cu:13-332)
// and forward/backward_dice_loss (src/cuda/dice_loss.cu:13-288): per-layer
// BCE (optionally focal) and dice of (L,B,C,H,W) logits against a (B,H_t,W_t)
// label map with classes in [0,C), every logit standing for an s x s block of
// target pixels (nearest upsampling).
//
// Layout: one block per (image, run of consecutive cells, slice of classes),
// one thread per cell (four for the dice forward, which amortises its warp
// sums over them).  A thread reads its cell's s*s labels once, keeps up to
// four (label, count) pairs in registers (cells with more labels count on
// demand), then streams the cell's logits of its class slice plane by plane
// -- coalesced across the block, each logit read once.  The class slices give
// the grid enough blocks to keep HBM busy at a few images.  All sums use
// fixed-order reductions (per-block partials, then a finalize pass), so the
// results are deterministic; the reference accumulates with atomics.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

namespace {

constexpr int kSemThreads = 256;
constexpr int kClassBatch = 8;       // class planes loaded together per thread
constexpr int kDiceClassBatch = 4;   // dice forward: x kDiceCells cells

struct CellLabels {
    int lab[4];
    int cnt[4];
    int n;
    bool over;  // more than four labels in the cell: count per class on demand
};

ML_INLINE void add_label(CellLabels& r, int64_t v, int C) {
    if (v < 0 || v >= C) return;  // out-of-range labels count for no class
    const int lab = (int)v;
    bool found = false;
#pragma unroll
    for (int k = 0; k < 4; ++k)
        if (k < r.n && r.lab[k] == lab) { ++r.cnt[k]; found = true; }
    if (found) return;
    if (r.n < 4) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (k == r.n) { r.lab[k] = lab; r.cnt[k] = 1; }
        ++r.n;
    } else {
        r.over = true;
    }
}

ML_INLINE CellLabels empty_labels() {
    CellLabels r;
#pragma unroll
    for (int k = 0; k < 4; ++k) { r.lab[k] = -1; r.cnt[k] = 0; }
    r.n = 0;
    r.over = false;
    return r;
}

// Small fixed factors: all S*S label loads are issued before any is used.
template <int S>
ML_INLINE CellLabels cell_labels_t(const int64_t* r0, int Wt, int C) {
    int64_t v[S * S];
#pragma unroll
    for (int dy = 0; dy < S; ++dy)
#pragma unroll
        for (int dx = 0; dx < S; ++dx) v[dy * S + dx] = r0[(int64_t)dy * Wt + dx];
    CellLabels r = empty_labels();
#pragma unroll
    for (int k = 0; k < S * S; ++k) add_label(r, v[k], C);
    return r;
}

ML_INLINE CellLabels cell_labels(const int64_t* tb, int cell, int W, int Wt, int s, int C) {
    const int ci = cell / W, cj = cell - ci * W;
    const int64_t* r0 = tb + (int64_t)(ci * s) * Wt + (int64_t)cj * s;
    switch (s) {
        case 1: return cell_labels_t<1>(r0, Wt, C);
        case 2: return cell_labels_t<2>(r0, Wt, C);
        case 3: return cell_labels_t<3>(r0, Wt, C);
        case 4: return cell_labels_t<4>(r0, Wt, C);
        default: break;
    }
    CellLabels r = empty_labels();
    for (int dy = 0; dy < s; ++dy)
        for (int dx = 0; dx < s; ++dx) add_label(r, r0[(int64_t)dy * Wt + dx], C);
    return r;
}

// Pixels of class c in the cell.
ML_INLINE float class_count(const CellLabels& cl, int c, const int64_t* tb, int cell, int W, int Wt,
                            int s) {
    if (!cl.over) {
        int n = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) n += cl.lab[k] == c ? cl.cnt[k] : 0;
        return (float)n;
    }
    const int ci = cell / W, cj = cell - ci * W;
    const int64_t* r0 = tb + (int64_t)(ci * s) * Wt + (int64_t)cj * s;
    int n = 0;
    for (int dy = 0; dy < s; ++dy)
        for (int dx = 0; dx < s; ++dx) n += r0[(int64_t)dy * Wt + dx] == c;
    return (float)n;
}

ML_INLINE double block_sum_d(double v, double* sh /* [32] */) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double t = 0.0;
    if (threadIdx.x == 0)
        for (int w = 0; w < nw; ++w) t += sh[w];
    return t;  // valid in thread 0
}

}  // namespace

// ---------------------------------------------------------------------------
// Sigmoid CE forward: per (l, b, block) the sum over the block's cells and all
// classes of  alpha+ * m+ * softplus(-x) * n_c + alpha- * m- * softplus(x) * (s^2 - n_c)
// (src/cuda/sigmoid_ce.cu:13-114).  part_d: (L, B, ncs, nblk) double.
// ---------------------------------------------------------------------------
template <bool FOC>
__device__ __forceinline__ void sce_fwd_body(const SemArgs& a) {
    __shared__ double sh[32];
    const int b = blockIdx.y;
    const int HW = a.H * a.W;
    const int cell = blockIdx.x * blockDim.x + threadIdx.x;
    const bool valid = cell < HW;
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;
    CellLabels cl;
    if (valid) cl = cell_labels(tb, cell, a.W, a.Wt, a.s, a.C);
    const Focal f = make_focal(a.gamma, a.alpha);
    const float N2 = (float)(a.s * a.s);
    const int c0 = blockIdx.z * a.cps, c1 = min(a.C, c0 + a.cps);
    for (int l = 0; l < a.L; ++l) {
        float acc = 0.0f;
        if (valid) {
            const float* x = a.logits + ((int64_t)l * a.B + b) * a.C * HW + cell;
            for (int cb = c0; cb < c1; cb += kClassBatch) {
                float xv[kClassBatch];  // all loads of the batch in flight first
#pragma unroll
                for (int k = 0; k < kClassBatch; ++k)
                    xv[k] = cb + k < c1 ? __ldcs(x + (int64_t)(cb + k) * HW) : 0.0f;
#pragma unroll
                for (int k = 0; k < kClassBatch; ++k) {
                    if (cb + k >= c1) break;
                    const Elem e = elem(xv[k]);
                    const float n = class_count(cl, cb + k, tb, cell, a.W, a.Wt, a.s);
                    const float lp = FOC ? focal_pos(f, e) : f.alpha_pos * e.pos;
                    const float ln = FOC ? focal_neg(f, e) : f.alpha_neg * e.neg;
                    acc += lp * n + ln * (N2 - n);
                }
            }
        }
        const double t = block_sum_d((double)acc, sh);
        if (threadIdx.x == 0)
            a.part_d[(((int64_t)l * a.B + b) * a.ncs + blockIdx.z) * gridDim.x + blockIdx.x] = t;
    }
}

__global__ void __launch_bounds__(kSemThreads) sce_fwd_kernel(SemArgs a) { sce_fwd_body<false>(a); }
__global__ void __launch_bounds__(kSemThreads) sce_fwd_focal_kernel(SemArgs a) { sce_fwd_body<true>(a); }

// out[l] = scale * sum_{b,blocks} part / (num_masks * H_t * W_t); grid = L.
__global__ void __launch_bounds__(kSemThreads) sce_finalize_kernel(SemArgs a, int nblk) {
    __shared__ double sh[32];
    const int l = blockIdx.x;
    double v = 0.0;
    const int64_t n = (int64_t)a.B * a.ncs * nblk;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) v += a.part_d[(int64_t)l * n + i];
    const double t = block_sum_d(v, sh);
    if (threadIdx.x == 0)
        a.out[l] = (float)(t * (double)a.scale) / (a.num_masks * (float)a.Ht * (float)a.Wt);
}

// ---------------------------------------------------------------------------
// Sigmoid CE backward (src/cuda/sigmoid_ce.cu:116-205): elementwise
// g = -a+ n m+ (gamma p ce+ + 1 - p) + a- (s^2 - n) m- (gamma (1-p) ce- + p),
// times grad_out[l] * scale / (num_masks * H_t * W_t).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kSemThreads) sce_bwd_kernel(SemArgs a) {
    const int b = blockIdx.y;
    const int HW = a.H * a.W;
    const int cell = blockIdx.x * blockDim.x + threadIdx.x;
    if (cell >= HW) return;
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;
    const CellLabels cl = cell_labels(tb, cell, a.W, a.Wt, a.s, a.C);
    const Focal f = make_focal(a.gamma, a.alpha);
    const float N2 = (float)(a.s * a.s);
    const float norm = a.scale / (a.num_masks * (float)a.Ht * (float)a.Wt);
    for (int l = 0; l < a.L; ++l) {
        const float go = a.grad_out[l] * norm;
        const int64_t base = ((int64_t)l * a.B + b) * a.C * HW + cell;
        const int c0 = blockIdx.z * a.cps, c1 = min(a.C, c0 + a.cps);
        for (int cb = c0; cb < c1; cb += kClassBatch) {
            float xv[kClassBatch];
#pragma unroll
            for (int k = 0; k < kClassBatch; ++k)
                xv[k] = cb + k < c1 ? __ldcs(a.logits + base + (int64_t)(cb + k) * HW) : 0.0f;
#pragma unroll
            for (int k = 0; k < kClassBatch; ++k) {
                if (cb + k >= c1) break;
                const Elem e = elem(xv[k]);
                const float n = class_count(cl, cb + k, tb, cell, a.W, a.Wt, a.s);
                const float om = 1.0f - e.p;
                const float mp = f.use_gamma ? __powf(om, f.gamma) : 1.0f;
                const float mn = f.use_gamma ? __powf(e.p, f.gamma) : 1.0f;
                const float gp = -f.alpha_pos * n * mp * (f.gamma * e.p * e.pos + om);
                const float gn = f.alpha_neg * (N2 - n) * mn * (f.gamma * om * e.neg + e.p);
                __stcs(a.grad + base + (int64_t)(cb + k) * HW, (gp + gn) * go);
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Dice forward (src/cuda/dice_loss.cu:13-82): per (l,b,c) the block's partial
// I = sum p n_c and sum p (P = s^2 * sum p), and (class slice 0) per (b,c) the
// block's label histogram (T).  A thread covers kDiceCells cells spaced one
// block apart, so each warp sum covers 32 * kDiceCells logits.
// Dynamic shared memory: (nwarps * 2 * cps + C) words.
// ---------------------------------------------------------------------------
constexpr int kDiceCells = 4;

__global__ void __launch_bounds__(kSemThreads) dice_fwd_kernel(SemArgs a) {
    extern __shared__ float dsm[];
    const int nw = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = a.C, cps = a.cps;
    float* ws = dsm;                                                 // [nw][2][cps]
    int* hist = reinterpret_cast<int*>(dsm + (size_t)nw * 2 * cps);  // [C]
    const int b = blockIdx.y;
    const int HW = a.H * a.W;
    const int nblk = gridDim.x;
    const int c0 = blockIdx.z * cps, c1 = min(C, c0 + cps);
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;
    const int cell0 = blockIdx.x * blockDim.x * kDiceCells + threadIdx.x;
    CellLabels cl[kDiceCells];
    bool valid[kDiceCells];
#pragma unroll
    for (int k = 0; k < kDiceCells; ++k) {
        const int cell = cell0 + k * blockDim.x;
        valid[k] = cell < HW;
        if (valid[k]) cl[k] = cell_labels(tb, cell, a.W, a.Wt, a.s, C);
    }
    if (blockIdx.z == 0) {
        for (int c = threadIdx.x; c < C; c += blockDim.x) hist[c] = 0;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kDiceCells; ++k) {
            if (!valid[k]) continue;
            if (!cl[k].over) {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (j < cl[k].n) atomicAdd(&hist[cl[k].lab[j]], cl[k].cnt[j]);
            } else {
                const int cell = cell0 + k * blockDim.x;
                const int ci = cell / a.W, cj = cell - ci * a.W;
                const int64_t* r0 = tb + (int64_t)(ci * a.s) * a.Wt + (int64_t)cj * a.s;
                for (int dy = 0; dy < a.s; ++dy)
                    for (int dx = 0; dx < a.s; ++dx) {
                        const int64_t v = r0[(int64_t)dy * a.Wt + dx];
                        if (v >= 0 && v < C) atomicAdd(&hist[(int)v], 1);
                    }
            }
        }
        __syncthreads();
        for (int c = threadIdx.x; c < C; c += blockDim.x)
            a.part_t[((int64_t)b * nblk + blockIdx.x) * C + c] = hist[c];
    }
    for (int l = 0; l < a.L; ++l) {
        const float* x = a.logits + ((int64_t)l * a.B + b) * C * HW;
        for (int cb = c0; cb < c1; cb += kDiceClassBatch) {
            float xv[kDiceClassBatch][kDiceCells];  // all loads of the batch in flight first
#pragma unroll
            for (int j = 0; j < kDiceClassBatch; ++j)
#pragma unroll
                for (int k = 0; k < kDiceCells; ++k)
                    xv[j][k] = (cb + j < c1 && valid[k])
                                   ? __ldcs(x + (int64_t)(cb + j) * HW + cell0 + k * blockDim.x)
                                   : 0.0f;
#pragma unroll
            for (int j = 0; j < kDiceClassBatch; ++j) {
                const int c = cb + j;
                if (c >= c1) break;
                float pi = 0.0f, pp = 0.0f;
#pragma unroll
                for (int k = 0; k < kDiceCells; ++k) {
                    if (!valid[k]) continue;
                    const float p = elem(xv[j][k]).p;
                    pi += p * class_count(cl[k], c, tb, cell0 + k * blockDim.x, a.W, a.Wt, a.s);
                    pp += p;
                }
                pi = warp_sum(pi);
                pp = warp_sum(pp);
                if (lane == 0) { ws[(warp * 2) * cps + (c - c0)] = pi; ws[(warp * 2 + 1) * cps + (c - c0)] = pp; }
            }
        }
        __syncthreads();
        const int64_t o = (((int64_t)l * a.B + b) * nblk + blockIdx.x) * C;
        for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
            float si = 0.0f, sp = 0.0f;
            for (int w = 0; w < nw; ++w) {
                si += ws[(w * 2) * cps + (c - c0)];
                sp += ws[(w * 2 + 1) * cps + (c - c0)];
            }
            a.part_f[2 * o + c] = si;
            a.part_f[2 * o + C + c] = sp;
        }
        __syncthreads();
    }
}

// I, P, T per (l,b,c) and the per-(l,b) sum of 1 - dice; grid = L*B.
__global__ void __launch_bounds__(kSemThreads) dice_reduce_kernel(SemArgs a, int nblk) {
    __shared__ double sh[32];
    const int lb = blockIdx.x, b = lb % a.B;
    const int C = a.C;
    const float N2 = (float)(a.s * a.s);
    double loss = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float I = 0.0f, P = 0.0f;
        int T = 0;
        for (int k = 0; k < nblk; ++k) {
            const int64_t o = ((int64_t)lb * nblk + k) * C;
            I += a.part_f[2 * o + c];
            P += a.part_f[2 * o + C + c];
            T += a.part_t[((int64_t)b * nblk + k) * C + c];
        }
        P *= N2;
        const float Tf = (float)T;
        a.I[(int64_t)lb * C + c] = I;
        a.P[(int64_t)lb * C + c] = P;
        a.T[(int64_t)lb * C + c] = Tf;
        const float dice = (2.0f * I + a.smooth) / (P + Tf + a.smooth);
        loss += (double)(1.0f - dice);
    }
    const double t = block_sum_d(loss, sh);
    if (threadIdx.x == 0) a.part_d[lb] = t;
}

// out[l] = scale * sum_b part[l,b] / num_masks; one block.
__global__ void dice_finalize_kernel(SemArgs a) {
    for (int l = threadIdx.x; l < a.L; l += blockDim.x) {
        double t = 0.0;
        for (int b = 0; b < a.B; ++b) t += a.part_d[(int64_t)l * a.B + b];
        a.out[l] = (float)t / a.num_masks * a.scale;
    }
}

// Dice backward (src/cuda/dice_loss.cu:84-157): elementwise
// -grad_out[l] * scale / num_masks * (2 n (P+T+smooth) - s^2 (2I+smooth)) / den^2 * p(1-p).
__global__ void __launch_bounds__(kSemThreads) dice_bwd_kernel(SemArgs a) {
    const int b = blockIdx.y;
    const int HW = a.H * a.W;
    const int cell = blockIdx.x * blockDim.x + threadIdx.x;
    if (cell >= HW) return;
    const int64_t* tb = a.targets + (int64_t)b * a.Ht * a.Wt;
    const CellLabels cl = cell_labels(tb, cell, a.W, a.Wt, a.s, a.C);
    const float N2 = (float)(a.s * a.s);
    for (int l = 0; l < a.L; ++l) {
        const float go = -a.grad_out[l] / a.num_masks * a.scale;
        const int64_t lb = (int64_t)l * a.B + b;
        const int64_t base = lb * a.C * HW + cell;
        const int c0 = blockIdx.z * a.cps, c1 = min(a.C, c0 + a.cps);
        for (int cb = c0; cb < c1; cb += kClassBatch) {
            float xv[kClassBatch];
#pragma unroll
            for (int k = 0; k < kClassBatch; ++k)
                xv[k] = cb + k < c1 ? __ldcs(a.logits + base + (int64_t)(cb + k) * HW) : 0.0f;
#pragma unroll
            for (int k = 0; k < kClassBatch; ++k) {
                const int c = cb + k;
                if (c >= c1) break;
                const float p = elem(xv[k]).p;
                const float n = class_count(cl, c, tb, cell, a.W, a.Wt, a.s);
                const float I = a.I[lb * a.C + c], P = a.P[lb * a.C + c], T = a.T[lb * a.C + c];
                const float den = P + T + a.smooth;
                const float d = (2.0f * n * den - N2 * (2.0f * I + a.smooth)) / (den * den);
                __stcs(a.grad + base + (int64_t)c * HW, go * d * (p * (1.0f - p)));
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Launchers (non-template entry points called from capi.cu).
// ---------------------------------------------------------------------------
int sem_blocks(const SemArgs& a) { return (a.H * a.W + kSemThreads - 1) / kSemThreads; }
int dice_blocks(const SemArgs& a) {
    return (a.H * a.W + kSemThreads * kDiceCells - 1) / (kSemThreads * kDiceCells);
}

// Class slices: about 4 blocks per SM of a 148-SM part (more slices re-read
// the labels more often than they add parallelism).
void sem_slices(SemArgs* a, int blocks_per_slice) {
    const int64_t want = 148 * 4;
    const int64_t per = (int64_t)blocks_per_slice * a->B;
    int ncs = (int)std::max<int64_t>(1, std::min<int64_t>(a->C, (want + per - 1) / std::max<int64_t>(per, 1)));
    if (ncs > 65535) ncs = 65535;
    a->cps = std::max(1, (a->C + ncs - 1) / ncs);
    a->ncs = std::max(1, (a->C + a->cps - 1) / a->cps);
}

cudaError_t launch_sce_forward(SemArgs a, cudaStream_t st) {
    const int nblk = sem_blocks(a);
    dim3 g(nblk, a.B, a.ncs);
    if (a.gamma > 0.0f) sce_fwd_focal_kernel<<<g, kSemThreads, 0, st>>>(a);
    else sce_fwd_kernel<<<g, kSemThreads, 0, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    sce_finalize_kernel<<<a.L, kSemThreads, 0, st>>>(a, nblk);
    return cudaGetLastError();
}

cudaError_t launch_sce_backward(SemArgs a, cudaStream_t st) {
    sce_bwd_kernel<<<dim3(sem_blocks(a), a.B, a.ncs), kSemThreads, 0, st>>>(a);
    return cudaGetLastError();
}

size_t dice_fwd_smem(int C, int cps) {
    return sizeof(float) * ((size_t)(kSemThreads / 32) * 2 * cps + C);
}

cudaError_t launch_dice_forward(SemArgs a, cudaStream_t st) {
    const int nblk = dice_blocks(a);
    const size_t smem = dice_fwd_smem(a.C, a.cps);
    cudaError_t e = cudaFuncSetAttribute(dice_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    dice_fwd_kernel<<<dim3(nblk, a.B, a.ncs), kSemThreads, smem, st>>>(a);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    dice_reduce_kernel<<<a.L * a.B, kSemThreads, 0, st>>>(a, nblk);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    dice_finalize_kernel<<<1, 128, 0, st>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_dice_backward(SemArgs a, cudaStream_t st) {
    dice_bwd_kernel<<<dim3(sem_blocks(a), a.B, a.ncs), kSemThreads, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace mlb
