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
// per-query row sums.  k is one-hot for s = H_t/H = 1 and for every "pure"
// cell when s > 1, so the contraction is a segmented sum over the cell
// stream.  Every query of a CTA walks the SAME label sequence, so label runs
// are uniform across the CTA: a thread (one query row, one half of each tile)
// accumulates the current run in registers and flushes it only when the label
// changes, with an ordered `red.add` into a CTA-private slice of a global
// partial buffer (a thread's same-address reductions apply in program order,
// so the sums are deterministic).  Tiles whose 32 cells carry one label --
// most of an image -- take a branch-free path.  Mixed cells (s > 1 on a label
// boundary) add the (column, pixel count) pairs of their table entry.
//
// Data movement: a prep kernel turns the int64 label map into one int32 code
// per low-res cell, the mixed-cell table (s > 1) and the per-image histogram
// once; the cost kernel then streams logits tiles of (qrows x 64 cells) with
// two cp.async.bulk.tensor boxes (128-byte swizzle for fp32, 64-byte for
// bf16/fp16; conflict-free 128-bit reads) plus the tile's 256 bytes of codes
// with one cp.async.bulk, all on one mbarrier, through a 2-stage pipeline.
// Logits are read from HBM exactly once.
//
// The HW axis is split into chunks across CTAs (grid.x) sized to whole waves
// of the 148 SMs; two finalize kernels reduce the chunk partials in fixed
// order.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

// ---------------------------------------------------------------------------
// Prep: per-cell code (pure output column / kNone / kMixed), the mixed-cell
// table (s > 1) and the per-image label histogram totals[b, lab], lab in
// [0, GT_total) (the counts.sum({2,3}) of src/cuda/pw_mask.cu:391).  Each of
// the three outputs may be null.  One low-res cell per thread; S is s at
// compile time (0: read from `s_rt`), so a thread issues all s*s label loads
// before it looks at any.  grid = (cell blocks, B).
// ---------------------------------------------------------------------------
template <int S>
__global__ void __launch_bounds__(256)
label_code_kernel(const int64_t* __restrict__ targets, int B, int H, int W, int Wt, int s_rt,
                  int gt_total, int bg, int32_t* __restrict__ codes, int32_t* __restrict__ totals,
                  uint4* __restrict__ mixtab) {
    extern __shared__ int32_t hist[];
    const int s = S > 0 ? S : s_rt;
    const int b = blockIdx.y;
    const bool use_sh = totals && gt_total <= kHistSmemMax;
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int HW = H * W;
    const int64_t* tb = targets + (int64_t)b * HW * s * s;
    int32_t* cb = codes ? codes + (int64_t)b * HW : nullptr;
    int32_t* tot = totals ? totals + (int64_t)b * gt_total : nullptr;
    int32_t* hc = use_sh ? hist : tot;  // null: no histogram
    const bool tab = mixtab != nullptr && s > 1;
    // even S, even row pitch and a 16-byte aligned map: 16-byte label loads
    const bool vec = (S % 2 == 0) && (Wt % 2 == 0) &&
                     (reinterpret_cast<uintptr_t>(targets) & 15) == 0;
    // every thread of the block runs the same number of iterations, so the
    // warp-aggregated count below sees the whole warp
    for (int base = blockIdx.x * blockDim.x; base < HW; base += gridDim.x * blockDim.x) {
        const int cell = base + threadIdx.x;
        int run = -1, rc = 0;  // this cell's last run of one in-range label
        if (cell < HW) {
            int c = -3;
            uint32_t e[4] = {0u, 0u, 0u, 0u};  // (col + 1, count) of the cell's columns
            bool wide = false;
            const int ci = cell / W, cj = cell - ci * W;
            const int64_t* r0 = tb + (int64_t)(ci * s) * Wt + (int64_t)cj * s;
            auto pixel = [&](int64_t lab) {  // histogram runs + cell code
                const int key = (lab >= 0 && lab < gt_total) ? (int)lab : -1;
                if (key != run) {
                    if (run >= 0 && hc) atomicAdd(&hc[run], rc);
                    run = key;
                    rc = 0;
                }
                ++rc;
                const int col = label_to_col(lab, gt_total, bg);
                c = (c == -3 || c == col) ? col : kMixed;
            };
            auto table = [&](int64_t lab) {  // mixed cells only
                const int col = label_to_col(lab, gt_total, bg);
                if (col < 0) return;
                // slots fill in order, so a column already held sits before
                // the first empty slot
                const uint32_t kc = (uint32_t)(col + 1) << 16;
                bool done = false;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    if (!done && (e[i] & 0xFFFF0000u) == kc) { e[i] += 1u; done = true; }
                    else if (!done && e[i] == 0u) { e[i] = kc | 1u; done = true; }
                }
                wide |= !done;
            };
            if (S > 0) {
                constexpr int N = S > 0 ? S * S : 1;
                int64_t v[N];
                if (vec) {  // rows of S labels as 16-byte pairs
#pragma unroll
                    for (int dy = 0; dy < S; ++dy)
#pragma unroll
                        for (int dx = 0; dx < S; dx += 2) {
                            const longlong2 t2 =
                                *reinterpret_cast<const longlong2*>(r0 + (int64_t)dy * Wt + dx);
                            v[dy * S + dx] = t2.x;
                            v[dy * S + dx + 1] = t2.y;
                        }
                } else {
#pragma unroll
                    for (int dy = 0; dy < S; ++dy)
#pragma unroll
                        for (int dx = 0; dx < S; ++dx) v[dy * S + dx] = r0[(int64_t)dy * Wt + dx];
                }
                bool same = true;
#pragma unroll
                for (int i = 1; i < N; ++i) same &= v[i] == v[0];
                if (same) {  // most cells: one label
                    run = (v[0] >= 0 && v[0] < gt_total) ? (int)v[0] : -1;
                    rc = N;
                    c = label_to_col(v[0], gt_total, bg);
                } else {
#pragma unroll
                    for (int i = 0; i < N; ++i) pixel(v[i]);
                    if (tab && c == kMixed) {
#pragma unroll
                        for (int i = 0; i < N; ++i) table(v[i]);
                    }
                }
            } else {
                for (int dy = 0; dy < s; ++dy)
                    for (int dx = 0; dx < s; ++dx) pixel(r0[(int64_t)dy * Wt + dx]);
                if (tab && c == kMixed)
                    for (int dy = 0; dy < s; ++dy)
                        for (int dx = 0; dx < s; ++dx) table(r0[(int64_t)dy * Wt + dx]);
            }
            if (cb) cb[cell] = c;
            if (tab && c == kMixed)
                mixtab[(int64_t)b * HW + cell] =
                    wide ? make_uint4(kMixWide, 0u, 0u, 0u) : make_uint4(e[0], e[1], e[2], e[3]);
        }
        // lanes whose last runs share a label add them with one atomic
        if (hc) {
            const unsigned peers = __match_any_sync(0xffffffffu, run);
            const int n = (int)__reduce_add_sync(peers, (unsigned)rc);
            if (run >= 0 && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hc[run], n);
        }
    }
    __syncthreads();
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x)
            if (hist[i]) atomicAdd(&tot[i], hist[i]);
}

// Histogram only, over the flat label map of each image (any shape): a thread
// counts 8 consecutive pixels as runs in registers; runs that end inside its
// pixels go straight to the shared histogram, and the warp adds the last runs
// with one atomic per label.  grid = (pixel blocks, B).
__global__ void __launch_bounds__(256)
label_hist_kernel(const int64_t* __restrict__ targets, int64_t npix, int gt_total,
                  int32_t* __restrict__ totals) {
    extern __shared__ int32_t hist[];
    const int b = blockIdx.y;
    const bool use_sh = gt_total <= kHistSmemMax;
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    const int64_t* tb = targets + (int64_t)b * npix;
    int32_t* tot = totals + (int64_t)b * gt_total;
    int32_t* hc = use_sh ? hist : tot;
    const bool vec = (reinterpret_cast<uintptr_t>(tb) & 15) == 0;
    const int64_t step = (int64_t)gridDim.x * blockDim.x * 8;
    for (int64_t base = ((int64_t)blockIdx.x * blockDim.x) * 8; base < npix; base += step) {
        const int64_t p0 = base + (int64_t)threadIdx.x * 8;
        int64_t v[8];
        if (vec && p0 + 8 <= npix) {
            const longlong2* q = reinterpret_cast<const longlong2*>(tb + p0);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const longlong2 t2 = q[i];
                v[2 * i] = t2.x;
                v[2 * i + 1] = t2.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = p0 + i < npix ? tb[p0 + i] : -1;
        }
        int run = -1, rc = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int key = (v[i] >= 0 && v[i] < gt_total) ? (int)v[i] : -1;
            if (key != run) {
                if (run >= 0) atomicAdd(&hc[run], rc);
                run = key;
                rc = 0;
            }
            ++rc;
        }
        const unsigned peers = __match_any_sync(0xffffffffu, run);
        const int n = (int)__reduce_add_sync(peers, (unsigned)rc);
        if (run >= 0 && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hc[run], n);
    }
    __syncthreads();
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x)
            if (hist[i]) atomicAdd(&tot[i], hist[i]);
}

cudaError_t launch_label_hist(const int64_t* targets, int B, int64_t npix, int gt_total,
                              int32_t* totals, cudaStream_t st) {
    if (B <= 0 || npix <= 0 || gt_total <= 0) return cudaSuccess;
    const int64_t want = (npix + 8 * 256 - 1) / (8 * 256);
    const int bx = (int)std::max<int64_t>(1, std::min<int64_t>(want, 65535));
    const size_t hs = gt_total <= kHistSmemMax ? sizeof(int32_t) * gt_total : 0;
    label_hist_kernel<<<dim3(bx, B), 256, hs, st>>>(targets, npix, gt_total, totals);
    return cudaGetLastError();
}

// s = 1 with H*W a multiple of 8 and 16-byte aligned maps: eight cells per
// thread (four 16-byte label loads issued together, two 16-byte code
// stores); the histogram counts the thread's runs in registers and adds the
// warp's last runs with one atomic per label, like label_hist_kernel.
__global__ void __launch_bounds__(256)
label_code_s1_kernel(const int64_t* __restrict__ targets, int HW, int gt_total, int bg,
                     int32_t* __restrict__ codes, int32_t* __restrict__ totals) {
    extern __shared__ int32_t hist[];
    const int b = blockIdx.y;
    const bool use_sh = totals && gt_total <= kHistSmemMax;
    if (use_sh)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x) hist[i] = 0;
    __syncthreads();
    int32_t* hc = use_sh ? hist : (totals ? totals + (int64_t)b * gt_total : nullptr);
    const int64_t* tb = targets + (int64_t)b * HW;
    int32_t* cb = codes + (int64_t)b * HW;
    for (int base = blockIdx.x * blockDim.x * 8; base < HW; base += gridDim.x * blockDim.x * 8) {
        const int c0 = base + (int)threadIdx.x * 8;
        int run = -1, rc = 0;
        if (c0 < HW) {
            int64_t v[8];
            const longlong2* q = reinterpret_cast<const longlong2*>(tb + c0);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const longlong2 t2 = q[i];
                v[2 * i] = t2.x;
                v[2 * i + 1] = t2.y;
            }
            int c[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                c[i] = label_to_col(v[i], gt_total, bg);
                const int key = (v[i] >= 0 && v[i] < gt_total) ? (int)v[i] : -1;
                if (key != run) {
                    if (run >= 0 && hc) atomicAdd(&hc[run], rc);
                    run = key;
                    rc = 0;
                }
                ++rc;
            }
            reinterpret_cast<int4*>(cb + c0)[0] = make_int4(c[0], c[1], c[2], c[3]);
            reinterpret_cast<int4*>(cb + c0)[1] = make_int4(c[4], c[5], c[6], c[7]);
        }
        if (hc) {
            const unsigned peers = __match_any_sync(0xffffffffu, run);
            const int n = (int)__reduce_add_sync(peers, (unsigned)rc);
            if (run >= 0 && (int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hc[run], n);
        }
    }
    __syncthreads();
    if (use_sh && totals)
        for (int i = threadIdx.x; i < gt_total; i += blockDim.x)
            if (hist[i]) atomicAdd(&totals[(int64_t)b * gt_total + i], hist[i]);
}

cudaError_t launch_label_code(const int64_t* targets, int B, int H, int W, int Wt, int s,
                              int gt_total, int bg, int32_t* codes, int32_t* totals, uint4* mixtab,
                              cudaStream_t st) {
    const int HW = H * W;
    if (B <= 0 || HW <= 0) return cudaSuccess;
    if (s == 1 && codes && HW % 8 == 0 && (reinterpret_cast<uintptr_t>(targets) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(codes) & 15) == 0) {
        const int bx = std::max(1, std::min((HW / 8 + 255) / 256, 65535));
        const size_t hs = (totals && gt_total <= kHistSmemMax) ? sizeof(int32_t) * gt_total : 0;
        label_code_s1_kernel<<<dim3(bx, B), 256, hs, st>>>(targets, HW, gt_total, bg, codes, totals);
        return cudaGetLastError();
    }
    const int bx = std::max(1, std::min((HW + 255) / 256, 65535));
    const size_t hs = (totals && gt_total <= kHistSmemMax) ? sizeof(int32_t) * gt_total : 0;
    const dim3 grid(bx, B);
    switch (s) {
        case 1: label_code_kernel<1><<<grid, 256, hs, st>>>(targets, B, H, W, Wt, s, gt_total, bg, codes, totals, mixtab); break;
        case 2: label_code_kernel<2><<<grid, 256, hs, st>>>(targets, B, H, W, Wt, s, gt_total, bg, codes, totals, mixtab); break;
        case 4: label_code_kernel<4><<<grid, 256, hs, st>>>(targets, B, H, W, Wt, s, gt_total, bg, codes, totals, mixtab); break;
        default: label_code_kernel<0><<<grid, 256, hs, st>>>(targets, B, H, W, Wt, s, gt_total, bg, codes, totals, mixtab); break;
    }
    return cudaGetLastError();
}

// Element pieces for the default path: fast_elem (common.cuh).

// red.add into the partial buffer (program order per address -> deterministic).
ML_INLINE void red_add(float* p, float v) {
    asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// Mixed cell (s > 1 on a label boundary) with table entry `e`: one red.add
// per column of the cell and accumulator, weighted by the column's pixel
// count.  Without a table (tab false) or for a wide cell, one red.add per
// pixel from the label map.
template <bool UNC>
__device__ __forceinline__ void mixed_cell(const int64_t* targets, const uint4& e, bool tab, int W,
                                           int Ht, int Wt, int s, int gt_total, int bg, float* part,
                                           int b, int cell, int t, int QP, int G, float dl, float wp,
                                           float w) {
    if (tab && e.x != kMixWide) {
        const uint32_t v[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (v[i] == 0u) break;
            const float n = mix_cnt(v[i]);
            float* pc = part + (int64_t)mix_col(v[i]) * QP + t;
            red_add(pc, n * dl);
            red_add(pc + (int64_t)G * QP, n * wp);
            if (UNC) red_add(pc + 2 * (int64_t)G * QP, n * w);
        }
        return;
    }
    const int ci = cell / W, cj = cell - ci * W;
    const int64_t* r0 = targets + ((int64_t)b * Ht + (int64_t)ci * s) * Wt + (int64_t)cj * s;
    for (int pp = 0; pp < s * s; ++pp) {
        const int col = label_to_col(r0[(int64_t)(pp / s) * Wt + (pp % s)], gt_total, bg);
        if (col >= 0) {
            float* pc = part + (int64_t)col * QP + t;
            red_add(pc, dl);
            red_add(pc + (int64_t)G * QP, wp);
            if (UNC) red_add(pc + 2 * (int64_t)G * QP, w);
        }
    }
}

// ---------------------------------------------------------------------------
// Shared-memory layout of one 32-cell box row, per logit type.  The TMA box
// rows are 128 bytes (fp32, 128-byte swizzle: 16-byte granule g of row r at
// g ^ (r & 7)) or 64 bytes (16-bit, 64-byte swizzle: g ^ ((r >> 1) & 3)); both
// keep a warp's 128-bit row reads conflict-free.  GR = elements per granule.
// ---------------------------------------------------------------------------
template <typename T> struct Tile {
    static constexpr int GR = 16 / (int)sizeof(T);
    ML_INLINE static int gran(int r, int g) {
        if constexpr (sizeof(T) == 4) return (g ^ (r & 7)) << 2;
        else return (g ^ ((r >> 1) & 3)) << 3;
    }
    ML_INLINE static float at(const T* row, int r, int k) { return to_f(row[gran(r, k / GR) + k % GR]); }
    // elements [8o, 8o + 8) of the row
    ML_INLINE static void octet(const T* row, int r, int o, float (&x)[8]) {
        if constexpr (sizeof(T) == 4) {
            const float* fr = reinterpret_cast<const float*>(row);
            const float4 v0 = *reinterpret_cast<const float4*>(fr + gran(r, 2 * o));
            const float4 v1 = *reinterpret_cast<const float4*>(fr + gran(r, 2 * o + 1));
            x[0] = v0.x; x[1] = v0.y; x[2] = v0.z; x[3] = v0.w;
            x[4] = v1.x; x[5] = v1.y; x[6] = v1.z; x[7] = v1.w;
        } else {
            const uint4 v = *reinterpret_cast<const uint4*>(row + gran(r, o));
            widen2(v.x, x[0], x[1], row);
            widen2(v.y, x[2], x[3], row);
            widen2(v.z, x[4], x[5], row);
            widen2(v.w, x[6], x[7], row);
        }
    }
};

// ---------------------------------------------------------------------------
// The streaming cost kernel.  grid = (nchunk, nqt, L*B); block = 2*qrows_pad
// consumer threads plus one producer warp.  The producer fills a 2-stage ring
// (full/empty mbarriers, no block-wide barrier in the loop); consumer thread
// (h, t) <-> query row qt*qrows + t, cells [h*32, h*32+32) of every 64-cell
// tile.  Inside a box the run starts are one ballot (bnd), so the element
// loop only branches on 4-cell groups that contain a start.  Template flags:
//   UNC   entropy weights on (uncertainty_gamma != 0)
//   FOC   focal gamma/alpha on the mask BCE
//   TMA   logits rows are 16-byte strided so the bulk-tensor path is legal
//   MIX   cells cover several target pixels (s > 1), so mixed cells occur
//   T     mask-logit element type (float, __nv_bfloat16, __half)
// ---------------------------------------------------------------------------
template <bool UNC, bool FOC, bool TMA, bool MIX, typename T>
__global__ void __launch_bounds__(kCostThreads, (MIX && !UNC && !FOC) ? 3 : 2)
cost_partial_kernel(const __grid_constant__ CUtensorMap tmap, CostArgs a) {
    pdl_enter();
    constexpr int NACC = UNC ? 3 : 2;
    constexpr int NROW = UNC ? 5 : 3;
    constexpr bool FAST = !UNC && !FOC;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int QP = a.qrows_pad;
    const int box_elems = QP * KBOX;                   // one 32-cell box
    T* xs = reinterpret_cast<T*>(base);                // [stage][2][QP][32]
    int32_t* cs = reinterpret_cast<int32_t*>(xs + kStages * 2 * box_elems);  // [stage][KC]
    uint64_t* full = reinterpret_cast<uint64_t*>(cs + kStages * KC);
    uint64_t* empty = full + kStages;

    const int tid = threadIdx.x;
    const int ncons = 2 * QP;                          // consumer threads
    const int n_cwarps = ncons / 32;
    const int lane = tid & 31;
    const int lb = blockIdx.z;
    const int b = lb % a.B;
    const int qt = blockIdx.y;
    const int HW = a.H * a.W;
    const int cell_begin = blockIdx.x * a.chunk_cells;
    const int cell_end = min(HW, cell_begin + a.chunk_cells);
    const int ntiles = (cell_end - cell_begin + KC - 1) / KC;
    const int row0 = lb * a.Q + qt * a.qrows;          // first global logits row
    const int32_t* codes_b = a.codes + (int64_t)b * HW;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], n_cwarps);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (tid >= ncons) {
        // ------------------------------ producer warp ------------------------------
        bool ok = true;
        for (int it = 0; it < ntiles && ok; ++it) {
            const int st = it % kStages;
            if (it >= kStages && !mbar_wait(&empty[st], (uint32_t)(((it / kStages) - 1) & 1))) {
                ok = false;
                break;
            }
            const int c0 = cell_begin + it * KC;
            const int nvalid = min(KC, cell_end - c0);
            if (TMA) {
                if (lane == 0) {
                    const uint32_t cbytes = (uint32_t)min(KC, HW - c0) * 4u;
                    mbar_arrive_expect_tx(&full[st], 2u * a.qrows * KBOX * (uint32_t)sizeof(T) + cbytes);
#pragma unroll
                    for (int bx = 0; bx < 2; ++bx)
                        asm volatile(
                            "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
                            " [%0], [%1, {%2, %3}], [%4];"
                            ::"r"(smem_u32(xs + (st * 2 + bx) * box_elems)), "l"(&tmap),
                              "r"(c0 + bx * KBOX), "r"(row0), "r"(smem_u32(&full[st])) : "memory");
                    bulk_g2s(cs + st * KC, codes_b + c0, cbytes, &full[st]);
                }
            } else {
                // plain loads into the same swizzled layout, then one arrive
                constexpr int GR = Tile<T>::GR;
                const T* lg = reinterpret_cast<const T*>(a.logits);
                for (int i = lane; i < 2 * a.qrows * (KBOX / GR); i += 32) {
                    const int bx = i / (a.qrows * (KBOX / GR));
                    const int rem = i - bx * a.qrows * (KBOX / GR);
                    const int r = rem / (KBOX / GR), c = rem - r * (KBOX / GR);
                    const T* src = lg + (int64_t)(row0 + r) * HW + c0 + bx * KBOX + c * GR;
                    // the last query tile can extend one row past Q (qrows =
                    // ceil(Q / nqt)): those rows read as zeros, like the TMA fill
                    const bool row_ok = qt * a.qrows + r < a.Q;
                    alignas(16) T vv[GR];
#pragma unroll
                    for (int u = 0; u < GR; ++u) {
                        const int k = bx * KBOX + c * GR + u;
                        vv[u] = (row_ok && k < nvalid) ? src[u] : from_f<T>(0.0f);
                    }
                    *reinterpret_cast<uint4*>(xs + (st * 2 + bx) * box_elems + r * KBOX +
                                              Tile<T>::gran(r, c)) = *reinterpret_cast<const uint4*>(vv);
                }
                for (int k = lane; k < KC; k += 32) cs[st * KC + k] = k < nvalid ? codes_b[c0 + k] : kNone;
                __syncwarp();
                if (lane == 0) mbar_arrive(&full[st]);
            }
        }
        if (!ok && lane == 0 && a.status) atomicOr(a.status, 2);
        return;
    }

    // ------------------------------- consumers -----------------------------------
    const int h = tid / QP;
    const int t = tid - h * QP;
    const int q = qt * a.qrows + t;
    const bool qvalid = (t < a.qrows) && (q < a.Q);
    const int G = a.gout;
    float* part = a.part + ((((int64_t)lb * a.nqt + qt) * a.nchunk + blockIdx.x) * 2 + h) *
                               (int64_t)a.part_stride;
    const float N2 = (float)(a.s * a.s);
    const Focal foc = make_focal(a.mask_gamma, a.mask_alpha);

    // this thread is the only writer of column t of its slot: clear it here
    // (program order puts these stores before its red.adds)
    for (int x = 0; x < NACC * G; ++x) part[(int64_t)x * QP + t] = 0.0f;
    float racc[NACC];
#pragma unroll
    for (int i = 0; i < NACC; ++i) racc[i] = 0.0f;
    float rows[NROW];
#pragma unroll
    for (int i = 0; i < NROW; ++i) rows[i] = 0.0f;
    int cur = kNone;     // code of the current run (uniform within a warp)
    float m = 0.0f;      // 1 while the current run belongs to an output column
    int run_tiles = 0;
    bool ok = true;

    auto flush = [&]() {
        if (cur >= 0 && qvalid) {
            float* pc = part + (int64_t)cur * QP + t;
            red_add(pc, FAST ? -racc[0] * N2 : racc[0] * N2);
            red_add(pc + (int64_t)G * QP, racc[1] * N2);
            if (UNC) red_add(pc + 2 * (int64_t)G * QP, racc[2] * N2);
        }
#pragma unroll
        for (int i = 0; i < NACC; ++i) racc[i] = 0.0f;
        run_tiles = 0;
    };

    // per-element update of the row sums and the run accumulators.  FAST keeps
    // only tile sums (x, |x|, p); a run's sums of x and p are differences of
    // the tile sums at its ends (close_run), which saves two FMAs per element.
    float trow[NROW] = {};
    float prod = 1.0f;
    float tabs = 0.0f, sx0 = 0.0f, sp0 = 0.0f;
    auto close_run = [&]() {
        if (FAST) {
            racc[0] = fmaf(m, trow[0] - sx0, racc[0]);
            racc[1] = fmaf(m, trow[1] - sp0, racc[1]);
            sx0 = trow[0];
            sp0 = trow[1];
        }
    };
    auto element = [&](float x) {
        if (FAST) {
            const Fast f = fast_elem(x);
            prod *= f.d;
            trow[0] += x;
            tabs += fabsf(x);
            trow[1] += f.p;
        } else {
            const Elem e = elem(x);
            const float w = UNC ? unc_weight(e.p, a.ug, a.ugmin) : 1.0f;
            const float nt = FOC ? focal_neg(foc, e) : e.neg;
            const float dl = FOC ? w * (focal_pos(foc, e) - nt) : -w * x;
            if (UNC) {
                trow[0] += w * nt; trow[1] += w * e.p; trow[2] += w;
                trow[3] += nt; trow[4] += e.p;
            } else {
                trow[0] += nt; trow[1] += e.p;
            }
            racc[0] = fmaf(m, dl, racc[0]);
            racc[1] = fmaf(m, w * e.p, racc[1]);
            if (UNC) racc[2] = fmaf(m, w, racc[2]);
        }
    };
    // A mixed cell is a one-cell run with m = 0 in the element loop (its row
    // sums count there); its contractions are added after the box from the
    // same shared-memory tile, outside the hot loop.
    // `mye` is lane k's table entry for cell k of the box (loaded before the
    // element loop); the warp walks the mixed cells together.
    const bool tab = MIX && a.mixtab != nullptr;
    auto mixed_cells = [&](uint32_t mb, const T* rowp, int cbase, const uint4& mye) {
        while (mb) {
            const int k = __ffs(mb) - 1;
            mb &= mb - 1u;
            uint4 ek;
            ek.x = __shfl_sync(0xffffffffu, mye.x, k);
            ek.y = __shfl_sync(0xffffffffu, mye.y, k);
            ek.z = __shfl_sync(0xffffffffu, mye.z, k);
            ek.w = __shfl_sync(0xffffffffu, mye.w, k);
            if (!qvalid) continue;
            const float x = Tile<T>::at(rowp, t, k);
            if (FAST) {
                const Fast f = fast_elem(x);
                mixed_cell<UNC>(a.targets, ek, tab, a.W, a.Ht, a.Wt, a.s, a.gt_total, a.bg, part, b,
                                cbase + k, t, QP, G, -x, f.p, 1.0f);
            } else {
                const Elem e = elem(x);
                const float w = UNC ? unc_weight(e.p, a.ug, a.ugmin) : 1.0f;
                const float dl = FOC ? w * (focal_pos(foc, e) - focal_neg(foc, e)) : -w * x;
                mixed_cell<UNC>(a.targets, ek, tab, a.W, a.Ht, a.Wt, a.s, a.gt_total, a.bg, part, b,
                                cbase + k, t, QP, G, dl, w * e.p, w);
            }
        }
    };

    for (int it = 0; it < ntiles; ++it) {
        const int st = it % kStages;
        const int cell0 = cell_begin + it * KC;
        const int nvalid = min(KC, cell_end - cell0);
        if (!mbar_wait(&full[st], (uint32_t)((it / kStages) & 1))) { ok = false; break; }
        // this thread's 32 cells: box h of the stage
        const int nv = min(KBOX, max(0, nvalid - h * KBOX));
        const int32_t* code = cs + st * KC + h * KBOX;
        const int my_code = lane < nv ? code[lane] : kNone;
        const int prev = __shfl_up_sync(0xffffffffu, my_code, 1);
        const bool starts = lane < nv && (my_code == kMixed || my_code != (lane == 0 ? cur : prev));
        const uint32_t bnd = __ballot_sync(0xffffffffu, starts);
        const uint32_t mixb = MIX ? __ballot_sync(0xffffffffu, my_code == kMixed) : 0u;
        uint4 mye = make_uint4(0u, 0u, 0u, 0u);
        if (tab && ((mixb >> lane) & 1u)) mye = a.mixtab[(int64_t)b * HW + cell0 + h * KBOX + lane];
        const T* rowp = xs + (st * 2 + h) * box_elems + t * KBOX;
#pragma unroll
        for (int i = 0; i < NROW; ++i) trow[i] = 0.0f;
        prod = 1.0f;
        tabs = sx0 = sp0 = 0.0f;
        if (nv == KBOX) {
            for (int o = 0; o < KBOX / 8; ++o) {
              float xo[8];
              Tile<T>::octet(rowp, t, o, xo);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const int c = 2 * o + j;
                const float xv[4] = {xo[4 * j], xo[4 * j + 1], xo[4 * j + 2], xo[4 * j + 3]};
                const uint32_t b4 = (bnd >> (4 * c)) & 0xFu;
                if (b4 == 0u) {
#pragma unroll
                    for (int u = 0; u < 4; ++u) element(xv[u]);
                } else if (FAST) {
                    // run starts but no mixed cell: the four elements first,
                    // then the run switches between the sums
                    Fast f[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        f[u] = fast_elem(xv[u]);
                        prod *= f[u].d;
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if ((b4 >> u) & 1u) {
                            close_run();
                            flush();
                            cur = __shfl_sync(0xffffffffu, my_code, 4 * c + u);
                            m = cur >= 0 ? 1.0f : 0.0f;
                        }
                        trow[0] += xv[u];
                        tabs += fabsf(xv[u]);
                        trow[1] += f[u].p;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        if ((b4 >> u) & 1u) {
                            close_run();
                            flush();
                            cur = __shfl_sync(0xffffffffu, my_code, 4 * c + u);
                            m = cur >= 0 ? 1.0f : 0.0f;
                        }
                        element(xv[u]);
                    }
                }
              }
              if (FAST) { trow[2] += lg2_approx(prod); prod = 1.0f; }
            }
        } else {  // last, partial tile of the image
            for (int k = 0; k < nv; ++k) {
                const float x = Tile<T>::at(rowp, t, k);
                if ((bnd >> k) & 1u) {
                    close_run();
                    flush();
                    cur = __shfl_sync(0xffffffffu, my_code, k);
                    m = cur >= 0 ? 1.0f : 0.0f;
                }
                element(x);
                if (FAST) { trow[2] += lg2_approx(prod); prod = 1.0f; }
            }
        }
        if (MIX && mixb != 0u) mixed_cells(mixb, rowp, cell0 + h * KBOX, mye);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        close_run();
        if (FAST) trow[0] = 0.5f * (trow[0] + tabs);  // sum of max(x, 0)
#pragma unroll
        for (int i = 0; i < NROW; ++i) rows[i] += trow[i];
        if (bnd != 0u) run_tiles = 0;
        if (++run_tiles >= kFlushTiles) flush();
    }
    flush();

    if (!ok && lane == 0 && a.status) atomicOr(a.status, 2);
    if (!qvalid) return;
    float* pr = part + (int64_t)NACC * G * QP + t;
#pragma unroll
    for (int i = 0; i < NROW; ++i) pr[(int64_t)i * QP] = rows[i];
}

// ---------------------------------------------------------------------------
// Finalize, per query: reduce the row partials, the per-query terms the loss
// needs, and the class row statistics.  One warp per query row.
// qstat layout: P, Wtot, um_mask, um_dice, um_cls, base, cls_row, -
// ---------------------------------------------------------------------------
template <bool UNC, bool FAST>
__global__ void __launch_bounds__(256) cost_rows_kernel(CostArgs a) {
    pdl_enter();
    constexpr int NACC = UNC ? 3 : 2;
    constexpr int NROW = UNC ? 5 : 3;
    const int64_t qi = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (qi >= (int64_t)a.L * a.B * a.Q) return;
    const int lb = (int)(qi / a.Q);
    const int q = (int)(qi - (int64_t)lb * a.Q);
    const int qt = q / a.qrows, t = q - qt * a.qrows;
    const int HW = a.H * a.W;
    const float N2 = (float)(a.s * a.s);
    // rows: lanes stride over the 2*nchunk partial slots, fixed-order warp sum
    float r[NROW];
#pragma unroll
    for (int i = 0; i < NROW; ++i) r[i] = 0.0f;
    const int nslot = 2 * a.nchunk;
    const float* pbase = a.part + (((int64_t)lb * a.nqt + qt) * nslot) * (int64_t)a.part_stride +
                         (int64_t)NACC * a.gout * a.qrows_pad + t;
    for (int sl = lane; sl < nslot; sl += 32) {
        const float* p = pbase + (int64_t)sl * a.part_stride;
#pragma unroll
        for (int i = 0; i < NROW; ++i) r[i] += p[(int64_t)i * a.qrows_pad];
    }
#pragma unroll
    for (int i = 0; i < NROW; ++i) r[i] = warp_sum(r[i]);
    // class row: lse (softmax) / sum of focal-neg terms (sigmoid), and the
    // unmatched class term (src/cuda/mask_matching_forward.cu:150-276)
    const float* z = a.cls_logits + qi * a.C;
    const Focal cf = make_focal(a.cls_gamma, a.cls_alpha);
    const Focal uf = make_focal(a.use_softmax ? 0.0f : a.cls_gamma, a.use_softmax ? -1.0f : a.cls_alpha);
    float m = -INFINITY;
    for (int c = lane; c < a.C; c += 32) m = fmaxf(m, z[c]);
    m = warp_max(m);
    float se = 0.0f, sn = 0.0f, snu = 0.0f;
    // the sigmoid sums only where a term below reads them (softmax with forced
    // unmatched classes and a void class, the Mask2Former setting, needs none)
    const bool need_sn = !a.use_softmax;
    const bool need_snu = a.force_cls && (!a.has_void || !a.use_softmax);
    if (need_sn || need_snu) {
        for (int c = lane; c < a.C; c += 32) {
            const float zc = z[c];
            se += __expf(zc - m);
            const Elem e = elem(zc);
            sn += focal_neg(cf, e);
            snu += focal_neg(uf, e);
        }
    } else {
        for (int c = lane; c < a.C; c += 32) se += __expf(z[c] - m);
    }
    se = warp_sum(se); sn = warp_sum(sn); snu = warp_sum(snu);
    if (lane != 0) return;
    float base, P, wt, su, pu;
    if (UNC) {
        base = r[0] * N2; P = r[1] * N2; wt = r[2] * N2; su = r[3]; pu = r[4];
    } else if (FAST) {
        su = r[0] + r[2] * 0.6931471805599453f;  // sum softplus(x) = sum max(x,0) + ln2 * sum log2(1+e)
        pu = r[1];
        base = su * N2; P = pu * N2; wt = (float)a.Ht * (float)a.Wt;
    } else {
        su = r[0]; pu = r[1];
        base = su * N2; P = pu * N2; wt = (float)a.Ht * (float)a.Wt;
    }
    if (!a.normalize_uncertainty) wt = (float)a.Ht * (float)a.Wt;
    wt = fmaxf(wt, 1e-12f);
    const float lse = __logf(fmaxf(se, 1e-20f)) + m;
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
    const float ps = pu * a.area_scale;
    float* o = a.qstat + qi * kQStat;
    o[0] = P;
    o[1] = wt;
    o[2] = a.sigmoid_scale * (su / (float)HW);     // unmatched: BCE mean against empty
    o[3] = a.dice_scale * (ps / (ps + a.smooth));  // unmatched: empty-mask dice
    o[4] = um * a.cls_scale;
    o[5] = base;
    o[6] = a.use_softmax ? lse : sn;
}

// ---------------------------------------------------------------------------
// Finalize, per (q, g) pair: fixed-order reduction of the run partials, cost
// formulas (src/cuda/pw_mask.cu:290-304), label cost, total cost.
// grid = (ceil(qrows*G / 256), nqt, L*B), q fastest within a block.
// ---------------------------------------------------------------------------
template <bool UNC>
__global__ void __launch_bounds__(256) cost_pairs_kernel(CostArgs a) {
    pdl_enter();
    constexpr int NACC = UNC ? 3 : 2;
    __shared__ float red[8][NACC][32];
    const int qt = blockIdx.y, lb = blockIdx.z, b = lb % a.B;
    const int nq = min(a.qrows, a.Q - qt * a.qrows);
    const int G = a.gout;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // 32 consecutive (g, t) pairs per block (lane), the 8 warps split the
    // chunk slots; the fixed-order combine keeps the sums deterministic
    const int i = blockIdx.x * 32 + lane;
    const bool pv = i < nq * G;
    const int g = pv ? i / nq : 0, t = pv ? i - g * nq : 0;
    const int nslot = 2 * a.nchunk;
    const float* p = a.part + (((int64_t)lb * a.nqt + qt) * nslot) * (int64_t)a.part_stride +
                     (int64_t)g * a.qrows_pad + t;
    float acc2[2][NACC];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int k = 0; k < NACC; ++k) acc2[j][k] = 0.0f;
    if (pv) {
        int sl = warp;
        for (; sl + 8 < nslot; sl += 16) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const float* ps = p + (int64_t)(sl + 8 * j) * a.part_stride;
#pragma unroll
                for (int k = 0; k < NACC; ++k) acc2[j][k] += ps[(int64_t)k * G * a.qrows_pad];
            }
        }
        if (sl < nslot) {
            const float* ps = p + (int64_t)sl * a.part_stride;
#pragma unroll
            for (int k = 0; k < NACC; ++k) acc2[0][k] += ps[(int64_t)k * G * a.qrows_pad];
        }
    }
#pragma unroll
    for (int k = 0; k < NACC; ++k) red[warp][k][lane] = acc2[0][k] + acc2[1][k];
    __syncthreads();
    if (warp != 0 || !pv) return;
    float acc[NACC];
#pragma unroll
    for (int k = 0; k < NACC; ++k)
        acc[k] = ((red[0][k][lane] + red[1][k][lane]) + (red[2][k][lane] + red[3][k][lane])) +
                 ((red[4][k][lane] + red[5][k][lane]) + (red[6][k][lane] + red[7][k][lane]));
    const int ga = g + (g >= a.bg ? 1 : 0);
    const int64_t qi = (int64_t)lb * a.Q + qt * a.qrows + t;
    const int64_t o = qi * G + g;
    const float* qs = a.qstat + qi * kQStat;
    const int32_t tc = a.totals[(int64_t)b * a.gt_total + ga];
    const float T = UNC ? acc[2] : (float)tc;
    // +inf where the GT id paints no pixel of the image (with point sampling
    // the presence comes from the full label map, T from the points)
    const bool absent = a.present ? a.present[(int64_t)b * a.gt_total + ga] == 0 : tc == 0;
    float bce, dice;
    if (absent) {
        bce = INFINITY; dice = INFINITY;
    } else {
        bce = (qs[5] + acc[0]) / qs[1] * a.sigmoid_scale;
        dice = (1.0f - (2.0f * acc[1] + a.smooth) / (qs[0] + T + a.smooth)) * a.dice_scale;
    }
    const int64_t y = a.cls_targets[(int64_t)b * a.gt_total + ga];
    float cls;
    if (y < 0 || y >= a.C) {
        cls = INFINITY;
    } else {
        const float zy = a.cls_logits[qi * a.C + y];
        if (a.use_softmax) {
            cls = (qs[6] - zy) * a.cls_scale;
        } else {
            const Focal cf = make_focal(a.cls_gamma, a.cls_alpha);
            const Elem e = elem(zy);
            cls = (qs[6] + focal_pos(cf, e) - focal_neg(cf, e)) / (float)a.C * a.cls_scale;
        }
    }
    const int64_t slice = (int64_t)a.L * a.B * a.Q * G;
    if (a.sep) {
        a.sep[o] = bce;
        a.sep[slice + o] = dice;
        a.sep[2 * slice + o] = cls;
    }
    if (a.total) a.total[o] = (bce + dice) + cls;
    if (a.rawI) { a.rawI[o] = acc[1]; a.rawT[o] = T; }
}

template __global__ void cost_partial_kernel<false, false, false, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, false, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, true, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, true, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true, false, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true, true, float>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, false, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, false, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, true, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, true, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true, false, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true, true, __nv_bfloat16>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, false, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, false, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, true, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, false, true, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, false, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<false, true, true, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, false, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, false, true, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, false, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true, false, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_partial_kernel<true, true, true, true, __half>(const __grid_constant__ CUtensorMap, CostArgs);
template __global__ void cost_rows_kernel<false, false>(CostArgs);
template __global__ void cost_rows_kernel<false, true>(CostArgs);
template __global__ void cost_rows_kernel<true, false>(CostArgs);
template __global__ void cost_pairs_kernel<false>(CostArgs);
template __global__ void cost_pairs_kernel<true>(CostArgs);

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
