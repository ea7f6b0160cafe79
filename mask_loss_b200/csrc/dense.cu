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
//                       (bf16 bit patterns, exact for counts <= 256,
//                       [b][GT_total][cell]) and per (image, GT) the
//                       mask area (the histogram the label path builds);
//   dense_cost_kernel   per (layer*image, query tile, cell chunk, GT chunk of up to 64)
//                       the chunk partials in the label path's layout: row
//                       sums, and per GT sum(val * count) from a per-tile list
//                       of the non-zero (GT, count) pairs of each cell; cells
//                       with equal lists form runs whose value sums are applied
//                       once per run (registers for the last two GTs, shared
//                       memory for the rest).  Deterministic: every
//                       accumulator has one owner thread.
#include <algorithm>

#include <type_traits>

#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

namespace {
constexpr int kDenseTile = 32;   // cells per staged tile
constexpr int kDenseGC = 64;     // GT columns per block (grid chunk)
}  // namespace

// grid = (ceil(HW / 256), B), block 256: thread per cell; eight GT planes'
// loads in flight per thread, areas summed per warp.
// F32: counts as fp32 (the tf32 tensor-core kernel's B operand), else bf16 bits.
template <bool F32>
__global__ void __launch_bounds__(256)
dense_count_kernel(const uint8_t* __restrict__ masks, int H, int W, int Ht, int Wt, int s,
                   int gt_total, void* __restrict__ cnt_out, int32_t* __restrict__ totals) {
    extern __shared__ int32_t area[];  // [gt_total]
    const int b = blockIdx.y;
    const int HW = H * W;
    for (int g = threadIdx.x; g < gt_total; g += blockDim.x) area[g] = 0;
    __syncthreads();
    const int cell = blockIdx.x * blockDim.x + threadIdx.x;
    const bool valid = cell < HW;
    const int ci = valid ? cell / W : 0, cj = valid ? cell - ci * W : 0;
    const int64_t off = (int64_t)(ci * s) * Wt + (int64_t)cj * s;
    for (int g0 = 0; g0 < gt_total; g0 += 8) {
        int n[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            n[u] = 0;
            const int g = g0 + u;
            if (valid && g < gt_total) {
                const uint8_t* mg = masks + ((int64_t)b * gt_total + g) * Ht * Wt + off;
                if (s == 1) {
                    n[u] = mg[0] != 0;
                } else {
                    for (int dy = 0; dy < s; ++dy)
                        for (int dx = 0; dx < s; ++dx) n[u] += mg[(int64_t)dy * Wt + dx] != 0;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int g = g0 + u;
            if (g >= gt_total) break;
            if (valid && cnt_out) {  // null: areas only
                const int64_t o = ((int64_t)b * gt_total + g) * HW + cell;
                if (F32) static_cast<float*>(cnt_out)[o] = (float)n[u];
                else static_cast<uint16_t*>(cnt_out)[o] = count_bits((float)n[u]);
            }
            const int sum = (int)__reduce_add_sync(0xffffffffu, (unsigned)n[u]);
            if ((threadIdx.x & 31) == 0 && sum) atomicAdd(&area[g], sum);
        }
    }
    __syncthreads();
    for (int g = threadIdx.x; g < gt_total; g += blockDim.x)
        if (area[g]) atomicAdd(&totals[(int64_t)b * gt_total + g], area[g]);
}

// s = 1 (one mask pixel per cell), H*W a multiple of 8: eight cells per
// thread, one 8-byte mask load and one 16-byte count store per GT plane,
// four planes in flight.  grid = (ceil(H*W / 2048), B), block 256.
template <bool F32>
__global__ void __launch_bounds__(256)
dense_count_s1_kernel(const uint8_t* __restrict__ masks, int HW, int gt_total,
                      void* __restrict__ cnt_out, int32_t* __restrict__ totals) {
    extern __shared__ int32_t area[];  // [gt_total]
    const int b = blockIdx.y;
    for (int g = threadIdx.x; g < gt_total; g += blockDim.x) area[g] = 0;
    __syncthreads();
    const int cell0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
    const bool valid = cell0 < HW;
    const uint32_t one = count_bits(1.0f);
    for (int g0 = 0; g0 < gt_total; g0 += 4) {
        uint2 m[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int g = g0 + u;
            m[u] = (valid && g < gt_total)
                       ? *reinterpret_cast<const uint2*>(masks + ((int64_t)b * gt_total + g) * HW + cell0)
                       : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int g = g0 + u;
            if (g >= gt_total) break;
            // 0xFF in every byte that is non-zero, then one bit per cell
            const uint32_t nz0 = __vcmpne4(m[u].x, 0u), nz1 = __vcmpne4(m[u].y, 0u);
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                w[k] = ((nz0 >> (16 * k)) & 1u ? one : 0u) | ((nz0 >> (16 * k + 8)) & 1u ? one << 16 : 0u);
                w[2 + k] = ((nz1 >> (16 * k)) & 1u ? one : 0u) | ((nz1 >> (16 * k + 8)) & 1u ? one << 16 : 0u);
            }
            if (valid && cnt_out) {  // null: areas only
                const int64_t o = ((int64_t)b * gt_total + g) * HW + cell0;
                if (F32) {
                    float c8[8];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        c8[k] = (nz0 >> (8 * k)) & 1u ? 1.0f : 0.0f;
                        c8[4 + k] = (nz1 >> (8 * k)) & 1u ? 1.0f : 0.0f;
                    }
                    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(cnt_out) + o);
                    dst[0] = make_float4(c8[0], c8[1], c8[2], c8[3]);
                    dst[1] = make_float4(c8[4], c8[5], c8[6], c8[7]);
                } else {
                    *reinterpret_cast<uint4*>(static_cast<uint16_t*>(cnt_out) + o) =
                        make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
            const int n = (__popc(nz0) + __popc(nz1)) >> 3;
            const int sum = (int)__reduce_add_sync(0xffffffffu, (unsigned)n);
            if ((threadIdx.x & 31) == 0 && sum) atomicAdd(&area[g], sum);
        }
    }
    __syncthreads();
    for (int g = threadIdx.x; g < gt_total; g += blockDim.x)
        if (area[g]) atomicAdd(&totals[(int64_t)b * gt_total + g], area[g]);
}

// grid = (nchunk * 2 halves * ngc, nqt, L*B), block = QP threads (query row t of the tile).
// Dynamic shared memory: see dense_cost_smem.
template <bool UNC, bool FOC, typename T>
__device__ __forceinline__ void dense_cost_body(const CostArgs& a, const uint16_t* cnt, int GC) {
    constexpr int NACC = UNC ? 3 : 2;
    constexpr int NROW = UNC ? 5 : 3;
    constexpr bool FAST = !UNC && !FOC;
    extern __shared__ __align__(16) float dsh[];
    const int QP = a.qrows_pad, G = a.gout;
    const int ngc = (G + GC - 1) / GC;
    const int slot = blockIdx.x / ngc, gc = blockIdx.x - slot * ngc;  // slot = 2 * chunk + half
    const int chunk = slot >> 1, half = slot & 1;
    const int g0 = gc * GC, g1 = min(G, g0 + GC), gn = g1 - g0;
    const int qt = blockIdx.y, lb = blockIdx.z, b = lb % a.B;
    const int t = threadIdx.x;
    const int q = qt * a.qrows + t;
    const bool qvalid = t < a.qrows && q < a.Q;
    const int HW = a.H * a.W;
    // each half of a chunk (a multiple of 64 cells) fills its own partial slot
    const int half_cells = a.chunk_cells / 2;
    const int cell_begin = min(HW, chunk * a.chunk_cells + half * half_cells);
    const int cell_end = min(HW, cell_begin + half_cells);
    float* xs = dsh;                                         // [QP][kDenseTile + 1]
    float* acc = xs + QP * (kDenseTile + 1);                 // [NACC][GC][QP]
    int* lcnt = reinterpret_cast<int*>(acc + NACC * GC * QP);  // [kDenseTile]
    int* lg = lcnt + kDenseTile;                             // [kDenseTile][GC]
    float* ln = reinterpret_cast<float*>(lg + kDenseTile * GC);  // [kDenseTile][GC]
    float* ct = ln + kDenseTile * GC;                        // [GC][kDenseTile]
    unsigned* rmask = reinterpret_cast<unsigned*>(ct + kDenseTile * GC);  // run starts of the tile
    for (int i = t; i < NACC * GC * QP; i += blockDim.x) acc[i] = 0.0f;
    const int row0 = lb * a.Q + qt * a.qrows;
    const Focal foc = make_focal(a.mask_gamma, a.mask_alpha);
    float rows[NROW];
#pragma unroll
    for (int i = 0; i < NROW; ++i) rows[i] = 0.0f;
    const int warp = t >> 5, lane = t & 31;
    // two register slots cache the running sums of the last two GTs seen (runs
    // of cells of one GT are the common case); others go to shared memory
    int cj0 = -1, cj1 = -1;
    float s0[NACC], s1[NACC];
#pragma unroll
    for (int z = 0; z < NACC; ++z) { s0[z] = 0.0f; s1[z] = 0.0f; }
    auto flush = [&](int j, const float (&c)[NACC]) {
        if (j < 0) return;
#pragma unroll
        for (int z = 0; z < NACC; ++z) acc[(z * GC + j) * QP + t] += c[z];
    };
    // a run's sums times each (GT, count) of its list, through the cache
    auto apply_run = [&](int kr, const float (&rsum)[NACC]) {
        const int m = lcnt[kr];
        for (int i = 0; i < m; ++i) {
            const int j = lg[kr * GC + i];
            const float n = ln[kr * GC + i];
            if (j == cj0) {
#pragma unroll
                for (int z = 0; z < NACC; ++z) s0[z] = fmaf(rsum[z], n, s0[z]);
            } else if (j == cj1) {
#pragma unroll
                for (int z = 0; z < NACC; ++z) s1[z] = fmaf(rsum[z], n, s1[z]);
            } else {
                flush(cj1, s1);
                cj1 = cj0;
#pragma unroll
                for (int z = 0; z < NACC; ++z) { s1[z] = s0[z]; s0[z] = rsum[z] * n; }
                cj0 = j;
            }
        }
    };
    // logits tile in registers: thread t holds float4 (t + m*QP), m < 8 --
    // row i >> 3, cells 4*(i & 7) .. +3 -- so the next tile's loads are in
    // flight while the current one is computed.  Four elements are one
    // 16-byte (fp32) or 8-byte (16-bit) access when vec (H*W % 4 == 0 and an
    // aligned base); T is the logit type, widened on load.
    // The registers keep the raw words (float4, or uint2 of four 16-bit
    // values) and are widened only when the tile goes to shared memory, so
    // the loads stay in flight through the current tile's compute.
    const T* xlog = reinterpret_cast<const T*>(a.logits);
    const bool vec = (HW % 4 == 0) && ((reinterpret_cast<uintptr_t>(xlog) & (4 * sizeof(T) - 1)) == 0);
    using Raw = typename std::conditional<sizeof(T) == 4, float4, uint2>::type;
    Raw pre[8];
    auto load_tile = [&](int c0n) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = t + m * QP, r = i >> 3, c = (i & 7) * 4;
            const int qq = qt * a.qrows + r;
            Raw v{};  // zeros (also +0.0 in 16 bits)
            if (r < a.qrows && qq < a.Q) {
                const T* src = xlog + (int64_t)(row0 + r) * HW + c0n + c;
                if (vec) {
                    if (c0n + c < cell_end) v = __ldcs(reinterpret_cast<const Raw*>(src));
                } else {
                    alignas(8) T e[4];
#pragma unroll
                    for (int u = 0; u < 4; ++u) e[u] = c0n + c + u < cell_end ? src[u] : from_f<T>(0.0f);
                    v = *reinterpret_cast<const Raw*>(e);
                }
            }
            pre[m] = v;
        }
    };
    if (cell_begin < cell_end) load_tile(cell_begin);
    for (int c0 = cell_begin; c0 < cell_end; c0 += kDenseTile) {
        const int nv = min(kDenseTile, cell_end - c0);
        __syncthreads();  // previous tile consumed
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = t + m * QP, r = i >> 3, c = (i & 7) * 4;
            float* d = xs + r * (kDenseTile + 1) + c;
            if constexpr (sizeof(T) == 4) {
                d[0] = pre[m].x; d[1] = pre[m].y; d[2] = pre[m].z; d[3] = pre[m].w;
            } else {
                widen2(pre[m].x, d[0], d[1], xlog);
                widen2(pre[m].y, d[2], d[3], xlog);
            }
        }
        // the tile's counts, coalesced per GT plane
        for (int i = t; i < gn * kDenseTile; i += blockDim.x) {
            const int j = i / kDenseTile, k = i - j * kDenseTile;
            const int g = g0 + j;
            ct[i] = k < nv ? count_value(cnt[((int64_t)b * a.gt_total + g + (g >= a.bg ? 1 : 0)) * HW + c0 + k])
                           : 0.0f;
        }
        __syncthreads();
        // non-zero (GT, count) list of every cell: warp 0, lane = cell
        if (warp == 0) {
            int m = 0;
            for (int j = 0; j < gn; ++j) {
                const float n = ct[j * kDenseTile + lane];
                if (n != 0.0f) {
                    lg[lane * GC + m] = j;
                    ln[lane * GC + m] = n;
                    ++m;
                }
            }
            lcnt[lane] = m;
            __syncwarp();
            // run starts: a cell whose list differs from the previous cell's
            bool start = lane == 0;
            if (lane > 0 && lane < nv) {
                const int mp = lcnt[lane - 1];
                start = mp != m;
                for (int i = 0; i < m && !start; ++i)
                    start = lg[lane * GC + i] != lg[(lane - 1) * GC + i] ||
                            ln[lane * GC + i] != ln[(lane - 1) * GC + i];
            }
            const unsigned rm = __ballot_sync(0xffffffffu, start && lane < nv);
            if (lane == 0) *rmask = rm;
        }
        __syncthreads();
        if (c0 + kDenseTile < cell_end) load_tile(c0 + kDenseTile);
        if (t < a.qrows) {
            const unsigned rm = *rmask;  // same for every thread: uniform branches
            float rs[NACC];               // this thread's sums over the current run
#pragma unroll
            for (int z = 0; z < NACC; ++z) rs[z] = 0.0f;
            int kr = 0;
#pragma unroll 4
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
                if (k > 0 && ((rm >> k) & 1u)) {
                    apply_run(kr, rs);
#pragma unroll
                    for (int z = 0; z < NACC; ++z) rs[z] = 0.0f;
                    kr = k;
                }
#pragma unroll
                for (int z = 0; z < NACC; ++z) rs[z] += v[z];
            }
            if (nv > 0) apply_run(kr, rs);
        }
    }
    flush(cj1, s1);
    flush(cj0, s0);
    __syncthreads();
    if (!qvalid) return;
    float* part = a.part + ((((int64_t)lb * a.nqt + qt) * a.nchunk + chunk) * 2 + half) * (int64_t)a.part_stride;
    for (int z = 0; z < NACC; ++z)
        for (int j = 0; j < gn; ++j)
            part[((int64_t)z * G + g0 + j) * QP + t] = acc[(z * GC + j) * QP + t];
    if (gc == 0) {
#pragma unroll
        for (int i = 0; i < NROW; ++i) part[(int64_t)NACC * G * QP + (int64_t)i * QP + t] = rows[i];
    }
}

template <typename T>
__global__ void __launch_bounds__(128) dense_cost_kernel(CostArgs a, const uint16_t* cnt, int GC) {
    dense_cost_body<false, false, T>(a, cnt, GC);
}
template <typename T>
__global__ void __launch_bounds__(128) dense_cost_unc_kernel(CostArgs a, const uint16_t* cnt, int GC) {
    dense_cost_body<true, false, T>(a, cnt, GC);
}
template <typename T>
__global__ void __launch_bounds__(128) dense_cost_foc_kernel(CostArgs a, const uint16_t* cnt, int GC) {
    dense_cost_body<false, true, T>(a, cnt, GC);
}
template <typename T>
__global__ void __launch_bounds__(128) dense_cost_unc_foc_kernel(CostArgs a, const uint16_t* cnt, int GC) {
    dense_cost_body<true, true, T>(a, cnt, GC);
}

// GT columns per block: all of them up to kDenseGC (shared memory scales with it).
int dense_gc(int gout) { return std::max(1, std::min(gout, kDenseGC)); }

size_t dense_cost_smem(int qrows_pad, bool unc, int gc) {
    const int nacc = unc ? 3 : 2;
    return sizeof(float) * ((size_t)qrows_pad * (kDenseTile + 1) + (size_t)nacc * gc * qrows_pad) +
           sizeof(int) * (kDenseTile + (size_t)kDenseTile * gc) + 2 * sizeof(float) * (size_t)kDenseTile * gc +
           16;
}

cudaError_t launch_dense_count(const uint8_t* masks, int B, int H, int W, int Ht, int Wt, int s,
                               int gt_total, void* cnt, int32_t* totals, cudaStream_t st, bool f32) {
    const int HW = H * W;
    const size_t hs = sizeof(int32_t) * (size_t)std::max(gt_total, 1);
    if (s == 1 && HW % 8 == 0 && (reinterpret_cast<uintptr_t>(masks) & 7) == 0 &&
        (reinterpret_cast<uintptr_t>(cnt) & 15) == 0) {
        dim3 g((HW / 8 + 255) / 256, B);
        if (f32) dense_count_s1_kernel<true><<<g, 256, hs, st>>>(masks, HW, gt_total, cnt, totals);
        else dense_count_s1_kernel<false><<<g, 256, hs, st>>>(masks, HW, gt_total, cnt, totals);
        return cudaGetLastError();
    }
    dim3 g((HW + 255) / 256, B);
    if (f32) dense_count_kernel<true><<<g, 256, hs, st>>>(masks, H, W, Ht, Wt, s, gt_total, cnt, totals);
    else dense_count_kernel<false><<<g, 256, hs, st>>>(masks, H, W, Ht, Wt, s, gt_total, cnt, totals);
    return cudaGetLastError();
}

template <typename T>
cudaError_t launch_dense_cost_t(const CostArgs& a, bool unc, bool foc, const uint16_t* cnt,
                                cudaStream_t st) {
    const int gc = dense_gc(a.gout);
    const size_t smem = dense_cost_smem(a.qrows_pad, unc, gc);
    const int ngc = (a.gout + gc - 1) / gc;
    dim3 g(a.nchunk * 2 * ngc, a.nqt, a.L * a.B);
    auto k = unc ? (foc ? dense_cost_unc_foc_kernel<T> : dense_cost_unc_kernel<T>)
                 : (foc ? dense_cost_foc_kernel<T> : dense_cost_kernel<T>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k<<<g, a.qrows_pad, smem, st>>>(a, cnt, gc);
    return cudaGetLastError();
}

cudaError_t launch_dense_cost(const CostArgs& a, bool unc, bool foc, const uint16_t* cnt,
                              cudaStream_t st, int ldt) {
    if (ldt == 1) return launch_dense_cost_t<__nv_bfloat16>(a, unc, foc, cnt, st);
    if (ldt == 2) return launch_dense_cost_t<__half>(a, unc, foc, cnt, st);
    return launch_dense_cost_t<float>(a, unc, foc, cnt, st);
}

}  // namespace mlb
