// match.cu -- on-device assignment solver, one warp per (l,b) slice.
//
// Replaces the host loop of src/cpu/matching.cpp:690-722 (D2H copy of each
// cost slice, C++ solve on a host thread, H2D of the results).  Restates
// assign_predictions_for_slice (src/cpu/matching.cpp:476-571) and its
// strategies (:95-463) so that, fed the same fp64 cost matrix, every output
// index is bit-identical:
//   * the shortest-augmenting-path Hungarian keeps the reference's operation
//     order in double precision (cur = (c - u[i0]) - v[j]; u += delta;
//     v -= delta; minv -= delta) with explicit _rn intrinsics, no FMA;
//   * the per-step argmin over columns is a warp-shuffle reduction on
//     (value, index) with ties to the lower index, which equals the
//     reference's sequential strict-< scan in increasing j;
//   * greedy scans keep the reference's first-minimum-in-valid-column-order.
// The cost slice is staged transposed ([col][query], fp32 or fp64) in shared
// memory when it fits, so the inner scan reads are conflict-free.
// Every loop is bounded by construction (at most n+1 Dijkstra steps per row);
// a step that finds no finite delta sets *status and abandons the slice.
#include "common.cuh"
#include "kernels.cuh"

namespace mlb {

namespace {

constexpr double kInf = __builtin_huge_val();

template <typename CT>
struct CostView {
    const CT* g;      // (Q, G) slice in global memory
    const CT* s;      // (G, Q) transposed copy in shared memory, or null
    int Q, G;
    ML_INLINE double at(int q, int col) const {
        return s ? static_cast<double>(s[col * Q + q]) : static_cast<double>(g[(int64_t)q * G + col]);
    }
};

ML_INLINE bool ok_cost(double c, double thr) { return isfinite(c) && c < thr; }

ML_INLINE double big_from(double x) {  // src/cpu/matching.cpp:71-83
    if (!isfinite(x) || x <= 0.0) return 1e15;
    double b = x * 0.5;
    if (!isfinite(b) || b < 1e6) b = 1e15;
    if (b > 1e290) b = 1e290;
    return b;
}

// (value, index) argmin across the warp; ties resolve to the lower index.
ML_INLINE void warp_argmin(double& v, int& j) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oj = __shfl_xor_sync(0xffffffffu, j, o);
        if (ov < v || (ov == v && oj < j)) { v = ov; j = oj; }
    }
}

struct SolverMem {
    double* u;     // [Q+1]  row potentials (rows <= Q)
    double* v;     // [Q+1]  column potentials
    double* minv;  // [Q+1]
    int* way;      // [Q+1]
    int* p;        // [Q+1]  row matched to column j (0 = free)
    int* used;     // [Q+1]
};

// Shortest augmenting path Hungarian, src/cpu/matching.cpp:95-186.
// rows = cols[0..M), columns = preds[0..n).  asg[k] = row slot of preds[k] or -1.
template <typename CT>
__device__ bool hungarian(const CostView<CT>& C, const int* preds, int n, const int* cols, int M,
                          double thr, double BIG, int* asg, SolverMem& m) {
    const int lane = threadIdx.x & 31;
    for (int k = lane; k < n; k += 32) asg[k] = -1;
    __syncwarp();
    if (M == 0 || n == 0 || n < M) return true;
    for (int i = lane; i <= M; i += 32) m.u[i] = 0.0;
    for (int j = lane; j <= n; j += 32) { m.v[j] = 0.0; m.p[j] = 0; m.way[j] = 0; }
    __syncwarp();
    for (int i = 1; i <= M; ++i) {
        if (lane == 0) m.p[0] = i;
        for (int j = lane; j <= n; j += 32) { m.minv[j] = kInf; m.used[j] = 0; }
        __syncwarp();
        int j0 = 0;
        int steps = 0;
        do {
            if (lane == 0) m.used[j0] = 1;
            __syncwarp();
            const int i0 = m.p[j0];
            const int col = cols[i0 - 1];
            const double ui0 = m.u[i0];
            double best = kInf;
            int bj = 0x7fffffff;
            for (int j = 1 + lane; j <= n; j += 32) {
                if (m.used[j]) continue;
                const double raw = C.at(preds[j - 1], col);
                const double cij = ok_cost(raw, thr) ? raw : BIG;
                const double cur = __dsub_rn(__dsub_rn(cij, ui0), m.v[j]);
                double mv = m.minv[j];
                if (cur < mv) { mv = cur; m.minv[j] = cur; m.way[j] = j0; }
                if (mv < best) { best = mv; bj = j; }
            }
            warp_argmin(best, bj);
            if (!isfinite(best) || bj > n) return false;
            const double delta = best;
            for (int j = lane; j <= n; j += 32) {
                if (m.used[j]) {
                    const int r = m.p[j];
                    m.u[r] = __dadd_rn(m.u[r], delta);
                    m.v[j] = __dsub_rn(m.v[j], delta);
                } else {
                    m.minv[j] = __dsub_rn(m.minv[j], delta);
                }
            }
            __syncwarp();
            j0 = bj;
            if (++steps > n + 1) return false;
        } while (m.p[j0] != 0);
        if (lane == 0) {
            int jj = j0;
            int guard = 0;
            do {
                const int j1 = m.way[jj];
                m.p[jj] = m.p[j1];
                jj = j1;
            } while (jj != 0 && ++guard <= n + 1);
        }
        __syncwarp();
    }
    for (int j = 1 + lane; j <= n; j += 32)
        if (m.p[j] > 0) asg[j - 1] = m.p[j] - 1;
    __syncwarp();
    return true;
}


// Register-resident variant of `hungarian` for n <= 32*NJ - 1 columns: lane
// `lane` owns columns j = lane + 32k (k < NJ) and keeps v, minv and the used
// flags in registers; u, p and way stay in shared memory (random access).
// Same operation order and tie rule as `hungarian`, so results are identical.
template <int NJ, typename CT>
__device__ bool hungarian_reg(const CostView<CT>& C, const int* preds, int n, const int* cols, int M,
                              double thr, double BIG, int* asg, SolverMem& m) {
    const int lane = threadIdx.x & 31;
    for (int k = lane; k < n; k += 32) asg[k] = -1;
    __syncwarp();
    if (M == 0 || n == 0 || n < M) return true;
    for (int i = lane; i <= M; i += 32) m.u[i] = 0.0;
    for (int j = lane; j <= n; j += 32) { m.p[j] = 0; m.way[j] = 0; }
    double v[NJ];
#pragma unroll
    for (int k = 0; k < NJ; ++k) v[k] = 0.0;
    __syncwarp();
    for (int i = 1; i <= M; ++i) {
        if (lane == 0) m.p[0] = i;
        double minv[NJ];
#pragma unroll
        for (int k = 0; k < NJ; ++k) minv[k] = kInf;
        uint32_t used = 0;
        __syncwarp();
        int j0 = 0;
        int steps = 0;
        do {
            if ((j0 & 31) == lane) used |= 1u << (j0 >> 5);
            const int i0 = m.p[j0];
            const int col = cols[i0 - 1];
            const double ui0 = m.u[i0];
            double best = kInf;
            int bj = 0x7fffffff;
#pragma unroll
            for (int k = 0; k < NJ; ++k) {
                const int j = lane + 32 * k;
                if (j < 1 || j > n || ((used >> k) & 1u)) continue;
                const double raw = C.at(preds[j - 1], col);
                const double cij = ok_cost(raw, thr) ? raw : BIG;
                const double cur = __dsub_rn(__dsub_rn(cij, ui0), v[k]);
                if (cur < minv[k]) { minv[k] = cur; m.way[j] = j0; }
                if (minv[k] < best) { best = minv[k]; bj = j; }
            }
            warp_argmin(best, bj);
            if (!isfinite(best) || bj > n) return false;
            const double delta = best;
#pragma unroll
            for (int k = 0; k < NJ; ++k) {
                const int j = lane + 32 * k;
                if (j > n) continue;
                if ((used >> k) & 1u) {
                    const int r = m.p[j];
                    m.u[r] = __dadd_rn(m.u[r], delta);
                    v[k] = __dsub_rn(v[k], delta);
                } else {
                    minv[k] = __dsub_rn(minv[k], delta);
                }
            }
            __syncwarp();
            j0 = bj;
            if (++steps > n + 1) return false;
        } while (m.p[j0] != 0);
        if (lane == 0) {
            int jj = j0;
            int guard = 0;
            do {
                const int j1 = m.way[jj];
                m.p[jj] = m.p[j1];
                jj = j1;
            } while (jj != 0 && ++guard <= n + 1);
        }
        __syncwarp();
    }
    for (int j = 1 + lane; j <= n; j += 32)
        if (m.p[j] > 0) asg[j - 1] = m.p[j] - 1;
    __syncwarp();
    return true;
}

template <typename CT>
__device__ bool solve(const CostView<CT>& C, const int* preds, int n, const int* cols, int M,
                      double thr, double BIG, int* asg, SolverMem& m) {
    if (n < 32) return hungarian_reg<1>(C, preds, n, cols, M, thr, BIG, asg, m);
    if (n < 64) return hungarian_reg<2>(C, preds, n, cols, M, thr, BIG, asg, m);
    if (n < 128) return hungarian_reg<4>(C, preds, n, cols, M, thr, BIG, asg, m);
    if (n < 256) return hungarian_reg<8>(C, preds, n, cols, M, thr, BIG, asg, m);
    return hungarian(C, preds, n, cols, M, thr, BIG, asg, m);
}

// Greedy fill with capacities, src/cpu/matching.cpp:193-229.
template <typename CT>
__device__ void greedy(const CostView<CT>& C, const int* preds, int np, const int* valid, int nv,
                       double thr, int* cap, int* p2g) {
    const int lane = threadIdx.x & 31;
    for (int k = 0; k < np; ++k) {
        const int q = preds[k];
        if (p2g[q] >= 0) continue;
        double best = kInf;
        int bt = 0x7fffffff;
        for (int t = lane; t < nv; t += 32) {
            const int a = valid[t];
            if (cap[a] <= 0) continue;
            const double c = C.at(q, a);
            if (!ok_cost(c, thr)) continue;
            if (c < best) { best = c; bt = t; }
        }
        warp_argmin(best, bt);
        if (bt < nv) {
            if (lane == 0) {
                const int a = valid[bt];
                p2g[q] = a;
                if (cap[a] > 0) cap[a] -= 1;
            }
        }
        __syncwarp();
    }
}

// Order-preserving warp compaction: out[k] for flag(k) true, returns count.
template <typename F>
ML_INLINE int warp_compact(int n, F flag, int* out, const int* in) {
    const int lane = threadIdx.x & 31;
    int total = 0;
    for (int base = 0; base < n; base += 32) {
        const int k = base + lane;
        const bool f = (k < n) && flag(k);
        const unsigned bal = __ballot_sync(0xffffffffu, f);
        if (f) out[total + __popc(bal & ((1u << lane) - 1u))] = in ? in[k] : k;
        total += __popc(bal);
    }
    __syncwarp();
    return total;
}

}  // namespace

// One warp per slice.  Dynamic shared memory holds the solver state and,
// when `stage_cost`, the transposed cost slice.
template <typename CT>
__global__ void __launch_bounds__(kMatchThreads) match_kernel(MatchArgs<CT> a) {
    extern __shared__ __align__(16) unsigned char msh[];
    const int slice = blockIdx.x;
    const int Q = a.Q, G = a.G;
    const int lane = threadIdx.x & 31;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const CT* cg = a.costs + (int64_t)slice * Q * G;
    int64_t* out_p = a.pred_to_gt + (int64_t)slice * Q;
    int64_t* out_r = a.pred_round + (int64_t)slice * Q;

    unsigned char* cur = msh;
    auto take = [&](size_t bytes) {
        unsigned char* r = cur;
        cur += (bytes + 15) & ~size_t(15);
        return r;
    };
    SolverMem m;
    m.u = reinterpret_cast<double*>(take(sizeof(double) * (Q + 1)));
    m.v = reinterpret_cast<double*>(take(sizeof(double) * (Q + 1)));
    m.minv = reinterpret_cast<double*>(take(sizeof(double) * (Q + 1)));
    m.way = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    m.p = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    m.used = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    int* valid = reinterpret_cast<int*>(take(sizeof(int) * (G + 1)));
    int* cap = reinterpret_cast<int*>(take(sizeof(int) * (G + 1)));
    int* cols = reinterpret_cast<int*>(take(sizeof(int) * ((Q > G ? Q : G) + 1)));
    int* preds = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    int* preds2 = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    int* asg = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    int* p2g = reinterpret_cast<int*>(take(sizeof(int) * (Q + 1)));
    CT* cs = nullptr;
    if (a.stage_cost) {
        cs = reinterpret_cast<CT*>(take(sizeof(CT) * (size_t)Q * G));
#pragma unroll 4
        for (int i = tid; i < Q * G; i += nthr) {
            const int q = i / G, g = i - q * G;
            cs[g * Q + q] = cg[i];
        }
    }
    CostView<CT> C{cg, cs, Q, G};
    const double thr = a.inf_thresh;
    const int64_t K = a.topk;
    __shared__ int failed;
    if (tid == 0) failed = 0;
    for (int q = tid; q < Q; q += nthr) p2g[q] = -1;
    __syncthreads();
    if (threadIdx.x >= 32) goto rank;  // warp 0 runs the strategies
    {

    bool good = true;
    if (Q > 0 && G > 0 && K > 0) {
        // valid columns: any finite cost below the threshold
        const int nv = warp_compact(G, [&](int g) {
            for (int q = 0; q < Q; ++q)
                if (ok_cost(C.at(q, g), thr)) return true;
            return false;
        }, valid, nullptr);
        if (nv > 0) {
            const double BIG = big_from(thr);
            for (int t = lane; t < nv; t += 32) cap[valid[t]] = (int)(K < (int64_t)(1 << 30) ? K : (int64_t)(1 << 30));
            for (int q = lane; q < Q; q += 32) preds[q] = q;
            __syncwarp();
            if (a.strategy == 0) {  // global, :239-286
                int M = 0;
                for (int64_t rep = 0; rep < K && M < Q; ++rep)
                    for (int t = 0; t < nv && M < Q; ++t) {
                        if (lane == 0) cols[M] = valid[t];
                        ++M;
                    }
                __syncwarp();
                good = solve(C, preds, Q, cols, M, thr, BIG, asg, m);
                if (good)
                    for (int q = lane; q < Q; q += 32)
                        if (asg[q] >= 0) {
                            const int c = cols[asg[q]];
                            if (ok_cost(C.at(q, c), thr)) p2g[q] = c;
                        }
                __syncwarp();
            } else if (a.strategy == 1) {  // round, :294-366
                int nrem = Q;
                int* pa = preds;
                int* pb = preds2;
                for (int64_t r = 0; r < K && good; ++r) {
                    int M = warp_compact(nv, [&](int t) { return cap[valid[t]] > 0; }, cols, valid);
                    if (M == 0 || nrem == 0) break;
                    if (M > nrem) M = nrem;
                    good = solve(C, pa, nrem, cols, M, thr, BIG, asg, m);
                    if (!good) break;
                    // assignments (distinct columns within a round)
                    for (int k = lane; k < nrem; k += 32) {
                        if (asg[k] >= 0) {
                            const int q = pa[k], c = cols[asg[k]];
                            if (ok_cost(C.at(q, c), thr)) {
                                p2g[q] = c;
                                if (cap[c] > 0) cap[c] -= 1;
                            }
                        }
                    }
                    __syncwarp();
                    const int nn = warp_compact(nrem, [&](int k) { return p2g[pa[k]] < 0; }, pb, pa);
                    int* tmp = pa; pa = pb; pb = tmp;
                    nrem = nn;
                    if (nrem == 0) break;
                }
            } else if (a.strategy == 2) {  // greedy, :372-393
                greedy(C, preds, Q, valid, nv, thr, cap, p2g);
            } else {  // pseudo-greedy, :400-463
                const int M = nv < Q ? nv : Q;
                for (int t = lane; t < M; t += 32) cols[t] = valid[t];
                __syncwarp();
                good = solve(C, preds, Q, cols, M, thr, BIG, asg, m);
                if (good) {
                    for (int q = lane; q < Q; q += 32)
                        if (asg[q] >= 0) {
                            const int c = cols[asg[q]];
                            if (ok_cost(C.at(q, c), thr)) {
                                p2g[q] = c;
                                if (cap[c] > 0) cap[c] -= 1;
                            }
                        }
                    __syncwarp();
                    const int nr = warp_compact(Q, [&](int q) { return p2g[q] < 0; }, preds2, nullptr);
                    if (nr > 0) greedy(C, preds2, nr, valid, nv, thr, cap, p2g);
                }
            }
        }
    }
    __syncwarp();
    if (!good && lane == 0) {
        atomicOr(a.status, 1);
        failed = 1;
    }
    }
rank:
    __syncthreads();
    if (failed) {
        for (int q = tid; q < Q; q += nthr) { out_p[q] = -1; out_r[q] = -1; }
        return;
    }
    // rank per GT by (cost, q), src/cpu/matching.cpp:538-565
    for (int q = tid; q < Q; q += nthr) {
        const int g = p2g[q];
        int64_t pr = -1;
        int64_t pg = -1;
        if (g >= 0 && ok_cost(C.at(q, g), thr)) {
            pg = g;
            const double c = C.at(q, g);
            int64_t rank = 0;
            for (int q2 = 0; q2 < Q; ++q2) {
                if (q2 == q || p2g[q2] != g) continue;
                const double c2 = C.at(q2, g);
                if (!ok_cost(c2, thr)) continue;
                if (c2 < c || (c2 == c && q2 < q)) ++rank;
            }
            if (rank < K) pr = rank;
        }
        out_p[q] = pg;
        out_r[q] = pr;
    }
}

template __global__ void match_kernel<float>(MatchArgs<float>);
template __global__ void match_kernel<double>(MatchArgs<double>);

size_t match_smem_bytes(int Q, int G, size_t cost_elem, bool stage) {
    auto r = [](size_t b) { return (b + 15) & ~size_t(15); };
    size_t s = 3 * r(sizeof(double) * (Q + 1)) + 3 * r(sizeof(int) * (Q + 1)) +
               2 * r(sizeof(int) * (G + 1)) + 4 * r(sizeof(int) * (Q + 1)) +
               r(sizeof(int) * ((Q > G ? Q : G) + 1));
    if (stage) s += r(cost_elem * (size_t)Q * G);
    return s;
}

}  // namespace mlb
