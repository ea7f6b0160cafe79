// match.cu -- on-device assignment solver, one thread block per (l,b) slice.
//
// Replaces the host loop of src/cpu/matching.cpp:690-722 (D2H copy of each
// cost slice, C++ solve on a host thread, H2D of the results).  Restates
// assign_predictions_for_slice (src/cpu/matching.cpp:476-571) and its
// strategies (:95-463) so that, fed the same fp64 cost matrix, every output
// index is bit-identical:
//   * the shortest-augmenting-path Hungarian keeps the reference's operation
//     order in double precision (cur = (c - u[i0]) - v[j]; u += delta;
//     v -= delta; minv -= delta) with explicit _rn intrinsics, no FMA;
//   * the per-step argmin over columns takes the smallest value with ties to
//     the lower index, which equals the reference's sequential strict-< scan
//     in increasing j;
//   * greedy scans keep the reference's first-minimum-in-valid-column-order.
// Up to 4 * blockDim.x - 1 prediction columns the Hungarian runs on the whole
// block with its per-column state in registers (hungarian_blk): fp64 issue is
// the limit of a Dijkstra step on this part, so the columns are spread over
// every SM sub-partition.  Larger slices use warp 0 and shared memory.
// The cost slice is staged transposed ([col][query]) in shared memory when it
// fits, with a double copy already mapped through ok_cost/BIG for the solver.
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


// Order-preserving 64-bit key of a double (never NaN here: ok_cost maps NaN
// to BIG); -0 and +0 get the same key, as they compare equal.
ML_INLINE uint64_t order_key(double v) {
    const uint64_t b = (uint64_t)__double_as_longlong(v + 0.0);  // -0 -> +0
    return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

ML_INLINE double from_key(uint64_t k) {
    return __longlong_as_double((long long)((k >> 63) ? (k & 0x7fffffffffffffffull) : ~k));
}

template <int NJ, typename T>
ML_INLINE T pick(const T (&a)[NJ], int k) {
    T r = a[0];
#pragma unroll
    for (int kk = 1; kk < NJ; ++kk)
        if (k == kk) r = a[kk];
    return r;
}

// One warp's best column of a Dijkstra step, with what the next step needs
// if it wins: p[j], u[p[j]] and cols[p[j] - 1].  Double-buffered by step
// parity, so a step needs one block barrier.
struct alignas(16) BlkCand {
    uint32_t hi, lo;  // order_key of the value
    int j;            // column (0x7fffffff: none)
    int i0;           // p[j]
    double u0;        // u[p[j]]
    int col;          // cols[p[j] - 1] (p[j] > 0)
    int pad;
};

struct BlkShared {
    BlkCand cand[2][kMatchMaxThreads / 32];
    int flag;
};

// Block-wide variant of `hungarian` for n + 1 <= NJ * blockDim.x columns:
// thread t owns columns j = t + blockDim.x * k and keeps, per column, its
// prediction row, v, minv, way, p (row matched to the column), the cost
// column of that row and its potential u in registers.  Every warp scans its
// columns in parallel; the argmin is a warp redux.sync on an order-preserving
// key, then a fixed-order pick over the warps' candidates, so the result is
// the smallest value with ties to the lower column index -- the reference's
// sequential strict-< scan.  u[p[j]] of the reference is uc[j] here: the same
// operations in the same order, moved along the augmenting path with p.
// `cd`, when set, is the transposed slice already mapped through ok_cost/BIG.
template <int NJ, typename CT>
__device__ bool hungarian_blk(const CostView<CT>& C, const double* cd, const int* preds, int n,
                              const int* cols, int M, double thr, double BIG, int* asg,
                              SolverMem& m, BlkShared& sh) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int lane = tid & 31, warp = tid >> 5, nw = nthr >> 5;
    for (int k = tid; k < n; k += nthr) asg[k] = -1;
    __syncthreads();
    if (M == 0 || n == 0 || n < M) return true;
    int pq[NJ], pc[NJ], wy[NJ], cc[NJ];
    double v[NJ], uc[NJ];
#pragma unroll
    for (int k = 0; k < NJ; ++k) {
        const int j = tid + nthr * k;
        pq[k] = (j >= 1 && j <= n) ? preds[j - 1] : 0;
        pc[k] = 0;
        wy[k] = 0;
        cc[k] = 0;
        v[k] = 0.0;
        uc[k] = 0.0;
    }
    const int Qs = C.Q;
    int par = 0;
    for (int i = 1; i <= M; ++i) {
        // column 0 holds the entering row i; u[i] is still 0
        int col = cols[i - 1];
        double ui0 = 0.0;
        if (tid == 0) { pc[0] = i; uc[0] = 0.0; cc[0] = col; }
        double minv[NJ];
#pragma unroll
        for (int k = 0; k < NJ; ++k) minv[k] = kInf;
        uint32_t used = 0;
        int j0 = 0;
        int steps = 0;
        while (true) {
            if (j0 % nthr == tid) used |= 1u << (j0 / nthr);
            double cij[NJ];
#pragma unroll
            for (int k = 0; k < NJ; ++k) {
                const int j = tid + nthr * k;
                if (j >= 1 && j <= n) {
                    if (cd) {
                        cij[k] = cd[col * Qs + pq[k]];
                    } else {
                        const double raw = C.at(pq[k], col);
                        cij[k] = ok_cost(raw, thr) ? raw : BIG;
                    }
                } else {
                    cij[k] = 0.0;
                }
            }
            double best = kInf;
            int bj = 0x7fffffff;
#pragma unroll
            for (int k = 0; k < NJ; ++k) {
                const int j = tid + nthr * k;
                if (j < 1 || j > n || ((used >> k) & 1u)) continue;
                const double cur = __dsub_rn(__dsub_rn(cij[k], ui0), v[k]);
                if (cur < minv[k]) { minv[k] = cur; wy[k] = j0; }
                if (minv[k] < best) { best = minv[k]; bj = j; }
            }
            {
                const uint64_t key = order_key(best);
                const uint32_t hi = (uint32_t)(key >> 32), lo = (uint32_t)key;
                const uint32_t mh = __reduce_min_sync(0xffffffffu, hi);
                const uint32_t ml = __reduce_min_sync(0xffffffffu, hi == mh ? lo : 0xffffffffu);
                const bool tie = hi == mh && lo == ml;
                const uint32_t mj = __reduce_min_sync(0xffffffffu, tie ? (uint32_t)bj : 0x7fffffffu);
                const uint32_t wl = __ballot_sync(0xffffffffu, tie && (uint32_t)bj == mj);
                if (lane == __ffs(wl) - 1) {
                    BlkCand c;
                    c.hi = mh; c.lo = ml; c.j = (int)mj;
                    const int k = bj <= n ? bj / nthr : 0;
                    c.i0 = pick(pc, k); c.u0 = pick(uc, k); c.col = pick(cc, k); c.pad = 0;
                    sh.cand[par][warp] = c;
                }
            }
            __syncthreads();
            BlkCand w = sh.cand[par][0];
            for (int x = 1; x < nw; ++x) {
                const BlkCand c = sh.cand[par][x];
                if (c.hi < w.hi || (c.hi == w.hi && (c.lo < w.lo || (c.lo == w.lo && c.j < w.j)))) w = c;
            }
            par ^= 1;
            best = from_key(((uint64_t)w.hi << 32) | w.lo);
            if (!isfinite(best) || w.j > n) return false;  // uniform across the block
            const double delta = best;
#pragma unroll
            for (int k = 0; k < NJ; ++k) {
                const int j = tid + nthr * k;
                if (j > n) continue;
                if ((used >> k) & 1u) {
                    uc[k] = __dadd_rn(uc[k], delta);
                    v[k] = __dsub_rn(v[k], delta);
                } else {
                    minv[k] = __dsub_rn(minv[k], delta);
                }
            }
            j0 = w.j;
            if (++steps > n + 1) return false;
            if (w.i0 == 0) break;  // free column reached
            col = w.col;           // the chosen column is unused: its u is unchanged
            ui0 = w.u0;
        }
        // augment along way[] (thread 0 walks the path in shared memory)
#pragma unroll
        for (int k = 0; k < NJ; ++k) {
            const int j = tid + nthr * k;
            if (j <= n) { m.way[j] = wy[k]; m.p[j] = pc[k]; m.minv[j] = uc[k]; m.used[j] = cc[k]; }
        }
        __syncthreads();
        if (tid == 0) {
            int jj = j0;
            int guard = 0;
            do {
                const int j1 = m.way[jj];
                m.p[jj] = m.p[j1];
                m.minv[jj] = m.minv[j1];
                m.used[jj] = m.used[j1];
                jj = j1;
            } while (jj != 0 && ++guard <= n + 1);
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < NJ; ++k) {
            const int j = tid + nthr * k;
            if (j <= n) { pc[k] = m.p[j]; uc[k] = m.minv[j]; cc[k] = m.used[j]; }
        }
        __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < NJ; ++k) {
        const int j = tid + nthr * k;
        if (j >= 1 && j <= n && pc[k] > 0) asg[j - 1] = pc[k] - 1;
    }
    __syncthreads();
    return true;
}

// Called by every thread of the block; returns the same value everywhere.
template <typename CT>
__device__ bool solve(const CostView<CT>& C, const double* cd, const int* preds, int n, const int* cols,
                      int M, double thr, double BIG, int* asg, SolverMem& m, BlkShared& sh) {
    const int nthr = blockDim.x;
    if (n + 1 <= nthr) return hungarian_blk<1>(C, cd, preds, n, cols, M, thr, BIG, asg, m, sh);
    if (n + 1 <= 2 * nthr) return hungarian_blk<2>(C, cd, preds, n, cols, M, thr, BIG, asg, m, sh);
    if (n + 1 <= 4 * nthr) return hungarian_blk<4>(C, cd, preds, n, cols, M, thr, BIG, asg, m, sh);
    bool r = true;
    if (threadIdx.x < 32) r = hungarian(C, preds, n, cols, M, thr, BIG, asg, m);
    if (threadIdx.x == 0) sh.flag = r ? 1 : 0;
    __syncthreads();
    r = sh.flag != 0;
    __syncthreads();
    return r;
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

// One block per slice; every strategy's control flow is block-uniform, the
// Hungarian runs on all threads (hungarian_blk) and the compactions and the
// greedy passes on warp 0.  Dynamic shared memory holds the solver state and,
// by `stage_cost`: 1 the transposed cost slice, 2 also its ok_cost/BIG-mapped
// copy in double for the solver.
template <typename CT>
__global__ void __launch_bounds__(kMatchMaxThreads) match_kernel(MatchArgs<CT> a) {
    pdl_enter();
    extern __shared__ __align__(16) unsigned char msh[];
    __shared__ BlkShared sh;
    __shared__ int sh_n, failed;
    const int slice = blockIdx.x;
    const int Q = a.Q, G = a.G;
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int lane = tid & 31;
    const CT* cg = a.costs + (int64_t)slice * Q * G;
    int64_t* out_p = a.pred_to_gt + (int64_t)slice * Q;
    int64_t* out_r = a.pred_round + (int64_t)slice * Q;
    const double thr = a.inf_thresh;
    const double BIG = big_from(thr);

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
    double* cd = nullptr;
    if (a.stage_cost >= 1) cs = reinterpret_cast<CT*>(take(sizeof(CT) * (size_t)Q * G));
    if (a.stage_cost >= 2) cd = reinterpret_cast<double*>(take(sizeof(double) * (size_t)Q * G));
    for (int g = tid; g < G; g += nthr) cap[g] = 0;  // valid-column flags first
    if (tid == 0) failed = 0;
    for (int q = tid; q < Q; q += nthr) p2g[q] = -1;
    __syncthreads();
    for (int i = tid; i < Q * G; i += nthr) {
        const int q = i / G, g = i - q * G;
        const CT c = cg[i];
        const bool ok = ok_cost((double)c, thr);
        if (cs) cs[g * Q + q] = c;
        if (cd) cd[g * Q + q] = ok ? (double)c : BIG;
        if (ok) cap[g] = 1;
    }
    __syncthreads();
    CostView<CT> C{cg, cs, Q, G};
    const int64_t K = a.topk;
    bool good = true;
    if (Q > 0 && G > 0 && K > 0) {
        // valid columns: any finite cost below the threshold
        if (tid < 32) {
            const int nv = warp_compact(G, [&](int g) { return cap[g] != 0; }, valid, nullptr);
            if (lane == 0) sh_n = nv;
        }
        __syncthreads();
        const int nv = sh_n;
        if (nv > 0) {
            const int kc = (int)(K < (int64_t)(1 << 30) ? K : (int64_t)(1 << 30));
            for (int t = tid; t < nv; t += nthr) cap[valid[t]] = kc;
            for (int q = tid; q < Q; q += nthr) preds[q] = q;
            __syncthreads();
            if (a.strategy == 0) {  // global, :239-286
                const int64_t kn = K * (int64_t)nv;
                const int M = (int)(kn < (int64_t)Q ? kn : (int64_t)Q);
                for (int t = tid; t < M; t += nthr) cols[t] = valid[t % nv];
                __syncthreads();
                good = solve(C, cd, preds, Q, cols, M, thr, BIG, asg, m, sh);
                if (good)
                    for (int q = tid; q < Q; q += nthr)
                        if (asg[q] >= 0) {
                            const int c = cols[asg[q]];
                            if (ok_cost(C.at(q, c), thr)) p2g[q] = c;
                        }
                __syncthreads();
            } else if (a.strategy == 1) {  // round, :294-366
                int nrem = Q;
                int* pa = preds;
                int* pb = preds2;
                for (int64_t r = 0; r < K && good; ++r) {
                    if (tid < 32) {
                        const int M = warp_compact(nv, [&](int t) { return cap[valid[t]] > 0; }, cols, valid);
                        if (lane == 0) sh_n = M;
                    }
                    __syncthreads();
                    int M = sh_n;
                    __syncthreads();
                    if (M == 0 || nrem == 0) break;
                    if (M > nrem) M = nrem;
                    good = solve(C, cd, pa, nrem, cols, M, thr, BIG, asg, m, sh);
                    if (!good) break;
                    // assignments (distinct columns within a round)
                    for (int k = tid; k < nrem; k += nthr) {
                        if (asg[k] >= 0) {
                            const int q = pa[k], c = cols[asg[k]];
                            if (ok_cost(C.at(q, c), thr)) {
                                p2g[q] = c;
                                if (cap[c] > 0) cap[c] -= 1;
                            }
                        }
                    }
                    __syncthreads();
                    if (tid < 32) {
                        const int nn = warp_compact(nrem, [&](int k) { return p2g[pa[k]] < 0; }, pb, pa);
                        if (lane == 0) sh_n = nn;
                    }
                    __syncthreads();
                    nrem = sh_n;
                    __syncthreads();
                    int* tmp = pa; pa = pb; pb = tmp;
                    if (nrem == 0) break;
                }
            } else if (a.strategy == 2) {  // greedy, :372-393
                if (tid < 32) greedy(C, preds, Q, valid, nv, thr, cap, p2g);
                __syncthreads();
            } else {  // pseudo-greedy, :400-463
                const int M = nv < Q ? nv : Q;
                for (int t = tid; t < M; t += nthr) cols[t] = valid[t];
                __syncthreads();
                good = solve(C, cd, preds, Q, cols, M, thr, BIG, asg, m, sh);
                if (good) {
                    for (int q = tid; q < Q; q += nthr)
                        if (asg[q] >= 0) {
                            const int c = cols[asg[q]];
                            if (ok_cost(C.at(q, c), thr)) {
                                p2g[q] = c;
                                if (cap[c] > 0) cap[c] -= 1;
                            }
                        }
                    __syncthreads();
                    if (tid < 32) {
                        const int nr = warp_compact(Q, [&](int q) { return p2g[q] < 0; }, preds2, nullptr);
                        if (nr > 0) greedy(C, preds2, nr, valid, nv, thr, cap, p2g);
                    }
                    __syncthreads();
                }
            }
        }
    }
    if (!good && tid == 0) {
        atomicOr(a.status, 1);
        failed = 1;
    }
    __syncthreads();
    if (failed) {
        for (int q = tid; q < Q; q += nthr) { out_p[q] = -1; out_r[q] = -1; }
        return;
    }
    // rank per GT by (cost, q), src/cpu/matching.cpp:538-565.  With K = 1
    // every strategy gives a GT at most one prediction, so each rank is 0.
    for (int q = tid; q < Q; q += nthr) {
        const int g = p2g[q];
        int64_t pr = -1;
        int64_t pg = -1;
        if (g >= 0 && ok_cost(C.at(q, g), thr)) {
            pg = g;
            int64_t rank = 0;
            if (K > 1) {
                const double c = C.at(q, g);
                for (int q2 = 0; q2 < Q; ++q2) {
                    if (q2 == q || p2g[q2] != g) continue;
                    const double c2 = C.at(q2, g);
                    if (!ok_cost(c2, thr)) continue;
                    if (c2 < c || (c2 == c && q2 < q)) ++rank;
                }
            }
            if (rank < K) pr = rank;
        }
        out_p[q] = pg;
        out_r[q] = pr;
    }
}

template __global__ void match_kernel<float>(MatchArgs<float>);
template __global__ void match_kernel<double>(MatchArgs<double>);

size_t match_smem_bytes(int Q, int G, size_t cost_elem, int stage) {
    auto r = [](size_t b) { return (b + 15) & ~size_t(15); };
    size_t s = 3 * r(sizeof(double) * (Q + 1)) + 3 * r(sizeof(int) * (Q + 1)) +
               2 * r(sizeof(int) * (G + 1)) + 4 * r(sizeof(int) * (Q + 1)) +
               r(sizeof(int) * ((Q > G ? Q : G) + 1));
    if (stage >= 1) s += r(cost_elem * (size_t)Q * G);
    if (stage >= 2) s += r(sizeof(double) * (size_t)Q * G);
    return s;
}

}  // namespace mlb
