// capi.cu -- extern "C" entry points declared in include/mask_loss_b200.h.
//
// Each entry validates its arguments with the reference's rules, carves the
// caller's workspace, and launches on the caller's stream.  No device memory
// is allocated here and nothing synchronises the device.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <map>
#include <mutex>
#include <vector>
#include <string>

#include "common.cuh"
#include "kernels.cuh"

using namespace mlb;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(ML_ECUDA, "CUDA error in %s: %s", where, cudaGetErrorString(e));
}

std::atomic<int64_t> g_launches{0};

#define ML_CHECK_LAUNCH(where)                                  \
    do {                                                        \
        g_launches.fetch_add(1, std::memory_order_relaxed);     \
        cudaError_t e_ = cudaGetLastError();                    \
        if (e_ != cudaSuccess) return cuda_fail(e_, where);     \
    } while (0)

// Optional per-launch CUDA-event timing of the hot kernels (ml_profile_*).
struct ProfRec {
    cudaEvent_t a, b;
    int kind;
};
std::mutex g_prof_mu;
std::vector<ProfRec> g_prof;
std::atomic<int> g_prof_on{0};

struct ProfScope {
    ProfRec r{nullptr, nullptr, -1};
    cudaStream_t st;
    ProfScope(int kind, cudaStream_t s) : st(s) {
        if (!g_prof_on.load(std::memory_order_relaxed)) return;
        if (cudaEventCreate(&r.a) != cudaSuccess || cudaEventCreate(&r.b) != cudaSuccess) return;
        r.kind = kind;
        cudaEventRecord(r.a, st);
    }
    ~ProfScope() {
        if (r.kind < 0) return;
        cudaEventRecord(r.b, st);
        std::lock_guard<std::mutex> g(g_prof_mu);
        g_prof.push_back(r);
    }
};

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Dense-mask costs run on the tensor-core kernel (dense_mma.cu) where it
// applies; MASK_LOSS_B200_DENSE_MMA=0 keeps them on the CUDA-core kernel
// (dense.cu), which also covers entropy weights, focal terms and GT_out > 64.
const bool g_dense_mma_off = [] {
    const char* v = getenv("MASK_LOSS_B200_DENSE_MMA");
    return v && v[0] == '0';
}();
// fp32 logits run on the kind::tf32 kernel (GT_total <= 64);
// MASK_LOSS_B200_DENSE_TF32=0 keeps them on the bf16 hi/lo one.
const bool g_dense_tf32_off = [] {
    const char* v = getenv("MASK_LOSS_B200_DENSE_TF32");
    return v && v[0] == '0';
}();

// Raise a kernel's dynamic shared-memory limit once per (kernel, device);
// later calls with the same or a smaller size touch no CUDA API (so they are
// safe inside stream capture).
std::mutex g_smem_mu;
std::map<std::pair<int, const void*>, int> g_smem_done;

template <typename K>
cudaError_t ensure_smem(K kernel, size_t bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const auto key = std::make_pair(dev, reinterpret_cast<const void*>(kernel));
    std::lock_guard<std::mutex> g(g_smem_mu);
    auto it = g_smem_done.find(key);
    if (it != g_smem_done.end() && (int)bytes <= it->second) return cudaSuccess;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) g_smem_done[key] = (int)bytes;
    return e;
}

int sm_count() {
    static int cached[64] = {};
    int dev = 0, n = 148;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return n;
    if (cached[dev]) return cached[dev];
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
        cached[dev] = n;
    else
        n = 148;
    return n > 0 ? n : 148;
}

// ---------------------------------------------------------------------------
// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// ---------------------------------------------------------------------------
// Forward plan: tiling, workspace layout.
// ---------------------------------------------------------------------------
// The mixed-cell table replaces per-pixel label reads for s > 1 (see
// common.cuh for its layout and limits).
bool mixtab_usable(int s, int gout) {
    return s > 1 && s <= 255 && gout <= kMixMaxCols;
}

size_t mixtab_bytes(int B, int HW) { return align256(sizeof(uint4) * (size_t)B * HW); }

struct FwdPlan {
    int L, B, Q, H, W, Ht, Wt, s, C, gt_total, gout, bg;
    bool unc, foc, tma_ok;
    int ldt, esize;  // mask-logit type (0 fp32, 1 bf16, 2 fp16) and its bytes
    int nacc, nrow;
    int qrows, qrows_pad, nqt, chunk_cells, nchunk, part_stride;
    size_t cost_smem;
    // workspace offsets
    size_t off_totals, off_codes, off_part, off_sep, off_total, off_rawI, off_rawT, off_qstat, bytes;
    size_t off_mixtab;  // mixed-cell table (s > 1), or SIZE_MAX when not used
};

size_t cost_smem_bytes(int qrows_pad, int esize) {
    return 1024 + (size_t)kStages * (2 * (size_t)qrows_pad * KBOX * esize + KC * 4) + 16 * kStages;
}

// Calls f(T{}) with T the plan's mask-logit element type.
template <typename F>
int with_logit_type(int ldt, F&& f) {
    if (ldt == 1) return f(__nv_bfloat16{});
    if (ldt == 2) return f(__half{});
    return f(float{});
}

int validate_dims(const ml_dims* d) {
    if (!d) return fail(ML_EINVAL, "dims is null");
    if (d->L < 0 || d->B < 0 || d->Q < 0 || d->C < 0 || d->GT_total < 0)
        return fail(ML_ESHAPE, "negative dimension");
    if (d->H <= 0 || d->W <= 0) return fail(ML_ESHAPE, "mask_logits must have positive spatial size");
    if (d->Ht % d->H != 0 || d->Wt % d->W != 0)
        return fail(ML_ESHAPE, "Target resolution must be an integer multiple of mask_logits resolution.");
    if (d->Ht / d->H != d->Wt / d->W)
        return fail(ML_ESHAPE, "Target downsample factors must be equal in both dimensions");
    if (d->Ht / d->H > 16) return fail(ML_EUNSUPPORTED, "downsample factor above 16 is not supported");
    const int64_t HW = d->H * d->W;
    if (HW >= (int64_t(1) << 31) || d->L * d->B * d->Q >= (int64_t(1) << 31) ||
        d->Ht * d->Wt >= (int64_t(1) << 31))
        return fail(ML_EUNSUPPORTED, "dimension product exceeds 2^31");
    if (d->GT_total >= 32767) return fail(ML_EUNSUPPORTED, "GT_total above 32766 is not supported");
    return ML_OK;
}

int validate_params(const ml_params* p, int64_t C) {
    if (!p) return fail(ML_EINVAL, "params is null");
    if (p->mask_gamma < 0.0f) return fail(ML_EINVAL, "mask focal_gamma must be non-negative");
    if (!(p->mask_alpha < 0.0f || p->mask_alpha <= 1.0f))
        return fail(ML_EINVAL, "mask focal_alpha must be in [0, 1] or negative to disable");
    if (p->cls_gamma < 0.0f) return fail(ML_EINVAL, "cls focal_gamma must be non-negative");
    if (!(p->cls_alpha < 0.0f || p->cls_alpha <= 1.0f))
        return fail(ML_EINVAL, "cls focal_alpha must be in [0, 1] or negative to disable");
    if (p->uncertainty_gamma < 0.0f) return fail(ML_EINVAL, "uncertainty_gamma must be non-negative");
    if (!(p->uncertainty_gamma_min >= 0.0f && p->uncertainty_gamma_min <= 1.0f))
        return fail(ML_EINVAL, "uncertainty_gamma_min must be in [0,1]");
    if (p->topk_matches < 0) return fail(ML_EINVAL, "K must be non-negative");
    if (p->strategy_id < 0 || p->strategy_id > 3) return fail(ML_EINVAL, "Invalid matching strategy id");
    if (p->logits_dtype < 0 || p->logits_dtype > 2)
        return fail(ML_EINVAL, "logits_dtype must be 0 (fp32), 1 (bf16) or 2 (fp16)");
    const bool has_void = p->void_class_index >= 0 && p->void_class_index < C;
    if (p->use_softmax_label_loss && p->force_unmatched_class_to_background && !has_void)
        return fail(ML_EINVAL,
                    "void_class_index must be provided when using softmax label loss and forcing "
                    "unmatched class logits");
    return ML_OK;
}

template <bool UNC, bool FOC, bool TMA, bool MIX, typename T>
int cost_blocks_per_sm_t(size_t smem, int threads) {
    auto k = cost_partial_kernel<UNC, FOC, TMA, MIX, T>;
    int n = 0;
    if (ensure_smem(k, smem) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, threads, smem) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

// Resident cost CTAs per SM for the kernel instance the plan launches (its
// registers and shared memory); without a device, the shared-memory bound.
int cost_blocks_per_sm(const FwdPlan& P, int threads) {
    const bool mix = P.s > 1;
    int n = with_logit_type(P.ldt, [&](auto tag) -> int {
        using T = decltype(tag);
        int r = 0;
#define ML_OCC(U, F) \
    r = P.tma_ok ? (mix ? cost_blocks_per_sm_t<U, F, true, true, T>(P.cost_smem, threads)      \
                        : cost_blocks_per_sm_t<U, F, true, false, T>(P.cost_smem, threads))    \
                 : (mix ? cost_blocks_per_sm_t<U, F, false, true, T>(P.cost_smem, threads)     \
                        : cost_blocks_per_sm_t<U, F, false, false, T>(P.cost_smem, threads))
        if (P.unc) { if (P.foc) ML_OCC(true, true); else ML_OCC(true, false); }
        else { if (P.foc) ML_OCC(false, true); else ML_OCC(false, false); }
#undef ML_OCC
        return r;
    });
    if (n < 1) n = (int)std::min<size_t>(228 * 1024 / (P.cost_smem + 1024), 2048 / threads);
    return n < 1 ? 1 : n;
}

int make_plan(const ml_dims* d, const ml_params* p, FwdPlan* P) {
    int rc = validate_dims(d);
    if (rc) return rc;
    P->L = (int)d->L; P->B = (int)d->B; P->Q = (int)d->Q; P->H = (int)d->H; P->W = (int)d->W;
    P->Ht = (int)d->Ht; P->Wt = (int)d->Wt; P->s = P->Ht / P->H; P->C = (int)d->C;
    P->gt_total = (int)d->GT_total;
    const bool skip = p->background_index >= 0 && p->background_index < d->GT_total;
    P->bg = skip ? (int)p->background_index : P->gt_total;
    P->gout = P->gt_total - (skip ? 1 : 0);
    P->unc = p->uncertainty_gamma != 0.0f;
    P->foc = p->mask_gamma > 0.0f || p->mask_alpha >= 0.0f;
    P->nacc = P->unc ? 3 : 2;
    P->nrow = P->unc ? 5 : 3;
    P->ldt = (int)p->logits_dtype;
    P->esize = P->ldt ? 2 : 4;
    const int HW = P->H * P->W;
    P->tma_ok = ((int64_t)HW * P->esize) % 16 == 0;  // TMA row pitch: a multiple of 16 bytes
    const int Q = P->Q > 0 ? P->Q : 1;
    P->nqt = (Q + 127) / 128;
    P->qrows = (Q + P->nqt - 1) / P->nqt;
    P->qrows_pad = (P->qrows + 31) / 32 * 32;
    P->cost_smem = cost_smem_bytes(P->qrows_pad, P->esize);
    const int threads = 2 * P->qrows_pad + 32;
    int per_sm = cost_blocks_per_sm(*P, threads);
    // chunks per (image, query tile): the smallest count whose CTAs fill the
    // SMs in whole waves to >= 95 % (else the best found up to 4 waves)
    const int64_t base = (int64_t)P->L * P->B * P->nqt;
    const int64_t slots = (int64_t)sm_count() * per_sm;
    const int64_t max_ch = std::max<int64_t>(1, (HW + KC - 1) / KC);
    int64_t best = 1;
    double best_eff = -1.0;
    const int64_t hi = base > 0 ? std::max<int64_t>(1, 4 * ((slots + base - 1) / base)) : 1;
    for (int64_t nch = 1; nch <= std::min<int64_t>(max_ch, hi); ++nch) {
        const int64_t total = base * nch;
        const int64_t waves = (total + slots - 1) / slots;
        const double eff = (double)total / (double)(waves * slots);
        if (eff > best_eff + 1e-9) { best_eff = eff; best = nch; }
        if (eff >= 0.95) { best = nch; break; }
    }
    if (best > max_ch) best = max_ch;
    P->chunk_cells = (int)(((HW + best - 1) / best + KC - 1) / KC * KC);
    P->nchunk = (HW + P->chunk_cells - 1) / P->chunk_cells;
    P->part_stride = (P->nacc * std::max(P->gout, 1) + P->nrow) * P->qrows_pad;
    // workspace
    const size_t LBQ = (size_t)P->L * P->B * P->Q;
    const size_t LBQG = LBQ * P->gout;
    size_t off = 0;
    P->off_totals = off; off += align256(sizeof(int32_t) * (size_t)P->B * P->gt_total);
    P->off_codes = off; off += align256(sizeof(int32_t) * (size_t)P->B * HW);
    P->off_mixtab = SIZE_MAX;
    if (mixtab_usable(P->s, P->gout)) {
        P->off_mixtab = off;
        off += mixtab_bytes(P->B, HW);
    }
    P->off_part = off;
    off += align256(sizeof(float) * (size_t)base * P->nchunk * 2 * P->part_stride);
    P->off_sep = off; off += align256(sizeof(float) * 3 * LBQG);
    P->off_total = off; off += align256(sizeof(float) * LBQG);
    P->off_rawI = off; off += align256(sizeof(float) * LBQG);
    P->off_rawT = off; off += align256(sizeof(float) * LBQG);
    P->off_qstat = off; off += align256(sizeof(float) * kQStat * LBQ);
    P->bytes = off + 256;
    return ML_OK;
}

unsigned char* ws_base(void* ws) {
    return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~uintptr_t(255));
}

CostArgs cost_args(const FwdPlan& P, const ml_params* p, const float* ml, const int64_t* mt,
                   const float* cl, const int64_t* ct, unsigned char* ws, int32_t* status) {
    CostArgs a{};
    a.logits = ml; a.targets = mt; a.cls_logits = cl; a.cls_targets = ct;
    a.totals = reinterpret_cast<int32_t*>(ws + P.off_totals);
    a.codes = reinterpret_cast<int32_t*>(ws + P.off_codes);
    a.mixtab = P.off_mixtab != SIZE_MAX ? reinterpret_cast<const uint4*>(ws + P.off_mixtab) : nullptr;
    a.part = reinterpret_cast<float*>(ws + P.off_part);
    a.sep = reinterpret_cast<float*>(ws + P.off_sep);
    a.total = reinterpret_cast<float*>(ws + P.off_total);
    a.rawI = reinterpret_cast<float*>(ws + P.off_rawI);
    a.rawT = reinterpret_cast<float*>(ws + P.off_rawT);
    a.qstat = reinterpret_cast<float*>(ws + P.off_qstat);
    a.status = status;
    a.L = P.L; a.B = P.B; a.Q = P.Q; a.H = P.H; a.W = P.W; a.Ht = P.Ht; a.Wt = P.Wt; a.s = P.s;
    a.C = P.C; a.gt_total = P.gt_total; a.gout = P.gout; a.bg = P.bg;
    a.qrows = P.qrows; a.qrows_pad = P.qrows_pad; a.nqt = P.nqt;
    a.chunk_cells = P.chunk_cells; a.nchunk = P.nchunk; a.part_stride = P.part_stride;
    a.smooth = p->smooth; a.sigmoid_scale = p->sigmoid_scale; a.dice_scale = p->dice_scale;
    a.cls_scale = p->cls_scale; a.ug = p->uncertainty_gamma; a.ugmin = p->uncertainty_gamma_min;
    a.mask_gamma = p->mask_gamma; a.mask_alpha = p->mask_alpha;
    a.cls_gamma = p->cls_gamma; a.cls_alpha = p->cls_alpha;
    a.area_scale = (float)(P.s * P.s);
    a.normalize_uncertainty = p->normalize_uncertainty;
    a.use_softmax = p->use_softmax_label_loss;
    a.force_cls = p->force_unmatched_class_to_background;
    a.has_void = (p->void_class_index >= 0 && p->void_class_index < P.C) ? 1 : 0;
    a.void_index = a.has_void ? (int)p->void_class_index : -1;
    return a;
}

template <bool UNC, bool FOC, bool TMA, typename T>
int launch_cost_t(const FwdPlan& P, const CUtensorMap& tm, const CostArgs& a, cudaStream_t st) {
    auto k = P.s > 1 ? cost_partial_kernel<UNC, FOC, TMA, true, T>
                     : cost_partial_kernel<UNC, FOC, TMA, false, T>;
    cudaError_t e = ensure_smem(k, P.cost_smem);
    if (e != cudaSuccess) return cuda_fail(e, "cost_partial_kernel attributes");
    dim3 grid(P.nchunk, P.nqt, P.L * P.B);
    ProfScope prof(0, st);
    launch_pdl(k, grid, dim3(2 * P.qrows_pad + 32), P.cost_smem, st, tm, a);
    ML_CHECK_LAUNCH("cost_partial_kernel");
    return ML_OK;
}

// Label codes + histogram (always), and when `costs` the chunk partials and
// both finalize kernels.  `a` decides which outputs are written.
int run_prep(const FwdPlan& P, const CostArgs& a, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(const_cast<int32_t*>(a.totals), 0,
                                    sizeof(int32_t) * (size_t)P.B * P.gt_total, st);
    if (e != cudaSuccess) return cuda_fail(e, "memset totals");
    cudaError_t le;
    ProfScope prof(3, st);
    if (a.codes) {
        le = launch_label_code(a.targets, P.B, P.H, P.W, P.Wt, P.s, P.gt_total, P.bg,
                               const_cast<int32_t*>(a.codes), const_cast<int32_t*>(a.totals),
                               const_cast<uint4*>(a.mixtab), st);
    } else {  // histogram only
        le = launch_label_hist(a.targets, P.B, (int64_t)P.Ht * P.Wt, P.gt_total,
                               const_cast<int32_t*>(a.totals), st);
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (le != cudaSuccess) return cuda_fail(le, a.codes ? "label_code_kernel" : "label_hist_kernel");
    return ML_OK;
}

int run_cost_core(const FwdPlan& P, CostArgs& a, const float* mask_logits, cudaStream_t st);

// 2-D tensor map over the mask logits (rows = L*B*Q, columns = H*W) with
// boxes of 32 cells x qrows rows: 128-byte rows with the 128-byte swizzle for
// fp32, 64-byte rows with the 64-byte swizzle for 16-bit logits.  False when
// the rows are not 16-byte strided or aligned (the kernels then load plainly).
bool logits_tensor_map(const FwdPlan& P, const float* mask_logits, CUtensorMap* tm) {
    memset(tm, 0, sizeof(*tm));
    const int64_t LBQ = (int64_t)P.L * P.B * P.Q;
    if (!P.tma_ok || (reinterpret_cast<uintptr_t>(mask_logits) % 16) != 0 || LBQ == 0) return false;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const CUtensorMapDataType dt = P.ldt == 1   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : P.ldt == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    const cuuint64_t dims[2] = {(cuuint64_t)P.H * P.W, (cuuint64_t)LBQ};
    const cuuint64_t strides[1] = {(cuuint64_t)P.H * P.W * P.esize};
    const cuuint32_t box[2] = {(cuuint32_t)KBOX, (cuuint32_t)P.qrows};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = enc(tm, dt, 2, const_cast<float*>(mask_logits), dims, strides, box, es,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     P.esize == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int run_finalize(const FwdPlan& P, CostArgs& a, cudaStream_t st);

int run_costs(const FwdPlan& P, CostArgs& a, const float* mask_logits, cudaStream_t st) {
    int rc = run_prep(P, a, st);
    if (rc) return rc;
    return run_cost_core(P, a, mask_logits, st);
}

// Chunk partials + both finalize kernels (codes and totals already built).
int run_cost_core(const FwdPlan& P, CostArgs& a, const float* mask_logits, cudaStream_t st) {
    int rc = ML_OK;
    const int64_t LBQ = (int64_t)P.L * P.B * P.Q;
    if (LBQ == 0 || P.gout == 0) return ML_OK;
    // the cost kernel clears its own partial slots (no memset)
    CUtensorMap tm;
    const bool tma = logits_tensor_map(P, mask_logits, &tm);
    rc = with_logit_type(P.ldt, [&](auto tag) -> int {
        using T = decltype(tag);
        if (P.unc) {
            if (P.foc) return tma ? launch_cost_t<true, true, true, T>(P, tm, a, st) : launch_cost_t<true, true, false, T>(P, tm, a, st);
            return tma ? launch_cost_t<true, false, true, T>(P, tm, a, st) : launch_cost_t<true, false, false, T>(P, tm, a, st);
        }
        if (P.foc) return tma ? launch_cost_t<false, true, true, T>(P, tm, a, st) : launch_cost_t<false, true, false, T>(P, tm, a, st);
        return tma ? launch_cost_t<false, false, true, T>(P, tm, a, st) : launch_cost_t<false, false, false, T>(P, tm, a, st);
    });
    if (rc) return rc;
    return run_finalize(P, a, st);
}

// Row statistics and pair costs from the chunk partials (both target modes).
int run_finalize(const FwdPlan& P, CostArgs& a, cudaStream_t st) {
    const int64_t LBQ = (int64_t)P.L * P.B * P.Q;
    const unsigned rb = (unsigned)((LBQ * 32 + 255) / 256);
    ProfScope prof(4, st);
    if (P.unc) launch_pdl(cost_rows_kernel<true, false>, dim3(rb), dim3(256), 0, st, a);
    else if (P.foc) launch_pdl(cost_rows_kernel<false, false>, dim3(rb), dim3(256), 0, st, a);
    else launch_pdl(cost_rows_kernel<false, true>, dim3(rb), dim3(256), 0, st, a);
    ML_CHECK_LAUNCH("cost_rows_kernel");
    dim3 pg((unsigned)((P.qrows * P.gout + 31) / 32), P.nqt, P.L * P.B);
    if (P.unc) launch_pdl(cost_pairs_kernel<true>, dim3(pg), dim3(256), 0, st, a);
    else launch_pdl(cost_pairs_kernel<false>, dim3(pg), dim3(256), 0, st, a);
    ML_CHECK_LAUNCH("cost_pairs_kernel");
    return ML_OK;
}

// Dense per-GT masks: counts + areas, then the dense cost kernel, then the
// same finalize.  The counts live after the plan's workspace.
// Counts take 4 bytes a cell and GT (fp32 for the tf32 kernel; the bf16
// forms use the first half).
size_t dense_count_bytes(const FwdPlan& P) {
    return align256(sizeof(float) * (size_t)P.B * P.H * P.W * std::max(P.gt_total, 1));
}

// 2-D tensor map over the dense counts (rows = B*GT_total GT planes, columns
// = H*W cells): boxes of 32 cells x the MMA's N rows; bf16 bit patterns with
// the 64-byte swizzle (bf16 tensor-core kernel) or fp32 with the 128-byte
// one (tf32 kernel), the layouts their B descriptors expect.
bool counts_tensor_map(const FwdPlan& P, const void* cnt, CUtensorMap* km, bool f32) {
    memset(km, 0, sizeof(*km));
    const int HW = P.H * P.W;
    if (HW % 8 != 0 || (reinterpret_cast<uintptr_t>(cnt) % 16) != 0) return false;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)HW, (cuuint64_t)P.B * P.gt_total};
    const cuuint64_t strides[1] = {(cuuint64_t)HW * (f32 ? 4 : 2)};
    const cuuint32_t box[2] = {32u, (cuuint32_t)dense_mma_n(P.gt_total)};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = enc(km, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                     const_cast<void*>(cnt), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 2-D tensor map over the uint8 masks themselves (s = 1; rows = B*GT_total
// planes, columns = H*W cells): boxes of 32 cells x the MMA's N rows, no
// swizzle -- the tf32 kernel turns them into its fp32 B tile.
bool masks_tensor_map(const FwdPlan& P, const uint8_t* masks, CUtensorMap* km) {
    memset(km, 0, sizeof(*km));
    const int HW = P.H * P.W;
    if (P.s != 1 || HW % 16 != 0 || (reinterpret_cast<uintptr_t>(masks) % 16) != 0) return false;
    EncodeTiledFn enc = encode_fn();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)HW, (cuuint64_t)P.B * P.gt_total};
    const cuuint64_t strides[1] = {(cuuint64_t)HW};
    const cuuint32_t box[2] = {32u, (cuuint32_t)dense_mma_n(P.gt_total)};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = enc(km, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(masks), dims, strides,
                     box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int run_dense_costs(const FwdPlan& P, CostArgs& a, const uint8_t* masks, unsigned char* ws,
                    cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(const_cast<int32_t*>(a.totals), 0,
                                    sizeof(int32_t) * (size_t)P.B * P.gt_total, st);
    if (e != cudaSuccess) return cuda_fail(e, "memset mask areas");
    uint16_t* cnt = reinterpret_cast<uint16_t*>(ws + (P.bytes - 256));
    const int64_t LBQ = (int64_t)P.L * P.B * P.Q;
    // which cost kernel, before the counts are written in its format
    CUtensorMap tm, km;
    const bool mma = LBQ > 0 && P.gout > 0 && !g_dense_mma_off && logits_tensor_map(P, a.logits, &tm) &&
                     dense_mma_usable(a, P.ldt, P.unc, P.foc, true);
    const bool tf32 = mma && !g_dense_tf32_off && dense_mma_tf32_usable(a, P.ldt);
    // s = 1: the tf32 kernel reads the masks themselves and sums the mask
    // areas as it goes, so no count pass runs
    // (the producers' 256 threads convert N x 32 mask bytes a block, 4 each:
    // N <= 32)
    const bool masks_b = (tf32 || (mma && P.ldt == 1 && dense_mma_n(P.gt_total) <= 32)) &&
                         masks_tensor_map(P, masks, &km);
    if (P.B > 0 && P.gt_total > 0 && !masks_b) {
        e = launch_dense_count(masks, P.B, P.H, P.W, P.Ht, P.Wt, P.s, P.gt_total,
                               masks_b ? nullptr : cnt, const_cast<int32_t*>(a.totals), st, tf32);
        g_launches.fetch_add(1);
        if (e != cudaSuccess) return cuda_fail(e, "dense_count_kernel");
    }
    if (LBQ == 0 || P.gout == 0) return ML_OK;
    {
        ProfScope prof(0, st);  // profiled as the cost stage
        if (masks_b && tf32)
            e = launch_dense_mma_tf32(tm, km, a, st, true);   // kind::tf32, B from the masks
        else if (masks_b)
            e = launch_dense_mma(tm, km, a, st, P.ldt, true);  // kind::f16 (bf16 logits), B from the masks
        else if (tf32 && counts_tensor_map(P, cnt, &km, true))
            e = launch_dense_mma_tf32(tm, km, a, st, false);  // kind::tf32, B from fp32 counts
        else if (mma && !tf32 && counts_tensor_map(P, cnt, &km, false))
            e = launch_dense_mma(tm, km, a, st, P.ldt, false);  // tensor cores, kind::f16
        else if (tf32)
            return fail(ML_EINVAL, "dense counts tensor map could not be encoded");
        else
            e = launch_dense_cost(a, P.unc, P.foc, cnt, st, P.ldt);
    }
    g_launches.fetch_add(1);
    if (e != cudaSuccess) return cuda_fail(e, "dense_cost_kernel");
    return run_finalize(P, a, st);
}

int check_ws(void* ws, size_t have, size_t need) {
    if (need == 0) return ML_OK;
    if (!ws) return fail(ML_EWORKSPACE, "workspace is null (need %zu bytes)", need);
    if (have < need) return fail(ML_EWORKSPACE, "workspace too small: %zu < %zu bytes", have, need);
    return ML_OK;
}

template <typename CT>
int launch_match(const CT* costs, int64_t N, int64_t Q, int64_t G, double thr, int64_t K, int64_t strat,
                 int64_t* p2g, int64_t* prnd, int32_t* status, cudaStream_t st) {
    if (N == 0 || Q == 0) return ML_OK;
    if (Q > 3000 || G > 32766) return fail(ML_EUNSUPPORTED, "solver supports Q <= 3000 and GT_out <= 32766");
    if (!status) return fail(ML_EINVAL, "dev_status is null");
    MatchArgs<CT> a;
    a.costs = costs; a.pred_to_gt = p2g; a.pred_round = prnd; a.status = status;
    a.Q = (int)Q; a.G = (int)G; a.inf_thresh = thr; a.topk = K; a.strategy = (int)strat;
    const size_t limit = 200 * 1024;
    a.stage_cost = 2;
    size_t smem = match_smem_bytes((int)Q, (int)G, sizeof(CT), a.stage_cost);
    while (a.stage_cost > 0 && smem > limit)
        smem = match_smem_bytes((int)Q, (int)G, sizeof(CT), --a.stage_cost);
    if (smem > 227 * 1024) return fail(ML_EUNSUPPORTED, "solver state does not fit shared memory");
    // one thread per solver column (Q + 1 of them) up to 256, whole warps
    const int threads = (int)std::min<int64_t>(kMatchMaxThreads, std::max<int64_t>(64, (Q + 1 + 31) / 32 * 32));
    auto k = match_kernel<CT>;
    cudaError_t e = ensure_smem(k, smem);
    if (e != cudaSuccess) return cuda_fail(e, "match_kernel attributes");
    {
        ProfScope prof(2, st);
        launch_pdl(k, dim3((unsigned)N), dim3(threads), smem, st, a);
    }
    ML_CHECK_LAUNCH("match_kernel");
    return ML_OK;
}

LossArgs loss_args(const FwdPlan& P, const ml_params* p) {
    LossArgs a{};
    a.L = P.L; a.B = P.B; a.Q = P.Q; a.H = P.H; a.W = P.W; a.Ht = P.Ht; a.Wt = P.Wt; a.s = P.s;
    a.C = P.C; a.G = P.gout; a.gt_total = P.gt_total; a.bg = P.bg;
    a.num_masks = (float)p->num_masks;
    a.smooth = p->smooth; a.sigmoid_scale = p->sigmoid_scale; a.dice_scale = p->dice_scale;
    a.cls_scale = p->cls_scale; a.ug = p->uncertainty_gamma; a.ugmin = p->uncertainty_gamma_min;
    a.mask_gamma = p->mask_gamma; a.mask_alpha = p->mask_alpha;
    a.cls_gamma = p->cls_gamma; a.cls_alpha = p->cls_alpha;
    a.force_masks = p->force_unmatched_masks_to_empty;
    a.force_cls = p->force_unmatched_class_to_background;
    a.has_void = (p->void_class_index >= 0 && p->void_class_index < P.C) ? 1 : 0;
    a.void_index = a.has_void ? (int)p->void_class_index : -1;
    a.use_softmax = p->use_softmax_label_loss;
    a.normalize_uncertainty = p->normalize_uncertainty;
    return a;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the pairwise-cost path.  Its scratch (label
// codes, per-image histogram, chunk partials, per-query statistics) lives in
// this fixed device array instead of a caller-provided workspace.  Every GPU
// that loads the library reserves it until the process exits.
// ---------------------------------------------------------------------------
constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.  The host-side
// symbol is only a stand-in; the real address comes from
// cudaGetSymbolAddress with the device current.  It is looked up on every
// call (it allocates nothing and is cheap), so a device or context reset
// between calls cannot leave a stale cached address behind.
int noalloc_scratch(unsigned char** out) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    *out = static_cast<unsigned char*>(ptr);
    return ML_OK;
}

// ---------------------------------------------------------------------------
// Point-sampled path.  The cost stage runs on a (L,B,Q,1,P) view of the
// sampled values: the plan is made for H=1, W=P, s=1.
// ---------------------------------------------------------------------------
struct SampledPlan {
    FwdPlan cp;          // cost-stage plan over the sampled values
    int H, W, Ht, Wt, P;
    size_t off_present, off_perm, off_scoords, off_zs, off_sort, bytes;
};

int make_sampled_plan(const ml_dims* d, const ml_params* p, int64_t P, SampledPlan* S) {
    int rc = validate_dims(d);
    if (rc) return rc;
    if (P <= 0 || P > kMaxSortPoints)
        return fail(ML_EUNSUPPORTED, "num_points must be in [1, %d]", kMaxSortPoints);
    if (p->force_unmatched_masks_to_empty)
        return fail(ML_EUNSUPPORTED, "force_unmatched_masks_to_empty is not supported with point sampling");
    if (p->uncertainty_gamma != 0.0f)
        return fail(ML_EUNSUPPORTED, "uncertainty weights are not used by point-sampled costs: pass uncertainty_gamma=0");
    ml_dims dv = *d;
    dv.H = 1; dv.W = P; dv.Ht = 1; dv.Wt = P;
    ml_params pf = *p;
    pf.logits_dtype = 0;  // the cost kernel reads the fp32 samples
    if ((rc = make_plan(&dv, &pf, &S->cp))) return rc;
    if (point_sort_smem((int)P, S->cp.gout) > 200 * 1024)
        return fail(ML_EUNSUPPORTED, "too many points x GT columns for the point sort");
    S->H = (int)d->H; S->W = (int)d->W; S->Ht = (int)d->Ht; S->Wt = (int)d->Wt; S->P = (int)P;
    const size_t LBQ = (size_t)d->L * d->B * d->Q;
    size_t off = S->cp.bytes;
    S->off_present = off; off += align256(sizeof(int32_t) * (size_t)d->B * d->GT_total);
    S->off_perm = off; off += align256(sizeof(int32_t) * (size_t)d->B * P);
    S->off_scoords = off; off += align256(sizeof(float) * 2 * (size_t)d->B * P);
    S->off_zs = off; off += align256(sizeof(float) * LBQ * P);
    S->off_sort = off; off += align256(point_sort_scratch_bytes((int)d->B, (int)P, S->cp.gout));
    S->bytes = off + 256;
    return ML_OK;
}

// present histogram, point sort (codes/totals of the cost plan), sampling.
int run_sampled_prep(const SampledPlan& S, const ml_params* p, const void* mask_logits, int dtype,
                     const int64_t* mask_targets, const float* coords, int align, unsigned char* ws,
                     CostArgs& a, cudaStream_t st) {
    const FwdPlan& P = S.cp;
    int32_t* present = reinterpret_cast<int32_t*>(ws + S.off_present);
    int32_t* perm = reinterpret_cast<int32_t*>(ws + S.off_perm);
    float* scoords = reinterpret_cast<float*>(ws + S.off_scoords);
    float* zs = reinterpret_cast<float*>(ws + S.off_zs);
    cudaError_t e = cudaMemsetAsync(present, 0, sizeof(int32_t) * (size_t)P.B * P.gt_total, st);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(const_cast<int32_t*>(a.totals), 0, sizeof(int32_t) * (size_t)P.B * P.gt_total, st);
    if (e != cudaSuccess) return cuda_fail(e, "memset histograms");
    const int HW = S.H * S.W;
    if (P.B > 0) {
        cudaError_t he = launch_label_hist(mask_targets, P.B, (int64_t)S.Ht * S.Wt, P.gt_total,
                                           present, st);
        g_launches.fetch_add(1, std::memory_order_relaxed);
        if (he != cudaSuccess) return cuda_fail(he, "label_hist_kernel");
        cudaError_t le = launch_point_sort(mask_targets, coords, P.B, S.Ht, S.Wt, S.P, P.gt_total, P.bg,
                                           P.gout, perm, const_cast<int32_t*>(a.codes), scoords,
                                           const_cast<int32_t*>(a.totals), st,
                                           reinterpret_cast<int32_t*>(ws + S.off_sort));
        g_launches.fetch_add(1);
        if (le != cudaSuccess) return cuda_fail(le, "point_sort_kernel");
    }
    const int64_t LB = (int64_t)P.L * P.B;
    if (LB > 0 && P.Q > 0) {
        cudaError_t le = launch_point_sample(dtype, mask_logits, scoords, P.B, P.L, P.Q, S.H, S.W,
                                             S.P, align, zs, st);
        g_launches.fetch_add(1);
        if (le != cudaSuccess) return cuda_fail(le, "point_sample_kernel");
        ML_CHECK_LAUNCH("point_sample_kernel");
    }
    a.present = present;
    a.logits = zs;
    (void)p;
    return ML_OK;
}

}  // namespace

extern "C" {

const char* ml_status_string(int status) {
    switch (status) {
        case ML_OK: return "ok";
        case ML_EINVAL: return "invalid argument";
        case ML_ESHAPE: return "invalid shape";
        case ML_EWORKSPACE: return "workspace missing or too small";
        case ML_ECUDA: return "CUDA error";
        case ML_ESOLVER: return "assignment solver failed";
        case ML_EUNSUPPORTED: return "unsupported size";
        default: return "unknown status";
    }
}

const char* ml_last_error(void) { return g_last_error.c_str(); }

int ml_version(void) { return 100; }

int64_t ml_launch_count(void) { return g_launches.load(); }

void ml_profile_enable(int on) { g_prof_on.store(on ? 1 : 0); }

int ml_profile_read(float* ms, int64_t* launches, int nkinds) {
    std::vector<ProfRec> recs;
    {
        std::lock_guard<std::mutex> g(g_prof_mu);
        recs.swap(g_prof);
    }
    for (int k = 0; k < nkinds; ++k) { ms[k] = 0.0f; launches[k] = 0; }
    int rc = ML_OK;
    for (auto& r : recs) {
        float t = 0.0f;
        if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess) {
            if (r.kind < nkinds) { ms[r.kind] += t; launches[r.kind] += 1; }
        } else {
            rc = fail(ML_ECUDA, "profile event read failed");
        }
        cudaEventDestroy(r.a);
        cudaEventDestroy(r.b);
    }
    return rc;
}

int64_t ml_gt_out(int64_t GT_total, int64_t bg) {
    return GT_total - ((bg >= 0 && bg < GT_total) ? 1 : 0);
}

size_t ml_mask_matching_workspace_size(const ml_dims* d, const ml_params* p) {
    FwdPlan P;
    if (!p || make_plan(d, p, &P)) return 0;
    return P.bytes;
}

size_t ml_match_workspace_size(int64_t, int64_t, int64_t, int64_t) { return 0; }

// Backward scratch: coef | statistics | (s > 1 label map) codes | mixed-cell table.
struct BwdLayout {
    size_t off_stats, off_codes, off_mixtab, bytes;
    bool cells;  // codes + table present
};

static BwdLayout bwd_layout(const ml_dims* d, const ml_params* p) {
    BwdLayout o{};
    const size_t LBQ = (size_t)d->L * d->B * d->Q;
    size_t off = align256(sizeof(float) * 3 * (size_t)d->L);
    o.off_stats = off;
    off += align256(sizeof(float) * kSaved * LBQ);
    const int s = d->H > 0 ? (int)(d->Ht / d->H) : 1;
    const bool skip = p && p->background_index >= 0 && p->background_index < d->GT_total;
    const int gout = (int)(d->GT_total - (skip ? 1 : 0));
    const int HW = (int)(d->H * d->W);
    o.cells = mixtab_usable(s, gout);
    if (o.cells) {
        o.off_codes = off;
        off += align256(sizeof(int32_t) * (size_t)d->B * HW);
        o.off_mixtab = off;
        off += mixtab_bytes((int)d->B, HW);
    }
    o.bytes = off + 256;
    return o;
}

size_t ml_mask_matching_backward_workspace_size(const ml_dims* d, const ml_params* p) {
    if (!d) return 0;
    return bwd_layout(d, p).bytes;
}

// Status word of the cost-only entries (which have no dev_status argument):
// the cost kernels OR bit 2 into it when a bounded pipeline wait runs out.
// Read (and cleared) by ml_cost_status.  Its address is looked up per call.
static __device__ int32_t g_cost_status;

int32_t* cost_status_ptr() {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_cost_status) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;  // the kernels then report nothing (as before)
    }
    return static_cast<int32_t*>(ptr);
}

int ml_pairwise_mask_loss_forward(const ml_dims* d, const ml_params* p, const float* mask_logits,
                                  const int64_t* mask_targets, const float* cls_logits,
                                  const int64_t* cls_targets, float* out, void* workspace,
                                  size_t workspace_bytes, ml_stream_t stream) {
    FwdPlan P;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if ((rc = make_plan(d, p, &P))) return rc;
    if ((rc = check_ws(workspace, workspace_bytes, P.bytes))) return rc;
    if (P.gout == 0) return ML_OK;
    unsigned char* ws = ws_base(workspace);
    CostArgs a = cost_args(P, p, mask_logits, mask_targets, cls_logits, cls_targets, ws,
                           cost_status_ptr());
    a.sep = out; a.total = nullptr; a.rawI = nullptr; a.rawT = nullptr;
    return run_costs(P, a, mask_logits, reinterpret_cast<cudaStream_t>(stream));
}

int ml_cost_status(int32_t* out) {
    if (!out) return fail(ML_EINVAL, "out is null");
    int32_t v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_cost_status, sizeof(v));
    if (e != cudaSuccess) return cuda_fail(e, "read the cost status word");
    if (v != 0) {
        const int32_t zero = 0;
        e = cudaMemcpyToSymbol(g_cost_status, &zero, sizeof(zero));
        if (e != cudaSuccess) return cuda_fail(e, "clear the cost status word");
    }
    *out = v;
    return ML_OK;
}

int ml_pairwise_mask_loss_forward_noalloc(const ml_dims* d, const ml_params* p,
                                          const float* mask_logits, const int64_t* mask_targets,
                                          const float* cls_logits, const int64_t* cls_targets,
                                          float* out, ml_stream_t stream) {
    FwdPlan P;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if (p->logits_dtype != 0)
        return fail(ML_EUNSUPPORTED, "ml_pairwise_mask_loss_forward_noalloc takes fp32 mask_logits");
    if ((rc = make_plan(d, p, &P))) return rc;
    // scratch layout: totals | codes | chunk partials | per-query statistics | mixed-cell table
    const size_t LBQ = (size_t)P.L * P.B * P.Q;
    const size_t n_tot = align256(sizeof(int32_t) * (size_t)P.B * P.gt_total);
    const size_t n_codes = align256(sizeof(int32_t) * (size_t)P.B * P.H * P.W);
    const size_t n_part =
        align256(sizeof(float) * (size_t)P.L * P.B * P.nqt * P.nchunk * 2 * P.part_stride);
    const size_t n_qstat = align256(sizeof(float) * kQStat * LBQ);
    const size_t n_mix = P.off_mixtab != SIZE_MAX ? mixtab_bytes(P.B, P.H * P.W) : 0;
    const size_t need = n_tot + n_codes + n_part + n_qstat + n_mix;
    if (need > kNoAllocScratchBytes)
        return fail(ML_EUNSUPPORTED,
                    "ml_pairwise_mask_loss_forward_noalloc: this call needs %zu bytes of scratch, "
                    "above the fixed %zu-byte limit; use ml_pairwise_mask_loss_forward with a "
                    "workspace instead", need, kNoAllocScratchBytes);
    if (P.gout == 0) return ML_OK;
    unsigned char* scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    CostArgs a = cost_args(P, p, mask_logits, mask_targets, cls_logits, cls_targets, scratch,
                           cost_status_ptr());
    a.totals = reinterpret_cast<int32_t*>(scratch);
    a.codes = reinterpret_cast<int32_t*>(scratch + n_tot);
    a.part = reinterpret_cast<float*>(scratch + n_tot + n_codes);
    a.qstat = reinterpret_cast<float*>(scratch + n_tot + n_codes + n_part);
    a.mixtab = n_mix ? reinterpret_cast<const uint4*>(scratch + n_tot + n_codes + n_part + n_qstat)
                     : nullptr;
    a.sep = out; a.total = nullptr; a.rawI = nullptr; a.rawT = nullptr;
    // run_costs clears the histogram and the partials before use (the array
    // keeps the previous call's contents); codes and statistics are fully
    // rewritten.
    return run_costs(P, a, mask_logits, reinterpret_cast<cudaStream_t>(stream));
}

size_t ml_noalloc_scratch_limit(void) { return kNoAllocScratchBytes; }

int ml_pairwise_label_loss_forward(int64_t L, int64_t B, int64_t Q, int64_t C, int64_t GT_total,
                                   int64_t bg, float scale, float gamma, float alpha,
                                   int32_t use_softmax, const float* cls_logits,
                                   const int64_t* cls_targets, float* out, ml_stream_t stream) {
    if (L < 0 || B < 0 || Q < 0 || C <= 0 || GT_total < 0)
        return fail(ML_ESHAPE, "class dimension must be positive");
    if (gamma < 0.0f) return fail(ML_EINVAL, "focal_gamma must be non-negative");
    if (!(alpha < 0.0f || alpha <= 1.0f)) return fail(ML_EINVAL, "focal_alpha must be in [0,1] or negative to disable");
    const bool skip = bg >= 0 && bg < GT_total;
    const int ibg = skip ? (int)bg : (int)GT_total;
    const int gout = (int)(GT_total - (skip ? 1 : 0));
    const int64_t rows = L * B * Q;
    if (gout == 0 || rows == 0) return ML_OK;
    const int64_t blocks = (rows * 32 + 255) / 256;
    label_cost_kernel<<<(unsigned)blocks, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        cls_logits, cls_targets, out, (int)L, (int)B, (int)Q, (int)C, (int)GT_total, ibg, gout, scale,
        gamma, alpha, use_softmax);
    ML_CHECK_LAUNCH("label_cost_kernel");
    return ML_OK;
}

int ml_match(const float* costs, int64_t L, int64_t B, int64_t Q, int64_t GT_out, double inf_thresh,
             int64_t topk, int64_t strategy_id, int64_t* pred_to_gt, int64_t* pred_round,
             int32_t* dev_status, void*, size_t, ml_stream_t stream) {
    if (topk < 0) return fail(ML_EINVAL, "K must be non-negative");
    if (strategy_id < 0 || strategy_id > 3) return fail(ML_EINVAL, "Invalid matching strategy id");
    return launch_match<float>(costs, L * B, Q, GT_out, inf_thresh, topk, strategy_id, pred_to_gt,
                               pred_round, dev_status, reinterpret_cast<cudaStream_t>(stream));
}

int ml_match_f64(const double* costs, int64_t N, int64_t Q, int64_t GT_out, double inf_thresh,
                 int64_t topk, int64_t strategy_id, int64_t* pred_to_gt, int64_t* pred_round,
                 int32_t* dev_status, ml_stream_t stream) {
    if (topk < 0) return fail(ML_EINVAL, "K must be non-negative");
    if (strategy_id < 0 || strategy_id > 3) return fail(ML_EINVAL, "Invalid matching strategy id");
    return launch_match<double>(costs, N, Q, GT_out, inf_thresh, topk, strategy_id, pred_to_gt,
                                pred_round, dev_status, reinterpret_cast<cudaStream_t>(stream));
}

static int mask_matching_impl(const ml_dims* d, const ml_params* p, const float* mask_logits,
                              const int64_t* mask_targets, const float* cls_logits,
                              const int64_t* cls_targets, const float* num_masks_dev,
                              int64_t* pred_to_gt, int64_t* pred_round, float* layer_means,
                              float* sep_costs, float* saved, int32_t* dev_status, void* workspace,
                              size_t workspace_bytes, ml_stream_t stream, cudaEvent_t loss_wait,
                              const uint8_t* dense_masks = nullptr,
                              cudaEvent_t costs_done = nullptr) {
    FwdPlan P;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if ((rc = make_plan(d, p, &P))) return rc;
    if (P.gout == 0)
        return fail(ML_ESHAPE, "pairwise_sigmoid_dice_loss_forward must return {3,L,B,Q,GT_out}");
    const size_t need = P.bytes + (dense_masks ? dense_count_bytes(P) : 0);
    if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
    if (!dev_status) return fail(ML_EINVAL, "dev_status is null");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* ws = ws_base(workspace);
    CostArgs a = cost_args(P, p, mask_logits, mask_targets, cls_logits, cls_targets, ws, dev_status);
    if (sep_costs) a.sep = sep_costs;
    if (dense_masks) rc = run_dense_costs(P, a, dense_masks, ws, st);
    else rc = run_costs(P, a, mask_logits, st);
    if (rc) return rc;
    if (costs_done) {  // the costs are final: work that needs only them may start
        cudaError_t e = cudaEventRecord(costs_done, st);
        if (e != cudaSuccess) return cuda_fail(e, "record costs_done_event");
    }
    if ((rc = launch_match<float>(a.total, (int64_t)P.L * P.B, P.Q, P.gout, p->inf_thresh,
                                  p->topk_matches, p->strategy_id, pred_to_gt, pred_round,
                                  dev_status, st)))
        return rc;
    if (P.L == 0) return ML_OK;
    LossArgs la = loss_args(P, p);
    la.pred_to_gt = pred_to_gt; la.sep = a.sep; la.qstat = a.qstat; la.rawI = a.rawI; la.rawT = a.rawT;
    la.num_masks_dev = num_masks_dev; la.saved = saved; la.layer_means = layer_means;
    if (p->num_masks == -2.0) {  // auto: counted on the device, written to num_masks_dev
        la.auto_num_masks = 1;
        la.totals = a.totals;
        la.num_masks_out = const_cast<float*>(num_masks_dev);
    }
    if (p->check_void_targets && la.has_void) {
        la.cls_targets = cls_targets;
        la.void_status = dev_status;
    }
    if (loss_wait) {  // e.g. the all-reduce that produces num_masks_dev
        cudaError_t e = cudaStreamWaitEvent(st, loss_wait, 0);
        if (e != cudaSuccess) return cuda_fail(e, "wait for loss_wait_event");
    }
    {
        ProfScope prof(5, st);
        launch_pdl(loss_fwd_kernel, dim3(P.L), dim3(1024), 0, st, la);
    }
    ML_CHECK_LAUNCH("loss_fwd_kernel");
    return ML_OK;
}

int ml_mask_matching(const ml_dims* d, const ml_params* p, const float* mask_logits,
                     const int64_t* mask_targets, const float* cls_logits, const int64_t* cls_targets,
                     const float* num_masks_dev, int64_t* pred_to_gt, int64_t* pred_round,
                     float* layer_means, float* sep_costs, float* saved, int32_t* dev_status,
                     void* workspace, size_t workspace_bytes, ml_stream_t stream) {
    return mask_matching_impl(d, p, mask_logits, mask_targets, cls_logits, cls_targets, num_masks_dev,
                              pred_to_gt, pred_round, layer_means, sep_costs, saved, dev_status,
                              workspace, workspace_bytes, stream, nullptr);
}

int ml_mask_matching_ex(const ml_dims* d, const ml_params* p, const float* mask_logits,
                        const int64_t* mask_targets, const float* cls_logits,
                        const int64_t* cls_targets, const float* num_masks_dev, int64_t* pred_to_gt,
                        int64_t* pred_round, float* layer_means, float* sep_costs, float* saved,
                        int32_t* dev_status, void* workspace, size_t workspace_bytes,
                        ml_stream_t stream, ml_event_t loss_wait_event) {
    return mask_matching_impl(d, p, mask_logits, mask_targets, cls_logits, cls_targets, num_masks_dev,
                              pred_to_gt, pred_round, layer_means, sep_costs, saved, dev_status,
                              workspace, workspace_bytes, stream,
                              reinterpret_cast<cudaEvent_t>(loss_wait_event));
}

int ml_mask_matching_ex2(const ml_dims* d, const ml_params* p, const float* mask_logits,
                         const int64_t* mask_targets, const float* cls_logits,
                         const int64_t* cls_targets, const float* num_masks_dev, int64_t* pred_to_gt,
                         int64_t* pred_round, float* layer_means, float* sep_costs, float* saved,
                         int32_t* dev_status, void* workspace, size_t workspace_bytes,
                         ml_stream_t stream, ml_event_t loss_wait_event, ml_event_t costs_done_event) {
    return mask_matching_impl(d, p, mask_logits, mask_targets, cls_logits, cls_targets, num_masks_dev,
                              pred_to_gt, pred_round, layer_means, sep_costs, saved, dev_status,
                              workspace, workspace_bytes, stream,
                              reinterpret_cast<cudaEvent_t>(loss_wait_event), nullptr,
                              reinterpret_cast<cudaEvent_t>(costs_done_event));
}

int ml_count_masks(const ml_dims* d, const ml_params* p, const int64_t* mask_targets,
                   float* num_masks_out, void* workspace, size_t workspace_bytes, ml_stream_t stream) {
    FwdPlan P;
    int rc;
    if (!p) return fail(ML_EINVAL, "params is null");
    if ((rc = make_plan(d, p, &P))) return rc;
    if ((rc = check_ws(workspace, workspace_bytes, P.bytes))) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* ws = ws_base(workspace);
    CostArgs a = cost_args(P, p, nullptr, mask_targets, nullptr, nullptr, ws, nullptr);
    a.codes = nullptr;  // histogram only
    if ((rc = run_prep(P, a, st))) return rc;
    const int32_t* totals = a.totals;
    count_masks_kernel<<<1, 256, 0, st>>>(totals, P.B, P.gt_total, P.bg, num_masks_out);
    ML_CHECK_LAUNCH("count_masks_kernel");
    return ML_OK;
}

static int backward_impl(const ml_dims* d, const ml_params* p, const float* grad_mask_mean,
                         const float* grad_dice_mean, const float* grad_cls_mean,
                         const float* mask_logits, const int64_t* mask_targets,
                         const float* cls_logits, const int64_t* cls_targets,
                         const int64_t* pred_to_gt, const float* saved,
                         const float* num_masks_dev, float* grad_mask_logits,
                         float* grad_cls_logits, void* workspace, size_t workspace_bytes,
                         ml_stream_t stream, const uint8_t* dense_masks,
                         const void* forward_workspace = nullptr, int rows_prezeroed = 0) {
    if (dense_masks && !saved)
        return fail(ML_EINVAL, "dense mask targets need the forward's saved statistics");
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    const int ldt = (int)p->logits_dtype;
    if ((rc = validate_dims(d))) return rc;
    const size_t need = ml_mask_matching_backward_workspace_size(d, p);
    if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
    FwdPlan P{};
    P.L = (int)d->L; P.B = (int)d->B; P.Q = (int)d->Q; P.H = (int)d->H; P.W = (int)d->W;
    P.Ht = (int)d->Ht; P.Wt = (int)d->Wt; P.s = P.Ht / P.H; P.C = (int)d->C;
    P.gt_total = (int)d->GT_total;
    const bool skip = p->background_index >= 0 && p->background_index < d->GT_total;
    // the backward maps pred_to_gt back through background_index only when it is >= 0
    P.bg = p->background_index >= 0 ? (int)std::min<int64_t>(p->background_index, 1 << 30) : P.gt_total;
    P.gout = P.gt_total - (skip ? 1 : 0);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* ws = ws_base(workspace);
    const BwdLayout lay = bwd_layout(d, p);
    float* coef = reinterpret_cast<float*>(ws);
    float* stats = reinterpret_cast<float*>(ws + lay.off_stats);
    const int64_t LBQ = (int64_t)P.L * P.B * P.Q;
    if (LBQ == 0) return ML_OK;
    LossArgs la = loss_args(P, p);
    la.mask_logits = mask_logits; la.targets = mask_targets; la.cls_logits = cls_logits;
    la.cls_targets = cls_targets; la.pred_to_gt = pred_to_gt; la.num_masks_dev = num_masks_dev;
    la.grad_mask = grad_mask_mean; la.grad_dice = grad_dice_mean; la.grad_cls = grad_cls_mean;
    la.coef = coef; la.grad_mask_logits = grad_mask_logits; la.grad_cls_logits = grad_cls_logits;
    la.masks = dense_masks;
    la.rows_zeroed = rows_prezeroed ? 1 : 0;
    const int HW = P.H * P.W;
    if (lay.cells && !dense_masks && HW > 0) {
        // per-cell column codes + mixed-cell table: the gradient kernels read
        // 4 bytes per cell (16 more on a label boundary) instead of s*s labels
        int32_t* codes = nullptr;
        uint4* mixtab = nullptr;
        FwdPlan FP;
        if (forward_workspace && make_plan(d, p, &FP) == ML_OK && FP.off_mixtab != SIZE_MAX) {
            // the forward of the same call built them already
            unsigned char* fws = ws_base(const_cast<void*>(forward_workspace));
            codes = reinterpret_cast<int32_t*>(fws + FP.off_codes);
            mixtab = reinterpret_cast<uint4*>(fws + FP.off_mixtab);
        } else {
            codes = reinterpret_cast<int32_t*>(ws + lay.off_codes);
            mixtab = reinterpret_cast<uint4*>(ws + lay.off_mixtab);
            cudaError_t ce = launch_label_code(mask_targets, P.B, P.H, P.W, P.Wt, P.s, P.gt_total,
                                               P.bg, codes, nullptr, mixtab, st);
            g_launches.fetch_add(1, std::memory_order_relaxed);
            if (ce != cudaSuccess) return cuda_fail(ce, "label_code_kernel");
        }
        la.codes = codes;
        la.mixtab = mixtab;
    }
    // coefficients + class-logit gradient first; the mask gradient reads coef
    {
        ProfScope prof(6, st);
        launch_pdl(bwd_cls_kernel, dim3((unsigned)((LBQ + 7) / 8)), dim3(256), 0, st, la);
    }
    ML_CHECK_LAUNCH("bwd_cls_kernel");
    const bool unc = p->uncertainty_gamma != 0.0f;
    const bool foc = p->mask_gamma > 0.0f || p->mask_alpha >= 0.0f;
    if (saved) {
        la.stats_in = saved;
    } else {
        la.stats_out = stats;
        la.stats_in = stats;
        dim3 g(P.Q, P.L * P.B);
        with_logit_type(ldt, [&](auto tag) -> int {
            using T = decltype(tag);
            if (unc) bwd_stats_kernel<true, T><<<g, 256, 0, st>>>(la);
            else bwd_stats_kernel<false, T><<<g, 256, 0, st>>>(la);
            return 0;
        });
        ML_CHECK_LAUNCH("bwd_stats_kernel");
    }
    // four elements per access: 16 bytes (fp32) or 8 bytes (16-bit)
    const uintptr_t va = ldt ? 8 : 16;
    const bool vec = (HW % 4 == 0) && (reinterpret_cast<uintptr_t>(mask_logits) % va == 0) &&
                     (reinterpret_cast<uintptr_t>(grad_mask_logits) % va == 0);
    // one block per (query row, contiguous range of cells)
    const int64_t ck = std::min<int64_t>(((HW + 3) / 4) * 4, 4096);
    la.chunk_cells = (int)ck;
    const int nchunk = (int)((HW + ck - 1) / ck);
    dim3 gg((unsigned)LBQ, nchunk);
    const size_t gs = 0;
#define ML_MG(U, F, V) launch_pdl(mask_grad_kernel<U, F, V, T>, dim3(gg), dim3(256), gs, st, la)
    {
    ProfScope prof(1, st);
    with_logit_type(ldt, [&](auto tag) -> int {
        using T = decltype(tag);
        if (unc) {
            if (foc) { if (vec) ML_MG(true, true, true); else ML_MG(true, true, false); }
            else { if (vec) ML_MG(true, false, true); else ML_MG(true, false, false); }
        } else {
            if (foc) { if (vec) ML_MG(false, true, true); else ML_MG(false, true, false); }
            else { if (vec) ML_MG(false, false, true); else ML_MG(false, false, false); }
        }
        return 0;
    });
    }
#undef ML_MG
    ML_CHECK_LAUNCH("mask_grad_kernel");
    return ML_OK;
}

int ml_mask_matching_backward(const ml_dims* d, const ml_params* p, const float* grad_mask_mean,
                              const float* grad_dice_mean, const float* grad_cls_mean,
                              const float* mask_logits, const int64_t* mask_targets,
                              const float* cls_logits, const int64_t* cls_targets,
                              const int64_t* pred_to_gt, const float* saved,
                              const float* num_masks_dev, float* grad_mask_logits,
                              float* grad_cls_logits, void* workspace, size_t workspace_bytes,
                              ml_stream_t stream) {
    return backward_impl(d, p, grad_mask_mean, grad_dice_mean, grad_cls_mean, mask_logits,
                         mask_targets, cls_logits, cls_targets, pred_to_gt, saved, num_masks_dev,
                         grad_mask_logits, grad_cls_logits, workspace, workspace_bytes, stream,
                         nullptr);
}

int ml_mask_matching_backward_ex(const ml_dims* d, const ml_params* p, const float* grad_mask_mean,
                                 const float* grad_dice_mean, const float* grad_cls_mean,
                                 const float* mask_logits, const int64_t* mask_targets,
                                 const float* cls_logits, const int64_t* cls_targets,
                                 const int64_t* pred_to_gt, const float* saved,
                                 const float* num_masks_dev, float* grad_mask_logits,
                                 float* grad_cls_logits, void* workspace, size_t workspace_bytes,
                                 ml_stream_t stream, const void* forward_workspace) {
    return backward_impl(d, p, grad_mask_mean, grad_dice_mean, grad_cls_mean, mask_logits,
                         mask_targets, cls_logits, cls_targets, pred_to_gt, saved, num_masks_dev,
                         grad_mask_logits, grad_cls_logits, workspace, workspace_bytes, stream,
                         nullptr, forward_workspace);
}

int ml_mask_matching_backward_ex2(const ml_dims* d, const ml_params* p, const float* grad_mask_mean,
                                  const float* grad_dice_mean, const float* grad_cls_mean,
                                  const float* mask_logits, const int64_t* mask_targets,
                                  const float* cls_logits, const int64_t* cls_targets,
                                  const int64_t* pred_to_gt, const float* saved,
                                  const float* num_masks_dev, float* grad_mask_logits,
                                  float* grad_cls_logits, void* workspace, size_t workspace_bytes,
                                  ml_stream_t stream, const void* forward_workspace,
                                  int grad_rows_prezeroed) {
    return backward_impl(d, p, grad_mask_mean, grad_dice_mean, grad_cls_mean, mask_logits,
                         mask_targets, cls_logits, cls_targets, pred_to_gt, saved, num_masks_dev,
                         grad_mask_logits, grad_cls_logits, workspace, workspace_bytes, stream,
                         nullptr, forward_workspace, grad_rows_prezeroed);
}

// ---------------------------------------------------------------------------
// Dense per-GT mask targets (no reference counterpart; dense.cu).
// ---------------------------------------------------------------------------
size_t ml_dense_workspace_size(const ml_dims* d, const ml_params* p) {
    FwdPlan P;
    if (!p || make_plan(d, p, &P)) return 0;
    return P.bytes + dense_count_bytes(P);
}

int ml_pairwise_mask_loss_dense_forward(const ml_dims* d, const ml_params* p, const float* mask_logits,
                                        const uint8_t* mask_masks, const float* cls_logits,
                                        const int64_t* cls_targets, float* out, void* workspace,
                                        size_t workspace_bytes, ml_stream_t stream) {
    FwdPlan P;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if ((rc = make_plan(d, p, &P))) return rc;
    if ((rc = check_ws(workspace, workspace_bytes, P.bytes + dense_count_bytes(P)))) return rc;
    if (P.gout == 0) return ML_OK;
    unsigned char* ws = ws_base(workspace);
    CostArgs a = cost_args(P, p, mask_logits, nullptr, cls_logits, cls_targets, ws,
                           cost_status_ptr());
    a.sep = out; a.total = nullptr; a.rawI = nullptr; a.rawT = nullptr;
    return run_dense_costs(P, a, mask_masks, ws, reinterpret_cast<cudaStream_t>(stream));
}

int ml_mask_matching_dense(const ml_dims* d, const ml_params* p, const float* mask_logits,
                           const uint8_t* mask_masks, const float* cls_logits,
                           const int64_t* cls_targets, const float* num_masks_dev,
                           int64_t* pred_to_gt, int64_t* pred_round, float* layer_means,
                           float* sep_costs, float* saved, int32_t* dev_status, void* workspace,
                           size_t workspace_bytes, ml_stream_t stream) {
    if (!mask_masks) return fail(ML_EINVAL, "mask_masks is null");
    return mask_matching_impl(d, p, mask_logits, nullptr, cls_logits, cls_targets, num_masks_dev,
                              pred_to_gt, pred_round, layer_means, sep_costs, saved, dev_status,
                              workspace, workspace_bytes, stream, nullptr, mask_masks);
}

int ml_mask_matching_dense_backward(const ml_dims* d, const ml_params* p, const float* grad_mask_mean,
                                    const float* grad_dice_mean, const float* grad_cls_mean,
                                    const float* mask_logits, const uint8_t* mask_masks,
                                    const float* cls_logits, const int64_t* cls_targets,
                                    const int64_t* pred_to_gt, const float* saved,
                                    const float* num_masks_dev, float* grad_mask_logits,
                                    float* grad_cls_logits, void* workspace,
                                    size_t workspace_bytes, ml_stream_t stream) {
    if (!mask_masks) return fail(ML_EINVAL, "mask_masks is null");
    return backward_impl(d, p, grad_mask_mean, grad_dice_mean, grad_cls_mean, mask_logits, nullptr,
                         cls_logits, cls_targets, pred_to_gt, saved, num_masks_dev,
                         grad_mask_logits, grad_cls_logits, workspace, workspace_bytes, stream,
                         mask_masks);
}


size_t ml_sampled_workspace_size(const ml_dims* d, const ml_params* p, int64_t num_points) {
    SampledPlan S;
    if (!p || make_sampled_plan(d, p, num_points, &S)) return 0;
    return S.bytes;
}

int ml_pairwise_mask_loss_sampled_forward(const ml_dims* d, const ml_params* p, int64_t num_points,
                                          int32_t align_corners, int32_t logits_dtype,
                                          const void* mask_logits, const int64_t* mask_targets,
                                          const float* cls_logits, const int64_t* cls_targets,
                                          const float* point_coords, float* out, void* workspace,
                                          size_t workspace_bytes, ml_stream_t stream) {
    SampledPlan S;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if ((rc = make_sampled_plan(d, p, num_points, &S))) return rc;
    if ((rc = check_ws(workspace, workspace_bytes, S.bytes))) return rc;
    if (S.cp.gout == 0) return ML_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* ws = ws_base(workspace);
    CostArgs a = cost_args(S.cp, p, nullptr, mask_targets, cls_logits, cls_targets, ws,
                           cost_status_ptr());
    if ((rc = run_sampled_prep(S, p, mask_logits, logits_dtype, mask_targets, point_coords,
                               align_corners, ws, a, st)))
        return rc;
    a.sep = out; a.total = nullptr; a.rawI = nullptr; a.rawT = nullptr;
    return run_cost_core(S.cp, a, a.logits, st);
}

int ml_mask_matching_sampled(const ml_dims* d, const ml_params* p, int64_t num_points,
                             int32_t align_corners, int32_t logits_dtype, const void* mask_logits,
                             const int64_t* mask_targets, const float* cls_logits,
                             const int64_t* cls_targets, const float* point_coords,
                             const float* num_masks_dev, int64_t* pred_to_gt, int64_t* pred_round,
                             float* layer_means, float* sep_costs, float* saved, int32_t* dev_status,
                             void* workspace, size_t workspace_bytes, ml_stream_t stream) {
    SampledPlan S;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if ((rc = make_sampled_plan(d, p, num_points, &S))) return rc;
    const FwdPlan& P = S.cp;
    if (P.gout == 0)
        return fail(ML_ESHAPE, "pairwise_sigmoid_dice_loss_forward must return {3,L,B,Q,GT_out}");
    if ((rc = check_ws(workspace, workspace_bytes, S.bytes))) return rc;
    if (!dev_status) return fail(ML_EINVAL, "dev_status is null");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* ws = ws_base(workspace);
    CostArgs a = cost_args(P, p, nullptr, mask_targets, cls_logits, cls_targets, ws, dev_status);
    if (sep_costs) a.sep = sep_costs;
    if ((rc = run_sampled_prep(S, p, mask_logits, logits_dtype, mask_targets, point_coords,
                               align_corners, ws, a, st)))
        return rc;
    if ((rc = run_cost_core(P, a, a.logits, st))) return rc;
    if ((rc = launch_match<float>(a.total, (int64_t)P.L * P.B, P.Q, P.gout, p->inf_thresh,
                                  p->topk_matches, p->strategy_id, pred_to_gt, pred_round,
                                  dev_status, st)))
        return rc;
    if (P.L == 0) return ML_OK;
    LossArgs la = loss_args(P, p);
    la.pred_to_gt = pred_to_gt; la.sep = a.sep; la.qstat = a.qstat; la.rawI = a.rawI; la.rawT = a.rawT;
    la.num_masks_dev = num_masks_dev; la.saved = saved; la.layer_means = layer_means;
    if (p->num_masks == -2.0) {  // auto: GT ids present in the full label maps
        la.auto_num_masks = 1;
        la.totals = a.present ? a.present : a.totals;
        la.num_masks_out = const_cast<float*>(num_masks_dev);
    }
    if (p->check_void_targets && la.has_void) {
        la.cls_targets = cls_targets;
        la.void_status = dev_status;
    }
    {
        ProfScope prof(5, st);
        launch_pdl(loss_fwd_kernel, dim3(P.L), dim3(1024), 0, st, la);
    }
    ML_CHECK_LAUNCH("loss_fwd_kernel");
    return ML_OK;
}

int ml_mask_matching_sampled_backward(const ml_dims* d, const ml_params* p, int64_t num_points,
                                      int32_t align_corners, int32_t logits_dtype,
                                      const float* grad_mask_mean, const float* grad_dice_mean,
                                      const float* grad_cls_mean, const void* mask_logits,
                                      const int64_t* mask_targets, const float* cls_logits,
                                      const int64_t* cls_targets, const float* point_coords,
                                      const int64_t* pred_to_gt, const float* saved,
                                      const float* num_masks_dev, const void* forward_workspace,
                                      void* grad_mask_logits, float* grad_cls_logits,
                                      void* workspace, size_t workspace_bytes, ml_stream_t stream) {
    SampledPlan S;
    int rc = validate_params(p, d ? d->C : 0);
    if (rc) return rc;
    if ((rc = make_sampled_plan(d, p, num_points, &S))) return rc;
    if (!saved) return fail(ML_EINVAL, "the sampled backward needs the forward's saved statistics");
    const FwdPlan& P = S.cp;
    const size_t LBQ = (size_t)P.L * P.B * P.Q;
    const size_t HWl = (size_t)S.H * S.W;
    const size_t need = ml_sampled_backward_workspace_size(d, p, num_points, logits_dtype);
    if ((rc = check_ws(workspace, workspace_bytes, need))) return rc;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char* ws = ws_base(workspace);
    // sorted points and samples: reuse the forward's when given, else rebuild
    unsigned char* fw = forward_workspace ? ws_base(const_cast<void*>(forward_workspace)) : ws;
    CostArgs a = cost_args(P, p, nullptr, mask_targets, cls_logits, cls_targets, fw, nullptr);
    if (!forward_workspace) {
        if ((rc = run_sampled_prep(S, p, mask_logits, logits_dtype, mask_targets, point_coords,
                                   align_corners, ws, a, st)))
            return rc;
    } else {
        a.logits = reinterpret_cast<float*>(fw + S.off_zs);
    }
    const float* scoords = reinterpret_cast<const float*>(fw + S.off_scoords);
    const size_t off_coef = S.bytes;
    const size_t off_gacc = off_coef + align256(sizeof(float) * 3 * (size_t)P.L);
    LossArgs la = loss_args(P, p);
    la.H = S.H; la.W = S.W; la.Ht = S.Ht; la.Wt = S.Wt;
    la.bg = p->background_index >= 0 ? (int)std::min<int64_t>(p->background_index, 1 << 30) : P.gt_total;
    la.cls_logits = cls_logits; la.cls_targets = cls_targets; la.pred_to_gt = pred_to_gt;
    la.num_masks_dev = num_masks_dev; la.grad_mask = grad_mask_mean; la.grad_dice = grad_dice_mean;
    la.grad_cls = grad_cls_mean; la.coef = reinterpret_cast<float*>(ws + off_coef);
    la.stats_in = saved; la.grad_cls_logits = grad_cls_logits;
    if (LBQ == 0) return ML_OK;
    // coefficients + class-logit gradient first; the mask gradient reads coef
    {
        ProfScope prof(6, st);
        launch_pdl(bwd_cls_kernel, dim3((unsigned)((LBQ + 7) / 8)), dim3(256), 0, st, la);
    }
    ML_CHECK_LAUNCH("bwd_cls_kernel");
    const bool foc = p->mask_gamma > 0.0f || p->mask_alpha >= 0.0f;
    float* gacc = logits_dtype == 1 ? reinterpret_cast<float*>(ws + off_gacc)
                                    : static_cast<float*>(grad_mask_logits);
    const bool rows_fit = HWl * 4 <= kRowMapMaxBytes;
    if (!rows_fit) {
        cudaError_t e = cudaMemsetAsync(gacc, 0, sizeof(float) * LBQ * HWl, st);
        if (e != cudaSuccess) return cuda_fail(e, "memset sampled gradient");
    }
    bool used_rows = false;
    cudaError_t e = launch_point_grad(foc, logits_dtype, la, a.logits, scoords, a.codes, S.P,
                                      align_corners, grad_mask_logits, gacc, (int64_t)LBQ,
                                      &used_rows, st);
    g_launches.fetch_add(1);
    if (e != cudaSuccess) return cuda_fail(e, "point_grad_kernel");
    if (!used_rows && logits_dtype == 1) {
        e = launch_to_bf16(gacc, grad_mask_logits, (int64_t)(LBQ * HWl), st);
        g_launches.fetch_add(1);
        if (e != cudaSuccess) return cuda_fail(e, "f32_to_bf16_kernel");
    }
    return ML_OK;
}

size_t ml_sampled_backward_workspace_size(const ml_dims* d, const ml_params* p, int64_t num_points,
                                          int32_t logits_dtype) {
    SampledPlan S;
    if (!p || make_sampled_plan(d, p, num_points, &S)) return 0;
    const size_t LBQ = (size_t)d->L * d->B * d->Q;
    const bool rows_fit = (size_t)d->H * d->W * 4 <= kRowMapMaxBytes;
    return S.bytes + align256(sizeof(float) * 3 * (size_t)d->L) +
           (logits_dtype == 1 && !rows_fit ? align256(sizeof(float) * LBQ * d->H * d->W) : 0) + 256;
}


// ---------------------------------------------------------------------------
// Standalone semantic losses (src/cuda/sigmoid_ce.cu, src/cuda/dice_loss.cu).
// ---------------------------------------------------------------------------
static int sem_setup(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                     SemArgs* a) {
    if (L < 0 || B < 0 || C < 0) return fail(ML_ESHAPE, "negative dimension");
    if (H <= 0 || W <= 0) return fail(ML_ESHAPE, "logits must have positive spatial size");
    if (Ht % H != 0 || Wt % W != 0 || Ht / H != Wt / W)
        return fail(ML_ESHAPE, "target size must be the same integer multiple of the logits size in both dimensions");
    if (Ht / H > 16) return fail(ML_EUNSUPPORTED, "downsample factor above 16 is not supported");
    if (C > 2048) return fail(ML_EUNSUPPORTED, "more than 2048 classes is not supported");
    if (H * W >= (int64_t(1) << 31) || B > 65535 || L * B > (int64_t(1) << 30) ||
        Ht * Wt >= (int64_t(1) << 31))
        return fail(ML_EUNSUPPORTED, "dimension product exceeds the supported range");
    *a = SemArgs{};
    a->L = (int)L; a->B = (int)B; a->C = (int)C; a->H = (int)H; a->W = (int)W;
    a->Ht = (int)Ht; a->Wt = (int)Wt; a->s = (int)(Ht / H);
    a->cps = a->C; a->ncs = 1;
    return ML_OK;
}

static size_t sem_ws(const SemArgs& a, int dice) {
    const size_t nblk = (size_t)sem_blocks(a), dblk = (size_t)dice_blocks(a);
    size_t n = align256(sizeof(double) * ((size_t)a.L * a.B * a.ncs * nblk + (size_t)a.L * a.B + 1));
    if (dice) {
        n += align256(sizeof(float) * (size_t)a.L * a.B * dblk * 2 * a.C);
        n += align256(sizeof(int32_t) * (size_t)a.B * dblk * a.C);
    }
    return n + 256;
}

static void sem_carve(SemArgs* a, void* ws, int dice) {
    unsigned char* w = ws_base(ws);
    const size_t nblk = (size_t)sem_blocks(*a), dblk = (size_t)dice_blocks(*a);
    a->part_d = reinterpret_cast<double*>(w);
    w += align256(sizeof(double) * ((size_t)a->L * a->B * a->ncs * nblk + (size_t)a->L * a->B + 1));
    if (dice) {
        a->part_f = reinterpret_cast<float*>(w);
        w += align256(sizeof(float) * (size_t)a->L * a->B * dblk * 2 * a->C);
        a->part_t = reinterpret_cast<int32_t*>(w);
    }
}

size_t ml_semantic_workspace_size(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht,
                                  int64_t Wt, int32_t dice) {
    SemArgs a;
    if (sem_setup(L, B, C, H, W, Ht, Wt, &a)) return 0;
    sem_slices(&a, dice ? dice_blocks(a) : sem_blocks(a));
    return sem_ws(a, dice);
}

int ml_sigmoid_ce_forward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                          const float* logits, const int64_t* targets, float num_masks, float scale,
                          float gamma, float alpha, float* out, void* workspace,
                          size_t workspace_bytes, ml_stream_t stream) {
    SemArgs a;
    int rc = sem_setup(L, B, C, H, W, Ht, Wt, &a);
    if (rc) return rc;
    sem_slices(&a, sem_blocks(a));
    if (gamma < 0.0f) return fail(ML_EINVAL, "focal_gamma must be non-negative");
    if (alpha > 1.0f) return fail(ML_EINVAL, "alpha must be in [0, 1]");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (L == 0) return ML_OK;
    if (B * C == 0) {  // the reference returns zeros for empty logits
        cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float) * (size_t)L, st);
        return e == cudaSuccess ? ML_OK : cuda_fail(e, "memset out");
    }
    if ((rc = check_ws(workspace, workspace_bytes, sem_ws(a, 0)))) return rc;
    a.logits = logits; a.targets = targets; a.num_masks = num_masks; a.scale = scale;
    a.gamma = gamma; a.alpha = alpha; a.out = out;
    sem_carve(&a, workspace, 0);
    cudaError_t e = launch_sce_forward(a, st);
    g_launches.fetch_add(2);
    return e == cudaSuccess ? ML_OK : cuda_fail(e, "sigmoid_ce forward");
}

int ml_sigmoid_ce_backward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                           const float* grad_out, const float* logits, const int64_t* targets,
                           float num_masks, float scale, float gamma, float alpha, float* grad_logits,
                           ml_stream_t stream) {
    SemArgs a;
    int rc = sem_setup(L, B, C, H, W, Ht, Wt, &a);
    if (rc) return rc;
    sem_slices(&a, sem_blocks(a));
    if (gamma < 0.0f) return fail(ML_EINVAL, "focal_gamma must be non-negative");
    if (alpha > 1.0f) return fail(ML_EINVAL, "alpha must be in [0, 1]");
    if (L * B * C == 0) return ML_OK;
    a.logits = logits; a.targets = targets; a.num_masks = num_masks; a.scale = scale;
    a.gamma = gamma; a.alpha = alpha; a.grad_out = grad_out; a.grad = grad_logits;
    cudaError_t e = launch_sce_backward(a, reinterpret_cast<cudaStream_t>(stream));
    g_launches.fetch_add(1);
    return e == cudaSuccess ? ML_OK : cuda_fail(e, "sigmoid_ce backward");
}

int ml_dice_forward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                    const float* logits, const int64_t* targets, float smooth, float num_masks,
                    float scale, float* out, float* int_sum, float* p_sum, float* t_sum,
                    void* workspace, size_t workspace_bytes, ml_stream_t stream) {
    SemArgs a;
    int rc = sem_setup(L, B, C, H, W, Ht, Wt, &a);
    if (rc) return rc;
    sem_slices(&a, dice_blocks(a));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (L == 0) return ML_OK;
    if (B * C == 0) {
        cudaError_t e = cudaMemsetAsync(out, 0, sizeof(float) * (size_t)L, st);
        return e == cudaSuccess ? ML_OK : cuda_fail(e, "memset out");
    }
    if ((rc = check_ws(workspace, workspace_bytes, sem_ws(a, 1)))) return rc;
    a.logits = logits; a.targets = targets; a.smooth = smooth; a.num_masks = num_masks;
    a.scale = scale; a.out = out; a.I = int_sum; a.P = p_sum; a.T = t_sum;
    sem_carve(&a, workspace, 1);
    cudaError_t e = launch_dice_forward(a, st);
    g_launches.fetch_add(3);
    return e == cudaSuccess ? ML_OK : cuda_fail(e, "dice forward");
}

int ml_dice_backward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                     const float* grad_out, const float* logits, const int64_t* targets,
                     const float* int_sum, const float* p_sum, const float* t_sum, float smooth,
                     float num_masks, float scale, float* grad_logits, ml_stream_t stream) {
    SemArgs a;
    int rc = sem_setup(L, B, C, H, W, Ht, Wt, &a);
    if (rc) return rc;
    sem_slices(&a, sem_blocks(a));
    if (L * B * C == 0) return ML_OK;
    a.logits = logits; a.targets = targets; a.smooth = smooth; a.num_masks = num_masks;
    a.scale = scale; a.grad_out = grad_out; a.grad = grad_logits;
    a.I = const_cast<float*>(int_sum); a.P = const_cast<float*>(p_sum); a.T = const_cast<float*>(t_sum);
    cudaError_t e = launch_dice_backward(a, reinterpret_cast<cudaStream_t>(stream));
    g_launches.fetch_add(1);
    return e == cudaSuccess ? ML_OK : cuda_fail(e, "dice backward");
}

}  // extern "C"
