// common.cuh -- shared device helpers for the mask_loss_b200 kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mask_loss_b200.h"

#define ML_INLINE __device__ __forceinline__

namespace mlb {

// Mask-logit element types (ml_params.logits_dtype): fp32, bf16, fp16.  All
// arithmetic is fp32; 16-bit values widen exactly and gradients round to
// nearest-even on the way out.
ML_INLINE float to_f(float x) { return x; }
ML_INLINE float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
ML_INLINE float to_f(__half x) { return __half2float(x); }
template <typename T> ML_INLINE T from_f(float x);
template <> ML_INLINE float from_f<float>(float x) { return x; }
template <> ML_INLINE __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> ML_INLINE __half from_f<__half>(float x) { return __float2half_rn(x); }

// two packed 16-bit values -> two floats (exact), and back (round to nearest)
ML_INLINE void widen2(uint32_t w, float& lo, float& hi, const __nv_bfloat16*) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xFFFF0000u);
}
ML_INLINE void widen2(uint32_t w, float& lo, float& hi, const __half*) {
    lo = __half2float(__ushort_as_half((unsigned short)(w & 0xFFFFu)));
    hi = __half2float(__ushort_as_half((unsigned short)(w >> 16)));
}
ML_INLINE uint32_t narrow2(float lo, float hi, const __nv_bfloat16*) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}
ML_INLINE uint32_t narrow2(float lo, float hi, const __half*) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Four consecutive elements with streaming (evict-first) accesses: one
// 16-byte access for fp32, one 8-byte access for 16-bit types.
template <typename T>
ML_INLINE float4 ld4cs(const T* p) {
    if constexpr (sizeof(T) == 4) {
        return __ldcs(reinterpret_cast<const float4*>(p));
    } else {
        const uint2 v = __ldcs(reinterpret_cast<const uint2*>(p));
        float4 r;
        widen2(v.x, r.x, r.y, p);
        widen2(v.y, r.z, r.w, p);
        return r;
    }
}
template <typename T>
ML_INLINE void st4cs(T* p, const float4& v) {
    if constexpr (sizeof(T) == 4) {
        __stcs(reinterpret_cast<float4*>(p), v);
    } else {
        __stcs(reinterpret_cast<uint2*>(p), make_uint2(narrow2(v.x, v.y, p), narrow2(v.z, v.w, p)));
    }
}

constexpr int kNone = -1;   // cell/pixel carries no output column
constexpr int kMixed = -2;  // cell holds more than one label (s > 1 only)

// ----------------------------------------------------------------------------
// Mixed-cell table (s > 1): one uint4 per low-res cell, written only for cells
// whose code is kMixed.  Each word packs one output column of the cell and its
// pixel count as ((col + 1) << 16) | count; 0 = empty slot.  A cell with more
// than four distinct columns is marked wide (x == kMixWide) and its readers
// count its pixels from the label map instead.  Needs gout < 65535 and
// s * s < 65536.
// ----------------------------------------------------------------------------
constexpr uint32_t kMixWide = 0xFFFFFFFFu;
constexpr int kMixMaxCols = 65534;

ML_INLINE int mix_col(uint32_t v) { return (int)(v >> 16) - 1; }
ML_INLINE float mix_cnt(uint32_t v) { return (float)(v & 0xFFFFu); }

// Pixels of column `col` in a table entry (the entry must not be wide).
ML_INLINE float mix_count(const uint4& e, int col) {
    const uint32_t key = (uint32_t)(col + 1) << 16;
    float n = 0.0f;
    n = ((e.x & 0xFFFF0000u) == key) ? mix_cnt(e.x) : n;
    n = ((e.y & 0xFFFF0000u) == key) ? mix_cnt(e.y) : n;
    n = ((e.z & 0xFFFF0000u) == key) ? mix_cnt(e.z) : n;
    n = ((e.w & 0xFFFF0000u) == key) ? mix_cnt(e.w) : n;
    return n;
}

// ----------------------------------------------------------------------------
// Label -> output column (GT_out index).  The background column is dropped
// and later columns shift down by one (src/cuda/utils.cuh:38-40 inverted);
// labels outside [0, GT_total) belong to no column (src/cuda/utils.cuh:27).
// `bg` is GT_total when no column is dropped.
// ----------------------------------------------------------------------------
ML_INLINE int label_to_col(int64_t lab, int gt_total, int bg) {
    if (lab < 0 || lab >= gt_total || lab == bg) return kNone;
    int l = static_cast<int>(lab);
    return l > bg ? l - 1 : l;
}

// ----------------------------------------------------------------------------
// Element math.  Logit x -> e = exp(-|x|), log1p(e), sigmoid p.
// MUFU forms (__expf, __logf, __fdividef); accuracy is far inside the 1e-4
// relative tolerance for the sums they feed.
// ----------------------------------------------------------------------------
// Single MUFU instructions (hardware approximations, flush-to-zero).
ML_INLINE float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

ML_INLINE float lg2_approx(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

ML_INLINE float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Dense-mask pixel counts are kept as bf16 bit patterns (exact up to 256,
// i.e. s <= 16): the CUDA-core kernel widens them, the tensor-core kernel
// feeds them to the MMA as they are.
ML_INLINE uint16_t count_bits(float n) { return __bfloat16_as_ushort(__float2bfloat16_rn(n)); }
ML_INLINE float count_value(uint16_t v) { return __uint_as_float((uint32_t)v << 16); }

// Element pieces for the default path (no entropy weight, no focal terms):
// e = exp(-|x|), d = 1 + e (log1p(e) = log(d) is summed through a product of
// several d's and one log2), p = sigmoid(x).
struct Fast {
    float d, p;
};

ML_INLINE Fast fast_elem(float x) {
    const float e = ex2_approx(-fabsf(x) * 1.4426950408889634f);
    const float d = 1.0f + e;
    const float r = rcp_approx(d);
    Fast f;
    f.d = d;
    f.p = x >= 0.0f ? r : e * r;
    return f;
}

struct Elem {
    float p;      // sigmoid(x)
    float sp;     // log1p(exp(-|x|))
    float neg;    // softplus(x)  = BCE against 0
    float pos;    // softplus(-x) = BCE against 1
};

ML_INLINE Elem elem(float x) {
    Elem r;
    const float ax = fabsf(x);
    const float e = __expf(-ax);
    const float d = 1.0f + e;
    r.sp = __logf(d);
    const float inv = __fdividef(1.0f, d);
    r.p = x >= 0.0f ? inv : e * inv;
    r.neg = r.sp + fmaxf(x, 0.0f);
    r.pos = r.sp + fmaxf(-x, 0.0f);
    return r;
}

// Entropy weight clamp(H(p)^gamma, gmin, 1).  Mirrors
// src/cuda/pw_mask.cu:131-136 including its fp32 saturation: where the
// clamped p rounds to 1.0f the entropy is NaN and fmaxf(NaN, gmin) = gmin.
ML_INLINE float unc_weight(float p, float ug, float ugmin) {
    const float pc = fminf(fmaxf(p, 1e-12f), 1.0f - 1e-12f);
    if (pc >= 1.0f) return fminf(1.0f, ugmin);
    float h = -(pc * __logf(pc) + (1.0f - pc) * __logf(1.0f - pc)) * 1.4426950408889634f;
    float w = __powf(h, ug);
    w = fmaxf(w, ugmin);
    return fminf(1.0f, w);
}

// Focal/alpha modulation of the BCE pieces (src/cuda/pw_mask.cu:242-247).
struct Focal {
    float alpha_pos, alpha_neg, gamma;
    bool use_gamma;
};

ML_INLINE Focal make_focal(float gamma, float alpha) {
    Focal f;
    f.alpha_pos = alpha >= 0.0f ? alpha : 1.0f;
    f.alpha_neg = alpha >= 0.0f ? 1.0f - alpha : 1.0f;
    f.gamma = gamma;
    f.use_gamma = gamma > 0.0f;
    return f;
}

ML_INLINE float focal_neg(const Focal& f, const Elem& t) {
    const float m = f.use_gamma ? __powf(t.p, f.gamma) : 1.0f;
    return f.alpha_neg * m * t.neg;
}

ML_INLINE float focal_pos(const Focal& f, const Elem& t) {
    const float m = f.use_gamma ? __powf(1.0f - t.p, f.gamma) : 1.0f;
    return f.alpha_pos * m * t.pos;
}

// ----------------------------------------------------------------------------
// Warp / block reductions (fixed order -> deterministic).
// ----------------------------------------------------------------------------
ML_INLINE float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

ML_INLINE float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ----------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (TMA engine, no tensor map): global -> shared.
// ----------------------------------------------------------------------------
ML_INLINE uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

ML_INLINE void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

ML_INLINE void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

ML_INLINE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// Raise the phase's expected transaction bytes without arriving (the arrival
// comes later, once the producer has also written its own shared data).
ML_INLINE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

ML_INLINE void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

ML_INLINE uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait on phase `parity` of an mbarrier, bounded in wall time (default 2 s):
// returns false when the bound is hit so the caller can flag an error
// instead of spinning forever.
ML_INLINE bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t max_ns = 2000000000ull) {
    const uint32_t a = smem_u32(bar);
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
        uint32_t done;
        asm volatile(
            "{\n .reg .pred p;\n"
            " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            " selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done) : "r"(a), "r"(parity) : "memory");
        if (done) return true;
        if ((it & 255) == 0) {
            const uint64_t now = global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > max_ns) return false;
        }
    }
}

// cp.async.bulk global->shared, completion signalled on `bar` (tx bytes).
ML_INLINE void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Programmatic dependent launch.  Kernels of the forward/backward chain are
// launched with launch_pdl, so a kernel's blocks can be scheduled while the
// previous kernel drains; pdl_enter, each such kernel's first statement,
// waits until the previous grid has completed and its writes are visible
// (a no-op when the kernel was launched without the attribute).  No kernel
// triggers its dependents early: measured on B200, an early trigger made
// the cfg2 step slower (0.2346 -> 0.2371 ms), the implicit trigger at block
// exit faster (0.2344 -> 0.2316 ms).
ML_INLINE void pdl_enter() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*k)(KArgs...), dim3 g, dim3 b, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t c = {};
    c.gridDim = g; c.blockDim = b; c.dynamicSmemBytes = smem; c.stream = st;
    c.attrs = at; c.numAttrs = 1;
    return cudaLaunchKernelEx(&c, k, static_cast<KArgs>(args)...);
}

}  // namespace mlb
