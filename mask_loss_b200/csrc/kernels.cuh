// kernels.cuh -- kernel argument blocks and declarations shared by the
// launchers in capi.cu.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "common.cuh"

namespace mlb {

constexpr int KBOX = 32;          // cells per TMA box row (128 bytes, one swizzle span)
constexpr int KC = 2 * KBOX;      // cells per pipeline tile (two boxes)
constexpr int kStages = 2;        // TMA pipeline depth (2 stages: 3 CTAs per SM)
constexpr int kFlushTiles = 8;    // longest register run (tiles) before a flush
constexpr int kCostThreads = 288; // 256 consumers + 1 producer warp (upper bound)
constexpr int kHistSmemMax = 8192;
constexpr int kMatchMaxThreads = 256;  // match block: one thread per solver column up to 255
constexpr int kQStat = 8;         // per-query: P, Wtot, um_mask, um_dice, um_cls, base, cls_row, -
constexpr int kSaved = 4;
constexpr int kSampleQ = 8;        // queries per thread in point_sample_kernel         // saved for backward: P, T, I, Wtot

struct CostArgs {
    const float* logits;
    const int64_t* targets;
    const float* cls_logits;
    const int64_t* cls_targets;
    const int32_t* totals;   // (B, GT_total)
    const int32_t* codes;    // (B, H*W) per-cell column code
    const uint4* mixtab;     // (B, H*W) mixed-cell table (s > 1), or null
    const int32_t* present;  // (B, GT_total) full-image label counts for the +inf mask, or null
    float* part;             // chunk partials
    float* sep;              // (3,L,B,Q,G) or null
    float* total;            // (L,B,Q,G) or null
    float* rawI;             // (L,B,Q,G) or null
    float* rawT;             // (L,B,Q,G) or null
    float* qstat;            // (L,B,Q,kQStat)
    int32_t* status;
    int L, B, Q, H, W, Ht, Wt, s, C;
    int gt_total, gout, bg;  // bg == gt_total when no column is dropped
    int qrows, qrows_pad, nqt;
    int chunk_cells, nchunk;
    int part_stride;         // floats per CTA partial
    float smooth, sigmoid_scale, dice_scale, cls_scale;
    float ug, ugmin;
    float mask_gamma, mask_alpha, cls_gamma, cls_alpha;
    float area_scale;
    int normalize_uncertainty;
    int use_softmax, force_cls, has_void, void_index;
};

// Per-cell codes, mixed-cell table and label histogram (each output nullable).
cudaError_t launch_label_code(const int64_t* targets, int B, int H, int W, int Wt, int s,
                              int gt_total, int bg, int32_t* codes, int32_t* totals, uint4* mixtab,
                              cudaStream_t st);
// Label histogram only, over B flat label maps of npix pixels each.
cudaError_t launch_label_hist(const int64_t* targets, int B, int64_t npix, int gt_total,
                              int32_t* totals, cudaStream_t st);

// T: mask-logit element type (float, __nv_bfloat16, __half); a.logits points
// at T values.
template <bool UNC, bool FOC, bool TMA, bool MIX, typename T = float>
__global__ void cost_partial_kernel(const __grid_constant__ CUtensorMap tmap, CostArgs a);

template <bool UNC, bool FAST>
__global__ void cost_rows_kernel(CostArgs a);

template <bool UNC>
__global__ void cost_pairs_kernel(CostArgs a);

}  // namespace mlb

namespace mlb {

template <typename CT>
struct MatchArgs {
    const CT* costs;       // (N, Q, G)
    int64_t* pred_to_gt;   // (N, Q)
    int64_t* pred_round;   // (N, Q)
    int32_t* status;
    int Q, G;
    double inf_thresh;
    int64_t topk;
    int strategy;
    int stage_cost;        // 0 none, 1 transposed slice, 2 also the solver's double copy
};

template <typename CT>
__global__ void match_kernel(MatchArgs<CT> a);

size_t match_smem_bytes(int Q, int G, size_t cost_elem, int stage);

}  // namespace mlb

namespace mlb {

struct LossArgs {
    // shapes
    int L, B, Q, H, W, Ht, Wt, s, C, G, gt_total, bg;
    int chunk_cells;
    // inputs
    const float* mask_logits;
    const int64_t* targets;
    const float* cls_logits;
    const int64_t* cls_targets;
    const int64_t* pred_to_gt;
    const float* sep;        // (3,L,B,Q,G)
    const float* qstat;      // (L,B,Q,kQStat)
    const float* rawI;
    const float* rawT;
    const float* num_masks_dev;
    const float* grad_mask;  // (L,)
    const float* grad_dice;
    const float* grad_cls;
    const float* stats_in;   // (L,B,Q,kSaved)
    // outputs
    float* saved;            // (L,B,Q,kSaved) or null
    float* layer_means;      // (3,L)
    float* coef;             // (L,3)
    float* stats_out;        // (L,B,Q,kSaved)
    float* grad_mask_logits;
    float* grad_cls_logits;
    // scalars
    float num_masks;
    int auto_num_masks;      // count present GT ids from `totals` (num_masks == -2)
    const int32_t* totals;   // (B, GT_total) label histogram (auto mode)
    float* num_masks_out;    // where the auto count is published, or null
    float smooth, sigmoid_scale, dice_scale, cls_scale;
    float ug, ugmin, mask_gamma, mask_alpha, cls_gamma, cls_alpha;
    int force_masks, force_cls, has_void, void_index, use_softmax, normalize_uncertainty;
    int32_t* void_status;    // forward: bit 4 set when cls_targets holds void_index, or null
    const uint8_t* masks;    // dense (B,GT_total,Ht,Wt) targets instead of the label map, or null
    const int32_t* codes;    // (B, H*W) per-cell column codes (s > 1 label map), or null
    const uint4* mixtab;     // (B, H*W) mixed-cell table beside `codes`, or null
    int rows_zeroed;         // backward: rows without a gradient already hold zeros
};

__global__ void loss_fwd_kernel(LossArgs a);
__global__ void count_masks_kernel(const int32_t* totals, int B, int gt_total, int bg, float* out);
// T: mask-logit element type; a.mask_logits / a.grad_mask_logits point at T.
template <bool UNC, typename T = float> __global__ void bwd_stats_kernel(LossArgs a);
template <bool UNC, bool FOC, bool VEC, typename T = float> __global__ void mask_grad_kernel(LossArgs a);
__global__ void bwd_cls_kernel(LossArgs a);

}  // namespace mlb

namespace mlb {
__global__ void label_cost_kernel(const float* z_all, const int64_t* y_all, float* out, int L, int B,
                                  int Q, int C, int gt_total, int bg, int gout, float scale,
                                  float gamma, float alpha, int use_softmax);
}  // namespace mlb

namespace mlb {
constexpr int kSortWarps = 16;
constexpr int kPointRowThreads = 512;  // block of the per-row point sample / gradient kernels
constexpr size_t kRowMapMaxBytes = 96 * 1024;  // per-row maps staged in shared memory up to this
constexpr int kMaxSortPoints = 40960;          // points per image (sort keys live in shared memory)
size_t point_sort_smem(int P, int gout);
constexpr int kSortBlockPts = 1024;            // points per block of the multi-block sort
// scratch (point_sort_scratch_bytes) selects the multi-block sort; null the
// one-block-per-image form.
size_t point_sort_scratch_bytes(int B, int P, int gout);
cudaError_t launch_point_sort(const int64_t* targets, const float* coords, int B, int Ht, int Wt,
                              int P, int gt_total, int bg, int gout, int32_t* perm, int32_t* scodes,
                              float* scoords, int32_t* ptotals, cudaStream_t st,
                              int32_t* scratch = nullptr);
cudaError_t launch_point_sample(int dtype, const void* logits, const float* scoords, int B, int L,
                                int Q, int H, int W, int P, int align, float* zs, cudaStream_t st);
cudaError_t launch_point_grad(bool foc, int dtype, const LossArgs& la, const float* zs,
                              const float* scoords, const int32_t* scodes, int P, int align,
                              void* grad_out, float* gacc, int64_t rows, bool* used_rows,
                              cudaStream_t st);
cudaError_t launch_to_bf16(const float* src, void* dst, int64_t n, cudaStream_t st);
}  // namespace mlb

namespace mlb {
// Standalone semantic losses (semantic.cu).
struct SemArgs {
    int L, B, C, H, W, Ht, Wt, s;
    int cps, ncs;            // classes per slice, class slices (grid.z)
    const float* logits;     // (L,B,C,H,W)
    const int64_t* targets;  // (B,Ht,Wt)
    float num_masks, scale, gamma, alpha, smooth;
    const float* grad_out;   // (L,) backward
    float* out;              // (L,) forward
    float* grad;             // (L,B,C,H,W) backward
    float *I, *P, *T;        // (L,B,C) dice sums (forward out, backward in)
    double* part_d;          // workspace: per-block / per-(l,b) double partials
    float* part_f;           // workspace: dice per-block partials (L,B,nblk,2,C)
    int32_t* part_t;         // workspace: dice per-block histograms (B,nblk,C)
};
int sem_blocks(const SemArgs& a);
int dice_blocks(const SemArgs& a);
void sem_slices(SemArgs* a, int blocks_per_slice);
size_t dice_fwd_smem(int C, int cps);
cudaError_t launch_sce_forward(SemArgs a, cudaStream_t st);
cudaError_t launch_sce_backward(SemArgs a, cudaStream_t st);
cudaError_t launch_dice_forward(SemArgs a, cudaStream_t st);
cudaError_t launch_dice_backward(SemArgs a, cudaStream_t st);
}  // namespace mlb

namespace mlb {
// Dense per-GT mask targets (dense.cu).
size_t dense_cost_smem(int qrows_pad, bool unc, int gc);
int dense_gc(int gout);
// cnt: [B][GT_total][H*W] counts, bf16 bits (f32 false) or fp32 (f32 true).
cudaError_t launch_dense_count(const uint8_t* masks, int B, int H, int W, int Ht, int Wt, int s,
                               int gt_total, void* cnt, int32_t* totals, cudaStream_t st, bool f32);
// ldt: mask-logit type (0 fp32, 1 bf16, 2 fp16)
cudaError_t launch_dense_cost(const CostArgs& a, bool unc, bool foc, const uint16_t* cnt,
                              cudaStream_t st, int ldt);
// The same partials on tcgen05 tensor cores (dense_mma.cu): no entropy
// weights or focal terms, GT_out <= 64, TMA-aligned logits (ldt: 0 fp32,
// 1 bf16, 2 fp16).
bool dense_mma_usable(const CostArgs& a, int ldt, bool unc, bool foc, bool tma);
int dense_mma_n(int gt_total);  // MMA N: GT_total rounded up to 16
// tm: the logits map (logits_tensor_map); km: the counts, bf16 [B*GT_total][H*W]
// with boxes of 32 cells x dense_mma_n(GT_total) rows and the 64-byte swizzle.
// masks_b (bf16 logits, s = 1): km covers the uint8 masks (boxes of 32 cells
// x N rows, no swizzle); the kernel builds its B tile and the mask areas.
cudaError_t launch_dense_mma(const CUtensorMap& tm, const CUtensorMap& km, const CostArgs& a,
                             cudaStream_t st, int ldt, bool masks_b);
// fp32 logits with GT_total <= 64 (and dense_mma_usable): the kind::tf32
// kernel; km: the counts as fp32 [B*GT_total][H*W], boxes of 32 cells x
// dense_mma_n(GT_total) rows with the 128-byte swizzle, or (masks_b, s = 1)
// the uint8 masks themselves with the same boxes and no swizzle.
bool dense_mma_tf32_usable(const CostArgs& a, int ldt);
cudaError_t launch_dense_mma_tf32(const CUtensorMap& tm, const CUtensorMap& km, const CostArgs& a,
                                  cudaStream_t st, bool masks_b);
}  // namespace mlb
