/*
 * mask_loss_b200.h -- C ABI of the B200-native mask matching + loss path.
 *
 * Plain pointers and sizes only: every tensor is a raw device pointer to a
 * contiguous buffer in the layout stated next to it, every launch goes on the
 * caller's stream, and nothing here allocates device memory (callers pass a
 * workspace sized by the *_workspace_size query).  Every entry returns an
 * ml_status; none of them calls exit() or synchronises the device.
 *
 * Each entry cites the reference interface it replaces
 * (AndyBarcia/mask_loss, path:line).
 */
#ifndef MASK_LOSS_B200_H
#define MASK_LOSS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* ml_stream_t; /* == cudaStream_t */
typedef struct CUevent_st* ml_event_t;   /* == cudaEvent_t */

typedef enum ml_status {
    ML_OK = 0,
    ML_EINVAL = 1,       /* an argument is out of its documented range */
    ML_ESHAPE = 2,       /* inconsistent or unsupported tensor shapes */
    ML_EWORKSPACE = 3,   /* workspace pointer null/misaligned or too small */
    ML_ECUDA = 4,        /* a CUDA launch or attribute call failed */
    ML_ESOLVER = 5,      /* the assignment solver reported failure (see dev_status) */
    ML_EUNSUPPORTED = 6  /* a size beyond what this build supports */
} ml_status;

/* Shapes of one call.  mask_logits (L,B,Q,H,W) of ml_params.logits_dtype
 * (fp32 by default), mask_targets (B,Ht,Wt) int64, cls_logits (L,B,Q,C) fp32,
 * cls_targets (B,GT_total) int64 (-1 pad). */
typedef struct ml_dims {
    int64_t L, B, Q, H, W;
    int64_t Ht, Wt;
    int64_t C;
    int64_t GT_total;
} ml_dims;

/* Scalar arguments of mask_loss.mask_matching (src/bindings.cpp:86-111), same
 * names and meaning.  Booleans are 0/1. */
typedef struct ml_params {
    float smooth, sigmoid_scale, dice_scale, cls_scale;
    int64_t background_index;          /* GT column dropped from the costs, or -1 */
    float uncertainty_gamma, uncertainty_gamma_min;
    double inf_thresh;                 /* costs >= this are treated as +inf */
    double num_masks;                  /* > 0: the normaliser; -2: count the present
                                          GT ids of this call on the device (the
                                          forward then writes the count to
                                          num_masks_dev when given); else <= 0:
                                          use the matched count */
    int32_t force_unmatched_class_to_background;
    int32_t force_unmatched_masks_to_empty;
    int64_t topk_matches;              /* K >= 0 */
    int64_t strategy_id;               /* 0 global, 1 round, 2 greedy, 3 pseudo-greedy */
    float mask_gamma, mask_alpha, cls_gamma, cls_alpha; /* alpha < 0 disables */
    int64_t void_class_index;          /* -1: none */
    int32_t use_softmax_label_loss;
    int32_t normalize_uncertainty;
    int32_t check_void_targets;        /* 1: ml_mask_matching sets bit 4 of dev_status
                                          when a cls_targets entry equals
                                          void_class_index (the check of
                                          functions/mask/matching.py:180-181, done on
                                          the device); 0: no check (the binding) */
    int32_t logits_dtype;              /* element type of mask_logits and
                                          grad_mask_logits in the label-map and
                                          dense entries (ml_pairwise_mask_loss_*
                                          forward, ml_mask_matching[_ex|_dense],
                                          ml_mask_matching[_dense]_backward[_ex]):
                                          0 fp32, 1 bf16, 2 fp16.  The pointers stay
                                          typed float* and point at values of this
                                          type; arithmetic is fp32 either way.  The
                                          no-alloc and semantic entries take fp32
                                          only; the sampled ones have their own
                                          dtype argument and ignore this field. */
} ml_params;

/* Human-readable text of a status code (static storage). */
const char* ml_status_string(int status);

/* Detail of the last failing call on this host thread ("" if none). */
const char* ml_last_error(void);

/* Library version as 10000*major + 100*minor + patch. */
int ml_version(void);

/* Number of kernels this library has launched in this process (monotonic). */
int64_t ml_launch_count(void);

/* Measurement hooks.  While enabled, the library records a CUDA event pair
 * on the launching stream around every launch of its kernels, by kind:
 * 0: pairwise-cost streaming kernel, 1: mask-gradient kernel, 2: assignment
 * solver, 3: label preparation (cell codes + histogram), 4: cost finalize
 * (row statistics + pair costs), 5: matched-loss forward, 6: class-logit
 * backward.  ml_profile_read waits for the recorded events,
 * returns the summed milliseconds and launch counts per kind (arrays of
 * nkinds entries) and clears the record.  No counterpart in the reference. */
void ml_profile_enable(int on);
int ml_profile_read(float* ms, int64_t* launches, int nkinds);

/* GT_out = GT_total minus the background column when it lies in range. */
int64_t ml_gt_out(int64_t GT_total, int64_t background_index);

/* ---------------------------------------------------------------------- */
/* Workspace sizes (bytes, 256-byte aligned pointers expected).             */
/* ---------------------------------------------------------------------- */
size_t ml_mask_matching_workspace_size(const ml_dims* d, const ml_params* p);
size_t ml_mask_matching_backward_workspace_size(const ml_dims* d, const ml_params* p);
size_t ml_match_workspace_size(int64_t L, int64_t B, int64_t Q, int64_t GT_out);

/* ---------------------------------------------------------------------- */
/* Pairwise costs.  Replaces pairwise_mask_loss_forward                    */
/* (src/bindings.cpp:64-82, src/cuda/pw_mask.cu:314-501).                   */
/* out: (3,L,B,Q,GT_out) fp32 -- sigmoid-CE, dice, label cost; +inf where   */
/* the GT id paints no pixel (mask slices) or its class is <0 or >=C.       */
/* Uses the same workspace as ml_mask_matching.                            */
/* ---------------------------------------------------------------------- */
int ml_pairwise_mask_loss_forward(const ml_dims* d, const ml_params* p,
                                  const float* mask_logits, const int64_t* mask_targets,
                                  const float* cls_logits, const int64_t* cls_targets,
                                  float* out, void* workspace, size_t workspace_bytes,
                                  ml_stream_t stream);

/* Same costs as ml_pairwise_mask_loss_forward, for callers that cannot
 * allocate device memory (for example code that runs inside a host-side
 * allocator, a memory pool or a callback that forbids cudaMalloc, or that
 * runs where device memory is fully reserved up front).  No counterpart in
 * the reference: it has no workspace argument, and its scratch lives in a
 * file-scope device array of ml_noalloc_scratch_limit() bytes (64 MiB) that
 * every GPU loading this library holds until the process exits.
 *   - Calls larger than that limit fail with ML_EUNSUPPORTED and a message
 *     (ml_last_error); use the workspace entry point for them.
 *   - It calls no cudaMalloc/cudaFree and no allocating library routine.
 *   - The array's device address is looked up (cudaGetSymbolAddress) with
 *     the device current on every call.  Under CUDA's lazy module loading the
 *     first call on a device also loads this library's device code there and
 *     with it the 64 MiB array, so make that first call before device memory
 *     is reserved up front, and before any stream capture.
 *   - Every call shares the one array: calls that can overlap on the GPU
 *     (different streams, or different host threads on one device) race
 *     and must be serialised by the caller. */
int ml_pairwise_mask_loss_forward_noalloc(const ml_dims* d, const ml_params* p,
                                          const float* mask_logits, const int64_t* mask_targets,
                                          const float* cls_logits, const int64_t* cls_targets,
                                          float* out, ml_stream_t stream);

/* Scratch capacity (bytes) of ml_pairwise_mask_loss_forward_noalloc. */
size_t ml_noalloc_scratch_limit(void);

/* The cost-only entries (ml_pairwise_mask_loss_forward, its dense, sampled
 * and no-alloc forms) have no dev_status argument: their kernels OR bit 2
 * into a library-wide device word when a bounded pipeline wait runs out.
 * ml_cost_status copies that word to *out and clears it.  It synchronises
 * with the device (a plain cudaMemcpyFromSymbol); call it when checking
 * results, not on a hot path.  No reference counterpart. */
int ml_cost_status(int32_t* out);

/* Pairwise label cost alone.  Replaces forward_pw_sigmoid_label_loss /     */
/* forward_pw_softmax_label_loss (src/bindings.cpp:141-155,                 */
/* src/cuda/pw_sigmoid_label_loss.cu:108-187, pw_softmax_label_loss.cu:105-174). */
/* out: (L,B,Q,GT_out) fp32.                                                */
int ml_pairwise_label_loss_forward(int64_t L, int64_t B, int64_t Q, int64_t C,
                                   int64_t GT_total, int64_t background_index,
                                   float scale, float gamma, float alpha, int32_t use_softmax,
                                   const float* cls_logits, const int64_t* cls_targets,
                                   float* out, ml_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Assignment solver alone, one thread-block per (l,b) slice.  Replaces    */
/* the host loop of src/cpu/matching.cpp:690-722 around                    */
/* assign_predictions_for_slice (:476-571).  costs: (L,B,Q,GT_out) fp32,    */
/* evaluated in fp64 exactly as the reference's kDouble copy.              */
/* pred_to_gt / pred_round: (L,B,Q) int64.  dev_status: one device int32    */
/* that stays 0 on success (nonzero: slice failed, outputs set to -1).      */
/* ---------------------------------------------------------------------- */
int ml_match(const float* costs, int64_t L, int64_t B, int64_t Q, int64_t GT_out,
             double inf_thresh, int64_t topk, int64_t strategy_id,
             int64_t* pred_to_gt, int64_t* pred_round, int32_t* dev_status,
             void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* Same solver fed fp64 cost slices directly (for bit-exact checks against
 * the reference solver on identical fp64 matrices). costs: (N,Q,GT_out). */
int ml_match_f64(const double* costs, int64_t N, int64_t Q, int64_t GT_out,
                 double inf_thresh, int64_t topk, int64_t strategy_id,
                 int64_t* pred_to_gt, int64_t* pred_round, int32_t* dev_status,
                 ml_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Fused forward: costs -> on-device matching -> matched-loss means.        */
/* Replaces mask_loss.mask_matching (src/bindings.cpp:86-111,              */
/* src/cpu/matching.cpp:592-752 + src/cuda/mask_matching_forward.cu:283-586). */
/*   pred_to_gt, pred_round : (L,B,Q) int64                                */
/*   layer_means            : (3,L) fp32 -- mask, dice, class means          */
/*   sep_costs  (nullable)  : (3,L,B,Q,GT_out) fp32 copy of the costs        */
/*   saved      (nullable)  : (L,B,Q,4) fp32 per-query statistics that let   */
/*                            ml_mask_matching_backward skip its stats pass  */
/*   num_masks_dev (nullable): device fp32 scalar overriding p->num_masks    */
/*                            (used by data-parallel callers after an        */
/*                            all-reduce, so no host sync is needed)         */
/*   dev_status             : one device int32, 0 on success; bits: 1 the   */
/*                            solver failed, 2 a device wait timed out, 4    */
/*                            cls_targets holds the void class (when         */
/*                            p->check_void_targets)                         */
/* ---------------------------------------------------------------------- */
int ml_mask_matching(const ml_dims* d, const ml_params* p,
                     const float* mask_logits, const int64_t* mask_targets,
                     const float* cls_logits, const int64_t* cls_targets,
                     const float* num_masks_dev,
                     int64_t* pred_to_gt, int64_t* pred_round, float* layer_means,
                     float* sep_costs, float* saved, int32_t* dev_status,
                     void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* ml_mask_matching with one more argument, no reference counterpart:
 * loss_wait_event (nullable) -- the stream waits on it after the assignment
 * and before the matched-loss kernel, the only one that reads num_masks_dev.
 * A data-parallel caller records it after the all-reduce of the GT count on
 * another stream, so the collective overlaps the cost and solver kernels. */
int ml_mask_matching_ex(const ml_dims* d, const ml_params* p,
                        const float* mask_logits, const int64_t* mask_targets,
                        const float* cls_logits, const int64_t* cls_targets,
                        const float* num_masks_dev,
                        int64_t* pred_to_gt, int64_t* pred_round, float* layer_means,
                        float* sep_costs, float* saved, int32_t* dev_status,
                        void* workspace, size_t workspace_bytes, ml_stream_t stream,
                        ml_event_t loss_wait_event);

/* ml_mask_matching_ex plus costs_done_event (nullable): recorded on `stream`
 * once the pairwise costs are final, before the solver launches, so that
 * work which needs only the costs (or nothing of this call, such as zeroing
 * the gradient buffer of ml_mask_matching_backward_ex2) can run on another
 * stream beside the solver.  No reference counterpart. */
int ml_mask_matching_ex2(const ml_dims* d, const ml_params* p,
                         const float* mask_logits, const int64_t* mask_targets,
                         const float* cls_logits, const int64_t* cls_targets,
                         const float* num_masks_dev,
                         int64_t* pred_to_gt, int64_t* pred_round, float* layer_means,
                         float* sep_costs, float* saved, int32_t* dev_status,
                         void* workspace, size_t workspace_bytes, ml_stream_t stream,
                         ml_event_t loss_wait_event, ml_event_t costs_done_event);

/* Per-image GT count (present, non-background GT ids) summed over the batch,
 * written as one fp32 to num_masks_out (device).  This is the num_masks a
 * data-parallel caller all-reduces.  Needs the forward workspace. */
int ml_count_masks(const ml_dims* d, const ml_params* p, const int64_t* mask_targets,
                   float* num_masks_out, void* workspace, size_t workspace_bytes,
                   ml_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Backward.  Replaces mask_loss.mask_matching_backward                     */
/* (src/bindings.cpp:113-139, src/cuda/mask_matching_backward.cu:378-621).   */
/*   grad_*_mean: (L,) fp32 device upstream gradients                       */
/*   saved (nullable): the forward's per-query statistics; when null a      */
/*                     statistics pass re-reads the logits (reference path) */
/*   grad_mask_logits (L,B,Q,H,W) of ml_params.logits_dtype, grad_cls_logits */
/*                     (L,B,Q,C) fp32: fully written (zeros where the loss  */
/*                     does not reach).                                     */
/* ---------------------------------------------------------------------- */
int ml_mask_matching_backward(const ml_dims* d, const ml_params* p,
                              const float* grad_mask_mean, const float* grad_dice_mean,
                              const float* grad_cls_mean,
                              const float* mask_logits, const int64_t* mask_targets,
                              const float* cls_logits, const int64_t* cls_targets,
                              const int64_t* pred_to_gt, const float* saved,
                              const float* num_masks_dev,
                              float* grad_mask_logits, float* grad_cls_logits,
                              void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* As ml_mask_matching_backward, plus forward_workspace (nullable): the      */
/* workspace of the ml_mask_matching / ml_mask_matching_ex call with the same */
/* dims and params, left untouched since.  With an s > 1 label map its per-  */
/* cell codes are reused instead of being rebuilt from the label map.  No    */
/* reference counterpart (the reference's backward has no workspace).       */
int ml_mask_matching_backward_ex(const ml_dims* d, const ml_params* p,
                                 const float* grad_mask_mean, const float* grad_dice_mean,
                                 const float* grad_cls_mean,
                                 const float* mask_logits, const int64_t* mask_targets,
                                 const float* cls_logits, const int64_t* cls_targets,
                                 const int64_t* pred_to_gt, const float* saved,
                                 const float* num_masks_dev,
                                 float* grad_mask_logits, float* grad_cls_logits,
                                 void* workspace, size_t workspace_bytes, ml_stream_t stream,
                                 const void* forward_workspace);

/* ml_mask_matching_backward_ex plus grad_rows_prezeroed: when non-zero, the
 * caller has already filled grad_mask_logits with zeros, and only the rows
 * that carry a gradient (matched queries, or every query with
 * force_unmatched_masks_to_empty) are written.  The zero fill can then run
 * beside the solver instead of after it.  No reference counterpart. */
int ml_mask_matching_backward_ex2(const ml_dims* d, const ml_params* p,
                                  const float* grad_mask_mean, const float* grad_dice_mean,
                                  const float* grad_cls_mean,
                                  const float* mask_logits, const int64_t* mask_targets,
                                  const float* cls_logits, const int64_t* cls_targets,
                                  const int64_t* pred_to_gt, const float* saved,
                                  const float* num_masks_dev,
                                  float* grad_mask_logits, float* grad_cls_logits,
                                  void* workspace, size_t workspace_bytes, ml_stream_t stream,
                                  const void* forward_workspace, int grad_rows_prezeroed);

/* ---------------------------------------------------------------------- */
/* Point-sampled costs and matching (config 3).  Replaces                    */
/* pairwise_sigmoid_cross_entropy_loss_sampling_py                           */
/* (functions/sigmoid/pw_sigmoid_ce.py:407-549) and                          */
/* pairwise_dice_loss_sampling_py (functions/dice/pw_dice_loss.py:174-268):  */
/* one shared set of num_points points per image, point_coords (B,P,2) fp32  */
/* in [0,1] (x, y), logits sampled bilinearly with zero padding (grid_sample, */
/* align_corners as given), labels read at floor(x*(W_t-1)), floor(y*(H_t-1)). */
/* BCE = (<c+,t> + <c-,1-t>)/P, dice over the points, +inf for GT ids absent */
/* from the whole label map; no entropy weights (uncertainty_gamma must be 0) */
/* and no forced-empty unmatched masks.  logits_dtype: 0 fp32, 1 bf16.        */
/* The matched losses and gradients of the sampled costs have no counterpart  */
/* in the reference (it never wires sampling into matching,                   */
/* functions/mask/matching.py:836).                                           */
/* ---------------------------------------------------------------------- */
size_t ml_sampled_workspace_size(const ml_dims* d, const ml_params* p, int64_t num_points);
size_t ml_sampled_backward_workspace_size(const ml_dims* d, const ml_params* p,
                                          int64_t num_points, int32_t logits_dtype);

int ml_pairwise_mask_loss_sampled_forward(const ml_dims* d, const ml_params* p, int64_t num_points,
                                          int32_t align_corners, int32_t logits_dtype,
                                          const void* mask_logits, const int64_t* mask_targets,
                                          const float* cls_logits, const int64_t* cls_targets,
                                          const float* point_coords, float* out, void* workspace,
                                          size_t workspace_bytes, ml_stream_t stream);

int ml_mask_matching_sampled(const ml_dims* d, const ml_params* p, int64_t num_points,
                             int32_t align_corners, int32_t logits_dtype, const void* mask_logits,
                             const int64_t* mask_targets, const float* cls_logits,
                             const int64_t* cls_targets, const float* point_coords,
                             const float* num_masks_dev, int64_t* pred_to_gt, int64_t* pred_round,
                             float* layer_means, float* sep_costs, float* saved, int32_t* dev_status,
                             void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* grad_mask_logits has the logits' dtype; gradients are accumulated with
 * atomics through the bilinear weights (order-dependent in the last ulp).
 * forward_workspace (nullable): the workspace of the ml_mask_matching_sampled
 * call with the same arguments, still unmodified; its sorted points and
 * samples are reused instead of being rebuilt. */
int ml_mask_matching_sampled_backward(const ml_dims* d, const ml_params* p, int64_t num_points,
                                      int32_t align_corners, int32_t logits_dtype,
                                      const float* grad_mask_mean, const float* grad_dice_mean,
                                      const float* grad_cls_mean, const void* mask_logits,
                                      const int64_t* mask_targets, const float* cls_logits,
                                      const int64_t* cls_targets, const float* point_coords,
                                      const int64_t* pred_to_gt, const float* saved,
                                      const float* num_masks_dev, const void* forward_workspace,
                                      void* grad_mask_logits, float* grad_cls_logits,
                                      void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Dense per-GT mask targets -- no counterpart in the reference, whose API  */
/* takes a label map only (src/bindings.cpp:66).  mask_masks: (B, GT_total,  */
/* Ht, Wt) uint8, nonzero = inside, aligned with cls_targets' columns; masks */
/* may overlap.  Costs, matching and losses follow the label-map entries     */
/* with each GT's pixel count per cell in place of the one-hot count; on     */
/* non-overlapping masks the results equal the label-map path.  d->GT_total  */
/* is the mask count.  Workspace: ml_dense_workspace_size (forwards); the    */
/* backward uses ml_mask_matching_backward_workspace_size and needs the     */
/* forward's saved statistics.                                               */
/* ---------------------------------------------------------------------- */
size_t ml_dense_workspace_size(const ml_dims* d, const ml_params* p);

int ml_pairwise_mask_loss_dense_forward(const ml_dims* d, const ml_params* p,
                                        const float* mask_logits, const uint8_t* mask_masks,
                                        const float* cls_logits, const int64_t* cls_targets,
                                        float* out, void* workspace, size_t workspace_bytes,
                                        ml_stream_t stream);

int ml_mask_matching_dense(const ml_dims* d, const ml_params* p,
                           const float* mask_logits, const uint8_t* mask_masks,
                           const float* cls_logits, const int64_t* cls_targets,
                           const float* num_masks_dev,
                           int64_t* pred_to_gt, int64_t* pred_round, float* layer_means,
                           float* sep_costs, float* saved, int32_t* dev_status,
                           void* workspace, size_t workspace_bytes, ml_stream_t stream);

int ml_mask_matching_dense_backward(const ml_dims* d, const ml_params* p,
                                    const float* grad_mask_mean, const float* grad_dice_mean,
                                    const float* grad_cls_mean, const float* mask_logits,
                                    const uint8_t* mask_masks, const float* cls_logits,
                                    const int64_t* cls_targets, const int64_t* pred_to_gt,
                                    const float* saved, const float* num_masks_dev,
                                    float* grad_mask_logits, float* grad_cls_logits,
                                    void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Standalone semantic losses of (L,B,C,H,W) fp32 logits against a         */
/* (B,Ht,Wt) int64 label map with classes in [0,C) (Ht = s*H, Wt = s*W,     */
/* s <= 16, C <= 2048; labels outside [0,C) count for no class).           */
/* Replace forward/backward_sigmoid_ce_loss (src/cuda/sigmoid_ce.cu:207-332, */
/* src/bindings.cpp:158-159) and forward/backward_dice_loss                 */
/* (src/cuda/dice_loss.cu:159-288, src/bindings.cpp:161-162).  Sums are     */
/* fixed-order (deterministic).                                              */
/* ---------------------------------------------------------------------- */
/* Workspace of the forwards (dice = 0: sigmoid CE, 1: dice). */
size_t ml_semantic_workspace_size(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W,
                                  int64_t Ht, int64_t Wt, int32_t dice);

/* out (L,): scale * sum of (focal) BCE over b, c and target pixels /
 * (num_masks * Ht * Wt).  alpha < 0 disables the alpha weights. */
int ml_sigmoid_ce_forward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht,
                          int64_t Wt, const float* logits, const int64_t* targets,
                          float num_masks, float scale, float gamma, float alpha, float* out,
                          void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* grad_logits (L,B,C,H,W) from grad_out (L,). */
int ml_sigmoid_ce_backward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht,
                           int64_t Wt, const float* grad_out, const float* logits,
                           const int64_t* targets, float num_masks, float scale, float gamma,
                           float alpha, float* grad_logits, ml_stream_t stream);

/* out (L,): scale * sum over (b,c) of 1 - (2I+smooth)/(P+T+smooth) / num_masks;
 * int_sum, p_sum, t_sum (L,B,C): I, P, T of every (l,b,c). */
int ml_dice_forward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                    const float* logits, const int64_t* targets, float smooth, float num_masks,
                    float scale, float* out, float* int_sum, float* p_sum, float* t_sum,
                    void* workspace, size_t workspace_bytes, ml_stream_t stream);

/* grad_logits (L,B,C,H,W) from grad_out (L,) and the forward's I, P, T. */
int ml_dice_backward(int64_t L, int64_t B, int64_t C, int64_t H, int64_t W, int64_t Ht, int64_t Wt,
                     const float* grad_out, const float* logits, const int64_t* targets,
                     const float* int_sum, const float* p_sum, const float* t_sum, float smooth,
                     float num_masks, float scale, float* grad_logits, ml_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MASK_LOSS_B200_H */
