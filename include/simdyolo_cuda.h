/*
 * simdyolo_cuda.h - C ABI of the B200 (sm_100a) detection-head fine-tuning path.
 *
 * The reference (SimdYolo, C#/.NET) trains the detection head one image at a time on the CPU
 * (src/SimdYolo.Training/YoloTrainer.cs:185-199) and offloads only large GEMMs through
 * IComputeBackend.MatMul (src/SimdYolo/Compute.cs:11-25).  This library moves the whole inner
 * batch loop behind one call: frozen backbone forward, Detect-head forward/backward with
 * per-image training BatchNorm, DFL + CIoU + BCE loss with the task-aligned assigner, the
 * optional NCCL gradient all-reduce and the SGD-momentum / AdamW update.
 *
 * Conventions: plain C types; host pointers unless a name says "device"; the caller owns every
 * buffer it passes and may reuse it as soon as a call returns (calls are synchronous).  Tensors
 * use the reference layouts: NCHW activations, OIHW weights, float32.  A session is not
 * reentrant (the C# host serialises calls, YoloTrainer.cs:163-168).
 *
 * Status codes map onto the reference's exceptions:
 *   SY_ERR_INVALID_ARGUMENT  -> ArgumentException            (e.g. DetectionLoss.cs:21,30,51)
 *   SY_ERR_UNSUPPORTED_SHAPE -> NotSupportedException        (HeadOperations.cs:34, TrainingHeadSchema.cs:44)
 *   SY_ERR_NONFINITE         -> ArithmeticException          (YoloTrainer.cs:193,196; TrainingParameter.cs:40)
 *   SY_ERR_COMM, SY_ERR_DEVICE, SY_ERR_OUT_OF_MEMORY -> InvalidOperationException (VulkanBackend.cs:323 style)
 */
#ifndef SIMDYOLO_CUDA_H
#define SIMDYOLO_CUDA_H
#include <stdint.h>

#if defined(__GNUC__)
#define SY_API __attribute__((visibility("default")))
#else
#define SY_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t sy_status;
#define SY_OK 0
#define SY_ERR_INVALID_ARGUMENT 1
#define SY_ERR_UNSUPPORTED_SHAPE 2
#define SY_ERR_NONFINITE 3
#define SY_ERR_COMM 4
#define SY_ERR_DEVICE 5
#define SY_ERR_OUT_OF_MEMORY 6

/* TrainingBox (src/SimdYolo.Training/TrainingTypes.cs:50): class id and xyxy in input pixels. */
typedef struct sy_box {
    int32_t class_id;
    float x1, y1, x2, y2;
} sy_box;

/* One block of a head branch (DetectionHead.cs:28-75, validated like TrainingHeadSchema.cs:36-46):
 * Conv/DWConv (has_bn = 1: conv without bias -> BatchNorm -> SiLU) or the final Conv2d
 * (has_bn = 0, has_bias = 1).  Kernel 1 or 3, stride 1, same padding.  groups must divide ic and oc:
 * groups = ic = oc is depthwise (up to 512 channels, BatchNorm, a multiple of 4 channels); other convs have
 * at most 256 output channels.  Anything else is SY_ERR_UNSUPPORTED_SHAPE at sy_cuda_create. */
typedef struct sy_block {
    int32_t ic, oc, k, groups, has_bn, has_bias;
} sy_block;

#define SY_OPT_SGD 0
#define SY_OPT_ADAMW 1
/* Tensor-core precision of every convolution in the step.  3xTF32 splits each FP32 operand into a
 * TF32 value and a TF32 residual and sums three products (small x big, big x small, big x big),
 * which restores FP32-level agreement with the reference's FP32 arithmetic at 3x the MMA work. */
#define SY_PRECISION_TF32 0
#define SY_PRECISION_3XTF32 1
#define SY_BACKBONE_NONE 0    /* features are supplied by the caller (cached features)       */
#define SY_BACKBONE_YOLOV8 1  /* YOLOv8 detection trunk (Conv, C2f, SPPF, Upsample, Concat) */
#define SY_BACKBONE_YOLO11 2  /* YOLO11 trunk (Conv, C3k2, C3k, SPPF, C2PSA attention, Upsample, Concat) */

typedef struct sy_config {
    int32_t struct_size;        /* sizeof(sy_config) */
    int32_t device;             /* CUDA device ordinal */
    int32_t rank, world_size;   /* data-parallel group: one process per GPU */
    uint8_t nccl_id[128];       /* from sy_cuda_nccl_unique_id on rank 0; ignored when world_size == 1 */
    int32_t image_size;         /* square input S (multiple of 32) */
    int32_t max_batch;          /* images per step on this rank */
    int32_t max_boxes;          /* ground-truth boxes per image (<= 100) */
    int32_t num_classes;        /* nc */
    int32_t reg_max;            /* 16 (DFL) or 1 (direct distances, end-to-end heads only) */
    int32_t backbone;           /* SY_BACKBONE_* */
    float width_mult, depth_mult;
    int32_t max_channels;
    int32_t feature_channels[3];/* P3/P4/P5 channels when backbone == SY_BACKBONE_NONE */
    int32_t n_box_blocks, n_cls_blocks;
    sy_block box_blocks[3][8];  /* cv2.{0,1,2} (and one2one_cv2.{0,1,2} with end_to_end) */
    sy_block cls_blocks[3][8];  /* cv3.{0,1,2} (and one2one_cv3.{0,1,2} with end_to_end) */
    float bn_eps, bn_momentum;  /* DetectionHead.cs:71 (PT defaults 1e-3 / 0.03) */
    int32_t optimizer;          /* SY_OPT_* */
    float lr, momentum, weight_decay;
    float beta1, beta2, adam_eps;
    int32_t precision;          /* SY_PRECISION_TF32, or SY_PRECISION_3XTF32 for the FP32 parity mode */
    /* TrainingHeadSchema (src/SimdYolo/TrainingHeadSchema.cs:7-21): end_to_end = 1 adds the
     * one2one_cv2 / one2one_cv3 branches (YOLOv10 / YOLO26 heads), trained with a second loss
     * (DetectionHead.cs:105-115); with reg_max 1 the loss is the progressive one whose one-to-many
     * weight follows DetectionHead.ProgressiveWeight(epoch, schedule_epochs). */
    int32_t end_to_end;
    int32_t schedule_epochs;    /* LossScheduleEpochs (YoloTrainer.cs:106): TrainingOptions.Epochs */
    /* Data-parallel sessions: a step whose collectives have not completed after comm_timeout_ms (0: 300000)
     * aborts the communicator (ncclCommAbort) and returns SY_ERR_COMM; the session then refuses further steps
     * and can only be destroyed. */
    int32_t comm_timeout_ms;
} sy_config;

/* Per-step results, summed over the global batch (all ranks). */
typedef struct sy_step_stats {
    double box, cls, dfl;       /* loss sums; YoloTrainer divides by the batch (YoloTrainer.cs:198) */
    int64_t positives;
    int32_t images;             /* global images in the step */
    int32_t box_has_grad;       /* bit 0: cv2 connected (any positive, DetectionLoss.cs:101); bit 1: one2one_cv2 */
    double grad_checksum;       /* sum of |g| over the averaged head gradient before the update */
    double device_ms;           /* device time of the step (CUDA events) */
    /* Assigner decisions taken by a margin of at most 16 ulp (GT boxes whose top-k boundary, and conflicted
     * anchors whose best and second overlap, lie that close): the reference computes the same quantities
     * with the platform libm (MathF.Exp / Atan / Pow, DetectionLoss.cs:63-65), which may decide these the
     * other way.  No counterpart in the reference. */
    int64_t near_ties;
} sy_step_stats;

typedef struct sy_tensor_info {
    char name[96];              /* DetectionHead.Snapshot name, e.g. "cv2.0.0.conv.weight" */
    int32_t kind;               /* 0 parameter, 1 buffer (BN running mean/var/num_batches_tracked) */
    int32_t rank;
    int32_t shape[4];
    int64_t numel;
} sy_tensor_info;

typedef struct sy_session sy_session;

/* Detection (src/SimdYolo/YoloDetector.cs:139): class, confidence and the box as top-left corner plus
 * size, in source-image pixels. */
typedef struct sy_detection {
    int32_t class_id;
    float confidence, x, y, width, height;
} sy_detection;

/* Letterbox (YoloDetector.cs:149): the preprocessing record that maps model pixels back to the source
 * image, x_source = (x_model - pad_x) / scale_x, clamped to [0, source_width]. */
typedef struct sy_letterbox {
    int32_t source_width, source_height, target_width, target_height;
    float scale_x, scale_y;
    int32_t pad_x, pad_y;
} sy_letterbox;

/* DetectorOptions' decode fields (YoloDetector.cs:88-105; defaults 0.25, 0.45, 300, 30000, 0).
 * DetectionEvaluator.Evaluate uses confidence 0.001, IoU 0.7, 300 detections (DetectionEvaluator.cs:50-51).
 * max_detections 1 .. 65536; max_candidates >= 1.  sy_cuda_detect* require confidence and iou_threshold in
 * [0, 1] (the YoloDetector constructor's check); sy_cuda_decode_detections, like the reference's static
 * decode, takes any value (NaN: no candidate is below the confidence threshold, no overlap above the IoU
 * threshold). */
typedef struct sy_detect_options {
    float confidence, iou_threshold;
    int32_t max_detections, max_candidates;
    int32_t class_agnostic;     /* ClassAgnosticNms */
} sy_detect_options;

#define SY_LAYOUT_AUTO 0            /* OutputLayout (YoloDetector.cs:49-59) */
#define SY_LAYOUT_CHANNELS_FIRST 1
#define SY_LAYOUT_CHANNELS_LAST 2
#define SY_LAYOUT_END_TO_END 3

/* ---- session (replaces YoloTrainer's inner batch loop, YoloTrainer.cs:185-199) ---- */
SY_API sy_status sy_cuda_nccl_unique_id(uint8_t out[128]);
SY_API sy_status sy_cuda_create(const sy_config *config, sy_session **out);
SY_API sy_status sy_cuda_destroy(sy_session *session);
SY_API const char *sy_cuda_last_error(const sy_session *session);   /* NULL session: last global error */

/* Snapshot-ordered tensors (DetectionHead.Snapshot / Restore, DetectionHead.cs:124-142). */
SY_API int32_t sy_cuda_tensor_count(const sy_session *session);
SY_API sy_status sy_cuda_tensor_info(const sy_session *session, int32_t index, sy_tensor_info *out);
SY_API sy_status sy_cuda_set_tensor(sy_session *session, int32_t index, const float *host, int64_t count);
SY_API sy_status sy_cuda_get_tensor(const sy_session *session, int32_t index, float *host, int64_t count);
/* Optimizer state of a parameter tensor (TrainingParameter.Velocity, YoloTrainer.cs:135-141);
 * moment 0 = SGD velocity / AdamW first moment, 1 = AdamW second moment. */
SY_API sy_status sy_cuda_set_optimizer_state(sy_session *session, int32_t index, int32_t moment, const float *host,
                                      int64_t count);
SY_API sy_status sy_cuda_get_optimizer_state(const sy_session *session, int32_t index, int32_t moment, float *host,
                                      int64_t count);
/* Frozen backbone weights with BatchNorm folded (PtModel.cs:128-144): for every conv in trunk
 * order, OIHW weight then bias. */
SY_API int64_t sy_cuda_backbone_param_count(const sy_session *session);
SY_API sy_status sy_cuda_set_backbone(sy_session *session, const float *host, int64_t count);

/* One optimizer step over `images` RGB24 images (images * S * S * 3 bytes, HWC, letterboxed to S)
 * with boxes[counts[0] + ... + counts[images-1]] in input pixels. */
SY_API sy_status sy_cuda_step(sy_session *session, const uint8_t *rgb, const sy_box *boxes, const int32_t *counts,
                       int32_t images, sy_step_stats *out);
/* Same step from cached frozen features (YoloTrainer.cs:257-261): features[l] is NCHW
 * [images][C_l][S/8/2^l][S/8/2^l]. */
SY_API sy_status sy_cuda_step_features(sy_session *session, const float *const features[3], const sy_box *boxes,
                                const int32_t *counts, int32_t images, sy_step_stats *out);
/* Same step with the RGB24 images already in device memory of the session's GPU (rgb_device:
 * images * S * S * 3 bytes, caller-owned). */
SY_API sy_status sy_cuda_step_device(sy_session *session, const uint8_t *rgb_device, const sy_box *boxes,
                                     const int32_t *counts, int32_t images, sy_step_stats *out);
/* Queues a batch of `images` RGB24 images (images * S * S * 3 bytes of host memory) for copying to the
 * session's GPU and returns at once.  The copy runs on a separate copy stream, started by the next call that
 * takes inputs (sy_cuda_step, sy_cuda_eval_loss, sy_cuda_detect and their variants) right after that call's
 * own small uploads, so a host loop that prefetches batch k + 1 before it steps batch k overlaps the copy
 * with batch k's device work; the call given the same rgb pointer and image count then uses the copy instead
 * of copying the images itself.  The two most recent prefetches are held; the memory must not change until
 * the call that uses it has returned.  Page-locked memory is copied directly, pageable memory is first copied
 * into a page-locked staging buffer of the session (inside this call).  No counterpart in the reference (its
 * trainer reads images on the host). */
SY_API sy_status sy_cuda_prefetch_images(sy_session *session, const uint8_t *rgb, int32_t images);
/* YoloTrainer.EvaluateLoss (YoloTrainer.cs:237-246): the head with BatchNorm in evaluation mode
 * (running mean / variance), the loss without gradients; no parameter, buffer or optimizer state
 * changes.  out->box / cls / dfl / positives are sums over the images of every rank (the reference
 * reports their mean total, (box + cls + dfl) / images); the gradient fields are zero. */
SY_API sy_status sy_cuda_eval_loss(sy_session *session, const uint8_t *rgb, const sy_box *boxes, const int32_t *counts,
                                   int32_t images, sy_step_stats *out);
SY_API sy_status sy_cuda_eval_loss_features(sy_session *session, const float *const features[3], const sy_box *boxes,
                                            const int32_t *counts, int32_t images, sy_step_stats *out);
/* The completed-epoch counter YoloTrainer passes to DetectionHead.Loss (YoloTrainer.cs:192); it only
 * matters for progressive end-to-end heads.  Evaluation always uses epoch 0 (YoloTrainer.cs:243). */
SY_API sy_status sy_cuda_set_epoch(sy_session *session, int32_t epoch);
/* AdamW steps taken per optimizer group: [0] class branches, [1] cv2, [2] one2one_cv2 (a box group steps only
 * when an image connected it).  AdamW is not in the reference; with sy_cuda_get/set_optimizer_state these
 * counts complete the state a resumed AdamW run needs. */
SY_API sy_status sy_cuda_get_optimizer_steps(const sy_session *session, int32_t steps[3]);
SY_API sy_status sy_cuda_set_optimizer_steps(sy_session *session, const int32_t steps[3]);
/* Gradient of the last step (summed over the images of every rank, before the update), parameter order. */
SY_API sy_status sy_cuda_get_last_gradients(const sy_session *session, float *host, int64_t count);
/* Frozen features of the last step (NCHW per level), for parity checks. */
SY_API sy_status sy_cuda_get_last_features(const sy_session *session, int32_t level, float *host, int64_t count);
/* Raw head outputs of the last step, evaluation or detection (NCHW per level): box logits
 * [images][4 * reg_max][H_l][W_l] and class logits [images][nc][H_l][W_l] of branch set `set` (0 cv2 / cv3,
 * 1 one2one_cv2 / one2one_cv3), for parity checks. */
SY_API sy_status sy_cuda_get_last_head_outputs(const sy_session *session, int32_t set, int32_t level, float *box,
                                               int64_t box_count, float *cls, int64_t cls_count);

/* ---- inference (YoloDetector.Detect on the session's model, YoloDetector.cs:327-376) ---- */

/* Detection on `images` RGB24 images of S x S (already letterboxed, as for sy_cuda_step): frozen trunk, head
 * with BatchNorm in evaluation mode (running statistics), decode (CpuHead.DecodeInto, CpuHead.cs:57-120),
 * then YoloDetector.DecodeIndexed (YoloDetector.cs:539-642): confidence filter, confidence order,
 * max_candidates, greedy NMS (class-aware unless class_agnostic), max_detections, and the mapping through
 * transforms[b] (NULL: identity, source S x S).  End-to-end heads use their one-to-one branches and
 * PtModel.EndToEndTopK (PtModel.cs:530-568, max_det 300) instead of NMS.  out holds
 * images * max_detections records, image b's counts[b] detections first in its block.  timing (optional,
 * no counterpart in the reference) receives [0] the call's device ms (upload to detections read back) and
 * [1] the device ms of the post-processing kernels.  Nothing in the session's parameters, buffers or
 * optimizer state changes. */
SY_API sy_status sy_cuda_detect(sy_session *session, const uint8_t *rgb, int32_t images,
                                const sy_letterbox *transforms, const sy_detect_options *options, sy_detection *out,
                                int32_t *counts, double *timing);
/* The same from cached frozen features (NCHW per level, as for sy_cuda_step_features). */
SY_API sy_status sy_cuda_detect_features(sy_session *session, const float *const features[3], int32_t images,
                                         const sy_letterbox *transforms, const sy_detect_options *options,
                                         sy_detection *out, int32_t *counts, double *timing);

/* ---- standalone operators (same algorithms as the session, host buffers) ---- */

/* DetectionLoss.Compute (DetectionLoss.cs:19-149) for a batch: boxes[l] NCHW [images][4*reg_max][H_l][W_l],
 * classes[l] NCHW [images][nc][H_l][W_l]; per-image losses out_loss[images][3] (box, cls, dfl),
 * positives[images]; optional assigned[images][A] (gt index or -1) and scores[images][A];
 * optional gradients with the same shapes as the inputs. */
SY_API sy_status sy_cuda_detection_loss(int32_t device, int32_t images, int32_t levels, const int32_t *hs, const int32_t *ws,
                                 const float *strides, int32_t nc, int32_t reg_max, const float *const *boxes,
                                 const float *const *classes, const sy_box *truth, const int32_t *counts,
                                 float *out_loss, int32_t *positives, int32_t *assigned, float *scores,
                                 float *const *box_grads, float *const *class_grads);
/* The same with the assigner's candidate counts (topk 1..15) and the gradient scale (DetectionLoss.Compute
 * arguments topk, topk2, gradientScale, DetectionLoss.cs:48-91): end-to-end heads call it with
 * (10, 10, w) for the one-to-many branch and (7 or 1, 1, 1 - w) for the one-to-one branch;
 * reg_max 1 is the L1 box loss of YOLO26 (DetectionLoss.cs:123-131). */
SY_API sy_status sy_cuda_detection_loss_ex(int32_t device, int32_t images, int32_t levels, const int32_t *hs,
                                           const int32_t *ws, const float *strides, int32_t nc, int32_t reg_max,
                                           const float *const *boxes, const float *const *classes, const sy_box *truth,
                                           const int32_t *counts, int32_t topk, int32_t topk2, float grad_scale,
                                           float *out_loss, int32_t *positives, int32_t *assigned, float *scores,
                                           float *const *box_grads, float *const *class_grads);

/* CpuHead.Decode / DecodeInto (CpuHead.cs:50-120) over joined levels, as PtModel.Detect joins them
 * (PtModel.cs:455-480): box[l] [images][4 * bins][hs[l]][ws[l]] (bins 1 or 16), cls[l] [images][nc][hs[l]][ws[l]]
 * -> out [images][4 + nc][anchors]: (cx, cy, w, h), or (x1, y1, x2, y2) with xyxy, in model pixels, then the
 * sigmoid class scores.  levels 1 .. 8. */
SY_API sy_status sy_cuda_head_decode(int32_t device, int32_t images, int32_t levels, const int32_t *hs,
                                     const int32_t *ws, const float *strides, int32_t bins, int32_t nc, int32_t xyxy,
                                     const float *const *box, const float *const *cls, float *out);
/* PtModel.EndToEndTopK (PtModel.cs:530-568): x [images][fields][anchors] (4 box fields, nc scores, extra
 * fields) -> out [images][k][6 + fields - nc - 4], k = min(maximum, anchors) (maximum 1 .. 1024): the k
 * anchors with the largest class maximum, then the k largest (anchor, class) scores among them, ordered by
 * score, anchor and class; rows (box fields, score, class, extra fields). */
SY_API sy_status sy_cuda_end_to_end_topk(int32_t device, const float *x, int32_t images, int32_t fields,
                                         int32_t anchors, int32_t nc, int32_t maximum, float *out);
/* YoloDetector.DecodeIndexed (YoloDetector.cs:539-642) per image on output [images][dim1][dim2] in
 * `layout` (SY_LAYOUT_*; AUTO is resolved from class_count and the shape as the reference does);
 * class_count 0 means every field after the box is a class score.  transforms[images] (NULL: identity with
 * a source of 2^20 x 2^20); out [images][max_detections], counts[images]. */
SY_API sy_status sy_cuda_decode_detections(int32_t device, const float *output, int32_t images, int32_t dim1,
                                           int32_t dim2, int32_t layout, int32_t class_count,
                                           const sy_letterbox *transforms, const sy_detect_options *options,
                                           sy_detection *out, int32_t *counts);

/* HeadOperations.Conv (HeadOperations.cs:29-82) batched: x NCHW [n][ic][h][w], w OIHW [oc][ic][k][k],
 * stride 1, padding k/2.  forward: y = conv(x, w) (+ bias);  backward_data: dx = conv^T(dy, w);
 * backward_filter: dw = sum_n dy (*) x (overwrites dw).  k in {1, 3}. */
SY_API sy_status sy_cuda_conv2d_forward(int32_t device, const float *x, int32_t n, int32_t ic, int32_t h, int32_t w,
                                 const float *weight, int32_t oc, int32_t k, const float *bias, float *y);
SY_API sy_status sy_cuda_conv2d_backward_data(int32_t device, const float *dy, int32_t n, int32_t oc, int32_t h, int32_t w,
                                       const float *weight, int32_t ic, int32_t k, float *dx);
SY_API sy_status sy_cuda_conv2d_backward_filter(int32_t device, const float *x, const float *dy, int32_t n, int32_t ic,
                                         int32_t oc, int32_t h, int32_t w, int32_t k, float *dw);

/* Allocation-free weight gradient: no counterpart in the reference.  For hosts that cannot let a library
 * call cudaMalloc (an embedding runtime or caching allocator that has reserved all device memory for its
 * own pool, or a serving loop that must not take the driver's allocation locks mid-request): same result as
 * sy_cuda_conv2d_backward_filter, but every buffer is caller-owned device memory and the split-K scratch is
 * a fixed 16 MiB static device array per GPU that loads the library (shapes needing more, or with more
 * than 256 output / 4096 input channels, return SY_ERR_UNSUPPORTED_SHAPE; the message is in
 * sy_cuda_last_error(NULL)).  x / dy use the library's padded channels-last layout: image b, pixel (y, x)
 * at row b * R + (y + 1) * (w + 2) + (x + 1) with R = round_up((h + 2) * (w + 2), 128), rows of
 * round_up(C, 4) floats, halo rows zero.  dw is OIHW.  The first call on a device looks up the static
 * array's device address.  Calls share the array, so calls that overlap on the GPU race; the call
 * returns after `stream` (NULL = legacy default stream) has finished it. */
SY_API sy_status sy_cuda_conv2d_backward_filter_static(int32_t device, const float *x_padded_device,
                                                       const float *dy_padded_device, int32_t n, int32_t ic,
                                                       int32_t oc, int32_t h, int32_t w, int32_t k, float *dw_device,
                                                       void *stream);

/* IComputeBackend.MatMul (Compute.cs:11-25): C[m,n] = A[m,k] * B[k,n], row-major, C overwritten. */
SY_API sy_status sy_cuda_matmul(int32_t device, const float *a, const float *b, float *c, int32_t m, int32_t n, int32_t k);

/* Measurement helpers (no counterpart in the reference, which times with Stopwatch).
 * sy_cuda_launch_count: kernels this library has launched in the process so far (a CUDA graph replay
 * counts every kernel node of the graph).
 * sy_cuda_bench_conv: device time in ms per launch (CUDA events, `iters` back-to-back launches after
 * one warm-up) of one convolution pass on device-resident data: kind 0 forward, 1 data gradient,
 * 2 weight gradient; shapes as in sy_cuda_conv2d_*. */
SY_API int64_t sy_cuda_launch_count(void);
/* sy_cuda_conv_profile: with enable != 0, the following steps of `session` record CUDA events around
 * every tensor-core convolution launch (trunk forward, head forward, head data gradients) on the
 * session stream.  Returns, and resets, the totals since the previous call: device ms, algorithmic
 * GFLOP (2 x MACs of the interior pixels) and the number of convolution launches. */
SY_API sy_status sy_cuda_conv_profile(sy_session *session, int32_t enable, double *ms, double *gflop,
                                      int64_t *launches);
/* Per-launch device ms, GFLOP and shape of the tensor-core conv launches of the most recent profiled
 * step, in launch order; shapes (optional) receives 6 ints per launch: pass (0 trunk stride 1, 1 trunk
 * stride 2, 2 head forward, 3 head data gradient), input channels, output channels, taps, output
 * height, output width.  *count receives the number of launches. */
SY_API sy_status sy_cuda_conv_profile_launches(const sy_session *session, double *ms, double *gflop,
                                               int32_t *shapes, int32_t capacity, int32_t *count);
SY_API sy_status sy_cuda_bench_conv(int32_t device, int32_t kind, int32_t n, int32_t ic, int32_t oc, int32_t h,
                                    int32_t w, int32_t k, int32_t iters, double *ms_per_launch);

/* Check of the bounded device waits (no counterpart in the reference, whose CPU loops cannot hang): one CTA
 * waits on an mbarrier that nothing arrives on, gives up after `spins` polls (1 .. 2^22), frees its TMEM and
 * exits, as every pipelined kernel here does after a timed-out wait.  Returns SY_ERR_DEVICE with *code set to
 * the wait's error code (21), and the context stays usable. */
SY_API sy_status sy_cuda_wait_limit_selftest(int32_t device, int32_t spins, int32_t *code);

/* TrainingParameter.Update (TrainingParameter.cs:21-43) on one tensor: returns SY_ERR_NONFINITE when
 * the result is not finite.  has_grad == 0 leaves everything untouched. */
SY_API sy_status sy_cuda_sgd_update(int32_t device, float *weight, float *velocity, float *grad, int64_t count, float lr,
                             float momentum, float weight_decay, int32_t images, int32_t has_grad);

#ifdef __cplusplus
}
#endif
#endif
