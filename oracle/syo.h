/*
 * CPU oracle for the SimdYolo.Training detection-head fine-tuning step.
 *
 * TEST INFRASTRUCTURE ONLY.  This library restates the reference's CPU algorithm in
 * plain C so that the CUDA path can be checked against it.  Only tests/, the smoke
 * check in __graft_entry__.py and bench.py's cpu_baseline leg may load it; the
 * product (simdyolo_b200/) never links, loads or calls it.
 *
 * Reference files restated (paths inside the reference project):
 *   src/SimdYolo.Training/HeadOperations.cs    conv / grouped conv / BatchNorm / SiLU
 *   src/SimdYolo.Training/DetectionLoss.cs     DFL decode, TAL assigner, BCE, CIoU, DFL
 *   src/SimdYolo.Training/TrainingParameter.cs SGD-momentum update, finiteness checks
 *   src/SimdYolo.Training/DetectionHead.cs     branch / block order, ProgressiveWeight
 *   src/SimdYolo.Training/YoloTrainer.cs       per-batch accumulate -> check -> update
 *   src/SimdYolo/PtModel.cs                    frozen backbone layer semantics (BN folded)
 *   src/SimdYolo/YoloDetector.cs               letterbox at identity scale (u8 / 255); DecodeIndexed, Iou
 *   src/SimdYolo/CpuHead.cs                    head decode (DFL expectation, boxes, sigmoid scores)
 *
 * Transcendental functions used by the assigner (exp, atan) come from detmath.c:
 * double-precision evaluations written from published methods, so the CUDA build can
 * reproduce them bit for bit.  The reference calls the platform libm (MathF.Exp /
 * MathF.Atan / MathF.Pow); detmath results are within one float ulp of those.
 */
#ifndef SYO_H
#define SYO_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- deterministic math (detmath.c) ---- */
double syo_exp_d(double x);
float syo_expf(float x);
double syo_atan_d(double x);
float syo_atanf(float x);
float syo_sigmoid(float x);            /* HeadOperations.cs:222 with syo_expf */
float syo_pow6(float x);               /* MathF.Pow(x, 6) restated as a rounded double product */

/* ---- head operations (head_ops.c), one image, NCHW, OIHW ---- */
void syo_conv_forward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                      const float *bias, float *y);
void syo_conv_backward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                       const float *dy, float *dw_acc, float *db_acc, float *dx_acc);
void syo_grouped_conv_forward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                              int groups, const float *bias, float *y);
void syo_grouped_conv_backward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                               int groups, const float *dy, float *dw_acc, float *db_acc, float *dx_acc);
void syo_batchnorm_forward(const float *x, int c, int spatial, const float *gamma, const float *beta,
                           float *rmean, float *rvar, float eps, float momentum, int training,
                           float *y, float *xhat, float *inv, float *batch_mean, float *batch_var);
void syo_batchnorm_backward(const float *dy, const float *xhat, const float *inv, const float *gamma,
                            int c, int spatial, float *dgamma_acc, float *dbeta_acc, float *dx_acc);
void syo_silu_forward(const float *x, int n, float *y, float *sig);
void syo_silu_backward(const float *x, const float *sig, const float *dy, int n, float *dx_acc);
void syo_right_transposed(const float *a, const float *b, float *c, int m, int n, int k);
int syo_all_finite(const float *v, long n);
/* TrainingParameter.Update; returns 0 ok, 1 non-finite (arrays already written, as in the reference) */
int syo_sgd_update(float *w, float *vel, float *grad, long n, float lr, float momentum, float wd,
                   int images, int has_grad);
/* torch.optim.AdamW restated (not in the reference); step is 1-based after increment */
int syo_adamw_update(float *w, float *m, float *v, float *grad, long n, float lr, float beta1,
                     float beta2, float eps, float wd, int step, int images, int has_grad);
float syo_progressive_weight(int epoch, int epochs);

/* ---- detection loss (loss.c), one image ---- */
typedef struct { int32_t cls; float x1, y1, x2, y2; } syo_box;
typedef struct { float box, cls, dfl; int32_t positives; int32_t connected; } syo_loss;

/* DetectionLoss.Compute.  box_levels[l]: [4*bins, H_l, W_l], cls_levels[l]: [nc, H_l, W_l].
 * dbox/dcls may be NULL when backward == 0; gradients are ACCUMULATED.
 * assigned/scores (length A) may be NULL.  Returns 0, or -1 on invalid arguments. */
int syo_detection_loss(const float *const *box_levels, const float *const *cls_levels,
                       const int *hs, const int *ws, const float *strides, int levels, int nc, int bins,
                       const syo_box *truth, int n_truth, int topk, int topk2, float grad_scale,
                       int backward, float *const *dbox_levels, float *const *dcls_levels,
                       syo_loss *out, int32_t *assigned, float *scores);

/* CIoU with forward-mode derivatives (DetectionLoss.cs:171-183). grad[4] may be NULL. */
float syo_ciou(const float p[4], const float t[4], float grad[4]);

/* ---- detection head (step.c) ----
 * Branch description: blocks in execution order.  A block is Conv(+BN+SiLU) or the final Conv2d. */
typedef struct { int32_t ic, oc, k, groups, has_bn, has_bias; } syo_block;

typedef struct {
    int32_t levels;             /* 3 */
    int32_t nc, bins;           /* classes, reg_max */
    int32_t hs[3], ws[3];       /* feature map sizes */
    float strides[3];
    int32_t n_box_blocks, n_cls_blocks;
    syo_block box_blocks[3][8]; /* per level */
    syo_block cls_blocks[3][8];
    float bn_eps, bn_momentum;
    /* TrainingHeadSchema (TrainingHeadSchema.cs:7-12): end_to_end adds one2one_cv2 / one2one_cv3
     * branches built like cv2 / cv3; bins == 1 with end_to_end is the progressive (YOLO26) loss.
     * epoch / schedule_epochs feed DetectionHead.ProgressiveWeight. */
    int32_t end_to_end;
    int32_t epoch, schedule_epochs;
} syo_head_desc;

/* Number of floats in the flat parameter array and in the flat buffer array (Snapshot order:
 * cv2.0, cv2.1, cv2.2, cv3.0, cv3.1, cv3.2, then with end_to_end one2one_cv2.0-2, one2one_cv3.0-2;
 * per block weight, [bias], [gamma, beta]). */
long syo_head_param_count(const syo_head_desc *d);
long syo_head_buffer_count(const syo_head_desc *d);

/* One image: head forward (training BN: running stats updated in place), loss, backward.
 * features[l]: [C_l, H_l, W_l].  grads accumulated into grad (flat, param order).
 * bn_stats (optional) receives per BN channel (mean, biased var) of this image in param order.
 * box_connected: bit 0 set when cv2 was connected for this image, bit 1 when one2one_cv2 was. */
int syo_head_image(const syo_head_desc *d, const float *params, float *buffers,
                   const float *const *features, const syo_box *truth, int n_truth,
                   float *grad, syo_loss *loss, int backward, int *box_connected);

int syo_head_eval_image(const syo_head_desc *d, const float *params, float *buffers, const float *const *features,
                        const syo_box *truth, int n_truth, syo_loss *loss);
/* The head's raw outputs in evaluation mode (BatchNorm with the running statistics), one image: branch set
 * `set` (0 cv2 / cv3, 1 one2one_cv2 / one2one_cv3); box[l] receives [4*bins][H_l][W_l], cls[l] [nc][H_l][W_l]. */
int syo_head_eval_outputs(const syo_head_desc *d, const float *params, const float *buffers,
                          const float *const *features, int set, float *const *box, float *const *cls);

/* ---- frozen backbone (backbone.c): YOLOv8-family detection trunk with folded BN ---- */
typedef struct {
    int32_t image;          /* square input size (multiple of 32) */
    float width_mult, depth_mult;
    int32_t max_channels;
    int32_t family;         /* 0 YOLOv8 (C2f trunk), 1 YOLO11 (C3k2 / SPPF / C2PSA trunk) */
} syo_backbone_desc;
long syo_backbone_param_count(const syo_backbone_desc *d);
void syo_backbone_feature_channels(const syo_backbone_desc *d, int32_t ch[3]);
/* rgb: HWC u8 image of size image x image; features out: NCHW per level */
void syo_backbone_forward(const syo_backbone_desc *d, const float *params, const uint8_t *rgb,
                          float *p3, float *p4, float *p5);

/* ---- detection post-processing (detect.c) ---- */
typedef struct { int32_t class_id; float confidence, x, y, width, height; } syo_detection;      /* Detection */
typedef struct { int32_t source_width, source_height, target_width, target_height;
                 float scale_x, scale_y; int32_t pad_x, pad_y; } syo_letterbox;                 /* Letterbox */
typedef struct { float confidence, iou_threshold; int32_t max_detections, max_candidates, class_agnostic; }
    syo_detect_options;

/* CpuHead.DecodeInto, one level: box [batch][4*bins][h][w], cls [batch][nc][h][w] into
 * out [batch][nc+4][out_anchors] at anchors out_start.. (cx, cy, w, h or x1, y1, x2, y2; sigmoid scores) */
void syo_head_decode(const float *box, const float *cls, int batch, int h, int w, int bins, int nc, float stride,
                     int xyxy, float *out, int out_anchors, int out_start);
/* PtModel.EndToEndTopK: x [batch][fields][anchors] -> out [batch][k][6 + fields - nc - 4]; returns k */
int syo_end_to_end_topk(const float *x, int batch, int fields, int anchors, int nc, int maximum, float *out);
/* YoloDetector.DecodeIndexed for one image; layout 1 channels-first, 2 channels-last, 3 end-to-end.
 * out holds max_detections entries; returns the count, -1 on invalid arguments, -2 when a class id of an
 * end-to-end row exceeds Int32 (the reference's checked conversion throws). */
int syo_decode_detections(const float *output, int dim1, int dim2, int layout, int class_count,
                          const syo_letterbox *t, const syo_detect_options *o, syo_detection *out);
float syo_detection_iou(const syo_detection *a, const syo_detection *b);

/* ---- full optimizer step (step.c) ---- */
typedef struct {
    float lr, momentum, weight_decay;
    int32_t optimizer;     /* 0 SGD, 1 AdamW */
    float beta1, beta2, adam_eps;
    int32_t adam_step[3];  /* AdamW steps already taken: [0] always-connected params, [1] cv2, [2] one2one_cv2 */
} syo_optim;

typedef struct { double box, cls, dfl; int64_t positives; int32_t box_has_grad; int32_t status; } syo_step_result;

/* images: B pointers to image x image RGB24.  truth: concatenated boxes, counts[B].
 * params/buffers/velocity (and adam second moment in velocity2) updated in place.
 * grad_out (optional) receives the summed (not yet divided) head gradient.
 * threads: OpenMP threads over images (0 = all). status: 0 ok, 3 non-finite. */
void syo_train_step(const syo_backbone_desc *bd, const float *backbone_params,
                    const syo_head_desc *hd, float *params, float *buffers, float *velocity,
                    float *velocity2, const syo_optim *opt, const uint8_t *const *images,
                    const syo_box *truth, const int32_t *counts, int batch, int threads,
                    float *grad_out, syo_step_result *result);

#ifdef __cplusplus
}
#endif
#endif
