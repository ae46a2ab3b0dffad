// Host-side launch interface of the sm_100a kernels.  All pointers are device pointers; all
// activations use the padded channels-last layout described in common.cuh (sy::Grid).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <stdexcept>
#include <string>

#include "common.cuh"

namespace sy {

// Raises when the most recent kernel launch on this thread failed (bad configuration, etc.).
// Every launch site calls it once, so it also counts this library's kernel launches.
void launch_check(const char* what);

// Per-device one-time set-up (kernel attributes, which CUDA keeps per device): `setup` runs the first
// time `once` is used while a given device is current.  The lock is held across the check, the set-up
// and the record, so a second host thread on the same device waits until the attributes are in place;
// a set-up that throws is not recorded and runs again on the next call.  Device ordinals of 64 and
// above run `setup` every time.
struct PerDeviceOnce {
    std::mutex mu;
    uint64_t done = 0;
};
template <class F>
void once_per_device(PerDeviceOnce& once, F&& setup) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    const uint64_t bit = (dev >= 0 && dev < 64) ? (1ull << dev) : 0;
    std::lock_guard<std::mutex> lock(once.mu);
    if (bit && (once.done & bit)) return;
    setup();
    once.done |= bit;
}
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) that raises on failure.
template <class K>
void set_max_dynamic_smem(K* kernel, int bytes, const char* what) {
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
long long launch_count();
// Kernels run by a CUDA graph replay (counted once at capture, so replays add their node count).
void add_launches(long long n);

// ---------------------------------------------------------------- tensor views
// A channels-last activation view: `base` points at channel 0 of the view in row 0,
// `pitch` floats between consecutive rows, `channels` channels visible, `rows` total rows.
struct View {
    float* base;
    int pitch;
    int channels;
    long rows;
};

// ---------------------------------------------------------------- convolution (tcgen05)
// Implicit-GEMM convolution over the padded layout, stride 1, k in {1,3}:
//   out[m, n] = epilogue( sum_t sum_c in[m + shift[t], c] * wk[n, t * kpad + c] )
// wk is K-major [n_rows][taps * kpad] (kpad = round_up(in.channels, 32)).  Used for forward
// convs (weights in [oc][tap][ic] order) and for data gradients (weights [ic][tap][oc] with
// negated shifts).  Halo / dead rows of `out` are written as zero.
// BatchNorm hooks of the epilogue (per-image training BatchNorm of the next / previous layer).
// Statistics are reduced per 32-row group (a group never spans two images, rows per image being a
// multiple of 128) and folded per (image, channel) in row-group order by bn_stats_fold /
// bn_backward_fold.
struct BnEpilogue {
    int channels = 0;                 // BN channels (stride of the partial and coefficient arrays)
    // forward: part[(group * channels + ch) * 3 + {0,1,2}] = (count, mean, M2) of the conv output
    float* stats_part = nullptr;
    // backward: the conv output is g = dL/da with a = SiLU(gamma * (y - mean) * inv + beta); the
    // epilogue stores dz = dL/dz instead and part[(group * channels + ch) * 2 + {0,1}] =
    // (sum dz, sum dz * xhat) over the group's interior rows.
    const float* y = nullptr;
    int y_pitch = 0;
    const float* mean = nullptr;      // [images][channels]
    const float* inv = nullptr;       // [images][channels] 1 / sqrt(var + eps)
    const float* gamma = nullptr;
    const float* beta = nullptr;
    float* grad_part = nullptr;
};

struct ConvEpilogue {
    const float* bias = nullptr;      // per output channel
    int silu = 0;
    const float* residual = nullptr;  // added after SiLU (Bottleneck shortcut)
    int res_pitch = 0;
    int mask_halo = 1;                // 0: every row is a valid output (plain GEMM use)
    const float* pre = nullptr;       // added to the accumulator before anything else (3xTF32 passes)
    int pre_pitch = 0;
    int round_tf32 = 0;               // store outputs rounded to the nearest TF32 (operands of a TF32 conv)
    BnEpilogue bn{};
};

// Parity-split copy of a feature map, the input format of a 3x3 stride-2 conv.  Padded pixel
// (py, px) of an H x W map (H, W even) goes to plane (py & 1) * 2 + (px & 1), cell (py / 2, px / 2),
// laid out like the consumer's (H/2 x W/2) padded output grid: plane q, image b, cell (sy, sx) is row
// q * plane_rows + b * consumer.rows + sy * consumer.wp + sx.  With this layout every tap of the
// stride-2 conv is a constant row offset, so it runs on the same implicit-GEMM kernel.
struct PhaseOut {
    float* base = nullptr;   // plane 0, row 0, first channel of this view
    int pitch = 0;
    Grid consumer{};         // output grid of the stride-2 consumer
    long plane_rows = 0;     // rows per plane (max batch * consumer.rows)
};

// shift_sign = +1 for a forward conv, -1 for the data gradient (taps read dy at m - shift[t]).
// `phase` (optional) also writes the parity-split copy of the output.
void conv_tc_forward(const View& in, const float* wk, int n_rows, int n_out, int taps, int shift_sign,
                     const Grid& grid, const View& out, const ConvEpilogue& ep, int* err, cudaStream_t stream,
                     const PhaseOut* phase = nullptr);
// 3x3 stride-2 conv on tensor cores: phase_in holds 4 planes of plane_rows rows (PhaseOut layout),
// m_rows = images * gout.rows output rows are computed.
void conv_tc_strided(const View& phase_in, long plane_rows, long m_rows, const float* wk, int oc, const Grid& gout,
                     const View& out, const ConvEpilogue& ep, int* err, cudaStream_t stream,
                     const PhaseOut* phase = nullptr);

// Centred weight gradient of a conv that reads the frozen features (the first conv of every head
// branch).  Those features carry a large per-(image, channel) mean against a BatchNorm gradient dy whose
// per-(image, channel) sum vanishes, so sum_m x dy cancels heavily and the tensor core's FP32
// accumulation loses accuracy in proportion.  With xc = x - mean at interior rows (0 at halo rows) the
// identity
//   sum_m x[m + s] dy[m] = sum_m xc[m + s] dy[m] + mean * T[s],  T[s] = sum of dy[m] over the interior m
//                                                                 whose tap source m + s is interior
// moves the mean into a small exact correction: conv_tc_wgrad runs on xc, the reduce adds
// sum_b mean[b][c] T[b][t][o].
struct WgradCenter {
    const float* mean = nullptr;   // [batch][ic]
    const float* tsum = nullptr;   // [batch][taps][oc]
    int batch = 0;
};
// mean[b][c] over the interior pixels of image b; xc = x - mean at interior rows, 0 at halo / tail rows
// (rounded to the nearest TF32 when round_tf32).  Any per-(image, channel) constant makes the identity
// exact; the mean makes xc small.  ws: center_workspace_floats(batch, channels) floats.
size_t center_workspace_floats(int batch, int channels);
void center_features(const View& x, int batch, const Grid& g, float* mean, float* ws, const View& xc, bool round_tf32,
                     cudaStream_t stream);
// T[b][t][o] of the identity above for dy (taps 1 or 9) from the four edge strips and corners of every
// (image, channel) and the sum over all interior pixels, which is taken as exactly 0 with zero_total (dy
// is the gradient of a conv followed by a per-image BatchNorm, whose backward sums to zero over the pixels
// of each (image, channel)).  ws: center_workspace_floats(batch, dy channels) floats.
void tap_border_sums(const View& dy, int batch, const Grid& g, int taps, bool zero_total, float* ws, float* tsum,
                     cudaStream_t stream);

// Weight gradient: dw[o, c, t] = sum_m dy[m, o] * x[m + shift[t], c], written to `dw` in OIHW order
// (dw[(o * ic + c) * taps + t]), fully overwritten.  `ws` is scratch of wgrad_workspace_floats() floats.
size_t wgrad_workspace_floats(int ic, int oc, int taps, long rows);
void conv_tc_wgrad(const View& x, const View& dy, int taps, const Grid& grid, float* dw, float* ws, int* err,
                   cudaStream_t stream, int accumulate = 0,   // accumulate: dw += instead of dw =
                   const WgradCenter* center = nullptr);      // x is centred: the reduce adds the correction
// 3xTF32 operand split of a view's channels: big = x rounded to TF32 (nearest, ties away), small =
// x - big (exact); both written with the view's pitch at the same row / channel positions.
void tf32_split(const View& src, float* big, float* small, cudaStream_t stream);

// ---------------------------------------------------------------- depthwise convolution (dwconv.cu)
// groups = channels (YOLO11 DWConv), k in {1, 3} (taps 1 or 9), FP32 on CUDA cores.  w: [c][taps].
// y[m] = sum_t w[c][t] x[m + shift_sign * shift_t] at interior rows, 0 elsewhere; shift_sign -1 is the
// data gradient.  `bn` as for the tensor-core epilogue: forward statistics partials, or the BatchNorm
// backward of the layer whose gradient this pass produces (y then receives dz).
// Optional per-channel `bias` and `residual` (same rows; may be y itself) are added after the sum.
// round_tf32: store y rounded to the nearest TF32 (when y feeds a TF32 tensor-core conv).
void dw_conv(const View& x, const float* w, int taps, int shift_sign, const Grid& g, const View& y, const BnEpilogue& bn,
             cudaStream_t stream, const float* bias = nullptr, const View* residual = nullptr, bool round_tf32 = false);
// Multi-head self-attention of the YOLO11 C2PSA block over the interior pixels of each image
// (PtModel.cs Attention, :429-439): qkv holds per head [q key_dim | k key_dim | v head_dim] channels;
// att[token][h * head_dim + d] = sum_j softmax_j(q_i . k_j * scale) v_j[d]; v_out receives v in that
// same channel order (the input of the positional depthwise conv).  key_dim 32, head_dim 64.
void attention(const View& qkv, int batch, const Grid& g, int heads, int key_dim, int head_dim, float scale,
               const View& att, const View& v_out, cudaStream_t stream);
// dw[c][t] = sum over rows of dy[m][c] * x[m + shift_t][c], overwritten; ws: dw_wgrad_workspace_floats.
size_t dw_wgrad_workspace_floats(int c, int taps, long rows);
void dw_wgrad(const View& x, const View& dy, int taps, const Grid& g, float* dw, float* ws, cudaStream_t stream);

// ---------------------------------------------------------------- layout helpers (layout.cu)
// round_tf32 (here and below): values stored rounded to the nearest TF32, for a TF32 tensor-core consumer.
void nchw_to_padded(const float* src, int batch, int c, const Grid& g, const View& dst, cudaStream_t stream,
                    bool round_tf32 = false);
void padded_to_nchw(const View& src, int batch, int c, const Grid& g, float* dst, cudaStream_t stream);
void rgb_to_padded(const uint8_t* rgb, int batch, int size, const Grid& g, const View& dst, cudaStream_t stream);
// Letterboxed RGB24 (identity scale, value / 255) written as the parity-split input of the stem.
void rgb_to_phase(const uint8_t* rgb, int batch, int size, const PhaseOut& dst, cudaStream_t stream);
// Stem of the trunk straight from RGB24: 3x3 stride-2 conv, 3 -> oc (<= 64) channels, folded-BN bias
// and SiLU, on CUDA cores (27 MACs per output channel is too narrow for the tensor cores).  Writes the
// padded output (skipped when out.base is null) and, when `phase` is given, its parity-split copy.
// w_host / bias_host: HOST copies, OIHW [oc][3][3][3] (they travel as kernel parameters).  rgb_ref: DEVICE
// memory holding the address of the device images (read by the kernel, so a captured launch serves any buffer).
void stem_conv(const uint8_t* const* rgb_ref, int batch, int size, const float* w_host, const float* bias_host, int oc,
               const View& out, const Grid& gout, const PhaseOut* phase, cudaStream_t stream, bool round_tf32 = false);
// Grouped conv weights [oc][ic / groups][taps] to block-diagonal dense [oc][ic][taps] (zeros between the
// groups), and the diagonal blocks of a dense [oc][ic][taps] weight gradient back to the grouped layout.
void grouped_to_dense(const float* w, int oc, int ic, int groups, int taps, float* dense, cudaStream_t stream);
void dense_to_grouped(const float* dense, int oc, int ic, int groups, int taps, float* w, cudaStream_t stream);
// OIHW -> [oc][t][kpad] (forward) and OIHW -> [ic][t][kpad_o] (data gradient)
void weights_fwd_layout(const float* oihw, int oc, int ic, int taps, int kpad, float* dst, cudaStream_t stream,
                        bool round_tf32 = false);
void weights_dgrad_layout(const float* oihw, int oc, int ic, int taps, int kpad_o, float* dst, cudaStream_t stream);
// Both layouts of many conv weights in one launch: table[i] describes weight tensor i (device array).
struct WeightLayoutJob {
    const float* oihw;
    int oc, ic, taps, kpad_in, kpad_out;
    float* fwd;     // [oc][taps][kpad_in]
    float* dgrad;   // [ic][taps][kpad_out]
};
void weights_layout_batch(const WeightLayoutJob* table_device, int jobs, long max_elems, cudaStream_t stream,
                          bool round_tf32 = false);

// One CTA that allocates TMEM, waits on an mbarrier nothing arrives on, gives up after `spins` polls,
// writes `code` to *err, frees the TMEM and exits: exercises the bounded-wait path of the pipelined
// kernels without anything asynchronous in flight.  spins in [1, kSpinLimit].
void wait_limit_selftest(uint32_t spins, int code, int* err, cudaStream_t stream);

// ---------------------------------------------------------------- backbone helpers
void maxpool5_padded(const View& in, const View& out, int batch, const Grid& g, cudaStream_t stream);
void upsample2_padded(const View& in, const Grid& gin, const View& out, const Grid& gout, int batch,
                      cudaStream_t stream);

// ---------------------------------------------------------------- BatchNorm (training, per image)
// Floats of the per-32-row-group partials the conv epilogue writes for `channels` channels.
size_t bn_partial_floats(int batch, const Grid& g, int channels);
// Fold the epilogue's (count, mean, M2) partials of every (image, channel) in row-group order
// (Chan's pairwise update, in double): stats[(b * c + ch) * 2 + {0,1}] = (mean, biased variance),
// coef = [mean plane | inv plane], each [batch][c], inv = 1 / sqrt(var + eps).
void bn_stats_fold(const float* part, int batch, const Grid& g, int c, float eps, float* stats, float* coef,
                   cudaStream_t stream);
// Evaluation-mode coefficients: the same [mean plane | inv plane] from the running statistics.
void bn_eval_coef(const float* rmean, const float* rvar, float eps, int batch, int c, float* coef,
                  cudaStream_t stream);
// a = SiLU(gamma * (y - mean) * inv + beta) at interior rows, 0 elsewhere (xhat is not stored).
void bn_silu_apply(const View& y, const float* coef, const float* gamma, const float* beta, int batch, const Grid& g,
                   const View& a, cudaStream_t stream, bool round_tf32 = false);
// Fold the epilogue's (sum dz, sum dz xhat) partials per (image, channel) over the row groups in order;
// dgamma / dbeta are accumulated over images in image order.  bcoef (3 x batch x c floats) receives
// [f plane | red], f = gamma inv / n, red[(b * c + ch) * 2 + {0,1}] = (sum dz, sum dz xhat).
void bn_backward_fold(const float* part, int batch, const Grid& g, int c, const float* coef, const float* gamma,
                      float* dgamma, float* dbeta, float* bcoef, cudaStream_t stream, bool param_grad = true);
// dy = f (n dz - sum dz - xhat sum dz xhat)  (HeadOperations.cs:185-189) at interior rows, 0 elsewhere.
void bn_backward_apply(const View& y, const View& dz, const float* coef, const float* bcoef, int batch, const Grid& g,
                       const View& dy, cudaStream_t stream, bool round_tf32 = false);
// Running statistics: for each BN channel, r <- (1-m) r + m * s_i for images i in order, over
// `ranks` blocks of `batch` images each `rank_stride` floats apart (all-gathered ranks).
// One BatchNorm layer of a batched fold (device table): statistics at `stats_off` floats into the
// statistics block, running buffers, and the backward sums / parameter gradients.
struct BnFoldJob {
    long stats_off;
    int c, spatial;
    float *rmean, *rvar, *tracked;
    const float* bcoef; // bn_backward_fold's output: [f plane (batch x c) | (sum dz, sum dz xhat) pairs]
    float *dgamma, *dbeta;
};
void bn_running_update_batch(const BnFoldJob* jobs, int njobs, int max_c, const float* stats, long rank_stride,
                             int ranks, int batch, float momentum, cudaStream_t stream);
void bn_param_grad_batch(const BnFoldJob* jobs, int njobs, int max_c, int batch, cudaStream_t stream);
void bn_running_update(const float* stats, long rank_stride, int ranks, int batch, int c, int spatial, float momentum,
                       float* rmean, float* rvar, float* tracked, cudaStream_t stream);

// ---------------------------------------------------------------- loss / assigner
struct LevelIO {
    const float* box;   // [rows][pitch] raw DFL logits (4 * bins channels)
    const float* cls;   // [rows][pitch] raw class logits
    float* dbox;        // gradients (same layout), may be null when !backward
    float* dcls;
    int box_pitch, cls_pitch;
    Grid grid;
    float stride;
    // optional (backward only): bias gradients of the convs that produce box / cls, accumulated (+=) here
    // as the loss writes their output gradients: per image the sum over its anchors, images added in order
    float* box_bias_grad = nullptr;
    float* cls_bias_grad = nullptr;
};
struct TruthBox {
    int cls;
    float x1, y1, x2, y2;
};
// Per image loss outputs: loss[b * 4 + {0,1,2}] = (box, cls, dfl), positives[b], connected[b].
struct LossOut {
    float* loss;
    int* positives;
    int* connected;
    int* assigned;     // [batch][anchors] (may be null)
    float* scores;     // [batch][anchors] (may be null)
    // [batch] (may be null): decisions of the assigner taken by a margin of at most kNearTieUlps ulp, i.e.
    // GT boxes whose top-k boundary (k-th against (k+1)-th alignment metric) and conflicted anchors whose
    // best and second overlap lie that close; another libm's exp / atan / pow could decide them the other way
    int* near_ties = nullptr;
};
constexpr unsigned kNearTieUlps = 16;
size_t loss_workspace_bytes(int batch, int anchors, int max_boxes, int topk, int nc);
// round_grad: the logit gradients are stored rounded to the nearest TF32 (operands of TF32 convs).
// serial_cls: the per-image class loss is the reference's float running sum (one term at a time, in its
// order) instead of the exact sum of the same terms (about 1e-3 apart at 640 x 640).
// Class part on a second stream: with `split`, the class-logit BCE, its bias-gradient fold and the per-image
// loss totals run on split->cls_stream once the assignment is done (event `assigned`), while `stream` goes on
// with the box terms and their gradients and records `box`; `cls_done` is recorded on cls_stream after the
// totals.  The caller orders later work on these events.
struct LossSplit {
    cudaStream_t cls_stream;
    cudaEvent_t assigned, box, cls_done;
};
void detection_loss(const LevelIO* levels, int nlevels, int batch, int nc, int bins, const TruthBox* truth,
                    const int* box_offsets, int max_boxes, int topk, int topk2, float grad_scale, int backward, void* workspace,
                    const LossOut& out, cudaStream_t stream, bool round_grad = false, bool serial_cls = false,
                    const LossSplit* split = nullptr);

// ---------------------------------------------------------------- inference post-processing (detect.cu)
constexpr int kMaxDetectLevels = 8;
constexpr int kMaxEndToEndTopk = 1024;
// One level of raw head outputs: element (image, channel, row, column) of the box (4 * bins channels) and
// class (nc channels) logits at base + the dot product of the index with the strides (in floats).
struct DetectLevelSrc {
    const float* box;
    const float* cls;
    long box_s[4];
    long cls_s[4];
    int h, w;
    float stride;
};
// Letterbox record (model pixels -> source pixels), pads and sizes converted to float.
struct DetectTransform {
    float scale_x, scale_y, pad_x, pad_y, source_w, source_h;
};
struct DetectOptions {
    float confidence, iou;
    int max_det, max_candidates, agnostic;
};
struct DetOut {   // same layout as sy_detection
    int class_id;
    float confidence, x, y, width, height;
};
// CpuHead.DecodeInto over the joined levels: out [batch][4 + nc][anchors]; xyxy for end-to-end heads.
void head_decode(const DetectLevelSrc* levels, int nlevels, int batch, int bins, int nc, int xyxy, float* out,
                 cudaStream_t stream);
// PtModel.EndToEndTopK: x [batch][fields][anchors] -> out [batch][min(k, anchors)][6 + fields - nc - 4];
// k <= kMaxEndToEndTopk, anchors * nc < 2^32.
size_t end_to_end_workspace_bytes(int batch, int anchors, int nc, int k);
void end_to_end_topk(const float* x, int batch, int fields, int anchors, int nc, int k, float* out, void* ws,
                     cudaStream_t stream);
// YoloDetector.DecodeIndexed per image: value (anchor a, field f) of image b at
// x[b * img_stride + a * a_stride + f * f_stride]; class_fields = 4 + classes (raw heads) or unused (e2e:
// fields x1, y1, x2, y2, score, class).  out [batch][o.max_det], counts [batch]; *err = 1 when an end-to-end
// class id exceeds Int32.  tf [batch] on the device.
size_t detections_workspace_bytes(int batch, int count, int max_det);
// The same candidates and NMS straight from raw head outputs in channels-last rows (levels[l].box / .cls with
// channel stride 1, 16-byte aligned rows of box_pitch / cls_pitch floats): CpuHead.DecodeInto's scores and
// boxes fused with DecodeIndexed (raw, non-end-to-end heads); workspace detections_workspace_bytes(batch,
// anchors, o.max_det).
void detect_raw(const DetectLevelSrc* levels, int nlevels, int batch, int bins, int nc, int cls_pitch, int box_pitch,
                const DetectTransform* tf, const DetectOptions& o, DetOut* out, int* counts, void* ws,
                cudaStream_t stream);
void decode_detections(const float* x, int batch, long img_stride, long a_stride, long f_stride, int count,
                       int class_fields, bool e2e, const DetectTransform* tf, const DetectOptions& o, DetOut* out,
                       int* counts, int* err, void* ws, cudaStream_t stream);

// ---------------------------------------------------------------- optimizer
struct ParamSegment {
    long offset, length;
    int decay;     // conv weights
    int group;     // 0: always connected, 1: box branch (skipped when no image connected it)
};
// SGD-momentum (TrainingParameter.Update) or AdamW over segments; flags[g] gates group g.
// Reports non-finite values through *nonfinite.  Gradients are zeroed after the update.
void optimizer_step(int optimizer, float* params, float* vel, float* vel2, float* grad, const ParamSegment* segs,
                    int nsegs, const int* group_has_grad, const int* group_steps, float lr, float momentum, float wd,
                    float beta1, float beta2, float adam_eps, float inv_images, int* nonfinite, cudaStream_t stream);
void check_finite(const float* v, long n, int* flag, cudaStream_t stream);
// part[kAbsSumBlocks] = block partial sums of |v| (fixed order, summed on the host)
constexpr int kAbsSumBlocks = 64;
void abs_sum_partials(const float* v, long n, double* part, cudaStream_t stream);

}  // namespace sy
