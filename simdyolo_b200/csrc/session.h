// Training session: owns the device state of one data-parallel rank and runs the fine-tuning step
// (YoloTrainer.Train inner loop, src/SimdYolo.Training/YoloTrainer.cs:185-199) on the GPU.
#pragma once
#include <array>
#include <map>
#include <tuple>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/simdyolo_cuda.h"
#include "kernels.h"

namespace sy {

// Error carrying an sy_status code; thrown inside the library, converted at the C ABI.
struct SyError : std::runtime_error {
    int code;
    SyError(int c, const std::string& m) : std::runtime_error(m), code(c) {}
};

// Records `message` as the process-wide last error returned by sy_cuda_last_error(NULL).
void set_last_error(const std::string& message);

struct TensorEntry {
    std::string name;
    int kind;            // 0 parameter, 1 buffer
    std::vector<int> shape;
    long offset;         // in params (kind 0) or buffers (kind 1)
    long numel;
    int group;           // parameters: 0 always connected, 1 box branch
    int decay;
};

struct HeadBlock {
    sy_block b;
    int taps;
    bool dw = false;            // depthwise (groups = channels): CUDA-core kernels, weights [c][taps]
    // other group counts: the tensor-core conv with block-diagonal dense weights (zeros between the groups);
    // the weight gradient is computed dense and its diagonal blocks are the parameter gradient
    bool grouped = false;
    float* w_dense = nullptr;   // [oc][ic][taps], refreshed from the [oc][ic / groups][taps] parameters
    float* wg_dense = nullptr;  // dense weight gradient [oc][ic][taps]
    long w_off = -1, b_off = -1, g_off = -1, be_off = -1;
    long rm_off = -1, rv_off = -1, nt_off = -1;
    float* w_fwd = nullptr;     // [oc][taps][kpad_in]
    float* w_dgrad = nullptr;   // [ic][taps][kpad_out]
    int kpad_in = 0, kpad_out = 0;
    View x{}, y{}, a{}, g{}, dy{};
    float* stats = nullptr;     // [B][oc][2] inside the session's contiguous statistics block
    long stats_off = 0;         // channel offset of this layer in that block
    float* coef = nullptr;      // [mean plane | inv plane], each [B][oc]
    float* bcoef = nullptr;     // backward: [f plane | (sum dz, sum dz xhat) per (image, channel)]
};

struct Branch {
    int level;
    bool box;
    int set = 0;                // 0 one-to-many (cv2 / cv3), 1 one-to-one (one2one_cv2 / one2one_cv3)
    int group = 0;              // optimizer group: 0 class branches, 1 cv2, 2 one2one_cv2
    std::vector<HeadBlock> blocks;
};

struct BackboneOp {
    int type;                   // 0 conv, 1 maxpool5, 2 upsample2, 3 depthwise conv, 4 attention
    int ic = 0, oc = 0, k = 0, stride = 1;
    int act = 1;                // conv: SiLU (1) or none (0, the YOLO11 attention's convs)
    View aux{};                 // attention: v in head-major channel order (input of the depthwise conv)
    int heads = 0;              // attention
    long w_off = 0, b_off = 0;
    float* wk = nullptr;        // K-major [oc][tap][round_up(ic, 32)]
    View in{}, out{}, res{};
    Grid gin{}, gout{};
    bool has_res = false;
    View phase_in{};            // stride 2: parity-split input (4 planes)
    long phase_plane_rows = 0;
    bool has_phase_out = false; // this conv's output feeds a stride-2 conv
    PhaseOut phase_out{};
    bool plain_out = true;      // false: only stride-2 convs read the output, so only the copy is written
};

struct NcclApi;

class Session {
public:
    explicit Session(const sy_config& cfg);
    ~Session();

    sy_config cfg;
    std::string error;

    // public operations (return sy_status)
    // rgb: host (or, with rgb_on_device, device) images; features: host NCHW features instead.
    int step(const uint8_t* rgb, bool rgb_on_device, const float* const* features, const sy_box* boxes,
             const int32_t* counts, int images, sy_step_stats* out);
    // YoloTrainer.EvaluateLoss: BatchNorm with running statistics, loss without gradients, no update.
    int evaluate(const uint8_t* rgb, bool rgb_on_device, const float* const* features, const sy_box* boxes,
                 const int32_t* counts, int images, sy_step_stats* out);
    // Inference (YoloDetector.Detect on this model, src/SimdYolo/YoloDetector.cs:327-376): frozen trunk, head
    // with BatchNorm in evaluation mode, decode, confidence filter, greedy NMS (none for end-to-end heads,
    // which take PtModel.EndToEndTopK instead) and letterbox mapping.  out [images][max_detections].
    // timing (optional): [0] device ms of the call (inputs up to the detections read back), [1] device ms of
    // the post-processing kernels (decode, top-k, candidates and NMS).
    int detect(const uint8_t* rgb, bool rgb_on_device, const float* const* features, int images,
               const sy_letterbox* transforms, const sy_detect_options* options, sy_detection* out, int32_t* counts,
               double* timing = nullptr);
    // Starts the host-to-device copy of a batch of RGB24 images on the copy stream; a later step / evaluate
    // / detect with the same host pointer and image count takes the copy instead of copying again.
    int prefetch_images(const uint8_t* rgb, int images);
    int set_epoch(int epoch);
    // AdamW steps taken per optimizer group (class branches, cv2, one2one_cv2)
    int get_optimizer_steps(int32_t steps[3]) const;
    int set_optimizer_steps(const int32_t steps[3]);
    int set_tensor(int index, const float* host, long count);
    int get_tensor(int index, float* host, long count) const;
    int set_opt_state(int index, int moment, const float* host, long count);
    int get_opt_state(int index, int moment, float* host, long count) const;
    int set_backbone(const float* host, long count);
    int get_last_gradients(float* host, long count) const;
    int get_last_features(int level, float* host, long count) const;
    // raw outputs (box and class logits, NCHW) of branch set `set` at `level` from the latest head forward
    int get_last_head_outputs(int set, int level, float* box, long box_count, float* cls, long cls_count) const;
    // Optional CUDA-event timing of every tensor-core convolution launch (forward, stride-2 and
    // data-gradient passes) on the session stream; returns the totals since the previous call.
    int conv_profile(int enable, double* ms, double* gflop, long* launches);
    // Per-launch (ms, GFLOP, shape) of the most recent profiled step, in launch order; shape =
    // (pass, input channels, output channels, taps, output height, output width) with pass 0 trunk
    // stride 1, 1 trunk stride 2, 2 head forward, 3 head data gradient.
    int conv_profile_launches(double* ms, double* gflop, int* shapes, int capacity, int* count) const;

    std::vector<TensorEntry> tensors;
    long n_params = 0, n_buffers = 0, n_backbone = 0;

private:
    void build_backbone();
    void build_trunk_v8();
    void build_trunk_11();
    // trunk builders shared by both families (parameters are taken in call order)
    void tk_conv(const View& in, const Grid& gin, int oc, int k, int s, const View& out, const Grid& gout,
                 const View* res, int act = 1);
    void tk_sppf(const View& in, const Grid& g, int c2, const View& out);
    void tk_upsample(const View& in, const Grid& gin, const View& out, const Grid& gout);
    long tk_poff_ = 0;
    void build_head();
    void forward_backbone(int batch);   // stem input: the images at *d_rgb_ref_
    void prepare_inputs(const uint8_t* rgb, bool rgb_on_device, const float* const* features, const sy_box* boxes,
                        const int32_t* counts, int images, bool defer_backbone = false);
    void forward_head(int batch, bool training = true);
    // DetectionHead.Loss: one loss per branch set, gradients scaled by the set's weight
    void launch_losses(int images, int backward, int epoch);
    void loss_weights(int epoch, float w[2]) const;
    // per-image weighted loss parts of one rank's exchange-record head, accumulated into the outputs
    void combine_losses(const float* head, int images, int epoch, double* box, double* cls, double* dfl,
                        long* positives, int* connected, bool* finite, long* near_ties) const;
    // host wait for the stream, bounded by comm_timeout_ms while collectives are in flight
    void wait_stream(const char* what);
    [[noreturn]] void abort_comm(const std::string& reason);
    void backward_head(int batch);
    // The head's three pyramid levels are independent between the trunk and the loss (forward) and between
    // the loss and the parameter-gradient fold (backward): in TF32 mode, unprofiled, each level runs on its
    // own stream with its own BatchNorm-partial, weight-gradient and centring scratch, forked from and joined back to
    // stream_ (inside the step's CUDA graph as well), so the small levels fill the SMs the large one leaves.
    struct LevelLane {
        cudaStream_t stream = nullptr;   // lane 0 is stream_
        float* bn_part = nullptr;
        float* wgrad_ws = nullptr;
        cudaEvent_t done = nullptr;
        float* tap_sums = nullptr;    // the first convs' centred weight gradient (tap_border_sums)
        float* center_ws = nullptr;
    };
    LevelLane lanes_[3];
    cudaEvent_t ev_fork_ = nullptr;
    // In the forward pass level l runs on lane (l + 1) % 3's stream (level 2, which needs the whole trunk,
    // stays on stream_), and when the trunk ran just before, levels 0 and 1 start as soon as the trunk op
    // that finishes their feature map has (ev_feat_), overlapping the trunk's remaining bottom-up layers.
    int feat_op_[3] = {-1, -1, -1};   // index in bops_ of the last op writing features_[l]
    cudaEvent_t ev_feat_[2] = {nullptr, nullptr};
    bool feat_events_ = false;        // ev_feat_ recorded by the trunk pass the next forward_head follows
    // The loss's class part (BCE, class-bias fold, per-image totals) runs on loss_stream_ beside its box part;
    // the backward starts the box branches after the box part and each level's class branches after
    // ev_cls_ (cls_pending_: the last launch_losses left that wait to the backward).
    cudaStream_t loss_stream_ = nullptr;
    cudaEvent_t ev_assigned_ = nullptr, ev_box_ = nullptr, ev_cls_ = nullptr;
    bool cls_pending_ = false;
    bool level_lanes() const { return lanes_[1].stream != nullptr && !x3_ && !prof_; }
    void fork_levels();
    void join_levels();
    void use_lane(int l, int stream_lane = -1);
    void refresh_head_weights();
    BnFoldJob* d_bn_jobs_ = nullptr;             // one job per head BatchNorm layer
    int n_bn_jobs_ = 0, bn_max_c_ = 0;
    WeightLayoutJob* d_layout_jobs_ = nullptr;   // one job per tensor-core head conv
    int n_layout_jobs_ = 0;
    long layout_max_elems_ = 0;
    View alloc_view(int channels, const Grid& g);
    // tensor-core convolutions, in TF32 or (precision 3xTF32) as three split-operand passes
    void conv_fwd(const View& in, const float* wk, long wk_floats, int n_rows, int n_out, int taps, int sign,
                  const Grid& grid, const View& out, const ConvEpilogue& ep, const PhaseOut* po);
    void conv_strided(const View& phase_in, long plane_rows, long m_rows, const float* wk, long wk_floats, int oc,
                      const Grid& gout, const View& out, const ConvEpilogue& ep, const PhaseOut* po);
    void conv_wgrad(const View& x, const View& dy, int taps, const Grid& grid, float* dw,
                    const WgradCenter* center = nullptr);
    View split_view(const View& v, int slot_big, View* small);
    const float* split_weights(const float* wk, long n, const float** small);
    void* dalloc(size_t bytes);

    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
    std::vector<void*> allocations_;
    int B_ = 0;
    Grid levels_[3];
    int feat_ch_[3] = {0, 0, 0};
    View features_[3];
    // 3xTF32 parity mode: centred copies of the features for the first head convs' weight gradients
    // (WgradCenter): xc = features - per-(image, channel) mean, the means, and the tap border sums of one
    // dy.  In TF32 the operand rounding, not the accumulation, sets the error, so TF32 runs without them.
    View feat_c_[3];
    float* feat_mean_[3] = {nullptr, nullptr, nullptr};
    float* tap_sums_ = nullptr;
    float* center_ws_ = nullptr;
    // backbone
    std::vector<BackboneOp> bops_;
    float* backbone_params_ = nullptr;
    std::vector<float> stem_host_;   // stem weights then bias (OIHW), host copy for the kernel parameters
    uint8_t* d_rgb_ = nullptr;
    uint8_t* h_rgb_ = nullptr;   // pinned staging
    View img_{};
    Grid img_grid_{};
    bool backbone_ready_ = false;
    // head
    std::vector<Branch> branches_;
    float* params_ = nullptr;
    float* grads_ = nullptr;
    float* last_grads_ = nullptr;
    float* vel_ = nullptr;
    float* vel2_ = nullptr;
    float* buffers_ = nullptr;
    float* wgrad_ws_ = nullptr;
    float* feat_stage_ = nullptr;
    float* bn_stats_all_ = nullptr;
    long bn_channels_ = 0;
    float* bn_part_ = nullptr;       // per-32-row-group BatchNorm partials written by conv epilogues
    void* loss_ws_ = nullptr;
    TruthBox* d_truth_ = nullptr;
    int* d_box_off_ = nullptr;
    TruthBox* h_truth_ = nullptr;
    int* h_box_off_ = nullptr;
    // exchange record (see build_head): head of loss parts / positives / connections / image count, then
    // the per-image BatchNorm statistics; its all-gathered copy; the heads on the host
    float* rec_ = nullptr;
    float* rec_gather_ = nullptr;
    long head_floats_ = 0, rec_floats_ = 0;
    float* h_rec_ = nullptr;
    int* h_images_ = nullptr;
    int* d_images_ = nullptr;
    // the current step's device image address, uploaded with the step's other small inputs: the stem reads
    // it from device memory, so one captured graph serves every image buffer
    const uint8_t** h_rgb_ref_ = nullptr;
    const uint8_t** d_rgb_ref_ = nullptr;
    int* d_ties_ = nullptr;
    int comm_timeout_ms_ = 300000;
    float* d_loss_ = nullptr;
    int* d_pos_ = nullptr;
    int* d_conn_ = nullptr;
    int* d_flags_ = nullptr;     // [0] device error, [1] nonfinite, [2..3] group has_grad, [4..5] adam steps
    int* h_flags_ = nullptr;
    double* d_abs_ = nullptr;
    double* h_abs_ = nullptr;
    ParamSegment* d_segs_ = nullptr;
    int nsegs_ = 0;
    int adam_steps_[3] = {0, 0, 0};   // AdamW steps per optimizer group
    int n_sets_ = 1;                  // 2 with the one-to-one branches
    bool progressive_ = false;        // end-to-end with reg_max 1 (TrainingHeadSchema.Progressive)
    int epoch_ = 0;
    // CUDA graphs of the device work of a training step (trunk forward, head forward, losses, head
    // backward), one per (images, image source, loss weights); a key is captured the second time it is
    // seen (the first run is eager and settles every one-time set-up).  Disabled while conv launches are
    // profiled, or with SIMDYOLO_CUDA_GRAPHS=0 in the environment.
    using GraphKey = std::tuple<int, const void*, float, float>;
    std::map<GraphKey, cudaGraphExec_t> graphs_;
    std::map<GraphKey, int> graph_seen_;
    std::map<GraphKey, long long> graph_nodes_;   // kernel launches inside each graph
    bool use_graphs_ = true;
    void clear_graphs();
    int last_batch_ = 0;
    // 3xTF32 operand split scratch: activations (4 buffers) and weights (2 buffers)
    bool x3_ = false;
    // TF32 mode: every tensor-core operand (weights, activations, gradients) is stored rounded to the
    // nearest TF32, so the tensor core's truncation of FP32 operands adds no systematic error
    bool rnd_ = false;
    float* sp_[4] = {nullptr, nullptr, nullptr, nullptr};
    size_t sp_floats_ = 0;
    float* wsp_[2] = {nullptr, nullptr};
    size_t wsp_floats_ = 0;
    // conv launch timing (conv_profile)
    bool prof_ = false;
    std::vector<cudaEvent_t> prof_ev_;
    std::vector<double> prof_flops_;
    int prof_n_ = 0;
    double prof_ms_ = 0.0, prof_gflop_ = 0.0;
    std::vector<double> prof_last_ms_, prof_last_gflop_;
    std::vector<std::array<int, 6>> prof_shape_, prof_last_shape_;
    long prof_launches_ = 0;
    void prof_begin();
    void prof_end(double flops, const std::array<int, 6>& shape);
    void prof_collect();
    NcclApi* nccl_ = nullptr;
    void* comm_ = nullptr;
    // Prefetched image batches: two slots, filled alternately by prefetch_images.  A slot's copy is issued on
    // copy_stream_ by the next call that prepares inputs, and starts after that call's own small uploads have
    // landed: the host-to-device copy engine serves one copy after another, so a large copy that got there
    // first would hold those uploads (and the step behind them) back for its whole length.  `copied` is recorded after a slot's copy, `released`
    // after the device work of the call that consumed it (the next copy into that slot waits for it).
    struct ImageSlot {
        uint8_t* dev = nullptr;
        uint8_t* pinned = nullptr;   // staging for pageable sources
        const uint8_t* host = nullptr;
        const uint8_t* src = nullptr;   // what the copy reads: host, or pinned
        int images = 0;
        bool ready = false, pending = false, used = false;
        cudaEvent_t copied = nullptr, released = nullptr;
    };
    void issue_prefetch(ImageSlot& sl);
    ImageSlot slots_[2];
    int next_slot_ = 0;
    cudaEvent_t ev_uploaded_ = nullptr;   // this call's small uploads, which a prefetch copy must not overtake
    ImageSlot* consuming_ = nullptr;   // slot read by the device work being enqueued
    cudaStream_t copy_stream_ = nullptr;
    void release_images();
    // inference buffers, allocated by the first detect call (the output and workspace grow with
    // max_detections): for end-to-end heads the decoded head [B][4 + nc][anchors] and the rows [B][k][6]
    // (raw heads decode inside the candidate kernel); letterbox records
    void ensure_detect(int max_det);
    int anchors_ = 0;
    float* det_dec_ = nullptr;
    float* det_e2e_ = nullptr;
    DetectTransform* det_tf_ = nullptr;
    int* det_counts_ = nullptr;
    cudaEvent_t ev_post_ = nullptr;     // start of the post-processing kernels
    int* det_err_ = nullptr;
    void* det_ws_ = nullptr;
    DetOut* det_out_ = nullptr;
    int det_cap_ = 0;
};

constexpr int kMaxDetections = 65536;   // max_detections accepted by detect / decode_detections
constexpr int kModelMaxDet = 300;        // max_det of an end-to-end head (PtModel.Detect's default)

// Validated conversions of the public inference records (YoloDetector option and Letterbox checks).
DetectOptions detect_options(const sy_detect_options* o, bool detector);
DetectTransform detect_transform(const sy_letterbox& t);

}  // namespace sy
