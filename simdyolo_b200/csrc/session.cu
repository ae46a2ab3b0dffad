// Session: model plan, device buffers and the fine-tuning step.
//
// Step order (one CUDA stream):
//   upload images + boxes -> frozen YOLOv8 trunk (PtModel.Run up to Detect, PtModel.cs:184-203)
//   -> head forward per level, box branch then class branch (DetectionHead.Forward, :89-98)
//   -> DetectionLoss on device -> head backward (reverse block order, GradientTape.Backward)
//   -> finiteness (YoloTrainer.cs:193,196) -> [NCCL all-reduce over ranks]
//   -> BN running statistics in image order -> SGD / AdamW (TrainingParameter.Update)
//   -> refresh the derived weight layouts used by the next step's convs.
#include <dlfcn.h>

#include <algorithm>
#include <functional>
#include <array>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>

#include "session.h"

namespace sy {


#define SY_CUDA(call)                                                                                    \
    do {                                                                                                 \
        cudaError_t e_ = (call);                                                                         \
        if (e_ != cudaSuccess)                                                                           \
            throw SyError(e_ == cudaErrorMemoryAllocation ? SY_ERR_OUT_OF_MEMORY : SY_ERR_DEVICE,        \
                          std::string(#call) + ": " + cudaGetErrorString(e_));                           \
    } while (0)

// ------------------------------------------------------------------ NCCL (loaded at run time)
typedef struct { char internal[128]; } nccl_unique_id_t;
struct NcclApi {
    void* lib = nullptr;
    int (*GetUniqueId)(nccl_unique_id_t*) = nullptr;
    int (*CommInitRank)(void**, int, nccl_unique_id_t, int) = nullptr;
    int (*AllReduce)(const void*, void*, size_t, int, int, void*, cudaStream_t) = nullptr;
    int (*AllGather)(const void*, void*, size_t, int, void*, cudaStream_t) = nullptr;
    int (*CommDestroy)(void*) = nullptr;
    int (*CommAbort)(void*) = nullptr;
    int (*CommGetAsyncError)(void*, int*) = nullptr;
    const char* (*GetErrorString)(int) = nullptr;
    bool load() {
        if (lib) return true;
        lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) return false;
        GetUniqueId = (decltype(GetUniqueId))dlsym(lib, "ncclGetUniqueId");
        CommInitRank = (decltype(CommInitRank))dlsym(lib, "ncclCommInitRank");
        AllReduce = (decltype(AllReduce))dlsym(lib, "ncclAllReduce");
        AllGather = (decltype(AllGather))dlsym(lib, "ncclAllGather");
        CommDestroy = (decltype(CommDestroy))dlsym(lib, "ncclCommDestroy");
        CommAbort = (decltype(CommAbort))dlsym(lib, "ncclCommAbort");
        CommGetAsyncError = (decltype(CommGetAsyncError))dlsym(lib, "ncclCommGetAsyncError");
        GetErrorString = (decltype(GetErrorString))dlsym(lib, "ncclGetErrorString");
        return GetUniqueId && CommInitRank && AllReduce && AllGather && CommDestroy && CommAbort && GetErrorString;
    }
};
static NcclApi g_nccl;
constexpr int kNcclFloat = 7, kNcclSum = 0, kNcclInProgress = 7;

int nccl_unique_id(uint8_t out[128]) {
    if (!g_nccl.load()) return SY_ERR_COMM;
    nccl_unique_id_t id;
    if (g_nccl.GetUniqueId(&id) != 0) return SY_ERR_COMM;
    std::memcpy(out, id.internal, 128);
    return SY_OK;
}

// ------------------------------------------------------------------ helpers
static View slice(const View& v, int c0, int n) { return View{v.base + c0, v.pitch, n, v.rows}; }
static int round_up(int v, int m) { return (v + m - 1) / m * m; }

void* Session::dalloc(size_t bytes) {
    void* p = nullptr;
    SY_CUDA(cudaMalloc(&p, std::max<size_t>(bytes, 256)));
    SY_CUDA(cudaMemsetAsync(p, 0, std::max<size_t>(bytes, 256), stream_));
    allocations_.push_back(p);
    return p;
}

View Session::alloc_view(int channels, const Grid& g) {
    const int pitch = round_up(channels, 4);
    const long rows = (long)B_ * g.rows;
    sp_floats_ = std::max(sp_floats_, (size_t)rows * pitch);
    float* p = static_cast<float*>(dalloc((size_t)rows * pitch * sizeof(float)));
    return View{p, pitch, channels, rows};
}

// ------------------------------------------------------------------ construction
Session::Session(const sy_config& c) : cfg(c) {
    if (c.struct_size != (int)sizeof(sy_config)) throw SyError(SY_ERR_INVALID_ARGUMENT, "sy_config size mismatch");
    if (c.image_size < 64 || c.image_size > 1280 || c.image_size % 32 != 0)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "image_size must be a multiple of 32 in [64, 1280]");
    if (c.max_batch < 1 || c.max_batch > 1024) throw SyError(SY_ERR_INVALID_ARGUMENT, "max_batch out of range");
    if (c.max_boxes < 0 || c.max_boxes > 100) throw SyError(SY_ERR_INVALID_ARGUMENT, "max_boxes out of range");
    if (c.num_classes < 1 || c.num_classes > 256) throw SyError(SY_ERR_INVALID_ARGUMENT, "num_classes out of range");
    // TrainingHeadSchema.Read (TrainingHeadSchema.cs:17-21): 16 bins, or 1 (direct distances) on
    // end-to-end heads only; end-to-end with one bin is the progressive loss
    if (c.reg_max != 16 && c.reg_max != 1)
        throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "reg_max must be 16 (DFL) or 1 (direct distances)");
    if (c.end_to_end != 0 && c.end_to_end != 1) throw SyError(SY_ERR_INVALID_ARGUMENT, "end_to_end must be 0 or 1");
    if (c.reg_max == 1 && !c.end_to_end)
        throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "reg_max 1 needs the one2one branches (end_to_end)");
    if (c.schedule_epochs < 0) throw SyError(SY_ERR_INVALID_ARGUMENT, "schedule_epochs must not be negative");
    n_sets_ = c.end_to_end ? 2 : 1;
    progressive_ = c.end_to_end && c.reg_max == 1;
    if (c.world_size < 1 || c.rank < 0 || c.rank >= c.world_size)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "bad rank / world_size");
    if (!(c.lr > 0) || !(c.momentum >= 0 && c.momentum < 1) || !(c.weight_decay >= 0))
        throw SyError(SY_ERR_INVALID_ARGUMENT, "bad optimizer hyper-parameters");
    if (c.comm_timeout_ms < 0) throw SyError(SY_ERR_INVALID_ARGUMENT, "comm_timeout_ms must not be negative");
    comm_timeout_ms_ = c.comm_timeout_ms > 0 ? c.comm_timeout_ms : 300000;
    if (c.precision != SY_PRECISION_TF32 && c.precision != SY_PRECISION_3XTF32)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "precision must be SY_PRECISION_TF32 or SY_PRECISION_3XTF32");
    x3_ = c.precision == SY_PRECISION_3XTF32;
    rnd_ = !x3_;
    if (const char* e = std::getenv("SIMDYOLO_CUDA_GRAPHS")) use_graphs_ = std::strcmp(e, "0") != 0;
    device_ = c.device;
    SY_CUDA(cudaSetDevice(device_));
    SY_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    SY_CUDA(cudaEventCreate(&ev0_));
    SY_CUDA(cudaEventCreate(&ev1_));
    SY_CUDA(cudaEventCreate(&ev_post_));
    B_ = c.max_batch;
    for (int l = 0; l < 3; l++) levels_[l] = make_grid(c.image_size >> (3 + l), c.image_size >> (3 + l));
    if (c.backbone == SY_BACKBONE_YOLOV8 || c.backbone == SY_BACKBONE_YOLO11) {
        build_backbone();
    } else if (c.backbone == SY_BACKBONE_NONE) {
        for (int l = 0; l < 3; l++) {
            if (c.feature_channels[l] < 1) throw SyError(SY_ERR_INVALID_ARGUMENT, "feature_channels required");
            feat_ch_[l] = c.feature_channels[l];
            features_[l] = alloc_view(feat_ch_[l], levels_[l]);
        }
        size_t most = 0;
        for (int l = 0; l < 3; l++) most = std::max(most, (size_t)B_ * feat_ch_[l] * levels_[l].h * levels_[l].w);
        feat_stage_ = static_cast<float*>(dalloc(most * sizeof(float)));
    } else {
        throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "unknown backbone");
    }
    build_head();
    if (x3_) {
        for (auto& p : sp_) p = static_cast<float*>(dalloc(sizeof(float) * sp_floats_));
        for (auto& p : wsp_) p = static_cast<float*>(dalloc(sizeof(float) * wsp_floats_));
    }
    // loss, truth, outputs
    const int anchors = levels_[0].h * levels_[0].w + levels_[1].h * levels_[1].w + levels_[2].h * levels_[2].w;
    anchors_ = anchors;
    loss_ws_ = dalloc(loss_workspace_bytes(B_, anchors, std::max(1, c.max_boxes), 10, c.num_classes));
    d_truth_ = static_cast<TruthBox*>(dalloc(sizeof(TruthBox) * (size_t)B_ * std::max(1, c.max_boxes)));
    d_box_off_ = static_cast<int*>(dalloc(sizeof(int) * (B_ + 1)));
    d_flags_ = static_cast<int*>(dalloc(sizeof(int) * 16));
    d_abs_ = static_cast<double*>(dalloc(sizeof(double) * kAbsSumBlocks));
    SY_CUDA(cudaMallocHost(&h_truth_, sizeof(TruthBox) * (size_t)B_ * std::max(1, c.max_boxes)));
    SY_CUDA(cudaMallocHost(&h_box_off_, sizeof(int) * (B_ + 1)));
    SY_CUDA(cudaMallocHost(&h_flags_, sizeof(int) * 16));
    SY_CUDA(cudaMallocHost(&h_rec_, sizeof(float) * (size_t)head_floats_ * c.world_size));
    SY_CUDA(cudaMallocHost(&h_images_, sizeof(int) * 4));
    SY_CUDA(cudaMallocHost(&h_rgb_ref_, sizeof(void*)));
    d_rgb_ref_ = static_cast<const uint8_t**>(dalloc(sizeof(void*)));
    SY_CUDA(cudaMallocHost(&h_abs_, sizeof(double) * kAbsSumBlocks));
    if (c.backbone != SY_BACKBONE_NONE) {
        SY_CUDA(cudaMallocHost(&h_rgb_, (size_t)B_ * c.image_size * c.image_size * 3));
        d_rgb_ = static_cast<uint8_t*>(dalloc((size_t)B_ * c.image_size * c.image_size * 3));
    }
    if (c.world_size > 1) {
        if (!g_nccl.load()) throw SyError(SY_ERR_COMM, "libnccl.so.2 not found");
        nccl_ = &g_nccl;
        nccl_unique_id_t id;
        std::memcpy(id.internal, c.nccl_id, 128);
        int r = g_nccl.CommInitRank(&comm_, c.world_size, id, c.rank);
        if (r != 0) throw SyError(SY_ERR_COMM, std::string("ncclCommInitRank: ") + g_nccl.GetErrorString(r));
    }
    SY_CUDA(cudaStreamSynchronize(stream_));
}

void Session::clear_graphs() {
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    graphs_.clear();
    graph_seen_.clear();
    graph_nodes_.clear();
}

Session::~Session() {
    if (stream_) cudaStreamSynchronize(stream_);
    clear_graphs();
    if (comm_ && nccl_) nccl_->CommDestroy(comm_);   // an aborted communicator is already gone
    for (void* p : allocations_) cudaFree(p);
    if (det_ws_) cudaFree(det_ws_);
    if (det_out_) cudaFree(det_out_);
    for (void* p : {(void*)h_truth_, (void*)h_box_off_, (void*)h_flags_, (void*)h_rec_, (void*)h_images_, (void*)h_rgb_ref_,
                    (void*)h_abs_, (void*)h_rgb_})
        if (p) cudaFreeHost(p);
    if (ev0_) cudaEventDestroy(ev0_);
    if (ev1_) cudaEventDestroy(ev1_);
    if (ev_post_) cudaEventDestroy(ev_post_);
    for (int l = 0; l < 3; l++) {
        if (l > 0 && lanes_[l].stream) cudaStreamDestroy(lanes_[l].stream);
        if (lanes_[l].done) cudaEventDestroy(lanes_[l].done);
    }
    if (ev_fork_) cudaEventDestroy(ev_fork_);
    for (cudaEvent_t e : {ev_assigned_, ev_box_, ev_cls_})
        if (e) cudaEventDestroy(e);
    if (loss_stream_) cudaStreamDestroy(loss_stream_);
    for (cudaEvent_t e : ev_feat_)
        if (e) cudaEventDestroy(e);
    for (ImageSlot& sl : slots_) {
        if (sl.dev) cudaFree(sl.dev);
        if (sl.pinned) cudaFreeHost(sl.pinned);
        if (sl.copied) cudaEventDestroy(sl.copied);
        if (sl.released) cudaEventDestroy(sl.released);
    }
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    if (ev_uploaded_) cudaEventDestroy(ev_uploaded_);
    for (cudaEvent_t e : prof_ev_) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
}

// ------------------------------------------------------------------ frozen trunk plan
// Trunk layer lists follow the public YOLOv8 / YOLO11 definitions: channel rule
// make_divisible(min(c, max) * width, 8), depth rule max(round(n * depth), 1); BatchNorm is already
// folded into every conv's weight + bias.  Parameters are taken in the order the builders call.
static int trunk_channels(const sy_config& c, int ch) {
    float x = (float)std::min(ch, c.max_channels) * c.width_mult;
    return (int)std::ceil(x / 8.0f) * 8;
}
static int trunk_depth(const sy_config& c, int n) { return std::max((int)std::lround(n * c.depth_mult), 1); }

void Session::tk_conv(const View& in, const Grid& gin, int oc, int k, int s, const View& out, const Grid& gout,
                      const View* res, int act) {
    BackboneOp op;
    op.type = 0;
    op.ic = in.channels;
    op.oc = oc;
    op.k = k;
    op.stride = s;
    op.act = act;
    op.w_off = tk_poff_;
    tk_poff_ += (long)oc * op.ic * k * k;
    op.b_off = tk_poff_;
    tk_poff_ += oc;
    op.in = in;
    op.out = out;
    op.gin = gin;
    op.gout = gout;
    if (res) {
        op.res = *res;
        op.has_res = true;
    }
    if (s == 2 && in.base != img_.base) {  // the stem reads the RGB24 image directly (stem_conv)
        // parity-split copy of the input, laid out on this conv's output grid
        if (gin.h != 2 * gout.h || gin.w != 2 * gout.w || k != 3)
            throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "stride-2 conv needs k 3 and an even input");
        const int pitch = round_up(op.ic, 4);
        op.phase_plane_rows = (long)B_ * gout.rows;
        float* buf = static_cast<float*>(dalloc(sizeof(float) * (size_t)pitch * 4 * op.phase_plane_rows));
        sp_floats_ = std::max(sp_floats_, (size_t)pitch * 4 * op.phase_plane_rows);
        op.phase_in = View{buf, pitch, op.ic, 4 * op.phase_plane_rows};
        const PhaseOut po{buf, pitch, gout, op.phase_plane_rows};
        // the most recent conv that wrote exactly this view also writes the parity copy
        bool found = false;
        for (auto it = bops_.rbegin(); it != bops_.rend(); ++it)
            if (it->type == 0 && it->out.base == in.base && it->out.channels == in.channels) {
                it->has_phase_out = true;
                it->phase_out = po;
                found = true;
                break;
            }
        if (!found) throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "stride-2 conv input has no producing conv");
    }
    bops_.push_back(op);
}

void Session::tk_sppf(const View& in, const Grid& g, int c2, const View& out) {
    const int c = in.channels / 2;
    View cat = alloc_view(4 * c, g);
    tk_conv(in, g, c, 1, 1, slice(cat, 0, c), g, nullptr);
    for (int i = 0; i < 3; i++) {
        BackboneOp op;
        op.type = 1;
        op.in = slice(cat, i * c, c);
        op.out = slice(cat, (i + 1) * c, c);
        op.gin = op.gout = g;
        bops_.push_back(op);
    }
    tk_conv(cat, g, c2, 1, 1, out, g, nullptr);
}

void Session::tk_upsample(const View& in, const Grid& gin, const View& out, const Grid& gout) {
    BackboneOp op;
    op.type = 2;
    op.in = in;
    op.out = out;
    op.gin = gin;
    op.gout = gout;
    bops_.push_back(op);
}

void Session::build_trunk_v8() {
    const int S = cfg.image_size;
    const int c64 = trunk_channels(cfg, 64), c128 = trunk_channels(cfg, 128), c256 = trunk_channels(cfg, 256);
    const int c512 = trunk_channels(cfg, 512), c1024 = trunk_channels(cfg, 1024);
    const int n3 = trunk_depth(cfg, 3), n6 = trunk_depth(cfg, 6);
    const Grid gS = make_grid(S, S), g2 = make_grid(S / 2, S / 2), g4 = make_grid(S / 4, S / 4);
    const Grid g8 = levels_[0], g16 = levels_[1], g32 = levels_[2];
    auto c2f = [&](const View& in, const Grid& g, int c2, int n, bool shortcut, const View& out) {
        const int c = c2 / 2;
        View cat = alloc_view((2 + n) * c, g);
        View tmp = alloc_view(c, g);
        tk_conv(in, g, 2 * c, 1, 1, slice(cat, 0, 2 * c), g, nullptr);
        for (int i = 0; i < n; i++) {
            View src = slice(cat, (1 + i) * c, c), dst = slice(cat, (2 + i) * c, c);
            tk_conv(src, g, c, 3, 1, tmp, g, nullptr);
            tk_conv(tmp, g, c, 3, 1, dst, g, shortcut ? &src : nullptr);
        }
        tk_conv(cat, g, c2, 1, 1, out, g, nullptr);
    };
    View b0 = alloc_view(c64, g2);
    tk_conv(img_, gS, c64, 3, 2, b0, g2, nullptr);
    View b1 = alloc_view(c128, g4);
    tk_conv(b0, g2, c128, 3, 2, b1, g4, nullptr);
    View b2 = alloc_view(c128, g4);
    c2f(b1, g4, c128, n3, true, b2);
    View b3 = alloc_view(c256, g8);
    tk_conv(b2, g4, c256, 3, 2, b3, g8, nullptr);
    View cat14 = alloc_view(c512 + c256, g8);
    View l4 = slice(cat14, c512, c256);
    c2f(b3, g8, c256, n6, true, l4);
    View b5 = alloc_view(c512, g16);
    tk_conv(l4, g8, c512, 3, 2, b5, g16, nullptr);
    View cat11 = alloc_view(c1024 + c512, g16);
    View l6 = slice(cat11, c1024, c512);
    c2f(b5, g16, c512, n6, true, l6);
    View b7 = alloc_view(c1024, g32);
    tk_conv(l6, g16, c1024, 3, 2, b7, g32, nullptr);
    View b8 = alloc_view(c1024, g32);
    c2f(b7, g32, c1024, n3, true, b8);
    View cat20 = alloc_view(c512 + c1024, g32);
    View l9 = slice(cat20, c512, c1024);
    tk_sppf(b8, g32, c1024, l9);
    tk_upsample(l9, g32, slice(cat11, 0, c1024), g16);
    View cat17 = alloc_view(c256 + c512, g16);
    View l12 = slice(cat17, c256, c512);
    c2f(cat11, g16, c512, n3, false, l12);
    tk_upsample(l12, g16, slice(cat14, 0, c512), g8);
    View p3 = alloc_view(c256, g8);
    c2f(cat14, g8, c256, n3, false, p3);
    tk_conv(p3, g8, c256, 3, 2, slice(cat17, 0, c256), g16, nullptr);
    View p4 = alloc_view(c512, g16);
    c2f(cat17, g16, c512, n3, false, p4);
    tk_conv(p4, g16, c512, 3, 2, slice(cat20, 0, c512), g32, nullptr);
    View p5 = alloc_view(c1024, g32);
    c2f(cat20, g32, c1024, n3, false, p5);
    features_[0] = p3;
    features_[1] = p4;
    features_[2] = p5;
}

// YOLO11 trunk (PtModel.cs cases C3k2, C3k, Bottleneck, C2PSA, PSABlock, Attention).
void Session::build_trunk_11() {
    const int S = cfg.image_size;
    const int c64 = trunk_channels(cfg, 64), c128 = trunk_channels(cfg, 128), c256 = trunk_channels(cfg, 256);
    const int c512 = trunk_channels(cfg, 512), c1024 = trunk_channels(cfg, 1024);
    const int n2 = trunk_depth(cfg, 2);
    const Grid gS = make_grid(S, S), g2 = make_grid(S / 2, S / 2), g4 = make_grid(S / 4, S / 4);
    const Grid g8 = levels_[0], g16 = levels_[1], g32 = levels_[2];
    // Bottleneck: cv2(cv1(x)) (+ x); `out` may be `x` itself (the residual is read before the write)
    auto bottleneck = [&](const View& x, const Grid& g, int c2, float e, bool shortcut, const View& out) {
        const int c_ = (int)(c2 * e);
        View t = alloc_view(c_, g);
        tk_conv(x, g, c_, 3, 1, t, g, nullptr);
        tk_conv(t, g, c2, 3, 1, out, g, (shortcut && x.channels == c2) ? &x : nullptr);
    };
    // C3k: cv3(cat(m(cv1(x)), cv2(x))), m = n Bottlenecks with e = 1
    auto c3k = [&](const View& x, const Grid& g, int c2, int n, const View& out) {
        const int c_ = (int)(c2 * 0.5f);
        View cat = alloc_view(2 * c_, g);
        View a = slice(cat, 0, c_), b = slice(cat, c_, c_);
        tk_conv(x, g, c_, 1, 1, a, g, nullptr);
        for (int i = 0; i < n; i++) bottleneck(a, g, c_, 1.0f, true, a);
        tk_conv(x, g, c_, 1, 1, b, g, nullptr);
        tk_conv(cat, g, c2, 1, 1, out, g, nullptr);
    };
    // C3k2: C2f layout whose modules are C3k(c, c, 2) or Bottleneck(c, c, e = 0.5)
    auto c3k2 = [&](const View& x, const Grid& g, int c2, bool use_c3k, float e, const View& out) {
        const int c = (int)(c2 * e);
        View cat = alloc_view((2 + n2) * c, g);
        tk_conv(x, g, 2 * c, 1, 1, slice(cat, 0, 2 * c), g, nullptr);
        for (int i = 0; i < n2; i++) {
            View src = slice(cat, (1 + i) * c, c), dst = slice(cat, (2 + i) * c, c);
            if (use_c3k) c3k(src, g, c, 2, dst);
            else bottleneck(src, g, c, 0.5f, true, dst);
        }
        tk_conv(cat, g, c2, 1, 1, out, g, nullptr);
    };
    // PSABlock in place on x: x += proj(attention(qkv(x)) + pe(v)); x += ffn(x)
    auto psablock = [&](const View& x, const Grid& g, int c, int heads) {
        const int hd = c / heads, kd = (int)(hd * 0.5f), hch = c + 2 * kd * heads;
        View qkv = alloc_view(hch, g), att = alloc_view(c, g), v = alloc_view(c, g), t = alloc_view(2 * c, g);
        tk_conv(x, g, hch, 1, 1, qkv, g, nullptr, 0);
        BackboneOp at;
        at.type = 4;
        at.in = qkv;
        at.out = att;
        at.aux = v;
        at.heads = heads;
        at.ic = hd;
        at.oc = kd;
        at.gin = at.gout = g;
        bops_.push_back(at);
        BackboneOp pe;   // depthwise 3x3 positional conv on v, added to the attention output
        pe.type = 3;
        pe.ic = pe.oc = c;
        pe.k = 3;
        pe.w_off = tk_poff_;
        tk_poff_ += (long)c * 9;
        pe.b_off = tk_poff_;
        tk_poff_ += c;
        pe.in = v;
        pe.out = att;
        pe.res = att;
        pe.has_res = true;
        pe.gin = pe.gout = g;
        bops_.push_back(pe);
        tk_conv(att, g, c, 1, 1, x, g, &x, 0);
        tk_conv(x, g, 2 * c, 1, 1, t, g, nullptr);
        tk_conv(t, g, c, 1, 1, x, g, &x, 0);
    };
    auto c2psa = [&](const View& x, const Grid& g, int c1, const View& out) {
        const int c = (int)(c1 * 0.5f);
        View cat = alloc_view(2 * c, g);
        tk_conv(x, g, 2 * c, 1, 1, cat, g, nullptr);
        for (int i = 0; i < n2; i++) psablock(slice(cat, c, c), g, c, std::max(c / 64, 1));
        tk_conv(cat, g, c1, 1, 1, out, g, nullptr);
    };
    View b0 = alloc_view(c64, g2);
    tk_conv(img_, gS, c64, 3, 2, b0, g2, nullptr);
    View b1 = alloc_view(c128, g4);
    tk_conv(b0, g2, c128, 3, 2, b1, g4, nullptr);
    View b2 = alloc_view(c256, g4);
    c3k2(b1, g4, c256, false, 0.25f, b2);
    View b3 = alloc_view(c256, g8);
    tk_conv(b2, g4, c256, 3, 2, b3, g8, nullptr);
    View cat15 = alloc_view(c512 + c512, g8);
    View l4 = slice(cat15, c512, c512);
    c3k2(b3, g8, c512, false, 0.25f, l4);
    View b5 = alloc_view(c512, g16);
    tk_conv(l4, g8, c512, 3, 2, b5, g16, nullptr);
    View cat12 = alloc_view(c1024 + c512, g16);
    View l6 = slice(cat12, c1024, c512);
    c3k2(b5, g16, c512, true, 0.5f, l6);
    View b7 = alloc_view(c1024, g32);
    tk_conv(l6, g16, c1024, 3, 2, b7, g32, nullptr);
    View b8 = alloc_view(c1024, g32);
    c3k2(b7, g32, c1024, true, 0.5f, b8);
    View b9 = alloc_view(c1024, g32);
    tk_sppf(b8, g32, c1024, b9);
    View cat21 = alloc_view(c512 + c1024, g32);
    View l10 = slice(cat21, c512, c1024);
    c2psa(b9, g32, c1024, l10);
    tk_upsample(l10, g32, slice(cat12, 0, c1024), g16);
    View cat18 = alloc_view(c256 + c512, g16);
    View l13 = slice(cat18, c256, c512);
    c3k2(cat12, g16, c512, false, 0.5f, l13);
    tk_upsample(l13, g16, slice(cat15, 0, c512), g8);
    View p3 = alloc_view(c256, g8);
    c3k2(cat15, g8, c256, false, 0.5f, p3);
    tk_conv(p3, g8, c256, 3, 2, slice(cat18, 0, c256), g16, nullptr);
    View p4 = alloc_view(c512, g16);
    c3k2(cat18, g16, c512, false, 0.5f, p4);
    tk_conv(p4, g16, c512, 3, 2, slice(cat21, 0, c512), g32, nullptr);
    View p5 = alloc_view(c1024, g32);
    c3k2(cat21, g32, c1024, true, 0.5f, p5);
    features_[0] = p3;
    features_[1] = p4;
    features_[2] = p5;
}

void Session::build_backbone() {
    img_grid_ = make_grid(cfg.image_size, cfg.image_size);
    // the image itself only exists as the stem's parity-split input; img_ just names it
    img_ = View{static_cast<float*>(dalloc(256)), 4, 3, 0};
    tk_poff_ = 0;
    if (cfg.backbone == SY_BACKBONE_YOLO11) build_trunk_11();
    else build_trunk_v8();
    for (int l = 0; l < 3; l++) feat_ch_[l] = features_[l].channels;
    // A conv whose output is read only through its parity-split copy (by stride-2 convs) skips the
    // plain write: no other op's input or residual, and no feature map, overlaps that output.
    auto span_of = [](const View& v) {
        return std::make_pair(v.base, v.base + (v.rows > 0 ? (v.rows - 1) * (long)v.pitch + v.channels : 0));
    };
    auto overlaps = [&](const View& a, const View& b) {
        const auto x = span_of(a), y = span_of(b);
        return x.first < y.second && y.first < x.second;
    };
    for (auto& op : bops_) {
        if (op.type != 0 || !op.has_phase_out) continue;
        bool read = false;
        for (const auto& q : bops_) {
            if (&q == &op) continue;
            if (q.type != 0 || q.stride == 1) read |= overlaps(q.in, op.out);
            if (q.has_res) read |= overlaps(q.res, op.out);
        }
        for (int l = 0; l < 3; l++) read |= overlaps(features_[l], op.out);
        op.plain_out = read || x3_;   // 3xTF32 passes accumulate in the plain output
    }
    for (int i = 0; i < (int)bops_.size(); i++)
        for (int l = 0; l < 3; l++)
            if (overlaps(features_[l], bops_[i].out)) feat_op_[l] = i;
    n_backbone = tk_poff_;
    backbone_params_ = static_cast<float*>(dalloc(sizeof(float) * (size_t)tk_poff_));
    for (auto& op : bops_) {
        if (op.type != 0) continue;
        const int taps = op.k * op.k;
        op.wk = static_cast<float*>(dalloc(sizeof(float) * (size_t)op.oc * taps * round_up(op.ic, 32)));
        wsp_floats_ = std::max(wsp_floats_, (size_t)op.oc * taps * round_up(op.ic, 32));
    }
}

int Session::set_backbone(const float* host, long count) {
    if (cfg.backbone == SY_BACKBONE_NONE || count != n_backbone)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "backbone parameter count mismatch");
    SY_CUDA(cudaMemcpyAsync(backbone_params_, host, sizeof(float) * count, cudaMemcpyHostToDevice, stream_));
    for (auto& op : bops_) {
        if (op.type != 0) continue;
        if (op.in.base == img_.base) {
            stem_host_.assign(host + op.w_off, host + op.w_off + (long)op.oc * op.ic * 9);
            stem_host_.insert(stem_host_.end(), host + op.b_off, host + op.b_off + op.oc);
        }
        const int taps = op.k * op.k;
        weights_fwd_layout(backbone_params_ + op.w_off, op.oc, op.ic, taps, round_up(op.ic, 32), op.wk, stream_, rnd_);
    }
    SY_CUDA(cudaStreamSynchronize(stream_));
    clear_graphs();   // the stem's weights travel by value inside captured launches
    backbone_ready_ = true;
    return SY_OK;
}

void Session::forward_backbone(int batch) {
    const bool events = level_lanes() && ev_feat_[0];
    for (int i = 0; i < (int)bops_.size(); i++) {
        const BackboneOp& op = bops_[i];
        View in = op.in, out = op.out;
        if (op.type == 0 && !op.plain_out) out.base = nullptr;
        if (op.type == 0 && in.base == img_.base) {
            stem_conv(d_rgb_ref_, batch, cfg.image_size, stem_host_.data(), stem_host_.data() + (long)op.oc * op.ic * 9,
                      op.oc, out, op.gout, op.has_phase_out ? &op.phase_out : nullptr, stream_, rnd_);
        } else if (op.type == 1) {
            maxpool5_padded(in, out, batch, op.gin, stream_);
        } else if (op.type == 2) {
            upsample2_padded(in, op.gin, out, op.gout, batch, stream_);
        } else if (op.type == 3) {
            View i2 = in, o2 = out, r2 = op.res;
            i2.rows = o2.rows = r2.rows = (long)batch * op.gin.rows;
            dw_conv(i2, backbone_params_ + op.w_off, op.k * op.k, 1, op.gin, o2, BnEpilogue{}, stream_,
                    backbone_params_ + op.b_off, op.has_res ? &r2 : nullptr, rnd_);
        } else if (op.type == 4) {
            View i2 = in, o2 = out, a2 = op.aux;
            i2.rows = o2.rows = a2.rows = (long)batch * op.gin.rows;
            attention(i2, batch, op.gin, op.heads, op.oc, op.ic, 1.0f / std::sqrt((float)op.oc), o2, a2, stream_);
        } else {
            ConvEpilogue ep;
            ep.bias = backbone_params_ + op.b_off;
            ep.silu = op.act;
            ep.round_tf32 = rnd_;
            if (op.has_res) {
                ep.residual = op.res.base;
                ep.res_pitch = op.res.pitch;
            }
            const PhaseOut* po = op.has_phase_out ? &op.phase_out : nullptr;
            if (op.stride == 1) {
                // the tcgen05 kernel works on whole 128-row tiles: restrict the views to `batch` images
                View i2 = in, o2 = out;
                i2.rows = o2.rows = (long)batch * op.gin.rows;
                prof_begin();
                conv_fwd(i2, op.wk, (long)op.oc * op.k * op.k * round_up(op.ic, 32), op.oc, op.oc, op.k * op.k, 1,
                         op.gin, o2, ep, po);
                prof_end(2.0 * batch * op.oc * op.ic * op.k * op.k * op.gin.h * op.gin.w,
                         {0, op.ic, op.oc, op.k * op.k, op.gin.h, op.gin.w});
            } else {
                prof_begin();
                conv_strided(op.phase_in, op.phase_plane_rows, (long)batch * op.gout.rows, op.wk,
                             (long)op.oc * 9 * round_up(op.ic, 32), op.oc, op.gout, out, ep, po);
                prof_end(2.0 * batch * op.oc * op.ic * 9 * op.gout.h * op.gout.w,
                         {1, op.ic, op.oc, 9, op.gout.h, op.gout.w});
            }
        }
        if (events)
            for (int l = 0; l < 2; l++)
                if (i == feat_op_[l]) SY_CUDA(cudaEventRecord(ev_feat_[l], stream_));
    }
    feat_events_ = events;
}

// ------------------------------------------------------------------ head plan
static std::string block_path(int i, int n) {
    if (n == 5) {
        static const char* p[5] = {"0.0", "0.1", "1.0", "1.1", "2"};
        return p[i];
    }
    return std::to_string(i);
}

// Branch name prefix in DetectionHead order (DetectionHead.cs:20-26, TrainingHeadSchema.cs:12).
static std::string branch_prefix(const Branch& b) {
    static const char* names[2][2] = {{"cv3.", "cv2."}, {"one2one_cv3.", "one2one_cv2."}};
    return std::string(names[b.set][b.box ? 1 : 0]) + std::to_string(b.level);
}

void Session::build_head() {
    long poff = 0, qoff = 0;
    // cv2.0-2, cv3.0-2, then for end-to-end heads one2one_cv2.0-2, one2one_cv3.0-2 with the same
    // block lists (the one-to-one branches are copies of the one-to-many ones in the source model)
    for (int br = 0; br < 6 * n_sets_; br++) {
        Branch branch;
        branch.level = br % 3;
        branch.box = (br / 3) % 2 == 0;
        branch.set = br / 6;
        branch.group = branch.box ? 1 + branch.set : 0;
        const int l = branch.level;
        const int n = branch.box ? cfg.n_box_blocks : cfg.n_cls_blocks;
        if (n < 1 || n > 8) throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "head branch needs 1..8 blocks");
        const sy_block* blocks = branch.box ? cfg.box_blocks[l] : cfg.cls_blocks[l];
        const std::string prefix = branch_prefix(branch);
        int ic = feat_ch_[l];
        for (int i = 0; i < n; i++) {
            HeadBlock hb;
            hb.b = blocks[i];
            const sy_block& b = hb.b;
            hb.dw = b.groups > 1 && b.groups == b.ic && b.ic == b.oc;
            hb.grouped = b.groups > 1 && !hb.dw;
            if (b.ic != ic || b.oc < 1 || b.oc > 512 || !(b.k == 1 || b.k == 3) || b.groups < 1 ||
                b.ic % b.groups != 0 || b.oc % b.groups != 0 || (!hb.dw && b.oc > 256))
                throw SyError(SY_ERR_UNSUPPORTED_SHAPE,
                              "head conv must be k 1 or 3 with groups dividing both channel counts, at most 256 output "
                              "channels (depthwise, groups = channels: 512), chained channels (" + prefix + ")");
            if (hb.dw && (b.has_bias || b.oc % 4 != 0))
                throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "depthwise head convs need BatchNorm and a multiple of 4 channels");
            if ((i == n - 1) == (b.has_bn != 0)) throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "only the last block is a Conv2d");
            hb.taps = b.k * b.k;
            const std::string path = prefix + "." + block_path(i, n);
            const long wn = (long)b.oc * (b.ic / b.groups) * b.k * b.k;
            auto add_param = [&](const std::string& name, std::vector<int> shape, long numel, int decay) {
                TensorEntry e{name, 0, shape, poff, numel, branch.group, decay};
                tensors.push_back(e);
                long off = poff;
                poff += numel;
                return off;
            };
            hb.w_off = add_param(path + (b.has_bn ? ".conv.weight" : ".weight"), {b.oc, b.ic / b.groups, b.k, b.k},
                                 wn, 1);
            if (b.has_bias) hb.b_off = add_param(path + (b.has_bn ? ".conv.bias" : ".bias"), {b.oc}, b.oc, 0);
            if (b.has_bn) {
                hb.g_off = add_param(path + ".bn.weight", {b.oc}, b.oc, 0);
                hb.be_off = add_param(path + ".bn.bias", {b.oc}, b.oc, 0);
            }
            ic = b.oc;
            branch.blocks.push_back(hb);
        }
        const int expect = branch.box ? 4 * cfg.reg_max : cfg.num_classes;
        if (branch.blocks.back().b.oc != expect)
            throw SyError(SY_ERR_UNSUPPORTED_SHAPE, "head output channels must be 4*reg_max (box) or nc (class)");
        branches_.push_back(std::move(branch));
    }
    n_params = poff;
    // buffers after all parameters (Snapshot order: parameters, then BN buffers)
    for (auto& branch : branches_) {
        const std::string prefix = branch_prefix(branch);
        const int n = (int)branch.blocks.size();
        for (int i = 0; i < n; i++) {
            HeadBlock& hb = branch.blocks[i];
            if (!hb.b.has_bn) continue;
            const std::string path = prefix + "." + block_path(i, n);
            hb.rm_off = qoff;
            tensors.push_back(TensorEntry{path + ".bn.running_mean", 1, {hb.b.oc}, qoff, hb.b.oc, 0, 0});
            qoff += hb.b.oc;
            hb.rv_off = qoff;
            tensors.push_back(TensorEntry{path + ".bn.running_var", 1, {hb.b.oc}, qoff, hb.b.oc, 0, 0});
            qoff += hb.b.oc;
            hb.nt_off = qoff;
            tensors.push_back(TensorEntry{path + ".bn.num_batches_tracked", 1, {}, qoff, 1, 0, 0});
            qoff += 1;
        }
    }
    n_buffers = qoff;
    params_ = static_cast<float*>(dalloc(sizeof(float) * n_params));
    grads_ = static_cast<float*>(dalloc(sizeof(float) * n_params));
    last_grads_ = static_cast<float*>(dalloc(sizeof(float) * n_params));
    vel_ = static_cast<float*>(dalloc(sizeof(float) * n_params));
    vel2_ = static_cast<float*>(dalloc(sizeof(float) * n_params));
    buffers_ = static_cast<float*>(dalloc(sizeof(float) * std::max(1L, n_buffers)));
    // running variance starts at 1 (fresh BatchNorm2d) until set_tensor overwrites it
    {
        std::vector<float> init(n_buffers, 0.0f);
        for (auto& br : branches_)
            for (auto& hb : br.blocks)
                if (hb.b.has_bn)
                    for (int c = 0; c < hb.b.oc; c++) init[hb.rv_off + c] = 1.0f;
        SY_CUDA(cudaMemcpy(buffers_, init.data(), sizeof(float) * n_buffers, cudaMemcpyHostToDevice));
    }
    // optimizer segments: one per parameter tensor
    std::vector<ParamSegment> segs;
    for (auto& t : tensors)
        if (t.kind == 0) segs.push_back(ParamSegment{t.offset, t.numel, t.decay, t.group});
    nsegs_ = (int)segs.size();
    d_segs_ = static_cast<ParamSegment*>(dalloc(sizeof(ParamSegment) * segs.size()));
    SY_CUDA(cudaMemcpy(d_segs_, segs.data(), sizeof(ParamSegment) * segs.size(), cudaMemcpyHostToDevice));
    // activations and gradients
    size_t ws = 0;
    size_t bn_part_floats = 0;
    size_t lvl_ws[3] = {0, 0, 0}, lvl_part[3] = {0, 0, 0};
    for (auto& branch : branches_) {
        const Grid& g = levels_[branch.level];
        View x = features_[branch.level];
        for (auto& hb : branch.blocks) {
            const sy_block& b = hb.b;
            hb.x = x;
            hb.y = alloc_view(b.oc, g);
            hb.g = alloc_view(b.oc, g);
            if (b.has_bn) {
                hb.a = alloc_view(b.oc, g);
                hb.dy = alloc_view(b.oc, g);
                hb.stats_off = bn_channels_;
                bn_channels_ += b.oc;
                hb.coef = static_cast<float*>(dalloc(sizeof(float) * 2 * B_ * b.oc));
                hb.bcoef = static_cast<float*>(dalloc(sizeof(float) * 3 * B_ * b.oc));
                bn_part_floats = std::max(bn_part_floats, bn_partial_floats(B_, g, b.oc));
                lvl_part[branch.level] = std::max(lvl_part[branch.level], bn_partial_floats(B_, g, b.oc));
            } else {
                hb.dy = hb.g;
            }
            if (hb.dw) {
                ws = std::max(ws, dw_wgrad_workspace_floats(b.oc, hb.taps, (long)B_ * g.rows));
                lvl_ws[branch.level] = std::max(lvl_ws[branch.level],
                                                dw_wgrad_workspace_floats(b.oc, hb.taps, (long)B_ * g.rows));
            } else {
                hb.kpad_in = round_up(b.ic, 32);
                hb.kpad_out = round_up(b.oc, 32);
                hb.w_fwd = static_cast<float*>(dalloc(sizeof(float) * (size_t)b.oc * hb.taps * hb.kpad_in));
                hb.w_dgrad = static_cast<float*>(dalloc(sizeof(float) * (size_t)b.ic * hb.taps * hb.kpad_out));
                if (hb.grouped) {
                    hb.w_dense = static_cast<float*>(dalloc(sizeof(float) * (size_t)b.oc * b.ic * hb.taps));
                    hb.wg_dense = static_cast<float*>(dalloc(sizeof(float) * (size_t)b.oc * b.ic * hb.taps));
                }
                wsp_floats_ = std::max(wsp_floats_, std::max((size_t)b.oc * hb.taps * hb.kpad_in,
                                                             (size_t)b.ic * hb.taps * hb.kpad_out));
                ws = std::max(ws, wgrad_workspace_floats(b.ic, b.oc, hb.taps, (long)B_ * g.rows));
                lvl_ws[branch.level] = std::max(lvl_ws[branch.level],
                                                wgrad_workspace_floats(b.ic, b.oc, hb.taps, (long)B_ * g.rows));
            }
            x = b.has_bn ? hb.a : hb.y;
        }
    }
    // per-image BN statistics of all layers in one block ([layer][image][channel][2]) so that
    // data-parallel ranks can exchange them with a single all-gather
    // This rank's exchange record, all-gathered once per data-parallel step: a head of per-image loss
    // parts ([set][image][4] floats), positives, box connections and assigner near ties ([set][image] ints)
    // and the image count, then the per-image BatchNorm statistics of every layer ([layer][image][channel][2]).
    head_floats_ = (8 * B_ + 2 * B_ + 2 * B_ + 2 * B_ + 1 + 3) / 4 * 4;
    rec_floats_ = head_floats_ + 2 * (long)B_ * std::max(1L, bn_channels_);
    rec_ = static_cast<float*>(dalloc(sizeof(float) * (size_t)rec_floats_));
    d_loss_ = rec_;
    d_pos_ = reinterpret_cast<int*>(rec_ + 8 * B_);
    d_conn_ = d_pos_ + 2 * B_;
    d_ties_ = d_conn_ + 2 * B_;
    d_images_ = d_ties_ + 2 * B_;
    bn_stats_all_ = rec_ + head_floats_;
    if (cfg.world_size > 1)
        rec_gather_ = static_cast<float*>(dalloc(sizeof(float) * (size_t)rec_floats_ * cfg.world_size));
    for (auto& branch : branches_)
        for (auto& hb : branch.blocks)
            if (hb.b.has_bn) hb.stats = bn_stats_all_ + 2 * (size_t)B_ * hb.stats_off;
    // batched folds over all BatchNorm layers (running statistics, parameter gradients)
    {
        std::vector<BnFoldJob> jobs;
        for (auto& branch : branches_)
            for (auto& hb : branch.blocks)
                if (hb.b.has_bn) {
                    const Grid& g = levels_[branch.level];
                    jobs.push_back(BnFoldJob{2L * B_ * hb.stats_off, hb.b.oc, g.h * g.w, buffers_ + hb.rm_off,
                                             buffers_ + hb.rv_off, buffers_ + hb.nt_off, hb.bcoef, grads_ + hb.g_off,
                                             grads_ + hb.be_off});
                    bn_max_c_ = std::max(bn_max_c_, hb.b.oc);
                }
        n_bn_jobs_ = (int)jobs.size();
        if (n_bn_jobs_ > 0) {
            d_bn_jobs_ = static_cast<BnFoldJob*>(dalloc(sizeof(BnFoldJob) * jobs.size()));
            SY_CUDA(cudaMemcpy(d_bn_jobs_, jobs.data(), sizeof(BnFoldJob) * jobs.size(), cudaMemcpyHostToDevice));
        }
    }
    wgrad_ws_ = static_cast<float*>(dalloc(sizeof(float) * ws));
    // 3xTF32: centred features for the weight gradients of the first tensor-core conv of every branch
    int max_first_oc = 0;
    for (auto& branch : branches_) {
        if (!x3_) break;
        const HeadBlock& hb = branch.blocks[0];
        if (hb.dw) continue;
        const int l = branch.level;
        if (!feat_mean_[l]) {
            feat_c_[l] = alloc_view(feat_ch_[l], levels_[l]);
            feat_mean_[l] = static_cast<float*>(dalloc(sizeof(float) * (size_t)B_ * feat_ch_[l]));
        }
        max_first_oc = std::max(max_first_oc, hb.b.oc);
    }
    const size_t center_ws_floats =
        center_workspace_floats(B_, std::max({max_first_oc, feat_ch_[0], feat_ch_[1], feat_ch_[2]}));
    if (max_first_oc > 0) {
        tap_sums_ = static_cast<float*>(dalloc(sizeof(float) * (size_t)B_ * 9 * max_first_oc));
        center_ws_ = static_cast<float*>(dalloc(sizeof(float) * center_ws_floats));
    }
    bn_part_ = static_cast<float*>(dalloc(sizeof(float) * std::max<size_t>(bn_part_floats, 1)));
    // level lanes (TF32 mode): lane 0 is stream_ with the shared scratch, lanes 1 and 2 get their own
    lanes_[0] = LevelLane{stream_, bn_part_, wgrad_ws_, nullptr, tap_sums_, center_ws_};
    if (!x3_) {
        SY_CUDA(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
        if (feat_op_[0] >= 0 && feat_op_[1] >= 0)
            for (int l = 0; l < 2; l++) SY_CUDA(cudaEventCreateWithFlags(&ev_feat_[l], cudaEventDisableTiming));
        SY_CUDA(cudaEventCreateWithFlags(&lanes_[0].done, cudaEventDisableTiming));
        SY_CUDA(cudaStreamCreateWithFlags(&loss_stream_, cudaStreamNonBlocking));
        for (cudaEvent_t* e : {&ev_assigned_, &ev_box_, &ev_cls_})
            SY_CUDA(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
        for (int l = 1; l < 3; l++) {
            SY_CUDA(cudaStreamCreateWithFlags(&lanes_[l].stream, cudaStreamNonBlocking));
            SY_CUDA(cudaEventCreateWithFlags(&lanes_[l].done, cudaEventDisableTiming));
            lanes_[l].bn_part = static_cast<float*>(dalloc(sizeof(float) * std::max<size_t>(lvl_part[l], 1)));
            lanes_[l].wgrad_ws = static_cast<float*>(dalloc(sizeof(float) * std::max<size_t>(lvl_ws[l], 1)));
            if (max_first_oc > 0) {
                lanes_[l].tap_sums = static_cast<float*>(dalloc(sizeof(float) * (size_t)B_ * 9 * max_first_oc));
                lanes_[l].center_ws = static_cast<float*>(dalloc(sizeof(float) * center_ws_floats));
            }
        }
    }
}

void Session::fork_levels() {
    SY_CUDA(cudaEventRecord(ev_fork_, lanes_[0].stream));
    for (int l = 1; l < 3; l++) SY_CUDA(cudaStreamWaitEvent(lanes_[l].stream, ev_fork_, 0));
}

void Session::join_levels() {
    use_lane(0);
    for (int l = 1; l < 3; l++) {
        SY_CUDA(cudaEventRecord(lanes_[l].done, lanes_[l].stream));
        SY_CUDA(cudaStreamWaitEvent(lanes_[0].stream, lanes_[l].done, 0));
    }
}

// Launches that follow go to lane stream_lane's stream (level l's own by default) with level l's scratch.
void Session::use_lane(int l, int stream_lane) {
    stream_ = lanes_[stream_lane < 0 ? l : stream_lane].stream;
    bn_part_ = lanes_[l].bn_part;
    wgrad_ws_ = lanes_[l].wgrad_ws;
    tap_sums_ = lanes_[l].tap_sums;
    center_ws_ = lanes_[l].center_ws;
}

void Session::refresh_head_weights() {
    if (!d_layout_jobs_) {
        // depthwise kernels read the [c][taps] parameters directly; every other head conv gets its
        // forward and data-gradient layouts from one batched launch
        std::vector<WeightLayoutJob> jobs;
        for (auto& branch : branches_)
            for (auto& hb : branch.blocks) {
                if (hb.dw) continue;
                jobs.push_back(WeightLayoutJob{hb.grouped ? hb.w_dense : params_ + hb.w_off, hb.b.oc, hb.b.ic, hb.taps,
                                               hb.kpad_in, hb.kpad_out, hb.w_fwd, hb.w_dgrad});
                layout_max_elems_ = std::max(layout_max_elems_, (long)hb.taps * (hb.b.oc * hb.kpad_in +
                                                                                  hb.b.ic * hb.kpad_out));
            }
        n_layout_jobs_ = (int)jobs.size();
        if (n_layout_jobs_ == 0) return;
        d_layout_jobs_ = static_cast<WeightLayoutJob*>(dalloc(sizeof(WeightLayoutJob) * jobs.size()));
        SY_CUDA(cudaMemcpy(d_layout_jobs_, jobs.data(), sizeof(WeightLayoutJob) * jobs.size(), cudaMemcpyHostToDevice));
    }
    for (auto& branch : branches_)
        for (auto& hb : branch.blocks)
            if (hb.grouped)
                grouped_to_dense(params_ + hb.w_off, hb.b.oc, hb.b.ic, hb.b.groups, hb.taps, hb.w_dense, stream_);
    if (n_layout_jobs_ > 0) weights_layout_batch(d_layout_jobs_, n_layout_jobs_, layout_max_elems_, stream_, rnd_);
}

static View rows_of(View v, int batch, const Grid& g) {
    v.rows = (long)batch * g.rows;
    return v;
}

// Puts stream_ and the scratch back to lane 0 when a head pass leaves early.
struct LaneGuard {
    std::function<void()> restore;
    ~LaneGuard() {
        if (restore) restore();
    }
};

void Session::forward_head(int batch, bool training) {
    const bool lanes = level_lanes();
    LaneGuard guard;
    if (lanes) {
        guard.restore = [this] { use_lane(0); };
        if (feat_events_) {
            for (int l = 0; l < 2; l++) SY_CUDA(cudaStreamWaitEvent(lanes_[l + 1].stream, ev_feat_[l], 0));
        } else {
            fork_levels();
        }
    }
    feat_events_ = false;
    for (int lv = 0; lv < 3; lv++)
    for (auto& branch : branches_) {
        if (branch.level != lv) continue;
        if (lanes) use_lane(lv, (lv + 1) % 3);
        const Grid& g = levels_[branch.level];
        for (auto& hb : branch.blocks) {
            ConvEpilogue ep;
            if (hb.b.has_bias) ep.bias = params_ + hb.b_off;
            if (hb.b.has_bn && training) {
                ep.bn.channels = hb.b.oc;
                ep.bn.stats_part = bn_part_;
            }
            if (hb.dw) {
                dw_conv(rows_of(hb.x, batch, g), params_ + hb.w_off, hb.taps, 1, g, rows_of(hb.y, batch, g), ep.bn,
                        stream_);
            } else {
                prof_begin();
                conv_fwd(rows_of(hb.x, batch, g), hb.w_fwd, (long)hb.b.oc * hb.taps * hb.kpad_in, hb.b.oc, hb.b.oc,
                         hb.taps, 1, g, rows_of(hb.y, batch, g), ep, nullptr);
                prof_end(2.0 * batch * hb.b.oc * hb.b.ic * hb.taps * g.h * g.w,
                         {2, hb.b.ic, hb.b.oc, hb.taps, g.h, g.w});
            }
            if (hb.b.has_bn) {
                if (training)
                    bn_stats_fold(bn_part_, batch, g, hb.b.oc, cfg.bn_eps, hb.stats, hb.coef, stream_);
                else
                    bn_eval_coef(buffers_ + hb.rm_off, buffers_ + hb.rv_off, cfg.bn_eps, batch, hb.b.oc, hb.coef,
                                 stream_);
                bn_silu_apply(rows_of(hb.y, batch, g), hb.coef, params_ + hb.g_off, params_ + hb.be_off, batch, g,
                              rows_of(hb.a, batch, g), stream_, rnd_);
            }
        }
    }
    if (lanes) join_levels();
}

void Session::backward_head(int batch) {
    for (int l = 0; l < 3; l++)
        if (feat_mean_[l])
            center_features(rows_of(features_[l], batch, levels_[l]), batch, levels_[l], feat_mean_[l], center_ws_,
                            rows_of(feat_c_[l], batch, levels_[l]), rnd_, stream_);
    const bool lanes = level_lanes();
    LaneGuard guard;
    if (lanes) {
        guard.restore = [this] { use_lane(0); };
        fork_levels();
    }
    // per level: box branches first (their gradient comes from the loss's box part), then the class
    // branches, which wait for the class part when it ran on its own stream
    for (int l = 2; l >= 0; l--) {
        bool cls_waited = false;
        for (int set = n_sets_ - 1; set >= 0; set--)
            for (int kind = 0; kind <= 1; kind++) {
                if (lanes) use_lane(l);
                if (kind == 1 && cls_pending_ && !cls_waited) {
                    SY_CUDA(cudaStreamWaitEvent(stream_, ev_cls_, 0));
                    cls_waited = true;
                }
                Branch& branch = branches_[set * 6 + kind * 3 + l];
                const Grid& g = levels_[l];
                for (int i = (int)branch.blocks.size() - 1; i >= 0; i--) {
                    HeadBlock& hb = branch.blocks[i];
                    if (hb.b.has_bn) {
                        // hb.g holds dz and bn_part_ its partial sums, written by the next block's data-gradient
                        // epilogue (every BN block is followed by another block)
                        bn_backward_fold(bn_part_, batch, g, hb.b.oc, hb.coef, params_ + hb.g_off, grads_ + hb.g_off,
                                         grads_ + hb.be_off, hb.bcoef, stream_, false);
                        bn_backward_apply(rows_of(hb.y, batch, g), rows_of(hb.g, batch, g), hb.coef, hb.bcoef, batch, g,
                                          rows_of(hb.dy, batch, g), stream_, rnd_);
                    }
                    // the final conv's bias gradient was accumulated by the loss kernels (LevelIO::*_bias_grad)
                    if (hb.dw)
                        dw_wgrad(rows_of(hb.x, batch, g), rows_of(hb.dy, batch, g), hb.taps, g, grads_ + hb.w_off,
                                 wgrad_ws_, stream_);
                    else if (i == 0 && feat_mean_[l]) {
                        // the first conv reads the frozen features: centred weight gradient (WgradCenter)
                        tap_border_sums(rows_of(hb.dy, batch, g), batch, g, hb.taps, hb.b.has_bn != 0, center_ws_,
                                        tap_sums_, stream_);
                        const WgradCenter center{feat_mean_[l], tap_sums_, batch};
                        conv_wgrad(rows_of(feat_c_[l], batch, g), rows_of(hb.dy, batch, g), hb.taps, g,
                                   hb.grouped ? hb.wg_dense : grads_ + hb.w_off, &center);
                    } else {
                        conv_wgrad(rows_of(hb.x, batch, g), rows_of(hb.dy, batch, g), hb.taps, g,
                                   hb.grouped ? hb.wg_dense : grads_ + hb.w_off);
                    }
                    if (hb.grouped)
                        dense_to_grouped(hb.wg_dense, hb.b.oc, hb.b.ic, hb.b.groups, hb.taps, grads_ + hb.w_off, stream_);
                    if (i > 0) {
                        HeadBlock& prev = branch.blocks[i - 1];
                        ConvEpilogue ep;
                        if (prev.b.has_bn) {
                            ep.bn.channels = prev.b.oc;
                            ep.bn.y = prev.y.base;
                            ep.bn.y_pitch = prev.y.pitch;
                            ep.bn.mean = prev.coef;
                            ep.bn.inv = prev.coef + (long)batch * prev.b.oc;
                            ep.bn.gamma = params_ + prev.g_off;
                            ep.bn.beta = params_ + prev.be_off;
                            ep.bn.grad_part = bn_part_;
                        }
                        if (hb.dw) {
                            dw_conv(rows_of(hb.dy, batch, g), params_ + hb.w_off, hb.taps, -1, g, rows_of(prev.g, batch, g),
                                    ep.bn, stream_);
                        } else {
                            prof_begin();
                            conv_fwd(rows_of(hb.dy, batch, g), hb.w_dgrad, (long)hb.b.ic * hb.taps * hb.kpad_out,
                                     hb.b.ic, hb.b.ic, hb.taps, -1, g, rows_of(prev.g, batch, g), ep, nullptr);
                            prof_end(2.0 * batch * hb.b.oc * hb.b.ic * hb.taps * g.h * g.w,
                                     {3, hb.b.oc, hb.b.ic, hb.taps, g.h, g.w});
                        }
                    }
                }
            }
    }
    cls_pending_ = false;
    if (lanes) join_levels();
    // BatchNorm gamma / beta gradients of every layer, images folded in order (deferred from the folds)
    if (n_bn_jobs_ > 0) bn_param_grad_batch(d_bn_jobs_, n_bn_jobs_, bn_max_c_, batch, stream_);
}

// ------------------------------------------------------------------ loss
// DetectionHead.ProgressiveWeight (DetectionHead.cs:120) for progressive heads, else both weights 1;
// the product and the sum round separately, as in the reference.
void Session::loss_weights(int epoch, float w[2]) const {
    if (!progressive_) {
        w[0] = w[1] = 1.0f;
        return;
    }
    const float t = std::max(1.0f - (float)epoch / (float)std::max(cfg.schedule_epochs - 1, 1), 0.0f);
    const float scaled = t * 0.7f;
    w[0] = scaled + 0.1f;
    w[1] = 1.0f - w[0];
}

// DetectionHead.Loss (DetectionHead.cs:105-115): the one-to-many set with the top-10 assigner; an
// end-to-end head adds the one-to-one set with top-k 1 (7 when progressive) and a second top-1 after
// conflicts.  Each set's output gradients are scaled by its weight.
void Session::launch_losses(int images, int backward, int epoch) {
    float w[2];
    loss_weights(epoch, w);
    const bool split = level_lanes() && loss_stream_;
    const LossSplit sp{loss_stream_, ev_assigned_, ev_box_, ev_cls_};
    for (int set = 0; set < n_sets_; set++) {
        LevelIO lv[3];
        for (int l = 0; l < 3; l++) {
            HeadBlock& bb = branches_[set * 6 + l].blocks.back();
            HeadBlock& cb = branches_[set * 6 + 3 + l].blocks.back();
            lv[l] = LevelIO{bb.y.base, cb.y.base, bb.g.base, cb.g.base, bb.y.pitch, cb.y.pitch, levels_[l],
                            (float)(8 << l), bb.b.has_bias ? grads_ + bb.b_off : nullptr,
                            cb.b.has_bias ? grads_ + cb.b_off : nullptr};
        }
        LossOut lo{d_loss_ + (size_t)4 * B_ * set, d_pos_ + (size_t)B_ * set, d_conn_ + (size_t)B_ * set, nullptr,
                   nullptr, d_ties_ + (size_t)B_ * set};
        const int topk = set == 0 ? 10 : (progressive_ ? 7 : 1), topk2 = set == 0 ? 10 : 1;
        detection_loss(lv, 3, images, cfg.num_classes, cfg.reg_max, d_truth_, d_box_off_, std::max(1, cfg.max_boxes),
                       topk, topk2, cfg.end_to_end ? w[set] : 1.0f, backward, loss_ws_, lo, stream_, rnd_, x3_,
                       split ? &sp : nullptr);
        // the next set reuses the workspace; without a backward nothing else waits for the class part
        if (split && (set + 1 < n_sets_ || !backward)) SY_CUDA(cudaStreamWaitEvent(stream_, ev_cls_, 0));
    }
    cls_pending_ = split && backward;
}

// Per image the reported parts are a.Part * w0 + b.Part * w1 in float (DetectionHead.cs:114), summed
// over the images in double; positives add up; `finite` checks every image's total (YoloTrainer.cs:193).
// `head` is one rank's exchange-record head ([set][image][4] loss parts, then [set][image] positives and
// box connections); the sums accumulate into the outputs, so ranks are added in rank order.
void Session::combine_losses(const float* head, int images, int epoch, double* box, double* cls, double* dfl,
                             long* positives, int* connected, bool* finite, long* near_ties) const {
    float w[2];
    loss_weights(epoch, w);
    const int* pos = reinterpret_cast<const int*>(head + 8 * B_);
    const int* conn = pos + 2 * B_;
    const int* ties = conn + 2 * B_;
    for (int b = 0; b < images; b++) {
        float part[3];
        for (int k = 0; k < 3; k++) {
            part[k] = head[4 * b + k];
            if (n_sets_ == 2) {
                const float one = head[4 * ((size_t)B_ + b) + k] * w[1];
                part[k] = part[k] * w[0] + one;
            }
        }
        *box += part[0];
        *cls += part[1];
        *dfl += part[2];
        if (!std::isfinite(part[0] + part[1] + part[2])) *finite = false;
        for (int set = 0; set < n_sets_; set++) {
            *positives += pos[(size_t)B_ * set + b];
            *near_ties += ties[(size_t)B_ * set + b];
            if (conn[(size_t)B_ * set + b]) *connected |= 1 << set;
        }
    }
}

int Session::get_optimizer_steps(int32_t steps[3]) const {
    if (!steps) throw SyError(SY_ERR_INVALID_ARGUMENT, "steps missing");
    for (int g = 0; g < 3; g++) steps[g] = adam_steps_[g];
    return SY_OK;
}

int Session::set_optimizer_steps(const int32_t steps[3]) {
    if (!steps) throw SyError(SY_ERR_INVALID_ARGUMENT, "steps missing");
    for (int g = 0; g < 3; g++)
        if (steps[g] < 0) throw SyError(SY_ERR_INVALID_ARGUMENT, "optimizer step counts must not be negative");
    for (int g = 0; g < 3; g++) adam_steps_[g] = steps[g];
    return SY_OK;
}

int Session::set_epoch(int epoch) {
    if (epoch < 0) throw SyError(SY_ERR_INVALID_ARGUMENT, "epoch must not be negative");
    epoch_ = epoch;
    return SY_OK;
}

// ------------------------------------------------------------------ step
// Validate and upload the step's ground truth and images, run the frozen trunk (or stage cached
// features); shared by the training step and the loss evaluation.
void Session::prepare_inputs(const uint8_t* rgb, bool rgb_on_device, const float* const* features,
                             const sy_box* boxes, const int32_t* counts, int images, bool defer_backbone) {
    if (cfg.world_size > 1 && !comm_)
        throw SyError(SY_ERR_COMM, "the data-parallel communicator was aborted after a failed step; destroy the session");
    if (images < 1 || images > B_) throw SyError(SY_ERR_INVALID_ARGUMENT, "images out of range");
    if (!counts || (!boxes && images > 0)) throw SyError(SY_ERR_INVALID_ARGUMENT, "counts / boxes missing");
    SY_CUDA(cudaSetDevice(device_));
    feat_events_ = false;
    // validate and stage ground truth (TrainingDataset.ParseLabels guarantees, DetectionLoss.cs:51)
    long k = 0;
    h_box_off_[0] = 0;
    for (int b = 0; b < images; b++) {
        if (counts[b] < 0 || counts[b] > cfg.max_boxes) throw SyError(SY_ERR_INVALID_ARGUMENT, "box count out of range");
        for (int j = 0; j < counts[b]; j++, k++) {
            const sy_box& bx = boxes[k];
            if (bx.class_id < 0 || bx.class_id >= cfg.num_classes)
                throw SyError(SY_ERR_INVALID_ARGUMENT, "class id out of range");
            if (!std::isfinite(bx.x1) || !std::isfinite(bx.y1) || !std::isfinite(bx.x2) || !std::isfinite(bx.y2))
                throw SyError(SY_ERR_INVALID_ARGUMENT, "box coordinates not finite");
            h_truth_[k] = TruthBox{bx.class_id, bx.x1, bx.y1, bx.x2, bx.y2};
        }
        h_box_off_[b + 1] = (int)k;
    }
    if (rgb && (cfg.backbone == SY_BACKBONE_NONE || !backbone_ready_))
        throw SyError(SY_ERR_INVALID_ARGUMENT, "backbone weights not set");
    // where this step's images come from: the caller's device buffer, a prefetched copy, or a copy made now
    // (pinned caller memory directly, pageable memory through pinned staging)
    const size_t bytes = rgb ? (size_t)images * cfg.image_size * cfg.image_size * 3 : 0;
    const uint8_t* src = nullptr;
    ImageSlot* slot = nullptr;
    bool copy_now = false;
    if (rgb) {
        if (!rgb_on_device)
            for (ImageSlot& sl : slots_)
                if (sl.ready && sl.host == rgb && sl.images == images) slot = &sl;
        if (rgb_on_device) {
            src = rgb;
        } else if (slot) {
            src = slot->dev;
        } else {
            cudaPointerAttributes attr;
            const bool pinned = cudaPointerGetAttributes(&attr, rgb) == cudaSuccess && attr.type == cudaMemoryTypeHost;
            cudaGetLastError();
            if (!pinned) {
                std::memcpy(h_rgb_, rgb, bytes);
                rgb = h_rgb_;
            }
            src = d_rgb_;
            copy_now = true;
        }
    }
    prof_n_ = 0;
    SY_CUDA(cudaEventRecord(ev0_, stream_));
    if (k > 0)
        SY_CUDA(cudaMemcpyAsync(d_truth_, h_truth_, sizeof(TruthBox) * k, cudaMemcpyHostToDevice, stream_));
    SY_CUDA(cudaMemcpyAsync(d_box_off_, h_box_off_, sizeof(int) * (images + 1), cudaMemcpyHostToDevice, stream_));
    SY_CUDA(cudaMemsetAsync(d_flags_, 0, sizeof(int) * 16, stream_));
    h_images_[0] = images;
    SY_CUDA(cudaMemcpyAsync(d_images_, h_images_, sizeof(int), cudaMemcpyHostToDevice, stream_));
    if (rgb) {
        *h_rgb_ref_ = src;
        SY_CUDA(cudaMemcpyAsync(d_rgb_ref_, h_rgb_ref_, sizeof(void*), cudaMemcpyHostToDevice, stream_));
    }
    if (copy_stream_) SY_CUDA(cudaEventRecord(ev_uploaded_, stream_));
    if (rgb) {
        if (slot) {
            // prefetched: the compute stream waits for the copy stream's copy of this batch
            issue_prefetch(*slot);
            SY_CUDA(cudaStreamWaitEvent(stream_, slot->copied, 0));
            slot->ready = false;
            consuming_ = slot;
        } else if (copy_now) {
            SY_CUDA(cudaMemcpyAsync(d_rgb_, rgb, bytes, cudaMemcpyHostToDevice, stream_));
        }
        // the copies of batches prefetched for later calls start now, behind this call's uploads
        for (ImageSlot& sl : slots_)
            if (sl.pending) issue_prefetch(sl);
        if (!defer_backbone) forward_backbone(images);
    } else {
        if (!features) throw SyError(SY_ERR_INVALID_ARGUMENT, "features missing");
        for (int l = 0; l < 3; l++) {
            const Grid& g = levels_[l];
            const size_t n = (size_t)images * feat_ch_[l] * g.h * g.w;
            SY_CUDA(cudaMemcpyAsync(feat_stage_, features[l], n * sizeof(float), cudaMemcpyHostToDevice, stream_));
            nchw_to_padded(feat_stage_, images, feat_ch_[l], g, features_[l], stream_, rnd_);
        }
    }
}

int Session::step(const uint8_t* rgb, bool rgb_on_device, const float* const* features, const sy_box* boxes,
                  const int32_t* counts, int images, sy_step_stats* out) {
    const bool graph = use_graphs_ && !prof_;
    prepare_inputs(rgb, rgb_on_device, features, boxes, counts, images, graph);
    const bool trunk = rgb != nullptr;
    auto device_work = [&] {
        if (graph && trunk) forward_backbone(images);
        forward_head(images);
        launch_losses(images, 1, epoch_);
        backward_head(images);
    };
    if (!graph) {
        device_work();
    } else {
        float w[2];
        loss_weights(epoch_, w);
        // the stem reads the image address from d_rgb_ref_: one graph for every image buffer
        const GraphKey key{images, trunk ? (const void*)d_rgb_ref_ : nullptr, w[0], w[1]};
        auto it = graphs_.find(key);
        bool captured = false;
        if (it == graphs_.end() && graph_seen_[key]++ > 0 && graphs_.size() < 16) {
            cudaGraph_t g = nullptr;
            const long long launches0 = launch_count();
            SY_CUDA(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            try {
                device_work();
            } catch (...) {
                cudaStreamEndCapture(stream_, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            SY_CUDA(cudaStreamEndCapture(stream_, &g));
            cudaGraphExec_t exec = nullptr;
            const cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
            cudaGraphDestroy(g);
            SY_CUDA(e);
            it = graphs_.emplace(key, exec).first;
            // the capture counted the graph's kernel nodes once (launch_count): replays add them again
            graph_nodes_[key] = launch_count() - launches0;
            captured = true;
        }
        if (it != graphs_.end()) {
            SY_CUDA(cudaGraphLaunch(it->second, stream_));
            if (!captured) add_launches(graph_nodes_[key]);
        } else {
            device_work();
        }
    }
    release_images();
    // Data-parallel exchange, all enqueued before one host wait: the gradient bucket summed over ranks
    // (so the finiteness check, the checksum and the kept copy all see the global gradient), then one
    // all-gather of every rank's exchange record (loss parts, positives, connections, image count and the
    // per-image BatchNorm statistics), whose heads come back to the host in one strided copy.
    const int ranks = comm_ ? cfg.world_size : 1;
    if (comm_) {
        int r = nccl_->AllReduce(grads_, grads_, (size_t)n_params, kNcclFloat, kNcclSum, comm_, stream_);
        if (r != 0) throw SyError(SY_ERR_COMM, std::string("ncclAllReduce: ") + nccl_->GetErrorString(r));
    }
    SY_CUDA(cudaMemcpyAsync(last_grads_, grads_, sizeof(float) * n_params, cudaMemcpyDeviceToDevice, stream_));
    check_finite(grads_, n_params, d_flags_ + 1, stream_);
    abs_sum_partials(grads_, n_params, d_abs_, stream_);
    const size_t head_bytes = sizeof(float) * (size_t)head_floats_;
    const float* records = rec_;
    if (comm_) {
        int r = nccl_->AllGather(rec_, rec_gather_, (size_t)rec_floats_, kNcclFloat, comm_, stream_);
        if (r != 0) throw SyError(SY_ERR_COMM, std::string("ncclAllGather: ") + nccl_->GetErrorString(r));
        records = rec_gather_;
        SY_CUDA(cudaMemcpy2DAsync(h_rec_, head_bytes, rec_gather_, sizeof(float) * (size_t)rec_floats_, head_bytes,
                                  ranks, cudaMemcpyDeviceToHost, stream_));
    } else {
        SY_CUDA(cudaMemcpyAsync(h_rec_, rec_, head_bytes, cudaMemcpyDeviceToHost, stream_));
    }
    SY_CUDA(cudaMemcpyAsync(h_flags_, d_flags_, sizeof(int) * 16, cudaMemcpyDeviceToHost, stream_));
    SY_CUDA(cudaMemcpyAsync(h_abs_, d_abs_, sizeof(double) * kAbsSumBlocks, cudaMemcpyDeviceToHost, stream_));
    wait_stream("the gradient all-reduce and record all-gather");
    if (h_flags_[0]) throw SyError(SY_ERR_DEVICE, "device wait limit exceeded (code " + std::to_string(h_flags_[0]) + ")");
    double box = 0, cls = 0, dfl = 0, abs_sum = 0;
    long positives = 0, near_ties = 0;
    int connected = 0;   // bit s: the box branch of set s received a gradient
    bool finite = h_flags_[1] == 0;
    bool same_images = true;
    for (int r = 0; r < ranks; r++) {
        const float* head = h_rec_ + (size_t)head_floats_ * r;
        const int n = reinterpret_cast<const int*>(head + 8 * B_)[6 * B_];
        // the running-statistics fold below walks `images` images of every rank in rank order
        if (n != images) {
            same_images = false;
            break;
        }
        combine_losses(head, images, epoch_, &box, &cls, &dfl, &positives, &connected, &finite, &near_ties);
    }
    for (int i = 0; i < kAbsSumBlocks; i++) abs_sum += h_abs_[i];
    const int global_images = images * ranks;
    if (!same_images) {
        SY_CUDA(cudaMemsetAsync(grads_, 0, sizeof(float) * n_params, stream_));
        SY_CUDA(cudaStreamSynchronize(stream_));
        throw SyError(SY_ERR_INVALID_ARGUMENT, "data-parallel ranks must step the same number of images");
    }
    if (!finite) {
        SY_CUDA(cudaMemsetAsync(grads_, 0, sizeof(float) * n_params, stream_));
        SY_CUDA(cudaStreamSynchronize(stream_));
        throw SyError(SY_ERR_NONFINITE, "non-finite loss or gradient; parameters not updated");
    }
    // BN running statistics, global images in order (HeadOperations.cs:164-165): every rank folds rank 0's
    // images, then rank 1's ..., from the gathered records
    if (n_bn_jobs_ > 0)
        bn_running_update_batch(d_bn_jobs_, n_bn_jobs_, bn_max_c_, records + head_floats_, rec_floats_, ranks, images,
                                cfg.bn_momentum, stream_);
    // update: flags [2..4] gate the optimizer groups (class branches, cv2, one2one_cv2), [5..7] hold
    // their AdamW step counts (TrainingParameter steps only when it received a gradient)
    const int has[3] = {1, connected & 1, (connected >> 1) & 1};
    for (int gi = 0; gi < 3; gi++) {
        h_flags_[2 + gi] = has[gi];
        if (cfg.optimizer == SY_OPT_ADAMW && has[gi]) adam_steps_[gi]++;
        h_flags_[5 + gi] = adam_steps_[gi];
    }
    h_flags_[1] = 0;
    SY_CUDA(cudaMemcpyAsync(d_flags_ + 1, h_flags_ + 1, sizeof(int) * 7, cudaMemcpyHostToDevice, stream_));
    optimizer_step(cfg.optimizer, params_, vel_, vel2_, grads_, d_segs_, nsegs_, d_flags_ + 2, d_flags_ + 5, cfg.lr,
                   cfg.momentum, cfg.weight_decay, cfg.beta1, cfg.beta2, cfg.adam_eps, 1.0f / (float)global_images,
                   d_flags_ + 1, stream_);
    refresh_head_weights();
    SY_CUDA(cudaMemcpyAsync(h_flags_, d_flags_, sizeof(int) * 2, cudaMemcpyDeviceToHost, stream_));
    SY_CUDA(cudaEventRecord(ev1_, stream_));
    SY_CUDA(cudaStreamSynchronize(stream_));
    prof_collect();
    last_batch_ = images;
    if (out) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev0_, ev1_);
        out->box = box;
        out->cls = cls;
        out->dfl = dfl;
        out->positives = positives;
        out->images = global_images;
        out->box_has_grad = connected;
        out->grad_checksum = abs_sum / global_images;
        out->device_ms = ms;
        out->near_ties = near_ties;
    }
    if (h_flags_[0]) throw SyError(SY_ERR_DEVICE, "device wait limit exceeded");
    if (h_flags_[1]) throw SyError(SY_ERR_NONFINITE, "non-finite parameters after the update");
    return SY_OK;
}

// ------------------------------------------------------------------ convolution passes
// 3xTF32: every FP32 operand x = big + small with big = x rounded to TF32 and small = x - big (exact);
// the tensor core's TF32 products of (small, big), (big, small) and (big, big) are accumulated in that
// order (smallest first) through the epilogue's pre-add, and only the last pass applies the layer's
// bias / activation / residual / BatchNorm hooks / parity copy.  The dropped small x small term is
// below FP32 rounding.
View Session::split_view(const View& v, int slot, View* small) {
    tf32_split(v, sp_[slot], sp_[slot + 1], stream_);
    *small = View{sp_[slot + 1], v.pitch, v.channels, v.rows};
    return View{sp_[slot], v.pitch, v.channels, v.rows};
}

const float* Session::split_weights(const float* wk, long n, const float** small) {
    tf32_split(View{const_cast<float*>(wk), (int)n, (int)n, 1}, wsp_[0], wsp_[1], stream_);
    *small = wsp_[1];
    return wsp_[0];
}

void Session::conv_fwd(const View& in, const float* wk, long wk_floats, int n_rows, int n_out, int taps, int sign,
                       const Grid& grid, const View& out, const ConvEpilogue& ep, const PhaseOut* po) {
    if (!x3_) {
        conv_tc_forward(in, wk, n_rows, n_out, taps, sign, grid, out, ep, d_flags_, stream_, po);
        return;
    }
    View as;
    const View ab = split_view(in, 0, &as);
    const float* ws = nullptr;
    const float* wb = split_weights(wk, wk_floats, &ws);
    ConvEpilogue raw;
    raw.mask_halo = ep.mask_halo;
    conv_tc_forward(as, wb, n_rows, n_out, taps, sign, grid, out, raw, d_flags_, stream_, nullptr);
    raw.pre = out.base;
    raw.pre_pitch = out.pitch;
    conv_tc_forward(ab, ws, n_rows, n_out, taps, sign, grid, out, raw, d_flags_, stream_, nullptr);
    ConvEpilogue last = ep;
    last.pre = out.base;
    last.pre_pitch = out.pitch;
    conv_tc_forward(ab, wb, n_rows, n_out, taps, sign, grid, out, last, d_flags_, stream_, po);
}

void Session::conv_strided(const View& phase_in, long plane_rows, long m_rows, const float* wk, long wk_floats,
                           int oc, const Grid& gout, const View& out, const ConvEpilogue& ep, const PhaseOut* po) {
    if (!x3_) {
        conv_tc_strided(phase_in, plane_rows, m_rows, wk, oc, gout, out, ep, d_flags_, stream_, po);
        return;
    }
    View as;
    const View ab = split_view(phase_in, 0, &as);
    const float* ws = nullptr;
    const float* wb = split_weights(wk, wk_floats, &ws);
    ConvEpilogue raw;
    raw.mask_halo = ep.mask_halo;
    conv_tc_strided(as, plane_rows, m_rows, wb, oc, gout, out, raw, d_flags_, stream_, nullptr);
    raw.pre = out.base;
    raw.pre_pitch = out.pitch;
    conv_tc_strided(ab, plane_rows, m_rows, ws, oc, gout, out, raw, d_flags_, stream_, nullptr);
    ConvEpilogue last = ep;
    last.pre = out.base;
    last.pre_pitch = out.pitch;
    conv_tc_strided(ab, plane_rows, m_rows, wb, oc, gout, out, last, d_flags_, stream_, po);
}

void Session::conv_wgrad(const View& x, const View& dy, int taps, const Grid& grid, float* dw,
                         const WgradCenter* center) {
    if (!x3_) {
        conv_tc_wgrad(x, dy, taps, grid, dw, wgrad_ws_, d_flags_, stream_, 0, center);
        return;
    }
    View xs, ds;
    const View xb = split_view(x, 0, &xs);
    const View db = split_view(dy, 2, &ds);
    conv_tc_wgrad(xs, db, taps, grid, dw, wgrad_ws_, d_flags_, stream_, 0, center);
    conv_tc_wgrad(xb, ds, taps, grid, dw, wgrad_ws_, d_flags_, stream_, 1);
    conv_tc_wgrad(xb, db, taps, grid, dw, wgrad_ws_, d_flags_, stream_, 1);
}

// ------------------------------------------------------------------ loss evaluation
int Session::evaluate(const uint8_t* rgb, bool rgb_on_device, const float* const* features, const sy_box* boxes,
                      const int32_t* counts, int images, sy_step_stats* out) {
    prepare_inputs(rgb, rgb_on_device, features, boxes, counts, images);
    forward_head(images, false);
    release_images();
    // EvaluateLoss passes epoch 0 to DetectionHead.Loss (YoloTrainer.cs:243)
    launch_losses(images, 0, 0);
    // every rank's record head (loss parts, positives, image count) in one all-gather, combined on the host
    // in global image order, so that every rank reports the same sums
    const int ranks = comm_ ? cfg.world_size : 1;
    const size_t head_bytes = sizeof(float) * (size_t)head_floats_;
    if (comm_) {
        int r = nccl_->AllGather(rec_, rec_gather_, (size_t)head_floats_, kNcclFloat, comm_, stream_);
        if (r != 0) throw SyError(SY_ERR_COMM, std::string("ncclAllGather: ") + nccl_->GetErrorString(r));
        SY_CUDA(cudaMemcpyAsync(h_rec_, rec_gather_, head_bytes * ranks, cudaMemcpyDeviceToHost, stream_));
    } else {
        SY_CUDA(cudaMemcpyAsync(h_rec_, rec_, head_bytes, cudaMemcpyDeviceToHost, stream_));
    }
    SY_CUDA(cudaMemcpyAsync(h_flags_, d_flags_, sizeof(int) * 16, cudaMemcpyDeviceToHost, stream_));
    SY_CUDA(cudaEventRecord(ev1_, stream_));
    wait_stream("the loss all-gather");
    if (h_flags_[0]) throw SyError(SY_ERR_DEVICE, "device wait limit exceeded (code " + std::to_string(h_flags_[0]) + ")");
    double box = 0, cls = 0, dfl = 0;
    long positives = 0, near_ties = 0;
    int connected = 0, total_images = 0;
    bool finite = true;
    for (int r = 0; r < ranks; r++) {
        const float* head = h_rec_ + (size_t)head_floats_ * r;
        const int n = reinterpret_cast<const int*>(head + 8 * B_)[6 * B_];
        if (n < 1 || n > B_) throw SyError(SY_ERR_COMM, "corrupt exchange record from rank " + std::to_string(r));
        combine_losses(head, n, 0, &box, &cls, &dfl, &positives, &connected, &finite, &near_ties);
        total_images += n;
    }
    last_batch_ = images;
    if (out) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ev0_, ev1_);
        *out = sy_step_stats{};
        out->box = box;
        out->cls = cls;
        out->dfl = dfl;
        out->positives = positives;
        out->images = total_images;
        out->near_ties = near_ties;
        out->device_ms = ms;
    }
    return SY_OK;
}

// ------------------------------------------------------------------ image prefetch
int Session::prefetch_images(const uint8_t* rgb, int images) {
    if (!rgb) throw SyError(SY_ERR_INVALID_ARGUMENT, "images missing");
    if (images < 1 || images > B_) throw SyError(SY_ERR_INVALID_ARGUMENT, "images out of range");
    if (cfg.backbone == SY_BACKBONE_NONE) throw SyError(SY_ERR_INVALID_ARGUMENT, "the session has no trunk");
    SY_CUDA(cudaSetDevice(device_));
    for (ImageSlot& sl : slots_)
        if (sl.ready && sl.host == rgb && sl.images == images) return SY_OK;   // already on its way
    const size_t cap = (size_t)B_ * cfg.image_size * cfg.image_size * 3;
    const size_t bytes = (size_t)images * cfg.image_size * cfg.image_size * 3;
    if (!copy_stream_) {
        SY_CUDA(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
        SY_CUDA(cudaEventCreateWithFlags(&ev_uploaded_, cudaEventDisableTiming));
        SY_CUDA(cudaEventRecord(ev_uploaded_, stream_));
    }
    ImageSlot& sl = slots_[next_slot_];
    next_slot_ ^= 1;
    if (!sl.dev) {
        SY_CUDA(cudaMalloc(&sl.dev, cap));
        SY_CUDA(cudaEventCreateWithFlags(&sl.copied, cudaEventDisableTiming));
        SY_CUDA(cudaEventCreateWithFlags(&sl.released, cudaEventDisableTiming));
    }
    sl.ready = false;
    sl.pending = false;
    cudaPointerAttributes attr;
    const bool pinned = cudaPointerGetAttributes(&attr, rgb) == cudaSuccess && attr.type == cudaMemoryTypeHost;
    cudaGetLastError();
    const uint8_t* src = rgb;
    if (!pinned) {
        // pageable memory: stage it (the staging buffer is free once the previous copy from it ended)
        if (!sl.pinned) SY_CUDA(cudaMallocHost(&sl.pinned, cap));
        SY_CUDA(cudaEventSynchronize(sl.copied));
        std::memcpy(sl.pinned, rgb, bytes);
        src = sl.pinned;
    }
    sl.host = rgb;
    sl.src = src;
    sl.images = images;
    sl.ready = true;
    sl.pending = true;
    return SY_OK;
}

void Session::issue_prefetch(ImageSlot& sl) {
    if (!sl.pending) return;
    // the previous batch in this slot has been read by its consumer's device work, and this call's small
    // uploads have landed (the copy engine serves eligible copies in turn, so a large copy that became
    // eligible first would hold them, and the step behind them, for its whole length)
    if (sl.used) SY_CUDA(cudaStreamWaitEvent(copy_stream_, sl.released, 0));
    SY_CUDA(cudaStreamWaitEvent(copy_stream_, ev_uploaded_, 0));
    const size_t bytes = (size_t)sl.images * cfg.image_size * cfg.image_size * 3;
    SY_CUDA(cudaMemcpyAsync(sl.dev, sl.src, bytes, cudaMemcpyHostToDevice, copy_stream_));
    SY_CUDA(cudaEventRecord(sl.copied, copy_stream_));
    sl.pending = false;
}

// After the device work that read a prefetched batch has been enqueued: the slot may be refilled once it ends.
void Session::release_images() {
    if (!consuming_) return;
    SY_CUDA(cudaEventRecord(consuming_->released, stream_));
    consuming_->used = true;
    consuming_ = nullptr;
}

// ------------------------------------------------------------------ inference
// DecodeIndexed's option checks (YoloDetector.cs:542); with `detector` also the YoloDetector constructor's
// (:214: confidence and IoU threshold finite and in [0, 1]).  The static decode takes any threshold, NaN
// included (no candidate is then below the confidence threshold, and no overlap above the IoU threshold).
DetectOptions detect_options(const sy_detect_options* o, bool detector) {
    if (!o) throw SyError(SY_ERR_INVALID_ARGUMENT, "detect options missing");
    if (detector && (!std::isfinite(o->confidence) || o->confidence < 0.0f || o->confidence > 1.0f))
        throw SyError(SY_ERR_INVALID_ARGUMENT, "confidence must be between 0 and 1");
    if (detector && (!std::isfinite(o->iou_threshold) || o->iou_threshold < 0.0f || o->iou_threshold > 1.0f))
        throw SyError(SY_ERR_INVALID_ARGUMENT, "iou_threshold must be between 0 and 1");
    if (o->max_detections < 1 || o->max_detections > kMaxDetections)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "max_detections must be in [1, 65536]");
    if (o->max_candidates < 1) throw SyError(SY_ERR_INVALID_ARGUMENT, "max_candidates must be positive");
    return DetectOptions{o->confidence, o->iou_threshold, o->max_detections, o->max_candidates,
                         o->class_agnostic ? 1 : 0};
}

DetectTransform detect_transform(const sy_letterbox& t) {
    if (t.source_width <= 0 || t.source_height <= 0 || t.target_width <= 0 || t.target_height <= 0 ||
        !std::isfinite(t.scale_x) || !std::isfinite(t.scale_y) || t.scale_x <= 0.0f || t.scale_y <= 0.0f)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "invalid letterbox transform");
    return DetectTransform{t.scale_x, t.scale_y, (float)t.pad_x, (float)t.pad_y, (float)t.source_width,
                           (float)t.source_height};
}

void Session::ensure_detect(int max_det) {
    const int nc = cfg.num_classes;
    if (!det_tf_) {
        if (cfg.end_to_end) {
            det_dec_ = static_cast<float*>(dalloc(sizeof(float) * (size_t)B_ * (nc + 4) * anchors_));
            det_e2e_ = static_cast<float*>(dalloc(sizeof(float) * (size_t)B_ * std::min(kModelMaxDet, anchors_) * 6));
        }
        det_tf_ = static_cast<DetectTransform*>(dalloc(sizeof(DetectTransform) * (size_t)B_));
        det_counts_ = static_cast<int*>(dalloc(sizeof(int) * (size_t)B_));
        det_err_ = static_cast<int*>(dalloc(sizeof(int)));
    }
    if (max_det <= det_cap_) return;
    if (det_ws_) cudaFree(det_ws_);
    if (det_out_) cudaFree(det_out_);
    det_ws_ = nullptr;
    det_out_ = nullptr;
    det_cap_ = 0;
    const int count = cfg.end_to_end ? std::min(kModelMaxDet, anchors_) : anchors_;
    size_t ws = detections_workspace_bytes(B_, count, max_det);
    if (cfg.end_to_end) ws = std::max(ws, end_to_end_workspace_bytes(B_, anchors_, nc, kModelMaxDet));
    SY_CUDA(cudaMalloc(&det_ws_, ws));
    SY_CUDA(cudaMalloc(&det_out_, sizeof(DetOut) * (size_t)B_ * max_det));
    det_cap_ = max_det;
}

// PtModel.Detect (PtModel.cs:444-503) on this head: the one-to-many branches, or the one-to-one branches of
// an end-to-end head (decoded as x1, y1, x2, y2 and passed through EndToEndTopK with the model's max_det of
// 300), then YoloDetector.DecodeIndexed with the channels-first (raw) or end-to-end layout.
int Session::detect(const uint8_t* rgb, bool rgb_on_device, const float* const* features, int images,
                    const sy_letterbox* transforms, const sy_detect_options* options, sy_detection* out,
                    int32_t* counts, double* timing) {
    static_assert(sizeof(DetOut) == sizeof(sy_detection), "DetOut mirrors sy_detection");
    if (!out || !counts) throw SyError(SY_ERR_INVALID_ARGUMENT, "detect: output missing");
    if (images < 1 || images > B_) throw SyError(SY_ERR_INVALID_ARGUMENT, "images out of range");
    const DetectOptions o = detect_options(options, true);
    std::vector<DetectTransform> tf(images);
    for (int b = 0; b < images; b++) {
        const int s = cfg.image_size;
        tf[b] = transforms ? detect_transform(transforms[b]) : detect_transform(sy_letterbox{s, s, s, s, 1.f, 1.f, 0, 0});
    }
    SY_CUDA(cudaSetDevice(device_));
    ensure_detect(o.max_det);
    const std::vector<int32_t> no_boxes(images, 0);
    const sy_box unused{};
    prepare_inputs(rgb, rgb_on_device, features, &unused, no_boxes.data(), images);
    forward_head(images, false);
    release_images();
    last_batch_ = images;
    const int nc = cfg.num_classes, set = n_sets_ - 1;
    const bool e2e = cfg.end_to_end != 0;
    DetectLevelSrc lv[3];
    for (int l = 0; l < 3; l++) {
        const Grid& g = levels_[l];
        const View& by = branches_[set * 6 + l].blocks.back().y;
        const View& cy = branches_[set * 6 + 3 + l].blocks.back().y;
        const long interior = (long)(g.wp + 1);
        lv[l] = DetectLevelSrc{by.base + interior * by.pitch, cy.base + interior * cy.pitch,
                               {(long)g.rows * by.pitch, 1, (long)g.wp * by.pitch, by.pitch},
                               {(long)g.rows * cy.pitch, 1, (long)g.wp * cy.pitch, cy.pitch}, g.h, g.w,
                               (float)(8 << l)};
    }
    SY_CUDA(cudaMemcpyAsync(det_tf_, tf.data(), sizeof(DetectTransform) * images, cudaMemcpyHostToDevice, stream_));
    SY_CUDA(cudaMemsetAsync(det_err_, 0, sizeof(int), stream_));
    SY_CUDA(cudaEventRecord(ev_post_, stream_));
    if (e2e) {
        const int k = std::min(kModelMaxDet, anchors_);
        head_decode(lv, 3, images, cfg.reg_max, nc, 1, det_dec_, stream_);
        end_to_end_topk(det_dec_, images, nc + 4, anchors_, nc, kModelMaxDet, det_e2e_, det_ws_, stream_);
        decode_detections(det_e2e_, images, (long)k * 6, 6, 1, k, 0, true, det_tf_, o, det_out_, det_counts_,
                          det_err_, det_ws_, stream_);
    } else {
        // decode fused into the candidate filter: no decoded [image][4 + nc][anchors] tensor
        detect_raw(lv, 3, images, cfg.reg_max, nc, branches_[set * 6 + 3].blocks.back().y.pitch,
                   branches_[set * 6].blocks.back().y.pitch, det_tf_, o, det_out_, det_counts_, det_ws_, stream_);
    }
    SY_CUDA(cudaMemcpyAsync(counts, det_counts_, sizeof(int) * images, cudaMemcpyDeviceToHost, stream_));
    SY_CUDA(cudaMemcpyAsync(out, det_out_, sizeof(DetOut) * (size_t)images * o.max_det, cudaMemcpyDeviceToHost,
                            stream_));
    SY_CUDA(cudaMemcpyAsync(h_flags_, det_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    SY_CUDA(cudaEventRecord(ev1_, stream_));
    SY_CUDA(cudaStreamSynchronize(stream_));
    if (h_flags_[0]) throw SyError(SY_ERR_DEVICE, "detect: class id out of Int32 range");
    if (timing) {
        float all = 0.0f, post = 0.0f;
        cudaEventElapsedTime(&all, ev0_, ev1_);
        cudaEventElapsedTime(&post, ev_post_, ev1_);
        timing[0] = all;
        timing[1] = post;
    }
    return SY_OK;
}

int Session::get_last_head_outputs(int set, int level, float* box, long box_count, float* cls, long cls_count) const {
    if (set < 0 || set >= n_sets_ || level < 0 || level > 2 || !box || !cls)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "set / level / buffers");
    const Grid& g = levels_[level];
    const View& by = branches_[set * 6 + level].blocks.back().y;
    const View& cy = branches_[set * 6 + 3 + level].blocks.back().y;
    const long nb = (long)last_batch_ * 4 * cfg.reg_max * g.h * g.w, nk = (long)last_batch_ * cfg.num_classes * g.h * g.w;
    if (box_count != nb || cls_count != nk) throw SyError(SY_ERR_INVALID_ARGUMENT, "head output size mismatch");
    float* tmp = nullptr;
    SY_CUDA(cudaMalloc(&tmp, sizeof(float) * std::max(nb, nk)));
    padded_to_nchw(by, last_batch_, 4 * cfg.reg_max, g, tmp, stream_);
    cudaError_t e = cudaMemcpyAsync(box, tmp, sizeof(float) * nb, cudaMemcpyDeviceToHost, stream_);
    if (e == cudaSuccess) {
        padded_to_nchw(cy, last_batch_, cfg.num_classes, g, tmp, stream_);
        e = cudaMemcpyAsync(cls, tmp, sizeof(float) * nk, cudaMemcpyDeviceToHost, stream_);
    }
    cudaStreamSynchronize(stream_);
    cudaFree(tmp);
    SY_CUDA(e);
    return SY_OK;
}

// ------------------------------------------------------------------ bounded waits on collectives
// With collectives in flight a peer that has died or stopped stepping would block the stream forever.
// The host polls the stream instead of blocking on it; NCCL's asynchronous error, or no completion within
// comm_timeout_ms, aborts the communicator (ncclCommAbort ends this rank's pending collectives), the stream
// is drained, and the step fails with SY_ERR_COMM.  Without a communicator this is a plain synchronize.
void Session::wait_stream(const char* what) {
    if (!comm_) {
        SY_CUDA(cudaStreamSynchronize(stream_));
        return;
    }
    using clock = std::chrono::steady_clock;
    const auto start = clock::now();
    const auto deadline = start + std::chrono::milliseconds(comm_timeout_ms_);
    for (;;) {
        const cudaError_t e = cudaStreamQuery(stream_);
        if (e == cudaSuccess) return;
        if (e != cudaErrorNotReady) SY_CUDA(e);
        int async = 0;
        if (nccl_->CommGetAsyncError && nccl_->CommGetAsyncError(comm_, &async) == 0 && async != 0 &&
            async != kNcclInProgress)
            abort_comm(std::string("NCCL reported ") + nccl_->GetErrorString(async) + " during " + what);
        if (clock::now() > deadline)
            abort_comm(std::string(what) + " did not complete within " + std::to_string(comm_timeout_ms_) +
                       " ms (a peer rank stopped or died)");
        // a step's device work takes milliseconds: poll without sleeping for the first 50 ms (a sleep would
        // add its own wake-up latency to every step), then every 50 us
        if (clock::now() - start < std::chrono::milliseconds(50))
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

void Session::abort_comm(const std::string& reason) {
    void* comm = comm_;
    comm_ = nullptr;   // no further collectives: later steps fail with SY_ERR_COMM
    nccl_->CommAbort(comm);
    // the aborted collectives return; give the stream a bounded time to drain
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(10);
    while (cudaStreamQuery(stream_) == cudaErrorNotReady && std::chrono::steady_clock::now() < deadline)
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    cudaGetLastError();
    throw SyError(SY_ERR_COMM, reason + "; the communicator was aborted");
}

// ------------------------------------------------------------------ conv launch timing
void Session::prof_begin() {
    if (!prof_) return;
    while ((int)prof_ev_.size() < 2 * (prof_n_ + 1)) {
        cudaEvent_t e;
        SY_CUDA(cudaEventCreate(&e));
        prof_ev_.push_back(e);
    }
    SY_CUDA(cudaEventRecord(prof_ev_[2 * prof_n_], stream_));
}

void Session::prof_end(double flops, const std::array<int, 6>& shape) {
    if (!prof_) return;
    SY_CUDA(cudaEventRecord(prof_ev_[2 * prof_n_ + 1], stream_));
    if ((int)prof_flops_.size() <= prof_n_) {
        prof_flops_.resize(prof_n_ + 1);
        prof_shape_.resize(prof_n_ + 1);
    }
    prof_flops_[prof_n_] = flops;
    prof_shape_[prof_n_] = shape;
    prof_n_++;
}

void Session::prof_collect() {
    if (prof_n_ > 0) {
        prof_last_ms_.assign(prof_n_, 0.0);
        prof_last_gflop_.assign(prof_n_, 0.0);
        prof_last_shape_.assign(prof_shape_.begin(), prof_shape_.begin() + prof_n_);
    }
    for (int k = 0; k < prof_n_; k++) {
        float ms = 0.0f;
        SY_CUDA(cudaEventElapsedTime(&ms, prof_ev_[2 * k], prof_ev_[2 * k + 1]));
        prof_ms_ += ms;
        prof_gflop_ += prof_flops_[k] * 1e-9;
        prof_last_ms_[k] = ms;
        prof_last_gflop_[k] = prof_flops_[k] * 1e-9;
    }
    prof_launches_ += prof_n_;
    prof_n_ = 0;
}

int Session::conv_profile_launches(double* ms, double* gflop, int* shapes, int capacity, int* count) const {
    const int n = (int)prof_last_ms_.size();
    if (count) *count = n;
    for (int k = 0; k < std::min(n, capacity); k++) {
        if (ms) ms[k] = prof_last_ms_[k];
        if (gflop) gflop[k] = prof_last_gflop_[k];
        if (shapes)
            for (int j = 0; j < 6; j++) shapes[6 * k + j] = prof_last_shape_[k][j];
    }
    return SY_OK;
}

int Session::conv_profile(int enable, double* ms, double* gflop, long* launches) {
    if (ms) *ms = prof_ms_;
    if (gflop) *gflop = prof_gflop_;
    if (launches) *launches = prof_launches_;
    prof_ms_ = prof_gflop_ = 0.0;
    prof_launches_ = 0;
    prof_ = enable != 0;
    return SY_OK;
}

// ------------------------------------------------------------------ tensors
int Session::set_tensor(int index, const float* host, long count) {
    if (index < 0 || index >= (int)tensors.size()) throw SyError(SY_ERR_INVALID_ARGUMENT, "tensor index");
    const TensorEntry& t = tensors[index];
    if (count != t.numel || !host) throw SyError(SY_ERR_INVALID_ARGUMENT, "tensor size mismatch");
    float* dst = (t.kind == 0 ? params_ : buffers_) + t.offset;
    SY_CUDA(cudaMemcpyAsync(dst, host, sizeof(float) * count, cudaMemcpyHostToDevice, stream_));
    if (t.kind == 0) refresh_head_weights();
    SY_CUDA(cudaStreamSynchronize(stream_));
    return SY_OK;
}

int Session::get_tensor(int index, float* host, long count) const {
    if (index < 0 || index >= (int)tensors.size()) throw SyError(SY_ERR_INVALID_ARGUMENT, "tensor index");
    const TensorEntry& t = tensors[index];
    if (count != t.numel || !host) throw SyError(SY_ERR_INVALID_ARGUMENT, "tensor size mismatch");
    const float* src = (t.kind == 0 ? params_ : buffers_) + t.offset;
    SY_CUDA(cudaMemcpy(host, src, sizeof(float) * count, cudaMemcpyDeviceToHost));
    return SY_OK;
}

int Session::set_opt_state(int index, int moment, const float* host, long count) {
    if (index < 0 || index >= (int)tensors.size() || tensors[index].kind != 0 || moment < 0 || moment > 1)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "optimizer state index");
    const TensorEntry& t = tensors[index];
    if (count != t.numel || !host) throw SyError(SY_ERR_INVALID_ARGUMENT, "tensor size mismatch");
    for (long i = 0; i < count; i++)
        if (!std::isfinite(host[i])) throw SyError(SY_ERR_INVALID_ARGUMENT, "optimizer state not finite");
    SY_CUDA(cudaMemcpy((moment ? vel2_ : vel_) + t.offset, host, sizeof(float) * count, cudaMemcpyHostToDevice));
    return SY_OK;
}

int Session::get_opt_state(int index, int moment, float* host, long count) const {
    if (index < 0 || index >= (int)tensors.size() || tensors[index].kind != 0 || moment < 0 || moment > 1)
        throw SyError(SY_ERR_INVALID_ARGUMENT, "optimizer state index");
    const TensorEntry& t = tensors[index];
    if (count != t.numel || !host) throw SyError(SY_ERR_INVALID_ARGUMENT, "tensor size mismatch");
    SY_CUDA(cudaMemcpy(host, (moment ? vel2_ : vel_) + t.offset, sizeof(float) * count, cudaMemcpyDeviceToHost));
    return SY_OK;
}

int Session::get_last_gradients(float* host, long count) const {
    if (count != n_params || !host) throw SyError(SY_ERR_INVALID_ARGUMENT, "gradient size mismatch");
    SY_CUDA(cudaMemcpy(host, last_grads_, sizeof(float) * count, cudaMemcpyDeviceToHost));
    return SY_OK;
}

int Session::get_last_features(int level, float* host, long count) const {
    if (level < 0 || level > 2 || !host) throw SyError(SY_ERR_INVALID_ARGUMENT, "level");
    const Grid& g = levels_[level];
    const long n = (long)last_batch_ * feat_ch_[level] * g.h * g.w;
    if (count != n) throw SyError(SY_ERR_INVALID_ARGUMENT, "feature size mismatch");
    float* tmp = nullptr;
    SY_CUDA(cudaMalloc(&tmp, sizeof(float) * n));
    padded_to_nchw(features_[level], last_batch_, feat_ch_[level], g, tmp, stream_);
    cudaError_t e = cudaMemcpyAsync(host, tmp, sizeof(float) * n, cudaMemcpyDeviceToHost, stream_);
    cudaStreamSynchronize(stream_);
    cudaFree(tmp);
    SY_CUDA(e);
    return SY_OK;
}

}  // namespace sy
