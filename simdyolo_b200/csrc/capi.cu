// extern "C" entry points declared in include/simdyolo_cuda.h.  Every call catches C++ exceptions
// and returns a status code; the message is kept for sy_cuda_last_error.
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "session.h"

namespace sy {
int nccl_unique_id(uint8_t out[128]);
}  // namespace sy

struct sy_session {
    std::unique_ptr<sy::Session> impl;
    std::string error;
};

namespace {

std::mutex g_err_mu;
std::string g_last_error;

void set_global_error(const std::string& m) {
    std::lock_guard<std::mutex> lock(g_err_mu);
    g_last_error = m;
}

}  // namespace

namespace sy {
void set_last_error(const std::string& message) { set_global_error(message); }
}  // namespace sy

namespace {

template <class F>
sy_status guarded(sy_session* s, F&& f) {
    try {
        return f();
    } catch (const sy::SyError& e) {
        if (s) s->error = e.what();
        set_global_error(e.what());
        return e.code;
    } catch (const std::bad_alloc& e) {
        if (s) s->error = "host allocation failed";
        set_global_error("host allocation failed");
        return SY_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        if (s) s->error = e.what();
        set_global_error(e.what());
        return SY_ERR_DEVICE;
    }
}

#define CK(call)                                                                                       \
    do {                                                                                               \
        cudaError_t e_ = (call);                                                                       \
        if (e_ != cudaSuccess)                                                                         \
            throw sy::SyError(e_ == cudaErrorMemoryAllocation ? SY_ERR_OUT_OF_MEMORY : SY_ERR_DEVICE,  \
                              std::string(#call) + ": " + cudaGetErrorString(e_));                     \
    } while (0)

// Device scratch owned by one standalone call.
struct Scratch {
    std::vector<void*> ptrs;
    ~Scratch() {
        for (void* p : ptrs) cudaFree(p);
    }
    template <class T>
    T* get(size_t count) {
        void* p = nullptr;
        CK(cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 256)));
        CK(cudaMemset(p, 0, std::max<size_t>(count * sizeof(T), 256)));
        ptrs.push_back(p);
        return static_cast<T*>(p);
    }
};

sy::View padded(Scratch& s, int n, int c, const sy::Grid& g) {
    const int pitch = (c + 3) / 4 * 4;
    const long rows = (long)n * g.rows;
    return sy::View{s.get<float>((size_t)rows * pitch), pitch, c, rows};
}

void conv_shape_check(int n, int ic, int oc, int h, int w, int k) {
    if (n < 1 || ic < 1 || oc < 1 || h < 1 || w < 1 || !(k == 1 || k == 3))
        throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "conv: batch, channels and size must be positive, k in {1,3}");
    if (ic > 4096 || oc > 4096) throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "conv: too many channels");
}

void check_device(int device) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count)
        throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "invalid CUDA device");
    CK(cudaSetDevice(device));
}

}  // namespace

extern "C" {

sy_status sy_cuda_nccl_unique_id(uint8_t out[128]) {
    if (!out) return SY_ERR_INVALID_ARGUMENT;
    return sy::nccl_unique_id(out);
}

sy_status sy_cuda_create(const sy_config* config, sy_session** out) {
    if (!config || !out) return SY_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    return guarded(nullptr, [&] {
        auto s = std::make_unique<sy_session>();
        s->impl = std::make_unique<sy::Session>(*config);
        *out = s.release();
        return SY_OK;
    });
}

sy_status sy_cuda_destroy(sy_session* session) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    delete session;
    return SY_OK;
}

const char* sy_cuda_last_error(const sy_session* session) {
    if (session) return session->error.c_str();
    std::lock_guard<std::mutex> lock(g_err_mu);
    return g_last_error.c_str();
}

int32_t sy_cuda_tensor_count(const sy_session* session) {
    return session ? (int32_t)session->impl->tensors.size() : 0;
}

sy_status sy_cuda_tensor_info(const sy_session* session, int32_t index, sy_tensor_info* out) {
    if (!session || !out || index < 0 || index >= (int32_t)session->impl->tensors.size())
        return SY_ERR_INVALID_ARGUMENT;
    const sy::TensorEntry& t = session->impl->tensors[index];
    std::memset(out, 0, sizeof(*out));
    std::strncpy(out->name, t.name.c_str(), sizeof(out->name) - 1);
    out->kind = t.kind;
    out->rank = (int32_t)t.shape.size();
    for (size_t i = 0; i < t.shape.size() && i < 4; i++) out->shape[i] = t.shape[i];
    out->numel = t.numel;
    return SY_OK;
}

sy_status sy_cuda_set_tensor(sy_session* session, int32_t index, const float* host, int64_t count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->set_tensor(index, host, (long)count); });
}

sy_status sy_cuda_get_tensor(const sy_session* session, int32_t index, float* host, int64_t count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] { return s->impl->get_tensor(index, host, (long)count); });
}

sy_status sy_cuda_set_optimizer_state(sy_session* session, int32_t index, int32_t moment, const float* host,
                                      int64_t count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->set_opt_state(index, moment, host, (long)count); });
}

sy_status sy_cuda_get_optimizer_state(const sy_session* session, int32_t index, int32_t moment, float* host,
                                      int64_t count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] { return s->impl->get_opt_state(index, moment, host, (long)count); });
}

int64_t sy_cuda_backbone_param_count(const sy_session* session) { return session ? session->impl->n_backbone : 0; }

sy_status sy_cuda_set_backbone(sy_session* session, const float* host, int64_t count) {
    if (!session || !host) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->set_backbone(host, (long)count); });
}

sy_status sy_cuda_step(sy_session* session, const uint8_t* rgb, const sy_box* boxes, const int32_t* counts,
                       int32_t images, sy_step_stats* out) {
    if (!session || !rgb) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->step(rgb, false, nullptr, boxes, counts, images, out); });
}

sy_status sy_cuda_step_device(sy_session* session, const uint8_t* rgb_device, const sy_box* boxes,
                              const int32_t* counts, int32_t images, sy_step_stats* out) {
    if (!session || !rgb_device) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session,
                   [&] { return session->impl->step(rgb_device, true, nullptr, boxes, counts, images, out); });
}

sy_status sy_cuda_step_features(sy_session* session, const float* const features[3], const sy_box* boxes,
                                const int32_t* counts, int32_t images, sy_step_stats* out) {
    if (!session || !features) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session,
                   [&] { return session->impl->step(nullptr, false, features, boxes, counts, images, out); });
}

sy_status sy_cuda_eval_loss(sy_session* session, const uint8_t* rgb, const sy_box* boxes, const int32_t* counts,
                             int32_t images, sy_step_stats* out) {
    if (!session || !rgb) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->evaluate(rgb, false, nullptr, boxes, counts, images, out); });
}

sy_status sy_cuda_eval_loss_features(sy_session* session, const float* const features[3], const sy_box* boxes,
                                     const int32_t* counts, int32_t images, sy_step_stats* out) {
    if (!session || !features) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session,
                   [&] { return session->impl->evaluate(nullptr, false, features, boxes, counts, images, out); });
}

sy_status sy_cuda_detect(sy_session* session, const uint8_t* rgb, int32_t images, const sy_letterbox* transforms,
                         const sy_detect_options* options, sy_detection* out, int32_t* counts, double* timing) {
    if (!session || !rgb) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] {
        return session->impl->detect(rgb, false, nullptr, images, transforms, options, out, counts, timing);
    });
}

sy_status sy_cuda_detect_features(sy_session* session, const float* const features[3], int32_t images,
                                  const sy_letterbox* transforms, const sy_detect_options* options, sy_detection* out,
                                  int32_t* counts, double* timing) {
    if (!session || !features) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] {
        return session->impl->detect(nullptr, false, features, images, transforms, options, out, counts, timing);
    });
}

sy_status sy_cuda_prefetch_images(sy_session* session, const uint8_t* rgb, int32_t images) {
    if (!session || !rgb) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->prefetch_images(rgb, images); });
}

int64_t sy_cuda_launch_count(void) { return sy::launch_count(); }

sy_status sy_cuda_conv_profile(sy_session* session, int32_t enable, double* ms, double* gflop, int64_t* launches) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] {
        long n = 0;
        const int r = session->impl->conv_profile(enable, ms, gflop, &n);
        if (launches) *launches = n;
        return r;
    });
}

sy_status sy_cuda_conv_profile_launches(const sy_session* session, double* ms, double* gflop, int32_t* shapes,
                                        int32_t capacity, int32_t* count) {
    if (!session || capacity < 0) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] {
        int n = 0;
        const int r = s->impl->conv_profile_launches(ms, gflop, shapes, capacity, &n);
        if (count) *count = n;
        return r;
    });
}

sy_status sy_cuda_bench_conv(int32_t device, int32_t kind, int32_t n, int32_t ic, int32_t oc, int32_t h, int32_t w,
                             int32_t k, int32_t iters, double* ms_per_launch) {
    return guarded(nullptr, [&] {
        if (!ms_per_launch || kind < 0 || kind > 2 || iters < 1)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "bench_conv: bad arguments");
        conv_shape_check(n, ic, oc, h, w, k);
        check_device(device);
        Scratch s;
        const sy::Grid g = sy::make_grid(h, w);
        const int taps = k * k;
        sy::View vx = padded(s, n, ic, g), vy = padded(s, n, oc, g);
        // deterministic non-trivial data (values do not matter for timing)
        {
            std::vector<float> hx((size_t)vx.rows * vx.pitch), hy((size_t)vy.rows * vy.pitch);
            for (size_t i = 0; i < hx.size(); i++) hx[i] = (float)((i * 2654435761u) % 1000) * 1e-3f - .5f;
            for (size_t i = 0; i < hy.size(); i++) hy[i] = (float)((i * 40503u) % 1000) * 1e-3f - .5f;
            CK(cudaMemcpy(vx.base, hx.data(), hx.size() * 4, cudaMemcpyHostToDevice));
            CK(cudaMemcpy(vy.base, hy.data(), hy.size() * 4, cudaMemcpyHostToDevice));
        }
        const int kpad_i = (ic + 31) / 32 * 32, kpad_o = (oc + 31) / 32 * 32;
        float* wfwd = s.get<float>((size_t)oc * taps * kpad_i);
        float* wdg = s.get<float>((size_t)ic * taps * kpad_o);
        float* dw = s.get<float>((size_t)oc * ic * taps);
        float* wsp = s.get<float>(sy::wgrad_workspace_floats(ic, oc, taps, vx.rows));
        int* err = s.get<int>(1);
        cudaStream_t st;
        CK(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        cudaEvent_t e0, e1;
        CK(cudaEventCreate(&e0));
        CK(cudaEventCreate(&e1));
        auto run = [&] {
            sy::ConvEpilogue ep;
            if (kind == 0) sy::conv_tc_forward(vx, wfwd, oc, oc, taps, 1, g, vy, ep, err, st);
            else if (kind == 1) sy::conv_tc_forward(vy, wdg, ic, ic, taps, -1, g, vx, ep, err, st);
            else sy::conv_tc_wgrad(vx, vy, taps, g, dw, wsp, err, st);
        };
        run();
        CK(cudaEventRecord(e0, st));
        for (int i = 0; i < iters; i++) run();
        CK(cudaEventRecord(e1, st));
        CK(cudaEventSynchronize(e1));
        float ms = 0.f;
        CK(cudaEventElapsedTime(&ms, e0, e1));
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
        cudaStreamDestroy(st);
        int e = 0;
        CK(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (e) throw sy::SyError(SY_ERR_DEVICE, "conv kernel wait limit exceeded");
        *ms_per_launch = ms / iters;
        return SY_OK;
    });
}

sy_status sy_cuda_set_epoch(sy_session* session, int32_t epoch) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->set_epoch(epoch); });
}

sy_status sy_cuda_get_optimizer_steps(const sy_session* session, int32_t steps[3]) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] { return s->impl->get_optimizer_steps(steps); });
}

sy_status sy_cuda_set_optimizer_steps(sy_session* session, const int32_t steps[3]) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    return guarded(session, [&] { return session->impl->set_optimizer_steps(steps); });
}

sy_status sy_cuda_wait_limit_selftest(int32_t device, int32_t spins, int32_t* code) {
    return guarded(nullptr, [&] {
        if (!code || spins < 1 || spins > (int32_t)sy::kSpinLimit)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "wait_limit_selftest: spins out of range");
        check_device(device);
        Scratch s;
        int* err = s.get<int>(1);
        CK(cudaMemset(err, 0, sizeof(int)));
        sy::wait_limit_selftest((uint32_t)spins, 21, err, 0);
        CK(cudaDeviceSynchronize());
        int e = 0;
        CK(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
        *code = e;
        if (e) throw sy::SyError(SY_ERR_DEVICE, "device wait limit exceeded (code " + std::to_string(e) + ")");
        return SY_OK;
    });
}

sy_status sy_cuda_get_last_gradients(const sy_session* session, float* host, int64_t count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] { return s->impl->get_last_gradients(host, (long)count); });
}

sy_status sy_cuda_get_last_features(const sy_session* session, int32_t level, float* host, int64_t count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] { return s->impl->get_last_features(level, host, (long)count); });
}

sy_status sy_cuda_get_last_head_outputs(const sy_session* session, int32_t set, int32_t level, float* box,
                                        int64_t box_count, float* cls, int64_t cls_count) {
    if (!session) return SY_ERR_INVALID_ARGUMENT;
    sy_session* s = const_cast<sy_session*>(session);
    return guarded(s, [&] {
        return s->impl->get_last_head_outputs(set, level, box, (long)box_count, cls, (long)cls_count);
    });
}

// ------------------------------------------------------------------ standalone operators

sy_status sy_cuda_head_decode(int32_t device, int32_t images, int32_t levels, const int32_t* hs, const int32_t* ws,
                              const float* strides, int32_t bins, int32_t nc, int32_t xyxy, const float* const* box,
                              const float* const* cls, float* out) {
    return guarded(nullptr, [&] {
        if (images < 1 || levels < 1 || levels > sy::kMaxDetectLevels || !hs || !ws || !strides || !box || !cls ||
            !out || nc < 0 || bins < 1)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "head_decode: bad arguments");
        check_device(device);
        Scratch s;
        long anchors = 0;
        for (int l = 0; l < levels; l++) {
            if (hs[l] < 1 || ws[l] < 1 || !box[l] || (nc > 0 && !cls[l]))
                throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "head_decode: bad level");
            anchors += (long)hs[l] * ws[l];
        }
        if ((nc + 4) * anchors * images > (1L << 31))
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "head_decode: output above 2^31 elements");
        sy::DetectLevelSrc lv[sy::kMaxDetectLevels];
        for (int l = 0; l < levels; l++) {
            const long hw = (long)hs[l] * ws[l];
            float* db = s.get<float>((size_t)images * 4 * bins * hw);
            float* dc = s.get<float>((size_t)images * std::max(nc, 1) * hw);
            CK(cudaMemcpy(db, box[l], sizeof(float) * images * 4 * bins * hw, cudaMemcpyHostToDevice));
            if (nc > 0) CK(cudaMemcpy(dc, cls[l], sizeof(float) * images * nc * hw, cudaMemcpyHostToDevice));
            lv[l] = sy::DetectLevelSrc{db, dc, {4L * bins * hw, hw, ws[l], 1}, {(long)nc * hw, hw, ws[l], 1}, hs[l],
                                       ws[l], strides[l]};
        }
        float* dout = s.get<float>((size_t)images * (nc + 4) * anchors);
        sy::head_decode(lv, levels, images, bins, nc, xyxy ? 1 : 0, dout, 0);
        CK(cudaMemcpy(out, dout, sizeof(float) * images * (nc + 4) * anchors, cudaMemcpyDeviceToHost));
        return SY_OK;
    });
}

sy_status sy_cuda_end_to_end_topk(int32_t device, const float* x, int32_t images, int32_t fields, int32_t anchors,
                                  int32_t nc, int32_t maximum, float* out) {
    return guarded(nullptr, [&] {
        if (!x || !out || images < 1 || nc < 1 || fields < nc + 4 || anchors < 1 || maximum < 1)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "end_to_end_topk: bad arguments");
        if (maximum > sy::kMaxEndToEndTopk)
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "end_to_end_topk: maximum above 1024");
        if ((long)anchors * nc >= 0xffffffffL || (long)images * fields * anchors > (1L << 31))
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "end_to_end_topk: input too large");
        check_device(device);
        Scratch s;
        const int k = std::min(maximum, anchors), width = 6 + fields - nc - 4;
        float* dx = s.get<float>((size_t)images * fields * anchors);
        float* dout = s.get<float>((size_t)images * k * width);
        void* ws_ = s.get<uint8_t>(sy::end_to_end_workspace_bytes(images, anchors, nc, k));
        CK(cudaMemcpy(dx, x, sizeof(float) * images * fields * anchors, cudaMemcpyHostToDevice));
        sy::end_to_end_topk(dx, images, fields, anchors, nc, k, dout, ws_, 0);
        CK(cudaMemcpy(out, dout, sizeof(float) * images * k * width, cudaMemcpyDeviceToHost));
        return SY_OK;
    });
}

sy_status sy_cuda_decode_detections(int32_t device, const float* output, int32_t images, int32_t dim1, int32_t dim2,
                                    int32_t layout, int32_t class_count, const sy_letterbox* transforms,
                                    const sy_detect_options* options, sy_detection* out, int32_t* counts) {
    return guarded(nullptr, [&] {
        if (!output || !out || !counts || images < 1 || dim1 < 1 || dim2 < 1 || class_count < 0)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "decode_detections: bad arguments");
        const sy::DetectOptions o = sy::detect_options(options, false);
        // OutputLayout.Auto (YoloDetector.cs:545-555)
        if (layout == SY_LAYOUT_AUTO) {
            const int expected = class_count > 0 ? 4 + class_count : 0;
            if (expected > 0 && dim1 == expected && dim2 != expected) layout = SY_LAYOUT_CHANNELS_FIRST;
            else if (expected > 0 && dim2 == expected && dim1 != expected) layout = SY_LAYOUT_CHANNELS_LAST;
            else if (dim2 == 6 && dim1 != 6) layout = SY_LAYOUT_END_TO_END;
            else if (dim1 >= 5 && dim1 < dim2) layout = SY_LAYOUT_CHANNELS_FIRST;
            else if (dim2 >= 5 && dim2 < dim1) layout = SY_LAYOUT_CHANNELS_LAST;
            else throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "ambiguous YOLO output layout; set the layout explicitly");
        }
        if (layout < SY_LAYOUT_CHANNELS_FIRST || layout > SY_LAYOUT_END_TO_END)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "decode_detections: unknown layout");
        const bool cf = layout == SY_LAYOUT_CHANNELS_FIRST, e2e = layout == SY_LAYOUT_END_TO_END;
        const int count = cf ? dim2 : dim1, fields = cf ? dim1 : dim2;
        if (fields < 5 || (e2e && fields != 6)) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "invalid detection output");
        const int class_fields = class_count > 0 ? 4 + class_count : fields;
        if (!e2e && (class_fields < 5 || class_fields > fields))
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "class count does not match the output");
        if ((long)images * dim1 * dim2 > (1L << 31))
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "decode_detections: output above 2^31 elements");
        std::vector<sy::DetectTransform> tf(images);
        for (int b = 0; b < images; b++)
            tf[b] = sy::detect_transform(transforms ? transforms[b]
                                                    : sy_letterbox{1 << 20, 1 << 20, 1 << 20, 1 << 20, 1.f, 1.f, 0, 0});
        check_device(device);
        Scratch s;
        float* dx = s.get<float>((size_t)images * dim1 * dim2);
        sy::DetectTransform* dtf = s.get<sy::DetectTransform>(images);
        sy::DetOut* dout = s.get<sy::DetOut>((size_t)images * o.max_det);
        int* dcounts = s.get<int>(images);
        int* derr = s.get<int>(1);
        void* ws_ = s.get<uint8_t>(sy::detections_workspace_bytes(images, count, o.max_det));
        CK(cudaMemcpy(dx, output, sizeof(float) * images * dim1 * dim2, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(dtf, tf.data(), sizeof(sy::DetectTransform) * images, cudaMemcpyHostToDevice));
        sy::decode_detections(dx, images, (long)dim1 * dim2, cf ? 1 : fields, cf ? count : 1, count, class_fields, e2e,
                              dtf, o, dout, dcounts, derr, ws_, 0);
        int err = 0;
        CK(cudaMemcpy(&err, derr, sizeof(int), cudaMemcpyDeviceToHost));
        if (err) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "decode_detections: class id out of Int32 range");
        CK(cudaMemcpy(counts, dcounts, sizeof(int) * images, cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(out, dout, sizeof(sy::DetOut) * images * o.max_det, cudaMemcpyDeviceToHost));
        return SY_OK;
    });
}

sy_status sy_cuda_detection_loss(int32_t device, int32_t images, int32_t levels, const int32_t* hs, const int32_t* ws,
                                 const float* strides, int32_t nc, int32_t reg_max, const float* const* boxes,
                                 const float* const* classes, const sy_box* truth, const int32_t* counts,
                                 float* out_loss, int32_t* positives, int32_t* assigned, float* scores,
                                 float* const* box_grads, float* const* class_grads) {
    return sy_cuda_detection_loss_ex(device, images, levels, hs, ws, strides, nc, reg_max, boxes, classes, truth, counts,
                                     10, 10, 1.0f, out_loss, positives, assigned, scores, box_grads, class_grads);
}

sy_status sy_cuda_detection_loss_ex(int32_t device, int32_t images, int32_t levels, const int32_t* hs,
                                    const int32_t* ws, const float* strides, int32_t nc, int32_t reg_max,
                                    const float* const* boxes, const float* const* classes, const sy_box* truth,
                                    const int32_t* counts, int32_t topk, int32_t topk2, float grad_scale,
                                    float* out_loss, int32_t* positives, int32_t* assigned, float* scores,
                                    float* const* box_grads, float* const* class_grads) {
    return guarded(nullptr, [&] {
        if (images < 1 || levels < 1 || levels > 3 || !hs || !ws || !strides || !boxes || !classes || !counts ||
            !out_loss || nc < 1 || !(reg_max == 16 || reg_max == 1) || topk < 1 || topk > 15 || topk2 < 1 ||
            topk2 > topk || !std::isfinite(grad_scale))
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "detection_loss: bad arguments");
        check_device(device);
        Scratch s;
        const bool backward = box_grads && class_grads;
        int max_boxes = 0, total = 0;
        for (int b = 0; b < images; b++) {
            if (counts[b] < 0 || counts[b] > 100) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "box count out of range");
            max_boxes = std::max(max_boxes, counts[b]);
            total += counts[b];
        }
        std::vector<sy::TruthBox> tb(std::max(1, total));
        std::vector<int> off(images + 1, 0);
        for (int b = 0, k = 0; b < images; b++) {
            for (int j = 0; j < counts[b]; j++, k++) {
                if (truth[k].class_id < 0 || truth[k].class_id >= nc)
                    throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "class id out of range");
                tb[k] = sy::TruthBox{truth[k].class_id, truth[k].x1, truth[k].y1, truth[k].x2, truth[k].y2};
            }
            off[b + 1] = off[b] + counts[b];
        }
        sy::LevelIO lv[3];
        std::vector<sy::Grid> grids(levels);
        std::vector<sy::View> vb(levels), vc(levels), gb(levels), gc(levels);
        int anchors = 0;
        for (int l = 0; l < levels; l++) {
            grids[l] = sy::make_grid(hs[l], ws[l]);
            anchors += hs[l] * ws[l];
            vb[l] = padded(s, images, 4 * reg_max, grids[l]);
            vc[l] = padded(s, images, nc, grids[l]);
            const size_t nbox = (size_t)images * 4 * reg_max * hs[l] * ws[l], ncls = (size_t)images * nc * hs[l] * ws[l];
            float* tmp = s.get<float>(std::max(nbox, ncls));
            CK(cudaMemcpy(tmp, boxes[l], nbox * sizeof(float), cudaMemcpyHostToDevice));
            sy::nchw_to_padded(tmp, images, 4 * reg_max, grids[l], vb[l], 0);
            CK(cudaMemcpy(tmp, classes[l], ncls * sizeof(float), cudaMemcpyHostToDevice));
            sy::nchw_to_padded(tmp, images, nc, grids[l], vc[l], 0);
            if (backward) {
                gb[l] = padded(s, images, 4 * reg_max, grids[l]);
                gc[l] = padded(s, images, nc, grids[l]);
            }
            lv[l] = sy::LevelIO{vb[l].base, vc[l].base, backward ? gb[l].base : nullptr, backward ? gc[l].base : nullptr,
                                vb[l].pitch, vc[l].pitch, grids[l], strides[l]};
        }
        sy::TruthBox* d_truth = s.get<sy::TruthBox>(tb.size());
        int* d_off = s.get<int>(images + 1);
        CK(cudaMemcpy(d_truth, tb.data(), tb.size() * sizeof(sy::TruthBox), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(d_off, off.data(), off.size() * sizeof(int), cudaMemcpyHostToDevice));
        void* ws_ = s.get<uint8_t>(sy::loss_workspace_bytes(images, anchors, std::max(1, max_boxes), topk, nc));
        sy::LossOut lo{s.get<float>(4 * images), s.get<int>(images), s.get<int>(images), s.get<int>((size_t)images * anchors),
                       s.get<float>((size_t)images * anchors)};
        if (max_boxes * topk > 1024) throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "detection_loss: boxes * topk > 1024");
        sy::detection_loss(lv, levels, images, nc, reg_max, d_truth, d_off, std::max(1, max_boxes), topk, topk2,
                           grad_scale, backward ? 1 : 0, ws_, lo, 0);
        CK(cudaGetLastError());
        std::vector<float> loss(4 * images);
        CK(cudaMemcpy(loss.data(), lo.loss, loss.size() * sizeof(float), cudaMemcpyDeviceToHost));
        for (int b = 0; b < images; b++)
            for (int j = 0; j < 3; j++) out_loss[b * 3 + j] = loss[4 * b + j];
        if (positives) CK(cudaMemcpy(positives, lo.positives, images * sizeof(int), cudaMemcpyDeviceToHost));
        if (assigned)
            CK(cudaMemcpy(assigned, lo.assigned, (size_t)images * anchors * sizeof(int), cudaMemcpyDeviceToHost));
        if (scores) CK(cudaMemcpy(scores, lo.scores, (size_t)images * anchors * sizeof(float), cudaMemcpyDeviceToHost));
        if (backward)
            for (int l = 0; l < levels; l++) {
                const size_t nbox = (size_t)images * 4 * reg_max * hs[l] * ws[l], ncls = (size_t)images * nc * hs[l] * ws[l];
                float* tmp = s.get<float>(std::max(nbox, ncls));
                sy::padded_to_nchw(gb[l], images, 4 * reg_max, grids[l], tmp, 0);
                CK(cudaMemcpy(box_grads[l], tmp, nbox * sizeof(float), cudaMemcpyDeviceToHost));
                sy::padded_to_nchw(gc[l], images, nc, grids[l], tmp, 0);
                CK(cudaMemcpy(class_grads[l], tmp, ncls * sizeof(float), cudaMemcpyDeviceToHost));
            }
        CK(cudaDeviceSynchronize());
        return SY_OK;
    });
}


sy_status sy_cuda_conv2d_forward(int32_t device, const float* x, int32_t n, int32_t ic, int32_t h, int32_t w,
                                 const float* weight, int32_t oc, int32_t k, const float* bias, float* y) {
    return guarded(nullptr, [&] {
        if (!x || !weight || !y) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "conv2d_forward: null buffer");
        conv_shape_check(n, ic, oc, h, w, k);
        check_device(device);
        Scratch s;
        const sy::Grid g = sy::make_grid(h, w);
        const int taps = k * k, kpad = (ic + 31) / 32 * 32;
        const size_t nx = (size_t)n * ic * h * w, ny = (size_t)n * oc * h * w, nw = (size_t)oc * ic * taps;
        float* tmp = s.get<float>(std::max(nx, ny));
        float* dw = s.get<float>(nw);
        float* wk = s.get<float>((size_t)oc * taps * kpad);
        float* db = bias ? s.get<float>(oc) : nullptr;
        sy::View vx = padded(s, n, ic, g), vy = padded(s, n, oc, g);
        CK(cudaMemcpy(tmp, x, nx * sizeof(float), cudaMemcpyHostToDevice));
        sy::nchw_to_padded(tmp, n, ic, g, vx, 0);
        CK(cudaMemcpy(dw, weight, nw * sizeof(float), cudaMemcpyHostToDevice));
        if (db) CK(cudaMemcpy(db, bias, oc * sizeof(float), cudaMemcpyHostToDevice));
        sy::weights_fwd_layout(dw, oc, ic, taps, kpad, wk, 0);
        int* err = s.get<int>(1);
        sy::ConvEpilogue ep;
        ep.bias = db;
        sy::conv_tc_forward(vx, wk, oc, oc, taps, 1, g, vy, ep, err, 0);
        sy::padded_to_nchw(vy, n, oc, g, tmp, 0);
        CK(cudaMemcpy(y, tmp, ny * sizeof(float), cudaMemcpyDeviceToHost));
        int e = 0;
        CK(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (e) throw sy::SyError(SY_ERR_DEVICE, "conv kernel wait limit exceeded");
        return SY_OK;
    });
}

sy_status sy_cuda_conv2d_backward_data(int32_t device, const float* dy, int32_t n, int32_t oc, int32_t h, int32_t w,
                                       const float* weight, int32_t ic, int32_t k, float* dx) {
    return guarded(nullptr, [&] {
        if (!dy || !weight || !dx) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "conv2d_backward_data: null buffer");
        conv_shape_check(n, ic, oc, h, w, k);
        check_device(device);
        Scratch s;
        const sy::Grid g = sy::make_grid(h, w);
        const int taps = k * k, kpad_o = (oc + 31) / 32 * 32;
        const size_t nx = (size_t)n * ic * h * w, ny = (size_t)n * oc * h * w, nw = (size_t)oc * ic * taps;
        float* tmp = s.get<float>(std::max(nx, ny));
        float* dw = s.get<float>(nw);
        float* wk = s.get<float>((size_t)ic * taps * kpad_o);
        sy::View vdy = padded(s, n, oc, g), vdx = padded(s, n, ic, g);
        CK(cudaMemcpy(tmp, dy, ny * sizeof(float), cudaMemcpyHostToDevice));
        sy::nchw_to_padded(tmp, n, oc, g, vdy, 0);
        CK(cudaMemcpy(dw, weight, nw * sizeof(float), cudaMemcpyHostToDevice));
        sy::weights_dgrad_layout(dw, oc, ic, taps, kpad_o, wk, 0);
        int* err = s.get<int>(1);
        sy::ConvEpilogue ep;
        sy::conv_tc_forward(vdy, wk, ic, ic, taps, -1, g, vdx, ep, err, 0);
        sy::padded_to_nchw(vdx, n, ic, g, tmp, 0);
        CK(cudaMemcpy(dx, tmp, nx * sizeof(float), cudaMemcpyDeviceToHost));
        int e = 0;
        CK(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (e) throw sy::SyError(SY_ERR_DEVICE, "conv kernel wait limit exceeded");
        return SY_OK;
    });
}

sy_status sy_cuda_conv2d_backward_filter(int32_t device, const float* x, const float* dy, int32_t n, int32_t ic,
                                         int32_t oc, int32_t h, int32_t w, int32_t k, float* dwout) {
    return guarded(nullptr, [&] {
        if (!x || !dy || !dwout) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "conv2d_backward_filter: null buffer");
        conv_shape_check(n, ic, oc, h, w, k);
        if (oc > 256) throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "conv2d_backward_filter: oc > 256");
        check_device(device);
        Scratch s;
        const sy::Grid g = sy::make_grid(h, w);
        const int taps = k * k;
        const size_t nx = (size_t)n * ic * h * w, ny = (size_t)n * oc * h * w, nw = (size_t)oc * ic * taps;
        float* tmp = s.get<float>(std::max(nx, ny));
        sy::View vx = padded(s, n, ic, g), vdy = padded(s, n, oc, g);
        CK(cudaMemcpy(tmp, x, nx * sizeof(float), cudaMemcpyHostToDevice));
        sy::nchw_to_padded(tmp, n, ic, g, vx, 0);
        CK(cudaMemcpy(tmp, dy, ny * sizeof(float), cudaMemcpyHostToDevice));
        sy::nchw_to_padded(tmp, n, oc, g, vdy, 0);
        float* dwd = s.get<float>(nw);
        float* wsp = s.get<float>(sy::wgrad_workspace_floats(ic, oc, taps, vx.rows));
        int* err = s.get<int>(1);
        sy::conv_tc_wgrad(vx, vdy, taps, g, dwd, wsp, err, 0);
        CK(cudaMemcpy(dwout, dwd, nw * sizeof(float), cudaMemcpyDeviceToHost));
        int e = 0;
        CK(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (e) throw sy::SyError(SY_ERR_DEVICE, "wgrad kernel wait limit exceeded");
        return SY_OK;
    });
}

sy_status sy_cuda_matmul(int32_t device, const float* a, const float* b, float* c, int32_t m, int32_t n, int32_t k) {
    return guarded(nullptr, [&] {
        if (!a || !b || !c || m < 1 || n < 1 || k < 1) throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "matmul: bad arguments");
        check_device(device);
        Scratch s;
        // A as a [rows][k] activation (rows rounded to 128), B^T as K-major weights [n][kpad]
        const long rows = ((long)m + 127) / 128 * 128;
        const int pitch = (k + 3) / 4 * 4, kpad = (k + 31) / 32 * 32, opitch = (n + 3) / 4 * 4;
        float* da = s.get<float>((size_t)rows * pitch);
        CK(cudaMemcpy2D(da, pitch * sizeof(float), a, k * sizeof(float), k * sizeof(float), m, cudaMemcpyHostToDevice));
        std::vector<float> bt((size_t)n * kpad, 0.0f);
        for (int i = 0; i < k; i++)
            for (int j = 0; j < n; j++) bt[(size_t)j * kpad + i] = b[(size_t)i * n + j];
        float* wk = s.get<float>(bt.size());
        CK(cudaMemcpy(wk, bt.data(), bt.size() * sizeof(float), cudaMemcpyHostToDevice));
        float* dc = s.get<float>((size_t)rows * opitch);
        int* err = s.get<int>(1);
        sy::Grid g = sy::make_grid(1, 1);
        g.rows = (int)rows;
        sy::ConvEpilogue ep;
        ep.mask_halo = 0;
        sy::conv_tc_forward(sy::View{da, pitch, k, rows}, wk, n, n, 1, 1, g, sy::View{dc, opitch, n, rows}, ep, err, 0);
        CK(cudaMemcpy2D(c, n * sizeof(float), dc, opitch * sizeof(float), n * sizeof(float), m, cudaMemcpyDeviceToHost));
        int e = 0;
        CK(cudaMemcpy(&e, err, sizeof(int), cudaMemcpyDeviceToHost));
        if (e) throw sy::SyError(SY_ERR_DEVICE, "matmul kernel wait limit exceeded");
        return SY_OK;
    });
}

sy_status sy_cuda_sgd_update(int32_t device, float* weight, float* velocity, float* grad, int64_t count, float lr,
                             float momentum, float weight_decay, int32_t images, int32_t has_grad) {
    return guarded(nullptr, [&] {
        if (!weight || !velocity || !grad || count < 1 || images < 1)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "sgd_update: bad arguments");
        if (!has_grad) return SY_OK;
        check_device(device);
        Scratch s;
        float* w = s.get<float>(count);
        float* v = s.get<float>(count);
        float* g = s.get<float>(count);
        CK(cudaMemcpy(w, weight, count * sizeof(float), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(v, velocity, count * sizeof(float), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(g, grad, count * sizeof(float), cudaMemcpyHostToDevice));
        sy::ParamSegment seg{0, (long)count, weight_decay != 0.0f ? 1 : 0, 0};
        sy::ParamSegment* dseg = s.get<sy::ParamSegment>(1);
        CK(cudaMemcpy(dseg, &seg, sizeof(seg), cudaMemcpyHostToDevice));
        int* flags = s.get<int>(4);
        const int one[2] = {1, 1};
        CK(cudaMemcpy(flags, one, sizeof(one), cudaMemcpyHostToDevice));
        sy::optimizer_step(0, w, v, nullptr, g, dseg, 1, flags, flags, lr, momentum, weight_decay, 0, 0, 0,
                           1.0f / (float)images, flags + 2, 0);
        int bad = 0;
        CK(cudaMemcpy(&bad, flags + 2, sizeof(int), cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(weight, w, count * sizeof(float), cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(velocity, v, count * sizeof(float), cudaMemcpyDeviceToHost));
        if (bad) throw sy::SyError(SY_ERR_NONFINITE, "sgd_update: non-finite parameters");
        CK(cudaMemcpy(grad, g, count * sizeof(float), cudaMemcpyDeviceToHost));
        return SY_OK;
    });
}

}  // extern "C"
