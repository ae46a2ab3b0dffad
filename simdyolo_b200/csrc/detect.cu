// Inference post-processing on device, in three kernels that the session's detection path runs back to
// back and the standalone C-ABI entry points expose one by one:
//
//   head_decode_kernel     CpuHead.DecodeInto (src/SimdYolo/CpuHead.cs:57-120): DFL expectation per side,
//                          anchor-point boxes (cx, cy, w, h, or x1, y1, x2, y2 for end-to-end heads) and
//                          sigmoid class scores, joined over the levels as PtModel.Detect does
//                          (src/SimdYolo/PtModel.cs:444-503); output [image][4 + nc][anchors].
//   e2e_topk_kernel        PtModel.EndToEndTopK (src/SimdYolo/PtModel.cs:530-568): the k anchors with the
//                          highest class maximum, then the k best (anchor, class) pairs among them, ordered
//                          by (score desc, anchor asc, class asc); output [image][k][6 + extra].
//   detections_kernel      YoloDetector.DecodeIndexed (src/SimdYolo/YoloDetector.cs:539-642): confidence
//                          filter, boxes to (x, y, w, h), confidence order (stable), MaxCandidates, greedy
//                          class-aware (or agnostic) NMS with YoloDetector.Iou (:648-652), MaxDetections,
//                          letterbox mapping with clamping; one block per image.
//
// Every float operation is an explicit round-to-nearest intrinsic in the reference's expression order, and
// exp is det_expf (common.cuh), so the results equal the CPU restatement bit for bit; the reference calls
// MathF.Exp (scalar) or its own vector exp approximation (SIMD lanes).  GPU arithmetic returns the
// canonical NaN, so NaN payloads and signs are not carried through as x86 code carries them.
//
// Ordering.  Candidates are ranked by one 64-bit key: the confidence's order-preserving bits above the
// complemented anchor (or anchor * nc + class) index, so that a larger key is exactly "earlier in the
// reference's order" (OrderByDescending is stable; the end-to-end queues break ties on lower anchor, then
// lower class).  Keys are distinct.  The k-th largest key comes from an MSB-first radix select (eight 8-bit
// digits, histogram in shared memory); greedy NMS repeatedly takes the largest remaining key and, in the
// same pass over the candidates, removes the ones it suppresses and finds the next largest, so no sort of
// the candidates is needed.
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kSelThreads = 1024;

// MathF.Max / MathF.Min: NaN if either operand is NaN; +0 above -0
__device__ __forceinline__ float net_max(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}
__device__ __forceinline__ float net_min(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    if (a < b) return a;
    if (b < a) return b;
    return signbit(a) ? a : b;
}

// TensorOps.Sigmoid (src/SimdYolo/Compute.cs:513): 1 / (1 + exp(-x))
__device__ __forceinline__ float infer_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, det_expf(-x))); }

// float.CompareTo order as unsigned bits: NaN lowest, -0 equal to +0
__device__ __forceinline__ uint32_t order_bits(float f) {
    if (f != f) return 0u;
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) == 0u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ uint64_t rank_key(float score, uint32_t index) {
    return ((uint64_t)order_bits(score) << 32) | (uint64_t)(0xffffffffu - index);
}
__device__ __forceinline__ uint32_t key_index(uint64_t key) { return 0xffffffffu - (uint32_t)key; }

// Largest value over the block; `red` is shared [33].
__device__ uint64_t block_max(uint64_t v, uint64_t* red) {
    for (int o = 16; o; o >>= 1) v = max(v, (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red[warp] = v;
    __syncthreads();
    if (warp == 0) {
        v = lane < (int)(blockDim.x >> 5) ? red[lane] : 0;
        for (int o = 16; o; o >>= 1) v = max(v, (uint64_t)__shfl_xor_sync(0xffffffffu, (unsigned long long)v, o));
        if (lane == 0) red[32] = v;
    }
    __syncthreads();
    return red[32];
}

struct SelectShared {
    unsigned hist[256];
    uint64_t prefix;
    int remaining;
};

// The K-th largest nonzero key of keys[0, n) (keys distinct, more than K of them nonzero): MSB-first radix
// select over eight 8-bit digits.  Every thread of the block calls it and gets the same key.
__device__ uint64_t block_select_kth(const uint64_t* keys, int n, int K, SelectShared& s) {
    uint64_t prefix = 0, mask = 0;
    int remaining = K;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) s.hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint64_t k = keys[i];
            if (k && (k & mask) == prefix) atomicAdd(&s.hist[(k >> shift) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int cum = 0, d = 255;
            for (; d > 0; d--) {
                if (cum + (int)s.hist[d] >= remaining) break;
                cum += (int)s.hist[d];
            }
            s.prefix = prefix | ((uint64_t)d << shift);
            s.remaining = remaining - cum;
        }
        __syncthreads();
        prefix = s.prefix;
        remaining = s.remaining;
        mask |= 0xffull << shift;
    }
    return prefix;
}

// ------------------------------------------------------------------ head decode
struct DecodeParams {
    DetectLevelSrc lv[kMaxDetectLevels];
    int start[kMaxDetectLevels + 1];
    int nlevels, bins, nc, anchors, xyxy;
    float* out;
};

__global__ void __launch_bounds__(128) head_decode_kernel(const __grid_constant__ DecodeParams p) {
    const int a = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (a >= p.anchors) return;
    int l = 0;
    while (l + 1 < p.nlevels && a >= p.start[l + 1]) l++;
    const DetectLevelSrc& L = p.lv[l];
    const int pix = a - p.start[l], y = pix / L.w, x = pix - y * L.w;
    float* dst = p.out + (size_t)b * (p.nc + 4) * p.anchors + a;
    const float* cls = L.cls + b * L.cls_s[0] + y * L.cls_s[2] + x * L.cls_s[3];
    for (int c = 0; c < p.nc; c++) dst[(size_t)(4 + c) * p.anchors] = infer_sigmoid(cls[c * L.cls_s[1]]);
    const float* box = L.box + b * L.box_s[0] + y * L.box_s[2] + x * L.box_s[3];
    float d[4];
    for (int side = 0; side < 4; side++) {
        const float* src = box + (long)side * p.bins * L.box_s[1];
        if (p.bins == 1) {
            d[side] = src[0];
            continue;
        }
        float mx = -INFINITY, sum = 0.0f, numerator = 0.0f;
        for (int r = 0; r < p.bins; r++) mx = net_max(mx, src[r * L.box_s[1]]);
        for (int r = 0; r < p.bins; r++) {
            const float e = det_expf(__fsub_rn(src[r * L.box_s[1]], mx));
            sum = __fadd_rn(sum, e);
            numerator = __fadd_rn(numerator, __fmul_rn(e, (float)r));
        }
        d[side] = __fdiv_rn(numerator, sum);
    }
    const float cx = __fadd_rn((float)x, 0.5f), cy = __fadd_rn((float)y, 0.5f);
    const float x1 = __fmul_rn(__fsub_rn(cx, d[0]), L.stride), y1 = __fmul_rn(__fsub_rn(cy, d[1]), L.stride);
    const float x2 = __fmul_rn(__fadd_rn(cx, d[2]), L.stride), y2 = __fmul_rn(__fadd_rn(cy, d[3]), L.stride);
    dst[0] = p.xyxy ? x1 : __fmul_rn(__fadd_rn(x1, x2), 0.5f);
    dst[(size_t)p.anchors] = p.xyxy ? y1 : __fmul_rn(__fadd_rn(y1, y2), 0.5f);
    dst[(size_t)2 * p.anchors] = p.xyxy ? x2 : __fsub_rn(x2, x1);
    dst[(size_t)3 * p.anchors] = p.xyxy ? y2 : __fsub_rn(y2, y1);
}

// ------------------------------------------------------------------ end-to-end top-k
__global__ void __launch_bounds__(kSelThreads) e2e_topk_kernel(const float* __restrict__ x, int fields, int anchors,
                                                               int nc, int k, float* __restrict__ out,
                                                               uint64_t* __restrict__ ws, long ws_stride) {
    __shared__ SelectShared sel_s;
    __shared__ int nsel;
    __shared__ int chosen[kMaxEndToEndTopk];
    __shared__ uint64_t top[kMaxEndToEndTopk];
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* data = x + (size_t)b * fields * anchors;
    uint64_t* keys = ws + (size_t)b * ws_stride;
    // the anchors: class maximum (MathF.Max from -inf), ties to the lower anchor
    for (int a = tid; a < anchors; a += blockDim.x) {
        float m = -INFINITY;
        for (int c = 0; c < nc; c++) m = net_max(m, data[(size_t)(4 + c) * anchors + a]);
        keys[a] = rank_key(m, (uint32_t)a);
    }
    if (tid == 0) nsel = 0;
    __syncthreads();
    const uint64_t t1 = k < anchors ? block_select_kth(keys, anchors, k, sel_s) : 1;
    for (int a = tid; a < anchors; a += blockDim.x)
        if (keys[a] >= t1) {
            const int j = atomicAdd(&nsel, 1);
            if (j < k) chosen[j] = a;   // exactly k keys reach t1 (keys are distinct)
        }
    __syncthreads();
    // the (anchor, class) pairs of the chosen anchors: ties to the lower anchor, then the lower class
    const int n2 = k * nc;
    for (int i = tid; i < n2; i += blockDim.x) {
        const int j = i / nc, c = i - j * nc, a = chosen[j];
        keys[i] = rank_key(data[(size_t)(4 + c) * anchors + a], (uint32_t)a * (uint32_t)nc + (uint32_t)c);
    }
    if (tid == 0) nsel = 0;
    __syncthreads();
    const uint64_t t2 = k < n2 ? block_select_kth(keys, n2, k, sel_s) : 1;
    for (int i = tid; i < n2; i += blockDim.x)
        if (keys[i] >= t2) {
            const int j = atomicAdd(&nsel, 1);
            if (j < k) top[j] = keys[i];
        }
    __syncthreads();
    int P = 1;
    while (P < k) P <<= 1;
    for (int i = k + tid; i < P; i += blockDim.x) top[i] = 0;
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < P; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const uint64_t u = top[i], v = top[j];
                    if ((i & size) == 0 ? u < v : u > v) {
                        top[i] = v;
                        top[j] = u;
                    }
                }
            }
            __syncthreads();
        }
    const int extra = fields - nc - 4, width = 6 + extra;
    for (int i = tid; i < k; i += blockDim.x) {
        const uint32_t idx = key_index(top[i]);
        const int a = (int)(idx / (uint32_t)nc), c = (int)(idx % (uint32_t)nc);
        float* row = out + ((size_t)b * k + i) * width;
        for (int f = 0; f < 4; f++) row[f] = data[(size_t)f * anchors + a];
        row[4] = data[(size_t)(4 + c) * anchors + a];
        row[5] = (float)c;
        for (int f = 0; f < extra; f++) row[6 + f] = data[(size_t)(4 + nc + f) * anchors + a];
    }
}

// ------------------------------------------------------------------ candidates, NMS, mapping
struct DetParams {
    const float* x;
    long img_stride, a_stride, f_stride;
    int count, class_fields, e2e;
    const DetectTransform* tf;
    DetectOptions o;
    DetOut* out;
    int* counts;
    int* err;
    uint64_t* keys;
    float4* boxes;
    float* conf;
    int* cls;
    int* kept;
};

// YoloDetector.Iou on (x, y, w, h)
__device__ __forceinline__ float det_iou(const float4& a, const float4& b) {
    const float w = net_max(0.0f, __fsub_rn(net_min(__fadd_rn(a.x, a.z), __fadd_rn(b.x, b.z)), net_max(a.x, b.x)));
    const float h = net_max(0.0f, __fsub_rn(net_min(__fadd_rn(a.y, a.w), __fadd_rn(b.y, b.w)), net_max(a.y, b.y)));
    const float inter = __fmul_rn(w, h);
    const float uni = __fsub_rn(__fadd_rn(__fmul_rn(a.z, a.w), __fmul_rn(b.z, b.w)), inter);
    return __fdiv_rn(inter, net_max(__int_as_float(1), uni));   // float.Epsilon, the smallest subnormal
}

// Math.Clamp(v, lo, hi)
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void __launch_bounds__(kSelThreads) detections_kernel(const __grid_constant__ DetParams p) {
    __shared__ SelectShared sel_s;
    __shared__ uint64_t red[33];
    __shared__ int nvalid;
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* X = p.x + (size_t)b * p.img_stride;
    uint64_t* keys = p.keys + (size_t)b * p.count;
    float4* boxes = p.boxes + (size_t)b * p.count;
    float* conf = p.conf + (size_t)b * p.count;
    int* cls = p.cls + (size_t)b * p.count;
    if (tid == 0) nvalid = 0;
    __syncthreads();
    int local = 0;
    for (int a = tid; a < p.count; a += blockDim.x) {
        const float* v = X + (size_t)a * p.a_stride;
        uint64_t key = 0;
        int c = 0;
        bool ok = true;
        float score;
        if (p.e2e) {
            score = v[4 * p.f_stride];
            const float cv = v[5 * p.f_stride];
            if (!isfinite(cv) || cv < 0.0f || cv != truncf(cv)) {
                ok = false;
            } else if (cv >= 2147483648.0f) {
                atomicExch(p.err, 1);   // checked((int)cv) throws OverflowException in the reference
                ok = false;
            } else {
                c = (int)cv;
            }
        } else {
            score = -INFINITY;
            for (int f = 4; f < p.class_fields; f++) {
                const float s = v[(size_t)f * p.f_stride];
                if (s > score) {
                    score = s;
                    c = f - 4;
                }
            }
        }
        float4 bx = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ok && isfinite(score) && !(score < p.o.confidence)) {
            float bxx = v[0], byy = v[p.f_stride], bw = v[2 * p.f_stride], bh = v[3 * p.f_stride];
            if (isfinite(bxx) && isfinite(byy) && isfinite(bw) && isfinite(bh)) {
                if (p.e2e) {
                    bw = __fsub_rn(bw, bxx);
                    bh = __fsub_rn(bh, byy);
                } else {
                    bxx = __fsub_rn(bxx, __fmul_rn(bw, 0.5f));
                    byy = __fsub_rn(byy, __fmul_rn(bh, 0.5f));
                }
                if (bw > 0.0f && bh > 0.0f) {
                    key = rank_key(score, (uint32_t)a);
                    bx = make_float4(bxx, byy, bw, bh);
                    local++;
                }
            }
        }
        keys[a] = key;
        boxes[a] = bx;
        conf[a] = score;
        cls[a] = c;
    }
    if (local) atomicAdd(&nvalid, local);
    __syncthreads();
    // Take(MaxCandidates) of the confidence order
    if (nvalid > p.o.max_candidates) {
        const uint64_t t = block_select_kth(keys, p.count, p.o.max_candidates, sel_s);
        for (int a = tid; a < p.count; a += blockDim.x)
            if (keys[a] < t) keys[a] = 0;
    }
    uint64_t lm = 0;
    for (int a = tid; a < p.count; a += blockDim.x) lm = max(lm, keys[a]);
    uint64_t best = block_max(lm, red);
    int nk = 0;
    int* kept = p.kept + (size_t)b * p.o.max_det;
    // greedy NMS: the best remaining candidate is kept; it removes itself and what it suppresses
    while (best != 0 && nk < p.o.max_det) {
        const int ab = (int)key_index(best);
        const float4 kb = boxes[ab];
        const int kc = cls[ab];
        if (tid == 0) kept[nk] = ab;
        nk++;
        lm = 0;
        for (int a = tid; a < p.count; a += blockDim.x) {
            const uint64_t k = keys[a];
            if (!k) continue;
            if (a == ab ||
                (!p.e2e && (p.o.agnostic || cls[a] == kc) && det_iou(kb, boxes[a]) > p.o.iou)) {
                keys[a] = 0;
                continue;
            }
            lm = max(lm, k);
        }
        best = block_max(lm, red);
    }
    if (tid == 0) {
        const DetectTransform t = p.tf[b];
        DetOut* out = p.out + (size_t)b * p.o.max_det;
        int m = 0;
        for (int i = 0; i < nk; i++) {
            const int a = kept[i];
            const float4 d = boxes[a];
            const float x1 = clampf(__fdiv_rn(__fsub_rn(d.x, t.pad_x), t.scale_x), 0.0f, t.source_w);
            const float y1 = clampf(__fdiv_rn(__fsub_rn(d.y, t.pad_y), t.scale_y), 0.0f, t.source_h);
            const float x2 = clampf(__fdiv_rn(__fsub_rn(__fadd_rn(d.x, d.z), t.pad_x), t.scale_x), 0.0f, t.source_w);
            const float y2 = clampf(__fdiv_rn(__fsub_rn(__fadd_rn(d.y, d.w), t.pad_y), t.scale_y), 0.0f, t.source_h);
            const float w = __fsub_rn(x2, x1), h = __fsub_rn(y2, y1);
            if (!(w > 0.0f && h > 0.0f)) continue;
            DetOut r;
            r.class_id = cls[a];
            r.confidence = conf[a];
            r.x = x1;
            r.y = y1;
            r.width = w;
            r.height = h;
            out[m] = r;
            m++;
        }
        p.counts[b] = m;
    }
}

}  // namespace

// ------------------------------------------------------------------ host launchers
void head_decode(const DetectLevelSrc* levels, int nlevels, int batch, int bins, int nc, int xyxy, float* out,
                 cudaStream_t stream) {
    if (nlevels < 1 || nlevels > kMaxDetectLevels) throw std::runtime_error("head_decode: 1..8 levels");
    DecodeParams p{};
    p.start[0] = 0;
    for (int l = 0; l < nlevels; l++) {
        p.lv[l] = levels[l];
        p.start[l + 1] = p.start[l] + levels[l].h * levels[l].w;
    }
    p.nlevels = nlevels;
    p.bins = bins;
    p.nc = nc;
    p.anchors = p.start[nlevels];
    p.xyxy = xyxy;
    p.out = out;
    dim3 grid((p.anchors + 127) / 128, batch);
    head_decode_kernel<<<grid, 128, 0, stream>>>(p);
    launch_check("head_decode_kernel");
}

size_t end_to_end_workspace_bytes(int batch, int anchors, int nc, int k) {
    const long per = std::max<long>(anchors, (long)std::min(k, anchors) * nc);
    return sizeof(uint64_t) * (size_t)batch * per;
}

void end_to_end_topk(const float* x, int batch, int fields, int anchors, int nc, int k, float* out, void* ws,
                     cudaStream_t stream) {
    if (k < 1 || k > kMaxEndToEndTopk) throw std::runtime_error("end_to_end_topk: k out of range");
    k = std::min(k, anchors);
    const long per = std::max<long>(anchors, (long)k * nc);
    e2e_topk_kernel<<<batch, kSelThreads, 0, stream>>>(x, fields, anchors, nc, k, out, static_cast<uint64_t*>(ws),
                                                       per);
    launch_check("e2e_topk_kernel");
}

size_t detections_workspace_bytes(int batch, int count, int max_det) {
    const size_t per = (size_t)count * (sizeof(uint64_t) + sizeof(float4) + sizeof(float) + sizeof(int));
    return (size_t)batch * per + sizeof(int) * (size_t)batch * max_det + 256;
}

void decode_detections(const float* x, int batch, long img_stride, long a_stride, long f_stride, int count,
                       int class_fields, bool e2e, const DetectTransform* tf, const DetectOptions& o, DetOut* out,
                       int* counts, int* err, void* ws, cudaStream_t stream) {
    DetParams p{};
    p.x = x;
    p.img_stride = img_stride;
    p.a_stride = a_stride;
    p.f_stride = f_stride;
    p.count = count;
    p.class_fields = class_fields;
    p.e2e = e2e ? 1 : 0;
    p.tf = tf;
    p.o = o;
    p.out = out;
    p.counts = counts;
    p.err = err;
    // workspace: boxes (16-byte aligned) first, then keys, confidences, classes, kept lists
    char* w = static_cast<char*>(ws);
    p.boxes = reinterpret_cast<float4*>(w);
    w += sizeof(float4) * (size_t)batch * count;
    p.keys = reinterpret_cast<uint64_t*>(w);
    w += sizeof(uint64_t) * (size_t)batch * count;
    p.conf = reinterpret_cast<float*>(w);
    w += sizeof(float) * (size_t)batch * count;
    p.cls = reinterpret_cast<int*>(w);
    w += sizeof(int) * (size_t)batch * count;
    p.kept = reinterpret_cast<int*>(w);
    detections_kernel<<<batch, kSelThreads, 0, stream>>>(p);
    launch_check("detections_kernel");
}

}  // namespace sy
