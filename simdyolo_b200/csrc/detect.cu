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
constexpr int kSortCap = 16384;   // candidates of one image sorted in shared memory (128 KB of keys)

// MathF.Max: NaN if either operand is NaN; +0 above -0
__device__ __forceinline__ float net_max(float a, float b) {
    if (a != a) return a;
    if (b != b) return b;
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
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

// ------------------------------------------------------------------ candidates
// Per-image candidate arrays, written by a candidate kernel for every anchor (key 0: not a candidate) and
// read by detections_kernel.
struct CandArrays {
    uint64_t* keys;   // [batch][count] rank keys (confidence, anchor)
    float4* boxes;    // (x, y, x + w, y + h) in model pixels, each sum rounded once as the reference rounds it
    float* area;      // w * h, rounded once
    float* conf;
    int* cls;
    int count;
};

// DecodeIndexed's AddCandidate (YoloDetector.cs:564-575) on the box fields of one anchor.
__device__ __forceinline__ void add_candidate(const CandArrays& c, size_t i, int a, float score, int cls, float x,
                                              float y, float w, float h, bool e2e) {
    uint64_t key = 0;
    float4 bx = make_float4(0.f, 0.f, 0.f, 0.f);
    if (isfinite(x) && isfinite(y) && isfinite(w) && isfinite(h)) {
        if (e2e) {
            w = __fsub_rn(w, x);
            h = __fsub_rn(h, y);
        } else {
            x = __fsub_rn(x, __fmul_rn(w, 0.5f));
            y = __fsub_rn(y, __fmul_rn(h, 0.5f));
        }
        if (w > 0.0f && h > 0.0f) {
            key = rank_key(score, (uint32_t)a);
            bx = make_float4(x, y, __fadd_rn(x, w), __fadd_rn(y, h));
            c.area[i] = __fmul_rn(w, h);
        }
    }
    c.keys[i] = key;
    c.boxes[i] = bx;
    c.conf[i] = score;
    c.cls[i] = cls;
}

__device__ __forceinline__ void no_candidate(const CandArrays& c, size_t i) {
    c.keys[i] = 0;
    c.cls[i] = 0;
}

// Candidates of a decoded output: value (anchor a, field f) of image b at x[b * img + a * as + f * fs].
struct DecodedCandParams {
    const float* x;
    long img_stride, a_stride, f_stride;
    int class_fields, e2e;
    float confidence;
    CandArrays c;
    int* err;
};

__global__ void __launch_bounds__(256) decoded_candidates_kernel(const __grid_constant__ DecodedCandParams p) {
    const int a = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (a >= p.c.count) return;
    const size_t i = (size_t)b * p.c.count + a;
    const float* v = p.x + (size_t)b * p.img_stride + (size_t)a * p.a_stride;
    int c = 0;
    float score;
    if (p.e2e) {
        score = v[4 * p.f_stride];
        const float cv = v[5 * p.f_stride];
        if (!isfinite(cv) || cv < 0.0f || cv != truncf(cv)) return no_candidate(p.c, i);
        if (cv >= 2147483648.0f) {
            atomicExch(p.err, 1);   // checked((int)cv) throws OverflowException in the reference
            return no_candidate(p.c, i);
        }
        c = (int)cv;
    } else {
        // strict comparison: the first class wins ties, NaN never wins (YoloDetector.cs:608-612)
        score = -INFINITY;
        for (int f = 4; f < p.class_fields; f++) {
            const float s = v[(size_t)f * p.f_stride];
            if (s > score) {
                score = s;
                c = f - 4;
            }
        }
    }
    if (!isfinite(score) || score < p.confidence) return no_candidate(p.c, i);
    add_candidate(p.c, i, a, score, c, v[0], v[p.f_stride], v[2 * p.f_stride], v[3 * p.f_stride], p.e2e != 0);
}

// Candidates straight from the raw head outputs of the session (channels-last rows of logits): CpuHead's
// sigmoid scores and, only for anchors whose confidence passes, its DFL boxes, then AddCandidate; the
// same values as head_decode_kernel followed by decoded_candidates_kernel, without the decoded tensor.
// A block stages the rows of kRawAnchors anchors in shared memory with coalesced float4 loads (classes
// first, then the box logits in the same buffer), one thread per anchor reads its row from there.
constexpr int kRawAnchors = 128;
constexpr int kMaxRawPitch = 256;   // staged floats per row: up to 256 classes, 64 box logits
struct RawCandParams {
    DetectLevelSrc lv[3];
    int start[4];
    int nlevels, bins, nc;
    int cls_pitch, box_pitch;   // floats per staged row (multiples of 4)
    float confidence;
    CandArrays c;
};

// Copies rows[an][0, 4 q) (an < n) to stage[an * stride + ...] with float4 loads, eight in flight per thread
// before their stores.
__device__ __forceinline__ void stage_rows(const float* const* rows, int n, int q, int stride, float* stage) {
    const int total = n * q;
    for (int base = threadIdx.x; base < total; base += 8 * kRawAnchors) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int idx = base + u * kRawAnchors;
            if (idx < total) {
                const int an = idx / q, k = idx - an * q;
                v[u] = __ldg(reinterpret_cast<const float4*>(rows[an]) + k);
            }
        }
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int idx = base + u * kRawAnchors;
            if (idx < total) {
                const int an = idx / q, k = idx - an * q;
                float* d = stage + an * stride + 4 * k;
                d[0] = v[u].x;
                d[1] = v[u].y;
                d[2] = v[u].z;
                d[3] = v[u].w;
            }
        }
    }
}

__global__ void __launch_bounds__(kRawAnchors) raw_candidates_kernel(const __grid_constant__ RawCandParams p) {
    extern __shared__ float stage[];
    __shared__ const float* row_c[kRawAnchors];
    __shared__ const float* row_b[kRawAnchors];
    const int t = threadIdx.x, b = blockIdx.y, a0 = blockIdx.x * kRawAnchors;
    const int a = a0 + t, n = min(kRawAnchors, p.c.count - a0);
    int l = 0, y = 0, x = 0;
    if (a < p.c.count) {
        while (l + 1 < p.nlevels && a >= p.start[l + 1]) l++;
        const int pix = a - p.start[l];
        y = pix / p.lv[l].w;
        x = pix - y * p.lv[l].w;
        const DetectLevelSrc& L = p.lv[l];
        row_c[t] = L.cls + b * L.cls_s[0] + y * L.cls_s[2] + x * L.cls_s[3];
        row_b[t] = L.box + b * L.box_s[0] + y * L.box_s[2] + x * L.box_s[3];
    }
    __syncthreads();
    // class rows
    const int qc = p.cls_pitch >> 2, cs = p.cls_pitch + 1;
    stage_rows(row_c, n, qc, cs, stage);
    __syncthreads();
    // Strict maximum of the sigmoid scores in class order (first class on ties, NaN never wins).  The
    // sigmoid is monotone (each step of 1 / (1 + exp(-x)) rounds monotonically), so a logit at or below the
    // largest one seen cannot raise the maximum: only logits that raise the running logit maximum are
    // evaluated, which gives the same class and score as evaluating all of them.
    float score = -INFINITY, top = 0.0f;
    int c = 0;
    bool seen = false;
    if (a < p.c.count)
        for (int k = 0; k < p.nc; k++) {
            const float v = stage[t * cs + k];
            if (v != v || (seen && !(v > top))) continue;
            const float s = infer_sigmoid(v);
            if (s > score) {
                score = s;
                c = k;
            }
            top = v;
            seen = true;
        }
    const bool pass = a < p.c.count && isfinite(score) && !(score < p.confidence);
    __syncthreads();
    // box rows (only those of passing anchors are needed, all are staged: the loads are coalesced)
    const int qb = p.box_pitch >> 2, bs = p.box_pitch + 1;
    stage_rows(row_b, n, qb, bs, stage);
    __syncthreads();
    if (a >= p.c.count) return;
    const size_t i = (size_t)b * p.c.count + a;
    if (!pass) return no_candidate(p.c, i);
    const float* src = stage + t * bs;
    float d[4];
    for (int side = 0; side < 4; side++) {
        if (p.bins == 1) {
            d[side] = src[side];
            continue;
        }
        const float* r = src + side * p.bins;
        float mx = -INFINITY, sum = 0.0f, numerator = 0.0f;
        for (int k = 0; k < p.bins; k++) mx = net_max(mx, r[k]);
        for (int k = 0; k < p.bins; k++) {
            const float e = det_expf(__fsub_rn(r[k], mx));
            sum = __fadd_rn(sum, e);
            numerator = __fadd_rn(numerator, __fmul_rn(e, (float)k));
        }
        d[side] = __fdiv_rn(numerator, sum);
    }
    const float stride = p.lv[l].stride;
    const float cx = __fadd_rn((float)x, 0.5f), cy = __fadd_rn((float)y, 0.5f);
    const float x1 = __fmul_rn(__fsub_rn(cx, d[0]), stride), y1 = __fmul_rn(__fsub_rn(cy, d[1]), stride);
    const float x2 = __fmul_rn(__fadd_rn(cx, d[2]), stride), y2 = __fmul_rn(__fadd_rn(cy, d[3]), stride);
    add_candidate(p.c, i, a, score, c, __fmul_rn(__fadd_rn(x1, x2), 0.5f), __fmul_rn(__fadd_rn(y1, y2), 0.5f),
                  __fsub_rn(x2, x1), __fsub_rn(y2, y1), false);
}

// ------------------------------------------------------------------ NMS and mapping
struct DetParams {
    CandArrays c;
    int e2e;
    const DetectTransform* tf;
    DetectOptions o;
    DetOut* out;
    int* counts;
    int* kept;      // [batch][max_det] anchors of the kept candidates, in order
    float4* kbox;   // [batch][max_det] their corners, areas and classes
    float* karea;
    int* kcls;
    int sort_cap;   // keys the dynamic shared memory holds (a power of two <= kSortCap)
};

// YoloDetector.Iou(a, b) > thr (YoloDetector.cs:648-652) on corner boxes (x1, y1, x2, y2) of positive finite
// size whose areas are given.  x2 = x + w is the reference's own rounded sum, so min / max / subtract give its
// overlap extents exactly (fminf / fmaxf differ from MathF.Min / Max only on NaN and on the sign of zero,
// neither of which changes the outcome here).  Boxes that do not overlap have intersection 0 and IoU 0 (the
// union is positive), which needs no division: most pairs of a greedy NMS are of that kind.
__device__ __forceinline__ bool iou_above(const float4& a, float area_a, const float4& b, float area_b, float thr) {
    const float w = fmaxf(0.0f, __fsub_rn(fminf(a.z, b.z), fmaxf(a.x, b.x)));
    const float h = fmaxf(0.0f, __fsub_rn(fminf(a.w, b.w), fmaxf(a.y, b.y)));
    const float inter = __fmul_rn(w, h);
    if (inter == 0.0f) return 0.0f > thr;
    const float uni = __fsub_rn(__fadd_rn(area_a, area_b), inter);
    return __fdiv_rn(inter, net_max(__int_as_float(1), uni)) > thr;   // float.Epsilon, the smallest subnormal
}

// Math.Clamp(v, lo, hi)
__device__ __forceinline__ float clampf(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Descending bitonic sort of keys[0, P) in shared memory (P a power of two), by the whole block.
__device__ void block_sort_desc(uint64_t* keys, int P) {
    for (int size = 2; size <= P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int j = i ^ stride;
                if (j > i) {
                    const uint64_t u = keys[i], v = keys[j];
                    if ((i & size) == 0 ? u < v : u > v) {
                        keys[i] = v;
                        keys[j] = u;
                    }
                }
            }
            __syncthreads();
        }
}

// Stable compaction rank: the number of threads below this one (in thread order) whose flag is set, and in
// *total the count over the block.  Every thread of the block calls it; `wsum` is shared [33].
__device__ int block_rank(bool flag, int* wsum, int* total) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = (int)(blockDim.x >> 5);
    const unsigned bal = __ballot_sync(0xffffffffu, flag);
    if (lane == 0) wsum[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
        const int v = lane < warps ? wsum[lane] : 0;
        int inc = v;
        for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += u;
        }
        if (lane < warps) wsum[lane] = inc - v;
        if (lane == 31) wsum[32] = inc;
    }
    __syncthreads();
    const int rank = wsum[warp] + __popc(bal & ((1u << lane) - 1u));
    *total = wsum[32];
    __syncthreads();
    return rank;
}

// The K-th largest of the keys in pool[0, n) that lie below `below` (keys distinct, more than K of them
// below): MSB-first radix select over eight 8-bit digits, the digit of each pass found by warp 0 (a lane
// per 8 bins, scanned from the top).  Every thread of the block calls it and gets the same key.
__device__ uint64_t pool_select_kth(const uint64_t* pool, int n, int K, uint64_t below, SelectShared& s) {
    uint64_t prefix = 0, mask = 0;
    int remaining = K;
    const int lane = threadIdx.x & 31;
    for (int shift = 56; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) s.hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint64_t k = pool[i];
            if (k < below && (k & mask) == prefix) atomicAdd(&s.hist[(k >> shift) & 255], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            // lane l holds bins 255 - 8 l - j (j = 0..7), i.e. lanes go down the digits
            int local = 0;
            for (int j = 0; j < 8; j++) local += (int)s.hist[255 - 8 * lane - j];
            int inc = local;
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += u;
            }
            const int before = inc - local;   // keys in higher digits than this lane's bins
            const unsigned hit = __ballot_sync(0xffffffffu, inc >= remaining && before < remaining);
            if (lane == __ffs(hit) - 1) {
                int cum = before, d = 255 - 8 * lane;
                for (int j = 0; j < 8; j++, d--) {
                    if (cum + (int)s.hist[d] >= remaining) break;
                    cum += (int)s.hist[d];
                }
                s.prefix = prefix | ((uint64_t)d << shift);
                s.remaining = remaining - cum;
            }
        }
        __syncthreads();
        prefix = s.prefix;
        remaining = s.remaining;
        mask |= 0xffull << shift;
    }
    return prefix;
}

constexpr int kWindow = kSelThreads;   // candidates per NMS window
constexpr int kKeptCache = 1024;       // kept boxes held in shared memory (the rest are read from global)

// Does any kept box of index [j0, k) whose class counts (agnostic NMS or the same class) suppress the
// candidate (bx, ar, c)?  Indices below kKeptCache are read from shared memory, the rest from global memory.
// Four tests per step without an early exit inside the step, so their loads and arithmetic overlap.
__device__ __forceinline__ bool suppressed_by(const float4* sbox, const float* sarea, const int* scls,
                                             const float4* gbox, const float* garea, const int* gcls, int j0, int k,
                                             const float4& bx, float ar, int c, const DetectOptions& o) {
    int j = j0;
    for (; j + 4 <= k; j += 4) {
        bool hit = false;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int i = j + q;
            const bool cached = i < kKeptCache;
            const float4 kb = cached ? sbox[i] : gbox[i];
            const float ka = cached ? sarea[i] : garea[i];
            const int kc = cached ? scls[i] : gcls[i];
            hit |= (o.agnostic || kc == c) && iou_above(kb, ka, bx, ar, o.iou);
        }
        if (hit) return true;
    }
    for (; j < k; j++) {
        const bool cached = j < kKeptCache;
        const float4 kb = cached ? sbox[j] : gbox[j];
        const float ka = cached ? sarea[j] : garea[j];
        const int kc = cached ? scls[j] : gcls[j];
        if ((o.agnostic || kc == c) && iou_above(kb, ka, bx, ar, o.iou)) return true;
    }
    return false;
}

__global__ void __launch_bounds__(kSelThreads) detections_kernel(const __grid_constant__ DetParams p) {
    extern __shared__ uint64_t pool[];     // p.sort_cap keys: every candidate of the image
    __shared__ SelectShared sel_s;
    __shared__ uint64_t red[33];
    __shared__ uint64_t window[kWindow];
    __shared__ int wsum[33];
    __shared__ int nvalid, nsel, kept_n, nnew;
    __shared__ float4 sbox[kKeptCache];   // the first kKeptCache kept boxes, areas and classes
    __shared__ float sarea[kKeptCache];
    __shared__ int scls[kKeptCache];
    const int b = blockIdx.x, tid = threadIdx.x, count = p.c.count;
    uint64_t* keys = p.c.keys + (size_t)b * count;
    const float4* boxes = p.c.boxes + (size_t)b * count;
    const float* area = p.c.area + (size_t)b * count;
    const float* conf = p.c.conf + (size_t)b * count;
    const int* cls = p.c.cls + (size_t)b * count;
    int* kept = p.kept + (size_t)b * p.o.max_det;
    float4* kbox = p.kbox + (size_t)b * p.o.max_det;
    float* karea = p.karea + (size_t)b * p.o.max_det;
    int* kcls = p.kcls + (size_t)b * p.o.max_det;
    if (tid == 0) {
        nvalid = 0;
        nsel = 0;
        kept_n = 0;
    }
    __syncthreads();
    int local = 0;
    for (int a = tid; a < count; a += blockDim.x) local += keys[a] != 0;
    if (local) atomicAdd(&nvalid, local);
    __syncthreads();
    const int nv = nvalid;
    int nk = 0;
    if (nv <= p.sort_cap) {
        // Pool path.  Every candidate key sits in shared memory; candidates are taken in rank order a window
        // at a time (the next kWindow keys by radix select below the previous window's last key, then a
        // bitonic sort of the window) until max_det are kept or MaxCandidates are used up.  In a window,
        // first all threads drop what the boxes kept so far suppress and move the survivors to the front,
        // in order; the survivors are then resolved 32 at a time: the warp that holds them keeps them in
        // lane order (a kept lane removes the later lanes it suppresses), and the later warps test their
        // candidates against those newly kept boxes.
        for (int a = tid; a < count; a += blockDim.x) {
            const uint64_t k = keys[a];
            if (k) {
                const int j = atomicAdd(&nsel, 1);
                if (j < p.sort_cap) pool[j] = k;
            }
        }
        __syncthreads();
        const int n = min(nv, p.o.max_candidates);   // Take(MaxCandidates)
        const int warp = tid >> 5, lane = tid & 31, warps = (int)(blockDim.x >> 5);
        uint64_t below = ~0ull;   // keys of the windows taken so far are >= below
        bool full = false;
        for (int base = 0; base < n && !full; base += kWindow) {
            const int take = min(kWindow, n - base);
            // the window's keys: the take largest keys below `below`
            const uint64_t lo = nv - base > take ? pool_select_kth(pool, nv, take, below, sel_s) : 1;
            if (tid == 0) nsel = 0;
            __syncthreads();
            for (int i = tid; i < nv; i += blockDim.x) {
                const uint64_t k = pool[i];
                if (k < below && k >= lo) {
                    const int j = atomicAdd(&nsel, 1);
                    if (j < kWindow) window[j] = k;
                }
            }
            int P = 1;
            while (P < take) P <<= 1;
            __syncthreads();
            for (int i = take + tid; i < P; i += blockDim.x) window[i] = 0;
            __syncthreads();
            block_sort_desc(window, P);
            below = lo;
            bool alive = tid < take;
            uint64_t key = 0;
            int c = 0;
            float4 bx = make_float4(0.f, 0.f, 0.f, 0.f);
            float ar = 0.0f;
            if (alive) {
                key = window[tid];
                const int a = (int)key_index(key);
                bx = boxes[a];
                ar = area[a];
                c = cls[a];
            }
            const int k0 = kept_n;
            if (!p.e2e && alive && suppressed_by(sbox, sarea, scls, kbox, karea, kcls, 0, k0, bx, ar, c, p.o))
                alive = false;
            int ns = 0;
            const int rank = block_rank(alive, wsum, &ns);
            if (alive) window[rank] = key;
            __syncthreads();
            alive = tid < ns;
            int a = 0;
            if (alive) {
                a = (int)key_index(window[tid]);
                bx = boxes[a];
                ar = area[a];
                c = cls[a];
            }
            for (int chunk = 0; chunk < warps; chunk++) {
                if (chunk * 32 >= ns) break;
                if (warp == chunk) {
                    unsigned m = __ballot_sync(0xffffffffu, alive);
                    const int kn = kept_n;
                    int added = 0;
                    while (m && kn + added < p.o.max_det) {
                        const int i = __ffs(m) - 1;
                        const float4 bi = make_float4(__shfl_sync(0xffffffffu, bx.x, i), __shfl_sync(0xffffffffu, bx.y, i),
                                                      __shfl_sync(0xffffffffu, bx.z, i), __shfl_sync(0xffffffffu, bx.w, i));
                        const float ai = __shfl_sync(0xffffffffu, ar, i);
                        const int ci = __shfl_sync(0xffffffffu, c, i);
                        if (lane == i) {
                            const int at = kn + added;
                            kept[at] = a;
                            if (at < kKeptCache) {
                                sbox[at] = bx;
                                sarea[at] = ar;
                                scls[at] = c;
                            } else {
                                kbox[at] = bx;
                                karea[at] = ar;
                                kcls[at] = c;
                            }
                        }
                        added++;
                        m &= ~(1u << i);
                        if (!p.e2e) {
                            const bool sup = ((m >> lane) & 1u) && (p.o.agnostic || ci == c) &&
                                             iou_above(bi, ai, bx, ar, p.o.iou);
                            if (sup) alive = false;
                            m &= ~__ballot_sync(0xffffffffu, sup);
                        }
                    }
                    if (lane == 0) {
                        nnew = kn;
                        kept_n = kn + added;
                    }
                }
                __syncthreads();
                // the later warps against the boxes this chunk kept (kept list entries [nnew, kept_n))
                if (!p.e2e && warp > chunk && alive) {
                    const int k1 = nnew, k2 = kept_n;
                    if (k2 > k1 && suppressed_by(sbox, sarea, scls, kbox, karea, kcls, k1, k2, bx, ar, c, p.o))
                        alive = false;
                }
                full = kept_n >= p.o.max_det;
                __syncthreads();
                if (full) break;
            }
        }
        nk = kept_n;
    } else {
        // More candidates than shared memory holds: Take(MaxCandidates) by radix select, then greedy NMS by
        // repeated maxima (the best remaining candidate is kept; it removes itself and what it suppresses,
        // and the same pass finds the next best).
        if (nv > p.o.max_candidates) {
            const uint64_t t = block_select_kth(keys, count, p.o.max_candidates, sel_s);
            for (int a = tid; a < count; a += blockDim.x)
                if (keys[a] < t) keys[a] = 0;
        }
        uint64_t lm = 0;
        for (int a = tid; a < count; a += blockDim.x) lm = max(lm, keys[a]);
        uint64_t best = block_max(lm, red);
        while (best != 0 && nk < p.o.max_det) {
            const int ab = (int)key_index(best);
            const float4 kb = boxes[ab];
            const float ka = area[ab];
            const int kc = cls[ab];
            if (tid == 0) kept[nk] = ab;
            nk++;
            lm = 0;
            for (int a = tid; a < count; a += blockDim.x) {
                const uint64_t k = keys[a];
                if (!k) continue;
                if (a == ab ||
                    (!p.e2e && (p.o.agnostic || cls[a] == kc) && iou_above(kb, ka, boxes[a], area[a], p.o.iou))) {
                    keys[a] = 0;
                    continue;
                }
                lm = max(lm, k);
            }
            best = block_max(lm, red);
        }
    }
    __syncthreads();
    // Letterbox mapping and clamping (YoloDetector.cs:636-641); boxes left without area are dropped, the
    // rest keep their order
    const DetectTransform t = p.tf[b];
    DetOut* out = p.out + (size_t)b * p.o.max_det;
    int m0 = 0;
    for (int base = 0; base < nk; base += blockDim.x) {
        const int i = base + tid;
        DetOut r{};
        bool ok = false;
        if (i < nk) {
            const int a = kept[i];
            const float4 d = boxes[a];   // (x, y, x + w, y + h)
            const float x1 = clampf(__fdiv_rn(__fsub_rn(d.x, t.pad_x), t.scale_x), 0.0f, t.source_w);
            const float y1 = clampf(__fdiv_rn(__fsub_rn(d.y, t.pad_y), t.scale_y), 0.0f, t.source_h);
            const float x2 = clampf(__fdiv_rn(__fsub_rn(d.z, t.pad_x), t.scale_x), 0.0f, t.source_w);
            const float y2 = clampf(__fdiv_rn(__fsub_rn(d.w, t.pad_y), t.scale_y), 0.0f, t.source_h);
            r.class_id = cls[a];
            r.confidence = conf[a];
            r.x = x1;
            r.y = y1;
            r.width = __fsub_rn(x2, x1);
            r.height = __fsub_rn(y2, y1);
            ok = r.width > 0.0f && r.height > 0.0f;
        }
        int total = 0;
        const int rank = block_rank(ok, wsum, &total);
        if (ok) out[m0 + rank] = r;
        m0 += total;
    }
    if (tid == 0) p.counts[b] = m0;
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
    const size_t per = (size_t)count * (sizeof(uint64_t) + sizeof(float4) + 2 * sizeof(float) + sizeof(int));
    const size_t kept = (size_t)max_det * (sizeof(float4) + sizeof(float) + 2 * sizeof(int));
    return (size_t)batch * (per + kept) + 256;
}

namespace {

// Carves the workspace (the 16-byte boxes first) and launches detections_kernel over the candidates.
DetParams carve(int batch, int count, const DetectOptions& o, void* ws, CandArrays* c) {
    DetParams p{};
    char* w = static_cast<char*>(ws);
    c->boxes = reinterpret_cast<float4*>(w);
    w += sizeof(float4) * (size_t)batch * count;
    p.kbox = reinterpret_cast<float4*>(w);
    w += sizeof(float4) * (size_t)batch * o.max_det;
    c->keys = reinterpret_cast<uint64_t*>(w);
    w += sizeof(uint64_t) * (size_t)batch * count;
    c->conf = reinterpret_cast<float*>(w);
    w += sizeof(float) * (size_t)batch * count;
    c->area = reinterpret_cast<float*>(w);
    w += sizeof(float) * (size_t)batch * count;
    c->cls = reinterpret_cast<int*>(w);
    w += sizeof(int) * (size_t)batch * count;
    p.kept = reinterpret_cast<int*>(w);
    w += sizeof(int) * (size_t)batch * o.max_det;
    p.kcls = reinterpret_cast<int*>(w);
    w += sizeof(int) * (size_t)batch * o.max_det;
    p.karea = reinterpret_cast<float*>(w);
    c->count = count;
    p.o = o;
    return p;
}

void launch_detections(DetParams& p, int batch, const CandArrays& c, bool e2e, const DetectTransform* tf,
                       DetOut* out, int* counts, cudaStream_t stream) {
    p.c = c;
    p.e2e = e2e ? 1 : 0;
    p.tf = tf;
    p.out = out;
    p.counts = counts;
    int cap = 1;
    while (cap < c.count && cap < kSortCap) cap <<= 1;
    p.sort_cap = cap;
    static PerDeviceOnce once;
    once_per_device(once, [] {
        set_max_dynamic_smem(detections_kernel, kSortCap * (int)sizeof(uint64_t), "detections_kernel");
    });
    detections_kernel<<<batch, kSelThreads, sizeof(uint64_t) * cap, stream>>>(p);
    launch_check("detections_kernel");
}

}  // namespace

void decode_detections(const float* x, int batch, long img_stride, long a_stride, long f_stride, int count,
                       int class_fields, bool e2e, const DetectTransform* tf, const DetectOptions& o, DetOut* out,
                       int* counts, int* err, void* ws, cudaStream_t stream) {
    CandArrays c{};
    DetParams p = carve(batch, count, o, ws, &c);
    DecodedCandParams q{};
    q.x = x;
    q.img_stride = img_stride;
    q.a_stride = a_stride;
    q.f_stride = f_stride;
    q.class_fields = class_fields;
    q.e2e = e2e ? 1 : 0;
    q.confidence = o.confidence;
    q.c = c;
    q.err = err;
    decoded_candidates_kernel<<<dim3((count + 255) / 256, batch), 256, 0, stream>>>(q);
    launch_check("decoded_candidates_kernel");
    launch_detections(p, batch, c, e2e, tf, out, counts, stream);
}

void detect_raw(const DetectLevelSrc* levels, int nlevels, int batch, int bins, int nc, int cls_pitch, int box_pitch,
                const DetectTransform* tf, const DetectOptions& o, DetOut* out, int* counts, void* ws,
                cudaStream_t stream) {
    if (nlevels < 1 || nlevels > 3) throw std::runtime_error("detect_raw: 1..3 levels");
    if (cls_pitch % 4 || box_pitch % 4 || cls_pitch < nc || box_pitch < 4 * bins)
        throw std::runtime_error("detect_raw: row pitches must cover the channels in whole float4s");
    RawCandParams q{};
    q.start[0] = 0;
    for (int l = 0; l < nlevels; l++) {
        const DetectLevelSrc& L = levels[l];
        if (L.box_s[1] != 1 || L.cls_s[1] != 1 || ((uintptr_t)L.box & 15) || ((uintptr_t)L.cls & 15) ||
            L.box_s[3] % 4 || L.cls_s[3] % 4 || L.box_s[2] % 4 || L.cls_s[2] % 4 || L.box_s[0] % 4 ||
            L.cls_s[0] % 4)
            throw std::runtime_error("detect_raw: channels-last rows aligned to 16 bytes expected");
        q.lv[l] = L;
        q.start[l + 1] = q.start[l] + L.h * L.w;
    }
    const int count = q.start[nlevels];
    CandArrays c{};
    DetParams p = carve(batch, count, o, ws, &c);
    q.nlevels = nlevels;
    q.bins = bins;
    q.nc = nc;
    q.cls_pitch = cls_pitch;
    q.box_pitch = box_pitch;
    q.confidence = o.confidence;
    q.c = c;
    if (std::max(cls_pitch, box_pitch) > kMaxRawPitch)
        throw std::runtime_error("detect_raw: rows above 256 floats");
    const int smem = (int)sizeof(float) * kRawAnchors * (std::max(cls_pitch, box_pitch) + 1);
    static PerDeviceOnce once;
    once_per_device(once, [] {
        set_max_dynamic_smem(raw_candidates_kernel, (int)sizeof(float) * kRawAnchors * (kMaxRawPitch + 1),
                             "raw_candidates_kernel");
    });
    raw_candidates_kernel<<<dim3((count + kRawAnchors - 1) / kRawAnchors, batch), kRawAnchors, smem, stream>>>(q);
    launch_check("raw_candidates_kernel");
    launch_detections(p, batch, c, false, tf, out, counts, stream);
}

}  // namespace sy
