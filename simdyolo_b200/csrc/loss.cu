// Detection loss on device: DFL decode, task-aligned assigner (TAL), BCE, CIoU and DFL with their
// gradients (DetectionLoss.Compute, src/SimdYolo.Training/DetectionLoss.cs:19-149; CIoU and its
// forward-mode derivatives BoxMath.Ciou / Differential, DetectionLoss.cs:154-183).
//
// Everything that decides the assignment (DFL softmax expectation, decoded boxes, inside test,
// CIoU value, sigmoid, metric, top-k order) is evaluated with round-to-nearest intrinsics and the
// deterministic exp / atan of common.cuh in the reference's expression order, so the assigned
// anchor sets equal the CPU restatement bit for bit.  Loss values and gradients use ordinary
// arithmetic (tolerance-checked).
//
// Kernels per step:  decode (image x anchor) -> topk (gt x image) -> assign (image) ->
//                    bce (anchor rows) -> box (positives) -> finalize (image).
#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kMaxLevels = 3;
constexpr int kMaxTopk = 16;
constexpr int kMaxBceSlots = 8;   // classes per lane in bce_kernel: 3 (nc <= 96) or 8 (nc <= 256)
constexpr int kMaxBatchFold = 64;   // images per pass of cls_bias_fold_kernel
constexpr int kMaxSel = 1024;  // max boxes * topk handled by one image's assignment

struct LossParams {
    LevelIO lv[kMaxLevels];
    int nlevels;
    int level_start[kMaxLevels + 1];
    int anchors;
    int batch, nc, bins, topk, topk2;
    float grad_scale;
    int backward;
    int round_grad;       // logit gradients stored rounded to the nearest TF32 (TF32 conv operands)
    int serial_cls;       // class loss summed in float one term at a time, in the reference's order
    const TruthBox* truth;
    const int* box_off;   // [batch + 1]
    int max_boxes;
    // workspace
    float* dec;           // [batch][anchors][4] decoded xyxy (pixels)
    float* expv;          // [batch][anchors][4] expected distances
    int* sel;             // [batch][max_boxes][topk] anchor or -1
    int* pos_anchor;      // [batch][kMaxSel]
    int* pos_gt;
    float* pos_score;
    int* pos_count;       // [batch]
    float* score_sum;     // [batch]
    double* bce_part;     // [batch][bce_blocks]
    int bce_blocks;
    float* cls_bias_part; // [batch][level][bce_blocks][nc] block partial sums of the class-logit gradient
    float* box_bias_part; // [batch][level][64] per-image sums of the box-logit gradient over the positives
    float* pos_box;       // [batch][kMaxSel] box loss term
    float* pos_dfl;       // [batch][kMaxSel] dfl loss term
    LossOut out;
};

// ---------------------------------------------------------------- exact float helpers
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }

// Differential (DetectionLoss.cs:154-164): value plus 4 partial derivatives.
struct Dif {
    float v, g[4];
};
__device__ __forceinline__ Dif dconst(float v) { return Dif{v, {0.f, 0.f, 0.f, 0.f}}; }
__device__ __forceinline__ Dif dvar(float v, int i) {
    Dif r{v, {0.f, 0.f, 0.f, 0.f}};
    r.g[i] = 1.f;
    return r;
}
__device__ __forceinline__ Dif dadd(const Dif& a, const Dif& b) {
    Dif r;
    r.v = fadd(a.v, b.v);
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fadd(a.g[i], b.g[i]);
    return r;
}
__device__ __forceinline__ Dif dsub(const Dif& a, const Dif& b) {
    Dif r;
    r.v = fsub(a.v, b.v);
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fsub(a.g[i], b.g[i]);
    return r;
}
__device__ __forceinline__ Dif dmul(const Dif& a, const Dif& b) {
    Dif r;
    r.v = fmul(a.v, b.v);
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fadd(fmul(a.g[i], b.v), fmul(b.g[i], a.v));
    return r;
}
__device__ __forceinline__ Dif ddiv(const Dif& a, const Dif& b) {
    Dif r;
    r.v = fdiv(a.v, b.v);
    const float d = fmul(b.v, b.v);
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fdiv(fsub(fmul(a.g[i], b.v), fmul(b.g[i], a.v)), d);
    return r;
}
__device__ __forceinline__ Dif dmin(const Dif& a, const Dif& b) {
    if (a.v < b.v) return a;
    if (a.v > b.v) return b;
    Dif r;
    r.v = a.v;
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fmul(fadd(a.g[i], b.g[i]), .5f);
    return r;
}
__device__ __forceinline__ Dif dmax(const Dif& a, const Dif& b) {
    if (a.v > b.v) return a;
    if (a.v < b.v) return b;
    Dif r;
    r.v = a.v;
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fmul(fadd(a.g[i], b.g[i]), .5f);
    return r;
}
__device__ __forceinline__ Dif datan(const Dif& a) {
    Dif r;
    r.v = det_atanf(a.v);
    const float d = fadd(1.f, fmul(a.v, a.v));
#pragma unroll
    for (int i = 0; i < 4; i++) r.g[i] = fdiv(a.g[i], d);
    return r;
}

// BoxMath.Ciou (DetectionLoss.cs:171-183); alpha is a stopped gradient.
__device__ float ciou(const float p[4], const float t[4], float* grad) {
    const float eps = 1e-7f;
    const Dif x1 = dvar(p[0], 0), y1 = dvar(p[1], 1), x2 = dvar(p[2], 2), y2 = dvar(p[3], 3);
    const Dif w1 = dsub(x2, x1), h1 = dadd(dsub(y2, y1), dconst(eps));
    const float w2 = fsub(t[2], t[0]), h2 = fadd(fsub(t[3], t[1]), eps);
    const Dif iw = dmax(dsub(dmin(x2, dconst(t[2])), dmax(x1, dconst(t[0]))), dconst(0.f));
    const Dif ih = dmax(dsub(dmin(y2, dconst(t[3])), dmax(y1, dconst(t[1]))), dconst(0.f));
    const Dif inter = dmul(iw, ih);
    const Dif uni = dadd(dsub(dadd(dmul(w1, h1), dconst(fmul(w2, h2))), inter), dconst(eps));
    const Dif iou = ddiv(inter, uni);
    const Dif cw = dsub(dmax(x2, dconst(t[2])), dmin(x1, dconst(t[0])));
    const Dif ch = dsub(dmax(y2, dconst(t[3])), dmin(y1, dconst(t[1])));
    const Dif dx = dsub(dsub(dconst(fadd(t[0], t[2])), x1), x2);
    const Dif dy = dsub(dsub(dconst(fadd(t[1], t[3])), y1), y2);
    const Dif rho = ddiv(dadd(dmul(dx, dx), dmul(dy, dy)), dconst(4.0f));
    const float pi = 3.14159265358979323846f;
    const float vscale = fdiv(4.0f, fmul(pi, pi));
    Dif v = dsub(datan(dconst(fdiv(w2, h2))), datan(ddiv(w1, h1)));
    v = dmul(dmul(v, v), dconst(vscale));
    const float alpha = fdiv(v.v, fadd(fadd(fsub(v.v, iou.v), 1.f), eps));
    const Dif c2 = dadd(dadd(dmul(cw, cw), dmul(ch, ch)), dconst(eps));
    const Dif res = dsub(dsub(iou, ddiv(rho, c2)), dmul(v, dconst(alpha)));
    if (grad)
        for (int i = 0; i < 4; i++) grad[i] = res.g[i];
    return res.v;
}

__device__ __forceinline__ void anchor_location(const LossParams& p, int a, int& level, int& row, float& cx, float& cy,
                                                float& stride) {
    level = 0;
    while (level + 1 < p.nlevels && a >= p.level_start[level + 1]) level++;
    const int pix = a - p.level_start[level];
    const Grid& g = p.lv[level].grid;
    const int y = pix / g.w, x = pix - y * g.w;
    row = g.row(y, x);
    stride = p.lv[level].stride;
    cx = fmul(fadd((float)x, .5f), stride);
    cy = fmul(fadd((float)y, .5f), stride);
}

// Inside test with small-box expansion (DetectionLoss.cs:57-60) and alignment metric (:62-63).
__device__ __forceinline__ void tal_metric(const LossParams& p, int b, int a, const TruthBox& box, bool& inside,
                                           float& overlap, float& metric) {
    int level, row;
    float cx, cy, st;
    anchor_location(p, a, level, row, cx, cy, st);
    const float s0 = p.lv[0].stride;
    const float s1 = p.nlevels > 1 ? p.lv[1].stride : fmul(s0, 2.f);
    const float bx = fmul(fadd(box.x1, box.x2), .5f), by = fmul(fadd(box.y1, box.y2), .5f);
    const float bw = fsub(box.x2, box.x1), bh = fsub(box.y2, box.y1);
    const float cw = bw < s0 ? s1 : bw, chh = bh < s0 ? s1 : bh;
    inside = fsub(cx, fsub(bx, fmul(cw, .5f))) > 1e-9f && fsub(fadd(bx, fmul(cw, .5f)), cx) > 1e-9f &&
             fsub(cy, fsub(by, fmul(chh, .5f))) > 1e-9f && fsub(fadd(by, fmul(chh, .5f)), cy) > 1e-9f;
    overlap = 0.f;
    metric = 0.f;
    if (!inside) return;
    const float* d = p.dec + ((long)b * p.anchors + a) * 4;
    const float pb[4] = {d[0], d[1], d[2], d[3]};
    const float tb[4] = {box.x1, box.y1, box.x2, box.y2};
    const float c = ciou(pb, tb, nullptr);
    overlap = fmaxf(0.f, c);
    const LevelIO& L = p.lv[level];
    const float s = det_sigmoid(L.cls[(long)b * L.grid.rows * L.cls_pitch + (long)row * L.cls_pitch + box.cls]);
    metric = fmul(__fsqrt_rn(s), det_pow6(overlap));
}

// ---------------------------------------------------------------- 1. decode
// One thread per (image, anchor, side): the DFL expectation of that side and its decoded coordinate.
__global__ void decode_kernel(LossParams p) {
    const long total = (long)p.batch * p.anchors * 4;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const long ia = i >> 2;
        const int d = (int)(i & 3);
        const int b = (int)(ia / p.anchors), a = (int)(ia - (long)b * p.anchors);
        int level, row;
        float cx, cy, st;
        anchor_location(p, a, level, row, cx, cy, st);
        const LevelIO& L = p.lv[level];
        const float* t = L.box + ((long)b * L.grid.rows + row) * L.box_pitch;
        float e;
        if (p.bins == 1) {
            e = t[d];
        } else {
            float maximum = -INFINITY;
            for (int k = 0; k < 16; k++) maximum = fmaxf(maximum, t[d * 16 + k]);
            float ex[16];
            float sum = 0.f;
            for (int k = 0; k < 16; k++) {
                ex[k] = det_expf(fsub(t[d * 16 + k], maximum));
                sum = fadd(sum, ex[k]);
            }
            float dist = 0.f;
            for (int k = 0; k < 16; k++) dist = fadd(dist, fmul(fdiv(ex[k], sum), (float)k));
            e = dist;
        }
        p.expv[i] = e;
        const float c = (d & 1) ? cy : cx;
        p.dec[i] = d < 2 ? fsub(c, fmul(e, st)) : fadd(c, fmul(e, st));
    }
}

// ---------------------------------------------------------------- 2. per-GT top-k
// Key order = (metric desc, anchor asc) as the bounded PriorityQueue of (metric, -anchor)
// (DetectionLoss.cs:65).  metric >= 0, so its bit pattern orders like the value.
__device__ __forceinline__ unsigned long long make_key(float metric, int a) {
    return ((unsigned long long)__float_as_uint(metric) << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)a);
}

__global__ void __launch_bounds__(256) topk_kernel(LossParams p) {
    const int g = blockIdx.x, b = blockIdx.y;
    const int n = p.box_off[b + 1] - p.box_off[b];
    int* sel = p.sel + ((long)b * p.max_boxes + g) * p.topk;
    if (g >= n) {
        for (int k = threadIdx.x; k < p.topk; k += blockDim.x) sel[k] = -1;
        return;
    }
    const TruthBox box = p.truth[p.box_off[b] + g];
    // each thread keeps its best topk + 1 keys (the extra one for the near-tie check); topk < kMaxTopk
    unsigned long long list[kMaxTopk];
    const int cap = p.topk + 1;
    int cnt = 0;
    for (int a = threadIdx.x; a < p.anchors; a += blockDim.x) {
        bool inside;
        float ov, m;
        tal_metric(p, b, a, box, inside, ov, m);
        const unsigned long long key = make_key(m, a);
        if (cnt == cap && key <= list[cnt - 1]) continue;
        int pos = cnt < cap ? cnt++ : cnt - 1;
        while (pos > 0 && list[pos - 1] < key) {
            list[pos] = list[pos - 1];
            pos--;
        }
        list[pos] = key;
    }
    __shared__ unsigned long long wbest[8];
    __shared__ unsigned long long best_s;
    int head = 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long kth = 0ull;   // key of the k-th (last) selected anchor
    // k = topk: one more round finds the (k+1)-th key, for the near-tie count only
    for (int k = 0; k <= p.topk; k++) {
        unsigned long long cand = head < cnt ? list[head] : 0ull;
        unsigned long long m = cand;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, m, o);
            m = other > m ? other : m;
        }
        if (lane == 0) wbest[warp] = m;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long bm = 0ull;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) bm = wbest[w] > bm ? wbest[w] : bm;
            best_s = bm;
        }
        __syncthreads();
        const unsigned long long bm = best_s;
        if (k == p.topk) {
            const unsigned m_k = (unsigned)(kth >> 32), m_next = (unsigned)(bm >> 32);
            if (threadIdx.x == 0 && p.out.near_ties && m_next > 0u && m_k - m_next <= kNearTieUlps)
                atomicAdd(&p.out.near_ties[b], 1);
            break;
        }
        if (k == p.topk - 1) kth = bm;
        if (bm != 0ull && cand == bm) {
            head++;
            const int a = (int)(0xFFFFFFFFu - (unsigned)(bm & 0xFFFFFFFFull));
            bool inside;
            float ov, mm;
            tal_metric(p, b, a, box, inside, ov, mm);
            sel[k] = inside ? a : -1;
        } else if (bm == 0ull && threadIdx.x == 0) {
            sel[k] = -1;
        }
        __syncthreads();
    }
}

// ---------------------------------------------------------------- 3. per-image assignment
// Conflicts (DetectionLoss.cs:69-81), max alignment / overlap per GT (:92-94), scores and their
// sum in anchor order (:95-98).
__global__ void __launch_bounds__(256) assign_kernel(LossParams p) {
    extern __shared__ int owner_s[];   // [anchors]: -1 unselected, g selected by GT g alone, -2 by several
    const int b = blockIdx.x;
    const int n = p.box_off[b + 1] - p.box_off[b];
    const TruthBox* truth = p.truth + p.box_off[b];
    __shared__ int anc[kMaxSel];
    __shared__ int own[kMaxSel];
    __shared__ float al[kMaxSel], ov[kMaxSel];
    __shared__ float max_al[128], max_ov[128];
    __shared__ int count_s;
    __shared__ bool keep_s[kMaxSel];
    // dense outputs of this image start cleared
    if (p.out.assigned)
        for (int a = threadIdx.x; a < p.anchors; a += blockDim.x) p.out.assigned[(long)b * p.anchors + a] = -1;
    if (p.out.scores)
        for (int a = threadIdx.x; a < p.anchors; a += blockDim.x) p.out.scores[(long)b * p.anchors + a] = 0.f;
    // the selected (gt, anchor) pairs, compacted in anchor order: an anchor picked by one GT keeps it as
    // owner, one picked by several is marked -2 (a conflict resolved below); the owner map does not
    // depend on the order in which the pairs are visited
    for (int a = threadIdx.x; a < p.anchors; a += blockDim.x) owner_s[a] = -1;
    __syncthreads();
    for (int i = threadIdx.x; i < n * p.topk; i += blockDim.x) {
        const int g = i / p.topk;
        const int a = p.sel[((long)b * p.max_boxes + g) * p.topk + (i - g * p.topk)];
        if (a < 0) continue;
        if (atomicCAS(&owner_s[a], -1, g) != -1) atomicExch(&owner_s[a], -2);
    }
    __syncthreads();
    {
        // block-wide exclusive scan of "selected" over contiguous anchor ranges per thread
        __shared__ int part_s[256];
        const int per = (p.anchors + blockDim.x - 1) / blockDim.x;
        const int a0 = min(p.anchors, (int)threadIdx.x * per), a1 = min(p.anchors, a0 + per);
        int cnt = 0;
        for (int a = a0; a < a1; a++) cnt += owner_s[a] != -1;
        part_s[threadIdx.x] = cnt;
        __syncthreads();
        if (threadIdx.x == 0) {
            int run = 0;
            for (int t = 0; t < (int)blockDim.x; t++) {
                const int v = part_s[t];
                part_s[t] = run;
                run += v;
            }
            count_s = min(run, kMaxSel);
        }
        __syncthreads();
        int pos = part_s[threadIdx.x];
        for (int a = a0; a < a1; a++)
            if (owner_s[a] != -1) {
                if (pos < kMaxSel) {
                    anc[pos] = a;
                    own[pos] = owner_s[a];
                }
                pos++;
            }
    }
    for (int g = threadIdx.x; g < 128; g += blockDim.x) {
        max_al[g] = 0.f;
        max_ov[g] = 0.f;
    }
    __syncthreads();
    const int c = count_s;
    // conflicts: argmax overlap over ALL gts, strict >, best starts at -1 (first max wins)
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
        const int a = anc[i];
        int chosen = own[i];
        if (chosen == -2) {
            float best = -1.f, second = -1.f;
            for (int g = 0; g < n; g++) {
                bool inside;
                float o, m;
                tal_metric(p, b, a, truth[g], inside, o, m);
                if (o > best) {
                    second = best;
                    best = o;
                    chosen = g;
                } else if (o > second) {
                    second = o;
                }
            }
            own[i] = chosen;
            if (p.out.near_ties && second > 0.f &&
                __float_as_uint(best) - __float_as_uint(second) <= kNearTieUlps)
                atomicAdd(&p.out.near_ties[b], 1);
        }
        bool inside;
        float o, m;
        tal_metric(p, b, a, truth[chosen], inside, o, m);
        al[i] = m;
        ov[i] = o;
    }
    __syncthreads();
    if (threadIdx.x == 0 && p.topk2 != p.topk) {
        // second top-k after the conflicts (DetectionLoss.cs:83-91): per GT keep the topk2 anchors
        // ranked by (alignment if selected else 0) descending, then by anchor index.  Selected anchors
        // with positive alignment come first; a selected anchor with zero alignment survives only if
        // it is among the lowest-index anchors of zero key that fill the remaining slots.
        for (int i = 0; i < c; i++) {
            const int g = own[i];
            int better = 0, pos_below = 0, npos = 0;
            for (int j = 0; j < c; j++) {
                if (own[j] != g || !(al[j] > 0.f)) continue;
                npos++;
                if (anc[j] < anc[i]) pos_below++;
                if (al[j] > al[i] || (al[j] == al[i] && anc[j] < anc[i])) better++;
            }
            if (al[i] > 0.f) keep_s[i] = better < p.topk2;
            else keep_s[i] = npos < p.topk2 && anc[i] - pos_below < p.topk2 - npos;
        }
        int kept = 0;   // compact after every decision (the decisions read the whole list)
        for (int i = 0; i < c; i++)
            if (keep_s[i]) {
                anc[kept] = anc[i];
                own[kept] = own[i];
                al[kept] = al[i];
                ov[kept] = ov[i];
                kept++;
            }
        count_s = kept;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int c = count_s;
        for (int i = 0; i < c; i++) {
            const int g = own[i];
            max_al[g] = fmaxf(max_al[g], al[i]);
            max_ov[g] = fmaxf(max_ov[g], ov[i]);
        }
        float sum = 0.f;
        for (int i = 0; i < c; i++) {
            const int g = own[i];
            const float s = fdiv(fmul(al[i], max_ov[g]), fadd(max_al[g], 1e-9f));
            sum = fadd(sum, s);
            p.pos_anchor[(long)b * kMaxSel + i] = anc[i];
            p.pos_gt[(long)b * kMaxSel + i] = g;
            p.pos_score[(long)b * kMaxSel + i] = s;
            if (p.out.assigned) p.out.assigned[(long)b * p.anchors + anc[i]] = g;
            if (p.out.scores) p.out.scores[(long)b * p.anchors + anc[i]] = s;
        }
        p.pos_count[b] = c;
        p.score_sum[b] = fmaxf(1.f, sum);
    }
}

// ---------------------------------------------------------------- 4. BCE over all anchors x classes
// (DetectionLoss.cs:104-111).  One warp per anchor row, lanes over classes.
template <int kBceSlots>
__global__ void __launch_bounds__(256) bce_kernel(LossParams p, const int* dense_assigned, const float* dense_scores) {
    const int b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const float inv = .5f / p.score_sum[b];
    const bool bias = p.backward && p.cls_bias_part;
    double acc = 0.0;
    // this lane's class-logit gradient sums per (level, class slot c = lane + 32 k), for the bias gradient
    float bsum[kMaxLevels][kBceSlots];
#pragma unroll
    for (int l = 0; l < kMaxLevels; l++)
#pragma unroll
        for (int k = 0; k < kBceSlots; k++) bsum[l][k] = 0.f;
    for (int a = blockIdx.x * 8 + warp; a < p.anchors; a += gridDim.x * 8) {
        int level, row;
        float cx, cy, st;
        anchor_location(p, a, level, row, cx, cy, st);
        const LevelIO& L = p.lv[level];
        const long off = ((long)b * L.grid.rows + row) * L.cls_pitch;
        const int g = dense_assigned[(long)b * p.anchors + a];
        const int tcls = g >= 0 ? p.truth[p.box_off[b] + g].cls : -1;
        const float w = g >= 0 ? dense_scores[(long)b * p.anchors + a] : 0.f;
        float part = 0.f;
#pragma unroll
        for (int k = 0; k < kBceSlots; k++) {
            const int c = lane + 32 * k;
            if (c >= p.nc) break;
            const float x = L.cls[off + c];
            const float t = c == tcls ? w : 0.f;
            // e = exp(-|x|) serves both the stable log-sum-exp and the sigmoid (HeadOperations.cs:222)
            const float e = __expf(-fabsf(x));
            part += (fmaxf(x, 0.f) - x * t + log1pf(e)) * inv;
            if (p.backward) {
                const float s = __fdividef(x >= 0.f ? 1.f : e, 1.f + e);
                const float gr = (s - t) * inv * p.grad_scale;
                L.dcls[off + c] = p.round_grad ? tf32_rna(gr) : gr;
#pragma unroll
                for (int l = 0; l < kMaxLevels; l++)
                    if (l == level) bsum[l][k] += gr;
            }
        }
        acc += (double)part;
    }
    acc = warp_sum_d(acc);
    __shared__ double red[8];
    __shared__ float bred[8][kMaxLevels][kBceSlots * 32];
    if (lane == 0) red[warp] = acc;
    if (bias)
#pragma unroll
        for (int l = 0; l < kMaxLevels; l++)
#pragma unroll
            for (int k = 0; k < kBceSlots; k++) bred[warp][l][lane + 32 * k] = bsum[l][k];
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; w++) t += red[w];
        p.bce_part[(long)b * p.bce_blocks + blockIdx.x] = t;
    }
    if (bias)
        for (int i = threadIdx.x; i < p.nlevels * p.nc; i += blockDim.x) {
            const int l = i / p.nc, c = i - l * p.nc;
            float t = 0.f;
            for (int w = 0; w < 8; w++) t += bred[w][l][c];   // warps in order
            p.cls_bias_part[(((long)b * kMaxLevels + l) * p.bce_blocks + blockIdx.x) * p.nc + c] = t;
        }
}

// Bias gradients of the class convs.  Block (level, 32 classes): lane = class, warp w sums the block partials
// of images w, w + 8, ... (each image's partials in block order), then warp 0 adds the images in order into
// the level's bias gradient.
__global__ void __launch_bounds__(256) cls_bias_fold_kernel(LossParams p) {
    __shared__ float img_s[kMaxBatchFold][32];
    const int l = blockIdx.y, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + lane;
    const bool on = c < p.nc && p.lv[l].cls_bias_grad != nullptr;
    for (int b0 = 0; b0 < p.batch; b0 += kMaxBatchFold) {
        const int nb = min(kMaxBatchFold, p.batch - b0);
        for (int i = warp; i < nb; i += 8) {
            float img = 0.f;
            if (on) {
                const float* part = p.cls_bias_part + ((long)(b0 + i) * kMaxLevels + l) * p.bce_blocks * p.nc + c;
#pragma unroll 8
                for (int k = 0; k < p.bce_blocks; k++) img += part[(long)k * p.nc];
            }
            img_s[i][lane] = img;
        }
        __syncthreads();
        if (warp == 0 && on) {
            float total = 0.f;
            for (int i = 0; i < nb; i++) total += img_s[i][lane];
            p.lv[l].cls_bias_grad[c] += total;
        }
        __syncthreads();
    }
}

// Bias gradients of the box convs: the box-logit gradient is zero except at the positives.  box_bias_image:
// block per image, thread per channel, the sum over the image's positives in anchor order per level;
// box_bias_fold: thread per (level, channel), images in order into the level's bias gradient.
__global__ void box_bias_image_kernel(LossParams p) {
    const int b = blockIdx.x, ch = threadIdx.x;
    if (ch >= 4 * p.bins) return;
    float acc[kMaxLevels] = {0.f, 0.f, 0.f};
    const int n = p.pos_count[b];
    for (int i = 0; i < n; i++) {
        const int a = p.pos_anchor[(long)b * kMaxSel + i];
        int level, row;
        float cx, cy, st;
        anchor_location(p, a, level, row, cx, cy, st);
        const LevelIO& L = p.lv[level];
        const float v = L.dbox[((long)b * L.grid.rows + row) * L.box_pitch + ch];
#pragma unroll
        for (int l = 0; l < kMaxLevels; l++)
            if (l == level) acc[l] += v;
    }
    for (int l = 0; l < p.nlevels; l++) p.box_bias_part[((long)b * kMaxLevels + l) * 64 + ch] = acc[l];
}

__global__ void box_bias_fold_kernel(LossParams p) {
    const int l = blockIdx.y, ch = threadIdx.x;
    if (ch >= 4 * p.bins || !p.lv[l].box_bias_grad) return;
    float total = 0.f;
    for (int b = 0; b < p.batch; b++) total += p.box_bias_part[((long)b * kMaxLevels + l) * 64 + ch];
    p.lv[l].box_bias_grad[ch] += total;
}

// ---------------------------------------------------------------- 5. CIoU + DFL for positives
// (DetectionLoss.cs:112-146).  One warp per positive; lane l handles bins of side l / 16 ... via loop.
__global__ void __launch_bounds__(256) box_kernel(LossParams p) {
    const int b = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = blockIdx.x * 8 + warp;
    if (i >= p.pos_count[b]) return;
    const int a = p.pos_anchor[(long)b * kMaxSel + i];
    const int g = p.pos_gt[(long)b * kMaxSel + i];
    const float weight = p.pos_score[(long)b * kMaxSel + i];
    const float ss = p.score_sum[b];
    const TruthBox tb = p.truth[p.box_off[b] + g];
    int level, row;
    float cx, cy, st;
    anchor_location(p, a, level, row, cx, cy, st);
    const LevelIO& L = p.lv[level];
    const float* dec = p.dec + ((long)b * p.anchors + a) * 4;
    const float* ex = p.expv + ((long)b * p.anchors + a) * 4;
    const float invs = 1.f / st;
    const float pg[4] = {dec[0] * invs, dec[1] * invs, dec[2] * invs, dec[3] * invs};
    const float tg[4] = {tb.x1 * invs, tb.y1 * invs, tb.x2 * invs, tb.y2 * invs};
    float cg[4];
    const float ci = ciou(pg, tg, cg);
    const float box_scale = 7.5f * weight / ss;
    float coord[4];
    for (int d = 0; d < 4; d++) coord[d] = -cg[d] * (box_scale * p.grad_scale);
    const float dist_grad[4] = {-coord[0], -coord[1], coord[2], coord[3]};
    const float dists[4] = {(cx - tb.x1) / st, (cy - tb.y1) / st, (tb.x2 - cx) / st, (tb.y2 - cy) / st};
    const long off = ((long)b * L.grid.rows + row) * L.box_pitch;
    const float* t = L.box + off;
    float dfl = 0.f;
    if (p.bins == 1) {
        for (int d = 0; d < 4; d++) {
            const float extent = (float)(d % 2 == 0 ? p.lv[0].grid.w : p.lv[0].grid.h) * p.lv[0].stride;
            const float norm = st / extent, delta = ex[d] - dists[d];
            const float l1 = 1.5f * weight / (4 * ss);
            dfl += fabsf(delta) * norm * l1;
            if (p.backward && lane == 0) {
                const float sign = delta > 0 ? 1.f : delta < 0 ? -1.f : 0.f;
                const float gr = dist_grad[d] + sign * norm * l1 * p.grad_scale;
                L.dbox[off + d] = p.round_grad ? tf32_rna(gr) : gr;
            }
        }
    } else {
        const float scale = 1.5f * weight / (4 * ss);
        for (int d = 0; d < 4; d++) {
            const float hi = 16 - 1 - .01f;
            float target = dists[d];
            target = target < 0 ? 0 : target > hi ? hi : target;
            const int left = (int)target;
            const float rw = target - left;
            // lanes 0..15 hold the bins of this side
            const float v = lane < 16 ? t[d * 16 + lane] : -INFINITY;
            float mx = v;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            mx = __shfl_sync(0xffffffffu, mx, 0);
            const float e = lane < 16 ? expf(v - mx) : 0.f;
            const float es = __shfl_sync(0xffffffffu, warp_sum(e), 0);
            const float log_sum = mx + logf(es);
            const float vl = t[d * 16 + left], vr = t[d * 16 + left + 1];
            dfl += scale * (log_sum - (1 - rw) * vl - rw * vr);
            if (p.backward && lane < 16) {
                // probabilities of the decode (det_expf softmax), as the reference reuses them
                float mxd = -INFINITY;
                for (int k = 0; k < 16; k++) mxd = fmaxf(mxd, t[d * 16 + k]);
                float sum = 0.f, mine = 0.f;
                for (int k = 0; k < 16; k++) {
                    const float ek = det_expf(fsub(t[d * 16 + k], mxd));
                    sum = fadd(sum, ek);
                    if (k == lane) mine = ek;
                }
                const float pr = fdiv(mine, sum);
                const float tp = lane == left ? 1 - rw : lane == left + 1 ? rw : 0.f;
                const float gr = pr * (lane - ex[d]) * dist_grad[d] + scale * (pr - tp) * p.grad_scale;
                L.dbox[off + d * 16 + lane] = p.round_grad ? tf32_rna(gr) : gr;
            }
        }
    }
    if (lane == 0) {
        p.pos_box[(long)b * kMaxSel + i] = (1 - ci) * box_scale;
        p.pos_dfl[(long)b * kMaxSel + i] = dfl;
    }
}

// ---------------------------------------------------------------- 6. per-image totals
__global__ void finalize_kernel(LossParams p) {
    const int b = blockIdx.x;
    if (threadIdx.x != 0) return;
    double cls = 0.0;
    for (int k = 0; k < p.bce_blocks; k++) cls += p.bce_part[(long)b * p.bce_blocks + k];
    float box = 0.f, dfl = 0.f;
    const int c = p.pos_count[b];
    for (int i = 0; i < c; i++) {
        box += p.pos_box[(long)b * kMaxSel + i];
        dfl += p.pos_dfl[(long)b * kMaxSel + i];
    }
    p.out.loss[b * 4 + 0] = box;
    p.out.loss[b * 4 + 1] = (float)cls;
    p.out.loss[b * 4 + 2] = dfl;
    p.out.loss[b * 4 + 3] = 0.f;
    p.out.positives[b] = c;
    p.out.connected[b] = (p.backward && c > 0) ? 1 : 0;
}

// The class loss as the reference accumulates it (DetectionLoss.cs:103-109): one float running sum over
// anchors in order, and per anchor over the classes in order, of
//   (max(x, 0) - x t + log(1 + exp(-|x|))) * (0.5 / scoreSum)
// each operation rounded to nearest, with full-precision expf / logf.  Over the 80 x 8400 terms of a
// 640-pixel image that sum differs from the exact one by about 1e-3 (each addition to a running sum near
// 5 rounds a term of about 1e-5 to the running sum's spacing); the reduction in bce_kernel returns the
// exact sum, this kernel the reference's value.  One block per image: threads 32.. compute the terms of
// the next chunk of anchors into shared memory while thread 0 adds up the current chunk.
constexpr int kSerialChunk = 32;   // anchors per chunk
__global__ void __launch_bounds__(256) bce_serial_kernel(LossParams p, const int* dense_assigned, const float* dense_scores) {
    extern __shared__ float terms[];   // [2][kSerialChunk * nc]
    const int b = blockIdx.x;
    const int per = kSerialChunk * p.nc;
    const float inv = __fdiv_rn(.5f, p.score_sum[b]);
    const int chunks = (p.anchors + kSerialChunk - 1) / kSerialChunk;
    auto fill = [&](int k, int tid, int nthreads) {
        float* dst = terms + (k & 1) * per;
        for (int i = tid; i < per; i += nthreads) {
            const int a = k * kSerialChunk + i / p.nc, c = i - (i / p.nc) * p.nc;
            float term = 0.f;
            if (a < p.anchors) {
                int level, row;
                float cx, cy, st;
                anchor_location(p, a, level, row, cx, cy, st);
                const LevelIO& L = p.lv[level];
                const float x = L.cls[((long)b * L.grid.rows + row) * L.cls_pitch + c];
                const int g = dense_assigned[(long)b * p.anchors + a];
                const float t = (g >= 0 && p.truth[p.box_off[b] + g].cls == c) ? dense_scores[(long)b * p.anchors + a]
                                                                                : 0.f;
                const float lg = logf(__fadd_rn(1.f, expf(-fabsf(x))));
                term = __fmul_rn(__fadd_rn(__fsub_rn(fmaxf(x, 0.f), __fmul_rn(x, t)), lg), inv);
            }
            dst[i] = term;
        }
    };
    fill(0, threadIdx.x, blockDim.x);
    __syncthreads();
    float acc = 0.f;
    for (int k = 0; k < chunks; k++) {
        if (threadIdx.x == 0) {
            const float* src = terms + (k & 1) * per;
            const int n = min(per, (p.anchors - k * kSerialChunk) * p.nc);
#pragma unroll 8
            for (int i = 0; i < n; i++) acc = __fadd_rn(acc, src[i]);
        } else if (threadIdx.x >= 32 && k + 1 < chunks) {
            fill(k + 1, threadIdx.x - 32, blockDim.x - 32);
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) p.out.loss[b * 4 + 1] = acc;
}

constexpr int kBceBlocks = 64;

size_t align_up(size_t v) { return (v + 255) & ~size_t(255); }

}  // namespace

size_t loss_workspace_bytes(int batch, int anchors, int max_boxes, int topk, int nc) {
    size_t s = 0;
    s += align_up((size_t)batch * anchors * 4 * sizeof(float)) * 2;  // dec, expv
    s += align_up((size_t)batch * max_boxes * topk * sizeof(int));   // sel
    s += align_up((size_t)batch * kMaxSel * sizeof(int)) * 2;        // pos anchor / gt
    s += align_up((size_t)batch * kMaxSel * sizeof(float)) * 3;      // score, box, dfl terms
    s += align_up((size_t)batch * sizeof(int));                      // pos count
    s += align_up((size_t)batch * sizeof(float));                    // score sum
    s += align_up((size_t)batch * kBceBlocks * sizeof(double));      // bce partials
    s += align_up((size_t)batch * kMaxLevels * kBceBlocks * nc * sizeof(float));   // class bias partials
    s += align_up((size_t)batch * kMaxLevels * 64 * sizeof(float));                // box bias per image
    s += align_up((size_t)batch * anchors * sizeof(int));            // dense assigned (if not given)
    s += align_up((size_t)batch * anchors * sizeof(float));          // dense scores (if not given)
    return s;
}

static void split_check(cudaError_t e) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("detection_loss: ") + cudaGetErrorString(e));
}

void detection_loss(const LevelIO* levels, int nlevels, int batch, int nc, int bins, const TruthBox* truth,
                    const int* box_offsets, int max_boxes, int topk, int topk2, float grad_scale, int backward, void* workspace,
                    const LossOut& out, cudaStream_t stream, bool round_grad, bool serial_cls, const LossSplit* split) {
    if (split && serial_cls) throw std::runtime_error("detection_loss: the serial class sum runs on one stream");
    LossParams p;
    p.round_grad = round_grad ? 1 : 0;
    p.serial_cls = serial_cls ? 1 : 0;
    p.nlevels = nlevels;
    p.level_start[0] = 0;
    for (int l = 0; l < nlevels; l++) {
        p.lv[l] = levels[l];
        p.level_start[l + 1] = p.level_start[l] + levels[l].grid.h * levels[l].grid.w;
    }
    p.anchors = p.level_start[nlevels];
    p.batch = batch;
    p.nc = nc;
    p.bins = bins;
    p.topk = topk;
    p.topk2 = topk2;
    if (topk2 < 1 || topk2 > topk) throw std::runtime_error("detection_loss: topk2 must be in [1, topk]");
    if (topk < 1 || topk >= kMaxTopk) throw std::runtime_error("detection_loss: topk must be in [1, 15]");
    p.grad_scale = grad_scale;
    p.backward = backward;
    p.truth = truth;
    p.box_off = box_offsets;
    p.max_boxes = max_boxes;
    uint8_t* w = static_cast<uint8_t*>(workspace);
    auto take = [&](size_t bytes) {
        uint8_t* r = w;
        w += align_up(bytes);
        return r;
    };
    p.dec = (float*)take((size_t)batch * p.anchors * 4 * sizeof(float));
    p.expv = (float*)take((size_t)batch * p.anchors * 4 * sizeof(float));
    p.sel = (int*)take((size_t)batch * max_boxes * topk * sizeof(int));
    p.pos_anchor = (int*)take((size_t)batch * kMaxSel * sizeof(int));
    p.pos_gt = (int*)take((size_t)batch * kMaxSel * sizeof(int));
    p.pos_score = (float*)take((size_t)batch * kMaxSel * sizeof(float));
    p.pos_box = (float*)take((size_t)batch * kMaxSel * sizeof(float));
    p.pos_dfl = (float*)take((size_t)batch * kMaxSel * sizeof(float));
    p.pos_count = (int*)take((size_t)batch * sizeof(int));
    p.score_sum = (float*)take((size_t)batch * sizeof(float));
    p.bce_part = (double*)take((size_t)batch * kBceBlocks * sizeof(double));
    p.bce_blocks = kBceBlocks;
    p.cls_bias_part = (float*)take((size_t)batch * kMaxLevels * kBceBlocks * nc * sizeof(float));
    p.box_bias_part = (float*)take((size_t)batch * kMaxLevels * 64 * sizeof(float));
    bool cls_bias = false, box_bias = false;
    for (int l = 0; l < nlevels; l++) {
        cls_bias |= backward && levels[l].cls_bias_grad != nullptr;
        box_bias |= backward && levels[l].box_bias_grad != nullptr;
    }
    if (!cls_bias) p.cls_bias_part = nullptr;
    if (nc > 32 * kMaxBceSlots) throw std::runtime_error("detection_loss: more than 256 classes");
    int* dense_a = (int*)take((size_t)batch * p.anchors * sizeof(int));
    float* dense_s = (float*)take((size_t)batch * p.anchors * sizeof(float));
    p.out = out;
    if (out.near_ties) cudaMemsetAsync(out.near_ties, 0, sizeof(int) * (size_t)batch, stream);
    if (!p.out.assigned) p.out.assigned = dense_a;
    if (!p.out.scores) p.out.scores = dense_s;

    const long total = (long)batch * p.anchors;
    decode_kernel<<<(int)std::min<long>(148L * 32, (4 * total + 255) / 256), 256, 0, stream>>>(p);
    launch_check("decode_kernel");
    if (max_boxes > 0) topk_kernel<<<dim3(max_boxes, batch), 256, 0, stream>>>(p);
    launch_check("topk_kernel");
    const size_t owner_bytes = sizeof(int) * (size_t)p.anchors;
    static PerDeviceOnce attr_once;   // devices whose kernel attribute is set
    once_per_device(attr_once, [] { set_max_dynamic_smem(assign_kernel, 160 * 1024, "assign_kernel attribute"); });
    if (owner_bytes > 160 * 1024) throw std::runtime_error("detection_loss: too many anchors");
    assign_kernel<<<batch, 256, owner_bytes, stream>>>(p);
    launch_check("assign_kernel");
    // class part (BCE, class bias fold) on cls, box part on stream; one stream unless split
    cudaStream_t cls = stream;
    if (split) {
        cls = split->cls_stream;
        split_check(cudaEventRecord(split->assigned, stream));
        split_check(cudaStreamWaitEvent(cls, split->assigned, 0));
    }
    if (backward)
        for (int l = 0; l < nlevels; l++) {
            const LevelIO& L = levels[l];
            // box gradients are sparse: clear the whole level, positives are scattered below
            cudaMemsetAsync(L.dbox, 0, (size_t)batch * L.grid.rows * L.box_pitch * sizeof(float), stream);
        }
    if (nc <= 96)
        bce_kernel<3><<<dim3(kBceBlocks, batch), 256, 0, cls>>>(p, p.out.assigned, p.out.scores);
    else
        bce_kernel<8><<<dim3(kBceBlocks, batch), 256, 0, cls>>>(p, p.out.assigned, p.out.scores);
    launch_check("bce_kernel");
    box_kernel<<<dim3((max_boxes * topk + 7) / 8 > 0 ? (max_boxes * topk + 7) / 8 : 1, batch), 256, 0, stream>>>(p);
    launch_check("box_kernel");
    if (cls_bias) {
        cls_bias_fold_kernel<<<dim3((nc + 31) / 32, nlevels), 256, 0, cls>>>(p);
        launch_check("cls_bias_fold_kernel");
    }
    if (box_bias) {
        box_bias_image_kernel<<<batch, 64, 0, stream>>>(p);
        launch_check("box_bias_image_kernel");
        box_bias_fold_kernel<<<dim3(1, nlevels), 64, 0, stream>>>(p);
        launch_check("box_bias_fold_kernel");
    }
    if (split) {
        // the per-image totals need both parts
        split_check(cudaEventRecord(split->box, stream));
        split_check(cudaStreamWaitEvent(cls, split->box, 0));
    }
    finalize_kernel<<<batch, 32, 0, cls>>>(p);
    launch_check("finalize_kernel");
    if (split) split_check(cudaEventRecord(split->cls_done, cls));
    if (serial_cls) {
        const size_t smem = 2 * (size_t)kSerialChunk * nc * sizeof(float);
        if (smem > 48 * 1024) throw std::runtime_error("detection_loss: too many classes for the serial class sum");
        bce_serial_kernel<<<batch, 256, smem, stream>>>(p, p.out.assigned, p.out.scores);
        launch_check("bce_serial_kernel");
    }
}

}  // namespace sy
