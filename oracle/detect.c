/*
 * Detection post-processing restated on the CPU: TEST INFRASTRUCTURE ONLY (see syo.h).
 *
 *   syo_head_decode        CpuHead.DecodeInto, scalar path (src/SimdYolo/CpuHead.cs:57-120)
 *   syo_end_to_end_topk    PtModel.EndToEndTopK, plain path (src/SimdYolo/PtModel.cs:530-568)
 *   syo_decode_detections  YoloDetector.DecodeIndexed (src/SimdYolo/YoloDetector.cs:539-642) with
 *                          YoloDetector.Iou (:648-652)
 *
 * Every float operation is written in the reference's expression order and compiled without
 * contraction (-ffp-contract=off), so each result is the IEEE single-precision value of the
 * reference's scalar code.  exp is syo_expf (detmath.c); the reference calls MathF.Exp.
 */
#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "syo.h"

/* MathF.Max: NaN if either operand is NaN, +0 above -0 */
static float net_max(float a, float b)
{
    if (a != a) return a;
    if (b != b) return b;
    if (a > b) return a;
    if (b > a) return b;
    return signbit(a) ? b : a;
}

/* TensorOps.Sigmoid (src/SimdYolo/Compute.cs:513): 1 / (1 + exp(-x)) */
static float infer_sigmoid(float x) { return 1.0f / (1.0f + syo_expf(-x)); }

void syo_head_decode(const float *box, const float *cls, int batch, int h, int w, int bins, int nc, float stride,
                     int xyxy, float *out, int out_anchors, int out_start)
{
    const int spatial = h * w;
    for (int b = 0; b < batch; b++) {
        float *dst = out + (size_t)b * (nc + 4) * out_anchors + out_start;
        for (int c = 0; c < nc; c++)
            for (int a = 0; a < spatial; a++)
                dst[(size_t)(4 + c) * out_anchors + a] = infer_sigmoid(cls[((size_t)b * nc + c) * spatial + a]);
        for (int a = 0; a < spatial; a++) {
            float dist[4];
            for (int side = 0; side < 4; side++) {
                const float *src = box + ((size_t)b * 4 + side) * bins * spatial + a;
                if (bins == 1) {
                    dist[side] = src[0];
                    continue;
                }
                float max = -INFINITY, sum = 0.0f, numerator = 0.0f;
                for (int r = 0; r < bins; r++) max = net_max(max, src[(size_t)r * spatial]);
                for (int r = 0; r < bins; r++) {
                    float e = syo_expf(src[(size_t)r * spatial] - max);
                    sum += e;
                    numerator += e * (float)r;
                }
                dist[side] = numerator / sum;
            }
            const float col = (float)(a % w), row = (float)(a / w);
            const float x1 = (col + .5f - dist[0]) * stride, y1 = (row + .5f - dist[1]) * stride;
            const float x2 = (col + .5f + dist[2]) * stride, y2 = (row + .5f + dist[3]) * stride;
            dst[a] = xyxy ? x1 : (x1 + x2) * .5f;
            dst[(size_t)out_anchors + a] = xyxy ? y1 : (y1 + y2) * .5f;
            dst[(size_t)2 * out_anchors + a] = xyxy ? x2 : x2 - x1;
            dst[(size_t)3 * out_anchors + a] = xyxy ? y2 : y2 - y1;
        }
    }
}

/* float.CompareTo order: NaN below every number, -0 equal to +0 */
static int compare_float(float a, float b)
{
    if (a != a) return b != b ? 0 : -1;
    if (b != b) return 1;
    return a < b ? -1 : a > b ? 1 : 0;
}

typedef struct { float score; int anchor, cls; } e2e_item;

/* descending (score, -anchor, -class): the priority queues' order and the final ordering */
static int e2e_desc(const void *pa, const void *pb)
{
    const e2e_item *a = (const e2e_item *)pa, *b = (const e2e_item *)pb;
    int c = compare_float(a->score, b->score);
    if (c) return -c;
    if (a->anchor != b->anchor) return a->anchor < b->anchor ? -1 : 1;
    return a->cls < b->cls ? -1 : a->cls > b->cls;
}

int syo_end_to_end_topk(const float *x, int batch, int fields, int anchors, int nc, int maximum, float *out)
{
    if (batch < 1 || nc < 1 || fields < nc + 4 || anchors < 1 || maximum < 1) return -1;
    const int k = maximum < anchors ? maximum : anchors, extra = fields - nc - 4, width = 6 + extra;
    e2e_item *items = (e2e_item *)malloc(sizeof(e2e_item) * (size_t)(anchors > k * nc ? anchors : k * nc));
    int *chosen = (int *)malloc(sizeof(int) * (size_t)k);
    for (int b = 0; b < batch; b++) {
        const float *data = x + (size_t)b * fields * anchors;
        for (int a = 0; a < anchors; a++) {
            float m = -INFINITY;
            for (int c = 0; c < nc; c++) m = net_max(m, data[(size_t)(4 + c) * anchors + a]);
            items[a] = (e2e_item){m, a, 0};
        }
        qsort(items, (size_t)anchors, sizeof(e2e_item), e2e_desc);
        for (int i = 0; i < k; i++) chosen[i] = items[i].anchor;
        int n = 0;
        for (int i = 0; i < k; i++)
            for (int c = 0; c < nc; c++) items[n++] = (e2e_item){data[(size_t)(4 + c) * anchors + chosen[i]], chosen[i], c};
        qsort(items, (size_t)n, sizeof(e2e_item), e2e_desc);
        for (int i = 0; i < k; i++) {
            float *row = out + ((size_t)b * k + i) * width;
            for (int j = 0; j < 4; j++) row[j] = data[(size_t)j * anchors + items[i].anchor];
            row[4] = items[i].score;
            row[5] = (float)items[i].cls;
            for (int j = 0; j < extra; j++) row[6 + j] = data[(size_t)(4 + nc + j) * anchors + items[i].anchor];
        }
    }
    free(items);
    free(chosen);
    return k;
}

typedef struct { syo_detection d; int anchor; } det_candidate;

/* OrderByDescending(confidence), stable: equal confidences keep anchor order */
static int candidate_desc(const void *pa, const void *pb)
{
    const det_candidate *a = (const det_candidate *)pa, *b = (const det_candidate *)pb;
    if (a->d.confidence != b->d.confidence) return a->d.confidence > b->d.confidence ? -1 : 1;
    return a->anchor < b->anchor ? -1 : a->anchor > b->anchor;
}

static float min_f(float a, float b) { return b < a ? b : a; }
static float max_f(float a, float b) { return b > a ? b : a; }

float syo_detection_iou(const syo_detection *a, const syo_detection *b)
{
    float w = max_f(0.0f, min_f(a->x + a->width, b->x + b->width) - max_f(a->x, b->x));
    float h = max_f(0.0f, min_f(a->y + a->height, b->y + b->height) - max_f(a->y, b->y));
    float intersection = w * h;
    return intersection / max_f(FLT_TRUE_MIN, a->width * a->height + b->width * b->height - intersection);
}

/* Math.Clamp(value, min, max) */
static float clamp_f(float v, float lo, float hi) { return v < lo ? lo : v > hi ? hi : v; }

int syo_decode_detections(const float *output, int dim1, int dim2, int layout, int class_count,
                          const syo_letterbox *t, const syo_detect_options *o, syo_detection *out)
{
    if (layout < 1 || layout > 3 || dim1 < 1 || dim2 < 1 || o->max_detections < 1 || o->max_candidates < 1) return -1;
    const int channels_first = layout == 1, end2end = layout == 3;
    const int count = channels_first ? dim2 : dim1, fields = channels_first ? dim1 : dim2;
    if (fields < 5 || (end2end && fields != 6)) return -1;
    const int class_fields = class_count > 0 ? 4 + class_count : fields;
    if (!end2end && (class_fields < 5 || class_fields > fields)) return -1;
#define AT(a, c) output[channels_first ? (size_t)(c) * count + (a) : (size_t)(a) * fields + (c)]
    det_candidate *cand = (det_candidate *)malloc(sizeof(det_candidate) * (size_t)count);
    int n = 0;
    for (int a = 0; a < count; a++) {
        int cls = 0;
        float confidence;
        if (end2end) {
            confidence = AT(a, 4);
            float cv = AT(a, 5);
            if (!isfinite(cv) || cv < 0 || cv != truncf(cv)) continue;
            if (cv >= 2147483648.0f) { free(cand); return -2; }   /* checked((int)cv) throws */
            cls = (int)cv;
        } else {
            confidence = -INFINITY;
            for (int c = 4; c < class_fields; c++) {
                float score = AT(a, c);
                if (score > confidence) { confidence = score; cls = c - 4; }
            }
        }
        if (!isfinite(confidence) || confidence < o->confidence) continue;
        float x = AT(a, 0), y = AT(a, 1), w = AT(a, 2), h = AT(a, 3);
        if (!isfinite(x) || !isfinite(y) || !isfinite(w) || !isfinite(h)) continue;
        if (end2end) { w -= x; h -= y; } else { x -= w * .5f; y -= h * .5f; }
        if (w <= 0 || h <= 0) continue;
        cand[n].d = (syo_detection){cls, confidence, x, y, w, h};
        cand[n].anchor = a;
        n++;
    }
#undef AT
    qsort(cand, (size_t)n, sizeof(det_candidate), candidate_desc);
    if (n > o->max_candidates) n = o->max_candidates;
    syo_detection *kept = (syo_detection *)malloc(sizeof(syo_detection) * (size_t)(o->max_detections));
    int nk = 0;
    for (int i = 0; i < n && nk < o->max_detections; i++) {
        const syo_detection *d = &cand[i].d;
        int suppressed = 0;
        if (!end2end)
            for (int j = 0; j < nk && !suppressed; j++)
                if ((o->class_agnostic || kept[j].class_id == d->class_id) &&
                    syo_detection_iou(&kept[j], d) > o->iou_threshold)
                    suppressed = 1;
        if (!suppressed) kept[nk++] = *d;
    }
    int m = 0;
    const float sw = (float)t->source_width, sh = (float)t->source_height;
    const float px = (float)t->pad_x, py = (float)t->pad_y;
    for (int i = 0; i < nk; i++) {
        const syo_detection *d = &kept[i];
        float x1 = clamp_f((d->x - px) / t->scale_x, 0, sw), y1 = clamp_f((d->y - py) / t->scale_y, 0, sh);
        float x2 = clamp_f((d->x + d->width - px) / t->scale_x, 0, sw);
        float y2 = clamp_f((d->y + d->height - py) / t->scale_y, 0, sh);
        syo_detection r = {d->class_id, d->confidence, x1, y1, x2 - x1, y2 - y1};
        if (r.width > 0 && r.height > 0) out[m++] = r;
    }
    free(kept);
    free(cand);
    return m;
}
