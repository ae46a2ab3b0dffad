/*
 * Oracle restatement of DetectionLoss.Compute (src/SimdYolo.Training/DetectionLoss.cs:19-149)
 * and BoxMath.Ciou / Differential (DetectionLoss.cs:154-183).  TEST INFRASTRUCTURE ONLY.
 *
 * Arithmetic follows the reference expression by expression in float (compiled with
 * -ffp-contract=off so nothing is fused).  exp / atan / pow come from detmath.c (see there).
 * Anchor order is level-major, pixel row-major (DetectionLoss.cs:27-33).  Top-k keeps the k
 * largest (metric, -anchor) pairs over ALL anchors, exactly like the bounded PriorityQueue
 * (DetectionLoss.cs:65), then intersects with the inside mask (:67).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include "syo.h"

/* ---- forward-mode differential with 4 partials (Differential, DetectionLoss.cs:154-164) ---- */
typedef struct { float v, g[4]; } dif;

static dif dconst(float v) { dif r = {v, {0, 0, 0, 0}}; return r; }
static dif dvar(float v, int i) { dif r = {v, {0, 0, 0, 0}}; r.g[i] = 1; return r; }
static dif dadd(dif a, dif b) { dif r; r.v = a.v + b.v; for (int i = 0; i < 4; i++) r.g[i] = a.g[i] + b.g[i]; return r; }
static dif dsub(dif a, dif b) { dif r; r.v = a.v - b.v; for (int i = 0; i < 4; i++) r.g[i] = a.g[i] - b.g[i]; return r; }
static dif dmul(dif a, dif b)
{
    dif r; r.v = a.v * b.v;
    for (int i = 0; i < 4; i++) r.g[i] = a.g[i] * b.v + b.g[i] * a.v;
    return r;
}
static dif ddiv(dif a, dif b)
{
    dif r; r.v = a.v / b.v;
    float d = b.v * b.v;
    for (int i = 0; i < 4; i++) r.g[i] = (a.g[i] * b.v - b.g[i] * a.v) / d;
    return r;
}
static dif dmin(dif a, dif b)
{
    if (a.v < b.v) return a;
    if (a.v > b.v) return b;
    dif r; r.v = a.v; for (int i = 0; i < 4; i++) r.g[i] = (a.g[i] + b.g[i]) * .5f; return r;
}
static dif dmax(dif a, dif b)
{
    if (a.v > b.v) return a;
    if (a.v < b.v) return b;
    dif r; r.v = a.v; for (int i = 0; i < 4; i++) r.g[i] = (a.g[i] + b.g[i]) * .5f; return r;
}
static dif datan(dif a)
{
    dif r; r.v = syo_atanf(a.v);
    float d = 1 + a.v * a.v;
    for (int i = 0; i < 4; i++) r.g[i] = a.g[i] / d;
    return r;
}

/* BoxMath.Ciou (DetectionLoss.cs:171-183): predicted p = x1,y1,x2,y2 (differentiated), target t. */
float syo_ciou(const float p[4], const float t[4], float grad[4])
{
    const float eps = 1e-7f;
    dif x1 = dvar(p[0], 0), y1 = dvar(p[1], 1), x2 = dvar(p[2], 2), y2 = dvar(p[3], 3);
    dif w1 = dsub(x2, x1), h1 = dadd(dsub(y2, y1), dconst(eps));
    float w2 = t[2] - t[0], h2 = t[3] - t[1] + eps;
    dif iw = dmax(dsub(dmin(x2, dconst(t[2])), dmax(x1, dconst(t[0]))), dconst(0));
    dif ih = dmax(dsub(dmin(y2, dconst(t[3])), dmax(y1, dconst(t[1]))), dconst(0));
    dif inter = dmul(iw, ih);
    dif uni = dadd(dsub(dadd(dmul(w1, h1), dconst(w2 * h2)), inter), dconst(eps));
    dif iou = ddiv(inter, uni);
    dif cw = dsub(dmax(x2, dconst(t[2])), dmin(x1, dconst(t[0])));
    dif ch = dsub(dmax(y2, dconst(t[3])), dmin(y1, dconst(t[1])));
    dif dx = dsub(dsub(dconst(t[0] + t[2]), x1), x2);
    dif dy = dsub(dsub(dconst(t[1] + t[3]), y1), y2);
    dif rho = ddiv(dadd(dmul(dx, dx), dmul(dy, dy)), dconst(4.0f));
    const float pi = 3.14159265358979323846f;
    dif v = dsub(datan(dconst(w2 / h2)), datan(ddiv(w1, h1)));
    v = dmul(dmul(v, v), dconst(4.0f / (pi * pi)));
    float alpha = v.v / (v.v - iou.v + 1 + eps);
    dif c2 = dadd(dadd(dmul(cw, cw), dmul(ch, ch)), dconst(eps));
    dif result = dsub(dsub(iou, ddiv(rho, c2)), dmul(v, dconst(alpha)));
    if (grad) for (int i = 0; i < 4; i++) grad[i] = result.g[i];
    return result.v;
}

/* heap-free exact top-k: key order (metric desc, anchor asc); k is small (<= 16) */
static int topk_select(const float *metric, int anchors, int k, int *out)
{
    int count = 0;
    for (int a = 0; a < anchors; a++) {
        float m = metric[a];
        if (count == k) {
            /* worst kept element is out[count-1] (smallest metric, largest index among ties) */
            int worst = out[count - 1];
            if (!(m > metric[worst])) continue;   /* equal metric: later (larger) index loses */
            count--;
        }
        int pos = count;
        while (pos > 0) {
            int prev = out[pos - 1];
            if (metric[prev] > m || (metric[prev] == m && prev < a)) break;
            out[pos] = prev;
            pos--;
        }
        out[pos] = a;
        count++;
    }
    return count;
}

int syo_detection_loss(const float *const *box_levels, const float *const *cls_levels,
                       const int *hs, const int *ws, const float *strides, int levels, int nc, int bins,
                       const syo_box *truth, int n_truth, int topk, int topk2, float grad_scale,
                       int backward, float *const *dbox_levels, float *const *dcls_levels,
                       syo_loss *out, int32_t *assigned_out, float *scores_out)
{
    if (!(bins == 1 || bins == 16) || topk < 1 || topk2 < 1 || topk2 > topk || topk > 64 || !isfinite(grad_scale))
        return -1;
    int anchors = 0;
    for (int l = 0; l < levels; l++) anchors += hs[l] * ws[l];
    int *lev = (int *)malloc(sizeof(int) * anchors), *pix = (int *)malloc(sizeof(int) * anchors);
    float *cx = (float *)malloc(sizeof(float) * anchors), *cy = (float *)malloc(sizeof(float) * anchors);
    float *st = (float *)malloc(sizeof(float) * anchors), *dec = (float *)malloc(sizeof(float) * anchors * 4);
    float *prob = (float *)malloc(sizeof(float) * (size_t)anchors * 4 * bins);
    float *expect = (float *)malloc(sizeof(float) * anchors * 4);
    int a = 0;
    for (int l = 0; l < levels; l++) {
        int h = hs[l], w = ws[l], spatial = h * w;
        const float *t = box_levels[l];
        for (int p = 0; p < spatial; p++, a++) {
            lev[a] = l; pix[a] = p;
            cx[a] = (p % w + .5f) * strides[l];
            cy[a] = (p / w + .5f) * strides[l];
            st[a] = strides[l];
            for (int d = 0; d < 4; d++) {
                if (bins == 1) { expect[a * 4 + d] = t[(size_t)d * spatial + p]; continue; }
                float maximum = -INFINITY;
                for (int b = 0; b < bins; b++) maximum = fmaxf(maximum, t[(size_t)(d * bins + b) * spatial + p]);
                float sum = 0;
                size_t start = ((size_t)a * 4 + d) * bins;
                for (int b = 0; b < bins; b++) {
                    float v = syo_expf(t[(size_t)(d * bins + b) * spatial + p] - maximum);
                    prob[start + b] = v;
                    sum += v;
                }
                float distance = 0;
                for (int b = 0; b < bins; b++) {
                    float pr = prob[start + b] / sum;
                    prob[start + b] = pr;
                    distance += pr * b;
                }
                expect[a * 4 + d] = distance;
            }
            dec[a * 4 + 0] = cx[a] - expect[a * 4 + 0] * strides[l];
            dec[a * 4 + 1] = cy[a] - expect[a * 4 + 1] * strides[l];
            dec[a * 4 + 2] = cx[a] + expect[a * 4 + 2] * strides[l];
            dec[a * 4 + 3] = cy[a] + expect[a * 4 + 3] * strides[l];
        }
    }
    size_t ga = (size_t)n_truth * anchors;
    unsigned char *selected = (unsigned char *)calloc(ga ? ga : 1, 1), *inside_m = (unsigned char *)calloc(ga ? ga : 1, 1);
    float *overlap = (float *)calloc(ga ? ga : 1, sizeof(float)), *align = (float *)calloc(ga ? ga : 1, sizeof(float));
    int *top = (int *)malloc(sizeof(int) * 64);
    int status = 0;
    for (int g = 0; g < n_truth; g++) {
        syo_box box = truth[g];
        if (box.cls < 0 || box.cls >= nc) { status = -1; break; }
        float tb[4] = {box.x1, box.y1, box.x2, box.y2};
        float *metric = align + (size_t)g * anchors;
        for (a = 0; a < anchors; a++) {
            size_t index = (size_t)g * anchors + a;
            float bx = (box.x1 + box.x2) * .5f, by = (box.y1 + box.y2) * .5f;
            float cwid = box.x2 - box.x1 < strides[0] ? (levels > 1 ? strides[1] : strides[0] * 2) : box.x2 - box.x1;
            float chei = box.y2 - box.y1 < strides[0] ? (levels > 1 ? strides[1] : strides[0] * 2) : box.y2 - box.y1;
            int inside = cx[a] - (bx - cwid * .5f) > 1e-9f && bx + cwid * .5f - cx[a] > 1e-9f &&
                         cy[a] - (by - chei * .5f) > 1e-9f && by + chei * .5f - cy[a] > 1e-9f;
            inside_m[index] = (unsigned char)inside;
            float iou = inside ? fmaxf(0, syo_ciou(dec + a * 4, tb, NULL)) : 0;
            overlap[index] = iou;
            float m = 0;
            if (inside) {
                int l = lev[a], spatial = hs[l] * ws[l];
                float s = syo_sigmoid(cls_levels[l][(size_t)box.cls * spatial + pix[a]]);
                m = sqrtf(s) * syo_pow6(iou);
            }
            metric[a] = m;
        }
        int kept = topk_select(metric, anchors, topk, top);
        for (int i = 0; i < kept; i++) {
            size_t index = (size_t)g * anchors + top[i];
            selected[index] = inside_m[index];
        }
    }
    syo_loss result = {0, 0, 0, 0, 0};
    if (status == 0) {
        int32_t *assigned = (int32_t *)malloc(sizeof(int32_t) * anchors);
        for (a = 0; a < anchors; a++) {
            int count = 0, chosen = -1;
            for (int g = 0; g < n_truth; g++)
                if (selected[(size_t)g * anchors + a]) { chosen = g; count++; }
            if (count > 1) {
                float best = -1;
                for (int g = 0; g < n_truth; g++)
                    if (overlap[(size_t)g * anchors + a] > best) { best = overlap[(size_t)g * anchors + a]; chosen = g; }
                for (int g = 0; g < n_truth; g++) selected[(size_t)g * anchors + a] = g == chosen;
            }
            assigned[a] = chosen;
        }
        if (topk2 != topk) {
            /* second top-k over kept matches, stable by anchor index (DetectionLoss.cs:83-91) */
            float *keyed = (float *)malloc(sizeof(float) * anchors);
            for (int g = 0; g < n_truth; g++) {
                for (a = 0; a < anchors; a++) {
                    size_t index = (size_t)g * anchors + a;
                    keyed[a] = selected[index] ? align[index] : 0;
                }
                int kept = topk_select(keyed, anchors, topk2, top);
                unsigned char *keep = (unsigned char *)calloc(anchors, 1);
                for (int i = 0; i < kept; i++) keep[top[i]] = 1;
                for (a = 0; a < anchors; a++) if (!keep[a]) selected[(size_t)g * anchors + a] = 0;
                free(keep);
            }
            free(keyed);
            for (a = 0; a < anchors; a++) {
                assigned[a] = -1;
                for (int g = 0; g < n_truth; g++) if (selected[(size_t)g * anchors + a]) { assigned[a] = g; break; }
            }
        }
        float *max_align = (float *)calloc(n_truth ? n_truth : 1, sizeof(float));
        float *max_ov = (float *)calloc(n_truth ? n_truth : 1, sizeof(float));
        for (int g = 0; g < n_truth; g++)
            for (a = 0; a < anchors; a++)
                if (selected[(size_t)g * anchors + a]) {
                    max_align[g] = fmaxf(max_align[g], align[(size_t)g * anchors + a]);
                    max_ov[g] = fmaxf(max_ov[g], overlap[(size_t)g * anchors + a]);
                }
        float *scores = (float *)calloc(anchors, sizeof(float));
        float score_sum = 0;
        int any = 0;
        for (a = 0; a < anchors; a++) {
            int g = assigned[a];
            if (g >= 0) {
                scores[a] = align[(size_t)g * anchors + a] * max_ov[g] / (max_align[g] + 1e-9f);
                score_sum += scores[a];
                any = 1;
            }
        }
        score_sum = fmaxf(1, score_sum);
        result.connected = backward && any;
        float box_loss = 0, class_loss = 0, dfl_loss = 0;
        int positives = 0;
        for (a = 0; a < anchors; a++) {
            int l = lev[a], p = pix[a], spatial = hs[l] * ws[l], g = assigned[a];
            float weight = scores[a];
            const float *logits = cls_levels[l];
            for (int c = 0; c < nc; c++) {
                size_t index = (size_t)c * spatial + p;
                float logit = logits[index];
                float target = g >= 0 && truth[g].cls == c ? weight : 0;
                class_loss += (fmaxf(logit, 0) - logit * target + logf(1 + expf(-fabsf(logit)))) * (.5f / score_sum);
                if (backward) dcls_levels[l][index] += (syo_sigmoid(logit) - target) * (.5f / score_sum) * grad_scale;
            }
            if (g < 0) continue;
            positives++;
            syo_box tb = truth[g];
            float inv = 1 / st[a];
            float pg[4] = {dec[a * 4] * inv, dec[a * 4 + 1] * inv, dec[a * 4 + 2] * inv, dec[a * 4 + 3] * inv};
            float tg[4] = {tb.x1 * inv, tb.y1 * inv, tb.x2 * inv, tb.y2 * inv};
            float cg[4];
            float ciou = syo_ciou(pg, tg, cg);
            float box_scale = 7.5f * weight / score_sum;
            box_loss += (1 - ciou) * box_scale;
            float coord[4];
            for (int i = 0; i < 4; i++) coord[i] = -cg[i] * (box_scale * grad_scale);
            float dist_grad[4] = {-coord[0], -coord[1], coord[2], coord[3]};
            float dists[4] = {(cx[a] - tb.x1) / st[a], (cy[a] - tb.y1) / st[a], (tb.x2 - cx[a]) / st[a], (tb.y2 - cy[a]) / st[a]};
            const float *bt = box_levels[l];
            for (int d = 0; d < 4; d++) {
                if (bins == 1) {
                    float extent = (d % 2 == 0 ? ws[0] : hs[0]) * strides[0];
                    float norm = st[a] / extent, delta = expect[a * 4 + d] - dists[d];
                    float l1 = 1.5f * weight / (4 * score_sum);
                    dfl_loss += fabsf(delta) * norm * l1;
                    if (backward) {
                        float sign = delta > 0 ? 1.0f : delta < 0 ? -1.0f : 0.0f;
                        dbox_levels[l][(size_t)d * spatial + p] += dist_grad[d] + sign * norm * l1 * grad_scale;
                    }
                    continue;
                }
                float target = dists[d];
                float hi = bins - 1 - .01f;
                target = target < 0 ? 0 : target > hi ? hi : target;
                int left = (int)target;
                float rw = target - left;
                size_t start = ((size_t)a * 4 + d) * bins;
                float scale = 1.5f * weight / (4 * score_sum);
                float max_logit = -INFINITY, exp_sum = 0;
                for (int b = 0; b < bins; b++) max_logit = fmaxf(max_logit, bt[(size_t)(d * bins + b) * spatial + p]);
                for (int b = 0; b < bins; b++) exp_sum += expf(bt[(size_t)(d * bins + b) * spatial + p] - max_logit);
                float log_sum = max_logit + logf(exp_sum);
                dfl_loss += scale * (log_sum - (1 - rw) * bt[(size_t)(d * bins + left) * spatial + p] -
                                     rw * bt[(size_t)(d * bins + left + 1) * spatial + p]);
                if (backward)
                    for (int b = 0; b < bins; b++) {
                        float pr = prob[start + b], tp = b == left ? 1 - rw : b == left + 1 ? rw : 0;
                        dbox_levels[l][(size_t)(d * bins + b) * spatial + p] +=
                            pr * (b - expect[a * 4 + d]) * dist_grad[d] + scale * (pr - tp) * grad_scale;
                    }
            }
        }
        result.box = box_loss; result.cls = class_loss; result.dfl = dfl_loss; result.positives = positives;
        if (assigned_out) memcpy(assigned_out, assigned, sizeof(int32_t) * anchors);
        if (scores_out) memcpy(scores_out, scores, sizeof(float) * anchors);
        free(scores); free(max_align); free(max_ov); free(assigned);
    }
    if (out) *out = result;
    free(top); free(selected); free(inside_m); free(overlap); free(align);
    free(lev); free(pix); free(cx); free(cy); free(st); free(dec); free(prob); free(expect);
    return status;
}
