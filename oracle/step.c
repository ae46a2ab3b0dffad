/*
 * Oracle restatement of the detection-head fine-tuning step.  TEST INFRASTRUCTURE ONLY.
 *
 *   syo_head_image   DetectionHead.Loss/Forward + Branch.Forward + GradientTape.Backward
 *                    (DetectionHead.cs:89-115,146-157; TrainingParameter.cs:70-78)
 *   syo_train_step   YoloTrainer.Train inner batch loop (YoloTrainer.cs:185-199):
 *                    per image letterbox -> frozen features -> head loss -> backward,
 *                    then AllFinite over all gradients and TrainingParameter.Update(images=B).
 *   syo_backbone_*   frozen YOLOv8-family trunk with BatchNorm folded into the convs
 *                    (PtModel.cs:128-144 fold, PtModel.cs:267-398 layer semantics: Conv, C2f,
 *                    Bottleneck, SPPF, Upsample nearest, Concat), stopped before Detect
 *                    (PtModel.cs:202-203).
 *
 * Parameters are one flat float array in DetectionHead.Snapshot order (DetectionHead.cs:124-130):
 * branches cv2.0, cv2.1, cv2.2, cv3.0, cv3.1, cv3.2 (then, for end-to-end heads, one2one_cv2.0-2 and
 * one2one_cv3.0-2); per block weight, [bias], [bn gamma, beta].
 * Buffers: per BN block running_mean, running_var, num_batches_tracked (one float).
 * Images run in parallel over OpenMP threads; BN running statistics and gradient sums are then
 * applied in image order, so the result equals the reference's sequential loop.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#include "syo.h"

/* ------------------------------------------------------------------ head layout */

/* Branch order (DetectionHead.cs:20-26): cv2.0-2, cv3.0-2, and with end_to_end one2one_cv2.0-2,
 * one2one_cv3.0-2 built from the same block lists. */
static int n_branches(const syo_head_desc *d) { return d->end_to_end ? 12 : 6; }

static const syo_block *branch_blocks(const syo_head_desc *d, int branch, int *count)
{
    int level = branch % 3;
    if ((branch / 3) % 2 == 0) { *count = d->n_box_blocks; return d->box_blocks[level]; }
    *count = d->n_cls_blocks;
    return d->cls_blocks[level];
}

/* gradient group of a branch: 0 class branches (always connected), 1 cv2, 2 one2one_cv2 (a box
 * branch receives a gradient only when its loss assigned a positive, DetectionLoss.cs:101) */
static int branch_group(int branch) { return branch < 3 ? 1 : (branch >= 6 && branch < 9) ? 2 : 0; }

static long block_weight_count(const syo_block *b) { return (long)b->oc * (b->ic / b->groups) * b->k * b->k; }

long syo_head_param_count(const syo_head_desc *d)
{
    long total = 0;
    for (int br = 0; br < n_branches(d); br++) {
        int n;
        const syo_block *blocks = branch_blocks(d, br, &n);
        for (int i = 0; i < n; i++) {
            total += block_weight_count(&blocks[i]);
            if (blocks[i].has_bias) total += blocks[i].oc;
            if (blocks[i].has_bn) total += 2L * blocks[i].oc;
        }
    }
    return total;
}

long syo_head_buffer_count(const syo_head_desc *d)
{
    long total = 0;
    for (int br = 0; br < n_branches(d); br++) {
        int n;
        const syo_block *blocks = branch_blocks(d, br, &n);
        for (int i = 0; i < n; i++)
            if (blocks[i].has_bn) total += 2L * blocks[i].oc + 1;
    }
    return total;
}

typedef struct {
    const syo_block *b;
    long w_off, b_off, g_off, be_off;   /* parameter offsets (-1 when absent) */
    long rm_off, rv_off, nt_off;        /* buffer offsets */
} block_slot;

static int slots_for_branch(const syo_head_desc *d, int branch, block_slot *out)
{
    long p = 0, q = 0;
    int n = 0;
    for (int br = 0; br < n_branches(d); br++) {
        int cnt;
        const syo_block *blocks = branch_blocks(d, br, &cnt);
        for (int i = 0; i < cnt; i++) {
            block_slot s;
            s.b = &blocks[i];
            s.w_off = p; p += block_weight_count(&blocks[i]);
            s.b_off = -1; s.g_off = s.be_off = s.rm_off = s.rv_off = s.nt_off = -1;
            if (blocks[i].has_bias) { s.b_off = p; p += blocks[i].oc; }
            if (blocks[i].has_bn) {
                s.g_off = p; p += blocks[i].oc;
                s.be_off = p; p += blocks[i].oc;
                s.rm_off = q; q += blocks[i].oc;
                s.rv_off = q; q += blocks[i].oc;
                s.nt_off = q; q += 1;
            }
            if (br == branch) out[n++] = s;
        }
    }
    return n;
}

/* saved state of one block during the forward (what the reference tape closures capture) */
typedef struct {
    float *x;        /* conv input (borrowed for block 0) */
    float *conv;     /* conv output (BN input) or branch output */
    float *xhat, *inv, *bn_out, *sig, *act;
    float *mean, *var;
} block_state;

static void conv_any(const syo_block *b, const float *x, int h, int w, const float *wt, const float *bias, float *y)
{
    if (b->groups == 1) syo_conv_forward(x, b->ic, h, w, wt, b->oc, b->k, bias, y);
    else syo_grouped_conv_forward(x, b->ic, h, w, wt, b->oc, b->k, b->groups, bias, y);
}

static void conv_any_backward(const syo_block *b, const float *x, int h, int w, const float *wt,
                              const float *dy, float *dw, float *db, float *dx)
{
    if (b->groups == 1) syo_conv_backward(x, b->ic, h, w, wt, b->oc, b->k, dy, dw, db, dx);
    else syo_grouped_conv_backward(x, b->ic, h, w, wt, b->oc, b->k, b->groups, dy, dw, db, dx);
}

/* Branch.Forward (DetectionHead.cs:146-157) with running statistics written to bn_stats slots:
 * stats[rm_off..] = this image's mean, stats[rv_off..] = biased variance. */
static float *branch_forward(const syo_head_desc *d, const block_slot *slots, int n, const float *params,
                             float *buffers, float *stats, const float *input, int h, int w, block_state *st,
                             int training)
{
    int spatial = h * w;
    const float *x = input;
    for (int i = 0; i < n; i++) {
        const syo_block *b = slots[i].b;
        block_state *s = &st[i];
        memset(s, 0, sizeof *s);
        s->x = (float *)x;
        s->conv = (float *)malloc(sizeof(float) * (size_t)b->oc * spatial);
        conv_any(b, x, h, w, params + slots[i].w_off, slots[i].b_off >= 0 ? params + slots[i].b_off : NULL, s->conv);
        if (!b->has_bn) { x = s->conv; continue; }
        size_t n_el = (size_t)b->oc * spatial;
        s->xhat = (float *)malloc(sizeof(float) * n_el);
        s->bn_out = (float *)malloc(sizeof(float) * n_el);
        s->sig = (float *)malloc(sizeof(float) * n_el);
        s->act = (float *)malloc(sizeof(float) * n_el);
        s->inv = (float *)malloc(sizeof(float) * b->oc);
        /* running statistics live in a per-image scratch copy; the caller folds them in order */
        float *rm = (float *)malloc(sizeof(float) * b->oc), *rv = (float *)malloc(sizeof(float) * b->oc);
        memcpy(rm, buffers + slots[i].rm_off, sizeof(float) * b->oc);
        memcpy(rv, buffers + slots[i].rv_off, sizeof(float) * b->oc);
        syo_batchnorm_forward(s->conv, b->oc, spatial, params + slots[i].g_off, params + slots[i].be_off, rm, rv,
                              d->bn_eps, d->bn_momentum, training, s->bn_out, s->xhat, s->inv,
                              stats + slots[i].rm_off, stats + slots[i].rv_off);
        free(rm);
        free(rv);
        syo_silu_forward(s->bn_out, (int)n_el, s->act, s->sig);
        x = s->act;
    }
    return (float *)x;
}

/* reverse replay of the branch closures; dout is d(loss)/d(branch output) */
static void branch_backward(const block_slot *slots, int n, const float *params, float *grad,
                            block_state *st, const float *dout, int h, int w)
{
    int spatial = h * w;
    float *g = (float *)dout;  /* gradient w.r.t. the current block output */
    float *owned = NULL;
    for (int i = n - 1; i >= 0; i--) {
        const syo_block *b = slots[i].b;
        block_state *s = &st[i];
        size_t n_el = (size_t)b->oc * spatial;
        float *dconv = g;
        float *tmp1 = NULL, *tmp2 = NULL;
        if (b->has_bn) {
            tmp1 = (float *)calloc(n_el, sizeof(float));
            syo_silu_backward(s->bn_out, s->sig, g, (int)n_el, tmp1);
            tmp2 = (float *)calloc(n_el, sizeof(float));
            syo_batchnorm_backward(tmp1, s->xhat, s->inv, params + slots[i].g_off, b->oc, spatial,
                                   grad + slots[i].g_off, grad + slots[i].be_off, tmp2);
            dconv = tmp2;
        }
        float *dx = NULL;
        if (i > 0) dx = (float *)calloc((size_t)b->ic * spatial, sizeof(float));
        conv_any_backward(b, s->x, h, w, params + slots[i].w_off, dconv, grad + slots[i].w_off,
                          slots[i].b_off >= 0 ? grad + slots[i].b_off : NULL, dx);
        free(tmp1);
        free(tmp2);
        free(owned);
        owned = dx;
        g = dx;
    }
    free(owned);
}

static void free_states(block_state *st, int n)
{
    for (int i = 0; i < n; i++) {
        free(st[i].conv); free(st[i].xhat); free(st[i].inv); free(st[i].bn_out); free(st[i].sig); free(st[i].act);
    }
}

/* Head loss of one image without touching running statistics; stats receives this image's
 * per-channel (mean, biased variance) at the buffer offsets of each BN block.
 * DetectionHead.Loss (DetectionHead.cs:105-115): the one-to-many branches with the top-10 assigner;
 * with end_to_end also the one-to-one branches (top-k 1, or 7 for the progressive loss, and a second
 * top-1 after conflicts), each loss's gradients scaled by its weight (ProgressiveWeight for the
 * progressive loss, else 1) and the reported parts summed with the same weights.
 * box_connected: bit 0 cv2, bit 1 one2one_cv2. */
static int head_image_core(const syo_head_desc *d, const float *params, float *buffers, float *stats,
                           const float *const *features, const syo_box *truth, int n_truth, float *grad,
                           syo_loss *loss, int backward, int *box_connected, int training)
{
    block_slot slots[12][8];
    int counts[12];
    block_state states[12][8];
    float *outs[12];
    const int nbr = n_branches(d), sets = nbr / 6;
    for (int br = 0; br < nbr; br++) counts[br] = slots_for_branch(d, br, slots[br]);
    for (int set = 0; set < sets; set++)
        for (int l = 0; l < 3; l++)
            for (int kind = 0; kind < 2; kind++) {
                int br = set * 6 + kind * 3 + l;
                outs[br] = branch_forward(d, slots[br], counts[br], params, buffers, stats, features[l], d->hs[l],
                                          d->ws[l], states[br], training);
            }
    const int progressive = d->end_to_end && d->bins == 1;
    const float many_w = progressive ? syo_progressive_weight(d->epoch, d->schedule_epochs) : 1.0f;
    const float one_w = progressive ? 1 - many_w : 1.0f;
    syo_loss parts[2];
    memset(parts, 0, sizeof parts);
    int rc = 0, connected = 0;
    for (int set = 0; set < sets && rc == 0; set++) {
        const int o = set * 6;
        const float *boxes[3] = {outs[o], outs[o + 1], outs[o + 2]};
        const float *classes[3] = {outs[o + 3], outs[o + 4], outs[o + 5]};
        float *dbox[3], *dcls[3];
        for (int l = 0; l < 3; l++) {
            size_t spatial = (size_t)d->hs[l] * d->ws[l];
            dbox[l] = (float *)calloc(4 * d->bins * spatial, sizeof(float));
            dcls[l] = (float *)calloc(d->nc * spatial, sizeof(float));
        }
        const int topk = set == 0 ? 10 : progressive ? 7 : 1, topk2 = set == 0 ? 10 : 1;
        const float weight = set == 0 ? many_w : one_w;
        rc = syo_detection_loss(boxes, classes, d->hs, d->ws, d->strides, 3, d->nc, d->bins, truth, n_truth, topk,
                                topk2, weight, backward, dbox, dcls, &parts[set], NULL, NULL);
        connected |= (parts[set].connected ? 1 : 0) << set;
        if (rc == 0 && backward) {
            for (int l = 2; l >= 0; l--) {
                branch_backward(slots[o + 3 + l], counts[o + 3 + l], params, grad, states[o + 3 + l], dcls[l],
                                d->hs[l], d->ws[l]);
                if (parts[set].connected)
                    branch_backward(slots[o + l], counts[o + l], params, grad, states[o + l], dbox[l], d->hs[l],
                                    d->ws[l]);
            }
        }
        for (int l = 0; l < 3; l++) { free(dbox[l]); free(dcls[l]); }
    }
    if (d->end_to_end) {
        loss->box = parts[0].box * many_w + parts[1].box * one_w;
        loss->cls = parts[0].cls * many_w + parts[1].cls * one_w;
        loss->dfl = parts[0].dfl * many_w + parts[1].dfl * one_w;
        loss->positives = parts[0].positives + parts[1].positives;
    } else {
        *loss = parts[0];
    }
    loss->connected = connected;
    if (box_connected) *box_connected = connected;
    for (int br = 0; br < nbr; br++) free_states(states[br], counts[br]);
    return rc;
}

/* fold one image's BN statistics into the running buffers (HeadOperations.cs:164-165, DetectionHead.cs:154) */
static void fold_running_stats(const syo_head_desc *d, float *buffers, const float *stats)
{
    for (int br = 0; br < n_branches(d); br++) {
        block_slot slots[8];
        int n = slots_for_branch(d, br, slots);
        for (int i = 0; i < n; i++) {
            if (!slots[i].b->has_bn) continue;
            int spatial = d->hs[br % 3] * d->ws[br % 3], oc = slots[i].b->oc;
            float m = d->bn_momentum;
            for (int c = 0; c < oc; c++) {
                float mean = stats[slots[i].rm_off + c], var = stats[slots[i].rv_off + c];
                buffers[slots[i].rm_off + c] = (1 - m) * buffers[slots[i].rm_off + c] + m * mean;
                buffers[slots[i].rv_off + c] = (1 - m) * buffers[slots[i].rv_off + c] +
                                               m * var * (spatial > 1 ? (float)spatial / (spatial - 1) : 1.0f);
            }
            buffers[slots[i].nt_off] += 1.0f;
        }
    }
}

int syo_head_image(const syo_head_desc *d, const float *params, float *buffers, const float *const *features,
                   const syo_box *truth, int n_truth, float *grad, syo_loss *loss, int backward, int *box_connected)
{
    long nb = syo_head_buffer_count(d);
    float *stats = (float *)calloc(nb ? nb : 1, sizeof(float));
    int rc = head_image_core(d, params, buffers, stats, features, truth, n_truth, grad, loss, backward, box_connected,
                             1);
    if (rc == 0) fold_running_stats(d, buffers, stats);
    free(stats);
    return rc;
}

/* YoloTrainer.EvaluateLoss (YoloTrainer.cs:237-246): the head with BatchNorm in evaluation mode
 * (running mean / variance, HeadOperations.cs:158-166 with training = false), the loss without
 * gradients; nothing is updated. */
int syo_head_eval_image(const syo_head_desc *d, const float *params, float *buffers, const float *const *features,
                        const syo_box *truth, int n_truth, syo_loss *loss)
{
    long nb = syo_head_buffer_count(d);
    float *stats = (float *)calloc(nb ? nb : 1, sizeof(float));
    int rc = head_image_core(d, params, buffers, stats, features, truth, n_truth, NULL, loss, 0, NULL, 0);
    free(stats);
    return rc;
}

/* The branch outputs of DetectionHead.Forward in evaluation mode (Branch.Forward, DetectionHead.cs:146-157,
 * BatchNorm with the running statistics), the input of the inference decode (PtModel.Detect). */
int syo_head_eval_outputs(const syo_head_desc *d, const float *params, const float *buffers,
                          const float *const *features, int set, float *const *box, float *const *cls)
{
    if (set < 0 || set >= n_branches(d) / 6) return -1;
    long nb = syo_head_buffer_count(d);
    float *stats = (float *)calloc(nb ? nb : 1, sizeof(float));
    float *scratch = (float *)malloc(sizeof(float) * (nb ? nb : 1));
    memcpy(scratch, buffers, sizeof(float) * (size_t)nb);
    for (int kind = 0; kind < 2; kind++)
        for (int l = 0; l < 3; l++) {
            const int br = set * 6 + kind * 3 + l;
            block_slot slots[8];
            block_state states[8];
            const int n = slots_for_branch(d, br, slots);
            const float *y = branch_forward(d, slots, n, params, scratch, stats, features[l], d->hs[l], d->ws[l],
                                            states, 0);
            const int oc = slots[n - 1].b->oc;
            memcpy(kind ? cls[l] : box[l], y, sizeof(float) * (size_t)oc * d->hs[l] * d->ws[l]);
            free_states(states, n);
        }
    free(scratch);
    free(stats);
    return 0;
}

/* ------------------------------------------------------------------ frozen backbone */

static int make_div8(float x)
{
    int v = (int)ceilf(x / 8.0f) * 8;
    return v;
}

static int bb_channels(const syo_backbone_desc *d, int c)
{
    float x = (float)(c < d->max_channels ? c : d->max_channels) * d->width_mult;
    return make_div8(x);
}

static int bb_depth(const syo_backbone_desc *d, int n)
{
    int v = (int)lroundf(n * d->depth_mult);
    return v > 1 ? v : 1;
}

typedef struct { const float *p; long off; int count_only; } bb_params;

static const float *take(bb_params *bp, long n)
{
    const float *r = bp->count_only ? NULL : bp->p + bp->off;
    bp->off += n;
    return r;
}

/* NCHW conv with folded BN bias and SiLU, or no activation (PtModel.cs Conv/DWConv; act=False convs
 * of the YOLO11 attention block have an Identity act) */
static void bb_conv_act(bb_params *bp, const float *x, int ic, int h, int w, int oc, int k, int s, int act, float *y);

static void bb_conv(bb_params *bp, const float *x, int ic, int h, int w, int oc, int k, int s, float *y)
{
    bb_conv_act(bp, x, ic, h, w, oc, k, s, 1, y);
}

static void bb_conv_act(bb_params *bp, const float *x, int ic, int h, int w, int oc, int k, int s, int act, float *y)
{
    const float *wt = take(bp, (long)oc * ic * k * k);
    const float *bias = take(bp, oc);
    if (bp->count_only) return;
    int pad = k / 2, ho = (h + 2 * pad - k) / s + 1, wo = (w + 2 * pad - k) / s + 1, so = ho * wo;
    int kk = ic * k * k;
    float *cols = (float *)malloc(sizeof(float) * (size_t)kk * so);
    for (int c = 0; c < ic; c++)
        for (int ky = 0; ky < k; ky++)
            for (int kx = 0; kx < k; kx++) {
                float *row = cols + (size_t)((c * k + ky) * k + kx) * so;
                for (int oy = 0; oy < ho; oy++) {
                    int iy = oy * s + ky - pad;
                    for (int ox = 0; ox < wo; ox++) {
                        int ix = ox * s + kx - pad;
                        row[oy * wo + ox] = (iy >= 0 && iy < h && ix >= 0 && ix < w) ? x[((size_t)c * h + iy) * w + ix] : 0.0f;
                    }
                }
            }
#pragma omp parallel for schedule(static) if (!omp_in_parallel() && (long)oc * kk * so > (1L << 20))
    for (int o = 0; o < oc; o++) {
        float *yr = y + (size_t)o * so;
        for (int p = 0; p < so; p++) yr[p] = 0;
        for (int q = 0; q < kk; q++) {
            float f = wt[(size_t)o * kk + q];
            const float *cr = cols + (size_t)q * so;
            for (int p = 0; p < so; p++) yr[p] += f * cr[p];
        }
        for (int p = 0; p < so; p++) {
            float v = yr[p] + bias[o];
            yr[p] = act ? v / (1.0f + expf(-v)) : v;
        }
    }
    free(cols);
}

/* C2f (PtModel.cs C2f case): cv1 -> split in two -> n bottlenecks on the last chunk -> concat -> cv2 */
static void bb_c2f(bb_params *bp, const float *x, int c1, int h, int w, int c2, int n, int shortcut, float *y)
{
    int c = c2 / 2, sp = h * w;
    float *cat = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)(2 + n) * c * sp);
    bb_conv(bp, x, c1, h, w, 2 * c, 1, 1, cat);
    float *tmp = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)c * sp);
    for (int i = 0; i < n; i++) {
        const float *in = bp->count_only ? NULL : cat + (size_t)(1 + i) * c * sp;
        float *out = bp->count_only ? NULL : cat + (size_t)(2 + i) * c * sp;
        bb_conv(bp, in, c, h, w, c, 3, 1, tmp);
        bb_conv(bp, tmp, c, h, w, c, 3, 1, out);
        if (shortcut && !bp->count_only)
            for (size_t q = 0; q < (size_t)c * sp; q++) out[q] += in[q];
    }
    bb_conv(bp, cat, (2 + n) * c, h, w, c2, 1, 1, y);
    free(tmp);
    free(cat);
}

/* MaxPool2d(5, stride 1, padding 2): padded taps never win (PyTorch pads with -inf) */
static void maxpool5(const float *x, int c, int h, int w, float *y)
{
    for (int ch = 0; ch < c; ch++)
        for (int yy = 0; yy < h; yy++)
            for (int xx = 0; xx < w; xx++) {
                float m = -INFINITY;
                for (int dy = -2; dy <= 2; dy++)
                    for (int dx = -2; dx <= 2; dx++) {
                        int iy = yy + dy, ix = xx + dx;
                        if (iy < 0 || iy >= h || ix < 0 || ix >= w) continue;
                        float v = x[((size_t)ch * h + iy) * w + ix];
                        if (v > m) m = v;
                    }
                y[((size_t)ch * h + yy) * w + xx] = m;
            }
}

static void bb_sppf(bb_params *bp, const float *x, int c1, int h, int w, int c2, float *y)
{
    int c = c1 / 2, sp = h * w;
    float *cat = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)4 * c * sp);
    bb_conv(bp, x, c1, h, w, c, 1, 1, cat);
    if (!bp->count_only)
        for (int i = 0; i < 3; i++) maxpool5(cat + (size_t)i * c * sp, c, h, w, cat + (size_t)(i + 1) * c * sp);
    bb_conv(bp, cat, 4 * c, h, w, c2, 1, 1, y);
    free(cat);
}

static void upsample2(const float *x, int c, int h, int w, float *y)
{
    for (int ch = 0; ch < c; ch++)
        for (int yy = 0; yy < 2 * h; yy++)
            for (int xx = 0; xx < 2 * w; xx++)
                y[((size_t)ch * 2 * h + yy) * 2 * w + xx] = x[((size_t)ch * h + yy / 2) * w + xx / 2];
}

static void run_backbone(const syo_backbone_desc *d, bb_params *bp, const uint8_t *rgb, float *p3out, float *p4out,
                         float *p5out)
{
    int S = d->image, co = bp->count_only;
    int c64 = bb_channels(d, 64), c128 = bb_channels(d, 128), c256 = bb_channels(d, 256);
    int c512 = bb_channels(d, 512), c1024 = bb_channels(d, 1024);
    int n3 = bb_depth(d, 3), n6 = bb_depth(d, 6);
    int s2 = S / 2, s4 = S / 4, s8 = S / 8, s16 = S / 16, s32 = S / 32;
#define ALLOC(n) (co ? NULL : (float *)malloc(sizeof(float) * (size_t)(n)))
    float *img = ALLOC(3 * S * S);
    if (!co)
        for (int c = 0; c < 3; c++)
            for (int p = 0; p < S * S; p++) img[(size_t)c * S * S + p] = (float)rgb[(size_t)p * 3 + c] / 255.0f;
    float *l0 = ALLOC(c64 * s2 * s2);
    bb_conv(bp, img, 3, S, S, c64, 3, 2, l0);
    free(img);
    float *l1 = ALLOC(c128 * s4 * s4);
    bb_conv(bp, l0, c64, s2, s2, c128, 3, 2, l1);
    free(l0);
    float *l2 = ALLOC(c128 * s4 * s4);
    bb_c2f(bp, l1, c128, s4, s4, c128, n3, 1, l2);
    free(l1);
    float *l3 = ALLOC(c256 * s8 * s8);
    bb_conv(bp, l2, c128, s4, s4, c256, 3, 2, l3);
    free(l2);
    float *l4 = ALLOC(c256 * s8 * s8);
    bb_c2f(bp, l3, c256, s8, s8, c256, n6, 1, l4);
    free(l3);
    float *l5 = ALLOC(c512 * s16 * s16);
    bb_conv(bp, l4, c256, s8, s8, c512, 3, 2, l5);
    float *l6 = ALLOC(c512 * s16 * s16);
    bb_c2f(bp, l5, c512, s16, s16, c512, n6, 1, l6);
    free(l5);
    float *l7 = ALLOC(c1024 * s32 * s32);
    bb_conv(bp, l6, c512, s16, s16, c1024, 3, 2, l7);
    float *l8 = ALLOC(c1024 * s32 * s32);
    bb_c2f(bp, l7, c1024, s32, s32, c1024, n3, 1, l8);
    free(l7);
    float *l9 = ALLOC(c1024 * s32 * s32);
    bb_sppf(bp, l8, c1024, s32, s32, c1024, l9);
    free(l8);
    /* neck */
    float *cat11 = ALLOC((c1024 + c512) * s16 * s16);
    if (!co) {
        upsample2(l9, c1024, s32, s32, cat11);
        memcpy(cat11 + (size_t)c1024 * s16 * s16, l6, sizeof(float) * (size_t)c512 * s16 * s16);
    }
    free(l6);
    float *l12 = ALLOC(c512 * s16 * s16);
    bb_c2f(bp, cat11, c1024 + c512, s16, s16, c512, n3, 0, l12);
    free(cat11);
    float *cat14 = ALLOC((c512 + c256) * s8 * s8);
    if (!co) {
        upsample2(l12, c512, s16, s16, cat14);
        memcpy(cat14 + (size_t)c512 * s8 * s8, l4, sizeof(float) * (size_t)c256 * s8 * s8);
    }
    free(l4);
    float *l15 = co ? NULL : p3out;
    bb_c2f(bp, cat14, c512 + c256, s8, s8, c256, n3, 0, l15);
    free(cat14);
    float *cat17 = ALLOC((c256 + c512) * s16 * s16);
    bb_conv(bp, l15, c256, s8, s8, c256, 3, 2, cat17);
    if (!co) memcpy(cat17 + (size_t)c256 * s16 * s16, l12, sizeof(float) * (size_t)c512 * s16 * s16);
    free(l12);
    float *l18 = co ? NULL : p4out;
    bb_c2f(bp, cat17, c256 + c512, s16, s16, c512, n3, 0, l18);
    free(cat17);
    float *cat20 = ALLOC((c512 + c1024) * s32 * s32);
    bb_conv(bp, l18, c512, s16, s16, c512, 3, 2, cat20);
    if (!co) memcpy(cat20 + (size_t)c512 * s32 * s32, l9, sizeof(float) * (size_t)c1024 * s32 * s32);
    free(l9);
    float *l21 = co ? NULL : p5out;
    bb_c2f(bp, cat20, c512 + c1024, s32, s32, c1024, n3, 0, l21);
    free(cat20);
#undef ALLOC
}

/* ---- YOLO11 trunk (PtModel.cs cases C3k2, C3k, Bottleneck, C2PSA, PSABlock, Attention; layer list
 * and channel / depth rules of the public YOLO11 definition).  Parameters in call order below. */

/* depthwise conv (groups = channels) with folded BN bias, no activation (the attention's pe conv) */
static void bb_dwconv(bb_params *bp, const float *x, int c, int h, int w, int k, float *y)
{
    const float *wt = take(bp, (long)c * k * k);
    const float *bias = take(bp, c);
    if (bp->count_only) return;
    syo_grouped_conv_forward(x, c, h, w, wt, c, k, c, bias, y);
}

/* Bottleneck: cv2(cv1(x)) (+ x when shortcut and c1 == c2); cv1 c1 -> c2*e, both 3x3 */
static void bb_bottleneck(bb_params *bp, const float *x, int c1, int c2, float e, int shortcut, int h, int w, float *y)
{
    int c_ = (int)(c2 * e), sp = h * w;
    float *t = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)c_ * sp);
    bb_conv(bp, x, c1, h, w, c_, 3, 1, t);
    bb_conv(bp, t, c_, h, w, c2, 3, 1, y);
    if (shortcut && c1 == c2 && !bp->count_only)
        for (size_t q = 0; q < (size_t)c2 * sp; q++) y[q] += x[q];
    free(t);
}

/* C3k: cv3(cat(m(cv1(x)), cv2(x))), m = n Bottlenecks (c_, c_, e = 1), c_ = c2 / 2; order cv1, m, cv2, cv3 */
static void bb_c3k(bb_params *bp, const float *x, int c1, int c2, int n, int shortcut, int h, int w, float *y)
{
    int c_ = (int)(c2 * 0.5f), sp = h * w;
    float *cat = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)2 * c_ * sp);
    float *t = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)c_ * sp);
    bb_conv(bp, x, c1, h, w, c_, 1, 1, cat);
    for (int i = 0; i < n; i++) {
        bb_bottleneck(bp, cat, c_, c_, 1.0f, shortcut, h, w, t);
        if (!bp->count_only) memcpy(cat, t, sizeof(float) * (size_t)c_ * sp);
    }
    bb_conv(bp, x, c1, h, w, c_, 1, 1, bp->count_only ? NULL : cat + (size_t)c_ * sp);
    bb_conv(bp, cat, 2 * c_, h, w, c2, 1, 1, y);
    free(t);
    free(cat);
}

/* C3k2: C2f layout (cv1 -> two chunks, n modules on the last chunk, concat, cv2) whose modules are
 * C3k(c, c, 2) or Bottleneck(c, c, e = 0.5), c = c2 * e */
static void bb_c3k2(bb_params *bp, const float *x, int c1, int c2, int n, int c3k, float e, int h, int w, float *y)
{
    int c = (int)(c2 * e), sp = h * w;
    float *cat = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)(2 + n) * c * sp);
    bb_conv(bp, x, c1, h, w, 2 * c, 1, 1, cat);
    for (int i = 0; i < n; i++) {
        const float *in = bp->count_only ? NULL : cat + (size_t)(1 + i) * c * sp;
        float *out = bp->count_only ? NULL : cat + (size_t)(2 + i) * c * sp;
        if (c3k) bb_c3k(bp, in, c, c, 2, 1, h, w, out);
        else bb_bottleneck(bp, in, c, c, 0.5f, 1, h, w, out);
    }
    bb_conv(bp, cat, (2 + n) * c, h, w, c2, 1, 1, y);
    free(cat);
}

/* Attention (PtModel.cs:429-439): qkv 1x1 (no act) -> per head [q kd | k kd | v hd] channels;
 * softmax over keys of q^T k * kd^-0.5; out = v attn^T + pe(v) (depthwise 3x3, no act); proj 1x1 (no
 * act).  Order: qkv, pe, proj. */
static void bb_attention(bb_params *bp, const float *x, int dim, int heads, int h, int w, float *y)
{
    int hd = dim / heads, kd = (int)(hd * 0.5f), n = h * w, hch = dim + 2 * kd * heads;
    float *qkv = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)hch * n);
    bb_conv_act(bp, x, dim, h, w, hch, 1, 1, 0, qkv);
    float *v = NULL, *att = NULL, *pe = NULL;
    if (!bp->count_only) {
        v = (float *)malloc(sizeof(float) * (size_t)dim * n);
        att = (float *)malloc(sizeof(float) * (size_t)dim * n);
        pe = (float *)malloc(sizeof(float) * (size_t)dim * n);
        float scale = 1.0f / sqrtf((float)kd);
        float *row = (float *)malloc(sizeof(float) * (size_t)n);
        for (int hh = 0; hh < heads; hh++) {
            const float *q = qkv + (size_t)hh * (2 * kd + hd) * n, *k = q + (size_t)kd * n, *vv = k + (size_t)kd * n;
            memcpy(v + (size_t)hh * hd * n, vv, sizeof(float) * (size_t)hd * n);
            for (int i = 0; i < n; i++) {
                float m = -INFINITY;
                for (int j = 0; j < n; j++) {
                    float sdot = 0.0f;
                    for (int d2 = 0; d2 < kd; d2++) sdot += q[(size_t)d2 * n + i] * k[(size_t)d2 * n + j];
                    row[j] = sdot * scale;
                    if (row[j] > m) m = row[j];
                }
                float sum = 0.0f;
                for (int j = 0; j < n; j++) {
                    row[j] = expf(row[j] - m);
                    sum += row[j];
                }
                for (int j = 0; j < n; j++) row[j] /= sum;
                for (int d2 = 0; d2 < hd; d2++) {
                    float a = 0.0f;
                    for (int j = 0; j < n; j++) a += vv[(size_t)d2 * n + j] * row[j];
                    att[((size_t)hh * hd + d2) * n + i] = a;
                }
            }
        }
        free(row);
    }
    bb_dwconv(bp, v, dim, h, w, 3, pe);
    if (!bp->count_only)
        for (size_t q = 0; q < (size_t)dim * n; q++) att[q] += pe[q];
    bb_conv_act(bp, att, dim, h, w, dim, 1, 1, 0, y);
    free(qkv);
    free(v);
    free(att);
    free(pe);
}

/* PSABlock: x + attn(x), then + ffn (Conv(c, 2c, 1) SiLU, Conv(2c, c, 1) no act) */
static void bb_psablock(bb_params *bp, const float *x, int c, int heads, int h, int w, float *y)
{
    int sp = h * w;
    float *t = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)2 * c * sp);
    bb_attention(bp, x, c, heads, h, w, y);
    if (!bp->count_only)
        for (size_t q = 0; q < (size_t)c * sp; q++) y[q] += x[q];
    bb_conv(bp, y, c, h, w, 2 * c, 1, 1, t);
    float *f = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)c * sp);
    bb_conv_act(bp, t, 2 * c, h, w, c, 1, 1, 0, f);
    if (!bp->count_only)
        for (size_t q = 0; q < (size_t)c * sp; q++) y[q] += f[q];
    free(t);
    free(f);
}

/* C2PSA: cv1 -> chunks (a, b), b through n PSABlocks (heads = c / 64), cv2(cat(a, b)) */
static void bb_c2psa(bb_params *bp, const float *x, int c1, int n, int h, int w, float *y)
{
    int c = (int)(c1 * 0.5f), sp = h * w;
    float *cat = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)2 * c * sp);
    float *t = bp->count_only ? NULL : (float *)malloc(sizeof(float) * (size_t)c * sp);
    bb_conv(bp, x, c1, h, w, 2 * c, 1, 1, cat);
    for (int i = 0; i < n; i++) {
        bb_psablock(bp, bp->count_only ? NULL : cat + (size_t)c * sp, c, c / 64 > 0 ? c / 64 : 1, h, w, t);
        if (!bp->count_only) memcpy(cat + (size_t)c * sp, t, sizeof(float) * (size_t)c * sp);
    }
    bb_conv(bp, cat, 2 * c, h, w, c1, 1, 1, y);
    free(t);
    free(cat);
}

static void run_backbone_11(const syo_backbone_desc *d, bb_params *bp, const uint8_t *rgb, float *p3out, float *p4out,
                            float *p5out)
{
    int S = d->image, co = bp->count_only;
    int c64 = bb_channels(d, 64), c128 = bb_channels(d, 128), c256 = bb_channels(d, 256);
    int c512 = bb_channels(d, 512), c1024 = bb_channels(d, 1024);
    int n2 = bb_depth(d, 2);
    int s2 = S / 2, s4 = S / 4, s8 = S / 8, s16 = S / 16, s32 = S / 32;
#define ALLOC(n) (co ? NULL : (float *)malloc(sizeof(float) * (size_t)(n)))
    float *img = ALLOC(3 * S * S);
    if (!co)
        for (int c = 0; c < 3; c++)
            for (int p = 0; p < S * S; p++) img[(size_t)c * S * S + p] = (float)rgb[(size_t)p * 3 + c] / 255.0f;
    float *l0 = ALLOC(c64 * s2 * s2);
    bb_conv(bp, img, 3, S, S, c64, 3, 2, l0);
    free(img);
    float *l1 = ALLOC(c128 * s4 * s4);
    bb_conv(bp, l0, c64, s2, s2, c128, 3, 2, l1);
    free(l0);
    float *l2 = ALLOC(c256 * s4 * s4);
    bb_c3k2(bp, l1, c128, c256, n2, 0, 0.25f, s4, s4, l2);
    free(l1);
    float *l3 = ALLOC(c256 * s8 * s8);
    bb_conv(bp, l2, c256, s4, s4, c256, 3, 2, l3);
    free(l2);
    float *l4 = ALLOC(c512 * s8 * s8);
    bb_c3k2(bp, l3, c256, c512, n2, 0, 0.25f, s8, s8, l4);
    free(l3);
    float *l5 = ALLOC(c512 * s16 * s16);
    bb_conv(bp, l4, c512, s8, s8, c512, 3, 2, l5);
    float *l6 = ALLOC(c512 * s16 * s16);
    bb_c3k2(bp, l5, c512, c512, n2, 1, 0.5f, s16, s16, l6);
    free(l5);
    float *l7 = ALLOC(c1024 * s32 * s32);
    bb_conv(bp, l6, c512, s16, s16, c1024, 3, 2, l7);
    float *l8 = ALLOC(c1024 * s32 * s32);
    bb_c3k2(bp, l7, c1024, c1024, n2, 1, 0.5f, s32, s32, l8);
    free(l7);
    float *l9 = ALLOC(c1024 * s32 * s32);
    bb_sppf(bp, l8, c1024, s32, s32, c1024, l9);
    free(l8);
    float *l10 = ALLOC(c1024 * s32 * s32);
    bb_c2psa(bp, l9, c1024, n2, s32, s32, l10);
    free(l9);
    /* neck */
    float *cat12 = ALLOC((c1024 + c512) * s16 * s16);
    if (!co) {
        upsample2(l10, c1024, s32, s32, cat12);
        memcpy(cat12 + (size_t)c1024 * s16 * s16, l6, sizeof(float) * (size_t)c512 * s16 * s16);
    }
    free(l6);
    float *l13 = ALLOC(c512 * s16 * s16);
    bb_c3k2(bp, cat12, c1024 + c512, c512, n2, 0, 0.5f, s16, s16, l13);
    free(cat12);
    float *cat15 = ALLOC((c512 + c512) * s8 * s8);
    if (!co) {
        upsample2(l13, c512, s16, s16, cat15);
        memcpy(cat15 + (size_t)c512 * s8 * s8, l4, sizeof(float) * (size_t)c512 * s8 * s8);
    }
    free(l4);
    float *l16 = co ? NULL : p3out;
    bb_c3k2(bp, cat15, c512 + c512, c256, n2, 0, 0.5f, s8, s8, l16);
    free(cat15);
    float *cat18 = ALLOC((c256 + c512) * s16 * s16);
    bb_conv(bp, l16, c256, s8, s8, c256, 3, 2, cat18);
    if (!co) memcpy(cat18 + (size_t)c256 * s16 * s16, l13, sizeof(float) * (size_t)c512 * s16 * s16);
    free(l13);
    float *l19 = co ? NULL : p4out;
    bb_c3k2(bp, cat18, c256 + c512, c512, n2, 0, 0.5f, s16, s16, l19);
    free(cat18);
    float *cat21 = ALLOC((c512 + c1024) * s32 * s32);
    bb_conv(bp, l19, c512, s16, s16, c512, 3, 2, cat21);
    if (!co) memcpy(cat21 + (size_t)c512 * s32 * s32, l10, sizeof(float) * (size_t)c1024 * s32 * s32);
    free(l10);
    float *l22 = co ? NULL : p5out;
    bb_c3k2(bp, cat21, c512 + c1024, c1024, n2, 1, 0.5f, s32, s32, l22);
    free(cat21);
#undef ALLOC
}

static void run_any_backbone(const syo_backbone_desc *d, bb_params *bp, const uint8_t *rgb, float *p3, float *p4,
                             float *p5)
{
    if (d->family == 1) run_backbone_11(d, bp, rgb, p3, p4, p5);
    else run_backbone(d, bp, rgb, p3, p4, p5);
}

long syo_backbone_param_count(const syo_backbone_desc *d)
{
    bb_params bp = {NULL, 0, 1};
    run_any_backbone(d, &bp, NULL, NULL, NULL, NULL);
    return bp.off;
}

void syo_backbone_feature_channels(const syo_backbone_desc *d, int32_t ch[3])
{
    ch[0] = bb_channels(d, 256);
    ch[1] = bb_channels(d, 512);
    ch[2] = bb_channels(d, 1024);
}

void syo_backbone_forward(const syo_backbone_desc *d, const float *params, const uint8_t *rgb, float *p3, float *p4,
                          float *p5)
{
    bb_params bp = {params, 0, 0};
    run_any_backbone(d, &bp, rgb, p3, p4, p5);
}

/* ------------------------------------------------------------------ full step */

/* segment flags per head parameter: box branch or not, decay (conv weights only, DetectionHead.cs:59-60) */
static void param_segments(const syo_head_desc *d, long *offs, long *lens, int *group, int *decay, int *count)
{
    int n = 0;
    long p = 0;
    for (int br = 0; br < n_branches(d); br++) {
        int cnt;
        const syo_block *blocks = branch_blocks(d, br, &cnt);
        for (int i = 0; i < cnt; i++) {
            long wl = block_weight_count(&blocks[i]);
            offs[n] = p; lens[n] = wl; group[n] = branch_group(br); decay[n] = 1; n++; p += wl;
            if (blocks[i].has_bias) { offs[n] = p; lens[n] = blocks[i].oc; group[n] = branch_group(br); decay[n] = 0; n++; p += blocks[i].oc; }
            if (blocks[i].has_bn) {
                offs[n] = p; lens[n] = blocks[i].oc; group[n] = branch_group(br); decay[n] = 0; n++; p += blocks[i].oc;
                offs[n] = p; lens[n] = blocks[i].oc; group[n] = branch_group(br); decay[n] = 0; n++; p += blocks[i].oc;
            }
        }
    }
    *count = n;
}

void syo_train_step(const syo_backbone_desc *bd, const float *backbone_params, const syo_head_desc *hd, float *params,
                    float *buffers, float *velocity, float *velocity2, const syo_optim *opt,
                    const uint8_t *const *images, const syo_box *truth, const int32_t *counts, int batch, int threads,
                    float *grad_out, syo_step_result *result)
{
    long np = syo_head_param_count(hd), nb = syo_head_buffer_count(hd);
    float *grads = (float *)calloc((size_t)np * batch, sizeof(float));
    float *stats = (float *)calloc((size_t)(nb ? nb : 1) * batch, sizeof(float));
    syo_loss *losses = (syo_loss *)calloc(batch, sizeof(syo_loss));
    int *connected = (int *)calloc(batch, sizeof(int)), *rcs = (int *)calloc(batch, sizeof(int));
    long *box_off = (long *)malloc(sizeof(long) * (batch + 1));
    box_off[0] = 0;
    for (int b = 0; b < batch; b++) box_off[b + 1] = box_off[b] + counts[b];
    int ch[3] = {0, 0, 0};
    syo_backbone_feature_channels(bd, ch);
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
    /* one image per thread; a single image instead spreads its GEMM rows over the threads */
    int team = threads < batch ? threads : batch;
    omp_set_num_threads(threads);
#pragma omp parallel for schedule(dynamic, 1) num_threads(team)
#endif
    for (int b = 0; b < batch; b++) {
        float *feat[3];
        for (int l = 0; l < 3; l++) feat[l] = (float *)malloc(sizeof(float) * (size_t)ch[l] * hd->hs[l] * hd->ws[l]);
        syo_backbone_forward(bd, backbone_params, images[b], feat[0], feat[1], feat[2]);
        const float *cf[3] = {feat[0], feat[1], feat[2]};
        rcs[b] = head_image_core(hd, params, buffers, stats + (size_t)b * nb, cf, truth + box_off[b], counts[b],
                                 grads + (size_t)b * np, &losses[b], 1, &connected[b], 1);
        for (int l = 0; l < 3; l++) free(feat[l]);
    }
    syo_step_result r;
    memset(&r, 0, sizeof r);
    float *grad = (float *)calloc(np, sizeof(float));
    int any_connected = 0, finite = 1;
    for (int b = 0; b < batch; b++) {
        if (rcs[b] != 0) { r.status = 1; break; }
        float total = losses[b].box + losses[b].cls + losses[b].dfl;
        if (!isfinite(total)) finite = 0;   /* YoloTrainer.cs:193 */
        r.box += losses[b].box; r.cls += losses[b].cls; r.dfl += losses[b].dfl; r.positives += losses[b].positives;
        any_connected |= connected[b];
        fold_running_stats(hd, buffers, stats + (size_t)b * nb);
        const float *g = grads + (size_t)b * np;
        for (long i = 0; i < np; i++) grad[i] += g[i];
    }
    r.box_has_grad = any_connected;
    if (r.status == 0 && (!finite || !syo_all_finite(grad, np))) r.status = 3;  /* YoloTrainer.cs:196 */
    if (grad_out) memcpy(grad_out, grad, sizeof(float) * np);
    if (r.status == 0) {
        long offs[1024], lens[1024];
        int group[1024], decay[1024], nseg = 0;
        param_segments(hd, offs, lens, group, decay, &nseg);
        for (int s = 0; s < nseg; s++) {
            int has = group[s] ? (any_connected >> (group[s] - 1)) & 1 : 1;
            int bad;
            if (opt->optimizer == 0)
                bad = syo_sgd_update(params + offs[s], velocity + offs[s], grad + offs[s], lens[s], opt->lr, opt->momentum,
                                     decay[s] ? opt->weight_decay : 0.0f, batch, has);
            else
                bad = syo_adamw_update(params + offs[s], velocity + offs[s], velocity2 + offs[s], grad + offs[s], lens[s],
                                       opt->lr, opt->beta1, opt->beta2, opt->adam_eps, decay[s] ? opt->weight_decay : 0.0f,
                                       opt->adam_step[group[s]] + 1, batch, has);
            if (bad) { r.status = 3; break; }
        }
    }
    *result = r;
    free(grad); free(grads); free(stats); free(losses); free(connected); free(rcs); free(box_off);
}
