/*
 * Oracle restatement of the detection-head operators.  TEST INFRASTRUCTURE ONLY.
 *
 *   syo_conv_forward / _backward        HeadOperations.Conv            HeadOperations.cs:29-82
 *   syo_grouped_conv_forward / _backward HeadOperations.GroupedConv    HeadOperations.cs:88-133
 *   syo_batchnorm_forward / _backward   HeadOperations.BatchNorm       HeadOperations.cs:153-193
 *   syo_silu_forward / _backward        HeadOperations.Silu            HeadOperations.cs:198-221
 *   syo_right_transposed                TrainingMatMul.RightTransposed TrainingMatMul.cs:14-49
 *   syo_sgd_update / syo_all_finite     TrainingParameter.Update / AllFinite  TrainingParameter.cs:21-55
 *   syo_progressive_weight              DetectionHead.ProgressiveWeight DetectionHead.cs:120
 *   syo_adamw_update                    torch.optim.AdamW (the reference has no AdamW)
 *
 * Batch is one image, layout NCHW, weights OIHW, stride 1, "same" padding k/2, as the
 * reference's shape guard requires (HeadOperations.cs:34).  The conv builds the same
 * im2col matrix (rows (c,ky,kx), columns pixels) and multiplies W[oc,K] x cols[K,HW].
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#else
static int omp_in_parallel(void) { return 1; }
#endif
#include "syo.h"

/* cols[(c*k+ky)*k+kx][y*w+x] = x[c][y+ky-p][x+kx-p] or 0 (HeadOperations.cs:39-45) */
static void im2col(const float *x, int ic, int h, int w, int k, float *cols)
{
    int pad = k / 2, spatial = h * w;
    memset(cols, 0, sizeof(float) * (size_t)ic * k * k * spatial);
    for (int c = 0; c < ic; c++)
        for (int ky = 0; ky < k; ky++)
            for (int kx = 0; kx < k; kx++) {
                float *row = cols + (size_t)((c * k + ky) * k + kx) * spatial;
                int left = pad - kx > 0 ? pad - kx : 0, right = w + pad - kx < w ? w + pad - kx : w;
                int y0 = pad - ky > 0 ? pad - ky : 0, y1 = h + pad - ky < h ? h + pad - ky : h;
                for (int y = y0; y < y1; y++)
                    memcpy(row + y * w + left, x + ((size_t)c * h + y + ky - pad) * w + left + kx - pad,
                           sizeof(float) * (size_t)(right - left));
            }
}

/* col2im scatter-add (HeadOperations.cs:73-79) */
static void col2im_add(const float *cols, int ic, int h, int w, int k, float *dx)
{
    int pad = k / 2, spatial = h * w;
    for (int c = 0; c < ic; c++)
        for (int ky = 0; ky < k; ky++)
            for (int kx = 0; kx < k; kx++) {
                const float *row = cols + (size_t)((c * k + ky) * k + kx) * spatial;
                int left = pad - kx > 0 ? pad - kx : 0, right = w + pad - kx < w ? w + pad - kx : w;
                int y0 = pad - ky > 0 ? pad - ky : 0, y1 = h + pad - ky < h ? h + pad - ky : h;
                for (int y = y0; y < y1; y++) {
                    float *dst = dx + ((size_t)c * h + y + ky - pad) * w + left + kx - pad;
                    const float *src = row + y * w + left;
                    for (int i = 0; i < right - left; i++) dst[i] += src[i];
                }
            }
}

/* C[m,n] = A[m,k] * B[k,n], row-major, overwrite (IComputeBackend.MatMul semantics, Compute.cs:11-25) */
static void matmul(const float *a, const float *b, float *c, int m, int n, int k)
{
    memset(c, 0, sizeof(float) * (size_t)m * n);
    /* rows are independent: split them over idle threads (each row keeps the serial k order) */
#pragma omp parallel for schedule(static) if (!omp_in_parallel() && (long)m * n * k > (1L << 20))
    for (int i = 0; i < m; i++) {
        float *crow = c + (size_t)i * n;
        for (int p = 0; p < k; p++) {
            float av = a[(size_t)i * k + p];
            const float *brow = b + (size_t)p * n;
            for (int j = 0; j < n; j++) crow[j] += av * brow[j];
        }
    }
}

/* TrainingMatMul.RightTransposed: C[m,n] = A[m,k] * B[n,k]^T (overwrite) */
void syo_right_transposed(const float *a, const float *b, float *c, int m, int n, int k)
{
#pragma omp parallel for schedule(static) if (!omp_in_parallel() && (long)m * n * k > (1L << 20))
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) {
            const float *ar = a + (size_t)i * k, *br = b + (size_t)j * k;
            float s0 = 0, s1 = 0, s2 = 0, s3 = 0, s4 = 0, s5 = 0, s6 = 0, s7 = 0;
            int p = 0;
            for (; p + 8 <= k; p += 8) {
                s0 += ar[p] * br[p]; s1 += ar[p + 1] * br[p + 1];
                s2 += ar[p + 2] * br[p + 2]; s3 += ar[p + 3] * br[p + 3];
                s4 += ar[p + 4] * br[p + 4]; s5 += ar[p + 5] * br[p + 5];
                s6 += ar[p + 6] * br[p + 6]; s7 += ar[p + 7] * br[p + 7];
            }
            float s = ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7));
            for (; p < k; p++) s += ar[p] * br[p];
            c[(size_t)i * n + j] = s;
        }
}

void syo_conv_forward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                      const float *bias, float *y)
{
    int spatial = h * w, kk = ic * k * k;
    float *cols = NULL;
    const float *b = x;
    if (k != 1) {
        cols = (float *)malloc(sizeof(float) * (size_t)kk * spatial);
        im2col(x, ic, h, w, k, cols);
        b = cols;
    }
    matmul(wt, b, y, oc, spatial, kk);
    if (bias)
        for (int c = 0; c < oc; c++)
            for (int p = 0; p < spatial; p++) y[(size_t)c * spatial + p] += bias[c];
    free(cols);
}

/* Backward closure of HeadOperations.Conv (HeadOperations.cs:49-80).  dx_acc == NULL mirrors a
 * frozen input (RequiresGradient == false, :67). */
void syo_conv_backward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                       const float *dy, float *dw_acc, float *db_acc, float *dx_acc)
{
    int spatial = h * w, kk = ic * k * k;
    float *cols = NULL;
    const float *b = x;
    if (k != 1) {
        cols = (float *)malloc(sizeof(float) * (size_t)kk * spatial);
        im2col(x, ic, h, w, k, cols);
        b = cols;
    }
    float *dw = (float *)malloc(sizeof(float) * (size_t)oc * kk);
    syo_right_transposed(dy, b, dw, oc, kk, spatial);
    for (size_t i = 0; i < (size_t)oc * kk; i++) dw_acc[i] += dw[i];
    free(dw);
    if (db_acc)
        for (int c = 0; c < oc; c++) {
            float s = 0;
            for (int p = 0; p < spatial; p++) s += dy[(size_t)c * spatial + p];
            db_acc[c] += s;
        }
    if (dx_acc) {
        float *wtt = (float *)malloc(sizeof(float) * (size_t)oc * kk);
        for (int r = 0; r < oc; r++)
            for (int c = 0; c < kk; c++) wtt[(size_t)c * oc + r] = wt[(size_t)r * kk + c];
        float *dcols = (float *)malloc(sizeof(float) * (size_t)kk * spatial);
        matmul(wtt, dy, dcols, kk, spatial, oc);
        if (k == 1)
            for (size_t i = 0; i < (size_t)kk * spatial; i++) dx_acc[i] += dcols[i];
        else
            col2im_add(dcols, ic, h, w, k, dx_acc);
        free(dcols);
        free(wtt);
    }
    free(cols);
}

void syo_grouped_conv_forward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                              int groups, const float *bias, float *y)
{
    int pad = k / 2, spatial = h * w, ig = ic / groups, og = oc / groups;
    for (int o = 0; o < oc; o++) {
        float *out = y + (size_t)o * spatial;
        for (int p = 0; p < spatial; p++) out[p] = bias ? bias[o] : 0.0f;
        int first = o / og * ig;
        for (int c = 0; c < ig; c++)
            for (int ky = 0; ky < k; ky++)
                for (int kx = 0; kx < k; kx++) {
                    float f = wt[((size_t)(o * ig + c) * k + ky) * k + kx];
                    int left = pad - kx > 0 ? pad - kx : 0, right = w + pad - kx < w ? w + pad - kx : w;
                    int y0 = pad - ky > 0 ? pad - ky : 0, y1 = h + pad - ky < h ? h + pad - ky : h;
                    for (int yy = y0; yy < y1; yy++) {
                        const float *src = x + (size_t)(first + c) * spatial + (yy + ky - pad) * w + left + kx - pad;
                        float *dst = out + yy * w + left;
                        for (int i = 0; i < right - left; i++) dst[i] += src[i] * f;
                    }
                }
    }
}

void syo_grouped_conv_backward(const float *x, int ic, int h, int w, const float *wt, int oc, int k,
                               int groups, const float *dy, float *dw_acc, float *db_acc, float *dx_acc)
{
    int pad = k / 2, spatial = h * w, ig = ic / groups, og = oc / groups;
    for (int o = 0; o < oc; o++) {
        const float *g = dy + (size_t)o * spatial;
        if (db_acc) {
            float s = 0;
            for (int p = 0; p < spatial; p++) s += g[p];
            db_acc[o] += s;
        }
        int first = o / og * ig;
        for (int c = 0; c < ig; c++)
            for (int ky = 0; ky < k; ky++)
                for (int kx = 0; kx < k; kx++) {
                    size_t wi = ((size_t)(o * ig + c) * k + ky) * k + kx;
                    float s = 0;
                    int left = pad - kx > 0 ? pad - kx : 0, right = w + pad - kx < w ? w + pad - kx : w;
                    int y0 = pad - ky > 0 ? pad - ky : 0, y1 = h + pad - ky < h ? h + pad - ky : h;
                    for (int yy = y0; yy < y1; yy++) {
                        size_t xi = (size_t)(first + c) * spatial + (yy + ky - pad) * w + left + kx - pad;
                        size_t yi = (size_t)o * spatial + yy * w + left;
                        for (int i = 0; i < right - left; i++) s += dy[yi + i] * x[xi + i];
                        if (dx_acc)
                            for (int i = 0; i < right - left; i++) dx_acc[xi + i] += dy[yi + i] * wt[wi];
                    }
                    dw_acc[wi] += s;
                }
    }
}

/* HeadOperations.BatchNorm forward (HeadOperations.cs:153-175).  xhat/inv keep what the
 * backward closure captures; batch_mean/batch_var (optional) report this image's statistics. */
void syo_batchnorm_forward(const float *x, int c, int spatial, const float *gamma, const float *beta,
                           float *rmean, float *rvar, float eps, float momentum, int training,
                           float *y, float *xhat, float *inv, float *batch_mean, float *batch_var)
{
    for (int ch = 0; ch < c; ch++) {
        const float *in = x + (size_t)ch * spatial;
        float mean = rmean[ch], variance = rvar[ch];
        if (training) {
            mean = 0;
            for (int q = 0; q < spatial; q++) mean += in[q];
            mean /= spatial;
            variance = 0;
            for (int q = 0; q < spatial; q++) {
                float d = in[q] - mean;
                variance += d * d;
            }
            variance /= spatial;
            rmean[ch] = (1 - momentum) * rmean[ch] + momentum * mean;
            rvar[ch] = (1 - momentum) * rvar[ch] +
                       momentum * variance * (spatial > 1 ? (float)spatial / (spatial - 1) : 1.0f);
            if (batch_mean) batch_mean[ch] = mean;
            if (batch_var) batch_var[ch] = variance;
        }
        inv[ch] = 1.0f / sqrtf(variance + eps);
        for (int p = 0; p < spatial; p++) {
            float v = (in[p] - mean) * inv[ch];
            xhat[(size_t)ch * spatial + p] = v;
            y[(size_t)ch * spatial + p] = v * gamma[ch] + beta[ch];
        }
    }
}

/* Backward closure of HeadOperations.BatchNorm (HeadOperations.cs:176-191) */
void syo_batchnorm_backward(const float *dy, const float *xhat, const float *inv, const float *gamma,
                            int c, int spatial, float *dgamma_acc, float *dbeta_acc, float *dx_acc)
{
    for (int ch = 0; ch < c; ch++) {
        size_t start = (size_t)ch * spatial;
        float sum = 0, weighted = 0;
        for (int q = 0; q < spatial; q++) {
            float d = dy[start + q];
            sum += d;
            weighted += d * xhat[start + q];
        }
        dgamma_acc[ch] += weighted;
        dbeta_acc[ch] += sum;
        float scale = gamma[ch] * inv[ch] / spatial;
        for (int p = 0; p < spatial; p++)
            dx_acc[start + p] += scale * (spatial * dy[start + p] - sum - xhat[start + p] * weighted);
    }
}

/* HeadOperations.Silu (HeadOperations.cs:198-221).  The reference's SIMD path uses its own fast
 * exp (CpuActivation.Exp); the value is the same function, evaluated with libm expf here. */
void syo_silu_forward(const float *x, int n, float *y, float *sig)
{
    for (int i = 0; i < n; i++) {
        float v = x[i];
        float e = expf(-fabsf(v));
        float s = v >= 0 ? 1.0f / (1.0f + e) : e / (1.0f + e);
        sig[i] = s;
        y[i] = v * s;
    }
}

void syo_silu_backward(const float *x, const float *sig, const float *dy, int n, float *dx_acc)
{
    for (int i = 0; i < n; i++) {
        float s = sig[i];
        dx_acc[i] += dy[i] * (s + x[i] * s * (1 - s));
    }
}

int syo_all_finite(const float *v, long n)
{
    for (long i = 0; i < n; i++)
        if (!isfinite(v[i])) return 0;
    return 1;
}

/* TrainingParameter.Update (TrainingParameter.cs:21-43) */
int syo_sgd_update(float *w, float *vel, float *grad, long n, float lr, float momentum, float wd,
                   int images, int has_grad)
{
    if (!has_grad) return 0;
    float inverse = 1.0f / images;
    int finite = 1;
    for (long i = 0; i < n; i++) {
        float v = vel[i] * momentum + grad[i] * inverse + w[i] * wd;
        float u = w[i] - lr * v;
        finite &= isfinite(v) && isfinite(u);
        vel[i] = v;
        w[i] = u;
    }
    if (!finite) return 1;
    memset(grad, 0, sizeof(float) * (size_t)n);
    return 0;
}

/* torch.optim.AdamW (decoupled decay, bias-corrected moments), gradient averaged over images.
 * step is the 1-based step count after this update.  Decay applies only where wd != 0. */
int syo_adamw_update(float *w, float *m, float *v, float *grad, long n, float lr, float beta1,
                     float beta2, float eps, float wd, int step, int images, int has_grad)
{
    if (!has_grad) return 0;
    float inverse = 1.0f / images;
    float bc1 = 1.0f - powf(beta1, (float)step), bc2 = 1.0f - powf(beta2, (float)step);
    float step_size = lr / bc1, bc2_sqrt = sqrtf(bc2);
    int finite = 1;
    for (long i = 0; i < n; i++) {
        float g = grad[i] * inverse;
        float p = w[i] * (1.0f - lr * wd);
        float mi = beta1 * m[i] + (1.0f - beta1) * g;
        float vi = beta2 * v[i] + (1.0f - beta2) * g * g;
        float denom = sqrtf(vi) / bc2_sqrt + eps;
        p = p - step_size * (mi / denom);
        finite &= isfinite(p) && isfinite(mi) && isfinite(vi);
        m[i] = mi;
        v[i] = vi;
        w[i] = p;
    }
    if (!finite) return 1;
    memset(grad, 0, sizeof(float) * (size_t)n);
    return 0;
}

/* DetectionHead.ProgressiveWeight (DetectionHead.cs:120); the product and the sum round separately
 * as in the reference, so no fused multiply-add */
__attribute__((optimize("fp-contract=off"))) float syo_progressive_weight(int epoch, int epochs)
{
    int denom = epochs - 1 > 1 ? epochs - 1 : 1;
    float t = 1 - (float)epoch / denom;
    return (t > 0 ? t : 0) * .7f + .1f;
}
