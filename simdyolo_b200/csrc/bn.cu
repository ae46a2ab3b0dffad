// Training-mode BatchNorm with per-image statistics, fused with SiLU, forward and backward
// (HeadOperations.BatchNorm HeadOperations.cs:153-193, HeadOperations.Silu :198-221), running
// statistics (HeadOperations.cs:164-165, num_batches_tracked DetectionHead.cs:154) and the bias
// gradient of the final conv (HeadOperations.cs:66).
//
// Each image normalises with its own mean / variance over H x W, exactly like the reference's
// batch-of-one convs, so a batch of B images needs B x C statistics.  The reductions happen in the
// epilogue of the conv that produces the data (forward: the conv output y; backward: the data
// gradient g of the next conv), which writes partials per 32-row group; the fold kernels here
// combine every (image, channel)'s groups in a fixed order (Chan's pairwise variance update for the
// statistics), so results do not depend on timing.  The apply passes stream float4s with
// per-(image, channel) coefficients prepared by the folds.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

__device__ __forceinline__ void split_range(int pixels, int splits, int s, int& p0, int& p1) {
    p0 = (int)((long)pixels * s / splits);
    p1 = (int)((long)pixels * (s + 1) / splits);
}

// Fold the (count, mean, M2) partials of every (image, channel) over its row groups: block
// (32 channels, image), warp w takes groups w, w + 8, ...; pass 1 sums count and count * mean, pass 2
// sums M2_q + n_q (mean_q - mean)^2 (the exact pooled-variance identity), both in double, and the
// eight warps' sums are added in warp order, so the result is deterministic.
constexpr int kFoldWarps = 8;
__global__ void __launch_bounds__(kFoldWarps * 32) bn_stats_fold_kernel(const float* part, int c, int groups,
                                                                        float eps, float* stats, float* mean_p,
                                                                        float* inv_p) {
    __shared__ double r1[kFoldWarps][32], r2[kFoldWarps][32];
    __shared__ double mean_s[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y;
    const bool on = ch < c;
    const float* pb = part + (long)b * groups * c * 3;
    double n = 0.0, sum = 0.0;
    if (on)
        for (int q = warp; q < groups; q += kFoldWarps) {
            const float* o = pb + ((long)q * c + ch) * 3;
            n += o[0];
            sum += (double)o[0] * o[1];
        }
    r1[warp][lane] = n;
    r2[warp][lane] = sum;
    __syncthreads();
    if (warp == 0) {
        double tn = 0.0, ts = 0.0;
        for (int w = 0; w < kFoldWarps; w++) {
            tn += r1[w][lane];
            ts += r2[w][lane];
        }
        mean_s[lane] = tn > 0.0 ? ts / tn : 0.0;
        r1[0][lane] = tn;
    }
    __syncthreads();
    const double mean = mean_s[lane], ntot = r1[0][lane];
    __syncthreads();
    double m2 = 0.0;
    if (on)
        for (int q = warp; q < groups; q += kFoldWarps) {
            const float* o = pb + ((long)q * c + ch) * 3;
            const double d = (double)o[1] - mean;
            m2 += (double)o[2] + (double)o[0] * d * d;
        }
    r2[warp][lane] = m2;
    __syncthreads();
    if (warp == 0 && on) {
        double t = 0.0;
        for (int w = 0; w < kFoldWarps; w++) t += r2[w][lane];
        const long i = (long)b * c + ch;
        const float mf = (float)mean, var = (float)(ntot > 0.0 ? t / ntot : 0.0);
        stats[i * 2 + 0] = mf;
        stats[i * 2 + 1] = var;
        mean_p[i] = mf;
        inv_p[i] = 1.0f / sqrtf(var + eps);
    }
}

// a = SiLU(gamma * (y - mean) * inv + beta) on interior rows, zero on halo / tail rows; one image per
// blockIdx.y.
template <bool kVec>
__global__ void bn_apply_kernel(const float* y, int ypitch, const float* mean_p, const float* inv_p,
                                const float* gamma, const float* beta, int c, Grid g, float* a, int apitch, int rnd) {
    const int b = blockIdx.y;
    const int per_row = kVec ? c / 4 : c;
    const int total = g.rows * per_row;   // < 2^22 (checked by the launcher)
    const float inv_row = 1.0f / (float)per_row, inv_wp = 1.0f / (float)g.wp;
    const long base = (long)b * g.rows;
    const float* mb = mean_p + (long)b * c;
    const float* ib = inv_p + (long)b * c;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = fast_div(i, inv_row), j = i - r * per_row;
        const long row = base + r;
        const int py = fast_div(r, inv_wp), px = r - py * g.wp;
        const bool in = py >= 1 && py <= g.h && px >= 1 && px <= g.w;
        if (kVec) {
            float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
            if (in) {
                const float4 v = *reinterpret_cast<const float4*>(y + row * ypitch + 4 * j);
                const float4 mv = *reinterpret_cast<const float4*>(mb + 4 * j);
                const float4 iv = *reinterpret_cast<const float4*>(ib + 4 * j);
                const int ch = 4 * j;
                out.x = silu_f((v.x - mv.x) * iv.x * gamma[ch] + beta[ch]);
                out.y = silu_f((v.y - mv.y) * iv.y * gamma[ch + 1] + beta[ch + 1]);
                out.z = silu_f((v.z - mv.z) * iv.z * gamma[ch + 2] + beta[ch + 2]);
                out.w = silu_f((v.w - mv.w) * iv.w * gamma[ch + 3] + beta[ch + 3]);
                if (rnd) out = make_float4(tf32_rna(out.x), tf32_rna(out.y), tf32_rna(out.z), tf32_rna(out.w));
            }
            *reinterpret_cast<float4*>(a + row * apitch + 4 * j) = out;
        } else {
            float out = 0.0f;
            if (in) out = silu_f((y[row * ypitch + j] - mb[j]) * ib[j] * gamma[j] + beta[j]);
            a[row * apitch + j] = rnd ? tf32_rna(out) : out;
        }
    }
}

// The same for channels in whole float4 groups: a thread keeps one channel group's coefficients in registers and
// walks the image's rows (blockDim.x / (c / 4) rows in flight per block), so each element costs one load, the
// arithmetic and one store.  SiLU as x / (1 + exp(-x)) with the fast exponential and division of the conv
// epilogues.
__global__ void __launch_bounds__(256) bn_apply_rows_kernel(const float* y, int ypitch, const float* mean_p,
                                                            const float* inv_p, const float* gamma, const float* beta,
                                                            int c, Grid g, float* a, int apitch, int rnd) {
    const int b = blockIdx.y, per_row = c >> 2;
    const int slots = blockDim.x / per_row;
    if ((int)threadIdx.x >= slots * per_row) return;
    const int j = threadIdx.x % per_row, r0 = threadIdx.x / per_row, ch = 4 * j;
    const float4 mv = *reinterpret_cast<const float4*>(mean_p + (long)b * c + ch);
    const float4 iv = *reinterpret_cast<const float4*>(inv_p + (long)b * c + ch);
    const float g0 = gamma[ch], g1 = gamma[ch + 1], g2 = gamma[ch + 2], g3 = gamma[ch + 3];
    const float b0 = beta[ch], b1 = beta[ch + 1], b2 = beta[ch + 2], b3 = beta[ch + 3];
    const float inv_wp = 1.0f / (float)g.wp;
    const long base = (long)b * g.rows;
    for (int r = blockIdx.x * slots + r0; r < g.rows; r += gridDim.x * slots) {
        const int py = fast_div(r, inv_wp), px = r - py * g.wp;
        const bool in = py >= 1 && py <= g.h && px >= 1 && px <= g.w;
        const long row = base + r;
        float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
        if (in) {
            const float4 v = *reinterpret_cast<const float4*>(y + row * ypitch + ch);
            out.x = silu_fast((v.x - mv.x) * iv.x * g0 + b0);
            out.y = silu_fast((v.y - mv.y) * iv.y * g1 + b1);
            out.z = silu_fast((v.z - mv.z) * iv.z * g2 + b2);
            out.w = silu_fast((v.w - mv.w) * iv.w * g3 + b3);
            if (rnd) out = make_float4(tf32_rna(out.x), tf32_rna(out.y), tf32_rna(out.z), tf32_rna(out.w));
        }
        *reinterpret_cast<float4*>(a + row * apitch + ch) = out;
    }
}

// Evaluation mode (HeadOperations.cs:158-166 with training = false): every image normalises with the
// running mean / variance.
__global__ void bn_eval_coef_kernel(const float* rm, const float* rv, float eps, long n, int c, float* mean_p,
                                    float* inv_p) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int ch = (int)(i % c);
    mean_p[i] = rm[ch];
    inv_p[i] = 1.0f / sqrtf(rv[ch] + eps);
}

// red[b][ch] = (sum dz, sum dz xhat) folded over the row groups; f = gamma inv / n.  Block (32 channels,
// image): warp w sums groups w, w + 8, ... and the eight warps' sums are added in warp order, so the
// result is deterministic.
__global__ void __launch_bounds__(kFoldWarps * 32) bn_bwd_fold_kernel(const float* part, int batch, int c, int groups,
                                                                      float n_pix, const float* inv_p,
                                                                      const float* gamma, float* red, float* f_p) {
    __shared__ float r1[kFoldWarps][32], r2[kFoldWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y;
    const bool on = ch < c;
    float t1 = 0.0f, t2 = 0.0f;
    if (on)
#pragma unroll 4
        for (int q = warp; q < groups; q += kFoldWarps) {
            const float* o = part + (((long)b * groups + q) * c + ch) * 2;
            t1 += o[0];
            t2 += o[1];
        }
    r1[warp][lane] = t1;
    r2[warp][lane] = t2;
    __syncthreads();
    if (warp == 0 && on) {
        float s1 = 0.0f, s2 = 0.0f;
        for (int w = 0; w < kFoldWarps; w++) {
            s1 += r1[w][lane];
            s2 += r2[w][lane];
        }
        const long i = (long)b * c + ch;
        red[i * 2 + 0] = s1;
        red[i * 2 + 1] = s2;
        f_p[i] = gamma[ch] * inv_p[i] / n_pix;
    }
}

// dgamma += sum_b red[b][ch][1], dbeta += sum_b red[b][ch][0], images in order.
__global__ void bn_param_grad_kernel(const float* red, int batch, int c, float* dgamma, float* dbeta) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= c) return;
    float dg = dgamma[ch], db = dbeta[ch];
#pragma unroll 8
    for (int b = 0; b < batch; b++) {
        db += red[((long)b * c + ch) * 2 + 0];
        dg += red[((long)b * c + ch) * 2 + 1];
    }
    dgamma[ch] = dg;
    dbeta[ch] = db;
}

// dy = gamma * inv / n * (n * dz - sum dz - xhat * sum dz xhat)  (HeadOperations.cs:185-189), with dz
// already formed by the data-gradient epilogue; one image per blockIdx.y.
template <bool kVec>
__global__ void bn_bwd_apply_kernel(const float* y, int ypitch, const float* dz, int zpitch, const float* mean_p,
                                    const float* inv_p, const float* f_p, const float* red, int c, float n, Grid g,
                                    float* dy, int dpitch, int rnd) {
    const int b = blockIdx.y;
    const int per_row = kVec ? c / 4 : c;
    const int total = g.rows * per_row;   // < 2^22 (checked by the launcher)
    const float inv_row = 1.0f / (float)per_row, inv_wp = 1.0f / (float)g.wp;
    const long base = (long)b * g.rows;
    const float* mb = mean_p + (long)b * c;
    const float* ib = inv_p + (long)b * c;
    const float* fb = f_p + (long)b * c;
    const float* rb = red + (long)b * c * 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = fast_div(i, inv_row), j = i - r * per_row;
        const long row = base + r;
        const int py = fast_div(r, inv_wp), px = r - py * g.wp;
        const bool in = py >= 1 && py <= g.h && px >= 1 && px <= g.w;
        if (kVec) {
            float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
            if (in) {
                const float4 yv = *reinterpret_cast<const float4*>(y + row * ypitch + 4 * j);
                const float4 zv = *reinterpret_cast<const float4*>(dz + row * zpitch + 4 * j);
                const float4 mv = *reinterpret_cast<const float4*>(mb + 4 * j);
                const float4 iv = *reinterpret_cast<const float4*>(ib + 4 * j);
                const float4 fv = *reinterpret_cast<const float4*>(fb + 4 * j);
                const float4 r0 = *reinterpret_cast<const float4*>(rb + 8 * j);
                const float4 r1 = *reinterpret_cast<const float4*>(rb + 8 * j + 4);
                out.x = fv.x * (n * zv.x - r0.x - (yv.x - mv.x) * iv.x * r0.y);
                out.y = fv.y * (n * zv.y - r0.z - (yv.y - mv.y) * iv.y * r0.w);
                out.z = fv.z * (n * zv.z - r1.x - (yv.z - mv.z) * iv.z * r1.y);
                out.w = fv.w * (n * zv.w - r1.z - (yv.w - mv.w) * iv.w * r1.w);
                if (rnd) out = make_float4(tf32_rna(out.x), tf32_rna(out.y), tf32_rna(out.z), tf32_rna(out.w));
            }
            *reinterpret_cast<float4*>(dy + row * dpitch + 4 * j) = out;
        } else {
            float out = 0.0f;
            if (in)
                out = fb[j] * (n * dz[row * zpitch + j] - rb[2 * j] - (y[row * ypitch + j] - mb[j]) * ib[j] * rb[2 * j + 1]);
            dy[row * dpitch + j] = rnd ? tf32_rna(out) : out;
        }
    }
}

// The same for channels in whole float4 groups, coefficients of one channel group per thread in registers
// (see bn_apply_rows_kernel).
__global__ void __launch_bounds__(256) bn_bwd_apply_rows_kernel(const float* y, int ypitch, const float* dz, int zpitch,
                                                                const float* mean_p, const float* inv_p, const float* f_p,
                                                                const float* red, int c, float n, Grid g, float* dy,
                                                                int dpitch, int rnd) {
    const int b = blockIdx.y, per_row = c >> 2;
    const int slots = blockDim.x / per_row;
    if ((int)threadIdx.x >= slots * per_row) return;
    const int j = threadIdx.x % per_row, r0 = threadIdx.x / per_row, ch = 4 * j;
    const float4 mv = *reinterpret_cast<const float4*>(mean_p + (long)b * c + ch);
    const float4 iv = *reinterpret_cast<const float4*>(inv_p + (long)b * c + ch);
    const float4 fv = *reinterpret_cast<const float4*>(f_p + (long)b * c + ch);
    const float4 q0 = *reinterpret_cast<const float4*>(red + (long)b * c * 2 + 8 * j);
    const float4 q1 = *reinterpret_cast<const float4*>(red + (long)b * c * 2 + 8 * j + 4);
    const float inv_wp = 1.0f / (float)g.wp;
    const long base = (long)b * g.rows;
    for (int r = blockIdx.x * slots + r0; r < g.rows; r += gridDim.x * slots) {
        const int py = fast_div(r, inv_wp), px = r - py * g.wp;
        const bool in = py >= 1 && py <= g.h && px >= 1 && px <= g.w;
        const long row = base + r;
        float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
        if (in) {
            const float4 yv = *reinterpret_cast<const float4*>(y + row * ypitch + ch);
            const float4 zv = *reinterpret_cast<const float4*>(dz + row * zpitch + ch);
            out.x = fv.x * (n * zv.x - q0.x - (yv.x - mv.x) * iv.x * q0.y);
            out.y = fv.y * (n * zv.y - q0.z - (yv.y - mv.y) * iv.y * q0.w);
            out.z = fv.z * (n * zv.z - q1.x - (yv.z - mv.z) * iv.z * q1.y);
            out.w = fv.w * (n * zv.w - q1.z - (yv.w - mv.w) * iv.w * q1.w);
            if (rnd) out = make_float4(tf32_rna(out.x), tf32_rna(out.y), tf32_rna(out.z), tf32_rna(out.w));
        }
        *reinterpret_cast<float4*>(dy + row * dpitch + ch) = out;
    }
}

__global__ void bn_running_kernel(const float* stats, long rank_stride, int ranks, int batch, int c, int spatial,
                                  float m, float* rmean, float* rvar, float* tracked) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch < c) {
        float rm = rmean[ch], rv = rvar[ch];
        const float unbias = spatial > 1 ? (float)spatial / (spatial - 1) : 1.0f;
        for (int r = 0; r < ranks; r++)
            for (int b = 0; b < batch; b++) {
                const float* s = stats + r * rank_stride + ((long)b * c + ch) * 2;
                rm = (1 - m) * rm + m * s[0];
                rv = (1 - m) * rv + m * s[1] * unbias;
            }
        rmean[ch] = rm;
        rvar[ch] = rv;
    }
    if (ch == 0 && tracked) tracked[0] += (float)batch * ranks;
}

// All BatchNorm layers of the head in one launch: blockIdx.y = layer (BnFoldJob table), threads over
// channels; per channel the images are folded in order, exactly as bn_running_kernel / bn_param_grad_kernel.
__global__ void bn_running_batch_kernel(const BnFoldJob* jobs, const float* stats, long rank_stride, int ranks,
                                        int batch, float m) {
    const BnFoldJob jb = jobs[blockIdx.y];
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch < jb.c) {
        const float* st = stats + jb.stats_off;
        float rm = jb.rmean[ch], rv = jb.rvar[ch];
        const float unbias = jb.spatial > 1 ? (float)jb.spatial / (jb.spatial - 1) : 1.0f;
        for (int r = 0; r < ranks; r++)
            for (int b = 0; b < batch; b++) {
                const float* s = st + r * rank_stride + ((long)b * jb.c + ch) * 2;
                rm = (1 - m) * rm + m * s[0];
                rv = (1 - m) * rv + m * s[1] * unbias;
            }
        jb.rmean[ch] = rm;
        jb.rvar[ch] = rv;
    }
    if (ch == 0 && jb.tracked) jb.tracked[0] += (float)batch * ranks;
}

__global__ void bn_param_grad_batch_kernel(const BnFoldJob* jobs, int batch) {
    const BnFoldJob jb = jobs[blockIdx.y];
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= jb.c) return;
    const float* red = jb.bcoef + (long)batch * jb.c;   // bcoef = [f plane | (sum dz, sum dz xhat) pairs]
    float dg = jb.dgamma[ch], db = jb.dbeta[ch];
    for (int b = 0; b < batch; b++) {
        db += red[((long)b * jb.c + ch) * 2 + 0];
        dg += red[((long)b * jb.c + ch) * 2 + 1];
    }
    jb.dgamma[ch] = dg;
    jb.dbeta[ch] = db;
}

// ---------------------------------------------------------------- centred weight gradient (kernels.h)
// Partial sums of x over a slice of the interior pixels of one image: block (32 channels, image, slice),
// lane = channel, warp w takes pixels w, w + 8, ... of the slice into four running sums (four loads in
// flight); the warps' sums are added in warp order.  part[(b * splits + s) * c + ch].
__global__ void __launch_bounds__(kThreads) feature_sum_kernel(const float* x, int pitch, int c, Grid g, int splits,
                                                               float* part) {
    __shared__ float red[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y, s = blockIdx.z;
    int p0, p1;
    split_range(g.h * g.w, splits, s, p0, p1);
    float acc = 0.0f;
    if (ch < c) {
        const float* img = x + (long)b * g.rows * pitch + ch;
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        int p = p0 + warp;
        for (; p + 3 * kWarps < p1; p += 4 * kWarps) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int q = p + k * kWarps, yy = q / g.w, xx = q - yy * g.w;
                a[k] += img[(long)g.row(yy, xx) * pitch];
            }
        }
        for (; p < p1; p += kWarps) {
            const int yy = p / g.w, xx = p - yy * g.w;
            a[0] += img[(long)g.row(yy, xx) * pitch];
        }
        acc = (a[0] + a[1]) + (a[2] + a[3]);
    }
    red[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && ch < c) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        part[((long)b * splits + s) * c + ch] = t;
    }
}

// mean[b][ch] = (sum of the slices in order) / pixels
__global__ void feature_mean_fold_kernel(const float* part, int batch, int c, int splits, float inv_pixels,
                                         float* mean) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)batch * c) return;
    const int b = (int)(i / c), ch = (int)(i - (long)b * c);
    double t = 0.0;
    for (int s = 0; s < splits; s++) t += part[((long)b * splits + s) * c + ch];
    mean[i] = (float)(t * inv_pixels);
}

// xc = x - mean[b][ch] at interior rows, 0 elsewhere; one image per blockIdx.y, float4 when kVec.
template <bool kVec>
__global__ void feature_center_kernel(const float* x, int xpitch, const float* mean, int c, Grid g, float* xc,
                                      int cpitch, int rnd) {
    const int b = blockIdx.y;
    const int per_row = kVec ? c / 4 : c;
    const int total = g.rows * per_row;   // < 2^22 (checked by the launcher)
    const float inv_row = 1.0f / (float)per_row, inv_wp = 1.0f / (float)g.wp;
    const long base = (long)b * g.rows;
    const float* mb = mean + (long)b * c;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int r = fast_div(i, inv_row), j = i - r * per_row;
        const long row = base + r;
        const int py = fast_div(r, inv_wp), px = r - py * g.wp;
        const bool in = py >= 1 && py <= g.h && px >= 1 && px <= g.w;
        if (kVec) {
            float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
            if (in) {
                const float4 v = *reinterpret_cast<const float4*>(x + row * xpitch + 4 * j);
                const float4 m = *reinterpret_cast<const float4*>(mb + 4 * j);
                out = make_float4(v.x - m.x, v.y - m.y, v.z - m.z, v.w - m.w);
                if (rnd) out = make_float4(tf32_rna(out.x), tf32_rna(out.y), tf32_rna(out.z), tf32_rna(out.w));
            }
            *reinterpret_cast<float4*>(xc + row * cpitch + 4 * j) = out;
        } else {
            float out = in ? x[row * xpitch + j] - mb[j] : 0.0f;
            xc[row * cpitch + j] = rnd ? tf32_rna(out) : out;
        }
    }
}

// Edge-strip sums of dy per (image, channel): block (32 channels, image), lane = channel; warp w takes
// strip elements w, w + 8, ... of the top row, bottom row, left column and right column (double, warps
// added in order).  With `part` the sum over all interior pixels is taken from its slices
// (feature_sum_kernel), else it is 0: the gradient of a conv that feeds a per-image BatchNorm sums to
// exactly zero over the pixels of each (image, channel), so the identity holds with the exact value 0,
// and the rounding of the stored dy then stays out of the correction.
// T[b][t][o]: tap t = (ky, kx) reads source offset (ky - 1, kx - 1), which leaves the map for the top row
// when ky = 0, the bottom row when ky = 2, and likewise for the columns (inclusion-exclusion adds the
// corner back).
__global__ void __launch_bounds__(kFoldWarps * 32) tap_border_sums_kernel(const float* dy, int pitch, int c, Grid g,
                                                                          int taps, const float* part, int splits,
                                                                          float* tsum) {
    __shared__ double r[4][kFoldWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y;
    const float* img = dy + (long)b * g.rows * pitch + ch;
    double e[4] = {0.0, 0.0, 0.0, 0.0};   // top, bottom, left, right
    if (ch < c && taps == 9) {
        const int n = 2 * g.w + 2 * g.h;
        for (int k = warp; k < n; k += kFoldWarps) {
            int yy, xx, side;
            if (k < g.w) {
                side = 0; yy = 0; xx = k;
            } else if (k < 2 * g.w) {
                side = 1; yy = g.h - 1; xx = k - g.w;
            } else if (k < 2 * g.w + g.h) {
                side = 2; yy = k - 2 * g.w; xx = 0;
            } else {
                side = 3; yy = k - 2 * g.w - g.h; xx = g.w - 1;
            }
            e[side] += img[(long)g.row(yy, xx) * pitch];
        }
    }
    for (int k = 0; k < 4; k++) r[k][warp][lane] = e[k];
    __syncthreads();
    if (warp != 0 || ch >= c) return;
    double t[4] = {0.0, 0.0, 0.0, 0.0};
    for (int k = 0; k < 4; k++)
        for (int w = 0; w < kFoldWarps; w++) t[k] += r[k][w][lane];
    double total = 0.0;
    if (part)
        for (int s = 0; s < splits; s++) total += part[((long)b * splits + s) * c + ch];
    float* out = tsum + (long)b * taps * c + ch;
    if (taps == 1) {
        out[0] = (float)total;
        return;
    }
    const double corner[2][2] = {{img[(long)g.row(0, 0) * pitch], img[(long)g.row(0, g.w - 1) * pitch]},
                                 {img[(long)g.row(g.h - 1, 0) * pitch], img[(long)g.row(g.h - 1, g.w - 1) * pitch]}};
    for (int ky = 0; ky < 3; ky++)
        for (int kx = 0; kx < 3; kx++) {
            double v = total;
            if (ky == 0) v -= t[0];
            if (ky == 2) v -= t[1];
            if (kx == 0) v -= t[2];
            if (kx == 2) v -= t[3];
            if (ky != 1 && kx != 1) v += corner[ky == 2][kx == 2];
            out[(long)(ky * 3 + kx) * c] = (float)v;
        }
}

}  // namespace

size_t bn_partial_floats(int batch, const Grid& g, int channels) {
    return (size_t)batch * (g.rows / 32) * channels * 3;
}

static dim3 image_grid(long per_image, int batch) {
    const long want = std::max<long>(1, (148L * 16 + batch - 1) / batch);
    return dim3((unsigned)std::min<long>(want, std::max<long>(1, (per_image + 255) / 256)), (unsigned)batch);
}

void bn_stats_fold(const float* part, int batch, const Grid& g, int c, float eps, float* stats, float* coef,
                   cudaStream_t stream) {
    const long n = (long)batch * c;
    bn_stats_fold_kernel<<<dim3((c + 31) / 32, batch), kFoldWarps * 32, 0, stream>>>(part, c, g.rows / 32, eps, stats,
                                                                                     coef, coef + n);
    launch_check("bn_stats_fold_kernel");
}

void bn_eval_coef(const float* rmean, const float* rvar, float eps, int batch, int c, float* coef,
                  cudaStream_t stream) {
    const long n = (long)batch * c;
    bn_eval_coef_kernel<<<(int)((n + 255) / 256), 256, 0, stream>>>(rmean, rvar, eps, n, c, coef, coef + n);
    launch_check("bn_eval_coef_kernel");
}

void bn_silu_apply(const View& y, const float* coef, const float* gamma, const float* beta, int batch, const Grid& g,
                   const View& a, cudaStream_t stream, bool round_tf32) {
    const int c = y.channels;
    const int rnd = round_tf32 ? 1 : 0;
    const bool vec = c % 4 == 0 && y.pitch % 4 == 0 && a.pitch % 4 == 0;
    const long per_image = (long)g.rows * (vec ? c / 4 : c);
    if (per_image >= (1L << 22)) throw std::runtime_error("bn_silu_apply: image too large");
    const float* inv = coef + (long)batch * c;
    if (vec && c / 4 <= 256)
        bn_apply_rows_kernel<<<image_grid(per_image, batch), 256, 0, stream>>>(y.base, y.pitch, coef, inv, gamma, beta,
                                                                                c, g, a.base, a.pitch, rnd);
    else if (vec)
        bn_apply_kernel<true><<<image_grid(per_image, batch), 256, 0, stream>>>(y.base, y.pitch, coef, inv, gamma,
                                                                                beta, c, g, a.base, a.pitch, rnd);
    else
        bn_apply_kernel<false><<<image_grid(per_image, batch), 256, 0, stream>>>(y.base, y.pitch, coef, inv, gamma,
                                                                                 beta, c, g, a.base, a.pitch, rnd);
    launch_check("bn_apply_kernel");
}

void bn_running_update_batch(const BnFoldJob* jobs, int njobs, int max_c, const float* stats, long rank_stride,
                             int ranks, int batch, float momentum, cudaStream_t stream) {
    bn_running_batch_kernel<<<dim3((max_c + 127) / 128, njobs), 128, 0, stream>>>(jobs, stats, rank_stride, ranks,
                                                                                   batch, momentum);
    launch_check("bn_running_batch_kernel");
}

void bn_param_grad_batch(const BnFoldJob* jobs, int njobs, int max_c, int batch, cudaStream_t stream) {
    bn_param_grad_batch_kernel<<<dim3((max_c + 127) / 128, njobs), 128, 0, stream>>>(jobs, batch);
    launch_check("bn_param_grad_batch_kernel");
}

void bn_backward_fold(const float* part, int batch, const Grid& g, int c, const float* coef, const float* gamma,
                      float* dgamma, float* dbeta, float* bcoef, cudaStream_t stream, bool param_grad) {
    const long n = (long)batch * c;
    float* red = bcoef + n;
    bn_bwd_fold_kernel<<<dim3((c + 31) / 32, batch), kFoldWarps * 32, 0, stream>>>(part, batch, c, g.rows / 32,
                                                                                  (float)(g.h * g.w), coef + n, gamma,
                                                                                  red, bcoef);
    launch_check("bn_bwd_fold_kernel");
    if (!param_grad) return;
    bn_param_grad_kernel<<<(c + 127) / 128, 128, 0, stream>>>(red, batch, c, dgamma, dbeta);
    launch_check("bn_param_grad_kernel");
}

void bn_backward_apply(const View& y, const View& dz, const float* coef, const float* bcoef, int batch, const Grid& g,
                       const View& dy, cudaStream_t stream, bool round_tf32) {
    const int c = y.channels;
    const int rnd = round_tf32 ? 1 : 0;
    const bool vec = c % 4 == 0 && y.pitch % 4 == 0 && dz.pitch % 4 == 0 && dy.pitch % 4 == 0;
    const long per_image = (long)g.rows * (vec ? c / 4 : c);
    if (per_image >= (1L << 22)) throw std::runtime_error("bn_backward_apply: image too large");
    const float* inv = coef + (long)batch * c;
    const float* red = bcoef + (long)batch * c;
    const float n = (float)(g.h * g.w);
    if (vec && c / 4 <= 256)
        bn_bwd_apply_rows_kernel<<<image_grid(per_image, batch), 256, 0, stream>>>(
            y.base, y.pitch, dz.base, dz.pitch, coef, inv, bcoef, red, c, n, g, dy.base, dy.pitch, rnd);
    else if (vec)
        bn_bwd_apply_kernel<true><<<image_grid(per_image, batch), 256, 0, stream>>>(
            y.base, y.pitch, dz.base, dz.pitch, coef, inv, bcoef, red, c, n, g, dy.base, dy.pitch, rnd);
    else
        bn_bwd_apply_kernel<false><<<image_grid(per_image, batch), 256, 0, stream>>>(
            y.base, y.pitch, dz.base, dz.pitch, coef, inv, bcoef, red, c, n, g, dy.base, dy.pitch, rnd);
    launch_check("bn_bwd_apply_kernel");
}

static int center_splits(int batch, int channels, const Grid& g) {
    const int cgroups = (channels + 31) / 32;
    const int want = (148 * 4 + cgroups * batch - 1) / (cgroups * batch);
    return std::max(1, std::min({want, 64, std::max(1, g.h * g.w / 256)}));
}

size_t center_workspace_floats(int batch, int channels) { return (size_t)batch * 64 * channels; }

void center_features(const View& x, int batch, const Grid& g, float* mean, float* ws, const View& xc,
                     bool round_tf32, cudaStream_t stream) {
    const int c = x.channels;
    const int splits = center_splits(batch, c, g);
    feature_sum_kernel<<<dim3((c + 31) / 32, batch, splits), kThreads, 0, stream>>>(x.base, x.pitch, c, g, splits, ws);
    launch_check("feature_sum_kernel");
    feature_mean_fold_kernel<<<(int)(((long)batch * c + 127) / 128), 128, 0, stream>>>(ws, batch, c, splits,
                                                                                         1.0f / (float)(g.h * g.w), mean);
    launch_check("feature_mean_fold_kernel");
    const bool vec = c % 4 == 0 && x.pitch % 4 == 0 && xc.pitch % 4 == 0;
    const long per_image = (long)g.rows * (vec ? c / 4 : c);
    if (per_image >= (1L << 22)) throw std::runtime_error("center_features: image too large");
    const int rnd = round_tf32 ? 1 : 0;
    if (vec)
        feature_center_kernel<true><<<image_grid(per_image, batch), 256, 0, stream>>>(x.base, x.pitch, mean, c, g,
                                                                                      xc.base, xc.pitch, rnd);
    else
        feature_center_kernel<false><<<image_grid(per_image, batch), 256, 0, stream>>>(x.base, x.pitch, mean, c, g,
                                                                                       xc.base, xc.pitch, rnd);
    launch_check("feature_center_kernel");
}

void tap_border_sums(const View& dy, int batch, const Grid& g, int taps, bool zero_total, float* ws, float* tsum,
                     cudaStream_t stream) {
    if (taps != 1 && taps != 9) throw std::runtime_error("tap_border_sums: taps must be 1 or 9");
    const int c = dy.channels;
    int splits = 0;
    if (!zero_total) {
        splits = center_splits(batch, c, g);
        feature_sum_kernel<<<dim3((c + 31) / 32, batch, splits), kThreads, 0, stream>>>(dy.base, dy.pitch, c, g, splits,
                                                                                      ws);
        launch_check("feature_sum_kernel");
    }
    tap_border_sums_kernel<<<dim3((c + 31) / 32, batch), kFoldWarps * 32, 0, stream>>>(
        dy.base, dy.pitch, c, g, taps, zero_total ? nullptr : ws, splits, tsum);
    launch_check("tap_border_sums_kernel");
}

void bn_running_update(const float* stats, long rank_stride, int ranks, int batch, int c, int spatial, float momentum,
                       float* rmean, float* rvar, float* tracked, cudaStream_t stream) {
    bn_running_kernel<<<(c + 127) / 128, 128, 0, stream>>>(stats, rank_stride, ranks, batch, c, spatial, momentum,
                                                           rmean, rvar, tracked);
    launch_check("bn_running_kernel");
}

}  // namespace sy
