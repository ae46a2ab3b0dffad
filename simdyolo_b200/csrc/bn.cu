// Training-mode BatchNorm with per-image statistics, fused with SiLU, forward and backward
// (HeadOperations.BatchNorm HeadOperations.cs:153-193, HeadOperations.Silu :198-221), running
// statistics (HeadOperations.cs:164-165, num_batches_tracked DetectionHead.cs:154) and the bias
// gradient of the final conv (HeadOperations.cs:66).
//
// Each image normalises with its own mean / variance over H x W, exactly like the reference's
// batch-of-one convs, so a batch of B images needs B x C statistics.  Reductions split every
// (image, channel group) over several blocks of pixels; each block writes (count, mean, M2) or plain
// sums and a second kernel folds the splits in a fixed order (Chan's pairwise variance update), so
// results do not depend on timing.  Elementwise passes move float4s and do one division per row.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct Split {
    int splits;     // pixel splits per (image, channel group)
    int cgroups;    // channel groups of 32
};

Split choose_split(int batch, int channels, const Grid& g) {
    Split s;
    s.cgroups = (channels + 31) / 32;
    const int pixels = g.h * g.w;
    const int want_blocks = 148 * 4;
    int splits = (want_blocks + s.cgroups * batch - 1) / (s.cgroups * batch);
    splits = std::min(splits, std::max(1, pixels / 64));
    s.splits = std::max(1, std::min(splits, 64));
    return s;
}

__device__ __forceinline__ void split_range(int pixels, int splits, int s, int& p0, int& p1) {
    p0 = (int)((long)pixels * s / splits);
    p1 = (int)((long)pixels * (s + 1) / splits);
}

// Partial (count, mean, M2) of one (image, 32 channels, pixel split): two passes over the split.
__global__ void __launch_bounds__(kThreads) bn_stats_partial_kernel(const float* y, int pitch, int c, Grid g,
                                                                    int splits, float* part) {
    __shared__ float red[kWarps][32];
    __shared__ float mean_s[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y, s = blockIdx.z;
    int p0, p1;
    split_range(g.h * g.w, splits, s, p0, p1);
    const float* base = y + (long)b * g.rows * pitch + ch;
    const bool on = ch < c;
    float acc = 0.0f;
    if (on)
        for (int p = p0 + warp; p < p1; p += kWarps) {
            const int yy = p / g.w, xx = p - yy * g.w;
            acc += base[(long)g.row(yy, xx) * pitch];
        }
    red[warp][lane] = acc;
    __syncthreads();
    const int n = p1 - p0;
    if (warp == 0) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        mean_s[lane] = n > 0 ? t / n : 0.0f;
    }
    __syncthreads();
    const float mean = mean_s[lane];
    float m2 = 0.0f;
    if (on)
        for (int p = p0 + warp; p < p1; p += kWarps) {
            const int yy = p / g.w, xx = p - yy * g.w;
            const float d = base[(long)g.row(yy, xx) * pitch] - mean;
            m2 += d * d;
        }
    red[warp][lane] = m2;
    __syncthreads();
    if (warp == 0 && on) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        float* o = part + (((long)b * splits + s) * c + ch) * 3;
        o[0] = (float)n;
        o[1] = mean;
        o[2] = t;
    }
}

// Fold the splits of every (image, channel) in order; stats = (mean, biased variance).
__global__ void bn_stats_final_kernel(const float* part, int batch, int c, int splits, float* stats) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)batch * c) return;
    const int b = (int)(i / c), ch = (int)(i - (long)b * c);
    double n = 0.0, mean = 0.0, m2 = 0.0;
    for (int s = 0; s < splits; s++) {
        const float* o = part + (((long)b * splits + s) * c + ch) * 3;
        const double nb = o[0];
        if (nb == 0.0) continue;
        const double delta = (double)o[1] - mean, tot = n + nb;
        mean += delta * nb / tot;
        m2 += (double)o[2] + delta * delta * n * nb / tot;
        n = tot;
    }
    stats[i * 2 + 0] = (float)mean;
    stats[i * 2 + 1] = (float)(n > 0 ? m2 / n : 0.0);
}

// a = SiLU(gamma * (y - mean) * inv + beta) on interior rows, zero on halo / tail rows.
template <bool kVec>
__global__ void bn_apply_kernel(const float* y, int ypitch, const float* stats, const float* gamma, const float* beta,
                                float eps, int c, long rows, Grid g, float* a, int apitch) {
    const int per_row = kVec ? c / 4 : c;
    const long total = rows * per_row;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const long row = i / per_row;
        const int j = (int)(i - row * per_row);
        const int b = (int)(row / g.rows), r = (int)(row - (long)b * g.rows);
        const bool in = g.interior(r);
        if (kVec) {
            float4 out = make_float4(0.f, 0.f, 0.f, 0.f);
            if (in) {
                const float4 v = *reinterpret_cast<const float4*>(y + row * ypitch + 4 * j);
                float o[4];
                const float vi[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int ch = 4 * j + k;
                    const float mean = stats[((long)b * c + ch) * 2], var = stats[((long)b * c + ch) * 2 + 1];
                    const float inv = 1.0f / sqrtf(var + eps);
                    o[k] = silu_f((vi[k] - mean) * inv * gamma[ch] + beta[ch]);
                }
                out = make_float4(o[0], o[1], o[2], o[3]);
            }
            *reinterpret_cast<float4*>(a + row * apitch + 4 * j) = out;
        } else {
            float out = 0.0f;
            if (in) {
                const float mean = stats[((long)b * c + j) * 2], var = stats[((long)b * c + j) * 2 + 1];
                const float inv = 1.0f / sqrtf(var + eps);
                out = silu_f((y[row * ypitch + j] - mean) * inv * gamma[j] + beta[j]);
            }
            a[row * apitch + j] = out;
        }
    }
}

__device__ __forceinline__ float bn_dz(float yv, float gv, float mean, float inv, float ga, float be, float& xh) {
    xh = (yv - mean) * inv;
    const float z = xh * ga + be;
    const float sg = 1.0f / (1.0f + __expf(-z));
    return gv * (sg + z * sg * (1.0f - sg));
}

// Partial sums of dz and dz * xhat for one (image, 32 channels, pixel split).
__global__ void __launch_bounds__(kThreads) bn_bwd_partial_kernel(const float* y, int ypitch, const float* gr,
                                                                  int gpitch, const float* stats, const float* gamma,
                                                                  const float* beta, float eps, int c, Grid g,
                                                                  int splits, float* part) {
    __shared__ float r1[kWarps][32], r2[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y, s = blockIdx.z;
    int p0, p1;
    split_range(g.h * g.w, splits, s, p0, p1);
    float s1 = 0.0f, s2 = 0.0f;
    if (ch < c) {
        const float mean = stats[((long)b * c + ch) * 2], var = stats[((long)b * c + ch) * 2 + 1];
        const float inv = 1.0f / sqrtf(var + eps), ga = gamma[ch], be = beta[ch];
        const long base = (long)b * g.rows;
        for (int p = p0 + warp; p < p1; p += kWarps) {
            const int yy = p / g.w, xx = p - yy * g.w;
            const long row = base + g.row(yy, xx);
            float xh;
            const float dz = bn_dz(y[row * ypitch + ch], gr[row * gpitch + ch], mean, inv, ga, be, xh);
            s1 += dz;
            s2 += dz * xh;
        }
    }
    r1[warp][lane] = s1;
    r2[warp][lane] = s2;
    __syncthreads();
    if (warp == 0 && ch < c) {
        float t1 = 0.0f, t2 = 0.0f;
        for (int w = 0; w < kWarps; w++) {
            t1 += r1[w][lane];
            t2 += r2[w][lane];
        }
        float* o = part + (((long)b * splits + s) * c + ch) * 2;
        o[0] = t1;
        o[1] = t2;
    }
}

// red[b][ch] = (sum dz, sum dz xhat) folded over the splits, one thread per (image, channel).
__global__ void bn_bwd_final_kernel(const float* part, int batch, int c, int splits, float* red) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)batch * c) return;
    const int b = (int)(i / c), ch = (int)(i - (long)b * c);
    float t1 = 0.0f, t2 = 0.0f;
    for (int s = 0; s < splits; s++) {
        const float* o = part + (((long)b * splits + s) * c + ch) * 2;
        t1 += o[0];
        t2 += o[1];
    }
    red[i * 2 + 0] = t1;
    red[i * 2 + 1] = t2;
}

// dgamma += sum_b red[b][ch][1], dbeta += sum_b red[b][ch][0], images in order.
__global__ void bn_param_grad_kernel(const float* red, int batch, int c, float* dgamma, float* dbeta) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= c) return;
    float dg = dgamma[ch], db = dbeta[ch];
    for (int b = 0; b < batch; b++) {
        db += red[((long)b * c + ch) * 2 + 0];
        dg += red[((long)b * c + ch) * 2 + 1];
    }
    dgamma[ch] = dg;
    dbeta[ch] = db;
}

// dy = gamma * inv / n * (n * dz - sum dz - xhat * sum dz xhat)  (HeadOperations.cs:185-189)
template <bool kVec>
__global__ void bn_bwd_apply_kernel(const float* y, int ypitch, const float* gr, int gpitch, const float* stats,
                                    const float* red, const float* gamma, const float* beta, float eps, int c,
                                    long rows, Grid g, float* dy, int dpitch) {
    const int per_row = kVec ? c / 4 : c;
    const long total = rows * per_row;
    const float n = (float)(g.h * g.w);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const long row = i / per_row;
        const int j = (int)(i - row * per_row);
        const int b = (int)(row / g.rows), r = (int)(row - (long)b * g.rows);
        const bool in = g.interior(r);
        const int lanes = kVec ? 4 : 1;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        if (in) {
            float yv[4] = {0.f, 0.f, 0.f, 0.f}, gv[4] = {0.f, 0.f, 0.f, 0.f};
            if (kVec) {
                const float4 a = *reinterpret_cast<const float4*>(y + row * ypitch + 4 * j);
                const float4 d = *reinterpret_cast<const float4*>(gr + row * gpitch + 4 * j);
                yv[0] = a.x;
                yv[1] = a.y;
                yv[2] = a.z;
                yv[3] = a.w;
                gv[0] = d.x;
                gv[1] = d.y;
                gv[2] = d.z;
                gv[3] = d.w;
            } else {
                yv[0] = y[row * ypitch + j];
                gv[0] = gr[row * gpitch + j];
            }
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (k >= lanes) break;
                const int ch = kVec ? 4 * j + k : j;
                const long s = ((long)b * c + ch) * 2;
                const float inv = 1.0f / sqrtf(stats[s + 1] + eps), ga = gamma[ch];
                float xh;
                const float dz = bn_dz(yv[k], gv[k], stats[s], inv, ga, beta[ch], xh);
                o[k] = ga * inv / n * (n * dz - red[s] - xh * red[s + 1]);
            }
        }
        if (kVec)
            *reinterpret_cast<float4*>(dy + row * dpitch + 4 * j) = make_float4(o[0], o[1], o[2], o[3]);
        else
            dy[row * dpitch + j] = o[0];
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

__global__ void __launch_bounds__(kThreads) bias_partial_kernel(const float* gr, int pitch, int c, Grid g, int splits,
                                                                float* part) {
    __shared__ float red[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y, s = blockIdx.z;
    int p0, p1;
    split_range(g.h * g.w, splits, s, p0, p1);
    float acc = 0.0f;
    if (ch < c)
        for (int p = p0 + warp; p < p1; p += kWarps) {
            const int yy = p / g.w, xx = p - yy * g.w;
            acc += gr[((long)b * g.rows + g.row(yy, xx)) * pitch + ch];
        }
    red[warp][lane] = acc;
    __syncthreads();
    if (warp == 0 && ch < c) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        part[((long)b * splits + s) * c + ch] = t;
    }
}

// per_image[b][ch] = sum over the splits of image b (one thread per (image, channel))
__global__ void bias_image_kernel(const float* part, int batch, int c, int splits, float* per_image) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)batch * c) return;
    const int b = (int)(i / c), ch = (int)(i - (long)b * c);
    float acc = 0.0f;
    for (int s = 0; s < splits; s++) acc += part[((long)b * splits + s) * c + ch];
    per_image[i] = acc;
}

__global__ void bias_fold_kernel(const float* per_image, int batch, int c, float* db) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= c) return;
    float acc = db[ch];
    for (int b = 0; b < batch; b++) acc += per_image[(long)b * c + ch];
    db[ch] = acc;
}

int blocks_for(long n) { return (int)std::min<long>(148L * 16, std::max<long>(1, (n + 255) / 256)); }

}  // namespace

size_t bn_workspace_floats(int batch, int channels) { return (size_t)batch * 64 * channels * 3; }

void bn_stats(const View& y, int batch, const Grid& g, float* stats, float* ws, cudaStream_t stream) {
    const Split sp = choose_split(batch, y.channels, g);
    bn_stats_partial_kernel<<<dim3(sp.cgroups, batch, sp.splits), kThreads, 0, stream>>>(y.base, y.pitch, y.channels,
                                                                                       g, sp.splits, ws);
    launch_check("bn_stats_partial_kernel");
    const long n = (long)batch * y.channels;
    bn_stats_final_kernel<<<(int)((n + 127) / 128), 128, 0, stream>>>(ws, batch, y.channels, sp.splits, stats);
    launch_check("bn_stats_final_kernel");
}

void bn_silu_apply(const View& y, const float* stats, const float* gamma, const float* beta, float eps, int batch,
                   const Grid& g, const View& a, cudaStream_t stream) {
    const long rows = (long)batch * g.rows;
    const bool vec = y.channels % 4 == 0;
    const long n = rows * (vec ? y.channels / 4 : y.channels);
    if (vec)
        bn_apply_kernel<true><<<blocks_for(n), 256, 0, stream>>>(y.base, y.pitch, stats, gamma, beta, eps, y.channels,
                                                                 rows, g, a.base, a.pitch);
    else
        bn_apply_kernel<false><<<blocks_for(n), 256, 0, stream>>>(y.base, y.pitch, stats, gamma, beta, eps, y.channels,
                                                                  rows, g, a.base, a.pitch);
    launch_check("bn_apply_kernel");
}

void bn_silu_backward(const View& y, const View& gv, const float* stats, const float* gamma, const float* beta,
                      float eps, int batch, const Grid& gr, float* red, const View& dy, float* dgamma, float* dbeta,
                      float* ws, cudaStream_t stream) {
    const int c = y.channels;
    const Split sp = choose_split(batch, c, gr);
    bn_bwd_partial_kernel<<<dim3(sp.cgroups, batch, sp.splits), kThreads, 0, stream>>>(
        y.base, y.pitch, gv.base, gv.pitch, stats, gamma, beta, eps, c, gr, sp.splits, ws);
    launch_check("bn_bwd_partial_kernel");
    bn_bwd_final_kernel<<<(int)(((long)batch * c + 127) / 128), 128, 0, stream>>>(ws, batch, c, sp.splits, red);
    launch_check("bn_bwd_final_kernel");
    bn_param_grad_kernel<<<(c + 127) / 128, 128, 0, stream>>>(red, batch, c, dgamma, dbeta);
    launch_check("bn_param_grad_kernel");
    const long rows = (long)batch * gr.rows;
    const bool vec = c % 4 == 0;
    const long n = rows * (vec ? c / 4 : c);
    if (vec)
        bn_bwd_apply_kernel<true><<<blocks_for(n), 256, 0, stream>>>(y.base, y.pitch, gv.base, gv.pitch, stats, red,
                                                                     gamma, beta, eps, c, rows, gr, dy.base, dy.pitch);
    else
        bn_bwd_apply_kernel<false><<<blocks_for(n), 256, 0, stream>>>(y.base, y.pitch, gv.base, gv.pitch, stats, red,
                                                                      gamma, beta, eps, c, rows, gr, dy.base, dy.pitch);
    launch_check("bn_bwd_apply_kernel");
}

void bn_running_update(const float* stats, long rank_stride, int ranks, int batch, int c, int spatial, float momentum,
                       float* rmean, float* rvar, float* tracked, cudaStream_t stream) {
    bn_running_kernel<<<(c + 127) / 128, 128, 0, stream>>>(stats, rank_stride, ranks, batch, c, spatial, momentum,
                                                           rmean, rvar, tracked);
    launch_check("bn_running_kernel");
}

void bias_grad(const View& gv, int batch, const Grid& gr, float* ws, float* db, cudaStream_t stream) {
    const Split sp = choose_split(batch, gv.channels, gr);
    bias_partial_kernel<<<dim3(sp.cgroups, batch, sp.splits), kThreads, 0, stream>>>(gv.base, gv.pitch, gv.channels,
                                                                                   gr, sp.splits, ws);
    launch_check("bias_partial_kernel");
    float* per_image = ws + (size_t)batch * sp.splits * gv.channels;
    bias_image_kernel<<<(int)(((long)batch * gv.channels + 127) / 128), 128, 0, stream>>>(ws, batch, gv.channels,
                                                                                         sp.splits, per_image);
    launch_check("bias_image_kernel");
    bias_fold_kernel<<<(gv.channels + 127) / 128, 128, 0, stream>>>(per_image, batch, gv.channels, db);
    launch_check("bias_fold_kernel");
}

}  // namespace sy
