// Training-mode BatchNorm with per-image statistics, fused with SiLU, forward and backward
// (HeadOperations.BatchNorm HeadOperations.cs:153-193, HeadOperations.Silu :198-221), running
// statistics (HeadOperations.cs:164-165, num_batches_tracked DetectionHead.cs:154) and the bias
// gradient of the final conv (HeadOperations.cs:66).
//
// Each image normalises with its own mean / variance over H x W, exactly like the reference's
// batch-of-one convs, so a batch of B images needs B x C statistics.  Reductions are written per
// (image, channel) and folded over images in image order, so results do not depend on timing.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kWarps = 8;

// One block per (channel group of 32, image); lane = channel, warps stride over interior pixels.
__global__ void __launch_bounds__(256) bn_stats_kernel(const float* y, int pitch, int c, Grid g, float* stats) {
    __shared__ float red[kWarps][32];
    __shared__ float mean_s[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y;
    const int n = g.h * g.w;
    const float* base = y + (long)b * g.rows * pitch + ch;
    float s = 0.0f;
    if (ch < c)
        for (int p = warp; p < n; p += kWarps) {
            int yy = p / g.w, xx = p - yy * g.w;
            s += base[(long)g.row(yy, xx) * pitch];
        }
    red[warp][lane] = s;
    __syncthreads();
    if (warp == 0) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        mean_s[lane] = t / n;
    }
    __syncthreads();
    const float mean = mean_s[lane];
    float v = 0.0f;
    if (ch < c)
        for (int p = warp; p < n; p += kWarps) {
            int yy = p / g.w, xx = p - yy * g.w;
            float d = base[(long)g.row(yy, xx) * pitch] - mean;
            v += d * d;
        }
    __syncthreads();
    red[warp][lane] = v;
    __syncthreads();
    if (warp == 0 && ch < c) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        stats[((long)b * c + ch) * 2 + 0] = mean;
        stats[((long)b * c + ch) * 2 + 1] = t / n;
    }
}

__global__ void bn_apply_kernel(const float* y, int ypitch, const float* stats, const float* gamma, const float* beta,
                                float eps, int c, int batch, Grid g, float* a, int apitch) {
    const long total = (long)batch * g.rows * c;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c);
        const long row = i / c;
        const int b = (int)(row / g.rows), r = (int)(row - (long)b * g.rows);
        float out = 0.0f;
        if (g.interior(r)) {
            const float mean = stats[((long)b * c + ch) * 2], var = stats[((long)b * c + ch) * 2 + 1];
            const float inv = 1.0f / sqrtf(var + eps);
            const float z = (y[row * ypitch + ch] - mean) * inv * gamma[ch] + beta[ch];
            out = silu_f(z);
        }
        a[row * apitch + ch] = out;
    }
}

// Per (channel group, image): sum dz and sum dz * xhat where dz is the gradient at the BN output.
__global__ void __launch_bounds__(256) bn_bwd_reduce_kernel(const float* y, int ypitch, const float* gr, int gpitch,
                                                            const float* stats, const float* gamma, const float* beta,
                                                            float eps, int c, Grid g, float* red_out) {
    __shared__ float r1[kWarps][32], r2[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y;
    const int n = g.h * g.w;
    float s = 0.0f, sx = 0.0f;
    if (ch < c) {
        const float mean = stats[((long)b * c + ch) * 2], var = stats[((long)b * c + ch) * 2 + 1];
        const float inv = 1.0f / sqrtf(var + eps), ga = gamma[ch], be = beta[ch];
        const long base = (long)b * g.rows;
        for (int p = warp; p < n; p += kWarps) {
            int yy = p / g.w, xx = p - yy * g.w;
            const long row = base + g.row(yy, xx);
            const float xh = (y[row * ypitch + ch] - mean) * inv;
            const float z = xh * ga + be;
            const float sg = 1.0f / (1.0f + __expf(-z));
            const float dz = gr[row * gpitch + ch] * (sg + z * sg * (1.0f - sg));
            s += dz;
            sx += dz * xh;
        }
    }
    r1[warp][lane] = s;
    r2[warp][lane] = sx;
    __syncthreads();
    if (warp == 0 && ch < c) {
        float t1 = 0.0f, t2 = 0.0f;
        for (int w = 0; w < kWarps; w++) {
            t1 += r1[w][lane];
            t2 += r2[w][lane];
        }
        red_out[((long)b * c + ch) * 2 + 0] = t1;
        red_out[((long)b * c + ch) * 2 + 1] = t2;
    }
}

// dy = gamma * inv / n * (n * dz - sum dz - xhat * sum dz xhat)  (HeadOperations.cs:185-189)
__global__ void bn_bwd_apply_kernel(const float* y, int ypitch, const float* gr, int gpitch, const float* stats,
                                    const float* red, const float* gamma, const float* beta, float eps, int c,
                                    int batch, Grid g, float* dy, int dpitch) {
    const long total = (long)batch * g.rows * c;
    const float n = (float)(g.h * g.w);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int ch = (int)(i % c);
        const long row = i / c;
        const int b = (int)(row / g.rows), r = (int)(row - (long)b * g.rows);
        float out = 0.0f;
        if (g.interior(r)) {
            const long k = ((long)b * c + ch) * 2;
            const float mean = stats[k], var = stats[k + 1];
            const float inv = 1.0f / sqrtf(var + eps), ga = gamma[ch];
            const float xh = (y[row * ypitch + ch] - mean) * inv;
            const float z = xh * ga + beta[ch];
            const float sg = 1.0f / (1.0f + __expf(-z));
            const float dz = gr[row * gpitch + ch] * (sg + z * sg * (1.0f - sg));
            const float scale = ga * inv / n;
            out = scale * (n * dz - red[k] - xh * red[k + 1]);
        }
        dy[row * dpitch + ch] = out;
    }
}

// dgamma[ch] += sum_b red[b][ch][1]; dbeta[ch] += sum_b red[b][ch][0], images in order.
__global__ void bn_param_grad_kernel(const float* red, int batch, int c, float* dgamma, float* dbeta) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= c) return;
    float g = dgamma[ch], bt = dbeta[ch];
    for (int b = 0; b < batch; b++) {
        g += red[((long)b * c + ch) * 2 + 1];
        bt += red[((long)b * c + ch) * 2 + 0];
    }
    dgamma[ch] = g;
    dbeta[ch] = bt;
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

__global__ void __launch_bounds__(256) bias_partial_kernel(const float* gr, int pitch, int c, Grid g, float* part) {
    __shared__ float red[kWarps][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int ch = blockIdx.x * 32 + lane, b = blockIdx.y;
    const int n = g.h * g.w;
    float s = 0.0f;
    if (ch < c)
        for (int p = warp; p < n; p += kWarps) {
            int yy = p / g.w, xx = p - yy * g.w;
            s += gr[((long)b * g.rows + g.row(yy, xx)) * pitch + ch];
        }
    red[warp][lane] = s;
    __syncthreads();
    if (warp == 0 && ch < c) {
        float t = 0.0f;
        for (int w = 0; w < kWarps; w++) t += red[w][lane];
        part[(long)b * c + ch] = t;
    }
}

__global__ void bias_fold_kernel(const float* part, int batch, int c, float* db) {
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= c) return;
    float s = db[ch];
    for (int b = 0; b < batch; b++) s += part[(long)b * c + ch];
    db[ch] = s;
}

int blocks_for(long n) { return (int)std::min<long>(148L * 64, std::max<long>(1, (n + 255) / 256)); }

}  // namespace

void bn_stats(const View& y, int batch, const Grid& g, float* stats, cudaStream_t stream) {
    dim3 grid((y.channels + 31) / 32, batch);
    bn_stats_kernel<<<grid, 256, 0, stream>>>(y.base, y.pitch, y.channels, g, stats);
    launch_check("bn_stats_kernel");
}

void bn_silu_apply(const View& y, const float* stats, const float* gamma, const float* beta, float eps, int batch,
                   const Grid& g, const View& a, cudaStream_t stream) {
    long n = (long)batch * g.rows * y.channels;
    bn_apply_kernel<<<blocks_for(n), 256, 0, stream>>>(y.base, y.pitch, stats, gamma, beta, eps, y.channels, batch, g,
                                                       a.base, a.pitch);
    launch_check("bn_apply_kernel");
}

void bn_silu_backward(const View& y, const View& gv, const float* stats, const float* gamma, const float* beta,
                      float eps, int batch, const Grid& gr, float* red, const View& dy, float* dgamma, float* dbeta,
                      cudaStream_t stream) {
    const int c = y.channels;
    dim3 grid((c + 31) / 32, batch);
    bn_bwd_reduce_kernel<<<grid, 256, 0, stream>>>(y.base, y.pitch, gv.base, gv.pitch, stats, gamma, beta, eps, c, gr,
                                                   red);
    launch_check("bn_bwd_reduce_kernel");
    long n = (long)batch * gr.rows * c;
    bn_bwd_apply_kernel<<<blocks_for(n), 256, 0, stream>>>(y.base, y.pitch, gv.base, gv.pitch, stats, red, gamma,
                                                           beta, eps, c, batch, gr, dy.base, dy.pitch);
    launch_check("bn_bwd_apply_kernel");
    bn_param_grad_kernel<<<(c + 127) / 128, 128, 0, stream>>>(red, batch, c, dgamma, dbeta);
    launch_check("bn_param_grad_kernel");
}

void bn_running_update(const float* stats, long rank_stride, int ranks, int batch, int c, int spatial, float momentum,
                       float* rmean, float* rvar, float* tracked, cudaStream_t stream) {
    bn_running_kernel<<<(c + 127) / 128, 128, 0, stream>>>(stats, rank_stride, ranks, batch, c, spatial, momentum,
                                                           rmean, rvar, tracked);
    launch_check("bn_running_kernel");
}

void bias_grad(const View& gv, int batch, const Grid& gr, float* part, float* db, cudaStream_t stream) {
    dim3 grid((gv.channels + 31) / 32, batch);
    bias_partial_kernel<<<grid, 256, 0, stream>>>(gv.base, gv.pitch, gv.channels, gr, part);
    launch_check("bias_partial_kernel");
    bias_fold_kernel<<<(gv.channels + 127) / 128, 128, 0, stream>>>(part, batch, gv.channels, db);
    launch_check("bias_fold_kernel");
}

}  // namespace sy
