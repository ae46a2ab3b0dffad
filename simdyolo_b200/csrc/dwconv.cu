// Depthwise convolution (groups = channels) of the YOLO11 class branch (DWConv, DetectionHead cv3;
// HeadOperations.GroupedConv HeadOperations.cs:88-133), forward, data gradient and weight gradient,
// on CUDA cores: with one input channel per output channel the work is a 9-tap stencil per element,
// bound by HBM traffic, not a contraction for the tensor cores.
//
// A block covers one 32-row group (the BatchNorm partial-sum unit, never spanning two images) and 32
// channels: thread (row ty, channel quad tx) moves float4s, 8 lanes cover 128 contiguous bytes of a row.
// Per-channel reductions over the 32 rows go through shared memory in a fixed order (deterministic).
#include <algorithm>
#include <stdexcept>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kDwThreads = 256;   // 32 rows x 8 channel quads

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// y[m] = sum_t w[c][t] x[m + sign * shift_t] at interior rows; BatchNorm partials as BnEpilogue says.
__global__ void __launch_bounds__(kDwThreads) dw_conv_kernel(const float* x, int xpitch, long xrows, const float* w,
                                                             int taps, int sign, int c, Grid g, float* y, int ypitch,
                                                             const float* bias, const float* res, int rpitch,
                                                             BnEpilogue bn, int rnd) {
    __shared__ float w_s[32 * 9];
    __shared__ float red[32][33];
    __shared__ float red2[32][33];
    const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
    const int cb = blockIdx.y * 32;
    for (int i = threadIdx.x; i < 32 * taps; i += kDwThreads) {
        const int ch = cb + i / taps;
        w_s[i] = ch < c ? w[(long)ch * taps + i % taps] : 0.0f;
    }
    __syncthreads();
    const long grp = blockIdx.x;
    const long m = grp * 32 + ty;
    const long img = m / g.rows;
    const int r = (int)(m - img * g.rows);
    const bool inside = g.interior(r);
    const int cl = tx * 4, ch = cb + cl;
    const bool on = ch < c;   // c is a multiple of 4
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (inside && on) {
        for (int t = 0; t < taps; t++) {
            const int shift = taps == 9 ? (t / 3 - 1) * g.wp + (t % 3 - 1) : 0;
            const long src = m + sign * shift;
            if (src < 0 || src >= xrows) continue;
            const float4 xv = ld4(x + src * xpitch + ch);
            v[0] = fmaf(w_s[(cl + 0) * taps + t], xv.x, v[0]);
            v[1] = fmaf(w_s[(cl + 1) * taps + t], xv.y, v[1]);
            v[2] = fmaf(w_s[(cl + 2) * taps + t], xv.z, v[2]);
            v[3] = fmaf(w_s[(cl + 3) * taps + t], xv.w, v[3]);
        }
    }
    if (inside && on && bias) {
#pragma unroll
        for (int k = 0; k < 4; k++) v[k] += bias[ch + k];
    }
    if (inside && on && res) {
        const float4 rv = ld4(res + m * rpitch + ch);   // may alias y: read before the store below
        v[0] += rv.x;
        v[1] += rv.y;
        v[2] += rv.z;
        v[3] += rv.w;
    }
    float xh[4] = {0.f, 0.f, 0.f, 0.f};
    if (bn.grad_part && inside && on) {
        // v is g = dL/da of the BatchNorm layer (y, mean, inv, gamma, beta): store dz = g SiLU'(z)
        const float4 yv = ld4(bn.y + m * bn.y_pitch + ch);
        const float yy[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const long s = img * bn.channels + ch + k;
            xh[k] = (yy[k] - bn.mean[s]) * bn.inv[s];
            const float z = xh[k] * bn.gamma[ch + k] + bn.beta[ch + k];
            const float sg = 1.0f / (1.0f + __expf(-z));
            v[k] = v[k] * (sg + z * sg * (1.0f - sg));
        }
    }
    if (on) {
        float4 o = make_float4(v[0], v[1], v[2], v[3]);
        if (rnd) o = make_float4(tf32_rna(o.x), tf32_rna(o.y), tf32_rna(o.z), tf32_rna(o.w));
        *reinterpret_cast<float4*>(y + m * ypitch + ch) = o;
    }
    if (!bn.stats_part && !bn.grad_part) return;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        red[ty][cl + k] = v[k];
        red2[ty][cl + k] = v[k] * xh[k];
    }
    __shared__ float cnt_s;
    if (threadIdx.x == 0) cnt_s = 0.0f;
    __syncthreads();
    if (tx == 0 && inside) atomicAdd(&cnt_s, 1.0f);   // integer counts: exact in any order
    __syncthreads();
    if (threadIdx.x < 32 && cb + (int)threadIdx.x < c) {
        const int cc = threadIdx.x;
        const long pc = grp * bn.channels + cb + cc;
        if (bn.stats_part) {
            const float cnt = cnt_s;
            float sum = 0.0f;
            for (int i = 0; i < 32; i++) sum += red[i][cc];
            const float mean = cnt > 0.0f ? sum / cnt : 0.0f;
            float m2 = 0.0f;
            for (int i = 0; i < 32; i++) {
                const long mi = grp * 32 + i;
                if (g.interior((int)(mi - (mi / g.rows) * g.rows))) {
                    const float d = red[i][cc] - mean;
                    m2 += d * d;
                }
            }
            float* o = bn.stats_part + pc * 3;
            o[0] = cnt;
            o[1] = mean;
            o[2] = m2;
        } else {
            float s1 = 0.0f, s2 = 0.0f;
            for (int i = 0; i < 32; i++) {
                s1 += red[i][cc];
                s2 += red2[i][cc];
            }
            float* o = bn.grad_part + pc * 2;
            o[0] = s1;
            o[1] = s2;
        }
    }
}

// part[(blockIdx.x * c + ch) * taps + t] = sum over the block's rows of dy[m][ch] * x[m + shift_t][ch].
__global__ void __launch_bounds__(kDwThreads) dw_wgrad_kernel(const float* x, int xpitch, long xrows,
                                                              const float* dy, int dpitch, int taps, int c, Grid g,
                                                              long rows, long rows_per_block, float* part) {
    __shared__ float acc_s[32][32 * 9 + 1];
    const int tx = threadIdx.x & 7, ty = threadIdx.x >> 3;
    const int cb = blockIdx.y * 32, cl = tx * 4, ch = cb + cl;
    const long r0 = (long)blockIdx.x * rows_per_block;
    const long r1 = r0 + rows_per_block < rows ? r0 + rows_per_block : rows;
    float acc[9][4];
#pragma unroll
    for (int t = 0; t < 9; t++)
#pragma unroll
        for (int k = 0; k < 4; k++) acc[t][k] = 0.0f;
    if (ch < c)
        for (long m = r0 + ty; m < r1; m += 32) {
            const float4 d = ld4(dy + m * dpitch + ch);   // zero at halo rows
#pragma unroll
            for (int t = 0; t < 9; t++) {
                if (t >= taps) break;
                const int shift = taps == 9 ? (t / 3 - 1) * g.wp + (t % 3 - 1) : 0;
                const long src = m + shift;
                if (src < 0 || src >= xrows) continue;
                const float4 xv = ld4(x + src * xpitch + ch);
                acc[t][0] = fmaf(d.x, xv.x, acc[t][0]);
                acc[t][1] = fmaf(d.y, xv.y, acc[t][1]);
                acc[t][2] = fmaf(d.z, xv.z, acc[t][2]);
                acc[t][3] = fmaf(d.w, xv.w, acc[t][3]);
            }
        }
#pragma unroll
    for (int t = 0; t < 9; t++)
#pragma unroll
        for (int k = 0; k < 4; k++) acc_s[ty][(cl + k) * 9 + t] = acc[t][k];
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * taps; i += kDwThreads) {
        const int cc = i / taps, t = i % taps;
        if (cb + cc >= c) continue;
        float s = 0.0f;
        for (int j = 0; j < 32; j++) s += acc_s[j][cc * 9 + t];
        part[((long)blockIdx.x * c + cb + cc) * taps + t] = s;
    }
}

__global__ void dw_wgrad_fold_kernel(const float* part, int blocks, int c, int taps, float* dw) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= c * taps) return;
    float s = 0.0f;
    for (int b = 0; b < blocks; b++) s += part[(long)b * c * taps + i];
    dw[i] = s;
}

int wgrad_blocks(int c, long rows) {
    const int slabs = (c + 31) / 32;
    long want = std::max<long>(1, (148L * 4 + slabs - 1) / slabs);
    return (int)std::min<long>(want, std::max<long>(1, rows / 256));
}

}  // namespace

static void check_dw(const View& x, const View& y, int taps) {
    if (x.channels != y.channels || x.channels % 4 != 0 || x.pitch % 4 != 0 || y.pitch % 4 != 0)
        throw std::runtime_error("dw_conv: depthwise channels must match and be a multiple of 4");
    if (taps != 1 && taps != 9) throw std::runtime_error("dw_conv: kernel 1 or 3");
    if ((reinterpret_cast<uintptr_t>(x.base) & 15) || (reinterpret_cast<uintptr_t>(y.base) & 15))
        throw std::runtime_error("dw_conv: views not 16-byte aligned");
}

void dw_conv(const View& x, const float* w, int taps, int shift_sign, const Grid& g, const View& y, const BnEpilogue& bn,
             cudaStream_t stream, const float* bias, const View* residual, bool round_tf32) {
    check_dw(x, y, taps);
    if (y.rows % 32 != 0) throw std::runtime_error("dw_conv: rows must be whole 32-row groups");
    if ((bn.stats_part || bn.grad_part) && bn.channels < y.channels)
        throw std::runtime_error("dw_conv: BatchNorm partials must cover every channel");
    const dim3 grid((unsigned)(y.rows / 32), (unsigned)((y.channels + 31) / 32));
    if (residual && (residual->pitch % 4 != 0 || (reinterpret_cast<uintptr_t>(residual->base) & 15)))
        throw std::runtime_error("dw_conv: residual not 16-byte aligned");
    dw_conv_kernel<<<grid, kDwThreads, 0, stream>>>(x.base, x.pitch, x.rows, w, taps, shift_sign, y.channels, g, y.base,
                                                   y.pitch, bias, residual ? residual->base : nullptr,
                                                   residual ? residual->pitch : 0, bn, round_tf32 ? 1 : 0);
    launch_check("dw_conv_kernel");
}

size_t dw_wgrad_workspace_floats(int c, int taps, long rows) { return (size_t)wgrad_blocks(c, rows) * c * taps; }

void dw_wgrad(const View& x, const View& dy, int taps, const Grid& g, float* dw, float* ws, cudaStream_t stream) {
    check_dw(x, dy, taps);
    const int c = x.channels;
    const int blocks = wgrad_blocks(c, dy.rows);
    const long per = (dy.rows + blocks - 1) / blocks;
    dw_wgrad_kernel<<<dim3(blocks, (c + 31) / 32), kDwThreads, 0, stream>>>(x.base, x.pitch, x.rows, dy.base, dy.pitch,
                                                                          taps, c, g, dy.rows, per, ws);
    launch_check("dw_wgrad_kernel");
    dw_wgrad_fold_kernel<<<(c * taps + 127) / 128, 128, 0, stream>>>(ws, blocks, c, taps, dw);
    launch_check("dw_wgrad_fold_kernel");
}

}  // namespace sy
