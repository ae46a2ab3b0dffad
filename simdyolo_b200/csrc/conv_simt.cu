// SIMT implicit-GEMM convolution (any stride), layout conversion and small backbone kernels.
//
// conv_simt_forward serves the frozen backbone's stride-2 3x3 convs and the 3-channel stem
// (PtModel.cs Conv with folded BN bias and fused SiLU, PtModel.cs:128-144); the stride-1 convs
// run on the tcgen05 kernels in conv_tc.cu.  maxpool5_padded is SPPF's MaxPool2d(5, 1, 2);
// upsample2_padded is nn.Upsample(scale 2, nearest) written into a concat slice.
#include <algorithm>
#include <atomic>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

constexpr int BM = 64, BN = 64, BK = 16;

struct SimtParams {
    const float* in;
    int in_pitch, ic;
    Grid gin;
    const float* w;  // [oc][taps][ic]
    int oc, k, stride, taps;
    float* out;
    int out_pitch;
    Grid gout;
    int batch;
    long m_total;    // batch * ho * wo
    const float* bias;
    int silu;
    const float* residual;
    int res_pitch;
};

__global__ void __launch_bounds__(256) conv_simt_kernel(const SimtParams p) {
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int tid = threadIdx.x;
    const long m0 = (long)blockIdx.x * BM;
    const int n0 = blockIdx.y * BN;
    const int K = p.taps * p.ic;
    const int pix_img = p.gout.h * p.gout.w;

    // loader coordinates: each thread loads 4 consecutive k of one row (A) / one output channel (B)
    const int lrow = tid >> 2, lk = (tid & 3) * 4;
    long in_row_base = -1;
    {
        long m = m0 + lrow;
        if (m < p.m_total) {
            int b = (int)(m / pix_img), rem = (int)(m - (long)b * pix_img);
            int oy = rem / p.gout.w, ox = rem - oy * p.gout.w;
            int pad = p.k / 2;
            // padded input coordinate of tap (0,0): oy*s - pad + 1
            int py = oy * p.stride - pad + 1, px = ox * p.stride - pad + 1;
            in_row_base = (long)b * p.gin.rows + (long)py * p.gin.wp + px;
        }
    }
    const int wn = n0 + lrow;

    const int ty = tid >> 4, tx = tid & 15;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += BK) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int kk = k0 + lk + j;
            float av = 0.0f, bv = 0.0f;
            if (kk < K) {
                int t = kk / p.ic, c = kk - t * p.ic;
                if (in_row_base >= 0) {
                    int ky = t / p.k, kx = t - ky * p.k;
                    av = p.in[(in_row_base + (long)ky * p.gin.wp + kx) * p.in_pitch + c];
                }
                if (wn < p.oc) bv = p.w[(long)wn * K + kk];
            }
            As[lk + j][lrow] = av;
            Bs[lk + j][lrow] = bv;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                a[i] = As[kk][ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        long m = m0 + ty * 4 + i;
        if (m >= p.m_total) continue;
        int b = (int)(m / pix_img), rem = (int)(m - (long)b * pix_img);
        int oy = rem / p.gout.w, ox = rem - oy * p.gout.w;
        long orow = (long)b * p.gout.rows + p.gout.row(oy, ox);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            int n = n0 + tx * 4 + j;
            if (n >= p.oc) continue;
            float v = acc[i][j];
            if (p.bias) v += p.bias[n];
            if (p.silu) v = silu_f(v);
            if (p.residual) v += p.residual[orow * p.res_pitch + n];
            p.out[orow * p.out_pitch + n] = v;
        }
    }
}

__global__ void nchw_to_padded_kernel(const float* src, int batch, int c, Grid g, float* dst, int pitch) {
    long total = (long)batch * c * g.h * g.w;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int x = (int)(i % g.w);
        long r = i / g.w;
        int y = (int)(r % g.h);
        r /= g.h;
        int ch = (int)(r % c);
        int b = (int)(r / c);
        dst[((long)b * g.rows + g.row(y, x)) * pitch + ch] = src[i];
    }
}

__global__ void padded_to_nchw_kernel(const float* src, int pitch, int batch, int c, Grid g, float* dst) {
    long total = (long)batch * c * g.h * g.w;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int x = (int)(i % g.w);
        long r = i / g.w;
        int y = (int)(r % g.h);
        r /= g.h;
        int ch = (int)(r % c);
        int b = (int)(r / c);
        dst[i] = src[((long)b * g.rows + g.row(y, x)) * pitch + ch];
    }
}

// ImagePreprocessor.Letterbox at identity scale (YoloDetector.cs:445-514): value / 255.
__global__ void rgb_to_padded_kernel(const uint8_t* rgb, int batch, int size, Grid g, float* dst, int pitch) {
    long total = (long)batch * size * size;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int x = (int)(i % size);
        long r = i / size;
        int y = (int)(r % size);
        int b = (int)(r / size);
        const uint8_t* px = rgb + i * 3;
        float* d = dst + ((long)b * g.rows + g.row(y, x)) * pitch;
        d[0] = __fdiv_rn((float)px[0], 255.0f);
        d[1] = __fdiv_rn((float)px[1], 255.0f);
        d[2] = __fdiv_rn((float)px[2], 255.0f);
    }
}

__global__ void weights_fwd_kernel(const float* w, int oc, int ic, int taps, int kpad, float* dst) {
    long total = (long)oc * taps * kpad;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int c = (int)(i % kpad);
        long r = i / kpad;
        int t = (int)(r % taps);
        int o = (int)(r / taps);
        dst[i] = c < ic ? w[((long)o * ic + c) * taps + t] : 0.0f;
    }
}

__global__ void weights_dgrad_kernel(const float* w, int oc, int ic, int taps, int kpad_o, float* dst) {
    long total = (long)ic * taps * kpad_o;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int o = (int)(i % kpad_o);
        long r = i / kpad_o;
        int t = (int)(r % taps);
        int c = (int)(r / taps);
        dst[i] = o < oc ? w[((long)o * ic + c) * taps + t] : 0.0f;
    }
}

__global__ void weights_ohwi_kernel(const float* w, int oc, int ic, int taps, float* dst) {
    long total = (long)oc * taps * ic;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int c = (int)(i % ic);
        long r = i / ic;
        int t = (int)(r % taps);
        int o = (int)(r / taps);
        dst[i] = w[((long)o * ic + c) * taps + t];
    }
}

// MaxPool2d(5, stride 1, padding 2); padded positions never win.
__global__ void maxpool5_kernel(const float* in, int in_pitch, float* out, int out_pitch, int c, int batch, Grid g) {
    long total = (long)batch * g.h * g.w * c;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int ch = (int)(i % c);
        long r = i / c;
        int x = (int)(r % g.w);
        r /= g.w;
        int y = (int)(r % g.h);
        int b = (int)(r / g.h);
        float m = -INFINITY;
        for (int dy = -2; dy <= 2; dy++) {
            int yy = y + dy;
            if (yy < 0 || yy >= g.h) continue;
            for (int dx = -2; dx <= 2; dx++) {
                int xx = x + dx;
                if (xx < 0 || xx >= g.w) continue;
                m = fmaxf(m, in[((long)b * g.rows + g.row(yy, xx)) * in_pitch + ch]);
            }
        }
        out[((long)b * g.rows + g.row(y, x)) * out_pitch + ch] = m;
    }
}

__global__ void upsample2_kernel(const float* in, int in_pitch, Grid gin, float* out, int out_pitch, Grid gout, int c,
                                 int batch) {
    long total = (long)batch * gout.h * gout.w * c;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int ch = (int)(i % c);
        long r = i / c;
        int x = (int)(r % gout.w);
        r /= gout.w;
        int y = (int)(r % gout.h);
        int b = (int)(r / gout.h);
        out[((long)b * gout.rows + gout.row(y, x)) * out_pitch + ch] =
            in[((long)b * gin.rows + gin.row(y / 2, x / 2)) * in_pitch + ch];
    }
}

int blocks_for(long n) { return (int)std::min<long>(65535L * 16, std::max<long>(1, (n + 255) / 256)); }

}  // namespace

static std::atomic<long long> g_launches{0};

void launch_check(const char* what) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

void conv_simt_forward(const View& in, const Grid& gin, const float* w_ohwi, int oc, int k, int stride,
                       const View& out, const Grid& gout, int batch, const ConvEpilogue& ep, cudaStream_t stream) {
    SimtParams p;
    p.in = in.base;
    p.in_pitch = in.pitch;
    p.ic = in.channels;
    p.gin = gin;
    p.w = w_ohwi;
    p.oc = oc;
    p.k = k;
    p.stride = stride;
    p.taps = k * k;
    p.out = out.base;
    p.out_pitch = out.pitch;
    p.gout = gout;
    p.batch = batch;
    p.m_total = (long)batch * gout.h * gout.w;
    p.bias = ep.bias;
    p.silu = ep.silu;
    p.residual = ep.residual;
    p.res_pitch = ep.res_pitch;
    dim3 grid((unsigned)((p.m_total + BM - 1) / BM), (unsigned)((oc + BN - 1) / BN));
    conv_simt_kernel<<<grid, 256, 0, stream>>>(p);
    launch_check("conv_simt_kernel");
}

void nchw_to_padded(const float* src, int batch, int c, const Grid& g, const View& dst, cudaStream_t stream) {
    long n = (long)batch * c * g.h * g.w;
    nchw_to_padded_kernel<<<blocks_for(n), 256, 0, stream>>>(src, batch, c, g, dst.base, dst.pitch);
    launch_check("nchw_to_padded_kernel");
}

void padded_to_nchw(const View& src, int batch, int c, const Grid& g, float* dst, cudaStream_t stream) {
    long n = (long)batch * c * g.h * g.w;
    padded_to_nchw_kernel<<<blocks_for(n), 256, 0, stream>>>(src.base, src.pitch, batch, c, g, dst);
    launch_check("padded_to_nchw_kernel");
}

void rgb_to_padded(const uint8_t* rgb, int batch, int size, const Grid& g, const View& dst, cudaStream_t stream) {
    long n = (long)batch * size * size;
    rgb_to_padded_kernel<<<blocks_for(n), 256, 0, stream>>>(rgb, batch, size, g, dst.base, dst.pitch);
    launch_check("rgb_to_padded_kernel");
}

void weights_fwd_layout(const float* oihw, int oc, int ic, int taps, int kpad, float* dst, cudaStream_t stream) {
    long n = (long)oc * taps * kpad;
    weights_fwd_kernel<<<blocks_for(n), 256, 0, stream>>>(oihw, oc, ic, taps, kpad, dst);
    launch_check("weights_fwd_kernel");
}

void weights_dgrad_layout(const float* oihw, int oc, int ic, int taps, int kpad_o, float* dst, cudaStream_t stream) {
    long n = (long)ic * taps * kpad_o;
    weights_dgrad_kernel<<<blocks_for(n), 256, 0, stream>>>(oihw, oc, ic, taps, kpad_o, dst);
    launch_check("weights_dgrad_kernel");
}

void weights_ohwi(const float* oihw, int oc, int ic, int taps, float* dst, cudaStream_t stream) {
    long n = (long)oc * taps * ic;
    weights_ohwi_kernel<<<blocks_for(n), 256, 0, stream>>>(oihw, oc, ic, taps, dst);
    launch_check("weights_ohwi_kernel");
}

void maxpool5_padded(const View& in, const View& out, int batch, const Grid& g, cudaStream_t stream) {
    long n = (long)batch * g.h * g.w * in.channels;
    maxpool5_kernel<<<blocks_for(n), 256, 0, stream>>>(in.base, in.pitch, out.base, out.pitch, in.channels, batch, g);
    launch_check("maxpool5_kernel");
}

void upsample2_padded(const View& in, const Grid& gin, const View& out, const Grid& gout, int batch,
                      cudaStream_t stream) {
    long n = (long)batch * gout.h * gout.w * in.channels;
    upsample2_kernel<<<blocks_for(n), 256, 0, stream>>>(in.base, in.pitch, gin, out.base, out.pitch, gout,
                                                        in.channels, batch);
    launch_check("upsample2_kernel");
}

}  // namespace sy
