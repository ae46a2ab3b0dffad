// Multi-head self-attention of the YOLO11 C2PSA block (PtModel.cs Attention, :429-439), part of the
// frozen trunk's forward pass, on CUDA cores: at the P5 map (20 x 20 tokens at 640 pixels) each
// (image, head) is a 400 x 400 score matrix with 32-wide keys, a few GFLOP for a whole batch.
//
// One thread per query token, 64 queries per block; keys and values stream through shared memory in
// tiles of 32 tokens with the running-maximum form of the softmax (scores scaled, exponentials
// rescaled when the maximum grows, one division at the end), so any token count fits.
#include <cmath>
#include <stdexcept>

#include "kernels.h"

namespace sy {

namespace {

constexpr int kKD = 32, kHD = 64;   // key_dim, head_dim (C2PSA: heads = channels / 64)
constexpr int kQ = 64, kKT = 32;    // queries per block, keys per tile

__device__ __forceinline__ long token_row(int t, int b, const Grid& g) {
    const int y = t / g.w, x = t - y * g.w;
    return (long)b * g.rows + (long)(y + 1) * g.wp + (x + 1);
}

__global__ void __launch_bounds__(kQ) attention_kernel(const float* qkv, int qpitch, Grid g, float scale, float* att,
                                                        int apitch, float* vout, int vpitch) {
    __shared__ __align__(16) float k_s[kKT][kKD];
    __shared__ __align__(16) float v_s[kKT][kHD];
    const int b = blockIdx.z, h = blockIdx.y, n = g.h * g.w;
    const int qi = blockIdx.x * kQ + threadIdx.x;
    const bool live = qi < n;
    const int base = h * (2 * kKD + kHD);   // this head's [q | k | v] channels
    const long qrow = live ? token_row(qi, b, g) : 0;
    float q[kKD], acc[kHD];
#pragma unroll
    for (int d = 0; d < kKD; d++) q[d] = live ? qkv[qrow * qpitch + base + d] : 0.0f;
#pragma unroll
    for (int d = 0; d < kHD; d++) acc[d] = 0.0f;
    if (live)
        for (int d = 0; d < kHD; d++) vout[qrow * vpitch + h * kHD + d] = qkv[qrow * qpitch + base + 2 * kKD + d];
    float m = -INFINITY, l = 0.0f;
    for (int j0 = 0; j0 < n; j0 += kKT) {
        __syncthreads();
        // k and v of a token are adjacent: channels base + kKD ... base + 2 kKD + kHD
        for (int i = threadIdx.x; i < kKT * (kKD + kHD); i += kQ) {
            const int j = i / (kKD + kHD), d = i - j * (kKD + kHD);
            const float val = j0 + j < n ? qkv[token_row(j0 + j, b, g) * qpitch + base + kKD + d] : 0.0f;
            if (d < kKD) k_s[j][d] = val;
            else v_s[j][d - kKD] = val;
        }
        __syncthreads();
        if (!live) continue;
        const int cnt = min(kKT, n - j0);
        float s[kKT];
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < kKT; j++) {
            float dot = 0.0f;
#pragma unroll
            for (int d = 0; d < kKD; d += 4) {
                const float4 kv = *reinterpret_cast<const float4*>(&k_s[j][d]);
                dot = fmaf(q[d], kv.x, dot);
                dot = fmaf(q[d + 1], kv.y, dot);
                dot = fmaf(q[d + 2], kv.z, dot);
                dot = fmaf(q[d + 3], kv.w, dot);
            }
            s[j] = j < cnt ? dot * scale : -INFINITY;
            tmax = fmaxf(tmax, s[j]);
        }
        const float mnew = fmaxf(m, tmax);
        const float corr = expf(m - mnew);   // 0 on the first tile (m = -inf)
        l *= corr;
#pragma unroll
        for (int d = 0; d < kHD; d++) acc[d] *= corr;
        for (int j = 0; j < cnt; j++) {
            const float p = expf(s[j] - mnew);
            l += p;
#pragma unroll
            for (int d = 0; d < kHD; d += 4) {
                const float4 vv = *reinterpret_cast<const float4*>(&v_s[j][d]);
                acc[d] = fmaf(p, vv.x, acc[d]);
                acc[d + 1] = fmaf(p, vv.y, acc[d + 1]);
                acc[d + 2] = fmaf(p, vv.z, acc[d + 2]);
                acc[d + 3] = fmaf(p, vv.w, acc[d + 3]);
            }
        }
        m = mnew;
    }
    if (live) {
        const float inv = 1.0f / l;
        for (int d = 0; d < kHD; d++) att[qrow * apitch + h * kHD + d] = acc[d] * inv;
    }
}

}  // namespace

void attention(const View& qkv, int batch, const Grid& g, int heads, int key_dim, int head_dim, float scale,
               const View& att, const View& v_out, cudaStream_t stream) {
    if (key_dim != kKD || head_dim != kHD)
        throw std::runtime_error("attention: key_dim 32 and head_dim 64 expected (C2PSA heads = channels / 64)");
    if (qkv.channels < heads * (2 * kKD + kHD) || att.channels < heads * kHD || v_out.channels < heads * kHD)
        throw std::runtime_error("attention: channel counts");
    const int n = g.h * g.w;
    const dim3 grid((unsigned)((n + kQ - 1) / kQ), (unsigned)heads, (unsigned)batch);
    attention_kernel<<<grid, kQ, 0, stream>>>(qkv.base, qkv.pitch, g, scale, att.base, att.pitch, v_out.base,
                                             v_out.pitch);
    launch_check("attention_kernel");
}

}  // namespace sy
