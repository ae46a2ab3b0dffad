// Fused optimizer over the flat head-parameter buffer.
//
// SGD-momentum restates TrainingParameter.Update (src/SimdYolo.Training/TrainingParameter.cs:21-43):
//   v = momentum * v + g / images + decay * w;  w = w - lr * v
// with decay only on conv weights (DetectionHead.cs:59-60), the whole update skipped for a
// parameter without gradient (the box branch when no image had a positive, :24), and non-finite
// results reported (:40).  AdamW follows torch.optim.AdamW (decoupled decay, bias correction);
// the reference has no AdamW.  Gradients are cleared after the update.
#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

struct OptParams {
    int optimizer;
    float* w;
    float* v;
    float* v2;
    float* g;
    const ParamSegment* segs;
    int nsegs;
    const int* has_grad;   // per group (device)
    const int* steps;      // per group, AdamW steps including this one (device)
    float lr, momentum, wd, beta1, beta2, eps, inv_images;
    int* nonfinite;
};

__global__ void optimizer_kernel(OptParams p) {
    const int s = blockIdx.y;
    const ParamSegment seg = p.segs[s];
    if (!p.has_grad[seg.group]) return;
    const float decay = seg.decay ? p.wd : 0.0f;
    bool bad = false;
    if (p.optimizer == 0) {
        for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < seg.length; i += (long)gridDim.x * blockDim.x) {
            const long k = seg.offset + i;
            const float w = p.w[k];
            const float v = p.v[k] * p.momentum + p.g[k] * p.inv_images + w * decay;
            const float u = w - p.lr * v;
            bad |= !(fabsf(v) <= 3.402823466e38f) || !(fabsf(u) <= 3.402823466e38f);
            p.v[k] = v;
            p.w[k] = u;
            p.g[k] = 0.0f;
        }
    } else {
        const int step = p.steps[seg.group];
        const float bc1 = 1.0f - powf(p.beta1, (float)step), bc2 = 1.0f - powf(p.beta2, (float)step);
        const float step_size = p.lr / bc1, bc2_sqrt = sqrtf(bc2);
        for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < seg.length; i += (long)gridDim.x * blockDim.x) {
            const long k = seg.offset + i;
            const float g = p.g[k] * p.inv_images;
            float w = p.w[k] * (1.0f - p.lr * decay);
            const float m = p.beta1 * p.v[k] + (1.0f - p.beta1) * g;
            const float v = p.beta2 * p.v2[k] + (1.0f - p.beta2) * g * g;
            const float denom = sqrtf(v) / bc2_sqrt + p.eps;
            w = w - step_size * (m / denom);
            bad |= !(fabsf(w) <= 3.402823466e38f) || !(fabsf(m) <= 3.402823466e38f) || !(fabsf(v) <= 3.402823466e38f);
            p.v[k] = m;
            p.v2[k] = v;
            p.w[k] = w;
            p.g[k] = 0.0f;
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicExch(p.nonfinite, 1);
}

__global__ void finite_kernel(const float* v, long n, int* flag) {
    bool bad = false;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        bad |= !(fabsf(v[i]) <= 3.402823466e38f);
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicExch(flag, 1);
}

__global__ void abs_sum_kernel(const float* v, long n, double* part) {
    double s = 0.0;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        s += fabs((double)v[i]);
    s = warp_sum_d(s);
    __shared__ double red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int w = 0; w < 8; w++) t += red[w];
        part[blockIdx.x] = t;
    }
}

}  // namespace

void abs_sum_partials(const float* v, long n, double* part, cudaStream_t stream) {
    abs_sum_kernel<<<kAbsSumBlocks, 256, 0, stream>>>(v, n, part);
    launch_check("abs_sum_kernel");
}

void optimizer_step(int optimizer, float* params, float* vel, float* vel2, float* grad, const ParamSegment* segs,
                    int nsegs, const int* group_has_grad, const int* group_steps, float lr, float momentum, float wd,
                    float beta1, float beta2, float adam_eps, float inv_images, int* nonfinite, cudaStream_t stream) {
    OptParams p;
    p.optimizer = optimizer;
    p.w = params;
    p.v = vel;
    p.v2 = vel2;
    p.g = grad;
    p.segs = segs;
    p.nsegs = nsegs;
    p.has_grad = group_has_grad;
    p.steps = group_steps;
    p.lr = lr;
    p.momentum = momentum;
    p.wd = wd;
    p.beta1 = beta1;
    p.beta2 = beta2;
    p.eps = adam_eps;
    p.inv_images = inv_images;
    p.nonfinite = nonfinite;
    optimizer_kernel<<<dim3(16, nsegs), 256, 0, stream>>>(p);
    launch_check("optimizer_kernel");
}

void check_finite(const float* v, long n, int* flag, cudaStream_t stream) {
    int blocks = (int)std::min<long>(148L * 8, std::max<long>(1, (n + 255) / 256));
    finite_kernel<<<blocks, 256, 0, stream>>>(v, n, flag);
    launch_check("finite_kernel");
}

}  // namespace sy
