// Layout conversions and the small memory-bound kernels of the frozen trunk.
//
// nchw_to_padded / padded_to_nchw convert between the reference layout and the padded
// channels-last layout; rgb_to_phase is the identity-scale letterbox (YoloDetector.cs:445-514)
// written as the stem's parity-split input; weights_*_layout build the K-major operands of the
// tensor-core convs; maxpool5_padded is SPPF's MaxPool2d(5, 1, 2); upsample2_padded is
// nn.Upsample(scale 2, nearest) written into a concat slice.  launch_check lives here too.
#include <algorithm>
#include <atomic>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

namespace {

__global__ void nchw_to_padded_kernel(const float* src, int batch, int c, Grid g, float* dst, int pitch, int rnd) {
    long total = (long)batch * c * g.h * g.w;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int x = (int)(i % g.w);
        long r = i / g.w;
        int y = (int)(r % g.h);
        r /= g.h;
        int ch = (int)(r % c);
        int b = (int)(r / c);
        dst[((long)b * g.rows + g.row(y, x)) * pitch + ch] = rnd ? tf32_rna(src[i]) : src[i];
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

__global__ void weights_fwd_kernel(const float* w, int oc, int ic, int taps, int kpad, float* dst, int rnd) {
    long total = (long)oc * taps * kpad;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        int c = (int)(i % kpad);
        long r = i / kpad;
        int t = (int)(r % taps);
        int o = (int)(r / taps);
        const float v = c < ic ? w[((long)o * ic + c) * taps + t] : 0.0f;
        dst[i] = rnd ? tf32_rna(v) : v;
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

// blockIdx.y = job; the forward layout then the data-gradient layout of that job's weights.
__global__ void weights_layout_batch_kernel(const WeightLayoutJob* table, int rnd) {
    const WeightLayoutJob jb = table[blockIdx.y];
    const long nf = (long)jb.oc * jb.taps * jb.kpad_in, nd = (long)jb.ic * jb.taps * jb.kpad_out;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < nf + nd; i += (long)gridDim.x * blockDim.x) {
        if (i < nf) {
            const int c = (int)(i % jb.kpad_in);
            const long r = i / jb.kpad_in;
            const int t = (int)(r % jb.taps), o = (int)(r / jb.taps);
            const float v = c < jb.ic ? jb.oihw[((long)o * jb.ic + c) * jb.taps + t] : 0.0f;
            jb.fwd[i] = rnd ? tf32_rna(v) : v;
        } else {
            const long k = i - nf;
            const int o = (int)(k % jb.kpad_out);
            const long r = k / jb.kpad_out;
            const int t = (int)(r % jb.taps), c = (int)(r / jb.taps);
            const float v = o < jb.oc ? jb.oihw[((long)o * jb.ic + c) * jb.taps + t] : 0.0f;
            jb.dgrad[k] = rnd ? tf32_rna(v) : v;
        }
    }
}

// Vector of V consecutive channels (V = 4 when channels and pitches allow float4 access).
template <int V>
struct Vec {
    float v[V];
};
template <int V>
__device__ __forceinline__ Vec<V> load_vec(const float* p) {
    Vec<V> r;
    if constexpr (V == 4) {
        const float4 t = *reinterpret_cast<const float4*>(p);
        r.v[0] = t.x;
        r.v[1] = t.y;
        r.v[2] = t.z;
        r.v[3] = t.w;
    } else {
        r.v[0] = *p;
    }
    return r;
}
template <int V>
__device__ __forceinline__ void store_vec(float* p, const Vec<V>& r) {
    if constexpr (V == 4)
        *reinterpret_cast<float4*>(p) = make_float4(r.v[0], r.v[1], r.v[2], r.v[3]);
    else
        *p = r.v[0];
}

// MaxPool2d(5, stride 1, padding 2); padded positions never win.
// SPPF max pool 5x5 / stride 1 / pad 2 (PtModel.cs SPPF): blockIdx.x = image * h + y (one output pixel
// row), blockIdx.y and the threads over (x, channel vector); 32-bit index math.
template <int V>
__global__ void maxpool5_kernel(const float* in, int in_pitch, float* out, int out_pitch, int c, int batch, Grid g,
                                float inv_cv) {
    const int cv = c / V;
    const int b = blockIdx.x / g.h, y = blockIdx.x - b * g.h;
    const long base = (long)b * g.rows;
    const int n = g.w * cv;
    for (int k = blockIdx.y * blockDim.x + threadIdx.x; k < n; k += gridDim.y * blockDim.x) {
        const int x = fast_div(k, inv_cv), ch = (k - x * cv) * V;
        Vec<V> m;
        for (int q = 0; q < V; q++) m.v[q] = -INFINITY;
        for (int dy = -2; dy <= 2; dy++) {
            const int yy = y + dy;
            if (yy < 0 || yy >= g.h) continue;
            for (int dx = -2; dx <= 2; dx++) {
                const int xx = x + dx;
                if (xx < 0 || xx >= g.w) continue;
                const Vec<V> t = load_vec<V>(in + (base + g.row(yy, xx)) * in_pitch + ch);
                for (int q = 0; q < V; q++) m.v[q] = fmaxf(m.v[q], t.v[q]);
            }
        }
        store_vec<V>(out + (base + g.row(y, x)) * out_pitch + ch, m);
    }
}

// Nearest 2x upsample into a (concatenation) slice: blockIdx.x = image * gout.h + y, blockIdx.y and the
// threads over (x, channel vector).
template <int V>
__global__ void upsample2_kernel(const float* in, int in_pitch, Grid gin, float* out, int out_pitch, Grid gout, int c,
                                 int batch, float inv_cv) {
    const int cv = c / V;
    const int b = blockIdx.x / gout.h, y = blockIdx.x - b * gout.h;
    const float* src = in + ((long)b * gin.rows + gin.row(y / 2, 0)) * in_pitch;
    float* dst = out + ((long)b * gout.rows + gout.row(y, 0)) * out_pitch;
    const int n = gout.w * cv;
    for (int k = blockIdx.y * blockDim.x + threadIdx.x; k < n; k += gridDim.y * blockDim.x) {
        const int x = fast_div(k, inv_cv), ch = (k - x * cv) * V;
        store_vec<V>(dst + (long)x * out_pitch + ch, load_vec<V>(src + (long)(x / 2) * in_pitch + ch));
    }
}

// x / 255 correctly rounded for an integer x in [0, 255]: the product with the rounded reciprocal
// is within one unit in the last place, and one FMA residual step (Markstein's correction) rounds
// it to the IEEE quotient; checked against IEEE division for every byte value.
__device__ __forceinline__ float byte_over_255(uint32_t v) {
    const float x = (float)v;
    const float r = 1.0f / 255.0f;
    const float q = __fmul_rn(x, r);
    const float e = __fmaf_rn(-q, 255.0f, x);
    return __fmaf_rn(e, r, q);
}

// Stem weights by value: kernel parameters live in the constant bank, so every FMA below takes
// its weight as a constant operand (no shared-memory traffic).
template <int OC>
struct StemParams {
    float w[OC * 27];   // OIHW [oc][3][3][3]
    float b[OC];
};

// One thread per output pixel of the stem: 27 inputs (u8 / 255) x OC outputs, bias, SiLU.  Grid (pixel
// blocks of one image, images): the pixel's row and column come from a float reciprocal of the output width
// (exact for fewer than 2^22 pixels an image) instead of 64-bit divisions, and each input row's address is
// formed once.
template <int OC>
__global__ void __launch_bounds__(256) stem_conv_kernel(const uint8_t* const* rgb_ref, int size,
                                                        const StemParams<OC> sp, float* out, int out_pitch, Grid gout,
                                                        PhaseOut phase, int has_phase, int rnd, float inv_wo) {
    const uint8_t* const rgb = *rgb_ref;
    const int ho = gout.h, wo = gout.w;
    const int rem = blockIdx.x * blockDim.x + threadIdx.x;
    if (rem >= ho * wo) return;
    const int b = blockIdx.y;
    const int oy = __float2int_rd(((float)rem + 0.5f) * inv_wo), ox = rem - oy * wo;
    float in[27];
#pragma unroll
    for (int ky = 0; ky < 3; ky++) {
        const int iy = 2 * oy + ky - 1;
        const bool row_ok = iy >= 0 && iy < size;
        const uint8_t* rp = rgb + ((long)b * size + (row_ok ? iy : 0)) * size * 3;
#pragma unroll
        for (int kx = 0; kx < 3; kx++) {
            const int ix = 2 * ox + kx - 1;
            const bool ok = row_ok && ix >= 0 && ix < size;
            const uint8_t* p = rp + (ok ? ix : 0) * 3;
#pragma unroll
            for (int c = 0; c < 3; c++) in[c * 9 + ky * 3 + kx] = ok ? byte_over_255(p[c]) : 0.0f;
        }
    }
    float acc[OC];
#pragma unroll
    for (int o = 0; o < OC; o++) {
        float s = 0.0f;
#pragma unroll
        for (int q = 0; q < 27; q++) s = fmaf(sp.w[o * 27 + q], in[q], s);
        acc[o] = silu_fast(s + sp.b[o]);
        if (rnd) acc[o] = tf32_rna(acc[o]);
    }
    if (out) {
        float* dst = out + ((long)b * gout.rows + gout.row(oy, ox)) * out_pitch;
#pragma unroll
        for (int o = 0; o < OC; o += 4)
            *reinterpret_cast<float4*>(dst + o) = make_float4(acc[o], acc[o + 1], acc[o + 2], acc[o + 3]);
    }
    if (has_phase) {
        const int py = oy + 1, px = ox + 1;
        float* pd = phase.base + (((py & 1) * 2 + (px & 1)) * phase.plane_rows + (long)b * phase.consumer.rows +
                                  (long)(py >> 1) * phase.consumer.wp + (px >> 1)) *
                                     phase.pitch;
#pragma unroll
        for (int o = 0; o < OC; o += 4)
            *reinterpret_cast<float4*>(pd + o) = make_float4(acc[o], acc[o + 1], acc[o + 2], acc[o + 3]);
    }
}

// Identity-scale letterbox written straight into the stem's parity-split input (PhaseOut layout),
// 4 floats per pixel (r, g, b, 0).
__global__ void rgb_to_phase_kernel(const uint8_t* rgb, int batch, int size, PhaseOut dst) {
    const long total = (long)batch * size * size;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int b = (int)(i / ((long)size * size));
        const int rem = (int)(i - (long)b * size * size);
        const int py = rem / size + 1, px = rem - (rem / size) * size + 1;
        const uint8_t* s = rgb + i * 3;
        const long row = ((py & 1) * 2 + (px & 1)) * dst.plane_rows + (long)b * dst.consumer.rows +
                         (long)(py >> 1) * dst.consumer.wp + (px >> 1);
        *reinterpret_cast<float4*>(dst.base + row * dst.pitch) =
            make_float4(__fdiv_rn((float)s[0], 255.0f), __fdiv_rn((float)s[1], 255.0f),
                        __fdiv_rn((float)s[2], 255.0f), 0.0f);
    }
}

// Bounded-wait check (wait_limit_selftest): the shape of every pipelined kernel here, with the producer
// missing.  Warp 0 allocates TMEM, warp 1 waits on an mbarrier that nothing arrives on, gives up after
// `spins` polls and records `code`; then every warp reaches the closing barrier and warp 0 frees the TMEM,
// as the conv kernels do after a timed-out wait.  Nothing asynchronous is in flight.
__global__ void wait_limit_selftest_kernel(uint32_t spins, int code, int* err) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    if (warp == 0) {
        tmem_alloc(&tmem_slot, 32);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 32) mbar_wait_limit(&bar, 0, err, code, spins);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_slot, 32);
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

// Grouped conv weights [oc][ic / groups][taps] <-> block-diagonal dense [oc][ic][taps]: output channel o
// belongs to group o / (oc / groups), which reads input channels [g ic / groups, (g + 1) ic / groups).
__global__ void grouped_to_dense_kernel(const float* w, int oc, int ic, int groups, int taps, float* dense) {
    const int icg = ic / groups, ocg = oc / groups;
    const long total = (long)oc * ic * taps;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i % taps);
        const long oc_c = i / taps;
        const int c = (int)(oc_c % ic), o = (int)(oc_c / ic);
        const int g = o / ocg;
        dense[i] = (c / icg == g) ? w[((long)o * icg + (c - g * icg)) * taps + t] : 0.0f;
    }
}

__global__ void dense_to_grouped_kernel(const float* dense, int oc, int ic, int groups, int taps, float* w) {
    const int icg = ic / groups, ocg = oc / groups;
    const long total = (long)oc * icg * taps;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i % taps);
        const long o_cl = i / taps;
        const int cl = (int)(o_cl % icg), o = (int)(o_cl / icg);
        w[i] = dense[((long)o * ic + (o / ocg) * icg + cl) * taps + t];
    }
}

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }
void add_launches(long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

void nchw_to_padded(const float* src, int batch, int c, const Grid& g, const View& dst, cudaStream_t stream,
                    bool round_tf32) {
    long n = (long)batch * c * g.h * g.w;
    nchw_to_padded_kernel<<<blocks_for(n), 256, 0, stream>>>(src, batch, c, g, dst.base, dst.pitch, round_tf32 ? 1 : 0);
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

void weights_fwd_layout(const float* oihw, int oc, int ic, int taps, int kpad, float* dst, cudaStream_t stream,
                        bool round_tf32) {
    long n = (long)oc * taps * kpad;
    weights_fwd_kernel<<<blocks_for(n), 256, 0, stream>>>(oihw, oc, ic, taps, kpad, dst, round_tf32 ? 1 : 0);
    launch_check("weights_fwd_kernel");
}

void weights_dgrad_layout(const float* oihw, int oc, int ic, int taps, int kpad_o, float* dst, cudaStream_t stream) {
    long n = (long)ic * taps * kpad_o;
    weights_dgrad_kernel<<<blocks_for(n), 256, 0, stream>>>(oihw, oc, ic, taps, kpad_o, dst);
    launch_check("weights_dgrad_kernel");
}

void weights_layout_batch(const WeightLayoutJob* table_device, int jobs, long max_elems, cudaStream_t stream,
                          bool round_tf32) {
    if (jobs < 1 || jobs > 65535) throw std::runtime_error("weights_layout_batch: job count");
    const int bx = (int)std::min<long>(64, std::max<long>(1, (max_elems + 255) / 256));
    weights_layout_batch_kernel<<<dim3(bx, jobs), 256, 0, stream>>>(table_device, round_tf32 ? 1 : 0);
    launch_check("weights_layout_batch_kernel");
}

void maxpool5_padded(const View& in, const View& out, int batch, const Grid& g, cudaStream_t stream) {
    const bool vec = in.channels % 4 == 0 && in.pitch % 4 == 0 && out.pitch % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(in.base) & 15) == 0 && (reinterpret_cast<uintptr_t>(out.base) & 15) == 0;
    const int cv = vec ? in.channels / 4 : in.channels;
    const int n = g.w * cv;
    if (n >= (1 << 22)) throw std::runtime_error("maxpool5: map too large");
    const dim3 grid((unsigned)(batch * g.h), (unsigned)((n + 255) / 256));
    if (vec)
        maxpool5_kernel<4><<<grid, 256, 0, stream>>>(in.base, in.pitch, out.base, out.pitch, in.channels, batch, g,
                                                     1.0f / (float)cv);
    else
        maxpool5_kernel<1><<<grid, 256, 0, stream>>>(in.base, in.pitch, out.base, out.pitch, in.channels, batch, g,
                                                     1.0f / (float)cv);
    launch_check("maxpool5_kernel");
}

void upsample2_padded(const View& in, const Grid& gin, const View& out, const Grid& gout, int batch,
                      cudaStream_t stream) {
    const bool vec = in.channels % 4 == 0 && in.pitch % 4 == 0 && out.pitch % 4 == 0 &&
                     (reinterpret_cast<uintptr_t>(in.base) & 15) == 0 && (reinterpret_cast<uintptr_t>(out.base) & 15) == 0;
    const int cv = vec ? in.channels / 4 : in.channels;
    const int n = gout.w * cv;
    if (n >= (1 << 22)) throw std::runtime_error("upsample2: map too large");
    const dim3 grid((unsigned)(batch * gout.h), (unsigned)((n + 255) / 256));
    if (vec)
        upsample2_kernel<4><<<grid, 256, 0, stream>>>(in.base, in.pitch, gin, out.base, out.pitch, gout, in.channels,
                                                      batch, 1.0f / (float)cv);
    else
        upsample2_kernel<1><<<grid, 256, 0, stream>>>(in.base, in.pitch, gin, out.base, out.pitch, gout, in.channels,
                                                      batch, 1.0f / (float)cv);
    launch_check("upsample2_kernel");
}

template <int OC>
static void launch_stem(const uint8_t* const* rgb_ref, int batch, int size, const float* w_host, const float* b_host,
                        const View& out, const Grid& gout, const PhaseOut& ph, int hp, cudaStream_t stream, int rnd) {
    StemParams<OC> sp;
    for (int i = 0; i < OC * 27; i++) sp.w[i] = w_host[i];
    for (int i = 0; i < OC; i++) sp.b[i] = b_host[i];
    const dim3 grid((unsigned)((gout.h * gout.w + 255) / 256), (unsigned)batch);
    stem_conv_kernel<OC><<<grid, 256, 0, stream>>>(rgb_ref, size, sp, out.base, out.pitch, gout, ph, hp, rnd,
                                                   1.0f / (float)gout.w);
}

void stem_conv(const uint8_t* const* rgb_ref, int batch, int size, const float* w_host, const float* bias_host, int oc,
               const View& out, const Grid& gout, const PhaseOut* phase, cudaStream_t stream, bool round_tf32) {
    if (out.pitch % 4 != 0 || (phase && phase->pitch % 4 != 0))
        throw std::runtime_error("stem_conv: pitches must be multiples of 4");
    if (!out.base && !phase) throw std::runtime_error("stem_conv: no output");
    if ((long)gout.h * gout.w >= (1L << 22) || batch > 65535) throw std::runtime_error("stem_conv: image too large");
    const PhaseOut ph = phase ? *phase : PhaseOut{};
    const int hp = phase ? 1 : 0;
    const int rnd = round_tf32 ? 1 : 0;
    switch (oc) {
        case 16: launch_stem<16>(rgb_ref, batch, size, w_host, bias_host, out, gout, ph, hp, stream, rnd); break;
        case 32: launch_stem<32>(rgb_ref, batch, size, w_host, bias_host, out, gout, ph, hp, stream, rnd); break;
        case 48: launch_stem<48>(rgb_ref, batch, size, w_host, bias_host, out, gout, ph, hp, stream, rnd); break;
        case 64: launch_stem<64>(rgb_ref, batch, size, w_host, bias_host, out, gout, ph, hp, stream, rnd); break;
        default: throw std::runtime_error("stem_conv: output channels must be 16, 32, 48 or 64");
    }
    launch_check("stem_conv_kernel");
}

__global__ void tf32_split_kernel(const float* src, int pitch, int channels, long rows, float* big, float* small) {
    const long total = rows * channels;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const long r = i / channels;
        const long idx = r * pitch + (i - r * channels);
        const float x = src[idx], b = tf32_rna(x);
        big[idx] = b;
        small[idx] = x - b;
    }
}

void tf32_split(const View& src, float* big, float* small, cudaStream_t stream) {
    const long n = src.rows * src.channels;
    tf32_split_kernel<<<blocks_for(n), 256, 0, stream>>>(src.base, src.pitch, src.channels, src.rows, big, small);
    launch_check("tf32_split_kernel");
}

void wait_limit_selftest(uint32_t spins, int code, int* err, cudaStream_t stream) {
    if (spins < 1 || spins > kSpinLimit) throw std::runtime_error("wait_limit_selftest: spins out of range");
    wait_limit_selftest_kernel<<<1, 64, 0, stream>>>(spins, code, err);
    launch_check("wait_limit_selftest_kernel");
}

void rgb_to_phase(const uint8_t* rgb, int batch, int size, const PhaseOut& dst, cudaStream_t stream) {
    if (dst.pitch != 4) throw std::runtime_error("rgb_to_phase: stem input pitch must be 4");
    const long n = (long)batch * size * size;
    rgb_to_phase_kernel<<<blocks_for(n), 256, 0, stream>>>(rgb, batch, size, dst);
    launch_check("rgb_to_phase_kernel");
}

void grouped_to_dense(const float* w, int oc, int ic, int groups, int taps, float* dense, cudaStream_t stream) {
    const long total = (long)oc * ic * taps;
    grouped_to_dense_kernel<<<(int)std::min<long>(148L * 8, (total + 255) / 256), 256, 0, stream>>>(w, oc, ic, groups,
                                                                                                 taps, dense);
    launch_check("grouped_to_dense_kernel");
}

void dense_to_grouped(const float* dense, int oc, int ic, int groups, int taps, float* w, cudaStream_t stream) {
    const long total = (long)oc * (ic / groups) * taps;
    dense_to_grouped_kernel<<<(int)std::min<long>(148L * 8, (total + 255) / 256), 256, 0, stream>>>(dense, oc, ic,
                                                                                                 groups, taps, w);
    launch_check("dense_to_grouped_kernel");
}

}  // namespace sy
