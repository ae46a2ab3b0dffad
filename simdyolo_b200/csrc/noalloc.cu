// Allocation-free variant of the weight-gradient convolution (sy_cuda_conv2d_backward_filter_static).
//
// Some hosts cannot let a library call cudaMalloc: an embedding runtime or caching allocator that has
// already reserved all device memory for its own pool (a further cudaMalloc fails, or bypasses the pool's
// accounting so that its limits no longer hold), or a latency-bound serving loop that must not take the
// driver's allocation locks and implicit synchronisation in the middle of a request.  Those hosts bring
// their own input and output buffers; the only extra device memory this kernel needs, its split-K partial
// sums, lives in the fixed array below instead of a per-call allocation, and the call makes no other
// allocation (no cudaMalloc, cudaFree or allocating library routine).
//
// The array is a file-scope __device__ variable: every GPU that loads this library holds its
// kStaticScratchFloats floats (16 MiB) until the process exits.  In host code `g_static_scratch`
// names a host-side stand-in, not device memory, so its device address is looked up once per device
// with cudaGetSymbolAddress (with that device current) and passed to the kernels.  That lookup
// happens on the first call on each device.
//
// All calls share the one array and leave the previous call's partial sums in it; nothing has to
// start at zero because the kernel writes every partial sum it later reads (the error flag beside it
// is cleared at the start of every call).  Calls that overlap on the GPU (different streams or host
// threads at the same time) race on the array and must be serialised by the caller.  Every call waits
// for its stream to finish before it returns, to read the kernels' error flag.
#include <mutex>
#include <stdexcept>
#include <string>

#include "session.h"

namespace {

constexpr size_t kStaticScratchFloats = size_t(4) << 20;  // 16 MiB of float32 partial sums
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_static_scratch[kStaticScratchFloats];
static __device__ __align__(256) int g_static_err[4];

struct StaticScratch {
    float* scratch = nullptr;
    int* err = nullptr;
};
StaticScratch g_addr[kMaxDevices];
std::mutex g_addr_mu;

// Device addresses of the static arrays for the current device (looked up once per device).
StaticScratch static_scratch(int device) {
    std::lock_guard<std::mutex> lock(g_addr_mu);
    StaticScratch& s = g_addr[device];
    if (!s.scratch) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            throw sy::SyError(SY_ERR_DEVICE, std::string("cudaGetSymbolAddress(scratch): ") + cudaGetErrorString(e));
        void* q = nullptr;
        e = cudaGetSymbolAddress(&q, g_static_err);
        if (e != cudaSuccess)
            throw sy::SyError(SY_ERR_DEVICE, std::string("cudaGetSymbolAddress(err): ") + cudaGetErrorString(e));
        s.scratch = static_cast<float*>(p);
        s.err = static_cast<int*>(q);
    }
    return s;
}

}  // namespace

extern "C" sy_status sy_cuda_conv2d_backward_filter_static(int32_t device, const float* x_padded_device,
                                                           const float* dy_padded_device, int32_t n, int32_t ic,
                                                           int32_t oc, int32_t h, int32_t w, int32_t k,
                                                           float* dw_device, void* stream) {
    try {
        if (!x_padded_device || !dy_padded_device || !dw_device || n < 1 || ic < 1 || oc < 1 || h < 1 || w < 1 ||
            !(k == 1 || k == 3))
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "conv2d_backward_filter_static: bad arguments");
        if (oc > 256)
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "conv2d_backward_filter_static: more than 256 output channels");
        if (ic > 4096)
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE, "conv2d_backward_filter_static: more than 4096 input channels");
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count || device >= kMaxDevices)
            throw sy::SyError(SY_ERR_INVALID_ARGUMENT, "invalid CUDA device");
        cudaError_t e = cudaSetDevice(device);
        if (e != cudaSuccess) throw sy::SyError(SY_ERR_DEVICE, cudaGetErrorString(e));
        const sy::Grid g = sy::make_grid(h, w);
        const long rows = (long)n * g.rows;
        const int taps = k * k;
        const size_t need = sy::wgrad_workspace_floats(ic, oc, taps, rows);
        if (need > kStaticScratchFloats)
            throw sy::SyError(SY_ERR_UNSUPPORTED_SHAPE,
                              "conv2d_backward_filter_static: needs " + std::to_string(need) +
                                  " scratch floats, the static scratch holds " + std::to_string(kStaticScratchFloats));
        const StaticScratch s = static_scratch(device);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        e = cudaMemsetAsync(s.err, 0, sizeof(int), st);
        if (e != cudaSuccess) throw sy::SyError(SY_ERR_DEVICE, cudaGetErrorString(e));
        const sy::View vx{const_cast<float*>(x_padded_device), (ic + 3) / 4 * 4, ic, rows};
        const sy::View vdy{const_cast<float*>(dy_padded_device), (oc + 3) / 4 * 4, oc, rows};
        sy::conv_tc_wgrad(vx, vdy, taps, g, dw_device, s.scratch, s.err, st);
        int flag = 0;
        e = cudaMemcpyAsync(&flag, s.err, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) throw sy::SyError(SY_ERR_DEVICE, cudaGetErrorString(e));
        if (flag) throw sy::SyError(SY_ERR_DEVICE, "wgrad kernel wait limit exceeded");
        return SY_OK;
    } catch (const sy::SyError& ex) {
        sy::set_last_error(ex.what());
        return ex.code;
    } catch (const std::exception& ex) {
        sy::set_last_error(ex.what());
        return SY_ERR_DEVICE;
    }
}
