// Shared device helpers for the sm_100a kernels: error plumbing, mbarrier / TMA / tcgen05 PTX
// wrappers, and the deterministic transcendental functions used by the task-aligned assigner.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdio>

namespace sy {

// ------------------------------------------------------------------------------------------
// Padded activation layout.  Every feature map of H x W pixels with C channels is stored
// channels-last with a one-pixel zero halo: image b, padded pixel (py, px) with
// py in [0, H+2), px in [0, W+2) lives at row b * rows_per_image + py * (W+2) + px.
// rows_per_image = round_up((H+2)*(W+2), 128) so that a 128-row GEMM tile never spans two
// images; the rows past (H+2)*(W+2) ("dead rows") and the halo stay zero.
// ------------------------------------------------------------------------------------------
struct Grid {
    int h, w;             // interior size
    int wp;               // w + 2
    int rows;             // rows per image (multiple of 128)
    __host__ __device__ int row(int y, int x) const { return (y + 1) * wp + (x + 1); }
    __host__ __device__ bool interior(int r) const {
        int py = r / wp, px = r - py * wp;
        return py >= 1 && py <= h && px >= 1 && px <= w;
    }
};

inline Grid make_grid(int h, int w) {
    Grid g;
    g.h = h;
    g.w = w;
    g.wp = w + 2;
    int used = (h + 2) * (w + 2);
    g.rows = (used + 127) / 128 * 128;
    return g;
}

// ------------------------------------------------------------------------------------------
// Deterministic math: the same published methods as the CPU checker, with explicit
// round-to-nearest intrinsics so that nvcc never contracts or reorders them.
//   exp : Cody-Waite reduction by ln 2 (two-part ln 2 split), Taylor series to r^13, exact 2^k.
//   atan: reduction to [0,1] (atan(x) = pi/2 - atan(1/x)) and to |t| <= tan(pi/12)
//         (atan(x) = pi/6 + atan((x*sqrt3-1)/(x+sqrt3))), odd Taylor series to t^25.
// Results are double values rounded once to float.
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ double det_exp_d(double x) {
    if (x != x) return x;
    x = fmin(fmax(x, -200.0), 200.0);
    const double LOG2E = 1.4426950408889634074;
    const double LN2_HI = 6.93147180369123816490e-01;
    const double LN2_LO = 1.90821492927058770002e-10;
    double k = rint(__dmul_rn(x, LOG2E));
    double r = __fma_rn(-k, LN2_HI, x);
    r = __fma_rn(-k, LN2_LO, r);
    double p = 1.0 / 6227020800.0;
    p = __fma_rn(p, r, 1.0 / 479001600.0);
    p = __fma_rn(p, r, 1.0 / 39916800.0);
    p = __fma_rn(p, r, 1.0 / 3628800.0);
    p = __fma_rn(p, r, 1.0 / 362880.0);
    p = __fma_rn(p, r, 1.0 / 40320.0);
    p = __fma_rn(p, r, 1.0 / 5040.0);
    p = __fma_rn(p, r, 1.0 / 720.0);
    p = __fma_rn(p, r, 1.0 / 120.0);
    p = __fma_rn(p, r, 1.0 / 24.0);
    p = __fma_rn(p, r, 1.0 / 6.0);
    p = __fma_rn(p, r, 0.5);
    p = __fma_rn(p, r, 1.0);
    p = __fma_rn(p, r, 1.0);
    long long e = (long long)k + 1023;
    double scale = __longlong_as_double(e << 52);
    return __dmul_rn(p, scale);
}

__device__ __forceinline__ float det_expf(float x) { return __double2float_rn(det_exp_d((double)x)); }

__device__ __forceinline__ double det_atan_d(double x) {
    if (x != x) return x;
    const double PI_2 = 1.57079632679489661923;
    const double PI_6 = 0.52359877559829887308;
    const double SQRT3 = 1.73205080756887729353;
    const double TAN_PI_12 = 0.26794919243112270647;
    bool negative = x < 0;
    if (negative) x = -x;
    bool inverted = false;
    if (x > 1.0) {
        inverted = true;
        x = __ddiv_rn(1.0, x);
    }
    double offset = 0.0;
    if (x > TAN_PI_12) {
        x = __ddiv_rn(__dadd_rn(__dmul_rn(x, SQRT3), -1.0), __dadd_rn(x, SQRT3));
        offset = PI_6;
    }
    double t2 = __dmul_rn(x, x);
    double p = 1.0 / 25.0;
    p = __fma_rn(p, t2, -1.0 / 23.0);
    p = __fma_rn(p, t2, 1.0 / 21.0);
    p = __fma_rn(p, t2, -1.0 / 19.0);
    p = __fma_rn(p, t2, 1.0 / 17.0);
    p = __fma_rn(p, t2, -1.0 / 15.0);
    p = __fma_rn(p, t2, 1.0 / 13.0);
    p = __fma_rn(p, t2, -1.0 / 11.0);
    p = __fma_rn(p, t2, 1.0 / 9.0);
    p = __fma_rn(p, t2, -1.0 / 7.0);
    p = __fma_rn(p, t2, 1.0 / 5.0);
    p = __fma_rn(p, t2, -1.0 / 3.0);
    double result = __fma_rn(__dmul_rn(x, t2), p, x);
    result = __dadd_rn(result, offset);
    if (inverted) result = __dadd_rn(PI_2, -result);
    return negative ? -result : result;
}

__device__ __forceinline__ float det_atanf(float x) { return __double2float_rn(det_atan_d((double)x)); }

// HeadOperations.Sigmoid (HeadOperations.cs:222) with det_expf.
__device__ __forceinline__ float det_sigmoid(float v) {
    if (v >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, det_expf(-v)));
    float e = det_expf(v);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

// MathF.Pow(x, 6) as a double product rounded once.
__device__ __forceinline__ float det_pow6(float x) {
    double t = (double)x;
    double t2 = __dmul_rn(t, t);
    double t4 = __dmul_rn(t2, t2);
    return __double2float_rn(__dmul_rn(t4, t2));
}

__device__ __forceinline__ float silu_f(float v) { return v / (1.0f + __expf(-v)); }
// The same with the fast division (within 2 ulp; v / inf = -0 for the very negative v)
__device__ __forceinline__ float silu_fast(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

// x rounded to the nearest TF32 value (10 explicit mantissa bits, ties away from zero).  The tensor
// core reads an FP32 operand of a kind::tf32 MMA by dropping its low 13 mantissa bits, which shrinks
// every product by about 2^-10 on average; operands stored already rounded make that error unbiased.
__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// ------------------------------------------------------------------------------------------
// Warp / block reductions
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------------------------------
// mbarrier / TMA / tcgen05 wrappers (PTX ISA 8.7, sm_100a)
// ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after `limit` polls and reports through *err (never traps).
// The limit is far above any legitimate wait (each try_wait already suspends for a while).
constexpr uint32_t kSpinLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, int* err, int code, uint32_t limit) {
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (++n > limit) {
            if (err) atomicExch(err, code);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
    return mbar_wait_limit(bar, parity, err, code, kSpinLimit);
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2D tiled TMA load into this CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// 2D tiled TMA store from this CTA's shared memory (bulk-group completion).  x, y >= 0 always.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// this thread's committed bulk stores have finished reading their shared-memory sources
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// this thread's committed bulk stores are complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on an mbarrier when all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// floor(n / d) for 0 <= n < 2^22 from inv = 1.0f / d (rounded): (n + 1/2) / d lies at least 1 / (2d)
// from an integer, and the float error is below (n + 1/2) 2^-23 / d, so rounding down is exact.
__device__ __forceinline__ int fast_div(int n, float inv) { return __float2int_rd(((float)n + 0.5f) * inv); }

// Warp-wide forms: the whole (converged) warp executes them and elect.sync picks the lane that issues
// the MMA / commit (always the same lane for a full warp, so commits track that lane's MMAs).  Issuing
// from warp-uniform code is much cheaper than from a single diverged lane.
__device__ __forceinline__ void mma_tf32_elect(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit_elect(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
}

// Named CTA barrier over `threads` threads (whole warps).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 bit, 32 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptors (sm_100 version bits).
//   K-major, SWIZZLE_128B (layout type 2): rows of 128 B (32 fp32 along K), 16 B chunks XOR-ed
//     with (row % 8), 8-row groups 1024 B apart (SBO); LBO unused.  Matches TMA SWIZZLE_128B.
//   MN-major fp32/tf32, SWIZZLE_128B_BASE32B (layout type 1): the only MN-major layout tf32
//     accepts.  Each K row holds 128 B (32 elements) along MN, 32 B chunks XOR-ed with (row % 4),
//     4-row K groups SBO apart, successive 128 B MN blocks LBO apart.  Matches TMA
//     SWIZZLE_128B_ATOM_32B.
constexpr uint32_t kLayoutSw128 = 2, kLayoutSw128Base32 = 1;
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version for sm_100
    d |= (uint64_t)layout << 61;
    return d;
}

// Instruction descriptor: D f32, A/B tf32, M = 128, given N and operand majors.
__host__ __device__ constexpr uint32_t idesc_tf32(int n, int a_mn_major, int b_mn_major) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)a_mn_major << 15) | ((uint32_t)b_mn_major << 16) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

}  // namespace sy
