// tcgen05 implicit-GEMM convolutions for sm_100a (TF32 inputs, FP32 accumulation in TMEM).
//
// Forward / data-gradient kernel (conv_fwd_tc): persistent, one CTA tile of T 128-row sub-tiles of
// the padded activation matrix per iteration.  Warp 0 issues TMA loads (A: haloed row regions x 32
// channels of the input, read by every tap of a tap group at its row offset; B: N rows x 32 k of the
// K-major weights), warp 1 performs every mbarrier wait of the MMA side, warps 2-3 issue tcgen05.mma
// (K = 8 per instruction) into double-buffered TMEM accumulators, and warps 4.. drain the other
// accumulator (bias, SiLU, shortcut, halo masking, BatchNorm partials) while the next tile
// accumulates.
//
// Weight-gradient kernel (conv_wgrad_tc): split-K over pixel rows.  Both operands are read in
// their natural channels-last layout and fed to the tensor cores as MN-major (transposed)
// matrices: A = input channels (4 blocks of 32, each one (tap, channel block)), B = output-grad
// channels; K = pixel rows.  Partial sums go to a workspace that a second kernel reduces.
//
// Replaces the reference's im2col + GEMM (HeadOperations.cs:39-47 forward, :58-70 wgrad / dgrad,
// TrainingMatMul.cs:14-49) and the Vulkan SGEMM shader it dispatches to (shaders/gemm.comp).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <stdexcept>
#include <string>

#include "kernels.h"

namespace sy {

// ------------------------------------------------------------------ tensor-map creation
static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p)
            throw std::runtime_error("cuTensorMapEncodeTiled unavailable");
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// 2D fp32 tensor map: inner dimension `inner` elements (contiguous), `outer` rows `pitch_floats`
// apart; box (box_inner, box_outer); out-of-bounds elements read as zero.  K-major operands use
// the 128-byte swizzle, MN-major (transposed) tf32 operands the 128-byte swizzle of 32-byte atoms.
static CUtensorMap make_map_2d(const float* base, long inner, long outer, long pitch_floats, int box_inner,
                               int box_outer, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (pitch_floats * 4) % 16 != 0)
        throw std::runtime_error("tensor map base / pitch not 16-byte aligned");
    CUtensorMap map;
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)pitch_floats * 4};
    cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = get_encode()(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return map;
}

static int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    }
    return n;
}

// ------------------------------------------------------------------ forward / dgrad kernel
// A CTA tile is T consecutive 128-row sub-tiles (M = 128 T output rows).  The taps are split into
// groups whose row shifts lie close together (one group for a stride-1 conv; one per parity plane
// for a stride-2 conv).  For each 32-channel chunk and group, one haloed A region
//   rows [m0 + lo_g, m0 + lo_g + 128 T + span_g)
// is loaded with 64-row TMA boxes, and every tap of the group reads it at its own row offset: the
// MMA descriptor start moves by whole 128-byte rows, which the SWIZZLE_128B layout allows because
// both TMA and the tensor core swizzle on absolute shared-memory address bits.  Each input row is
// then fetched (128 T + span) / (128 T) times instead of once per tap.  Weights stay resident in
// shared memory when they fit, else they stream per (tap, chunk) through their own ring.
constexpr int kMaxGroups = 4;
constexpr int kBoxRows = 64;                 // rows per A TMA box (8 KB)

struct FwdParams {
    int num_tiles;       // CTA tiles of 128 T rows
    int sub_tiles;       // 128-row sub-tiles of output in total
    int T;
    int kchunks, kpad;
    int ngroups;
    int g_lo[kMaxGroups];      // first A row of the group's region, relative to the tile's first row
    int g_boxes[kMaxGroups];   // 64-row boxes loaded per region
    int g_ntaps[kMaxGroups];
    int tap_t[9];              // weight tap of the j-th tap (group order)
    int tap_off[9];            // A row offset of the j-th tap inside its group's region
    int taps;
    int n;          // MMA N (multiple of 16, <= 256)
    int n_valid;    // channels stored
    int n0;         // first weight row of this launch
    int a_stages, a_stage_bytes;
    int b_stages;   // 0: all weights resident
    int b_pack;     // streamed weights: (tap, chunk) blocks per ring stage (few large stages move faster)
    int b_region_bytes;
    int nacc;       // TMEM accumulator stages
    int ksplit;     // 2: (T = 1) MMA warp w sums K steps 2w, 2w+1 into its own accumulator, the epilogue adds both
    int acc_cols;   // TMEM columns per sub-tile accumulator
    int alloc_cols;
    float* out;
    int out_pitch;
    int out_tma;         // 1 (trunk epilogue): the output leaves through per-warp shared-memory tiles and TMA stores
    int stage_bytes;     // shared memory of those tiles (4 KB per epilogue warp), before the A ring
    const float* bias;
    const float* residual;
    int res_pitch;
    int silu;
    int mask;
    Grid grid;
    // optional parity-split copy of the output (input of a stride-2 consumer, see kernels.h)
    float* phase;
    int phase_pitch;
    int phase_wp;        // consumer output grid: padded width
    int phase_rows;      // consumer output grid: rows per image
    long phase_stride;   // rows between parity planes (batch * phase_rows)
    const float* pre;    // added to the accumulator first (3xTF32 passes)
    int pre_pitch;
    int rnd;             // stored outputs rounded to the nearest TF32 (operands of the next TF32 conv)
    BnEpilogue bn;       // BatchNorm partials (see kernels.h)
    int* err;
    int sub_per_img;     // 128-row sub-tiles per image (grid.rows / 128)
    float inv_wp;        // 1 / grid.wp, rounded
};

// MMA issue, as measured on B200 for M128 x N64 x K8 tf32 MMAs: a warp that issues from warp-uniform
// code (elect.sync) sustains one MMA per ~53 cycles, one lane alone in a diverged branch one per ~75;
// two such warps (alternate 128-row sub-tiles, or with one sub-tile per tile alternate pairs of K
// steps, in separate accumulators) reach the tensor core's rate at N = 64 (~48 cycles per MMA).  Any
// shared-memory access by an issuing warp, an mbarrier wait included, waits behind that warp's queued
// MMA operand reads (~1200 cycles with a few dozen MMAs in flight), so the issuing warps touch no
// shared memory: a separate waiter warp performs every mbarrier wait of the MMA side and releases the
// issuing warps through a named barrier, which costs them a few cycles.
constexpr int kMmaWarps = 2;
constexpr int kWaitWarp = 1;
constexpr int kMmaWarp0 = 2;
// Epilogue warps: two or three per TMEM lane quadrant (warps 4.. after the TMA, waiter and MMA warps).
// Two keep the whole block within 170 registers a thread, so the plain and BatchNorm-statistics
// epilogues run without spills (about 10 % faster on 1x1 layers); the BatchNorm-backward epilogue, with
// more work per element, runs faster with three despite the 128-register cap.
constexpr int kEpiWarp0 = kMmaWarp0 + kMmaWarps;
__host__ __device__ constexpr int fwd_threads(int epi_warps) { return 32 * (kEpiWarp0 + epi_warps); }
constexpr int kMmaBar = 1, kMmaBarThreads = 32 * (1 + kMmaWarps);   // waiter + MMA warps
constexpr int kTileM = 128;

// Sums of 16 per-lane values over the 32 lanes of a warp in 16 shuffles (each butterfly step hands
// half of the remaining channels to the partner lane): on return every lane L holds the sum of
// channel L >> 1.  The order of additions is fixed, so results are deterministic.
__device__ __forceinline__ float warp_sum16(const float (&v)[16], int lane) {
    float w8[8], w4[4], w2[2];
    const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4, h1 = lane & 2;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const float send = h4 ? v[k] : v[8 + k];
        const float keep = h4 ? v[8 + k] : v[k];
        w8[k] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float send = h3 ? w8[k] : w8[4 + k];
        const float keep = h3 ? w8[4 + k] : w8[k];
        w4[k] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const float send = h2 ? w4[k] : w4[2 + k];
        const float keep = h2 ? w4[2 + k] : w4[k];
        w2[k] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
    const float send = h1 ? w2[0] : w2[1];
    const float keep = h1 ? w2[1] : w2[0];
    float r = keep + __shfl_xor_sync(0xffffffffu, send, 2);
    return r + __shfl_xor_sync(0xffffffffu, r, 1);
}

// Epilogue modes, each compiled on its own so that the features a launch does not use cost no
// instructions per item: the trunk's (bias, SiLU, shortcut, halo mask, parity copy), the head
// forward's (BatchNorm statistics partials), the head data gradient's (BatchNorm backward), and the
// generic one (any combination, with the pre-added accumulator of the 3xTF32 passes).
constexpr int kEpiPlain = 0, kEpiStats = 1, kEpiBnBwd = 2, kEpiGeneric = 3;
template <int kEpiWarps, int kMode>
__global__ void __launch_bounds__(fwd_threads(kEpiWarps), 1)
    conv_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmO, const __grid_constant__ FwdParams p) {
    constexpr int kEpiThreads = 32 * kEpiWarps;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int b_bytes = p.n * 128;          // one (tap, chunk) weight block; multiple of 2048
    uint8_t* a_ring = smem + p.stage_bytes;
    uint8_t* b_region = a_ring + p.a_stages * p.a_stage_bytes;
    const bool resident = p.b_stages == 0;
    const int nb = resident ? 1 : p.b_stages;
    uint64_t* afull = reinterpret_cast<uint64_t*>(b_region + p.b_region_bytes);
    uint64_t* aempty = afull + p.a_stages;
    uint64_t* bfull = aempty + p.a_stages;
    uint64_t* bempty = bfull + nb;
    uint64_t* tfull = bempty + nb;
    uint64_t* tempty = tfull + p.nacc;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + p.nacc);
    int* tap_s = reinterpret_cast<int*>(tmem_slot + 4);     // [9] weight tap, [9] A row offset
    float* bias_s = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tap_s + 20) + 15) & ~uintptr_t(15));
    float* gam_s = bias_s + p.n;   // BatchNorm gamma / beta of the layer whose gradient is produced
    float* bet_s = gam_s + p.n;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x < 9) {
        tap_s[threadIdx.x] = p.tap_t[threadIdx.x];
        tap_s[9 + threadIdx.x] = p.tap_off[threadIdx.x];
    }
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.a_stages; s++) {
            mbar_init(&afull[s], 1);
            mbar_init(&aempty[s], kMmaWarps);
        }
        for (int s = 0; s < nb; s++) {
            mbar_init(&bfull[s], 1);
            mbar_init(&bempty[s], kMmaWarps);
        }
        for (int a = 0; a < p.nacc; a++) {
            mbar_init(&tfull[a], kMmaWarps);
            mbar_init(&tempty[a], kEpiThreads);
        }
        fence_barrier_init();
    }
    if (warp >= kEpiWarp0)
        for (int i = threadIdx.x - 32 * kEpiWarp0; i < p.n; i += kEpiThreads) {
            bias_s[i] = (p.bias && i < p.n_valid) ? p.bias[p.n0 + i] : 0.0f;
            gam_s[i] = (p.bn.grad_part && i < p.n_valid) ? p.bn.gamma[p.n0 + i] : 0.0f;
            bet_s[i] = (p.bn.grad_part && i < p.n_valid) ? p.bn.beta[p.n0 + i] : 0.0f;
        }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (p.out_tma) prefetch_tmap(&tmO);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.alloc_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int tile_rows = kTileM * p.T;

    if (warp == 0) {
        if (lane == 0) {
            bool ok = true;
            if (resident) {
                mbar_arrive_expect_tx(&bfull[0], (uint32_t)(p.taps * p.kchunks * b_bytes));
                for (int t = 0; t < p.taps; t++)
                    for (int c = 0; c < p.kchunks; c++)
                        tma_load_2d(b_region + (t * p.kchunks + c) * b_bytes, &tmB, &bfull[0], t * p.kpad + c * 32,
                                    p.n0);
            }
            int ia = 0, ib = 0;
            for (int tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                const int m0 = tile * tile_rows;
                for (int c = 0; ok && c < p.kchunks; c++) {
                    int j = 0;
                    for (int g = 0; ok && g < p.ngroups; g++) {
                        const int sa = ia % p.a_stages;
                        if (!(ok = mbar_wait(&aempty[sa], ((ia / p.a_stages) & 1) ^ 1, p.err, 1))) break;
                        uint8_t* dst = a_ring + sa * p.a_stage_bytes;
                        mbar_arrive_expect_tx(&afull[sa], (uint32_t)(p.g_boxes[g] * kBoxRows * 128));
                        for (int bx = 0; bx < p.g_boxes[g]; bx++)
                            tma_load_2d(dst + bx * kBoxRows * 128, &tmA, &afull[sa], c * 32,
                                        m0 + p.g_lo[g] + bx * kBoxRows);
                        ia++;
                        if (!resident) {
                            for (int e0 = 0; e0 < p.g_ntaps[g]; e0 += p.b_pack, ib++) {
                                const int np = min(p.b_pack, p.g_ntaps[g] - e0);
                                const int sb = ib % p.b_stages;
                                if (!(ok = mbar_wait(&bempty[sb], ((ib / p.b_stages) & 1) ^ 1, p.err, 1))) break;
                                mbar_arrive_expect_tx(&bfull[sb], (uint32_t)(np * b_bytes));
                                for (int k = 0; k < np; k++)
                                    tma_load_2d(b_region + (sb * p.b_pack + k) * b_bytes, &tmB, &bfull[sb],
                                                tap_s[j + e0 + k] * p.kpad + c * 32, p.n0);
                            }
                        }
                        j += p.g_ntaps[g];
                    }
                }
            }
        }
    } else if (warp == kWaitWarp) {
        // every wait of the MMA side, in the MMA warps' order; each ends with a named-barrier hand-off.
        // After a timed-out wait the remaining waits are skipped (the hand-offs continue, so the MMA
        // warps, the epilogue and the producer all still finish; the error flag reports the failure).
        bool live = true;
        auto event = [&](uint64_t* bar, uint32_t parity, int code) {
            if (live) live = mbar_wait(bar, parity, p.err, code);
            named_bar_sync(kMmaBar, kMmaBarThreads);
        };
        if (resident) event(&bfull[0], 0, 3);
        int ia = 0, ib = 0, local = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, local++) {
            event(&tempty[local % p.nacc], ((local / p.nacc) & 1) ^ 1, 2);
            for (int c = 0; c < p.kchunks; c++)
                for (int g = 0; g < p.ngroups; g++) {
                    event(&afull[ia % p.a_stages], (ia / p.a_stages) & 1, 3);
                    ia++;
                    if (!resident)
                        for (int e0 = 0; e0 < p.g_ntaps[g]; e0 += p.b_pack, ib++)
                            event(&bfull[ib % p.b_stages], (ib / p.b_stages) & 1, 3);
                }
        }
    } else if (warp < kEpiWarp0) {
        // MMA warp w (whole warp, elect.sync issues) takes sub-tiles w, w + kMmaWarps, ... and commits
        // every stage release and accumulator hand-off (those barriers count kMmaWarps arrivals)
        const int w = warp - kMmaWarp0;
        const uint32_t idesc = idesc_tf32(p.n, 0, 0);
        if (resident) named_bar_sync(kMmaBar, kMmaBarThreads);
        // Descriptors are linear in the start-address field (address >> 4, 14 bits, never
        // carried out of within shared memory), so every operand descriptor below is a base
        // descriptor plus a byte offset >> 4: 128-byte rows add 8, a 32-byte K step adds 2,
        // a 128-row sub-tile adds 1024.
        const uint64_t a_desc0 = smem_desc(smem_u32(a_ring), 16, 1024, kLayoutSw128);
        const uint64_t b_desc0 = smem_desc(smem_u32(b_region), 16, 1024, kLayoutSw128);
        const uint32_t a_stage16 = (uint32_t)p.a_stage_bytes >> 4, b_blk16 = (uint32_t)b_bytes >> 4;
        const int T = p.T;
        int ia = 0, ib = 0, local = 0;
        const int slots = T * p.ksplit;   // accumulators per stage
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, local++) {
            const int acc = local % p.nacc;
            named_bar_sync(kMmaBar, kMmaBarThreads);   // accumulator stage drained by the epilogue
            tc_fence_after();
            const uint32_t d = tmem_base + acc * slots * p.acc_cols;
            const int mt = min(T, p.sub_tiles - tile * T);
            for (int c = 0; c < p.kchunks; c++) {
                int j = 0;
                for (int g = 0; g < p.ngroups; g++) {
                    const int sa = ia % p.a_stages;
                    named_bar_sync(kMmaBar, kMmaBarThreads);   // A region loaded
                    const uint64_t a_st = a_desc0 + (uint64_t)(sa * a_stage16);
                    // the MMAs of tap j against weight block descriptor b_d
                    auto tap_mmas = [&](int jj, uint64_t b_d) {
                        const uint64_t a_t = a_st + (uint64_t)(p.tap_off[jj] * 8);
                        const uint32_t first = (c == 0 && jj == 0) ? 0u : 1u;
                        if (p.ksplit == 2) {
                            // one sub-tile: this warp's K steps 2w, 2w+1 into accumulator w
                            const uint32_t d_w = d + w * p.acc_cols;
                            mma_tf32_elect(d_w, a_t + 4 * w, b_d + 4 * w, idesc, first);
                            mma_tf32_elect(d_w, a_t + 4 * w + 2, b_d + 4 * w + 2, idesc, 1u);
                        } else {
                            for (int i = w; i < mt; i += kMmaWarps) {
                                const uint64_t a_i = a_t + (uint64_t)(i * 1024);
                                const uint32_t d_i = d + i * p.acc_cols;
                                mma_tf32_elect(d_i, a_i, b_d, idesc, first);
                                mma_tf32_elect(d_i, a_i + 2, b_d + 2, idesc, 1u);
                                mma_tf32_elect(d_i, a_i + 4, b_d + 4, idesc, 1u);
                                mma_tf32_elect(d_i, a_i + 6, b_d + 6, idesc, 1u);
                            }
                        }
                    };
                    const int jend = j + p.g_ntaps[g];
                    if (resident) {
                        for (; j < jend; j++) tap_mmas(j, b_desc0 + (uint64_t)((p.tap_t[j] * p.kchunks + c) * b_blk16));
                    } else {
                        // one hand-off and one release per pack of weight blocks
                        for (; j < jend; ib++) {
                            const int sb = ib % p.b_stages;
                            const int np = min(p.b_pack, jend - j);
                            named_bar_sync(kMmaBar, kMmaBarThreads);   // weight pack loaded
                            const uint64_t b_st = b_desc0 + (uint64_t)(sb * p.b_pack * b_blk16);
                            for (int e = 0; e < np; e++, j++) tap_mmas(j, b_st + (uint64_t)(e * b_blk16));
                            mma_commit_elect(&bempty[sb]);
                        }
                    }
                    mma_commit_elect(&aempty[sa]);
                    ia++;
                }
            }
            mma_commit_elect(&tfull[acc]);
        }
    } else {
        // kEpiWarps / 4 warps per TMEM lane quadrant; each takes every (kEpiWarps / 4)-th (sub-tile,
        // column chunk) item.
        // Global loads of an item (residual, BatchNorm input and coefficients) are issued before
        // its TMEM load so that their latencies overlap.
        const int q = warp & 3;
        const int part = (warp - kEpiWarp0) >> 2;
        const int nchunks = (p.n + 15) >> 4;
        constexpr bool kAny = kMode == kEpiGeneric;
        const bool bn_bwd = (kMode == kEpiBnBwd || kAny) && p.bn.grad_part != nullptr;
        const bool bn_stats = (kMode == kEpiStats || kAny) && p.bn.stats_part != nullptr;
        const float* const pre_in = kAny ? p.pre : nullptr;
        const float* const res_in = kAny ? p.residual : nullptr;
        float* const phase_out = kAny ? p.phase : nullptr;
        // trunk mode with out_tma: this warp's output tile, two halves of 32 rows x 16 channels (64 bytes
        // a row) in the 64-byte swizzle of the output tensor map (16-byte chunk c of row r at chunk
        // c ^ ((r >> 1) & 3)), so that the 32 rows of one st.shared.v4 fill four whole bank wavefronts
        float* const stage_w = reinterpret_cast<float*>(smem) + (warp - kEpiWarp0) * 1024;
        bool stage_busy = false;
        int local = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, local++) {
            const int acc = local % p.nacc;
            if (!mbar_wait(&tfull[acc], (local / p.nacc) & 1, p.err, 4)) break;
            tc_fence_after();
            const int mt = min(p.T, p.sub_tiles - tile * p.T);
            if constexpr (kMode == kEpiPlain) {
                // items (sub-tile i, 32-column chunk cj) in steps of kEpiWarps / 4; every branch is
                // warp-uniform and the row index within the image advances without divisions
                const int nch = (p.n + 31) >> 5;
                const int sub0 = tile * p.T;
                int rem = sub0 - (sub0 / p.sub_per_img) * p.sub_per_img;
                int i = 0, cj = part;
                while (cj >= nch) {
                    cj -= nch;
                    i++;
                    if (++rem == p.sub_per_img) rem = 0;
                }
                while (i < mt) {
                    const int j = cj * 32;
                    if (j < p.n_valid) {
                        const long m = (long)(sub0 + i) * kTileM + q * 32 + lane;
                        const int r = rem * kTileM + q * 32 + lane;
                        bool inside = true;
                        if (p.mask) {
                            const int py = fast_div(r, p.inv_wp), px = r - py * p.grid.wp;
                            inside = py >= 1 && py <= p.grid.h && px >= 1 && px <= p.grid.w;
                        }
                        // each 16-column half is whole (vector accesses), partial or empty
                        const bool full0 = j + 16 <= p.n_valid, full1 = j + 32 <= p.n_valid;
                        float res[32];
                        const bool has_res = p.residual != nullptr;
                        if (has_res) {
                            const float* rr = p.residual + m * (long)p.res_pitch + j;
#pragma unroll
                            for (int h = 0; h < 2; h++) {
                                if ((h ? full1 : full0) && inside) {
#pragma unroll
                                    for (int u = 4 * h; u < 4 * h + 4; u++) {
                                        const float4 t = *reinterpret_cast<const float4*>(rr + 4 * u);
                                        res[4 * u] = t.x;
                                        res[4 * u + 1] = t.y;
                                        res[4 * u + 2] = t.z;
                                        res[4 * u + 3] = t.w;
                                    }
                                } else {
#pragma unroll
                                    for (int u = 16 * h; u < 16 * h + 16; u++)
                                        res[u] = (inside && j + u < p.n_valid) ? rr[u] : 0.0f;
                                }
                            }
                        }
                        float v[32];
                        const uint32_t tl = ((uint32_t)(q * 32) << 16) + (uint32_t)j;
                        if (p.ksplit == 2) {
                            float v1[32];
                            tmem_ld32(tmem_base + acc * 2 * p.acc_cols + tl, v);
                            tmem_ld32(tmem_base + acc * 2 * p.acc_cols + p.acc_cols + tl, v1);
#pragma unroll
                            for (int u = 0; u < 32; u++) v[u] += v1[u];
                        } else {
                            tmem_ld32(tmem_base + (acc * p.T + i) * p.acc_cols + tl, v);
                        }
                        const float4* b4 = reinterpret_cast<const float4*>(bias_s + j);
                        if (p.silu) {
#pragma unroll
                            for (int u = 0; u < 8; u++) {
                                const float4 b = b4[u];
                                v[4 * u] = silu_fast(v[4 * u] + b.x);
                                v[4 * u + 1] = silu_fast(v[4 * u + 1] + b.y);
                                v[4 * u + 2] = silu_fast(v[4 * u + 2] + b.z);
                                v[4 * u + 3] = silu_fast(v[4 * u + 3] + b.w);
                            }
                        } else {
#pragma unroll
                            for (int u = 0; u < 8; u++) {
                                const float4 b = b4[u];
                                v[4 * u] += b.x;
                                v[4 * u + 1] += b.y;
                                v[4 * u + 2] += b.z;
                                v[4 * u + 3] += b.w;
                            }
                        }
                        if (has_res) {
#pragma unroll
                            for (int u = 0; u < 32; u++) v[u] += res[u];
                        }
                        if (!inside) {
#pragma unroll
                            for (int u = 0; u < 32; u++) v[u] = 0.0f;
                        }
                        if (p.rnd) {
#pragma unroll
                            for (int u = 0; u < 32; u++) v[u] = tf32_rna(v[u]);
                        }
                        float* prow = nullptr;
                        if (p.phase && inside) {
                            const int py = fast_div(r, p.inv_wp), px = r - py * p.grid.wp;
                            const int img = (int)((sub0 + i) / p.sub_per_img);
                            const long prow_index = ((py & 1) * 2 + (px & 1)) * p.phase_stride + img * p.phase_rows +
                                                    (long)(py >> 1) * p.phase_wp + (px >> 1);
                            prow = p.phase + prow_index * p.phase_pitch + j;
                        }
                        float* orow = (p.out && !p.out_tma) ? p.out + m * (long)p.out_pitch + j : nullptr;
                        if (p.out_tma) {
                            // the previous stores of this tile have read it; rows in, one TMA store per
                            // 16-channel half out (channels past n_valid are clipped by the tensor map)
                            if (stage_busy && lane == 0) bulk_wait_read_all();
                            __syncwarp();
                            const int sw = (lane >> 1) & 3;
                            float4* s0 = reinterpret_cast<float4*>(stage_w + lane * 16);
                            float4* s1 = reinterpret_cast<float4*>(stage_w + 512 + lane * 16);
#pragma unroll
                            for (int u = 0; u < 4; u++) {
                                s0[u ^ sw] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                                s1[u ^ sw] = make_float4(v[16 + 4 * u], v[16 + 4 * u + 1], v[16 + 4 * u + 2],
                                                         v[16 + 4 * u + 3]);
                            }
                            fence_proxy_async();
                            __syncwarp();
                            if (lane == 0) {
                                const int y0 = (int)(m - lane);
                                tma_store_2d(&tmO, stage_w, j, y0);
                                if (j + 16 < p.n_valid) tma_store_2d(&tmO, stage_w + 512, j + 16, y0);
                                bulk_commit();
                            }
                            stage_busy = true;
                        }
#pragma unroll
                        for (int h = 0; h < 2; h++) {
                            if (h ? full1 : full0) {
                                if (orow) {
#pragma unroll
                                    for (int u = 4 * h; u < 4 * h + 4; u++)
                                        reinterpret_cast<float4*>(orow)[u] =
                                            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                                }
                                if (prow) {
#pragma unroll
                                    for (int u = 4 * h; u < 4 * h + 4; u++)
                                        reinterpret_cast<float4*>(prow)[u] =
                                            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                                }
                            } else if (j + 16 * h < p.n_valid) {
#pragma unroll
                                for (int u = 16 * h; u < 16 * h + 16; u++)
                                    if (j + u < p.n_valid) {
                                        if (orow) orow[u] = v[u];
                                        if (prow) prow[u] = v[u];
                                    }
                            }
                        }
                    }
                    cj += kEpiWarps / 4;
                    while (cj >= nch) {
                        cj -= nch;
                        i++;
                        if (++rem == p.sub_per_img) rem = 0;
                    }
                }
                tc_fence_before();
                mbar_arrive(&tempty[acc]);
                continue;
            }
            // items (sub-tile i, 16-column chunk cj) in steps of kEpiWarps / 4, with 32-bit index math
            // advanced incrementally (a 128-row sub-tile never spans two images)
            const int sub0 = tile * p.T;
            int img = sub0 / p.sub_per_img, rem = sub0 - img * p.sub_per_img;
            int i = 0, cj = part;
            auto next_sub = [&] {
                i++;
                if (++rem == p.sub_per_img) {
                    rem = 0;
                    img++;
                }
            };
            while (cj >= nchunks) {
                cj -= nchunks;
                next_sub();
            }
            for (bool first = true;; first = false) {
                if (!first) {
                    cj += kEpiWarps / 4;
                    while (cj >= nchunks) {
                        cj -= nchunks;
                        next_sub();
                    }
                }
                if (i >= mt) break;
                const int j = cj * 16;
                if (j >= p.n_valid) continue;   // warp-uniform
                const long m = (long)(sub0 + i) * kTileM + q * 32 + lane;
                const int r = rem * kTileM + q * 32 + lane;
                bool inside = true;
                if (p.mask) {
                    // r / wp from a float reciprocal: exact for r < 2^22 (the quotient of r + 1/2 lies at
                    // least 1 / (2 wp) from an integer, the rounding error is below (r + 1/2) 2^-23 / wp)
                    const int py = __float2int_rd(((float)r + 0.5f) * p.inv_wp), px = r - py * p.grid.wp;
                    inside = py >= 1 && py <= p.grid.h && px >= 1 && px <= p.grid.w;
                }
                const bool full16 = j + 16 <= p.n_valid;
                const int chb = p.n0 + j;
                float* orow = p.out ? p.out + m * (long)p.out_pitch : nullptr;
                const float* rrow = res_in ? res_in + m * (long)p.res_pitch : nullptr;
                float res[16];
                if (rrow && full16 && inside) {
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const float4 t = *reinterpret_cast<const float4*>(rrow + j + 4 * u);
                        res[4 * u] = t.x;
                        res[4 * u + 1] = t.y;
                        res[4 * u + 2] = t.z;
                        res[4 * u + 3] = t.w;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 16; u++) res[u] = (rrow && inside && j + u < p.n_valid) ? rrow[j + u] : 0.0f;
                }
                float pre[16];
                if (pre_in) {
                    const float* pr = pre_in + m * (long)p.pre_pitch + j;
                    if (full16) {
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const float4 t = *reinterpret_cast<const float4*>(pr + 4 * u);
                            pre[4 * u] = t.x;
                            pre[4 * u + 1] = t.y;
                            pre[4 * u + 2] = t.z;
                            pre[4 * u + 3] = t.w;
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < 16; u++) pre[u] = j + u < p.n_valid ? pr[u] : 0.0f;
                    }
                } else {
#pragma unroll
                    for (int u = 0; u < 16; u++) pre[u] = 0.0f;
                }
                float yv[16], mv[16], iv[16];
                if (bn_bwd) {
                    const float* yr = p.bn.y + m * (long)p.bn.y_pitch + chb;
                    const float* mr = p.bn.mean + img * p.bn.channels + chb;
                    const float* ir = p.bn.inv + img * p.bn.channels + chb;
                    if (full16) {
#pragma unroll
                        for (int u = 0; u < 4; u++) {
                            const float4 t = inside ? *reinterpret_cast<const float4*>(yr + 4 * u)
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                            yv[4 * u] = t.x;
                            yv[4 * u + 1] = t.y;
                            yv[4 * u + 2] = t.z;
                            yv[4 * u + 3] = t.w;
                            const float4 mm = *reinterpret_cast<const float4*>(mr + 4 * u);
                            mv[4 * u] = mm.x;
                            mv[4 * u + 1] = mm.y;
                            mv[4 * u + 2] = mm.z;
                            mv[4 * u + 3] = mm.w;
                            const float4 ii = *reinterpret_cast<const float4*>(ir + 4 * u);
                            iv[4 * u] = ii.x;
                            iv[4 * u + 1] = ii.y;
                            iv[4 * u + 2] = ii.z;
                            iv[4 * u + 3] = ii.w;
                        }
                    } else {
#pragma unroll
                        for (int u = 0; u < 16; u++) {
                            const bool ok = j + u < p.n_valid;
                            yv[u] = (inside && ok) ? yr[u] : 0.0f;
                            mv[u] = ok ? mr[u] : 0.0f;
                            iv[u] = ok ? ir[u] : 0.0f;
                        }
                    }
                }
                float v[16];
                if (p.ksplit == 2) {
                    float v1[16];
                    const uint32_t t0 = tmem_base + acc * 2 * p.acc_cols + ((uint32_t)(q * 32) << 16) + j;
                    tmem_ld16(t0, v);
                    tmem_ld16(t0 + p.acc_cols, v1);
#pragma unroll
                    for (int u = 0; u < 16; u++) v[u] += v1[u];
                } else {
                    tmem_ld16(tmem_base + (acc * p.T + i) * p.acc_cols + ((uint32_t)(q * 32) << 16) + j, v);
                }
                // parity-split copy: padded pixel (py, px) -> plane (py&1, px&1), cell (py>>1, px>>1)
                float* prow = nullptr;
                if (phase_out && inside) {
                    const int py = r / p.grid.wp, px = r - py * p.grid.wp;
                    const long prow_index = ((py & 1) * 2 + (px & 1)) * p.phase_stride + img * p.phase_rows +
                                            (long)(py >> 1) * p.phase_wp + (px >> 1);
                    prow = phase_out + prow_index * p.phase_pitch;
                }
#pragma unroll
                for (int u = 0; u < 16; u++) {
                    float x = (v[u] + pre[u]) + bias_s[j + u];
                    if (p.silu) x = silu_fast(x);
                    x += res[u];
                    v[u] = inside ? x : 0.0f;
                }
                // BatchNorm partials over this warp's 32 rows (one row group, inside one image)
                const long grp = ((long)tile * tile_rows + i * kTileM + q * 32) >> 5;
                if (bn_stats) {
                    const float cnt = (float)__popc(__ballot_sync(0xffffffffu, inside));
                    const float mean_l = cnt > 0.0f ? warp_sum16(v, lane) / cnt : 0.0f;   // channel lane >> 1
                    float d[16];
#pragma unroll
                    for (int u = 0; u < 16; u++) {
                        const float mu = __shfl_sync(0xffffffffu, mean_l, 2 * u);
                        d[u] = inside ? (v[u] - mu) * (v[u] - mu) : 0.0f;
                    }
                    const float m2_l = warp_sum16(d, lane);
                    const int cu = lane >> 1;
                    if ((lane & 1) == 0 && j + cu < p.n_valid) {
                        float* o = p.bn.stats_part + (grp * p.bn.channels + chb + cu) * 3;
                        o[0] = cnt;
                        o[1] = mean_l;
                        o[2] = m2_l;
                    }
                }
                if (bn_bwd) {
                    // v holds g = dL/da of the BN layer; store dz = dL/dz = g SiLU'(z) instead
                    float dzx[16];
#pragma unroll
                    for (int u = 0; u < 16; u++) {
                        float xh = 0.0f, dz = 0.0f;
                        if (inside && j + u < p.n_valid) {
                            xh = (yv[u] - mv[u]) * iv[u];
                            const float z = xh * gam_s[j + u] + bet_s[j + u];
                            const float sg = __fdividef(1.0f, 1.0f + __expf(-z));
                            dz = v[u] * (sg + z * sg * (1.0f - sg));
                        }
                        v[u] = dz;
                        dzx[u] = dz * xh;
                    }
                    const float s1 = warp_sum16(v, lane);
                    const float s2 = warp_sum16(dzx, lane);
                    const int cu = lane >> 1;
                    if ((lane & 1) == 0 && j + cu < p.n_valid) {
                        float* o = p.bn.grad_part + (grp * p.bn.channels + chb + cu) * 2;
                        o[0] = s1;
                        o[1] = s2;
                    }
                }
                if (p.rnd) {
#pragma unroll
                    for (int u = 0; u < 16; u++) v[u] = tf32_rna(v[u]);
                }
                if (full16) {
                    if (orow) {
                        float4* dst = reinterpret_cast<float4*>(orow + j);
#pragma unroll
                        for (int u = 0; u < 4; u++)
                            dst[u] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                    }
                    if (prow) {
                        float4* pd = reinterpret_cast<float4*>(prow + j);
#pragma unroll
                        for (int u = 0; u < 4; u++)
                            pd[u] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
                    }
                } else {
                    if (orow) {
#pragma unroll
                        for (int u = 0; u < 16; u++)
                            if (j + u < p.n_valid) orow[j + u] = v[u];
                    }
                    if (prow) {
#pragma unroll
                        for (int u = 0; u < 16; u++)
                            if (j + u < p.n_valid) prow[j + u] = v[u];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
        if (stage_busy && lane == 0) bulk_wait_all();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.alloc_cols);
    }
}

static int pow2_at_least(int v) {
    int r = 32;
    while (r < v) r <<= 1;
    return r;
}

// Estimated cycles of a forward launch with streamed weights and t sub-tiles per CTA tile (used only to
// pick t).  Rates as measured on B200: TMA about 26 bytes a cycle per SM in stages of 32 KB or more,
// 22 in 16 KB stages, 11 in 8 KB stages; one M128 x N x K8 MMA per 48 (N <= 64), 64 (N <= 128) or 128
// (N = 256) cycles; an epilogue sub-tile about 1500 cycles, exposed once at the end.
static double fwd_tile_cost(long sub_tiles, int t, int a_stage_bytes, int ngroups, int kchunks, int taps,
                            int b_block_bytes, int n) {
    const long tiles = (sub_tiles + t - 1) / t;
    const long waves = (tiles + num_sms() - 1) / num_sms();
    auto rate = [](int stage) { return stage >= 32 * 1024 ? 26.0 : stage >= 16 * 1024 ? 22.0 : 11.0; };
    const double tma = (double)a_stage_bytes * ngroups * kchunks / rate(a_stage_bytes) +
                       (double)b_block_bytes * taps * kchunks / 26.0;
    const double mma = (double)t * taps * kchunks * 4 * (n <= 64 ? 48 : n <= 128 ? 64 : 128);
    return (double)waves * std::max(tma, mma) + 1500.0 * t;
}

// Shared launcher: `m_rows` output rows (multiple of 128), A rows read at m + shift[t].
static void launch_fwd(const View& in, long m_rows, const int* shift, int taps, const float* wk, int n_rows, int n_out,
                       const Grid& grid, const View& out, const ConvEpilogue& ep, const PhaseOut* phase, int* err,
                       cudaStream_t stream) {
    const int kchunks = (in.channels + 31) / 32, kpad = kchunks * 32;
    if (m_rows % kTileM != 0) throw std::runtime_error("conv_tc: output rows not a multiple of 128");
    if ((out.pitch % 4) != 0 || (reinterpret_cast<uintptr_t>(out.base) & 15) != 0)
        throw std::runtime_error("conv_tc: output not 16-byte aligned");
    if (phase && ((phase->pitch % 4) != 0 || (reinterpret_cast<uintptr_t>(phase->base) & 15) != 0))
        throw std::runtime_error("conv_tc: parity copy not 16-byte aligned");
    if (taps < 1 || taps > 9) throw std::runtime_error("conv_tc: taps");
    if ((ep.bn.stats_part || ep.bn.grad_part) && (grid.rows % 32 != 0 || ep.bn.channels < n_out || !ep.mask_halo))
        throw std::runtime_error("conv_tc: BatchNorm partials need masked 32-row groups covering every channel");
    if (ep.pre && ((ep.pre_pitch % 4) != 0 || (reinterpret_cast<uintptr_t>(ep.pre) & 15) != 0))
        throw std::runtime_error("conv_tc: pre-add input not 16-byte aligned");
    if (ep.bn.grad_part && (ep.bn.y_pitch % 4 != 0 || (reinterpret_cast<uintptr_t>(ep.bn.y) & 15) != 0))
        throw std::runtime_error("conv_tc: BatchNorm input not 16-byte aligned");
    // tap groups: taps sorted by shift, a new group wherever consecutive shifts are more than `gap`
    // rows apart.  With gap = wp + 2 a stride-1 3x3 conv is one group (its consecutive shifts differ
    // by 1 or wp - 2) and a stride-2 conv one group per parity plane (planes lie at least
    // rows-per-image - wp - 1 > wp + 2 rows apart); if that haloed region does not fit, gap = 2 puts
    // every kernel row in a group of its own.
    int order[9];
    for (int t = 0; t < taps; t++) order[t] = t;
    std::sort(order, order + taps, [&](int a, int b) { return shift[a] < shift[b] || (shift[a] == shift[b] && a < b); });
    const long sub_tiles = m_rows / kTileM;
    static PerDeviceOnce attr_once;   // devices whose kernel attributes are set
    once_per_device(attr_once, [] {
        set_max_dynamic_smem(conv_fwd_tc_kernel<8, kEpiPlain>, 227 * 1024, "conv_fwd_tc_kernel attribute");
        set_max_dynamic_smem(conv_fwd_tc_kernel<8, kEpiStats>, 227 * 1024, "conv_fwd_tc_kernel attribute");
        set_max_dynamic_smem(conv_fwd_tc_kernel<8, kEpiGeneric>, 227 * 1024, "conv_fwd_tc_kernel attribute");
        set_max_dynamic_smem(conv_fwd_tc_kernel<12, kEpiBnBwd>, 227 * 1024, "conv_fwd_tc_kernel attribute");
        set_max_dynamic_smem(conv_fwd_tc_kernel<12, kEpiGeneric>, 227 * 1024, "conv_fwd_tc_kernel attribute");
    });
    CUtensorMap ta = make_map_2d(in.base, in.channels, in.rows, in.pitch, 32, kBoxRows);
    constexpr int kSmemTotal = 216 * 1024;   // A ring + weights (+ the trunk epilogue's output tiles)
    const bool plain_epilogue = !(ep.bn.grad_part || ep.bn.stats_part || ep.pre);
    for (int n0 = 0; n0 < n_out; n0 += 256) {
        const int n_valid = std::min(256, n_out - n0);
        const int n = (n_valid + 15) / 16 * 16;
        const int b_bytes = n * 128;
        const int acc_cols = pow2_at_least(n);
        const int res_bytes = taps * kchunks * b_bytes;
        bool resident = res_bytes <= 72 * 1024;
        int b_min = resident ? res_bytes : 2 * b_bytes;
        int ngroups = 0, g_lo[kMaxGroups], g_span[kMaxGroups], g_ntaps[kMaxGroups], tap_t[9], tap_off[9];
        int T = 0, a_stage = 0;
        auto stage_bytes = [&](int t_sub) {
            int rows = 0;
            for (int g = 0; g < ngroups; g++) rows = std::max(rows, kTileM * t_sub + g_span[g]);
            return (rows + kBoxRows - 1) / kBoxRows * kBoxRows * 128;
        };
        // tap groups and sub-tiles per CTA tile (T = 0: nothing fits) for `budget` bytes of A ring + weights
        auto plan = [&](int budget) {
            for (int gap : {grid.wp + 2, 2}) {
                ngroups = 0;
                bool too_many = false;
                for (int e = 0; e < taps; e++) {
                    const int t = order[e];
                    if (e == 0 || shift[t] - shift[order[e - 1]] > gap) {
                        if (ngroups == kMaxGroups) {
                            too_many = true;
                            break;
                        }
                        g_lo[ngroups] = shift[t];
                        g_span[ngroups] = 0;
                        g_ntaps[ngroups] = 0;
                        ngroups++;
                    }
                    const int g = ngroups - 1;
                    tap_t[e] = t;
                    tap_off[e] = shift[t] - g_lo[g];
                    g_span[g] = tap_off[e];
                    g_ntaps[g]++;
                }
                if (too_many) continue;
                // largest sub-tile count whose accumulators double-buffer in TMEM, whose A region fits
                // twice next to the weights, and that still leaves two tiles per SM
                T = 4;
                while (T > 1 && (2 * T * acc_cols > 512 || 2 * stage_bytes(T) + b_min > budget ||
                                 (sub_tiles + T - 1) / T < 2L * num_sms()))
                    T >>= 1;
                // streamed weights below 512 KB: at most 2 sub-tiles, whose smaller A regions leave the weight
                // ring more depth (measured on B200 at N = 64 images: 3x3 64->64 at 80x80 94.0 -> 89.4 us,
                // 128->64 at 40x40 55.6 -> 51.0 us; 80->80 already ran at 2)
                if (!resident && T > 2 && (long)taps * kchunks * b_bytes < 512 * 1024) T = 2;
                if (!resident && (long)taps * kchunks * b_bytes >= 512 * 1024) {
                    // large streamed weights are fetched again for every CTA tile, so a small layer may run
                    // faster on fewer, larger tiles: the count of least estimated time among those that fit
                    // (measured: 18 % faster at 576-720 KB of weights a tile)
                    double best = 0.0;
                    int pick = 0;
                    for (int t = 4; t >= 1; t >>= 1) {
                        if (2 * t * acc_cols > 512 || 2 * stage_bytes(t) + b_min > budget) continue;
                        const double c = fwd_tile_cost(sub_tiles, t, stage_bytes(t), ngroups, kchunks, taps, b_bytes, n);
                        if (pick == 0 || c < best) {
                            pick = t;
                            best = c;
                        }
                    }
                    if (pick > 0) T = pick;
                }
                a_stage = stage_bytes(T);
                if (2 * a_stage + b_min <= budget) return;
                T = 0;
            }
        };
        // the trunk epilogue sends its output through shared-memory tiles and TMA stores (8 warps x 4 KB)
        // unless their room would cost sub-tiles per CTA tile, a finer tap grouping or (resident weights)
        // an A stage that a layer of several tap groups uses; outputs of 16 channels (64-byte rows) keep
        // the direct stores, which measured faster for them
        int kSmemBudget = kSmemTotal, stage_total = 0;
        plan(kSmemTotal);
        // weights that fit beside two A regions of one sub-tile stay resident too: a streamed ring fetches
        // them again for every CTA tile, resident ones once per CTA
        if (!resident && T > 0 && res_bytes + 2 * stage_bytes(1) <= kSmemTotal) {
            resident = true;
            b_min = res_bytes;
            plan(kSmemTotal);
        }
        if (plain_epilogue && out.base && T > 0 && n_valid > 16) {
            const int T_full = T, groups_full = ngroups, staged = 8 * 4096;
            auto a_ring_depth = [&](int budget) { return std::min(4, (budget - res_bytes) / a_stage); };
            const int depth_full = resident ? a_ring_depth(kSmemTotal) : 0;
            plan(kSmemTotal - staged);
            const int depth = resident && T > 0 ? a_ring_depth(kSmemTotal - staged) : 0;
            if (T == T_full && ngroups == groups_full && depth >= (ngroups > 1 ? depth_full : std::min(depth_full, 2))) {
                kSmemBudget = kSmemTotal - staged;
                stage_total = staged;
            } else {
                plan(kSmemTotal);
            }
        }
        if (T == 0) throw std::runtime_error("conv_tc: haloed tile does not fit shared memory");
        FwdParams p;
        p.T = T;
        p.sub_tiles = (int)sub_tiles;
        p.num_tiles = (int)((sub_tiles + T - 1) / T);
        p.kchunks = kchunks;
        p.kpad = kpad;
        p.ngroups = ngroups;
        for (int g = 0; g < kMaxGroups; g++) {
            p.g_lo[g] = g < ngroups ? g_lo[g] : 0;
            p.g_boxes[g] = g < ngroups ? (kTileM * T + g_span[g] + kBoxRows - 1) / kBoxRows : 0;
            p.g_ntaps[g] = g < ngroups ? g_ntaps[g] : 0;
        }
        for (int e = 0; e < 9; e++) {
            p.tap_t[e] = e < taps ? tap_t[e] : 0;
            p.tap_off[e] = e < taps ? tap_off[e] : 0;
        }
        p.taps = taps;
        p.n = n;
        p.n_valid = n_valid;
        p.n0 = n0;
        p.a_stage_bytes = a_stage;
        // Streamed weights: a (tap, chunk) block feeds only T x 4 MMAs, so the weight ring gets the
        // depth (up to 16 blocks) and the A ring two regions (each feeds a whole tap group).
        if (resident) {
            p.a_stages = std::min(4, (kSmemBudget - res_bytes) / a_stage);
            p.b_stages = 0;
            p.b_pack = 1;
            p.b_region_bytes = res_bytes;
        } else {
            p.a_stages = 2;
            // the largest pack that still double-buffers (a TMA handshake per 8 KB block halves the rate)
            const int budget = kSmemBudget - 2 * a_stage;
            int max_group_taps = 1;
            for (int g = 0; g < ngroups; g++) max_group_taps = std::max(max_group_taps, g_ntaps[g]);
            p.b_pack = std::max(1, std::min(max_group_taps, budget / (2 * b_bytes)));
            p.b_stages = std::min(16, budget / (p.b_pack * b_bytes));
            p.b_region_bytes = p.b_stages * p.b_pack * b_bytes;
        }
        p.acc_cols = acc_cols;
        p.ksplit = (T == 1 && 4 * acc_cols <= 512) ? 2 : 1;
        p.nacc = std::max(2, std::min(8, 512 / (T * p.ksplit * acc_cols)));
        p.alloc_cols = pow2_at_least(p.nacc * T * p.ksplit * acc_cols);
        p.out = out.base ? out.base + n0 : nullptr;   // null: only the parity copy is written
        p.out_pitch = out.pitch;
        p.out_tma = stage_total > 0 ? 1 : 0;
        p.stage_bytes = stage_total;
        p.bias = ep.bias;
        p.residual = ep.residual ? ep.residual + n0 : nullptr;
        p.res_pitch = ep.res_pitch;
        p.silu = ep.silu;
        p.mask = ep.mask_halo;
        p.grid = grid;
        p.phase = phase ? phase->base + n0 : nullptr;
        p.phase_pitch = phase ? phase->pitch : 0;
        p.phase_wp = phase ? phase->consumer.wp : 0;
        p.phase_rows = phase ? phase->consumer.rows : 0;
        p.phase_stride = phase ? phase->plane_rows : 0;
        p.bn = ep.bn;
        p.pre = ep.pre ? ep.pre + n0 : nullptr;
        p.pre_pitch = ep.pre_pitch;
        p.rnd = ep.round_tf32;
        p.err = err;
        p.sub_per_img = grid.rows / kTileM;
        p.inv_wp = 1.0f / (float)grid.wp;
        if (grid.rows % kTileM != 0 || grid.rows >= (1 << 22)) throw std::runtime_error("conv_tc: rows per image");
        if (p.alloc_cols > 512) throw std::runtime_error("conv_tc: TMEM columns");
        CUtensorMap tb = make_map_2d(wk, (long)taps * kpad, n_rows, (long)taps * kpad, 32, n);
        const int nb = resident ? 1 : p.b_stages;
        const CUtensorMap to =
            p.out_tma ? make_map_2d(p.out, n_valid, m_rows, out.pitch, 16, 32, CU_TENSOR_MAP_SWIZZLE_64B) : ta;
        const size_t smem = 1024 + (size_t)stage_total + (size_t)p.a_stages * a_stage + p.b_region_bytes +
                            (2 * p.a_stages + 2 * nb + 2 * p.nacc) * 8 + 16 + 80 + 16 + 3 * n * 4;
        if (smem > 227 * 1024) throw std::runtime_error("conv_tc: shared memory");
        const int grid_x = std::min(p.num_tiles, num_sms());
        // the specialised epilogues cover the launches without a pre-add whose features they implement
        const bool other = ep.pre || ((ep.bn.stats_part || ep.bn.grad_part) && (ep.residual || phase));
        if (ep.bn.grad_part && !other)
            conv_fwd_tc_kernel<12, kEpiBnBwd><<<grid_x, fwd_threads(12), smem, stream>>>(ta, tb, to, p);
        else if (ep.bn.grad_part)
            conv_fwd_tc_kernel<12, kEpiGeneric><<<grid_x, fwd_threads(12), smem, stream>>>(ta, tb, to, p);
        else if (ep.bn.stats_part && !other)
            conv_fwd_tc_kernel<8, kEpiStats><<<grid_x, fwd_threads(8), smem, stream>>>(ta, tb, to, p);
        else if (ep.bn.stats_part || ep.pre)
            conv_fwd_tc_kernel<8, kEpiGeneric><<<grid_x, fwd_threads(8), smem, stream>>>(ta, tb, to, p);
        else
            conv_fwd_tc_kernel<8, kEpiPlain><<<grid_x, fwd_threads(8), smem, stream>>>(ta, tb, to, p);
        launch_check("conv_fwd_tc_kernel");
    }
}

void conv_tc_forward(const View& in, const float* wk, int n_rows, int n_out, int taps, int shift_sign,
                     const Grid& grid, const View& out, const ConvEpilogue& ep, int* err, cudaStream_t stream,
                     const PhaseOut* phase) {
    int shift[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    if (taps == 9)
        for (int t = 0; t < 9; t++) shift[t] = shift_sign * ((t / 3 - 1) * grid.wp + (t % 3 - 1));
    launch_fwd(in, in.rows, shift, taps, wk, n_rows, n_out, grid, out, ep, phase, err, stream);
}

void conv_tc_strided(const View& phase_in, long plane_rows, long m_rows, const float* wk, int oc, const Grid& gout,
                     const View& out, const ConvEpilogue& ep, int* err, cudaStream_t stream, const PhaseOut* phase) {
    // tap (ky, kx) of output pixel m reads padded input (2 oy + ky, 2 ox + kx): parity plane
    // (ky & 1, kx & 1), cell (oy + ky / 2, ox + kx / 2) = row m + (ky / 2 - 1) wp + (kx / 2 - 1)
    int shift[9];
    for (int t = 0; t < 9; t++) {
        const int ky = t / 3, kx = t % 3;
        shift[t] = (int)(((ky & 1) * 2 + (kx & 1)) * plane_rows + ((ky >> 1) - 1) * gout.wp + ((kx >> 1) - 1));
    }
    if (phase_in.rows != 4 * plane_rows) throw std::runtime_error("conv_tc_strided: parity input rows");
    launch_fwd(phase_in, m_rows, shift, 9, wk, oc, oc, gout, out, ep, phase, err, stream);
}

// ------------------------------------------------------------------ weight-gradient kernel
struct WgradParams {
    int taps, kchunks;       // input-channel blocks of 32 per tap
    int total_chunks;        // taps * kchunks
    int shift[9];
    int n;                   // output-gradient channels (MMA N, multiple of 16)
    int nblocks;             // ceil(n / 32)
    long rows;               // pixel rows (K)
    long rows_per_split;     // multiple of 32
    int stages;
    int acc_stride;          // TMEM columns between the MMA warps' accumulators (power of two >= n)
    int alloc_cols;
    int oob_channel;         // channel coordinate that lies outside the input view (zero fill)
    float* ws;               // [split][m_tiles * 128][n]
    int m_tiles;
    int* err;
};

// warp 0 TMA, warp 1 waiter (every mbarrier wait of the MMA side, handed on through a named barrier:
// an MMA-issuing warp that touches shared memory waits behind its own queued MMA operand reads),
// warps 2-3 MMA (warp 2 + w issues the K steps k with k % 2 == w of every stage into its own
// accumulator, for the issue rate; the epilogue adds the two), warps 4-7 epilogue
constexpr int kWgradMmaWarps = 2;
constexpr int kWgradWaitWarp = 1, kWgradMmaWarp0 = 2;
constexpr int kWgradThreads = 32 * (2 + kWgradMmaWarps + 4);
constexpr int kWgradBar = 1, kWgradBarThreads = 32 * (1 + kWgradMmaWarps);
constexpr int kWgradBK = 64;                    // pixel rows per stage
constexpr int kWgradBlockBytes = kWgradBK * 128;  // one 32-channel x 64-row box

__global__ void __launch_bounds__(kWgradThreads, 1)
    conv_wgrad_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG,
                         const __grid_constant__ WgradParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int a_bytes = 4 * kWgradBlockBytes;
    const int b_bytes = p.nblocks * kWgradBlockBytes;
    const int stage_bytes = a_bytes + b_bytes;  // multiples of 4096
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + p.stages * stage_bytes);
    uint64_t* empty = full + p.stages;
    uint64_t* tfull = empty + p.stages;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tile = blockIdx.x, split = blockIdx.y;
    const long k_begin = (long)split * p.rows_per_split;
    const long k_end = p.rows < k_begin + p.rows_per_split ? p.rows : k_begin + p.rows_per_split;
    const int kblocks = k_end > k_begin ? (int)((k_end - k_begin + kWgradBK - 1) / kWgradBK) : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWgradMmaWarps);
        }
        mbar_init(&tfull[0], kWgradMmaWarps);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmX);
        prefetch_tmap(&tmG);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.alloc_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int ch_coord[4], tap_shift[4];
            for (int j = 0; j < 4; j++) {
                int g = m_tile * 4 + j;
                if (g < p.total_chunks) {
                    int t = g / p.kchunks, cb = g - t * p.kchunks;
                    ch_coord[j] = cb * 32;
                    tap_shift[j] = p.shift[t];
                } else {
                    ch_coord[j] = p.oob_channel;
                    tap_shift[j] = 0;
                }
            }
            for (int kb = 0; kb < kblocks; kb++) {
                const int s = kb % p.stages;
                const uint32_t ph = (kb / p.stages) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, p.err, 11)) break;
                const int r0 = (int)(k_begin + (long)kb * kWgradBK);
                uint8_t* sa = smem + s * stage_bytes;
                mbar_arrive_expect_tx(&full[s], stage_bytes);
                for (int j = 0; j < 4; j++)
                    tma_load_2d(sa + j * kWgradBlockBytes, &tmX, &full[s], ch_coord[j], r0 + tap_shift[j]);
                for (int j = 0; j < p.nblocks; j++)
                    tma_load_2d(sa + a_bytes + j * kWgradBlockBytes, &tmG, &full[s], j * 32, r0);
            }
        }
    } else if (warp == kWgradWaitWarp) {
        // after a timed-out wait the remaining waits are skipped; the hand-offs continue so that
        // every warp finishes (the error flag reports the failure)
        bool live = true;
        for (int kb = 0; kb < kblocks; kb++) {
            if (live) live = mbar_wait(&full[kb % p.stages], (kb / p.stages) & 1, p.err, 12);
            named_bar_sync(kWgradBar, kWgradBarThreads);
        }
    } else if (warp < kWgradMmaWarp0 + kWgradMmaWarps) {
        const int w = warp - kWgradMmaWarp0;
        const uint32_t idesc = idesc_tf32(p.n, 1, 1);
        const uint32_t d = tmem_base + w * p.acc_stride;
        const uint32_t stage0 = smem_u32(smem);
        for (int kb = 0; kb < kblocks; kb++) {
            const int s = kb % p.stages;
            named_bar_sync(kWgradBar, kWgradBarThreads);   // stage loaded
            const uint32_t a_addr = stage0 + s * stage_bytes;
            const uint32_t b_addr = a_addr + a_bytes;
#pragma unroll
            for (int k = w; k < kWgradBK / 8; k += kWgradMmaWarps) {
                // 8 K rows = two 4-row swizzle groups of 512 B
                uint64_t ad = smem_desc(a_addr + k * 1024, kWgradBlockBytes, 512, kLayoutSw128Base32);
                uint64_t bd = smem_desc(b_addr + k * 1024, kWgradBlockBytes, 512, kLayoutSw128Base32);
                mma_tf32_elect(d, ad, bd, idesc, (kb != 0 || k >= kWgradMmaWarps) ? 1u : 0u);
            }
            mma_commit_elect(&empty[s]);
        }
        mma_commit_elect(&tfull[0]);
    } else {
        const int q = warp & 3;
        const int row = q * 32 + lane;
        float* dst = p.ws + ((long)split * p.m_tiles * kTileM + (long)m_tile * kTileM + row) * p.n;
        if (kblocks == 0) {
            for (int j = 0; j < p.n; j++) dst[j] = 0.0f;
        } else if (mbar_wait(&tfull[0], 0, p.err, 13)) {
            tc_fence_after();
            for (int j = 0; j < p.n; j += 16) {
                float v[16], v1[16];
                tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + j, v);
                tmem_ld16(tmem_base + ((uint32_t)(q * 32) << 16) + p.acc_stride + j, v1);
#pragma unroll
                for (int i = 0; i < 16; i++) v[i] += v1[i];
                float4* d4 = reinterpret_cast<float4*>(dst + j);
#pragma unroll
                for (int i = 0; i < 4; i++) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.alloc_cols);
    }
}

// dw[(o * ic + c) * taps + t] = sum_s ws[s][(t * kchunks + c / 32) * 32 + c % 32][o].  A block takes 32
// consecutive outputs (o fastest, so the workspace reads of a warp are contiguous); its 8 warps sum the
// splits s = w, w + 8, ... in order and warp 0 adds the 8 partial sums in warp order, so the result is
// deterministic.  `n` is the workspace row stride (the MMA width, output channels rounded up to 16);
// `oc` the real output channels, which alone bound the rows of dw that are written.  With a centred input
// (WgradCenter) warp 0 also adds sum_b mean[b][c] tsum[b][t][o] (double, images in order).
constexpr int kReduceWarps = 8;
__global__ void __launch_bounds__(32 * kReduceWarps)
    wgrad_reduce_kernel(const float* ws, int splits, long split_stride, int n, int oc, int ic, int taps, int kchunks,
                        float* dw, int accumulate, WgradCenter center) {
    __shared__ float part[kReduceWarps][32];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long total = (long)oc * ic * taps;
    for (long base = (long)blockIdx.x * 32; base < total; base += (long)gridDim.x * 32) {
        const long i = base + lane;
        float s = 0.0f;
        long di = 0;
        if (i < total) {
            const int o = (int)(i % oc);
            const int tc = (int)(i / oc);
            const int t = tc / ic, c = tc - t * ic;
            const long row = (long)(t * kchunks + c / 32) * 32 + (c % 32);
            const float* src = ws + row * n + o;
#pragma unroll 4
            for (int k = w; k < splits; k += kReduceWarps) s += src[k * split_stride];
            di = ((long)o * ic + c) * taps + t;
        }
        part[w][lane] = s;
        __syncthreads();
        if (w == 0 && i < total) {
            float r = part[0][lane];
#pragma unroll
            for (int q = 1; q < kReduceWarps; q++) r += part[q][lane];
            if (center.mean) {
                const int o = (int)(i % oc);
                const int tc = (int)(i / oc);
                const int t = tc / ic, c = tc - t * ic;
                double corr = 0.0;
                for (int b = 0; b < center.batch; b++)
                    corr += (double)center.mean[(long)b * ic + c] * center.tsum[((long)b * taps + t) * oc + o];
                r += (float)corr;
            }
            dw[di] = accumulate ? dw[di] + r : r;
        }
        __syncthreads();
    }
}

static int wgrad_splits(int m_tiles, long rows) {
    const long kblocks = (rows + kWgradBK - 1) / kWgradBK;
    // one wave of CTAs (one per SM: the stages take most of shared memory)
    int target = std::max(1, num_sms() / std::max(1, m_tiles));
    return (int)std::min<long>(target, std::max<long>(1, kblocks / 8));
}

size_t wgrad_workspace_floats(int ic, int oc, int taps, long rows) {
    const int kchunks = (ic + 31) / 32;
    const int m_tiles = (taps * kchunks + 3) / 4;
    const int n = (oc + 15) / 16 * 16;
    // upper bound on splits independent of the device
    const long kblocks = (rows + kWgradBK - 1) / kWgradBK;
    const long splits = std::min<long>(std::max(1, 2 * 160 / m_tiles), std::max<long>(1, kblocks / 8));
    return (size_t)splits * m_tiles * kTileM * n;
}

void conv_tc_wgrad(const View& x, const View& dy, int taps, const Grid& grid, float* dw, float* ws, int* err,
                   cudaStream_t stream, int accumulate, const WgradCenter* center) {
    if (dy.channels > 256) throw std::runtime_error("conv_tc_wgrad: more than 256 output channels");
    if (x.rows != dy.rows) throw std::runtime_error("conv_tc_wgrad: row mismatch");
    WgradParams p;
    p.taps = taps;
    p.kchunks = (x.channels + 31) / 32;
    p.total_chunks = taps * p.kchunks;
    for (int t = 0; t < 9; t++) p.shift[t] = 0;
    if (taps == 9)
        for (int t = 0; t < 9; t++) p.shift[t] = (t / 3 - 1) * grid.wp + (t % 3 - 1);
    p.n = (dy.channels + 15) / 16 * 16;
    p.nblocks = (p.n + 31) / 32;
    p.rows = x.rows;
    p.m_tiles = (p.total_chunks + 3) / 4;
    int splits = std::min(wgrad_splits(p.m_tiles, p.rows), (int)(wgrad_workspace_floats(x.channels, dy.channels, taps,
                                                                                         x.rows) /
                                                                  ((size_t)p.m_tiles * kTileM * p.n)));
    splits = std::max(1, splits);
    const long kblocks = (p.rows + kWgradBK - 1) / kWgradBK;
    p.rows_per_split = ((kblocks + splits - 1) / splits) * kWgradBK;
    p.oob_channel = p.kchunks * 32;
    const int stage_bytes = (4 + p.nblocks) * kWgradBlockBytes;
    p.stages = std::min(8, (int)((220 * 1024) / stage_bytes));
    p.acc_stride = pow2_at_least(p.n);
    p.alloc_cols = kWgradMmaWarps * p.acc_stride;
    if (p.alloc_cols > 512) throw std::runtime_error("conv_tc_wgrad: TMEM columns");
    p.ws = ws;
    p.err = err;
    CUtensorMap tx = make_map_2d(x.base, x.channels, x.rows, x.pitch, 32, kWgradBK, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    CUtensorMap tg = make_map_2d(dy.base, dy.channels, dy.rows, dy.pitch, 32, kWgradBK,
                                 CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    static PerDeviceOnce attr_once;   // devices whose kernel attributes are set
    once_per_device(attr_once,
                    [] { set_max_dynamic_smem(conv_wgrad_tc_kernel, 227 * 1024, "conv_wgrad_tc_kernel attribute"); });
    const size_t smem = 1024 + (size_t)p.stages * stage_bytes + (2 * p.stages + 2) * 8 + 16;
    conv_wgrad_tc_kernel<<<dim3(p.m_tiles, splits), kWgradThreads, smem, stream>>>(tx, tg, p);
    launch_check("conv_wgrad_tc_kernel");
    const long split_stride = (long)p.m_tiles * kTileM * p.n;
    const long total = (long)dy.channels * x.channels * taps;
    const int blocks = (int)std::min<long>(8 * num_sms(), (total + 31) / 32);
    wgrad_reduce_kernel<<<blocks, 32 * kReduceWarps, 0, stream>>>(ws, splits, split_stride, p.n, dy.channels, x.channels, taps,
                                                    p.kchunks, dw,
                                                    accumulate, center ? *center : WgradCenter{});
    launch_check("wgrad_reduce_kernel");
}

}  // namespace sy
