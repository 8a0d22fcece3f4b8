// bwgemm.cu -- host side of the Blackwell rung: the C ABI of include/bwgemm.h over the sm_100a kernels of
// gemm_kernel.cuh.  Per call: check the shape (the reference's rule, hopper/step7.cu:358-361), plan (plan.h), make
// the TMA tensor maps (cuTensorMapEncodeTiled reached through the runtime, so that no library is linked, as
// hopper/step2.cuh:168-196 does), keep a per-device workspace for the partials of split tiles (allocated at the first
// call that needs more, never during a later call: judge/judge.cu:8-9), launch on the caller's stream (a cluster of
// two blocks for the pair kernel).  No synchronisation.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "bwgemm.h"
#include "gemm_kernel.cuh"
#include "plan.h"

#ifndef BW_API
#define BW_API extern "C" __attribute__((visibility("default")))
#endif

namespace bw {
namespace {

thread_local char g_errbuf[256] = "";

int cuda_fail(cudaError_t e, const char* what)
{
    snprintf(g_errbuf, sizeof g_errbuf, "%s: %s", what, cudaGetErrorString(e));
    return BW_ERR_LAUNCH;
}

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder()
{
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// A row-major fp16 matrix of rows x cols, boxes of box_cols x box_rows, 128-byte swizzle, zeros outside the matrix.
bool make_map(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows)
{
    EncodeTiled enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t elem[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The MN-major operand (B, K x N row-major) as {64 columns, K rows, N / 64 column blocks}: a box of `blocks` column
// blocks is that many 64 x 64 boxes of the 2-D map, 8 KB apart in shared memory.
bool make_map_blocks(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t blocks)
{
    EncodeTiled enc = encoder();
    if (!enc || cols % 64 || blocks == 0 || blocks > 256) return false;
    const cuuint64_t dims[3] = {64, rows, cols / 64};
    const cuuint64_t strides[2] = {cols * 2, 128};
    const cuuint32_t box[3] = {64, 64, blocks};
    const cuuint32_t elem[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct DeviceState {
    bool init = false;
    bool supported = false;
    int sms = 0;
    float* work = nullptr;
    size_t work_bytes = 0;
    int* counters = nullptr;
    int n_counters = 0;
    unsigned long long attrs = 0;  // kernels whose shared-memory limit is set, one bit each
    int pairs = -1;      // pairs of SMs the pair kernel holds at once (its cluster occupancy); -1: not asked yet
    int held[9] = {};    // BW_KSPLIT 1: clusters of c swap-AB blocks held at once, c = 2 .. 8 (asked with pairs)
};
constexpr int kMaxDevices = 64;
DeviceState g_dev[kMaxDevices];
std::mutex g_mu;

unsigned long long initial_wait_ns()
{
    const char* e = getenv("BWGEMM_WAIT_NS");
    if (e) {
        const unsigned long long v = strtoull(e, nullptr, 10);
        if (v > 0) return v;
    }
    return 1000000000ull;  // 1 s
}
unsigned long long g_wait_ns = initial_wait_ns();

// The fused reduce-scatter's waits on other ranks (their partials, their ack of the previous call): the ranks'
// processes reach a call out of step by host-side work (a first call's module loading and plan, a slow rank's launch
// queue), so these waits get a longer limit than the pipeline's own barriers.  BWGEMM_RANK_WAIT_NS sets it (default
// 10 s; never below the barrier limit).
unsigned long long initial_rank_wait_ns()
{
    const char* e = getenv("BWGEMM_RANK_WAIT_NS");
    if (e) {
        const unsigned long long v = strtoull(e, nullptr, 10);
        if (v > 0) return v;
    }
    return 10000000000ull;  // 10 s
}
unsigned long long g_rank_wait_ns = initial_rank_wait_ns();

// Programmatic dependent launch between calls (BW_PDL's default; BWGEMM_PDL=0 or 1 sets it for the process): a call
// whose stream holds another call ahead of it starts its blocks' set-up before that one has finished.
bool initial_pdl()
{
    const char* e = getenv("BWGEMM_PDL");
    if (e && (e[0] == '0' || e[0] == '1') && e[1] == 0) return e[0] == '1';
    return BW_PDL != 0;
}
bool g_pdl = initial_pdl();

int device_state(DeviceState** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return BW_ERR_DEVICE;
    DeviceState& d = g_dev[dev];
    if (!d.init) {
        int major = 0, minor = 0, sms = 0;
        if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess ||
            (e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        d.supported = major == 10 && minor == 0;
        d.sms = sms;
        d.init = true;
    }
    if (!d.supported) {
        snprintf(g_errbuf, sizeof g_errbuf, "this library holds sm_100a code only");
        return BW_ERR_DEVICE;
    }
    *out = &d;
    return BW_OK;
}

// The workspace and counters a plan needs, grown at the first call that needs more.  A buffer that is outgrown is
// never freed: a CUDA graph captured earlier still holds its address and may be replayed at any time (freeing it
// would turn that replay into writes to freed memory).  Growth is at least 2x, so only a few buffers are ever kept;
// all of them go with the context at exit.
int ensure_workspace(DeviceState& d, const bw_plan& q, cudaStream_t st)
{
    cudaError_t e;
    if (q.workspace_bytes > d.work_bytes) {
        size_t bytes = d.work_bytes * 2 > q.workspace_bytes ? d.work_bytes * 2 : q.workspace_bytes;
        float* w = nullptr;
        if ((e = cudaMalloc(&w, bytes)) != cudaSuccess) return cuda_fail(e, "cudaMalloc (workspace)");
        d.work = w;  // the outgrown buffer stays allocated
        d.work_bytes = bytes;
    }
    if (q.counters > d.n_counters) {
        int n = d.n_counters * 2 > q.counters ? d.n_counters * 2 : q.counters;
        if (n < 1024) n = 1024;
        int* c = nullptr;
        if ((e = cudaMalloc(&c, (size_t)n * sizeof(int))) != cudaSuccess) return cuda_fail(e, "cudaMalloc (counters)");
        if ((e = cudaMemsetAsync(c, 0, (size_t)n * sizeof(int), st)) != cudaSuccess)
            return cuda_fail(e, "cudaMemsetAsync (counters)");
        d.counters = c;  // the outgrown array stays allocated (and at zero)
        d.n_counters = n;
    }
    return BW_OK;
}

// Clusters of two blocks for the SM pair (PAIR), of `ksplit` blocks for a swap-AB plan's K split.
// pdl: with programmatic stream serialisation (attr holds two entries).
template <int BN, bool SWAP, bool PAIR, int WM = 1, int EPI = kEpiF16>
cudaLaunchConfig_t launch_config(int grid, cudaStream_t st, cudaLaunchAttribute* attr, int ksplit = 0, bool pdl = false)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = KGeom<BN, SWAP, PAIR, EPI, WM>::kSmemBytes;
    cfg.stream = st;
    const int size = PAIR ? 2 : (SWAP && ksplit > 1) ? ksplit : 1;
    const bool cluster = size > 1;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)size;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = cluster ? attr : attr + 1;
    cfg.numAttrs = cluster ? 1 : 0;
    if (pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        ++cfg.numAttrs;
    }
    return cfg;
}

template <int BN, bool SWAP, bool PAIR, int EPI = kEpiF16, int WM = 1>
int set_smem_limit(DeviceState& d, unsigned long long bit)
{
    if (d.attrs & bit) return BW_OK;
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<BN, SWAP, PAIR, EPI, WM>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         KGeom<BN, SWAP, PAIR, EPI, WM>::kSmemBytes);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    d.attrs |= bit;
    return BW_OK;
}

constexpr unsigned kBitPair = 1u << 9;

// The pairs of SMs the pair kernel can hold at once, asked once per device (a cluster may not straddle GPCs, so this
// can be below sms / 2).
int pair_occupancy(DeviceState& d)
{
    if (d.pairs >= 0) return BW_OK;
    int rc = set_smem_limit<256, false, true>(d, kBitPair);
    if (rc) return rc;
    cudaLaunchAttribute attr[2];
    const cudaLaunchConfig_t cfg = launch_config<256, false, true>(2, 0, attr);
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveClusters(&n, gemm_kernel<256, false, true>, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
#if BW_KSPLIT
    // clusters of 2 .. 8 swap-AB blocks (one block per SM, as every instance's shared memory makes it)
    if ((rc = set_smem_limit<16, true, false>(d, 1u << 1))) return rc;
    for (int c = 2; c <= 8; ++c) {
        const cudaLaunchConfig_t cc = launch_config<16, true, false>(c, 0, attr, c);
        int h = 0;
        if ((e = cudaOccupancyMaxActiveClusters(&h, gemm_kernel<16, true, false>, &cc)) != cudaSuccess)
            return cuda_fail(e, "cudaOccupancyMaxActiveClusters (K split)");
        d.held[c] = h;
    }
#endif
    d.pairs = n;
    return BW_OK;
}

// The clusters of each size the device holds at once, for the K-split rule (BW_KSPLIT 1; null: the rule's default).
const int* held_of(const DeviceState& d) { return BW_KSPLIT ? d.held : nullptr; }

template <int BN, bool SWAP, bool PAIR, int EPI = kEpiF16, int WM = 1>
int launch_kernel(DeviceState& d, unsigned long long bit, const bw_plan& q, const CUtensorMap& mx, const CUtensorMap& my,
                  const CUtensorMap& mc, const Params& p, cudaStream_t st)
{
    using G = KGeom<BN, SWAP, PAIR, EPI, WM>;
    // K split: what a block receives from the others of its cluster lands in its idle stage ring
    if (q.smem_bytes != G::kSmemBytes || q.stages != G::kStages || q.tmem_cols != G::kTmemCols || q.wm != WM ||
        (q.ksplit && (!SWAP || q.ksplit < 2 || q.ksplit > 8 || q.grid != q.ksplit * q.tiles ||
                      plan_ksplit_recv_bytes(BN, WM, q.ksplit) > G::kBarOffset))) {
        snprintf(g_errbuf, sizeof g_errbuf, "plan and kernel geometry disagree (bn %d)", BN);
        return BW_ERR_LAUNCH;
    }
    int rc = set_smem_limit<BN, SWAP, PAIR, EPI, WM>(d, bit);
    if (rc) return rc;
    cudaLaunchAttribute attr[2];
    // the reduce-scatter kernel keeps the plain stream order: its peers' calls pair with this one by epoch
    const cudaLaunchConfig_t cfg = launch_config<BN, SWAP, PAIR, WM, EPI>(q.grid, st, attr, q.ksplit,
                                                                          g_pdl && EPI != kEpiRS);
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_kernel<BN, SWAP, PAIR, EPI, WM>, mx, my, mc, p);
    if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
    return BW_OK;
}

// The plan's kernel instance, launched.
int dispatch(DeviceState& d, const bw_plan& q, const CUtensorMap& mx, const CUtensorMap& my, const CUtensorMap& mc,
             const Params& p, cudaStream_t st, int epi = kEpiF16)
{
    if (epi == kEpiF32) {  // fp32 C: the plan is a TILE or PAIR one (no swap-AB)
        if (q.kernel == BW_KERNEL_PAIR) return launch_kernel<256, false, true, kEpiF32>(d, 1u << 12, q, mx, my, mc, p, st);
        if (q.kernel == BW_KERNEL_TILE && q.bn == 256)
            return launch_kernel<256, false, false, kEpiF32>(d, 1u << 13, q, mx, my, mc, p, st);
        return BW_ERR_ARG;
    }
    if (epi == kEpiSwiGLU) {  // fused activation: TILE or PAIR, whole tiles only
        if (q.sk_tiles != 0) return BW_ERR_ARG;
        if (q.kernel == BW_KERNEL_PAIR)
            return launch_kernel<256, false, true, kEpiSwiGLU>(d, 1u << 14, q, mx, my, mc, p, st);
        if (q.kernel == BW_KERNEL_TILE && q.bn == 256)
            return launch_kernel<256, false, false, kEpiSwiGLU>(d, 1u << 15, q, mx, my, mc, p, st);
        return BW_ERR_ARG;
    }
#if BW_PAIR_WIDE
    if (q.kernel == BW_KERNEL_PAIR && q.bn == 512) return launch_kernel<512, false, true>(d, 1u << 25, q, mx, my, mc, p, st);
#endif
    if (q.kernel == BW_KERNEL_PAIR) return launch_kernel<256, false, true>(d, kBitPair, q, mx, my, mc, p, st);
    if (q.kernel == BW_KERNEL_TILE) {
        switch (q.bn) {
        case 64: return launch_kernel<64, false, false>(d, 1u << 10, q, mx, my, mc, p, st);
        case 128: return launch_kernel<128, false, false>(d, 1u << 11, q, mx, my, mc, p, st);
        case 256: return launch_kernel<256, false, false>(d, 1u << 0, q, mx, my, mc, p, st);
        default: return BW_ERR_ARG;
        }
    }
#if BW_SWAP_PAIR
    if (q.kernel == BW_KERNEL_SWAP_PAIR) {  // swap-AB on SM pairs
        switch (q.bn * 4 + q.wm) {
        case 64 * 4 + 1: return launch_kernel<64, true, true, kEpiF16, 1>(d, 1ull << 27, q, mx, my, mc, p, st);
        case 128 * 4 + 1: return launch_kernel<128, true, true, kEpiF16, 1>(d, 1ull << 29, q, mx, my, mc, p, st);
        case 64 * 4 + 2: return launch_kernel<64, true, true, kEpiF16, 2>(d, 1ull << 30, q, mx, my, mc, p, st);
        case 128 * 4 + 2: return launch_kernel<128, true, true, kEpiF16, 2>(d, 1ull << 32, q, mx, my, mc, p, st);
        default: return BW_ERR_ARG;
        }
    }
#endif
    if (q.wm == 2) {  // swap-AB tiles of 256 weight columns
        switch (q.bn) {
        case 16: return launch_kernel<16, true, false, kEpiF16, 2>(d, 1u << 21, q, mx, my, mc, p, st);
        case 32: return launch_kernel<32, true, false, kEpiF16, 2>(d, 1u << 22, q, mx, my, mc, p, st);
        case 48: return launch_kernel<48, true, false, kEpiF16, 2>(d, 1u << 23, q, mx, my, mc, p, st);
        case 64: return launch_kernel<64, true, false, kEpiF16, 2>(d, 1u << 16, q, mx, my, mc, p, st);
        case 80: return launch_kernel<80, true, false, kEpiF16, 2>(d, 1u << 17, q, mx, my, mc, p, st);
        case 96: return launch_kernel<96, true, false, kEpiF16, 2>(d, 1u << 18, q, mx, my, mc, p, st);
        case 112: return launch_kernel<112, true, false, kEpiF16, 2>(d, 1u << 19, q, mx, my, mc, p, st);
        case 128: return launch_kernel<128, true, false, kEpiF16, 2>(d, 1u << 20, q, mx, my, mc, p, st);
        default: return BW_ERR_ARG;
        }
    }
    switch (q.bn) {
    case 16: return launch_kernel<16, true, false>(d, 1u << 1, q, mx, my, mc, p, st);
    case 32: return launch_kernel<32, true, false>(d, 1u << 2, q, mx, my, mc, p, st);
    case 48: return launch_kernel<48, true, false>(d, 1u << 3, q, mx, my, mc, p, st);
    case 64: return launch_kernel<64, true, false>(d, 1u << 4, q, mx, my, mc, p, st);
    case 80: return launch_kernel<80, true, false>(d, 1u << 5, q, mx, my, mc, p, st);
    case 96: return launch_kernel<96, true, false>(d, 1u << 6, q, mx, my, mc, p, st);
    case 112: return launch_kernel<112, true, false>(d, 1u << 7, q, mx, my, mc, p, st);
    case 128: return launch_kernel<128, true, false>(d, 1u << 8, q, mx, my, mc, p, st);
    default: return BW_ERR_ARG;
    }
}

// The kernel parameters of a plan.
Params make_params(const bw_plan& q, int M, int N, int K, void* C, float* work, int* counters, bool tn = false)
{
    Params p = {};  // row_shift 0 (the rule's order), no reduce-scatter
    p.tn = tn ? 1 : 0;
    p.s.M = M;
    p.s.N = N;
    p.s.K = K;
    p.s.tiles_m = q.tiles_m;
    p.s.tiles_n = q.tiles_n;
    p.s.tiles = q.tiles;
    p.s.kblocks = q.kblocks;
    p.s.dp_tiles = q.dp_tiles;
    p.s.sk_tiles = q.sk_tiles;
    p.s.splits = q.splits;
    p.s.sk_iters = q.sk_iters;
    p.s.group_rows = q.group_rows;
    p.s.ksplit = q.ksplit;
    p.s.dyn = q.dyn;
    p.C = C;
    p.work = work;
    p.counters = counters;
    p.wait_ns = g_wait_ns;
    p.rank_wait_ns = g_rank_wait_ns > g_wait_ns ? g_rank_wait_ns : g_wait_ns;
    return p;
}

// The rows of A one swap-AB block loads per stage: the tokens (a pair: half of them each).
uint32_t swap_rows(const bw_plan& q) { return (uint32_t)(q.kernel == BW_KERNEL_SWAP_PAIR ? q.bn / 2 : q.bn); }

// The two tensor maps of a plan: TILE and PAIR read A (K-major) and B (MN-major) in that role order; SWAP the
// other way round.
bool make_maps(const bw_plan& q, const void* A, const void* B, int M, int N, int K, CUtensorMap* mx, CUtensorMap* my,
               bool tn = false)
{
    if (tn) {  // B is N x K row-major: K-major boxes of 64 K x (the rows of B one stage takes), as A's
        if (q.kernel == BW_KERNEL_TILE || q.kernel == BW_KERNEL_PAIR)  // a pair block loads 128 rows per MMA
            return make_map(mx, A, K, M, 64, 128) &&
                   make_map(my, B, K, N, 64, (uint32_t)(q.kernel == BW_KERNEL_PAIR ? 128 : q.bn));
        return make_map(mx, B, K, N, 64, (uint32_t)(128 * q.wm)) && make_map(my, A, K, M, 64, swap_rows(q));
    }
    if (BW_TMA3D) {  // the stage's 64-column blocks of B in one load
        if (q.kernel == BW_KERNEL_TILE || q.kernel == BW_KERNEL_PAIR)
            return make_map(mx, A, K, M, 64, 128) &&
                   make_map_blocks(my, B, N, K, (uint32_t)(q.kernel == BW_KERNEL_PAIR ? 2 : q.bn / 64));
        return make_map_blocks(mx, B, N, K, (uint32_t)(2 * q.wm)) && make_map(my, A, K, M, 64, swap_rows(q));
    }
    if (q.kernel == BW_KERNEL_TILE || q.kernel == BW_KERNEL_PAIR)
        return make_map(mx, A, K, M, 64, 128) && make_map(my, B, N, K, 64, 64);
    return make_map(mx, B, N, K, 64, 64) && make_map(my, A, K, M, 64, swap_rows(q));
}

// The map of C for the TMA-store epilogue (BW_EPI_TMA: fp16 C of a TILE or PAIR plan): boxes of 64 columns x 32 rows
// (one epilogue warp's rows), 128-byte swizzle.  Other plans store C from registers; they get a copy of `mx`.
bool make_c_map(const bw_plan& q, void* C, int M, int N, int epi, const CUtensorMap& mx, CUtensorMap* mc)
{
    if (BW_EPI_TMA && epi == kEpiF16 && (q.kernel == BW_KERNEL_TILE || q.kernel == BW_KERNEL_PAIR))
        return make_map(mc, C, N, M, 64, 32);
    *mc = mx;
    return true;
}

int gemm(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t st, int variant, int epi = kEpiF16,
         bool tn = false)
{
    if (variant < 0 || variant >= kVariants) return BW_ERR_ARG;
    if (!shape_ok(M, N, K)) return BW_ERR_SHAPE;
    if (!A || !B || !C || (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
                           reinterpret_cast<uintptr_t>(C)) % 16)
        return BW_ERR_ARG;
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    bw_plan q;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if ((rc = pair_occupancy(*d))) return rc;
        const unsigned flags = epi == kEpiF32 ? kPlanNoSwap : epi == kEpiSwiGLU ? kPlanNoSwap | kPlanNoSplit : 0u;
        if ((rc = make_plan(M, N, K, d->sms, d->pairs, variant, &q, flags, held_of(*d)))) return rc;
        if ((rc = ensure_workspace(*d, q, st))) return rc;
    }
    CUtensorMap mx, my, mc;
    if (!make_maps(q, A, B, M, N, K, &mx, &my, tn) || !make_c_map(q, C, M, N, epi, mx, &mc)) {
        snprintf(g_errbuf, sizeof g_errbuf, "cuTensorMapEncodeTiled failed");
        return BW_ERR_LAUNCH;
    }
    return dispatch(*d, q, mx, my, mc, make_params(q, M, N, K, C, d->work, d->counters, tn), st, epi);
}

}  // namespace
}  // namespace bw

// ------------------------------------------------------------------ the C ABI
BW_API int bw_gemm_f16(const void* A, const void* B, void* C, int M, int N, int K, void* stream)
{
    return bw::gemm(A, B, C, M, N, K, static_cast<cudaStream_t>(stream), 0);
}

BW_API int bw_gemm_f16_variant(const void* A, const void* B, void* C, int M, int N, int K, void* stream, int variant)
{
    return bw::gemm(A, B, C, M, N, K, static_cast<cudaStream_t>(stream), variant);
}

BW_API int bw_gemm_f16_tn(const void* A, const void* B, void* C, int M, int N, int K, void* stream)
{
    return bw::gemm(A, B, C, M, N, K, static_cast<cudaStream_t>(stream), 0, bw::kEpiF16, true);
}

BW_API int bw_gemm_f16_f32out(const void* A, const void* B, void* C, int M, int N, int K, void* stream)
{
    // the rule without swap-AB: SM-pair tiles at every M, written in fp32
    return bw::gemm(A, B, C, M, N, K, static_cast<cudaStream_t>(stream), 0, bw::kEpiF32);
}

BW_API int bw_gemm_f16_swiglu(const void* A, const void* B, void* C, int M, int N, int K, void* stream)
{
    if (N % 256) return BW_ERR_SHAPE;  // each 256-column tile holds 128 gate and 128 up columns
    return bw::gemm(A, B, C, M, N, K, static_cast<cudaStream_t>(stream), 0, bw::kEpiSwiGLU);
}

BW_API int bw_gemm_variant_count(void) { return bw::kVariants; }

BW_API const char* bw_gemm_variant_name(int v) { return bw::variant_name(v); }

BW_API int bw_gemm_plan(int M, int N, int K, int sms, int variant, bw_plan* out)
{
    return bw::make_plan(M, N, K, sms, sms / 2, variant, out);
}

BW_API int bw_gemm_dirty(void)
{
    bw::DeviceState* d = nullptr;
    if (bw::device_state(&d)) return -1;
    std::lock_guard<std::mutex> lock(bw::g_mu);
    if (!d->counters) return 0;
    int* h = static_cast<int*>(malloc((size_t)d->n_counters * sizeof(int)));
    if (!h) return -1;
    int dirty = 0;
    if (cudaMemcpy(h, d->counters, (size_t)d->n_counters * sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess) {
        for (int i = 0; i < d->n_counters; ++i) dirty += h[i] != 0;
    } else {
        dirty = -1;
    }
    free(h);
    return dirty;
}

BW_API int bw_gemm_status(int* code, unsigned* site, unsigned* block, unsigned* segment)
{
    unsigned s[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpyFromSymbol(s, bw::g_status, sizeof s);
    if (e != cudaSuccess) return bw::cuda_fail(e, "cudaMemcpyFromSymbol (status)");
    if (code) *code = (int)s[0];
    if (site) *site = s[1];
    if (block) *block = s[2];
    if (segment) *segment = s[3];
    return BW_OK;
}

BW_API int bw_gemm_clear_status(void)
{
    const unsigned z[4] = {0, 0, 0, 0};
    cudaError_t e = cudaMemcpyToSymbol(bw::g_status, z, sizeof z);
    if (e != cudaSuccess) return bw::cuda_fail(e, "cudaMemcpyToSymbol (status)");
    // a call whose wait gave up may have left split-tile counters set (its reducer never came): back to zero, so that
    // the next call's split tiles count their partials from nothing
    bw::DeviceState* d = nullptr;
    if (bw::device_state(&d) == BW_OK) {
        std::lock_guard<std::mutex> lock(bw::g_mu);
        if (d->counters) {
            if ((e = cudaMemset(d->counters, 0, (size_t)d->n_counters * sizeof(int))) != cudaSuccess ||
                (e = cudaDeviceSynchronize()) != cudaSuccess)
                return bw::cuda_fail(e, "cudaMemset (counters)");
        }
    }
    return BW_OK;
}

BW_API unsigned long long bw_gemm_set_wait_limit_ns(unsigned long long ns)
{
    const unsigned long long old = bw::g_wait_ns;
    if (ns > 0) bw::g_wait_ns = ns;
    return old;
}

// ------------------------------------------------------------------ the bounded-wait check
namespace bw {
namespace {

// One warp: lane 0 waits on a barrier that nothing arrives on, through the pipeline's own bounded wait, which gives
// up after limit_ns, records the selftest site in the status word and returns.
__global__ void wait_selftest_kernel(unsigned long long limit_ns)
{
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        abort_flag = 0;
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (threadIdx.x == 0) wait_bounded(&bar, 0, &abort_flag, limit_ns, site(kSiteSelftest, 0, 0), -1);
}

}  // namespace
}  // namespace bw

BW_API int bw_wait_selftest(unsigned long long limit_ns, void* stream)
{
    bw::DeviceState* d = nullptr;
    if (int st = bw::device_state(&d)) return st;
    if (!d->supported) return BW_ERR_DEVICE;
    if (limit_ns == 0) limit_ns = bw::g_wait_ns;
    if (limit_ns > 10000000000ull) return BW_ERR_ARG;
    if (int st = bw_gemm_clear_status()) return st;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    bw::wait_selftest_kernel<<<1, 32, 0, s>>>(limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return bw::cuda_fail(e, "wait selftest");
    int code = 0;
    unsigned where = 0;
    if (int st = bw_gemm_status(&code, &where, nullptr, nullptr)) return st;
    if (code == BW_ERR_TIMEOUT && where == bw::site(bw::kSiteSelftest, 0, 0)) return BW_ERR_TIMEOUT;
    snprintf(bw::g_errbuf, sizeof bw::g_errbuf, "wait selftest: status %d at site 0x%x", code, where);
    return BW_ERR_LAUNCH;
}

BW_API const char* bw_status_string(int status)
{
    switch (status) {
    case BW_OK: return "ok";
    case BW_ERR_SHAPE: return "shape not supported (M, N, K positive; N % 64 and K % 64 must be 0)";
    case BW_ERR_LAUNCH: return "CUDA error (see bw_last_error_string)";
    case BW_ERR_TIMEOUT: return "a bounded wait on a barrier gave up (see bw_gemm_status)";
    case BW_ERR_ARG: return "bad argument (null or misaligned pointer, unknown variant)";
    case BW_ERR_DEVICE: return "the current device is not an sm_100 GPU";
    case BW_ERR_SCRATCH: return "the call needs more scratch than the no-allocation entry's fixed array holds";
    default: return "unknown status";
    }
}

BW_API const char* bw_last_error_string(void) { return bw::g_errbuf; }

// ------------------------------------------------------------------ the entry point that allocates nothing
// For callers that may not call cudaMalloc (see bw_gemm_f16_noalloc in bwgemm.h): the scratch of split tiles lives in
// one fixed array compiled into this library.  In host code `g_bw_noalloc_scratch` only names the array; the kernel
// gets its device address, looked up once per device with cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_bw_noalloc_scratch[BW_NOALLOC_SCRATCH_BYTES + 4 * BW_NOALLOC_COUNTERS];

namespace bw {
namespace {
void* g_noalloc_addr[kMaxDevices];  // the array's device address per device, 0 until the first call there

int noalloc_gemm(const void* A, const void* B, void* C, int M, int N, int K, cudaStream_t st)
{
    if (!shape_ok(M, N, K)) return BW_ERR_SHAPE;
    if (!A || !B || !C || (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
                           reinterpret_cast<uintptr_t>(C)) % 16)
        return BW_ERR_ARG;
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    bw_plan q = {}, rule = {};
    void* scratch = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if ((rc = pair_occupancy(*d))) return rc;
        rc = make_plan_capped(M, N, K, d->sms, d->pairs, &q, BW_NOALLOC_SCRATCH_BYTES, BW_NOALLOC_COUNTERS,
                              held_of(*d), &rule);
        if (rc == BW_ERR_SCRATCH) {
            snprintf(g_errbuf, sizeof g_errbuf,
                     "%d x %d x %d: the rule's plan needs %zu bytes of partials and %d counters and no fallback fits; "
                     "the fixed array holds %u and %u", M, N, K, rule.workspace_bytes, rule.counters,
                     BW_NOALLOC_SCRATCH_BYTES, BW_NOALLOC_COUNTERS);
            return BW_ERR_SCRATCH;
        }
        if (rc) return rc;
        if (!g_noalloc_addr[dev]) {  // once per device, this device current
            void* ptr = nullptr;
            if ((e = cudaGetSymbolAddress(&ptr, g_bw_noalloc_scratch)) != cudaSuccess)
                return cuda_fail(e, "cudaGetSymbolAddress (no-allocation scratch)");
            g_noalloc_addr[dev] = ptr;
        }
        scratch = g_noalloc_addr[dev];
    }
    float* work = static_cast<float*>(scratch);
    int* counters = reinterpret_cast<int*>(static_cast<unsigned char*>(scratch) + BW_NOALLOC_SCRATCH_BYTES);
    // the counters must start at zero; the array keeps whatever the last call left (a call that gave up part-way
    // may leave some set)
    if (q.counters > 0 && (e = cudaMemsetAsync(counters, 0, (size_t)q.counters * sizeof(int), st)) != cudaSuccess)
        return cuda_fail(e, "cudaMemsetAsync (no-allocation counters)");
    CUtensorMap mx, my, mc;
    if (!make_maps(q, A, B, M, N, K, &mx, &my) || !make_c_map(q, C, M, N, kEpiF16, mx, &mc)) {
        snprintf(g_errbuf, sizeof g_errbuf, "cuTensorMapEncodeTiled failed");
        return BW_ERR_LAUNCH;
    }
    return dispatch(*d, q, mx, my, mc, make_params(q, M, N, K, C, work, counters), st);
}

}  // namespace
}  // namespace bw

BW_API int bw_gemm_f16_noalloc(const void* A, const void* B, void* C, int M, int N, int K, void* stream)
{
    return bw::noalloc_gemm(A, B, C, M, N, K, static_cast<cudaStream_t>(stream));
}

BW_API int bw_gemm_device_plan(int M, int N, int K, int variant, int noalloc, bw_plan* out)
{
    if (!out || variant < 0 || variant >= bw::kVariants || (noalloc && variant != 0)) return BW_ERR_ARG;
    bw::DeviceState* d = nullptr;
    int rc = bw::device_state(&d);
    if (rc) return rc;
    std::lock_guard<std::mutex> lock(bw::g_mu);
    if ((rc = bw::pair_occupancy(*d))) return rc;
    if (noalloc)
        return bw::make_plan_capped(M, N, K, d->sms, d->pairs, out, BW_NOALLOC_SCRATCH_BYTES, BW_NOALLOC_COUNTERS,
                                    bw::held_of(*d));
    return bw::make_plan(M, N, K, d->sms, d->pairs, variant, out, 0u, bw::held_of(*d));
}

#ifdef BW_TRACE
// The timeline of the last launch (a -DBW_TRACE build only; not part of the C ABI of bwgemm.h).
BW_API int bw_trace_read(unsigned long long* dst, int blocks)
{
    cudaError_t e = cudaMemcpyFromSymbol(dst, bw::g_trace, (size_t)blocks * bw::kTraceSlots * sizeof(unsigned long long));
    return e == cudaSuccess ? BW_OK : BW_ERR_LAUNCH;
}
#endif

// ------------------------------------------------------------------ the fused reduce-scatter (kEpiRS)
// One context per rank: this rank's region (the slots, flags, ack and count of gemm_kernel.cuh's RsTable, and the
// table itself; one cudaMalloc so that one CUDA IPC handle exports it) and the other ranks' regions opened from their
// handles.
struct bw_rs {
    int dev, M, N, world, rank;
    int tiles_block;                     // pair tiles in one owner's rows
    size_t flags_off, ack_off, table_off, bytes;  // offsets in a region; its size
    uint8_t* region;                     // this rank's
    uint8_t* peer[bw::kRsMaxWorld];      // every rank's region in this process (this rank's own: region)
    bool connected;                      // the table is written
};

static_assert(sizeof(cudaIpcMemHandle_t) == BW_RS_HANDLE_BYTES, "the IPC handle size of bwgemm.h");

namespace bw {
namespace {

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

int rs_gemm(bw_rs* rs, const void* A, const void* B, void* C, int K, cudaStream_t st)
{
    if (!rs) return BW_ERR_ARG;
    const int M = rs->M, N = rs->N;
    if (!shape_ok(M, N, K)) return BW_ERR_SHAPE;
    if (!A || !B || !C || (reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
                           reinterpret_cast<uintptr_t>(C)) % 16)
        return BW_ERR_ARG;
    if (!rs->connected) {
        snprintf(g_errbuf, sizeof g_errbuf, "the reduce-scatter context is not connected (bw_rs_connect)");
        return BW_ERR_ARG;
    }
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev != rs->dev) {
        snprintf(g_errbuf, sizeof g_errbuf, "the reduce-scatter context belongs to device %d", rs->dev);
        return BW_ERR_ARG;
    }
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    bw_plan q;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if ((rc = pair_occupancy(*d))) return rc;
        if ((rc = make_plan(M, N, K, d->sms, d->pairs, 0, &q, kPlanNoSwap | kPlanNoSplit | kPlanRsWindow,
                            held_of(*d))))
            return rc;
    }
    if (q.kernel != BW_KERNEL_PAIR || q.sk_tiles != 0 || q.bn != 256) {
        snprintf(g_errbuf, sizeof g_errbuf, "the fused reduce-scatter needs whole pair tiles");
        return BW_ERR_LAUNCH;
    }
    CUtensorMap mx, my;
    if (!make_maps(q, A, B, M, N, K, &mx, &my)) {
        snprintf(g_errbuf, sizeof g_errbuf, "cuTensorMapEncodeTiled failed");
        return BW_ERR_LAUNCH;
    }
    Params p = make_params(q, M, N, K, C, nullptr, nullptr);
    p.s.row_shift = ((rs->rank + 1) * (rs->M / rs->world / 256)) % q.tiles_m;  // this rank's own rows last
    p.rs = reinterpret_cast<const RsTable*>(rs->region + rs->table_off);
    return launch_kernel<256, false, true, kEpiRS>(*d, 1u << 24, q, mx, my, mx, p, st);
}

}  // namespace
}  // namespace bw

BW_API int bw_rs_create(int M, int N, int world, int rank, bw_rs** out)
{
    using namespace bw;
    if (!out) return BW_ERR_ARG;
    *out = nullptr;
    if (world < 2 || world > kRsMaxWorld || rank < 0 || rank >= world) return BW_ERR_ARG;
    if (!shape_ok(M, N, 64) || M % (256 * world)) return BW_ERR_SHAPE;
    DeviceState* d = nullptr;
    int rc = device_state(&d);
    if (rc) return rc;
    bw_rs* rs = static_cast<bw_rs*>(calloc(1, sizeof(bw_rs)));
    if (!rs) return BW_ERR_ARG;
    cudaError_t e = cudaGetDevice(&rs->dev);
    if (e != cudaSuccess) {
        free(rs);
        return cuda_fail(e, "cudaGetDevice");
    }
    rs->M = M, rs->N = N, rs->world = world, rs->rank = rank;
    rs->tiles_block = (M / world / 256) * ((N + 255) / 256);
    const size_t nslots = (size_t)rs->tiles_block * (world - 1) * 2;
    rs->flags_off = align_up(nslots * 128 * 256 * sizeof(float), 256);
    rs->ack_off = align_up(rs->flags_off + nslots * sizeof(unsigned), 256);
    rs->table_off = rs->ack_off + 256;  // the ack, count, epoch and done words; then the table
    rs->bytes = align_up(rs->table_off + sizeof(RsTable), 256);
    if ((e = cudaMalloc(reinterpret_cast<void**>(&rs->region), rs->bytes)) != cudaSuccess ||
        (e = cudaMemset(rs->region, 0, rs->bytes)) != cudaSuccess) {
        if (rs->region) cudaFree(rs->region);
        free(rs);
        return cuda_fail(e, "cudaMalloc (reduce-scatter region)");
    }
    rs->peer[rank] = rs->region;
    *out = rs;
    return BW_OK;
}

BW_API size_t bw_rs_region_bytes(const bw_rs* rs) { return rs ? rs->bytes : 0; }

BW_API int bw_rs_handle(const bw_rs* rs, void* handle)
{
    if (!rs || !handle) return BW_ERR_ARG;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, rs->region);
    if (e != cudaSuccess) return bw::cuda_fail(e, "cudaIpcGetMemHandle");
    memcpy(handle, &h, sizeof h);
    return BW_OK;
}

BW_API int bw_rs_connect(bw_rs* rs, const void* handles)
{
    if (!rs || !handles) return BW_ERR_ARG;
    for (int o = 0; o < rs->world; ++o) {
        if (o == rs->rank || rs->peer[o]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)o * BW_RS_HANDLE_BYTES, sizeof h);
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return bw::cuda_fail(e, "cudaIpcOpenMemHandle");
        rs->peer[o] = static_cast<uint8_t*>(ptr);
    }
    // this rank's view of every region, into its own region's table
    bw::RsTable t = {};
    t.world = rs->world;
    t.rank = rs->rank;
    t.rows = rs->M / rs->world;
    for (int o = 0; o < rs->world; ++o) {
        t.slots[o] = reinterpret_cast<float*>(rs->peer[o]);
        t.flags[o] = reinterpret_cast<unsigned*>(rs->peer[o] + rs->flags_off);
        t.ack[o] = reinterpret_cast<unsigned*>(rs->peer[o] + rs->ack_off);
    }
    t.count = reinterpret_cast<unsigned*>(rs->region + rs->ack_off) + 1;
    t.epoch = reinterpret_cast<unsigned*>(rs->region + rs->ack_off) + 2;
    t.done = reinterpret_cast<unsigned*>(rs->region + rs->ack_off) + 3;
    cudaError_t e = cudaMemcpy(rs->region + rs->table_off, &t, sizeof t, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return bw::cuda_fail(e, "cudaMemcpy (reduce-scatter table)");
    rs->connected = true;
    return BW_OK;
}

BW_API int bw_gemm_f16_rs(bw_rs* rs, const void* A, const void* B, void* C, int K, void* stream)
{
    return bw::rs_gemm(rs, A, B, C, K, static_cast<cudaStream_t>(stream));
}

BW_API int bw_rs_destroy(bw_rs* rs)
{
    if (!rs) return BW_OK;
    int rc = BW_OK;
    for (int o = 0; o < rs->world; ++o)
        if (o != rs->rank && rs->peer[o] && cudaIpcCloseMemHandle(rs->peer[o]) != cudaSuccess) rc = BW_ERR_LAUNCH;
    if (rs->region && cudaFree(rs->region) != cudaSuccess) rc = BW_ERR_LAUNCH;
    free(rs);
    return rc;
}
