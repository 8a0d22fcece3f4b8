// emu.cpp -- the host emulator of the rung's kernel (test infrastructure): gemm_kernel.cuh, unchanged, compiled as
// host C++ with -DBW_EMULATE over emu_runtime.h / ptx_emu.h, and a launcher that plans a call exactly as the library
// does (plan.h), builds the same tensor maps and parameters as csrc/bwgemm.cu, and runs the plan's kernel instance on
// the CPU, clusters in concurrent batches.
//
//   g++ -std=c++20 -O2 -pthread -DBW_EMULATE -fPIC -shared -I<cuda>/include -Iinclude -Igemm-ladder_b200/csrc \
//       gemm-ladder_b200/emu/emu.cpp -o libbwemu.so        (tests/test_emulator.py builds and drives it)
//
// C entry (the same arguments as the library's entries, plus the emulated GPU's SM count):
//   bw_emu_gemm(A, B, C, M, N, K, sms, variant, epi, tn, status[4], &dirty, finding, finding_len)
//     epi: 0 fp16 C, 1 fp32 C, 2 SwiGLU (C is M x N/2);  tn: B given as N x K.
//     Returns a BW_* status; status = the device status word, dirty = counters left non-zero, findings = the number
//     of emulator findings and finding = the first one's text (empty if none).
//   bw_emu_set(name, value): the knobs below.
//   bw_emu_plan(M, N, K, sms, variant, &plan): the plan a call takes.
// Built with -DBW_KSPLIT=1 it runs the K split over clusters of 2 to 8 blocks (plan.h) in place of the halves.
#include <algorithm>
#include <functional>
#include <future>
#include <string>
#include <thread>
#include <vector>

#include "gemm_kernel.cuh"

namespace bw {
namespace {

// ------------------------------------------------------------------ the library's maps and parameters, emulated
void map2(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t box_cols, uint32_t box_rows)
{
    const uint64_t dims[2] = {cols, rows}, strides[2] = {2, cols * 2};
    const uint32_t box[2] = {box_cols, box_rows};
    emu::make_map(m, base, 2, dims, strides, box);
}
void map_blocks(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows, uint32_t blocks)
{
    const uint64_t dims[3] = {64, rows, cols / 64}, strides[3] = {2, cols * 2, 128};
    const uint32_t box[3] = {64, 64, blocks};
    emu::make_map(m, base, 3, dims, strides, box);
}
uint32_t swap_rows(const bw_plan& q) { return (uint32_t)(q.kernel == BW_KERNEL_SWAP_PAIR ? q.bn / 2 : q.bn); }
// the same choice as csrc/bwgemm.cu's make_c_map: C's map for the TMA-store epilogue (fp16 TILE / PAIR plans)
void make_c_map(const bw_plan& q, void* C, int M, int N, int epi, const CUtensorMap& mx, CUtensorMap* mc)
{
    if (BW_EPI_TMA && epi == kEpiF16 && (q.kernel == BW_KERNEL_TILE || q.kernel == BW_KERNEL_PAIR))
        map2(mc, C, N, M, 64, 32);
    else
        *mc = mx;
}
// the same choices as csrc/bwgemm.cu's make_maps
void make_maps(const bw_plan& q, const void* A, const void* B, int M, int N, int K, CUtensorMap* mx, CUtensorMap* my,
               bool tn)
{
    const bool ab = q.kernel == BW_KERNEL_TILE || q.kernel == BW_KERNEL_PAIR;
    if (tn) {
        if (ab) {
            map2(mx, A, K, M, 64, 128);
            map2(my, B, K, N, 64, (uint32_t)(q.kernel == BW_KERNEL_PAIR ? 128 : q.bn));
        } else {
            map2(mx, B, K, N, 64, (uint32_t)(128 * q.wm));
            map2(my, A, K, M, 64, swap_rows(q));
        }
        return;
    }
    if (BW_TMA3D) {
        if (ab) {
            map2(mx, A, K, M, 64, 128);
            map_blocks(my, B, N, K, (uint32_t)(q.kernel == BW_KERNEL_PAIR ? 2 : q.bn / 64));
        } else {
            map_blocks(mx, B, N, K, (uint32_t)(2 * q.wm));
            map2(my, A, K, M, 64, swap_rows(q));
        }
        return;
    }
    if (ab) {
        map2(mx, A, K, M, 64, 128);
        map2(my, B, N, K, 64, 64);
    } else {
        map2(mx, B, N, K, 64, 64);
        map2(my, A, K, M, 64, swap_rows(q));
    }
}

Params make_params(const bw_plan& q, int M, int N, int K, void* C, float* work, int* counters, bool tn)
{
    Params p = {};
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
    p.wait_ns = emu::g_wait_ns;  // long by default (the emulator is slow): a wait that runs out is a protocol fault
    p.rank_wait_ns = emu::g_rank_wait_ns ? emu::g_rank_wait_ns : emu::g_wait_ns;
    return p;
}

// ------------------------------------------------------------------ a launch: clusters in batches
// Blocks of different clusters never wait on one another in a launch (a split tile is summed by whichever block
// finishes it last), so clusters run in concurrent batches across the host's cores, as many at once as keeps the
// host threads to a few thousand (g_cluster_batch, 0: that many; 1: one after another).
inline long long g_cluster_batch = 0;
inline bool g_dry_run = false;  // dispatch and check a plan's instance and geometry, launch nothing
inline long long g_noalloc_cap = -1;  // >= 0: bw_emu_gemm plans as bw_gemm_f16_noalloc does, with this many bytes

template <int BN, bool SWAP, bool PAIR, int EPI, int WM>
int launch(const bw_plan& q, const CUtensorMap& mx, const CUtensorMap& my, const CUtensorMap& mc, const Params& p)
{
    using G = KGeom<BN, SWAP, PAIR, EPI, WM>;
    if (q.smem_bytes != G::kSmemBytes || q.stages != G::kStages || q.tmem_cols != G::kTmemCols || q.wm != WM) {
        emu::finding("plan and kernel geometry disagree (bn %d)", BN);
        return BW_ERR_LAUNCH;
    }
    const int cs = PAIR ? 2 : (SWAP && q.ksplit) ? q.ksplit : 1;
    if (q.grid % cs || cs > emu::kMaxCluster ||
        (q.ksplit && (!SWAP || q.grid != q.ksplit * q.tiles ||
                      plan_ksplit_recv_bytes(BN, WM, q.ksplit) > G::kBarOffset))) {
        emu::finding("a launch the library would refuse (cluster %d, grid %d)", cs, q.grid);
        return BW_ERR_LAUNCH;
    }
    if (g_dry_run) return BW_OK;
    emu::g_smem_limit = q.smem_bytes - 1024;
    const unsigned seq = emu::g_launch_seq++;
    const int cores = (int)std::max(1u, std::thread::hardware_concurrency());
    const int batch = g_cluster_batch > 0 ? (int)g_cluster_batch
                                          : std::max(1, std::min(cores, 4096 / (cs * emu::kCtaThreads)));
    for (int b0 = 0; b0 < q.grid; b0 += batch * cs) {
        const int b1 = std::min(q.grid, b0 + batch * cs);
        std::vector<std::unique_ptr<emu::Cluster>> clusters;
        std::vector<std::unique_ptr<emu::Cta>> ctas;
        for (int c0 = b0; c0 < b1; c0 += cs) {
            clusters.emplace_back(new emu::Cluster());
            emu::Cluster* cl = clusters.back().get();
            cl->size = cs;
            for (int r = 0; r < cs; ++r) {
                ctas.emplace_back(new emu::Cta());
                ctas.back()->rank = r;
                ctas.back()->cluster = cs > 1 ? cl : nullptr;
                cl->cta[r] = ctas.back().get();
            }
        }
        std::vector<std::thread> threads;
        threads.reserve((size_t)(b1 - b0) * emu::kCtaThreads);
        // every thread of the batch waits at a gate until all exist, so that the blocks start together (the order of
        // thread creation gives no block a head start), then by its block's start jitter
        std::promise<void> gate;
        std::shared_future<void> open = gate.get_future().share();
        for (int blk = b0; blk < b1; ++blk)
            for (int t = 0; t < emu::kCtaThreads; ++t)
                threads.emplace_back([&, blk, t, open] {
                    open.wait();
                    emu::t_cta = ctas[(size_t)(blk - b0)].get();
                    emu::t_tid = t;
                    threadIdx = dim3((unsigned)t);
                    blockIdx = dim3((unsigned)blk);
                    gridDim = dim3((unsigned)q.grid);
                    blockDim = dim3((unsigned)emu::kCtaThreads);
                    emu::start_jitter((unsigned)blk, seq);
                    if (emu::g_lead_skew_us > 0 && cs > 1 && blk % cs == 0)
                        std::this_thread::sleep_for(std::chrono::microseconds(emu::g_lead_skew_us));
                    if (emu::g_block_ramp_us > 0)
                        std::this_thread::sleep_for(std::chrono::microseconds((long long)emu::g_block_ramp_us * blk));
                    gemm_kernel<BN, SWAP, PAIR, EPI, WM>(mx, my, mc, p);
                });
        gate.set_value();
        for (auto& th : threads) th.join();
        // every block's queued work (an st.async into another block among it) done before any block goes away
        for (auto& c : ctas) {
            c->tma.finish();
            c->tc.finish();
        }
    }
    return BW_OK;
}

// the plan's kernel instance (csrc/bwgemm.cu's dispatch)
int dispatch(const bw_plan& q, const CUtensorMap& mx, const CUtensorMap& my, const CUtensorMap& mc, const Params& p,
             int epi)
{
    if (epi == kEpiF32) {
        if (q.kernel == BW_KERNEL_PAIR) return launch<256, false, true, kEpiF32, 1>(q, mx, my, mc, p);
        if (q.kernel == BW_KERNEL_TILE && q.bn == 256) return launch<256, false, false, kEpiF32, 1>(q, mx, my, mc, p);
        return BW_ERR_ARG;
    }
    if (epi == kEpiSwiGLU) {
        if (q.sk_tiles != 0) return BW_ERR_ARG;
        if (q.kernel == BW_KERNEL_PAIR) return launch<256, false, true, kEpiSwiGLU, 1>(q, mx, my, mc, p);
        if (q.kernel == BW_KERNEL_TILE && q.bn == 256) return launch<256, false, false, kEpiSwiGLU, 1>(q, mx, my, mc, p);
        return BW_ERR_ARG;
    }
#if BW_PAIR_WIDE
    if (q.kernel == BW_KERNEL_PAIR && q.bn == 512) return launch<512, false, true, kEpiF16, 1>(q, mx, my, mc, p);
#endif
    if (q.kernel == BW_KERNEL_PAIR) return launch<256, false, true, kEpiF16, 1>(q, mx, my, mc, p);
    if (q.kernel == BW_KERNEL_TILE) {
        switch (q.bn) {
        case 64: return launch<64, false, false, kEpiF16, 1>(q, mx, my, mc, p);
        case 128: return launch<128, false, false, kEpiF16, 1>(q, mx, my, mc, p);
        case 256: return launch<256, false, false, kEpiF16, 1>(q, mx, my, mc, p);
        default: return BW_ERR_ARG;
        }
    }
#if BW_SWAP_PAIR
    if (q.kernel == BW_KERNEL_SWAP_PAIR) {
        switch (q.bn * 4 + q.wm) {
        case 64 * 4 + 1: return launch<64, true, true, kEpiF16, 1>(q, mx, my, mc, p);
        case 128 * 4 + 1: return launch<128, true, true, kEpiF16, 1>(q, mx, my, mc, p);
        case 64 * 4 + 2: return launch<64, true, true, kEpiF16, 2>(q, mx, my, mc, p);
        case 128 * 4 + 2: return launch<128, true, true, kEpiF16, 2>(q, mx, my, mc, p);
        default: return BW_ERR_ARG;
        }
    }
#endif
    if (q.wm == 2) {
        switch (q.bn) {
        case 16: return launch<16, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 32: return launch<32, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 48: return launch<48, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 64: return launch<64, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 80: return launch<80, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 96: return launch<96, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 112: return launch<112, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        case 128: return launch<128, true, false, kEpiF16, 2>(q, mx, my, mc, p);
        default: return BW_ERR_ARG;
        }
    }
    switch (q.bn) {
    case 16: return launch<16, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 32: return launch<32, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 48: return launch<48, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 64: return launch<64, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 80: return launch<80, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 96: return launch<96, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 112: return launch<112, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    case 128: return launch<128, true, false, kEpiF16, 1>(q, mx, my, mc, p);
    default: return BW_ERR_ARG;
    }
}

}  // namespace
}  // namespace bw

// Sets a knob of the emulator: "wait_ns" (the kernel's limit of one bounded wait), "rank_wait_ns" (the limit of a wait
// for another rank's flag; 0: wait_ns), "drop_tma" (the n-th TMA / bulk
// completion of each launch never arrives, -1 none), "barrier_limit_ms" (a thread barrier never completed: a finding
// after this long), "cluster_batch" (clusters run at once; 0: as many as the host's cores take), "noalloc_cap"
// (>= 0: fp16 calls of variant 0 plan as bw_gemm_f16_noalloc does, its array this many bytes; -1: the rule),
// "ld_delay_us" (a random pause of up to this long before each tensor-memory load), "start_jitter_us" (each block starts
// up to this much later), "lead_skew_us" (the first block of every cluster starts this much later), "block_ramp_us"
// (block b starts b times this much later), "engine_delay_us"
// (the asynchronous units' longest delay), "force_ksplit" (c * 16 + wm: the K split takes clusters of c and tiles of
// 128 wm columns where they fit; 0: the rule).  Returns 0, or -1 for an unknown name.
extern "C" __attribute__((visibility("default"))) int bw_emu_set(const char* name, long long value)
{
    using namespace bw::emu;
    const std::string n = name ? name : "";
    if (n == "wait_ns") g_wait_ns = (unsigned long long)value;
    else if (n == "rank_wait_ns") g_rank_wait_ns = (unsigned long long)value;
    else if (n == "cluster_batch") bw::g_cluster_batch = value;
    else if (n == "drop_tma") g_drop_tma = value;
    else if (n == "barrier_limit_ms") g_barrier_limit_ms = value;
    else if (n == "noalloc_cap") bw::g_noalloc_cap = value;
    else if (n == "ld_delay_us") g_ld_delay_us = (int)value;
    else if (n == "start_jitter_us") g_start_jitter_us = (int)value;
    else if (n == "lead_skew_us") g_lead_skew_us = (int)value;
    else if (n == "block_ramp_us") g_block_ramp_us = (int)value;
    else if (n == "engine_delay_us") g_engine_delay_us = (int)value;
    else if (n == "force_ksplit") bw::g_emu_force_ksplit = (int)value;
    else return -1;
    return 0;
}

// Plans a call as bw_emu_gemm does (epi kEpiRS: as bw_emu_gemm_rs does, variant and tn unused), makes its tensor maps
// and dispatches the plan to its kernel instance without running it: BW_OK if the maps are within the driver's limits
// and an instance exists whose geometry is the plan's (BW_ERR_ARG / BW_ERR_LAUNCH otherwise; for kEpiRS,
// BW_ERR_LAUNCH also for a plan of other than whole 256 x 256 pair tiles), or the plan's own status.
extern "C" __attribute__((visibility("default"))) int bw_emu_check_plan(int M, int N, int K, int sms, int variant,
                                                                        int epi, int tn)
{
    using namespace bw;
    bw_plan q = {};
    const unsigned flags = epi == kEpiF32      ? kPlanNoSwap
                           : epi == kEpiSwiGLU ? kPlanNoSwap | kPlanNoSplit
                           : epi == kEpiRS     ? kPlanNoSwap | kPlanNoSplit | kPlanRsWindow
                                               : 0u;
    if (epi == kEpiSwiGLU && N % 256) return BW_ERR_SHAPE;
    if (epi == kEpiRS) variant = 0, tn = 0;
    int rc = make_plan(M, N, K, sms, sms / 2, variant, &q, flags);
    if (rc) return rc;
    if (epi == kEpiRS && (q.kernel != BW_KERNEL_PAIR || q.sk_tiles != 0 || q.bn != 256)) return BW_ERR_LAUNCH;
    alignas(64) static const unsigned char dummy[64] = {};
    CUtensorMap mx, my;
    emu::g_findings = 0;
    make_maps(q, dummy, dummy, M, N, K, &mx, &my, tn != 0);  // the driver's limits on a tensor map: findings
    const Params p = make_params(q, M, N, K, nullptr, nullptr, nullptr, tn != 0);
    g_dry_run = true;
    CUtensorMap mc;
    make_c_map(q, const_cast<unsigned char*>(dummy), M, N, epi, mx, &mc);
    rc = epi == kEpiRS ? launch<256, false, true, kEpiRS, 1>(q, mx, my, mx, p) : dispatch(q, mx, my, mc, p, epi);
    g_dry_run = false;
    return rc ? rc : emu::g_findings ? BW_ERR_LAUNCH : BW_OK;
}

// The plan bw_gemm_f16_noalloc takes on the emulated GPU of `sms` SMs, its scratch a fixed array of `work_cap` bytes
// of partials and `counter_cap` counters (the library's: BW_NOALLOC_SCRATCH_BYTES, BW_NOALLOC_COUNTERS): BW_OK, or
// BW_ERR_SCRATCH if no plan fits.
extern "C" __attribute__((visibility("default"))) int bw_emu_noalloc_plan(int M, int N, int K, int sms,
                                                                          long long work_cap, int counter_cap,
                                                                          bw_plan* out)
{
    return bw::make_plan_capped(M, N, K, sms, sms / 2, out, (size_t)work_cap, (unsigned)counter_cap);
}

// The plan the launcher takes for a call on the emulated GPU of `sms` SMs (the rule of this build).
extern "C" __attribute__((visibility("default"))) int bw_emu_plan(int M, int N, int K, int sms, int variant,
                                                                  bw_plan* out)
{
    return bw::make_plan(M, N, K, sms, sms / 2, variant, out);
}

// Runs one call of the rung on the emulated GPU of `sms` SMs.  status[4]: the device status word after the call;
// *dirty: split-tile counters left non-zero; *findings: the emulator's findings (the first one's text in `finding`).
extern "C" __attribute__((visibility("default"))) int bw_emu_gemm(const void* A, const void* B, void* C, int M, int N,
                                                                  int K, int sms, int variant, int epi, int tn,
                                                                  unsigned* status, int* dirty, int* findings,
                                                                  char* finding, int finding_len)
{
    using namespace bw;
    emu::g_findings = 0;
    emu::g_first_finding[0] = 0;
    emu::g_tma_count = 0;
    std::memset(g_status, 0, sizeof g_status);
    bw_plan q = {};
    const unsigned flags = epi == kEpiF32 ? kPlanNoSwap : epi == kEpiSwiGLU ? kPlanNoSwap | kPlanNoSplit : 0u;
    if (epi == kEpiSwiGLU && N % 256) return BW_ERR_SHAPE;
    int rc = g_noalloc_cap >= 0 && epi == kEpiF16 && variant == 0
                 ? make_plan_capped(M, N, K, sms, sms / 2, &q, (size_t)g_noalloc_cap, BW_NOALLOC_COUNTERS)
                 : make_plan(M, N, K, sms, sms / 2, variant, &q, flags);
    if (rc) return rc;
    std::vector<float> work(q.workspace_bytes / sizeof(float) + 4, 0.f);
    std::vector<int> counters((size_t)q.counters + 1, 0);
    CUtensorMap mx, my;
    make_maps(q, A, B, M, N, K, &mx, &my, tn != 0);
    const Params p = make_params(q, M, N, K, C, work.data(), counters.data(), tn != 0);
    CUtensorMap mc;
    make_c_map(q, C, M, N, epi, mx, &mc);
    rc = dispatch(q, mx, my, mc, p, epi);
    if (status) std::memcpy(status, g_status, sizeof g_status);
    if (dirty) *dirty = (int)std::count_if(counters.begin(), counters.begin() + q.counters, [](int v) { return v != 0; });
    if (findings) *findings = emu::g_findings.load();
    if (finding && finding_len > 0) snprintf(finding, (size_t)finding_len, "%s", emu::g_first_finding);
    return rc;
}

// ------------------------------------------------------------------ the fused reduce-scatter over emulated GPUs
// `world` emulated GPUs in one process, each with its own region (the layout of csrc/bwgemm.cu's bw_rs) and status
// word.  Every block of every rank runs at once: an owner's blocks wait for other ranks' blocks.
namespace bw {
namespace {

struct EmuRank {
    std::vector<uint8_t> raw;
    uint8_t* region = nullptr;
    RsTable table = {};
    unsigned status[4] = {0, 0, 0, 0};
};

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

int launch_rs(const bw_plan& q, int world, std::vector<EmuRank>& ranks, const std::vector<CUtensorMap>& mx,
              const std::vector<CUtensorMap>& my, const std::vector<Params>& p, int absent)
{
    using G = KGeom<256, false, true, kEpiRS, 1>;
    if (q.smem_bytes != G::kSmemBytes || q.stages != G::kStages || q.tmem_cols != G::kTmemCols || q.grid % 2) {
        emu::finding("plan and kernel geometry disagree (reduce-scatter)");
        return BW_ERR_LAUNCH;
    }
    emu::g_smem_limit = q.smem_bytes - 1024;
    const unsigned seq = emu::g_launch_seq++;
    std::vector<std::unique_ptr<emu::Cluster>> clusters;
    std::vector<std::unique_ptr<emu::Cta>> ctas;
    std::vector<std::thread> threads;
    std::promise<void> gate;  // as in launch: the threads start together once all exist
    std::shared_future<void> open = gate.get_future().share();
    for (int r = 0; r < world; ++r) {
        if (r == absent) continue;
        for (int c0 = 0; c0 < q.grid; c0 += 2) {
            clusters.emplace_back(new emu::Cluster());
            emu::Cluster* cl = clusters.back().get();
            cl->size = 2;
            for (int k = 0; k < 2; ++k) {
                ctas.emplace_back(new emu::Cta());
                ctas.back()->rank = k;
                ctas.back()->cluster = cl;
                cl->cta[k] = ctas.back().get();
            }
            for (int k = 0; k < 2; ++k)
                for (int t = 0; t < emu::kCtaThreads; ++t)
                    threads.emplace_back([&, r, c0, k, t, cl, open] {
                        open.wait();
                        emu::t_cta = cl->cta[k];
                        emu::t_tid = t;
                        t_status = ranks[r].status;
                        threadIdx = dim3((unsigned)t);
                        blockIdx = dim3((unsigned)(c0 + k));
                        gridDim = dim3((unsigned)q.grid);
                        blockDim = dim3((unsigned)emu::kCtaThreads);
                        emu::start_jitter((unsigned)(r * q.grid + c0 + k), seq);
                        gemm_kernel<256, false, true, kEpiRS, 1>(mx[r], my[r], mx[r], p[r]);
                    });
        }
    }
    gate.set_value();
    for (auto& th : threads) th.join();
    for (auto& c : ctas) {
        c->tma.finish();
        c->tc.finish();
    }
    return BW_OK;
}

}  // namespace
}  // namespace bw

// The fused reduce-scatter on `world` emulated GPUs of `sms` SMs each: rank r's C[r] (M / world x N fp16) = its rows
// of sum_r A[r] B[r], `calls` calls in a row (the epochs and acks of call-to-call reuse); in the last call rank
// `absent` (-1: none) does not run, as a rank that died between calls.  status: world x 4 words (each rank's status
// word after the last call).  Returns a BW_* status.
extern "C" __attribute__((visibility("default"))) int bw_emu_gemm_rs(int world, const void* const* A,
                                                                     const void* const* B, void* const* C, int M,
                                                                     int N, int K, int sms, int calls, int absent,
                                                                     unsigned* status, int* findings, char* finding,
                                                                     int finding_len)
{
    using namespace bw;
    emu::g_findings = 0;
    emu::g_first_finding[0] = 0;
    emu::g_tma_count = 0;
    if (world < 2 || world > kRsMaxWorld || M % (256 * world) || !shape_ok(M, N, K)) return BW_ERR_SHAPE;
    bw_plan q = {};
    int rc = make_plan(M, N, K, sms, sms / 2, 0, &q, kPlanNoSwap | kPlanNoSplit | kPlanRsWindow);
    if (rc) return rc;
    if (q.kernel != BW_KERNEL_PAIR || q.sk_tiles != 0 || q.bn != 256) return BW_ERR_LAUNCH;
    // the regions, laid out as bwgemm.cu's bw_rs_create does
    const int tiles_block = (M / world / 256) * ((N + 255) / 256);
    const size_t nslots = (size_t)tiles_block * (world - 1) * 2;
    const size_t flags_off = align256(nslots * 128 * 256 * sizeof(float));
    const size_t ack_off = align256(flags_off + nslots * sizeof(unsigned));
    const size_t bytes = ack_off + 256;
    std::vector<EmuRank> ranks((size_t)world);
    for (auto& r : ranks) {
        r.raw.assign(bytes + 256, 0);
        r.region = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(r.raw.data()) + 255) & ~uintptr_t(255));
    }
    for (int r = 0; r < world; ++r) {
        RsTable& t = ranks[r].table;
        t.world = world;
        t.rank = r;
        t.rows = M / world;
        for (int o = 0; o < world; ++o) {
            t.slots[o] = reinterpret_cast<float*>(ranks[o].region);
            t.flags[o] = reinterpret_cast<unsigned*>(ranks[o].region + flags_off);
            t.ack[o] = reinterpret_cast<unsigned*>(ranks[o].region + ack_off);
        }
        t.count = reinterpret_cast<unsigned*>(ranks[r].region + ack_off) + 1;
        t.epoch = reinterpret_cast<unsigned*>(ranks[r].region + ack_off) + 2;
        t.done = reinterpret_cast<unsigned*>(ranks[r].region + ack_off) + 3;
    }
    std::vector<CUtensorMap> mx((size_t)world), my((size_t)world);
    std::vector<Params> p((size_t)world);
    for (int e = 1; e <= calls && rc == BW_OK; ++e) {
        for (int r = 0; r < world; ++r) {
            make_maps(q, A[r], B[r], M, N, K, &mx[r], &my[r], false);
            p[r] = make_params(q, M, N, K, C[r], nullptr, nullptr, false);
            p[r].s.row_shift = ((r + 1) * (M / world / 256)) % q.tiles_m;
            p[r].rs = &ranks[r].table;
        }
        rc = launch_rs(q, world, ranks, mx, my, p, e == calls ? absent : -1);
    }
    if (status)
        for (int r = 0; r < world; ++r) std::memcpy(status + 4 * r, ranks[r].status, sizeof ranks[r].status);
    if (findings) *findings = emu::g_findings.load();
    if (finding && finding_len > 0) snprintf(finding, (size_t)finding_len, "%s", emu::g_first_finding);
    return rc;
}
