// kernel_common.cuh -- what the rung's kernel and its epilogue helpers share: the block's shape and roles, the
// output modes, the kernel parameters, the geometry of each instance (Geom), the TMA load forms, the wait sites and
// the shared-memory matrix descriptors of the stage tiles.  gemm_kernel.cuh describes the kernel as a whole.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include "plan.h"
#include "ptx.cuh"
#include "schedule.h"

namespace bw {

constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiThread0 = 64;  // the first epilogue thread
constexpr int kBK = 64;          // K per stage: one 128-byte swizzle row of fp16

// Epilogue modes: what the kernel writes.
enum : int {
    kEpiF16 = 0,     // C = A B in fp16
    kEpiF32 = 1,     // C = A B in fp32 (row-parallel partial sums)
    kEpiSwiGLU = 2,  // B's tiles of BN columns hold BN/2 gate then BN/2 up columns: C = silu(gate) * up in fp16,
                     // M x N/2 (a gated MLP's activation, from the accumulators: the gateup result never exists)
    kEpiRS = 3,      // the fused reduce-scatter: C (fp16, this rank's M / world rows) = the sum over the ranks of
                     // their A_r B_r, the partials exchanged tile by tile through the ranks' memory (RsTable)
};

constexpr int kRsMaxWorld = 8;

// The fused reduce-scatter of a row-parallel layer (kEpiRS, pair tiles of 256 x 256, whole tiles): every rank computes
// every tile of its partial A_r B_r; owner o = the rank whose rows [o rows, (o + 1) rows) hold the tile.  Owner o's
// region (one allocation, mapped into the other ranks' address spaces):
//   slots  [tile of o's rows][sender j: the other ranks in rank order][block of the pair] x 128 x 256 fp32, each
//          laid out [col / 4][row][4] (a warp's 16-byte stores contiguous)
//   flags  one per slot: the epoch of the call whose partial it holds
//   ack    the last epoch whose slots o has consumed (a sender waits for epoch - 1 before writing)
//   count  tile halves o has consumed in this call
//   epoch  o's calls so far: every block of a call reads it at entry (the call's epoch is one more), the call's last
//          block to finish advances it, so a call replayed from a CUDA graph carries a new epoch each time
//   done   blocks of the current call that have finished
// The table lives in this rank's device memory (written once, when the ranks connect); a call passes its address.
struct RsTable {
    int world, rank;                 // ranks; this one
    int rows;                        // rows of C per owner (M / world, a multiple of 256)
    float* slots[kRsMaxWorld];       // owner o's slots, as this rank addresses them
    unsigned* flags[kRsMaxWorld];    // owner o's flags
    unsigned* ack[kRsMaxWorld];      // owner o's ack word
    unsigned* count;                 // this rank's count
    unsigned* epoch;                 // this rank's epoch word
    unsigned* done;                  // this rank's finished-block count
};

struct Params {
    Sched s;
    void* C;                     // fp16; fp32 for kEpiF32; M x N/2 fp16 for kEpiSwiGLU
    float* work;                 // the partials: workspace_slots() x (PAIR ? 2 : 1) slots of 128 x BN fp32, row-major
    int* counters;               // one per split tile (per block of the pair), zero between calls
    unsigned long long wait_ns;  // the limit of any single wait on a barrier
    unsigned long long rank_wait_ns;  // kEpiRS: the limit of a wait on another rank (its partials, its ack), longer
                                      // than wait_ns: the ranks' processes reach their first call out of step
    int tn;                      // 1: B is N x K row-major (K-major for the tensor core, like A); 0: K x N
    const RsTable* rs;           // kEpiRS only: the ranks' regions
};

__host__ __device__ constexpr int pow2_at_least(int v, int p) { return p >= v ? p : pow2_at_least(v, 2 * p); }

// Optional timeline (compiled in with -DBW_TRACE only): per block, %globaltimer at kernel entry, after set-up, the
// MMA's first full stage, its last commit, the epilogue's end, and the exit.
#ifdef BW_TRACE
constexpr int kTraceSlots = 16;
__device__ unsigned long long g_trace[1024 * kTraceSlots];
#define BW_TRACE_AT(slot) (g_trace[blockIdx.x * kTraceSlots + (slot)] = globaltimer_ns())
#define BW_TRACE_VAL(slot, v) (g_trace[blockIdx.x * kTraceSlots + (slot)] = (unsigned long long)(v))
// a block's slots from an earlier launch are cleared at its entry (a slot no role of this block stamps reads 0)
#define BW_TRACE_CLEAR() \
    for (int i_ = 1; i_ < kTraceSlots; ++i_) g_trace[blockIdx.x * kTraceSlots + i_] = 0ull
#else
#define BW_TRACE_CLEAR() ((void)0)
#define BW_TRACE_VAL(slot, v) ((void)0)
#define BW_TRACE_AT(slot) ((void)0)
#endif

// RSV: bytes of shared memory reserved after the stage ring (the fused reduce-scatter's window).
template <int BN, bool SWAP, bool PAIR, int WM = 1, int RSV = 0>
struct Geom {
    static constexpr int kRanks = PAIR ? 2 : 1;
    static constexpr int kTileM = PAIR ? 256 : 128;          // rows of C per tile (TILE, PAIR)
    static constexpr int kAccN = WM * BN;                    // TMEM columns of one accumulator (SWAP: WM weight
                                                             // blocks of 128 columns, BN tokens each)
    static constexpr int kWN = PAIR && BN > 256 ? BN / 256 : 1;  // PAIR: MMAs of N = 256 across a 512-column tile
    static constexpr int kMmaN = BN / kWN;                       // N of one MMA
    static constexpr int kBPart = BN / kRanks / kWN;             // this block's B columns per MMA (PAIR: 128)
    static constexpr int kXBytes = 128 * WM * kBK * 2;       // this block's MMA-A operand: 128 (x WM) rows x 64 K
    static constexpr int kYBytes = (BN / kRanks) * kBK * 2;  // this block's MMA-B operand: BN (PAIR: BN / 2) x 64 K
    static constexpr int kStageBytes = kXBytes + kYBytes;
    static constexpr int kCStageBytes = SWAP ? 2 * 16 * 128 * 2 : 0;  // swap-AB epilogue transpose buffers
    static constexpr int kRingFit = (BW_SMEM_LIMIT - 1024 - 512 - kCStageBytes - RSV) / kStageBytes;
    static constexpr int kStages = kRingFit < BW_MAX_STAGES ? kRingFit : BW_MAX_STAGES;
    static constexpr int kAccBufs = 2 * kAccN <= 512 ? 2 : 1;  // two accumulators, or one of 512 columns
    // one accumulator of two 256-column halves (a wide pair tile): the halves are released and refilled separately
    static constexpr bool kHalves = kAccBufs == 1 && kWN == 2;
    static constexpr int kTmemCols = pow2_at_least(kAccBufs * kAccN < 32 ? 32 : kAccBufs * kAccN, 32);
    static constexpr int kRingBytes = kStages * kStageBytes;
    static constexpr int kWindowOffset = kRingBytes;         // RSV bytes (kEpiRS: the owner's window)
    static constexpr int kBarOffset = kRingBytes + RSV;
    static constexpr int kNumBars = 2 * kStages + 8 + 2 * kPlanUnitQ;  // full, empty, tmem full x2, tmem empty x2,
                                                                       // drain, reduce, the K split's go / receive,
                                                                       // the unit queue's full and empty
    static constexpr int kSlotBytes = 128 * kAccN * 4;  // one partial of this block's rows
    static constexpr int kRingSlots = kRingBytes / kSlotBytes;  // partials the idle ring holds at once
    static constexpr int kMaxSum = kRingSlots + 1 < 8 ? kRingSlots + 1 : 8;  // partials the bulk reduction sums
    static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
    // swap-AB: the epilogue transposes each 16-column chunk through two 16 x 128 fp16 buffers
    static constexpr int kCStageOffset = (kMiscOffset + 64 + 127) / 128 * 128;
    static constexpr int kSmemBytes = 1024 + kCStageOffset + kCStageBytes;  // + slack to align the stages to 1024 B
    static_assert(BN % 16 == 0 && BN >= 16 && (BN <= 256 || (PAIR && BN == 512 && WM == 1)),
                  "MMA N: a multiple of 16 in [16, 256] (pair tiles of 512 columns: two MMAs of 256)");
    static_assert(SWAP || BN % (64 * kRanks) == 0, "B tiles are boxes of 64 columns (per block)");
    static_assert(!(SWAP && PAIR) || BN == 64 || BN == 128, "swap-AB on a pair: MMA N of 64 or 128, half per block");
    static_assert(WM == 1 || (SWAP && WM == 2), "two weight blocks per tile: swap-AB only");
    static_assert(kYBytes % 1024 == 0 && kXBytes % 1024 == 0, "operand tiles on 1024-byte swizzle atoms");
    static_assert(kStages >= 2 && kSmemBytes <= BW_SMEM_LIMIT, "shared memory");
    static_assert(kTmemCols <= 512, "tensor memory");
};

// The geometry of a kernel instance: the fused reduce-scatter's reserves its window, the fp16 TILE / PAIR epilogue its
// staging buffers for TMA stores of C (BW_EPI_TMA).
template <int BN, bool SWAP, bool PAIR, int EPI>
constexpr bool kEpiTma = BW_EPI_TMA && !SWAP && EPI == kEpiF16;
template <int BN, bool SWAP, bool PAIR, int EPI, int WM = 1>
using KGeom = Geom<BN, SWAP, PAIR, WM,
                   EPI == kEpiRS ? kPlanRsWindowBytes : kEpiTma<BN, SWAP, PAIR, EPI> ? kPlanEpiStageBytes : 0>;

// The 3-D form for the MN-major operand (BW_TMA3D): `n64` is the first 64-column block; the map's box holds the
// stage's blocks.
template <bool PAIR, int HINT>
__device__ __forceinline__ void load_blocks(void* dst, const void* tmap, int n64, int k, uint64_t* bar,
                                            uint32_t bar_cluster, uint64_t policy)
{
    if (PAIR)
        tma_load_3d_pair(dst, tmap, 0, k, n64, bar_cluster);  // (the pair form takes no cache hint here)
    else if (HINT)
        tma_load_3d_hint(dst, tmap, 0, k, n64, bar, policy);
    else
        tma_load_3d(dst, tmap, 0, k, n64, bar);
}

// The L2 policy of a hint setting (0 none, 1 evict-last, 2 evict-first).
__device__ __forceinline__ uint64_t l2_policy(int hint) { return hint == 1 ? policy_evict_last() : policy_evict_first(); }

// A tile load with an optional L2 policy; `bar` is this block's barrier (or, PAIR, the leader's shared::cluster one).
template <bool PAIR, int HINT>
__device__ __forceinline__ void load_tile(void* dst, const void* tmap, int x, int y, uint64_t* bar, uint32_t bar_cluster,
                                          uint64_t policy)
{
    if (PAIR) {
        if (HINT) tma_load_2d_pair_hint(dst, tmap, x, y, bar_cluster, policy);
        else tma_load_2d_pair(dst, tmap, x, y, bar_cluster);
    } else {
        if (HINT) tma_load_2d_hint(dst, tmap, x, y, bar, policy);
        else tma_load_2d(dst, tmap, x, y, bar);
    }
}

// Where a wait gave up: role (0 producer, 1 MMA, 2 epilogue, 7 the wait selftest) << 16 | barrier kind << 8 | index.
enum : uint32_t { kSiteSelftest = 7u };
__host__ __device__ __forceinline__ uint32_t site(uint32_t role, uint32_t kind, uint32_t idx)
{
    return role << 16 | kind << 8 | idx;
}

// A wait on a barrier that only bounds time (used to drain copies and MMAs in flight after an abort, before the
// shared and tensor memory they write is given up).  What it waits for is already issued, so it waits at least 1 s
// whatever the limit of the pipeline's waits: a short limit that caught a stall must not cut the drain short.
__device__ __forceinline__ void wait_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns)
{
    const uint32_t b = smem_u32(bar);
    const uint64_t t0 = globaltimer_ns();
    if (limit_ns < 1000000000ull) limit_ns = 1000000000ull;
    while (!mbar_try_wait(b, parity))
        if (globaltimer_ns() - t0 > limit_ns) return;
}

// ------------------------------------------------------------------ descriptors of the stage tiles
// K-major tile (rows of 64 fp16 = 128 bytes, 8-row swizzle atoms of 1024 bytes): the k-th K16 slice starts 32 bytes in.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int k) { return smem_desc_sw128(tile + 32u * k, 16u, 1024u); }
// MN-major tile (boxes of 64 MN x 64 K, 8 KB each; within a box K-row r at 128 r): the k-th K16 slice is 16 rows on;
// leading byte offset = the next 64 MN (8192), stride byte offset = the next 8 K-rows (1024).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int k) { return smem_desc_sw128(tile + 2048u * k, 8192u, 1024u); }

}  // namespace bw
