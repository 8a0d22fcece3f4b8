// plan.h -- the rung's rule (host only, no CUDA): which kernel, tile and schedule a call takes.
//
// The reference picks a kernel per class of shape (step7::choose, hopper/step7.cuh:921-949; step6::choose,
// hopper/step6.cuh:468-488; its 128 x 320 tile where waves x area are smaller, rows7c :921-933).  On the B200:
//   M <= 128   swap-AB (BW_KERNEL_SWAP): the weights' 128 columns per tile fill the MMA's 128 rows and the M tokens its
//              N (rounded up to 16), so small M wastes no tensor-core rows.  The shape streams B from HBM once:
//              - if every tile's two K halves fit the SMs at once (clusters of two), each half on one block and the
//                two sums added through distributed shared memory (ksplit = 2), with tiles of 128 weight columns,
//                else of 256 (wm = 2, two MMAs on each stage of A) if those fit (BW_KSPLIT 1: K cut over clusters
//                of 2 to 8 blocks, the cluster size and tile width of the least estimated time, ksplit_cost);
//              - otherwise the K-blocks of all tiles cut evenly over the SMs (stream-K), with tiles of 256 weight
//                columns from 64 tokens while they outnumber the SMs (A is re-read from L2 once per tile).
//   M > 128    256 x 256 tiles on pairs of SMs (BW_KERNEL_PAIR, tcgen05 cta_group::2), persistent: per SM the
//              operand traffic of a 128 x 128 tile for the work of a 128 x 256 one.  Whole waves of tiles go
//              round-robin (data-parallel); the tiles of the last, partial wave are split in K into `splits` ranges
//              (split-K) when that fills the pairs better than leaving them idle, the cost of each extra partial
//              included -- or, when the tiles make one wave and a part, all of them are cut evenly (stream-K).
//              Options built but not yet measured: stream-K also over a part wave (BW_SK_PART_WAVE 1), and pair tiles
//              of 256 x 512 where their estimated time is lower (BW_PAIR_WIDE 1, pair_time); at M <= 128, the
//              stream-K swap-AB tiles on SM pairs (BW_SWAP_PAIR 1).
// Variants take one mechanism out each, for ablations (the reference's g_var, hopper/step7.cu:1-11).
#pragma once
#include <cstddef>
#include "bwgemm.h"
#include "schedule.h"

// Tuning constants (compile-time; measured on the B200 unless marked as estimates).
#ifndef BW_GROUP_ROWS
#define BW_GROUP_ROWS 8        // rows of tiles per serpentine group (8 vs 16: -20 % DRAM reads at 8192^3)
#endif
#ifndef BW_FIXUP_KB
#define BW_FIXUP_KB 12.0       // the cost of one extra partial of a 256-column tile, in K-blocks of MMA work
#endif
#ifndef BW_SMEM_LIMIT
#define BW_SMEM_LIMIT 232448   // dynamic shared memory per block on sm_100 (227 KB)
#endif
#ifndef BW_MAX_STAGES
#define BW_MAX_STAGES 12
#endif
#ifndef BW_HINT_A
#define BW_HINT_A 0            // L2 policy of the A tiles: 0 none, 1 evict-last, 2 evict-first
#endif
#ifndef BW_HINT_B
#define BW_HINT_B 0            // L2 policy of the B tiles: 0 none, 1 evict-last, 2 evict-first
#endif
#ifndef BW_SWAP_HINT_B
#define BW_SWAP_HINT_B 2       // swap-AB (M <= 128): the weights are read once, evict first (measured: o_m128 -11 %)
#endif

#ifndef BW_EPI_LDW
#define BW_EPI_LDW 64          // epilogue: accumulator columns loaded from tensor memory per wait (16, 32 or 64;
                               // measured: 64 cuts the last tile's epilogue, o_m512 -3 %)
#endif
#ifndef BW_EPI_LINES
#define BW_EPI_LINES 1         // TILE / PAIR epilogue: whole-line stores of C after an in-warp transpose (0: a row
                               // per thread)
#endif
#ifndef BW_SWAP_WM2_MIN
#define BW_SWAP_WM2_MIN 64     // swap-AB tiles of 256 weight columns (two MMAs on one stage of A) from this many tokens:
                               // every 128-column tile re-reads all of A from L2 (0: never)
#endif
#ifndef BW_TMA3D
#define BW_TMA3D 1             // the MN-major operand's 64-column boxes of a stage in one 3-D TMA load (0: one 2-D
                               // load per box; measured: the swap-AB shapes 0.5-3 % faster, the pair shapes even)
#endif
#ifndef BW_PAIR_WIDE
#define BW_PAIR_WIDE 1         // pair tiles of 256 x 512 (two MMAs of N = 256 per K step into one 512-column accumulator)
                               // where their estimated time beats the 256 x 256 tiles' (pair_time) and their schedule
                               // needs no stream-K: a block takes in 48 KB per K-block for twice the math of the 32 KB of
                               // a 256 x 256 tile (measured in back-to-back CUDA graphs under the power cap: config 1
                               // -7 %, 8192^3 -5 %, gateup_m2048 -5 %; stream-K over 512-column tiles, whose partials
                               // are 256 KB per block, +37 % at o_m2048)
#endif
#ifndef BW_PAIR_KB_NS
#define BW_PAIR_KB_NS 409.0        // a 256 x 256 pair tile's K-block (measured: its intake-bound mainloop at 1965 MHz)
#endif
#ifndef BW_PAIR_WIDE_KB_NS
#define BW_PAIR_WIDE_KB_NS 748.0   // a 256 x 512 one's: twice the MMA time of the measured cuBLAS peak (an estimate; with
                                   // it the rule takes the wide tile where it measured faster -- config 1, 8192^3,
                                   // gateup_m2048 -- and not at qkv_m2048 (1 % slower wide) or 4096 x 6144 (even))
#endif
#ifndef BW_PAIR_WIDE_EPI_NS
#define BW_PAIR_WIDE_EPI_NS 1200.0 // the 256 x 512 tile's exposed epilogue, once per wave: the first half's drain (the
                                   // next tile's first-half MMAs overlap the second's) and the catch-up (an estimate)
#endif
#ifndef BW_SWAP_PAIR
#define BW_SWAP_PAIR 0         // swap-AB on SM pairs (cta_group::2, M = 256: each block 128 x wm weight columns, the
                               // tokens, 33 to 128 of them as N = 64 or 128, split over the pair) where the swap-AB
                               // tiles go to stream-K: each block takes in half the tokens (run on the host emulator;
                               // not yet measured)
#endif
#ifndef BW_SK_PART_WAVE
#define BW_SK_PART_WAVE 0      // stream-K over every pair when the tiles make more than half a wave but not a whole one
                               // (o and down at M = 512: 64 tiles on 74 pairs leave 10 idle; run on the host emulator,
                               // not yet measured)
#endif
#ifndef BW_KSPLIT
#define BW_KSPLIT 1            // swap-AB K cut over the blocks of a cluster: 1, clusters of 2 to BW_KSPLIT_MAX blocks,
                               // each summing the cluster's partials of its own run of the accumulator's 16-column
                               // chunks, the cluster size and tile width of the least estimated time (ksplit_cost;
                               // measured against the halves: qkv_m128 -9 %, down_m128 -9 %, o_m16 -5 %); 0, halves
                               // on clusters of two, the second block's sum added by the first
#endif
#ifndef BW_KSPLIT_MAX
#define BW_KSPLIT_MAX 8        // BW_KSPLIT 1: the largest cluster (8, the portable limit)
#endif
// BW_KSPLIT 1's choice of cluster size and tile width: the estimated time of a call (plan.h, ksplit_cost).  The five
// constants were fitted to the times of every valid (cluster size, tile width) of the qkv, o and down weights at
// M = 1 .. 128 on a B200 (back-to-back CUDA graphs): with them the rule's choice is within 1 % of the fastest on 13 of
// the 18 shapes and within 4 % on all (0.55 % slower than the fastest on average).
#ifndef BW_HBM_GBS
#define BW_HBM_GBS 6450.0      // HBM copy bandwidth (measured on this pool's B200s)
#endif
#ifndef BW_SM_INGEST_GBS
#define BW_SM_INGEST_GBS 70.0  // operand bytes one swap-AB block takes in from L2 per second (fitted; the pair kernel's
                               // mainloop measured ~80: 32 KB per K-block in ~400 ns)
#endif
#ifndef BW_DSMEM_GBS
#define BW_DSMEM_GBS 10.0      // bytes one block hands over to the others of its cluster per second (fitted: the whole
                               // hand-over, st.async into their rings and the wait for it)
#endif
#ifndef BW_KS_BLOCK_US
#define BW_KS_BLOCK_US 0.1     // per block of the grid (fitted: more blocks streaming the weights at once cost time)
#endif
#ifndef BW_KS_CLUSTER_US
#define BW_KS_CLUSTER_US 0.5   // per block of a cluster beyond two (fitted: the larger clusters' longer hand-over)
#endif
#ifndef BW_EPI_TMA
#define BW_EPI_TMA 0           // TILE / PAIR fp16 epilogue: each warp's 32 rows x 64 columns of C through a swizzled 4 KB
                               // quarter of a shared-memory staging buffer (two buffers of 16 KB after the stage ring,
                               // alternating by 64-column chunk) and one TMA store per warp and chunk, in place of
                               // whole-line stores from registers (0); the ring loses what the buffers take
#endif
#ifndef BW_PDL
#define BW_PDL 0               // launch with programmatic stream serialisation (not the reduce-scatter kernel): a call's
                               // blocks start on SMs the call ahead of it has left, do their setup (barriers, tensor
                               // memory, descriptor prefetch) and wait (griddepcontrol.wait) for that call to finish
                               // before their first access to global memory (0: the launch waits, as streams do; the
                               // environment's BWGEMM_PDL overrides it).  Measured in back-to-back CUDA graphs: +1.3 %
                               // on the 17 shapes' geomean, up to 6 % on the pair-tile shapes whose last wave leaves
                               // SMs idle, even on the small-M ones.  Off by default: the reference's judge turns such
                               // dependencies between calls into ordinary ones, so the rung's figures are without it
#endif
#ifndef BW_DYN_UNITS
#define BW_DYN_UNITS 0         // swap-AB shapes whose tiles outnumber the clusters (stream-K otherwise): every tile cut
                               // in units of BW_DYN_UNIT_KB K-blocks, each unit taken by whichever block asks next (the
                               // producer's atomic on a counter in global memory), the partials summed in unit order by
                               // the tile's last unit (the same bits whoever ran them).  Static stream-K shares leave the
                               // slowest tenth of the blocks 8-10 us behind the median at gateup_m16, but the units
                               // measured slower still (160.1 against 144.7 us there: 352 against 318 ns per K-block
                               // streamed, and 5.6 us of waits for a free accumulator per block), so off
#endif
#ifndef BW_DYN_UNIT_KB
#define BW_DYN_UNIT_KB 16      // K-blocks per unit (a unit's MMAs take ~5 us at M = 16)
#endif
#ifndef BW_DYN_MAX_COLS
#define BW_DYN_MAX_COLS 64     // only where the accumulator is at most this many columns (a unit's partial <= 32 KB)
#endif
#ifndef BW_DYN_MAX_BYTES
#define BW_DYN_MAX_BYTES (32u << 20)  // the units' partials of a call at most this many bytes (longer units if need be;
                                      // so that the no-allocation entry's array holds them too)
#endif
#ifndef BW_SK_ONE_WAVE
#define BW_SK_ONE_WAVE 1       // stream-K over every tile when they make one full wave and part of another (the
                               // split-K tail's units then double a block's work: measured qkv_m512 -12 %)
#endif

namespace bw {

#ifdef BW_EMULATE
// The host emulator's test knob (emu.cpp, bw_emu_set "force_ksplit"): c * 16 + wm restricts the BW_KSPLIT 1 choice to
// that cluster size and tile width where they fit (0: the rule).  Not compiled into the library.
inline int g_emu_force_ksplit = 0;
#endif

constexpr int kVariants = 8;
inline const char* variant_name(int v)
{
    switch (v) {
    case 0: return "v0: the rule (swap-AB + cluster K halves or stream-K at M <= 128; 256x256 pair tiles + split-K tail above)";
    case 1: return "v1: without split-K / stream-K (whole tiles only, round-robin)";
    case 2: return "v2: without swap-AB (pair tiles at every M)";
    case 3: return "v3: without the serpentine order (tiles row after row)";
    case 4: return "v4: stream-K in place of the split-K tail, of the cluster K halves and of 256-column swap tiles";
    case 5: return "v5: without the SM pair (128x256 tiles on single SMs)";
    case 6: return "v6: 128x64 tiles on single SMs at every M (no swap-AB, no pair)";
    case 7: return "v7: 128x128 tiles on single SMs at every M (no swap-AB, no pair)";
    default: return nullptr;
    }
}

// The kernels' geometry, as gemm_kernel.cuh's Geom computes it (checked against it at launch in bwgemm.cu): the ring
// takes what the 227 KB leave after the alignment slack, the barriers and the swap-AB epilogue's transpose buffers.
inline int plan_stage_bytes(int bn, int ranks, int wm = 1) { return 128 * wm * 64 * 2 + (bn / ranks) * 64 * 2; }
inline int plan_cstage_bytes(bool swap) { return swap ? 2 * 16 * 128 * 2 : 0; }
// The fused reduce-scatter's window (two 32 KB buffers) for the owner's partials, after the stage ring.
constexpr int kPlanRsWindowBytes = 2 * 32768;
// The TMA-store epilogue's staging (BW_EPI_TMA): two buffers of 128 rows x 64 fp16 columns, after the stage ring.
constexpr int kPlanEpiStageBytes = 2 * 16384;
// Entries of a block's queue of units (BW_DYN_UNITS: its producer takes units and passes them to the MMA issuer and the
// epilogue), each with a full and an empty barrier.
constexpr int kPlanUnitQ = 4;
inline int plan_stages(int bn, int ranks, bool swap, int wm = 1, int reserve = 0)
{
    const int s = (BW_SMEM_LIMIT - 1024 - 512 - plan_cstage_bytes(swap) - reserve) / plan_stage_bytes(bn, ranks, wm);
    return s < BW_MAX_STAGES ? s : BW_MAX_STAGES;
}
// Tensor-memory columns for accumulators of acc_n columns: two of them, or one of 512.
inline int plan_tmem_cols(int acc_n)
{
    const int need = 2 * acc_n <= 512 ? 2 * acc_n : acc_n;
    int c = 32;
    while (c < need) c *= 2;
    return c;
}
inline int plan_smem_bytes(int bn, int ranks, bool swap, int wm = 1, int reserve = 0)
{
    const int st = plan_stages(bn, ranks, swap, wm, reserve);
    const int misc = st * plan_stage_bytes(bn, ranks, wm) + reserve + (2 * st + 8 + 2 * kPlanUnitQ) * 8;
    const int cstage = (misc + 64 + 127) / 128 * 128;
    return 1024 + cstage + plan_cstage_bytes(swap);
}

// A K-split cluster of c blocks (swap-AB): the bytes one block receives into its idle stage ring.  BW_KSPLIT 0: the
// second block's whole accumulator (128 x bn x wm fp32) at the first.  BW_KSPLIT 1: the other c - 1 blocks' parts
// of the longest run of 16-column chunks (8 KB each) that one block owns (runs of floor or ceil(chunks / c)).
inline int plan_ksplit_recv_bytes(int bn, int wm, int c)
{
    if (!BW_KSPLIT) return 128 * bn * wm * 4;
    const int chunks = bn * wm / 16;
    return (c - 1) * ((chunks + c - 1) / c) * 8192;
}
inline bool plan_ksplit_fits(int bn, int wm, int c)
{
    return plan_ksplit_recv_bytes(bn, wm, c) <= plan_stages(bn, 1, true, wm) * plan_stage_bytes(bn, 1, wm);
}

// The estimated time (us) of a K-split plan with clusters of c blocks and tiles of 128 wm weight columns: the larger
// of the weights' HBM time and the busiest block's operand intake (its K range of 128 wm weight columns and of the bn
// tokens, both re-read per block), plus that block's hand-over of the chunks it does not own, plus a cost per block of
// the grid and per block of a cluster beyond two.  Every K-split plan streams the weights once, so the intake decides
// between them where it exceeds the HBM time: at M = 128 the tokens cost as much intake per block as the weights of a
// 128-column tile.
inline double ksplit_cost(int M, int N, int K, int bn, int wm, int c)
{
    const double kb = (double)((K / 64 + c - 1) / c);                      // the longest K range, in K-blocks
    const double intake = (128.0 * wm + bn) * 64 * 2 * kb;                  // bytes into the busiest block
    const double hbm = ((double)N * K + (double)M * K + (double)M * N) * 2;  // bytes from / to HBM
    const int chunks = bn * wm / 16;
    const double sent = (double)(chunks - chunks / c) * 8192;               // the busiest sender's pieces
    const int blocks = (N + 128 * wm - 1) / (128 * wm) * c;
    const double t_hbm = hbm / (BW_HBM_GBS * 1e3), t_in = intake / (BW_SM_INGEST_GBS * 1e3);
    return (t_hbm > t_in ? t_hbm : t_in) + sent / (BW_DSMEM_GBS * 1e3) + BW_KS_BLOCK_US * blocks +
           BW_KS_CLUSTER_US * (c - 2);
}

// The shapes the library serves: N and K multiples of 64 (the TMA boxes' widths), any M >= 1.  Rows of A past M
// reach the tensor core as the TMA engine's zero fill and rows of C past M are never stored, so the tokens of a decode
// step (M = 1, 8, ...) need no padding in the caller's memory.
inline bool shape_ok(int M, int N, int K) { return M > 0 && N > 0 && K > 0 && N % 64 == 0 && K % 64 == 0; }

// The reference's candidate rule (hopper/step7.cu:358-361): M % 16 too.  candidate.cu keeps it, so the reference's
// harnesses see the reference's behaviour.
inline bool reference_shape_ok(int M, int N, int K) { return shape_ok(M, N, K) && M % 16 == 0; }

// The split-K factor for a tail of `tail` tiles on P blocks: minimises the tail's time in tile-times,
// ceil(tail s / P) / s, plus the reduction of s partials (each about fixup_kb K-blocks of work for the last block).
inline int tail_splits(int tail, int P, int kblocks, double fixup_kb, int max_sp = 16)
{
    int best = 1;
    double best_cost = 1.0;
    for (int sp = 2; sp <= 16 && sp <= max_sp && sp <= kblocks; ++sp) {
        const double waves = (double)((tail * sp + P - 1) / P);
        const double cost = waves / sp + sp * fixup_kb / kblocks;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = sp;
        }
    }
    return best;
}

// BW_PAIR_WIDE: the estimated time (ns) of `tiles` pair tiles of `bn` columns on `units` pairs, as the rule below
// schedules them: whole waves, then stream-K over one wave and a part (even shares plus one fix-up) or the split-K tail
// tail_splits picks; each wave at kblocks K-blocks of the tile's measured or estimated time, each partial's fix-up at
// BW_FIXUP_KB K-blocks of the 256-column tile per 256 columns (its bytes), and the 512-column tile's exposed epilogue
// once per wave.
inline double pair_time(int tiles, int units, int kblocks, int bn)
{
    const bool wide = bn > 256;
    const double kb_ns = wide ? BW_PAIR_WIDE_KB_NS : BW_PAIR_KB_NS;
    const double fixup_kb = BW_FIXUP_KB * bn / 256;                // as the rule weighs a partial
    const double fixup_ns = BW_FIXUP_KB * bn / 256 * BW_PAIR_KB_NS;  // a partial's write and read
    double t;
    if (tiles % units == 0) {
        t = (double)(tiles / units) * kblocks * kb_ns;
    } else if ((BW_SK_ONE_WAVE && tiles > units && tiles < 2 * units) ||
               (BW_SK_PART_WAVE && 2 * tiles > units && tiles < units)) {
        t = (double)tiles / units * kblocks * kb_ns + fixup_ns;
    } else {
        const int tail = tiles % units;
        const int sp = tail_splits(tail, units, kblocks, fixup_kb);
        const double tail_waves = (double)((tail * sp + units - 1) / units) / sp;
        t = (tiles / units + tail_waves) * kblocks * kb_ns + (sp > 1 ? sp * fixup_ns : 0.0);
    }
    return t + (wide ? (double)((tiles + units - 1) / units) * BW_PAIR_WIDE_EPI_NS : 0.0);
}

// Plan constraints of the entries that need them (on top of the variant).
enum : unsigned {
    kPlanNoSwap = 1u,   // A is the MMA's A operand (fp32 and fused outputs are written by TILE and PAIR only)
    kPlanNoSplit = 2u,  // whole tiles only (a fused epilogue needs the complete sums)
    kPlanNarrow = 4u,   // swap-AB tiles of 128 weight columns, pair tiles of 256 (half the partials' scratch)
    kPlanRsWindow = 8u, // shared memory for the fused reduce-scatter's window (kPlanRsWindowBytes), fewer stages
};

// sms: the SMs; pairs: the pairs of SMs the pair kernel can hold at once (its cluster occupancy); held (BW_KSPLIT 1,
// may be null): held[c], c = 2 .. 8, the clusters of c swap-AB blocks the device holds at once (null: sms / c).
inline int make_plan(int M, int N, int K, int sms, int pairs, int variant, bw_plan* p, unsigned flags = 0,
                     const int* held = nullptr, size_t work_cap = 0)
{
    if (!p || variant < 0 || variant >= kVariants || sms <= 0) return BW_ERR_ARG;
    if (!shape_ok(M, N, K)) return BW_ERR_SHAPE;
    bw_plan q = {};
    q.kblocks = K / 64;
    if (flags & kPlanNoSplit) variant = variant == 0 || variant == 2 ? 1 : variant;
    const bool swap = M <= 128 && variant != 2 && variant < 6 && !(flags & kPlanNoSwap);
    const bool pair = !swap && variant != 5 && variant < 6 && pairs > 0;
    int ranks = 1, units = sms;  // the blocks (or pairs) of the persistent grid
    if (swap) {
        q.kernel = BW_KERNEL_SWAP;
        q.bn = (M + 15) / 16 * 16;
        q.tiles_m = 1;
        q.tiles_n = (N + 127) / 128;
        q.group_rows = 0;
    } else {
        q.kernel = pair ? BW_KERNEL_PAIR : BW_KERNEL_TILE;
        q.bn = variant == 6 ? 64 : variant == 7 ? 128 : 256;
        ranks = pair ? 2 : 1;
        units = pair ? pairs : sms;
        q.tiles_m = (M + 128 * ranks - 1) / (128 * ranks);
        // pair tiles of 512 columns for the fp16 entries, where their estimated time is 2 % below the 256-column ones'
        // and they make no stream-K schedule (whose partials would be 256 KB per block)
        const int tw = q.tiles_m * ((N + 511) / 512);
        const bool wide_sk = (BW_SK_ONE_WAVE && tw > units && tw < 2 * units) ||
                             (BW_SK_PART_WAVE && 2 * tw > units && tw < units);
        if (BW_PAIR_WIDE && pair && (variant == 0 || variant == 3) && !(flags & (kPlanNoSwap | kPlanNarrow)) &&
            N > 256 && units > 0 && !wide_sk &&
            pair_time(tw, units, q.kblocks, 512) < 0.98 * pair_time(q.tiles_m * ((N + 255) / 256), units, q.kblocks, 256))
            q.bn = 512;
        q.tiles_n = (N + q.bn - 1) / q.bn;
        q.group_rows = variant == 3 ? 0 : BW_GROUP_ROWS;
    }
    q.tiles = q.tiles_m * q.tiles_n;
    const long long kb = q.kblocks;
    const bool one_wave = (BW_SK_ONE_WAVE && !swap && q.tiles > units && q.tiles < 2 * units) ||
                          (BW_SK_PART_WAVE && !swap && 2 * q.tiles > units && q.tiles < units);
    const bool stream_k = swap ? variant != 1 : variant == 4 || (variant == 0 && one_wave);
    // swap-AB with every tile at once on clusters of blocks, each block one equal K range of its tile, the blocks'
    // sums added through distributed shared memory (no partials in memory, no counters).  BW_KSPLIT 0: clusters of
    // two, tiles of 128 weight columns if they all fit at once, else of 256 (two MMAs on each stage of A) if those do.
    // BW_KSPLIT 1: clusters of c = 2 .. BW_KSPLIT_MAX, the (c, tile width) of the least estimated time (ksplit_cost;
    // an exact tie goes to the smaller c, then to the narrower tile); c > 2 wants 4 K-blocks per block at least.
    const bool wide_ok = (variant == 0 || variant == 3) && !(flags & kPlanNarrow);
    const int tiles256 = (N + 255) / 256;
    int ks = 0, ks_wm = 0;
    if (swap && variant != 1 && variant != 4 && q.kblocks >= 2) {
#if BW_KSPLIT
        double best = 0.0;
        for (int c = 2; c <= BW_KSPLIT_MAX && c <= 8; ++c) {
            for (int wm = 1; wm <= (wide_ok ? 2 : 1); ++wm) {
#ifdef BW_EMULATE
                if (g_emu_force_ksplit && (c != g_emu_force_ksplit / 16 || wm != g_emu_force_ksplit % 16)) continue;
#endif
                const int tiles = (N + 128 * wm - 1) / (128 * wm);
                const int at_once = held ? held[c] : (c == 2 && pairs > 0) ? pairs : sms / c;
                if (tiles > at_once || (c > 2 && q.kblocks < 4 * c) || !plan_ksplit_fits(q.bn, wm, c)) continue;
                const double t = ksplit_cost(M, N, K, q.bn, wm, c);
                if (!ks || t < best) {
                    best = t;
                    ks = c;
                    ks_wm = wm;
                }
            }
        }
#else
        (void)held;
        const int clusters = pairs > 0 ? pairs : sms / 2;  // clusters of two blocks held at once
        ks_wm = q.tiles <= clusters ? 1 : (wide_ok && tiles256 <= clusters) ? 2 : 0;
        ks = ks_wm ? 2 : 0;
#endif
    }
    if (ks) {
        q.ksplit = ks;
        q.wm = ks_wm;
        q.tiles_n = (N + 128 * q.wm - 1) / (128 * q.wm);
        q.tiles = q.tiles_n;
        q.dp_tiles = 0;
        q.sk_tiles = q.tiles;
        q.splits = ks;
        q.grid = ks * q.tiles;
        q.stages = plan_stages(q.bn, 1, true, q.wm);
        q.smem_bytes = plan_smem_bytes(q.bn, 1, true, q.wm);
        q.tmem_cols = plan_tmem_cols(q.bn * q.wm);
        *p = q;
        return BW_OK;
    }
    // stream-K: tiles of 256 weight columns while they still outnumber the SMs (fewer, larger partials otherwise)
    q.wm = 1;
    if (swap && wide_ok && BW_SWAP_WM2_MIN > 0 && q.bn >= BW_SWAP_WM2_MIN && tiles256 >= sms) {
        q.wm = 2;
        q.tiles_n = tiles256;
        q.tiles = q.tiles_n;
    }
    // BW_SWAP_PAIR: the stream-K swap-AB tiles on SM pairs instead, from 33 tokens, the MMA's N rounded up to 64 or
    // 128 (half per block; the pair MMA's N kept to those two); tiles of 2 x 128 weight columns, or 2 x 256 while those
    // still outnumber the pairs
    if (BW_SWAP_PAIR && swap && wide_ok && pairs > 0 && q.bn > 32 && variant != 1) {
        q.kernel = BW_KERNEL_SWAP_PAIR;
        q.bn = q.bn <= 64 ? 64 : 128;
        ranks = 2;
        units = pairs;
        const int tiles512 = (N + 511) / 512;
        q.wm = BW_SWAP_WM2_MIN > 0 && q.bn >= BW_SWAP_WM2_MIN && tiles512 >= pairs ? 2 : 1;
        q.tiles_n = (N + 256 * q.wm - 1) / (256 * q.wm);
        q.tiles = q.tiles_n;
    }
    // BW_DYN_UNITS: the swap-AB stream-K shapes with small accumulators as units of fixed K ranges, taken dynamically
    const size_t dyn_split_bytes = (size_t)q.tiles * 128 * q.bn * q.wm * sizeof(float);  // one partial of every tile
    int dyn_splits = (q.kblocks + BW_DYN_UNIT_KB - 1) / BW_DYN_UNIT_KB;
    if ((size_t)dyn_splits * dyn_split_bytes > BW_DYN_MAX_BYTES) dyn_splits = (int)(BW_DYN_MAX_BYTES / dyn_split_bytes);
    const bool dyn = BW_DYN_UNITS && swap && stream_k && q.kernel == BW_KERNEL_SWAP && (variant == 0 || variant == 3) &&
                     q.bn * q.wm <= BW_DYN_MAX_COLS && dyn_splits >= 2 && q.tiles % units != 0 &&
                     (!work_cap || dyn_splits * dyn_split_bytes <= work_cap);
    if (variant == 1 || q.tiles % units == 0) {
        q.dp_tiles = q.tiles;  // whole tiles only
    } else if (dyn) {
        q.dp_tiles = 0;
        q.sk_tiles = q.tiles;
        q.splits = dyn_splits;
        q.dyn = 1;
    } else if (stream_k) {
        // stream-K: at M <= 128 over every tile; above, over the last full wave and the partial one
        const int waves = q.tiles / units;
        q.dp_tiles = swap ? 0 : (waves >= 1 ? waves - 1 : 0) * units;
        q.sk_tiles = q.tiles - q.dp_tiles;
        q.sk_iters = (long long)q.sk_tiles * kb;
    } else {
        // split-K over the partial wave, if it pays
        const int tail = q.tiles % units;
        // a fixed scratch of work_cap bytes (0: none) holds at most work_cap / (tail x one partial) splits of the tail
        int max_sp = 16;
        if (work_cap) {
            const size_t per = (size_t)tail * ranks * 128 * q.bn * q.wm * sizeof(float);
            max_sp = work_cap / per < 16 ? (int)(work_cap / per) : 16;
        }
        const int sp = tail_splits(tail, units, q.kblocks, /*fixup_kb=*/BW_FIXUP_KB * q.bn / 256, max_sp);
        if (sp > 1) {
            q.dp_tiles = q.tiles - tail;
            q.sk_tiles = tail;
            q.splits = sp;
        } else {
            q.dp_tiles = q.tiles;
        }
    }
    int P;  // blocks, or pairs, of the grid
    if (q.sk_tiles == 0) {
        P = q.tiles < units ? q.tiles : units;
    } else if (q.splits > 0) {
        const int u = q.sk_tiles * q.splits;
        P = q.dp_tiles > 0 ? units : (u < units ? u : units);
    } else {
        P = q.dp_tiles > 0 ? units : (q.sk_iters < units ? (int)q.sk_iters : units);
        if (q.sk_iters < P) return BW_ERR_ARG;  // every block owns at least one stream-K K-block
    }
    q.grid = P * ranks;
    // shared memory after the ring: the fused reduce-scatter's window, or the fp16 TILE / PAIR epilogue's staging
    const bool epi_tma = BW_EPI_TMA && !swap && !(flags & (kPlanNoSwap | kPlanRsWindow));
    const int reserve = (flags & kPlanRsWindow) ? kPlanRsWindowBytes : epi_tma ? kPlanEpiStageBytes : 0;
    q.stages = plan_stages(q.bn, ranks, swap, q.wm, reserve);
    q.smem_bytes = plan_smem_bytes(q.bn, ranks, swap, q.wm, reserve);
    q.tmem_cols = plan_tmem_cols(q.bn * q.wm);
    q.counters = q.sk_tiles * ranks + (q.dyn ? 2 : 0);  // dyn: the next unit to take, the blocks that finished
    Sched sc = {};
    sc.sk_tiles = q.sk_tiles;
    sc.splits = q.splits;
    q.workspace_bytes = (size_t)workspace_slots(sc, P) * ranks * 128 * q.bn * q.wm * sizeof(float);
    *p = q;
    return BW_OK;
}

// The plan of a call whose split-tile scratch is a fixed array of `work_cap` bytes of partials and `counter_cap`
// counters (bw_gemm_f16_noalloc), the first of these that fits: the rule's plan (variant 0); where the rule's partials
// are twice as large (256-column swap tiles, 512-column pair tiles, swap-AB pairs), the plan on the narrower tiles
// (kPlanNarrow); the plan so far with its split-K tail cut to the splits the array holds; whole tiles (kPlanNoSplit),
// which keep no partials.  BW_ERR_SCRATCH if none fits (whole tiles always do); *rule, if given, receives the rule's
// own plan (what the call would have taken with scratch enough, for the error text and for callers comparing them).
inline int make_plan_capped(int M, int N, int K, int sms, int pairs, bw_plan* p, size_t work_cap,
                            unsigned counter_cap, const int* held = nullptr, bw_plan* rule = nullptr)
{
    auto fits = [&] { return p->workspace_bytes <= work_cap && (unsigned)p->counters <= counter_cap; };
    int rc = make_plan(M, N, K, sms, pairs, 0, p, 0u, held);
    if (rule) *rule = *p;
    if (rc || fits()) return rc;
    unsigned narrow = 0u;  // kPlanNarrow once the rule's double-width tiles have been given up
    if (p->wm > 1 || p->bn > 256 || p->kernel == BW_KERNEL_SWAP_PAIR) {
        narrow = kPlanNarrow;
        if ((rc = make_plan(M, N, K, sms, pairs, 0, p, narrow, held)) || fits()) return rc;
    }
    if ((rc = make_plan(M, N, K, sms, pairs, 0, p, narrow, held, work_cap ? work_cap : 1)) || fits()) return rc;
    if ((rc = make_plan(M, N, K, sms, pairs, 0, p, kPlanNoSplit, held))) return rc;
    return fits() ? BW_OK : BW_ERR_SCRATCH;
}

}  // namespace bw
