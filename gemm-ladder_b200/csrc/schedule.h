// schedule.h -- the work of one block of the rung's persistent kernel: which tiles, and which K-blocks of them, in
// which order, and where the partial sums of a tile split over several blocks go.  Host and device: the kernel runs
// it, and the CPU tests run the same code to check that every K-block of every tile is computed exactly once and that
// the partial counts and workspace slots the reducer uses are the ones the writers used.
//
// A block's work: data-parallel whole tiles c, c + P, c + 2P, ... below dp_tiles (P blocks; consecutive tiles run at
// the same time, so blocks that share rows of A or columns of B read them from L2 together), and the other sk_tiles
// tiles, either
//      split-K (splits > 0), done before the whole tiles: each tile's K-blocks cut in `splits` equal ranges; unit
//        u = split * sk_tiles + tile goes to block u % P, so the units running together are the same K range of
//        neighbouring tiles (the shared operands stay shared in L2), or
//      stream-K (splits == 0), done after the whole tiles: the sk_tiles * kblocks K-blocks cut evenly over the P
//        blocks, block c taking
//        [sk_iters c / P, sk_iters (c + 1) / P) -- every block the same work whatever the tile count (used where the
//        operands are streamed once from HBM anyway: the swap-AB path at M <= 128).
// A tile computed by several blocks: each writes its fp32 partial to a workspace slot; the last to finish (a counter
// per tile) sums the partials in a fixed order (split order, or block order) -- so the result is the same bits
// whichever block finishes last -- and writes C.
// Or (ksplit = c > 0, swap-AB only, every tile at once): block c t + r of the grid's clusters of c blocks takes K
// range r of tile t (of c equal ranges), its only segment; the blocks of the cluster add their sums through
// distributed shared memory, no workspace involved.
#pragma once
#if defined(__CUDACC__)
#define BW_HD __host__ __device__
#else
#define BW_HD
#endif

namespace bw {

// The schedule, computed on the host (plan.h) and passed by value.
struct Sched {
    int M, N, K;
    int tiles_m, tiles_n, tiles;
    int kblocks;          // K / 64
    int dp_tiles;         // tiles [0, dp_tiles): whole tiles, round-robin over the blocks
    int sk_tiles;         // tiles [dp_tiles, tiles): split-K or stream-K
    int splits;           // > 0: split-K into this many K ranges; 0: stream-K
    long long sk_iters;   // stream-K: sk_tiles * kblocks, split evenly over the blocks
    int group_rows;       // serpentine group height in rows of tiles; 0: row after row
    int ksplit;           // > 0: each tile's K cut in ksplit ranges on the blocks of a cluster of ksplit (one
                          // segment per block); 0: none
    int row_shift;        // rows of tiles the order is rotated by (the fused reduce-scatter: a rank's own rows last)
    int dyn;              // 1: the split-K units (every tile split, dp_tiles 0) go to whichever block asks next (a
                          // counter in global memory, read by each block's producer), not round-robin
};

// The segment of split-K unit u (split-major: u = split * sk_tiles + tile - dp_tiles).
BW_HD inline void unit_seg(const Sched& s, int u, int& tile, int& k0, int& k1)
{
    const int sp = u / s.sk_tiles, rel = u - sp * s.sk_tiles;
    tile = s.dp_tiles + rel;
    k0 = (int)((long long)sp * s.kblocks / s.splits);
    k1 = (int)((long long)(sp + 1) * s.kblocks / s.splits);
}

// ------------------------------------------------------------------ stream-K bookkeeping
BW_HD inline long long sk_begin(const Sched& s, int c, int P) { return s.sk_iters * c / P; }
// The block whose stream-K share holds iteration g (the largest c with sk_begin(c) <= g).
BW_HD inline int sk_owner(const Sched& s, long long g, int P)
{
    return (int)(((g + 1) * (long long)P - 1) / s.sk_iters);
}
// Block cc's slot for stream-K tile `tile`: 2 cc for the tile its share starts in, 2 cc + 1 for the one it ends in
// (a share covers whole tiles in between, which need no slot).
BW_HD inline int sk_slot(const Sched& s, int cc, int P, int tile)
{
    const int first = s.dp_tiles + (int)(sk_begin(s, cc, P) / s.kblocks);
    return 2 * cc + (tile == first ? 0 : 1);
}

// ------------------------------------------------------------------ tile order
// Serpentine order of hopper/step5.cuh:149-163: groups of group_rows rows of tiles, column after column within a
// group, the odd groups from the last column back; then the rows rotated by row_shift.
BW_HD inline void tile_coords(const Sched& s, int t, int& tm, int& tn)
{
    if (s.group_rows <= 0) {
        tm = t / s.tiles_n;
        tn = t - tm * s.tiles_n;
    } else {
        const int per = s.group_rows * s.tiles_n;
        const int g = t / per, r = t - g * per;
        const int left = s.tiles_m - g * s.group_rows;
        const int rows = left < s.group_rows ? left : s.group_rows;
        tm = g * s.group_rows + r % rows;
        tn = r / rows;
        if (g & 1) tn = s.tiles_n - 1 - tn;
    }
    if (s.row_shift) tm = (tm + s.row_shift) % s.tiles_m;
}

// ------------------------------------------------------------------ one block's segments
struct Seg {
    int tile, k0, k1;
    int unit;  // split-K unit index (split * sk_tiles + tile - dp_tiles), -1 otherwise
};

struct SegIter {
    int next_dp, next_u;
    long long g, g_end;
    BW_HD SegIter(const Sched& s, int c, int P)
        : next_dp(c), next_u(c), g(s.splits > 0 ? 0 : sk_begin(s, c, P)), g_end(s.splits > 0 ? 0 : sk_begin(s, c + 1, P))
    {
    }
    BW_HD bool next(const Sched& s, int P, Seg& seg)
    {
        if (s.ksplit) {  // block c: K range c % ksplit of tile c / ksplit, once
            if (next_u < 0 || next_u >= s.ksplit * s.tiles) return false;
            const int r = next_u % s.ksplit;
            seg.tile = next_u / s.ksplit;
            seg.k0 = (int)((long long)r * s.kblocks / s.ksplit);
            seg.k1 = (int)((long long)(r + 1) * s.kblocks / s.ksplit);
            seg.unit = r * s.tiles + seg.tile;
            next_u = -1;
            return true;
        }
        // split-K units first: the reduction of a split tile then overlaps the block's next tiles (the epilogue
        // of one segment runs while the MMAs of the next fill the other accumulator), not the end of the kernel
        if (s.splits > 0 && next_u < s.sk_tiles * s.splits) {
            const int u = next_u;
            unit_seg(s, u, seg.tile, seg.k0, seg.k1);
            seg.unit = u;
            next_u += P;
            return true;
        }
        if (next_dp < s.dp_tiles) {
            seg.tile = next_dp;
            seg.k0 = 0;
            seg.k1 = s.kblocks;
            seg.unit = -1;
            next_dp += P;
            return true;
        }
        if (s.splits > 0) return false;
        if (g < g_end) {
            const long long rel = g / s.kblocks;
            seg.k0 = (int)(g - rel * s.kblocks);
            const long long left = g_end - g;
            seg.k1 = left < (long long)(s.kblocks - seg.k0) ? seg.k0 + (int)left : s.kblocks;
            seg.tile = s.dp_tiles + (int)rel;
            seg.unit = -1;
            g += seg.k1 - seg.k0;
            return true;
        }
        return false;
    }
};

// ------------------------------------------------------------------ the partials of one tile
// A segment that is not a whole tile: how many partials its tile has (nseg), which of them is this block's (mine),
// and where partial i (in summation order) lives.
struct Fixup {
    int nseg, mine;
    int first;  // stream-K: the first block of the tile
};

BW_HD inline Fixup fixup_of(const Sched& s, int c, int P, const Seg& seg)
{
    Fixup f;
    if (s.splits > 0) {
        f.nseg = s.splits;
        f.mine = seg.unit / s.sk_tiles;
        f.first = 0;
    } else {
        const long long gf = (long long)(seg.tile - s.dp_tiles) * s.kblocks;
        f.first = sk_owner(s, gf, P);
        f.nseg = sk_owner(s, gf + s.kblocks - 1, P) - f.first + 1;
        f.mine = c - f.first;
    }
    return f;
}

BW_HD inline int fixup_slot(const Sched& s, int P, int tile, const Fixup& f, int i)
{
    if (s.splits > 0) return i * s.sk_tiles + (tile - s.dp_tiles);
    return sk_slot(s, f.first + i, P, tile);
}

// ------------------------------------------------------------------ the chunks of a K-split cluster (BW_KSPLIT 1)
// The accumulator's n 16-column chunks in runs, block o of a cluster of c owning [ksplit_run(o), ksplit_run(o + 1))
// (runs of floor or ceil(n / c) chunks, empty ones where n < c).  The owner of chunk ch is the largest o whose run
// starts at or before it: o n / c < ch + 1, so o = ceil((ch + 1) c / n) - 1.
BW_HD inline int ksplit_run(int o, int n, int c) { return o * n / c; }
BW_HD inline int ksplit_owner(int ch, int n, int c) { return ((ch + 1) * c + n - 1) / n - 1; }

// The number of workspace slots a schedule needs.
BW_HD inline long long workspace_slots(const Sched& s, int P)
{
    if (s.sk_tiles <= 0 || s.ksplit) return 0;
    return s.splits > 0 ? (long long)s.sk_tiles * s.splits : 2LL * P;
}

}  // namespace bw
