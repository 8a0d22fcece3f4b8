// schedule.h -- the work of one block of the rung's persistent kernel: which tiles, and which K-blocks of them, in
// which order.  Host and device: the kernel runs it, and the CPU tests run the same code to check that every K-block
// of every tile is computed exactly once and that the stream-K partial counts and slots agree.
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
    long long sk_iters;   // (tiles - dp_tiles) * kblocks: K-blocks split evenly over the blocks (stream-K)
    int group_rows;       // serpentine group height in rows of tiles; 0: row after row
};

// ------------------------------------------------------------------ the schedule
BW_HD inline long long sk_begin(const Sched& s, int c, int P) { return s.sk_iters * c / P; }
// The block whose stream-K share holds iteration g (the largest c with sk_begin(c) <= g).
BW_HD inline int sk_owner(const Sched& s, long long g, int P)
{
    return (int)(((g + 1) * (long long)P - 1) / s.sk_iters);
}

BW_HD inline void tile_coords(const Sched& s, int t, int& tm, int& tn)
{
    if (s.group_rows <= 0) {
        tm = t / s.tiles_n;
        tn = t - tm * s.tiles_n;
        return;
    }
    const int per = s.group_rows * s.tiles_n;
    const int g = t / per, r = t - g * per;
    const int left = s.tiles_m - g * s.group_rows;
    const int rows = left < s.group_rows ? left : s.group_rows;
    tm = g * s.group_rows + r % rows;
    tn = r / rows;
    if (g & 1) tn = s.tiles_n - 1 - tn;
}

// The segments of block c, in order: its data-parallel tiles, then its stream-K share cut at tile boundaries.
struct SegIter {
    int next_dp;
    long long g, g_end;
    BW_HD SegIter(const Sched& s, int c, int P) : next_dp(c), g(sk_begin(s, c, P)), g_end(sk_begin(s, c + 1, P)) {}
    BW_HD bool next(const Sched& s, int P, int& tile, int& k0, int& k1)
    {
        if (next_dp < s.dp_tiles) {
            tile = next_dp;
            k0 = 0;
            k1 = s.kblocks;
            next_dp += P;
            return true;
        }
        if (g < g_end) {
            const long long rel = g / s.kblocks;
            k0 = (int)(g - rel * s.kblocks);
            const long long left = g_end - g;
            k1 = left < (long long)(s.kblocks - k0) ? k0 + (int)left : s.kblocks;
            tile = s.dp_tiles + (int)rel;
            g += k1 - k0;
            return true;
        }
        return false;
    }
};

// Block cc's workspace slot for stream-K tile `tile`: 2 cc for the tile its share starts in, 2 cc + 1 for the one it
// ends in (a share covers whole tiles in between, which need no slot).
BW_HD inline int sk_slot(const Sched& s, int cc, int P, int tile)
{
    const int first = s.dp_tiles + (int)(sk_begin(s, cc, P) / s.kblocks);
    return 2 * cc + (tile == first ? 0 : 1);
}


}  // namespace bw
