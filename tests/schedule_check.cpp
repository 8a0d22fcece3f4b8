// schedule_check.cpp -- CPU check of the rung's schedule (gemm-ladder_b200/csrc/schedule.h, the code the kernel runs)
// under the host rule (plan.h): for a shape and a variant, every K-block of every tile is computed by exactly one block,
// the serpentine order is a bijection onto the tile grid, the stream-K partial counts the reducer expects equal the
// partials written, and no two partials share a workspace slot.  Prints "OK <shape>" or the first fault; exit 1 on a fault.
//   schedule_check M N K sms variant [M N K sms variant ...]
#include <cstdio>
#include <cstdlib>
#include <map>
#include <set>
#include <vector>

#include "plan.h"
#include "schedule.h"

static int check(int M, int N, int K, int sms, int variant)
{
    bw_plan q;
    const int rc = bw::make_plan(M, N, K, sms, variant, &q);
    if (rc) {
        printf("FAULT %d %d %d sms %d v%d: plan status %d\n", M, N, K, sms, variant, rc);
        return 1;
    }
    bw::Sched s;
    s.M = M, s.N = N, s.K = K, s.tiles_m = q.tiles_m, s.tiles_n = q.tiles_n, s.tiles = q.tiles;
    s.kblocks = q.kblocks, s.dp_tiles = q.dp_tiles, s.sk_iters = q.sk_iters, s.group_rows = q.group_rows;
    const int P = q.grid;
    if (P < 1 || P > sms) {
        printf("FAULT %dx%dx%d v%d: grid %d\n", M, N, K, variant, P);
        return 1;
    }
    // the tile order: a bijection
    if (q.kernel == BW_KERNEL_TILE) {
        std::vector<int> seen((size_t)q.tiles, 0);
        for (int t = 0; t < q.tiles; ++t) {
            int tm, tn;
            bw::tile_coords(s, t, tm, tn);
            if (tm < 0 || tm >= q.tiles_m || tn < 0 || tn >= q.tiles_n || seen[(size_t)tm * q.tiles_n + tn]++) {
                printf("FAULT %dx%dx%d v%d: tile order at %d\n", M, N, K, variant, t);
                return 1;
            }
        }
    }
    std::vector<unsigned char> cover((size_t)q.tiles * q.kblocks, 0);
    std::map<int, int> partials;        // stream-K tile -> partials written
    std::set<int> slots;
    for (int c = 0; c < P; ++c) {
        bw::SegIter it(s, c, P);
        int tile, k0, k1;
        while (it.next(s, P, tile, k0, k1)) {
            if (tile < 0 || tile >= q.tiles || k0 < 0 || k1 > q.kblocks || k0 >= k1) {
                printf("FAULT %dx%dx%d v%d: block %d segment tile %d k %d..%d\n", M, N, K, variant, c, tile, k0, k1);
                return 1;
            }
            for (int k = k0; k < k1; ++k) cover[(size_t)tile * q.kblocks + k]++;
            const bool whole = k0 == 0 && k1 == q.kblocks;
            if (!whole) {
                if (tile < q.dp_tiles) {
                    printf("FAULT %dx%dx%d v%d: a data-parallel tile in part\n", M, N, K, variant);
                    return 1;
                }
                partials[tile]++;
                const int slot = bw::sk_slot(s, c, P, tile);
                if (slot < 0 || slot >= 2 * P || !slots.insert(slot).second) {
                    printf("FAULT %dx%dx%d v%d: slot %d of block %d tile %d\n", M, N, K, variant, slot, c, tile);
                    return 1;
                }
                if ((size_t)(slot + 1) * 128 * q.bn * sizeof(float) > q.workspace_bytes) {
                    printf("FAULT %dx%dx%d v%d: slot %d outside the workspace\n", M, N, K, variant, slot);
                    return 1;
                }
            }
        }
    }
    for (size_t i = 0; i < cover.size(); ++i)
        if (cover[i] != 1) {
            printf("FAULT %dx%dx%d v%d: tile %zu K-block %zu computed %d times\n", M, N, K, variant, i / q.kblocks,
                   i % q.kblocks, cover[i]);
            return 1;
        }
    for (int t = q.dp_tiles; t < q.tiles; ++t) {
        const long long gf = (long long)(t - q.dp_tiles) * q.kblocks;
        const int cf = bw::sk_owner(s, gf, P), cl = bw::sk_owner(s, gf + q.kblocks - 1, P);
        const int expect = cl - cf + 1;
        const int got = partials.count(t) ? partials[t] : 0;
        if (expect == 1 ? got != 0 : got != expect) {
            printf("FAULT %dx%dx%d v%d: stream-K tile %d: %d partials, the reducer expects %d\n", M, N, K, variant, t,
                   got, expect);
            return 1;
        }
        if (t - q.dp_tiles >= q.counters && expect > 1) {
            printf("FAULT %dx%dx%d v%d: tile %d has no counter\n", M, N, K, variant, t);
            return 1;
        }
        // the reducer's slots are the writers' slots
        for (int cc = cf; expect > 1 && cc <= cl; ++cc)
            if (!slots.count(bw::sk_slot(s, cc, P, t))) {
                printf("FAULT %dx%dx%d v%d: tile %d reads slot of block %d never written\n", M, N, K, variant, t, cc);
                return 1;
            }
    }
    printf("OK %d %d %d sms %d v%d kernel %d bn %d grid %d dp %d sk %lld\n", M, N, K, sms, variant, q.kernel, q.bn, P,
           q.dp_tiles, q.sk_iters);
    return 0;
}

int main(int argc, char** argv)
{
    if (argc < 6 || (argc - 1) % 5) {
        fprintf(stderr, "usage: %s M N K sms variant [...]\n", argv[0]);
        return 2;
    }
    int bad = 0;
    for (int i = 1; i + 4 < argc; i += 5)
        bad |= check(atoi(argv[i]), atoi(argv[i + 1]), atoi(argv[i + 2]), atoi(argv[i + 3]), atoi(argv[i + 4]));
    return bad;
}
