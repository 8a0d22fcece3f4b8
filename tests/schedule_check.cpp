// schedule_check.cpp -- CPU check of the rung's schedule (gemm-ladder_b200/csrc/schedule.h, the code the kernel runs)
// under the host rule (plan.h): for a shape and a variant, every K-block of every tile is computed by exactly one block,
// the serpentine order is a bijection onto the tile grid, the stream-K partial counts the reducer expects equal the
// partials written, and no two partials share a workspace slot.  Prints "OK <shape>" or the first fault; exit 1 on a fault.
//   schedule_check M N K sms variant [M N K sms variant ...]
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <map>
#include <set>
#include <vector>

#include "plan.h"
#include "schedule.h"

static int check(int M, int N, int K, int sms, int variant)
{
    bw_plan q;
    const int rc = bw::make_plan(M, N, K, sms, sms / 2, variant, &q);
    if (rc) {
        printf("FAULT %d %d %d sms %d v%d: plan status %d\n", M, N, K, sms, variant, rc);
        return 1;
    }
    bw::Sched s = {};
    s.M = M, s.N = N, s.K = K, s.tiles_m = q.tiles_m, s.tiles_n = q.tiles_n, s.tiles = q.tiles;
    s.kblocks = q.kblocks, s.dp_tiles = q.dp_tiles, s.sk_tiles = q.sk_tiles, s.splits = q.splits;
    s.sk_iters = q.sk_iters, s.group_rows = q.group_rows, s.ksplit = q.ksplit;
    if (q.dp_tiles + q.sk_tiles != q.tiles || (q.splits > 0) == (q.sk_iters > 0) && q.sk_tiles > 0) {
        printf("FAULT %dx%dx%d v%d: inconsistent plan\n", M, N, K, variant);
        return 1;
    }
    const int R = q.kernel == BW_KERNEL_PAIR || q.kernel == BW_KERNEL_SWAP_PAIR ? 2 : 1;
    const int P = q.grid / R;
    if (P < 1 || q.grid > sms || q.grid % R) {
        printf("FAULT %dx%dx%d v%d: grid %d\n", M, N, K, variant, P);
        return 1;
    }
    // the tile order: a bijection
    if (q.kernel != BW_KERNEL_SWAP) {
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
    std::map<int, std::vector<int>> partials;  // split tile -> the `mine` index of each partial written
    std::set<int> slots;
    const long long nslots = bw::workspace_slots(s, P);
    for (int c = 0; c < P; ++c) {
        bw::SegIter it(s, c, P);
        bw::Seg sg;
        while (it.next(s, P, sg)) {
            if (sg.tile < 0 || sg.tile >= q.tiles || sg.k0 < 0 || sg.k1 > q.kblocks || sg.k0 >= sg.k1) {
                printf("FAULT %dx%dx%d v%d: block %d segment tile %d k %d..%d\n", M, N, K, variant, c, sg.tile, sg.k0,
                       sg.k1);
                return 1;
            }
            for (int k = sg.k0; k < sg.k1; ++k) cover[(size_t)sg.tile * q.kblocks + k]++;
            const bool whole = sg.k0 == 0 && sg.k1 == q.kblocks;
            if (q.ksplit) {
                // K range r of tile t on block c t + r of one cluster of c = ksplit blocks (block r of the cluster),
                // the ranges in block order, no workspace
                const int ks = q.ksplit, r = c % ks;
                if (q.kernel != BW_KERNEL_SWAP || q.workspace_bytes || q.counters || sg.tile != c / ks || ks < 2 ||
                    ks > 8 || sg.k0 != (int)((long long)r * q.kblocks / ks) ||
                    sg.k1 != (int)((long long)(r + 1) * q.kblocks / ks) || q.grid != ks * q.tiles) {
                    printf("FAULT %dx%dx%d v%d: ksplit block %d tile %d k %d..%d\n", M, N, K, variant, c, sg.tile, sg.k0,
                           sg.k1);
                    return 1;
                }
                continue;
            }
            if (!whole) {
                if (sg.tile < q.dp_tiles) {
                    printf("FAULT %dx%dx%d v%d: a data-parallel tile in part\n", M, N, K, variant);
                    return 1;
                }
                const bw::Fixup f = bw::fixup_of(s, c, P, sg);
                if (f.mine < 0 || f.mine >= f.nseg) {
                    printf("FAULT %dx%dx%d v%d: block %d is partial %d of %d\n", M, N, K, variant, c, f.mine, f.nseg);
                    return 1;
                }
                partials[sg.tile].push_back(f.mine);
                const int slot = bw::fixup_slot(s, P, sg.tile, f, f.mine);
                if (slot < 0 || slot >= nslots || !slots.insert(slot).second) {
                    printf("FAULT %dx%dx%d v%d: slot %d of block %d tile %d\n", M, N, K, variant, slot, c, sg.tile);
                    return 1;
                }
                if ((size_t)(slot + 1) * R * 128 * q.bn * sizeof(float) > q.workspace_bytes) {
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
    for (auto& kv : partials) {
        const int t = kv.first;
        std::vector<int> mine = kv.second;
        std::sort(mine.begin(), mine.end());
        // the reducer's view: nseg partials, indices 0 .. nseg-1 each written once, slots as the writers used
        bw::Seg probe = {t, 0, 0, -1};
        int c0 = -1;
        for (int c = 0; c < P && c0 < 0; ++c) {
            bw::SegIter it(s, c, P);
            bw::Seg sg;
            while (it.next(s, P, sg))
                if (sg.tile == t && !(sg.k0 == 0 && sg.k1 == q.kblocks)) {
                    probe = sg;
                    c0 = c;
                    break;
                }
        }
        const bw::Fixup f = bw::fixup_of(s, c0, P, probe);
        if ((int)mine.size() != f.nseg || (t - q.dp_tiles + 1) * R > q.counters) {
            printf("FAULT %dx%dx%d v%d: tile %d: %zu partials, the reducer expects %d\n", M, N, K, variant, t,
                   mine.size(), f.nseg);
            return 1;
        }
        for (int i = 0; i < f.nseg; ++i)
            if (mine[i] != i || !slots.count(bw::fixup_slot(s, P, t, f, i))) {
                printf("FAULT %dx%dx%d v%d: tile %d partial %d missing\n", M, N, K, variant, t, i);
                return 1;
            }
    }
    printf("OK %d %d %d sms %d v%d kernel %d bn %d grid %d dp %d sk_tiles %d splits %d sk_iters %lld\n", M, N, K, sms,
           variant, q.kernel, q.bn, P, q.dp_tiles, q.sk_tiles, q.splits, q.sk_iters);
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
