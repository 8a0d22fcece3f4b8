// plan.h -- the rung's rule (host only, no CUDA): which kernel, tile and schedule a call takes.
//
// The reference picks a kernel per class of shape (step7::choose, hopper/step7.cuh:921-949; step6::choose,
// hopper/step6.cuh:468-488; its 128 x 320 tile where waves x area are smaller, rows7c :921-933).  On the B200 the
// classes are:
//   M <= 128   swap-AB (BW_KERNEL_SWAP): the weights' 128 columns per tile fill the MMA's 128 rows and the M tokens its
//              N (rounded up to 16), so small M wastes no tensor-core rows; the K-blocks of all tiles are split evenly
//              over the SMs (stream-K), so every SM streams the same share of B from HBM whatever N / 128 is.
//   M > 128    128 x 256 tiles (BW_KERNEL_TILE), persistent; whole waves of tiles round-robin (data-parallel), the
//              last one to two waves' K-blocks split evenly over the SMs (stream-K), so no wave runs part-empty.
// Variants take one mechanism out each, for ablations (the reference's g_var, hopper/step7.cu:1-11).
#pragma once
#include <cstddef>
#include "bwgemm.h"

namespace bw {

constexpr int kVariants = 5;
inline const char* variant_name(int v)
{
    switch (v) {
    case 0: return "v0: the rule (swap-AB + stream-K at M <= 128; 128x256 tiles, data-parallel + stream-K tail above)";
    case 1: return "v1: without stream-K (whole tiles only, round-robin)";
    case 2: return "v2: without swap-AB (128x256 tiles at every M)";
    case 3: return "v3: without the serpentine order (tiles row after row)";
    case 4: return "v4: stream-K over every tile (no data-parallel waves)";
    default: return nullptr;
    }
}

// The kernels' geometry, as gemm_kernel.cuh's Geom computes it (checked against it at compile time in bwgemm.cu).
inline int plan_stage_bytes(int bn) { return 128 * 64 * 2 + bn * 64 * 2; }
inline int plan_stages(int bn)
{
    const int s = 204800 / plan_stage_bytes(bn);
    return s < 12 ? s : 12;
}
inline int plan_tmem_cols(int bn)
{
    int c = 32;
    while (c < 2 * bn) c *= 2;
    return c;
}
inline int plan_smem_bytes(int bn) { return 1024 + plan_stages(bn) * plan_stage_bytes(bn) + (2 * plan_stages(bn) + 5) * 8 + 32; }

inline bool shape_ok(int M, int N, int K)
{
    return M > 0 && N > 0 && K > 0 && M % 16 == 0 && N % 64 == 0 && K % 64 == 0;
}

inline int make_plan(int M, int N, int K, int sms, int variant, bw_plan* p)
{
    if (!p || variant < 0 || variant >= kVariants || sms <= 0) return BW_ERR_ARG;
    if (!shape_ok(M, N, K)) return BW_ERR_SHAPE;
    bw_plan q = {};
    q.kblocks = K / 64;
    const bool swap = M <= 128 && variant != 2;
    if (swap) {
        q.kernel = BW_KERNEL_SWAP;
        q.bn = (M + 15) / 16 * 16;
        q.tiles_m = 1;
        q.tiles_n = (N + 127) / 128;
        q.group_rows = 0;
    } else {
        q.kernel = BW_KERNEL_TILE;
        q.bn = 256;
        q.tiles_m = (M + 127) / 128;
        q.tiles_n = (N + 255) / 256;
        q.group_rows = variant == 3 ? 0 : 16;
    }
    q.tiles = q.tiles_m * q.tiles_n;
    const long long kb = q.kblocks;
    if (variant == 1 || (!swap && variant != 4 && q.tiles % sms == 0)) {
        q.dp_tiles = q.tiles;  // whole tiles only
        q.sk_iters = 0;
        q.grid = q.tiles < sms ? q.tiles : sms;
    } else if (swap || variant == 4) {
        q.dp_tiles = 0;  // every tile's K-blocks split evenly
        q.sk_iters = (long long)q.tiles * kb;
        q.grid = q.sk_iters < sms ? (int)q.sk_iters : sms;
    } else {
        const int waves = q.tiles / sms;  // full waves; keep one of them for stream-K with the partial wave
        q.dp_tiles = (waves >= 1 ? waves - 1 : 0) * sms;
        q.sk_iters = (long long)(q.tiles - q.dp_tiles) * kb;
        q.grid = q.dp_tiles > 0 ? sms : (q.sk_iters < sms ? (int)q.sk_iters : sms);
    }
    // every block owns at least one stream-K K-block (the partial counts rely on it)
    if (q.sk_iters > 0 && q.sk_iters < q.grid) return BW_ERR_ARG;
    q.stages = plan_stages(q.bn);
    q.smem_bytes = plan_smem_bytes(q.bn);
    q.tmem_cols = plan_tmem_cols(q.bn);
    q.counters = q.sk_iters > 0 ? q.tiles - q.dp_tiles : 0;
    q.workspace_bytes = q.sk_iters > 0 ? (size_t)2 * q.grid * 128 * q.bn * sizeof(float) : 0;
    *p = q;
    return BW_OK;
}

}  // namespace bw
