// gemm_kernel.cuh -- the rung's sm_100a GEMM kernel: C = A B, A (M x K) and B (K x N) fp16 row-major, fp32
// accumulation in tensor memory, C (M x N) fp16 row-major (the judge's convention, judge/judge.cu:5-7).
//
// One persistent block per SM, 6 warps with fixed roles:
//   warp 0      TMA producer: fills a ring of STAGES shared-memory stages (full / empty mbarriers).
//   warp 1      allocates tensor memory, then one thread issues tcgen05.mma (128 x BN x 16 per instruction) into one
//               of two accumulators and commits each stage back to the producer and each finished tile to the
//               epilogue.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32 (w % 4) .. +31), fp32 -> fp16
//               round-to-nearest, stores to C; the accumulator is released as soon as it is read, so the next tile's
//               MMA overlaps this tile's stores.
//
// Two operand forms (the reference's tiles and transposed bands, hopper/step7.cuh:429-631 and :671-910):
//   SWAP = false  MMA-A = a 128-row tile of A (K-major), MMA-B = a BN-column tile of B (MN-major: B is K x N with N
//                 contiguous).  TMEM lane = row of C, TMEM column = column of C.
//   SWAP = true   for M <= 128: C^T = B^T A^T.  MMA-A = 128 columns of B (MN-major), MMA-B = the M rows of A (K-major,
//                 BN = M rounded up to 16).  TMEM lane = column of C, TMEM column = row of C.  The weights fill the
//                 128-row MMA dimension whatever the number of tokens.
//
// Work: tiles in the serpentine order of hopper/step5.cuh:149-163 (groups of rows of tiles, column after column, odd
// groups backwards).  The first dp_tiles tiles go round-robin to the blocks (data-parallel); the K-blocks of the other
// tiles are split evenly over the blocks (stream-K).  A block whose share covers a tile only in part writes an fp32
// partial to its workspace slot; the last block to finish a tile (a counter per tile) sums the tile's partials in
// block order -- a fixed order, so results are bit-for-bit repeatable -- writes C and puts the counter back to zero.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include "ptx.cuh"
#include "schedule.h"

namespace bw {

constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiThread0 = 64;  // the first epilogue thread
constexpr int kBK = 64;          // K per stage: one 128-byte swizzle row of fp16

struct Params {
    Sched s;
    __half* C;
    float* work;               // 2 * gridDim.x slots of 128 * BN floats (stream-K partials)
    int* counters;             // one per stream-K tile, zero between calls
    unsigned long long wait_ns;  // the limit of any single wait on a barrier
};

__host__ __device__ constexpr int pow2_at_least(int v, int p) { return p >= v ? p : pow2_at_least(v, 2 * p); }

template <int BN, bool SWAP>
struct Geom {
    static constexpr int kXBytes = 128 * kBK * 2;  // MMA-A operand tile: 128 rows x 64 K
    static constexpr int kYBytes = BN * kBK * 2;   // MMA-B operand tile: BN rows x 64 K
    static constexpr int kStageBytes = kXBytes + kYBytes;
    static constexpr int kStages = (204800 / kStageBytes) < 12 ? (204800 / kStageBytes) : 12;
    static constexpr int kTmemCols = pow2_at_least(2 * BN < 32 ? 32 : 2 * BN, 32);  // two accumulators
    static constexpr int kBarOffset = kStages * kStageBytes;
    static constexpr int kNumBars = 2 * kStages + 5;  // full, empty, tmem full x2, tmem empty x2, drain
    static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
    static constexpr int kSmemBytes = 1024 + kMiscOffset + 32;  // + slack to align the stages to 1024 bytes
    static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "MMA N: a multiple of 16 in [16, 256] at M = 128");
    static_assert(SWAP || BN % 64 == 0, "B tiles are boxes of 64 columns");
    static_assert(kYBytes % 1024 == 0 && kXBytes % 1024 == 0, "operand tiles on 1024-byte swizzle atoms");
    static_assert(kStages >= 2 && kSmemBytes <= 227 * 1024, "shared memory");
    static_assert(kTmemCols <= 512, "tensor memory");
};

// Where a wait gave up: role (0 producer, 1 MMA, 2 epilogue) << 16 | barrier kind << 8 | index.
__device__ __forceinline__ uint32_t site(uint32_t role, uint32_t kind, uint32_t idx) { return role << 16 | kind << 8 | idx; }

// A wait on a barrier that only bounds time (used to drain copies in flight after an abort).
__device__ __forceinline__ void wait_drain(uint64_t* bar, uint32_t parity, uint64_t limit_ns)
{
    const uint32_t b = smem_u32(bar);
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(b, parity))
        if (globaltimer_ns() - t0 > limit_ns) return;
}

// ------------------------------------------------------------------ descriptors of the stage tiles
// K-major tile (rows of 64 fp16 = 128 bytes, 8-row swizzle atoms of 1024 bytes): the k-th K16 slice starts 32 bytes in.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int k) { return smem_desc_sw128(tile + 32u * k, 16u, 1024u); }
// MN-major tile (boxes of 64 MN x 64 K, 8 KB each; within a box K-row r at 128 r): the k-th K16 slice is 16 rows on;
// leading byte offset = the next 64 MN (8192), stride byte offset = the next 8 K-rows (1024).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int k) { return smem_desc_sw128(tile + 2048u * k, 8192u, 1024u); }

// ------------------------------------------------------------------ the epilogue's stores
// 16 accumulator columns of TMEM lane `lane` (v) -> C.  Not swapped: C[m0 + lane][n0 + c0 .. +15], two 16-byte stores.
// Swapped: C[c0 + j][n0 + lane] for j < 16, one fp16 each (a warp writes 64 contiguous bytes per row of C).
template <int BN, bool SWAP>
__device__ __forceinline__ void store_chunk(const Params& p, int tm, int tn, int lane, int c0, const float (&v)[16])
{
    const Sched& s = p.s;
    if (!SWAP) {
        const int m = tm * 128 + lane, n = tn * BN + c0;
        if (m >= s.M || n >= s.N) return;
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const __half2 x = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            h[j] = *reinterpret_cast<const uint32_t*>(&x);
        }
        uint4* dst = reinterpret_cast<uint4*>(p.C + (size_t)m * s.N + n);
        dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
        dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
    } else {
        const int n = tn * 128 + lane;
        if (n >= s.N) return;
        __half* col = p.C + n;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int m = c0 + j;
            if (m < s.M) col[(size_t)m * s.N] = __float2half_rn(v[j]);
        }
    }
}

// ------------------------------------------------------------------ the kernel
template <int BN, bool SWAP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmy, const Params p)
{
    using G = Geom<BN, SWAP>;
    constexpr int S = G::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kBarOffset);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kMiscOffset);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* reduce_flag = abort_flag + 1;
    volatile int* epi_go = abort_flag + 2;  // two slots, alternating by segment

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Sched& s = p.s;
    const int P = gridDim.x, c = blockIdx.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);   // the producer's arrive.expect_tx; the TMA bytes complete it
            mbar_init(&empty[i], 1);  // one tcgen05.commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);     // one tcgen05.commit at the end of a segment
            mbar_init(&tempty[i], 128);  // every epilogue thread, once its loads of the accumulator are done
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        *reduce_flag = 0;
        epi_go[0] = epi_go[1] = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmx);
        prefetch_tmap(&tmy);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, G::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer (one thread)
        if (lane == 0) {
            SegIter it(s, c, P);
            int stage = 0, issued = 0, seg = 0, tile, k0, k1;
            uint32_t ph = 0;
            bool ok = true;
            while (ok && it.next(s, P, tile, k0, k1)) {
                int tm, tn;
                if (SWAP) {
                    tm = 0;
                    tn = tile;
                } else {
                    tile_coords(s, tile, tm, tn);
                }
                for (int kb = k0; kb < k1; ++kb) {
                    if (!wait_bounded(&empty[stage], ph ^ 1u, abort_flag, p.wait_ns, site(0, 1, stage), seg)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sx = smem + stage * G::kStageBytes;
                    uint8_t* sy = sx + G::kXBytes;
                    mbar_arrive_expect_tx(&full[stage], G::kStageBytes);
                    if (!SWAP) {
                        tma_load_2d(sx, &tmx, kb * kBK, tm * 128, &full[stage]);  // A: 64 K x 128 rows
#pragma unroll
                        for (int j = 0; j < BN / 64; ++j)  // B: 64 columns x 64 K per box
                            tma_load_2d(sy + j * 8192, &tmy, tn * BN + 64 * j, kb * kBK, &full[stage]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 2; ++j)  // B: 128 columns as two boxes of 64 columns x 64 K
                            tma_load_2d(sx + j * 8192, &tmx, tn * 128 + 64 * j, kb * kBK, &full[stage]);
                        tma_load_2d(sy, &tmy, kb * kBK, 0, &full[stage]);  // A: 64 K x BN rows (M <= BN)
                    }
                    ++issued;
                    if (++stage == S) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
                ++seg;
            }
            if (!ok) {  // let the loads in flight land before the block leaves
                const int n = issued < S ? issued : S;
                for (int i = 1; i <= n; ++i) {
                    const int q = issued - i;
                    wait_drain(&full[q % S], (uint32_t)((q / S) & 1), p.wait_ns);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer (one thread)
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16_f32(128, BN, SWAP, !SWAP);
            SegIter it(s, c, P);
            int stage = 0, acc = 0, seg = 0, tile, k0, k1;
            uint32_t ph = 0, aph = 0;
            bool ok = true;
            while (ok && it.next(s, P, tile, k0, k1)) {
                if (!wait_bounded(&tempty[acc], aph ^ 1u, abort_flag, p.wait_ns, site(1, 3, acc), seg)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * BN);
                for (int kb = k0; kb < k1; ++kb) {
                    if (!wait_bounded(&full[stage], ph, abort_flag, p.wait_ns, site(1, 0, stage), seg)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sx = smem_u32(smem + stage * G::kStageBytes), sy = sx + G::kXBytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        const uint64_t ad = SWAP ? desc_mnmajor(sx, k) : desc_kmajor(sx, k);
                        const uint64_t bd = SWAP ? desc_kmajor(sy, k) : desc_mnmajor(sy, k);
                        mma_f16(d, ad, bd, idesc, (kb > k0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(&empty[stage]);  // the stage is free once these MMAs have read it
                    if (++stage == S) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                mma_commit(&tfull[acc]);  // the accumulator is complete once every MMA so far has finished
                if (++acc == 2) {
                    acc = 0;
                    aph ^= 1u;
                }
                ++seg;
            }
            if (!ok) {  // let the MMAs in flight finish before the tensor memory is freed
                mma_commit(drain);
                wait_drain(drain, 0, p.wait_ns);
            }
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------- epilogue (warps 2-5, 128 threads)
        const int q = warp & 3;         // the TMEM lane quarter this warp may access
        const int row = q * 32 + lane;  // accumulator row = TMEM lane
        SegIter it(s, c, P);
        int acc = 0, seg = 0, tile, k0, k1;
        uint32_t aph = 0;
        while (it.next(s, P, tile, k0, k1)) {
            // one thread waits (bounded); a named barrier hands its outcome to the other 127, so that an abort
            // takes the whole group out together and no thread is left at a later barrier
            if (threadIdx.x == kEpiThread0)
                epi_go[seg & 1] = wait_bounded(&tfull[acc], aph, abort_flag, p.wait_ns, site(2, 2, acc), seg) ? 1 : 0;
            named_bar_sync(1, 128);
            if (!epi_go[seg & 1]) break;
            tc_fence_after();
            int tm, tn;
            if (SWAP) {
                tm = 0;
                tn = tile;
            } else {
                tile_coords(s, tile, tm, tn);
            }
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
            if (k0 == 0 && k1 == s.kblocks) {
                // a whole tile: straight to C
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    uint32_t r[16];
                    tmem_ld16(tbase + (uint32_t)c0, r);
                    tmem_wait_ld();
                    float v[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
                    store_chunk<BN, SWAP>(p, tm, tn, row, c0, v);
                }
                tc_fence_before();
                mbar_arrive(&tempty[acc]);
            } else {
                // part of a stream-K tile: the fp32 partial to this block's slot, column-major (a warp's 32 lanes
                // write 128 contiguous bytes per column)
                float* w = p.work + (size_t)sk_slot(s, c, P, tile) * (128 * BN);
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 16) {
                    uint32_t r[16];
                    tmem_ld16(tbase + (uint32_t)c0, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) __stcg(w + (size_t)(c0 + j) * 128 + row, __uint_as_float(r[j]));
                }
                tc_fence_before();
                mbar_arrive(&tempty[acc]);
                __threadfence();
                named_bar_sync(1, 128);
                const long long gf = (long long)(tile - s.dp_tiles) * s.kblocks;
                const int cf = sk_owner(s, gf, P), cl = sk_owner(s, gf + s.kblocks - 1, P);
                if (threadIdx.x == kEpiThread0) {
                    const int old = atomicAdd(&p.counters[tile - s.dp_tiles], 1);
                    *reduce_flag = (old == cl - cf) ? 1 : 0;
                }
                named_bar_sync(1, 128);
                if (*reduce_flag) {
                    // the last block of this tile: sum the partials in block order, then C
                    __threadfence();
#pragma unroll 1
                    for (int c0 = 0; c0 < BN; c0 += 16) {
                        float v[16];
                        const float* w0 = p.work + (size_t)sk_slot(s, cf, P, tile) * (128 * BN);
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = __ldcg(w0 + (size_t)(c0 + j) * 128 + row);
                        for (int cc = cf + 1; cc <= cl; ++cc) {
                            const float* wc = p.work + (size_t)sk_slot(s, cc, P, tile) * (128 * BN);
#pragma unroll
                            for (int j = 0; j < 16; ++j) v[j] += __ldcg(wc + (size_t)(c0 + j) * 128 + row);
                        }
                        store_chunk<BN, SWAP>(p, tm, tn, row, c0, v);
                    }
                    if (threadIdx.x == kEpiThread0) p.counters[tile - s.dp_tiles] = 0;
                }
                named_bar_sync(1, 128);
            }
            if (++acc == 2) {
                acc = 0;
                aph ^= 1u;
            }
            ++seg;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, G::kTmemCols);
    }
}

}  // namespace bw
