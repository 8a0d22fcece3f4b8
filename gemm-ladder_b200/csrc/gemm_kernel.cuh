// gemm_kernel.cuh -- the rung's sm_100a GEMM kernel: C = A B, A (M x K) and B (K x N) fp16 row-major, fp32
// accumulation in tensor memory, C (M x N) fp16 row-major (the judge's convention, judge/judge.cu:5-7).
//
// One persistent block per SM (PAIR: one block pair per two SMs), 6 warps with fixed roles:
//   warp 0      TMA producer: fills a ring of shared-memory stages (full / empty mbarriers).
//   warp 1      allocates tensor memory; one thread issues tcgen05.mma into one of two accumulators (one, for a
//               512-column pair tile) and commits each stage back to the producer and each finished segment to the
//               epilogue.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32 (w % 4) .. +31), fp32 -> fp16
//               round-to-nearest, stores to C (TILE / PAIR: whole lines after an in-warp transpose; SWAP: through a
//               shared-memory transpose); the accumulator is released as soon as it is read, so the next tile's MMA
//               overlaps this tile's stores.
//
// Three operand forms (the reference's tiles and transposed bands, hopper/step7.cuh:429-631 and :671-910):
//   TILE  (SWAP = false, PAIR = false)  MMA 128 x BN x 16: A = a 128-row tile of A (K-major), B = a BN-column tile of
//         B (MN-major: B is K x N with N contiguous).  TMEM lane = row of C, TMEM column = column of C.
//   PAIR  (SWAP = false, PAIR = true)   MMA 256 x BN x 16 on a cluster of two blocks (cta_group::2): each block loads
//         its own 128 rows of A and BN / 2 columns of B, the leader block issues the MMA that reads both blocks'
//         shared memory, each block's tensor memory holds its 128 rows x BN.  Per SM the operand traffic of a
//         256 x 256 tile is that of a 128 x 128 tile.  BN = 512 (BW_PAIR_WIDE): two MMAs of N = 256 per K step, each
//         block holding 128 columns of each, so that accumulator column c is tile column c.
//   SWAP  (SWAP = true)   for M <= 128: C^T = B^T A^T.  MMA-A = 128 columns of B (MN-major), MMA-B = the M rows of A
//         (K-major, BN = M rounded up to 16).  TMEM lane = column of C, TMEM column = row of C.  The weights fill the
//         128-row MMA dimension whatever the number of tokens.  WM = 2: tiles of 256 weight columns, two MMAs on each
//         stage of A, accumulator columns [w * BN, (w + 1) * BN) for weight block w.
//
// Work (schedule.h): data-parallel whole tiles in serpentine order, then split-K or stream-K segments; a tile split
// over several blocks is summed by the last of them in a fixed order, so results are bit-for-bit repeatable.  Or
// (ksplit, SWAP) each tile's K ranges on the blocks of a cluster, their sums exchanged through distributed shared
// memory (st.async into idle stage rings) and added in a fixed order: BW_KSPLIT 0, halves on clusters of two, the
// second block's sum added by the first; BW_KSPLIT 1, clusters of 2 to 8, each block summing its own run of the
// accumulator's 16-column chunks.
// Outputs (EPI): fp16 C; fp32 C; the SwiGLU activation of a gate / up tile; or the fused reduce-scatter of a
// row-parallel layer (kEpiRS: partial tiles of other ranks' rows pushed into their memory, this rank's rows summed).
// Every wait on a barrier is bounded (ptx.cuh, wait_bounded): a stalled pipeline ends the kernel with an error status
// instead of hanging the GPU.
#pragma once
#include "epilogue.cuh"

namespace bw {

// ------------------------------------------------------------------ the kernel
template <int BN, bool SWAP, bool PAIR, int EPI = kEpiF16, int WM = 1>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmy,
                const __grid_constant__ CUtensorMap tmc, const Params p)
{
    using G = KGeom<BN, SWAP, PAIR, EPI, WM>;
    constexpr int AN = G::kAccN;  // accumulator columns (TMEM)
    static_assert(!SWAP || EPI == kEpiF16, "fp32 and SwiGLU outputs are written by the TILE and PAIR forms");
    static_assert(EPI != kEpiSwiGLU || BN % 32 == 0, "SwiGLU pairs the two halves of a tile");
    static_assert(EPI != kEpiRS || (PAIR && BN == 256 && WM == 1), "the fused reduce-scatter runs on pair tiles");
    constexpr int S = G::kStages;
    constexpr int R = G::kRanks;
#ifdef BW_EMULATE
    uint8_t* smem_raw = emu::cta_smem();  // the emulated block's shared memory
#else
    extern __shared__ uint8_t smem_raw[];
#endif
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kBarOffset);
    uint64_t* empty = full + S;
    uint64_t* tfull = empty + S;
    uint64_t* tempty = tfull + 2;
    uint64_t* drain = tempty + 2;
    uint64_t* rbar = drain + 1;  // the bulk reduction's copies of partials
    uint64_t* kgo = rbar + 1;    // K split: the other blocks' rings may take this block's sums
    uint64_t* krecv = rbar + 2;  // K split: the other blocks' sums for this block have arrived
    uint64_t* uq_full = rbar + 3;             // s.dyn: the unit queue's entries, filled by the producer
    uint64_t* uq_empty = uq_full + kPlanUnitQ;  // and read by the MMA issuer and the epilogue
    __half* cst = reinterpret_cast<__half*>(smem + G::kCStageOffset);  // swap-AB epilogue transpose buffers
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kMiscOffset);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* reduce_flag = abort_flag + 1;
    volatile int* epi_go = abort_flag + 2;  // two slots, alternating by segment
    volatile int* recv_flag = abort_flag + 4;  // K split: the other blocks' parts arrived
    volatile int* epi_unit = abort_flag + 5;   // s.dyn: two slots, alternating by segment, beside epi_go
    volatile int* uq = abort_flag + 7;         // s.dyn: the unit queue (kPlanUnitQ entries; -1: no unit left)

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifdef BW_TRACE
    const long long clk0 = clock64();  // SM cycles from entry to exit (slot 15): the block's mean SM clock
#endif
    if (threadIdx.x == 0) {
        BW_TRACE_CLEAR();
        BW_TRACE_AT(0);
    }
    const Sched& s = p.s;
    const int rank = PAIR ? (int)cluster_ctarank() : 0;
    const bool leader = rank == 0;
    const bool kp = SWAP && s.ksplit;                // swap-AB K ranges on the blocks of a cluster
    const int kr = kp ? (int)cluster_ctarank() : 0;  // this block's K range (0: the first)
    const int P = gridDim.x / R, c = blockIdx.x / R;  // the two blocks of a pair share their segments

    // the next call on the stream (launched with programmatic serialisation) may start its setup on free SMs now
    griddep_launch();
    if (threadIdx.x == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], 1);   // the (leader's) producer's arrive.expect_tx; the TMA bytes complete it
            mbar_init(&empty[i], 1);  // one tcgen05.commit
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&tfull[i], 1);       // one tcgen05.commit at the end of a segment
            mbar_init(&tempty[i], 4 * R);  // one arrival per epilogue warp (of both blocks of a pair)
        }
        mbar_init(drain, 1);
        mbar_init(rbar, 1);
        for (int i = 0; i < kPlanUnitQ; ++i) {
            mbar_init(&uq_full[i], 1);   // the producer's arrival once the entry is written
            mbar_init(&uq_empty[i], 2);  // the MMA issuer's and the epilogue's, once they have read it
        }
        mbar_init(kgo, kp ? s.ksplit - 1 : 1);  // a remote arrival from each other block of the cluster
        mbar_init(krecv, 1);  // this block's arrive.expect_tx; the other blocks' st.async bytes complete it
        *abort_flag = 0;
        *reduce_flag = 0;
        epi_go[0] = epi_go[1] = 0;
        *recv_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmx);
        prefetch_tmap(&tmy);
        if (kEpiTma<BN, SWAP, PAIR, EPI>) prefetch_tmap(&tmc);
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, G::kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, G::kTmemCols);
            tmem_relinquish();
        }
    }
    __syncwarp();
    tc_fence_before();
    if (PAIR || kp)
        cluster_sync();  // the leader's barriers exist before the other block's loads and arrivals reach them
    else
        __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // nothing above touches global memory: from here on the call ahead of this one (operands, counters, status word,
    // workspace) has finished and its writes are visible
    griddep_wait();
    if (threadIdx.x == 0) BW_TRACE_AT(1);

    if (warp == 0) {
        // ---------------------------------------------------------- TMA producer (one thread per block)
        if (lane == 0) {
            SegIter it(s, c, P);
            Seg sg;
            const uint64_t pol_a = BW_HINT_A ? l2_policy(BW_HINT_A) : 0ull;
            const uint64_t pol_b = BW_HINT_B ? l2_policy(BW_HINT_B) : 0ull;
            const uint64_t pol_sb = BW_SWAP_HINT_B ? l2_policy(BW_SWAP_HINT_B) : 0ull;
            int stage = 0, issued = 0, seg = 0, qi = 0;
            uint32_t ph = 0;
            bool ok = true;
            // s.dyn: the next unit from the call's counter, passed on through the queue (-1 once none is left)
            auto next = [&](Seg& g) -> bool {
                if (!s.dyn) return it.next(s, P, g);
                const int qs = qi % kPlanUnitQ;
                if (!wait_bounded(&uq_empty[qs], (uint32_t)((qi / kPlanUnitQ) & 1) ^ 1u, abort_flag, p.wait_ns,
                                  site(0, 9, (uint32_t)qs), seg)) {
                    ok = false;
                    return false;
                }
                int u = atomicAdd(p.counters + s.sk_tiles * R, 1);
                if (u >= s.sk_tiles * s.splits) u = -1;
                uq[qs] = u;
                mbar_arrive(&uq_full[qs]);  // release: the readers see the entry after their wait
                ++qi;
                if (u < 0) return false;
                unit_seg(s, u, g.tile, g.k0, g.k1);
                g.unit = u;
                return true;
            };
            while (ok && next(sg)) {
                int tm, tn;
                if (SWAP) {
                    tm = 0;
                    tn = sg.tile;
                } else {
                    tile_coords(s, sg.tile, tm, tn);
                }
                for (int kb = sg.k0; kb < sg.k1; ++kb) {
                    if (!wait_bounded(&empty[stage], ph ^ 1u, abort_flag, p.wait_ns, site(0, 1, stage), seg)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sx = smem + stage * G::kStageBytes;
                    uint8_t* sy = sx + G::kXBytes;
                    // both blocks of a pair complete their halves on the leader's barrier, which expects them all
                    const uint32_t barc = PAIR ? mapa_shared(smem_u32(&full[stage]), 0) : 0u;
                    if (!PAIR || leader) mbar_arrive_expect_tx(&full[stage], R * G::kStageBytes);
                    if (!SWAP) {
                        // A: 64 K x 128 rows (this block's rows of a pair tile)
                        load_tile<PAIR, BW_HINT_A>(sx, &tmx, kb * kBK, tm * G::kTileM + rank * 128, &full[stage], barc,
                                                   pol_a);
                        // B: this block's kBPart columns of each MMA's 256 (w: a wide pair tile's MMA), so that
                        // accumulator column c is tile column c
#pragma unroll
                        for (int w = 0; w < G::kWN; ++w) {
                            uint8_t* syw = sy + w * G::kBPart * kBK * 2;
                            const int n = tn * BN + w * 256 + rank * G::kBPart;
                            if (p.tn) {  // B (N x K): kBPart rows of B, 64 K each, one load
                                load_tile<PAIR, BW_HINT_B>(syw, &tmy, kb * kBK, n, &full[stage], barc, pol_b);
                            } else if (BW_TMA3D) {  // B: kBPart columns, one load
                                load_blocks<PAIR, BW_HINT_B>(syw, &tmy, n / 64, kb * kBK, &full[stage], barc, pol_b);
                            } else {
#pragma unroll
                                for (int j = 0; j < G::kBPart / 64; ++j)  // B: kBPart columns, 64 x 64 K boxes
                                    load_tile<PAIR, BW_HINT_B>(syw + j * 8192, &tmy, n + 64 * j, kb * kBK,
                                                               &full[stage], barc, pol_b);
                            }
                        }
                    } else {
                        // this block's weight columns (a pair: block r holds the tile's r-th run of 128 x WM), and
                        // its tokens (a pair: block r the r-th half of the BN, the MMA's N split over the pair)
                        const int wcol = (tn * R + rank) * 128 * WM;
                        if (p.tn) {  // B (N x K): 128 (x WM) rows of B, 64 K each, one load
                            load_tile<PAIR, BW_SWAP_HINT_B>(sx, &tmx, kb * kBK, wcol, &full[stage], barc, pol_sb);
                        } else if (BW_TMA3D) {  // B: 128 (x WM) columns, one load
                            load_blocks<PAIR, BW_SWAP_HINT_B>(sx, &tmx, wcol / 64, kb * kBK, &full[stage], barc, pol_sb);
                        } else {
#pragma unroll
                            for (int j = 0; j < 2 * WM; ++j)  // B: 128 (x WM) columns as boxes of 64 columns x 64 K
                                load_tile<PAIR, BW_SWAP_HINT_B>(sx + j * 8192, &tmx, wcol + 64 * j, kb * kBK,
                                                                &full[stage], barc, pol_sb);
                        }
                        // A: 64 K x BN (a pair: BN / 2) rows
                        load_tile<PAIR, BW_HINT_A>(sy, &tmy, kb * kBK, rank * (BN / R), &full[stage], barc, pol_a);
                    }
                    ++issued;
                    if (++stage == S) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
                ++seg;
            }
            // let the loads in flight land (a pair's land on the leader's barriers) before the block may leave: after
            // this thread's abort, and after an abort elsewhere that left its last stages unconsumed (on the normal
            // path they have all landed: no wait)
            if (leader) {
                const int n = issued < S ? issued : S;
                for (int i = 1; i <= n; ++i) {
                    const int q = issued - i;
                    wait_drain(&full[q % S], (uint32_t)((q / S) & 1), p.wait_ns);
                }
            }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------- MMA issuer (one thread; the leader of a pair)
        if (lane == 0 && leader) {
            // B (the MMA's A operand in swap-AB) is MN-major when K x N, K-major when N x K (p.tn)
            constexpr uint32_t idesc_nn = idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, SWAP, !SWAP);
            constexpr uint32_t idesc_tn = idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, false, false);
            const uint32_t idesc = p.tn ? idesc_tn : idesc_nn;
            const bool bk = p.tn != 0;
            SegIter it(s, c, P);
            Seg sg;
            int stage = 0, acc = 0, seg = 0, qi = 0;
            uint32_t ph = 0, aph = 0;
            bool ok = true;
#ifdef BW_TRACE
            unsigned long long w_full = 0, w_acc = 0, n_kb = 0;
#endif
            // s.dyn: the producer's next unit from the queue
            auto next = [&](Seg& g) -> bool {
                if (!s.dyn) return it.next(s, P, g);
                const int qs = qi % kPlanUnitQ;
                if (!wait_bounded(&uq_full[qs], (uint32_t)((qi / kPlanUnitQ) & 1), abort_flag, p.wait_ns,
                                  site(1, 9, (uint32_t)qs), seg)) {
                    ok = false;
                    return false;
                }
                const int u = uq[qs];
                mbar_arrive(&uq_empty[qs]);
                ++qi;
                if (u < 0) return false;
                unit_seg(s, u, g.tile, g.k0, g.k1);
                g.unit = u;
                return true;
            };
            while (ok && next(sg)) {
#ifdef BW_TRACE
                const unsigned long long ta0 = globaltimer_ns();
#endif
                if (!wait_bounded(&tempty[acc], aph ^ 1u, abort_flag, p.wait_ns, site(1, 3, acc), seg)) {
                    ok = false;
                    break;
                }
#ifdef BW_TRACE
                w_acc += globaltimer_ns() - ta0;
#endif
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(acc * AN);
                // the MMAs of stage st (K-block kb) into parts [w0, w1) of the accumulator: SWAP, each 128-column
                // weight block of A into its BN columns; a wide pair tile, each 256-column part of B into its columns
                auto issue = [&](int st, int kb, int w0, int w1) {
                    const uint32_t sx = smem_u32(smem + st * G::kStageBytes), sy = sx + G::kXBytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k) {
                        const uint32_t accumulate = (kb > sg.k0 || k > 0) ? 1u : 0u;
#pragma unroll
                        for (int w = 0; w < WM * G::kWN; ++w) {
                            if (w < w0 || w >= w1) continue;
                            const uint32_t xw = sx + (uint32_t)((SWAP ? w : 0) * 128 * kBK * 2);
                            const uint32_t yw = sy + (uint32_t)((SWAP ? 0 : w) * G::kBPart * kBK * 2);
                            const uint64_t ad = (SWAP && !bk) ? desc_mnmajor(xw, k) : desc_kmajor(xw, k);
                            const uint64_t bd = (SWAP || bk) ? desc_kmajor(yw, k) : desc_mnmajor(yw, k);
                            const uint32_t dw = d + (uint32_t)(w * (SWAP ? BN : G::kMmaN));
                            if (PAIR)
                                mma_f16_pair(dw, ad, bd, idesc, accumulate);
                            else
                                mma_f16(dw, ad, bd, idesc, accumulate);
                        }
                    }
                };
                // the stage is free (in both blocks of a pair) once the MMAs so far have read it
                auto free_stage = [&](int st) {
                    if (PAIR) {
                        mma_commit_pair(mapa_shared(smem_u32(&empty[st]), 0));
                        mma_commit_pair(mapa_shared(smem_u32(&empty[st]), 1));
                    } else {
                        mma_commit(&empty[st]);
                    }
                };
                // kHalves: the epilogue has released the accumulator's first half (tempty[0]); until it releases the
                // second (tempty[1]) the stages get their first-half MMAs only and are held, at most S - 1 of them,
                // then get their second-half MMAs in K order and are freed
                int held = 0, held_stage = 0, held_kb = 0;
                bool half1 = !G::kHalves;
                auto catch_up = [&]() -> bool {
                    if (!wait_bounded(&tempty[1], aph ^ 1u, abort_flag, p.wait_ns, site(1, 3, 1), seg)) return false;
                    tc_fence_after();
                    for (int i = 0; i < held; ++i) {
                        const int st = (held_stage + i) % S;
                        issue(st, held_kb + i, 1, 2);
                        free_stage(st);
                    }
                    held = 0;
                    half1 = true;
                    return true;
                };
                for (int kb = sg.k0; kb < sg.k1; ++kb) {
#ifdef BW_TRACE
                    const unsigned long long tf0 = globaltimer_ns();
#endif
                    if (!wait_bounded(&full[stage], ph, abort_flag, p.wait_ns, site(1, 0, stage), seg)) {
                        ok = false;
                        break;
                    }
#ifdef BW_TRACE
                    if (seg == 0 && kb == sg.k0) BW_TRACE_AT(2);
                    else w_full += globaltimer_ns() - tf0;
                    ++n_kb;
#endif
                    tc_fence_after();
                    if (G::kHalves && !half1) {
                        issue(stage, kb, 0, 1);
                        if (held++ == 0) {
                            held_stage = stage;
                            held_kb = kb;
                        }
                        if ((mbar_try_wait(smem_u32(&tempty[1]), aph ^ 1u) || held == S - 1) && !catch_up()) {
                            ok = false;
                            break;
                        }
                    } else {
                        issue(stage, kb, 0, WM * G::kWN);
                        free_stage(stage);
                    }
                    if (++stage == S) {
                        stage = 0;
                        ph ^= 1u;
                    }
                }
                if (ok && !half1 && !catch_up()) ok = false;  // a segment shorter than the held stages
                if (!ok) break;
                // the accumulator (both blocks' halves) is complete once every MMA so far has finished
                if (PAIR) {
                    mma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 0));
                    mma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
                } else {
                    mma_commit(&tfull[acc]);
                }
                if (++acc == G::kAccBufs) {
                    acc = 0;
                    aph ^= 1u;
                }
                ++seg;
            }
            BW_TRACE_AT(3);
            BW_TRACE_VAL(12, w_full);
            BW_TRACE_VAL(13, w_acc);
            BW_TRACE_VAL(14, n_kb);
            // the MMAs in flight finish before the tensor memory is freed: after this thread's own abort, and after
            // an abort elsewhere in the block that left the epilogue without waiting for the last accumulator (on the
            // normal path the last segment's MMAs, which the epilogue is about to wait for anyway)
            if (PAIR)
                mma_commit_pair(mapa_shared(smem_u32(drain), 0));
            else
                mma_commit(drain);
            wait_drain(drain, 0, p.wait_ns);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------- epilogue (warps 2-5, 128 threads per block)
        const int q = warp & 3;         // the TMEM lane quarter this warp may access
        const int row = q * 32 + lane;  // accumulator row = TMEM lane
        const uint32_t tempty_leader0 = PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : smem_u32(&tempty[0]);
        SegIter it(s, c, P);
        Seg sg;
        int acc = 0, seg = 0, qi = 0;
        uint32_t aph = 0;
        unsigned epi_chunks = 0;  // BW_EPI_TMA: 64-column chunks this warp has stored (the staging buffer alternates)
        unsigned rs_acked = 0;  // kEpiRS: owners whose ack of the previous call this block has seen
        uint32_t win_ph = 0;    // kEpiRS: the window's buffers (rbar, krecv): the parity each waits for next
        int win_next = 0;       // kEpiRS: the buffer the next copy into the window goes to
        // kEpiRS: this call's epoch (the rank's epoch word moves on only once every block has finished, below)
        unsigned rs_epoch = 0u;
        if constexpr (EPI == kEpiRS) rs_epoch = *static_cast<volatile unsigned*>(p.rs->epoch) + 1u;
        // the accumulator is read: one arrival per warp on the (leader's) tmem-empty barrier
        auto release_acc = [&](int a) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (PAIR)
                    mbar_arrive_cluster(tempty_leader0 + 8u * (uint32_t)a);
                else
                    mbar_arrive(&tempty[a]);
            }
        };
        // the whole accumulator (kHalves: its two halves, tempty[0] and tempty[1])
        auto release_all = [&](int a) {
            if constexpr (G::kHalves) {
                release_acc(0);
                release_acc(1);
            } else {
                release_acc(a);
            }
        };
        for (;;) {
            if (!s.dyn && !it.next(s, P, sg)) break;
            // one thread waits (bounded); a named barrier hands its outcome to the other 127, so that an abort
            // takes the whole group out together and no thread is left at a later barrier.  s.dyn: that thread first
            // takes the segment's unit from the queue (go 2: none left)
            if (threadIdx.x == kEpiThread0) {
                int go = 1, u = 0;
                if (s.dyn) {
                    const int qs = qi % kPlanUnitQ;
                    if (!wait_bounded(&uq_full[qs], (uint32_t)((qi / kPlanUnitQ) & 1), abort_flag, p.wait_ns,
                                      site(2, 9, (uint32_t)qs), seg)) {
                        go = 0;
                    } else {
                        u = uq[qs];
                        mbar_arrive(&uq_empty[qs]);
                        ++qi;
                        if (u < 0) go = 2;
                    }
                }
                if (go == 1) go = wait_bounded(&tfull[acc], aph, abort_flag, p.wait_ns, site(2, 2, acc), seg) ? 1 : 0;
                epi_unit[seg & 1] = u;
                epi_go[seg & 1] = go;
            }
            named_bar_sync(1, 128);
            if (epi_go[seg & 1] != 1) break;
            if (s.dyn) {
                sg.unit = epi_unit[seg & 1];
                unit_seg(s, sg.unit, sg.tile, sg.k0, sg.k1);
            }
            if (threadIdx.x == kEpiThread0) {
                BW_TRACE_AT(6);  // the last segment's accumulator is ready (kept: overwritten per segment)
                BW_TRACE_VAL(8, 0);
            }
            tc_fence_after();
            int m0, n0;
            if (SWAP) {
                m0 = 0;
                n0 = (sg.tile * R + rank) * 128 * WM;  // this block's weight columns (a pair: its run of the tile)
            } else {
                int tm, tn;
                tile_coords(s, sg.tile, tm, tn);
                m0 = tm * G::kTileM + rank * 128;
                n0 = tn * BN;
            }
            const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * AN);
            if constexpr (EPI == kEpiRS) {
                int tm, tn;
                tile_coords(s, sg.tile, tm, tn);
                rs_tile(p, rs_epoch, tm, tn, rank, tbase, row, lane, q, abort_flag, recv_flag, reduce_flag, rs_acked,
                        smem + G::kWindowOffset, rbar, krecv, win_ph, win_next, seg);
                release_all(acc);
            } else if (EPI == kEpiSwiGLU) {
                // a whole tile (the plan splits none): gate columns [0, BN/2), up columns [BN/2, BN) of the tile,
                // silu(gate) * up to columns [n0 / 2, n0 / 2 + BN / 2) of the M x N/2 output
#pragma unroll 1
                for (int c0 = 0; c0 < BN / 2; c0 += 16) {
                    uint32_t gr[16], ur[16];
                    tmem_ld16(tbase + (uint32_t)c0, gr);
                    tmem_ld16(tbase + (uint32_t)(BN / 2 + c0), ur);
                    tmem_wait_ld();
                    const int m = m0 + row, n = n0 / 2 + c0;
                    if (m < s.M && n < s.N / 2) {
                        uint32_t h[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const float g0 = __uint_as_float(gr[2 * j]), g1 = __uint_as_float(gr[2 * j + 1]);
                            const float a0 = g0 / (1.0f + __expf(-g0)) * __uint_as_float(ur[2 * j]);
                            const float a1 = g1 / (1.0f + __expf(-g1)) * __uint_as_float(ur[2 * j + 1]);
                            const __half2 x = __floats2half2_rn(a0, a1);
                            h[j] = *reinterpret_cast<const uint32_t*>(&x);
                        }
                        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.C) + (size_t)m * (s.N / 2) + n);
                        dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
                        dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
                    }
                }
                release_all(acc);
            } else if (kp) {
#if BW_KSPLIT
                // a tile's K ranges on the kc blocks of this cluster (their only segment, so every block's stage ring
                // is idle once its accumulator is complete).  The accumulator's 16-column chunks are dealt out in
                // runs, block o owning [ksplit_run(o), ksplit_run(o + 1)).  Each block sends every chunk it does not
                // own into the owner's idle ring (16 bytes per st.async, counted on the owner's krecv barrier), as
                // piece (source block, chunk of the run) of 8 KB laid out [col / 4][row][4]; then sums the kc partials
                // of its own chunks in block order (its own from tensor memory) and writes them to C.  A block sends
                // once every other block has arrived on its kgo barrier (their rings are idle and they expect the
                // bytes).  One thread waits (bounded) and hands each outcome to the other 127.
                constexpr int kChunks = AN / 16;
                const int kc = s.ksplit;
                const int own0 = ksplit_run(kr, kChunks, kc), own1 = ksplit_run(kr + 1, kChunks, kc);
                const uint32_t recv_bytes = (uint32_t)((kc - 1) * (own1 - own0)) * 8192u;
                if (threadIdx.x == kEpiThread0) {
                    if (recv_bytes) mbar_arrive_expect_tx(krecv, recv_bytes);
                    for (int o = 0; o < kc; ++o)
                        if (o != kr) mbar_arrive_cluster(mapa_shared(smem_u32(kgo), (uint32_t)o));
                    const bool ok = wait_bounded(kgo, 0, abort_flag, p.wait_ns, site(2, 6, 0), seg);
                    if (ok) fence_acq_rel_cluster();  // after the others' arrivals (release, cluster scope)
                    *reduce_flag = ok ? 1 : 0;
                }
                named_bar_sync(1, 128);
                const bool go = *reduce_flag != 0;
                if (threadIdx.x == kEpiThread0) {
                    BW_TRACE_AT(7);  // the others' rings are idle
                    BW_TRACE_VAL(8, 4 | kc << 8);
                }
                if (go) {
#pragma unroll 1
                    for (int ch = 0; ch < kChunks; ++ch) {
                        if (ch >= own0 && ch < own1) continue;
                        const int o = ksplit_owner(ch, kChunks, kc);
                        const int r0 = ksplit_run(o, kChunks, kc), len = ksplit_run(o + 1, kChunks, kc) - r0;
                        const int piece = (kr < o ? kr : kr - 1) * len + (ch - r0);
                        const uint32_t dst = mapa_shared(smem_u32(smem), (uint32_t)o) + (uint32_t)piece * 8192u +
                                             (uint32_t)row * 16u;
                        const uint32_t bar = mapa_shared(smem_u32(krecv), (uint32_t)o);
                        uint32_t r[16];
                        tmem_ld16(tbase + (uint32_t)(ch * 16), r);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            st_async_v4(dst + (uint32_t)(j * 128 * 16), r[4 * j], r[4 * j + 1], r[4 * j + 2],
                                        r[4 * j + 3], bar);
                    }
                }
                if (threadIdx.x == kEpiThread0) BW_TRACE_AT(9);  // this thread's parts sent
                bool have = go;
                if (recv_bytes) {
                    // the others' parts of this block's chunks (after a failure, bytes still on their way land first)
                    if (threadIdx.x == kEpiThread0) {
                        const bool ok = go && wait_bounded(krecv, 0, abort_flag, p.wait_ns, site(2, 5, 0), seg);
                        if (!ok) wait_drain(krecv, 0, p.wait_ns);
                        *recv_flag = ok ? 1 : 0;
                    }
                    named_bar_sync(1, 128);
                    have = *recv_flag != 0;
                    if (have) mbar_try_wait(smem_u32(krecv), 0);  // complete: each thread acquires the bytes
                }
                if (threadIdx.x == kEpiThread0) BW_TRACE_AT(10);  // the others' parts of this block's chunks are in
                if (have) {
                    const float4* ring = reinterpret_cast<const float4*>(smem) + row;  // [piece][col / 4][row][4]
#pragma unroll 1
                    for (int ch = own0; ch < own1; ++ch) {
                        float v[16];
#pragma unroll 1
                        for (int sb = 0; sb < kc; ++sb) {
                            float x[16];
                            if (sb == kr) {
                                uint32_t r[16];
                                tmem_ld16(tbase + (uint32_t)(ch * 16), r);
                                tmem_wait_ld();
#pragma unroll
                                for (int e = 0; e < 16; ++e) x[e] = __uint_as_float(r[e]);
                            } else {
                                const float4* src = ring + (size_t)((sb < kr ? sb : sb - 1) * (own1 - own0) +
                                                                    (ch - own0)) * 512;
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const float4 w = src[j * 128];
                                    x[4 * j] = w.x;
                                    x[4 * j + 1] = w.y;
                                    x[4 * j + 2] = w.z;
                                    x[4 * j + 3] = w.w;
                                }
                            }
#pragma unroll
                            for (int e = 0; e < 16; ++e) v[e] = sb == 0 ? x[e] : v[e] + x[e];
                        }
                        store_chunk<SWAP, EPI, BN>(p, m0, n0, row, ch * 16, v, cst);
                    }
                }
                if (threadIdx.x == kEpiThread0) BW_TRACE_AT(11);  // this block's chunks summed and stored
                release_all(acc);
                named_bar_sync(1, 128);  // the flags are read by all before the block goes on
#else
                // a tile's K halves on the two blocks of this cluster (their only segment, so the first block's stage
                // ring is idle once its accumulator is complete): the second block sends its sum into that ring, 16
                // bytes per st.async, counted on the first block's krecv barrier; the first adds it to its own sum in
                // a fixed order and writes C.  One thread waits (bounded) and hands the outcome to the other 127.
                const float4* peer = reinterpret_cast<const float4*>(smem) + row;  // [col / 4][row][4]
                if (kr == 0) {
                    if (threadIdx.x == kEpiThread0) {
                        mbar_arrive_expect_tx(krecv, 128u * AN * 4u);
                        mbar_arrive_cluster(mapa_shared(smem_u32(kgo), 1));  // the ring may take the other sum now
                        const bool ok = wait_bounded(krecv, 0, abort_flag, p.wait_ns, site(2, 5, 0), seg);
                        if (!ok) wait_drain(krecv, 0, p.wait_ns);  // st.async bytes still on their way land first
                        *reduce_flag = ok ? 1 : 0;
                    }
                    named_bar_sync(1, 128);
                    if (*reduce_flag) {
                        mbar_try_wait(smem_u32(krecv), 0);  // complete: each thread acquires the bytes that arrived
#pragma unroll 1
                        for (int c0 = 0; c0 < AN; c0 += 16) {
                            uint32_t r[16];
                            tmem_ld16(tbase + (uint32_t)c0, r);
                            tmem_wait_ld();
                            float v[16];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float4 w = peer[(c0 / 4 + j) * 128];
                                v[4 * j] = __uint_as_float(r[4 * j]) + w.x;
                                v[4 * j + 1] = __uint_as_float(r[4 * j + 1]) + w.y;
                                v[4 * j + 2] = __uint_as_float(r[4 * j + 2]) + w.z;
                                v[4 * j + 3] = __uint_as_float(r[4 * j + 3]) + w.w;
                            }
                            store_chunk<SWAP, EPI, BN>(p, m0, n0, row, c0, v, cst);
                        }
                    }
                } else {
                    if (threadIdx.x == kEpiThread0) {
                        const bool ok = wait_bounded(kgo, 0, abort_flag, p.wait_ns, site(2, 6, 0), seg);
                        if (ok) fence_acq_rel_cluster();  // after the first block's arrival (release, cluster scope)
                        *reduce_flag = ok ? 1 : 0;
                    }
                    named_bar_sync(1, 128);
                    if (*reduce_flag) {
                        const uint32_t dst = mapa_shared(smem_u32(smem), 0) + (uint32_t)row * 16u;
                        const uint32_t bar = mapa_shared(smem_u32(krecv), 0);
#pragma unroll 1
                        for (int c0 = 0; c0 < AN; c0 += 16) {
                            uint32_t r[16];
                            tmem_ld16(tbase + (uint32_t)c0, r);
                            tmem_wait_ld();
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                st_async_v4(dst + (uint32_t)((c0 / 4 + j) * 128 * 16), r[4 * j], r[4 * j + 1],
                                            r[4 * j + 2], r[4 * j + 3], bar);
                        }
                    }
                }
                release_all(acc);
                named_bar_sync(1, 128);  // reduce_flag is read by all before the next segment writes it
#endif
            } else if (sg.k0 == 0 && sg.k1 == s.kblocks) {
                // a whole tile: straight to C, kLdw columns per wait on the tensor-memory loads
                constexpr int kLdw = AN % BW_EPI_LDW == 0 ? BW_EPI_LDW : 16;
#pragma unroll 1
                for (int c0 = 0; c0 < AN; c0 += kLdw) {
                    uint32_t r[kLdw / 16][16];
#pragma unroll
                    for (int h = 0; h < kLdw / 16; ++h) tmem_ld16(tbase + (uint32_t)(c0 + 16 * h), r[h]);
                    tmem_wait_ld();
                    if (G::kHalves && c0 + kLdw == AN / 2) release_acc(0);  // the first half is read
                    if (kEpiTma<BN, SWAP, PAIR, EPI> && kLdw == 64) {  // a TMA store per warp (store_rows64_tma)
                        float v[64];
#pragma unroll
                        for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j / 16][j % 16]);
                        uint8_t* quarter = smem + G::kWindowOffset + (epi_chunks++ & 1u) * 16384u + q * 4096;
                        store_rows64_tma(&tmc, quarter, m0 + q * 32, n0 + c0, s.M, s.N, lane, v);
                    } else if (!SWAP && kLdw == 64 && BW_EPI_LINES) {  // whole lines of C (store_rows64)
                        float v[64];
#pragma unroll
                        for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j / 16][j % 16]);
                        store_rows64<EPI == kEpiF32 ? kEpiF32 : kEpiF16>(p, m0 + q * 32, n0 + c0, lane, v);
                    } else {
#pragma unroll
                        for (int h = 0; h < kLdw / 16; ++h) {
                            float v[16];
#pragma unroll
                            for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[h][j]);
                            store_chunk<SWAP, EPI, BN>(p, m0, n0, row, c0 + 16 * h, v, cst);
                        }
                    }
                }
                if constexpr (G::kHalves)
                    release_acc(1);  // the first half went at the middle
                else
                    release_acc(acc);
            } else {
                // part of a split tile
                const Fixup f = fixup_of(s, c, P, sg);
                int* counter = p.counters + (sg.tile - s.dp_tiles) * R + rank;
                // this block's last segment: its stage ring is idle and can take the partials by bulk copy (s.dyn:
                // not known in advance, so never)
                SegIter peek = it;
                Seg nx;
                const bool last_seg = !s.dyn && !peek.next(s, P, nx);
                // the reduction may copy the partials into the stage ring only when no later segment streams into it
                const bool bulk = last_seg && f.nseg <= G::kMaxSum;
                // every other partial already written: this block is the last; sum them with its own accumulator
                // straight from tensor memory (no round trip of its own partial)
                if (threadIdx.x == kEpiThread0) *reduce_flag = ld_acquire_gpu(counter) == f.nseg - 1 ? 2 : 0;
                named_bar_sync(1, 128);
                const int fast = *reduce_flag;
                if (threadIdx.x == kEpiThread0) {
                    BW_TRACE_AT(7);
                    BW_TRACE_VAL(8, (fast == 2 ? 2 : 3) | f.nseg << 8 | seg << 16);
                }
                if (fast == 2) {
                    if (bulk)
                        reduce_tile_bulk<AN, SWAP, R, G::kMaxSum, EPI, BN>(p, P, sg.tile, rank, f, true, tbase, row, m0, n0,
                                                                  cst, smem, rbar, abort_flag, seg);
                    else
                        reduce_tile<AN, SWAP, R, EPI, BN>(p, P, sg.tile, rank, f, true, tbase, row, m0, n0, cst);
                    release_all(acc);
                    if (threadIdx.x == kEpiThread0) atomicExch(counter, 0);
                } else {
                    // this block's partial to its slot; the last block to finish the tile sums them
                    const long long myslot = (long long)fixup_slot(s, P, sg.tile, f, f.mine) * R + rank;
#pragma unroll 1
                    for (int c0 = 0; c0 < AN; c0 += 16) {
                        uint32_t r[16];
                        tmem_ld16(tbase + (uint32_t)c0, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            __stcg(slot_vec<AN>(p, myslot, row, c0 / 4 + j),
                                   make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                               __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
                    }
                    // at the last segment the accumulator stays (no later MMA needs it): the reduction reads this
                    // block's own partial from tensor memory
                    if (!last_seg) release_all(acc);
                    __threadfence();
                    named_bar_sync(1, 128);
                    if (threadIdx.x == kEpiThread0) {
                        const int old = atomicAdd(counter, 1);
                        if (old == f.nseg - 1) __threadfence();
                        *reduce_flag = old == f.nseg - 1 ? 1 : 0;
                    }
                    named_bar_sync(1, 128);
                    if (*reduce_flag == 1) {
                        if (threadIdx.x == kEpiThread0) {
                            BW_TRACE_AT(9);
                            BW_TRACE_VAL(8, 1 | f.nseg << 8 | seg << 16);
                        }
                        if (bulk)
                            reduce_tile_bulk<AN, SWAP, R, G::kMaxSum, EPI, BN>(p, P, sg.tile, rank, f, true, tbase, row, m0, n0,
                                                                      cst, smem, rbar, abort_flag, seg);
                        else
                            reduce_tile<AN, SWAP, R, EPI, BN>(p, P, sg.tile, rank, f, false, tbase, row, m0, n0, cst);
                        if (threadIdx.x == kEpiThread0) atomicExch(counter, 0);
                    }
                    if (last_seg) release_all(acc);
                }
                named_bar_sync(1, 128);  // reduce_flag is read by all before the next segment writes it
            }
            if (++acc == G::kAccBufs) {
                acc = 0;
                aph ^= 1u;
            }
            ++seg;
        }
        if constexpr (EPI == kEpiRS) {
            // the call's last block to finish moves the rank's epoch word on; every block read it at entry (this
            // block's 128 threads have all passed that read at this barrier)
            named_bar_sync(1, 128);
            if (threadIdx.x == kEpiThread0) {
                __threadfence();
                if (atomicAdd(p.rs->done, 1u) == gridDim.x - 1u) {
                    *p.rs->done = 0u;
                    __threadfence();
                    *static_cast<volatile unsigned*>(p.rs->epoch) = rs_epoch;
                }
            }
        }
        // the TMA stores of C complete before the block leaves (their sources are this block's shared memory)
        if (kEpiTma<BN, SWAP, PAIR, EPI> && lane == 0) bulk_wait<0>();
        if (threadIdx.x == kEpiThread0) BW_TRACE_AT(4);
    }

    __syncwarp();
    tc_fence_before();
    if (PAIR || kp)
        cluster_sync();  // neither block leaves while the other may still read its memory or arrive on its barriers
    else
        __syncthreads();
    if (s.dyn && threadIdx.x == 0) {
        // this block's producer has taken its last unit: the call's last block to get here puts the counter of the
        // next unit, and its own count, back to zero for the next call
        int* next_unit = p.counters + s.sk_tiles * R;
        __threadfence();
        if (atomicAdd(next_unit + 1, 1) == (int)gridDim.x - 1) {
            atomicExch(next_unit, 0);
            atomicExch(next_unit + 1, 0);
        }
    }
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        if (PAIR)
            tmem_dealloc_pair(tmem_base, G::kTmemCols);
        else
            tmem_dealloc(tmem_base, G::kTmemCols);
    }
    if (threadIdx.x == 0) {
        BW_TRACE_AT(5);
        BW_TRACE_VAL(15, clock64() - clk0);
    }
}

}  // namespace bw
