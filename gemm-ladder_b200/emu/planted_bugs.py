"""Planted-bug test of the Blackwell host emulator -- TEST INFRASTRUCTURE (nothing here is part of the library).

The emulator (emu.cpp, emu_runtime.h, ptx_emu.h) is only worth its findings if it catches the mistakes a kernel of this
kind is prone to.  This script plants them: each entry of MUTATIONS is one small edit of the kernel's own source
(csrc/gemm_kernel.cuh, epilogue.cuh, kernel_common.cuh, schedule.h, plan.h) -- a wait taken out, a barrier parity
flipped, a transaction count off, a tcgen05 commit dropped, a tensor-memory column or lane off, a descriptor's swizzle
stride wrong, a coordinate or a store bound off by one, a reduction's order or count changed.  For each, a copy of the
sources with that one edit is compiled into the emulator and run on a set of calls that covers every plan form
(SM-pair tiles whole, with a split-K tail and stream-K; swap-AB with K halves on clusters of two and stream-K; M not a
multiple of 16; fp32 and SwiGLU outputs; B as N x K; the single-SM tile variants).  The mutation is REPORTED if any
call of the set ends with a non-zero status, an emulator finding (an access out of bounds, an mbarrier misuse, a wait
that gave up, a thread barrier never completed), a split-tile counter left set, an element written past row M, a
result outside the oracle's gates (the fp64 i-k-j GEMM of oracle/oracle.c: per element 2 ulp16 + 1e-3 sqrt(K), and
normwise 2e-3), two calls that differ bit for bit, or a crash or hang of the emulator process.  The unmodified sources
must pass every call.  The reference holds its emulators to the same standard (hopper/emu/planted_bugs.py:820-867:
every one of its mutations reported, the unmodified copy clean).

    python gemm-ladder_b200/emu/planted_bugs.py [--jobs 8] [--only name,...] [--list] [--out FILE]

Each mutation names the build it needs ("library": the kernel as the library builds it; the others: BUILDS, below), so
that code compiled only there is mutated where it runs.
"""
import argparse
import concurrent.futures
import ctypes
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
CUDA_INCLUDE = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
BUILDS = {
    "library": (),
    # the options built but off by default (stream-K over a part wave of pair tiles, swap-AB on SM pairs)
    "next": ("BW_SK_PART_WAVE=1", "BW_SWAP_PAIR=1"),
    # the swap-AB K halves on clusters of two (BW_KSPLIT 0, the rule's form before the K split over 2 to 8 blocks)
    "halves": ("BW_KSPLIT=0",),
    # the 256 x 512 pair tile wherever the rule allows it, so that small emulated shapes run the wide kernel
    "wide": ("BW_PAIR_WIDE=1", "BW_PAIR_WIDE_KB_NS=1", "BW_PAIR_WIDE_EPI_NS=0", "BW_FIXUP_KB=0"),
    # the TMA-store epilogue
    "tma": ("BW_EPI_TMA=1",),
    # the dynamic units of K for swap-AB stream-K shapes (measured slower than static stream-K, off in the library)
    "dyn": ("BW_DYN_UNITS=1",),
}

GK, EP, KC, SC, PL = "csrc/gemm_kernel.cuh", "csrc/epilogue.cuh", "csrc/kernel_common.cuh", "csrc/schedule.h", "csrc/plan.h"

# (name, file, before, after, occurrence of `before` (0: the first), build)
MUTATIONS = [
    # ---------------------------------------------------------------- the producer (TMA warp)
    ("prod_empty_wait_gone", GK, "if (!wait_bounded(&empty[stage], ph ^ 1u, abort_flag, p.wait_ns, site(0, 1, stage), seg)) {",
     "if (false) {", 0, "library"),
    ("prod_empty_parity", GK, "&empty[stage], ph ^ 1u,", "&empty[stage], ph,", 0, "library"),
    ("prod_expect_tx_half_pair", GK, "mbar_arrive_expect_tx(&full[stage], R * G::kStageBytes);",
     "mbar_arrive_expect_tx(&full[stage], G::kStageBytes);", 0, "library"),
    ("prod_expect_tx_over", GK, "mbar_arrive_expect_tx(&full[stage], R * G::kStageBytes);",
     "mbar_arrive_expect_tx(&full[stage], R * G::kStageBytes + 16);", 0, "library"),
    ("prod_a_rows_no_rank", GK, "kb * kBK, tm * G::kTileM + rank * 128,", "kb * kBK, tm * G::kTileM,", 0, "library"),
    ("prod_a_rows_off", GK, "kb * kBK, tm * G::kTileM + rank * 128,", "kb * kBK, tm * G::kTileM + rank * 128 + 8,", 0,
     "library"),
    ("prod_a_k_block", GK, "load_tile<PAIR, BW_HINT_A>(sx, &tmx, kb * kBK,", "load_tile<PAIR, BW_HINT_A>(sx, &tmx, (kb ^ 1) * kBK,",
     0, "library"),
    ("prod_b_cols_no_rank", GK, "const int n = tn * BN + w * 256 + rank * G::kBPart;", "const int n = tn * BN + w * 256;", 0,
     "library"),
    ("prod_b_tn_rows", GK, "load_tile<PAIR, BW_HINT_B>(syw, &tmy, kb * kBK, n, &full[stage], barc, pol_b);",
     "load_tile<PAIR, BW_HINT_B>(syw, &tmy, kb * kBK, n + 64, &full[stage], barc, pol_b);", 0, "library"),
    ("prod_b_3d_block", GK, "load_blocks<PAIR, BW_HINT_B>(syw, &tmy, n / 64, kb * kBK,",
     "load_blocks<PAIR, BW_HINT_B>(syw, &tmy, n / 64 + 1, kb * kBK,", 0, "library"),
    ("prod_b_3d_k", GK, "load_blocks<PAIR, BW_HINT_B>(syw, &tmy, n / 64, kb * kBK,",
     "load_blocks<PAIR, BW_HINT_B>(syw, &tmy, n / 64, (kb ^ 1) * kBK,", 0, "library"),
    ("prod_swap_wcol_wm", GK, "const int wcol = (tn * R + rank) * 128 * WM;", "const int wcol = (tn * R + rank) * 128;", 0,
     "library"),
    ("prod_swap_tokens_off", GK, "load_tile<PAIR, BW_HINT_A>(sy, &tmy, kb * kBK, rank * (BN / R),",
     "load_tile<PAIR, BW_HINT_A>(sy, &tmy, kb * kBK, 16 + rank * (BN / R),", 0, "library"),
    ("prod_swap_tokens_k", GK, "load_tile<PAIR, BW_HINT_A>(sy, &tmy, kb * kBK, rank * (BN / R),",
     "load_tile<PAIR, BW_HINT_A>(sy, &tmy, (kb ^ 1) * kBK, rank * (BN / R),", 0, "library"),
    ("prod_swap_tn_rows", GK, "load_tile<PAIR, BW_SWAP_HINT_B>(sx, &tmx, kb * kBK, wcol,",
     "load_tile<PAIR, BW_SWAP_HINT_B>(sx, &tmx, kb * kBK, wcol + 64,", 0, "library"),
    ("prod_swap_3d_block", GK, "load_blocks<PAIR, BW_SWAP_HINT_B>(sx, &tmx, wcol / 64, kb * kBK,",
     "load_blocks<PAIR, BW_SWAP_HINT_B>(sx, &tmx, wcol / 64 + 1, kb * kBK,", 0, "library"),
    ("prod_stage_bytes", GK, "uint8_t* sx = smem + stage * G::kStageBytes;", "uint8_t* sx = smem + (stage ^ 1) * G::kStageBytes;",
     0, "library"),
    ("prod_phase_never_flips", GK, "ph ^= 1u;", "(void)0;", 0, "library"),
    ("prod_leader_only_expects", GK, "if (!PAIR || leader) mbar_arrive_expect_tx(&full[stage], R * G::kStageBytes);",
     "mbar_arrive_expect_tx(&full[stage], R * G::kStageBytes);", 0, "library"),
    # ---------------------------------------------------------------- the MMA issuer
    ("mma_full_wait_gone", GK, "if (!wait_bounded(&full[stage], ph, abort_flag, p.wait_ns, site(1, 0, stage), seg)) {",
     "if (false) {", 0, "library"),
    ("mma_full_parity", GK, "wait_bounded(&full[stage], ph,", "wait_bounded(&full[stage], ph ^ 1u,", 0, "library"),
    ("mma_acc_free_wait_gone", GK,
     "if (!wait_bounded(&tempty[acc], aph ^ 1u, abort_flag, p.wait_ns, site(1, 3, acc), seg)) {", "if (false) {", 0,
     "library"),
    ("mma_acc_free_parity", GK, "&tempty[acc], aph ^ 1u,", "&tempty[acc], aph,", 0, "library"),
    ("mma_idesc_b_major", GK, "idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, SWAP, !SWAP)",
     "idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, SWAP, SWAP)", 0, "library"),
    ("mma_idesc_tn", GK, "idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, false, false)",
     "idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, false, true)", 0, "library"),
    ("mma_idesc_n", GK, "idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN, SWAP, !SWAP)",
     "idesc_f16_f32(PAIR ? 256 : 128, G::kMmaN / 2, SWAP, !SWAP)", 0, "library"),
    ("mma_accumulate_from_zero", GK, "(kb > sg.k0 || k > 0) ? 1u : 0u", "(kb > 0 || k > 0) ? 1u : 0u", 0, "library"),
    ("mma_accumulate_slice", GK, "(kb > sg.k0 || k > 0) ? 1u : 0u", "(kb > sg.k0 || k > 1) ? 1u : 0u", 0, "library"),
    ("mma_weight_block_a", GK, "(uint32_t)((SWAP ? w : 0) * 128 * kBK * 2)", "(uint32_t)((SWAP ? 0 : 0) * 128 * kBK * 2)",
     0, "library"),
    ("mma_a_desc_k", GK, "(SWAP && !bk) ? desc_mnmajor(xw, k) : desc_kmajor(xw, k)",
     "(SWAP && !bk) ? desc_mnmajor(xw, 0) : desc_kmajor(xw, k)", 0, "library"),
    ("mma_a_desc_k_kmajor", GK, "(SWAP && !bk) ? desc_mnmajor(xw, k) : desc_kmajor(xw, k)",
     "(SWAP && !bk) ? desc_mnmajor(xw, k) : desc_kmajor(xw, k ^ 1)", 0, "library"),
    ("mma_b_desc_k", GK, "(SWAP || bk) ? desc_kmajor(yw, k) : desc_mnmajor(yw, k)",
     "(SWAP || bk) ? desc_kmajor(yw, k) : desc_mnmajor(yw, k ^ 2)", 0, "library"),
    ("mma_b_desc_kmajor", GK, "(SWAP || bk) ? desc_kmajor(yw, k) : desc_mnmajor(yw, k)",
     "(SWAP || bk) ? desc_kmajor(yw, 0) : desc_mnmajor(yw, k)", 0, "library"),
    ("mma_weight_block_columns", GK, "d + (uint32_t)(w * (SWAP ? BN : G::kMmaN))", "d + (uint32_t)(w * (SWAP ? 16 : G::kMmaN))",
     0, "library"),
    ("mma_free_stage_pair_one", GK, "mma_commit_pair(mapa_shared(smem_u32(&empty[st]), 1));", "(void)st;", 0, "library"),
    ("mma_free_stage_single", GK, "mma_commit(&empty[st]);", "(void)st;", 0, "library"),
    ("mma_free_stage_before_issue", GK, "issue(stage, kb, 0, WM * G::kWN);\n                        free_stage(stage);",
     "free_stage(stage);\n                        issue(stage, kb, 0, WM * G::kWN);", 0, "library"),
    ("mma_acc_done_pair_one", GK, "mma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));", "(void)acc;", 0, "library"),
    ("mma_acc_done_single", GK, "mma_commit(&tfull[acc]);", "(void)acc;", 0, "library"),
    ("mma_acc_phase_never_flips", GK, "aph ^= 1u;", "(void)0;", 0, "library"),
    ("mma_stage_phase_never_flips", GK, "ph ^= 1u;", "(void)0;", 1, "library"),
    ("mma_one_accumulator", GK, "const uint32_t d = tmem_base + (uint32_t)(acc * AN);", "const uint32_t d = tmem_base;", 0,
     "library"),
    ("sched_block_index", GK, "const int P = gridDim.x / R, c = blockIdx.x / R;",
     "const int P = gridDim.x / R, c = blockIdx.x / R + (blockIdx.x >= (unsigned)R && blockIdx.x + R < gridDim.x);", 0,
     "library"),
    # ---------------------------------------------------------------- barrier set-up
    ("init_acc_free_count", GK, "mbar_init(&tempty[i], 4 * R);", "mbar_init(&tempty[i], 4 * R + 1);", 0, "library"),
    ("init_acc_free_count_low", GK, "mbar_init(&tempty[i], 4 * R);", "mbar_init(&tempty[i], 4 * R - 1);", 0, "library"),
    ("init_full_count", GK, "mbar_init(&full[i], 1);", "mbar_init(&full[i], 2);", 0, "library"),
    ("init_empty_count", GK, "mbar_init(&empty[i], 1);", "mbar_init(&empty[i], 2);", 0, "library"),
    ("init_acc_done_count", GK, "mbar_init(&tfull[i], 1);", "mbar_init(&tfull[i], 2);", 0, "library"),
    ("init_kgo_count", GK, "mbar_init(kgo, kp ? s.ksplit - 1 : 1);", "mbar_init(kgo, kp ? s.ksplit : 1);", 0, "library"),
    ("init_no_pair_sync", GK, "if (PAIR || kp)\n        cluster_sync();  // the leader's barriers exist",
     "if (false)\n        cluster_sync();  // the leader's barriers exist", 0, "library"),
    # ---------------------------------------------------------------- the epilogue: accumulators and whole tiles
    ("epi_acc_wait_gone", GK,
     "if (go == 1) go = wait_bounded(&tfull[acc], aph, abort_flag, p.wait_ns, site(2, 2, acc), seg) ? 1 : 0;",
     "(void)aph;", 0, "library"),
    ("epi_acc_parity", GK, "wait_bounded(&tfull[acc], aph,", "wait_bounded(&tfull[acc], aph ^ 1u,", 0, "library"),
    ("epi_whole_tile_kept", GK, "                else\n                    release_acc(acc);\n",
     "                else\n                    (void)acc;\n", 0, "library"),
    ("epi_release_early", GK, "if (G::kHalves && c0 + kLdw == AN / 2) release_acc(0);  // the first half is read",
     "if (G::kHalves ? c0 + kLdw == AN / 2 : c0 == 0) release_acc(G::kHalves ? 0 : acc);", 0, "library"),
    ("epi_split_acc_kept", GK, "if (!last_seg) release_all(acc);", "if (false) release_all(acc);", 0, "library"),
    ("epi_lane_quarter", GK, "const int q = warp & 3;         // the TMEM lane quarter this warp may access",
     "const int q = (warp + 1) & 3;", 0, "library"),
    ("epi_tmem_acc_column", GK, "((uint32_t)(q * 32) << 16) + (uint32_t)(acc * AN)",
     "((uint32_t)(q * 32) << 16) + (uint32_t)(acc * AN / 2)", 0, "library"),
    ("epi_pair_rows_no_rank", GK, "m0 = tm * G::kTileM + rank * 128;", "m0 = tm * G::kTileM;", 0, "library"),
    ("epi_cols_off", GK, "n0 = tn * BN;", "n0 = tn * BN + 64;", 0, "library"),
    ("epi_swap_cols_wm", GK, "n0 = (sg.tile * R + rank) * 128 * WM;", "n0 = (sg.tile * R + rank) * 128;", 0, "library"),
    ("epi_whole_tile_test", GK, "} else if (sg.k0 == 0 && sg.k1 == s.kblocks) {", "} else if (sg.k0 == 0) {", 0,
     "library"),
    ("epi_lines_column", GK, "store_rows64<EPI == kEpiF32 ? kEpiF32 : kEpiF16>(p, m0 + q * 32, n0 + c0, lane, v);",
     "store_rows64<EPI == kEpiF32 ? kEpiF32 : kEpiF16>(p, m0 + q * 32, n0, lane, v);", 0, "library"),
    ("epi_lines_order", GK, "for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j / 16][j % 16]);",
     "for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j % 4][j / 4]);", 1, "library"),
    ("tma_lines_order", GK, "for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j / 16][j % 16]);",
     "for (int j = 0; j < 64; ++j) v[j] = __uint_as_float(r[j % 4][j / 4]);", 0, "tma"),
    ("epi_chunk_column", GK, "store_chunk<SWAP, EPI, BN>(p, m0, n0, row, c0 + 16 * h, v, cst);",
     "store_chunk<SWAP, EPI, BN>(p, m0, n0, row, c0, v, cst);", 0, "library"),
    ("epi_swiglu_up_half", GK, "tmem_ld16(tbase + (uint32_t)(BN / 2 + c0), ur);", "tmem_ld16(tbase + (uint32_t)(c0), ur);", 0,
     "library"),
    ("epi_swiglu_row_bound", GK, "if (m < s.M && n < s.N / 2) {", "if (m <= s.M && n < s.N / 2) {", 0, "library"),
    # ---------------------------------------------------------------- split tiles: partials, counters, reductions
    ("split_counter_shared_by_pair", GK, "int* counter = p.counters + (sg.tile - s.dp_tiles) * R + rank;",
     "int* counter = p.counters + (sg.tile - s.dp_tiles) * R;", 0, "library"),
    ("split_fast_path_early", GK, "*reduce_flag = ld_acquire_gpu(counter) == f.nseg - 1 ? 2 : 0;",
     "*reduce_flag = ld_acquire_gpu(counter) >= f.nseg - 2 ? 2 : 0;", 0, "library"),
    ("split_slot_shared_by_pair", GK, "(long long)fixup_slot(s, P, sg.tile, f, f.mine) * R + rank;",
     "(long long)fixup_slot(s, P, sg.tile, f, f.mine) * R;", 0, "library"),
    ("split_slot_other_partial", GK, "(long long)fixup_slot(s, P, sg.tile, f, f.mine) * R + rank;",
     "(long long)fixup_slot(s, P, sg.tile, f, f.mine ^ 1) * R + rank;", 0, "library"),
    ("split_partial_columns", GK, "__stcg(slot_vec<AN>(p, myslot, row, c0 / 4 + j),",
     "__stcg(slot_vec<AN>(p, myslot, row, c0 / 4 + (j ^ 1)),", 0, "library"),
    ("split_count_by_two", GK, "const int old = atomicAdd(counter, 1);", "const int old = atomicAdd(counter, 2);", 0,
     "library"),
    ("split_reducer_never", GK, "*reduce_flag = old == f.nseg - 1 ? 1 : 0;", "*reduce_flag = old == f.nseg ? 1 : 0;", 0,
     "library"),
    ("split_reducer_early", GK, "*reduce_flag = old == f.nseg - 1 ? 1 : 0;", "*reduce_flag = old == f.nseg - 2 ? 1 : 0;",
     0, "library"),
    ("split_counter_kept_fast", GK, "if (threadIdx.x == kEpiThread0) atomicExch(counter, 0);", "(void)counter;", 0,
     "library"),
    ("split_counter_kept_slow", GK, "if (threadIdx.x == kEpiThread0) atomicExch(counter, 0);", "(void)counter;", 1,
     "library"),
    ("split_bulk_not_last", GK, "const bool bulk = last_seg && f.nseg <= G::kMaxSum;",
     "const bool bulk = f.nseg <= G::kMaxSum;", 0, "library"),
    # ---------------------------------------------------------------- K halves on clusters of two (swap-AB)
    ("khalf_expect_half", GK, "mbar_arrive_expect_tx(krecv, 128u * AN * 4u);", "mbar_arrive_expect_tx(krecv, 128u * AN * 2u);",
     0, "halves"),
    ("khalf_go_to_self", GK, "mbar_arrive_cluster(mapa_shared(smem_u32(kgo), 1));  // the ring may take the other sum now",
     "mbar_arrive_cluster(mapa_shared(smem_u32(kgo), 0));", 0, "halves"),
    ("khalf_recv_wait_gone", GK, "const bool ok = wait_bounded(krecv, 0, abort_flag, p.wait_ns, site(2, 5, 0), seg);\n                        if (!ok) wait_drain(krecv, 0, p.wait_ns);  // st.async",
     "const bool ok = true;\n                        if (!ok) wait_drain(krecv, 0, p.wait_ns);  // st.async", 0, "halves"),
    ("khalf_other_half_dropped", GK, "v[4 * j] = __uint_as_float(r[4 * j]) + w.x;", "v[4 * j] = __uint_as_float(r[4 * j]);",
     0, "halves"),
    ("khalf_send_stride", GK, "st_async_v4(dst + (uint32_t)((c0 / 4 + j) * 128 * 16), r[4 * j], r[4 * j + 1],",
     "st_async_v4(dst + (uint32_t)((c0 / 4 + j) * 128 * 8), r[4 * j], r[4 * j + 1],", 0, "halves"),
    ("khalf_peer_row", GK, "const float4* peer = reinterpret_cast<const float4*>(smem) + row;  // [col / 4][row][4]",
     "const float4* peer = reinterpret_cast<const float4*>(smem) + (row ^ 1);", 0, "halves"),
    ("khalf_send_before_go", GK, "const bool ok = wait_bounded(kgo, 0, abort_flag, p.wait_ns, site(2, 6, 0), seg);\n                        if (ok) fence_acq_rel_cluster();  // after the first block's arrival",
     "const bool ok = true;\n                        if (ok) fence_acq_rel_cluster();  // after the first block's arrival", 0, "halves"),
    # ---------------------------------------------------------------- descriptors and loads (kernel_common.cuh)
    ("desc_kmajor_k_step", KC, "smem_desc_sw128(tile + 32u * k, 16u, 1024u)", "smem_desc_sw128(tile + 16u * k, 16u, 1024u)", 0,
     "library"),
    ("desc_kmajor_sbo", KC, "smem_desc_sw128(tile + 32u * k, 16u, 1024u)", "smem_desc_sw128(tile + 32u * k, 16u, 512u)", 0,
     "library"),
    ("desc_mnmajor_k_step", KC, "smem_desc_sw128(tile + 2048u * k, 8192u, 1024u)",
     "smem_desc_sw128(tile + 1024u * k, 8192u, 1024u)", 0, "library"),
    ("desc_mnmajor_lbo", KC, "smem_desc_sw128(tile + 2048u * k, 8192u, 1024u)", "smem_desc_sw128(tile + 2048u * k, 4096u, 1024u)",
     0, "library"),
    ("desc_mnmajor_sbo", KC, "smem_desc_sw128(tile + 2048u * k, 8192u, 1024u)", "smem_desc_sw128(tile + 2048u * k, 8192u, 2048u)",
     0, "library"),
    ("load_3d_pair_x", KC, "tma_load_3d_pair(dst, tmap, 0, k, n64, bar_cluster);", "tma_load_3d_pair(dst, tmap, 64, k, n64, bar_cluster);",
     0, "library"),
    ("load_3d_k", KC, "tma_load_3d(dst, tmap, 0, k, n64, bar);", "tma_load_3d(dst, tmap, 0, k + 64, n64, bar);", 0, "library"),
    ("load_2d_pair_rows", KC, "else tma_load_2d_pair(dst, tmap, x, y, bar_cluster);",
     "else tma_load_2d_pair(dst, tmap, x, y + 64, bar_cluster);", 0, "library"),
    ("load_2d_x_y_swapped", KC, "else tma_load_2d(dst, tmap, x, y, bar);", "else tma_load_2d(dst, tmap, y, x, bar);", 0,
     "library"),
    ("geom_b_part", KC, "static constexpr int kBPart = BN / kRanks / kWN;", "static constexpr int kBPart = BN / kWN;", 0,
     "library"),
    # ---------------------------------------------------------------- stores of C, reductions (epilogue.cuh)
    ("store_f32_row_bound", EP, "if (m >= s.M || n >= s.N) return;", "if (m > s.M || n >= s.N) return;", 0, "library"),
    ("store_f16_row_bound", EP, "if (m >= s.M || n >= s.N) return;", "if (m > s.M || n >= s.N) return;", 1, "library"),
    ("store_f16_pair_order", EP, "const __half2 x = __floats2half2_rn(v[2 * j], v[2 * j + 1]);",
     "const __half2 x = __floats2half2_rn(v[2 * j + 1], v[2 * j]);", 0, "library"),
    ("store_swap_lane", EP, "buf[j * 128 + lane] = __float2half_rn(v[j]);", "buf[j * 128 + (lane ^ 1)] = __float2half_rn(v[j]);",
     0, "library"),
    ("store_swap_piece", EP, "const int mm = piece >> 4, nn = (piece & 15) * 8;", "const int mm = piece >> 4, nn = (piece & 7) * 8;",
     0, "library"),
    ("store_swap_row_bound", EP, "if (m < s.M && n < s.N)\n", "if (m <= s.M && n < s.N)\n", 0, "library"),
    ("store_swap_tokens_wm", EP, "const int wb = BT ? c0 / BT : 0, tok = c0 - wb * BT;", "const int wb = BT ? c0 / BT : 0, tok = c0;",
     0, "library"),
    ("store_swap_no_barrier", EP, "buf[j * 128 + lane] = __float2half_rn(v[j]);\n        named_bar_sync(1, 128);",
     "buf[j * 128 + lane] = __float2half_rn(v[j]);", 0, "library"),
    ("transpose_direction", EP, "const bool hi = (q & m) != 0;", "const bool hi = (q & m) == 0;", 0, "library"),
    ("transpose_partner", EP, "const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, m);",
     "const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, m == 1 ? 2 : m);", 0, "library"),
    ("lines_group_rows", EP, "const int q = lane & (P - 1), g = lane / P;", "const int q = lane & (P - 1), g = (lane / P) ^ 1;",
     0, "library"),
    ("lines_row_bound", EP, "if (m < s.M) {", "if (m <= s.M) {", 0, "library"),
    ("lines_f16_pair_order", EP, "__floats2half2_rn(v[8 * i + 2 * w], v[8 * i + 2 * w + 1])",
     "__floats2half2_rn(v[8 * i + 2 * w], v[8 * i + 2 * w])", 0, "library"),
    ("reduce_column_group", EP, "w[q] = __ldcg(slot_vec<BN>(p, slot, row, chunk * 4 + q));",
     "w[q] = __ldcg(slot_vec<BN>(p, slot, row, chunk * 4 + (q ^ 1)));", 0, "library"),
    ("reduce_reads_own_slot", EP, "const int L = f.nseg - (own_mine ? 1 : 0);  // partials read from memory",
     "const int L = f.nseg;", 0, "library"),
    ("reduce_skips_own_index", EP, "auto index_of = [&](int j) { return (own_mine && j >= f.mine) ? j + 1 : j; };",
     "auto index_of = [&](int j) { return j; };", 0, "library"),
    ("reduce_overwrites", EP, "for (int e = 0; e < 16; ++e) v[e] += x[e];", "for (int e = 0; e < 16; ++e) v[e] = x[e];", 0,
     "library"),
    ("reduce_own_dropped", EP, "for (int e = 0; e < 16; ++e) v[e] += own[e];", "for (int e = 0; e < 16; ++e) v[e] += 0.f;", 1,
     "library"),
    ("bulk_expect_short", EP, "mbar_arrive_expect_tx(rbar, (uint32_t)(L * kSlotBytes));",
     "mbar_arrive_expect_tx(rbar, (uint32_t)(L * kSlotBytes / 2));", 0, "library"),
    ("bulk_piece_short", EP, "const int n = kSlotBytes - off < 32768 ? kSlotBytes - off : 32768;",
     "const int n = kSlotBytes - off < 32768 ? kSlotBytes - off : 16384;", 0, "library"),
    ("bulk_ring_place", EP, "const int j = (own_mine && i > f.mine) ? i - 1 : i;  // its place in the ring",
     "const int j = i;", 0, "library"),
    ("bulk_sum_sign", EP, "acc[q].x += w[q].x;", "acc[q].x -= w[q].x;", 0, "library"),
    ("bulk_wait_gone", EP, "if (!wait_bounded(rbar, 0, abort_flag, p.wait_ns, site(2, 4, 0), seg)) return false;",
     "(void)seg;", 0, "library"),
    ("bulk_wait_parity", EP, "if (!wait_bounded(rbar, 0, abort_flag, p.wait_ns, site(2, 4, 0), seg)) return false;",
     "if (!wait_bounded(rbar, 1, abort_flag, p.wait_ns, site(2, 4, 0), seg)) return false;", 0, "library"),
    ("bulk_source_offset", EP, "bulk_load(ring + (size_t)j * kSlotBytes + off, src + off, (uint32_t)n, rbar);",
     "bulk_load(ring + (size_t)j * kSlotBytes + off, src + off / 2, (uint32_t)n, rbar);", 0, "library"),
    ("bulk_lines_lane", EP, "store_rows64<EPI>(p, m0 + (row & ~31), n0 + c0, row & 31, v);",
     "store_rows64<EPI>(p, m0 + (row & ~31), n0 + c0, row & 15, v);", 0, "library"),
    # ---------------------------------------------------------------- the schedule (schedule.h)
    ("sched_group_row", SC, "tm = g * s.group_rows + r % rows;", "tm = g * s.group_rows + r % rows / 2;", 0, "library"),
    ("sched_group_col", SC, "tn = r / rows;", "tn = r % rows;", 0, "library"),
    ("sched_reverse_off", SC, "if (g & 1) tn = s.tiles_n - 1 - tn;", "if (g & 1) tn = s.tiles_n - tn;", 0, "library"),
    ("sched_split_stride", SC, "next_u += P;", "next_u += P + 1;", 0, "library"),
    ("sched_dp_stride", SC, "next_dp += P;", "next_dp += 2 * P;", 0, "library"),
    ("sched_sk_last_kblock", SC, "seg.k1 = left < (long long)(s.kblocks - seg.k0) ? seg.k0 + (int)left : s.kblocks;",
     "seg.k1 = left < (long long)(s.kblocks - seg.k0) ? seg.k0 + (int)left : s.kblocks - 1;", 0, "library"),
    ("sched_sk_begin", SC, "BW_HD inline long long sk_begin(const Sched& s, int c, int P) { return s.sk_iters * c / P; }",
     "BW_HD inline long long sk_begin(const Sched& s, int c, int P) { return s.sk_iters * c / P + (c == 1); }", 0,
     "library"),
    ("sched_fixup_nseg", SC, "f.nseg = sk_owner(s, gf + s.kblocks - 1, P) - f.first + 1;",
     "f.nseg = sk_owner(s, gf + s.kblocks - 1, P) - f.first;", 0, "library"),
    ("sched_split_slot", SC, "if (s.splits > 0) return i * s.sk_tiles + (tile - s.dp_tiles);",
     "if (s.splits > 0) return i * s.sk_tiles;", 0, "library"),
    ("sched_sk_slot", SC, "return 2 * cc + (tile == first ? 0 : 1);", "return 2 * cc;", 0, "library"),
    ("sched_khalf_k0", SC, "seg.k0 = (int)((long long)r * s.kblocks / s.ksplit);", "seg.k0 = 0;", 0, "library"),
    ("sched_split_mine", SC, "f.mine = seg.unit / s.sk_tiles;", "f.mine = seg.unit % s.sk_tiles;", 0, "library"),
    # ---------------------------------------------------------------- the rule (plan.h)
    ("plan_tokens_rounding", PL, "q.bn = (M + 15) / 16 * 16;", "q.bn = (M + 7) / 16 * 16;", 0, "library"),
    ("plan_swap_tiles_ragged", PL, "q.tiles_n = (N + 127) / 128;", "q.tiles_n = N / 128;", 0, "library"),
    ("plan_pair_rows", PL, "q.tiles_m = (M + 128 * ranks - 1) / (128 * ranks);", "q.tiles_m = (M + 127) / (128 * ranks);", 0,
     "library"),
    ("plan_sk_tiles", PL, "q.sk_tiles = q.tiles - q.dp_tiles;", "q.sk_tiles = q.tiles - q.dp_tiles - 1;", 0, "library"),
    # ---------------------------------------------------------------- options of the next build
    ("ksplit_recv_bytes", GK, "const uint32_t recv_bytes = (uint32_t)((kc - 1) * (own1 - own0)) * 8192u;",
     "const uint32_t recv_bytes = (uint32_t)((kc - 1) * (own1 - own0)) * 4096u;", 0, "library"),
    ("ksplit_piece", GK, "const int piece = (kr < o ? kr : kr - 1) * len + (ch - r0);", "const int piece = (kr < o ? kr : kr - 1) * len;",
     0, "library"),
    ("ksplit_sum_order", GK, "const float4* src = ring + (size_t)((sb < kr ? sb : sb - 1) * (own1 - own0) +",
     "const float4* src = ring + (size_t)((sb < kr ? sb : sb) * (own1 - own0) +", 0, "library"),
    ("ksplit_owner_run", SC, "BW_HD inline int ksplit_run(int o, int n, int c) { return o * n / c; }",
     "BW_HD inline int ksplit_run(int o, int n, int c) { return o * n / c + (o == 1); }", 0, "library"),
    ("wide_first_half_early", GK, "if (G::kHalves && c0 + kLdw == AN / 2) release_acc(0);  // the first half is read",
     "if (G::kHalves && c0 == 0) release_acc(0);", 0, "wide"),
    ("wide_catch_up_k", GK, "issue(st, held_kb + i, 1, 2);", "issue(st, held_kb, 1, 2);", 0, "wide"),
    ("wide_second_half_cols", GK, "const uint32_t yw = sy + (uint32_t)((SWAP ? 0 : w) * G::kBPart * kBK * 2);",
     "const uint32_t yw = sy;", 0, "wide"),
    ("wide_catch_up_wait", GK, "if (!wait_bounded(&tempty[1], aph ^ 1u, abort_flag, p.wait_ns, site(1, 3, 1), seg)) return false;",
     "(void)0;", 0, "wide"),
    # ---------------------------------------------------------------- dynamic units (BW_DYN_UNITS)
    ("dyn_unit_overrun", GK, "if (u >= s.sk_tiles * s.splits) u = -1;", "if (u > s.sk_tiles * s.splits) u = -1;", 0,
     "dyn"),
    ("dyn_empty_count", GK, "mbar_init(&uq_empty[i], 2);", "mbar_init(&uq_empty[i], 1);", 0, "dyn"),
    ("dyn_full_parity", GK, "if (!wait_bounded(&uq_full[qs], (uint32_t)((qi / kPlanUnitQ) & 1), abort_flag, p.wait_ns,\n                                  site(1, 9",
     "if (!wait_bounded(&uq_full[qs], (uint32_t)((qi / kPlanUnitQ) & 1) ^ 1u, abort_flag, p.wait_ns,\n                                  site(1, 9", 0, "dyn"),
    ("dyn_epi_slot", GK, "                sg.unit = epi_unit[seg & 1];", "                sg.unit = epi_unit[0];", 0,
     "dyn"),
    ("dyn_no_reset", GK, "            atomicExch(next_unit, 0);\n", "", 0, "dyn"),
    ("dyn_epi_queue_slot", GK, "                        u = uq[qs];", "                        u = uq[(qs + 1) % kPlanUnitQ];", 0,
     "dyn"),
    ("dyn_unit_k", SC, "    k1 = (int)((long long)(sp + 1) * s.kblocks / s.splits);\n}",
     "    k1 = (int)((long long)(sp + 1) * s.kblocks / s.splits) - (sp == 0);\n}", 0, "dyn"),
    # ---------------------------------------------------------------- the TMA-store epilogue (BW_EPI_TMA)
    ("tma_no_read_wait", EP, "if (lane == 0) bulk_wait_read<1>();", "(void)0;", 0, "tma"),
    ("tma_one_buffer", GK, "(epi_chunks++ & 1u) * 16384u", "(epi_chunks++ & 0u) * 16384u", 0, "tma"),
    ("tma_swizzle_off", EP, "row[j ^ (lane & 7)] = make_uint4(h[0], h[1], h[2], h[3]);",
     "row[j] = make_uint4(h[0], h[1], h[2], h[3]);", 0, "tma"),
    ("tma_box_rows", EP, "tma_store_2d(tmc, quarter, n, r0);", "tma_store_2d(tmc, quarter, n, r0 + 8);", 0, "tma"),
    ("tma_quarter_overlap", GK, "(epi_chunks++ & 1u) * 16384u + q * 4096", "(epi_chunks++ & 1u) * 16384u + q * 2048", 0,
     "tma"),
    ("tma_uncommitted", EP, "tma_store_2d(tmc, quarter, n, r0);\n        bulk_commit();",
     "tma_store_2d(tmc, quarter, n, r0);", 0, "tma"),
    ("tma_pair_order", EP, "const __half2 x = __floats2half2_rn(v[8 * j + 2 * w], v[8 * j + 2 * w + 1]);",
     "const __half2 x = __floats2half2_rn(v[8 * j + 2 * w + 1], v[8 * j + 2 * w]);", 0, "tma"),
    ("swap_pair_weights", GK, "const int wcol = (tn * R + rank) * 128 * WM;", "const int wcol = (tn * R) * 128 * WM;", 0,
     "next"),
    ("swap_pair_tokens", GK, "load_tile<PAIR, BW_HINT_A>(sy, &tmy, kb * kBK, rank * (BN / R),",
     "load_tile<PAIR, BW_HINT_A>(sy, &tmy, kb * kBK, 0,", 0, "next"),
]

# The calls each build's mutants run, in order; a mutant stops at its first reported call.  (M, N, K, emulated SMs,
# variant, epi: 0 fp16 / 1 fp32 / 2 SwiGLU, B as N x K[, the K split forced to clusters of c and tiles of 128 wm
# columns: c * 16 + wm])
CASES = {
    "library": [
        (256, 256, 128, 8, 0, 0, False),    # one pair tile
        (512, 2048, 128, 8, 0, 0, False),   # four pair tiles per pair: both accumulators reused twice
        (512, 1280, 4096, 8, 0, 0, False),  # pair tiles, a split-K tail (bulk and plain reductions)
        (256, 1280, 256, 8, 0, 0, False),   # pair tiles, stream-K over one wave and a part
        (16, 256, 128, 8, 0, 0, False),     # swap-AB, K halves on a cluster of two
        (16, 1280, 256, 8, 0, 0, False),    # swap-AB stream-K
        (64, 2304, 256, 8, 0, 0, False),    # swap-AB stream-K, 256-column tiles
        (16, 1024, 384, 8, 0, 0, False),    # swap-AB K halves, 256-column tiles
        (128, 2176, 128, 16, 0, 0, False),  # swap-AB stream-K, bn 128, ragged N
        (1, 256, 128, 8, 0, 0, False),      # one token
        (24, 1024, 384, 8, 0, 0, False),    # 24 tokens in bn 32
        (130, 320, 192, 8, 0, 0, False),    # a ragged pair tile, odd K-blocks
        (300, 1280, 4096, 8, 0, 0, False),  # ragged rows with a split-K tail
        (512, 1024, 256, 8, 0, 1, False),   # fp32 output
        (512, 1024, 256, 8, 0, 2, False),   # SwiGLU output
        (256, 256, 128, 8, 0, 0, True),     # B as N x K: a pair tile
        (16, 1280, 256, 8, 0, 0, True),     # B as N x K: swap-AB stream-K
        (16, 256, 128, 8, 0, 0, True),      # B as N x K: K halves
        (256, 512, 256, 8, 5, 0, False),    # 128 x 256 single-SM tiles
        (256, 512, 256, 8, 6, 0, False),    # 128 x 64 tiles
        (256, 512, 256, 8, 1, 0, False),    # whole pair tiles only
        (2304, 512, 128, 8, 0, 0, False),   # nine rows of pair tiles: a second, reversed serpentine group
        (512, 2560, 4096, 16, 0, 0, False), # four two-way split tiles, each pair's unit before its whole tiles
        (512, 256, 4096, 8, 0, 0, False),   # two two-way split tiles, no whole tiles: the reductions by bulk copies
        (256, 1280, 8192, 16, 0, 0, False), # five three-way split tiles, 15 units on 8 pairs
        (16, 1280, 4096, 8, 0, 0, False),   # swap-AB stream-K: 10 tiles on 8 blocks, partial segments before the last
        (24, 3200, 2048, 16, 0, 0, True),   # swap-AB stream-K, bn 32, a half tile
        (128, 1024, 1024, 8, 0, 0, False),  # the K split over clusters of 2 to 8 (the rule's, then forced sizes)
        (96, 640, 1024, 16, 0, 0, False, 3 * 16 + 1),
        (64, 704, 1024, 16, 0, 0, False, 4 * 16 + 2),
        (112, 256, 4096, 16, 0, 0, False, 8 * 16 + 1),
        (96, 448, 2624, 16, 0, 0, True, 7 * 16 + 2),
        (128, 512, 2048, 16, 0, 0, False, 8 * 16 + 2),  # 16 chunks over 8 blocks of 256-column tiles
        (16, 256, 2048, 8, 0, 0, False),    # K halves deeper than the stage ring
        (256, 512, 1024, 8, 5, 0, False),   # single-SM tiles deeper than the stage ring
        (64, 2304, 1024, 8, 0, 0, False),   # swap-AB stream-K, 256-column tiles, several tiles per block
        (128, 2112, 128, 16, 0, 0, False),  # swap-AB stream-K, N not a multiple of 128
        (300, 1024, 256, 8, 0, 2, False),   # SwiGLU output, ragged rows
        (300, 1280, 4096, 8, 0, 1, False),  # fp32 output, ragged rows, a split-K tail
    ],
    "next": [
        (48, 2304, 256, 8, 0, 0, False),    # swap-AB on SM pairs (stream-K swap shapes from 33 tokens)
        (80, 2304, 256, 8, 0, 0, False),
        (128, 4096, 256, 8, 0, 0, False),
        (16, 1280, 256, 8, 0, 0, True),
        (80, 2304, 256, 8, 0, 0, True),
    ],
    "halves": [
        (16, 256, 128, 8, 0, 0, False),     # K halves on a cluster of two
        (16, 256, 2048, 8, 0, 0, False),    # deeper than the stage ring
        (16, 1024, 384, 8, 0, 0, False),    # 256-column tiles
        (96, 448, 320, 8, 0, 0, False),     # bn 96, odd K-blocks
        (1, 256, 128, 8, 0, 0, False),      # one token
        (16, 256, 128, 8, 0, 0, True),      # B as N x K
    ],
    "tma": [
        (256, 256, 128, 8, 0, 0, False),    # one pair tile
        (512, 2048, 128, 8, 0, 0, False),   # four pair tiles per pair
        (130, 320, 192, 8, 0, 0, False),    # ragged rows (the map clips them)
        (256, 512, 1024, 8, 5, 0, False),   # single-SM tiles
        (256, 512, 256, 8, 6, 0, False),    # 128 x 64 tiles
        (256, 256, 128, 8, 0, 0, True),     # B as N x K
    ],
    "dyn": [
        (16, 1280, 4096, 8, 0, 0, False),   # dynamic units: 10 tiles x 4 units on 8 blocks
        (24, 3200, 2048, 16, 0, 0, True),   # dynamic units, bn 32, a half tile
        (1, 2304, 2048, 8, 0, 0, False),    # one token, 18 tiles x 2 units
        (64, 2304, 1024, 8, 0, 0, False),   # large accumulators: static stream-K beside the option
    ],
    "wide": [
        (256, 1024, 256, 8, 0, 0, False),   # 256 x 512 pair tiles, whole waves
        (512, 2048, 512, 8, 0, 0, False),
        (256, 1536, 1024, 8, 0, 0, False),  # with stream-K
        (300, 1280, 384, 8, 0, 0, False),   # ragged
        (512, 2048, 512, 8, 0, 0, True),
    ],
}


# ------------------------------------------------------------------------------------------------------ one mutant
def locate(text, mutation):
    """Where occurrence `nth` of the mutation's text starts in `text` (ValueError if it is not there)."""
    name, rel, before, _, nth, _ = mutation
    at = -1
    for _ in range(nth + 1):
        at = text.find(before, at + 1)
        if at < 0:
            raise ValueError(f"{name}: occurrence {nth} of its text is not in {rel}")
    return at


def apply(tree, mutation):
    name, rel, before, after, nth, _ = mutation
    path = os.path.join(tree, "gemm-ladder_b200", rel)
    with open(path) as f:
        text = f.read()
    at = locate(text, mutation)
    with open(path, "w") as f:
        f.write(text[:at] + after + text[at + len(before):])


def build(tree, build_name, out):
    cmd = ["g++", "-std=c++20", "-O1", "-pthread", "-DBW_EMULATE", *[f"-D{d}" for d in BUILDS[build_name]], "-fPIC",
           "-shared", "-w", f"-I{CUDA_INCLUDE}", f"-I{os.path.join(tree, 'include')}",
           f"-I{os.path.join(tree, 'gemm-ladder_b200', 'csrc')}", os.path.join(tree, "gemm-ladder_b200", "emu", "emu.cpp"),
           "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.returncode == 0, r.stderr[-2000:]


def snapshot(dst):
    """The sources every mutant starts from, copied once when a run starts (later edits of the tree do not reach it)."""
    os.makedirs(os.path.join(dst, "gemm-ladder_b200"))
    shutil.copytree(os.path.join(PKG, "csrc"), os.path.join(dst, "gemm-ladder_b200", "csrc"))
    shutil.copytree(os.path.join(PKG, "emu"), os.path.join(dst, "gemm-ladder_b200", "emu"),
                    ignore=shutil.ignore_patterns("*.py", "__pycache__"))
    shutil.copytree(os.path.join(ROOT, "include"), os.path.join(dst, "include"))


def run_one(mutation, build_name, timeout_s, cluster_batch, base):
    """Compile the sources of `base` (a snapshot) with `mutation` (None: unmodified) and run the build's calls in a
    child process.  Returns a dict: name, build, reported (bool), why."""
    name = mutation[0] if mutation else "unmodified"
    with tempfile.TemporaryDirectory(prefix="bwpb_") as tmp:
        os.rmdir(tmp)
        shutil.copytree(base, tmp)
        if mutation:
            apply(tmp, mutation)
        lib = os.path.join(tmp, "libbwemu.so")
        ok, err = build(tmp, build_name, lib)
        if not ok:
            return {"name": name, "build": build_name, "reported": True, "why": "does not compile",
                    "detail": err.strip().splitlines()[-1] if err.strip() else ""}
        t0 = time.time()
        try:
            r = subprocess.run([sys.executable, os.path.abspath(__file__), "--check", lib, "--build", build_name,
                                "--cluster-batch", str(cluster_batch)],
                               capture_output=True, text=True, timeout=timeout_s)
        except subprocess.TimeoutExpired:
            return {"name": name, "build": build_name, "reported": True, "why": f"the emulator hung ({timeout_s} s)"}
        lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
        if r.returncode != 0 or not lines:
            return {"name": name, "build": build_name, "reported": True,
                    "why": f"the emulator process ended with status {r.returncode}",
                    "detail": (r.stderr or r.stdout).strip()[-300:]}
        res = json.loads(lines[-1])
        res.update({"name": name, "build": build_name, "seconds": round(time.time() - t0, 1)})
        return res


# ------------------------------------------------------------------------------------------------------ the check
def check(lib_path, build_name, cluster_batch):
    """Runs the build's calls on the emulator library at lib_path; prints one JSON line: reported, why."""
    import numpy as np

    sys.path.insert(0, ROOT)
    from oracle import oracle

    L = ctypes.CDLL(lib_path)
    vp, i = ctypes.c_void_p, ctypes.c_int
    L.bw_emu_gemm.argtypes = [vp, vp, vp, i, i, i, i, i, i, i, ctypes.POINTER(ctypes.c_uint),
                              ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, i]
    L.bw_emu_gemm.restype = i
    L.bw_emu_set.argtypes = [ctypes.c_char_p, ctypes.c_longlong]
    L.bw_emu_set(b"wait_ns", 4_000_000_000)        # a wait that gives up is a report, so no need to wait long
    L.bw_emu_set(b"barrier_limit_ms", 8000)
    L.bw_emu_set(b"cluster_batch", cluster_batch)
    L.bw_emu_set(b"ld_delay_us", 30)               # a slow epilogue: an MMA that does not wait for it overwrites
    L.bw_emu_set(b"start_jitter_us", 50000)        # blocks start apart: a peer's barriers unset show
    if build_name == "tma":                        # TMA stores that lag behind the epilogue: a staging buffer rewritten
        L.bw_emu_set(b"engine_delay_us", 2000)     # before its store has read it shows in C

    def call(A, B, M, N, K, sms, variant, epi, tn):
        Bx = np.ascontiguousarray(np.asarray(B).reshape(K, N).T) if tn else np.ascontiguousarray(B)
        cols = N // 2 if epi == 2 else N
        Cp = np.full((M + 16, cols), np.nan, np.float32) if epi == 1 else np.full((M + 16, cols), 0xFFFF, np.uint16)
        st = (ctypes.c_uint * 4)()
        dirty, nf = ctypes.c_int(), ctypes.c_int()
        msg = ctypes.create_string_buffer(256)
        rc = L.bw_emu_gemm(np.ascontiguousarray(A).ctypes.data, Bx.ctypes.data, Cp.ctypes.data, M, N, K, sms, variant,
                           epi, int(tn), st, ctypes.byref(dirty), ctypes.byref(nf), msg, 256)
        return rc, Cp, list(st), dirty.value, nf.value, msg.value.decode()

    def report(why):
        print(json.dumps({"reported": True, "why": why}), flush=True)

    for case in CASES[build_name]:
        M, N, K, sms, variant, epi, tn = case[:7]
        L.bw_emu_set(b"force_ksplit", case[7] if len(case) > 7 else 0)
        tag = f"{M}x{N}x{K} on {sms} SMs, v{variant}, epi {epi}{', B as N x K' if tn else ''}"
        A, B = oracle.lcg_inputs(M, N, K)
        ref = oracle.gemm_f64(A, B)
        first = None
        for rep in range(3):
            # the second launch starts each cluster's first block 20 ms after the others: a block that sends its sums
            # into the first block's ring before that block says its ring is idle then overwrites live stages.  The
            # third starts block b 100 b ms after block 0 (longer than a segment takes here): a split tile's later
            # block then finishes its part last while it has segments to come, and reduces the tile with its stage
            # ring busy
            L.bw_emu_set(b"lead_skew_us", 20000 if rep == 1 else 0)
            L.bw_emu_set(b"block_ramp_us", 100000 if rep == 2 else 0)
            rc, Cp, st, dirty, nf, msg = call(A, B, M, N, K, sms, variant, epi, tn)
            L.bw_emu_set(b"lead_skew_us", 0)
            L.bw_emu_set(b"block_ramp_us", 0)
            C, pad = Cp[:M], Cp[M:]
            if rc != 0:
                return report(f"{tag}: status {rc}")
            if nf:
                return report(f"{tag}: emulator finding: {msg}")
            if st[0] != 0:
                return report(f"{tag}: device status {st[0]} at site {st[1]:#x} (a bounded wait gave up)")
            if dirty:
                return report(f"{tag}: {dirty} split-tile counters left set")
            if not (np.isnan(pad).all() if epi == 1 else (pad == 0xFFFF).all()):
                return report(f"{tag}: an element written past row M")
            if epi == 0:
                r = oracle.check(C, ref, K)
                if r["nonfinite"] or r["violations"] or r["normwise"] > 2e-3:
                    return report(f"{tag}: result outside the gates ({r['nonfinite']} not finite, {r['violations']} "
                                  f"over the per-element bound, normwise {r['normwise']:.2e})")
            elif epi == 1:
                if not np.isfinite(C).all() or np.abs(C - ref).max() > 1e-5 * np.abs(ref).max():
                    return report(f"{tag}: fp32 result wrong")
            else:
                g = ref.reshape(M, -1, 2, 128)
                gate, up = g[:, :, 0, :].reshape(M, -1), g[:, :, 1, :].reshape(M, -1)
                act = gate / (1.0 + np.exp(-gate)) * up
                got = C.view(np.float16).astype(np.float64)
                if not np.isfinite(got).all() or np.abs(got - act).max() > 2e-3 * np.abs(act).max():
                    return report(f"{tag}: SwiGLU result wrong")
            if first is None:
                first = C.copy()
            elif not np.array_equal(first.view(np.uint8), C.view(np.uint8)):
                return report(f"{tag}: two calls differ bit for bit")
    print(json.dumps({"reported": False, "why": "every call passed"}), flush=True)


# ------------------------------------------------------------------------------------------------------ main
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=max(1, (os.cpu_count() or 2) // 2))
    ap.add_argument("--only", default=None, help="names, comma-separated")
    ap.add_argument("--list", action="store_true")
    ap.add_argument("--out", default=None, help="also write the results here (text)")
    ap.add_argument("--timeout", type=int, default=600)
    ap.add_argument("--cluster-batch", type=int, default=2)
    ap.add_argument("--check", default=None, help=argparse.SUPPRESS)
    ap.add_argument("--build", default="library", help=argparse.SUPPRESS)
    a = ap.parse_args()
    if a.check:
        check(a.check, a.build, a.cluster_batch)
        return 0
    names = [m[0] for m in MUTATIONS]
    assert len(names) == len(set(names)), "mutation names must be unique"
    if a.list:
        for m in MUTATIONS:
            print(f"{m[0]:34s} {m[5]:8s} {m[1]}")
        print(f"{len(MUTATIONS)} mutations")
        return 0
    todo = [m for m in MUTATIONS if not a.only or m[0] in a.only.split(",")]
    # every mutation's text must be where it says in the unmodified sources, before anything is compiled
    for m in todo:
        with open(os.path.join(PKG, m[1])) as f:
            text = f.read()
        at = -1
        for _ in range(m[4] + 1):
            at = text.find(m[2], at + 1)
            if at < 0:
                raise SystemExit(f"{m[0]}: occurrence {m[4]} of its text is not in {m[1]}")
    t0 = time.time()
    results = []
    builds = sorted({m[5] for m in todo})
    base_dir = tempfile.mkdtemp(prefix="bwpb_base_")
    base = os.path.join(base_dir, "src")
    snapshot(base)
    with concurrent.futures.ThreadPoolExecutor(max_workers=a.jobs) as ex:
        futs = [ex.submit(run_one, None, b, a.timeout, a.cluster_batch, base) for b in builds]
        futs += [ex.submit(run_one, m, m[5], a.timeout, a.cluster_batch, base) for m in todo]
        for f in concurrent.futures.as_completed(futs):
            r = f.result()
            results.append(r)
            mark = "REPORTED" if r["reported"] else "missed  "
            if r["name"] == "unmodified":
                mark = "CLEAN   " if not r["reported"] else "BROKEN  "
            print(f"{mark} {r['name']:34s} [{r['build']}] {r['why']}", flush=True)
    shutil.rmtree(base_dir, ignore_errors=True)
    clean = [r for r in results if r["name"] == "unmodified"]
    muts = [r for r in results if r["name"] != "unmodified"]
    caught = sum(r["reported"] for r in muts)
    ok = all(not r["reported"] for r in clean) and caught == len(muts)
    summary = (f"{caught} of {len(muts)} planted bugs reported; unmodified sources "
               f"{'clean' if all(not r['reported'] for r in clean) else 'NOT clean'} in {', '.join(builds)}; "
               f"{time.time() - t0:.0f} s: {'PLANTED-BUG TEST OK' if ok else 'PLANTED-BUG TEST FAILED'}")
    print(summary)
    if a.out:
        order = {m[0]: k for k, m in enumerate(MUTATIONS)}
        with open(a.out, "w") as f:
            f.write("# python gemm-ladder_b200/emu/planted_bugs.py --out " + os.path.relpath(a.out, ROOT) + "\n")
            for r in sorted(results, key=lambda r: (r["name"] != "unmodified", order.get(r["name"], -1), r["build"])):
                mark = ("clean" if not r["reported"] else "BROKEN") if r["name"] == "unmodified" else (
                    "reported" if r["reported"] else "MISSED")
                f.write(f"{mark:8s} {r['name']:34s} [{r['build']}] {r['why']}\n")
            f.write(summary + "\n")
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
