// ptx_emu.h -- the host emulator's version of csrc/ptx.cuh: the same functions, carried out on the CPU by the
// execution model of emu_runtime.h (each block's 192 threads as host threads, a cluster's blocks side by side).
//
// What each instruction does here:
//   mbarrier         a table per block (arrival count, pending arrivals, transaction bytes, completed phases);
//                    try_wait.parity(p) is true once the phase of parity p has completed.
//   TMA tiled load   queued to the block's TMA engine (emu_runtime.h, Engine), which later copies the box element by
//                    element from the tensor map's global array (zeros outside it) into shared memory in the 128-byte
//                    swizzle (16-byte chunk c of 128-byte row r at c ^ (r % 8)), then completes its bytes on the
//                    barrier (a pair's on the leader block's barrier).  Bulk copies likewise.
//   tcgen05.mma      queued to the block's tensor core, which later reads the operands through the shared-memory
//                    descriptors (start, leading and stride byte offsets, 128-byte swizzle; K-major or MN-major from the
//                    instruction descriptor) and multiplies them in fp32 into the block's tensor memory (128 lanes x 512
//                    columns); the pair form takes A's rows and B's columns from both blocks and writes each block's
//                    rows to its own tensor memory.
//   tcgen05.commit   queued behind the MMAs: an arrival on the barrier once they have run.
//   tcgen05.ld       lane (address lane + the thread's lane in its warp), 16 consecutive columns.
//   clusters         rank, mapa (the rank in the address's top byte), barrier.cluster, remote arrivals, st.async (queued
//                    like a copy: its bytes land in the other block, and complete on its barrier, later).
// Every access to shared or tensor memory is bounds-checked, and the checks that fail are recorded as findings
// (emu::finding) instead of being carried out.
#pragma once
#include <cuda.h>

#include "emu_runtime.h"

namespace bw {

// ------------------------------------------------------------------ addresses and timers
inline uint32_t smem_u32(const void* p) { return emu::offset_of(p); }
inline uint64_t globaltimer_ns() { return emu::now_ns(); }
inline uint32_t lane_id() { return (uint32_t)(emu::t_tid & 31); }

// ------------------------------------------------------------------ mbarrier
inline void mbar_init(uint64_t* bar, uint32_t count) { emu::mb_init(emu::t_cta, emu::offset_of(bar), (int)count); }
inline void fence_barrier_init() {}
inline void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    emu::mb_arrive(emu::t_cta, emu::offset_of(bar), (long long)bytes);
}
inline void mbar_arrive(uint64_t* bar) { emu::mb_arrive(emu::t_cta, emu::offset_of(bar), 0); }
inline bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    return emu::mb_try_wait(emu::cta_of(bar), emu::off_of(bar), parity);
}

inline unsigned int g_status[4];
inline thread_local unsigned int* t_status = g_status;  // the status word of the emulated GPU this thread runs on
enum : uint32_t { kStatusTimeout = 3u };

inline void record_timeout(volatile int* abort_flag, uint32_t where, int seg)
{
    *abort_flag = 1;
    unsigned expected = 0u;
    if (__atomic_compare_exchange_n(&t_status[0], &expected, (unsigned)kStatusTimeout, false, __ATOMIC_SEQ_CST,
                                    __ATOMIC_SEQ_CST)) {
        t_status[1] = where;
        t_status[2] = blockIdx.x;
        t_status[3] = (unsigned)seg;
    }
}

// A spinning thread gives way to the other emulated threads: a yield at first, then short sleeps (thousands of host
// threads spinning on yields alone spend most of their time in the scheduler).
inline void spin_pause(uint32_t i)
{
    if (i < 64)
        std::this_thread::yield();
    else
        std::this_thread::sleep_for(std::chrono::microseconds(20));
}

// The bounded wait of ptx.cuh, with a pause in the spin so that the other emulated threads run.
inline bool wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, uint64_t limit_ns, uint32_t where, int seg)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        spin_pause(i);
        if ((i & 31u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                record_timeout(abort_flag, where, seg);
                return false;
            }
        }
    }
}

// ------------------------------------------------------------------ system scope (the emulated GPUs of one process)
inline unsigned ld_acquire_sys(const unsigned* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void st_release_sys(unsigned* p, unsigned v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
inline void fence_sys() { std::atomic_thread_fence(std::memory_order_seq_cst); }
inline bool wait_flag(const unsigned* p, unsigned want, volatile int* abort_flag, uint64_t limit_ns, uint32_t where,
                      int seg)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if ((int)(ld_acquire_sys(p) - want) >= 0) return true;
        spin_pause(i);
        if ((i & 15u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                record_timeout(abort_flag, where, seg);
                return false;
            }
        }
    }
}

inline bool wait_bounded(uint64_t* barp, uint32_t parity, volatile int* abort_flag, uint64_t limit_ns, uint32_t where,
                         int seg)
{
    const uint32_t bar = smem_u32(barp);
    if (mbar_try_wait(bar, parity)) return true;
    return wait_slow(bar, parity, abort_flag, limit_ns, where, seg);
}

// ------------------------------------------------------------------ TMA
inline void prefetch_tmap(const void*) {}
// One launch at a time here: a grid never starts before the one ahead of it has finished.
inline void griddep_launch() {}
inline void griddep_wait() {}
// A tiled load into this block's shared memory, carried out later by its TMA engine; its bytes complete on `bar`
// (a shared::cluster address: possibly the pair leader's) when it lands.
inline void tma_post(void* dst, const void* tmap, int x, int y, int z, uint32_t bar)
{
    emu::Cta* c = emu::t_cta;
    const bool keep = emu::keep_completion();
    CUtensorMap map;
    std::memcpy(&map, tmap, sizeof map);  // the map lives in the kernel's parameters: copied as the TMA unit would
    c->tma.post([=] {
        const long long bytes = emu::tma_copy(dst, &map, x, y, z);
        if (keep) emu::mb_complete_tx(emu::cta_of(bar), emu::off_of(bar), bytes);
    });
}
inline void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar)
{
    tma_post(dst, tmap, x, y, 0, emu::offset_of(bar));
}
inline void tma_load_2d_hint(void* dst, const void* tmap, int x, int y, uint64_t* bar, uint64_t)
{
    tma_load_2d(dst, tmap, x, y, bar);
}
inline void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar)
{
    tma_post(dst, tmap, x, y, z, emu::offset_of(bar));
}
inline void tma_load_3d_hint(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar, uint64_t)
{
    tma_load_3d(dst, tmap, x, y, z, bar);
}
// One memory model for every access here: the proxy fences are ordinary full fences.
inline void fence_proxy_async_global() { std::atomic_thread_fence(std::memory_order_seq_cst); }
inline void fence_proxy_async_shared() { std::atomic_thread_fence(std::memory_order_seq_cst); }
inline void tma_store_2d(const void* tmap, const void* src, int x, int y) { emu::tma_store(tmap, src, x, y); }
inline void bulk_commit() { emu::store_commit(); }
template <int N>
inline void bulk_wait_read() { emu::store_wait(N); }
template <int N>
inline void bulk_wait() { emu::store_wait(N); }
inline uint64_t policy_evict_first() { return 0; }
inline uint64_t policy_evict_last() { return 0; }
inline void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    emu::Cta* c = emu::t_cta;
    const bool keep = emu::keep_completion();
    const uint32_t boff = emu::offset_of(bar);
    c->tma.post([=] {
        emu::bulk_copy(dst, src, bytes);
        if (keep) emu::mb_complete_tx(c, boff, bytes);
    });
}

// ------------------------------------------------------------------ clusters
inline uint32_t cluster_ctarank() { return (uint32_t)emu::t_cta->rank; }
inline uint32_t mapa_shared(uint32_t saddr, uint32_t rank) { return emu::mapa(saddr, rank); }
inline void cluster_sync() { emu::cluster_sync(); }
inline void mbar_arrive_cluster(uint32_t cluster_addr) { emu::mb_arrive(emu::cta_of(cluster_addr), emu::off_of(cluster_addr), 0); }
// st.async: the 16 bytes land in the other block later (queued to this block's TMA engine, standing for the path
// between the blocks), then complete on that block's barrier.
inline void st_async_v4(uint32_t dst, uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t bar)
{
    emu::t_cta->tma.post([=] {
        const uint32_t v[4] = {a, b, c, d};
        emu::remote_store(dst, v, 16);
        emu::mb_complete_tx(emu::cta_of(bar), emu::off_of(bar), 16);
    });
}
inline void fence_acq_rel_cluster() { std::atomic_thread_fence(std::memory_order_seq_cst); }
inline void tma_load_2d_pair(void* dst, const void* tmap, int x, int y, uint32_t bar)
{
    tma_post(dst, tmap, x, y, 0, bar);
}
inline void tma_load_3d_pair(void* dst, const void* tmap, int x, int y, int z, uint32_t bar)
{
    tma_post(dst, tmap, x, y, z, bar);
}
inline void tma_load_2d_pair_hint(void* dst, const void* tmap, int x, int y, uint32_t bar, uint64_t)
{
    tma_load_2d_pair(dst, tmap, x, y, bar);
}

// ------------------------------------------------------------------ tensor memory and the tensor core
inline void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) { emu::tmem_alloc(dst_smem, ncols); }
inline void tmem_relinquish() {}
inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) { emu::tmem_dealloc(taddr, ncols); }
inline void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) { emu::tmem_alloc(dst_smem, ncols); }
inline void tmem_relinquish_pair() {}
inline void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) { emu::tmem_dealloc(taddr, ncols); }
inline void tc_fence_before() {}
inline void tc_fence_after() {}
// MMAs and their commits go to the block's tensor core, which carries them out later and in order: a commit arrives
// once the MMAs issued before it have run.
inline void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
    emu::Engine& tc = emu::t_cta->tc;
    ++tc.mmas;
    tc.post([=, &tc] {
        emu::mma(d_tmem, adesc, bdesc, idesc, accumulate != 0, false);
        --tc.mmas;
    });
}
inline void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate)
{
    emu::Engine& tc = emu::t_cta->tc;
    ++tc.mmas;
    tc.post([=, &tc] {
        emu::mma(d_tmem, adesc, bdesc, idesc, accumulate != 0, true);
        --tc.mmas;
    });
}
inline void mma_commit_pair(uint32_t bar)
{
    emu::t_cta->tc.post([=] { emu::mb_arrive(emu::cta_of(bar), emu::off_of(bar), 0); });
}
inline void mma_commit(uint64_t* bar)
{
    const uint32_t off = emu::offset_of(bar);
    emu::Cta* c = emu::t_cta;
    c->tc.post([=] { emu::mb_arrive(c, off, 0); });
}
inline void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) { emu::tmem_ld(taddr, r); }
inline void tmem_wait_ld() {}

// ------------------------------------------------------------------ descriptors (the same encodings as ptx.cuh)
inline uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
constexpr uint32_t idesc_f16_f32(int m, int n, bool a_mn_major, bool b_mn_major)
{
    return (1u << 4) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

// ------------------------------------------------------------------ global memory ordering, named barriers
inline int ld_acquire_gpu(const int* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
inline void named_bar_sync(uint32_t id, uint32_t count) { emu::named_sync((int)id, (int)count); }

}  // namespace bw
