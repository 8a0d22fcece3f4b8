// ptx.cuh -- the sm_100a instructions the rung's kernels use, as thin inline-PTX wrappers.
//
// mbarrier (arrive / expect_tx / try_wait.parity), TMA tiled loads (cp.async.bulk.tensor), the 5th-generation tensor
// core (tcgen05.alloc / mma / commit / ld / wait / fence / dealloc) and the shared-memory matrix descriptors it reads.
// Every spin on an mbarrier goes through wait_bounded(): it gives up after a time limit, records where in the device
// status word and raises the block's abort flag, so a kernel whose pipeline stalls returns an error instead of hanging
// the GPU.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifdef BW_EMULATE
// The host emulator (gemm-ladder_b200/emu/): the same functions, carried out on the CPU.
#include "../emu/ptx_emu.h"
#else

namespace bw {

// ------------------------------------------------------------------ addresses and timers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes the barriers' initialisation visible to the async proxy (TMA, tensor core) and to the cluster.
__device__ __forceinline__ void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// True once the phase of parity `parity` has completed (a fresh barrier counts its phase "1" as completed).
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// ------------------------------------------------------------------ the device status word
// [0]: status code (0 ok, 3 a bounded wait gave up); [1]: the first site that gave up (role << 16 | barrier id);
// [2]: blockIdx.x of that block; [3]: the segment it was on.  Cleared by the host.
__device__ unsigned int g_status[4];

enum : uint32_t { kStatusTimeout = 3u };

// A wait that gave up: the first one since the host cleared the status word records `where`, the block's abort flag
// rises.
__device__ __forceinline__ void record_timeout(volatile int* abort_flag, uint32_t where, int seg)
{
    *abort_flag = 1;
    if (atomicCAS(&g_status[0], 0u, kStatusTimeout) == 0u) {
        g_status[1] = where;
        g_status[2] = blockIdx.x;
        g_status[3] = (unsigned)seg;
    }
    __threadfence();
}

// Spins on (bar, parity) until the phase completes, the block's abort flag rises, or `limit_ns` pass. On a timeout it
// records `where` and raises the abort flag; returns false on timeout or abort.
__device__ __noinline__ bool wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, uint64_t limit_ns,
                                       uint32_t where, int seg)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                record_timeout(abort_flag, where, seg);
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool wait_bounded(uint64_t* barp, uint32_t parity, volatile int* abort_flag,
                                             uint64_t limit_ns, uint32_t where, int seg)
{
    const uint32_t bar = smem_u32(barp);
    if (mbar_try_wait(bar, parity)) return true;
    return wait_slow(bar, parity, abort_flag, limit_ns, where, seg);
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void prefetch_tmap(const void* tmap)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// A 2-D tiled load of one box into shared memory, completing `bytes` on `bar` (x: the innermost coordinate).
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// The same with an L2 cache policy (createpolicy), e.g. evict-first for a stream of weights read once.
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const void* tmap, int x, int y, uint64_t* bar,
                                                 uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// A 3-D tiled load (x innermost): with the map {64 columns, K rows, column blocks of 64} of a row-major matrix, one
// load brings several 64-column boxes, each 8 KB, one after the other -- the layout of as many 2-D boxes.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar,
                                                 uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Orders this thread's generic-proxy view of global memory before its later async-proxy operations (TMA, bulk copies):
// after an acquire that made other threads' ordinary stores visible to this thread, a bulk copy it issues next reads
// those stores, not older data.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Programmatic dependent launch.  griddep_launch: this block no longer holds back the grid launched after it on the
// stream with programmatic serialisation (once every block of this grid has said so or exited, that grid's blocks may
// start on free SMs and do their setup).  griddep_wait: waits until every grid this one depends on has completed and
// its memory writes are visible; it returns at once when the launch had no programmatic dependency.
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// A contiguous copy of `bytes` (a multiple of 16) from global to this block's shared memory by the TMA engine,
// completing on `bar` (both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// ------------------------------------------------------------------ TMA stores (the epilogue's C tiles)
// A 2-D tiled store of one box from this block's shared memory (in the map's swizzle) to global memory; the map's
// bounds clip the box (rows or columns past the tensor are not written).  It joins the thread's open bulk-async group.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(tmap)),
                 "r"(x), "r"(y), "r"(smem_u32(src))
                 : "memory");
}
// Closes the thread's open bulk-async group.
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N of the thread's committed groups are still reading their shared-memory sources (the sources of
// the others may be overwritten).  A store's read of shared memory always completes; it depends on no other agent.
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N of the thread's committed groups are incomplete (their writes to global memory done).
template <int N>
__device__ __forceinline__ void bulk_wait()
{
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Makes this thread's ordinary writes to shared memory visible to the async proxy (a TMA store that reads them next).
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ clusters (the CTA pair of cta_group::2)
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of the same shared variable in block `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}

// Every thread of every block of the cluster (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// One arrival on a barrier of another block of the cluster (a shared::cluster address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 16 bytes into another block's shared memory (`dst`, a shared::cluster address), counted as transaction bytes on
// that block's barrier `bar` (a shared::cluster address in the same block): the receiver waits on its barrier alone.
__device__ __forceinline__ void st_async_v4(uint32_t dst, uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t bar)
{
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(dst),
                 "r"(a), "r"(b), "r"(c), "r"(d), "r"(bar)
                 : "memory");
}

// Orders this thread's accesses after an acquire at cluster scope (after a wait on a barrier another block arrived on).
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }

// A 2-D tiled load into this block's shared memory whose bytes complete on a barrier of either block of the pair
// (`bar`: a shared::cluster address) -- each block of the pair loads its own halves, the leader's barrier counts both.
// No multicast: each block reads only what it holds.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, int x, int y, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// The 3-D form (several 64-column boxes in one load), completing on the leader's barrier.  No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const void* tmap, int x, int y, int z, uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
        "%4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}

// The same with an L2 cache policy.
__device__ __forceinline__ void tma_load_2d_pair_hint(void* dst, const void* tmap, int x, int y, uint32_t bar,
                                                      uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], "
        "[%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}

// ------------------------------------------------------------------ tcgen05: tensor memory
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// The pair forms: one warp of each block of the pair executes them; the columns are the same in both blocks.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] x B[smem desc], kind::f16 (fp16 inputs, fp32 accumulators); accumulate = 0 overwrites.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The pair's MMA, issued by the leader block only: A = 128 rows from each block's shared memory (the same
// descriptor address in both), B = N / 2 columns from each, D = each block's 128 TMEM lanes x N columns.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrives once on the barrier at shared::cluster address `bar` (this block's or the other block's of the pair) when
// every tcgen05 operation the leader has issued so far has completed.  The pair's barriers in both blocks are reached
// by one such commit each (no multicast form is used anywhere in this library).
__device__ __forceinline__ void mma_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Arrives once on `bar` when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 16 columns of 32 bits: thread t of the warp gets lane (taddr.lane + t), columns taddr.col .. +15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ descriptors
// Shared-memory matrix descriptor (sm_100 layout): start >> 4 in bits [0,14), leading byte offset >> 4 in [16,30),
// stride byte offset >> 4 in [32,46), version 1 in [46,48), base offset 0, swizzle mode in [61,64) (2 = 128-byte).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, kind::f16: fp32 accumulators (bits [4,6) = 1), fp16 A and B (formats 0), A major in bit 15
// and B major in bit 16 (0: K-major, 1: MN-major), N >> 3 in bits [17,23), M >> 4 in bits [24,29).
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool a_mn_major, bool b_mn_major)
{
    return (1u << 4) | ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

// ------------------------------------------------------------------ global memory ordering
__device__ __forceinline__ int ld_acquire_gpu(const int* p)
{
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ------------------------------------------------------------------ system scope: flags in another GPU's memory
// (reached through a CUDA IPC mapping over NVLink) or in this GPU's memory written by another GPU
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Orders this thread's earlier stores (to any GPU's memory) before its later ones, at system scope.
__device__ __forceinline__ void fence_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Spins until the flag at p reaches `want` (epochs count up from 1; compared modulo 2^32), the block's abort flag
// rises, or `limit_ns` pass; a timeout is recorded like wait_slow's.  One thread calls it.
__device__ __noinline__ bool wait_flag(const unsigned* p, unsigned want, volatile int* abort_flag, uint64_t limit_ns,
                                       uint32_t where, int seg)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if ((int)(ld_acquire_sys(p) - want) >= 0) return true;
        if ((i & 15u) == 0) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > limit_ns) {
                record_timeout(abort_flag, where, seg);
                return false;
            }
            __nanosleep(256);
        }
    }
}

// ------------------------------------------------------------------ named barriers
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t count)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

}  // namespace bw

#endif  // BW_EMULATE
