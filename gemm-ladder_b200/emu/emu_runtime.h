// emu_runtime.h -- the host emulator's execution model for the rung's kernel (gemm_kernel.cuh compiled as host C++
// with -DBW_EMULATE; test infrastructure, never part of the library).
//
// A launch runs its clusters in concurrent batches (blocks of different clusters meet only through global memory:
// the split tiles' counters and partials, which the kernel orders with atomics and fences; none waits on another).
// The fused reduce-scatter runs every block of every emulated GPU at once.  Inside a cluster every thread
// of every block is a host thread, so the kernel's own barriers, mbarrier waits and warp-synchronous code run as they
// are written.  State per block: its shared memory, its tensor memory (128 lanes x 512 fp32 columns), its mbarriers,
// named barriers, warp barriers and shuffle slots.
//
// Findings: an access outside shared or tensor memory, an arrival on an uninitialised or already complete barrier, a
// TMA box that breaks the 128-byte swizzle's rules, an MMA shape the kernel does not use -- each is recorded
// (first one kept as text) and not carried out, so a wrong index shows as a finding, not as a crash.
#pragma once
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <random>
#include <thread>
#include <vector>

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

// ------------------------------------------------------------------ CUDA built-ins, per emulated thread
inline thread_local dim3 threadIdx, blockIdx, gridDim, blockDim;

namespace bw {
namespace emu {

constexpr int kCtaThreads = 192;
constexpr int kSmemBytes = 232448 + 1024;  // the kernel's dynamic shared memory limit and alignment slack
constexpr int kTmemLanes = 128, kTmemCols = 512;

// ------------------------------------------------------------------ findings
inline std::atomic<int> g_findings{0};
inline char g_first_finding[512] = "";
inline std::mutex g_finding_mu;

inline void finding(const char* fmt, ...)
{
    std::lock_guard<std::mutex> l(g_finding_mu);
    if (g_findings.fetch_add(1) == 0) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(g_first_finding, sizeof g_first_finding, fmt, ap);
        va_end(ap);
    }
}

// ------------------------------------------------------------------ knobs (bw_emu_set)
inline long long g_barrier_limit_ms = 120000;  // a thread barrier that never completes: a finding, then on
inline long long g_drop_tma = -1;              // the n-th TMA / bulk completion of a launch is dropped (-1: none)
inline std::atomic<long long> g_tma_count{0};

// ------------------------------------------------------------------ barriers between host threads
// A thread barrier the kernel's threads never all reach (a deadlock in the kernel's own control flow) ends with a
// finding after g_barrier_limit_ms instead of hanging the emulator.
struct Barrier {
    std::mutex m;
    std::condition_variable cv;
    int arrived = 0;
    unsigned gen = 0;
    void sync(int count)
    {
        std::unique_lock<std::mutex> l(m);
        const unsigned g = gen;
        if (++arrived >= count) {
            arrived = 0;
            ++gen;
            cv.notify_all();
        } else if (!cv.wait_for(l, std::chrono::milliseconds(g_barrier_limit_ms), [&] { return gen != g; })) {
            finding("a thread barrier of %d threads that %d reached (a deadlock in the kernel's control flow)", count,
                    arrived);
            arrived = 0;
            ++gen;
            cv.notify_all();
        }
    }
};

// a TMA or bulk completion that the drop_tma knob takes away (its bytes never arrive: a stall, made on purpose)
inline bool keep_completion() { return g_tma_count.fetch_add(1) != g_drop_tma; }
inline unsigned long long g_wait_ns = 60ull * 1000000000ull;  // the kernel's limit of one bounded wait
inline unsigned long long g_rank_wait_ns = 0;  // the limit of a wait for another rank's flag (0: g_wait_ns)

struct MBar {
    int count = 0, pending = 0;
    long long tx = 0;
    unsigned phase = 0;  // phases completed
};

struct Cluster;
struct Cta;

// The longest delay (microseconds) before an asynchronous unit carries out an item of work.
inline int g_engine_delay_us = 20;
// The longest random pause (microseconds) a thread takes before each tensor-memory load (0: none): an epilogue that
// reads its accumulator slowly, so that an MMA that does not wait for the accumulator to be released overwrites it.
inline int g_ld_delay_us = 0;
// The longest random delay (microseconds) before a block's threads start the kernel (0: none; each block its own),
// so that a block whose cluster peer has not yet set up its barriers or tensor memory meets them unset.
inline int g_start_jitter_us = 0;
inline int g_lead_skew_us = 0;  // the first block of every cluster starts this much later than the others
inline int g_block_ramp_us = 0;  // block b starts b times this much later than block 0

// One of a block's asynchronous units (its TMA engine, or its tensor core): work issued to it runs later, in issue
// order, on a host thread of its own, each item after a random delay of up to g_engine_delay_us -- so the kernel sees
// its copies land and its MMAs finish only when their barriers say so, as on the GPU, and a read that does not wait
// for them finds stale data.
struct Engine {
    Cta* owner = nullptr;
    std::mutex m;
    std::condition_variable cv;
    std::deque<std::function<void()>> q;
    bool stop = false;
    std::thread th;
    std::atomic<int> mmas{0};  // the tensor core: MMAs issued and not yet carried out
    void start(Cta* c);
    void post(std::function<void()> f)
    {
        {
            std::lock_guard<std::mutex> l(m);
            q.push_back(std::move(f));
        }
        cv.notify_one();
    }
    void finish()  // carries out what is queued, then ends
    {
        {
            std::lock_guard<std::mutex> l(m);
            stop = true;
        }
        cv.notify_one();
        if (th.joinable()) th.join();
    }
};

struct Cta {
    std::unique_ptr<uint8_t[]> raw;
    uint8_t* smem = nullptr;  // 1024-byte aligned
    std::vector<uint32_t> tmem;
    int rank = 0;
    Cluster* cluster = nullptr;
    std::map<uint32_t, MBar> mbars;
    Barrier named[16];
    Barrier warp[kCtaThreads / 32];
    uint32_t shfl[kCtaThreads / 32][32];
    int tmem_cols = 0;  // allocated columns (0: none)
    Engine tma, tc;     // the TMA engine (tiled loads, bulk copies) and the tensor core (MMAs, their commits)
    Cta() : raw(new uint8_t[kSmemBytes + 1024]), tmem((size_t)kTmemLanes * kTmemCols, 0u)
    {
        smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw.get()) + 1023) & ~uintptr_t(1023));
        std::memset(smem, 0xA5, kSmemBytes);  // not zero: a read of shared memory nothing wrote shows in the result
        tma.start(this);
        tc.start(this);
    }
    ~Cta()
    {
        tma.finish();
        tc.finish();
    }
};

constexpr int kMaxCluster = 8;  // the portable cluster limit

struct Cluster {
    int size = 1;
    Cta* cta[kMaxCluster] = {};
    Barrier all;
};

// The shared memory a launch's layout may use: its dynamic size less the 1024 bytes of slack the kernel keeps for
// aligning its base (on the GPU the slack is spent on alignment; here the base is aligned already).
inline int g_smem_limit = kSmemBytes;

inline thread_local Cta* t_cta = nullptr;
inline thread_local int t_tid = 0;
inline std::mutex g_mb;  // every mbarrier operation

inline void Engine::start(Cta* c)
{
    owner = c;
    th = std::thread([this] {
        t_cta = owner;  // the work runs as its block's
        std::minstd_rand rng((unsigned)reinterpret_cast<uintptr_t>(this));
        for (;;) {
            std::function<void()> f;
            {
                std::unique_lock<std::mutex> l(m);
                cv.wait(l, [&] { return stop || !q.empty(); });
                if (q.empty()) return;
                f = std::move(q.front());
                q.pop_front();
            }
            const int d = g_engine_delay_us > 0 ? (int)(rng() % (unsigned)(g_engine_delay_us + 1)) : 0;
            if (d > 0) std::this_thread::sleep_for(std::chrono::microseconds(d));
            f();
        }
    });
}

// A block's start delay under g_start_jitter_us: the same for every thread of the block, drawn from the block's index
// and the launch's sequence number (so the blocks of a cluster start in another order on each launch): none for about
// half the blocks, up to g_start_jitter_us for the others; plus a few microseconds per thread.
inline std::atomic<unsigned> g_launch_seq{0};
inline void start_jitter(unsigned block, unsigned seq)
{
    if (g_start_jitter_us <= 0) return;
    std::minstd_rand rng((block + 1u) * 2654435761u ^ (seq * 40503u + 1u));
    rng.discard(3);
    const unsigned r = rng();
    const unsigned d = ((r >> 7) & 1u ? r % (unsigned)(g_start_jitter_us + 1) : 0u) + (unsigned)(t_tid % 8);
    std::this_thread::sleep_for(std::chrono::microseconds(d));
}

inline uint64_t now_ns()
{
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

inline uint8_t* cta_smem() { return t_cta->smem; }

// ------------------------------------------------------------------ shared-memory addresses
// A shared::cta address is the offset in the block's shared memory; a shared::cluster address (mapa) carries the
// block's rank + 1 in its top byte.
inline uint32_t offset_of(const void* p)
{
    const std::ptrdiff_t o = static_cast<const uint8_t*>(p) - t_cta->smem;
    if (o < 0 || o >= g_smem_limit) {
        finding("a shared-memory address outside the launch's shared memory (offset %td)", o);
        return 0;
    }
    return (uint32_t)o;
}
inline uint32_t off_of(uint32_t a) { return a & 0xFFFFFFu; }
inline Cta* cta_of(uint32_t a)
{
    const unsigned r = a >> 24;
    if (r == 0) return t_cta;
    if (!t_cta->cluster || (int)r > t_cta->cluster->size) {
        finding("a shared::cluster address of rank %u outside the cluster", r - 1);
        return t_cta;
    }
    return t_cta->cluster->cta[r - 1];
}
inline uint32_t mapa(uint32_t a, uint32_t rank)
{
    if (!t_cta->cluster || (int)rank >= t_cta->cluster->size) finding("mapa to rank %u outside the cluster", rank);
    return off_of(a) | ((rank + 1u) << 24);
}

// ------------------------------------------------------------------ mbarrier
constexpr long long kTxLimit = (1 << 20) - 1;  // an mbarrier's pending transaction bytes, either way

// A copy into [off, off + bytes) of block c's shared memory that would overwrite one of its mbarriers.
inline bool over_mbar(Cta* c, uint32_t off, uint32_t bytes)
{
    std::lock_guard<std::mutex> l(g_mb);
    auto it = c->mbars.lower_bound(off >= 7 ? off - 7 : 0);
    return it != c->mbars.end() && it->first < off + bytes;
}

inline void mb_settle(MBar& b)
{
    if (b.pending == 0 && b.tx == 0) {
        ++b.phase;
        b.pending = b.count;
    }
}
inline void mb_init(Cta* c, uint32_t off, int count)
{
    std::lock_guard<std::mutex> l(g_mb);
    MBar b;
    b.count = b.pending = count;
    c->mbars[off] = b;
}
inline MBar* mb_find(Cta* c, uint32_t off, const char* what)
{
    auto it = c->mbars.find(off);
    if (it == c->mbars.end()) {
        finding("%s on an mbarrier never initialised (block rank %d, offset %u)", what, c->rank, off);
        return nullptr;
    }
    return &it->second;
}
inline void mb_arrive(Cta* c, uint32_t off, long long tx_add)
{
    std::lock_guard<std::mutex> l(g_mb);
    MBar* b = mb_find(c, off, "an arrival");
    if (!b) return;
    if (b->pending <= 0) {
        finding("an arrival beyond an mbarrier's count (offset %u)", off);
        return;
    }
    b->tx += tx_add;
    if (b->tx > kTxLimit || b->tx < -kTxLimit) finding("an mbarrier transaction count of %lld bytes", b->tx);
    --b->pending;
    mb_settle(*b);
}
inline void mb_complete_tx(Cta* c, uint32_t off, long long bytes)
{
    std::lock_guard<std::mutex> l(g_mb);
    MBar* b = mb_find(c, off, "transaction bytes");
    if (!b) return;
    b->tx -= bytes;
    if (b->tx > kTxLimit || b->tx < -kTxLimit) finding("an mbarrier transaction count of %lld bytes", b->tx);
    mb_settle(*b);
}
inline bool mb_try_wait(Cta* c, uint32_t off, uint32_t parity)
{
    std::lock_guard<std::mutex> l(g_mb);
    MBar* b = mb_find(c, off, "a wait");
    if (!b) return true;
    return (b->phase & 1u) != (parity & 1u);
}

// ------------------------------------------------------------------ thread barriers, shuffles
inline void named_sync(int id, int count)
{
    if (id < 0 || id >= 16 || count <= 0 || count % 32 || count > kCtaThreads) {  // bar.sync: whole warps, ids 0..15
        finding("named barrier %d of %d threads", id, count);
        return;
    }
    t_cta->named[id].sync(count);
}
inline void cluster_sync()
{
    Cluster* cl = t_cta->cluster;
    if (!cl) {
        t_cta->named[0].sync(kCtaThreads);
        return;
    }
    cl->all.sync(kCtaThreads * cl->size);
}

// ------------------------------------------------------------------ the tensor map (the 128-byte CUtensorMap, reused)
struct Map {
    const uint8_t* base;
    int rank;
    uint64_t dims[3];
    uint64_t strides[3];  // bytes per step of each dimension (strides[0] = the element size, 2)
    uint32_t box[3];
};
static_assert(sizeof(Map) <= sizeof(CUtensorMap), "the emulated map fits the opaque one");

inline void make_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                     const uint32_t* box)
{
    std::memset(m, 0, sizeof *m);
    // what cuTensorMapEncodeTiled refuses (the library's maps are encoded by the driver, which checks these): a base
    // not on 16 bytes, row strides not multiples of 16 bytes, boxes outside 1 .. 256, or (128-byte swizzle) an inner
    // box wider than 128 bytes
    if (reinterpret_cast<uintptr_t>(base) % 16) finding("a tensor map whose base is not on 16 bytes");
    for (int i = 0; i < rank; ++i) {
        if (box[i] < 1 || box[i] > 256) finding("a tensor map box of %u in dimension %d", box[i], i);
        if (i > 0 && strides[i] % 16) finding("a tensor map stride of %llu bytes", (unsigned long long)strides[i]);
    }
    if (box[0] * 2 > 128) finding("a 128-byte-swizzled tensor map box %u elements wide", box[0]);
    Map e;
    e.base = static_cast<const uint8_t*>(base);
    e.rank = rank;
    for (int i = 0; i < 3; ++i) {
        e.dims[i] = i < rank ? dims[i] : 1;
        e.strides[i] = i < rank ? strides[i] : 0;
        e.box[i] = i < rank ? box[i] : 1;
    }
    std::memcpy(m, &e, sizeof e);
}

// the 128-byte swizzle: 16-byte chunk c of 128-byte row r (within each 1024-byte atom) sits at chunk c ^ (r % 8)
inline uint32_t swizzle128(uint32_t off) { return off ^ (((off >> 7) & 7u) << 4); }

inline long long tma_copy(void* dst, const void* tmap, int x, int y, int z)
{
    Map m;
    std::memcpy(&m, tmap, sizeof m);
    Cta* c = t_cta;
    const uint32_t base = offset_of(dst);
    if (m.box[0] * 2 != 128) finding("a TMA box whose inner extent is %u bytes (128-byte swizzle needs 128)", m.box[0] * 2);
    if (((long long)x * 2) % 16) finding("a TMA load at x = %d, not on a 16-byte boundary", x);
    if (base % 1024) finding("a TMA destination not on a 1024-byte swizzle atom (offset %u)", base);
    const long long bytes = (long long)m.box[0] * m.box[1] * m.box[2] * 2;
    if (base + bytes > (long long)g_smem_limit || over_mbar(c, base, (uint32_t)bytes)) {
        finding("a TMA load past the launch's shared memory or over an mbarrier (offset %u, %lld bytes)", base, bytes);
        return bytes;
    }
    for (uint32_t zz = 0; zz < m.box[2]; ++zz)
        for (uint32_t rr = 0; rr < m.box[1]; ++rr)
            for (uint32_t cc = 0; cc < m.box[0]; ++cc) {
                const long long gx = (long long)x + cc, gy = (long long)y + rr, gz = (long long)z + zz;
                uint16_t v = 0;
                if (gx >= 0 && gy >= 0 && gz >= 0 && gx < (long long)m.dims[0] && gy < (long long)m.dims[1] &&
                    gz < (long long)m.dims[2])
                    std::memcpy(&v, m.base + gz * m.strides[2] + gy * m.strides[1] + gx * 2, 2);
                const uint32_t lin = base + ((zz * m.box[1] + rr) * m.box[0] + cc) * 2;
                const uint32_t off = swizzle128(lin);
                if (off + 2 > (uint32_t)kSmemBytes) {
                    finding("a TMA load past the end of shared memory");
                    return bytes;
                }
                std::memcpy(c->smem + off, &v, 2);
            }
    return bytes;
}

// TMA stores: each issued store is queued to the block's TMA engine, which later reads the box out of shared memory
// (through the 128-byte swizzle, as the map says) and writes the part of it inside the tensor to global memory -- so a
// kernel that overwrites a store's source before waiting for the store's read sends the new data, as on the GPU.  A
// thread's stores join its open group until it commits; a wait for the groups counts the committed ones still pending.
using StoreFlag = std::shared_ptr<std::atomic<bool>>;
inline thread_local std::vector<StoreFlag> t_open_stores;
inline thread_local std::deque<std::vector<StoreFlag>> t_store_groups;

inline void tma_store(const void* tmap, const void* src, int x, int y)
{
    Map m;
    std::memcpy(&m, tmap, sizeof m);
    Cta* c = t_cta;
    const uint32_t base = offset_of(src);
    if (m.rank != 2 || m.box[0] * 2 != 128) finding("a TMA store through a map that is not 2-D with 128-byte rows");
    if (((long long)x * 2) % 16 || x < 0 || y < 0) finding("a TMA store at (%d, %d): not on 16 bytes, or negative", x, y);
    if (base % 1024) finding("a TMA store source not on a 1024-byte swizzle atom (offset %u)", base);
    const uint32_t bytes = m.box[0] * m.box[1] * 2;
    if (base + bytes > (uint32_t)g_smem_limit || over_mbar(c, base, bytes)) {
        finding("a TMA store source past the launch's shared memory or over an mbarrier (offset %u)", base);
        return;
    }
    StoreFlag done = std::make_shared<std::atomic<bool>>(false);
    t_open_stores.push_back(done);
    c->tma.post([=] {
        uint8_t* g = const_cast<uint8_t*>(m.base);
        for (uint32_t rr = 0; rr < m.box[1]; ++rr)
            for (uint32_t cc = 0; cc < m.box[0]; ++cc) {
                const long long gx = (long long)x + cc, gy = (long long)y + rr;
                if (gx >= (long long)m.dims[0] || gy >= (long long)m.dims[1]) continue;  // clipped
                std::memcpy(g + gy * m.strides[1] + gx * 2, c->smem + swizzle128(base + (rr * m.box[0] + cc) * 2), 2);
            }
        done->store(true);
    });
}
inline void store_commit()
{
    t_store_groups.push_back(std::move(t_open_stores));
    t_open_stores.clear();
}
// Waits until at most n committed groups are pending (reads and writes alike: here a store is done when both are).
inline void store_wait(int n)
{
    while ((int)t_store_groups.size() > n) {
        for (const StoreFlag& f : t_store_groups.front())
            while (!f->load()) std::this_thread::sleep_for(std::chrono::microseconds(5));
        t_store_groups.pop_front();
    }
}

inline void bulk_copy(void* dst, const void* src, uint32_t bytes)
{
    const uint32_t off = offset_of(dst);
    if (off % 16 || bytes % 16 || reinterpret_cast<uintptr_t>(src) % 16)
        finding("a bulk copy not on 16-byte boundaries");
    if (off + bytes > (uint32_t)g_smem_limit || over_mbar(t_cta, off, bytes)) {
        finding("a bulk copy past the launch's shared memory or over an mbarrier");
        return;
    }
    std::memcpy(t_cta->smem + off, src, bytes);
}

inline void remote_store(uint32_t dst, const uint32_t* v, uint32_t bytes)
{
    Cta* c = cta_of(dst);
    const uint32_t off = off_of(dst);
    if (off + bytes > (uint32_t)g_smem_limit || off % bytes || over_mbar(c, off, bytes)) {
        finding("an st.async outside the destination block's shared memory, unaligned or over an mbarrier");
        return;
    }
    std::memcpy(c->smem + off, v, bytes);
}

// ------------------------------------------------------------------ tensor memory and the MMA
// A fresh allocation holds what earlier kernels left, not zeros: here a NaN in every column, so that an MMA chain
// that accumulates onto an accumulator it never cleared (accumulate set on its first MMA) shows in the result.
constexpr uint32_t kTmemStale = 0x7FC0DEADu;
inline void tmem_alloc(uint32_t* slot, uint32_t ncols)
{
    if (ncols < 32 || ncols > (uint32_t)kTmemCols || (ncols & (ncols - 1))) finding("tcgen05.alloc of %u columns", ncols);
    t_cta->tmem_cols = (int)ncols;
    std::fill(t_cta->tmem.begin(), t_cta->tmem.end(), kTmemStale);
    *slot = 0u;  // lane 0, column 0
}
inline void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    if (taddr != 0u || (int)ncols != t_cta->tmem_cols) finding("tcgen05.dealloc of %u columns at %#x", ncols, taddr);
    // the MMAs that write this block's tensor memory: its own, and its pair leader's (cta_group::2)
    const Cta* writers[2] = {t_cta, t_cta->cluster && t_cta->rank ? t_cta->cluster->cta[0] : t_cta};
    for (const Cta* w : writers)
        if (w->tc.mmas.load() > 0) finding("tensor memory freed while %d MMAs are still in flight", w->tc.mmas.load());
}

// operand element (row, k) of a K16 slice through a 128-byte-swizzled shared-memory descriptor
inline float operand(const Cta* c, uint64_t desc, bool mn_major, int row, int k)
{
    const uint32_t start = (uint32_t)(desc & 0x3FFFu) << 4;
    const uint32_t lbo = (uint32_t)((desc >> 16) & 0x3FFFu) << 4;
    const uint32_t sbo = (uint32_t)((desc >> 32) & 0x3FFFu) << 4;
    const uint32_t off = mn_major ? start + (uint32_t)(row >> 6) * lbo + (uint32_t)(k >> 3) * sbo + (uint32_t)(k & 7) * 128u +
                                        (uint32_t)(row & 63) * 2u
                                  : start + (uint32_t)(row >> 3) * sbo + (uint32_t)(row & 7) * 128u + (uint32_t)k * 2u;
    const uint32_t p = swizzle128(off);
    if (p + 2 > (uint32_t)kSmemBytes) {
        finding("an MMA operand read past the end of shared memory");
        return 0.f;
    }
    __half h;
    std::memcpy(&h, c->smem + p, 2);
    return __half2float(h);
}

// D (tensor memory at d) (+)= A B over one K16 slice; pair: a cluster of two blocks, A's rows and D's rows split by
// block rank (128 each), B's N columns split in halves, each block's half in its own shared memory.
inline void mma(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate, bool pair)
{
    for (uint64_t desc : {adesc, bdesc})
        if ((desc >> 61) != 2u || ((desc >> 46) & 3u) != 1u) finding("a descriptor that is not sm_100 128-byte swizzle");
    const bool a_mn = (idesc >> 15) & 1u, b_mn = (idesc >> 16) & 1u;
    const int N = (int)((idesc >> 17) & 0x3Fu) << 3, M = (int)((idesc >> 24) & 0x1Fu) << 4;
    if (((idesc >> 4) & 3u) != 1u) finding("an MMA whose accumulator is not fp32");
    const int ranks = pair ? 2 : 1;
    // cta_group::1 with M = 128: N in 16 .. 256 by 16; cta_group::2 (M = 256): N in 32 .. 256 by 32, half per block
    if (M != 128 * ranks || N < 16 * ranks || N > 256 || N % (16 * ranks)) {
        finding("an MMA of M %d N %d (cta_group::%d)", M, N, ranks);
        return;
    }
    Cta* cta[2] = {t_cta, t_cta};
    if (pair) {
        if (!t_cta->cluster || t_cta->cluster->size != 2) {
            finding("a cta_group::2 MMA outside a cluster of two");
            return;
        }
        cta[0] = t_cta->cluster->cta[0];
        cta[1] = t_cta->cluster->cta[1];
    }
    const uint32_t lane0 = d >> 16, col0 = d & 0xFFFFu;
    if (lane0 != 0 || col0 + (uint32_t)N > (uint32_t)kTmemCols) {
        finding("an MMA accumulator at lane %u column %u (N %d) outside tensor memory", lane0, col0, N);
        return;
    }
    // B: N rows of K16, the first N / ranks from block 0's shared memory, the rest from block 1's
    std::vector<float> b((size_t)N * 16);
    for (int n = 0; n < N; ++n) {
        const int r = n / (N / ranks), local = n % (N / ranks);
        for (int k = 0; k < 16; ++k) b[(size_t)n * 16 + k] = operand(cta[r], bdesc, b_mn, local, k);
    }
    std::vector<float> a(128 * 16);
    for (int r = 0; r < ranks; ++r) {
        for (int m = 0; m < 128; ++m)
            for (int k = 0; k < 16; ++k) a[(size_t)m * 16 + k] = operand(cta[r], adesc, a_mn, m, k);
        if (cta[r]->tmem_cols < (int)(col0 + N)) finding("an MMA into tensor memory not allocated");
        for (int m = 0; m < 128; ++m) {
            uint32_t* row = cta[r]->tmem.data() + (size_t)m * kTmemCols + col0;
            for (int n = 0; n < N; ++n) {
                float s = 0.f;
                for (int k = 0; k < 16; ++k) s += a[(size_t)m * 16 + k] * b[(size_t)n * 16 + k];
                float acc;
                std::memcpy(&acc, &row[n], 4);
                acc = accumulate ? acc + s : s;
                std::memcpy(&row[n], &acc, 4);
            }
        }
    }
}

// tcgen05.ld 32x32b.x16: lane = the address's lane + the thread's lane in its warp, 16 columns
inline void tmem_ld(uint32_t taddr, uint32_t (&r)[16])
{
    if (g_ld_delay_us > 0) {
        thread_local std::minstd_rand rng((unsigned)(t_tid * 7919 + 17));
        std::this_thread::sleep_for(std::chrono::microseconds(rng() % (unsigned)(g_ld_delay_us + 1)));
    }
    const uint32_t lane = (taddr >> 16) + (uint32_t)(t_tid & 31), col = taddr & 0xFFFFu;
    if (lane >= (uint32_t)kTmemLanes || col + 16 > (uint32_t)t_cta->tmem_cols) {
        finding("tcgen05.ld of lane %u column %u outside the allocation", lane, col);
        std::memset(r, 0, sizeof r);
        return;
    }
    if (((uint32_t)(t_tid >> 5) & 3u) != ((taddr >> 16) >> 5)) finding("a warp reading a TMEM lane quarter not its own");
    std::memcpy(r, t_cta->tmem.data() + (size_t)lane * kTmemCols + col, sizeof r);
}

}  // namespace emu
}  // namespace bw

// ------------------------------------------------------------------ the other CUDA built-ins the kernel calls
inline void __syncthreads() { bw::emu::named_sync(0, bw::emu::kCtaThreads); }
inline void __syncwarp(unsigned = 0xffffffffu) { bw::emu::t_cta->warp[bw::emu::t_tid >> 5].sync(32); }
inline uint32_t __shfl_xor_sync(unsigned, uint32_t v, int m)
{
    bw::emu::Cta* c = bw::emu::t_cta;
    const int w = bw::emu::t_tid >> 5, lane = bw::emu::t_tid & 31;
    c->shfl[w][lane] = v;
    c->warp[w].sync(32);
    const uint32_t r = c->shfl[w][lane ^ (m & 31)];
    c->warp[w].sync(32);
    return r;
}
inline void __threadfence() { std::atomic_thread_fence(std::memory_order_seq_cst); }
inline float4 __ldcg(const float4* p)
{
    std::atomic_thread_fence(std::memory_order_acquire);
    return *p;
}
inline void __stcg(float4* p, float4 v) { *p = v; }
inline float __expf(float x) { return std::exp(x); }
inline float __uint_as_float(uint32_t u)
{
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
inline uint32_t __float_as_uint(float f)
{
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
}
inline int atomicAdd(int* p, int v) { return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST); }
inline unsigned atomicAdd(unsigned* p, unsigned v) { return __atomic_fetch_add(p, v, __ATOMIC_SEQ_CST); }
inline int atomicExch(int* p, int v) { return __atomic_exchange_n(p, v, __ATOMIC_SEQ_CST); }
inline unsigned atomicCAS(unsigned* p, unsigned cmp, unsigned val)
{
    __atomic_compare_exchange_n(p, &cmp, val, false, __ATOMIC_SEQ_CST, __ATOMIC_SEQ_CST);
    return cmp;
}

// the two qualifiers the host compiler does not define (every system header is included above)
#ifndef __noinline__
#define __noinline__ __attribute__((noinline))
#endif
#ifndef __launch_bounds__
#define __launch_bounds__(...)
#endif
