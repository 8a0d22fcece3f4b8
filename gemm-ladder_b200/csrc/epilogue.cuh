// epilogue.cuh -- the epilogue helpers of the rung's kernel (gemm_kernel.cuh): stores of C from the accumulator
// (whole lines after an in-warp transpose, or through the swap-AB transpose buffers), the reductions of tiles split over
// several blocks, and the fused reduce-scatter's per-tile exchange between GPUs.
#pragma once
#include "kernel_common.cuh"

namespace bw {

// ------------------------------------------------------------------ the epilogue's stores
// 16 accumulator columns of TMEM lane `lane` (v) -> C, by all 128 epilogue threads together.
// Not swapped: C[m0 + lane][n0 + c0 .. +15], two 16-byte stores per thread.
// Swapped: the values are column n0 + lane of rows c0 .. c0 + 15 of C.  They go through shared memory (cst: two
// 16 x 128 fp16 buffers, alternating by chunk), so that C is written by 16-byte stores, a warp covering two rows of
// 256 contiguous bytes, instead of 16 scattered 2-byte stores per thread.  One named barrier per chunk; the buffer of
// chunk i + 2 is written only after every thread has passed the barrier of chunk i + 1, so after it read chunk i.
template <bool SWAP, int EPI = kEpiF16, int BT = 0>
__device__ __forceinline__ void store_chunk(const Params& p, int m0, int n0, int lane, int c0, const float (&v)[16],
                                            __half* cst)
{
    const Sched& s = p.s;
    if (EPI == kEpiF32) {  // fp32 C (not swapped): four 16-byte stores
        const int m = m0 + lane, n = n0 + c0;
        if (m >= s.M || n >= s.N) return;
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.C) + (size_t)m * s.N + n);
#pragma unroll
        for (int q = 0; q < 4; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        return;
    }
    if (!SWAP) {
        const int m = m0 + lane, n = n0 + c0;
        if (m >= s.M || n >= s.N) return;
        uint32_t h[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const __half2 x = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            h[j] = *reinterpret_cast<const uint32_t*>(&x);
        }
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(p.C) + (size_t)m * s.N + n);
        dst[0] = make_uint4(h[0], h[1], h[2], h[3]);
        dst[1] = make_uint4(h[4], h[5], h[6], h[7]);
    } else {
        __half* buf = cst + ((c0 >> 4) & 1) * (16 * 128);
#pragma unroll
        for (int j = 0; j < 16; ++j) buf[j * 128 + lane] = __float2half_rn(v[j]);
        named_bar_sync(1, 128);
        const int t = threadIdx.x - kEpiThread0;
        // accumulator column c0: token c0 % BT of weight block c0 / BT (BT tokens per block; 0: one block)
        const int wb = BT ? c0 / BT : 0, tok = c0 - wb * BT;
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int piece = t + 128 * k;  // 256 pieces of 8 fp16: 16 rows x 16 pieces
            const int mm = piece >> 4, nn = (piece & 15) * 8;
            const int m = tok + mm, n = n0 + wb * 128 + nn;
            if (m < s.M && n < s.N)
                *reinterpret_cast<uint4*>(static_cast<__half*>(p.C) + (size_t)m * s.N + n) =
                    *reinterpret_cast<const uint4*>(buf + mm * 128 + nn);
        }
    }
}

// 64 columns of C from the 32 rows of one epilogue warp (TILE and PAIR; lane l holds row r0 + l, as the accumulator's
// TMEM lanes give it), stored as whole lines.  A thread writing its own row would touch 32 rows per warp store, half a
// sector each (measured: 16 GB/s per SM for a 128 x 256 fp16 tile); instead the 16-byte pieces are transposed within
// groups of P lanes (P = pieces per row of 64 columns: 8 in fp16, 16 in fp32) by log2(P) rounds of shfl_xor, after
// which lane q of a group holds piece q of the group's P rows, and each store writes 32 / P rows of 128 (256) bytes
// (measured: 53 GB/s per SM).
template <int P>
__device__ __forceinline__ void transpose_pieces(uint32_t (&x)[P][4], int lane)
{
    const int q = lane & (P - 1);
#pragma unroll
    for (int m = P / 2; m >= 1; m >>= 1) {
        const bool hi = (q & m) != 0;
#pragma unroll
        for (int e = 0; e < P; ++e) {
            if (e & m) continue;
#pragma unroll
            for (int w = 0; w < 4; ++w) {  // the lower lane keeps piece e and takes e | m; the upper the other way
                const uint32_t send = hi ? x[e][w] : x[e | m][w];
                const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, m);
                if (hi)
                    x[e][w] = recv;
                else
                    x[e | m][w] = recv;
            }
        }
    }
}

template <int EPI>
__device__ __forceinline__ void store_rows64(const Params& p, int r0, int n, int lane, const float (&v)[64])
{
    static_assert(EPI == kEpiF16 || EPI == kEpiF32, "fp16 or fp32 C");
    constexpr int P = EPI == kEpiF32 ? 16 : 8;
    const Sched& s = p.s;
    uint32_t x[P][4];
#pragma unroll
    for (int i = 0; i < P; ++i)
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            if (EPI == kEpiF32) {
                x[i][w] = __float_as_uint(v[4 * i + w]);
            } else {
                const __half2 h = __floats2half2_rn(v[8 * i + 2 * w], v[8 * i + 2 * w + 1]);
                x[i][w] = *reinterpret_cast<const uint32_t*>(&h);
            }
        }
    transpose_pieces<P>(x, lane);
    const int q = lane & (P - 1), g = lane / P;
    if (n >= s.N) return;  // N % 64 == 0: the 64 columns are all in C or all outside
#pragma unroll
    for (int e = 0; e < P; ++e) {
        const int m = r0 + g * P + e;
        if (m < s.M) {
            uint4* dst = EPI == kEpiF32
                             ? reinterpret_cast<uint4*>(static_cast<float*>(p.C) + (size_t)m * s.N + n) + q
                             : reinterpret_cast<uint4*>(static_cast<__half*>(p.C) + (size_t)m * s.N + n) + q;
            *dst = make_uint4(x[e][0], x[e][1], x[e][2], x[e][3]);
        }
    }
}

// The same 64 columns of C from one warp's 32 rows by a TMA store (TILE and PAIR, fp16, BW_EPI_TMA): the warp writes
// its rows into `quarter`, its 4 KB of a staging buffer (128-byte rows; the 16-byte pieces of row l at piece
// j ^ (l % 8), the map's 128-byte swizzle, so that the 8 rows a quarter-warp writes at once fall in distinct banks),
// makes them visible to the async proxy, and lane 0 stores the box of 64 columns x 32 rows at (n, r0) -- the map
// clips the rows past M.  The buffer was last read by this warp's store of two chunks before: lane 0 first waits until
// at most one of its stores (the previous chunk's, from the other buffer) is still reading shared memory.
__device__ __forceinline__ void store_rows64_tma(const CUtensorMap* tmc, uint8_t* quarter, int r0, int n, int M,
                                                 int N, int lane, const float (&v)[64])
{
    if (n >= N || r0 >= M) return;  // the whole box outside C (warp-uniform): nothing to store
    if (lane == 0) bulk_wait_read<1>();
    __syncwarp();
    uint4* row = reinterpret_cast<uint4*>(quarter + lane * 128);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint32_t h[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const __half2 x = __floats2half2_rn(v[8 * j + 2 * w], v[8 * j + 2 * w + 1]);
            h[w] = *reinterpret_cast<const uint32_t*>(&x);
        }
        row[j ^ (lane & 7)] = make_uint4(h[0], h[1], h[2], h[3]);
    }
    fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(tmc, quarter, n, r0);
        bulk_commit();
    }
}

// ------------------------------------------------------------------ the partials of a split tile
// Slot layout: 128 rows x BN columns of fp32, interleaved by groups of 4 columns: [col / 4][row][col % 4].  TMEM lane
// `row`'s 4-column group is one 16-byte vector, and the 32 lanes of a warp touch 512 contiguous bytes per vector
// access (stores of a partial and loads of the reduction alike).  A block of a pair keeps its half in slot
// 2 s + rank.
template <int BN>
__device__ __forceinline__ float4* slot_vec(const Params& p, long long slot, int row, int col4)
{
    return reinterpret_cast<float4*>(p.work + (size_t)slot * 128 * BN) + (size_t)col4 * 128 + row;
}

// The last block of a split tile: for its row of the tile, sums the tile's nseg partials in their fixed order
// (p_0 + p_1 + ... : the same bits whichever block is last) and stores the result to C.  Partial f.mine comes from
// this block's accumulator in tensor memory when own_mine (tbase: its row's TMEM address), from its slot otherwise.
// The loads from memory are a stream of (16-column chunk, partial) pairs in chunk order, kept kWin deep in flight:
// with one partial in memory four chunks are on their way at once, instead of one L2 round trip per chunk.
template <int BN, bool SWAP, int RANKS, int EPI, int BT = 0>
__device__ __noinline__ void reduce_tile(const Params& p, int P, int tile, int rank, Fixup f, bool own_mine,
                                            uint32_t tbase, int row, int m0, int n0, __half* cst)
{
    constexpr int kWin = 4;
    constexpr int kChunks = BN / 16;
    const Sched& s = p.s;
    const int L = f.nseg - (own_mine ? 1 : 0);  // partials read from memory
    const int total = kChunks * L;
    // the memory partial j (in order) is partial index i: j, or j + 1 past this block's own
    auto index_of = [&](int j) { return (own_mine && j >= f.mine) ? j + 1 : j; };
    auto issue = [&](int idx, float4 (&w)[4]) {
        const int chunk = idx / L, j = idx - chunk * L;
        const long long slot = (long long)fixup_slot(s, P, tile, f, index_of(j)) * RANKS + rank;
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = __ldcg(slot_vec<BN>(p, slot, row, chunk * 4 + q));
    };
    float4 win[kWin][4];
#pragma unroll
    for (int q = 0; q < kWin; ++q)
        if (q < total) issue(q, win[q]);
    float v[16], own[16];
    bool own_added = false;
    for (int base = 0; base < total; base += kWin) {
#pragma unroll
        for (int q = 0; q < kWin; ++q) {
            const int idx = base + q;
            if (idx < total) {
                const int chunk = idx / L, j = idx - chunk * L;
                const int i = index_of(j);
                if (j == 0) {
                    own_added = false;
                    if (own_mine) {
                        uint32_t r[16];
                        tmem_ld16(tbase + (uint32_t)(chunk * 16), r);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 16; ++e) own[e] = __uint_as_float(r[e]);
                    }
                }
                // this block's own partial goes in at its place in the order
                if (own_mine && !own_added && f.mine < i) {
                    if (f.mine == 0) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) v[e] = own[e];
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e) v[e] += own[e];
                    }
                    own_added = true;
                }
                float x[16];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    x[4 * e] = win[q][e].x;
                    x[4 * e + 1] = win[q][e].y;
                    x[4 * e + 2] = win[q][e].z;
                    x[4 * e + 3] = win[q][e].w;
                }
                if (idx + kWin < total) issue(idx + kWin, win[q]);  // refill this window slot
                if (i == 0) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[e] = x[e];
                } else {
#pragma unroll
                    for (int e = 0; e < 16; ++e) v[e] += x[e];
                }
                if (j == L - 1) {  // the chunk is complete
                    if (own_mine && !own_added) {
#pragma unroll
                        for (int e = 0; e < 16; ++e) v[e] += own[e];
                    }
                    store_chunk<SWAP, EPI, BT>(p, m0, n0, row, chunk * 16, v, cst);
                }
            }
        }
    }
}

// The same at a block's last segment, when its stage ring is idle (every load consumed, none to come): the partials
// in memory are copied into the ring by the TMA engine at once (cp.async.bulk, one per partial), then summed from
// shared memory.  The sum runs over at most kMaxSum partials, unrolled and predicated, so that everything stays in
// registers.  Returns false if the copy did not complete within the wait limit (the block's abort flag is up).
template <int BN, bool SWAP, int RANKS, int kMaxSum, int EPI, int BT = 0>
__device__ __noinline__ bool reduce_tile_bulk(const Params& p, int P, int tile, int rank, Fixup f, bool own_mine,
                                              uint32_t tbase, int row, int m0, int n0, __half* cst, uint8_t* ring,
                                              uint64_t* rbar, volatile int* abort_flag, int seg)
{
    constexpr int kSlotBytes = 128 * BN * 4;
    constexpr int kChunks = BN / 16;
    const Sched& s = p.s;
    const int L = f.nseg - (own_mine ? 1 : 0);
    if (threadIdx.x == kEpiThread0) {
        // the other blocks' partials were written by ordinary stores, made visible to this thread by its acquire of
        // the tile's counter; the bulk copies below read through the async proxy, so order them after that view
        fence_proxy_async_global();
        mbar_arrive_expect_tx(rbar, (uint32_t)(L * kSlotBytes));
        for (int j = 0; j < L; ++j) {
            const int i = (own_mine && j >= f.mine) ? j + 1 : j;
            const long long slot = (long long)fixup_slot(s, P, tile, f, i) * RANKS + rank;
            const uint8_t* src = reinterpret_cast<const uint8_t*>(p.work + (size_t)slot * 128 * BN);
            for (int off = 0; off < kSlotBytes; off += 32768) {
                const int n = kSlotBytes - off < 32768 ? kSlotBytes - off : 32768;
                bulk_load(ring + (size_t)j * kSlotBytes + off, src + off, (uint32_t)n, rbar);
            }
        }
    }
    if (!wait_bounded(rbar, 0, abort_flag, p.wait_ns, site(2, 4, 0), seg)) return false;
    if (threadIdx.x == kEpiThread0) BW_TRACE_AT(10);
    // [col / 4][row][4] within a slot: consecutive rows are consecutive 16-byte vectors
    const float4* base = reinterpret_cast<const float4*>(ring) + row;
    // the sum of 16 columns (chunk) of this row, in summation order
    auto sum_chunk = [&](int chunk, float4 (&acc)[4]) {
        float4 own[4];
        if (own_mine) {
            uint32_t r[16];
            tmem_ld16(tbase + (uint32_t)(chunk * 16), r);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 4; ++q)
                own[q] = make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                     __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3]));
        }
#pragma unroll
        for (int i = 0; i < kMaxSum; ++i) {
            if (i < f.nseg) {
                float4 w[4];
                if (own_mine && i == f.mine) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) w[q] = own[q];
                } else {
                    const int j = (own_mine && i > f.mine) ? i - 1 : i;  // its place in the ring
                    const float4* src = base + (size_t)j * (kSlotBytes / 16) + (size_t)chunk * 4 * 128;
#pragma unroll
                    for (int q = 0; q < 4; ++q) w[q] = src[q * 128];
                }
                if (i == 0) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[q] = w[q];
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        acc[q].x += w[q].x;
                        acc[q].y += w[q].y;
                        acc[q].z += w[q].z;
                        acc[q].w += w[q].w;
                    }
                }
            }
        }
    };
    if constexpr (!SWAP && BN % 64 == 0 && BW_EPI_LINES && (EPI == kEpiF16 || EPI == kEpiF32)) {
        // 64 columns at a time, stored as whole lines of C (store_rows64)
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 64) {
            float v[64];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                float4 acc[4];
                sum_chunk(c0 / 16 + h, acc);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    v[16 * h + 4 * q] = acc[q].x;
                    v[16 * h + 4 * q + 1] = acc[q].y;
                    v[16 * h + 4 * q + 2] = acc[q].z;
                    v[16 * h + 4 * q + 3] = acc[q].w;
                }
            }
            store_rows64<EPI>(p, m0 + (row & ~31), n0 + c0, row & 31, v);
        }
    } else {
#pragma unroll 1
        for (int chunk = 0; chunk < kChunks; ++chunk) {
            float4 acc[4];
            sum_chunk(chunk, acc);
            float v[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                v[4 * q] = acc[q].x;
                v[4 * q + 1] = acc[q].y;
                v[4 * q + 2] = acc[q].z;
                v[4 * q + 3] = acc[q].w;
            }
            store_chunk<SWAP, EPI, BT>(p, m0, n0, row, chunk * 16, v, cst);
        }
    }
    if (threadIdx.x == kEpiThread0) BW_TRACE_AT(11);
    return true;
}

// ------------------------------------------------------------------ the fused reduce-scatter's epilogue
// One pair tile's half (this block's 128 rows x 256 columns, accumulator at tbase) under kEpiRS.  Not this rank's
// rows: the partial goes into the owner's slot by 16-byte stores (over NVLink), then the slot's flag takes the epoch
// (each thread's stores ordered before it by a system-scope fence).  The first time a block sends to an owner in a
// call it waits for the owner's ack of the previous call (the slot is free).  This rank's rows: the other ranks'
// flags for the tile, then, 64 columns at a time, the sum in rank order (this rank's own partial from tensor memory)
// rounded to fp16 into C, then a count; the block that consumes the call's last tile half acks the epoch.  The other
// ranks' partials reach the sum through the window (two 32 KB buffers of shared memory after the ring): each 64-column
// piece of a partial (32 KB, contiguous in the slot layout) is copied in by the TMA engine (cp.async.bulk, measured
// 90-98 GB/s per SM against ~35 for 16-byte loads) while the one before it is summed.  win_bar: the buffers' barriers;
// win_ph: the parity each waits for next (bit b); win_next: the buffer the next copy goes to.  Every wait is bounded;
// one thread waits and hands the outcome to the other 127 through `go` (two slots, alternating).  Returns false after
// a wait gave up.
__device__ __noinline__ bool rs_tile(const Params& p, unsigned epoch, int tm, int tn, int pr, uint32_t tbase, int row,
                                     int lane, int q, volatile int* abort_flag, volatile int* go, volatile int* go2,
                                     unsigned& acked, uint8_t* window, uint64_t* win_bar0, uint64_t* win_bar1,
                                     uint32_t& win_ph, int& win_next, int seg)
{
    const RsTable& rs = *p.rs;
    const Sched& s = p.s;
    const int o = tm * 256 / rs.rows;                        // the owner of the tile's rows
    const int tl = (tm - o * (rs.rows / 256)) * s.tiles_n + tn;  // the tile among the owner's
    if (o != rs.rank) {
        if (!(acked >> o & 1u)) {
            if (threadIdx.x == kEpiThread0)
                *go = wait_flag(rs.ack[o], epoch - 1u, abort_flag, p.rank_wait_ns, site(2, 8, (uint32_t)o), seg) ? 1 : 0;
            named_bar_sync(1, 128);
            const bool ok = *go != 0;
            named_bar_sync(1, 128);  // `go` is read by all before it is written again
            if (!ok) return false;
            acked |= 1u << o;
        }
        const int j = rs.rank < o ? rs.rank : rs.rank - 1;
        const size_t idx = ((size_t)tl * (rs.world - 1) + j) * 2 + pr;
        float4* slot = reinterpret_cast<float4*>(rs.slots[o] + idx * 128 * 256);
#pragma unroll 1
        for (int c0 = 0; c0 < 256; c0 += 16) {
            uint32_t r[16];
            tmem_ld16(tbase + (uint32_t)c0, r);
            tmem_wait_ld();
#pragma unroll
            for (int k = 0; k < 4; ++k)
                slot[(size_t)(c0 / 4 + k) * 128 + row] =
                    make_float4(__uint_as_float(r[4 * k]), __uint_as_float(r[4 * k + 1]), __uint_as_float(r[4 * k + 2]),
                                __uint_as_float(r[4 * k + 3]));
        }
        fence_sys();
        named_bar_sync(1, 128);
        if (threadIdx.x == kEpiThread0) st_release_sys(rs.flags[o] + idx, epoch);
        return true;
    }
    // this rank's rows: the others' partials of the tile
    if (threadIdx.x == kEpiThread0) {
        bool ok = true;
        for (int j = 0; j < rs.world - 1 && ok; ++j)
            ok = wait_flag(rs.flags[o] + ((size_t)tl * (rs.world - 1) + j) * 2 + pr, epoch, abort_flag,
                           p.rank_wait_ns, site(2, 7, (uint32_t)j), seg);
        // the peers' partials came by ordinary stores over NVLink, visible to this thread after its acquires of their
        // flags; this thread's bulk copies of them (fetch) go through the async proxy, so order them after that view
        if (ok) fence_proxy_async_global();
        *go = ok ? 1 : 0;
    }
    named_bar_sync(1, 128);
    const bool ok = *go != 0;
    named_bar_sync(1, 128);
    if (!ok) return false;
    const int m_local = tm * 256 + pr * 128 - o * rs.rows;  // the block's first row in this rank's C
    const int others = rs.world - 1;
    uint64_t* const wbar[2] = {win_bar0, win_bar1};
    // the 64-column piece c0 of the j-th other rank's partial (j in rank order), into buffer b of the window
    auto fetch = [&](int j, int c0, int b) {
        if (threadIdx.x == kEpiThread0) {
            const uint8_t* src = reinterpret_cast<const uint8_t*>(
                                     rs.slots[o] + (((size_t)tl * others + j) * 2 + pr) * 128 * 256) +
                                 (size_t)(c0 / 4) * 128 * 16;
            mbar_arrive_expect_tx(wbar[b], 32768u);
            bulk_load(window + b * 32768, src, 32768u, wbar[b]);
        }
    };
    int turn = 0;  // alternates the `go` slots
#pragma unroll 1
    for (int c0 = 0; c0 < 256; c0 += 64) {
        float v[64];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            uint32_t r[16];
            tmem_ld16(tbase + (uint32_t)(c0 + 16 * h), r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) v[16 * h + e] = __uint_as_float(r[e]);
        }
        // the sum in rank order: rank 0's partial first, this rank's (v) at its place
        float acc[64];
        bool own_in = false;
        fetch(0, c0, win_next);
#pragma unroll 1
        for (int j = 0; j < others; ++j) {
            const int b = win_next;
            const int src = j < rs.rank ? j : j + 1;
            if (j + 1 < others) fetch(j + 1, c0, b ^ 1);  // the other buffer was read by every thread before
            volatile int* slot = (turn++ & 1) ? go2 : go;
            if (threadIdx.x == kEpiThread0) {
                const bool okw = wait_bounded(wbar[b], (win_ph >> b) & 1u, abort_flag, p.wait_ns, site(2, 4, b), seg);
                if (!okw && j + 1 < others)  // the next piece is on its way: let it land before giving up
                    wait_drain(wbar[b ^ 1], (win_ph >> (b ^ 1)) & 1u, p.wait_ns);
                *slot = okw ? 1 : 0;
            }
            named_bar_sync(1, 128);
            if (!*slot) return false;
            mbar_try_wait(smem_u32(wbar[b]), (win_ph >> b) & 1u);  // complete: each thread acquires the bytes
            win_ph ^= 1u << b;
            win_next = b ^ 1;
            if (!own_in && rs.rank < src) {
#pragma unroll
                for (int e = 0; e < 64; ++e) acc[e] = rs.rank == 0 ? v[e] : acc[e] + v[e];
                own_in = true;
            }
            const float4* w4 = reinterpret_cast<const float4*>(window + b * 32768) + row;  // [col / 4][row][4]
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const float4 w = w4[k * 128];
                const float x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[4 * k + e] = src == 0 ? x[e] : acc[4 * k + e] + x[e];
            }
            named_bar_sync(1, 128);  // buffer b read by every thread: it may be refilled
        }
        if (!own_in) {  // this rank is the last
#pragma unroll
            for (int e = 0; e < 64; ++e) acc[e] = acc[e] + v[e];
        }
        store_rows64<kEpiF16>(p, m_local + q * 32, tn * 256 + c0, lane, acc);
    }
    named_bar_sync(1, 128);
    if (threadIdx.x == kEpiThread0) {
        // every rank's tile halves of this rank's rows: 2 per tile
        const unsigned total = 2u * (unsigned)((rs.rows / 256) * s.tiles_n);
        __threadfence();
        if (atomicAdd(rs.count, 1u) == total - 1u) {
            *rs.count = 0u;
            __threadfence();
            st_release_sys(rs.ack[rs.rank], epoch);
        }
    }
    return true;
}

}  // namespace bw
