/*
 * bwgemm.h -- the C ABI of the Blackwell (sm_100a) rung of gemm-ladder: C = A B, A (M x K) and B (K x N) fp16
 * row-major, fp32 accumulation, C (M x N) fp16 row-major.
 *
 * Plain pointers and sizes only: device pointers for A, B and C, a cudaStream_t passed as void*.  The library is
 * gemm-ladder_b200/lib/libbwgemm.so; gemm-ladder_b200/blackwell/candidate.cu wraps it in the reference's C++
 * candidate interface so the reference's judge, probe and verif drive it unchanged.
 *
 * Each entry names the reference interface it replaces (paths inside the reference project).
 */
#ifndef BWGEMM_H
#define BWGEMM_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference prints and aborts on an unsupported shape (hopper/step7.cu:358-361); the C ABI returns
 * a code instead and candidate.cu turns a non-zero code into that print-and-abort.  The reference's candidates also
 * want M % 16 == 0; this library serves any M >= 1 (the tokens of a decode step, M = 1 or 8, included: rows past M
 * are the TMA engine's zero fill inside the kernel, never padding in the caller's memory), and candidate.cu keeps the
 * reference's M % 16 rule for the reference's harnesses. */
#define BW_OK 0
#define BW_ERR_SHAPE 1     /* M, N, K not positive, or N % 64, K % 64 not 0 (any M >= 1 is served) */
#define BW_ERR_LAUNCH 2    /* a CUDA call failed (the CUDA error string: bw_last_error_string) */
#define BW_ERR_TIMEOUT 3   /* a kernel's bounded wait on a barrier gave up; see bw_gemm_status */
#define BW_ERR_ARG 4       /* null or misaligned pointer, unknown variant */
#define BW_ERR_DEVICE 5    /* the current device is not an sm_100 (B200-class) GPU */
#define BW_ERR_SCRATCH 6   /* bw_gemm_f16_noalloc: no plan's scratch fits its fixed array (whole tiles always do) */

/* Kernels of the rule (bw_plan.kernel). */
#define BW_KERNEL_TILE 0   /* 128 x bn tiles of C, A as the MMA's A operand */
#define BW_KERNEL_SWAP 1   /* M <= 128: C^T = B^T A^T, 128 columns of B as the MMA's A operand, bn = M rounded to 16 */
#define BW_KERNEL_PAIR 2   /* 256 x bn tiles on a pair of SMs (tcgen05 cta_group::2) */
#define BW_KERNEL_SWAP_PAIR 3 /* swap-AB on a pair of SMs: 128 (x wm) weight columns per SM, the tokens (bn 64 or 128)
                                split over the pair (built with BW_SWAP_PAIR 1 only) */

/*
 * C = A B on `stream` (a cudaStream_t, 0 for the legacy default stream), with the current device.
 * Replaces: void candidate_gemm(const half* A, const half* B, half* C, int M, int N, int K, cudaStream_t s)
 *   (declared judge/judge.cu:73, probe/probe.cu:38, hopper/verif.cu:35; defined by each step, e.g.
 *   hopper/step7.cu:355-374).
 * Same rules as the reference's candidate (judge/judge.cu:5-10): asynchronous (no synchronisation), no allocation
 * except at the first call of a larger shape (a workspace kept until exit), capturable in a CUDA graph, A and B not
 * modified.  A, B and C 16-byte aligned.  Not for concurrent calls from several host threads on one device.
 */
int bw_gemm_f16(const void* A, const void* B, void* C, int M, int N, int K, void* stream);

/*
 * The same with a variant of the rule, for ablations (0 = the rule itself).
 * Replaces: the weak `int g_var` read by candidate_gemm (probe/probe.cu:39, hopper/verif.cu:37, hopper/step7.cu:15).
 */
int bw_gemm_f16_variant(const void* A, const void* B, void* C, int M, int N, int K, void* stream, int variant);

/*
 * C = A B^T-stored: the same product with B given as N x K row-major (each row of B one output column's weights, the
 * layout of a linear layer's weight matrix; K-major, the tensor core's native operand form), A M x K and C M x N as
 * above, the same rule and plans.  Replaces nothing in the reference: its candidates take B as K x N only.
 */
int bw_gemm_f16_tn(const void* A, const void* B, void* C, int M, int N, int K, void* stream);

/*
 * C = A B with C written in fp32 (M x N row-major, 16-byte aligned), A and B fp16 as above: the partial sums of a
 * row-parallel layer, reduced across GPUs by a reduce-scatter before they are rounded (the tensor-parallel MLP block
 * of the B200 configs: down = H_r W2_r on each rank, then an NCCL reduce-scatter of the fp32 partials).  SM-pair tiles
 * at every M.  No reference counterpart: the reference's candidates write fp16 only.
 */
int bw_gemm_f16_f32out(const void* A, const void* B, void* C, int M, int N, int K, void* stream);

/*
 * A gated MLP's activation in one GEMM: with B (K x N, N a multiple of 256) laid out so that each group of 256
 * columns holds 128 gate columns then the 128 matching up columns, C (M x N/2 fp16) = silu(A B_gate) * (A B_up),
 * computed from the fp32 accumulators in the epilogue (the M x N gateup result is never written).  Whole SM-pair tiles.
 * No reference counterpart: the tensor-parallel MLP block of the B200 configs (gateup, then down).
 */
int bw_gemm_f16_swiglu(const void* A, const void* B, void* C, int M, int N, int K, void* stream);

/* The number of variants.  Replaces: the weak `int g_nvar` (probe/probe.cu:40, hopper/verif.cu:38,
 * hopper/step7.cu:16). */
int bw_gemm_variant_count(void);

/* A one-line description of variant v (NULL if v is out of range).  Replaces: the variant list in the header comment
 * of each step (hopper/step7.cu:1-11). */
const char* bw_gemm_variant_name(int v);

/*
 * Words of the rung's state across calls left non-zero (the stream-K tile counters), after the caller has
 * synchronised.  0 means the state is back as the call found it.
 * Replaces: the weak `int candidate_dirty()` (hopper/verif.cu:41, :216-222; ampere/step7.cu:277-292).
 */
int bw_gemm_dirty(void);

/*
 * C = A B like bw_gemm_f16, for callers that cannot allocate device memory: a serving process whose memory is all
 * handed out up front by its own allocator (a cudaMalloc there would take memory outside its budget, and the first one
 * can stall every stream of the device), or a plugin that runs inside someone else's process and may not call
 * cudaMalloc / cudaFree at all.  No reference counterpart: the reference's candidates allocate their workspace at the
 * first call of a shape.
 *
 * The scratch this call needs (the fp32 partials and counters of tiles split over several SMs) lives in one fixed
 * array of BW_NOALLOC_SCRATCH_BYTES + 4 * BW_NOALLOC_COUNTERS bytes, compiled into the library: every GPU that loads
 * the library holds it until the process exits.  The first call on a device looks up that array's device address
 * (once, with the device current); make that first call before any stream capture.  Calls never allocate or free.
 * The array holds the stream-K partials of any plan on a GPU of up to 160 SMs (two 256 x 256 fp32 slots per SM pair,
 * 37 MiB on a B200), so on a B200's 74 pairs every judge, ladder and decode shape takes the rule's own plan (on a
 * device that holds fewer pairs at once, down_m2048's split-K tail can take fewer splits).  A call whose plan needs
 * more than the array holds takes the first of these that fits: the narrower tiles (where the rule's are 256-column
 * swap tiles, 512-column pair tiles or swap-AB pairs), the same plan with its split-K tail cut to the splits the
 * array holds, whole tiles (no partials).  So no call is refused for scratch; BW_ERR_SCRATCH is kept for a plan that
 * somehow still does not fit.
 * Every call shares the one array and clears the counters it uses on its stream first: two calls that overlap on
 * the GPU (different streams, or several host threads) race on it; order them, or use bw_gemm_f16.
 */
#define BW_NOALLOC_SCRATCH_BYTES (40u << 20) /* fp32 partials: 40 MiB */
#define BW_NOALLOC_COUNTERS 4096u            /* split-tile counters */
int bw_gemm_f16_noalloc(const void* A, const void* B, void* C, int M, int N, int K, void* stream);

/*
 * The fused reduce-scatter of a row-parallel layer, on `world` GPUs of one node (2 to 8, one process each, the same
 * M and N everywhere): rank r holds A_r (M x K) and B_r (K x N) and receives C_r, rows [r M/world, (r+1) M/world) of
 * the sum over the ranks of A_r B_r, in fp16 (M/world x N row-major).  One kernel per rank computes its pair tiles;
 * a tile of another rank's rows goes as fp32 into that rank's memory over NVLink (its receive slots, reached through
 * CUDA IPC), and each rank sums the ranks' partials of its own tiles in rank order (bit-for-bit the same on every
 * run) as they arrive.  No NCCL call: it replaces the fp32-output GEMM + reduce-scatter collective of the tensor-
 * parallel MLP block (gemm-ladder_b200/tp_mlp.py).  No reference counterpart (the reference runs on one GPU).
 *
 *   bw_rs_create     this rank's context and receive region (M % (256 world) == 0), on the current device; the
 *                    region holds (world - 1) fp32 partials of this rank's rows (bw_rs_region_bytes)
 *   bw_rs_handle     the region's CUDA IPC handle (BW_RS_HANDLE_BYTES bytes), for the other ranks
 *   bw_rs_connect    opens the other ranks' regions from all ranks' handles (world x BW_RS_HANDLE_BYTES bytes, in
 *                    rank order); every rank connects before any rank calls bw_gemm_f16_rs
 *   bw_gemm_f16_rs   C_r as above, on `stream`; every rank makes the same calls in the same order.  A call waits
 *                    (bounded) for the other ranks' partials and, before reusing a rank's slots, for that rank to
 *                    have consumed the previous call's; a rank that never comes ends the others' calls with
 *                    BW_ERR_TIMEOUT in the status word (site kinds 7 and 8).  Capturable in a CUDA graph (each call
 *                    takes its number from the device, so every replay is a new call); every rank replays the same
 *                    calls.  After a BW_ERR_TIMEOUT destroy the contexts and create new ones.
 *   bw_rs_destroy    closes the peers' regions and frees this rank's
 */
#define BW_RS_HANDLE_BYTES 64
typedef struct bw_rs bw_rs;
int bw_rs_create(int M, int N, int world, int rank, bw_rs** out);
size_t bw_rs_region_bytes(const bw_rs* rs);
int bw_rs_handle(const bw_rs* rs, void* handle);
int bw_rs_connect(bw_rs* rs, const void* handles);
int bw_gemm_f16_rs(bw_rs* rs, const void* A, const void* B, void* C, int K, void* stream);
int bw_rs_destroy(bw_rs* rs);

/* The plan of one call: the kernel, its tile and its schedule (host only, no GPU needed). */
typedef struct bw_plan {
    int kernel;          /* BW_KERNEL_TILE or BW_KERNEL_SWAP */
    int bn;              /* MMA N: the tile's columns (TILE) or the tokens rounded up to 16 (SWAP) */
    int stages;          /* shared-memory stages of the TMA ring */
    int tiles_m, tiles_n, tiles;
    int kblocks;         /* K / 64 */
    int grid;            /* persistent blocks, one per SM at most */
    int dp_tiles;        /* tiles done whole, round-robin over the blocks */
    int sk_tiles;        /* the other tiles: split-K or stream-K */
    int splits;          /* > 0: each of them split into this many K ranges (split-K); 0: stream-K */
    long long sk_iters;  /* stream-K: their K-blocks, split evenly over the blocks */
    int group_rows;      /* rows of tiles per serpentine group (0: row after row) */
    size_t workspace_bytes; /* fp32 partials of the split tiles */
    int counters;        /* one counter per split tile */
    int smem_bytes;      /* dynamic shared memory per block */
    int tmem_cols;       /* tensor-memory columns per block */
    int ksplit;          /* > 0: SWAP with each tile's K cut in ksplit ranges on the blocks of a cluster of ksplit
                            (grid = ksplit x tiles); 0: none */
    int wm;              /* SWAP: 128-column weight blocks per tile (1 or 2; 2 = two MMAs on each stage of A) */
    int dyn;             /* 1: the split-K units (splits per tile, every tile split) go to whichever block asks next
                            (a counter in global memory), their partials summed in unit order; 0: a static order */
} bw_plan;

/*
 * The rule: which kernel, tile and schedule a call at M x N x K takes on a GPU of `sms` SMs (sms / 2 pairs of SMs
 * held at once), for variant `variant`.  On a device the library uses the pairs its occupancy query reports.
 * Replaces: step7::choose / step6::choose / rows7c (hopper/step7.cuh:921-949, hopper/step6.cuh:468-488).
 */
int bw_gemm_plan(int M, int N, int K, int sms, int variant, bw_plan* out);

/*
 * The plan a call on the current device takes: bw_gemm_f16_variant's with `variant` (noalloc 0), or
 * bw_gemm_f16_noalloc's (noalloc 1, variant 0) -- the rule on the pairs of SMs the device holds at once (its cluster
 * occupancy, asked once), and for the no-allocation entry the fallback that fits its fixed array, if the rule's plan
 * does not.  Host work only (no launch), but it needs the device.  No reference counterpart.
 */
int bw_gemm_device_plan(int M, int N, int K, int variant, int noalloc, bw_plan* out);

/*
 * The device status word of the current device, after the caller has synchronised: *code = 0, or BW_ERR_TIMEOUT if
 * a bounded wait gave up since the last clear; *site = role << 16 | barrier kind << 8 | index of the first wait that
 * gave up, *block its block, *segment the segment that block was on.  Kinds: 0 a full stage, 1 an empty stage, 2 a
 * finished accumulator, 3 a free accumulator, 4 partials copied in, 5 and 6 a K-split cluster's pieces and go signal,
 * 7 another rank's partial of the fused reduce-scatter (index: the sender), 8 a rank's ack of the previous call, 9 an
 * entry of the block's queue of units (a plan with dyn 1).
 * Returns a CUDA error as BW_ERR_LAUNCH.
 * No reference counterpart as a function: the reference traps in its guarded wait (hopper/step2.cuh:128-145); this
 * rung's waits return instead and leave the context usable.
 */
int bw_gemm_status(int* code, unsigned* site, unsigned* block, unsigned* segment);

/* Clears the status word and puts back to zero the split-tile counters of the current device that a call whose wait
 * gave up may have left set (call it after handling BW_ERR_TIMEOUT, with the device idle; it synchronises the
 * device).  No reference counterpart. */
int bw_gemm_clear_status(void);

/* The limit of any single wait on a barrier, in nanoseconds (default 1 s; the BWGEMM_WAIT_NS environment variable
 * sets it at load).  Returns the previous limit.
 * BWGEMM_PDL=1 in the environment at load launches every call but bw_gemm_f16_rs with programmatic stream
 * serialisation: its blocks may start their set-up before the call ahead of it on the stream has finished, and wait
 * for it before their first access to global memory.  Off by default. */
unsigned long long bw_gemm_set_wait_limit_ns(unsigned long long ns);

/*
 * The bounded-wait check, for a caller's health check: one warp waits, through the same bounded wait as the GEMM's
 * pipeline, on a shared-memory barrier that nothing arrives on, for `limit_ns` (0: the current wait limit; at most
 * 10 s).  The wait gives up, records site 7 << 16 in the status word and the kernel returns.  Clears the status word
 * first, synchronises `stream` (unlike the GEMM entries) and returns BW_ERR_TIMEOUT -- the expected outcome: a stall
 * ends with a status and a usable context, not a hang.  Any other return is a failure.
 * No reference counterpart: the reference's guarded wait traps (hopper/step2.cuh:128-145).
 */
int bw_wait_selftest(unsigned long long limit_ns, void* stream);

/* Text of a status code, and of the last CUDA error met by the library on this thread. */
const char* bw_status_string(int status);
const char* bw_last_error_string(void);

#ifdef __cplusplus
}
#endif

#endif /* BWGEMM_H */
