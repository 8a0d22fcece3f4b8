/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY.  The CPU restatement of the reference's host-side GEMM arithmetic, used as the
 * checker of the sm_100a path.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it; the
 * product (libbwgemm.so) never links or calls it.
 *
 * What it restates (paths inside the reference project):
 *   - oracle_lcg_fill      : the LCG `rnd` that draws verif.cu's and the emulator's inputs, seed 7, converted to fp16
 *                            round-to-nearest-even (hopper/verif.cu:74, :168-170; hopper/emu/emu.cpp:2048-2052,
 *                            :2568-2570).
 *   - oracle_judge_fill    : the judge's `fill` hash, uniform in [-1, 1) (judge/judge.cu:127-134; the same kernel in
 *                            probe/probe.cu and hopper/verif.cu).
 *   - oracle_gemm_f64      : the fp64 reference, i-k-j loop, double accumulation from the fp16 inputs, C = A B with A
 *                            M x K and B K x N row-major (hopper/verif.cu:171-178; hopper/emu/emu.cpp:2571-2576).
 *   - oracle_check         : the normwise gate max|C - ref| / max|ref| <= 2e-3 with every element finite
 *                            (hopper/verif.cu:179-196, :227; judge/judge.cu:12,78,138-154), plus the per-element
 *                            bound |C - ref16| <= 2 ulp16(|ref16|) + 1e-3 sqrt(K), ref16 = ref rounded to fp16.
 *
 * fp16 conversions are written here from the IEEE 754 binary16 definition (round to nearest, ties to even), not taken
 * from any library.  Pinning: tests/test_oracle.py checks these functions against fixtures dumped by the reference's
 * own emulator (oracle/ref_emu_dump.cpp) and against gcc's _Float16 conversions.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

/* ------------------------------------------------------------------ binary16 conversions */

float oracle_f16_to_f32(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1f;
    const uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        float v = ldexpf((float)man, -24); /* subnormal or zero: man * 2^-24, exact in binary32 */
        memcpy(&bits, &v, 4);
        bits |= sign;
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13); /* infinity or NaN (payload kept) */
    } else {
        bits = sign | ((exp + 112u) << 23) | (man << 13); /* rebias 15 -> 127 */
    }
    float v;
    memcpy(&v, &bits, 4);
    return v;
}

/* Round a double to binary16, nearest-even, with overflow to infinity.  Works from the exact double value, so
 * float -> half and double -> half both round once. */
uint16_t oracle_f64_to_f16(double x)
{
    uint16_t sign = 0;
    if (signbit(x)) {
        sign = 0x8000;
        x = -x;
    }
    if (isnan(x)) return (uint16_t)(sign | 0x7e00);
    if (isinf(x)) return (uint16_t)(sign | 0x7c00);
    /* Smallest subnormal 2^-24; the representable grid below 2^-14 is k * 2^-24. */
    if (x < 0x1p-14) {
        const double q = x * 0x1p24;      /* exact: scaling by a power of two */
        double r = nearbyint(q);          /* default rounding mode: nearest-even */
        return (uint16_t)(sign | (uint16_t)r); /* r <= 1024; 1024 is the smallest normal, bits 0x0400 */
    }
    int e;
    (void)frexp(x, &e);                   /* x = f * 2^e, f in [0.5, 1): unit in [2^(e-1), 2^e) */
    const int unbiased = e - 1;           /* x in [2^unbiased, 2^(unbiased+1)) */
    if (unbiased > 15) return (uint16_t)(sign | 0x7c00);
    const double q = ldexp(x, 10 - unbiased); /* in [1024, 2048): 11 significant bits */
    double r = nearbyint(q);
    int ub = unbiased;
    if (r >= 2048.0) {                    /* rounded up into the next binade */
        r = 1024.0;
        ub += 1;
        if (ub > 15) return (uint16_t)(sign | 0x7c00);
    }
    const uint16_t man = (uint16_t)((int)r - 1024);
    return (uint16_t)(sign | (uint16_t)((ub + 15) << 10) | man);
}

uint16_t oracle_f32_to_f16(float x) { return oracle_f64_to_f16((double)x); }

/* The spacing of binary16 values at |x| (x itself a binary16 value): 2^(e-10) in the binade [2^e, 2^(e+1)),
 * 2^-24 among the subnormals. */
double oracle_ulp16(double ax)
{
    ax = fabs(ax);
    if (ax < 0x1p-14) return 0x1p-24;
    int e;
    (void)frexp(ax, &e);
    return ldexp(1.0, e - 1 - 10);
}

/* ------------------------------------------------------------------ the seeded generators */

/* verif.cu's / the emulator's rnd: s = s * 1664525 + 1013904223; ((s >> 9) & 0xffff) / 32768 - 1 in float, then
 * stored as fp16 (hopper/verif.cu:74 with __float2half at :169; hopper/emu/emu.cpp:2048-2052 with (half) at :2569).
 * The state carries over from one array to the next (A then B from one seed). */
void oracle_lcg_fill(uint16_t* out, size_t n, uint32_t* state)
{
    uint32_t s = *state;
    for (size_t i = 0; i < n; i++) {
        s = s * 1664525u + 1013904223u;
        const float v = (float)((s >> 9) & 0xffffu) / 32768.0f - 1.0f;
        out[i] = oracle_f32_to_f16(v);
    }
    *state = s;
}

/* The judge's fill: a hash of the index and the seed, 24 bits of it scaled to [0, 2), minus 1 (judge/judge.cu:127-134). */
static inline uint16_t judge_value(size_t i, uint32_t seed)
{
    uint32_t x = ((uint32_t)i * 2654435761u) ^ (seed * 0x9e3779b9u) ^ (uint32_t)(i >> 32);
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    const float v = (float)(x >> 8) * (1.0f / 8388608.0f) - 1.0f;
    return oracle_f32_to_f16(v);
}

void oracle_judge_fill(uint16_t* out, size_t n, uint32_t seed)
{
    for (size_t i = 0; i < n; i++) out[i] = judge_value(i, seed);
}

/* Element i of the judge's fill, for spot checks at sizes too large to draw on the CPU. */
uint16_t oracle_judge_value(uint64_t i, uint32_t seed) { return judge_value((size_t)i, seed); }

/* ------------------------------------------------------------------ the fp64 reference GEMM */

typedef struct {
    const uint16_t* A;
    const uint16_t* B;
    double* ref;
    int M, N, K;
    int row0, row1;
    const float* bf; /* B converted once to float (exact) */
} GemmJob;

static void* gemm_rows(void* p)
{
    const GemmJob* j = (const GemmJob*)p;
    const int N = j->N, K = j->K;
    for (int i = j->row0; i < j->row1; i++) {
        double* r = j->ref + (size_t)i * N;
        for (int c = 0; c < N; c++) r[c] = 0.0;
        for (int k = 0; k < K; k++) {
            const double a = (double)oracle_f16_to_f32(j->A[(size_t)i * K + k]);
            const float* b = j->bf + (size_t)k * N;
            for (int c = 0; c < N; c++) r[c] += a * (double)b[c];
        }
    }
    return NULL;
}

/* ref (M x N doubles) = A B in double, the i-k-j order of hopper/verif.cu:171-178, rows split over `threads`
 * threads (each row's sums are in the same order whatever the thread count).  bf_scratch: K*N floats. */
void oracle_gemm_f64(const uint16_t* A, const uint16_t* B, double* ref, int M, int N, int K, int threads,
                     float* bf_scratch)
{
    for (size_t i = 0; i < (size_t)K * N; i++) bf_scratch[i] = oracle_f16_to_f32(B[i]);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > M) threads = M > 0 ? M : 1;
    pthread_t tid[256];
    GemmJob job[256];
    for (int t = 0; t < threads; t++) {
        job[t].A = A;
        job[t].B = B;
        job[t].ref = ref;
        job[t].M = M;
        job[t].N = N;
        job[t].K = K;
        job[t].bf = bf_scratch;
        job[t].row0 = (int)((long)M * t / threads);
        job[t].row1 = (int)((long)M * (t + 1) / threads);
    }
    if (threads == 1) {
        gemm_rows(&job[0]);
        return;
    }
    int started = 0;
    for (int t = 0; t < threads; t++)
        if (pthread_create(&tid[t], NULL, gemm_rows, &job[t]) == 0) started = t + 1;
        else { gemm_rows(&job[t]); tid[t] = 0; }
    for (int t = 0; t < started; t++)
        if (tid[t]) pthread_join(tid[t], NULL);
}

/* One element of the fp64 reference, C[i][j], in the same k order: for spot checks at full sizes. */
double oracle_dot_f64(const uint16_t* A, const uint16_t* B, int N, int K, int i, int j)
{
    double s = 0.0;
    for (int k = 0; k < K; k++)
        s += (double)oracle_f16_to_f32(A[(size_t)i * K + k]) * (double)oracle_f16_to_f32(B[(size_t)k * N + j]);
    return s;
}

/* ------------------------------------------------------------------ the checks */

typedef struct {
    double max_err;        /* max |C - ref| over finite elements */
    double max_ref;        /* max |ref| */
    double normwise;       /* max_err / max_ref, or 1e30 with a non-finite element */
    long long nonfinite;   /* elements not finite (unwritten: NaN pattern 0xffff) */
    long long violations;  /* elements over the per-element bound */
    long long first_bad;   /* index of the first violation, -1 if none */
    double worst_ratio;    /* max over elements of |C - ref16| / bound */
} OracleCheck;

/* C: fp16 bits (M*N), ref: fp64 (M*N).  Per-element bound: |C - ref16| <= 2 ulp16(|ref16|) + 1e-3 sqrt(K). */
void oracle_check(const uint16_t* C, const double* ref, long long n, int K, OracleCheck* out)
{
    OracleCheck r;
    r.max_err = 0;
    r.max_ref = 0;
    r.nonfinite = 0;
    r.violations = 0;
    r.first_bad = -1;
    r.worst_ratio = 0;
    const double slack = 1e-3 * sqrt((double)K);
    for (long long i = 0; i < n; i++) {
        const double c = (double)oracle_f16_to_f32(C[i]);
        const double rf = ref[i];
        if (fabs(rf) > r.max_ref) r.max_ref = fabs(rf);
        if (!isfinite(c)) {
            r.nonfinite++;
            if (r.first_bad < 0) r.first_bad = i;
            r.violations++;
            continue;
        }
        const double d = fabs(c - rf);
        if (d > r.max_err) r.max_err = d;
        const double r16 = (double)oracle_f16_to_f32(oracle_f64_to_f16(rf));
        const double bound = 2.0 * oracle_ulp16(r16) + slack;
        const double e16 = fabs(c - r16);
        const double q = e16 / bound;
        if (q > r.worst_ratio) r.worst_ratio = q;
        if (e16 > bound) {
            r.violations++;
            if (r.first_bad < 0) r.first_bad = i;
        }
    }
    r.normwise = r.nonfinite ? 1e30 : (r.max_ref > 0 ? r.max_err / r.max_ref : r.max_err);
    *out = r;
}

/* ref rounded to fp16 bits (the "C_ref accumulated in fp64 then rounded"). */
void oracle_round_f16(const double* ref, uint16_t* out, long long n)
{
    for (long long i = 0; i < n; i++) out[i] = oracle_f64_to_f16(ref[i]);
}
