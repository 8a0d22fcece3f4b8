// ref_emu_dump.cpp -- TEST INFRASTRUCTURE ONLY (never part of the product).
//
// Builds the reference's own Hopper host emulator from its sources where they lie (hopper/emu/emu.cpp, compiled in
// place through the include path that ref.mk gives; nothing of it is copied into this repository) and runs ONE of its
// kernels at ONE shape on the emulator's own inputs, then writes what the reference computed:
//
//   <out>.A.u16   the fp16 bits of A as the emulator drew them (LCG seed 7, hopper/emu/emu.cpp:2568-2570)
//   <out>.B.u16   the fp16 bits of B (the same LCG state carried on)
//   <out>.C.u16   the fp16 bits of C written by the reference's Hopper kernel, run by the emulator in forward order
//   <out>.ref.f64 the emulator's own fp64 reference (hopper/emu/emu.cpp:2571-2576)
//
// These files pin the oracle (oracle.c): its generator must reproduce A and B bit for bit, its fp64 GEMM the reference
// to rounding, and its checks must accept the reference kernel's C.  tests/golden/make_golden.py turns them into the
// committed fixtures.
//
// Usage: ref_emu_dump --list
//        ref_emu_dump "<kernel label>" M N K <out prefix>
#define main gemm_ladder_hopper_emu_main
#include "emu.cpp"
#undef main

#include <cstdio>
#include <string>

static bool write_file(const std::string& path, const void* p, size_t bytes)
{
    FILE* f = fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = fwrite(p, 1, bytes, f) == bytes;
    return fclose(f) == 0 && ok;
}

int main(int argc, char** argv)
{
    setvbuf(stdout, nullptr, _IOLBF, 0);
    const std::vector<Kernel> all = kernels();
    if (argc == 2 && std::string(argv[1]) == "--list") {
        for (const Kernel& k : all) printf("%s\n", k.label);
        return 0;
    }
    if (argc != 6) {
        fprintf(stderr, "usage: %s --list | \"<kernel label>\" M N K <out prefix>\n", argv[0]);
        return 2;
    }
    const std::string label = argv[1];
    const int M = atoi(argv[2]), N = atoi(argv[3]), K = atoi(argv[4]);
    const std::string out = argv[5];
    const Kernel* kern = nullptr;
    for (const Kernel& k : all)
        if (label == k.label) kern = &k;
    if (!kern) {
        fprintf(stderr, "no kernel labelled \"%s\" (try --list)\n", label.c_str());
        return 2;
    }
    if (M <= 0 || N <= 0 || K <= 0 || M > kern->maxM || N % kern->nMultiple) {
        fprintf(stderr, "%s cannot take %d x %d x %d\n", kern->label, M, N, K);
        return 2;
    }

    // The emulator's coroutine stacks (each above a PROT_NONE page) and its fault handler on a stack of its own: the
    // set-up its run() expects, as the emulator's main does it.
    g_stacks = (char*)mmap(nullptr, kMaxThreads * (kPage + kStackBytes), PROT_READ | PROT_WRITE,
                           MAP_PRIVATE | MAP_ANONYMOUS | MAP_NORESERVE, -1, 0);
    if (g_stacks == MAP_FAILED) {
        perror("mmap");
        return 2;
    }
    for (int t = 0; t < kMaxThreads; t++) mprotect(g_stacks + t * (kPage + kStackBytes), kPage, PROT_NONE);
    static char faultStack[64 << 10];
    stack_t ss = {};
    ss.ss_sp = faultStack;
    ss.ss_size = sizeof faultStack;
    sigaltstack(&ss, nullptr);
    struct sigaction sa = {};
    sa.sa_sigaction = on_fault;
    sa.sa_flags = SA_SIGINFO | SA_ONSTACK;
    sigemptyset(&sa.sa_mask);
    sigaction(SIGSEGV, &sa, nullptr);
    sigaction(SIGBUS, &sa, nullptr);
    sigaction(SIGFPE, &sa, nullptr);

    // The emulator's inputs and reference, drawn by its own functions (allocate, rnd).
    allocate(g_A, M, K, false);
    allocate(g_B, K, N, false);
    allocate(g_C, M, N, true);
    unsigned seed = 7;
    for (size_t i = 0; i < (size_t)M * K; i++) g_A.p[i] = (half)rnd(seed);
    for (size_t i = 0; i < (size_t)K * N; i++) g_B.p[i] = (half)rnd(seed);
    std::vector<double> ref((size_t)M * N, 0.0);
    for (int i = 0; i < M; i++)
        for (int k = 0; k < K; k++) {
            const double a = (double)g_A.p[(size_t)i * K + k];
            for (int j = 0; j < N; j++) ref[(size_t)i * N + j] += a * (double)g_B.p[(size_t)k * N + j];
        }
    double mref = 0;
    for (const double r : ref) mref = std::max(mref, std::fabs(r));

    std::vector<uint16_t> forward;
    std::map<unsigned, SameBits> same;
    Totals totals;
    const bool ok = run(*kern, M, N, K, kForward, forward, same, ref, mref, totals);
    if (!ok) {
        fprintf(stderr, "the emulator reported a failure for %s at %d x %d x %d\n", kern->label, M, N, K);
        return 1;
    }
    const size_t nA = (size_t)M * K, nB = (size_t)K * N, nC = (size_t)M * N;
    if (!write_file(out + ".A.u16", g_A.p, nA * 2) || !write_file(out + ".B.u16", g_B.p, nB * 2) ||
        !write_file(out + ".C.u16", g_C.p, nC * 2) || !write_file(out + ".ref.f64", ref.data(), nC * 8)) {
        perror("write");
        return 2;
    }
    printf("dumped %s at %d x %d x %d to %s.*\n", kern->label, M, N, K, out.c_str());
    return 0;
}
