"""Parity of the sm_100a path with the oracle, through the C ABI, on a B200.

- The reference's own fixtures (tests/golden, dumped from its Hopper emulator): the same inputs, and C within the
  per-element bound of the fp64 reference; the reference kernel's C and ours within twice that bound of each other,
  and most elements bit-identical.
- The reference's 26 verif shapes (hopper/verif.cu:158-163) on its LCG inputs, every variant: per element
  |C - ref16| <= 2 ulp16(|ref16|) + 1e-3 sqrt(K) and normwise <= 2e-3 against the fp64 oracle, 8 calls compared bit for
  bit (hopper/verif.cu:197-215), the stream-K counters back at zero (candidate_dirty, :216-222).
- This rung's own edges (half tiles in N, every swap-AB width, stream-K shares inside one tile).
- The judge's 17 B200 shapes and the BASELINE configs at full size on the judge's fill: the judge's gate against an
  fp32 GEMM (max|C - ref| / max|ref| <= 2e-3, every element finite; judge/judge.cu:12,138-154) and 2048 elements
  against the fp64 oracle per element.
- Streams, CUDA-graph capture with new contents at the same addresses (judge/judge.cu:13-18), A and B unchanged.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

import bwgemm  # noqa: E402
from shapes import B200_EDGES, CONFIG1, DECODE_M, DECODE_WEIGHTS, JUDGE_B200, LADDER_4096, RAGGED_M, VERIF  # noqa: E402

pytestmark = pytest.mark.gpu

NAN16 = 0xFFFF  # the pattern an unwritten element keeps


@pytest.fixture(scope="module", autouse=True)
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    assert torch.cuda.get_device_capability(0) == (10, 0), "an sm_100 (B200) device is required"
    torch.cuda.set_device(0)
    bwgemm.clear_status()
    yield
    torch.cuda.synchronize()
    assert bwgemm.status()[0] == 0


def to_dev(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.float16)).cuda()


def run(A, B, variant=0, C=None):
    M, K = A.shape
    N = B.shape[1]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    C.view(torch.int16).fill_(-1)  # NaN: an element left unwritten shows
    bwgemm.gemm(A, B, C, variant=variant)
    torch.cuda.synchronize()
    code = bwgemm.status()
    assert code[0] == 0, f"device status {code}"
    return C


def bits(C):
    return C.cpu().numpy().view(np.uint16)


_ref_cache = {}


def lcg_case(M, N, K, oracle_mod):
    key = (M, N, K)
    if key not in _ref_cache:
        _ref_cache.clear()
        A, B = oracle_mod.lcg_inputs(M, N, K)
        _ref_cache[key] = (A, B, oracle_mod.gemm_f64(A, B))
    return _ref_cache[key]


def assert_parity(C_bits, ref, K, oracle_mod, what):
    r = oracle_mod.check(C_bits, ref, K)
    assert r["nonfinite"] == 0, f"{what}: {r['nonfinite']} elements not finite (unwritten?), first at {r['first_bad']}"
    assert r["violations"] == 0, f"{what}: {r['violations']} elements over the per-element bound, first at " \
                                 f"{r['first_bad']} (worst ratio {r['worst_ratio']:.2f})"
    assert r["normwise"] <= 2e-3, f"{what}: normwise {r['normwise']:.3e}"
    return r


# ---------------------------------------------------------------------------------------------- the reference's own
def test_smoke_one_tile(oracle_mod):
    A, B, ref = lcg_case(128, 256, 64, oracle_mod)
    C = run(to_dev(A), to_dev(B))
    assert_parity(bits(C), ref, 64, oracle_mod, "128x256x64")


def test_smoke_swap(oracle_mod):
    A, B, ref = lcg_case(16, 256, 64, oracle_mod)
    C = run(to_dev(A), to_dev(B))
    assert_parity(bits(C), ref, 64, oracle_mod, "16x256x64")


def golden_files():
    import glob
    import os
    return sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


@pytest.mark.parametrize("path", golden_files(), ids=lambda p: p.rsplit("/", 1)[-1][:-4])
def test_golden_reference_fixtures(path, oracle_mod):
    g = np.load(path)
    M, N, K = (int(x) for x in g["shape"])
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    for v in range(bwgemm.lib().bw_gemm_variant_count()):
        C = bits(run(to_dev(A), to_dev(B), variant=v))
        assert_parity(C, ref, K, oracle_mod, f"{path} v{v}")
        # ours and the reference kernel's C: each within the bound of the fp64 result, so within twice the bound of
        # each other (both round fp32 sums of a different order; near zero that is many ulp of the value itself)
        ours = C.view(np.float16).astype(np.float64)
        theirs = g["c"].view(np.float16).astype(np.float64)
        L = oracle_mod.lib()
        bound = np.array([2 * L.oracle_ulp16(float(x)) for x in np.abs(theirs).ravel()]).reshape(theirs.shape)
        bound += 1e-3 * np.sqrt(K)
        assert np.all(np.abs(ours - theirs) <= 2 * bound), f"v{v}: farther from the reference kernel's C than 2 bounds"
        same = np.mean(C == g["c"])
        assert same > 0.5, f"v{v}: only {same:.1%} of C bit-identical to the reference kernel's"


@pytest.mark.parametrize("shape", VERIF, ids=lambda s: "x".join(map(str, s)))
def test_verif_shapes_every_variant_bit_for_bit(shape, oracle_mod):
    M, N, K = shape
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    dA, dB = to_dev(A), to_dev(B)
    for v in range(bwgemm.lib().bw_gemm_variant_count()):
        first = bits(run(dA, dB, variant=v))
        assert_parity(first, ref, K, oracle_mod, f"{shape} v{v}")
        for _ in range(7):  # 8 calls in all, compared bit for bit
            assert np.array_equal(bits(run(dA, dB, variant=v)), first), f"{shape} v{v}: calls differ (a race)"
        assert bwgemm.dirty() == 0, f"{shape} v{v}: stream-K counters left non-zero"
    assert np.array_equal(bits(dA), A) and np.array_equal(bits(dB), B), "A or B modified"


@pytest.mark.parametrize("shape", B200_EDGES, ids=lambda s: "x".join(map(str, s)))
def test_b200_edges(shape, oracle_mod):
    M, N, K = shape
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    dA, dB = to_dev(A), to_dev(B)
    for v in range(bwgemm.lib().bw_gemm_variant_count()):
        first = bits(run(dA, dB, variant=v))
        assert_parity(first, ref, K, oracle_mod, f"{shape} v{v}")
        assert np.array_equal(bits(run(dA, dB, variant=v)), first)
    assert bwgemm.dirty() == 0


@pytest.mark.parametrize("shape", RAGGED_M, ids=lambda s: "x".join(map(str, s)))
def test_ragged_m_every_variant(shape, oracle_mod):
    """M not a multiple of 16 (decode steps of 1 or 8 tokens, ragged last tiles): every variant against the fp64
    oracle under both gates, 2 calls bit for bit, nothing written past row M (C's padding rows keep their NaN)."""
    M, N, K = shape
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    dA, dB = to_dev(A), to_dev(B)
    pad = torch.empty((M + 16, N), dtype=torch.float16, device="cuda")
    for v in range(bwgemm.lib().bw_gemm_variant_count()):
        pad.view(torch.int16).fill_(-1)
        first = bits(run(dA, dB, variant=v, C=pad[:M]))
        assert_parity(first, ref, K, oracle_mod, f"{shape} v{v}")
        assert np.all(bits(pad[M:]) == NAN16), f"{shape} v{v}: rows past M written"
        assert np.array_equal(bits(run(dA, dB, variant=v)), first), f"{shape} v{v}: calls differ"
    assert bwgemm.dirty() == 0


# ---------------------------------------------------------------------------------------------- full sizes
def judge_inputs_dev(M, N, K, oracle_mod):
    A, B = oracle_mod.judge_inputs(M, N, K)
    return A, B, to_dev(A), to_dev(B)


def judge_gate(C, dA, dB):
    """judge/judge.cu's gate against an fp32 GEMM: max|C - ref| / max|ref| <= 2e-3, every element finite."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = torch.matmul(dA.float(), dB.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    c = C.float()
    assert bool(torch.isfinite(c).all()), "an element not finite (unwritten?)"
    gap = ((c - ref).abs().max() / ref.abs().max()).item()
    return gap


def spot_check(C_bits, A, B, K, oracle_mod, n=2048, seed=0):
    M, N = C_bits.shape
    rng = np.random.default_rng(seed)
    ii = rng.integers(0, M, n)
    jj = rng.integers(0, N, n)
    # always the corners and the last rows / columns of the edge tiles
    ii = np.concatenate([ii, [0, 0, M - 1, M - 1]])
    jj = np.concatenate([jj, [0, N - 1, 0, N - 1]])
    ref = np.array([oracle_mod.dot_f64(A, B, int(i), int(j)) for i, j in zip(ii, jj)])
    got = C_bits[ii, jj]
    assert_parity(got, ref, K, oracle_mod, "spot check")


FULL = [(n, m, nn, k) for n, m, nn, k in JUDGE_B200] + [LADDER_4096, CONFIG1]


@pytest.mark.parametrize("case", FULL, ids=lambda c: c[0])
def test_full_size_judge_gate_and_spot_check(case, oracle_mod):
    name, M, N, K = case
    A, B, dA, dB = judge_inputs_dev(M, N, K, oracle_mod)
    C = run(dA, dB)
    gap = judge_gate(C, dA, dB)
    assert gap <= 2e-3, f"{name}: judge gap {gap:.3e}"
    Cb = bits(C)
    spot_check(Cb, A, B, K, oracle_mod)
    assert np.array_equal(bits(run(dA, dB)), Cb), f"{name}: calls differ"
    assert bwgemm.dirty() == 0


@pytest.mark.parametrize("weight", DECODE_WEIGHTS, ids=lambda w: w[0])
def test_decode_regime(weight, oracle_mod):
    name, N, K = weight
    B = oracle_mod.judge_fill(K * N, 2).reshape(K, N)
    dB = to_dev(B)
    for M in DECODE_M:
        A = oracle_mod.judge_fill(M * K, 1).reshape(M, K)
        dA = to_dev(A)
        C = run(dA, dB)
        assert judge_gate(C, dA, dB) <= 2e-3
        spot_check(bits(C), A, B, K, oracle_mod, n=512, seed=M)


# ---------------------------------------------------------------------------------------------- the judge's rules
def test_side_stream_and_graph_capture(oracle_mod):
    M, N, K = 272, 5376, 128  # stream-K tail + data-parallel tiles
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    dA, dB = to_dev(A), to_dev(B)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        bwgemm.gemm(dA, dB, C)  # first call of the shape: outside the capture
    s.synchronize()
    assert_parity(bits(C), ref, K, oracle_mod, "side stream")
    g = torch.cuda.CUDAGraph()
    C.view(torch.int16).fill_(-1)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        for _ in range(3):
            bwgemm.gemm(dA, dB, C)
    g.replay()
    torch.cuda.synchronize()
    assert_parity(bits(C), ref, K, oracle_mod, "graph")
    # new contents at the same addresses, the graph again (a kept result would fail)
    A2, B2 = oracle_mod.judge_inputs(M, N, K, seed_a=11, seed_b=12)
    dA.copy_(to_dev(A2))
    dB.copy_(to_dev(B2))
    C.view(torch.int16).fill_(-1)
    g.replay()
    torch.cuda.synchronize()
    assert_parity(bits(C), oracle_mod.gemm_f64(A2, B2), K, oracle_mod, "graph, new contents")
    assert bwgemm.dirty() == 0
    assert bwgemm.status()[0] == 0


def test_graph_survives_a_later_workspace_growth(oracle_mod):
    """A graph captured at one shape replays correctly after a call at another shape needed a larger workspace: the
    library never frees a workspace that a captured graph may hold."""
    M, N, K = 16, 1024, 1024  # swap-AB + stream-K: a small workspace
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    dA, dB = to_dev(A), to_dev(B)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    bwgemm.gemm(dA, dB, C)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        bwgemm.gemm(dA, dB, C)
    M2, N2, K2 = 256, 9728, 8192  # a split-K tail of 38 pair tiles x 3: a much larger workspace
    assert bwgemm.plan(M2, N2, K2)["workspace_bytes"] > 20 << 20
    X = torch.rand((M2, K2), device="cuda").half()
    Y = torch.rand((K2, N2), device="cuda").half()
    Z = torch.empty((M2, N2), dtype=torch.float16, device="cuda")
    bwgemm.gemm(X, Y, Z)
    torch.cuda.synchronize()
    for _ in range(2):
        C.view(torch.int16).fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        assert bwgemm.status()[0] == 0
        assert_parity(bits(C), ref, K, oracle_mod, "graph replayed after a workspace growth")
    assert bwgemm.dirty() == 0


@pytest.mark.parametrize("shape", [(256, 512, 1024), (2048, 8192, 28672 // 8), (4608, 5632, 8192), (144, 640, 320)],
                         ids=lambda s: "x".join(map(str, s)))
def test_f32out_partials(shape, oracle_mod):
    """bw_gemm_f16_f32out: fp32 C within fp32 accumulation error of the fp64 oracle, and, where the fp16 entry takes the
    same plan (above M = 128 on 256-column pair tiles: the fp32 entry never takes the 512-column ones), rounded to fp16
    it is the fp16 entry's result bit for bit."""
    M, N, K = shape
    A, B = oracle_mod.judge_inputs(M, N, K)
    dA, dB = to_dev(A), to_dev(B)
    C32 = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
    bwgemm.gemm_f32out(dA, dB, C32)
    torch.cuda.synchronize()
    assert bwgemm.status()[0] == 0
    got = C32.cpu().numpy().astype(np.float64)
    assert np.isfinite(got).all()
    rng = np.random.default_rng(3)
    for i, j in zip(rng.integers(0, M, 512), rng.integers(0, N, 512)):
        ref = oracle_mod.dot_f64(A, B, int(i), int(j))
        assert abs(got[i, j] - ref) <= 1e-4 * K ** 0.5, (i, j, got[i, j], ref)
    C16 = run(dA, dB)
    if M > 128 and bwgemm.device_plan(M, N, K)["bn"] == 256:
        assert torch.equal(C32.half(), C16), "fp32 partials rounded differ from the fp16 entry's result"
    assert bwgemm.dirty() == 0


def test_tp_mlp_block_on_one_gpu():
    """The tensor-parallel block at one rank (no collective) through the rung's GEMMs, against torch in fp32."""
    import tp_mlp

    M, hidden, f = 512, 1024, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    X = (torch.rand((M, hidden), generator=g, device="cuda") * 2 - 1).half()
    W1 = ((torch.rand((hidden, 2 * f), generator=g, device="cuda") * 2 - 1) / hidden ** 0.5).half()
    W2 = ((torch.rand((f, hidden), generator=g, device="cuda") * 2 - 1) / f ** 0.5).half()
    blk = tp_mlp.TPMLP(tp_mlp.shard_gateup(W1, 0, 1), tp_mlp.shard_down(W2, 0, 1), 0, 1, bwgemm.gemm,
                       bwgemm.gemm_f32out)
    Y = blk.forward(X)
    torch.cuda.synchronize()
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        H = (X.float() @ W1.float()).half()
        A = (torch.nn.functional.silu(H[:, :f].float()) * H[:, f:].float()).half()
        ref = A.float() @ W2.float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    gap = ((Y.float() - ref).abs().max() / ref.abs().max()).item()
    assert gap <= 2e-3, gap


@pytest.mark.parametrize("shape", [(512, 2048, 1024), (2048, 7168, 8192), (144, 512, 320)],
                         ids=lambda s: "x".join(map(str, s)))
def test_swiglu_fused_epilogue(shape):
    """bw_gemm_f16_swiglu against silu(gate) * up computed from an fp32 GEMM (no TF32) on the interleaved layout."""
    import tp_mlp

    M, N, K = shape
    g = torch.Generator(device="cuda")
    g.manual_seed(M + N)
    X = (torch.rand((M, K), generator=g, device="cuda") * 2 - 1).half()
    W = ((torch.rand((K, N), generator=g, device="cuda") * 2 - 1) / K ** 0.5).half()
    A = bwgemm.gemm_swiglu(X, W)
    torch.cuda.synchronize()
    assert bwgemm.status()[0] == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        ref = tp_mlp.swiglu_reference(X, W).float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert A.shape == (M, N // 2) and bool(torch.isfinite(A.float()).all())
    gap = ((A.float() - ref).abs().max() / ref.abs().max()).item()
    assert gap <= 2e-3, gap
    assert torch.equal(bwgemm.gemm_swiglu(X, W), A), "calls differ"


def test_tp_mlp_block_fused_on_one_gpu():
    """The block with the activation fused into the gateup GEMM equals the unfused block within fp16 rounding."""
    import tp_mlp

    M, hidden, f = 512, 1024, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(10)
    X = (torch.rand((M, hidden), generator=g, device="cuda") * 2 - 1).half()
    W1 = ((torch.rand((hidden, 2 * f), generator=g, device="cuda") * 2 - 1) / hidden ** 0.5).half()
    W2 = ((torch.rand((f, hidden), generator=g, device="cuda") * 2 - 1) / f ** 0.5).half()
    fused = tp_mlp.TPMLP(tp_mlp.shard_gateup_interleaved(W1, 0, 1), tp_mlp.shard_down(W2, 0, 1), 0, 1, bwgemm.gemm,
                         bwgemm.gemm_f32out, gemm_swiglu=bwgemm.gemm_swiglu).forward(X)
    plain = tp_mlp.TPMLP(tp_mlp.shard_gateup(W1, 0, 1), tp_mlp.shard_down(W2, 0, 1), 0, 1, bwgemm.gemm,
                         bwgemm.gemm_f32out).forward(X)
    torch.cuda.synchronize()
    gap = ((fused.float() - plain.float()).abs().max() / plain.float().abs().max()).item()
    assert gap <= 4e-3, gap


def test_a_wait_that_runs_out_returns_a_status_and_the_context_stays_usable(oracle_mod):
    """The pipeline's bounded wait, on a barrier that nothing arrives on (bw_wait_selftest): it gives up after its
    limit, the kernel returns, the host reads BW_ERR_TIMEOUT and the wait's site from the status word, and the next
    GEMM on the same context is correct.  No fault, trap or endless loop is involved."""
    import time

    t0 = time.monotonic()
    assert bwgemm.wait_selftest(50_000_000) == 3  # a 50 ms limit
    assert time.monotonic() - t0 < 10
    code, where, block, _ = bwgemm.status()
    assert (code, where, block) == (3, 7 << 16, 0)
    assert bwgemm.lib().bw_wait_selftest(20_000_000_000, None) == 4  # a limit over 10 s is refused
    bwgemm.clear_status()
    A, B, ref = lcg_case(256, 512, 1024, oracle_mod)
    C = run(to_dev(A), to_dev(B))
    assert_parity(bits(C), ref, 1024, oracle_mod, "256x512x1024 after the selftest")


# ------------------------------------------------------------------ B given as N x K (bw_gemm_f16_tn)
TN_SHAPES = sorted(set(VERIF[::2]) | set(B200_EDGES) | {(16, 8192, 1024), (128, 10240, 512), (64, 38080, 128)})


@pytest.mark.parametrize("shape", TN_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_tn_layout_against_the_oracle(shape, oracle_mod):
    """The N x K layout of B (K-major for the tensor core) through every plan form: the same gates against the fp64
    oracle as the K x N entry, 2 calls bit for bit, counters back at zero."""
    M, N, K = shape
    A, B, ref = lcg_case(M, N, K, oracle_mod)
    Bt = np.ascontiguousarray(np.asarray(B).reshape(K, N).T)
    dA, dBt = to_dev(A), to_dev(Bt)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    C.view(torch.int16).fill_(-1)
    bwgemm.gemm_tn(dA, dBt, C)
    torch.cuda.synchronize()
    assert bwgemm.status()[0] == 0
    Cb = bits(C)
    assert_parity(Cb, ref, K, oracle_mod, f"tn {M}x{N}x{K}")
    bwgemm.gemm_tn(dA, dBt, C)
    torch.cuda.synchronize()
    assert np.array_equal(bits(C), Cb), "calls differ"
    assert bwgemm.dirty() == 0


@pytest.mark.parametrize("case", [c for c in FULL if c[0] in ("o_m16", "qkv_m16", "gateup_m128", "o_m2048", "config1")],
                         ids=lambda c: c[0])
def test_tn_layout_full_size(case, oracle_mod):
    """Full-size judge shapes of each plan form (kpair at 128 and 256 columns, stream-K, pair tiles with a split-K
    tail) with B given as N x K: the judge's gate and a spot check against the fp64 oracle."""
    name, M, N, K = case
    A, B, dA, dB = judge_inputs_dev(M, N, K, oracle_mod)
    C = bwgemm.gemm_tn(dA, dB.t().contiguous())
    torch.cuda.synchronize()
    assert bwgemm.status()[0] == 0
    gap = judge_gate(C, dA, dB)
    assert gap <= 2e-3, f"{name}: judge gap {gap:.3e}"
    spot_check(bits(C), A, B, K, oracle_mod)
