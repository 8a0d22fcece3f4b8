"""ctypes view of oracle/liboracle.so -- TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's fp64 GEMM, its seeded generators and its checks (see oracle.c for the reference
lines each function follows).  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module;
the product path (gemm-ladder_b200/) never does.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


class OracleCheck(ctypes.Structure):
    _fields_ = [
        ("max_err", ctypes.c_double),
        ("max_ref", ctypes.c_double),
        ("normwise", ctypes.c_double),
        ("nonfinite", ctypes.c_longlong),
        ("violations", ctypes.c_longlong),
        ("first_bad", ctypes.c_longlong),
        ("worst_ratio", ctypes.c_double),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


_lib = None


def build():
    """Compile liboracle.so from oracle.c (gcc; seconds)."""
    subprocess.check_call(["make", "-s", "-C", HERE], stdout=subprocess.DEVNULL)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(os.path.join(HERE, "oracle.c")):
            build()
        L = ctypes.CDLL(LIB_PATH)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        f64p = ctypes.POINTER(ctypes.c_double)
        f32p = ctypes.POINTER(ctypes.c_float)
        L.oracle_f16_to_f32.restype = ctypes.c_float
        L.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.oracle_f32_to_f16.restype = ctypes.c_uint16
        L.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        L.oracle_f64_to_f16.restype = ctypes.c_uint16
        L.oracle_f64_to_f16.argtypes = [ctypes.c_double]
        L.oracle_ulp16.restype = ctypes.c_double
        L.oracle_ulp16.argtypes = [ctypes.c_double]
        L.oracle_lcg_fill.restype = None
        L.oracle_lcg_fill.argtypes = [u16p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint32)]
        L.oracle_judge_fill.restype = None
        L.oracle_judge_fill.argtypes = [u16p, ctypes.c_size_t, ctypes.c_uint32]
        L.oracle_judge_value.restype = ctypes.c_uint16
        L.oracle_judge_value.argtypes = [ctypes.c_uint64, ctypes.c_uint32]
        L.oracle_gemm_f64.restype = None
        L.oracle_gemm_f64.argtypes = [u16p, u16p, f64p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, f32p]
        L.oracle_dot_f64.restype = ctypes.c_double
        L.oracle_dot_f64.argtypes = [u16p, u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.oracle_check.restype = None
        L.oracle_check.argtypes = [u16p, f64p, ctypes.c_longlong, ctypes.c_int, ctypes.POINTER(OracleCheck)]
        L.oracle_round_f16.restype = None
        L.oracle_round_f16.argtypes = [f64p, u16p, ctypes.c_longlong]
        _lib = L
    return _lib


def _u16(a):
    a = np.ascontiguousarray(a, dtype=np.uint16)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16))


def _f64(a):
    a = np.ascontiguousarray(a, dtype=np.float64)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_double))


def lcg_inputs(M, N, K, seed=7):
    """A (M x K) and B (K x N) fp16 bits from verif.cu's / the emulator's LCG, A first then B from one state."""
    A = np.empty(M * K, dtype=np.uint16)
    B = np.empty(K * N, dtype=np.uint16)
    st = ctypes.c_uint32(seed)
    lib().oracle_lcg_fill(A.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), A.size, ctypes.byref(st))
    lib().oracle_lcg_fill(B.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), B.size, ctypes.byref(st))
    return A.reshape(M, K), B.reshape(K, N)


def judge_fill(n, seed):
    """n fp16 bits of the judge's fill (uniform in [-1, 1))."""
    out = np.empty(n, dtype=np.uint16)
    lib().oracle_judge_fill(out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), n, seed)
    return out


def judge_inputs(M, N, K, seed_a=1, seed_b=2):
    """A and B as the reference's verif.cu one-shot mode and the judge draw them (fill with seeds 1 and 2)."""
    return judge_fill(M * K, seed_a).reshape(M, K), judge_fill(K * N, seed_b).reshape(K, N)


def gemm_f64(A, B, threads=None):
    """The fp64 reference C = A B (i-k-j order), A and B as fp16 bits."""
    A, pa = _u16(A)
    B, pb = _u16(B)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    ref = np.empty((M, N), dtype=np.float64)
    scratch = np.empty(K * N, dtype=np.float32)
    if threads is None:
        threads = os.cpu_count() or 1
    lib().oracle_gemm_f64(pa, pb, ref.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), M, N, K, threads,
                          scratch.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return ref


def dot_f64(A, B, i, j):
    """One element of the fp64 reference (same k order)."""
    A, pa = _u16(A)
    B, pb = _u16(B)
    return lib().oracle_dot_f64(pa, pb, B.shape[1], A.shape[1], i, j)


def check(C, ref, K):
    """Normwise and per-element checks of fp16 bits C against the fp64 reference."""
    C, pc = _u16(C)
    ref, pr = _f64(ref)
    assert C.size == ref.size
    out = OracleCheck()
    lib().oracle_check(pc, pr, C.size, K, ctypes.byref(out))
    return out.as_dict()


def round_f16(ref):
    ref, pr = _f64(ref)
    out = np.empty(ref.shape, dtype=np.uint16)
    lib().oracle_round_f16(pr, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint16)), ref.size)
    return out


def f16_bits_to_f32(h):
    L = lib()
    return np.array([L.oracle_f16_to_f32(int(x)) for x in np.asarray(h).ravel()], dtype=np.float32)


def tolerance(ref16_value, K):
    """The per-element bound at one fp16 reference value: 2 ulp16(|ref|) + 1e-3 sqrt(K)."""
    return 2.0 * lib().oracle_ulp16(float(ref16_value)) + 1e-3 * float(K) ** 0.5
