"""Python view of the Blackwell rung's C ABI (include/bwgemm.h) over gemm-ladder_b200/lib/libbwgemm.so.

The product is the native library; this module only binds it with ctypes for Python callers (tests, bench.py) and
passes torch tensors' device pointers and torch's current CUDA stream.  There is no fallback: if the library is
missing or the device is not an sm_100 GPU, calls raise.

    import bwgemm
    C = bwgemm.gemm(A, B)          # A (M x K), B (K x N) fp16 CUDA tensors, row-major; C (M x N) fp16
"""
import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
# BWGEMM_LIB picks another build of the library in lib/ (e.g. libbwgemm_next.so from build.py --next), or a path
LIB_PATH = os.path.join(HERE, "lib", os.environ.get("BWGEMM_LIB") or "libbwgemm.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "bwgemm.h")

BW_OK, BW_ERR_SHAPE, BW_ERR_LAUNCH, BW_ERR_TIMEOUT, BW_ERR_ARG, BW_ERR_DEVICE = 0, 1, 2, 3, 4, 5
BW_KERNEL_TILE, BW_KERNEL_SWAP, BW_KERNEL_PAIR = 0, 1, 2


class Plan(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int),
        ("bn", ctypes.c_int),
        ("stages", ctypes.c_int),
        ("tiles_m", ctypes.c_int),
        ("tiles_n", ctypes.c_int),
        ("tiles", ctypes.c_int),
        ("kblocks", ctypes.c_int),
        ("grid", ctypes.c_int),
        ("dp_tiles", ctypes.c_int),
        ("sk_tiles", ctypes.c_int),
        ("splits", ctypes.c_int),
        ("sk_iters", ctypes.c_longlong),
        ("group_rows", ctypes.c_int),
        ("workspace_bytes", ctypes.c_size_t),
        ("counters", ctypes.c_int),
        ("smem_bytes", ctypes.c_int),
        ("tmem_cols", ctypes.c_int),
        ("ksplit", ctypes.c_int),
        ("wm", ctypes.c_int),
        ("dyn", ctypes.c_int),
    ]

    def as_dict(self):
        return {name: getattr(self, name) for name, _ in self._fields_}


class BwError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(msg)
        self.status = status


_lib = None


def lib():
    """The loaded library (raises if it was not built: python gemm-ladder_b200/build.py)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with python gemm-ladder_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        vp, i = ctypes.c_void_p, ctypes.c_int
        L.bw_gemm_f16.argtypes = [vp, vp, vp, i, i, i, vp]
        L.bw_gemm_f16.restype = i
        L.bw_gemm_f16_variant.argtypes = [vp, vp, vp, i, i, i, vp, i]
        L.bw_gemm_f16_variant.restype = i
        L.bw_gemm_f16_tn.argtypes = [vp, vp, vp, i, i, i, vp]
        L.bw_gemm_f16_tn.restype = i
        L.bw_gemm_f16_f32out.argtypes = [vp, vp, vp, i, i, i, vp]
        L.bw_gemm_f16_f32out.restype = i
        L.bw_gemm_f16_swiglu.argtypes = [vp, vp, vp, i, i, i, vp]
        L.bw_gemm_f16_swiglu.restype = i
        L.bw_gemm_variant_count.argtypes = []
        L.bw_gemm_variant_count.restype = i
        L.bw_gemm_variant_name.argtypes = [i]
        L.bw_gemm_variant_name.restype = ctypes.c_char_p
        L.bw_gemm_dirty.argtypes = []
        L.bw_gemm_dirty.restype = i
        L.bw_gemm_plan.argtypes = [i, i, i, i, i, ctypes.POINTER(Plan)]
        L.bw_gemm_plan.restype = i
        L.bw_gemm_device_plan.argtypes = [i, i, i, i, i, ctypes.POINTER(Plan)]
        L.bw_gemm_device_plan.restype = i
        L.bw_gemm_f16_noalloc.argtypes = [vp, vp, vp, i, i, i, vp]
        L.bw_gemm_f16_noalloc.restype = i
        u = ctypes.POINTER(ctypes.c_uint)
        L.bw_gemm_status.argtypes = [ctypes.POINTER(ctypes.c_int), u, u, u]
        L.bw_gemm_status.restype = i
        L.bw_gemm_clear_status.argtypes = []
        L.bw_gemm_clear_status.restype = i
        L.bw_gemm_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
        L.bw_gemm_set_wait_limit_ns.restype = ctypes.c_ulonglong
        L.bw_wait_selftest.argtypes = [ctypes.c_ulonglong, vp]
        L.bw_wait_selftest.restype = i
        L.bw_rs_create.argtypes = [i, i, i, i, ctypes.POINTER(vp)]
        L.bw_rs_create.restype = i
        L.bw_rs_region_bytes.argtypes = [vp]
        L.bw_rs_region_bytes.restype = ctypes.c_size_t
        L.bw_rs_handle.argtypes = [vp, ctypes.c_char_p]
        L.bw_rs_handle.restype = i
        L.bw_rs_connect.argtypes = [vp, ctypes.c_char_p]
        L.bw_rs_connect.restype = i
        L.bw_gemm_f16_rs.argtypes = [vp, vp, vp, vp, i, vp]
        L.bw_gemm_f16_rs.restype = i
        L.bw_rs_destroy.argtypes = [vp]
        L.bw_rs_destroy.restype = i
        L.bw_status_string.argtypes = [i]
        L.bw_status_string.restype = ctypes.c_char_p
        L.bw_last_error_string.argtypes = []
        L.bw_last_error_string.restype = ctypes.c_char_p
        _lib = L
    return _lib


def declared_symbols():
    """The functions include/bwgemm.h declares."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(bw_\w+)\s*\(", text, flags=re.M)))


def check(status):
    if status != BW_OK:
        L = lib()
        msg = L.bw_status_string(status).decode()
        if status == BW_ERR_LAUNCH:
            msg += ": " + L.bw_last_error_string().decode()
        raise BwError(status, msg)


def variants():
    L = lib()
    return [L.bw_gemm_variant_name(v).decode() for v in range(L.bw_gemm_variant_count())]


def plan(M, N, K, sms=148, variant=0):
    p = Plan()
    check(lib().bw_gemm_plan(M, N, K, sms, variant, ctypes.byref(p)))
    return p.as_dict()


def device_plan(M, N, K, variant=0, noalloc=False):
    """The plan a call takes on the current device (bw_gemm_device_plan): the rule on the device's own pair count, or
    the no-allocation entry's plan (the rule's, or the fallback that fits its fixed array)."""
    p = Plan()
    check(lib().bw_gemm_device_plan(M, N, K, variant, 1 if noalloc else 0, ctypes.byref(p)))
    return p.as_dict()


def gemm_ptr(a_ptr, b_ptr, c_ptr, M, N, K, stream_handle=0, variant=0):
    """C = A B on raw device pointers (the C ABI as it is); returns the status code."""
    return lib().bw_gemm_f16_variant(a_ptr, b_ptr, c_ptr, M, N, K, stream_handle, variant)


def gemm(A, B, C=None, variant=0, stream=None):
    """C = A B for fp16 CUDA tensors: A (M x K) and B (K x N) row-major (contiguous); C (M x N) is made if not given."""
    import torch

    M, K = A.shape
    K2, N = B.shape
    if K2 != K:
        raise ValueError(f"A is {M} x {K} but B is {K2} x {N}")
    for t in (A, B):
        if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("A and B must be contiguous fp16 CUDA tensors")
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A.device)
    elif C.shape != (M, N) or C.dtype != torch.float16 or not C.is_contiguous():
        raise ValueError("C must be a contiguous fp16 M x N tensor")
    s = stream if stream is not None else torch.cuda.current_stream(A.device)
    with torch.cuda.device(A.device):
        check(gemm_ptr(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, s.cuda_stream, variant))
    return C


def gemm_tn(A, Bt, C=None, stream=None):
    """C (fp16, M x N) = A Bt^T for fp16 CUDA tensors, Bt being N x K row-major (a linear layer's weight layout)."""
    import torch

    M, K = A.shape
    N, K2 = Bt.shape
    if K2 != K:
        raise ValueError(f"A is {M} x {K} but Bt is {N} x {K2}")
    for t in (A, Bt):
        if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("A and Bt must be contiguous fp16 CUDA tensors")
    if C is None:
        C = torch.empty((M, N), dtype=torch.float16, device=A.device)
    elif C.shape != (M, N) or C.dtype != torch.float16 or not C.is_contiguous():
        raise ValueError("C must be a contiguous fp16 M x N tensor")
    s = stream if stream is not None else torch.cuda.current_stream(A.device)
    with torch.cuda.device(A.device):
        check(lib().bw_gemm_f16_tn(A.data_ptr(), Bt.data_ptr(), C.data_ptr(), M, N, K, s.cuda_stream))
    return C


def gemm_f32out(A, B, C=None, stream=None):
    """C (fp32, M x N) = A B for fp16 CUDA tensors: the partial sums of a row-parallel layer."""
    import torch

    M, K = A.shape
    K2, N = B.shape
    if K2 != K:
        raise ValueError(f"A is {M} x {K} but B is {K2} x {N}")
    for t in (A, B):
        if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("A and B must be contiguous fp16 CUDA tensors")
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    elif C.shape != (M, N) or C.dtype != torch.float32 or not C.is_contiguous():
        raise ValueError("C must be a contiguous fp32 M x N tensor")
    s = stream if stream is not None else torch.cuda.current_stream(A.device)
    with torch.cuda.device(A.device):
        check(lib().bw_gemm_f16_f32out(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, s.cuda_stream))
    return C


def gemm_swiglu(A, B, C=None, stream=None):
    """C (M x N/2, fp16) = silu(A B_gate) * (A B_up), B's 256-column groups being 128 gate then 128 up columns."""
    import torch

    M, K = A.shape
    K2, N = B.shape
    if K2 != K:
        raise ValueError(f"A is {M} x {K} but B is {K2} x {N}")
    for t in (A, B):
        if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
            raise ValueError("A and B must be contiguous fp16 CUDA tensors")
    if C is None:
        C = torch.empty((M, N // 2), dtype=torch.float16, device=A.device)
    elif C.shape != (M, N // 2) or C.dtype != torch.float16 or not C.is_contiguous():
        raise ValueError("C must be a contiguous fp16 M x N/2 tensor")
    s = stream if stream is not None else torch.cuda.current_stream(A.device)
    with torch.cuda.device(A.device):
        check(lib().bw_gemm_f16_swiglu(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K, s.cuda_stream))
    return C


def status():
    """The device status word of the current device (after a synchronisation): (code, site, block, segment)."""
    code = ctypes.c_int()
    site, block, seg = ctypes.c_uint(), ctypes.c_uint(), ctypes.c_uint()
    check(lib().bw_gemm_status(ctypes.byref(code), ctypes.byref(site), ctypes.byref(block), ctypes.byref(seg)))
    return code.value, site.value, block.value, seg.value


def clear_status():
    check(lib().bw_gemm_clear_status())


def dirty():
    return lib().bw_gemm_dirty()


def set_wait_limit_ns(ns):
    return lib().bw_gemm_set_wait_limit_ns(ns)


def wait_selftest(limit_ns=0, stream=None):
    """Runs the bounded-wait check (a wait on a barrier that nothing arrives on) and returns the C status: 3
    (BW_ERR_TIMEOUT) is the expected outcome; the status word then holds the selftest site."""
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return lib().bw_wait_selftest(limit_ns, s.cuda_stream)


RS_HANDLE_BYTES = 64


class ReduceScatterGemm:
    """The fused reduce-scatter of a row-parallel layer on this rank (bw_rs_* of bwgemm.h): for fp16 A_r (M x K) and
    B_r (K x N), C_r = this rank's rows [r M/world, (r+1) M/world) of sum_r A_r B_r in fp16, one kernel per rank that
    pushes the partial tiles of the other ranks' rows into their memory and sums its own rows' partials in rank order.

    Every rank of `group` constructs it with the same M and N (its receive region's CUDA IPC handle is exchanged with
    all_gather_object, then every rank opens the others' and a barrier follows), and calls it with the same shapes in
    the same order.  Capturable in a CUDA graph (every rank then replays the same graphs).  After a BW_ERR_TIMEOUT
    (another rank never came), close it and make a new one."""

    def __init__(self, M, N, group=None):
        import torch.distributed as dist

        L = lib()
        self.M, self.N = M, N
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self._ctx = ctypes.c_void_p()
        check(L.bw_rs_create(M, N, self.world, self.rank, ctypes.byref(self._ctx)))
        try:
            h = ctypes.create_string_buffer(RS_HANDLE_BYTES)
            check(L.bw_rs_handle(self._ctx, h))
            handles = [None] * self.world
            dist.all_gather_object(handles, h.raw, group=group)
            check(L.bw_rs_connect(self._ctx, b"".join(handles)))
            dist.barrier(group=group)
        except Exception:
            self.close()
            raise

    def region_bytes(self):
        return lib().bw_rs_region_bytes(self._ctx)

    def __call__(self, A, B, C=None, stream=None):
        import torch

        M, K = A.shape
        K2, N = B.shape
        if (M, N) != (self.M, self.N) or K2 != K:
            raise ValueError(f"A {tuple(A.shape)} and B {tuple(B.shape)} do not make the context's {self.M} x {self.N}")
        for t in (A, B):
            if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("A and B must be contiguous fp16 CUDA tensors")
        rows = M // self.world
        if C is None:
            C = torch.empty((rows, N), dtype=torch.float16, device=A.device)
        elif C.shape != (rows, N) or C.dtype != torch.float16 or not C.is_contiguous():
            raise ValueError(f"C must be a contiguous fp16 {rows} x {N} tensor")
        s = stream if stream is not None else torch.cuda.current_stream(A.device)
        with torch.cuda.device(A.device):
            check(lib().bw_gemm_f16_rs(self._ctx, A.data_ptr(), B.data_ptr(), C.data_ptr(), K, s.cuda_stream))
        return C

    def close(self):
        if self._ctx:
            lib().bw_rs_destroy(self._ctx)
            self._ctx = ctypes.c_void_p()
