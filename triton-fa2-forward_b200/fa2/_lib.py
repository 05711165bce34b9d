"""ctypes binding of the C ABI in include/fa2_sm100.h (libfa2_sm100.so, built in-tree).

This is the whole host<->native boundary: plain pointers, sizes and strides go in, a
status code comes out. The library is required; there is no CPU or library fallback.
"""

import ctypes
import os

LIB_NAME = "libfa2_sm100.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

ABI_VERSION = 5

FA2_DTYPE_FP16 = 0
FA2_DTYPE_BF16 = 1

FA2_CAUSAL_TOP_LEFT = 0
FA2_CAUSAL_BOTTOM_RIGHT = 1

FA2_OK = 0
FA2_ERR_NULL = 1
FA2_ERR_SHAPE = 2
FA2_ERR_DTYPE = 3
FA2_ERR_HEAD_DIM = 4
FA2_ERR_GQA = 5
FA2_ERR_PACK = 6
FA2_ERR_SCALE = 7
FA2_ERR_LAYOUT = 8
FA2_ERR_TMA_ENCODE = 9
FA2_ERR_LAUNCH = 10
FA2_ERR_DEVICE = 11
FA2_ERR_TIMEOUT = 12
FA2_ERR_WORKSPACE = 13
FA2_ERR_SCRATCH_LIMIT = 14
NOALLOC_SCRATCH_BYTES = 32 << 20

# Every symbol the header declares (the ABI test checks the library exports all of them).
EXPORTED = (
    "fa2_fwd_sm100_check",
    "fa2_fwd_sm100",
    "fa2_fwd_sm100_config",
    "fa2_fwd_sm100_workspace_bytes",
    "fa2_fwd_sm100_noalloc",
    "fa2_sm100_strerror",
    "fa2_sm100_abi_version",
    "fa2_sm100_params_size",
)


class Fa2FwdParams(ctypes.Structure):
    """Mirror of `Fa2FwdParams` (include/fa2_sm100.h)."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("o", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 4),
        ("k_stride", ctypes.c_int64 * 4),
        ("v_stride", ctypes.c_int64 * 4),
        ("o_stride", ctypes.c_int64 * 4),
        ("batch", ctypes.c_int32),
        ("heads_q", ctypes.c_int32),
        ("heads_kv", ctypes.c_int32),
        ("seqlen_q", ctypes.c_int32),
        ("seqlen_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("causal", ctypes.c_int32),
        ("pack_gqa", ctypes.c_int32),
        ("qk_scale", ctypes.c_float),
        ("err_flag", ctypes.c_void_p),
        ("timeout_cycles", ctypes.c_int64),
        ("gate", ctypes.c_void_p),
        ("num_splits", ctypes.c_int32),
        ("causal_align", ctypes.c_int32),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_int64),
        ("cu_seqlens_q", ctypes.c_void_p),
        ("cu_seqlens_kv", ctypes.c_void_p),
        ("total_q", ctypes.c_int32),
        ("total_kv", ctypes.c_int32),
        ("block_table", ctypes.c_void_p),
        ("seqlens_kv", ctypes.c_void_p),
        ("block_table_stride", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("reserved1", ctypes.c_int32),
    ]


class Fa2Error(RuntimeError):
    """A non-zero Fa2Status returned by the native library."""

    def __init__(self, status, text):
        super().__init__(f"fa2_sm100 status {status}: {text}")
        self.status = status


_lib = None


def lib():
    """Load (once) and return the native library, checking its ABI version and struct size."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python triton-fa2-forward_b200/build.py` "
            "(there is no non-CUDA implementation of fa2.kernel.attention)"
        )
    L = ctypes.CDLL(LIB_PATH)
    L.fa2_fwd_sm100_check.argtypes = [ctypes.POINTER(Fa2FwdParams)]
    L.fa2_fwd_sm100_check.restype = ctypes.c_int
    L.fa2_fwd_sm100.argtypes = [ctypes.POINTER(Fa2FwdParams), ctypes.c_void_p]
    L.fa2_fwd_sm100.restype = ctypes.c_int
    i32p = ctypes.POINTER(ctypes.c_int32)
    L.fa2_fwd_sm100_config.argtypes = [ctypes.c_int32, i32p, i32p, i32p, i32p, i32p]
    L.fa2_fwd_sm100_config.restype = ctypes.c_int
    L.fa2_sm100_strerror.argtypes = [ctypes.c_int]
    L.fa2_sm100_strerror.restype = ctypes.c_char_p
    L.fa2_sm100_abi_version.argtypes = []
    L.fa2_sm100_abi_version.restype = ctypes.c_int
    L.fa2_fwd_sm100_noalloc.argtypes = [ctypes.POINTER(Fa2FwdParams), ctypes.c_void_p]
    L.fa2_fwd_sm100_noalloc.restype = ctypes.c_int
    L.fa2_fwd_sm100_workspace_bytes.argtypes = [ctypes.POINTER(Fa2FwdParams)]
    L.fa2_fwd_sm100_workspace_bytes.restype = ctypes.c_int64
    L.fa2_sm100_params_size.argtypes = []
    L.fa2_sm100_params_size.restype = ctypes.c_int64
    if L.fa2_sm100_abi_version() != ABI_VERSION:
        raise ImportError(f"{LIB_PATH}: ABI version {L.fa2_sm100_abi_version()} != {ABI_VERSION}")
    if L.fa2_sm100_params_size() != ctypes.sizeof(Fa2FwdParams):
        raise ImportError(
            f"{LIB_PATH}: sizeof(Fa2FwdParams) {L.fa2_sm100_params_size()} != "
            f"ctypes mirror {ctypes.sizeof(Fa2FwdParams)}"
        )
    _lib = L
    return L


def strerror(status):
    return lib().fa2_sm100_strerror(int(status)).decode()


def config(head_dim):
    """(block_m, block_n, threads, stages, smem_bytes) of the compiled kernel for head_dim."""
    vals = [ctypes.c_int32() for _ in range(5)]
    rc = lib().fa2_fwd_sm100_config(int(head_dim), *[ctypes.byref(x) for x in vals])
    if rc != FA2_OK:
        raise Fa2Error(rc, strerror(rc))
    return tuple(int(x.value) for x in vals)


def make_params(q_ptr, k_ptr, v_ptr, o_ptr, q_stride, k_stride, v_stride, o_stride,
                batch, heads_q, heads_kv, seqlen_q, seqlen_kv, head_dim, dtype, causal,
                pack_gqa, qk_scale, err_flag=0, timeout_cycles=0, gate=0, num_splits=1,
                workspace=0, workspace_bytes=0, causal_align=FA2_CAUSAL_TOP_LEFT,
                cu_seqlens_q=0, cu_seqlens_kv=0, total_q=0, total_kv=0, block_table=0, seqlens_kv=0,
                block_table_stride=0, page_size=0, num_pages=0):
    p = Fa2FwdParams()
    p.q, p.k, p.v, p.o = q_ptr, k_ptr, v_ptr, o_ptr
    p.q_stride[:] = list(q_stride)
    p.k_stride[:] = list(k_stride)
    p.v_stride[:] = list(v_stride)
    p.o_stride[:] = list(o_stride)
    p.batch, p.heads_q, p.heads_kv = batch, heads_q, heads_kv
    p.seqlen_q, p.seqlen_kv, p.head_dim = seqlen_q, seqlen_kv, head_dim
    p.dtype, p.causal, p.pack_gqa = dtype, int(bool(causal)), int(bool(pack_gqa))
    p.qk_scale = float(qk_scale)
    p.err_flag = err_flag or None
    p.timeout_cycles = int(timeout_cycles)
    p.gate = gate or None
    p.num_splits = int(num_splits)
    p.causal_align = int(causal_align)
    p.workspace = workspace or None
    p.workspace_bytes = int(workspace_bytes)
    p.cu_seqlens_q = cu_seqlens_q or None
    p.cu_seqlens_kv = cu_seqlens_kv or None
    p.total_q, p.total_kv = int(total_q), int(total_kv)
    p.block_table = block_table or None
    p.seqlens_kv = seqlens_kv or None
    p.block_table_stride, p.page_size, p.num_pages = int(block_table_stride), int(page_size), int(num_pages)
    return p


def workspace_bytes(params):
    return int(lib().fa2_fwd_sm100_workspace_bytes(ctypes.byref(params)))


def check(params):
    return lib().fa2_fwd_sm100_check(ctypes.byref(params))


def launch(params, stream_handle):
    return lib().fa2_fwd_sm100(ctypes.byref(params), ctypes.c_void_p(stream_handle or None))
