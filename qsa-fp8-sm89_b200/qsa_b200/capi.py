"""ctypes bindings of the C ABI (include/qsa_b200.h).

This is the binding a Python maintainer of the reference would add to call
``libqsa_b200.so`` the way the reference's CUDA library is meant to be called
(``launch_qsa_cuda``, sm89_cuda.cu:232-253, "Shared library (for Python /
PyTorch ctypes)", sm89_cuda.cu:21-22). Pointers are raw device addresses
(``tensor.data_ptr()``); streams are ``torch.cuda.Stream.cuda_stream``
integers.
"""

from __future__ import annotations

import ctypes
import math
from ctypes import c_float, c_int, c_int32, c_int64, c_size_t, c_void_p

from ._lib import load_clib

OK = 0
ERR_NULL_POINTER = -1
ERR_BAD_SHAPE = -2
ERR_UNSUPPORTED = -3
ERR_MISALIGNED = -4
ERR_WORKSPACE = -5
ERR_DEVICE = -6
ERR_LAUNCH = -7
ERR_KERNEL = -8
ERR_TOO_LARGE = -9
ERR_BAD_VALUE = -10

# Fixed split scratch of qsa_b200_decode_noalloc (QSA_B200_NOALLOC_SCRATCH_BYTES).
NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024

KERNEL_AUTO = 0
KERNEL_TC = 1
KERNEL_SIMT = 2

DTYPE_BF16 = 0
DTYPE_F16 = 1
DTYPE_F32 = 2

LOG2E = 1.4426950408889634

# Names of every function include/qsa_b200.h declares.
EXPORTED = (
    "qsa_b200_workspace_bytes",
    "qsa_b200_decode",
    "qsa_b200_slots",
    "launch_qsa_cuda",
    "qsa_b200_last_status",
    "qsa_b200_device_error",
    "qsa_b200_status_string",
    "qsa_b200_abi_version",
    "qsa_b200_decode_noalloc",
    "qsa_b200_cache_write",
    "qsa_b200_topk_select",
)
# test hook (include/qsa_b200_testing.h), not part of the decode interface
TESTING_EXPORTED = ("qsa_b200_testing_set_wait_limit_ns",)


class DecodeArgs(ctypes.Structure):
    """Mirror of ``qsa_b200_decode_args``."""

    _fields_ = [
        ("q", c_void_p),
        ("k_cache", c_void_p),
        ("v_cache", c_void_p),
        ("indices", c_void_p),
        ("counts", c_void_p),
        ("btable", c_void_p),
        ("t2r", c_void_p),
        ("gate", c_void_p),
        ("out", c_void_p),
        ("softmax_scale", c_float),
        ("k_scale", c_float),
        ("v_scale", c_float),
        ("rows", c_int32),
        ("num_q_heads", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("page_size", c_int32),
        ("pages_per_req", c_int32),
        ("num_reqs", c_int32),
        ("num_pages", c_int64),
        ("topk", c_int32),
        ("indices_stride", c_int64),
        ("count_column", c_int32),
        ("btable_stride", c_int64),
        ("kernel", c_int32),
    ]


class CacheWriteArgs(ctypes.Structure):
    """Mirror of ``qsa_b200_cache_write_args``."""

    _fields_ = [
        ("k", c_void_p),
        ("v", c_void_p),
        ("slots", c_void_p),
        ("k_cache", c_void_p),
        ("v_cache", c_void_p),
        ("k_scale", c_float),
        ("v_scale", c_float),
        ("tokens", c_int32),
        ("num_kv_heads", c_int32),
        ("head_dim", c_int32),
        ("page_size", c_int32),
        ("num_pages", c_int64),
        ("token_stride", c_int64),
        ("input_dtype", c_int32),
    ]


class TopkArgs(ctypes.Structure):
    """Mirror of ``qsa_b200_topk_args``."""

    _fields_ = [
        ("scores", c_void_p),
        ("lengths", c_void_p),
        ("out", c_void_p),
        ("rows", c_int32),
        ("ctx", c_int32),
        ("k", c_int32),
        ("score_stride", c_int64),
        ("out_stride", c_int64),
    ]


_configured = False


def lib() -> ctypes.CDLL:
    """The loaded library with argument / return types declared."""
    global _configured
    L = load_clib()
    if not _configured:
        P = ctypes.POINTER(DecodeArgs)
        L.qsa_b200_workspace_bytes.argtypes = [P]
        L.qsa_b200_workspace_bytes.restype = c_int64
        L.qsa_b200_decode.argtypes = [P, c_void_p, c_size_t, c_void_p]
        L.qsa_b200_decode.restype = c_int
        L.qsa_b200_slots.argtypes = [P, c_void_p, c_void_p]
        L.qsa_b200_slots.restype = c_int
        L.launch_qsa_cuda.argtypes = [c_void_p] * 8 + [c_float, c_float] + [c_int32] * 9 + [c_void_p]
        L.launch_qsa_cuda.restype = None
        L.qsa_b200_last_status.argtypes = []
        L.qsa_b200_last_status.restype = c_int
        L.qsa_b200_device_error.argtypes = [c_int]
        L.qsa_b200_device_error.restype = c_int
        L.qsa_b200_status_string.argtypes = [c_int]
        L.qsa_b200_status_string.restype = ctypes.c_char_p
        L.qsa_b200_abi_version.argtypes = []
        L.qsa_b200_abi_version.restype = c_int
        L.qsa_b200_decode_noalloc.argtypes = [P, c_void_p]
        L.qsa_b200_decode_noalloc.restype = c_int
        L.qsa_b200_cache_write.argtypes = [ctypes.POINTER(CacheWriteArgs), c_void_p]
        L.qsa_b200_cache_write.restype = c_int
        L.qsa_b200_topk_select.argtypes = [ctypes.POINTER(TopkArgs), c_void_p]
        L.qsa_b200_topk_select.restype = c_int
        L.qsa_b200_testing_set_wait_limit_ns.argtypes = [ctypes.c_uint64]
        L.qsa_b200_testing_set_wait_limit_ns.restype = ctypes.c_uint64
        _configured = True
    return L


def testing_set_wait_limit_ns(ns: int) -> int:
    """Test hook: the limit of the tensor-core kernel's pipeline waits for
    the launches that follow (0 = the 1 s default); returns the previous one."""
    return int(lib().qsa_b200_testing_set_wait_limit_ns(int(ns)))


def check_device_error(clear: bool = True) -> None:
    """Raises RuntimeError (QSA_B200_ERR_KERNEL's text and the error word)
    when a kernel has reported a device-side failure, such as a bounded wait
    that ran out; clears the word first when ``clear``. Synchronous."""
    word = device_error(clear=clear)
    if word < 0:
        raise RuntimeError(f"reading the device error word failed: {status_string(word)}")
    if word != 0:
        raise RuntimeError(f"{status_string(ERR_KERNEL)} (device error word {word})")


def status_string(status: int) -> str:
    return lib().qsa_b200_status_string(int(status)).decode()


def _ptr(t):
    return None if t is None else c_void_p(t.data_ptr())


def make_args(q, k, v, btable, t2r, indices, gate, out, *, counts=None, softmax_scale=None,
              k_scale=1.0, v_scale=1.0, topk=None, count_column=False, kernel=KERNEL_AUTO) -> DecodeArgs:
    """Fills ``qsa_b200_decode_args`` from torch tensors (no checks: the C
    side validates). ``q``/``gate``/``out`` may be None for ``slots``."""
    a = DecodeArgs()
    a.q, a.k_cache, a.v_cache = _ptr(q), _ptr(k), _ptr(v)
    a.indices, a.counts, a.btable, a.t2r = _ptr(indices), _ptr(counts), _ptr(btable), _ptr(t2r)
    a.gate, a.out = _ptr(gate), _ptr(out)
    ref = q if q is not None else None
    hd = ref.shape[2] if ref is not None else 128
    a.softmax_scale = float(hd ** -0.5 if softmax_scale is None else softmax_scale)
    a.k_scale = float(k_scale)
    a.v_scale = float(v_scale)
    a.rows = int(indices.shape[0])
    a.num_q_heads = int(q.shape[1]) if q is not None else 1
    a.num_kv_heads = int(k.shape[2]) if k is not None else 1
    a.head_dim = int(hd)
    a.page_size = int(k.shape[1]) if k is not None else 1
    a.pages_per_req = int(btable.shape[1])
    a.num_reqs = int(btable.shape[0])
    a.num_pages = int(k.shape[0]) if k is not None else 1
    a.topk = int(indices.shape[1] - (1 if count_column else 0) if topk is None else topk)
    a.indices_stride = int(indices.stride(0))
    a.count_column = 1 if count_column else 0
    a.btable_stride = int(btable.stride(0))
    a.kernel = int(kernel)
    return a


def workspace_bytes(args: DecodeArgs) -> int:
    return int(lib().qsa_b200_workspace_bytes(ctypes.byref(args)))


def decode(args: DecodeArgs, workspace=None, workspace_bytes_: int = 0, stream: int = 0) -> int:
    """Calls ``qsa_b200_decode``; returns its status."""
    ws = None if workspace is None else c_void_p(workspace.data_ptr())
    return int(lib().qsa_b200_decode(ctypes.byref(args), ws, c_size_t(workspace_bytes_), c_void_p(stream)))


def decode_noalloc(args: DecodeArgs, stream: int = 0) -> int:
    """Calls ``qsa_b200_decode_noalloc`` (split scratch from the library's
    fixed device array, no workspace); returns its status."""
    return int(lib().qsa_b200_decode_noalloc(ctypes.byref(args), c_void_p(stream)))


def slots(args: DecodeArgs, out, stream: int = 0) -> int:
    return int(lib().qsa_b200_slots(ctypes.byref(args), c_void_p(out.data_ptr()), c_void_p(stream)))


def launch_qsa_cuda(q, k, v, indices, btable, t2r, gate, out, k_scale, v_scale, stream: int = 0) -> int:
    """Calls the reference-compatible launcher exactly as the reference's own
    ``main`` does (sm89_cuda.cu:369-385): log2-domain softmax scale, indices
    with the count column, rows == nreqs. Returns qsa_b200_last_status()."""
    L = lib()
    hd = q.shape[2]
    ss = (1.0 / math.sqrt(hd)) * k_scale * LOG2E
    nreqs, max_pages = btable.shape
    L.launch_qsa_cuda(
        _ptr(q), _ptr(k), _ptr(v), _ptr(indices), _ptr(btable), _ptr(t2r), _ptr(gate), _ptr(out),
        c_float(ss), c_float(v_scale), c_int32(k.shape[0]), c_int32(nreqs), c_int32(q.shape[1]),
        c_int32(k.shape[2]), c_int32(indices.shape[1] - 1), c_int32(k.shape[1]), c_int32(max_pages),
        c_int32(hd), c_int32(q.shape[1] // k.shape[2]), c_void_p(stream))
    return int(L.qsa_b200_last_status())


_DTYPES = {"torch.bfloat16": DTYPE_BF16, "torch.float16": DTYPE_F16, "torch.float32": DTYPE_F32}


def make_cache_write_args(k_new, v_new, slots, k_cache, v_cache, k_scale=1.0, v_scale=1.0) -> CacheWriteArgs:
    """Fills ``qsa_b200_cache_write_args`` from torch tensors: new keys and
    values ``[tokens, Hkv, 128]`` (bf16, fp16 or fp32, unit stride inside a
    token), int64 ``slots[tokens]``, caches ``[num_pages, P, Hkv, 128]``. No
    checks: the C side validates."""
    a = CacheWriteArgs()
    a.k, a.v, a.slots = _ptr(k_new), _ptr(v_new), _ptr(slots)
    a.k_cache, a.v_cache = _ptr(k_cache), _ptr(v_cache)
    a.k_scale, a.v_scale = float(k_scale), float(v_scale)
    a.tokens = int(k_new.shape[0])
    a.num_kv_heads = int(k_cache.shape[2])
    a.head_dim = int(k_cache.shape[3])
    a.page_size = int(k_cache.shape[1])
    a.num_pages = int(k_cache.shape[0])
    a.token_stride = int(k_new.stride(0))
    a.input_dtype = _DTYPES.get(str(k_new.dtype), -1)
    return a


def cache_write(args: CacheWriteArgs, stream: int = 0) -> int:
    """Calls ``qsa_b200_cache_write``; returns its status."""
    return int(lib().qsa_b200_cache_write(ctypes.byref(args), c_void_p(stream)))


def make_topk_args(scores, k, out, lengths=None) -> TopkArgs:
    """Fills ``qsa_b200_topk_args`` from torch tensors: fp32 ``scores[rows,
    ctx]`` and int32 ``out[rows, k]`` with unit inner stride, optional int32
    ``lengths[rows]``. No data is touched."""
    a = TopkArgs()
    a.scores = c_void_p(scores.data_ptr())
    a.lengths = c_void_p(lengths.data_ptr()) if lengths is not None else None
    a.out = c_void_p(out.data_ptr())
    a.rows, a.ctx, a.k = scores.shape[0], scores.shape[1], int(k)
    a.score_stride = scores.stride(0)
    a.out_stride = out.stride(0)
    return a


def topk_select(args: TopkArgs, stream: int = 0) -> int:
    """Calls ``qsa_b200_topk_select``; returns its status."""
    return int(lib().qsa_b200_topk_select(ctypes.byref(args), c_void_p(stream)))


def device_error(clear: bool = False) -> int:
    return int(lib().qsa_b200_device_error(1 if clear else 0))
