"""ctypes binding of the C ABI in include/trs.h (libtrs_b200.so).

This is the Python-side caller of the library: tests and the benchmark go
through exactly the entry points a Rust `-sys` crate would bind.  Loading
fails loudly when the library has not been built; there is no fallback.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_double, c_int32, c_int64, c_size_t, c_uint8, c_uint64, c_void_p
from pathlib import Path

MAX_DIMS = 8
LIB_PATH = Path(__file__).resolve().with_name("libtrs_b200.so")

# trs_dtype
F32, F64, I32, I64 = 0, 1, 2, 3
DTYPE_SIZE = {F32: 4, F64: 8, I32: 4, I64: 8}

# trs_status
OK, NONE = 0, 1
ERR_SHAPE, ERR_AXIS, ERR_EMPTY_AXIS, ERR_VIEW, ERR_DTYPE, ERR_ALIAS = 2, 3, 4, 5, 6, 7
ERR_OOM, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_ARG, ERR_DIV_ZERO, ERR_UNAVAILABLE = 8, 9, 10, 11, 12, 13, 14

# trs_binop
ADD, SUB, MUL, DIV, POW = 0, 1, 2, 3, 4
BINOPS = {"add": ADD, "sub": SUB, "mul": MUL, "div": DIV, "pow": POW}

# trs_unop
UNOPS = {
    "none": 0, "neg": 1, "relu": 2, "sigmoid": 3, "tanh": 4, "elu": 5, "leaky_relu": 6,
    "selu": 7, "exp": 8, "ln": 9, "abs": 10, "sign": 11, "clamp": 12, "add_scalar": 13,
    "sub_scalar": 14, "rsub_scalar": 15, "mul_scalar": 16, "div_scalar": 17,
    "pow_scalar": 18, "rpow_scalar": 19,
}


class View(ctypes.Structure):
    """trs_view: a strided view of a device buffer (element units)."""

    _fields_ = [
        ("data", c_void_p),
        ("storage_len", c_int64),
        ("dtype", c_int32),
        ("ndim", c_int32),
        ("shape", c_int64 * MAX_DIMS),
        ("strides", c_int64 * MAX_DIMS),
        ("offset", c_int64),
    ]


class Scalar(ctypes.Structure):
    _fields_ = [("f", c_double), ("i", c_int64)]


class Program(ctypes.Structure):
    _fields_ = [
        ("n_in", c_int32),
        ("op1", c_int32),
        ("op2", c_int32),
        ("epilogue", c_int32),
        ("p0", Scalar),
        ("p1", Scalar),
    ]


class TrsError(RuntimeError):
    """A non-OK status; `status` is the trs_status, the message is the library's."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status
        self.message = message


_V = POINTER(View)
_SIGNATURES = {
    "trs_abi_version": (c_int32, []),
    "trs_last_error": (c_size_t, [ctypes.c_char_p, c_size_t]),
    "trs_status_string": (ctypes.c_char_p, [c_int32]),
    "trs_launch_count": (c_uint64, []),
    "trs_scratch_alloc_count": (c_uint64, []),
    "trs_async_error": (c_int32, [POINTER(c_int32)]),
    "trs_broadcast_shape": (c_int32, [POINTER(c_int64), c_int32, POINTER(c_int64), c_int32,
                                      POINTER(c_int64), POINTER(c_int32)]),
    "trs_plan_elementwise": (c_int32, [POINTER(Program), _V, _V, POINTER(c_int32), POINTER(c_int32),
                                       POINTER(c_int64), POINTER(c_int64), POINTER(c_int32)]),
    "trs_binary": (c_int32, [c_int32, _V, _V, _V, c_void_p]),
    "trs_unary": (c_int32, [c_int32, _V, POINTER(Scalar), _V, c_void_p]),
    "trs_elementwise": (c_int32, [POINTER(Program), _V, _V, c_void_p]),
    "trs_elementwise_sum": (c_int32, [POINTER(Program), _V, _V, _V, c_void_p]),
    "trs_elementwise_row_sums": (c_int32, [POINTER(Program), _V, _V, _V, _V, c_void_p]),
    "trs_pack": (c_int32, [_V, _V, c_void_p]),
    "trs_sum": (c_int32, [_V, _V, c_void_p]),
    "trs_sum_noalloc": (c_int32, [_V, _V, c_void_p]),
    "trs_sum_axis": (c_int32, [_V, c_int32, c_int32, _V, c_void_p]),
    "trs_mean_axis": (c_int32, [_V, c_int32, c_int32, _V, c_void_p]),
    "trs_max_axis": (c_int32, [_V, c_int32, _V, c_void_p]),
    "trs_argmax_axis": (c_int32, [_V, c_int32, _V, c_void_p]),
    "trs_reduce_broadcast_grad": (c_int32, [_V, POINTER(c_int64), c_int32, _V, c_void_p]),
    "trs_sum_to_shape_fused": (c_int32, [_V, _V, _V, POINTER(c_int64), c_int32, _V, c_void_p]),
    "trs_affine_relu_backward": (c_int32, [_V, _V, _V, _V, _V, _V, c_void_p]),
    "trs_softmax_lastdim": (c_int32, [_V, _V, c_void_p]),
    "trs_layer_norm_lastdim": (c_int32, [_V, _V, _V, c_double, _V, c_void_p]),
    "trs_sgd_step": (c_int32, [_V, _V, c_double, c_void_p]),
    "trs_rmsprop_step": (c_int32, [_V, _V, _V, c_double, c_double, c_double, c_void_p]),
    "trs_adam_step": (c_int32, [_V, _V, _V, _V, c_double, c_double, c_double, c_double, c_int64, c_void_p]),
    "trs_max_pool2d": (c_int32, [_V, c_int64, c_int64, c_int64, c_int64, _V, c_void_p]),
    "trs_avg_pool2d": (c_int32, [_V, c_int64, c_int64, c_int64, c_int64, _V, c_void_p]),
    "trs_max_pool2d_backward": (c_int32, [_V, _V, c_int64, c_int64, c_int64, c_int64, c_int32, _V, c_void_p]),
    "trs_matmul": (c_int32, [_V, _V, _V, c_void_p]),
    "trs_matmul_tf32x3": (c_int32, [_V, _V, _V, c_void_p]),
    "trs_unfold_2d": (c_int32, [_V, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _V, c_void_p]),
    "trs_fold_2d": (c_int32, [_V, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, _V, c_void_p]),
    "trs_fill_uniform": (c_int32, [_V, c_uint64, c_uint64, c_double, c_double, c_void_p]),
    "trs_fill_normal": (c_int32, [_V, c_uint64, c_uint64, c_void_p]),
    "trs_set_device": (c_int32, [c_int32]),
    "trs_malloc": (c_int32, [POINTER(c_void_p), c_size_t]),
    "trs_free": (c_int32, [c_void_p]),
    "trs_memcpy_htod": (c_int32, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "trs_memcpy_dtoh": (c_int32, [c_void_p, c_void_p, c_size_t, c_void_p]),
    "trs_stream_synchronize": (c_int32, [c_void_p]),
    "trs_comm_unique_id": (c_int32, [POINTER(c_uint8)]),
    "trs_comm_init_rank": (c_int32, [POINTER(c_uint8), c_int32, c_int32, c_int32, POINTER(c_void_p)]),
    "trs_comm_destroy": (c_int32, [c_void_p]),
    "trs_comm_peer_exchange": (c_int32, [c_void_p, POINTER(c_int32)]),
    "trs_comm_abort": (c_int32, [c_void_p]),
    "trs_sharded_sum": (c_int32, [c_void_p, _V, _V, c_void_p]),
    "trs_sharded_elementwise_sum": (c_int32, [c_void_p, POINTER(Program), _V, _V, _V, c_void_p]),
    "trs_sharded_sum_axis0": (c_int32, [c_void_p, _V, _V, c_void_p]),
    "trs_sharded_max_axis0": (c_int32, [c_void_p, _V, _V, c_void_p]),
    "trs_sharded_argmax_axis0": (c_int32, [c_void_p, _V, _V, c_void_p]),
}

_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads libtrs_b200.so once and declares every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is not built: run `python -m tensorrs_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def exported_names() -> list[str]:
    return list(_SIGNATURES)


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(4096)
    lib.trs_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int) -> int:
    """Raises TrsError for a failing status; returns OK or NONE."""
    if status in (OK, NONE):
        return status
    raise TrsError(status, last_error())


def make_view(ptr: int, dtype: int, shape, strides=None, offset: int = 0,
              storage_len: int | None = None) -> View:
    """A trs_view; strides default to row-major, storage_len to the extent the view reaches."""
    shape = [int(s) for s in shape]
    if strides is None:
        strides, step = [0] * len(shape), 1
        for i in range(len(shape) - 1, -1, -1):
            strides[i] = step
            step *= shape[i]
    strides = [int(s) for s in strides]
    if storage_len is None:
        hi = offset
        for s, st in zip(shape, strides):
            if s > 0 and st > 0:
                hi += (s - 1) * st
        storage_len = hi + 1
    v = View()
    v.data = ptr
    v.storage_len = storage_len
    v.dtype = dtype
    v.ndim = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        v.shape[i] = s
        v.strides[i] = st
    v.offset = offset
    return v


def program(n_in: int, op1: int = ADD, op2: int = ADD, epilogue: str | int = "none",
            p0: float | int = 0.0, p1: float | int = 0.0) -> Program:
    pr = Program()
    pr.n_in = n_in
    pr.op1 = op1
    pr.op2 = op2
    pr.epilogue = UNOPS[epilogue] if isinstance(epilogue, str) else epilogue
    pr.p0 = scalar(p0)
    pr.p1 = scalar(p1)
    return pr


def scalar(v: float | int) -> Scalar:
    s = Scalar()
    s.f = float(v)
    s.i = int(v) if float(v).is_integer() else 0
    return s


def views_array(views) -> ctypes.Array:
    arr = (View * len(views))()
    for i, v in enumerate(views):
        arr[i] = v
    return arr
