"""ctypes binding of the CPU oracle (oracle/oracle.cpp).

TEST INFRASTRUCTURE ONLY: the checker that tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg compare against.  The shipped library never loads
it.  `build()` compiles it with oracle/Makefile into oracle/_build/.

Every function takes host numpy arrays and describes views of them the same
way the C ABI does (storage + shape + signed strides + offset, in elements).
"""
from __future__ import annotations

import ctypes
import subprocess
from ctypes import POINTER, c_double, c_int, c_int32, c_int64, c_uint64, c_void_p
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle.so"
MAX_DIMS = 8

NP_TO_DT = {np.dtype(np.float32): 0, np.dtype(np.float64): 1, np.dtype(np.int32): 2, np.dtype(np.int64): 3}
DT_TO_NP = {v: k for k, v in NP_TO_DT.items()}
BINOPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "pow": 4}
UNOPS = {
    "none": 0, "neg": 1, "relu": 2, "sigmoid": 3, "tanh": 4, "elu": 5, "leaky_relu": 6,
    "selu": 7, "exp": 8, "ln": 9, "abs": 10, "sign": 11, "clamp": 12, "add_scalar": 13,
    "sub_scalar": 14, "rsub_scalar": 15, "mul_scalar": 16, "div_scalar": 17,
    "pow_scalar": 18, "rpow_scalar": 19,
}
STATUS_NONE = 1


class OView(ctypes.Structure):
    _fields_ = [
        ("data", c_void_p), ("storage_len", c_int64), ("dtype", c_int32), ("ndim", c_int32),
        ("shape", c_int64 * MAX_DIMS), ("strides", c_int64 * MAX_DIMS), ("offset", c_int64),
    ]


class OracleError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{message} (status {status})")
        self.status = status
        self.message = message


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


_lib = None


def load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        V = POINTER(OView)
        I64P = POINTER(c_int64)
        sig = {
            "orc_last_message": (ctypes.c_char_p, []),
            "orc_set_threads": (None, [c_int]),
            "orc_get_max_threads": (c_int, []),
            "orc_storage_indices": (c_int, [V, I64P]),
            "orc_broadcast_shape": (c_int, [I64P, c_int, I64P, c_int, I64P, POINTER(c_int32)]),
            "orc_binary": (c_int, [c_int, V, V, c_void_p, I64P, POINTER(c_int32)]),
            "orc_unary": (c_int, [c_int, V, c_double, c_int64, c_double, c_int64, c_void_p]),
            "orc_program": (c_int, [c_int, c_int, c_int, c_int, c_double, c_int64, c_double, c_int64, V,
                                    c_void_p, I64P, POINTER(c_int32)]),
            "orc_sum": (c_int, [V, c_void_p]),
            "orc_sum_axis": (c_int, [V, c_int, c_int, c_void_p, I64P, POINTER(c_int32)]),
            "orc_mean_axis": (c_int, [V, c_int, c_int, c_void_p, I64P, POINTER(c_int32)]),
            "orc_max_axis": (c_int, [V, c_int, c_void_p, I64P]),
            "orc_reduce_broadcast_grad": (c_int, [V, I64P, c_int, c_void_p, I64P, POINTER(c_int32)]),
            "orc_softmax_lastdim": (c_int, [V, c_void_p]),
            "orc_sum_f64": (c_int, [V, POINTER(c_double), POINTER(c_double)]),
            "orc_fill_uniform": (c_int, [c_int, c_void_p, c_int64, c_uint64, c_double, c_double]),
            "orc_fill_uniform_at": (c_int, [c_int, c_void_p, c_int64, c_int64, c_uint64, c_double, c_double]),
            "orc_fill_normal": (c_int, [c_int, c_void_p, c_int64, c_uint64]),
            "orc_fill_normal_at": (c_int, [c_int, c_void_p, c_int64, c_int64, c_uint64]),
            "orc_fma_sum_stream": (c_int, [c_int64, c_int64, c_uint64, c_uint64, c_uint64, POINTER(c_double),
                                           POINTER(c_double), POINTER(ctypes.c_float), c_void_p]),
            "orc_opt_step": (c_int, [c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_double,
                                     c_double, c_double, c_double, c_int64]),
            "orc_pool2d": (c_int, [c_int, V, c_int64, c_int64, c_int64, c_int64, c_void_p, I64P]),
            "orc_matmul": (c_int, [V, V, c_void_p, I64P, POINTER(c_int32)]),
            "orc_unfold_2d": (c_int, [V, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p, I64P]),
            "orc_fold_2d": (c_int, [V, I64P, c_int64, c_int64, c_int64, c_int64, c_int64, c_int64, c_void_p]),
            "orc_max_pool2d_backward": (c_int, [V, V, c_int64, c_int64, c_int64, c_int64, c_void_p, c_void_p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class HostView:
    """A view into a contiguous numpy storage array (keeps the array alive)."""

    def __init__(self, storage: np.ndarray, shape, strides=None, offset: int = 0):
        assert storage.flags["C_CONTIGUOUS"]
        self.storage = storage
        self.shape = [int(s) for s in shape]
        if strides is None:
            strides, step = [0] * len(self.shape), 1
            for i in range(len(self.shape) - 1, -1, -1):
                strides[i] = step
                step *= self.shape[i]
        self.strides = [int(s) for s in strides]
        self.offset = int(offset)

    @property
    def dtype(self) -> np.dtype:
        return self.storage.dtype

    def numel(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) if self.shape else 1

    def c(self) -> OView:
        v = OView()
        v.data = self.storage.ctypes.data
        v.storage_len = self.storage.size
        v.dtype = NP_TO_DT[self.storage.dtype]
        v.ndim = len(self.shape)
        for i, (s, st) in enumerate(zip(self.shape, self.strides)):
            v.shape[i] = s
            v.strides[i] = st
        v.offset = self.offset
        return v


def contiguous(a: np.ndarray) -> HostView:
    a = np.ascontiguousarray(a)
    return HostView(a.reshape(-1), a.shape)


def _check(st: int) -> int:
    if st not in (0, STATUS_NONE):
        raise OracleError(st, load().orc_last_message().decode())
    return st


def set_threads(n: int) -> None:
    load().orc_set_threads(n)


def max_threads() -> int:
    return load().orc_get_max_threads()


def _out_buf(dtype, n):
    return np.empty(max(int(n), 1), dtype=dtype)


def binary(op: str, a: HostView, b: HostView) -> np.ndarray:
    lib = load()
    shp = (c_int64 * MAX_DIMS)()
    nd = c_int32()
    _check(lib.orc_broadcast_shape((c_int64 * MAX_DIMS)(*a.shape), len(a.shape), (c_int64 * MAX_DIMS)(*b.shape),
                                   len(b.shape), shp, ctypes.byref(nd)))
    shape = [shp[i] for i in range(nd.value)]
    out = _out_buf(a.dtype, np.prod(shape, dtype=np.int64) if shape else 1)
    _check(lib.orc_binary(BINOPS[op], ctypes.byref(a.c()), ctypes.byref(b.c()), out.ctypes.data, shp,
                          ctypes.byref(nd)))
    return out[: int(np.prod(shape, dtype=np.int64))].reshape(shape)


def unary(op: str, x: HostView, p0=0.0, p1=0.0) -> np.ndarray:
    out = _out_buf(x.dtype, x.numel())
    _check(load().orc_unary(UNOPS[op], ctypes.byref(x.c()), float(p0), int(p0), float(p1), int(p1),
                            out.ctypes.data))
    return out[: x.numel()].reshape(x.shape)


def program(n_in: int, op1: str, op2: str, epi: str, ins: list[HostView], p0=0.0, p1=0.0) -> np.ndarray:
    lib = load()
    arr = (OView * len(ins))(*[v.c() for v in ins])
    shape = list(ins[0].shape)
    for v in ins[1:n_in]:
        shape = list(np.broadcast_shapes(tuple(shape), tuple(v.shape)))
    n = int(np.prod(shape, dtype=np.int64)) if shape else 1
    out = _out_buf(ins[0].dtype, n)
    shp = (c_int64 * MAX_DIMS)()
    nd = c_int32()
    _check(lib.orc_program(n_in, BINOPS[op1], BINOPS[op2], UNOPS[epi], float(p0), int(p0), float(p1), int(p1),
                           arr, out.ctypes.data, shp, ctypes.byref(nd)))
    return out[:n].reshape([shp[i] for i in range(nd.value)])


def sum_all(x: HostView):
    out = np.empty(1, dtype=x.dtype)
    _check(load().orc_sum(ctypes.byref(x.c()), out.ctypes.data))
    return out[0]


def sum_axis(x: HostView, axis: int, keepdim: bool) -> np.ndarray:
    shp = (c_int64 * MAX_DIMS)()
    nd = c_int32()
    n = x.numel() // max(x.shape[axis], 1) if x.shape[axis] else int(np.prod([s for i, s in enumerate(x.shape) if i != axis]))
    out = _out_buf(x.dtype, n)
    _check(load().orc_sum_axis(ctypes.byref(x.c()), axis, int(keepdim), out.ctypes.data, shp, ctypes.byref(nd)))
    shape = [shp[i] for i in range(nd.value)]
    return out[: int(np.prod(shape, dtype=np.int64))].reshape(shape)


def mean_axis(x: HostView, axis: int, keepdim: bool) -> np.ndarray:
    shp = (c_int64 * MAX_DIMS)()
    nd = c_int32()
    n = int(np.prod([s for i, s in enumerate(x.shape) if i != axis], dtype=np.int64))
    out = _out_buf(x.dtype, n)
    _check(load().orc_mean_axis(ctypes.byref(x.c()), axis, int(keepdim), out.ctypes.data, shp, ctypes.byref(nd)))
    shape = [shp[i] for i in range(nd.value)]
    return out[: int(np.prod(shape, dtype=np.int64))].reshape(shape)


def max_argmax_axis(x: HostView, axis: int):
    oshape = [s for i, s in enumerate(x.shape) if i != axis]
    n = int(np.prod(oshape, dtype=np.int64)) if oshape else 1
    vals = _out_buf(x.dtype, n)
    idx = np.empty(max(n, 1), dtype=np.int64)
    _check(load().orc_max_axis(ctypes.byref(x.c()), axis, vals.ctypes.data,
                               idx.ctypes.data_as(POINTER(c_int64))))
    return vals[:n].reshape(oshape), idx[:n].reshape(oshape)


def reduce_broadcast_grad(g: HostView, target: list[int]):
    """Returns the reduced array, or None where the reference returns None."""
    shp = (c_int64 * MAX_DIMS)()
    nd = c_int32()
    n = max(g.numel(), int(np.prod(target, dtype=np.int64)) if target else 1)
    out = _out_buf(g.dtype, n)
    st = _check(load().orc_reduce_broadcast_grad(ctypes.byref(g.c()), (c_int64 * MAX_DIMS)(*target), len(target),
                                                 out.ctypes.data, shp, ctypes.byref(nd)))
    if st == STATUS_NONE:
        return None
    shape = [shp[i] for i in range(nd.value)]
    return out[: int(np.prod(shape, dtype=np.int64))].reshape(shape)


def softmax_lastdim(x: HostView) -> np.ndarray:
    out = _out_buf(x.dtype, x.numel())
    _check(load().orc_softmax_lastdim(ctypes.byref(x.c()), out.ctypes.data))
    return out[: x.numel()].reshape(x.shape)


def opt_step(kind: str, p: np.ndarray, g: np.ndarray, m: np.ndarray | None, v: np.ndarray | None, lr: float,
             b1: float = 0.9, b2: float = 0.999, eps: float = 1e-8, t: int = 1) -> None:
    """One SGD / RMSprop / Adam step in place on contiguous host arrays, as the
    reference's chain of calls computes it (alpha goes in b2 for RMSprop)."""
    k = {"sgd": 0, "rmsprop": 1, "adam": 2}[kind]
    dt = {np.dtype(np.float32): 0, np.dtype(np.float64): 1}[p.dtype]
    for a in (p, g, m, v):
        assert a is None or (a.flags.c_contiguous and a.dtype == p.dtype and a.size == p.size)
    nul = None
    _check(load().orc_opt_step(k, dt, p.ctypes.data, g.ctypes.data, m.ctypes.data if m is not None else nul,
                               v.ctypes.data if v is not None else nul, p.size, lr, b1, b2, eps, t))


def pool2d(kind: str, x: HostView, kernel, stride=None) -> np.ndarray:
    """MaxPool2d / AvgPool2d forward ("max" / "avg") of an [N, C, H, W] view, as
    the reference computes it (reshape, unfold_2d, max_axis or sum_axis / k)."""
    kh, kw = kernel
    sh, sw = stride if stride is not None else kernel
    n_out = 1
    if len(x.shape) == 4 and sh > 0 and sw > 0 and x.shape[2] >= kh >= 0 and x.shape[3] >= kw >= 0:
        N, C, H, W = x.shape
        n_out = N * C * ((H - kh) // sh + 1) * ((W - kw) // sw + 1)
    out = _out_buf(x.dtype, max(n_out, 1))
    shp = (c_int64 * 4)()
    _check(load().orc_pool2d(1 if kind == "max" else 0, ctypes.byref(x.c()), kh, kw, sh, sw, out.ctypes.data, shp))
    shape = [shp[i] for i in range(4)]
    return out[: int(np.prod(shape, dtype=np.int64))].reshape(shape)


def max_pool2d_backward(x: HostView, g: HostView, kernel, stride=None, current: np.ndarray | None = None):
    """The gradient MaxPool2d passes to x (max_axis backward, fold_2d), added to
    `current` (same shape as x) when given."""
    kh, kw = kernel
    sh, sw = stride if stride is not None else kernel
    out = _out_buf(x.dtype, max(x.numel(), 1))
    cur = None
    if current is not None:
        cur = np.ascontiguousarray(current, dtype=x.dtype)
        assert cur.size == x.numel()
    _check(load().orc_max_pool2d_backward(ctypes.byref(x.c()), ctypes.byref(g.c()), kh, kw, sh, sw,
                                          cur.ctypes.data if cur is not None else None, out.ctypes.data))
    return out[: x.numel()].reshape(x.shape)


def matmul(a: HostView, b: HostView) -> np.ndarray:
    """Tensor::matmul (linalg/tensor/base.rs:896-1013)."""
    batch = list(np.broadcast_shapes(tuple(a.shape[:-2]), tuple(b.shape[:-2]))) if len(a.shape) >= 2 and \
        len(b.shape) >= 2 else []
    n = int(np.prod(batch, dtype=np.int64)) * (a.shape[-2] if len(a.shape) >= 2 else 1) * \
        (b.shape[-1] if len(b.shape) >= 2 else 1)
    out = _out_buf(a.dtype, max(n, 1))
    shp = (c_int64 * (MAX_DIMS + 2))()
    nd = c_int32()
    _check(load().orc_matmul(ctypes.byref(a.c()), ctypes.byref(b.c()), out.ctypes.data, shp, ctypes.byref(nd)))
    shape = [shp[i] for i in range(nd.value)]
    return out[: int(np.prod(shape, dtype=np.int64))].reshape(shape)


def unfold_2d(x: HostView, kernel, stride, padding=(0, 0)) -> np.ndarray:
    """Tensor::unfold_2d (linalg/tensor/conv.rs:360-418)."""
    (kh, kw), (sh, sw), (ph, pw) = kernel, stride, padding
    n = 1
    if len(x.shape) == 4 and sh > 0 and sw > 0 and x.shape[2] + 2 * ph >= kh and x.shape[3] + 2 * pw >= kw:
        N, C, H, W = x.shape
        n = N * ((H + 2 * ph - kh) // sh + 1) * ((W + 2 * pw - kw) // sw + 1) * C * kh * kw
    out = _out_buf(x.dtype, max(n, 1))
    shp = (c_int64 * 2)()
    _check(load().orc_unfold_2d(ctypes.byref(x.c()), kh, kw, sh, sw, ph, pw, out.ctypes.data, shp))
    return out[: shp[0] * shp[1]].reshape(shp[0], shp[1])


def fold_2d(cols: HostView, shape, kernel, stride, padding=(0, 0)) -> np.ndarray:
    """Tensor::fold_2d (linalg/tensor/conv.rs:434-488) into [batch, channels, height, width]."""
    (kh, kw), (sh, sw), (ph, pw) = kernel, stride, padding
    n = int(np.prod(shape, dtype=np.int64))
    out = _out_buf(cols.dtype, max(n, 1))
    _check(load().orc_fold_2d(ctypes.byref(cols.c()), (c_int64 * 4)(*shape), kh, kw, sh, sw, ph, pw,
                              out.ctypes.data))
    return out[:n].reshape(shape)


def sum_f64(x: HostView) -> tuple[float, float]:
    """(compensated sum, sum of |x|) in extended precision, for error bounds."""
    s, a = c_double(), c_double()
    _check(load().orc_sum_f64(ctypes.byref(x.c()), ctypes.byref(s), ctypes.byref(a)))
    return s.value, a.value


def fill_uniform(dtype, n: int, seed: int, lo: float = -1.0, hi: float = 1.0, first: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=dtype)
    _check(load().orc_fill_uniform_at(NP_TO_DT[np.dtype(dtype)], out.ctypes.data, first, n, seed, lo, hi))
    return out


def fill_normal(dtype, n: int, seed: int, first: int = 0) -> np.ndarray:
    """Elements first .. first + n - 1 of the seeded N(0, 1) stream."""
    out = np.empty(n, dtype=dtype)
    _check(load().orc_fill_normal_at(NP_TO_DT[np.dtype(dtype)], out.ctypes.data, first, n, seed))
    return out


def fma_sum_stream(rows: int, cols: int, seed_a: int, seed_b: int, seed_c: int, row_bits: bool = False):
    """The sharded workload Y = A & B + c, sum(Y) (A, B [rows, cols], c [cols],
    U(-1, 1) from the three seeds) checked by regenerating every element:
    returns (reference's sequential f32 fold of Y, exact sum, sum of |y|,
    per-row int64 sums of y's int32 bit patterns or None)."""
    ex, sa, fold = c_double(), c_double(), ctypes.c_float()
    bits = np.zeros(rows, dtype=np.int64) if row_bits else None
    _check(load().orc_fma_sum_stream(rows, cols, seed_a, seed_b, seed_c, ctypes.byref(ex), ctypes.byref(sa),
                                     ctypes.byref(fold), bits.ctypes.data if bits is not None else None))
    return np.float32(fold.value), ex.value, sa.value, bits
