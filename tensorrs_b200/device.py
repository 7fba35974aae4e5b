"""trs_views over PyTorch CUDA tensors, and thin callers of the C ABI that
allocate their outputs with PyTorch.

PyTorch only provides device memory and the current stream here; every
computation is a libtrs_b200.so kernel.  Views are described over a tensor's
underlying storage, so any strides the reference can express (including the
negative strides of step_slice, which PyTorch views cannot hold) are passed as
explicit (shape, strides, offset) triples.
"""
from __future__ import annotations

import ctypes

import torch

from . import abi

TORCH_TO_TRS = {torch.float32: abi.F32, torch.float64: abi.F64, torch.int32: abi.I32, torch.int64: abi.I64}


def stream_handle() -> int:
    return torch.cuda.current_stream().cuda_stream


def view_of(t: torch.Tensor, shape=None, strides=None, offset=None) -> abi.View:
    """A trs_view into t's storage.  Without overrides it describes t itself."""
    if t.device.type != "cuda":
        raise ValueError("view_of needs a CUDA tensor")
    st = t.untyped_storage()
    es = t.element_size()
    base = st.data_ptr()
    storage_len = st.nbytes() // es
    if shape is None:
        shape = list(t.shape)
    if strides is None:
        strides = list(t.stride()) if shape is not None and list(shape) == list(t.shape) else None
    if offset is None:
        offset = t.storage_offset()
    return abi.make_view(base, TORCH_TO_TRS[t.dtype], shape, strides, offset, storage_len)


def _call(name: str, *args) -> int:
    lib = abi.load()
    return abi.check(getattr(lib, name)(*args))


def binary(op: str, a: abi.View, b: abi.View, out: torch.Tensor) -> torch.Tensor:
    _call("trs_binary", abi.BINOPS[op], ctypes.byref(a), ctypes.byref(b), ctypes.byref(view_of(out)),
          stream_handle())
    return out


def unary(op: str, x: abi.View, out: torch.Tensor, p0=0.0, p1=0.0) -> torch.Tensor:
    params = (abi.Scalar * 2)(abi.scalar(p0), abi.scalar(p1))
    _call("trs_unary", abi.UNOPS[op], ctypes.byref(x), params, ctypes.byref(view_of(out)), stream_handle())
    return out


def elementwise(prog: abi.Program, ins: list[abi.View], out: torch.Tensor | None,
                sum_out: torch.Tensor | None = None) -> None:
    arr = abi.views_array(ins)
    ov = ctypes.byref(view_of(out)) if out is not None else None
    if sum_out is None:
        _call("trs_elementwise", ctypes.byref(prog), arr, ov, stream_handle())
    else:
        _call("trs_elementwise_sum", ctypes.byref(prog), arr, ov, ctypes.byref(view_of(sum_out)),
              stream_handle())


def elementwise_row_sums(prog: abi.Program, ins: list[abi.View], out: torch.Tensor,
                         row_sums: torch.Tensor | None, total: torch.Tensor | None) -> None:
    """Y = prog(ins) into `out`, its sums along the last axis into `row_sums`
    and its total into `total`, in one pass (trs_elementwise_row_sums)."""
    arr = abi.views_array(ins)
    rv = ctypes.byref(view_of(row_sums)) if row_sums is not None else None
    tv = ctypes.byref(view_of(total)) if total is not None else None
    _call("trs_elementwise_row_sums", ctypes.byref(prog), arr, ctypes.byref(view_of(out)), rv, tv,
          stream_handle())


def pack(x: abi.View, out: torch.Tensor) -> torch.Tensor:
    _call("trs_pack", ctypes.byref(x), ctypes.byref(view_of(out)), stream_handle())
    return out


def sum_all(x: abi.View, out: torch.Tensor) -> torch.Tensor:
    _call("trs_sum", ctypes.byref(x), ctypes.byref(view_of(out)), stream_handle())
    return out


def sum_axis(x: abi.View, axis: int, keepdim: bool, out: torch.Tensor) -> torch.Tensor:
    _call("trs_sum_axis", ctypes.byref(x), axis, int(keepdim), ctypes.byref(view_of(out)), stream_handle())
    return out


def mean_axis(x: abi.View, axis: int, keepdim: bool, out: torch.Tensor) -> torch.Tensor:
    _call("trs_mean_axis", ctypes.byref(x), axis, int(keepdim), ctypes.byref(view_of(out)), stream_handle())
    return out


def max_axis(x: abi.View, axis: int, out: torch.Tensor) -> torch.Tensor:
    _call("trs_max_axis", ctypes.byref(x), axis, ctypes.byref(view_of(out)), stream_handle())
    return out


def argmax_axis(x: abi.View, axis: int, out: torch.Tensor) -> torch.Tensor:
    _call("trs_argmax_axis", ctypes.byref(x), axis, ctypes.byref(view_of(out)), stream_handle())
    return out


def reduce_broadcast_grad(g: abi.View, target: list[int], out: torch.Tensor) -> int:
    """Returns abi.OK, or abi.NONE where the reference returns None."""
    t = (ctypes.c_int64 * max(1, len(target)))(*target)
    return _call("trs_reduce_broadcast_grad", ctypes.byref(g), t, len(target), ctypes.byref(view_of(out)),
                 stream_handle())


def sum_to_shape_fused(g: abi.View, gate: abi.View | None, mul: abi.View | None, target: list[int],
                       out: torch.Tensor) -> int:
    t = (ctypes.c_int64 * max(1, len(target)))(*target)
    return _call("trs_sum_to_shape_fused", ctypes.byref(g), ctypes.byref(gate) if gate is not None else None,
                 ctypes.byref(mul) if mul is not None else None, t, len(target), ctypes.byref(view_of(out)),
                 stream_handle())


def affine_relu_backward(g: abi.View, x: abi.View, scale: abi.View, bias: abi.View,
                         grad_scale: torch.Tensor | None, grad_bias: torch.Tensor | None) -> None:
    _call("trs_affine_relu_backward", ctypes.byref(g), ctypes.byref(x), ctypes.byref(scale), ctypes.byref(bias),
          ctypes.byref(view_of(grad_scale)) if grad_scale is not None else None,
          ctypes.byref(view_of(grad_bias)) if grad_bias is not None else None, stream_handle())


def softmax_lastdim(x: abi.View, out: torch.Tensor) -> torch.Tensor:
    _call("trs_softmax_lastdim", ctypes.byref(x), ctypes.byref(view_of(out)), stream_handle())
    return out


def layer_norm_lastdim(x: abi.View, gamma: abi.View, beta: abi.View, eps: float, out: torch.Tensor) -> torch.Tensor:
    """LayerNorm::forward over the last axis (nn/layer_norm.rs:20-33)."""
    _call("trs_layer_norm_lastdim", ctypes.byref(x), ctypes.byref(gamma), ctypes.byref(beta), float(eps),
          ctypes.byref(view_of(out)), stream_handle())
    return out


def sgd_step(param: torch.Tensor, grad: torch.Tensor, lr: float) -> None:
    """SGD::step for one parameter (optim/sgd.rs:29-37), in place."""
    _call("trs_sgd_step", ctypes.byref(view_of(param)), ctypes.byref(view_of(grad)), float(lr), stream_handle())


def rmsprop_step(param: torch.Tensor, grad: torch.Tensor, v: torch.Tensor, lr: float, alpha: float = 0.99,
                 eps: float = 1e-8) -> None:
    """RMSprop::step for one parameter (optim/rmsprop.rs:30-46), in place."""
    _call("trs_rmsprop_step", ctypes.byref(view_of(param)), ctypes.byref(view_of(grad)), ctypes.byref(view_of(v)),
          float(lr), float(alpha), float(eps), stream_handle())


def adam_step(param: torch.Tensor, grad: torch.Tensor, m: torch.Tensor, v: torch.Tensor, lr: float, t: int,
              beta1: float = 0.9, beta2: float = 0.999, eps: float = 1e-8) -> None:
    """Adam::step for one parameter at step t >= 1 (optim/adam.rs:119-144), in place."""
    _call("trs_adam_step", ctypes.byref(view_of(param)), ctypes.byref(view_of(grad)), ctypes.byref(view_of(m)),
          ctypes.byref(view_of(v)), float(lr), float(beta1), float(beta2), float(eps), int(t), stream_handle())


def pooled_size(size: tuple[int, int], kernel: tuple[int, int], stride: tuple[int, int]) -> tuple[int, int]:
    """The spatial size a pooling layer turns `size` into (pooled_size, nn/pool.rs:8-17;
    MaxPool2d::output_size / AvgPool2d::output_size).  No padding: a window that
    would hang over the edge is not taken."""
    if stride[0] <= 0 or stride[1] <= 0:
        raise ValueError("!!!MaxPool2d: stride must be positive!!!")
    if size[0] < kernel[0] or size[1] < kernel[1]:
        raise ValueError("the input is smaller than one window")
    return (size[0] - kernel[0]) // stride[0] + 1, (size[1] - kernel[1]) // stride[1] + 1


def max_pool2d(x: abi.View, kernel: tuple[int, int], out: torch.Tensor,
               stride: tuple[int, int] | None = None) -> torch.Tensor:
    """MaxPool2d::forward (nn/pool.rs:137-144) of an [N, C, H, W] view; the stride
    defaults to the kernel (MaxPool2d::new)."""
    sh, sw = stride if stride is not None else kernel
    _call("trs_max_pool2d", ctypes.byref(x), int(kernel[0]), int(kernel[1]), int(sh), int(sw),
          ctypes.byref(view_of(out)), stream_handle())
    return out


def avg_pool2d(x: abi.View, kernel: tuple[int, int], out: torch.Tensor,
               stride: tuple[int, int] | None = None) -> torch.Tensor:
    """AvgPool2d::forward (nn/pool.rs:223-233)."""
    sh, sw = stride if stride is not None else kernel
    _call("trs_avg_pool2d", ctypes.byref(x), int(kernel[0]), int(kernel[1]), int(sh), int(sw),
          ctypes.byref(view_of(out)), stream_handle())
    return out


def max_pool2d_backward(x: abi.View, grad_out: abi.View, kernel: tuple[int, int], grad_x: torch.Tensor,
                        stride: tuple[int, int] | None = None, accumulate: bool = False) -> torch.Tensor:
    """The gradient MaxPool2d passes back to x (max_axis backward, then fold_2d);
    with accumulate, added to what grad_x holds."""
    sh, sw = stride if stride is not None else kernel
    _call("trs_max_pool2d_backward", ctypes.byref(x), ctypes.byref(grad_out), int(kernel[0]), int(kernel[1]),
          int(sh), int(sw), int(bool(accumulate)), ctypes.byref(view_of(grad_x)), stream_handle())
    return grad_x


def matmul_shape(a: abi.View, b: abi.View) -> list[int]:
    """The shape Tensor::matmul returns for a [..., M, K] and b [..., K, N]."""
    sa = [a.shape[i] for i in range(a.ndim)]
    sb = [b.shape[i] for i in range(b.ndim)]
    batch = [max(x, y) for x, y in zip([1] * (len(sb) - len(sa)) + sa[:-2], [1] * (len(sa) - len(sb)) + sb[:-2])]
    return batch + [sa[-2], sb[-1]]


def matmul(a: abi.View, b: abi.View, out: torch.Tensor) -> torch.Tensor:
    """Tensor::matmul (linalg/tensor/base.rs:896-1013), bit-identical to the reference."""
    _call("trs_matmul", ctypes.byref(a), ctypes.byref(b), ctypes.byref(view_of(out)), stream_handle())
    return out


def matmul_tf32x3(a: abi.View, b: abi.View, out: torch.Tensor) -> torch.Tensor:
    """Tensor::matmul for f32 on the tensor cores (split-TF32, within the sum tolerance)."""
    _call("trs_matmul_tf32x3", ctypes.byref(a), ctypes.byref(b), ctypes.byref(view_of(out)), stream_handle())
    return out


def unfold_2d(x: abi.View, kernel, stride, padding, out: torch.Tensor) -> torch.Tensor:
    """Tensor::unfold_2d (linalg/tensor/conv.rs:360-418) into out [B*OH*OW, C*kh*kw]."""
    (kh, kw), (sh, sw), (ph, pw) = kernel, stride, padding
    _call("trs_unfold_2d", ctypes.byref(x), kh, kw, sh, sw, ph, pw, ctypes.byref(view_of(out)), stream_handle())
    return out


def fold_2d(cols: abi.View, kernel, stride, padding, out: torch.Tensor) -> torch.Tensor:
    """Tensor::fold_2d (linalg/tensor/conv.rs:434-488) into out [B, C, H, W]."""
    (kh, kw), (sh, sw), (ph, pw) = kernel, stride, padding
    _call("trs_fold_2d", ctypes.byref(cols), kh, kw, sh, sw, ph, pw, ctypes.byref(view_of(out)), stream_handle())
    return out


def fill_uniform(out: torch.Tensor, seed: int, lo: float = -1.0, hi: float = 1.0, first: int = 0) -> torch.Tensor:
    _call("trs_fill_uniform", ctypes.byref(view_of(out)), seed, first, lo, hi, stream_handle())
    return out


def fill_normal(out: torch.Tensor, seed: int, first: int = 0) -> torch.Tensor:
    _call("trs_fill_normal", ctypes.byref(view_of(out)), seed, first, stream_handle())
    return out
