"""Helpers for GPU tests: host arrays <-> device views through the C ABI."""
from __future__ import annotations

import numpy as np
import torch

from tensorrs_b200 import abi, device

NP_TO_TORCH = {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
               np.dtype(np.int32): torch.int32, np.dtype(np.int64): torch.int64}


class DevView:
    """A device copy of a host storage array plus a view description."""

    def __init__(self, storage: np.ndarray, shape, strides=None, offset: int = 0):
        self.host = np.ascontiguousarray(storage).reshape(-1)
        self.t = torch.from_numpy(self.host.copy()).cuda()
        self.shape = [int(s) for s in shape]
        self.strides = None if strides is None else [int(s) for s in strides]
        self.offset = int(offset)

    @property
    def view(self) -> abi.View:
        return device.view_of(self.t, self.shape, self.strides, self.offset)

    def host_view(self):
        import oracle
        return oracle.HostView(self.host, self.shape, self.strides, self.offset)


def contiguous(a: np.ndarray) -> DevView:
    a = np.ascontiguousarray(a)
    return DevView(a.reshape(-1), a.shape)


def empty(shape, dtype) -> torch.Tensor:
    return torch.empty([int(s) for s in shape], dtype=NP_TO_TORCH[np.dtype(dtype)], device="cuda")


def to_host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    return t.cpu().numpy()
