"""Array plumbing between the caller's arrays and the device.

Callers hand the API numpy arrays (as with the reference) or torch tensors.
Kernels only ever see device memory: numpy inputs are copied to the current
CUDA device, torch CUDA tensors are used in place.  Results come back in the
caller's kind: numpy for numpy inputs, a CUDA tensor if any input was on the
device, a (pinned) CPU tensor for CPU tensors.

Element types: the kernels compute in float32 or float64.  float32 features
stay float32 (the B200 path); float64 stays float64 (the reference's own
precision, ``python/mojodgl/_lib.py:127-163``); every other input goes through
the reference's ``f64()`` rules -- complex is rejected, integers that float64
cannot hold exactly are rejected, the rest widen to float64.  Half and bf16
tensors compute in float32, except in segment_mm/gather_mm, which take bf16.
"""

from __future__ import annotations

import numpy as np
import torch

from ._lib import BGL_BF16, BGL_F32, BGL_F64
from .base import DGLError

NUMPY, TORCH_CPU, TORCH_CUDA = 0, 1, 2


def device() -> torch.device:
    if not torch.cuda.is_available():
        raise DGLError("mojodgl (B200 build) needs a CUDA device; it has no CPU fallback")
    return torch.device("cuda", torch.cuda.current_device())


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def kind_of(*xs) -> int:
    k = NUMPY
    for x in xs:
        if isinstance(x, torch.Tensor):
            k = max(k, TORCH_CUDA if x.is_cuda else TORCH_CPU)
    return k


def is_torch(x) -> bool:
    return isinstance(x, torch.Tensor)


# ----------------------------------------------------------------- id arrays
def ids(a):
    """Node ids / segment lengths as int64 (numpy, or torch if given torch).

    Non-integral floats are rejected rather than truncated
    (python/mojodgl/_lib.py:166-180)."""
    if is_torch(a):
        if a.is_floating_point() and a.numel() and not bool((a == a.floor()).all()):
            raise DGLError("node ids and segment lengths must be whole numbers, got {}".format(a.dtype))
        return a.to(torch.int64).contiguous()
    a = np.asanyarray(a)
    if np.issubdtype(a.dtype, np.floating) and a.size:
        if not bool(np.all(a == np.floor(a))):
            raise DGLError("node ids and segment lengths must be whole numbers, got {}".format(a.dtype))
    return np.ascontiguousarray(a, dtype=np.int64)


# ------------------------------------------------------------ feature arrays
def _check_lossless_np(a: np.ndarray) -> None:
    if np.iscomplexobj(a):
        raise DGLError("the kernels are real-valued; complex input is not supported")
    if np.issubdtype(a.dtype, np.integer) and a.dtype != np.int64 and a.size:
        with np.errstate(invalid="ignore"):
            back = a.astype(np.float64).astype(a.dtype)
        if not bool(np.array_equal(back, a)):
            raise DGLError("{} values do not survive the conversion to float64 exactly".format(a.dtype))


def feature(a):
    """A contiguous float32/float64 feature array of the caller's kind."""
    if is_torch(a):
        if a.is_complex():
            raise DGLError("the kernels are real-valued; complex input is not supported")
        if a.dtype in (torch.float32, torch.float64):
            return a.contiguous()
        if a.dtype in (torch.float16, torch.bfloat16):
            return a.to(torch.float32).contiguous()
        if a.dtype != torch.int64 and a.numel() and not a.dtype.is_floating_point:
            back = a.to(torch.float64).to(a.dtype)
            if not bool(torch.equal(back, a)):
                raise DGLError("{} values do not survive the conversion to float64 exactly".format(a.dtype))
        return a.to(torch.float64).contiguous()
    a = np.asanyarray(a)
    if a.dtype == np.float32 or a.dtype == np.float64:
        return np.ascontiguousarray(a)
    _check_lossless_np(a)
    return np.ascontiguousarray(a, dtype=np.float64)


def common_float(*xs):
    """float32 if every present operand is float32, else float64."""
    present = [x for x in xs if x is not None]
    if present and all(str(x.dtype).endswith("float32") for x in present):
        return torch.float32
    return torch.float64


def code_of(dtype: torch.dtype) -> int:
    if dtype == torch.float32:
        return BGL_F32
    if dtype == torch.float64:
        return BGL_F64
    if dtype == torch.bfloat16:
        return BGL_BF16
    raise DGLError("unsupported element type {}".format(dtype))


_NP2T = {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64,
         np.dtype(np.int64): torch.int64, np.dtype(np.int32): torch.int32,
         np.dtype(np.int8): torch.int8}


def to_dev(a, dtype: torch.dtype = None) -> torch.Tensor:
    """The array as a contiguous tensor on the current CUDA device."""
    dev = device()
    if is_torch(a):
        t = a
        if dtype is not None and t.dtype != dtype:
            t = t.to(dtype)
        if t.device != dev:
            t = t.to(dev, non_blocking=t.is_pinned())
        return t.contiguous()
    arr = np.ascontiguousarray(a)
    t = torch.from_numpy(arr) if arr.dtype in _NP2T else torch.from_numpy(arr.astype(np.float64))
    if dtype is not None and t.dtype != dtype:
        t = t.to(dtype)
    return t.to(dev)


def result(t: torch.Tensor, kind: int):
    """Hand a device result back in the caller's kind."""
    if kind == TORCH_CUDA:
        return t
    if kind == TORCH_CPU:
        out = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        out.copy_(t, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return out
    return t.cpu().numpy()


def ptr(t) -> int:
    """Device address of a tensor, or None (NULL) for an absent/empty one."""
    if t is None or t.numel() == 0:
        return None
    return t.data_ptr()


def workspace(nbytes: int) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device())


def shape_of(a):
    return tuple(a.shape)


def reshape(a, shape):
    return a.reshape(shape)


def zeros_like_kind(shape, dtype, kind):
    if kind == NUMPY:
        return np.zeros(shape, dtype=np.float32 if dtype == torch.float32 else np.float64)
    dev = device() if kind == TORCH_CUDA else "cpu"
    return torch.zeros(shape, dtype=dtype, device=dev)
