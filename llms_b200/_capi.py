"""ctypes binding of ``libb200mm.so`` (declared in ``include/b200mm.h``).

This module is the only place Python touches the C ABI.  It loads the
in-tree library built by ``llms_b200/csrc/Makefile`` and raises at import
time if it is missing: there is no Python or CPU fallback for the kernels.
"""

from __future__ import annotations

import contextlib
import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("B200MM_LIB", Path(__file__).resolve().parent / "_lib" / "libb200mm.so"))

B200MM_OK = 0
DTYPE_CODES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

_c_i64 = ctypes.c_int64
_c_p = ctypes.c_void_p


class MlaShape(ctypes.Structure):
    """Mirror of ``b200mm_mla_shape``."""

    _fields_ = [
        ("B", ctypes.c_int32),
        ("H", ctypes.c_int32),
        ("KV", ctypes.c_int32),
        ("D", ctypes.c_int32),
        ("DR", ctypes.c_int32),
        ("R", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
        ("eps", ctypes.c_float),
    ]


class PeerOut(ctypes.Structure):
    """Mirror of ``b200mm_peer_out``."""

    _fields_ = [
        ("dst", ctypes.c_void_p * 8),
        ("ld_dst", ctypes.c_int64),
        ("part_widths", ctypes.c_int64 * 3),
        ("nparts", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("world", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("flags", ctypes.c_void_p * 8),
        ("ticket", ctypes.c_void_p),
        ("seen", ctypes.c_void_p),
        ("err", ctypes.c_void_p),
    ]


# name -> (restype, argtypes); kept in the order of include/b200mm.h
SIGNATURES: dict[str, tuple] = {
    "b200mm_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "b200mm_abi_version": (ctypes.c_int, []),
    "b200mm_launch_count": (ctypes.c_uint64, []),
    "b200mm_force_generic": (ctypes.c_int, [ctypes.c_int]),
    "b200mm_gate_up_silu": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p],
    ),
    "b200mm_qkv": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p],
    ),
    "b200mm_gate_up_silu_w8": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p],
    ),
    "b200mm_qkv_w8": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p],
    ),
    "b200mm_linear": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p],
    ),
    "b200mm_linear_w8": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _c_p],
    ),
    "b200mm_gqa_decode_workspace_size": (ctypes.c_size_t, [_c_i64] * 5),
    "b200mm_gqa_decode": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
         _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_float, ctypes.c_int, _c_p, ctypes.c_size_t, _c_p],
    ),
    "b200mm_mla_append": (
        ctypes.c_int,
        [ctypes.POINTER(MlaShape), _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p,
         _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_p],
    ),
    "b200mm_mla_decode_workspace_size": (ctypes.c_size_t, [ctypes.POINTER(MlaShape), _c_i64]),
    "b200mm_mla_decode": (
        ctypes.c_int,
        [ctypes.POINTER(MlaShape), _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, ctypes.c_float, _c_i64, _c_p, _c_i64,
         _c_p, ctypes.c_size_t, _c_p],
    ),
    "b200mm_mla_decode_partial": (
        ctypes.c_int,
        [ctypes.POINTER(MlaShape), _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, ctypes.c_float, _c_i64, _c_i64, _c_i64, _c_p, _c_p,
         _c_p, ctypes.c_size_t, _c_p],
    ),
    "b200mm_mla_combine_partials": (
        ctypes.c_int,
        [ctypes.POINTER(MlaShape), _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_i64, _c_p, ctypes.c_size_t,
         _c_p],
    ),
    "b200mm_rmsnorm": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_i64, _c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, ctypes.c_float, ctypes.c_int,
         _c_p],
    ),
    "b200mm_qk_norm_rope": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_i64, _c_i64, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_p,
         _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, ctypes.c_float,
         ctypes.c_int, _c_p],
    ),
    "b200mm_linear_peer": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.POINTER(PeerOut), _c_p],
    ),
    "b200mm_linear_w8_peer": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.POINTER(PeerOut), _c_p],
    ),
    "b200mm_gate_up_silu_w8_peer": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_p, _c_p, _c_p, _c_p, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int,
         ctypes.POINTER(PeerOut), _c_p],
    ),
    "b200mm_peer_gather": (
        ctypes.c_int,
        [_c_p, _c_i64, _c_i64, ctypes.POINTER(ctypes.c_int64), ctypes.c_int, ctypes.POINTER(_c_p), _c_i64,
         ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.POINTER(_c_p), _c_p, _c_p, ctypes.c_int, _c_p],
    ),
    "b200mm_mla_decode_noalloc": (
        ctypes.c_int,
        [ctypes.POINTER(MlaShape), _c_p, _c_i64, _c_p, _c_i64, _c_i64, _c_p, _c_i64, _c_i64,
         _c_p, _c_i64, _c_i64, _c_p, _c_p, _c_p, _c_p, ctypes.c_float, _c_i64, _c_p, _c_i64, _c_p],
    ),
}


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH} is not built; run `make -C llms_b200/csrc -j8` or "
            "`python -c 'import __graft_entry__ as g; g.build()'`"
        )
    lib = ctypes.CDLL(os.fspath(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()


class KernelError(RuntimeError):
    """A b200mm entry point returned a non-zero status."""


def check(status: int, what: str) -> None:
    if status != B200MM_OK:
        msg = lib.b200mm_status_string(status).decode()
        raise KernelError(f"{what} failed with status {status}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}; expected float32, float16 or bfloat16") from None


_SAME_DEVICE = contextlib.nullcontext()


def on_device(t: torch.Tensor):
    """``torch.cuda.device(t.device)`` when ``t`` is not on the current device,
    else a no-op context (entering the device context costs more host time
    than the kernel launch it guards, on every eager call)."""
    idx = t.device.index
    if idx is None or idx == torch.cuda.current_device():
        return _SAME_DEVICE
    return torch.cuda.device(t.device)


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def launch_count() -> int:
    return int(lib.b200mm_launch_count())


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError(
                "b200mm kernels run on CUDA (sm_100a) tensors only; got a tensor on "
                f"{t.device}. There is no CPU path."
            )
