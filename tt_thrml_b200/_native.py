"""ctypes binding of libtthrml_b200.so (the C ABI declared in include/tthrml.h).

There is no CPU fallback: every compute call goes to the CUDA library, and
loading fails loudly when the library is missing.  Structures below mirror the
C layouts field for field.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_NAME = "libtthrml_b200.so"
LIB_PATH = Path(__file__).resolve().parent / LIB_NAME

OK = 0
SPIN, CATEGORICAL, GAUSSIAN = 0, 1, 2
KIND_LINEAR, KIND_PRECISION = 0, 1
STATE_F32, STATE_I8, STATE_BITS = 0, 1, 2
MAX_CAT_SOURCES = 4
MAX_CATEGORIES = 64

c_i32 = ctypes.c_int32
c_i64 = ctypes.c_int64
c_u32 = ctypes.c_uint32
c_u64 = ctypes.c_uint64
c_vp = ctypes.c_void_p


class Interaction(ctypes.Structure):
    _fields_ = [
        ("row_ptr", c_vp),
        ("weights", c_vp),
        ("sources", c_vp),
        ("nnz", c_i64),
        ("n_sources", c_i32),
        ("n_categorical", c_i32),
        ("kind", c_i32),
        ("w_inner", c_i32),
        ("cat_q", c_i32 * MAX_CAT_SOURCES),
    ]


class BlockDesc(ctypes.Structure):
    _fields_ = [
        ("family", c_i32),
        ("n_categories", c_i32),
        ("n_interactions", c_i32),
        ("reserved", c_i32),
        ("n_nodes", c_i64),
        ("row_start", c_i64),
        ("interactions", c_vp),
        ("variates", c_vp),
        ("variates_sweeps", c_i64),
    ]


class HaloExport(ctypes.Structure):
    """tthrml_halo_export (include/tthrml.h)."""

    _fields_ = [
        ("up", ctypes.c_void_p),
        ("down", ctypes.c_void_p),
        ("up_row0", ctypes.c_int64),
        ("down_row0", ctypes.c_int64),
        ("rows", ctypes.c_int64),
        ("slot_bytes", ctypes.c_int64),
        ("sweeps_per_period", ctypes.c_uint32),
        ("reserved", ctypes.c_uint32),
    ]


class GroupDesc(ctypes.Structure):
    _fields_ = [
        ("blocks", c_vp),
        ("n_blocks", c_i32),
        ("state_dtype", c_i32),
        ("group_rows", c_i64),
        ("n_chains", c_i64),
        ("chain_offset", c_i64),
        ("state", c_vp),
        ("scratch", c_vp),
        ("in_place", c_i32),
        ("use_variates", c_i32),
        ("seed", c_u64),
        ("sweep", c_u32),
        ("reserved", c_u32),
        ("ctl", c_vp),
    ]


# (name, restype, argtypes) of every exported entry point.
_SIGNATURES = {
    "tthrml_group_step": (c_i32, [ctypes.POINTER(GroupDesc), c_vp]),
    "tthrml_group_step_static_scratch": (c_i32, [ctypes.POINTER(GroupDesc), c_vp]),
    "tthrml_spin_csr_step": (
        c_i32,
        [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_u64, c_u32, c_vp, c_vp],
    ),
    "tthrml_spin_bits_step": (
        c_i32,
        [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_u64, c_u32, c_vp, c_vp],
    ),
    "tthrml_spin_bits_step_ordered": (
        c_i32,
        [c_vp, c_vp, c_vp, c_vp, c_i64, c_i64, c_vp, c_i64, c_i64, c_vp, c_i64, c_u64, c_u32, c_vp, c_vp, c_vp],
    ),
    "tthrml_dense_field_sample": (
        c_i32,
        [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, ctypes.c_float, c_vp, c_vp, c_i32, c_i64, c_i64, c_vp,
         c_i64, c_u64, c_u32, c_vp, c_vp, c_vp],
    ),
    "tthrml_dense_field_sample_ties": (
        c_i32,
        [c_vp, c_vp, c_i64, c_i64, c_i64, c_vp, c_i32, ctypes.c_float, c_vp, c_vp, c_i32, c_i64, c_i64, c_vp,
         c_i64, c_u64, c_u32, c_vp, c_vp, c_vp, c_i64, c_vp],
    ),
    "tthrml_potts3d_step": (
        c_i32,
        [c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_vp, c_vp, c_i32, c_i64, c_vp, c_i64, c_u64, c_u32,
         c_vp, c_vp],
    ),
    "tthrml_potts3d_step_weights": (
        c_i32,
        [c_vp, c_i64, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_vp, c_vp, c_i32, c_i64, c_vp, c_i64, c_u64, c_u32,
         c_vp, c_vp, c_vp],
    ),
    "tthrml_potts3d_bias_weights": (c_i32, [c_vp, c_i64, c_i32, c_vp, c_vp]),
    "tthrml_ising2d_halfsweep": (
        c_i32,
        [c_vp, c_vp, c_i64, c_i64, c_i32, c_i64, c_i64, c_i64, c_i64, c_i32, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64,
         c_u64, c_u32, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp],
    ),
    "tthrml_moments_accumulate": (c_i32, [c_vp, c_i32, c_i64, c_vp, c_vp, c_i32, c_i64, c_i32, c_vp, c_vp]),
    "tthrml_ising2d_halfsweep_x": (
        c_i32,
        [c_vp, c_vp, c_i64, c_i64, c_i32, c_i64, c_i64, c_i64, c_i64, c_i32, c_i64, c_vp, c_vp, c_vp, c_i64, c_i64,
         c_u64, c_u32, c_vp, c_i64, c_i64, c_vp, c_i64, c_vp, c_vp],
    ),
    "tthrml_ising2d_halfsweep_planes": (
        c_i32,
        [c_vp, c_vp, c_i64, c_i64, c_i32, c_i64, c_i64, c_i64, c_i64, c_i32, c_i64, c_vp, c_i64, c_u64, c_u32, c_vp,
         c_i64, c_i64, c_vp, c_i64, c_vp, c_vp],
    ),
    "tthrml_ising2d_halfsweep_bits": (
        c_i32,
        [c_vp, c_vp, c_i64, c_i64, c_i32, c_i64, c_i64, c_i64, c_i64, c_i32, c_i64, c_vp, c_i64, c_u64, c_u32, c_vp,
         c_i64, c_i64, c_vp, c_i64, c_vp, c_vp],
    ),
    "tthrml_ipc_malloc": (c_i32, [c_i64, c_vp, c_vp]),
    "tthrml_ipc_open": (c_i32, [c_vp, c_vp]),
    "tthrml_ipc_close": (c_i32, [c_vp]),
    "tthrml_free": (c_i32, [c_vp]),
    "tthrml_memcpy": (c_i32, [c_vp, c_vp, c_i64, c_vp]),
    "tthrml_halo_signal": (c_i32, [c_vp, c_vp, c_u32, c_u32, c_vp, c_vp]),
    "tthrml_halo_import": (c_i32, [c_vp, c_vp, c_i64, c_i64, c_i64, c_i64, c_vp, c_vp, c_u32, c_u32, c_vp, c_vp, c_vp]),
    "tthrml_ising2d_resident": (
        c_i32,
        [c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_u64, c_u32, c_i32, c_i64, c_vp, c_i64, c_i64, c_i64, c_i32,
         c_i64, c_vp, c_vp, c_vp],
    ),
    "tthrml_ising2d_resident_planes": (
        c_i32,
        [c_vp, c_i64, c_i32, c_i32, c_i64, c_i64, c_vp, c_u64, c_u32, c_i32, c_i64, c_vp, c_i64, c_i64, c_i64, c_i32,
         c_i64, c_vp, c_vp, c_vp],
    ),
    "tthrml_ctl_advance": (c_i32, [c_vp, c_u32, c_vp]),
    "tthrml_decode_rows": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_i32, c_vp, c_vp]),
    "tthrml_encode_rows": (c_i32, [c_vp, c_i32, c_i32, c_i64, c_i32, c_i64, c_i64, c_vp, c_vp]),
    "tthrml_sum_rows": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_vp]),
    "tthrml_greedy_colouring": (c_i32, [c_i64, c_vp, c_vp, c_vp, ctypes.POINTER(c_i32)]),
    "tthrml_set_device": (c_i32, [c_i32]),
    "tthrml_last_error": (ctypes.c_char_p, []),
    "tthrml_abi_version": (c_i32, []),
}

_lib = None
_lock = threading.Lock()


class NativeError(RuntimeError):
    """A libtthrml_b200 entry point returned a non-zero status."""


def exported_symbols() -> tuple[str, ...]:
    return tuple(_SIGNATURES)


def lib() -> ctypes.CDLL:
    """Loads the CUDA library once; raises when it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("TTHRML_LIB", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build the CUDA extension first "
                "(python -m tt_thrml_b200.build). There is no CPU fallback."
            )
        handle = ctypes.CDLL(str(path))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        if handle.tthrml_abi_version() != 1:
            raise RuntimeError(f"{path}: unexpected ABI version {handle.tthrml_abi_version()}")
        _lib = handle
    return _lib


def check(rc: int, what: str) -> None:
    if rc != OK:
        msg = lib().tthrml_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed ({rc}): {msg}")


def ptr(t) -> int | None:
    """Device (or host) address of a torch tensor, None for None."""
    if t is None:
        return None
    return t.data_ptr()


def stream_handle(stream) -> int | None:
    return None if stream is None else stream.cuda_stream


_bound = threading.local()


def bind_device(index: int) -> None:
    """Makes `index` current for the library's CUDA runtime on this thread (cached)."""
    if getattr(_bound, "device", None) != index:
        check(lib().tthrml_set_device(int(index)), "tthrml_set_device")
        _bound.device = index
