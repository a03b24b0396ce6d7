"""Core data structures, configuration and device helpers.

Mirrors tt_thrml/core.py of the reference: the same dataclass names and
fields (Family, FusedInteractionSpec, FusedBlockSpec, CompiledFusedBlock,
CompiledSamplingGroup, CompiledProgram, RNGSpec, BulkRNGBuffers) and the same
device helpers (open_device/open_devices/open_mesh_device/close_*,
is_mesh_device, device_ids, core.py:178-228).  The TT-MLIR configuration
becomes a CUDA configuration (`make_cuda_config`); `make_ttmlir_config`
accepts the reference's keyword arguments so existing callers keep working.
"""

from __future__ import annotations

import hashlib
import json
import os
import tempfile
from dataclasses import dataclass, field
from enum import Enum
from pathlib import Path
from typing import Any, Iterable, Sequence, cast

import numpy as np


class Family(str, Enum):
    SPIN = "spin"
    CATEGORICAL = "categorical"
    GAUSSIAN = "gaussian"


RNG_MODES = ("philox", "parity")
# State layout of all-spin programs: "bits" packs one bit per chain (needs a
# multiple of 256 chains), "int8" one byte per chain; "auto" picks bits when
# the chain count allows.
SPIN_LAYOUTS = ("auto", "bits", "int8")
DENSE_PRECISIONS = ("auto", "bf16", "fp32")


@dataclass(frozen=True)
class CUDAConfig:
    """Execution configuration (replaces TTMLIRConfig, tt_thrml/core.py:21-40).

    rng_mode: "philox" draws variates on device from a counter-based Philox
      stream keyed by (seed, sweep, row, chain); "parity" uploads host-made
      variates following thrml's key tree (tt_thrml/rng.py:132-200).
    n_chains: independent chains per executor (the reference has one).
    cuda_graphs: capture multi-sweep runs in CUDA graphs.
    spin_layout: state layout of all-spin programs ("auto", "bits", "int8").
    dense_precision: tensor-core path of dense bipartite programs. "bf16"
      keeps gaussian block states as bf16 GEMM operands; "fp32" keeps them
      float32, fed to the GEMM as three bf16 pieces against the weights
      repeated along K (the float32 field up to summation order); "auto" is
      "fp32" in parity mode and "bf16" in Philox mode.
    stencil: run lattice programs on the stencil kernels (False: their tables).
    dense_detect: look for dense bipartite structure in lowered programs (an RBM
      written with thrml factors) and run it on the tensor-core kernel.
    dense_round_weights: allow that path to round the detected weights to bf16
      (otherwise only bf16-representable weights qualify).
    """

    artifact_root: Path
    arch: str = "sm_100a"
    rng_mode: str = "philox"
    n_chains: int = 1
    cuda_graphs: bool = True
    spin_layout: str = "auto"
    dense_precision: str = "auto"
    stencil: bool = True
    dense_detect: bool = True
    dense_round_weights: bool = False

    def __post_init__(self) -> None:
        object.__setattr__(self, "artifact_root", Path(self.artifact_root).resolve())
        if self.rng_mode not in RNG_MODES:
            raise ValueError(f"rng_mode must be one of {RNG_MODES}, got {self.rng_mode!r}")
        if int(self.n_chains) < 1:
            raise ValueError("n_chains must be >= 1")
        if self.arch != "sm_100a":
            raise ValueError(f"only sm_100a is supported, got {self.arch!r}")
        if self.spin_layout not in SPIN_LAYOUTS:
            raise ValueError(f"spin_layout must be one of {SPIN_LAYOUTS}, got {self.spin_layout!r}")
        if self.dense_precision not in DENSE_PRECISIONS:
            raise ValueError(f"dense_precision must be one of {DENSE_PRECISIONS}, got {self.dense_precision!r}")

    @property
    def resolved_dense_precision(self) -> str:
        if self.dense_precision != "auto":
            return self.dense_precision
        return "fp32" if self.rng_mode == "parity" else "bf16"

    def cache_key(self) -> str:
        payload = {"arch": self.arch, "rng_mode": self.rng_mode}
        return hashlib.sha256(json.dumps(payload, sort_keys=True).encode()).hexdigest()[:16]

    def plan_key(self) -> tuple:
        """The fields that decide a program's kernels and device tables (the plan cache's part of the key)."""
        return (self.arch, self.rng_mode, self.spin_layout, self.resolved_dense_precision, bool(self.stencil),
                bool(self.dense_detect), bool(self.dense_round_weights))


# Drop-in name for callers written against the reference.
TTMLIRConfig = CUDAConfig


@dataclass(frozen=True)
class FusedInteractionSpec:
    """One lowered interaction (tt_thrml/core.py:43-57).

    Dense form (row_ptr is None): weighted_mask has shape
    (n_nodes, n_terms, *inner) and each gather_indices entry (n_nodes, n_terms),
    exactly as the reference builds them.  Ragged form (row_ptr given, length
    n_nodes + 1): weighted_mask is (nnz, *inner) and each gather entry (nnz,);
    the terms of node i are row_ptr[i]:row_ptr[i+1].  Gather entries hold flat
    block-ordered state rows.
    """

    weighted_mask: np.ndarray
    gather_indices: tuple[np.ndarray, ...]
    n_spin: int
    n_categorical: int
    n_terms: int
    contribution_kind: str
    row_ptr: np.ndarray | None = None

    def ragged(self, n_nodes: int) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(row_ptr int64 [n+1], weights float32 [nnz, inner], sources int32 [n_src, nnz])."""
        wm = np.asarray(self.weighted_mask, dtype=np.float32)
        if self.row_ptr is not None:
            rp = np.asarray(self.row_ptr, dtype=np.int64)
            nnz = int(rp[-1])
            w = wm.reshape(nnz, -1) if nnz else wm.reshape(0, max(1, int(np.prod(wm.shape[1:]))))
            src = (
                np.stack([np.asarray(g, dtype=np.int32).reshape(nnz) for g in self.gather_indices])
                if self.gather_indices
                else np.zeros((0, nnz), dtype=np.int32)
            )
            return rp, np.ascontiguousarray(w), np.ascontiguousarray(src)
        t = int(self.n_terms)
        rp = np.arange(n_nodes + 1, dtype=np.int64) * t
        w = wm.reshape(n_nodes * t, -1)
        src = (
            np.stack([np.asarray(g, dtype=np.int32).reshape(n_nodes * t) for g in self.gather_indices])
            if self.gather_indices
            else np.zeros((0, n_nodes * t), dtype=np.int32)
        )
        return rp, np.ascontiguousarray(w), np.ascontiguousarray(src)


@dataclass(frozen=True)
class FusedBlockSpec:
    """Specification of one block (tt_thrml/core.py:60-70)."""

    block_index: int
    family: Family
    n_nodes: int
    n_categories: int | None
    block_global_start: int
    total_nodes: int
    interactions: tuple[FusedInteractionSpec, ...]


@dataclass(frozen=True)
class CompiledFusedBlock:
    """One block and its device plan (tt_thrml/core.py:73-78).

    kernel_artifact holds the block's device tables (None for clamped blocks).
    """

    spec: FusedBlockSpec
    kernel_artifact: Any | None


@dataclass(frozen=True)
class CompiledSamplingGroup:
    """One sampling group and its device plan (tt_thrml/core.py:81-86)."""

    block_indices: tuple[int, ...]
    kernel_artifact: Any


@dataclass(frozen=True)
class CompiledProgram:
    """Compiled program (tt_thrml/core.py:89-102).

    state_dtype is "int8" or "float32"; layout is "rows x chains" (chain
    innermost); index_dtype is the int32 gather index type.
    """

    blocks: tuple[CompiledFusedBlock, ...]
    sampling_groups: tuple[CompiledSamplingGroup, ...]
    n_free_blocks: int
    total_nodes: int
    block_global_starts: tuple[int, ...]
    sampling_order: tuple[tuple[int, ...], ...]
    state_dtype: object
    index_dtype: object
    layout: object
    rng_spec: "RNGSpec"
    n_chains: int = 1
    device: Any = None


@dataclass(frozen=True)
class RNGSpec:
    """Specification of the per-(block, sweep) variates (tt_thrml/core.py:105-114)."""

    n_sweeps: int
    spin_blocks: tuple[int, ...]
    categorical_blocks: tuple[int, ...]
    gaussian_blocks: tuple[int, ...]
    nodes_per_block: tuple[int, ...]
    categories_per_block: tuple[int | None, ...]


@dataclass(frozen=True)
class BulkRNGBuffers:
    """Device variates per block (tt_thrml/core.py:117-123).

    Each dict maps a block index to one device tensor [n_sweeps, n_nodes, qv,
    n_chains] (qv = q for categorical, else 1); in Philox mode all three are
    None and `seed` keys the on-device stream.
    """

    spin_threshold_logits: dict[int, Any] | None
    categorical_gumbel: dict[int, Any] | None
    gaussian_noise: dict[int, Any] | None
    seed: int | None = None
    n_sweeps: int = 0


def make_cuda_config(
    *,
    artifact_root: Path | str | None = None,
    arch: str = "sm_100a",
    rng_mode: str = "philox",
    n_chains: int = 1,
    cuda_graphs: bool = True,
    spin_layout: str = "auto",
    dense_precision: str = "auto",
    stencil: bool = True,
    dense_detect: bool = True,
    dense_round_weights: bool = False,
) -> CUDAConfig:
    """Create a CUDA configuration (the CUDA counterpart of make_ttmlir_config)."""
    root = Path(artifact_root if artifact_root is not None else Path(tempfile.gettempdir()) / "tt-thrml-b200")
    return CUDAConfig(
        artifact_root=root,
        arch=arch,
        rng_mode=rng_mode,
        n_chains=int(n_chains),
        cuda_graphs=cuda_graphs,
        spin_layout=spin_layout,
        dense_precision=dense_precision,
        stencil=stencil,
        dense_detect=dense_detect,
        dense_round_weights=dense_round_weights,
    )


def make_ttmlir_config(
    *,
    system_desc_path: Path | str | None = None,
    artifact_root: Path | str | None = None,
    build_dir: Path | str | None = None,
    ttmlir_opt: Path | str | None = None,
    ttmlir_translate: Path | str | None = None,
    **cuda_kwargs,
) -> CUDAConfig:
    """Reference-compatible factory (tt_thrml/core.py:134-175).

    The TT-MLIR tool paths have no meaning on CUDA; the argument checks the
    reference performs on them are kept so misuse fails the same way.
    """
    if build_dir is not None and (ttmlir_opt is not None or ttmlir_translate is not None):
        raise ValueError("Pass either build_dir or explicit tool paths, not both.")
    if (ttmlir_opt is None) != (ttmlir_translate is None):
        raise ValueError("Pass both ttmlir_opt and ttmlir_translate together.")
    del system_desc_path
    return make_cuda_config(artifact_root=artifact_root, **cuda_kwargs)


# --------------------------------------------------------------------------
# Devices.  `ttnn` is the backend object.  The reference passes the ttnn
# module; here any object exposing open_device/close_device (e.g. the CUDA
# backend in tt_thrml_b200.backend, or a test double) is delegated to, and
# None means the CUDA backend.
# --------------------------------------------------------------------------


def _backend(ttnn):
    if ttnn is None:
        from .backend import cuda

        return cuda
    return ttnn


def open_device(ttnn=None, *, device_id: int = 0) -> object:
    return _backend(ttnn).open_device(device_id=device_id)


def open_devices(ttnn=None, *, device_ids: Sequence[int]) -> tuple[object, ...]:
    if not device_ids:
        raise ValueError("At least one device id required.")
    be = _backend(ttnn)
    return tuple(be.open_device(device_id=int(d)) for d in device_ids)


def open_mesh_device(
    ttnn=None,
    *,
    mesh_shape: tuple[int, int],
    device_ids: Sequence[int] | None = None,
    num_command_queues: int = 1,
    offset=None,
) -> object:
    be = _backend(ttnn)
    kwargs: dict = {"mesh_shape": be.MeshShape(*mesh_shape), "num_command_queues": num_command_queues}
    if device_ids is not None:
        kwargs["physical_device_ids"] = [int(d) for d in device_ids]
    if offset is not None:
        kwargs["offset"] = offset
    return be.open_mesh_device(**kwargs)


def close_device(ttnn, device) -> None:
    _backend(ttnn).close_device(device)


def close_mesh_device(ttnn, device) -> None:
    _backend(ttnn).close_mesh_device(device)


def close_devices(ttnn, devices) -> None:
    be = _backend(ttnn)
    for device in devices:
        be.close_device(device)


def is_mesh_device(device) -> bool:
    return len(device_ids(device)) > 1


def device_ids(device) -> tuple[int, ...]:
    get_ids = getattr(device, "get_device_ids", None)
    if callable(get_ids):
        return tuple(int(d) for d in cast(Iterable[Any], get_ids()))
    return ()


def env_flag(name: str, default: bool = False) -> bool:
    v = os.environ.get(name)
    if v is None:
        return default
    return v not in ("0", "", "false", "False")
