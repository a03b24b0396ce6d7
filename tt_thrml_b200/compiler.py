"""Program compilation: thrml program -> per-group device plans.

The reference lowers each sampling group to a TT-MLIR flatbuffer with every
weight and gather index baked in as IR constants (tt_thrml/compiler.py:1-7,
453-521).  Here each group lowers to static device tables plus a block
descriptor, and runs as one precompiled sm_100a kernel per sweep:

* the lowering of a thrml `BlockSamplingProgram` to `FusedBlockSpec`s keeps
  the reference's semantics (flat block-ordered layout, family inference,
  interaction lowering, weighted masks; tt_thrml/compiler.py:39-271);
* each group is then planned onto one of two kernels:
  - `spin_csr`: blocks of spins whose field is one bias plus one pairwise
    spin coupling (Ising-type programs), int8 state, CSR neighbour tables;
  - `generic`: anything else (categorical sources, gaussian blocks, mixed
    superblocks, multi-source terms), ragged-ELL tables.

Programs may also lower themselves (native table programs such as the
synthetic workloads in `tt_thrml_b200.workloads`) by providing
`tt_lower_blocks()`; they skip the per-node thrml layout loop.
"""

from __future__ import annotations

import dataclasses
import hashlib
import threading
import weakref
from collections import OrderedDict
from dataclasses import dataclass
from enum import Enum
from typing import Any

import numpy as np

from . import _native as nat
from .core import (
    CompiledFusedBlock,
    CompiledProgram,
    CompiledSamplingGroup,
    CUDAConfig,
    Family,
    FusedBlockSpec,
    FusedInteractionSpec,
)
from .rng import make_rng_spec

# --------------------------------------------------------------------------
# Lowering of thrml programs (semantics of tt_thrml/compiler.py:39-271).
# --------------------------------------------------------------------------


@dataclass(frozen=True)
class _GlobalStateLayout:
    """Flat block-ordered layout (tt_thrml/compiler.py:39-50)."""

    block_starts: tuple[int, ...]
    global_to_flat: tuple[np.ndarray, ...]
    total_nodes: int

    def flatten_slices(self, global_inds, global_slices) -> tuple[np.ndarray, ...]:
        flat = []
        for global_ind, global_slice in zip(global_inds, global_slices, strict=True):
            index_map = self.global_to_flat[int(global_ind)]
            flat.append(index_map[np.asarray(global_slice, dtype=np.int64)].astype(np.int32))
        return tuple(flat)


def _infer_family(block, gibbs_spec) -> Family:
    """tt_thrml/compiler.py:53-70."""
    explicit = getattr(block, "family", None)
    if explicit is not None:
        return Family(explicit)
    node_type = type(block.nodes[0]).__name__.lower()
    if "spin" in node_type or "bool" in node_type:
        return Family.SPIN
    if "categorical" in node_type or "discrete" in node_type:
        return Family.CATEGORICAL
    if "gaussian" in node_type or "continuous" in node_type:
        return Family.GAUSSIAN
    sds = getattr(gibbs_spec, "node_shape_dtypes", None) or {}
    sd = sds.get(type(block.nodes[0]))
    if sd is not None:
        dtype = getattr(sd, "dtype", None)
        if dtype is None:
            dtype = sd[0][0].dtype
        kind = np.dtype(dtype).kind
        if kind == "b":
            return Family.SPIN
        if kind in ("i", "u"):
            return Family.CATEGORICAL
        if kind == "f":
            return Family.GAUSSIAN
    return Family.SPIN


def _get_n_categories(block, family: Family) -> int | None:
    """tt_thrml/compiler.py:73-79."""
    if family != Family.CATEGORICAL:
        return None
    n = getattr(block.nodes[0], "n_categories", None)
    return int(n) if n is not None else 2


def _lower_interaction(interaction, family: Family) -> dict:
    """tt_thrml/compiler.py:82-114 (same hook, attribute and error contract)."""
    hook = getattr(interaction, "tt_interaction_contribution", None)
    if callable(hook):
        contrib = hook(parameter_family=family.value)
        return {
            "weights": np.asarray(getattr(contrib, "weights")),
            "n_spin": int(getattr(contrib, "n_spin")),
            "n_categorical": getattr(contrib, "n_categorical", None),
            "contribution_kind": str(getattr(contrib, "contribution_kind", "default")),
        }
    if hasattr(interaction, "n_spin") and hasattr(interaction, "weights"):
        return {
            "weights": np.asarray(interaction.weights),
            "n_spin": int(interaction.n_spin),
            "n_categorical": None,
            "contribution_kind": "default",
        }
    if family == Family.GAUSSIAN:
        if hasattr(interaction, "weights"):
            return {
                "weights": np.asarray(interaction.weights),
                "n_spin": 0,
                "n_categorical": 0,
                "contribution_kind": "linear",
            }
        if hasattr(interaction, "inverse_weights"):
            return {
                "weights": np.reciprocal(np.asarray(interaction.inverse_weights, dtype=np.float32)),
                "n_spin": 0,
                "n_categorical": 0,
                "contribution_kind": "precision",
            }
    raise TypeError(f"Cannot lower interaction of type {type(interaction)}")


def _build_block_global_starts(gibbs_spec) -> tuple[tuple[int, ...], int]:
    starts, offset = [], 0
    for block in gibbs_spec.blocks:
        starts.append(offset)
        offset += len(block.nodes)
    return tuple(starts), offset


def _build_global_state_layout(gibbs_spec) -> _GlobalStateLayout:
    """tt_thrml/compiler.py:126-153: free blocks first, then clamped."""
    block_starts, total_nodes = _build_block_global_starts(gibbs_spec)
    loc_map = gibbs_spec.node_global_location_map
    per_block = []
    max_gi = -1
    for bi, block in enumerate(gibbs_spec.blocks):
        locs = np.asarray([loc_map[node] for node in block.nodes], dtype=np.int64).reshape(-1, 2)
        per_block.append(locs)
        if len(locs):
            max_gi = max(max_gi, int(locs[:, 0].max()))
    sizes = [0] * (max_gi + 1)
    for locs in per_block:
        for gi in np.unique(locs[:, 0]):
            sizes[gi] = max(sizes[gi], int(locs[locs[:, 0] == gi, 1].max()) + 1)
    maps = [np.full(s, -1, dtype=np.int64) for s in sizes]
    for bi, locs in enumerate(per_block):
        flat = block_starts[bi] + np.arange(len(locs), dtype=np.int64)
        for gi in np.unique(locs[:, 0]):
            sel = locs[:, 0] == gi
            maps[gi][locs[sel, 1]] = flat[sel]
    for m in maps:
        if (m < 0).any():
            raise ValueError("THRML global state map is not dense.")
    return _GlobalStateLayout(block_starts=block_starts, global_to_flat=tuple(maps), total_nodes=total_nodes)


def _build_interaction_spec(
    interaction, active_mask, global_inds, global_slices, family: Family, n_nodes: int, layout: _GlobalStateLayout
) -> FusedInteractionSpec:
    """tt_thrml/compiler.py:156-217."""
    lowered = _lower_interaction(interaction, family)
    weights = np.asarray(lowered["weights"], dtype=np.float32)
    mask = np.asarray(active_mask, dtype=np.float32)
    if weights.ndim == 1:
        weights = weights.reshape(n_nodes, -1)
    if mask.ndim == 1:
        mask = mask.reshape(n_nodes, -1)
    if weights.shape[:2] == mask.shape:
        n_terms = int(mask.shape[1])
        weighted_mask = (weights * mask.reshape(mask.shape + (1,) * (weights.ndim - 2))).astype(np.float32)
    elif weights.shape == mask.shape:
        weighted_mask = (weights * mask).astype(np.float32)
        n_terms = int(weighted_mask.shape[-1])
    else:
        raise ValueError(f"weights shape {weights.shape} does not match mask shape {mask.shape}")

    n_spin = int(lowered["n_spin"])
    explicit = lowered.get("n_categorical")
    if explicit is not None:
        n_cat = int(explicit)
    elif family == Family.CATEGORICAL:
        n_cat = max(0, weights.ndim - 3)
    elif lowered["contribution_kind"] == "default":
        n_cat = max(0, weights.ndim - 2)
    else:
        n_cat = 0

    gathers = []
    for gslice in layout.flatten_slices(global_inds, global_slices):
        arr = np.asarray(gslice, dtype=np.int32)
        if arr.shape != (n_nodes, n_terms):
            raise ValueError(f"gather slice shape {arr.shape} does not match ({n_nodes}, {n_terms})")
        gathers.append(arr)
    if len(gathers) < n_spin + n_cat:
        raise ValueError(
            f"too few gather slices: need at least {n_spin + n_cat} "
            f"(n_spin={n_spin} + n_categorical_sources={n_cat}), got {len(gathers)}"
        )
    return FusedInteractionSpec(
        weighted_mask=weighted_mask,
        gather_indices=tuple(gathers),
        n_spin=n_spin,
        n_categorical=n_cat,
        n_terms=n_terms,
        contribution_kind=lowered["contribution_kind"],
    )


def _build_fused_block_spec(program, block_index, block, family, block_global_start, total_nodes, layout):
    """tt_thrml/compiler.py:220-271."""
    n_nodes = len(block.nodes)
    n_categories = _get_n_categories(block, family)
    interactions = tuple(
        _build_interaction_spec(inter, active, ginds, gslices, family, n_nodes, layout)
        for inter, active, ginds, gslices in zip(
            program.per_block_interactions[block_index],
            program.per_block_interaction_active[block_index],
            program.per_block_interaction_global_inds[block_index],
            program.per_block_interaction_global_slices[block_index],
            strict=True,
        )
    )
    if family == Family.CATEGORICAL and interactions:
        n_categories = _infer_n_categories(interactions, n_categories)
    return FusedBlockSpec(block_index, family, n_nodes, n_categories, block_global_start, total_nodes, interactions)


def _infer_n_categories(interactions, default):
    """Category count from the weight shapes (tt_thrml/compiler.py:252-261)."""
    q = default
    for ispec in interactions:
        wm = ispec.weighted_mask
        if ispec.row_ptr is None:
            if wm.ndim >= 3:
                return int(wm.shape[2])
            if ispec.n_terms > 0:
                q = wm.shape[-1] // ispec.n_terms
        elif wm.ndim >= 2:
            return int(wm.shape[1])
    return q


@dataclass
class LoweredProgram:
    specs: tuple[FusedBlockSpec, ...]
    sampling_order: tuple[tuple[int, ...], ...]
    n_free_blocks: int
    total_nodes: int
    block_global_starts: tuple[int, ...]


def lower_program(program) -> LoweredProgram:
    """Lowers a thrml program (or a native table program) to block specs."""
    native = getattr(program, "tt_lower_blocks", None)
    gibbs_spec = program.gibbs_spec
    sampling_order = tuple(tuple(int(i) for i in g) for g in gibbs_spec.sampling_order)
    n_free = len(gibbs_spec.free_blocks)
    if callable(native):
        specs = tuple(native())
        starts = tuple(s.block_global_start for s in specs)
        total = specs[0].total_nodes if specs else 0
        return LoweredProgram(specs, sampling_order, n_free, total, starts)
    layout = _build_global_state_layout(gibbs_spec)
    specs = []
    for bi, block in enumerate(gibbs_spec.blocks):
        family = _infer_family(block, gibbs_spec)
        if bi < n_free:
            specs.append(
                _build_fused_block_spec(
                    program, bi, block, family, layout.block_starts[bi], layout.total_nodes, layout
                )
            )
        else:
            specs.append(
                FusedBlockSpec(bi, family, len(block.nodes), None, layout.block_starts[bi], layout.total_nodes, ())
            )
    return LoweredProgram(tuple(specs), sampling_order, n_free, layout.total_nodes, layout.block_starts)


# --------------------------------------------------------------------------
# Planning: block specs -> device tables + kernel choice per group.
# --------------------------------------------------------------------------

_FAMILY_CODE = {Family.SPIN: nat.SPIN, Family.CATEGORICAL: nat.CATEGORICAL, Family.GAUSSIAN: nat.GAUSSIAN}


def _torch():
    import torch

    return torch


def resolve_torch_device(device):
    torch = _torch()
    if device is None:
        return torch.device("cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
    if isinstance(device, torch.device):
        return device
    if isinstance(device, int):
        return torch.device("cuda", device)
    if isinstance(device, str):
        return torch.device(device)
    td = getattr(device, "torch_device", None)
    if td is not None:
        return td
    devs = getattr(device, "devices", None)
    if devs:
        return devs[0].torch_device
    raise TypeError(f"cannot interpret {device!r} as a CUDA device")


def _to_dev(arr: np.ndarray, device):
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(arr)).to(device)


def _cat_axes(spec: FusedBlockSpec, it: FusedInteractionSpec) -> tuple[int, tuple[int, ...]]:
    """(q_target, categorical source sizes) of an interaction's weight table."""
    wm = np.asarray(it.weighted_mask)
    lead = 1 if it.row_ptr is not None else 2
    trailing = tuple(int(d) for d in wm.shape[lead:])
    if spec.family == Family.CATEGORICAL:
        q = int(spec.n_categories or 2)
        if not trailing or trailing[0] != q:
            raise ValueError(
                f"block {spec.block_index}: categorical weights need a category axis of size {q}, got {wm.shape}"
            )
        cat = trailing[1:]
        q_t = q
    else:
        cat = trailing
        q_t = 1
    if len(cat) != it.n_categorical:
        raise ValueError(
            f"block {spec.block_index}: weight shape {wm.shape} has {len(cat)} source axes, "
            f"n_categorical={it.n_categorical}"
        )
    if it.n_categorical > nat.MAX_CAT_SOURCES:
        raise ValueError(f"at most {nat.MAX_CAT_SOURCES} categorical sources per interaction are supported")
    return q_t, cat


@dataclass
class GenericGroupPlan:
    """Device tables of a group run by tthrml_group_step."""

    block_indices: tuple[int, ...]
    family_label: str
    in_place: bool
    group_rows: int
    interaction_tables: list  # keeps device tensors alive
    block_fields: list  # (family, q, n_inter, n_nodes, row_start, inter_desc_tensor)
    device: Any
    kind: str = "generic"
    _desc: Any = None
    _desc_variates: tuple = ()

    def descriptor(self, variates: dict | None, n_sweeps: int):
        """Device array of block descriptors (rebuilt when the variates change)."""
        key = tuple(
            (bi, 0 if variates is None or variates.get(bi) is None else variates[bi].data_ptr())
            for bi in self.block_indices
        )
        if self._desc is not None and self._desc_variates == key:
            return self._desc
        arr = (nat.BlockDesc * len(self.block_fields))()
        for k, (bi, (fam, q, n_inter, n_nodes, row_start, inter_t)) in enumerate(
            zip(self.block_indices, self.block_fields)
        ):
            d = arr[k]
            d.family, d.n_categories, d.n_interactions = fam, q, n_inter
            d.n_nodes, d.row_start = n_nodes, row_start
            d.interactions = inter_t.data_ptr() if inter_t is not None else None
            v = None if variates is None else variates.get(bi)
            d.variates = v.data_ptr() if v is not None else None
            d.variates_sweeps = n_sweeps if v is not None else 0
        torch = _torch()
        raw = torch.frombuffer(bytearray(bytes(arr)), dtype=torch.uint8)
        self._desc = raw.to(self.device)
        torch.cuda.synchronize(self.device)  # visible to kernels on any stream
        self._desc_variates = key
        return self._desc


@dataclass
class SpinCSRBlock:
    block_index: int
    row_start: int
    n_rows: int
    row_ptr: Any
    cols: Any
    vals: Any
    bias: Any
    nnz: int
    # rows in processing order for the bit-packed kernel: sorted by degree, so the two rows a warp
    # handles together need equally many neighbour terms (the order does not change any sample)
    row_order: Any = None


@dataclass
class SpinCSRGroupPlan:
    """Device tables of a group of spin blocks run by tthrml_spin_csr_step."""

    block_indices: tuple[int, ...]
    blocks: list[SpinCSRBlock]
    family_label: str = "spin"
    kind: str = "spin_csr"
    in_place: bool = True
    group_rows: int = 0
    device: Any = None


def _ragged_tables(spec: FusedBlockSpec):
    out = []
    for it in spec.interactions:
        rp, w, src = it.ragged(spec.n_nodes)
        out.append((it, rp, w, src))
    return out


def _validate_sources(spec: FusedBlockSpec, tables, total_nodes: int) -> None:
    for it, rp, w, src in tables:
        if rp.shape != (spec.n_nodes + 1,) or rp[0] != 0 or (np.diff(rp) < 0).any():
            raise ValueError(f"block {spec.block_index}: malformed term offsets")
        if src.size and (src.min() < 0 or src.max() >= total_nodes):
            raise ValueError(f"block {spec.block_index}: gather index outside the {total_nodes}-row state")
        if w.shape[0] != rp[-1]:
            raise ValueError(f"block {spec.block_index}: {w.shape[0]} weight rows for {rp[-1]} terms")


def _group_reads_itself(specs, tables_by_block, total_nodes: int) -> bool:
    """True when a term with a non-zero weight reads a row of the group (the superblock then needs
    staging).  Masked terms (all weights zero, e.g. the padding of an interaction's term axis) add an
    exact zero whatever the state holds, so where they point does not matter."""
    inside = np.zeros(total_nodes, dtype=bool)
    for s in specs:
        inside[s.block_global_start : s.block_global_start + s.n_nodes] = True
    for s in specs:
        for it, rp, w, src in tables_by_block[s.block_index]:
            if not src.size:
                continue
            live = np.any(w != 0.0, axis=1)  # per term
            if (inside[src] & live[None, :]).any():
                return True
    return False


def _spin_csr_eligible(specs, tables_by_block, state_dtype: str, n_chains: int) -> bool:
    if state_dtype != "int8" or n_chains % 32:
        return False
    for s in specs:
        if s.family != Family.SPIN:
            return False
        n_bias = n_pair = 0
        for it, rp, w, src in tables_by_block[s.block_index]:
            if it.n_categorical or w.shape[1] != 1:
                return False
            if src.shape[0] == 0:
                n_bias += 1
            elif src.shape[0] == 1:
                n_pair += 1
            else:
                return False
        if n_bias + n_pair == 0:
            return False
    return True


def _sequential_row_sum(rp: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Per-row float32 sum of terms in order (the bias of a spin block)."""
    n = rp.shape[0] - 1
    counts = np.diff(rp)
    out = np.zeros(n, dtype=np.float32)
    if n == 0:
        return out
    vals = w[:, 0].astype(np.float32)
    maxc = int(counts.max()) if n else 0
    first = True
    for t in range(maxc):
        has = counts > t
        idx = rp[:-1][has] + t
        if first:
            out[has] = vals[idx]
            first = False
        else:
            out[has] = (out[has] + vals[idx]).astype(np.float32)
    return out


def _merge_rows(parts, n_rows: int):
    """Concatenates per-row term lists [(row_ptr, vals, cols), ...] row by row, in the given order."""
    counts = sum(np.diff(rp) for rp, _, _ in parts)
    rp_out = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
    vals = np.empty(int(rp_out[-1]), dtype=np.float32)
    cols = np.empty(int(rp_out[-1]), dtype=np.int32)
    fill = rp_out[:-1].copy()
    for rp, v, c in parts:
        cnt = np.diff(rp)
        dst = np.repeat(fill, cnt) + (np.arange(int(rp[-1]), dtype=np.int64) - np.repeat(rp[:-1], cnt))
        vals[dst], cols[dst] = v, c
        fill += cnt
    return rp_out, vals, cols


def _plan_spin_csr(group, specs, tables_by_block, device) -> SpinCSRGroupPlan:
    """Sparse spin plan.  A block's bias interactions collapse into one per-row bias and its pair
    interactions into one CSR row per node (terms in program order): with one of each the field is the
    reference's float32 sum exactly; with several (thrml's IsingEBM gives a block two pair interactions,
    one per edge side) the grouping of the sum differs by rounding only."""
    blocks = []
    for s in specs:
        bias = None
        pairs = []
        for it, rp, w, src in tables_by_block[s.block_index]:
            if src.shape[0] == 0:
                b = _sequential_row_sum(rp, w)
                bias = b if bias is None else (bias + b).astype(np.float32)
            else:
                pairs.append((rp, w[:, 0], src[0]))
        pair = None
        if len(pairs) == 1:
            pair = pairs[0]
        elif pairs:
            pair = _merge_rows(pairs, s.n_nodes)
        if pair is None:
            rp = np.zeros(s.n_nodes + 1, dtype=np.int64)
            cols = np.zeros(1, dtype=np.int32)
            vals = np.zeros(1, dtype=np.float32)
        else:
            rp, vals, cols = pair
            keep = vals != 0.0
            if not keep.all():
                # masked terms add +-0 to the field: dropping them is exact
                row_of_term = np.repeat(np.arange(s.n_nodes, dtype=np.int64), np.diff(rp))
                counts = np.bincount(row_of_term[keep], minlength=s.n_nodes)
                rp = np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)
                vals, cols = vals[keep], cols[keep]
            if len(vals) == 0:
                cols = np.zeros(1, dtype=np.int32)
                vals = np.zeros(1, dtype=np.float32)
        blocks.append(
            SpinCSRBlock(
                block_index=s.block_index,
                row_start=s.block_global_start,
                n_rows=s.n_nodes,
                row_ptr=_to_dev(rp.astype(np.int64), device),
                cols=_to_dev(cols.astype(np.int32), device),
                vals=_to_dev(vals.astype(np.float32), device),
                bias=None if bias is None else _to_dev(bias, device),
                nnz=int(rp[-1]),
                row_order=_to_dev(np.argsort(np.diff(rp), kind="stable").astype(np.int32), device),
            )
        )
    return SpinCSRGroupPlan(
        block_indices=tuple(group), blocks=blocks, group_rows=sum(s.n_nodes for s in specs), device=device
    )


def _plan_generic(group, specs, tables_by_block, in_place: bool, device) -> GenericGroupPlan:
    torch = _torch()
    keep = []
    fields = []
    for s in specs:
        if s.family == Family.CATEGORICAL and int(s.n_categories or 2) > nat.MAX_CATEGORIES:
            raise ValueError(f"at most {nat.MAX_CATEGORIES} categories are supported")
        descs = (nat.Interaction * max(1, len(s.interactions)))()
        for k, (it, rp, w, src) in enumerate(tables_by_block[s.block_index]):
            q_t, cat = _cat_axes(s, it)
            rp_d, w_d, src_d = _to_dev(rp, device), _to_dev(w.astype(np.float32), device), _to_dev(src, device)
            keep += [rp_d, w_d, src_d]
            d = descs[k]
            d.row_ptr, d.weights, d.sources = rp_d.data_ptr(), w_d.data_ptr(), src_d.data_ptr()
            d.nnz = int(rp[-1])
            d.n_sources = int(src.shape[0])
            d.n_categorical = int(it.n_categorical)
            d.kind = nat.KIND_PRECISION if it.contribution_kind == "precision" else nat.KIND_LINEAR
            d.w_inner = int(w.shape[1])
            for j, qj in enumerate(cat):
                d.cat_q[j] = int(qj)
            if d.n_sources < d.n_categorical:
                raise ValueError(f"block {s.block_index}: fewer sources than categorical sources")
            if d.w_inner != q_t * int(np.prod(cat, dtype=np.int64)):
                raise ValueError(f"block {s.block_index}: weight inner size mismatch")
        if s.family in (Family.SPIN, Family.CATEGORICAL) and not s.interactions:
            raise ValueError("Block has no interactions; cannot build kernel")
        inter_t = torch.frombuffer(bytearray(bytes(descs)), dtype=torch.uint8).to(device)
        keep.append(inter_t)
        q = int(s.n_categories or 2) if s.family == Family.CATEGORICAL else 1
        fields.append((_FAMILY_CODE[s.family], q, len(s.interactions), s.n_nodes, s.block_global_start, inter_t))
    label = "+".join(s.family.value for s in specs)
    return GenericGroupPlan(
        block_indices=tuple(group),
        family_label=label,
        in_place=in_place,
        group_rows=sum(s.n_nodes for s in specs),
        interaction_tables=keep,
        block_fields=fields,
        device=device,
    )


def choose_state_dtype(specs) -> str:
    for s in specs:
        if s.family == Family.GAUSSIAN:
            return "float32"
        if s.family == Family.CATEGORICAL and int(s.n_categories or 2) > 127:
            return "float32"
    return "int8"


def plan_program(
    lowered: LoweredProgram, n_chains: int, device, *, force_generic: bool = False, spin_layout: str = "auto"
):
    """Builds the per-group device plans of a lowered program.

    Returns (state dtype, plans).  Programs whose every group runs on the
    sparse spin kernel keep their state bit-packed ("bits") when the chain
    count is a multiple of 256 and spin_layout allows it.
    """
    specs = lowered.specs
    state_dtype = choose_state_dtype(specs[: lowered.n_free_blocks])
    tables = {}
    for s in specs[: lowered.n_free_blocks]:
        t = _ragged_tables(s)
        _validate_sources(s, t, lowered.total_nodes)
        tables[s.block_index] = t
    plans = []
    for group in lowered.sampling_order:
        gspecs = [specs[i] for i in group]
        for s in gspecs:
            if s.block_index >= lowered.n_free_blocks:
                raise ValueError(f"sampling group {group} contains clamped block {s.block_index}")
        reads_itself = _group_reads_itself(gspecs, tables, lowered.total_nodes)
        if not force_generic and not reads_itself and _spin_csr_eligible(gspecs, tables, state_dtype, n_chains):
            plans.append(_plan_spin_csr(group, gspecs, tables, device))
        else:
            plans.append(_plan_generic(group, gspecs, tables, not reads_itself, device))
    if (
        spin_layout in ("auto", "bits")
        and plans
        and all(p.kind == "spin_csr" for p in plans)
        and n_chains % 256 == 0
    ):
        state_dtype = "bits"
        for p in plans:
            p.kind = "spin_bits"
    elif spin_layout == "bits":
        raise ValueError("spin_layout='bits' needs an all-spin program on the sparse kernel and n_chains % 256 == 0")
    return state_dtype, plans


@dataclass
class DenseGroupPlan:
    """A block whose field is one dense GEMM over the chain batch (tthrml_dense_field_sample)."""

    block_indices: tuple[int, ...]
    source: int
    family: Family
    n_units: int
    n_sources: int
    row0: int
    precision: float
    weights_nk: Any  # bf16 [n_units][source_pieces * n_sources] device tensor (K-repeated per piece)
    bias: Any  # float32 [n_units] device tensor
    source_pieces: int = 1  # bf16 pieces per source value in the source block's state
    out_pieces: int = 1  # bf16 pieces per value written for the target block
    family_label: str = ""
    kind: str = "dense"
    in_place: bool = True
    group_rows: int = 0
    device: Any = None
    rng_layout: str = "row4"  # Philox counter (chain, row / 4, sweep), word row % 4


DENSE_CHAIN_MULTIPLE = 128
DENSE_UNIT_MULTIPLE = 256


def dense_eligible(program, n_chains: int) -> bool:
    """True when the program lowers to the tensor-core dense plan at this chain count."""
    couplings = getattr(program, "tt_dense_couplings", None)
    if not callable(couplings) or n_chains % DENSE_CHAIN_MULTIPLE:
        return False
    gs = program.gibbs_spec
    if gs.clamped_blocks or any(len(g) != 1 for g in gs.sampling_order):
        return False
    for bi, c in couplings().items():
        if c["n_units"] % DENSE_UNIT_MULTIPLE or Family(c["family"]) not in (Family.SPIN, Family.GAUSSIAN):
            return False
    return True


def dense_pieces(program, precision: str) -> dict[int, int]:
    """bf16 pieces per value of each block's state: 3 for gaussian blocks at fp32, else 1."""
    return _pieces_of(program.tt_dense_couplings(), precision)


def _pieces_of(couplings: dict, precision: str) -> dict[int, int]:
    return {
        bi: 3 if precision == "fp32" and Family(c["family"]) == Family.GAUSSIAN else 1 for bi, c in couplings.items()
    }


def detect_dense_couplings(lowered: LoweredProgram, n_chains: int, round_weights: bool = False):
    """Dense bipartite structure found in lowered tables, as tt_dense_couplings() would give it, or None.

    Two free blocks sampled one per group, spin or gaussian, where every node of
    a block has exactly one pair term per node of the other block, in row order
    (per-node weight rows over a whole block: the RBM case of
    tt_thrml/compiler.py:173-176), plus one-term bias interactions and, for
    gaussian blocks, a precision that is the same for every node.  This is how
    an RBM written with thrml factors reaches the tensor-core kernel.  The
    weights must be bf16-representable unless round_weights is set.
    """
    if len(lowered.specs) != 2 or lowered.n_free_blocks != 2 or n_chains % DENSE_CHAIN_MULTIPLE:
        return None
    if sorted(lowered.sampling_order) != [(0,), (1,)]:
        return None
    out = {}
    for bi, spec in enumerate(lowered.specs):
        other = lowered.specs[1 - bi]
        if spec.family not in (Family.SPIN, Family.GAUSSIAN) or spec.n_nodes % DENSE_UNIT_MULTIPLE:
            return None
        n, m = spec.n_nodes, other.n_nodes
        bias = np.zeros(n, dtype=np.float32)
        precision = None
        pair = None
        for it in spec.interactions:
            if it.n_categorical:
                return None
            rp, w, src = it.ragged(n)
            if src.shape[0] == 0:  # one constant term per node
                if w.shape[1] != 1 or not np.array_equal(np.diff(rp), np.ones(n, np.int64)):
                    return None
                if it.contribution_kind == "precision":
                    if spec.family != Family.GAUSSIAN or not np.all(w[:, 0] == w[0, 0]):
                        return None
                    precision = np.float32(w[0, 0]) if precision is None else np.float32(precision + w[0, 0])
                else:
                    bias = (bias + w[:, 0]).astype(np.float32)
            elif src.shape[0] == 1 and it.contribution_kind != "precision" and pair is None:
                if w.shape[1] != 1 or not np.array_equal(np.diff(rp), np.full(n, m, np.int64)):
                    return None
                rows = np.arange(other.block_global_start, other.block_global_start + m, dtype=np.int32)
                if not np.array_equal(src[0], np.tile(rows, n)):
                    return None
                pair = w[:, 0].reshape(n, m)
            else:
                return None
        if pair is None:
            return None
        pair = np.ascontiguousarray(pair, dtype=np.float32)
        rounded = _bf16_round(pair)
        if not round_weights and not np.array_equal(rounded, pair):
            return None
        out[bi] = {"family": spec.family, "row0": spec.block_global_start, "n_units": n, "source": 1 - bi,
                   "weights_nk": rounded, "bias": bias, "precision": 1.0 if precision is None else float(precision)}
    return out


def _bf16_round(x: np.ndarray) -> np.ndarray:
    torch = _torch()
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(torch.bfloat16).float().numpy()


def _plan_dense(program, device, precision: str = "bf16"):
    return _plan_dense_couplings(program.tt_dense_couplings(), program.gibbs_spec.sampling_order, device, precision)


def _plan_dense_couplings(couplings: dict, sampling_order, device, precision: str = "bf16"):
    torch = _torch()
    pieces = _pieces_of(couplings, precision)
    plans = []
    for group in sampling_order:
        bi = int(group[0])
        c = couplings[bi]
        w = np.ascontiguousarray(c["weights_nk"], dtype=np.float32)
        wt = torch.from_numpy(w).to(device=device, dtype=torch.bfloat16).contiguous()
        if not torch.equal(wt.float().cpu(), torch.from_numpy(w)):
            raise ValueError(
                f"block {bi}: dense couplings must be bf16-representable (round them with "
                "workloads.bf16_representable) so the tensor-core operands are the model's weights"
            )
        fam = Family(c["family"])
        src_pieces = pieces[int(c["source"])]
        if src_pieces > 1:
            wt = wt.repeat(1, src_pieces).contiguous()
        plans.append(
            DenseGroupPlan(
                block_indices=(bi,),
                source=int(c["source"]),
                family=fam,
                n_units=int(c["n_units"]),
                n_sources=int(w.shape[1]) * src_pieces,
                row0=int(c["row0"]),
                precision=float(c.get("precision", 1.0)),
                weights_nk=wt,
                source_pieces=src_pieces,
                out_pieces=pieces[bi],
                bias=torch.from_numpy(np.asarray(c["bias"], np.float32)).to(device),
                family_label=fam.value,
                group_rows=int(c["n_units"]),
                device=device,
            )
        )
    return plans


def _dense_specs(program):
    """Light block specs (no tables) of a dense program: family, size, flat start."""
    couplings = program.tt_dense_couplings()
    blocks = program.gibbs_spec.blocks
    total = sum(len(b.nodes) for b in blocks)
    return tuple(
        FusedBlockSpec(bi, Family(couplings[bi]["family"]), len(b.nodes), None, int(couplings[bi]["row0"]), total, ())
        for bi, b in enumerate(blocks)
    )


@dataclass
class PottsStencilGroupPlan:
    """One checkerboard colour of a 3-D Potts lattice (tthrml_potts3d_step)."""

    block_indices: tuple[int, ...]
    dims: tuple[int, int, int]
    colour: int
    q: int
    target_row0: int
    source_row0: int
    J: Any  # float32 [3][q][q] device tensor
    bias: Any  # float32 [n_rows][q] device tensor (target block rows)
    bias_w: Any = None  # float32 [n_rows][8] e^(b - max b) per site (q = 8), made by the executor
    family: Family = Family.CATEGORICAL
    family_label: str = "categorical"
    kind: str = "potts3d"
    in_place: bool = True
    group_rows: int = 0
    device: Any = None


POTTS_MAX_Q = 8


@dataclass
class IsingResidentGroupPlan:
    """One checkerboard colour of a small 2-D Ising lattice with many chains (tthrml_ising2d_resident)."""

    block_indices: tuple[int, ...]
    dims: tuple[int, int]
    colour: int
    block_rows: tuple[int, int]
    thresholds: Any  # uint32 [16] device tensor
    family: Family = Family.SPIN
    family_label: str = "spin"
    kind: str = "ising2d_resident"
    in_place: bool = True
    group_rows: int = 0
    device: Any = None
    # Philox draws: "planes8" (bit-sliced kernel, count-symmetric tables and width % 8 == 0) or the split
    # uniforms "chain8s" (16 bits of counter (chain / 8, row, sweep, "LSPI") + 7 refill bits)
    rng_layout: str = "chain8s"


@dataclass
class IsingStencilGroupPlan:
    """One checkerboard colour of a single-chain 2-D Ising lattice (tthrml_ising2d_halfsweep)."""

    block_indices: tuple[int, ...]
    dims: tuple[int, int]
    colour: int
    target_row0: int
    source_row0: int
    thresholds: Any  # uint32 [16] device tensor (Philox mode)
    fields: Any  # float32 [16] device tensor (variates mode)
    family: Family = Family.SPIN
    family_label: str = "spin"
    kind: str = "ising2d"
    in_place: bool = True
    group_rows: int = 0
    device: Any = None
    # Philox draws: "planes" (bit-sliced kernel, count-symmetric tables) or the split uniforms "row8s"
    # (16 bits of counter (chain, row / 8, sweep, "LSPI") + 7 refill bits)
    rng_layout: str = "row8s"


def ising_pattern_tables(edge_weight, site_bias) -> tuple[np.ndarray, np.ndarray]:
    """(fields float32 [16], thresholds uint32 [16]) of a uniform lattice site.

    Pattern bit k (k = 0..3: left, right, up, down) set means neighbour k is
    -1.  field = b + (((w s_0 + w s_1) + w s_2) + w s_3) in float32 -- the
    bias interaction first, then the pair interaction summed over its terms
    (tt_thrml/compiler.py:303-318).  threshold = ceil((sigmoid(2 field) 2^24 -
    1) / 2): with u = (2m + 1) / 2^24 the Philox uniform of the 23-bit draw
    m, u < sigmoid(2 field) exactly when m < threshold.
    """
    w, b = np.float32(edge_weight), np.float32(site_bias)
    fields = np.empty(16, np.float32)
    for idx in range(16):
        terms = [np.float32(-w) if (idx >> k) & 1 else w for k in range(4)]
        acc = terms[0]
        for t in terms[1:]:
            acc = np.float32(acc + t)
        fields[idx] = np.float32(b + acc)
    p = 1.0 / (1.0 + np.exp(-2.0 * fields.astype(np.float64)))
    thr = np.ceil((p * 2.0**24 - 1.0) / 2.0)
    return fields, np.clip(thr, 0, 2**23).astype(np.uint32)


def ising_count_symmetric(thresholds) -> bool:
    """True when the 16-entry threshold table depends only on the number of -1
    neighbours (uniform couplings: the bit-sliced lattice kernels apply)."""
    thr = np.asarray(thresholds).astype(np.int64)
    by_count = {}
    for idx in range(16):
        by_count.setdefault(bin(idx).count("1"), set()).add(int(thr[idx]))
    return all(len(v) == 1 for v in by_count.values())


def ising_stencil_layout(thresholds, width: int) -> str:
    """Philox layout of the single-chain lattice kernel: "planes" (bit-sliced
    over 32 sites) for count-symmetric tables and width % 64 == 0, else the
    split uniforms "row8s"."""
    return "planes" if width % 64 == 0 and ising_count_symmetric(thresholds) else "row8s"


RESIDENT_MAX_SITES = 96 * 1024  # one byte per site of 8 chains in a CTA's shared memory


def stencil_eligible(program, n_chains: int, rng_mode: str = "philox") -> bool:
    """True when the program is a lattice the stencil kernels run at this chain count."""
    stencil = getattr(program, "tt_stencil", None)
    if not callable(stencil):
        return False
    st = stencil()
    if st.get("kind") == "potts3d":
        return 1 <= int(st["q"]) <= POTTS_MAX_Q and n_chains % 4 == 0
    if st.get("kind") == "ising2d":
        H, W = st["dims"]
        if n_chains == 1:
            return W % 32 == 0 and H % 2 == 0
        return resident_eligible(st, n_chains, rng_mode)
    return False


def resident_eligible(st: dict, n_chains: int, rng_mode: str) -> bool:
    """Small 2-D lattices with many chains run shared-memory resident (Philox mode, chains % 32 == 0)."""
    H, W = st["dims"]
    return rng_mode == "philox" and n_chains % 32 == 0 and H * W <= RESIDENT_MAX_SITES


def _plan_stencil(program, device, n_chains: int = 1):
    torch = _torch()
    st = program.tt_stencil()
    if st["kind"] == "ising2d" and n_chains > 1:
        _, thr = ising_pattern_tables(st["edge_weight"], st["site_bias"])
        t_dev = torch.from_numpy(thr.view(np.int32)).to(device)
        H, W = st["dims"]
        rows = tuple(int(r) for r in st["block_rows"])
        layout = "planes8" if W % 8 == 0 and all(r % 4 == 0 for r in rows) and ising_count_symmetric(thr) \
            else "chain8s"
        return [
            IsingResidentGroupPlan(
                block_indices=(int(g[0]),), dims=(int(H), int(W)), colour=int(g[0]), block_rows=rows,
                thresholds=t_dev, group_rows=H * W // 2, device=device, rng_layout=layout,
            )
            for g in program.gibbs_spec.sampling_order
        ]
    if st["kind"] == "ising2d":
        fields, thr = ising_pattern_tables(st["edge_weight"], st["site_bias"])
        f_dev = torch.from_numpy(fields).to(device)
        t_dev = torch.from_numpy(thr.view(np.int32)).to(device)
        rows = st["block_rows"]
        H, W = st["dims"]
        layout = ising_stencil_layout(thr, int(W))
        return [
            IsingStencilGroupPlan(
                block_indices=(int(g[0]),), dims=(int(H), int(W)), colour=int(g[0]), target_row0=int(rows[int(g[0])]),
                source_row0=int(rows[1 - int(g[0])]), thresholds=t_dev, fields=f_dev, group_rows=H * W // 2,
                device=device, rng_layout=layout,
            )
            for g in program.gibbs_spec.sampling_order
        ]
    if st["kind"] != "potts3d":
        raise ValueError(f"unknown stencil kind {st['kind']!r}")
    J = torch.from_numpy(np.ascontiguousarray(st["J"], dtype=np.float32)).to(device)
    rows = st["block_rows"]
    plans = []
    for group in program.gibbs_spec.sampling_order:
        c = int(group[0])
        bias = torch.from_numpy(np.ascontiguousarray(st["bias"][c], dtype=np.float32)).to(device)
        plans.append(
            PottsStencilGroupPlan(
                block_indices=(c,), dims=tuple(int(d) for d in st["dims"]), colour=c, q=int(st["q"]),
                target_row0=int(rows[c]), source_row0=int(rows[1 - c]), J=J, bias=bias,
                group_rows=int(bias.shape[0]), device=device,
            )
        )
    return plans


def detect_ising_lattice(lowered) -> dict | None:
    """The stencil description of a lowered program that is a periodic 2-D Ising lattice, else None.

    A thrml program of a lattice (e.g. an IsingEBM over an H x W grid with periodic edges) lowers to
    per-term tables; the stencil kernels run it when: two free spin blocks of n/2 nodes, block 0 the
    colour-0 sites (x + y even) in row-major order and block 1 the colour-1 sites, one sampling group
    each; every node with a bias (the same value everywhere) and exactly four non-zero pair terms of one
    common weight whose sources are its four lattice neighbours.  Then the field of every node is
    bias + weight * (sum of the neighbours' spins), which is what the stencil tables hold (the float32
    grouping of the sum may differ from the lowered program's by rounding, inside the threshold band)."""
    specs = lowered.specs
    if lowered.n_free_blocks != 2 or len(specs) != 2 or any(s.family != Family.SPIN for s in specs):
        return None
    half = specs[0].n_nodes
    if specs[1].n_nodes != half or specs[0].block_global_start != 0 or specs[1].block_global_start != half:
        return None
    if sorted(tuple(int(i) for i in g) for g in lowered.sampling_order) != [(0,), (1,)]:
        return None
    n = 2 * half
    biases, nbrs, weights = [], [], []
    for s in specs:
        bias = np.zeros(half, dtype=np.float32)
        pairs = []
        for it, rp, w, src in _ragged_tables(s):
            if it.n_categorical or w.shape[1] != 1 or src.shape[0] > 1:
                return None
            if src.shape[0] == 0:
                bias = (bias + _sequential_row_sum(rp, w)).astype(np.float32)
            else:
                pairs.append((rp, w[:, 0], src[0]))
        if not pairs:
            return None
        rp, vals, cols = _merge_rows(pairs, half) if len(pairs) > 1 else pairs[0]
        keep = vals != 0.0
        row_of = np.repeat(np.arange(half, dtype=np.int64), np.diff(rp))[keep]
        if not (np.bincount(row_of, minlength=half) == 4).all():
            return None
        v = vals[keep]
        if not (v == v[0]).all():
            return None
        weights.append(v[0])
        biases.append(bias)
        nbrs.append(np.sort(cols[keep].astype(np.int64).reshape(half, 4), axis=1))
    if weights[0] != weights[1] or not (biases[0] == biases[0][0]).all() or not (biases[1] == biases[0][0]).all():
        return None
    # block-0 row 0 is site (0, 0): its neighbours sit at block-1 rows {0, W/2 - 1, W/2, (H - 1) W / 2}
    W = 2 * int(nbrs[0][0][2] - half)
    if W < 4 or n % W or (n // W) < 4 or (n // W) % 2:
        return None
    H = n // W
    for c in range(2):
        r = np.arange(half, dtype=np.int64)
        y = (2 * r) // W
        x = (2 * r) % W + ((y + c) & 1)
        L = np.stack([y * W + (x - 1) % W, y * W + (x + 1) % W, ((y - 1) % H) * W + x, ((y + 1) % H) * W + x], 1)
        if not np.array_equal(np.sort((1 - c) * half + L // 2, axis=1), nbrs[c]):
            return None
    return {"kind": "ising2d", "dims": (H, W), "edge_weight": np.float32(weights[0]),
            "site_bias": np.float32(biases[0][0]), "block_rows": (0, half)}


def _potts_geometry(dims, half: int):
    """Per colour c: (n/2, 6) flat rows of the neighbours (x-, x+, y-, y+, z-, z+) of block c's sites."""
    X, Y, Z = dims
    out = []
    for c in range(2):
        even = 2 * np.arange(half, dtype=np.int64)
        yy = (even // X) % Y
        zz = even // (X * Y)
        L = even + ((yy + zz + c) & 1)
        x, y, z = L % X, (L // X) % Y, L // (X * Y)
        nb = [(((z + dz) % Z) * Y + (y + dy) % Y) * X + (x + dx) % X
              for dx, dy, dz in ((-1, 0, 0), (1, 0, 0), (0, -1, 0), (0, 1, 0), (0, 0, -1), (0, 0, 1))]
        out.append((1 - c) * half + np.stack(nb, axis=1) // 2)
    return out


def detect_potts_lattice(lowered) -> dict | None:
    """The stencil description of a lowered program that is a periodic 3-D Potts lattice, else None.

    The counterpart of `detect_ising_lattice` for categorical programs (e.g. CategoricalEBMFactors over
    the x, y and z edges of a periodic grid): two free categorical blocks of n/2 nodes with q <= 8, block
    c the colour-c sites (x + y + z = c mod 2) in row-major order, one sampling group each; per node a
    bias q-vector (any values) and exactly six pair terms with one categorical source each, whose
    sources are its six lattice neighbours and whose q x q matrices are one matrix per axis, the same for
    both directions and for every node."""
    specs = lowered.specs
    if lowered.n_free_blocks != 2 or len(specs) != 2 or any(s.family != Family.CATEGORICAL for s in specs):
        return None
    q = int(specs[0].n_categories or 2)
    half = specs[0].n_nodes
    if int(specs[1].n_categories or 2) != q or not 1 <= q <= POTTS_MAX_Q or specs[1].n_nodes != half:
        return None
    if specs[0].block_global_start != 0 or specs[1].block_global_start != half:
        return None
    if sorted(tuple(int(i) for i in g) for g in lowered.sampling_order) != [(0,), (1,)]:
        return None
    n = 2 * half
    biases, srcs, mats = [], [], []
    for s in specs:
        bias = np.zeros((half, q), dtype=np.float32)
        parts = []
        for it in s.interactions:
            rp, w, src = it.ragged(s.n_nodes)
            if src.shape[0] == 0 and it.n_categorical == 0 and w.shape[1] == q:
                for t in range(int(np.diff(rp).max()) if half else 0):
                    has = np.diff(rp) > t
                    bias[has] = (bias[has] + w[rp[:-1][has] + t]).astype(np.float32)
            elif src.shape[0] == 1 and it.n_categorical == 1 and w.shape[1] == q * q:
                parts.append((rp, w, src[0]))
            else:
                return None
        if not parts:
            return None
        counts = sum(np.diff(rp) for rp, _, _ in parts)
        rows = np.concatenate([np.repeat(np.arange(half), np.diff(rp)) for rp, _, _ in parts])
        ws = np.concatenate([w for _, w, _ in parts])
        cs = np.concatenate([c for _, _, c in parts]).astype(np.int64)
        live = np.any(ws != 0.0, axis=1)
        if not (np.bincount(rows[live], minlength=half) == 6).all():
            return None
        order = np.argsort(rows[live], kind="stable")
        biases.append(bias)
        srcs.append(cs[live][order].reshape(half, 6))
        mats.append(ws[live][order].reshape(half, 6, q, q))
    # dims from site (0, 0, 0) = block-0 row 0: its neighbour rows in block 1 hold X/2 - 1 and X/2
    r0 = set((srcs[0][0] - half).tolist())
    for X in sorted(2 * (r + 1) for r in r0 if r + 1 in r0):
        for r in sorted(r0):
            if r <= 0 or X < 4 or 2 * r % X or n % (2 * r) or 2 * r // X < 4:
                continue
            Y = 2 * r // X
            if n % (X * Y) or (n // (X * Y)) < 4 or (n // (X * Y)) % 2 or Y % 2:
                continue
            dims = (X, Y, n // (X * Y))
            geo = _potts_geometry(dims, half)
            if not all(np.array_equal(np.sort(geo[c], 1), np.sort(srcs[c], 1)) for c in range(2)):
                continue
            J = np.zeros((3, q, q), dtype=np.float32)
            for c in range(2):
                # which lattice direction each term points to
                d = np.argmax(srcs[c][:, :, None] == geo[c][:, None, :], axis=2)  # [half][term] -> direction
                for a in range(3):
                    for sgn in range(2):
                        sel = mats[c][d == 2 * a + sgn]
                        if not (sel == sel[0]).all():
                            return None
                        if c == 0 and sgn == 0:
                            J[a] = sel[0]
                        elif not np.array_equal(sel[0], J[a]):
                            return None
            return {"kind": "potts3d", "dims": dims, "q": q, "J": J, "bias": biases, "block_rows": (0, half)}
    return None


class _DetectedStencil:
    """A lowered program recognised as a lattice, seen through the stencil planner's interface."""

    def __init__(self, lowered, stencil: dict):
        from types import SimpleNamespace

        self.gibbs_spec = SimpleNamespace(sampling_order=[list(g) for g in lowered.sampling_order])
        self._stencil = stencil

    def tt_stencil(self) -> dict:
        return self._stencil


def _stencil_specs(program):
    """Light block specs (no tables) of a stencil program: family, size, flat start."""
    st = program.tt_stencil()
    blocks = program.gibbs_spec.blocks
    total = sum(len(b.nodes) for b in blocks)
    if st["kind"] == "ising2d":
        fam, q = Family.SPIN, None
    else:
        fam, q = Family.CATEGORICAL, int(st["q"])
    return tuple(
        FusedBlockSpec(bi, fam, len(b.nodes), q, int(st["block_rows"][bi]), total, ()) for bi, b in enumerate(blocks)
    )


# ---------------------------------------------------------------------------
# Plan cache (the counterpart of the reference's artifact cache,
# tt_thrml/compiler.py:398-433, 457-463): compiled plans -- the lowered
# program, the state layout and the group plans with their device tables --
# keyed by a SHA-256 signature of the program's contents plus the device, the
# chain count and the configuration fields that shape the plans.  A second
# executor (or a second `sample_states` call) over the same program reuses the
# tables instead of lowering and uploading them again.  Programs are taken as
# immutable once compiled, as thrml's are.  The cache holds device memory, so
# it keeps the most recent PLAN_CACHE_SIZE entries; `clear_plan_cache()` drops
# them.  Thread-safe.
# ---------------------------------------------------------------------------

PLAN_CACHE_SIZE = 8
_PLAN_CACHE_LOCK = threading.Lock()
_PLAN_CACHE: "OrderedDict[tuple, tuple]" = OrderedDict()  # key -> (lowered, state_dtype, plans)
_PROGRAM_SIGNATURES: dict = {}  # id(program) -> (weakref to program, signature, lowered or None)


def clear_plan_cache() -> None:
    with _PLAN_CACHE_LOCK:
        _PLAN_CACHE.clear()
        _PROGRAM_SIGNATURES.clear()


def plan_cache_size() -> int:
    with _PLAN_CACHE_LOCK:
        return len(_PLAN_CACHE)


def _hash_into(h, obj) -> None:
    torch = _torch()
    if isinstance(obj, torch.Tensor):
        obj = obj.detach().cpu().numpy()
    if isinstance(obj, np.ndarray) or isinstance(obj, np.generic):
        a = np.ascontiguousarray(obj)
        h.update(f"nd{a.dtype.str}{a.shape}".encode())
        h.update(a.tobytes())
    elif isinstance(obj, dict):
        h.update(b"{")
        for k in sorted(obj, key=str):
            h.update(str(k).encode())
            _hash_into(h, obj[k])
        h.update(b"}")
    elif isinstance(obj, (list, tuple)):
        h.update(b"[")
        for x in obj:
            _hash_into(h, x)
        h.update(b"]")
    elif isinstance(obj, Enum):
        h.update(repr(obj.value).encode())
    elif dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        h.update(type(obj).__name__.encode())
        for f in dataclasses.fields(obj):
            h.update(f.name.encode())
            _hash_into(h, getattr(obj, f.name))
    else:
        h.update(repr(obj).encode())


def _structure(program) -> list:
    gs = program.gibbs_spec
    return [[len(b.nodes) for b in gs.free_blocks], [len(b.nodes) for b in gs.clamped_blocks],
            [[int(i) for i in g] for g in gs.sampling_order]]


def program_signature(program) -> tuple[str, Any]:
    """(SHA-256 signature of the program's contents, its lowering when one was needed to compute it).

    Lattice programs are signed by their stencil description, dense bipartite programs by their
    coupling matrices, table programs by their tables and any other program (a thrml program) by its
    lowering, like the reference's kernel signature keys (tt_thrml/compiler.py:398-433)."""
    h = hashlib.sha256()
    lowered = None
    _hash_into(h, _structure(program))
    if callable(getattr(program, "tt_stencil", None)):
        h.update(b"stencil")
        _hash_into(h, program.tt_stencil())
    if callable(getattr(program, "tt_dense_couplings", None)):
        h.update(b"dense")
        _hash_into(h, program.tt_dense_couplings())
    elif callable(getattr(program, "tt_lower_blocks", None)) and not callable(getattr(program, "tt_stencil", None)):
        h.update(b"tables")
        _hash_into(h, list(program.tt_lower_blocks()))
    elif not callable(getattr(program, "tt_stencil", None)):
        lowered = lower_program(program)
        h.update(b"lowered")
        _hash_into(h, list(lowered.specs))
    return h.hexdigest(), lowered


def _signature_of(program) -> tuple[str, Any]:
    """program_signature, remembered per live program object (a repeated call does not lower again)."""
    with _PLAN_CACHE_LOCK:
        hit = _PROGRAM_SIGNATURES.get(id(program))
        if hit is not None and hit[0]() is program:
            return hit[1], hit[2]
    sig, lowered = program_signature(program)
    try:
        ref = weakref.ref(program)
    except TypeError:
        return sig, lowered
    with _PLAN_CACHE_LOCK:
        for k in [k for k, v in _PROGRAM_SIGNATURES.items() if v[0]() is None]:
            del _PROGRAM_SIGNATURES[k]
        _PROGRAM_SIGNATURES[id(program)] = (ref, sig, lowered)
    return sig, lowered


def _copy_plans(plans) -> list:
    """Per-executor plan objects sharing the cached device tables (descriptor caches stay private)."""
    out = []
    for p in plans:
        q = dataclasses.replace(p)
        if isinstance(q, GenericGroupPlan):
            q._desc, q._desc_variates = None, ()
        out.append(q)
    return out


def compile_program(
    ttnn,
    device,
    program,
    config: CUDAConfig,
    *,
    n_sweeps: int = 100,
    n_chains: int | None = None,
    force_generic: bool = False,
    cache: bool = True,
) -> CompiledProgram:
    """Compile a thrml program for the CUDA executor (tt_thrml/compiler.py:524-592).

    cache: reuse the plans (device tables) of an earlier compilation of a program with the same
    signature for the same device, chain count and configuration."""
    del ttnn
    n_chains = int(n_chains if n_chains is not None else config.n_chains)
    tdev = resolve_torch_device(device)
    key, pre_lowered = None, None
    if cache:
        sig, pre_lowered = _signature_of(program)
        key = (sig, tdev.type, tdev.index, n_chains, config.plan_key(), bool(force_generic))
        with _PLAN_CACHE_LOCK:
            hit = _PLAN_CACHE.get(key)
            if hit is not None:
                _PLAN_CACHE.move_to_end(key)
        if hit is not None:
            lowered, state_dtype, plans = hit
            return _assemble(lowered, state_dtype, _copy_plans(plans), n_sweeps, n_chains, tdev)
    lowered, state_dtype, plans = _build_plans(program, config, n_chains, tdev, force_generic, pre_lowered)
    if key is not None:
        with _PLAN_CACHE_LOCK:
            _PLAN_CACHE[key] = (lowered, state_dtype, plans)
            _PLAN_CACHE.move_to_end(key)
            while len(_PLAN_CACHE) > PLAN_CACHE_SIZE:
                _PLAN_CACHE.popitem(last=False)
        plans = _copy_plans(plans)
    return _assemble(lowered, state_dtype, plans, n_sweeps, n_chains, tdev)


def _build_plans(program, config: CUDAConfig, n_chains: int, tdev, force_generic: bool, pre_lowered=None):
    if not force_generic and config.stencil and stencil_eligible(program, n_chains, config.rng_mode):
        specs = _stencil_specs(program)
        order = tuple(tuple(int(i) for i in g) for g in program.gibbs_spec.sampling_order)
        lowered = LoweredProgram(specs, order, len(program.gibbs_spec.free_blocks), specs[0].total_nodes,
                                 tuple(s.block_global_start for s in specs))
        plans = _plan_stencil(program, tdev, n_chains)
        state_dtype = "bits" if plans[0].kind == "ising2d_resident" else "int8"
    elif not force_generic and dense_eligible(program, n_chains):
        specs = _dense_specs(program)
        order = tuple(tuple(int(i) for i in g) for g in program.gibbs_spec.sampling_order)
        lowered = LoweredProgram(specs, order, len(program.gibbs_spec.free_blocks), specs[0].total_nodes,
                                 tuple(s.block_global_start for s in specs))
        state_dtype, plans = "dense_bf16", _plan_dense(program, tdev, config.resolved_dense_precision)
    else:
        lowered = pre_lowered if pre_lowered is not None else lower_program(program)
        if not force_generic and config.stencil:
            st = detect_ising_lattice(lowered) or detect_potts_lattice(lowered)
            view = _DetectedStencil(lowered, st) if st is not None else None
            if view is not None and stencil_eligible(view, n_chains, config.rng_mode):
                plans = _plan_stencil(view, tdev, n_chains)
                _torch().cuda.synchronize(tdev)
                return lowered, ("bits" if plans[0].kind == "ising2d_resident" else "int8"), plans
        couplings = None
        if not force_generic and config.dense_detect and not callable(getattr(program, "tt_stencil", None)):
            couplings = detect_dense_couplings(lowered, n_chains, round_weights=config.dense_round_weights)
        if couplings is not None:
            state_dtype = "dense_bf16"
            plans = _plan_dense_couplings(couplings, lowered.sampling_order, tdev, config.resolved_dense_precision)
        else:
            state_dtype, plans = plan_program(
                lowered, n_chains, tdev, force_generic=force_generic, spin_layout=config.spin_layout
            )
    _torch().cuda.synchronize(tdev)  # tables uploaded before any stream uses them
    return lowered, state_dtype, plans


def _assemble(lowered, state_dtype, plans, n_sweeps: int, n_chains: int, tdev) -> CompiledProgram:
    blocks = tuple(CompiledFusedBlock(spec=s, kernel_artifact=None) for s in lowered.specs)
    groups = tuple(
        CompiledSamplingGroup(block_indices=tuple(g), kernel_artifact=p) for g, p in zip(lowered.sampling_order, plans)
    )
    rng_spec = make_rng_spec(blocks[: lowered.n_free_blocks], n_sweeps)
    return CompiledProgram(
        blocks=blocks,
        sampling_groups=groups,
        n_free_blocks=lowered.n_free_blocks,
        total_nodes=lowered.total_nodes,
        block_global_starts=lowered.block_global_starts,
        sampling_order=lowered.sampling_order,
        state_dtype=state_dtype,
        index_dtype="int32",
        layout="rows x chains",
        rng_spec=rng_spec,
        n_chains=n_chains,
        device=tdev,
    )


__all__ = [
    "compile_program",
    "clear_plan_cache",
    "plan_cache_size",
    "program_signature",
    "PLAN_CACHE_SIZE",
    "lower_program",
    "plan_program",
    "LoweredProgram",
    "GenericGroupPlan",
    "SpinCSRGroupPlan",
    "DenseGroupPlan",
    "PottsStencilGroupPlan",
    "IsingStencilGroupPlan",
    "IsingResidentGroupPlan",
    "detect_dense_couplings",
    "detect_ising_lattice",
    "detect_potts_lattice",
    "ising_pattern_tables",
]
