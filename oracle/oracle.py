"""CPU oracle for the block-Gibbs sweep path — TEST INFRASTRUCTURE ONLY.

Only tests, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg may
import this module, and only as the checker.  It restates the reference
algorithm independently of the product package:

* `lower_program` restates the reference's lowering of a thrml program to
  per-block tables (tt_thrml/compiler.py:39-271): flat block-ordered layout,
  family inference, interaction lowering, weighted masks, gather slices;
* `OracleSampler.group_step` runs one sampling group through the C
  restatement in oracle.c (tt_thrml/compiler.py:274-450), on a float32 state
  [rows, chains] like the reference's flat float32 global state
  (tt_thrml/executor.py:104-136) with a chain axis;
* `OracleSampler.sample_with_observation` follows the reference's schedule
  (tt_thrml/executor.py:367-409).

Parity status: pinned to the reference's own known-answer tests
(tests/test_compiler_lowering.py, scripts/probe_gather_pipeline.py of the
reference) through tests/golden; upstream thrml/JAX cannot run here, so
sample-level parity with upstream thrml itself is unpinned.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

SPIN, CATEGORICAL, GAUSSIAN = 0, 1, 2
_FAMILY = {"spin": SPIN, "categorical": CATEGORICAL, "gaussian": GAUSSIAN}


class _Inter(ctypes.Structure):
    _fields_ = [
        ("row_ptr", ctypes.c_void_p),
        ("weights", ctypes.c_void_p),
        ("sources", ctypes.c_void_p),
        ("nnz", ctypes.c_int64),
        ("n_sources", ctypes.c_int32),
        ("n_categorical", ctypes.c_int32),
        ("kind", ctypes.c_int32),
        ("w_inner", ctypes.c_int32),
        ("cat_q", ctypes.c_int32 * 4),
    ]


class _Block(ctypes.Structure):
    _fields_ = [
        ("family", ctypes.c_int32),
        ("q", ctypes.c_int32),
        ("n_interactions", ctypes.c_int32),
        ("rng_layout", ctypes.c_int32),
        ("n_nodes", ctypes.c_int64),
        ("row_start", ctypes.c_int64),
        ("inter", ctypes.c_void_p),
        ("variates", ctypes.c_void_p),
    ]


_lib = None


def build() -> Path:
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        _lib.oracle_group_step.restype = ctypes.c_int32
        _lib.oracle_group_step.argtypes = [
            ctypes.c_void_p,
            ctypes.c_int32,
            ctypes.c_void_p,
            ctypes.c_int64,
            ctypes.c_int64,
            ctypes.c_int32,
            ctypes.c_uint64,
            ctypes.c_uint32,
            ctypes.c_void_p,
            ctypes.c_int32,
        ]
        _lib.oracle_philox4x32_10.restype = None
        _lib.oracle_philox4x32_10.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        # (model, colour/block, state, C, chain_offset, variates, [rng_layout], seed, sweep, margin, threads)
        i64, i32, vp = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
        _lib.oracle_ising2d_step.restype = i32
        _lib.oracle_ising2d_step.argtypes = [vp, i32, vp, i64, i64, vp, i32, ctypes.c_uint64, ctypes.c_uint32, vp, i32]
        _lib.oracle_potts3d_step.restype = i32
        _lib.oracle_potts3d_step.argtypes = [vp, i32, vp, i64, i64, vp, ctypes.c_uint64, ctypes.c_uint32, vp, i32]
        _lib.oracle_dense_step.restype = i32
        _lib.oracle_dense_step.argtypes = [vp, i32, vp, i64, i64, vp, i32, ctypes.c_uint64, ctypes.c_uint32, vp, i32]
        _lib.oracle_greedy_colouring.restype = i32
        _lib.oracle_greedy_colouring.argtypes = [i64, vp, vp, vp, vp]
    return _lib


def philox4x32_10(ctr, key) -> np.ndarray:
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    out = np.zeros(4, dtype=np.uint32)
    lib().oracle_philox4x32_10(c.ctypes.data, k.ctypes.data, out.ctypes.data)
    return out


# ----------------------------------------------------------------------------
# Lowering restatement (tt_thrml/compiler.py:39-271).
# ----------------------------------------------------------------------------


@dataclass
class OInteraction:
    row_ptr: np.ndarray  # int64 [n+1]
    weights: np.ndarray  # float32 [nnz, inner]
    sources: np.ndarray  # int32 [n_sources, nnz]
    n_categorical: int
    kind: str  # "default" | "linear" | "precision"
    cat_q: tuple
    n_terms: int
    q_axis: int | None = None  # size of weight axis 2 of the dense table, when it has one


@dataclass
class OBlock:
    index: int
    family: str
    n_nodes: int
    q: int
    start: int
    interactions: list


@dataclass
class OProgram:
    blocks: list
    sampling_order: list
    n_free: int
    total: int
    model: object = None  # a model path of oracle/models.py (stencil / dense), or None for the table path


class Lattice2D(ctypes.Structure):
    _fields_ = [("height", ctypes.c_int64), ("width", ctypes.c_int64), ("edge_weight", ctypes.c_float),
                ("site_bias", ctypes.c_float)]


class Potts3D(ctypes.Structure):
    _fields_ = [("dims", ctypes.c_int64 * 3), ("q", ctypes.c_int32), ("J", ctypes.c_void_p), ("bias0", ctypes.c_void_p),
                ("bias1", ctypes.c_void_p)]


class Dense(ctypes.Structure):
    _fields_ = [("n_visible", ctypes.c_int64), ("n_hidden", ctypes.c_int64), ("W", ctypes.c_void_p),
                ("b_v", ctypes.c_void_p), ("b_h", ctypes.c_void_p), ("visible_family", ctypes.c_int32),
                ("store_bf16", ctypes.c_int32)]


def _family_of(block, gibbs_spec) -> str:
    fam = getattr(block, "family", None)
    if fam is not None:
        return getattr(fam, "value", fam)
    name = type(block.nodes[0]).__name__.lower()
    if "spin" in name or "bool" in name:
        return "spin"
    if "categorical" in name or "discrete" in name:
        return "categorical"
    if "gaussian" in name or "continuous" in name:
        return "gaussian"
    sds = getattr(gibbs_spec, "node_shape_dtypes", None) or {}
    sd = sds.get(type(block.nodes[0]))
    if sd is not None:
        kind = np.dtype(getattr(sd, "dtype", None) or sd[0][0].dtype).kind
        return {"b": "spin", "i": "categorical", "u": "categorical", "f": "gaussian"}.get(kind, "spin")
    return "spin"


def _lower_one(inter, family: str) -> dict:
    hook = getattr(inter, "tt_interaction_contribution", None)
    if callable(hook):
        c = hook(parameter_family=family)
        return dict(w=np.asarray(c.weights), n_spin=int(c.n_spin), n_cat=getattr(c, "n_categorical", None),
                    kind=str(getattr(c, "contribution_kind", "default")))
    if hasattr(inter, "n_spin") and hasattr(inter, "weights"):
        return dict(w=np.asarray(inter.weights), n_spin=int(inter.n_spin), n_cat=None, kind="default")
    if family == "gaussian":
        if hasattr(inter, "weights"):
            return dict(w=np.asarray(inter.weights), n_spin=0, n_cat=0, kind="linear")
        if hasattr(inter, "inverse_weights"):
            return dict(w=np.reciprocal(np.asarray(inter.inverse_weights, dtype=np.float32)), n_spin=0, n_cat=0,
                        kind="precision")
    raise TypeError(f"Cannot lower interaction of type {type(inter)}")


def layout_of(gibbs_spec):
    """(block_starts, global_to_flat, total) — literal per-node restatement."""
    starts, off = [], 0
    for b in gibbs_spec.blocks:
        starts.append(off)
        off += len(b.nodes)
    locmap = gibbs_spec.node_global_location_map
    g2f: dict[int, dict[int, int]] = {}
    for bi, b in enumerate(gibbs_spec.blocks):
        for k, node in enumerate(b.nodes):
            gi, go = locmap[node]
            g2f.setdefault(int(gi), {})[int(go)] = starts[bi] + k
    maps = []
    for gi in range(max(g2f) + 1 if g2f else 0):
        d = g2f.get(gi, {})
        size = max(d) + 1 if d else 0
        if len(d) != size:
            raise ValueError("THRML global state map is not dense.")
        maps.append(np.array([d[i] for i in range(size)], dtype=np.int64))
    return starts, maps, off


def _interaction(inter, active, ginds, gslices, family, n, maps) -> OInteraction:
    lo = _lower_one(inter, family)
    w = np.asarray(lo["w"], dtype=np.float32)
    mask = np.asarray(active, dtype=np.float32)
    if w.ndim == 1:
        w = w.reshape(n, -1)
    if mask.ndim == 1:
        mask = mask.reshape(n, -1)
    if w.shape[:2] == mask.shape:
        T = mask.shape[1]
        wm = (w * mask.reshape(mask.shape + (1,) * (w.ndim - 2))).astype(np.float32)
    elif w.shape == mask.shape:
        wm = (w * mask).astype(np.float32)
        T = wm.shape[-1]
    else:
        raise ValueError("weights/mask shape mismatch")
    if lo["n_cat"] is not None:
        n_cat = int(lo["n_cat"])
    elif family == "categorical":
        n_cat = max(0, w.ndim - 3)
    elif lo["kind"] == "default":
        n_cat = max(0, w.ndim - 2)
    else:
        n_cat = 0
    srcs = [maps[int(g)][np.asarray(s, dtype=np.int64)].astype(np.int32) for g, s in zip(ginds, gslices)]
    for s in srcs:
        if s.shape != (n, T):
            raise ValueError("gather slice shape mismatch")
    if len(srcs) < int(lo["n_spin"]) + n_cat:
        raise ValueError("too few gather slices")
    inner = wm.shape[2:]
    cat_q = tuple(int(d) for d in (inner[1:] if family == "categorical" else inner))
    return OInteraction(
        row_ptr=np.arange(n + 1, dtype=np.int64) * T,
        weights=np.ascontiguousarray(wm.reshape(n * T, -1)),
        sources=np.ascontiguousarray(np.stack(srcs).reshape(len(srcs), n * T) if srcs else np.zeros((0, n * T), np.int32)),
        n_categorical=n_cat,
        kind=lo["kind"],
        cat_q=cat_q,
        n_terms=T,
        q_axis=int(wm.shape[2]) if wm.ndim >= 3 else None,
    )


def _from_spec(spec) -> OBlock:
    """Block tables handed over as FusedBlockSpec-shaped data (native table programs)."""
    fam = getattr(spec.family, "value", spec.family)
    inters = []
    for it in spec.interactions:
        wm = np.asarray(it.weighted_mask, dtype=np.float32)
        if it.row_ptr is not None:
            rp = np.asarray(it.row_ptr, dtype=np.int64)
            nnz = int(rp[-1])
            inner = wm.shape[1:]
            w2 = wm.reshape(nnz, -1)
            src = np.stack([np.asarray(g, np.int32).reshape(nnz) for g in it.gather_indices]) if it.gather_indices \
                else np.zeros((0, nnz), np.int32)
        else:
            n, T = spec.n_nodes, int(it.n_terms)
            rp = np.arange(n + 1, dtype=np.int64) * T
            inner = wm.shape[2:]
            w2 = wm.reshape(n * T, -1)
            src = np.stack([np.asarray(g, np.int32).reshape(n * T) for g in it.gather_indices]) if it.gather_indices \
                else np.zeros((0, n * T), np.int32)
        cat_q = tuple(int(d) for d in (inner[1:] if fam == "categorical" else inner))
        inters.append(OInteraction(rp, np.ascontiguousarray(w2), np.ascontiguousarray(src), int(it.n_categorical),
                                   it.contribution_kind, cat_q, int(it.n_terms)))
    q = int(spec.n_categories or 2) if fam == "categorical" else 1
    return OBlock(spec.block_index, fam, spec.n_nodes, q, spec.block_global_start, inters)


def lower_program(program, *, tables: bool = False) -> OProgram:
    """The oracle's program.  Synthetic models (lattices, random graphs, RBMs) are built from their raw
    parameters by oracle/models.py (stencil / dense paths unless `tables`); a program given directly as
    block tables (a plain table program) is read as given; a thrml program is lowered as the reference
    lowers it."""
    from . import models

    own = models.from_raw_parameters(program, tables=tables)
    if own is not None:
        return own
    gs = program.gibbs_spec
    order = [list(map(int, g)) for g in gs.sampling_order]
    n_free = len(gs.free_blocks)
    specs = getattr(program, "specs", None)
    if isinstance(specs, (list, tuple)) and callable(getattr(program, "tt_lower_blocks", None)):
        blocks = [_from_spec(s) for s in specs]
        return OProgram(blocks, order, n_free, specs[0].total_nodes if specs else 0)
    starts, maps, total = layout_of(gs)
    blocks = []
    for bi, b in enumerate(gs.blocks):
        fam = _family_of(b, gs)
        n = len(b.nodes)
        inters = []
        if bi < n_free:
            for inter, active, gi, gsl in zip(program.per_block_interactions[bi],
                                              program.per_block_interaction_active[bi],
                                              program.per_block_interaction_global_inds[bi],
                                              program.per_block_interaction_global_slices[bi]):
                inters.append(_interaction(inter, active, gi, gsl, fam, n, maps))
        q = 1
        if fam == "categorical":
            q = int(getattr(b.nodes[0], "n_categories", None) or 2)
            for it in inters:  # tt_thrml/compiler.py:252-261
                if it.q_axis is not None:
                    q = it.q_axis
                    break
                if it.n_terms > 0:
                    q = it.weights.shape[1] // it.n_terms
        blocks.append(OBlock(bi, fam, n, q, starts[bi], inters))
    return OProgram(blocks, order, n_free, total)


def bf16_round(x) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (ties to even), as float32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


# ----------------------------------------------------------------------------
# Sampler.
# ----------------------------------------------------------------------------


class OracleSampler:
    """Runs lowered programs on the CPU over a float32 [rows, chains] state."""

    def __init__(self, program, n_chains: int = 1, chain_offset: int = 0, n_threads: int | None = None,
                 rng_layout="chain4", gaussian_storage: str = "f32", tables: bool = False):
        """rng_layout: Philox counter layout of Philox-mode draws, one name for
        every block or a dict block index -> name.  "chain4": counter (chain/4,
        row, sweep), word chain % 4 (the sparse, generic and Potts kernels);
        "row4": counter (chain, row/4, sweep), word row % 4 (the tensor-core
        dense kernel; its gaussians take Box-Muller on words 2p, 2p+1 for rows
        4j+2p (cosine) and 4j+2p+1 (sine)); "row8s" / "chain8s": the lattice kernels' split uniforms
        (spin blocks: 16 bits of counter (chain, row/8, sweep) resp.
        (chain/8, row, sweep), "LSPI", and 7 refill bits of (chain, row, sweep),
        "LREF"; the single-chain stencil and the resident lattice kernel);
        "planes": bit-plane draws of the bit-sliced lattice kernel (bit 22 - b
        of the draw of row r: bit 8 (r % 4) + (r % 32) / 4 of word b % 4 of
        counter (chain, r / 32, sweep, "LPL0" + b / 4)); "planes8": those of the
        bit-sliced resident kernel (bit 8 (r % 4) + chain % 8 of word b % 4 of
        counter (chain / 8, r / 4, sweep, "LPL0" + b / 4)).
        gaussian_storage: "f32", or "bf16" for a dense model whose gaussian
        block is stored as bfloat16 (the tensor-core kernel's operand).
        tables: build synthetic models as per-term tables instead of the
        stencil / dense paths."""
        names = {"chain4": 0, "row4": 1, "row8s": 2, "chain8s": 3, "planes": 4, "planes8": 5}
        layouts = rng_layout if isinstance(rng_layout, dict) else None
        for v in (layouts.values() if layouts is not None else [rng_layout]):
            if v not in names:
                raise ValueError(f"rng_layout must be one of {sorted(names)}, got {v!r}")
        self._rng_layout = {int(k): names[v] for k, v in layouts.items()} if layouts is not None else {}
        self._rng_default = 0 if layouts is not None else names[rng_layout]
        if gaussian_storage not in ("f32", "bf16"):
            raise ValueError(f"gaussian_storage must be 'f32' or 'bf16', got {gaussian_storage!r}")
        self.gaussian_storage = gaussian_storage
        self.prog = program if isinstance(program, OProgram) else lower_program(program, tables=tables)
        self.program = program
        self.C = int(n_chains)
        self.chain_offset = int(chain_offset)
        self.n_threads = int(n_threads or os.cpu_count() or 1)
        self.state = np.zeros((self.prog.total, self.C), dtype=np.float32)
        self._keep = []
        self._inter_structs = {}
        for b in self.prog.blocks[: self.prog.n_free]:
            arr = (_Inter * max(1, len(b.interactions)))()
            for k, it in enumerate(b.interactions):
                d = arr[k]
                self._keep += [it.row_ptr, it.weights, it.sources]
                d.row_ptr, d.weights, d.sources = it.row_ptr.ctypes.data, it.weights.ctypes.data, it.sources.ctypes.data
                d.nnz = int(it.row_ptr[-1])
                d.n_sources = it.sources.shape[0]
                d.n_categorical = it.n_categorical
                d.kind = 1 if it.kind == "precision" else 0
                d.w_inner = it.weights.shape[1]
                for j, q in enumerate(it.cat_q):
                    d.cat_q[j] = q
            self._inter_structs[b.index] = arr

    def layout_of(self, block_index: int) -> int:
        """Philox counter layout code of a block's draws."""
        return self._rng_layout.get(int(block_index), self._rng_default)

    # state -----------------------------------------------------------------
    def load_state(self, state_free, state_clamp=()):
        states = list(state_free) + list(state_clamp)
        for b, s in zip(self.prog.blocks, states):
            a = np.asarray(s)
            if b.family == "spin":
                a = np.where(a.astype(np.float32) > 0, 1.0, -1.0)
            a = a.astype(np.float32).reshape(-1, b.n_nodes)
            if b.family == "gaussian" and self.gaussian_storage == "bf16":
                a = bf16_round(a)
            if a.shape[0] == 1:
                a = np.broadcast_to(a, (self.C, b.n_nodes))
            self.state[b.start : b.start + b.n_nodes] = a.T

    def block_state(self, bi: int) -> np.ndarray:
        """Chain-major (C, n) decoded like tt_thrml/executor.py:433-438."""
        b = self.prog.blocks[bi]
        raw = self.state[b.start : b.start + b.n_nodes].T
        if b.family == "spin":
            return raw > 0
        if b.family == "categorical":
            return np.round(raw).astype(np.int32)
        return raw.astype(np.float32)

    # steps -----------------------------------------------------------------
    def group_step(self, group_index: int, sweep: int, *, seed: int = 0, variates: dict | None = None,
                   return_margin: bool = False):
        """One sampling group; variates: block index -> [n, qv, C] float32 for this sweep."""
        group = self.prog.sampling_order[group_index]
        if self.prog.model is not None:
            rows = sum(self.prog.blocks[bi].n_nodes for bi in group)
            margin = np.zeros((rows, self.C), dtype=np.float64) if return_margin else None
            self.prog.model.group_step(self, group_index, sweep, seed, variates, margin)
            return margin
        arr = (_Block * len(group))()
        keep = []
        rows = 0
        for k, bi in enumerate(group):
            b = self.prog.blocks[bi]
            d = arr[k]
            d.family = _FAMILY[b.family]
            d.q = b.q
            d.n_interactions = len(b.interactions)
            d.n_nodes = b.n_nodes
            d.row_start = b.start
            d.rng_layout = self._rng_layout.get(int(bi), self._rng_default)
            d.inter = ctypes.addressof(self._inter_structs[bi])
            if variates is not None:
                v = np.ascontiguousarray(variates[bi], dtype=np.float32)
                keep.append(v)
                d.variates = v.ctypes.data
            rows += b.n_nodes
        margin = np.zeros((rows, self.C), dtype=np.float64) if return_margin else None
        rc = lib().oracle_group_step(
            ctypes.addressof(arr), len(group), self.state.ctypes.data, self.C, self.chain_offset,
            1 if variates is not None else 0, int(seed), int(sweep),
            None if margin is None else margin.ctypes.data, self.n_threads,
        )
        if rc != 0:
            raise MemoryError("oracle_group_step failed")
        return margin

    def sweep(self, sweep: int, *, seed: int = 0, variates_for=None, return_margins: bool = False):
        """All groups in order; variates_for(block_index) -> [n, qv, C] of this sweep (parity mode)."""
        margins = []
        for gi, group in enumerate(self.prog.sampling_order):
            v = None if variates_for is None else {bi: variates_for(bi) for bi in group}
            m = self.group_step(gi, sweep, seed=seed, variates=v, return_margin=return_margins)
            margins.append(m)
        return margins
