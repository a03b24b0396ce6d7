"""Native table programs and the seeded synthetic workloads.

A thrml program describes every node as a Python object; the layout pass over
them (tt_thrml/compiler.py:126-153) is O(N) Python, which is infeasible for
the million-node and billion-site workloads.  A *table program* carries the
already-lowered block tables instead (the same `FusedBlockSpec` /
`FusedInteractionSpec` data the compiler would build, in flat block-ordered
rows) and exposes the parts of thrml's program surface the executor uses:
`gibbs_spec.blocks / free_blocks / clamped_blocks / sampling_order`, plus
`tt_lower_blocks()`.

Generators (all seeded, numpy only):
* `ising_lattice_2d`: periodic 2-D Ising lattice, two checkerboard blocks;
* `erdos_renyi_ising`: sparse random-graph Ising, greedy colouring into k
  blocks (native host colouring in libtthrml_b200).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .core import Family, FusedBlockSpec, FusedInteractionSpec


class IndexBlock:
    """A block of nodes addressed by position (stands in for thrml.Block)."""

    def __init__(self, n_nodes: int, family: Family = Family.SPIN, n_categories: int | None = None, name: str = ""):
        self.nodes = range(int(n_nodes))
        self.family = Family(family)
        self.n_categories = n_categories
        self.name = name

    def __len__(self) -> int:
        return len(self.nodes)

    def __repr__(self) -> str:
        return f"IndexBlock({self.name or ''}{len(self.nodes)} {self.family.value})"


@dataclass
class TableGibbsSpec:
    free_blocks: list
    clamped_blocks: list
    sampling_order: list

    @property
    def blocks(self) -> list:
        return list(self.free_blocks) + list(self.clamped_blocks)


@dataclass
class TableProgram:
    """A program given directly by its lowered block tables."""

    gibbs_spec: TableGibbsSpec
    specs: list
    meta: dict = field(default_factory=dict)

    def tt_lower_blocks(self):
        return list(self.specs)


def _bias_interaction(values: np.ndarray) -> FusedInteractionSpec:
    v = np.asarray(values, dtype=np.float32).reshape(-1, 1)
    return FusedInteractionSpec(
        weighted_mask=v, gather_indices=(), n_spin=0, n_categorical=0, n_terms=1, contribution_kind="default"
    )


def _pair_interaction(row_ptr, cols, vals) -> FusedInteractionSpec:
    rp = np.asarray(row_ptr, dtype=np.int64)
    counts = np.diff(rp)
    return FusedInteractionSpec(
        weighted_mask=np.asarray(vals, dtype=np.float32),
        gather_indices=(np.asarray(cols, dtype=np.int32),),
        n_spin=1,
        n_categorical=0,
        n_terms=int(counts.max()) if len(counts) else 0,
        contribution_kind="default",
        row_ptr=rp,
    )


def spin_graph_program(row_ptr, cols, J, h, colours, *, beta: float = 1.0, name: str = "spin-graph") -> TableProgram:
    """Ising program on a graph given as symmetric CSR over original node ids.

    colours[i] is the block of node i; nodes are renumbered block by block
    (stable in original order) into flat rows, and each block gets one bias
    interaction (beta*h) and one pair interaction (beta*J over CSR edges).
    """
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    cols = np.asarray(cols, dtype=np.int64)
    n = row_ptr.shape[0] - 1
    colours = np.asarray(colours, dtype=np.int64)
    k = int(colours.max()) + 1 if n else 0
    order = np.argsort(colours, kind="stable")
    flat_of = np.empty(n, dtype=np.int64)
    flat_of[order] = np.arange(n, dtype=np.int64)
    counts = np.bincount(colours, minlength=k)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]]).astype(np.int64)
    deg = np.diff(row_ptr)
    Jb = (np.float32(beta) * np.asarray(J, dtype=np.float32)).astype(np.float32)
    hb = (np.float32(beta) * np.asarray(h, dtype=np.float32)).astype(np.float32)
    blocks, specs = [], []
    for b in range(k):
        nodes = order[starts[b] : starts[b] + counts[b]]
        d = deg[nodes]
        rp = np.concatenate([[0], np.cumsum(d)]).astype(np.int64)
        # edge ids of the block's rows, row by row in CSR order
        eidx = np.repeat(row_ptr[nodes], d) + (np.arange(rp[-1], dtype=np.int64) - np.repeat(rp[:-1], d))
        c_flat = flat_of[cols[eidx]].astype(np.int32)
        spec = FusedBlockSpec(
            block_index=b,
            family=Family.SPIN,
            n_nodes=int(counts[b]),
            n_categories=None,
            block_global_start=int(starts[b]),
            total_nodes=n,
            interactions=(_bias_interaction(hb[nodes]), _pair_interaction(rp, c_flat, Jb[eidx])),
        )
        blocks.append(IndexBlock(int(counts[b]), Family.SPIN, name=f"colour{b}:"))
        specs.append(spec)
    gspec = TableGibbsSpec(free_blocks=blocks, clamped_blocks=[], sampling_order=[[b] for b in range(k)])
    meta = {"name": name, "n_nodes": n, "n_edges": int(row_ptr[-1]) // 2, "n_blocks": k, "flat_of": flat_of}
    return TableProgram(gspec, specs, meta)


def lattice_2d_csr(height: int, width: int, periodic: bool = True):
    """CSR of the 4-neighbour lattice, neighbour order (left, right, up, down)."""
    idx = np.arange(height * width, dtype=np.int64).reshape(height, width)
    nbrs = []
    for dy, dx in ((0, -1), (0, 1), (-1, 0), (1, 0)):
        nb = np.roll(idx, shift=(-dy, -dx), axis=(0, 1))
        if not periodic:
            y = np.arange(height)[:, None] + dy
            x = np.arange(width)[None, :] + dx
            nb = np.where((y >= 0) & (y < height) & (x >= 0) & (x < width), nb, -1)
        nbrs.append(nb.reshape(-1))
    nb = np.stack(nbrs, axis=1)
    valid = nb >= 0
    row_ptr = np.concatenate([[0], np.cumsum(valid.sum(1))]).astype(np.int64)
    return row_ptr, nb[valid]


def ising_lattice_2d(
    height: int = 64, width: int = 64, *, J: float = 1.0, h: float = 0.0, beta: float = 0.44, periodic: bool = True
) -> TableProgram:
    """2-D Ising lattice with two checkerboard blocks, one per sampling group."""
    row_ptr, cols = lattice_2d_csr(height, width, periodic)
    n = height * width
    colours = ((np.arange(n) // width + np.arange(n) % width) % 2).astype(np.int64)
    Jv = np.full(cols.shape[0], J, dtype=np.float32)
    hv = np.full(n, h, dtype=np.float32)
    prog = spin_graph_program(row_ptr, cols, Jv, hv, colours, beta=beta, name=f"ising2d-{height}x{width}")
    prog.meta.update(height=height, width=width, J=J, h=h, beta=beta)
    return prog


def greedy_colouring(row_ptr, cols) -> np.ndarray:
    """Greedy colouring in node order via the native host helper."""
    import ctypes

    from . import _native as nat

    rp = np.ascontiguousarray(row_ptr, dtype=np.int64)
    cc = np.ascontiguousarray(cols, dtype=np.int32)
    n = rp.shape[0] - 1
    out = np.empty(n, dtype=np.int32)
    k = ctypes.c_int32(0)
    nat.check(
        nat.lib().tthrml_greedy_colouring(n, rp.ctypes.data, cc.ctypes.data, out.ctypes.data, ctypes.byref(k)),
        "tthrml_greedy_colouring",
    )
    return out


def erdos_renyi_edges(n: int, mean_degree: float, seed: int):
    """Undirected G(n, p) edge list (i < j), p = mean_degree / (n - 1), seeded."""
    rng = np.random.default_rng(seed)
    p = mean_degree / (n - 1)
    pairs = n * (n - 1) // 2
    m = int(rng.binomial(pairs, p))
    got = np.zeros(0, dtype=np.int64)
    while got.size < m:
        need = int((m - got.size) * 1.01) + 16
        i = rng.integers(0, n, need, dtype=np.int64)
        j = rng.integers(0, n, need, dtype=np.int64)
        keep = i != j
        a, b = np.minimum(i, j)[keep], np.maximum(i, j)[keep]
        got = np.unique(np.concatenate([got, a * n + b]))
    if got.size > m:
        got = got[rng.permutation(got.size)[:m]]
        got.sort()
    return got // n, got % n


def symmetric_csr(n: int, ei, ej, w):
    """Symmetric CSR (both directions) sorted by (row, col)."""
    rows = np.concatenate([ei, ej])
    cols = np.concatenate([ej, ei])
    vals = np.concatenate([w, w]).astype(np.float32)
    order = np.lexsort((cols, rows))
    rows, cols, vals = rows[order], cols[order], vals[order]
    row_ptr = np.concatenate([[0], np.cumsum(np.bincount(rows, minlength=n))]).astype(np.int64)
    return row_ptr, cols, vals


def erdos_renyi_ising(
    n: int = 1 << 20,
    mean_degree: float = 8.0,
    *,
    seed: int = 0,
    beta: float = 1.0,
    j_variance: float = 1.0 / 8.0,
    h_variance: float = 0.1,
) -> TableProgram:
    """Sparse random-graph Ising: G(n, p) with mean degree `mean_degree`,
    J_ij ~ N(0, j_variance) per undirected edge (symmetric), h_i ~ N(0,
    h_variance), inverse temperature beta folded into the tables, greedy
    colouring into blocks (each block its own sampling group)."""
    ei, ej = erdos_renyi_edges(n, mean_degree, seed)
    rng = np.random.default_rng(seed + 1)
    J = (rng.standard_normal(ei.shape[0]) * np.sqrt(j_variance)).astype(np.float32)
    h = (rng.standard_normal(n) * np.sqrt(h_variance)).astype(np.float32)
    row_ptr, cols, vals = symmetric_csr(n, ei, ej, J)
    colours = greedy_colouring(row_ptr, cols)
    prog = spin_graph_program(row_ptr, cols, vals, h, colours, beta=beta, name=f"er-ising-{n}")
    prog.meta.update(mean_degree=mean_degree, seed=seed, beta=beta, j_variance=j_variance, h_variance=h_variance)
    return prog


def random_spin_state(program: TableProgram, n_chains: int, seed: int = 0) -> list[np.ndarray]:
    """Uniform ±1 initial states per free block, (n_chains, n) bool, seeded."""
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 2, size=(n_chains, len(b.nodes)), dtype=np.int8).astype(bool)
            for b in program.gibbs_spec.free_blocks]
