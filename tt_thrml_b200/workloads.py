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
    meta = {"name": name, "n_nodes": n, "n_edges": int(row_ptr[-1]) // 2, "n_blocks": k, "flat_of": flat_of,
            # the model's raw parameters (before beta and the block renumbering), for independent checkers
            "graph": {"row_ptr": row_ptr, "cols": cols, "J": np.asarray(J, dtype=np.float32),
                      "h": np.asarray(h, dtype=np.float32), "beta": float(beta), "colours": colours}}
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


class IsingLattice2D(TableProgram):
    """Periodic H x W Ising lattice with uniform coupling J and field h, two checkerboard blocks.

    Site (y, x) has linear index L = y*W + x and colour (x + y) % 2; block c
    holds the colour-c sites in increasing L, so site L sits at block row L // 2
    (W even) and each block is the split-colour array [H][W/2].  Couplings are
    beta*J per edge and beta*h per site in float32, neighbours in the order
    (left, right, up, down), i.e. exactly the tables `spin_graph_program`
    builds from `lattice_2d_csr` -- `tt_lower_blocks()` materialises them on
    demand (small lattices; a 32768^2 lattice would need ~32 GB of tables).
    `tt_stencil()` describes the lattice for the single-chain stencil kernel.
    """

    MAX_TABLE_SITES = 1 << 24

    def __init__(self, height: int, width: int, *, J: float = 1.0, h: float = 0.0, beta: float = 0.44,
                 name: str | None = None):
        height, width = int(height), int(width)
        if height % 2 or width % 2:
            raise ValueError("the checkerboard colouring of a periodic lattice needs even dimensions")
        n = height * width
        blocks = [IndexBlock(n // 2, Family.SPIN, name=f"colour{c}:") for c in range(2)]
        gspec = TableGibbsSpec(free_blocks=blocks, clamped_blocks=[], sampling_order=[[0], [1]])
        meta = {"name": name or f"ising2d-{height}x{width}", "n_nodes": n, "n_blocks": 2, "height": height,
                "width": width, "J": J, "h": h, "beta": beta}
        super().__init__(gspec, [], meta)
        self.height, self.width = height, width
        self.J, self.h, self.beta = float(J), float(h), float(beta)
        self._specs = None

    @property
    def n_sites(self) -> int:
        return self.height * self.width

    def edge_weight(self) -> np.float32:
        return np.float32(self.beta) * np.float32(self.J)

    def site_bias(self) -> np.float32:
        return np.float32(self.beta) * np.float32(self.h)

    def tt_stencil(self) -> dict:
        return {
            "kind": "ising2d",
            "dims": (self.height, self.width),
            "edge_weight": self.edge_weight(),
            "site_bias": self.site_bias(),
            "block_rows": (0, self.n_sites // 2),
        }

    def tt_lower_blocks(self):
        if self._specs is None:
            if self.n_sites > self.MAX_TABLE_SITES:
                raise ValueError(
                    f"per-edge tables of a {self.height}x{self.width} lattice take "
                    f"{self.n_sites * 4 * 12 / 2**30:.0f} GiB; the stencil kernel runs it without them"
                )
            row_ptr, cols = lattice_2d_csr(self.height, self.width, True)
            n = self.n_sites
            colours = ((np.arange(n) // self.width + np.arange(n) % self.width) % 2).astype(np.int64)
            Jv = np.full(cols.shape[0], self.J, dtype=np.float32)
            hv = np.full(n, self.h, dtype=np.float32)
            self._specs = spin_graph_program(row_ptr, cols, Jv, hv, colours, beta=self.beta).specs
        return list(self._specs)

    @property
    def specs(self):
        return self.tt_lower_blocks()

    @specs.setter
    def specs(self, value):  # TableProgram's constructor assigns an empty list
        pass


def ising_lattice_2d(
    height: int = 64, width: int = 64, *, J: float = 1.0, h: float = 0.0, beta: float = 0.44, periodic: bool = True
):
    """2-D Ising lattice with two checkerboard blocks, one per sampling group.

    Periodic lattices are `IsingLattice2D` programs (tables built on demand,
    stencil description for the single-chain kernel); open boundaries give a
    table program."""
    if periodic:
        return IsingLattice2D(height, width, J=J, h=h, beta=beta)
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
    prog.meta["graph"]["colouring"] = "greedy"
    return prog


def random_spin_state(program: TableProgram, n_chains: int, seed: int = 0) -> list[np.ndarray]:
    """Uniform ±1 initial states per free block, (n_chains, n) bool, seeded."""
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 2, size=(n_chains, len(b.nodes)), dtype=np.int8).astype(bool)
            for b in program.gibbs_spec.free_blocks]


def bf16_representable(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to the nearest bfloat16 (ties to even), kept as float32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = ((b + np.uint32(0x7FFF) + ((b >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    return rounded.view(np.float32)


class DenseBipartiteProgram(TableProgram):
    """Two blocks coupled through a dense weight matrix (a restricted Boltzmann machine).

    Block 0: `n_visible` units (gaussian with unit precision, or spins), flat
    rows [0, n_visible); block 1: `n_hidden` spins, rows [n_visible, n_visible
    + n_hidden).  Field of visible unit i: b_v[i] + sum_j W[i, j] h_j; of hidden
    unit j: b_h[j] + sum_i W[i, j] v_i.  The tensor-core plan reads W directly
    (`tt_dense_couplings`); `tt_lower_blocks` builds the equivalent per-node
    tables (every unit has one term per unit of the other block) for the
    generic kernel and the oracle.
    """

    def __init__(self, W, b_v, b_h, *, visible_family: Family = Family.GAUSSIAN, sampling_order=((1,), (0,)),
                 name: str = "rbm"):
        W = np.ascontiguousarray(W, dtype=np.float32)
        V, H = W.shape
        blocks = [IndexBlock(V, visible_family, name="visible:"), IndexBlock(H, Family.SPIN, name="hidden:")]
        gspec = TableGibbsSpec(free_blocks=blocks, clamped_blocks=[], sampling_order=[list(g) for g in sampling_order])
        super().__init__(gspec, [], {"name": name, "n_visible": V, "n_hidden": H})
        self.W = W
        self.b_v = np.asarray(b_v, dtype=np.float32).reshape(V)
        self.b_h = np.asarray(b_h, dtype=np.float32).reshape(H)
        self.visible_family = Family(visible_family)
        self._specs = None

    def tt_dense_couplings(self) -> dict:
        V, H = self.W.shape
        return {
            0: {"family": self.visible_family, "row0": 0, "n_units": V, "source": 1, "weights_nk": self.W,
                "bias": self.b_v, "precision": 1.0},
            1: {"family": Family.SPIN, "row0": V, "n_units": H, "source": 0, "weights_nk": self.W.T,
                "bias": self.b_h, "precision": 1.0},
        }

    def tt_lower_blocks(self):
        if self._specs is None:
            V, H = self.W.shape
            total = V + H

            def block(bi, family, n, start, bias, w_nk, src0, n_src):
                rp = np.arange(n + 1, dtype=np.int64) * n_src
                cols = np.tile(np.arange(src0, src0 + n_src, dtype=np.int32), n)
                pair = FusedInteractionSpec(
                    weighted_mask=np.ascontiguousarray(w_nk, dtype=np.float32).reshape(-1),
                    gather_indices=(cols,),
                    n_spin=1,
                    n_categorical=0,
                    n_terms=n_src,
                    contribution_kind="default" if family == Family.SPIN else "linear",
                    row_ptr=rp,
                )
                b = FusedInteractionSpec(
                    weighted_mask=np.asarray(bias, np.float32).reshape(n, 1),
                    gather_indices=(),
                    n_spin=0,
                    n_categorical=0,
                    n_terms=1,
                    contribution_kind="default" if family == Family.SPIN else "linear",
                )
                return FusedBlockSpec(bi, family, n, None, start, total, (b, pair))

            self._specs = [
                block(0, self.visible_family, V, 0, self.b_v, self.W, V, H),
                block(1, Family.SPIN, H, V, self.b_h, self.W.T, 0, V),
            ]
        return list(self._specs)


def gaussian_bernoulli_rbm(
    n_visible: int = 4096,
    n_hidden: int = 8192,
    *,
    seed: int = 0,
    w_std: float = 0.01,
    visible_bias_variance: float = 0.1,
) -> DenseBipartiteProgram:
    """Gauss-Bernoulli RBM: unit-precision gaussian visible units with bias ~
    N(0, visible_bias_variance), +-1 hidden spins without bias, couplings
    W ~ N(0, w_std^2) rounded to bf16-representable values (the tensor cores
    then multiply the model's exact weights)."""
    rng = np.random.default_rng(seed)
    W = bf16_representable((rng.standard_normal((n_visible, n_hidden)) * w_std).astype(np.float32))
    b_v = (rng.standard_normal(n_visible) * np.sqrt(visible_bias_variance)).astype(np.float32)
    b_h = np.zeros(n_hidden, dtype=np.float32)
    prog = DenseBipartiteProgram(W, b_v, b_h, name=f"gb-rbm-{n_visible}x{n_hidden}")
    prog.meta.update(seed=seed, w_std=w_std, visible_bias_variance=visible_bias_variance)
    return prog


class PottsLattice3D(TableProgram):
    """q-state Potts model on a periodic X x Y x Z lattice, two checkerboard blocks.

    Site (x, y, z) has linear index L = (z*Y + y)*X + x and colour (x+y+z) % 2;
    block c holds the colour-c sites in increasing L, so site L sits at block
    row L // 2 (X even).  Field of category k at a site:
        theta_k = ((b[k] + (Jx[k][s_x-] + Jx[k][s_x+])) + (Jy[k][s_y-] + Jy[k][s_y+]))
                  + (Jz[k][s_z-] + Jz[k][s_z+])
    i.e. four interactions (bias, x pair, y pair, z pair), each summed over its
    terms first, in the order the reference accumulates interactions
    (tt_thrml/compiler.py:289-318).  `tt_stencil()` describes the lattice for
    the stencil kernel; `tt_lower_blocks()` builds the equivalent per-term
    tables (each term carries a q x q matrix) for the generic kernel and the
    oracle, which is only reasonable for small lattices.
    """

    MAX_TABLE_SITES = 1 << 18

    def __init__(self, dims, J, bias, *, name: str = "potts3d"):
        X, Y, Z = (int(d) for d in dims)
        if X % 2 or Y % 2 or Z % 2:
            raise ValueError("the checkerboard colouring of a periodic lattice needs even dimensions")
        J = np.ascontiguousarray(J, dtype=np.float32)
        q = int(J.shape[-1])
        if J.shape != (3, q, q):
            raise ValueError(f"J must have shape (3, q, q), got {J.shape}")
        n = X * Y * Z
        bias = np.ascontiguousarray(bias, dtype=np.float32).reshape(n, q)
        blocks = [IndexBlock(n // 2, Family.CATEGORICAL, q, name=f"colour{c}:") for c in range(2)]
        gspec = TableGibbsSpec(free_blocks=blocks, clamped_blocks=[], sampling_order=[[0], [1]])
        super().__init__(gspec, [], {"name": name, "dims": (X, Y, Z), "q": q, "n_sites": n})
        self.dims = (X, Y, Z)
        self.q = q
        self.J = J
        self.site_bias = bias
        self._specs = None

    def sites_of_block(self, c: int) -> np.ndarray:
        """Linear site indices of block c, in block-row order."""
        X, Y, Z = self.dims
        r = np.arange(X * Y * Z // 2, dtype=np.int64)
        even = 2 * r
        y = (even // X) % Y
        z = even // (X * Y)
        return even + ((y + z + c) & 1)

    def tt_stencil(self) -> dict:
        return {
            "kind": "potts3d",
            "dims": self.dims,
            "q": self.q,
            "J": self.J,
            "bias": [self.site_bias[self.sites_of_block(c)] for c in range(2)],
            "block_rows": (0, self.n_sites // 2),
        }

    @property
    def n_sites(self) -> int:
        X, Y, Z = self.dims
        return X * Y * Z

    def neighbour_rows(self, c: int) -> np.ndarray:
        """(n/2, 6) flat state rows of the neighbours (x-, x+, y-, y+, z-, z+) of block c's sites."""
        X, Y, Z = self.dims
        L = self.sites_of_block(c)
        x, y, z = L % X, (L // X) % Y, L // (X * Y)
        half = self.n_sites // 2
        other = (1 - c) * half
        out = []
        for dx, dy, dz in ((-1, 0, 0), (1, 0, 0), (0, -1, 0), (0, 1, 0), (0, 0, -1), (0, 0, 1)):
            Ln = (((z + dz) % Z) * Y + (y + dy) % Y) * X + (x + dx) % X
            out.append(other + Ln // 2)
        return np.stack(out, axis=1)

    def tt_lower_blocks(self):
        if self._specs is None:
            n, q = self.n_sites, self.q
            if n > self.MAX_TABLE_SITES:
                raise ValueError(
                    f"per-term tables of a {self.dims} Potts lattice take {n * 6 * q * q * 4 / 2**30:.1f} GiB; "
                    "the stencil kernel runs it without them"
                )
            half = n // 2
            specs = []
            for c in range(2):
                nb = self.neighbour_rows(c).astype(np.int32)
                inters = [
                    FusedInteractionSpec(
                        weighted_mask=self.site_bias[self.sites_of_block(c)].reshape(half, 1, q),
                        gather_indices=(), n_spin=0, n_categorical=0, n_terms=1, contribution_kind="default",
                    )
                ]
                for a in range(3):
                    wm = np.broadcast_to(self.J[a], (half, 2, q, q)).copy()
                    inters.append(
                        FusedInteractionSpec(
                            weighted_mask=wm, gather_indices=(np.ascontiguousarray(nb[:, 2 * a : 2 * a + 2]),),
                            n_spin=0, n_categorical=1, n_terms=2, contribution_kind="default",
                        )
                    )
                specs.append(FusedBlockSpec(c, Family.CATEGORICAL, half, q, c * half, n, tuple(inters)))
            self._specs = specs
        return list(self._specs)


def potts_lattice_3d(
    side: int = 128, q: int = 8, *, seed: int = 0, j_std: float = 1.0, bias_variance: float = 0.5
) -> PottsLattice3D:
    """3-D q-state Potts lattice side^3 (periodic): per axis one q x q matrix with
    entries ~ N(0, j_std^2), symmetrised as (A + A^T) / 2; per-site bias
    q-vectors ~ N(0, bias_variance) (0.5 read as the variance)."""
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((3, q, q)) * j_std).astype(np.float32)
    J = ((A + A.transpose(0, 2, 1)) * np.float32(0.5)).astype(np.float32)
    bias = (rng.standard_normal((side**3, q)) * np.sqrt(bias_variance)).astype(np.float32)
    prog = PottsLattice3D((side, side, side), J, bias, name=f"potts3d-{side}-q{q}")
    prog.meta.update(seed=seed, j_std=j_std, bias_variance=bias_variance)
    return prog
