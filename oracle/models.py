"""The oracle's own construction of the synthetic models — TEST INFRASTRUCTURE ONLY.

Each benchmark configuration is a seeded synthetic model given by raw
parameters (an edge list with couplings and biases, lattice dimensions with
J, h and beta, q x q coupling matrices with per-site biases, a weight matrix
with unit biases).  This module builds the oracle's program for each of them
from those raw parameters alone, without the product's lowering:

* `graph_ising`: a spin graph (symmetric CSR over node ids, J per edge entry,
  h per node, beta, block = colour) -> per-block tables: a bias interaction
  beta*h and a pair interaction over the node's edges, beta*J times the
  neighbour's spin, flat rows block by block in node order.  This is the
  reference's lowering of an Ising program (tt_thrml/compiler.py:156-271)
  written out for this model.
* `er_edges`, `er_ising_raw`: the sparse random-graph configuration's seeded
  G(n, p) graph and parameters, and `greedy_colouring` (oracle.c) for its
  blocks, so a CPU-only run needs nothing of the product.
* `ising2d`: the periodic 2-D lattice, as per-edge tables (`tables=True`) or
  as the stencil path of oracle.c (no tables: billion-site lattices).
* `potts3d`: the periodic 3-D Potts lattice, per-term tables or stencil path.
* `dense_bipartite`: the restricted Boltzmann machine, per-term tables or the
  dense path of oracle.c (fields summed in double precision).

The stencil and dense paths are checked against the table path on small
models by the CPU tests, so each full-size check rests on the same restated
group math (tt_thrml/compiler.py:274-450).
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import oracle as orc


# ----------------------------------------------------------------------------
# raw synthetic inputs
# ----------------------------------------------------------------------------


def er_edges(n: int, mean_degree: float, seed: int):
    """Undirected G(n, p) edge list (i < j, sorted by i * n + j), p = mean_degree / (n - 1).

    The number of edges is Binomial(n (n - 1) / 2, p); pairs are drawn
    uniformly without replacement by rejection of self-loops and repeats,
    and a surplus is thinned by a seeded permutation."""
    rng = np.random.default_rng(seed)
    p = mean_degree / (n - 1)
    m = int(rng.binomial(n * (n - 1) // 2, p))
    keys = np.zeros(0, dtype=np.int64)
    while keys.size < m:
        draw = int((m - keys.size) * 1.01) + 16
        a = rng.integers(0, n, draw, dtype=np.int64)
        b = rng.integers(0, n, draw, dtype=np.int64)
        ok = a != b
        lo, hi = np.minimum(a, b)[ok], np.maximum(a, b)[ok]
        keys = np.unique(np.concatenate([keys, lo * n + hi]))
    if keys.size > m:
        keys = np.sort(keys[rng.permutation(keys.size)[:m]])
    return keys // n, keys % n


def er_ising_raw(n: int = 1 << 20, mean_degree: float = 8.0, *, seed: int = 0, beta: float = 1.0,
                 j_variance: float = 1.0 / 8.0, h_variance: float = 0.1) -> dict:
    """Raw parameters of the sparse random-graph Ising configuration: symmetric CSR (row-major, columns
    ascending), J per CSR entry (both directions of an edge share it), h per node, beta, greedy colours."""
    ei, ej = er_edges(n, mean_degree, seed)
    rng = np.random.default_rng(seed + 1)
    J_edge = (rng.standard_normal(ei.shape[0]) * np.sqrt(j_variance)).astype(np.float32)
    h = (rng.standard_normal(n) * np.sqrt(h_variance)).astype(np.float32)
    src = np.concatenate([ei, ej])
    dst = np.concatenate([ej, ei])
    val = np.concatenate([J_edge, J_edge])
    order = np.lexsort((dst, src))
    row_ptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.bincount(src, minlength=n), out=row_ptr[1:])
    cols = dst[order].astype(np.int32)
    return {"row_ptr": row_ptr, "cols": cols, "J": val[order].astype(np.float32), "h": h, "beta": float(beta),
            "colours": greedy_colouring(row_ptr, cols)}


def rbm_raw(n_visible: int = 4096, n_hidden: int = 8192, *, seed: int = 0, w_std: float = 0.01,
            visible_bias_variance: float = 0.1) -> dict:
    """Raw parameters of the Gauss-Bernoulli RBM configuration: W ~ N(0, w_std^2) rounded to bf16, visible
    bias ~ N(0, visible_bias_variance), no hidden bias."""
    rng = np.random.default_rng(seed)
    W = orc.bf16_round((rng.standard_normal((n_visible, n_hidden)) * w_std).astype(np.float32))
    b_v = (rng.standard_normal(n_visible) * np.sqrt(visible_bias_variance)).astype(np.float32)
    return {"W": W, "b_v": b_v, "b_h": np.zeros(n_hidden, dtype=np.float32)}


def potts_raw(side: int = 128, q: int = 8, *, seed: int = 0, j_std: float = 1.0, bias_variance: float = 0.5) -> dict:
    """Raw parameters of the 3-D Potts configuration: per axis (A + A^T) / 2 with A ~ N(0, j_std^2), site
    biases ~ N(0, bias_variance)."""
    rng = np.random.default_rng(seed)
    A = (rng.standard_normal((3, q, q)) * j_std).astype(np.float32)
    J = ((A + A.transpose(0, 2, 1)) * np.float32(0.5)).astype(np.float32)
    bias = (rng.standard_normal((side**3, q)) * np.sqrt(bias_variance)).astype(np.float32)
    return {"dims": (side, side, side), "J": J, "bias": bias}


def greedy_colouring(row_ptr, cols) -> np.ndarray:
    rp = np.ascontiguousarray(row_ptr, dtype=np.int64)
    cc = np.ascontiguousarray(cols, dtype=np.int32)
    n = rp.shape[0] - 1
    out = np.empty(max(n, 1), dtype=np.int32)
    k = ctypes.c_int32(0)
    if orc.lib().oracle_greedy_colouring(n, rp.ctypes.data, cc.ctypes.data, out.ctypes.data, ctypes.byref(k)) != 0:
        raise MemoryError("oracle_greedy_colouring failed")
    return out[:n]


# ----------------------------------------------------------------------------
# table programs built from raw parameters
# ----------------------------------------------------------------------------


def _single_block_order(k: int):
    return [[b] for b in range(k)]


def graph_ising(row_ptr, cols, J, h, colours, beta: float) -> orc.OProgram:
    """Spin graph -> per-block tables (bias beta*h, then beta*J_e * s_col(e) over the node's CSR entries)."""
    row_ptr = np.asarray(row_ptr, dtype=np.int64)
    cols = np.asarray(cols, dtype=np.int64)
    colours = np.asarray(colours, dtype=np.int64)
    n = row_ptr.shape[0] - 1
    k = int(colours.max()) + 1 if n else 0
    b32 = np.float32(beta)
    wJ = (b32 * np.asarray(J, dtype=np.float32)).astype(np.float32)
    wh = (b32 * np.asarray(h, dtype=np.float32)).astype(np.float32)
    # flat row of every node: blocks in colour order, nodes of a block in index order
    members = [np.flatnonzero(colours == b) for b in range(k)]
    flat = np.empty(n, dtype=np.int64)
    start = 0
    starts = []
    for b in range(k):
        flat[members[b]] = start + np.arange(members[b].size)
        starts.append(start)
        start += members[b].size
    deg = np.diff(row_ptr)
    blocks = []
    for b in range(k):
        nodes = members[b]
        d = deg[nodes]
        rp = np.zeros(nodes.size + 1, dtype=np.int64)
        np.cumsum(d, out=rp[1:])
        # CSR entries of the block's nodes, node by node
        first = np.repeat(row_ptr[nodes], d)
        within = np.arange(rp[-1], dtype=np.int64) - np.repeat(rp[:-1], d)
        e = first + within
        bias = orc.OInteraction(
            row_ptr=np.arange(nodes.size + 1, dtype=np.int64), weights=wh[nodes].reshape(-1, 1).copy(),
            sources=np.zeros((0, nodes.size), np.int32), n_categorical=0, kind="default", cat_q=(), n_terms=1)
        pair = orc.OInteraction(
            row_ptr=rp, weights=np.ascontiguousarray(wJ[e].reshape(-1, 1)),
            sources=np.ascontiguousarray(flat[cols[e]].astype(np.int32).reshape(1, -1)), n_categorical=0,
            kind="default", cat_q=(), n_terms=int(d.max()) if d.size else 0)
        blocks.append(orc.OBlock(b, "spin", int(nodes.size), 1, starts[b], [bias, pair]))
    return orc.OProgram(blocks, _single_block_order(k), k, n)


def lattice2d_csr(height: int, width: int):
    """Periodic 4-neighbour lattice CSR over site ids y*width + x, neighbours (left, right, up, down)."""
    y, x = np.divmod(np.arange(height * width, dtype=np.int64), width)
    nb = np.stack([y * width + (x - 1) % width, y * width + (x + 1) % width,
                   ((y - 1) % height) * width + x, ((y + 1) % height) * width + x], axis=1)
    return np.arange(height * width + 1, dtype=np.int64) * 4, nb.reshape(-1).astype(np.int32)


class Ising2DModel:
    """oracle.c's 2-D lattice path for a program whose blocks are the two colours."""

    def __init__(self, height, width, J, h, beta):
        self.height, self.width = int(height), int(width)
        b32 = np.float32(beta)
        self.struct = orc.Lattice2D(self.height, self.width, float(b32 * np.float32(J)), float(b32 * np.float32(h)))

    def group_step(self, sampler, gi, sweep, seed, variates, margin_out):
        (bi,) = sampler.prog.sampling_order[gi]
        v = None if variates is None else np.ascontiguousarray(variates[bi], dtype=np.float32).reshape(-1, sampler.C)
        rc = orc.lib().oracle_ising2d_step(
            ctypes.byref(self.struct), int(bi), sampler.state.ctypes.data, sampler.C, sampler.chain_offset,
            None if v is None else v.ctypes.data, sampler.layout_of(bi), int(seed), int(sweep),
            None if margin_out is None else margin_out.ctypes.data, sampler.n_threads)
        if rc != 0:
            raise ValueError("oracle_ising2d_step rejected the lattice")


def ising2d(height: int, width: int, *, J: float = 1.0, h: float = 0.0, beta: float = 0.44,
            tables: bool = False) -> orc.OProgram:
    """Periodic 2-D Ising lattice, two checkerboard blocks (colour (x + y) % 2, sites in index order)."""
    n = height * width
    blocks = [orc.OBlock(c, "spin", n // 2, 1, c * n // 2, []) for c in range(2)]
    if tables:
        rp, cols = lattice2d_csr(height, width)
        colours = ((np.arange(n) // width + np.arange(n) % width) % 2).astype(np.int64)
        prog = graph_ising(rp, cols, np.full(cols.size, J, np.float32), np.full(n, h, np.float32), colours, beta)
        return prog
    return orc.OProgram(blocks, [[0], [1]], 2, n, model=Ising2DModel(height, width, J, h, beta))


def _potts_block_sites(dims, c):
    X, Y, Z = dims
    even = 2 * np.arange(X * Y * Z // 2, dtype=np.int64)
    y = (even // X) % Y
    z = even // (X * Y)
    return even + ((y + z + c) & 1)


def _potts_neighbours(dims, c):
    """(n/2, 6) site ids of the neighbours (x-, x+, y-, y+, z-, z+) of block c's sites."""
    X, Y, Z = dims
    L = _potts_block_sites(dims, c)
    x, y, z = L % X, (L // X) % Y, L // (X * Y)
    out = []
    for dx, dy, dz in ((-1, 0, 0), (1, 0, 0), (0, -1, 0), (0, 1, 0), (0, 0, -1), (0, 0, 1)):
        out.append((((z + dz) % Z) * Y + (y + dy) % Y) * X + (x + dx) % X)
    return np.stack(out, axis=1)


class Potts3DModel:
    def __init__(self, dims, J, bias):
        self.dims = tuple(int(d) for d in dims)
        self.J = np.ascontiguousarray(J, dtype=np.float32)
        q = self.J.shape[-1]
        bias = np.asarray(bias, dtype=np.float32).reshape(-1, q)
        self.bias = [np.ascontiguousarray(bias[_potts_block_sites(self.dims, c)]) for c in range(2)]
        self.struct = orc.Potts3D((ctypes.c_int64 * 3)(*self.dims), q, self.J.ctypes.data,
                                  self.bias[0].ctypes.data, self.bias[1].ctypes.data)

    def group_step(self, sampler, gi, sweep, seed, variates, margin_out):
        (bi,) = sampler.prog.sampling_order[gi]
        v = None if variates is None else np.ascontiguousarray(variates[bi], dtype=np.float32)
        rc = orc.lib().oracle_potts3d_step(
            ctypes.byref(self.struct), int(bi), sampler.state.ctypes.data, sampler.C, sampler.chain_offset,
            None if v is None else v.ctypes.data, int(seed), int(sweep),
            None if margin_out is None else margin_out.ctypes.data, sampler.n_threads)
        if rc != 0:
            raise ValueError("oracle_potts3d_step rejected the lattice")


def potts3d(dims, J, bias, *, tables: bool = False) -> orc.OProgram:
    """Periodic 3-D q-state Potts lattice, two checkerboard blocks; J [3][q][q], bias [sites][q]."""
    dims = tuple(int(d) for d in dims)
    J = np.ascontiguousarray(J, dtype=np.float32)
    q = int(J.shape[-1])
    n = int(np.prod(dims))
    half = n // 2
    bias = np.asarray(bias, dtype=np.float32).reshape(n, q)
    if not tables:
        blocks = [orc.OBlock(c, "categorical", half, q, c * half, []) for c in range(2)]
        return orc.OProgram(blocks, [[0], [1]], 2, n, model=Potts3DModel(dims, J, bias))
    blocks = []
    for c in range(2):
        nb = _potts_neighbours(dims, c)
        nb_rows = ((1 - c) * half + nb // 2).astype(np.int32)
        inters = [orc.OInteraction(
            row_ptr=np.arange(half + 1, dtype=np.int64), weights=np.ascontiguousarray(bias[_potts_block_sites(dims, c)]),
            sources=np.zeros((0, half), np.int32), n_categorical=0, kind="default", cat_q=(), n_terms=1, q_axis=q)]
        for a in range(3):
            # each term: the q x q matrix of the axis, selected by the neighbour's category (weights [k][s])
            w = np.broadcast_to(J[a].reshape(1, q * q), (2 * half, q * q))
            inters.append(orc.OInteraction(
                row_ptr=np.arange(half + 1, dtype=np.int64) * 2, weights=np.ascontiguousarray(w),
                sources=np.ascontiguousarray(nb_rows[:, 2 * a : 2 * a + 2].reshape(1, -1)), n_categorical=1,
                kind="default", cat_q=(q,), n_terms=2, q_axis=q))
        blocks.append(orc.OBlock(c, "categorical", half, q, c * half, inters))
    return orc.OProgram(blocks, [[0], [1]], 2, n)


class DenseModel:
    def __init__(self, W, b_v, b_h, visible_family):
        self.W = np.ascontiguousarray(W, dtype=np.float32)
        V, H = self.W.shape
        self.b_v = np.ascontiguousarray(b_v, dtype=np.float32).reshape(V)
        self.b_h = np.ascontiguousarray(b_h, dtype=np.float32).reshape(H)
        self.visible_family = visible_family

    def group_step(self, sampler, gi, sweep, seed, variates, margin_out):
        (bi,) = sampler.prog.sampling_order[gi]
        V, H = self.W.shape
        st = orc.Dense(V, H, self.W.ctypes.data, self.b_v.ctypes.data, self.b_h.ctypes.data,
                       orc._FAMILY[self.visible_family], 1 if sampler.gaussian_storage == "bf16" else 0)
        v = None if variates is None else np.ascontiguousarray(variates[bi], dtype=np.float32).reshape(-1, sampler.C)
        rc = orc.lib().oracle_dense_step(
            ctypes.byref(st), int(bi), sampler.state.ctypes.data, sampler.C, sampler.chain_offset,
            None if v is None else v.ctypes.data, sampler.layout_of(bi), int(seed), int(sweep),
            None if margin_out is None else margin_out.ctypes.data, sampler.n_threads)
        if rc != 0:
            raise MemoryError("oracle_dense_step failed")


def dense_bipartite(W, b_v, b_h, *, visible_family: str = "gaussian", sampling_order=((1,), (0,)),
                    tables: bool = False) -> orc.OProgram:
    """Restricted Boltzmann machine: visible block rows [0, V), hidden spins [V, V + H)."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    V, H = W.shape
    order = [list(g) for g in sampling_order]
    if not tables:
        blocks = [orc.OBlock(0, visible_family, V, 1, 0, []), orc.OBlock(1, "spin", H, 1, V, [])]
        return orc.OProgram(blocks, order, 2, V + H, model=DenseModel(W, b_v, b_h, visible_family))
    kind_v = "default" if visible_family == "spin" else "linear"

    def block(bi, family, kind, n, start, bias, w_nk, src0, n_src):
        b = orc.OInteraction(np.arange(n + 1, dtype=np.int64), np.asarray(bias, np.float32).reshape(n, 1).copy(),
                             np.zeros((0, n), np.int32), 0, kind, (), 1)
        pair = orc.OInteraction(np.arange(n + 1, dtype=np.int64) * n_src,
                                np.ascontiguousarray(w_nk, dtype=np.float32).reshape(-1, 1),
                                np.tile(np.arange(src0, src0 + n_src, dtype=np.int32), n).reshape(1, -1),
                                0, kind, (), n_src)
        return orc.OBlock(bi, family, n, 1, start, [b, pair])

    blocks = [block(0, visible_family, kind_v, V, 0, b_v, W, V, H), block(1, "spin", "default", H, V, b_h, W.T, 0, V)]
    return orc.OProgram(blocks, order, 2, V + H)


# ----------------------------------------------------------------------------
# a product program's raw parameters -> the oracle's program
# ----------------------------------------------------------------------------


def from_raw_parameters(program, *, tables: bool = False):
    """The oracle's program for a synthetic-model program, read from its raw parameters; None when the
    program is not one of the synthetic models (thrml programs and plain table programs)."""
    meta = getattr(program, "meta", None) or {}
    if all(hasattr(program, a) for a in ("height", "width", "J", "h", "beta")):
        return ising2d(program.height, program.width, J=program.J, h=program.h, beta=program.beta, tables=tables)
    if all(hasattr(program, a) for a in ("dims", "J", "site_bias")):
        return potts3d(program.dims, program.J, program.site_bias, tables=tables)
    if all(hasattr(program, a) for a in ("W", "b_v", "b_h", "visible_family")):
        fam = getattr(program.visible_family, "value", program.visible_family)
        order = [tuple(int(b) for b in g) for g in program.gibbs_spec.sampling_order]
        return dense_bipartite(program.W, program.b_v, program.b_h, visible_family=fam, sampling_order=order,
                               tables=tables)
    g = meta.get("graph")
    if g is not None:
        colours = greedy_colouring(g["row_ptr"], g["cols"]) if g.get("colouring") == "greedy" else g["colours"]
        return graph_ising(g["row_ptr"], g["cols"], g["J"], g["h"], colours, g["beta"])
    return None
