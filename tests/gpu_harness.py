"""Shared GPU-vs-oracle comparison helpers for the -m gpu tests."""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from oracle import oracle as orc
from tt_thrml_b200 import BulkRNGBuffers, Executor, make_cuda_config
from tt_thrml_b200.core import Family

BAND = 1e-5  # spin / categorical decisions this close to the threshold are ties, not mismatches
GAUSS_RTOL = 1e-4
# Absolute floor of the gaussian criterion |gpu - oracle| <= GAUSS_ATOL + GAUSS_RTOL * |oracle|: a float32 sum of
# K terms carries an error that scales with the sum of the terms' magnitudes, not with the result, so a value
# near zero cannot be matched relatively.  1e-5 is a few times the float32 accumulation error of the
# largest fields checked here (8192 products of size ~0.01: ~1e-6 rms, ~5e-6 at the extremes).
GAUSS_ATOL = 1e-5


@dataclass
class ParityReport:
    sites: int = 0
    band: int = 0
    hard_mismatches: int = 0
    gauss_max_rel: float = 0.0
    notes: list = field(default_factory=list)

    @property
    def band_fraction(self) -> float:
        return self.band / max(1, self.sites)


def rng_layouts(compiled) -> dict:
    """Block index -> Philox counter layout of the kernel that samples it."""
    out = {}
    for g in compiled.sampling_groups:
        for bi in g.block_indices:
            out[int(bi)] = getattr(g.kernel_artifact, "rng_layout", "chain4")
    return out


def gaussian_storage(compiled) -> str:
    """"bf16" when the tensor-core plans hold gaussian blocks as single bf16 operands, else "f32"."""
    plans = [g.kernel_artifact for g in compiled.sampling_groups]
    if plans and all(p.kind == "dense" and p.source_pieces == 1 and p.out_pieces == 1 for p in plans):
        return "bf16"
    return "f32"


def random_init(program, C, seed=0, clamp=None):
    rng = np.random.default_rng(seed)
    out = []
    for b in program.gibbs_spec.free_blocks:
        n = len(b.nodes)
        fam = getattr(b, "family", None)
        out.append(rng.integers(0, 2, (C, n)).astype(bool) if fam in (None, Family.SPIN) else rng.integers(0, 2, (C, n)))
    return out


def make_variates(executor: Executor, n_sweeps: int, seed: int = 7):
    """Host variates per free block [S, n, qv, C] like the reference's bulk buffers (logits / Gumbel / normal)."""
    import torch

    rng = np.random.default_rng(seed)
    C = executor.n_chains
    spin, cat, gauss = {}, {}, {}
    for cb in executor.compiled.blocks[: executor.compiled.n_free_blocks]:
        s = cb.spec
        if s.family == Family.SPIN:
            u = rng.uniform(1e-7, 1 - 1e-7, (n_sweeps, s.n_nodes, 1, C)).astype(np.float32)
            spin[s.block_index] = np.log(u / (np.float32(1) - u)).astype(np.float32)
        elif s.family == Family.CATEGORICAL:
            q = int(s.n_categories or 2)
            u = rng.uniform(1e-7, 1.0, (n_sweeps, s.n_nodes, q, C))
            cat[s.block_index] = (-np.log(-np.log(u))).astype(np.float32)
        else:
            gauss[s.block_index] = rng.standard_normal((n_sweeps, s.n_nodes, 1, C)).astype(np.float32)
    dev = executor.compiled.device
    to = lambda d: {k: torch.from_numpy(v).to(dev) for k, v in d.items()} or None  # noqa: E731
    buffers = BulkRNGBuffers(to(spin), to(cat), to(gauss), seed=None, n_sweeps=n_sweeps)
    host = {**spin, **cat, **gauss}
    return buffers, host


def gpu_state(executor: Executor) -> np.ndarray:
    """Device state decoded to float32 [rows, chains] (any layout)."""
    return executor.raw_state()


def set_gpu_state(executor: Executor, state: np.ndarray) -> None:
    executor.set_raw_state(state)


def compare_group(report: ParityReport, ex: Executor, o: orc.OracleSampler, gi: int, margin: np.ndarray,
                  *, gauss_rtol: float = GAUSS_RTOL, follow_gpu: bool = False) -> None:
    """Compares the rows of group gi, then re-syncs the two states.

    Default: the GPU is reset to the oracle's state (tie sites, float32
    gaussians).  follow_gpu: the oracle adopts the GPU's state instead (a
    GPU state stored at lower precision, e.g. bf16 gaussian blocks, stays
    exactly representable and the next group starts from identical inputs).
    """
    g = gpu_state(ex)
    rows = []
    for bi in o.prog.sampling_order[gi]:
        b = o.prog.blocks[bi]
        rows.append((b, np.arange(b.start, b.start + b.n_nodes)))
    off = 0
    for b, r in rows:
        gg, oo = g[r], o.state[r]
        m = margin[off : off + len(r)]
        off += len(r)
        report.sites += gg.size
        if b.family == "gaussian":
            err = np.abs(gg - oo)
            rel = float(np.max(err / (np.abs(oo) + GAUSS_ATOL / gauss_rtol))) if err.size else 0.0
            report.gauss_max_rel = max(report.gauss_max_rel, rel)
            continue
        tie = np.abs(m) < BAND
        report.band += int(tie.sum())
        diff = gg != oo
        hard = diff & ~tie
        report.hard_mismatches += int(hard.sum())
        if hard.any():  # the decision margins (oracle, logit units) of the sites that disagree
            report.notes.append(("hard mismatch margins", sorted(float(x) for x in np.abs(m[hard]))[:8]))
    if follow_gpu:
        o.state[...] = g
    elif not np.array_equal(g, o.state):
        set_gpu_state(ex, o.state)


def run_parity(program, C: int, n_sweeps: int, *, mode: str, seed: int = 11, init=None, clamp=(), force_generic=False,
               dense_precision: str = "auto", gauss_rtol: float = GAUSS_RTOL, follow_gpu: bool = False,
               stencil: bool = True):
    """Runs n_sweeps group by group on the GPU and in the oracle from the same state and variates."""
    from tt_thrml_b200.compiler import compile_program

    cfg = make_cuda_config(rng_mode="parity" if mode == "variates" else "philox", n_chains=C, cuda_graphs=False,
                           dense_precision=dense_precision, stencil=stencil)
    compiled = compile_program(None, 0, program, cfg, n_sweeps=n_sweeps, n_chains=C, force_generic=force_generic)
    ex = Executor(None, 0, program, cfg, compiled, n_sweeps=n_sweeps, n_chains=C)
    o = orc.OracleSampler(program, n_chains=C, rng_layout=rng_layouts(compiled),
                          gaussian_storage=gaussian_storage(compiled))
    init = init if init is not None else random_init(program, C, seed)
    ex.load_state(init, clamp)
    o.load_state(init, clamp)
    if mode == "variates":
        buffers, host = make_variates(ex, n_sweeps, seed)
        ex._install_rng(buffers, n_sweeps)
    else:
        ex.prepare_rng(seed)
        from tt_thrml_b200.rng import seed_from_key

        philox_seed = seed_from_key(seed)
    report = ParityReport()
    set_gpu_state(ex, o.state)  # both start from the oracle's float32 encoding
    if follow_gpu:
        o.state[...] = gpu_state(ex)  # ... as stored on the GPU
    for sweep in range(n_sweeps):
        for gi, group in enumerate(ex.compiled.sampling_groups):
            ex._run_sampling_group(group, sweep)
            if mode == "variates":
                v = {bi: host[bi][sweep] for bi in o.prog.sampling_order[gi]}
                m = o.group_step(gi, sweep, variates=v, return_margin=True)
            else:
                m = o.group_step(gi, sweep, seed=philox_seed, return_margin=True)
            compare_group(report, ex, o, gi, m, gauss_rtol=gauss_rtol, follow_gpu=follow_gpu)
        ex._sweep_counter += 1
    return report, ex, o


def exact_spin_distribution(weights_bias, pairs, n):
    """Exact Boltzmann distribution p(s) ~ exp(sum h s + sum J s s) over 2^n spin states (bit i = node i up)."""
    states = ((np.arange(2**n)[:, None] >> np.arange(n)[None, :]) & 1) * 2 - 1
    e = states @ np.asarray(weights_bias, np.float64)
    for (i, j), w in pairs.items():
        e = e + w * states[:, i] * states[:, j]
    p = np.exp(e - e.max())
    return p / p.sum()
