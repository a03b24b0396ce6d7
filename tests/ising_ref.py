"""Host restatement of the single-chain 2-D Ising half-sweep (test infrastructure).

Mirrors tthrml_ising2d_halfsweep on numpy arrays so the strip decomposition
of tt_thrml_b200.domain can be checked on CPU ranks (gloo): split-colour
int8 arrays [rows][W/2], neighbour-sign pattern (left, right, up, down), the
pattern's Philox threshold and the 23-bit draw of the strips' layout
(lattice_draws: bit-planes for count-symmetric tables, else split uniforms).
It is itself checked against the oracle (the reference's group math on the
lattice's per-edge tables) in test_domain_cpu.py.
"""

from __future__ import annotations

import numpy as np

M32 = np.uint64(0xFFFFFFFF)
SALT_LATTICE_SPIN = 0x4C535049
SALT_LATTICE_REFILL = 0x4C524546
SALT_LATTICE_PLANES = 0x4C504C30


def philox4x32_10(c0, c1, c2, c3, k0: int, k1: int):
    """Vectorised Philox4x32-10 on uint64 arrays holding 32-bit words."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint64) & M32 for c in (c0, c1, c2, c3))
    k0, k1 = np.uint64(k0 & 0xFFFFFFFF), np.uint64(k1 & 0xFFFFFFFF)
    for _ in range(10):
        p0 = np.uint64(0xD2511F53) * c0
        p1 = np.uint64(0xCD9E8D57) * c2
        c0, c1, c2, c3 = (p1 >> np.uint64(32)) ^ c1 ^ k0, p1 & M32, (p0 >> np.uint64(32)) ^ c3 ^ k1, p0 & M32
        k0 = (k0 + np.uint64(0x9E3779B9)) & M32
        k1 = (k1 + np.uint64(0xBB67AE85)) & M32
    return c0, c1, c2, c3


def lattice_draws(layout: str, flat, chain: int, sweep: int, seed: int) -> np.ndarray:
    """The 23-bit Philox draws m of the sites at flat rows `flat` (int64 array) of one chain.

    "row8s": top 16 bits half flat % 2 of word (flat / 2) % 4 of counter (chain,
    flat / 8, sweep, "LSPI"), low 7 bits word 0 >> 25 of (chain, flat, sweep,
    "LREF").  "planes": bit 22 - b is bit 8 (flat % 4) + (flat % 32) / 4 of word
    b % 4 of counter (chain, flat / 32, sweep, "LPL0" + b / 4)."""
    flat = np.asarray(flat, dtype=np.int64)
    k0, k1 = seed & 0xFFFFFFFF, seed >> 32
    cs, ss = np.full(flat.shape, chain), np.full(flat.shape, sweep)
    if layout == "planes":
        pos = (8 * (flat & 3) + ((flat & 31) >> 2)).astype(np.uint64)
        m = np.zeros(flat.shape, dtype=np.int64)
        for ch in range(6):
            words = philox4x32_10(cs, flat >> 5, ss, np.full(flat.shape, SALT_LATTICE_PLANES + ch), k0, k1)
            for q in range(4):
                b = 4 * ch + q
                if b < 23:
                    m |= ((words[q] >> pos) & np.uint64(1)).astype(np.int64) << (22 - b)
        return m
    words = philox4x32_10(cs, flat >> 3, ss, np.full(flat.shape, SALT_LATTICE_SPIN), k0, k1)
    w = np.choose(((flat >> 1) & 3).astype(np.int64), words)
    h = (w >> (np.uint64(16) * (flat & 1).astype(np.uint64))) & np.uint64(0xFFFF)
    f = philox4x32_10(cs, flat, ss, np.full(flat.shape, SALT_LATTICE_REFILL), k0, k1)[0] >> np.uint64(25)
    return ((h << np.uint64(7)) | f).astype(np.int64)


def make_halfsweep(strips, *, chain: int = 0):
    """A `halfsweep` callable for LatticeStrips that updates its CPU tensors in place."""
    H, W = strips.H, strips.W
    hw = W // 2
    thr = strips.thresholds_host.astype(np.int64)

    def halfsweep(colour, row_lo, row_hi, sweep, stream, ctl_ptr=None):
        cc = strips.colours[colour].numpy()
        co = strips.colours[1 - colour].numpy()
        rows = np.arange(row_lo, row_hi)
        Y = (strips.global_row0 + rows) % H
        p = ((Y + colour) & 1)[:, None]
        j = np.arange(hw)[None, :]
        mid = co[rows].astype(np.int64)
        left = np.where(p == 0, co[rows][:, (j[0] - 1) % hw], mid)
        right = np.where(p == 0, mid, co[rows][:, (j[0] + 1) % hw])
        upv = co[rows - 1].astype(np.int64)
        dnv = co[rows + 1].astype(np.int64)
        idx = (left < 0) * 1 + (right < 0) * 2 + (upv < 0) * 4 + (dnv < 0) * 8
        flat = strips.block_rows[colour] + Y[:, None] * hw + j
        m = lattice_draws(strips.rng_layout, flat, chain, sweep, strips.seed)
        up = m < thr[idx]
        new = np.where(up, 1, -1).astype(np.int8)
        cc[rows] = new
        # observables of the counted rows
        sel = (rows >= strips.D) & (rows < strips.D + strips.h)
        if strips._trace is not None and sweep < strips._trace.shape[0]:
            tr = strips._trace.numpy()
            tr[sweep, 0] += int(new[sel].astype(np.int64).sum())
            if colour == 1:
                nsum = left + right + upv + dnv
                tr[sweep, 1] += int((new.astype(np.int64) * nsum)[sel].sum())

    return halfsweep


def lattice_energy_magnetisation(spins: np.ndarray, J: float = 1.0, h: float = 0.0):
    """(bond sum, magnetisation) of a periodic +-1 lattice: bonds = sum_i s_i (s_right + s_down)... counted once."""
    s = spins.astype(np.int64)
    bonds = int((s * np.roll(s, -1, axis=1)).sum() + (s * np.roll(s, -1, axis=0)).sum())
    return bonds, int(s.sum())
