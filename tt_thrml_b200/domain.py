"""Domain decomposition of one large single-chain 2-D Ising lattice over GPUs.

The lattice (H x W, periodic, split-colour int8 layout: colour c is an
[H][W/2] array, see csrc/ising2d.cu) is cut into G row strips of h = H/G
rows, one per rank (one process per GPU, torch.distributed over NCCL).  Each
rank keeps its strip with D halo rows above and below, for both colours:
local row i holds lattice row (y0 - D + i) mod H.

Deep halos: right after an exchange every local row of both colours is
current.  The k-th half-sweep after it updates local rows [k, h + 2D - k):
their neighbours at rows k-1 and h + 2D - k are still current, and the rows
that go stale move inwards by one row per half-sweep.  After D half-sweeps
exactly the own rows [D, D + h) are current, and one exchange of D rows per
colour with each neighbour restores the halos.  The redundant halo updates
repeat the owner's computation bit for bit (Philox counters are keyed by the
global site and sweep), so the result does not depend on G or D: a G-GPU run
reproduces the 1-GPU run exactly.  One exchange per D/2 sweeps (D even)
instead of one per half-sweep keeps the NCCL latency off the critical path;
the redundant work is 2D/h of a strip.

Exchange of a period (per colour; `up` = rank - 1, `down` = rank + 1, mod G):
send own rows [h, h + D) to `down` and [D, 2D) to `up`; receive `up`'s into
local rows [0, D) and `down`'s into [h + D, h + 2D).  On one GPU the same
copies are local.  The reference has no exchange at all (its MeshExecutor
replicates one state, tt_thrml/mesh.py:29-46); this is the one real
collective of the sweep path.

Observables: the kernel adds, per sweep, the magnetisation of the own rows
and the bond sum sum_i s_i (sum of the 4 neighbours) into an int64 trace
[n_sweeps][2]; `trace()` all-reduces it over ranks once at the end.
Energy = -J * bonds - h * magnetisation (J, h the lattice's couplings).
"""

from __future__ import annotations

import ctypes
from typing import Callable

import numpy as np

from . import _native as nat
from .compiler import ising_pattern_tables, ising_stencil_layout
from .rng import seed_from_key


def _torch():
    import torch

    return torch


def _dist():
    try:
        import torch.distributed as dist
    except ImportError:
        return None
    return dist if dist.is_available() and dist.is_initialized() else None


class LatticeStrips:
    """Row-strip domain decomposition of an `IsingLattice2D` with one chain.

    program: the lattice (its tt_stencil() gives size and couplings).
    device: torch device of this rank.  halo: D, even, 2 <= D <= h.
    process_group: the ranks sharing the lattice (default: the world group
    when torch.distributed is initialised, else this process alone).
    halfsweep: the half-sweep implementation (default: the CUDA kernel
    tthrml_ising2d_halfsweep); tests substitute a host restatement to check
    the decomposition logic on CPU ranks.
    storage: "int8" (one byte per site, [rows][W/2] per colour) or "bits" (32
    sites per 32-bit word, [rows][W/64] per colour, site s of a word at bit
    8 (s % 4) + s / 4, bit set = -1; the bit-sliced kernel reads and writes
    them directly, 8x fewer bytes).  Default: "bits" for a count-symmetric
    lattice of width % 256 == 0 with the CUDA kernel, else "int8".
    exchange: "p2p" (default with the CUDA kernel): the last two half-sweeps
    of a period store the boundary rows straight into the neighbours'
    mailboxes in peer memory (CUDA IPC over NVLink), a flag publishes the
    period and the next period imports -- no host step, one CUDA graph for
    any number of periods; "nccl": the host posts NCCL (or gloo) send/recv
    of the halo rows between periods.
    """

    def __init__(self, program, *, device=None, halo: int = 32, process_group=None,
                 halfsweep: Callable | None = None, cuda_graphs: bool = True, exchange: str = "p2p",
                 storage: str | None = None):
        torch = _torch()
        st = program.tt_stencil()
        if st.get("kind") != "ising2d":
            raise ValueError("LatticeStrips runs 2-D Ising lattice programs")
        self.program = program
        self.H, self.W = (int(d) for d in st["dims"])
        dist = _dist()
        self.group = process_group
        if dist is not None:
            self.world, self.rank = dist.get_world_size(process_group), dist.get_rank(process_group)
        else:
            self.world, self.rank = 1, 0
        G = self.world
        if self.H % G or (self.H // G) % 2:
            raise ValueError(f"{self.H} rows do not split into {G} strips of an even number of rows")
        self.h = self.H // G
        D = int(halo)
        if D < 2 or D % 2 or D > self.h:
            raise ValueError(f"halo must be even and in [2, {self.h}], got {D}")
        if self.W % 32:
            raise ValueError("the lattice width must be a multiple of 32")
        self.D = D
        self.y0 = self.rank * self.h
        self.rows_local = self.h + 2 * D
        self.global_row0 = (self.y0 - D) % self.H
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.block_rows = tuple(int(r) for r in st["block_rows"])
        self.J, self.h_field = float(program.J), float(program.h)
        self._halfsweep = halfsweep or self._cuda_halfsweep
        self._custom = halfsweep is not None
        if exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange must be 'p2p' or 'nccl', got {exchange!r}")
        self.exchange = "nccl" if self._custom else exchange
        self._p2p = None
        self.cuda_graphs = bool(cuda_graphs) and not self._custom
        fields, thr = ising_pattern_tables(st["edge_weight"], st["site_bias"])
        self.fields_host, self.thresholds_host = fields, thr
        # Philox layout of the half-sweeps, the same as the executor's single-chain lattice plan
        self.rng_layout = ising_stencil_layout(thr, self.W)
        bits_ok = self.rng_layout == "planes" and self.W % 256 == 0
        if storage is None:
            storage = "bits" if bits_ok and not self._custom else "int8"
        if storage not in ("int8", "bits") or (storage == "bits" and not bits_ok):
            raise ValueError(f"storage must be 'int8' or, for a count-symmetric lattice of width % 256 == 0, "
                             f"'bits' (got {storage!r})")
        self.storage = storage
        self.row_bytes = self.W // 2 if storage == "int8" else self.W // 16
        if storage == "int8":
            self.colours = [torch.empty((self.rows_local, self.W // 2), dtype=torch.int8, device=self.device)
                            for _ in range(2)]
        else:
            self.colours = [torch.empty((self.rows_local, self.W // 64), dtype=torch.int32, device=self.device)
                            for _ in range(2)]
        self.fields = torch.from_numpy(fields).to(self.device)
        self.thresholds = torch.from_numpy(thr.view(np.int32)).to(self.device)
        self.seed = 0
        self.sweep = 0
        self._trace = None
        self._graphs: dict = {}
        self._ctl = None
        if not self._custom:
            self._lib = nat.lib()
            self._stream = torch.cuda.Stream(self.device)
        else:
            self._stream = None

    # ------------------------------------------------------------------ state
    def _rows_of_local(self) -> np.ndarray:
        return (self.global_row0 + np.arange(self.rows_local)) % self.H

    def load_lattice(self, spins: np.ndarray) -> None:
        """Loads a full lattice of +-1 (or bool, True = +1) spins [H][W] into this rank's strip and halos."""
        torch = _torch()
        a = np.asarray(spins)
        if a.shape != (self.H, self.W):
            raise ValueError(f"expected a ({self.H}, {self.W}) lattice, got {a.shape}")
        s = np.where(a.astype(np.float32) > 0, 1, -1).astype(np.int8)
        rows = self._rows_of_local()
        for c in range(2):
            cols = (np.arange(self.W // 2)[None, :] * 2) + ((rows[:, None] + c) & 1)
            part = np.take_along_axis(s[rows], cols, axis=1)
            self._store_rows(c, 0, torch.from_numpy(np.ascontiguousarray(part)))
        self._after_load()

    # bit-packed rows: site s of a 32-site group at bit 8 (s % 4) + s / 4, bit set = -1
    _PACK_ROWS = 1024  # rows per packing chunk (bounds the int64 temporaries)

    @staticmethod
    def _bit_shifts(device):
        torch = _torch()
        j = torch.arange(8, device=device, dtype=torch.int64)[:, None]
        k = torch.arange(4, device=device, dtype=torch.int64)[None, :]
        return 8 * k + j  # [j][k] for site 4j + k

    @classmethod
    def pack_rows(cls, rows):
        """int8 +-1 rows [n][W/2] -> int32 words [n][W/64] (bit-packed storage order)."""
        torch = _torch()
        n, half = rows.shape
        b = (rows < 0).reshape(n, half // 32, 8, 4).to(torch.int64)
        words = (b << cls._bit_shifts(rows.device)).sum(dim=(-1, -2))
        return torch.where(words >= 2**31, words - 2**32, words).to(torch.int32)

    @classmethod
    def unpack_rows(cls, words):
        """int32 words [n][W/64] -> int8 +-1 rows [n][W/2]."""
        torch = _torch()
        n, nw = words.shape
        w = words.to(torch.int64) & 0xFFFFFFFF
        bits = (w[:, :, None, None] >> cls._bit_shifts(words.device)) & 1
        return (1 - 2 * bits).to(torch.int8).reshape(n, nw * 32)

    def _store_rows(self, c: int, row0: int, rows) -> None:
        """Writes int8 +-1 rows [n][W/2] (any device) into local rows [row0, row0 + n) of colour c."""
        if self.storage == "int8":
            self.colours[c][row0 : row0 + rows.shape[0]].copy_(rows, non_blocking=True)
            return
        for a in range(0, rows.shape[0], self._PACK_ROWS):
            part = rows[a : a + self._PACK_ROWS].to(self.device, non_blocking=True)
            self.colours[c][row0 + a : row0 + a + part.shape[0]].copy_(self.pack_rows(part))

    def _own_rows(self, c: int):
        """The own rows [D, D + h) of colour c as int8 +-1 rows [h][W/2] on the device."""
        torch = _torch()
        own = self.colours[c][self.D : self.D + self.h]
        if self.storage == "int8":
            return own
        return torch.cat([self.unpack_rows(own[a : a + self._PACK_ROWS])
                          for a in range(0, self.h, self._PACK_ROWS)])

    def load_split_colours(self, colour0, colour1) -> None:
        """Loads the lattice from its two split-colour arrays [H][W/2] (host, ideally pinned, or device)."""
        torch = _torch()
        rows = self._rows_of_local()
        # the local rows are a few contiguous runs of lattice rows (the halos may wrap around the lattice)
        breaks = np.flatnonzero(np.diff(rows) != 1) + 1
        runs = np.split(np.arange(self.rows_local), breaks)
        ctx = torch.cuda.stream(self._stream) if self._stream is not None else _null()
        with ctx:
            for c, src in enumerate((colour0, colour1)):
                t = src if isinstance(src, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(src))
                if tuple(t.shape) != (self.H, self.W // 2) or t.dtype != torch.int8:
                    raise ValueError(f"expected an int8 ({self.H}, {self.W // 2}) array, got {tuple(t.shape)}")
                for run in runs:
                    y = int(rows[run[0]])
                    self._store_rows(c, int(run[0]), t[y : y + len(run)])
        self._after_load()

    def load_random(self, seed: int) -> None:
        """Uniform +-1 spins from a hash of (seed, site): identical for every strip decomposition."""
        torch = _torch()
        all_rows = torch.from_numpy(self._rows_of_local().astype(np.int64)).to(self.device)
        j = torch.arange(self.W // 2, device=self.device, dtype=torch.int64)
        for c in range(2):
            for a in range(0, self.rows_local, self._PACK_ROWS):
                rows = all_rows[a : a + self._PACK_ROWS]
                x = 2 * j[None, :] + ((rows[:, None] + c) & 1)
                z = rows[:, None] * self.W + x + (int(seed) & 0x3FFFFFFF) * 0x9E3779B1
                # 64-bit mix (splitmix64 finaliser constants), wrapping arithmetic
                z = (z ^ (z >> 30)) * -4658895280553007687
                z = (z ^ (z >> 27)) * -7723592293110705685
                z = z ^ (z >> 31)
                self._store_rows(c, a, torch.where((z & 1) == 1, 1, -1).to(torch.int8))
        self._after_load()

    def _after_load(self) -> None:
        if self.device.type == "cuda":
            _torch().cuda.synchronize(self.device)  # loads may run on the default stream

    def gather_lattice(self) -> np.ndarray:
        """The full lattice [H][W] of +-1 spins (all-gathered over ranks)."""
        torch = _torch()
        self._sync()
        own = [self._own_rows(c).cpu().numpy() for c in range(2)]
        strip = np.empty((self.h, self.W), dtype=np.int8)
        rows = self.y0 + np.arange(self.h)
        for c in range(2):
            cols = (np.arange(self.W // 2)[None, :] * 2) + ((rows[:, None] + c) & 1)
            np.put_along_axis(strip, cols, own[c], axis=1)
        dist = _dist()
        if self.world == 1 or dist is None:
            return strip
        t = torch.from_numpy(strip)
        if self._backend_is_nccl():
            t = t.to(self.device)
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t, group=self.group)
        return np.concatenate([p.cpu().numpy() for p in parts], axis=0)

    # -------------------------------------------------------------------- rng
    def prepare_rng(self, key, n_sweeps: int) -> None:
        """Philox seed from `key` (int or key data) and a trace of n_sweeps sweeps starting at sweep 0."""
        torch = _torch()
        self.seed = seed_from_key(key)
        self.sweep = 0
        if self._trace is not None and self._trace.shape[0] == int(n_sweeps):
            self._sync()
            self._trace.zero_()  # same buffer: captured graphs stay valid
        else:
            self._trace = torch.zeros((int(n_sweeps), 2), dtype=torch.int64, device=self.device)
            self._graphs.clear()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        self._ctl_value = None
        if self.exchange == "p2p":
            self._prime_p2p()

    # ----------------------------------------------------------------- sweeps
    def _cuda_halfsweep(self, colour: int, row_lo: int, row_hi: int, sweep: int, stream, ctl_ptr=None,
                        export=None) -> None:
        c, o = self.colours[colour], self.colours[1 - colour]
        trace = self._trace
        if self.storage == "bits":
            nat.check(
                self._lib.tthrml_ising2d_halfsweep_bits(
                    c.data_ptr(), o.data_ptr(), self.W, self.rows_local, 0, row_lo, row_hi, self.global_row0, self.H,
                    colour, self.block_rows[colour], self.thresholds.data_ptr(), 0, self.seed, sweep, ctl_ptr,
                    self.D, self.D + self.h, None if trace is None else trace.data_ptr(),
                    0 if trace is None else trace.shape[0], None if export is None else ctypes.byref(export),
                    nat.stream_handle(stream),
                ),
                "tthrml_ising2d_halfsweep_bits",
            )
            return
        if self.rng_layout == "planes":
            nat.check(
                self._lib.tthrml_ising2d_halfsweep_planes(
                    c.data_ptr(), o.data_ptr(), self.W, self.rows_local, 0, row_lo, row_hi, self.global_row0, self.H,
                    colour, self.block_rows[colour], self.thresholds.data_ptr(), 0, self.seed, sweep, ctl_ptr,
                    self.D, self.D + self.h, None if trace is None else trace.data_ptr(),
                    0 if trace is None else trace.shape[0], None if export is None else ctypes.byref(export),
                    nat.stream_handle(stream),
                ),
                "tthrml_ising2d_halfsweep_planes",
            )
            return
        nat.check(
            self._lib.tthrml_ising2d_halfsweep_x(
                c.data_ptr(), o.data_ptr(), self.W, self.rows_local, 0, row_lo, row_hi, self.global_row0, self.H,
                colour, self.block_rows[colour], self.thresholds.data_ptr(), self.fields.data_ptr(), None, 0, 0,
                self.seed, sweep, ctl_ptr, self.D, self.D + self.h,
                None if trace is None else trace.data_ptr(), 0 if trace is None else trace.shape[0],
                None if export is None else ctypes.byref(export), nat.stream_handle(stream),
            ),
            "tthrml_ising2d_halfsweep_x",
        )

    def _period(self, sweep0: int, stream, ctl_ptr=None) -> None:
        """One exchange period starting at sweep sweep0 (colour 0): D half-sweeps; with the peer-memory
        exchange also the halo import before them, the fused boundary-row export in the last two and the
        flag signal after them."""
        p2p = self.exchange == "p2p"
        per = self.D // 2
        h = stream if stream is None else nat.stream_handle(stream)
        if p2p:
            m = self._p2p
            nat.check(
                self._lib.tthrml_halo_import(  # rows of row_bytes bytes: "width" 2 * row_bytes
                    self.colours[0].data_ptr(), self.colours[1].data_ptr(), 2 * self.row_bytes, self.D, 0,
                    self.h + self.D,
                    m["own"], m["own"] + m["flags_off"], per, sweep0, ctl_ptr, m["error"].data_ptr(), h,
                ),
                "tthrml_halo_import",
            )
        for k in range(1, self.D + 1):
            colour = (k - 1) & 1
            sweep = sweep0 + (k - 1) // 2
            if p2p and k >= self.D - 1:
                self._halfsweep(colour, k, self.rows_local - k, sweep, stream, ctl_ptr, self._p2p["export"][colour])
            else:
                self._halfsweep(colour, k, self.rows_local - k, sweep, stream, ctl_ptr)
        if p2p:
            m = self._p2p
            nat.check(
                self._lib.tthrml_halo_signal(m["up"] + m["flags_off"] + 4, m["down"] + m["flags_off"], per, sweep0,
                                             ctl_ptr, h),
                "tthrml_halo_signal",
            )

    # ------------------------------------------------------ peer-memory exchange
    def _setup_p2p(self) -> None:
        """Mailboxes in IPC-exported device memory, the neighbours' opened, export descriptors."""
        if self._p2p is not None:
            return
        nat.bind_device(self.device.index)
        D = self.D
        plane = D * self.row_bytes
        mb_bytes = 8 * plane  # [2 slots][2 directions][2 colours][D][row bytes]
        flags_off = (mb_bytes + 255) // 256 * 256
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * 64)()
        nat.check(self._lib.tthrml_ipc_malloc(flags_off + 256, ctypes.byref(own), handle), "tthrml_ipc_malloc")
        ptrs = {self.rank: own.value}
        opened = []
        up = (self.rank - 1) % self.world
        down = (self.rank + 1) % self.world
        if self.world > 1:
            dist = _dist()
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=self.group)
            for r in {up, down} - {self.rank}:
                p = ctypes.c_void_p()
                buf = (ctypes.c_char * 64).from_buffer_copy(handles[r])
                nat.check(self._lib.tthrml_ipc_open(buf, ctypes.byref(p)), "tthrml_ipc_open")
                ptrs[r] = p.value
                opened.append(p.value)
        exports = []
        for c in range(2):
            ex = nat.HaloExport()
            ex.up = ptrs[up] + (1 * 2 + c) * plane  # up neighbour's "from down" mailbox
            ex.down = ptrs[down] + (0 * 2 + c) * plane  # down neighbour's "from up" mailbox
            ex.up_row0, ex.down_row0, ex.rows = D, self.h, D
            ex.slot_bytes = 4 * plane
            ex.sweeps_per_period = D // 2
            exports.append(ex)
        torch = _torch()
        self._p2p = {
            "own": own.value, "up": ptrs[up], "down": ptrs[down], "opened": opened, "flags_off": flags_off,
            "export": exports, "error": torch.zeros(1, dtype=torch.int32, device=self.device), "plane": plane,
        }

    def _prime_p2p(self) -> None:
        """Resets this rank's flags and, when resuming mid-run, replays the exchange of the period that
        completed last (its own boundary rows into the neighbours' mailboxes, then the signal), so the
        next period's import finds current halos.  Collective over the ranks."""
        torch = _torch()
        self._setup_p2p()
        m = self._p2p
        per = self.D // 2
        cuda_rt = torch.cuda
        cuda_rt.synchronize(self.device)
        dist = _dist()
        flags = (ctypes.c_uint32 * 2)(0, 0)
        nat.bind_device(self.device.index)
        nat.check(self._lib.tthrml_memcpy(ctypes.c_void_p(m["own"] + m["flags_off"]), flags, 8, None),
                  "tthrml_memcpy")
        m["error"].zero_()
        cuda_rt.synchronize(self.device)
        if self.world > 1 and dist is not None:
            dist.barrier(group=self.group)
        if self.sweep > 0:
            p_done = self.sweep // per
            slot = (p_done & 1) * 4 * m["plane"]
            for c in range(2):
                ex = m["export"][c]
                top = self.colours[c][self.D : 2 * self.D]
                bottom = self.colours[c][self.h : self.h + self.D]
                for dst, src in ((ex.up + slot, top.data_ptr()), (ex.down + slot, bottom.data_ptr())):
                    nat.check(self._lib.tthrml_memcpy(ctypes.c_void_p(dst), ctypes.c_void_p(src),
                                                      self.D * self.row_bytes, None), "tthrml_memcpy")
            nat.check(
                self._lib.tthrml_halo_signal(m["up"] + m["flags_off"] + 4, m["down"] + m["flags_off"], per,
                                             self.sweep - per, None, None),
                "tthrml_halo_signal",
            )
            cuda_rt.synchronize(self.device)
            if self.world > 1 and dist is not None:
                dist.barrier(group=self.group)

    def check_errors(self) -> None:
        """Raises if a halo import gave up waiting for a neighbour (peer-memory exchange)."""
        if self._p2p is not None:
            self._sync()
            if int(self._p2p["error"].item()):
                raise RuntimeError("halo exchange: a neighbour's period flag did not arrive in time")

    def close(self) -> None:
        """Releases the peer mappings and the mailbox (collective when several ranks share the lattice)."""
        if self._p2p is None:
            return
        self._sync()
        dist = _dist()
        if self.world > 1 and dist is not None:
            dist.barrier(group=self.group)
        nat.bind_device(self.device.index)
        for p in self._p2p["opened"]:
            self._lib.tthrml_ipc_close(ctypes.c_void_p(p))
        self._lib.tthrml_free(ctypes.c_void_p(self._p2p["own"]))
        self._p2p = None
        self._graphs.clear()

    def run_sweeps(self, n: int) -> None:
        """n sweeps (n a multiple of D/2), one halo exchange per D/2 sweeps."""
        per = self.D // 2
        if n % per:
            raise ValueError(f"sweeps must come in multiples of halo/2 = {per}")
        if self._trace is None:
            raise RuntimeError("prepare_rng must be called before running sweeps")
        torch = _torch()
        if self.exchange == "p2p":
            if self._p2p is None:
                self._prime_p2p()
            if self.cuda_graphs:
                self._replay_periods(n // per)
            else:
                nat.bind_device(self.device.index)
                with torch.cuda.stream(self._stream):
                    for _ in range(n // per):
                        self._period(self.sweep, self._stream)
                        self.sweep += per
            return
        for _ in range(n // per):
            if self.cuda_graphs:
                self._replay_periods(1)
            elif self._custom:
                self._period(self.sweep, None)
                self.sweep += per
            else:
                nat.bind_device(self.device.index)
                with torch.cuda.stream(self._stream):
                    self._period(self.sweep, self._stream)
                self.sweep += per
            self._exchange()

    def _replay_periods(self, n_periods: int) -> None:
        """Replays the graph of n_periods consecutive periods (captured once per count); advances self.sweep."""
        torch = _torch()
        nat.bind_device(self.device.index)
        per = self.D // 2
        if self._ctl is None:
            self._ctl = torch.zeros(2, dtype=torch.int64, device=self.device)
            self._ctl_host = torch.zeros(2, dtype=torch.int64, pin_memory=True)
            self._ctl_value = None
        g = self._graphs.get(n_periods)
        if g is None:
            g = torch.cuda.CUDAGraph()
            self._stream.synchronize()
            with torch.cuda.graph(g, stream=self._stream):
                s = torch.cuda.current_stream(self.device)
                for j in range(n_periods):
                    self._period(j * per, s, self._ctl.data_ptr())
                nat.check(self._lib.tthrml_ctl_advance(self._ctl.data_ptr(), n_periods * per, nat.stream_handle(s)),
                          "tthrml_ctl_advance")
            self._graphs[n_periods] = g
        want = (self.sweep, self.seed)
        with torch.cuda.stream(self._stream):
            if self._ctl_value != want:
                self._stream.synchronize()
                lo = self.seed & 0xFFFFFFFFFFFFFFFF
                self._ctl_host[0] = self.sweep
                self._ctl_host[1] = lo - (1 << 64) if lo >= (1 << 63) else lo
                self._ctl.copy_(self._ctl_host, non_blocking=True)
            g.replay()
        self.sweep += n_periods * per
        self._ctl_value = (self.sweep, self.seed)

    def _backend_is_nccl(self) -> bool:
        dist = _dist()
        return dist is not None and dist.get_backend(self.group) == "nccl"

    def _exchange(self) -> None:
        """Restores the D halo rows of both colours from the neighbouring strips."""
        torch = _torch()
        D, h = self.D, self.h
        if self.world == 1:
            ctx = torch.cuda.stream(self._stream) if self._stream is not None else _null()
            with ctx:
                for a in self.colours:
                    a[0:D].copy_(a[h : h + D])
                    a[h + D : h + 2 * D].copy_(a[D : 2 * D])
            return
        dist = _dist()
        up = (self.rank - 1) % self.world
        down = (self.rank + 1) % self.world
        ranks = dist.get_process_group_ranks(self.group) if self.group is not None else list(range(self.world))
        g_up, g_down = ranks[up], ranks[down]
        ops = []
        for a in self.colours:
            # pairwise order: what a rank sends to `down` first is what `down` receives from `up` first
            ops.append(dist.P2POp(dist.isend, a[h : h + D], g_down, group=self.group))
            ops.append(dist.P2POp(dist.irecv, a[0:D], g_up, group=self.group))
            ops.append(dist.P2POp(dist.isend, a[D : 2 * D], g_up, group=self.group))
            ops.append(dist.P2POp(dist.irecv, a[h + D : h + 2 * D], g_down, group=self.group))
        ctx = torch.cuda.stream(self._stream) if self._stream is not None else _null()
        with ctx:
            for req in dist.batch_isend_irecv(ops):
                req.wait()

    def _sync(self) -> None:
        if self._stream is not None:
            self._stream.synchronize()

    def synchronize(self) -> None:
        self._sync()

    # ------------------------------------------------------------ checkpoint
    def checkpoint(self) -> dict:
        """This rank's strip (both colours, halos included), sweep, seed and trace: enough to continue
        bit for bit.  Taken between run_sweeps calls, i.e. right after a halo exchange."""
        self._sync()
        return {
            "format": "tt_thrml_b200.strips/1",
            "dims": (self.H, self.W),
            "strips": self.world,
            "rank": self.rank,
            "halo": self.D,
            "storage": self.storage,
            "colours": [c.cpu().numpy() for c in self.colours],
            "sweep": int(self.sweep),
            "seed": int(self.seed),
            "trace": None if self._trace is None else self._trace.cpu().numpy(),
        }

    def restore(self, ckpt: dict) -> None:
        torch = _torch()
        want = ("tt_thrml_b200.strips/1", (self.H, self.W), self.world, self.rank, self.D, self.storage)
        got = (ckpt.get("format"), tuple(ckpt["dims"]), ckpt["strips"], ckpt["rank"], ckpt["halo"],
               ckpt.get("storage", "int8"))
        if want != got:
            raise ValueError(f"checkpoint {got} does not match this decomposition {want}")
        for dst, src in zip(self.colours, ckpt["colours"]):
            dst.copy_(torch.from_numpy(np.ascontiguousarray(src)))
        self.seed = int(ckpt["seed"])
        if ckpt["trace"] is not None:
            t = torch.from_numpy(np.ascontiguousarray(ckpt["trace"])).to(self.device)
            if self._trace is None or self._trace.shape != t.shape:
                self._trace = t
                self._graphs.clear()
            else:
                self._trace.copy_(t)
        self.sweep = int(ckpt["sweep"])
        self._ctl_value = None
        self._after_load()
        if self.exchange == "p2p":
            self._prime_p2p()

    # ------------------------------------------------------------ observables
    def trace(self) -> np.ndarray:
        """int64 [sweeps run][2]: (magnetisation, bond sum) of the whole lattice after each sweep."""
        torch = _torch()
        self._sync()
        t = self._trace[: self.sweep].clone()
        dist = _dist()
        if self.world > 1 and dist is not None:
            if not self._backend_is_nccl():
                t = t.cpu()
            dist.all_reduce(t, group=self.group)
        return t.cpu().numpy()

    def energy_magnetisation(self) -> np.ndarray:
        """float64 [sweeps][2]: energy -J*bonds - h*M and magnetisation per site after each sweep."""
        tr = self.trace().astype(np.float64)
        n = float(self.H * self.W)
        energy = -self.J * tr[:, 1] - self.h_field * tr[:, 0]
        return np.stack([energy / n, tr[:, 0] / n], axis=1)


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


__all__ = ["LatticeStrips"]
