"""Minimal stand-in for upstream thrml's program construction (test fixture).

thrml 0.1.3 is not installed here (no JAX either), so the tests build
reference-style programs with this restatement of the parts of thrml's
public model the reference consumes (tt_thrml/compiler.py:220-271,
536-568): nodes, `Block`, `BlockGibbsSpec` (free super-blocks, clamped
blocks, node_shape_dtypes, global state locations), `InteractionGroup`,
the discrete EBM factors, `FactorSamplingProgram` and its per-block
interaction tables, and `SamplingSchedule`.  The gaussian factors mirror the
definitions in the reference's parity runner (tests/parity/_parity_runner.py
:44-109).  Sampling itself is not restated here: the CPU oracle does that.
"""

from __future__ import annotations

from dataclasses import dataclass
from types import SimpleNamespace

import numpy as np


class AbstractNode:
    pass


class SpinNode(AbstractNode):
    pass


class CategoricalNode(AbstractNode):
    pass


class ContinuousNode(AbstractNode):
    pass


def sd(dtype, shape=()):
    return SimpleNamespace(shape=shape, dtype=np.dtype(dtype))


DEFAULT_NODE_SHAPE_DTYPES = {SpinNode: sd(np.bool_), CategoricalNode: sd(np.uint8)}


class Block:
    def __init__(self, nodes):
        self.nodes = tuple(nodes)

    def __len__(self):
        return len(self.nodes)


@dataclass(frozen=True)
class SamplingSchedule:
    n_warmup: int
    n_samples: int
    steps_per_sample: int


class BlockGibbsSpec:
    """Free super-blocks (Block or tuple of Blocks) + clamped blocks.

    Global state: one array per distinct node shape/dtype, in order of first
    appearance over blocks; node_global_location_map[node] = (array index,
    position in that array).
    """

    def __init__(self, free_super_blocks, clamped_blocks, node_shape_dtypes=None):
        self.node_shape_dtypes = dict(DEFAULT_NODE_SHAPE_DTYPES if node_shape_dtypes is None else node_shape_dtypes)
        self.free_blocks, self.sampling_order = [], []
        for sb in free_super_blocks:
            group = (sb,) if isinstance(sb, Block) else tuple(sb)
            self.sampling_order.append([len(self.free_blocks) + i for i in range(len(group))])
            self.free_blocks.extend(group)
        self.clamped_blocks = list(clamped_blocks)
        self.blocks = self.free_blocks + self.clamped_blocks
        keys, counts = [], []
        self.node_global_location_map = {}
        for b in self.blocks:
            s = self.node_shape_dtypes[type(b.nodes[0])]
            key = (tuple(s.shape), np.dtype(s.dtype).str)
            if key not in keys:
                keys.append(key)
                counts.append(0)
            gi = keys.index(key)
            for node in b.nodes:
                self.node_global_location_map[node] = (gi, counts[gi])
                counts[gi] += 1
        self.global_sd_order = keys


class InteractionGroup:
    def __init__(self, interaction, head_nodes: Block, tail_nodes):
        self.interaction = interaction
        self.head_nodes = head_nodes
        self.tail_nodes = list(tail_nodes)
        for t in self.tail_nodes:
            assert len(t.nodes) == len(head_nodes.nodes)


class DiscreteEBMInteraction:
    """n_spin spin tails multiply; trailing weight axes index categorical tails."""

    def __init__(self, n_spin: int, weights):
        self.n_spin = int(n_spin)
        self.weights = np.asarray(weights, dtype=np.float32)

    def take(self, inds):
        return DiscreteEBMInteraction(self.n_spin, self.weights[inds])


class LinearInteraction:
    def __init__(self, weights):
        self.weights = np.asarray(weights, dtype=np.float32)

    def take(self, inds):
        return LinearInteraction(self.weights[inds])


class QuadraticInteraction:
    def __init__(self, inverse_weights):
        self.inverse_weights = np.asarray(inverse_weights, dtype=np.float32)

    def take(self, inds):
        return QuadraticInteraction(self.inverse_weights[inds])


class DiscreteEBMFactor:
    def __init__(self, spin_node_groups, categorical_node_groups, weights):
        self.spin = list(spin_node_groups)
        self.cat = list(categorical_node_groups)
        self.weights = np.asarray(weights, dtype=np.float32)

    def to_interaction_groups(self):
        groups = []
        ns = len(self.spin)
        for i, head in enumerate(self.spin):
            tails = self.spin[:i] + self.spin[i + 1 :] + self.cat
            groups.append(InteractionGroup(DiscreteEBMInteraction(ns - 1, self.weights), head, tails))
        for i, head in enumerate(self.cat):
            tails = self.spin + self.cat[:i] + self.cat[i + 1 :]
            w = np.moveaxis(self.weights, 1 + i, 1)
            groups.append(InteractionGroup(DiscreteEBMInteraction(ns, w), head, tails))
        return groups


class SpinEBMFactor(DiscreteEBMFactor):
    def __init__(self, node_groups, weights):
        super().__init__(node_groups, [], weights)


class CategoricalEBMFactor(DiscreteEBMFactor):
    def __init__(self, node_groups, weights):
        super().__init__([], node_groups, weights)


class LinearFactor:
    def __init__(self, weights, block):
        self.weights, self.block = np.asarray(weights, np.float32), block

    def to_interaction_groups(self):
        return [InteractionGroup(LinearInteraction(self.weights), self.block, [])]


class QuadraticFactor:
    def __init__(self, inverse_weights, block):
        self.inverse_weights, self.block = np.asarray(inverse_weights, np.float32), block

    def to_interaction_groups(self):
        return [InteractionGroup(QuadraticInteraction(self.inverse_weights), self.block, [])]


class CouplingFactor:
    def __init__(self, weights, blocks):
        self.weights, self.blocks = np.asarray(weights, np.float32), tuple(blocks)

    def to_interaction_groups(self):
        a, b = self.blocks
        return [
            InteractionGroup(LinearInteraction(self.weights), a, [b]),
            InteractionGroup(LinearInteraction(self.weights), b, [a]),
        ]


class SpinGibbsConditional:
    pass


class CategoricalGibbsConditional:
    def __init__(self, n_categories):
        self.n_categories = n_categories


class GaussianSampler:
    pass


class FactorSamplingProgram:
    """Per free block, the interaction groups with heads in the block, sliced
    to (n_block_nodes, k) with k = most head occurrences of one node; unused
    slots point at edge 0 and are inactive."""

    def __init__(self, gibbs_spec, samplers, factors, other_interaction_groups):
        self.gibbs_spec = gibbs_spec
        self.samplers = list(samplers)
        groups = [g for f in factors for g in f.to_interaction_groups()] + list(other_interaction_groups)
        loc = gibbs_spec.node_global_location_map
        self.per_block_interactions = []
        self.per_block_interaction_active = []
        self.per_block_interaction_global_inds = []
        self.per_block_interaction_global_slices = []
        for block in gibbs_spec.free_blocks:
            pos = {node: i for i, node in enumerate(block.nodes)}
            inters, actives, ginds, gslices = [], [], [], []
            for g in groups:
                occ = [[] for _ in block.nodes]
                for e, node in enumerate(g.head_nodes.nodes):
                    if node in pos:
                        occ[pos[node]].append(e)
                k = max((len(o) for o in occ), default=0)
                if k == 0:
                    continue
                inds = np.zeros((len(block.nodes), k), dtype=np.int64)
                active = np.zeros((len(block.nodes), k), dtype=bool)
                for i, o in enumerate(occ):
                    inds[i, : len(o)] = o
                    active[i, : len(o)] = True
                inters.append(g.interaction.take(inds))
                actives.append(active)
                gi_list, gs_list = [], []
                for tail in g.tail_nodes:
                    gi_list.append(loc[tail.nodes[0]][0])
                    gs_list.append(np.array([[loc[tail.nodes[e]][1] for e in row] for row in inds], dtype=np.int32))
                ginds.append(gi_list)
                gslices.append(gs_list)
            self.per_block_interactions.append(inters)
            self.per_block_interaction_active.append(actives)
            self.per_block_interaction_global_inds.append(ginds)
            self.per_block_interaction_global_slices.append(gslices)


class IsingEBM:
    """Ising model as two spin factors (bias and pairwise), beta folded in."""

    def __init__(self, nodes, edges, biases, weights, beta):
        self.nodes = list(nodes)
        self.edges = list(edges)
        self.biases = np.asarray(biases, np.float32)
        self.weights = np.asarray(weights, np.float32)
        self.beta = np.float32(beta)

    @property
    def factors(self):
        return [
            SpinEBMFactor([Block(self.nodes)], self.beta * self.biases),
            SpinEBMFactor([Block([u for u, _ in self.edges]), Block([v for _, v in self.edges])], self.beta * self.weights),
        ]


def IsingSamplingProgram(model, free_blocks, clamped_blocks):
    spec = BlockGibbsSpec(free_blocks, clamped_blocks)
    return FactorSamplingProgram(spec, [SpinGibbsConditional() for _ in spec.free_blocks], model.factors, [])


# ----------------------------------------------------------------------------
# The reference's parity scenarios (tests/parity/_parity_runner.py:202-621),
# rebuilt with the same parameters; initial states are seeded numpy draws.
# ----------------------------------------------------------------------------


@dataclass(frozen=True)
class SampleCase:
    program: FactorSamplingProgram
    schedule: SamplingSchedule
    init_state_free: list
    state_clamp: list
    nodes_to_sample: list


def make_spin_case() -> SampleCase:
    nodes = [SpinNode() for _ in range(4)]
    bias = SpinEBMFactor([Block(nodes)], [0.35, -0.25, 0.2, -0.15])
    pair = SpinEBMFactor([Block(nodes[:-1]), Block(nodes[1:])], [0.75, -0.45, 0.3])
    free = [Block(nodes[0::2]), Block(nodes[1::2])]
    prog = FactorSamplingProgram(BlockGibbsSpec(free, []), [SpinGibbsConditional()] * 2, [bias, pair], [])
    rng = np.random.default_rng(1001)
    init = [rng.integers(0, 2, len(b.nodes)).astype(bool) for b in free]
    return SampleCase(prog, SamplingSchedule(12, 96, 2), init, [], [Block(nodes)])


def make_categorical_case(n_categories: int = 3) -> SampleCase:
    nodes = [CategoricalNode() for _ in range(4)]
    bias = CategoricalEBMFactor(
        [Block(nodes)],
        [[0.4, -0.15, 0.0], [-0.1, 0.25, -0.2], [0.05, -0.35, 0.3], [0.2, -0.05, -0.1]],
    )
    pair = CategoricalEBMFactor(
        [Block(nodes[:-1]), Block(nodes[1:])],
        [
            [[0.9, -0.3, 0.2], [-0.1, 0.4, -0.2], [0.15, -0.05, 0.25]],
            [[0.25, -0.4, 0.1], [0.35, 0.2, -0.3], [-0.15, 0.1, 0.45]],
            [[0.5, -0.2, -0.1], [0.05, 0.3, -0.25], [-0.2, 0.15, 0.35]],
        ],
    )
    free = [Block(nodes[0::2]), Block(nodes[1::2])]
    sampler = CategoricalGibbsConditional(n_categories)
    prog = FactorSamplingProgram(BlockGibbsSpec(free, []), [sampler, sampler], [bias, pair], [])
    rng = np.random.default_rng(2002)
    init = [rng.integers(0, n_categories, len(b.nodes)).astype(np.uint8) for b in free]
    return SampleCase(prog, SamplingSchedule(12, 256, 2), init, [], [Block(nodes)])


def make_gaussian_case() -> SampleCase:
    nodes = [ContinuousNode() for _ in range(3)]
    free = [Block(nodes[0::2]), Block(nodes[1::2])]
    sds = {ContinuousNode: sd(np.float32)}
    prog = FactorSamplingProgram(
        BlockGibbsSpec(free, [], sds),
        [GaussianSampler(), GaussianSampler()],
        [
            LinearFactor([0.15, -0.35, 0.2], Block(nodes)),
            QuadraticFactor([0.7, 0.9, 0.8], Block(nodes)),
            CouplingFactor([0.12, -0.08], (Block(nodes[:-1]), Block(nodes[1:]))),
        ],
        [],
    )
    rng = np.random.default_rng(3003)
    init = [(0.2 * rng.standard_normal(len(b.nodes))).astype(np.float32) for b in free]
    return SampleCase(prog, SamplingSchedule(16, 128, 3), init, [], [Block(nodes)])


def make_mixed_case(n_categories: int = 3) -> SampleCase:
    spin = [SpinNode() for _ in range(2)]
    cat = [CategoricalNode() for _ in range(2)]
    cont = [ContinuousNode() for _ in range(2)]
    free_super = [
        (Block([spin[0]]), Block([cat[0]]), Block([cont[0]])),
        (Block([spin[1]]), Block([cat[1]]), Block([cont[1]])),
    ]
    sds = {SpinNode: sd(np.bool_), CategoricalNode: sd(np.uint8), ContinuousNode: sd(np.float32)}
    prog = FactorSamplingProgram(
        BlockGibbsSpec(free_super, [], sds),
        [SpinGibbsConditional(), CategoricalGibbsConditional(n_categories), GaussianSampler()] * 2,
        [
            SpinEBMFactor([Block(spin)], [0.25, -0.2]),
            CategoricalEBMFactor([Block(cat)], [[0.2, -0.1, 0.0], [-0.15, 0.3, -0.05]]),
            DiscreteEBMFactor([Block(spin)], [Block(cat)], [[0.55, -0.25, 0.15], [-0.2, 0.4, 0.1]]),
            LinearFactor([0.1, -0.2], Block(cont)),
            QuadraticFactor([0.85, 0.75], Block(cont)),
            CouplingFactor([0.11], (Block([cont[0]]), Block([cont[1]]))),
        ],
        [],
    )
    rng = np.random.default_rng(4004)
    init = [
        rng.integers(0, 2, 1).astype(bool),
        rng.integers(0, n_categories, 1).astype(np.uint8),
        (0.2 * rng.standard_normal(1)).astype(np.float32),
        rng.integers(0, 2, 1).astype(bool),
        rng.integers(0, n_categories, 1).astype(np.uint8),
        (0.2 * rng.standard_normal(1)).astype(np.float32),
    ]
    return SampleCase(prog, SamplingSchedule(14, 96, 2), init, [], [Block(spin), Block(cat), Block(cont)])


def make_clamp_case():
    nodes = [SpinNode() for _ in range(3)]
    free = [Block([nodes[0]]), Block([nodes[1]])]
    clamped = [Block([nodes[2]])]
    prog = FactorSamplingProgram(
        BlockGibbsSpec(free, clamped),
        [SpinGibbsConditional(), SpinGibbsConditional()],
        [
            SpinEBMFactor([Block(nodes)], [0.15, -0.25, 0.4]),
            SpinEBMFactor([Block(nodes[:-1]), Block(nodes[1:])], [0.55, -0.35]),
        ],
        [],
    )
    schedule = SamplingSchedule(10, 96, 2)
    init = [np.array([True]), np.array([False])]
    clamp = [np.array([True])]
    return prog, schedule, init, clamp, nodes


def two_spin_superblock_program():
    """Two coupled spins (J = -1) in one superblock (tests/test_compiler_lowering.py:59-77)."""
    nodes = [SpinNode(), SpinNode()]
    free = (Block([nodes[0]]), Block([nodes[1]]))
    return FactorSamplingProgram(
        BlockGibbsSpec([free], []),
        [SpinGibbsConditional(), SpinGibbsConditional()],
        [SpinEBMFactor([Block([nodes[0]]), Block([nodes[1]])], [-1.0])],
        [],
    )


def ising_grid_program(height: int, width: int, *, J: float = 1.0, h: float = 0.0, beta: float = 0.44,
                       periodic: bool = True, colour_blocks: bool = True):
    """An IsingEBM over a height x width grid (edges to the right and lower neighbours, wrapping when
    periodic; J a scalar or one coupling per edge), free blocks = the two checkerboard colours with sites
    in row-major order."""
    nodes = [SpinNode() for _ in range(height * width)]
    edges = []
    for y in range(height):
        for x in range(width):
            if periodic or x + 1 < width:
                edges.append((nodes[y * width + x], nodes[y * width + (x + 1) % width]))
            if periodic or y + 1 < height:
                edges.append((nodes[y * width + x], nodes[((y + 1) % height) * width + x]))
    Jv = np.broadcast_to(np.asarray(J, np.float32), (len(edges),)).copy()
    model = IsingEBM(nodes, edges, np.full(len(nodes), h, np.float32), Jv, beta)
    colour = [(i // width + i % width) % 2 for i in range(len(nodes))]
    if colour_blocks:
        free = [Block([nd for nd, c in zip(nodes, colour) if c == k]) for k in range(2)]
    else:  # rows split in halves: not a checkerboard
        free = [Block(nodes[: len(nodes) // 2]), Block(nodes[len(nodes) // 2 :])]
    return IsingSamplingProgram(model, free, []), nodes


def potts_grid_program(dims, J, bias):
    """A q-state Potts model over a periodic X x Y x Z grid written with thrml factors: one
    CategoricalEBMFactor per axis over the (site, site + unit step) edges with that axis's q x q matrix,
    one for the site biases; free blocks = the two checkerboard colours with sites in row-major order."""
    X, Y, Z = (int(d) for d in dims)
    J = np.asarray(J, np.float32)
    q = J.shape[-1]
    nodes = [CategoricalNode() for _ in range(X * Y * Z)]
    idx = lambda x, y, z: ((z % Z) * Y + (y % Y)) * X + (x % X)  # noqa: E731
    factors = [CategoricalEBMFactor([Block(nodes)], np.asarray(bias, np.float32).reshape(len(nodes), q))]
    for a, (dx, dy, dz) in enumerate(((1, 0, 0), (0, 1, 0), (0, 0, 1))):
        us, vs = [], []
        for z in range(Z):
            for y in range(Y):
                for x in range(X):
                    us.append(nodes[idx(x, y, z)])
                    vs.append(nodes[idx(x + dx, y + dy, z + dz)])
        factors.append(CategoricalEBMFactor([Block(us), Block(vs)], np.broadcast_to(J[a], (len(us), q, q)).copy()))
    colour = [((i % X) + (i // X) % Y + i // (X * Y)) % 2 for i in range(len(nodes))]
    free = [Block([nd for nd, c in zip(nodes, colour) if c == k]) for k in range(2)]
    spec = BlockGibbsSpec(free, [], {CategoricalNode: sd(np.uint8)})
    sampler = CategoricalGibbsConditional(q)
    return FactorSamplingProgram(spec, [sampler, sampler], factors, []), nodes
