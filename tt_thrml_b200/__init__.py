"""B200 execution backend for thrml block-Gibbs sampling.

One hand-written sm_100a CUDA kernel per sampling group per sweep, state kept
on the GPU, same public surface as tt-thrml (tt_thrml/__init__.py:1-96):
sample_states, sample_with_observation, make_executor/Executor,
make_mesh_executor/MeshExecutor, GaussianConditional, the device helpers and
the configuration factory (make_cuda_config; make_ttmlir_config kept for
drop-in callers).
"""

from .compiler import compile_program
from .conditional_samplers import GaussianConditional
from .core import (
    BulkRNGBuffers,
    CompiledFusedBlock,
    CompiledProgram,
    CUDAConfig,
    Family,
    FusedBlockSpec,
    FusedInteractionSpec,
    RNGSpec,
    TTMLIRConfig,
    close_device,
    close_devices,
    close_mesh_device,
    device_ids,
    is_mesh_device,
    make_cuda_config,
    make_ttmlir_config,
    open_device,
    open_devices,
    open_mesh_device,
)
from .executor import Executor, make_executor
from .mesh import MeshExecutor, make_mesh_executor, mesh_barrier, mesh_device_ids, mesh_size
from .rng import generate_bulk_rng, make_rng_spec, slice_rng_for_sweep


def sample_states(
    key, program, schedule, init_state_free, state_clamp, nodes_to_sample, *, ttnn=None, device=None, config=None
):
    """High-level sampling API matching thrml.sample_states (tt_thrml/__init__.py:31-51)."""
    config = config if config is not None else make_cuda_config()
    executor = make_executor(ttnn, device, program, config)
    return executor.sample_states(
        key, schedule, nodes_to_sample, init_state_free=init_state_free, state_clamp=state_clamp
    )


def sample_with_observation(
    key,
    program,
    schedule,
    init_state_free,
    state_clamp,
    observation_carry_init,
    f_observe,
    *,
    ttnn=None,
    device=None,
    config=None,
):
    """High-level observer API matching thrml.sample_with_observation (tt_thrml/__init__.py:54-77)."""
    config = config if config is not None else make_cuda_config()
    executor = make_executor(ttnn, device, program, config)
    return executor.sample_with_observation(
        key,
        schedule,
        f_observe,
        init_state_free=init_state_free,
        state_clamp=state_clamp,
        observation_carry_init=observation_carry_init,
    )


__all__ = [
    "CUDAConfig",
    "TTMLIRConfig",
    "make_cuda_config",
    "make_ttmlir_config",
    "open_device",
    "open_devices",
    "open_mesh_device",
    "close_device",
    "close_mesh_device",
    "close_devices",
    "Executor",
    "make_executor",
    "MeshExecutor",
    "make_mesh_executor",
    "sample_states",
    "sample_with_observation",
    "GaussianConditional",
]
