"""Drop-in import name: `import tt_thrml` resolves to the B200 backend.

Scripts and tests written against tt-thrml import `tt_thrml`; this alias
re-exports tt_thrml_b200 and maps its submodules (tt_thrml.compiler,
tt_thrml.executor, tt_thrml.core, tt_thrml.rng, tt_thrml.mesh,
tt_thrml.conditional_samplers) onto the B200 implementations.
"""

import sys as _sys

import tt_thrml_b200 as _impl
from tt_thrml_b200 import *  # noqa: F401,F403
from tt_thrml_b200 import __all__  # noqa: F401

for _name in ("compiler", "executor", "core", "rng", "mesh", "conditional_samplers", "observers", "backend"):
    _mod = __import__(f"tt_thrml_b200.{_name}", fromlist=[_name])
    _sys.modules[f"{__name__}.{_name}"] = _mod
    globals()[_name] = _mod

sample_states = _impl.sample_states
sample_with_observation = _impl.sample_with_observation
