"""pytest plugin (loaded with ``-p _reference_alias``): makes ``import stratum.X``
resolve to this package's module for each reference module on the NF4 path, so
the reference's own test files run against this build unmodified."""

import importlib
import sys
import types

ALIASES = {  # reference module -> stratum_b200 module
    "upload": "upload",
    "assign": "assign",
    "stage": "stage",
    "pipeline": "pipeline",
    "host_staging": "boundary",
    "grad_hooks": "boundary",
    "nf4_linear": "nf4_linear",
    "scheduler": "scheduler",
    "runtime": "runtime",
    "layer_transfer": "upload",
}

_pkg = types.ModuleType("stratum")
_pkg.__path__ = []
sys.modules["stratum"] = _pkg
for _name, _target in ALIASES.items():
    _mod = importlib.import_module(f"stratum_b200.{_target}")
    sys.modules[f"stratum.{_name}"] = _mod
    setattr(_pkg, _name, _mod)
