"""B200-native token sampler: a drop-in for llama.zig's src/sampler.zig.

The product is ``libb200_sampler.so`` (CUDA kernels for sm_100a behind the C
ABI in include/b200_sampler.h).  This package holds its sources (csrc/), the
build step (build.py), the Python mirror of the reference interface
(sampler.py), the batch sharding across ranks (sharding.py) and the benchmark
workloads (workloads.py).

The directory name contains a dot, so it is loaded by path, e.g.::

    import importlib.util, sys
    spec = importlib.util.spec_from_file_location(
        "llama_zig_b200", "llama.zig_b200/__init__.py",
        submodule_search_locations=["llama.zig_b200"])
    pkg = importlib.util.module_from_spec(spec); sys.modules["llama_zig_b200"] = pkg
    spec.loader.exec_module(pkg)
"""
from . import build, sharding, workloads  # noqa: F401
from .sampler import (  # noqa: F401
    EXPORTS, Sampler, SamplerConfig, SamplerError, lib, sample_argmax, status_string,
)
