"""B200-native token sampler for qwen600_engine.

``sampler`` mirrors the reference's sampler API over the C ABI of
``libqwen600_sampler.so`` (include/qwen600_sampler.h); ``workloads`` makes the
seeded synthetic logit batches used by the tests and the benchmark.
"""
from . import workloads  # noqa: F401

__version__ = "0.1.0"


def _sampler_module():
    import importlib
    return importlib.import_module(__name__ + ".sampler")


def __getattr__(name):
    # The CUDA library is loaded on first use so that the synthetic-workload
    # helpers import on machines without the built library.
    if name in ("sampler", "Sampler", "SamplingConfig", "build_sampler", "sample",
                "reset_sampler_history", "free_sampler"):
        mod = _sampler_module()
        return mod if name == "sampler" else getattr(mod, name)
    raise AttributeError(name)
