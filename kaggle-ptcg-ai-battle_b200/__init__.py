"""ptcg_b200 -- B200-native (sm_100a) policy-learning hot path for the
dipamc/kaggle-ptcg-ai-battle PPO trainer.

The directory is imported under the module name ``ptcg_b200`` (see
``__graft_entry__.load_package``).  Pure-Python pieces (shape config,
synthetic inputs) import without a GPU; everything that computes goes through
the CUDA C-ABI library ``libptcg_b200.so`` (``native.lib()``), which raises
when the library is missing -- there is no CPU fallback.
"""
from . import config, synth  # noqa: F401

__all__ = ["config", "synth"]


def __getattr__(name):
    # computing pieces import lazily so config / synth work without the .so
    if name in ("native", "policy", "build", "smoke", "dp", "feed"):
        import importlib
        return importlib.import_module(f"{__name__}.{name}")
    if name == "PTCGPolicy":
        from .policy import PTCGPolicy
        return PTCGPolicy
    raise AttributeError(name)
