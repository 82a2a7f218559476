"""libra_b200: a Blackwell-native asynchronous agentic-RL (GRPO) post-training framework.

Public API (same names as the reference package ``RL_Framework``):
``AsyncRLTrainer``, ``HeterogeneousRolloutEngine``, ``load_config``.
The heavy classes are imported lazily so that ``import libra_b200`` stays cheap.
"""

__version__ = "0.2.0"

from libra_b200.config import AsyncRLConfig, load_config, parse_args_and_load_config  # noqa: F401

_LAZY = {
    "AsyncRLTrainer": ("libra_b200.trainer.async_rl_trainer", "AsyncRLTrainer"),
    "HeterogeneousRolloutEngine": ("libra_b200.engine.heterogeneous_engine", "HeterogeneousRolloutEngine"),
    "B200TrainEngine": ("libra_b200.engine.train_engine", "B200TrainEngine"),
}


def __getattr__(name):
    if name in _LAZY:
        import importlib

        module, attr = _LAZY[name]
        return getattr(importlib.import_module(module), attr)
    raise AttributeError(f"module 'libra_b200' has no attribute {name!r}")


__all__ = ["AsyncRLConfig", "load_config", "parse_args_and_load_config", *sorted(_LAZY)]
