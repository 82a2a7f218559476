"""Scheduler registry (reference ``infra/scheduling/factory.py``)."""

from __future__ import annotations

from typing import Any, Dict, List, Type

from libra_b200.infra.scheduling.base import BaseScheduler

_REGISTRY: Dict[str, Type[BaseScheduler]] = {}


def register_scheduler(name: str, cls: Type[BaseScheduler]) -> None:
    _REGISTRY[name] = cls


def _builtin() -> None:
    if _REGISTRY:
        return
    from libra_b200.infra.scheduling.baselines import LAMLFQScheduler, LengthAwareScheduler, LoadBalanceScheduler
    from libra_b200.infra.scheduling.cmlfq_scheduler import CMLFQScheduler

    for name, cls in (("length_aware", LengthAwareScheduler), ("la_mlfq", LAMLFQScheduler),
                      ("cmlfq", CMLFQScheduler), ("load_balance", LoadBalanceScheduler)):
        register_scheduler(name, cls)


class SchedulerFactory:
    @staticmethod
    def create(scheduler_type: str, hetero_config: Any) -> BaseScheduler:
        _builtin()
        cls = _REGISTRY.get(scheduler_type)
        if cls is None:
            raise ValueError(f"Unknown scheduler type: '{scheduler_type}'. Available types: "
                             f"{', '.join(sorted(_REGISTRY))}")
        return cls.from_config(hetero_config)

    @staticmethod
    def available_types() -> List[str]:
        _builtin()
        return sorted(_REGISTRY)
