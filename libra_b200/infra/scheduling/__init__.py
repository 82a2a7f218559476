"""Rollout request schedulers: C-MLFQ and the baselines it is compared with."""

from libra_b200.infra.scheduling.base import BaseScheduler, InstanceHandle, SchedulingResult  # noqa: F401
from libra_b200.infra.scheduling.factory import SchedulerFactory, register_scheduler  # noqa: F401
