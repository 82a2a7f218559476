"""Run history, phase tracing and run analysis."""

from libra_b200.infra.observability.history_collector import HistoryDataCollector, StepRecord  # noqa: F401
from libra_b200.infra.observability.phase_tracer import DeviceSpan, PhaseTracer  # noqa: F401
