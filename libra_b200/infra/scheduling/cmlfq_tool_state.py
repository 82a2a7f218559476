"""Tool-return state abstraction for C-MLFQ (reference ``infra/scheduling/cmlfq_tool_state.py``).

A tool return is reduced to ``tool_type:size_class:status``; the size class
uses payload thresholds (small <= 500, large > 5000 by default, configurable)
and the status is success / failure / timeout detected from common dict fields.
The key string is part of the persisted prefix-tree format.
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from dataclasses import dataclass
from enum import Enum
from typing import Any, List


class PayloadSizeClass(Enum):
    SizeSmall = "small"
    SizeMedium = "medium"
    SizeLarge = "large"


class ExecutionStatus(Enum):
    ToolSuccess = "success"
    ToolFailure = "failure"
    ToolTimeout = "timeout"


@dataclass(frozen=True)
class ToolReturnState:
    tool_type: str
    payload_size_class: PayloadSizeClass
    execution_status: ExecutionStatus
    raw_payload_size: int = 0

    def to_key(self) -> str:
        return f"{self.tool_type}:{self.payload_size_class.value}:{self.execution_status.value}"

    @classmethod
    def from_key(cls, key: str) -> "ToolReturnState":
        parts = key.split(":")
        if len(parts) != 3:
            raise ValueError(f"Invalid ToolReturnState key: {key}")
        return cls(parts[0], PayloadSizeClass(parts[1]), ExecutionStatus(parts[2]))


class ToolStateExtractor(ABC):
    @abstractmethod
    def extract(self, tool_result: Any) -> ToolReturnState: ...

    @abstractmethod
    def can_handle(self, tool_result: Any) -> bool: ...


_FAIL_WORDS = {"error", "failure", "failed"}
_TIMEOUT_WORDS = {"timeout", "timed_out"}
_SIZE_NAMES = {c.value: c for c in PayloadSizeClass}


class DefaultToolStateExtractor(ToolStateExtractor):
    SMALL_THRESHOLD = 500
    LARGE_THRESHOLD = 5000

    def __init__(self, small_threshold: int = SMALL_THRESHOLD, large_threshold: int = LARGE_THRESHOLD):
        if small_threshold < 0 or large_threshold < small_threshold:
            raise ValueError("invalid payload size thresholds")
        self.small_threshold = small_threshold
        self.large_threshold = large_threshold

    def can_handle(self, tool_result: Any) -> bool:
        return isinstance(tool_result, (str, dict))

    def size_class(self, n: int) -> PayloadSizeClass:
        if n <= self.small_threshold:
            return PayloadSizeClass.SizeSmall
        return PayloadSizeClass.SizeMedium if n <= self.large_threshold else PayloadSizeClass.SizeLarge

    def extract(self, tool_result: Any) -> ToolReturnState:
        if isinstance(tool_result, str):
            status = ExecutionStatus.ToolFailure if "error" in tool_result.lower() else ExecutionStatus.ToolSuccess
            return ToolReturnState("text", self.size_class(len(tool_result)), status, len(tool_result))
        if isinstance(tool_result, dict):
            return self._from_dict(tool_result)
        return ToolReturnState("unknown", PayloadSizeClass.SizeMedium, ExecutionStatus.ToolSuccess)

    def _from_dict(self, d: dict) -> ToolReturnState:
        kind = str(d.get("tool_type", d.get("tool", "unknown")))
        body = d.get("output", d.get("result", d.get("content", "")))
        text = body if isinstance(body, str) else str(body)
        n = int(d.get("payload_tokens", len(text)))
        size = _SIZE_NAMES.get(str(d.get("payload_size_class", "")).lower()) or self.size_class(n)
        declared = str(d.get("status", "")).lower()
        if declared in _TIMEOUT_WORDS:
            status = ExecutionStatus.ToolTimeout
        elif (declared in _FAIL_WORDS or any(k in d for k in ("error", "exception", "traceback"))
              or (isinstance(body, str) and "error" in body.lower())):
            status = ExecutionStatus.ToolFailure
        else:
            status = ExecutionStatus.ToolSuccess
        return ToolReturnState(kind, size, status, n)


class ToolStateExtractorRegistry:
    """Most recently registered extractor that can handle the value wins."""

    def __init__(self):
        self._extractors: List[ToolStateExtractor] = []

    def register(self, extractor: ToolStateExtractor) -> None:
        self._extractors.append(extractor)

    def extract(self, tool_result: Any) -> ToolReturnState:
        for ex in reversed(self._extractors):
            if ex.can_handle(tool_result):
                return ex.extract(tool_result)
        return DefaultToolStateExtractor().extract(tool_result)

    @staticmethod
    def create_default_registry(small_threshold: int = DefaultToolStateExtractor.SMALL_THRESHOLD,
                                large_threshold: int = DefaultToolStateExtractor.LARGE_THRESHOLD):
        reg = ToolStateExtractorRegistry()
        reg.register(DefaultToolStateExtractor(small_threshold, large_threshold))
        return reg
