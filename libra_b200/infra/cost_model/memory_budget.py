"""Per-device temporary memory of a logprob recompute (reference
``infra/cost_model/memory_budget.py``): b * (L - 1) * ceil(V / tp) * bytes *
workspace factor.  With the fused vocab log-softmax of this framework the
logits stay bf16 and only action rows are materialised, so callers pass
``logits_dtype_bytes=2`` and the action-row count when they use it.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass


@dataclass(frozen=True)
class RecomputeLogprobsMemoryEstimate:
    batch_size: int
    sequence_length: int
    local_vocab_size: int
    logits_dtype_bytes: int
    workspace_factor: float
    logits_bytes: int
    total_bytes: int

    def to_dict(self) -> dict:
        return asdict(self)


def estimate_recompute_logprobs_memory(*, batch_size: int, sequence_length: int, vocab_size: int,
                                       tensor_parallel_size: int, logits_dtype_bytes: int = 4,
                                       workspace_factor: float = 1.5) -> RecomputeLogprobsMemoryEstimate:
    b = max(1, int(batch_size))
    L = max(1, int(sequence_length))
    tp = max(1, int(tensor_parallel_size))
    nbytes = max(1, int(logits_dtype_bytes))
    factor = max(1.0, float(workspace_factor))
    local_v = -(-max(1, int(vocab_size)) // tp)
    logits = b * max(1, L - 1) * local_v * nbytes
    return RecomputeLogprobsMemoryEstimate(b, L, local_v, nbytes, factor, logits, int(logits * factor))
