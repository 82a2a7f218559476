"""Per-step run history (JSONL) feeding the planner and the analysis tools.

Each ``StepRecord`` line has the reference's key layout
(``infra/observability/history_collector.py``): ``sequence_stats`` (p25..p99 of
prompt / generation / total lengths), ``timing`` (rollout, train, weight sync,
advantage, recompute, total and derived overhead), ``resource_config``,
``training_metrics``, ``pipeline_stats``, ``control_plane``, optional
``cost_model_comparison`` and per-sequence records.  The same length pairs are
also appended to ``runtime_length_profile.jsonl`` for online planning.
B200 addition: ``timing.device_train_time`` (CUDA-event time of the update,
max over ranks) next to the host wall-clock figures.
"""

from __future__ import annotations

import json
import os
import statistics
import threading
import time
from dataclasses import asdict, dataclass, field
from typing import Any, Dict, List, Optional, Tuple


def _pct(sorted_vals: List[float], q: float) -> float:
    pos = (len(sorted_vals) - 1) * q / 100.0
    lo = int(pos)
    hi = min(lo + 1, len(sorted_vals) - 1)
    return sorted_vals[lo] + (sorted_vals[hi] - sorted_vals[lo]) * (pos - lo)


@dataclass
class SequenceLengthStats:
    count: int = 0
    mean: float = 0.0
    std: float = 0.0
    min: int = 0
    max: int = 0
    p25: float = 0.0
    p50: float = 0.0
    p75: float = 0.0
    p90: float = 0.0
    p95: float = 0.0
    p99: float = 0.0

    @classmethod
    def from_lengths(cls, lengths: List[int]) -> "SequenceLengthStats":
        if not lengths:
            return cls()
        v = sorted(float(x) for x in lengths)
        return cls(len(v), round(statistics.fmean(v), 2), round(statistics.pstdev(v), 2), int(v[0]), int(v[-1]),
                   *(round(_pct(v, q), 1) for q in (25, 50, 75, 90, 95, 99)))


@dataclass
class TimingRecord:
    rollout_time: float = 0.0
    train_time: float = 0.0
    weight_sync_time: float = 0.0
    advantage_time: float = 0.0
    recompute_logprob_time: float = 0.0
    step_total_time: float = 0.0
    device_train_time: float = 0.0

    @property
    def overhead_time(self) -> float:
        used = (self.rollout_time + self.train_time + self.weight_sync_time + self.advantage_time
                + self.recompute_logprob_time)
        return max(0.0, self.step_total_time - used)


@dataclass
class ResourceConfig:
    n_total_gpus: int = 0
    train_gpus: int = 0
    rollout_gpus: int = 0
    train_backend: str = "b200"
    train_tp: int = 1
    train_pp: int = 1
    train_dp: int = 1
    rollout_tp_list: List[int] = field(default_factory=list)
    vllm_tp_size: int = 1
    vllm_num_instances: int = 1
    batch_size: int = 32
    micro_batch_size: int = 4
    B_global: int = 32
    max_new_tokens: int = 1024
    max_seq_length: int = 2048
    n_samples: int = 4
    temperature: float = 1.0
    model_path: str = ""
    model_params: float = 0.0


@dataclass
class CostModelComparison:
    predicted_rollout_time: float = 0.0
    actual_rollout_time: float = 0.0
    rollout_ratio: float = 0.0
    rollout_abs_error: float = 0.0
    predicted_train_time: float = 0.0
    actual_train_time: float = 0.0
    train_ratio: float = 0.0
    train_abs_error: float = 0.0
    eta_comp: float = 0.5
    eta_mem: float = 0.5
    gamma_overlap: float = 0.3


@dataclass
class PipelineStats:
    running_rollouts: int = 0
    accepted_rollouts: int = 0
    rejected_rollouts: int = 0
    model_version: int = 0


@dataclass
class TrainingMetrics:
    loss: float = 0.0
    pg_loss: float = 0.0
    kl: float = 0.0
    reward_mean: float = 0.0
    reward_std: float = 0.0
    reward_min: float = 0.0
    reward_max: float = 0.0
    n_trajectories: int = 0
    grpo_num_groups: int = 0
    grpo_mean_group_size: float = 0.0
    grpo_singleton_groups: int = 0
    grpo_zero_variance_groups: int = 0


@dataclass
class StepRecord:
    step: int = 0
    timestamp: float = 0.0
    timestamp_iso: str = ""
    wall_clock_elapsed: float = 0.0
    sequence_stats: Dict[str, Any] = field(default_factory=dict)
    timing: TimingRecord = field(default_factory=TimingRecord)
    resource_config: ResourceConfig = field(default_factory=ResourceConfig)
    training_metrics: TrainingMetrics = field(default_factory=TrainingMetrics)
    pipeline_stats: PipelineStats = field(default_factory=PipelineStats)
    control_plane: Dict[str, Any] = field(default_factory=dict)
    cost_model_comparison: Optional[CostModelComparison] = None
    sequences: List[dict] = field(default_factory=list)
    raw_prompt_lengths: List[int] = field(default_factory=list)
    raw_gen_lengths: List[int] = field(default_factory=list)

    def to_dict(self) -> dict:
        timing = {k: round(v, 6) for k, v in asdict(self.timing).items()}
        timing["overhead_time"] = round(self.timing.overhead_time, 6)
        d = {"step": self.step, "timestamp": self.timestamp, "timestamp_iso": self.timestamp_iso,
             "wall_clock_elapsed": round(self.wall_clock_elapsed, 3),
             "sequence_stats": {k: asdict(v) if isinstance(v, SequenceLengthStats) else v
                                for k, v in self.sequence_stats.items()},
             "sequences": self.sequences, "timing": timing, "resource_config": asdict(self.resource_config),
             "training_metrics": asdict(self.training_metrics), "pipeline_stats": asdict(self.pipeline_stats)}
        if self.control_plane:
            d["control_plane"] = self.control_plane
        if self.cost_model_comparison is not None:
            d["cost_model_comparison"] = asdict(self.cost_model_comparison)
        if self.raw_prompt_lengths:
            d["raw_prompt_lengths"] = self.raw_prompt_lengths
        if self.raw_gen_lengths:
            d["raw_gen_lengths"] = self.raw_gen_lengths
        return d


class HistoryDataCollector:
    def __init__(self, output_dir: str = "./logs/history", save_raw_lengths: bool = False, flush_interval: int = 10,
                 experiment_name: str = "", length_profile_path: str = ""):
        self.output_dir = output_dir
        self.save_raw_lengths = save_raw_lengths
        self.flush_interval = max(1, flush_interval)
        self.experiment_name = experiment_name
        self.length_profile_path = length_profile_path
        self._records: List[StepRecord] = []
        self._lock = threading.Lock()
        self._fh = None
        self._profile_fh = None
        self._start = 0.0
        self._initialized = False
        self._resource = ResourceConfig()

    def initialize(self) -> None:
        os.makedirs(self.output_dir, exist_ok=True)
        ts = time.strftime("%Y%m%d_%H%M%S")
        prefix = f"{self.experiment_name}_" if self.experiment_name else ""
        self.jsonl_path = os.path.join(self.output_dir, f"{prefix}history_{ts}.jsonl")
        self.summary_path = os.path.join(self.output_dir, f"{prefix}summary_{ts}.json")
        self._fh = open(self.jsonl_path, "w", encoding="utf-8")
        if self.length_profile_path:
            os.makedirs(os.path.dirname(self.length_profile_path) or ".", exist_ok=True)
            self._profile_fh = open(self.length_profile_path, "w", encoding="utf-8")
        self._start = time.time()
        self._initialized = True

    @staticmethod
    def _sequences(sequence_records, sequence_pairs, prompt_lengths, gen_lengths) -> List[dict]:
        if sequence_records:
            out = []
            for s in sequence_records:
                item = dict(s)
                item["input_len"], item["output_len"] = int(item.get("input_len", 0)), int(item.get("output_len", 0))
                if "total_output_tokens" in item:
                    item["total_output_tokens"] = int(item["total_output_tokens"])
                out.append(item)
            return out
        if sequence_pairs:
            return [{"input_len": int(p), "output_len": int(g)} for p, g in sequence_pairs]
        if prompt_lengths and gen_lengths and len(prompt_lengths) == len(gen_lengths):
            return [{"input_len": int(p), "output_len": int(g)} for p, g in zip(prompt_lengths, gen_lengths)]
        return []

    def record_step(self, step: int, sequence_pairs: Optional[List[Tuple[int, int]]] = None,
                    sequence_records: Optional[List[dict]] = None, prompt_lengths: Optional[List[int]] = None,
                    gen_lengths: Optional[List[int]] = None, rollout_time: float = 0.0, train_time: float = 0.0,
                    weight_sync_time: float = 0.0, advantage_time: float = 0.0,
                    recompute_logprob_time: float = 0.0, step_total_time: float = 0.0,
                    training_stats: Optional[dict] = None, pipeline_running: int = 0, pipeline_accepted: int = 0,
                    pipeline_rejected: int = 0, model_version: int = 0, predicted_rollout_time: float = 0.0,
                    predicted_train_time: float = 0.0, eta_comp: float = 0.5, eta_mem: float = 0.5,
                    gamma_overlap: float = 0.3, resource_config: Optional[ResourceConfig] = None,
                    control_plane: Optional[dict] = None, device_train_time: float = 0.0) -> StepRecord:
        if not self._initialized:
            self.initialize()
        now = time.time()
        seqs = self._sequences(sequence_records, sequence_pairs, prompt_lengths, gen_lengths)
        pl = [s["input_len"] for s in seqs] if seqs else [int(x) for x in (prompt_lengths or [])]
        gl = [s["output_len"] for s in seqs] if seqs else [int(x) for x in (gen_lengths or [])]
        st = dict(training_stats or {})
        rewards = st.get("rewards")
        if rewards is not None and len(rewards):
            rv = [float(x) for x in rewards]
            r_mean, r_std, r_min, r_max = statistics.fmean(rv), statistics.pstdev(rv), min(rv), max(rv)
        else:
            r_mean, r_std = st.get("reward_mean", 0.0), st.get("reward_std", 0.0)
            r_min, r_max = st.get("reward_min", 0.0), st.get("reward_max", 0.0)
        cmp = None
        if predicted_rollout_time > 0 or predicted_train_time > 0:
            cmp = CostModelComparison(
                predicted_rollout_time, rollout_time,
                round(predicted_rollout_time / rollout_time, 4) if rollout_time > 0 else 0.0,
                round(abs(predicted_rollout_time - rollout_time), 6), predicted_train_time, train_time,
                round(predicted_train_time / train_time, 4) if train_time > 0 else 0.0,
                round(abs(predicted_train_time - train_time), 6), eta_comp, eta_mem, gamma_overlap)
        if resource_config is not None:
            self._resource = resource_config
        rec = StepRecord(
            step=step, timestamp=now, timestamp_iso=time.strftime("%Y-%m-%dT%H:%M:%S", time.localtime(now)),
            wall_clock_elapsed=now - self._start,
            sequence_stats={"prompt": SequenceLengthStats.from_lengths(pl),
                            "generation": SequenceLengthStats.from_lengths(gl),
                            "total": SequenceLengthStats.from_lengths([p + g for p, g in zip(pl, gl)])},
            timing=TimingRecord(rollout_time, train_time, weight_sync_time, advantage_time, recompute_logprob_time,
                                step_total_time, device_train_time),
            resource_config=self._resource,
            training_metrics=TrainingMetrics(
                float(st.get("loss", 0.0)), float(st.get("pg_loss", 0.0)), float(st.get("kl", 0.0)), float(r_mean),
                float(r_std), float(r_min), float(r_max), int(st.get("n_trajectories", len(pl))),
                int(st.get("grpo_num_groups", 0)), float(st.get("grpo_mean_group_size", 0.0)),
                int(st.get("grpo_singleton_groups", 0)), int(st.get("grpo_zero_variance_groups", 0))),
            pipeline_stats=PipelineStats(pipeline_running, pipeline_accepted, pipeline_rejected, model_version),
            control_plane=dict(control_plane or {}), cost_model_comparison=cmp, sequences=seqs,
            raw_prompt_lengths=pl if self.save_raw_lengths else [], raw_gen_lengths=gl if self.save_raw_lengths else [])
        with self._lock:
            self._records.append(rec)
            self._fh.write(json.dumps(rec.to_dict(), default=str) + "\n")
            if self._profile_fh is not None:
                for i, s in enumerate(seqs):
                    self._profile_fh.write(json.dumps({"step": step, "timestamp": now, "sequence_index": i,
                                                       **{k: v for k, v in s.items()}}) + "\n")
            if len(self._records) % self.flush_interval == 0:
                self._flush()
        return rec

    @staticmethod
    def snapshot_resource_config(config) -> ResourceConfig:
        h = getattr(config, "heterogeneous_rollout", None)
        hetero = bool(getattr(h, "enabled", False))
        return ResourceConfig(
            n_total_gpus=getattr(config, "n_total_gpus", 0) or getattr(config, "train_gpus", 0) + getattr(config, "rollout_gpus", 0),
            train_gpus=getattr(config, "train_gpus", 0), rollout_gpus=getattr(config, "rollout_gpus", 0),
            train_backend=getattr(config, "train_backend", "b200"),
            train_tp=getattr(config, "train_tp_size", getattr(config, "tp_size", 1)),
            train_pp=getattr(config, "train_pp_size", 1), train_dp=getattr(config, "train_dp_size", 1),
            rollout_tp_list=list(h.tp_list) if hetero else [], vllm_tp_size=getattr(config, "vllm_tp_size", 1),
            vllm_num_instances=h.n_instances if hetero else getattr(config, "vllm_num_instances", 1),
            batch_size=getattr(config, "batch_size", 32), micro_batch_size=getattr(config, "micro_batch_size", 4),
            B_global=getattr(config, "batch_size", 32), max_new_tokens=getattr(config, "max_new_tokens", 1024),
            max_seq_length=getattr(config, "max_seq_length", 2048), n_samples=getattr(config, "n_samples", 4),
            temperature=getattr(config, "temperature", 1.0), model_path=getattr(config, "model_path", ""),
            model_params=getattr(getattr(config, "model_arch", None), "num_params", 0.0))

    def get_summary(self) -> dict:
        recs = self._records
        if not recs:
            return {"total_steps": 0}
        step_t = [r.timing.step_total_time for r in recs]
        tokens = sum(s["input_len"] + s["output_len"] for r in recs for s in r.sequences)
        out = {"total_steps": len(recs), "total_tokens": tokens,
               "mean_step_time": statistics.fmean(step_t), "tokens_per_second": tokens / max(sum(step_t), 1e-9),
               "mean_rollout_time": statistics.fmean(r.timing.rollout_time for r in recs),
               "mean_train_time": statistics.fmean(r.timing.train_time for r in recs)}
        sync = [r.timing.weight_sync_time for r in recs if r.timing.weight_sync_time > 0]
        out["mean_weight_sync_time"] = statistics.fmean(sync) if sync else 0.0
        ratios = [r.cost_model_comparison.train_ratio for r in recs if r.cost_model_comparison]
        if ratios:
            out["cost_model_train_ratio_mean"] = statistics.fmean(ratios)
        return out

    def compute_cost_model_accuracy(self) -> dict:
        cmp = [r.cost_model_comparison for r in self._records if r.cost_model_comparison is not None]
        if not cmp:
            return {}
        mape = lambda pairs: statistics.fmean(abs(p - a) / a for p, a in pairs if a > 0) if any(a > 0 for _, a in pairs) else 0.0  # noqa: E731
        return {"n": len(cmp),
                "rollout_mape": mape([(c.predicted_rollout_time, c.actual_rollout_time) for c in cmp]),
                "train_mape": mape([(c.predicted_train_time, c.actual_train_time) for c in cmp])}

    def _flush(self) -> None:
        if self._fh:
            self._fh.flush()
        if self._profile_fh:
            self._profile_fh.flush()

    def close(self) -> None:
        with self._lock:
            self._flush()
            if self._initialized:
                with open(self.summary_path, "w", encoding="utf-8") as fh:
                    json.dump(self.get_summary(), fh, indent=2)
            for f in (self._fh, self._profile_fh):
                if f:
                    f.close()
            self._fh = self._profile_fh = None
