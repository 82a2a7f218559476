"""External-simulator adapters behind a CostModel-compatible facade.

Command contract (same placeholders and result markers as the reference,
``infra/cost_model/simulator_adapters.py``, so existing Sailor/Vidur wrapper
scripts keep working):

* training: ``sailor_train_command`` with ``{input_json} {output_json}
  {sailor_path} {rl_framework_path} {python}``; the command writes
  ``output_json`` or prints ``SAILOR_RESULT_JSON=<json>`` containing one of
  ``t_train / iteration_time / iteration_time_s / iteration_time_sec /
  throughput`` and optionally ``is_oom``.
* rollout: ``vidur_rollout_command`` with ``{trace_csv} {output_json}
  {output_dir} {vidur_path} {rl_framework_path} {python} {tp_list}
  {num_replicas} {tensor_parallel_size}``; result ``VIDUR_RESULT_JSON=`` or
  ``output_json`` with ``makespan / t_rollout / ...`` or a Vidur
  ``request_metrics.csv``.

``HybridSimulatorCostModel`` picks the backend per side from
``global_resource_planner.{train,rollout}_backend`` ("analytic", "sailor",
"vidur", "hybrid") and falls back to the B200 analytic model when a simulator
fails (unless ``simulator_allow_fallback`` is false).
"""

from __future__ import annotations

import csv
import json
import math
import os
import shlex
import subprocess
import tempfile
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional, Tuple

from libra_b200.infra.cost_model.model import CostModel, RequestInfo, RolloutClusterConfig, TrainParallelConfig

PKG_ROOT = Path(__file__).resolve().parents[2]


class SimulatorBackendError(RuntimeError):
    pass


@dataclass
class SimulatorEstimate:
    seconds: float
    details: Dict[str, Any]
    is_oom: bool = False


TRAIN_KEYS = ("t_train", "iteration_time", "iteration_time_s", "iteration_time_sec")
ROLLOUT_KEYS = ("makespan", "t_rollout", "makespan_s", "total_time", "total_time_s")


def _seconds(payload: Dict[str, Any], keys: Tuple[str, ...]) -> float:
    for k in keys:
        v = payload.get(k)
        if v is not None and math.isfinite(float(v)) and float(v) >= 0:
            return float(v)
    if float(payload.get("throughput", 0) or 0) > 0:
        return 1.0 / float(payload["throughput"])
    raise SimulatorBackendError(f"Simulator output does not contain any time key from {keys}")


def _abs(path: str) -> Path:
    p = Path(path).expanduser()
    return p if p.is_absolute() else (PKG_ROOT.parent / p).resolve()


def _cache_dir(planner_cfg) -> str:
    p = _abs(planner_cfg.simulator_cache_dir)
    p.mkdir(parents=True, exist_ok=True)
    return str(p)


def _run(cmd: str, cwd: Optional[Path], timeout: float, env_extra: Optional[Dict[str, str]] = None):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run(cmd, shell=True, cwd=str(cwd) if cwd else None, env=env, text=True, capture_output=True,
                          timeout=timeout, check=False)


def _marker(stdout: str, marker: str) -> Optional[dict]:
    for line in stdout.splitlines():
        if line.startswith(marker):
            return json.loads(line[len(marker):])
    return None


class SailorTrainingSimulatorAdapter:
    def __init__(self, planner_config, rl_config):
        self.pc, self.rc = planner_config, rl_config
        self.path = _abs(planner_config.sailor_path)
        self.timeout = float(planner_config.simulator_timeout_s)

    def evaluate_training(self, tc: TrainParallelConfig, B_global: int, L: int) -> SimulatorEstimate:
        cmd = (self.pc.sailor_train_command or "").strip()
        if not cmd:
            raise SimulatorBackendError("sailor_train_command is empty")
        if not self.path.exists():
            raise SimulatorBackendError(f"Sailor path does not exist: {self.path}")
        with tempfile.TemporaryDirectory(prefix="sailor_train_", dir=_cache_dir(self.pc)) as td:
            inp, out = Path(td) / "input.json", Path(td) / "output.json"
            inp.write_text(json.dumps({"train_config": asdict(tc), "batch_size": B_global, "avg_sequence_length": L,
                                       "hardware": asdict(self.rc.hardware), "model_arch": asdict(self.rc.model_arch),
                                       "profiling": asdict(self.rc.profiling)}, indent=2))
            full = cmd.format(input_json=shlex.quote(str(inp)), output_json=shlex.quote(str(out)),
                              sailor_path=shlex.quote(str(self.path)), rl_framework_path=shlex.quote(str(PKG_ROOT)),
                              python=shlex.quote(self.pc.sailor_python))
            proc = _run(full, self.path, self.timeout, {"PYTHONPATH": str(self.path)})
            if proc.returncode != 0:
                raise SimulatorBackendError(f"Sailor training simulator failed (code={proc.returncode}): "
                                            f"{proc.stderr[-1000:]}")
            res = json.loads(out.read_text()) if out.exists() else _marker(proc.stdout, "SAILOR_RESULT_JSON=")
            if res is None:
                raise SimulatorBackendError("Sailor simulator did not write output_json or SAILOR_RESULT_JSON")
            return SimulatorEstimate(_seconds(res, TRAIN_KEYS), {"backend": "sailor", "command": full, "raw": res},
                                     bool(res.get("is_oom", res.get("oom", False))))


class VidurRolloutSimulatorAdapter:
    def __init__(self, planner_config, rl_config):
        self.pc, self.rc = planner_config, rl_config
        self.path = _abs(planner_config.vidur_path)
        self.timeout = float(planner_config.simulator_timeout_s)

    def _default_command(self, trace: Path, outdir: Path, rc: RolloutClusterConfig) -> str:
        tp = max(1, max(rc.tp_list or [1]))
        max_tokens = max(2, int(self.rc.max_seq_length or self.rc.max_new_tokens))
        parts = [shlex.quote(self.pc.vidur_python), "-m", "vidur.main",
                 "--replica_config_device", shlex.quote(self.pc.vidur_device),
                 "--replica_config_model_name", shlex.quote(self.pc.vidur_model_name),
                 "--cluster_config_num_replicas", str(max(1, rc.n_gpus // tp)),
                 "--replica_config_tensor_parallel_size", str(tp),
                 "--request_generator_config_type", "trace_replay",
                 "--trace_request_generator_config_trace_file", shlex.quote(str(trace)),
                 "--trace_request_generator_config_max_tokens", str(max_tokens),
                 "--replica_scheduler_config_type", shlex.quote(self.pc.vidur_scheduler),
                 f"--{self.pc.vidur_scheduler}_scheduler_config_batch_size_cap", str(self.pc.vidur_batch_size_cap),
                 f"--{self.pc.vidur_scheduler}_scheduler_config_chunk_size", str(self.pc.vidur_chunk_size),
                 "--metrics_config_output_dir", shlex.quote(str(outdir))]
        if self.pc.vidur_time_limit_s > 0:
            parts += ["--time_limit", str(self.pc.vidur_time_limit_s)]
        return " ".join(parts)

    def evaluate_rollout(self, rc: RolloutClusterConfig, requests: List[RequestInfo]) -> SimulatorEstimate:
        if not requests:
            return SimulatorEstimate(0.0, {"backend": "vidur", "reason": "empty_requests"})
        if not self.path.exists():
            raise SimulatorBackendError(f"Vidur path does not exist: {self.path}")
        with tempfile.TemporaryDirectory(prefix="vidur_rollout_", dir=_cache_dir(self.pc)) as td:
            work = Path(td)
            trace, out, outdir = work / "request_trace.csv", work / "output.json", work / "vidur_output"
            outdir.mkdir()
            with trace.open("w", newline="") as fh:
                w = csv.DictWriter(fh, fieldnames=["arrived_at", "num_prefill_tokens", "num_decode_tokens"])
                w.writeheader()
                for r in requests:
                    w.writerow({"arrived_at": 0.0, "num_prefill_tokens": r.prompt_length,
                                "num_decode_tokens": r.gen_length})
            cmd = (self.pc.vidur_rollout_command or "").strip()
            full = cmd.format(trace_csv=shlex.quote(str(trace)), output_json=shlex.quote(str(out)),
                              output_dir=shlex.quote(str(outdir)), vidur_path=shlex.quote(str(self.path)),
                              rl_framework_path=shlex.quote(str(PKG_ROOT)), python=shlex.quote(self.pc.vidur_python),
                              tp_list=shlex.quote(",".join(map(str, rc.tp_list))), num_replicas=max(1, rc.n_instances),
                              tensor_parallel_size=max(1, max(rc.tp_list or [1]))) if cmd else \
                self._default_command(trace, outdir, rc)
            proc = _run(full, self.path, self.timeout, {"PYTHONPATH": str(self.path)})
            if proc.returncode != 0:
                raise SimulatorBackendError(f"Vidur rollout simulator failed (code={proc.returncode}): "
                                            f"{proc.stderr[-1000:]}")
            res = json.loads(out.read_text()) if out.exists() else _marker(proc.stdout, "VIDUR_RESULT_JSON=")
            if res is None:
                res = self._from_metrics(outdir)
            return SimulatorEstimate(_seconds(res, ROLLOUT_KEYS), {"backend": "vidur", "command": full, "raw": res})

    @staticmethod
    def _from_metrics(outdir: Path) -> dict:
        for name, cols in (("request_metrics.csv", ("request_completed_at", "completed_at", "request_e2e_time")),
                           ("batch_metrics.csv", ("batch_completed_at", "completed_at", "time"))):
            for path in outdir.glob(f"**/{name}"):
                with path.open(newline="") as fh:
                    rows = list(csv.DictReader(fh))
                for col in cols:
                    vals = [float(r[col]) for r in rows if r.get(col) not in (None, "")]
                    if vals:
                        return {"makespan": max(vals), "source": str(path), "column": col}
        raise SimulatorBackendError("Vidur produced no output_json, VIDUR_RESULT_JSON, request_metrics.csv or "
                                    "batch_metrics.csv")


class HybridSimulatorCostModel:
    """The evaluator the planner calls; analytic-B200 by default."""

    def __init__(self, config: Any, analytic: Optional[CostModel] = None):
        self.config = config
        self.planner_config = pc = config.global_resource_planner
        self.analytic = analytic or CostModel(
            hardware=config.hardware, model_arch=config.model_arch, profiling=config.profiling,
            max_seq_length=config.max_seq_length, recompute_logprobs=config.recompute_logprobs,
            recompute_micro_batch_size=config.recompute_micro_batch_size,
            recompute_logits_dtype_bytes=pc.memory_budget_logits_dtype_bytes,
            recompute_workspace_factor=pc.memory_budget_workspace_factor,
            memory_safety_margin_bytes=pc.memory_budget_safety_margin_bytes)
        self.train_backend = str(pc.train_backend or "analytic").lower()
        self.rollout_backend = str(pc.rollout_backend or "analytic").lower()
        self.sailor = SailorTrainingSimulatorAdapter(pc, config) if self.train_backend in ("sailor", "hybrid") else None
        self.vidur = VidurRolloutSimulatorAdapter(pc, config) if self.rollout_backend in ("vidur", "hybrid") else None
        self.fallback_events: List[dict] = []

    def _fallback(self, side: str, exc: Exception) -> None:
        if not self.planner_config.simulator_allow_fallback:
            raise exc
        self.fallback_events.append({"side": side, "error": str(exc)[-500:]})

    def evaluate_training(self, tc: TrainParallelConfig, B_global: int, L: int) -> Tuple[float, dict]:
        if self.sailor is not None:
            try:
                est = self.sailor.evaluate_training(tc, B_global, L)
                return (float("inf") if est.is_oom else est.seconds), est.details
            except (SimulatorBackendError, subprocess.TimeoutExpired, OSError, ValueError) as exc:
                self._fallback("train", exc)
        t, d = self.analytic.evaluate_training(tc, B_global, L)
        return t, dict(d, backend="analytic")

    def evaluate_rollout(self, rc: RolloutClusterConfig, requests: List[RequestInfo]) -> Tuple[float, dict]:
        if self.vidur is not None:
            try:
                est = self.vidur.evaluate_rollout(rc, requests)
                return est.seconds, est.details
            except (SimulatorBackendError, subprocess.TimeoutExpired, OSError, ValueError) as exc:
                self._fallback("rollout", exc)
        t, d = self.analytic.evaluate_rollout(rc, requests)
        return t, dict(d, backend="analytic")

    def check_train_oom(self, tc: TrainParallelConfig, B_global: int, L: int) -> bool:
        return self.analytic.check_train_oom(tc, B_global, L)
