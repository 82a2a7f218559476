"""Online calibration of the cost model from measured step times.

Keeps exponential moving averages of the compute efficiency (eta_comp: how
much of the modelled FLOP rate training reaches), memory efficiency (eta_mem:
rollout), the comm/compute overlap gamma and the prompt/generation length
statistics; a 3-sigma jump in the training-time prediction error or in the
mean generation length is treated as a change point and switches to a fast
EMA (reference ``infra/cost_model/calibrator.py``).

Unlike the reference (where it is exported but unused), the trainer wires this
into the planner here: ``apply_to_cost_model`` rescales the B200 training MFU
and decode bandwidth utilisation of the analytic model.
"""

from __future__ import annotations

import logging
import statistics
from collections import deque
from dataclasses import dataclass, field, replace
from typing import Any, Dict, List

log = logging.getLogger(__name__)


@dataclass
class EpochRunData:
    t_train_real: float = 0.0
    t_rollout_real: float = 0.0
    t_train_predicted: float = 0.0
    t_rollout_predicted: float = 0.0
    gen_lengths: List[float] = field(default_factory=list)
    prompt_lengths: List[float] = field(default_factory=list)
    epoch_id: int = 0


@dataclass
class CalibratedParams:
    eta_comp: float = 0.5
    eta_mem: float = 0.5
    gamma_overlap: float = 0.3
    mu_gen: float = 512.0
    sigma_gen: float = 256.0
    mu_prompt: float = 256.0
    confidence: float = 0.0


def _clip(x: float, lo: float, hi: float) -> float:
    return max(lo, min(hi, x))


def _ema(old: float, new: float, a: float) -> float:
    return a * new + (1.0 - a) * old


class ShadowCalibrator:
    def __init__(self, alpha_default: float = 0.1, alpha_emergency: float = 0.8, change_point_threshold: float = 3.0,
                 history_window: int = 20, min_epochs_for_calibration: int = 2):
        self.alpha_default, self.alpha_emergency = alpha_default, alpha_emergency
        self.change_point_threshold = change_point_threshold
        self.history_window = history_window
        self.min_epochs = min_epochs_for_calibration
        self.reset()

    def reset(self) -> None:
        self.params = CalibratedParams()
        self.history: deque = deque(maxlen=self.history_window)
        self._train_err: deque = deque(maxlen=self.history_window)
        self._roll_err: deque = deque(maxlen=self.history_window)
        self._gen_means: deque = deque(maxlen=self.history_window)
        self._is_change_point = False
        self._change_points = 0

    @staticmethod
    def _rel(real: float, pred: float) -> float:
        return (real - pred) / pred

    def _outlier(self, value: float, series) -> bool:
        mu = statistics.fmean(series)
        sd = statistics.pstdev(series) + 1e-8
        return abs(value - mu) > self.change_point_threshold * sd

    def _detect(self, e: EpochRunData) -> None:
        self._is_change_point = False
        if len(self.history) < self.min_epochs:
            return
        if e.t_train_predicted > 0 and len(self._train_err) >= 3 and \
                self._outlier(self._rel(e.t_train_real, e.t_train_predicted), self._train_err):
            self._is_change_point = True
        if e.gen_lengths and len(self._gen_means) >= 3 and self._outlier(statistics.fmean(e.gen_lengths), self._gen_means):
            self._is_change_point = True
        self._change_points += int(self._is_change_point)

    def update(self, e: EpochRunData) -> CalibratedParams:
        self.history.append(e)
        self._detect(e)
        a = self.alpha_emergency if self._is_change_point else self.alpha_default
        p = self.params
        if e.t_train_predicted > 0 and e.t_train_real > 0:
            ratio = e.t_train_predicted / e.t_train_real
            p.eta_comp = _ema(p.eta_comp, _clip(p.eta_comp * ratio, 0.05, 0.95), a)
            step = min(0.05, abs(e.t_train_real / e.t_train_predicted - 1.0))
            target = p.gamma_overlap + step if e.t_train_real > e.t_train_predicted else p.gamma_overlap - step
            p.gamma_overlap = _ema(p.gamma_overlap, _clip(target, 0.0, 1.0), a)
        if e.t_rollout_predicted > 0 and e.t_rollout_real > 0:
            p.eta_mem = _ema(p.eta_mem, _clip(p.eta_mem * e.t_rollout_predicted / e.t_rollout_real, 0.05, 0.95), a)
        if e.gen_lengths:
            mu = statistics.fmean(e.gen_lengths)
            p.mu_gen = _ema(p.mu_gen, mu, a)
            p.sigma_gen = _ema(p.sigma_gen, statistics.pstdev(e.gen_lengths) + 1e-8, a)
            self._gen_means.append(mu)
        if e.prompt_lengths:
            p.mu_prompt = _ema(p.mu_prompt, statistics.fmean(e.prompt_lengths), a)
        p.confidence = min(1.0, len(self.history) / max(2 * self.min_epochs, 1))
        if e.t_train_predicted > 0:
            self._train_err.append(self._rel(e.t_train_real, e.t_train_predicted))
        if e.t_rollout_predicted > 0:
            self._roll_err.append(self._rel(e.t_rollout_real, e.t_rollout_predicted))
        return self.params

    def get_calibrated_params(self) -> CalibratedParams:
        return replace(self.params)

    def get_statistics(self) -> Dict[str, Any]:
        p = self.params
        out = {"n_epochs": len(self.history), "eta_comp": p.eta_comp, "eta_mem": p.eta_mem,
               "gamma_overlap": p.gamma_overlap, "mu_gen": p.mu_gen, "sigma_gen": p.sigma_gen,
               "confidence": p.confidence, "change_point_count": self._change_points,
               "is_change_point": self._is_change_point}
        if self._train_err:
            out["train_error_mean"] = statistics.fmean(self._train_err)
            out["train_error_std"] = statistics.pstdev(self._train_err)
        if self._roll_err:
            out["rollout_error_mean"] = statistics.fmean(self._roll_err)
            out["rollout_error_std"] = statistics.pstdev(self._roll_err)
        return out

    def apply_to_cost_model(self, cost_model, baseline_mfu: float, baseline_bw_util: float) -> None:
        """Scale the analytic model's efficiencies by the calibrated ratios (eta / 0.5)."""
        if self.params.confidence <= 0:
            return
        tm = cost_model.training_model
        rm = cost_model.rollout_model
        tm.train_mfu = _clip(baseline_mfu * self.params.eta_comp / 0.5, 0.05, 1.0)
        rm.decode_bw_util = _clip(baseline_bw_util * self.params.eta_mem / 0.5, 0.05, 1.0)


# ------------------------------------------------------------------ offline fit of the B200 decode profile
def fit_decode_profile(samples: List[Dict[str, float]], n_layers: int, mem_bw: float) -> Dict[str, float]:
    """Fit the rollout model's decode-step terms to measured whole-step times.

    Each sample is one measured decode step of the engine: ``batch`` running
    sequences, ``weight_bytes`` and ``kv_bytes`` read, ``ms`` per step (the
    decode microbenchmark's CUDA-event time).  Model:
    ``ms = n_layers * (layer_overhead + batch * row_layer) + bytes / (mem_bw * util)``,
    solved by least squares for (layer_overhead, row_layer, 1/util).  Returns
    the ``profiling`` keys ``decode_layer_overhead_s``, ``decode_row_layer_s``
    and ``decode_bw_util`` plus the fit's largest relative error."""
    import numpy as np

    if len(samples) < 3:
        raise ValueError("need at least three measured decode steps")
    A = np.array([[n_layers, n_layers * s["batch"], (s["weight_bytes"] + s["kv_bytes"]) / mem_bw] for s in samples])
    y = np.array([s["ms"] / 1e3 for s in samples])
    (a, r, inv_u), *_ = np.linalg.lstsq(A, y, rcond=None)
    a, r = max(float(a), 0.0), max(float(r), 0.0)
    util = 1.0 / float(inv_u) if inv_u > 0 else 1.0
    util = min(max(util, 0.05), 1.0)
    pred = A @ np.array([a, r, 1.0 / util])
    err = float(np.max(np.abs(pred - y) / y))
    return {"decode_layer_overhead_s": a, "decode_row_layer_s": r, "decode_bw_util": util, "max_rel_error": err}


def fit_train_mfu(measured_s: float, predicted_s: float, mfu_used: float) -> float:
    """Training MFU that makes the FLOP-based prediction match a measured step
    (the time is inverse in the MFU)."""
    if measured_s <= 0 or predicted_s <= 0:
        raise ValueError("times must be positive")
    return _clip(mfu_used * predicted_s / measured_s, 0.05, 1.0)
