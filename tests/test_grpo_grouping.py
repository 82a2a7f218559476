"""GRPO grouping in the trainer's host logic (reference tests/test_grpo_grouping.py):
contiguous groups from the data generator, per-group advantage normalisation,
and batches made of complete groups only."""

import itertools
from types import SimpleNamespace

import torch

from libra_b200.trainer.async_rl_trainer import AsyncRLTrainer, compute_group_advantages


class _Engine:
    def get_data_parallel_world_size(self):
        return 1

    def get_data_parallel_rank(self):
        return 0

    def get_version(self):
        return 3


def _trainer(n_samples=4):
    tr = object.__new__(AsyncRLTrainer)
    grp = SimpleNamespace(runtime_batch_collection_timeout_s=0, runtime_batch_collection_max_retries=0)
    tr.config = SimpleNamespace(n_samples=n_samples, seed=0, global_resource_planner=grp)
    tr.train_engine = _Engine()
    tr._single_batch_source = True
    tr._task_counter = itertools.count()
    tr._pending_groups = {}
    return tr


def test_data_generator_repeats_each_prompt_as_a_contiguous_group():
    tasks = list(itertools.islice(_trainer(4)._data_generator([{"x": 1}, {"x": 2}]), 8))
    assert len({t.group_id for t in tasks[:4]}) == 1 and len({t.group_id for t in tasks[4:]}) == 1
    assert tasks[0].group_id != tasks[4].group_id
    assert [t.rollout_index for t in tasks[:4]] == [0, 1, 2, 3]
    assert len({t.data["x"] for t in tasks[:4]}) == 1 and {t.data["x"] for t in tasks} == {1, 2}
    assert all(t.version == 3 for t in tasks)


def test_advantages_are_normalised_within_groups():
    ts = [{"grpo_group_id": "easy", "rewards": torch.tensor([0.8])},
          {"grpo_group_id": "easy", "rewards": torch.tensor([1.0])},
          {"grpo_group_id": "hard", "rewards": torch.tensor([0.0])},
          {"grpo_group_id": "hard", "rewards": torch.tensor([0.2])},
          {"grpo_group_id": "same", "rewards": torch.tensor([0.5])},
          {"grpo_group_id": "same", "rewards": torch.tensor([0.5])}]
    stats = compute_group_advantages(ts)
    easy = torch.cat([ts[0]["advantages"], ts[1]["advantages"]])
    hard = torch.cat([ts[2]["advantages"], ts[3]["advantages"]])
    assert torch.allclose(easy, hard, atol=1e-5) and abs(float(easy.mean())) < 1e-6
    assert float(ts[4]["advantages"]) == 0.0 == float(ts[5]["advantages"])
    assert stats["grpo_mean_group_size"] == 2.0 and stats["grpo_zero_variance_groups"] == 1


def test_batch_keeps_only_complete_groups_after_a_rejection_gap():
    """Group a lost a member to a rejection: it never completes, b completes
    across two dispatches, and every collected trajectory counts as consumed."""
    tr = _trainer(4)

    class Dispatcher:
        chunks = [[{"grpo_group_id": "a"}] * 3 + [{"grpo_group_id": "b"}],
                  [{"grpo_group_id": "b"}] * 3 + [{"grpo_group_id": "c"}]]

        def active_submit_and_wait(self, data_gen, batch_size, timeout):
            return self.chunks.pop(0)

    class Staleness:
        consumed = 0

        def on_batch_consumed(self, n):
            self.consumed += n

    tr.dispatcher, tr.staleness_manager = Dispatcher(), Staleness()
    batch = tr._collect_complete_grpo_batch(iter(()), batch_size=4)
    assert [t["grpo_group_id"] for t in batch] == ["b"] * 4
    assert tr.staleness_manager.consumed == 8
    assert set(tr._pending_groups) == {"a", "c"}
