"""C-MLFQ KV migration from an in-process engine into a TP-2 server group
(two gloo processes on CPU): the prefix's KV goes through a safetensors file,
each server rank takes its own KV heads, the next turn there reuses the
prefix and decodes what the source engine decodes."""

import json
import os
import urllib.request

import torch

from libra_b200.engine.rollout.llm_engine import LLMEngine
from libra_b200.engine.rollout.sampler import SamplingParams
from libra_b200.engine.tp_bucket import TPServerGroup
from libra_b200.engine.train_engine import B200TrainEngine


def _metrics(url):
    with urllib.request.urlopen(url + "/metrics", timeout=10) as r:
        return json.loads(r.read())


def test_prefix_kv_migrates_into_tp2_server_group(tmp_path):
    from safetensors.torch import save_file

    from libra_b200.engine.checkpointing import hf_config_dict, to_hf

    eng = B200TrainEngine("tiny", device="cpu", seed=13)
    eng.initialize()
    ck = tmp_path / "ck"
    ck.mkdir()
    save_file({k: v.contiguous() for k, v in to_hf({n: p.detach() for n, p in eng.params.items()}, eng.cfg).items()},
              str(ck / "model.safetensors"))
    (ck / "config.json").write_text(json.dumps(hf_config_dict(eng.cfg)))
    src = LLMEngine(eng.cfg, {k: v.detach() for k, v in eng.params.items()}, kv_blocks=128, block_size=16)
    greedy = SamplingParams(max_tokens=6, temperature=0.0)
    prompt = list(range(200, 260))
    first = src.generate_sync([prompt], greedy)[0]
    ctx = prompt + first.output_tokens
    turn2 = ctx + [5, 6, 7]
    want = src.generate_sync([turn2], greedy)[0].output_tokens
    group = TPServerGroup("tiny", 2, [], device="cpu", checkpoint=str(ck), startup_timeout=240,
                          log_path=str(tmp_path / "group.log"))
    try:
        client = group.client()
        path = str(tmp_path / "kv.safetensors")
        payload = src.export_prefix(ctx, path)
        assert payload["tokens"] == ctx[:(len(ctx) // 16) * 16] and os.path.exists(path)
        # a payload from another weight version is refused (imports nothing)
        assert client.import_prefix(dict(payload, version=payload["version"] + 1)) == 0
        n = client.import_prefix(payload)
        assert n == len(payload["tokens"])
        before = _metrics(group.base_url)
        out = group.post("/v1/completions", {"prompt": turn2, "max_tokens": 6, "temperature": 0.0})
        after = _metrics(group.base_url)
        assert after["cached_prefix_tokens"] - before["cached_prefix_tokens"] >= n
        assert after.get("migrated_in_tokens", 0) == n
        assert out["choices"][0]["token_ids"] == want
    finally:
        group.close()
