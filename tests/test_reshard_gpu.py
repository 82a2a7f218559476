"""weight_reshard kernel on one GPU: the planned copies (sources as separate
buffers standing in for the trainer's TP ranks) equal slicing the full tensors."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(cfg, src_tp, dtype=torch.bfloat16, seed=0):
    from libra_b200.models.qwen3 import ParamLayout, param_shapes
    from libra_b200.parallel.tensor_parallel import shard_full_params

    g = torch.Generator(device="cuda").manual_seed(seed)
    lay1 = ParamLayout(param_shapes(cfg, 1, 0))
    full = {n: torch.randn(lay1.shapes[n], generator=g, device="cuda").to(dtype) for n in lay1.order}

    def flat(tp, rank, dt):
        lay = ParamLayout(param_shapes(cfg, tp, rank))
        f = torch.zeros(lay.numel, dtype=dt, device="cuda")
        views = lay.views(f)
        for n, v in shard_full_params(full, cfg, tp, rank).items():
            views[n].copy_(v)
        return f

    return full, flat


@pytest.mark.parametrize("src_tp,dst_tp", [(2, 1), (1, 4), (4, 2), (2, 2)])
def test_reshard_kernel_matches_slices(src_tp, dst_tp):
    from libra_b200 import ops
    from libra_b200.infra.sync.reshard import DeviceReshard
    from libra_b200.models.qwen3 import get_config

    cfg = get_config("tiny-gpu")
    _, flat = _setup(cfg, src_tp)
    srcs = [flat(src_tp, r, torch.bfloat16) for r in range(src_tp)]
    for dst_rank in range(dst_tp):
        want = flat(dst_tp, dst_rank, torch.bfloat16)
        got = torch.full_like(want, float("nan"))
        plan = DeviceReshard(cfg, src_tp, dst_tp, dst_rank, [s.data_ptr() for s in srcs], got)
        moved = plan.run()
        torch.cuda.synchronize()
        ops.check_kernel_errors()
        # padding between parameters is not part of any slice
        from libra_b200.models.qwen3 import ParamLayout, param_shapes
        lay = ParamLayout(param_shapes(cfg, dst_tp, dst_rank))
        for n in lay.order:
            a, b = lay.segment(n)
            assert torch.equal(got[a:b], want[a:b]), n
        assert moved == 2 * sum(lay.segment(n)[1] - lay.segment(n)[0] for n in lay.order)


def test_reshard_kernel_casts_fp32_sources():
    from libra_b200.infra.sync.reshard import DeviceReshard
    from libra_b200.models.qwen3 import get_config

    cfg = get_config("tiny-gpu")
    _, flat = _setup(cfg, 1, dtype=torch.float32, seed=4)
    src = flat(1, 0, torch.float32)
    want = flat(2, 1, torch.float32).bfloat16()
    got = torch.zeros_like(want)
    DeviceReshard(cfg, 1, 2, 1, [src.data_ptr()], got, src_elem_bytes=[4]).run()
    torch.cuda.synchronize()
    assert torch.equal(got, want)
