"""Device-side failure detection: a bounded wait that nobody satisfies runs out,
the kernel returns, the host reads the error code, and the context stays usable.

The fused AdamW + parameter all-gather kernel waits (in CTA 0) for every CTA of
every rank to arrive on its counters.  Launched on one rank with an epoch one
ahead of the counters, its target can never be reached: the wait must give up
after the shortened budget set through the error word, record the peer-flag
timeout code, and leave the GPU in a state where the next launch succeeds.
No fault, trap or endless loop is involved.
"""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_runs_out_and_reports():
    from libra_b200 import ops

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    n = 1 << 16
    torch.manual_seed(0)
    master0 = torch.randn(n, device=dev)
    grad = torch.randn(n, device=dev) * 1e-2
    flat = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    err = ops.error_flag(dev)
    ops.check_kernel_errors(dev)
    hp = (1e-3, 0.9, 0.95, 1e-8, 0.0, 1, None, 0.0, 1.0)
    grid = 8
    ops.set_wait_limit_ms(dev, 20)
    try:
        master, m, v = master0.clone(), torch.zeros_like(master0), torch.zeros_like(master0)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        # epoch 2 on fresh counters: the kernel waits for 2 x grid arrivals and only grid arrive
        ops.ext().adamw_step_allgather(master, grad, m, v, *hp, [flat.data_ptr()], [flags.data_ptr()], 0, 2, err, grid)
        torch.cuda.synchronize()
        waited = time.perf_counter() - t0
        with pytest.raises(ops.KernelError) as info:
            ops.check_kernel_errors(dev)
        assert info.value.code == ops.TIMEOUT_PEER_FLAG
        assert waited < 1.0, f"the 20 ms budget was not applied (kernel took {waited:.3f}s)"
        assert int(err[0]) == 0  # check_kernel_errors cleared the code

        # the context is still usable: a reachable target completes and matches plain AdamW
        flags.zero_()
        master, m, v = master0.clone(), torch.zeros_like(master0), torch.zeros_like(master0)
        ops.ext().adamw_step_allgather(master, grad, m, v, *hp, [flat.data_ptr()], [flags.data_ptr()], 0, 1, err, grid)
        torch.cuda.synchronize()
        ops.check_kernel_errors(dev)
        ref_master, rm, rv = master0.clone(), torch.zeros_like(master0), torch.zeros_like(master0)
        ref_param = torch.zeros(n, dtype=torch.bfloat16, device=dev)
        ops.adamw_step(ref_master, grad, rm, rv, ref_param, lr=hp[0], beta1=hp[1], beta2=hp[2], eps=hp[3],
                       weight_decay=hp[4], step=hp[5])
        assert torch.equal(flat, ref_param)
        assert int(flags[0]) == grid
    finally:
        ops.set_wait_limit_ms(dev, 0)
