"""A bounded device wait runs out and the host sees it, without hanging the GPU.

The fused all-reduce waits for a flag from every peer.  Here one GPU plays rank 0 of a
two-rank group whose "peer" region is a second local allocation that no kernel ever
signals from, so the wait for peer 1 can only end by its limit (1 ms here).  The kernel
must return, record kWaitTimeout (1002) in the status word, and leave the context usable;
the host check must raise."""

import pytest
import torch

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 1002  # kWaitTimeout, csrc/common.cuh


@pytest.mark.parametrize("ll", [0, 1])
def test_allreduce_wait_runs_out_and_host_raises(ll):
    """ll=0: the wait for the peer's release flag runs out; ll=1: the polls of the peer's LL
    units (data with the epoch inside) run out."""
    from vllm_neuron_b200.ops import check_device_status, device_status
    from vllm_neuron_b200.ops._ext import load

    assert load()
    ops = torch.ops.b200
    dev = torch.device("cuda", torch.cuda.current_device())
    T, H, world, blocks = 4, 256, 2, 4
    slot_bytes = world * T * H * (4 if ll else 2)
    mine = ops.comm_alloc(slot_bytes)
    silent_peer = ops.comm_alloc(slot_bytes)  # nobody ever raises this rank's flags
    try:
        status = device_status(dev)
        status.zero_()
        x = torch.randn(T, H, device=dev).bfloat16()
        out = torch.empty_like(x)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        ops.allreduce_fused([mine, silent_peer], 0, slot_bytes, x, out, None, None, None, 0.0, blocks, status,
                            1_000_000, None, 0, 0, ll)
        end.record()
        torch.cuda.synchronize()
        assert int(status[0].item()) == WAIT_TIMEOUT
        assert start.elapsed_time(end) < 500.0, "the 1 ms limit was not honoured"
        with pytest.raises(RuntimeError, match="timed out"):
            check_device_status(dev)
        assert int(status[0].item()) == 0  # the check clears the word
        # the context is still usable
        y = (x.float() * 2).sum()
        torch.cuda.synchronize()
        assert torch.isfinite(y)
    finally:
        torch.cuda.synchronize()
        ops.comm_free(mine)
        ops.comm_free(silent_peer)
