"""Bounded device-side waits end with an error status instead of hanging.

The fused collectives wait on flags that other ranks release through NVLink.
Here one GPU plays rank 0 of a two-rank group whose buffers and signal pads all
live in its own memory, and the "peer" never releases its flag.  Each wait is
given a 1 ms limit: the kernel records kErrPeerWait (code 5) in the status word,
skips its remaining work and returns, the host turns the word into an exception,
and the CUDA context stays usable for the next kernel.  No GPU is faulted or hung:
the waits are bounded and nothing is left in flight.
"""

import pytest
import torch

from online_speculation_b200.ops import _ext, workspace
from online_speculation_b200.ops import kernels as K

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000   # 1 ms


def _context_still_usable(dev):
    x = torch.randn(4, 256, device=dev).bfloat16()
    w = torch.ones(256, device=dev).bfloat16()
    out = K.rmsnorm(x, w, 1e-6)
    ref = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.cuda.synchronize()
    assert float((out.float() - ref).abs().max()) < 5e-2
    workspace.check_status(dev)   # the error was consumed: nothing new is reported


@pytest.mark.parametrize("algorithm", [1, 2], ids=["oneshot", "twoshot"])
def test_allreduce_peer_wait_times_out(algorithm):
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    workspace.check_status(dev)
    T, H, world = 8, 512, 2
    parts = [torch.randn(T, H, device=dev).bfloat16() for _ in range(world)]
    rows = [torch.zeros(T, H, device=dev, dtype=torch.bfloat16) for _ in range(world)]
    pads = [torch.zeros(64, device=dev, dtype=torch.int32) for _ in range(world)]   # slots x 8 rank words
    epoch = torch.zeros(4, device=dev, dtype=torch.int32)
    h = torch.randn(T, H, device=dev).bfloat16()
    h0 = h.clone()
    w = torch.ones(H, device=dev).bfloat16()
    x = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    _ext.require().allreduce_add_rmsnorm([p.data_ptr() for p in parts], [r.data_ptr() for r in rows],
                                         [p.data_ptr() for p in pads], epoch, h, w, x, T, 0, 1e-6, 4,
                                         workspace.status(dev), algorithm, LIMIT_NS)
    stop.record()
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device kernel error 5"):
        workspace.check_status(dev)
    # the wait gave up after about the limit, not the two-second default
    assert start.elapsed_time(stop) < 200.0
    # rank 0 published its own flag; the peer's word stayed zero
    assert int(pads[0][2 * 8 + 0]) == 1 and int(pads[0][2 * 8 + 1]) == 0
    if algorithm == 1:
        assert torch.equal(h, h0)   # the one-shot kernel skipped the reduction
    _context_still_usable(dev)


def test_expert_parallel_count_exchange_times_out():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    workspace.check_status(dev)
    world, E, k, T, H = 2, 8, 2, 4, 256
    r_max = T * k * world
    i32 = dict(dtype=torch.int32, device=dev)
    tables = [torch.zeros(world * E, **i32) for _ in range(world)]
    recv_x = [torch.zeros(r_max, H, device=dev, dtype=torch.bfloat16) for _ in range(world)]
    recv_y = [torch.zeros(r_max, H, device=dev, dtype=torch.bfloat16) for _ in range(world)]
    pads = [torch.zeros(64, **i32) for _ in range(world)]
    epoch = torch.zeros(2, **i32)
    topk_idx = torch.tensor([0, 5, 1, 6, 2, 7, 3, 4], **i32)
    counts = torch.bincount(topk_idx.long(), minlength=E).int()
    topk_w = torch.full((T * k,), 0.5, device=dev)
    x = torch.randn(T, H, device=dev).bfloat16()
    h = torch.zeros(T, H, device=dev, dtype=torch.bfloat16)
    cursor = torch.zeros(E, **i32)
    slot_of = torch.full((T * k,), -1, **i32)
    local_offsets = torch.zeros(E // world + 1, **i32)
    _ext.require().ep_exchange([t.data_ptr() for t in tables], [t.data_ptr() for t in recv_x],
                               [t.data_ptr() for t in recv_y], [p.data_ptr() for p in pads], epoch, r_max, counts,
                               topk_idx, topk_w, x, cursor, slot_of, local_offsets, h, E, k, 0, 2, 0,
                               workspace.status(dev), LIMIT_NS)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="device kernel error 5"):
        workspace.check_status(dev)
    assert bool((slot_of == -1).all())          # no row was dispatched
    assert bool((cursor == 0).all())            # the scratch cursors are left at rest
    assert int(pads[0][0]) == 1 and int(pads[0][1]) == 0
    _context_still_usable(dev)
