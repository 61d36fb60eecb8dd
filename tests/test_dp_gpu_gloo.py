"""The multi-rank train step on the GPU kernels: two ranks share cuda:0 and
reduce over gloo (host-side, so no kernel waits on another process). Both
forms of the step run: the graphed one (flat gradient buffer all-reduced
between two CUDA graphs, the flag carried in the buffer) and the eager DDP
one (flag MAX-reduced). A poisoned batch on one rank must make every rank
skip, leave the weights as they were, and clean steps afterwards must keep
the ranks identical."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(T, cfg, rank, world, graphed, batches):
    step = T.TrainStep(cfg, "cuda", cuda_graph=graphed)
    assert step.world == 2 and step.lagged and step.graphed == graphed
    params = lambda: torch.cat([p.detach().reshape(-1) for p in step.model.parameters()])
    poisoned = batches[rank][0].clone()
    poisoned[0, 0, 0] = float("nan")
    before = params()
    # a poisoned batch on rank 1 only: every rank skips (flag reduced over ranks)
    step.step(poisoned if rank == 1 else batches[rank][0], batches[rank][1])
    assert step.skipped == 1
    assert torch.equal(before, params())
    assert step.sched.last_epoch == 0
    # clean steps: eager warm-up, then (graphed) capture and replays. The
    # schedule's first step runs at LR factor 0 (as the reference's warmup
    # does), the next ones at the full rate.
    for _ in range(3):
        step.step(*batches[rank])
    assert step.skipped == 1 and step.sched.last_epoch == 3
    after3 = params()
    if graphed:
        assert step._gA is not None
        # the same skip from a replayed graph
        before = params()
        step.step(poisoned if rank == 1 else batches[rank][0], batches[rank][1])
        assert step.skipped == 2 and torch.equal(before, params())
        step.step(*batches[rank])
        assert step.skipped == 2 and step.sched.last_epoch == 4
    flat = params()
    assert torch.isfinite(flat).all()
    other = flat.clone()
    dist.broadcast(other, src=0)
    assert torch.equal(flat, other)               # the ranks stay identical
    assert not torch.equal(flat, before)
    step.reset_graph()
    del step
    torch.cuda.empty_cache()
    return after3


def _worker(rank, world, port, tests_dir):
    import sys
    sys.path.insert(0, tests_dir)
    sys.path.insert(0, os.path.dirname(tests_dir))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(0)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        from tau_dxb_b200 import train as T
        cfg = T.StepConfig(batch=2, frames=400, label_len=40, min_label=10, encoder_layers=2,
                           decoder_layers=2, d_model=128, heads=2, ffn=512, vocab=700, warmup_steps=1)
        batches = [T.synthetic_batch(cfg, "cuda", torch.Generator().manual_seed(300 + r)) for r in range(world)]
        graphed = _run(T, cfg, rank, world, True, batches)
        eager = _run(T, cfg, rank, world, False, batches)
        # the graphed flat-buffer all-reduce and DDP's bucketed one train alike
        # (after the same skipped step and three updates), up to the summation
        # order of the attention backward's atomics
        assert torch.allclose(graphed, eager, rtol=1e-4, atol=1e-6), float((graphed - eager).abs().max())
    finally:
        dist.destroy_process_group()


def test_two_ranks_skip_together_on_gpu():
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    mp.spawn(_worker, args=(2, _free_port(), tests_dir), nprocs=2, join=True)
