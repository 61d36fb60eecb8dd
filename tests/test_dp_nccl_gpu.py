"""The multi-rank train step over NCCL on two GPUs: the gradient buckets are
all-reduced from the backward's hooks while it runs, and those calls are
captured in graph A. Checked against eager DistributedDataParallel on the
same batches: a poisoned batch on one rank makes both ranks skip (eagerly and
from a replayed graph), the ranks stay bitwise identical, and the two forms
train alike. Skipped with fewer than two GPUs."""
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


def _run(T, cfg, rank, graphed, batches):
    step = T.TrainStep(cfg, "cuda", cuda_graph=graphed, bucket_mb=1)
    assert step.world == 2 and step.lagged and step.graphed == graphed
    params = lambda: torch.cat([p.detach().reshape(-1) for p in step.model.parameters()])
    poisoned = batches[rank][0].clone()
    poisoned[0, 0, 0] = float("nan")
    before = params()
    step.step(poisoned if rank == 1 else batches[rank][0], batches[rank][1])
    assert step.skipped == 1 and torch.equal(before, params())
    for _ in range(3):
        step.step(*batches[rank])
    assert step.skipped == 1 and step.sched.last_epoch == 3
    after3 = params()
    if graphed:
        assert step._gA is not None and step._reduced_in_backward
        assert len(step._buckets) > 2                  # 1 MB buckets: several per backward
        before = params()
        step.step(poisoned if rank == 1 else batches[rank][0], batches[rank][1])
        assert step.skipped == 2 and torch.equal(before, params())
        step.step(*batches[rank])
        assert step.skipped == 2 and step.sched.last_epoch == 4
    flat = params()
    assert torch.isfinite(flat).all()
    other = flat.clone()
    dist.broadcast(other, src=0)
    assert torch.equal(flat, other)
    assert not torch.equal(flat, before)
    step.close()
    del step
    torch.cuda.empty_cache()
    return after3


def _worker(rank, world, port, tests_dir):
    import sys
    from datetime import timedelta
    sys.path.insert(0, tests_dir)
    sys.path.insert(0, os.path.dirname(tests_dir))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from tau_dxb_b200 import train as T
        cfg = T.StepConfig(batch=2, frames=400, label_len=40, min_label=10, encoder_layers=2,
                           decoder_layers=2, d_model=128, heads=2, ffn=512, vocab=700, warmup_steps=1)
        batches = [T.synthetic_batch(cfg, "cuda", torch.Generator().manual_seed(300 + r)) for r in range(world)]
        graphed = _run(T, cfg, rank, True, batches)
        eager = _run(T, cfg, rank, False, batches)
        # NCCL's average of the buckets and DDP's bucketed sum train alike, up
        # to summation order (the attention backward's atomics, NCCL's reduction)
        assert torch.allclose(graphed, eager, rtol=1e-4, atol=1e-6), float((graphed - eager).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_nccl_buckets_in_graph():
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    mp.spawn(_worker, args=(2, _free_port(), tests_dir), nprocs=2, join=True)
