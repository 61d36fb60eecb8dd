"""The multi-rank train step on the GPU kernels: two ranks share cuda:0 and
reduce over gloo (host-side, so no kernel waits on another process). With
more than one rank the step settles its non-finite flag one step late with a
MAX all-reduce; a poisoned batch on one rank must make every rank skip, leave
the weights as they were, and a clean step afterwards must keep the ranks
identical."""
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
        step = T.TrainStep(cfg, "cuda")
        assert step.world == 2 and step.lagged and not step.graphed
        batches = [T.synthetic_batch(cfg, "cuda", torch.Generator().manual_seed(300 + r)) for r in range(world)]
        before = [p.detach().clone() for p in step.model.parameters()]
        mel, labels = batches[rank]
        if rank == 1:
            mel = mel.clone()
            mel[0, 0, 0] = float("nan")
        step.step(mel, labels)
        assert step.skipped == 1                 # settles the flag (MAX over ranks)
        for a, p in zip(before, step.model.parameters()):
            assert torch.equal(a, p.detach())
        assert step.sched.last_epoch == 0
        # the schedule's first step runs at LR factor 0 (as the reference's
        # warmup does), the next one at the full rate
        for _ in range(2):
            step.step(*batches[rank])
        assert step.skipped == 1 and step.sched.last_epoch == 2
        flat = torch.cat([p.detach().reshape(-1) for p in step.model.parameters()])
        assert torch.isfinite(flat).all()
        other = flat.clone()
        dist.broadcast(other, src=0)
        assert torch.equal(flat, other)
        assert not torch.equal(flat, torch.cat([a.reshape(-1) for a in before]))
    finally:
        dist.destroy_process_group()


def test_two_ranks_skip_together_on_gpu():
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    mp.spawn(_worker, args=(2, _free_port(), tests_dir), nprocs=2, join=True)
