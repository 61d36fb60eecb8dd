"""Data-parallel train step on 2 CPU ranks (gloo): DDP-averaged gradients equal
the average of per-batch gradients, parameters stay identical across ranks,
and a non-finite loss on one rank makes every rank skip the step."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _route_to_oracle():
    import oracle_ops as O
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import patch_whisper_stau as ST
    ST.STauOpusAttentionFunction = O.OracleAttention
    ST.STauOpusCausalFunction = O.OracleCausalAttention
    SG.SparseGradWTA_Function = O.OracleSparseGrad
    SG._WTAFusedCounting = O.OracleWTA


def _worker(rank, world, port, tests_dir, mode):
    import sys
    sys.path.insert(0, tests_dir)
    sys.path.insert(0, os.path.dirname(tests_dir))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.set_num_threads(2)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=120))
    try:
        _route_to_oracle()
        from tau_dxb_b200 import train as T
        cfg = T.StepConfig(batch=1, frames=200, label_len=16, min_label=6, encoder_layers=1,
                           decoder_layers=1, d_model=128, heads=2, ffn=256, vocab=300)
        step = T.TrainStep(cfg, "cpu")
        batches = [T.synthetic_batch(cfg, "cpu", torch.Generator().manual_seed(100 + r))
                   for r in range(world)]
        if mode == "grads":
            loss, _ = step.loss(*batches[rank])
            loss.backward()
            ddp = {n: p.grad.clone() for n, p in step.model.named_parameters() if p.grad is not None}
            # single-process reference on the same weights: mean of per-batch grads
            ref = {}
            for b in batches:
                step.model.zero_grad(set_to_none=True)
                l, _ = T.TrainStep.loss(type("S", (), {"net": T.PaddedHeadLoss(step.model),
                                                       "device": step.device, "cfg": cfg})(), *b)
                l.backward()
                for n, p in step.model.named_parameters():
                    if p.grad is not None:
                        ref[n] = ref.get(n, 0) + p.grad / world
            assert set(ddp) == set(ref)
            for n in ddp:
                assert torch.allclose(ddp[n], ref[n], rtol=1e-4, atol=1e-6), n
            for key in ("log_tau", "log_alpha", "logit_k"):
                assert any(key in n for n in ddp), key
        else:  # "nan": rank 1 feeds a poisoned batch; everyone must skip
            before = [p.detach().clone() for p in step.model.parameters()]
            mel, labels = batches[rank]
            if rank == 1:
                mel = mel.clone()
                mel[0, 0, 0] = float("nan")
            step.step(mel, labels)
            assert step.skipped == 1
            for a, p in zip(before, step.model.parameters()):
                assert torch.equal(a, p.detach())
            # a clean step afterwards moves every rank identically
            step.step(*batches[rank])
            flat = torch.cat([p.detach().reshape(-1) for p in step.model.parameters()])
            other = flat.clone()
            dist.broadcast(other, src=0)
            assert torch.equal(flat, other)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["grads", "nan"])
def test_two_rank_gloo(mode):
    tests_dir = os.path.dirname(os.path.abspath(__file__))
    mp.spawn(_worker, args=(2, _free_port(), tests_dir, mode), nprocs=2, join=True)
