"""The gradient buckets of the data-parallel step, on the host (no GPU, no
process group): the NCCL call is replaced by a recorder, and the step's own
forward/backward (_dp_local) runs on a small Whisper. Checked: the first
backward only records the order in which gradients finish and then averages
everything after it; later backwards issue every bucket from inside the
backward as soon as its last gradient is in, in the recorded order; each
parameter with a gradient is in exactly one bucket; the non-finite flag rides
with the first bucket; buckets have about the requested size. The tau-opus /
WTA operators run on the oracle here (tests/oracle_ops.py), as in the other
host-side model tests."""
import pytest
import torch

from oracle_ops import use_oracle_ops
from tau_dxb_b200 import train as T


_BUILT = []


@pytest.fixture(autouse=True)
def _oracle_ops(monkeypatch):
    use_oracle_ops(monkeypatch)
    yield
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import patch_whisper_stau as ST
    while _BUILT:
        step = _BUILT.pop()
        step.close()
        ST.remove_stau(step.model)
        SG.remove_sparse_grad(step.model)


class _Work:
    def wait(self):
        pass


def _step_with_recorder(bucket_mb=1):
    cfg = T.StepConfig(batch=2, frames=200, label_len=16, min_label=6, encoder_layers=2, decoder_layers=2,
                       d_model=128, heads=2, ffn=512, vocab=300)
    step = T.TrainStep(cfg, "cpu", cuda_graph=False)
    _BUILT.append(step)
    step._init_buckets(bucket_mb)
    calls = []

    def record(tensors):
        calls.append((list(tensors), step._bucket_open))
        return _Work()
    step._allreduce_avg = record
    batch = T.synthetic_batch(cfg, "cpu", torch.Generator().manual_seed(4))
    return step, calls, batch


def test_first_backward_records_then_reduces_after():
    step, calls, batch = _step_with_recorder()
    loss = step._dp_local(*batch)
    assert torch.isfinite(loss)
    assert step._buckets and len(step._buckets) > 2
    # every call happened after the backward (the order was still being recorded)
    assert calls and all(not inside for _, inside in calls)
    assert any(t is step._flag for t in calls[0][0])
    assert step._reduced_in_backward


def test_later_backwards_issue_buckets_inside_the_backward():
    step, calls, batch = _step_with_recorder(bucket_mb=1)
    step._dp_local(*batch)
    calls.clear()
    step._dp_local(*batch)
    n_b = len(step._buckets)
    assert len(calls) == n_b
    assert all(inside for _, inside in calls)          # issued by the hooks, during the backward
    # the first issued bucket carries the flag, and only it
    assert any(t is step._flag for t in calls[0][0])
    assert not any(t is step._flag for c, _ in calls[1:] for t in c)
    # each gradient exactly once, in the order of the buckets
    grads = [t for c, _ in calls for t in c if t is not step._flag]
    params = [p for p in step.model.parameters() if p.grad is not None]
    assert len(grads) == len(params)
    assert {id(t) for t in grads} == {id(p.grad) for p in params}
    order = [p.grad for bk in step._buckets for p in bk["params"] if p.grad is not None]
    assert [id(t) for t in grads] == [id(t) for t in order]
    # about 1 MB per bucket (the last one may be smaller; a large tensor may make one larger)
    sizes = [sum(p.numel() * 4 for p in bk["params"]) for bk in step._buckets]
    assert all(s >= (1 << 20) for s in sizes[:-1])


def test_flag_carries_non_finite_loss():
    step, calls, batch = _step_with_recorder()
    step._dp_local(*batch)
    mel, labels = batch
    bad = mel.clone()
    bad[0, 0, 0] = float("nan")
    calls.clear()
    step._dp_local(bad, labels)
    assert float(step._flag[0]) == 1.0
    assert any(t is step._flag for t in calls[0][0])
    step.close()
    assert step._hook_handles == []
