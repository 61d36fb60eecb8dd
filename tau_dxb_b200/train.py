"""Whisper-small tau-opus + WTA fine-tune step, data-parallel over NCCL.

One optimiser step of echo/train_echo_opus1.py:405-434 on B200:
  bf16 autocast forward with fp32 master weights, loss = CE + lambda * mean
  sigmoid(logit_k), backward through the fused tau-opus attention (36 sites)
  and WTA / sparse_grad (24 FFNs), gradient all-reduce (NCCL, bucketed and
  overlapped with the backward by DistributedDataParallel), clip_grad_norm 1.0,
  AdamW with the reference's two parameter groups (base lr / tau lr for
  log_tau and log_alpha, weight decay 0.01), the LR schedule (linear warmup,
  then cosine with warm restarts, echo/train_echo_opus1.py:230-244) and the
  weight EMA (decay 0.999, echo/train_echo_opus1.py:199-213) as one
  multi-tensor lerp. grad_accum micro-batches per optimiser step (the
  reference's GRAD_ACCUM; 1 here by default).

Data parallelism shards by batch: every rank holds a replica and its own
16-sample batch; the all-reduce averages every gradient, log_tau, log_alpha
and logit_k included. A non-finite loss skips the step on every rank (the
flag is all-reduced with the loss), as the reference skips NaN batches
(echo/train_echo_opus1.py:422-425).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from . import layernorm as LN
from . import linear as LIN
from . import patch_whisper_sparse_grad as SG
from . import patch_whisper_stau as ST

SIGMA_MAP = {"encoder_self": "softplus", "decoder_self": "sigmoid", "decoder_cross": "exp"}


@dataclass
class StepConfig:
    batch: int = 16                 # per rank
    n_mels: int = 80
    frames: int = 3000
    label_len: int = 448
    min_label: int = 64
    lr: float = 5e-6
    tau_lr: float = 3e-4
    weight_decay: float = 0.01
    sparsity_lambda: float = 0.01
    init_k_ratio: float = 0.4
    clip: float = 1.0
    grad_accum: int = 1
    ema_decay: float = 0.999        # 0 disables the EMA
    warmup_steps: int = 100
    t0_steps: int = 400
    t_mult: int = 2
    encoder_layers: int = 12
    decoder_layers: int = 12
    d_model: int = 768
    heads: int = 12
    ffn: int = 3072
    vocab: int = 51865
    seed: int = 0
    extra: dict = field(default_factory=dict)


def whisper_config(cfg: StepConfig):
    from transformers import WhisperConfig
    special = {}
    if cfg.vocab < 51865:   # reduced test vocabularies: keep the special tokens inside it
        special = dict(pad_token_id=cfg.vocab - 1, bos_token_id=cfg.vocab - 2,
                       eos_token_id=cfg.vocab - 1, decoder_start_token_id=cfg.vocab - 3)
    c = WhisperConfig(vocab_size=cfg.vocab, d_model=cfg.d_model, encoder_layers=cfg.encoder_layers,
                      decoder_layers=cfg.decoder_layers, encoder_attention_heads=cfg.heads,
                      decoder_attention_heads=cfg.heads, encoder_ffn_dim=cfg.ffn,
                      decoder_ffn_dim=cfg.ffn, max_source_positions=cfg.frames // 2,
                      max_target_positions=cfg.label_len, num_mel_bins=cfg.n_mels, **special)
    c._attn_implementation = "eager"
    return c


def synthetic_tau_init(cfg: StepConfig, seed: int = 1234):
    """Seeded per-head tau initial values shaped like a tau* estimate: encoder
    self-attention in [1.1, 1.9], decoder self-attention in [1.0, 4.6],
    cross-attention 1.0."""
    g = torch.Generator().manual_seed(seed)
    out = {k: {} for k in ST.SITE_KINDS}
    for layer in range(max(cfg.encoder_layers, cfg.decoder_layers)):
        out["encoder_self"][layer] = (1.1 + 0.8 * torch.rand(cfg.heads, generator=g) ** 2).tolist()
        out["decoder_self"][layer] = (1.0 + 3.6 * torch.rand(cfg.heads, generator=g) ** 3).tolist()
        out["decoder_cross"][layer] = [1.0] * cfg.heads
    return out


def build_model(cfg: StepConfig, device, tau_init=None):
    """Random-init Whisper with both patches applied (fp32 master weights)."""
    from transformers import WhisperForConditionalGeneration
    torch.manual_seed(cfg.seed)
    model = WhisperForConditionalGeneration(whisper_config(cfg)).to(device)
    ST.apply_learnable_stau(model, tau_init=tau_init if tau_init is not None else synthetic_tau_init(cfg),
                            alpha_init=1.0, sigma_name=SIGMA_MAP, assume_causal_decoder=True, fuse_qkv=True)
    SG.apply_sparse_grad_wta(model, target="encoder+decoder", encoder_mode="wta_activation",
                             decoder_mode="sparse_grad", learnable_k=True,
                             init_k_ratio=cfg.init_k_ratio, track_wins=True)
    model._tau_dxb_encoder_hook = contiguous_encoder_stream(model)
    LN.patch_layer_norms(model, bf16_out=single_gemm_norm)
    LIN.patch_linears(model)
    if torch.device(device).type == "cuda":
        SG.fuse_gelu_into_wta(model)        # encoder MLPs: GELU inside the WTA kernels
    model.train()
    return model


def single_gemm_norm(name: str) -> bool:
    """Norms of the patched Whisper whose output feeds one GEMM: each layer's
    self-attention norm (the fused q/k/v projection), cross-attention norm
    (q_proj), final norm (fc1), and the decoder's last norm (the LM head).
    The encoder's last norm feeds every cross-attention k/v projection."""
    return name.endswith(("self_attn_layer_norm", "encoder_attn_layer_norm", "final_layer_norm")) \
        or name.endswith("decoder.layer_norm")


def contiguous_encoder_stream(model):
    """Make the encoder's residual stream row-major once, before its first layer.

    Whisper's encoder forms it as conv2(x).permute(0, 2, 1) + positions, a
    [B, L, d] tensor laid out as [B, d, L]; every residual add keeps that
    layout, so each encoder layer norm copies its input to a contiguous buffer
    in the forward and again in the backward, and the adds and the casts of
    their gradients run as strided kernels. One copy here leaves the values
    unchanged and the rest of the encoder row-major."""
    def pre_hook(module, args):
        if args and isinstance(args[0], torch.Tensor) and not args[0].is_contiguous():
            return (args[0].contiguous(),) + tuple(args[1:])
        return None
    return model.model.encoder.layers[0].register_forward_pre_hook(pre_hook)


def lr_lambda(warmup_steps: int, t0_steps: int, t_mult: int):
    """LR factor of the reference's schedule (echo/train_echo_opus1.py:230-244):
    linear warmup over warmup_steps, then cosine annealing restarted after
    t0_steps, t0_steps * t_mult, ... steps."""
    def fn(step: int) -> float:
        if step < warmup_steps:
            return step / max(1, warmup_steps)
        s, length = step - warmup_steps, t0_steps
        while s >= length > 0:
            s -= length
            length *= t_mult
        if length <= 0:
            return 1.0
        return 0.5 * (1.0 + math.cos(math.pi * s / length))
    return fn


class WeightEMA:
    """Shadow copies of the trainable weights, shadow += (1 - decay) (w - shadow)
    after every optimiser step (echo/train_echo_opus1.py:199-213) -- one
    multi-tensor lerp over all of them instead of a per-parameter loop."""

    def __init__(self, model, decay: float):
        self.decay = decay
        self.names = [n for n, p in model.named_parameters() if p.requires_grad]
        self.params = [p for p in model.parameters() if p.requires_grad]
        self.shadow = [p.detach().clone() for p in self.params]

    @torch.no_grad()
    def update(self):
        torch._foreach_lerp_(self.shadow, [p.detach() for p in self.params], 1.0 - self.decay)

    def state_dict(self):
        return dict(zip(self.names, self.shadow))


def make_optimizer(model, cfg: StepConfig, capturable: bool = False):
    """AdamW with the reference's groups (echo/train_echo_opus1.py:344-355).
    capturable: fused AdamW whose step can be recorded in a CUDA graph, with
    the learning rates as device tensors (the LR schedule fills them)."""
    base, taup = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (taup if ("log_tau" in name or "log_alpha" in name) else base).append(p)
    fused = all(p.is_cuda for p in base + taup)
    if capturable and fused:
        dev = base[0].device
        return torch.optim.AdamW([{"params": base, "lr": torch.tensor(cfg.lr, device=dev)},
                                  {"params": taup, "lr": torch.tensor(cfg.tau_lr, device=dev)}],
                                 weight_decay=cfg.weight_decay, fused=True, capturable=True)
    return torch.optim.AdamW([{"params": base, "lr": cfg.lr}, {"params": taup, "lr": cfg.tau_lr}],
                             weight_decay=cfg.weight_decay, fused=fused)


def synthetic_batch(cfg: StepConfig, device, generator: torch.Generator):
    """log-mel [B, 80, 3000] ~ N(0,1); labels uniform over the vocabulary with
    lengths uniform in [64, 448], padded with -100 to 448."""
    mel = torch.randn(cfg.batch, cfg.n_mels, cfg.frames, generator=generator)
    labels = torch.randint(0, cfg.vocab, (cfg.batch, cfg.label_len), generator=generator)
    lens = torch.randint(cfg.min_label, cfg.label_len + 1, (cfg.batch,), generator=generator)
    labels[torch.arange(cfg.label_len)[None, :] >= lens[:, None]] = -100
    return mel.to(device, non_blocking=True), labels.to(device, non_blocking=True)


class PaddedHeadLoss(torch.nn.Module):
    """Whisper forward + the reference's loss (echo/train_echo_opus1.py:405-420:
    cross-entropy of the LM head over the vocabulary, labels -100 ignored), with
    the tied LM head evaluated over a vocabulary padded to a multiple of 64.

    The 51865-wide logits of the plain head have an odd row pitch, which keeps
    the three head GEMMs (logits, their input and weight gradients; ~0.57 TFLOP
    each at batch 16) off the aligned tensor-core kernels. Here the head weight
    gets zero rows and a bias of -inf on the pad columns: the pad logits drop
    out of the softmax exactly, so the loss and every gradient equal the
    unpadded head's."""

    def __init__(self, model, multiple: int = 64):
        super().__init__()
        self.whisper = model
        v = model.config.vocab_size
        self.vocab = v
        self.pad = (-v) % multiple
        bias = torch.zeros(v + self.pad)
        bias[v:] = float("-inf")
        self.register_buffer("head_bias", bias, persistent=False)
        self._mask_key, self._mask = None, None

    def causal_mask(self, B, L, device):
        """[B, 1, L, L] additive causal mask with the values transformers builds
        for eager attention (0 where key <= query, fp32 min above), made once
        per shape. The decoder takes a ready 4D mask as it is, so no mask is
        built inside the step (nor a host-to-device scalar copy)."""
        key = (B, L, str(device))
        if self._mask_key != key:
            i = torch.arange(L, device=device)
            m = torch.where(i[None, :] <= i[:, None], 0.0, torch.finfo(torch.float32).min)
            self._mask = m.expand(B, 1, L, L)
            self._mask_key = key
        return self._mask

    def forward(self, input_features, labels):
        from transformers.models.whisper.modeling_whisper import shift_tokens_right
        cfg = self.whisper.config
        dec_in = shift_tokens_right(labels, cfg.pad_token_id, cfg.decoder_start_token_id)
        # no KV cache in training (it would copy every decoder layer's keys and values)
        mask = self.causal_mask(dec_in.shape[0], dec_in.shape[1], dec_in.device)
        h = self.whisper.model(input_features, decoder_input_ids=dec_in, decoder_attention_mask=mask,
                               use_cache=False).last_hidden_state
        w = self.whisper.proj_out.weight
        if self.pad:
            w = torch.nn.functional.pad(w, (0, 0, 0, self.pad))
        logits = torch.nn.functional.linear(h, w, self.head_bias.to(w.dtype))
        return LIN.cross_entropy(logits.view(-1, logits.shape[-1]), labels.reshape(-1))


class TrainStep:
    """One fine-tune step on this rank (DDP-wrapped when a process group exists)."""

    def __init__(self, cfg: StepConfig, device, tau_init=None, bucket_mb: int = 64, cuda_graph: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.model = build_model(cfg, self.device, tau_init)
        self.world = dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1
        self.net = PaddedHeadLoss(self.model).to(self.device)
        # one CUDA graph pair for the whole step: no accumulation (LayerDrop
        # draws on the host in every forward, which a graph would freeze)
        layerdrop = getattr(self.model.config, "encoder_layerdrop", 0.0) or getattr(self.model.config,
                                                                                "decoder_layerdrop", 0.0)
        self.graphed = bool(cuda_graph) and self.device.type == "cuda" and cfg.grad_accum == 1 \
            and not layerdrop
        # With more than one rank, the graphed step averages the gradients over
        # NCCL in buckets from inside the backward (captured in graph A); over
        # other backends it all-reduces one flat fp32 gradient buffer between
        # its two graphs (every .grad a view of it). Ungraphed, it is
        # DistributedDataParallel.
        self._flat = None
        self._reduce_avg = False
        self._buckets = None            # in-backward gradient buckets (NCCL), see _init_buckets
        self._reduced_in_backward = False
        if self.world > 1:
            if self.graphed:
                for t in list(self.net.parameters()) + list(self.net.buffers()):
                    dist.broadcast(t.data, src=0)        # the replicas start identical, as DDP makes them
                self._reduce_avg = dist.get_backend() == "nccl"
                if self._reduce_avg:
                    self._init_buckets(bucket_mb)
            else:
                from torch.nn.parallel import DistributedDataParallel as DDP
                self.net = DDP(self.net, device_ids=[self.device.index] if self.device.type == "cuda" else None,
                               bucket_cap_mb=bucket_mb, gradient_as_bucket_view=True,
                               broadcast_buffers=False)
        self.opt = make_optimizer(self.model, cfg, capturable=self.graphed)
        self.sched = torch.optim.lr_scheduler.LambdaLR(
            self.opt, lr_lambda=lr_lambda(cfg.warmup_steps, cfg.t0_steps, cfg.t_mult))
        # float base rates: the schedule then fills the tensor rates of a
        # capturable AdamW without reading a device value back
        self.sched.base_lrs = [cfg.lr, cfg.tau_lr]
        self.ema = WeightEMA(self.model, cfg.ema_decay) if cfg.ema_decay > 0 else None
        self._skipped = 0
        self.micro = 0                  # micro-batches since the last optimiser step
        # Non-finite steps are skipped without a host sync when AdamW is fused
        # (it skips on the device given found_inf) and there is no
        # accumulation: the host reads a step's flag one step later.
        self.lagged = bool(self.opt.defaults.get("fused")) and cfg.grad_accum == 1
        self._pending = None            # (pinned flag, event) of the last step, not yet settled
        if self.lagged:
            self._flag_host = torch.zeros(1, dtype=torch.float32).pin_memory()
        self.graph_warmup = 2           # eager steps (on a side stream) before the capture
        # When a list, every replayed step appends {phase: (start, end)} CUDA
        # events: "fwd_bwd" (graph A), "all_reduce" (world > 1), "update" (graph B)
        self.phase_events = None
        self.reset_graph()

    def reset_graph(self):
        """Drop the captured step; the next calls warm up and capture again.
        Needed after anything the capture froze changes: batch shapes, or the
        sparse-grad patch's settings (k ratios, win collection, prune masks)."""
        self._gA = self._gB = None
        self._eager_calls = 0
        self._static = None

    def close(self):
        """Release the captured graphs (before destroy_process_group when they
        hold NCCL calls) and the gradient hooks."""
        self.reset_graph()
        for h in getattr(self, "_hook_handles", ()):
            h.remove()
        self._hook_handles = []
    @property
    def skipped(self) -> int:
        """Steps skipped for a non-finite loss (settles the last step first)."""
        self.flush()
        return self._skipped

    def flush(self):
        """Settle the last step: when its loss was finite, its LR-schedule step
        and weight EMA; otherwise count it as skipped."""
        if self._pending is None:
            return
        ev = self._pending
        self._pending = None
        ev.synchronize()
        if float(self._flag_host[0]) > 0:
            self._skipped += 1
            return
        self.sched.step()
        if self.ema is not None:
            self.ema.update()

    def loss(self, mel, labels):
        amp = torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.device.type == "cuda")
        with amp:
            ce = self.net(mel, labels)
            sp = SG.get_sparsity_loss().to(ce.device)
            return ce + self.cfg.sparsity_lambda * sp, ce

    def step(self, mel, labels):
        """One micro-batch: forward, backward (+ all-reduce); every grad_accum
        micro-batches clip, AdamW, LR schedule and EMA. Returns the loss.
        A step whose loss is not finite (on any rank) changes nothing: no
        AdamW update, no LR-schedule step, no EMA update."""
        if self.graphed and self.lagged:
            return self._step_graphed(mel, labels)
        if self.lagged:
            return self._step_lagged(mel, labels)
        import contextlib
        accumulate = self.world > 1 and self.micro + 1 < self.cfg.grad_accum
        with self.net.no_sync() if accumulate else contextlib.nullcontext():   # all-reduce on the last
            loss, ce = self.loss(mel, labels)
            (loss / self.cfg.grad_accum).backward()
        bad = (~torch.isfinite(loss.detach())).float().reshape(1)
        if self.world > 1:
            dist.all_reduce(bad)
        if float(bad.item()) > 0:       # every rank skips together
            self.opt.zero_grad(set_to_none=True)
            self.micro = 0
            self._skipped += 1
            return loss.detach()
        self.micro += 1
        if self.micro < self.cfg.grad_accum:
            return loss.detach()
        self.micro = 0
        torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.clip)
        self.opt.step()
        self.sched.step()
        self.opt.zero_grad(set_to_none=True)
        if self.ema is not None:
            self.ema.update()
        return loss.detach()


    def _step_lagged(self, mel, labels):
        """The same step without waiting for the GPU. The non-finite flag goes
        to AdamW as found_inf (the fused kernel leaves weights, moments and step
        counts alone when it is set) and to pinned host memory. The host reads
        it one step later, when this step's work has long finished while the
        next step's is queued. At that point (before the next AdamW update, so
        the weights are still this step's) it runs this step's LR-schedule
        step and EMA update, or counts the skip. Same results as checking at
        once; the GPU queue never drains."""
        loss, _ = self.loss(mel, labels)
        loss.backward()
        bad = (~torch.isfinite(loss.detach())).float().reshape(())    # 0-dim, like AdamW's step counts
        if self.world > 1:
            dist.all_reduce(bad, op=dist.ReduceOp.MAX)     # exactly 1.0 when any rank is bad
        self.flush()                     # the previous step: schedule and EMA, or skip
        torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.clip)
        self.opt.found_inf = bad
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        self._flag_host.copy_(bad, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._pending = ev
        return loss.detach()


    def _fwd_bwd(self, mel, labels):
        """Forward, backward, clip; the non-finite flag as a 0-dim tensor."""
        loss, _ = self.loss(mel, labels)
        loss.backward()
        bad = (~torch.isfinite(loss.detach())).float().reshape(())
        torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.clip)
        return loss.detach(), bad

    def _post(self, bad):
        self._flag_host.copy_(bad, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._pending = ev

    # ---- data parallel over a flat gradient buffer (graphed, world > 1) ----

    def _dp_local(self, mel, labels):
        """Forward and backward. With buckets (NCCL), the gradients stay where
        autograd puts them and are averaged bucket by bucket while the backward
        runs, this rank's non-finite-loss flag riding with the first bucket.
        Otherwise they go into the flat buffer (zeroed first), whose last slot
        carries the flag through the all-reduce after the backward."""
        if self._buckets is not None:
            self.opt.zero_grad(set_to_none=True)
            loss, _ = self.loss(mel, labels)
            self._flag.copy_((~torch.isfinite(loss.detach())).float().reshape(1))
            self._bucket_begin()
            loss.backward()
            self._bucket_end()
            return loss.detach()
        first = self._flat is None
        if first:
            self.opt.zero_grad(set_to_none=True)
        else:
            self._flat.zero_()
        loss, _ = self.loss(mel, labels)
        loss.backward()
        if first:
            self._build_flat()
        self._flat[-1:].copy_((~torch.isfinite(loss.detach())).float().reshape(1))
        return loss.detach()

    def _build_flat(self):
        """After the first backward: one fp32 buffer holding every gradient the
        step produced, each parameter's .grad becoming a view of it (the values
        copied in). Parameters without a gradient keep .grad None, so AdamW
        leaves them alone, as in the eager step."""
        used = [p for p in self.model.parameters() if p.requires_grad and p.grad is not None]
        n = sum(p.numel() for p in used)
        flat = torch.zeros(n + 4, dtype=torch.float32, device=self.device)   # + the flag slot, 16-byte padded
        off = 0
        for p in used:
            view = flat[off:off + p.numel()].view_as(p)
            view.copy_(p.grad)
            p.grad = view
            off += p.numel()
        self._flat = flat

    # ---- gradient buckets averaged inside the backward (NCCL) ----

    def _init_buckets(self, bucket_mb: int):
        """Hooks that see each parameter's gradient finished. The first
        backward records the order in which they finish and is averaged in one
        coalesced call after it; later ones average a bucket (about bucket_mb
        MB of gradients, in that order) as soon as its last gradient is in:
        one coalesced NCCL call per bucket on NCCL's stream, overlapping the
        rest of the backward. The calls run on the autograd thread in the
        same order on every rank, and are captured in graph A."""
        self._bucket_bytes = max(1, int(bucket_mb)) << 20
        self._pg = dist.group.WORLD
        self._ready_order = []
        self._buckets = []
        self._pbucket = {}
        self._works = []
        self._bucket_open = False
        self._flag_pending = False
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)
        self._hook_handles = [p.register_post_accumulate_grad_hook(self._grad_ready)
                              for p in self.model.parameters() if p.requires_grad]

    def _build_buckets(self):
        """Cut the recorded order into buckets of about bucket_bytes."""
        buckets, cur, size = [], [], 0
        seen = set()
        for p in self._ready_order:
            if id(p) in seen:
                continue
            seen.add(id(p))
            self._pbucket[id(p)] = len(buckets)
            cur.append(p)
            size += p.numel() * 4
            if size >= self._bucket_bytes:
                buckets.append({"params": cur, "seen": 0, "issued": False})
                cur, size = [], 0
        if cur:
            buckets.append({"params": cur, "seen": 0, "issued": False})
        self._buckets = buckets

    def _grad_ready(self, p):
        if not self._bucket_open:
            if self._recording:
                self._ready_order.append(p)
            return
        b = self._pbucket.get(id(p))
        if b is None:
            return
        bk = self._buckets[b]
        bk["seen"] += 1
        if bk["seen"] == len(bk["params"]):
            self._issue_bucket(bk)

    def _issue_bucket(self, bk):
        bk["issued"] = True
        tensors = [p.grad for p in bk["params"] if p.grad is not None]
        if self._flag_pending:
            tensors.append(self._flag)
            self._flag_pending = False
        if tensors:
            self._works.append(self._allreduce_avg(tensors))

    def _allreduce_avg(self, tensors):
        opts = dist.AllreduceCoalescedOptions()
        opts.reduceOp = dist.ReduceOp.AVG
        opts.asyncOp = True
        return self._pg.allreduce_coalesced(tensors, opts)

    @property
    def _recording(self):
        return not self._buckets

    def _bucket_begin(self):
        self._flag_pending = True
        if self._recording:
            return                       # the first backward only records the order
        for bk in self._buckets:
            bk["seen"], bk["issued"] = 0, False
        self._bucket_open = True

    def _bucket_end(self):
        """Average what the backward did not (all of it the first time; a
        bucket some of whose parameters got no gradient), in bucket order, then
        make the current stream wait for every reduction."""
        self._bucket_open = False
        if self._recording:
            self._build_buckets()
        for bk in self._buckets:
            if not bk["issued"]:
                self._issue_bucket(bk)
        if self._flag_pending:
            self._issue_bucket({"params": []})
        for w in self._works:
            w.wait()
        self._works = []
        self._reduced_in_backward = True

    def _dp_reduce(self):
        """Average the gradients over the ranks (the flag slot becomes the
        fraction of ranks with a non-finite loss). NCCL averages in the
        collective; other backends sum, and the step scales afterwards. A
        no-op when the buckets already did it inside the backward."""
        if self._reduced_in_backward:
            return
        dist.all_reduce(self._flat, op=dist.ReduceOp.AVG if self._reduce_avg else dist.ReduceOp.SUM)

    def _dp_finish(self):
        """Scale (when the collective summed), the flag of the whole job as a
        0-dim tensor, and clipping; returns the flag."""
        if self._buckets is not None:
            bad = (self._flag[0] > 0).float()
        else:
            if not self._reduce_avg:
                self._flat.mul_(1.0 / self.world)
            bad = (self._flat[-1] > 0).float()
        torch.nn.utils.clip_grad_norm_(self.model.parameters(), self.cfg.clip)
        return bad

    def _step_graphed_dp(self, mel, labels):
        """The graphed step on each of several ranks: graph A = forward and
        backward, with the gradient average inside it (NCCL buckets issued
        from the backward) or, over other backends, one all-reduce of the flat
        gradient buffer issued between the replays; graph B = scaling, flag,
        clipping and the AdamW update. The previous step is settled while A
        runs, before B changes the weights."""
        if self._gA is None and self._eager_calls < self.graph_warmup:
            self._eager_calls += 1
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                loss = self._dp_local(mel, labels)
                self._dp_reduce()
                self.flush()
                bad = self._dp_finish()
                self.opt.found_inf = bad
                self.opt.step()
                self._post(bad)
            torch.cuda.current_stream(self.device).wait_stream(side)
            return loss
        if self._gA is None:
            self.flush()
            torch.cuda.synchronize(self.device)
            self._static = (mel.clone(), labels.clone())
            gA, gB = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            tracker = SG._TRACKER
            steps0 = dict(tracker.total_steps) if tracker is not None else {}
            with torch.cuda.graph(gA):
                self._sloss = self._dp_local(*self._static)
            self._host_deltas = {k: v - steps0.get(k, 0) for k, v in tracker.total_steps.items()} \
                if tracker is not None else {}
            self._replays = 0
            with torch.cuda.graph(gB, pool=gA.pool()):
                self._sbad = self._dp_finish()
                self.opt.found_inf = self._sbad
                self.opt.step()
            self._gA, self._gB = gA, gB
        self._load_static(mel, labels)
        ev = self._phase_begin()
        self._gA.replay()
        self._phase_mark(ev, "fwd_bwd")
        self._dp_reduce()
        self._phase_mark(ev, "all_reduce")
        self.flush()
        self._gB.replay()
        self._phase_mark(ev, "update")
        self._post(self._sbad)
        return self._sloss.clone()

    def _phase_begin(self):
        if self.phase_events is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        rec = {"_last": e}
        self.phase_events.append(rec)
        return rec

    @staticmethod
    def _phase_mark(rec, name):
        if rec is None:
            return
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        rec[name] = (rec["_last"], e)
        rec["_last"] = e

    def _load_static(self, mel, labels):
        smel, slab = self._static
        if mel.shape != smel.shape or labels.shape != slab.shape:
            raise ValueError("TrainStep: batch shapes changed since the CUDA graph was captured "
                             f"({tuple(smel.shape)}, {tuple(slab.shape)}); call reset_graph()")
        smel.copy_(mel, non_blocking=True)
        slab.copy_(labels, non_blocking=True)
        if self._replays and SG._TRACKER is not None:
            for k, d in self._host_deltas.items():
                SG._TRACKER.total_steps[k] += d
        self._replays += 1

    def _step_graphed(self, mel, labels):
        """The lagged step replayed from two CUDA graphs: A = forward, backward,
        clip and flag; B = the AdamW update (found_inf = the flag). The previous
        step is settled between them (host waits while A runs; its EMA reads
        the weights before B changes them). The batch is copied into static
        buffers. The first graph_warmup calls are ordinary steps on a side
        stream; the next one captures both graphs, then replays them."""
        if self.world > 1:
            return self._step_graphed_dp(mel, labels)
        if self._gA is None and self._eager_calls < self.graph_warmup:
            self._eager_calls += 1
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                loss, bad = self._fwd_bwd(mel, labels)
                self.flush()
                self.opt.found_inf = bad
                self.opt.step()
                self.opt.zero_grad(set_to_none=True)
                self._post(bad)
            torch.cuda.current_stream(self.device).wait_stream(side)
            return loss
        if self._gA is None:
            self.flush()
            torch.cuda.synchronize(self.device)
            self._static = (mel.clone(), labels.clone())
            self.opt.zero_grad(set_to_none=True)
            gA, gB = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
            tracker = SG._TRACKER
            steps0 = dict(tracker.total_steps) if tracker is not None else {}
            with torch.cuda.graph(gA):
                self._sloss, self._sbad = self._fwd_bwd(*self._static)
            # Python-side counters the forward advanced while being captured
            # (the win tracker's per-layer step counts): a replay does not run
            # Python, so each later replay adds the same amounts
            self._host_deltas = {k: v - steps0.get(k, 0) for k, v in tracker.total_steps.items()} \
                if tracker is not None else {}
            self._replays = 0
            self.opt.found_inf = self._sbad
            with torch.cuda.graph(gB, pool=gA.pool()):
                self.opt.step()
            self._gA, self._gB = gA, gB
        self._load_static(mel, labels)
        ev = self._phase_begin()
        self._gA.replay()
        self._phase_mark(ev, "fwd_bwd")
        self.flush()
        self._gB.replay()
        self._phase_mark(ev, "update")
        self._post(self._sbad)
        return self._sloss.clone()


def model_flops_per_step(cfg: StepConfig) -> float:
    """Algorithmic FLOPs of one step (6 * weights * tokens for the linears, the
    conv stem, and 3.5x the forward attention-score work)."""
    d, f, T_enc, T_dec, B = cfg.d_model, cfg.ffn, cfg.frames // 2, cfg.label_len, cfg.batch
    enc_lin = cfg.encoder_layers * (4 * d * d + 2 * d * f)
    dec_self = cfg.decoder_layers * (4 * d * d + 2 * d * f)
    dec_cross_qo = cfg.decoder_layers * 2 * d * d
    dec_cross_kv = cfg.decoder_layers * 2 * d * d
    head = cfg.vocab * d
    lin = 6 * B * (enc_lin * T_enc + (dec_self + dec_cross_qo + head) * T_dec + dec_cross_kv * T_enc)
    conv = 6 * B * (cfg.n_mels * d * 3 * cfg.frames + d * d * 3 * T_enc)
    attn = 3.5 * 4 * B * cfg.heads * 64 * (
        cfg.encoder_layers * T_enc * T_enc + cfg.decoder_layers * (0.5 * T_dec * T_dec + T_dec * T_enc))
    return float(lin + conv + attn)
