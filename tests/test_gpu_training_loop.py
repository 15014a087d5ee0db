"""The drop-in inside a real training loop on a GPU.

A small causal decoder (written here; the reference's MiniGPT is not on the GPU box) trains with
the reference loop's sequence (``train.py:445-491``): ``set_optimizer_lr`` -> ``zero_grad(
set_to_none=True)`` -> loss-scaled backward -> ``unscale_`` -> ``clip_grad_norm_`` -> ``step`` ->
``update``.  Gradients come from autograd and are reallocated every step.  The bf16 model with
this package's optimizer must track the fp32 model with torch's own AdamW/GradScaler/clip.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


class TinyDecoder(nn.Module):
    def __init__(self, vocab=97, d=64, n_layer=2, n_head=4, block=32):
        super().__init__()
        self.tok = nn.Embedding(vocab, d)
        self.pos = nn.Embedding(block, d)
        self.layers = nn.ModuleList()
        for _ in range(n_layer):
            self.layers.append(nn.ModuleDict({
                "ln1": nn.LayerNorm(d), "qkv": nn.Linear(d, 3 * d), "out": nn.Linear(d, d),
                "ln2": nn.LayerNorm(d), "fc": nn.Linear(d, 4 * d), "proj": nn.Linear(4 * d, d)}))
        self.ln_f = nn.LayerNorm(d)
        self.head = nn.Linear(d, vocab, bias=False)
        self.head.weight = self.tok.weight
        self.n_head = n_head
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, 0.0, 0.02)
                if isinstance(m, nn.Linear) and m.bias is not None:
                    nn.init.zeros_(m.bias)

    def forward(self, x):
        b, t = x.shape
        h = self.tok(x) + self.pos(torch.arange(t, device=x.device))
        for L in self.layers:
            a = L["qkv"](L["ln1"](h)).view(b, t, 3, self.n_head, -1).permute(2, 0, 3, 1, 4)
            y = F.scaled_dot_product_attention(a[0], a[1], a[2], is_causal=True)
            h = h + L["out"](y.transpose(1, 2).reshape(b, t, -1))
            h = h + L["proj"](F.gelu(L["fc"](L["ln2"](h))))
        return self.head(self.ln_f(h))


def _cosine(step, base=3e-3, warm=5, total=40, low=3e-4):
    if step < warm:
        return base * (step + 1) / warm
    p = min(1.0, (step - warm) / max(1, total - warm))
    return low + 0.5 * (1 + math.cos(math.pi * p)) * (base - low)


def _train(fused: bool, steps=40):
    from minigpt_train_infra_b200 import (FusedAdamW, GradScaler, build_adamw_param_groups,
                                          clip_grad_norm_)
    torch.manual_seed(0)
    model = TinyDecoder().to(DEV)
    fp32_init = {n: p.detach().clone() for n, p in model.named_parameters()}
    if fused:
        model = model.to(torch.bfloat16)
        opt = FusedAdamW(build_adamw_param_groups(model, 0.1), lr=3e-3, betas=(0.9, 0.95),
                         eps=1e-8, fused=True)
        for n, p in model.named_parameters():
            opt.set_master_(p, fp32_init[n])
        scaler = GradScaler("cuda", init_scale=2.0 ** 12)
        clip = clip_grad_norm_
    else:
        opt = torch.optim.AdamW(build_adamw_param_groups(model, 0.1), lr=3e-3, betas=(0.9, 0.95),
                                eps=1e-8, fused=True)
        scaler = torch.amp.GradScaler("cuda", init_scale=2.0 ** 12)
        clip = torch.nn.utils.clip_grad_norm_
    gen = torch.Generator(device=DEV).manual_seed(1)
    # a learnable sequence task: next token = (token * 3 + 1) mod vocab
    losses, norms, plans = [], [], 0  # plans: how many times the optimizer built chunk tables
    for step in range(steps):
        for g in opt.param_groups:
            g["lr"] = _cosine(step)
        opt.zero_grad(set_to_none=True)
        x = torch.randint(0, 97, (16, 32), generator=gen, device=DEV)
        y = (x * 3 + 1) % 97
        logits = model(x)
        loss = F.cross_entropy(logits.float().view(-1, 97), y.view(-1))
        scaler.scale(loss).backward()
        scaler.unscale_(opt)
        norm = clip(model.parameters(), 1.0)
        scaler.step(opt)
        scaler.update()
        losses.append(float(loss.detach()))
        norms.append(float(norm))
        if fused:
            plans = opt._plan_builds
    return losses, norms, plans, opt


def test_training_loop_tracks_torch_reference():
    ours, our_norms, n_plans, opt = _train(fused=True)
    ref, ref_norms, _, _ = _train(fused=False)
    assert ours[-1] < 0.35 * ours[0], "the bf16 model must learn the task"
    assert ref[-1] < 0.35 * ref[0]
    # bf16 forward/backward against fp32: the trajectories agree to bf16 accuracy
    for a, b in zip(ours, ref):
        assert abs(a - b) <= 0.1 * abs(b) + 0.1
    assert abs(our_norms[0] - ref_norms[0]) <= 0.03 * ref_norms[0]
    assert n_plans == 1  # autograd's reallocated gradients only patch the pointers
    steps = {float(s["step"]) for s in opt.state.values()}
    assert steps == {40.0}


def test_fp16_autocast_loop_follows_the_scaler_contract():
    """The reference's own mixed-precision mode (``train.py:366-370,479-491``; GradScaler enabled
    for fp16 autocast): fp32 parameters, fp16 activations, scaled fp32 gradients.  A large initial
    scale forces overflow skips and a short growth interval forces growth; every step's skip
    decision must equal the gradients' own finiteness, a skipped step must leave parameters and
    step counters untouched, and the scale must follow backoff/growth exactly.  As in the
    reference loop, each step accumulates two micro-batches (``loss / 2``) and keeps a running
    maximum of the returned norm tensor."""
    from minigpt_train_infra_b200 import (FusedAdamW, GradScaler, build_adamw_param_groups,
                                          clip_grad_norm_)
    torch.manual_seed(0)
    model = TinyDecoder().to(DEV)
    opt = FusedAdamW(build_adamw_param_groups(model, 0.1), lr=3e-3, betas=(0.9, 0.95), eps=1e-8)
    scaler = GradScaler("cuda", init_scale=2.0 ** 24, growth_interval=4)
    gen = torch.Generator(device=DEV).manual_seed(1)
    scale, tracker, skips, growths, losses = 2.0 ** 24, 0, 0, 0, []
    params = list(model.parameters())
    for step in range(40):
        for g in opt.param_groups:
            g["lr"] = _cosine(step)
        opt.zero_grad(set_to_none=True)
        for _micro in range(2):  # gradient accumulation (train.py's micro-step loop)
            x = torch.randint(0, 97, (16, 32), generator=gen, device=DEV)
            with torch.autocast("cuda", dtype=torch.float16):
                logits = model(x)
                loss = F.cross_entropy(logits.float().view(-1, 97), ((x * 3 + 1) % 97).view(-1))
            scaler.scale(loss / 2).backward()
        bad = not all(bool(torch.isfinite(p.grad).all()) for p in params)
        before = [p.detach().clone() for p in params]
        scaler.unscale_(opt)
        norm = clip_grad_norm_(params, 1.0)
        norm_max = norm.detach().float() if step == 0 else torch.maximum(
            norm_max, norm.detach().float())
        scaler.step(opt)
        scaler.update()
        if bad:
            skips += 1
            scale, tracker = scale * 0.5, 0
            assert all(torch.equal(a, p) for a, p in zip(before, params))
        else:
            losses.append(float(loss.detach()))
            tracker += 1
            if tracker == 4:
                scale, tracker, growths = scale * 2.0, 0, growths + 1
            assert not any(torch.equal(a, p) for a, p in zip(before, params[:1]))
        assert scaler.get_scale() == scale
        assert int(scaler._growth_tracker) == tracker
        assert {float(s["step"]) for s in opt.state.values()} <= {float(step + 1 - skips)}
    assert skips >= 1 and growths >= 1
    assert not bool(torch.isfinite(norm_max))  # an overflowing step's norm is inf or NaN
    assert {float(s["step"]) for s in opt.state.values()} == {40.0 - skips}
    assert losses[-1] < 0.6 * losses[0], "the fp16-autocast model must learn the task"


def test_tiny_gpu_config_bf16_autocast_tracks_torch():
    """The reference's ``configs/tiny_gpu.json`` recipe: 4 layers, 4 heads, 128 wide, block 128,
    batch 16, 4 accumulation micro-steps, bf16 autocast over fp32 parameters with the scaler
    disabled (GradScaler is enabled for fp16 only, ``train.py:366-370``), lr 6e-4 with 20 warm-up
    steps, weight decay 0.01 on matrices, betas (0.9, 0.95), clip 1.0.  Against torch's own
    ``AdamW(fused=True)`` + ``GradScaler(enabled=False)`` + ``clip_grad_norm_`` from the same
    initial weights and batches: after the first step the weights agree to the rounding of the
    two update implementations; over 30 steps the losses and norms track to 2e-3 and the
    weights on average to 1e-5 (an element whose gradient is near zero may take Adam's full
    +-lr step one way in one run and the other way in the other)."""
    from minigpt_train_infra_b200 import (FusedAdamW, GradScaler, build_adamw_param_groups,
                                          clip_grad_norm_)

    def run(fused):
        torch.manual_seed(1337)
        model = TinyDecoder(vocab=65, d=128, n_layer=4, n_head=4, block=128).to(DEV)
        groups = build_adamw_param_groups(model, 0.01)
        if fused:
            opt = FusedAdamW(groups, lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
            scaler, clip = GradScaler("cuda", enabled=False), clip_grad_norm_
        else:
            opt = torch.optim.AdamW(groups, lr=6e-4, betas=(0.9, 0.95), eps=1e-8, fused=True)
            scaler = torch.amp.GradScaler("cuda", enabled=False)
            clip = torch.nn.utils.clip_grad_norm_
        gen = torch.Generator(device=DEV).manual_seed(7)
        losses, norms = [], []
        for step in range(30):
            for g in opt.param_groups:
                g["lr"] = _cosine(step, base=6e-4, warm=20, total=200, low=6e-5)
            opt.zero_grad(set_to_none=True)
            for _micro in range(4):
                x = torch.randint(0, 65, (16, 128), generator=gen, device=DEV)
                with torch.autocast("cuda", dtype=torch.bfloat16):
                    logits = model(x)
                    loss = F.cross_entropy(logits.float().view(-1, 65), ((x * 3 + 1) % 65).view(-1))
                scaler.scale(loss / 4).backward()
            scaler.unscale_(opt)
            norms.append(float(clip(model.parameters(), 1.0)))
            scaler.step(opt)
            scaler.update()
            losses.append(float(loss.detach()))
            if step == 0:
                first = [p.detach().clone() for p in model.parameters()]
        return losses, norms, [p.detach().clone() for p in model.parameters()], opt, first

    ours, our_norms, our_w, opt, our_first = run(True)
    ref, ref_norms, ref_w, _, ref_first = run(False)
    for a, b in zip(our_first, ref_first):
        assert float((a - b).abs().max()) <= 1e-6
    assert ours[-1] < ours[0], "the loss must fall"
    for a, b in zip(ours, ref):
        assert abs(a - b) <= 2e-3 * abs(b)
    for a, b in zip(our_norms, ref_norms):
        assert abs(a - b) <= 2e-3 * abs(b)
    diffs = torch.cat([(a - b).abs().flatten() for a, b in zip(our_w, ref_w)])
    assert float(diffs.mean()) <= 1e-5
    assert float(diffs.max()) <= 2e-2
    assert {float(s["step"]) for s in opt.state.values()} == {30.0}
