"""The drop-in inside the reference's own training loop, checkpoint and resume code.

The reference's ``train.py`` is a script (it is not part of the installable ``minigpt`` package),
so these tests drive the loop body of ``train.py:343-491`` with the reference's own modules --
``MiniGPT``, ``RandomTokenBatcher``, ``RuntimeContext``, ``build_adamw_param_groups``,
``cosine_lr``/``set_optimizer_lr``, ``next_token_cross_entropy``, ``build_checkpoint_payload``,
``load_optimizer_state``, ``load_grad_scaler_state``, ``restore_rng_state`` -- imported from the
reference installed under ``baseline/_ref`` (``python -m pip install --no-index
--no-build-isolation --no-deps --target baseline/_ref <reference checkout>``).  The tests skip,
saying so, when it is not installed.  The only change between the two arms is the three-line swap:
``torch.optim.AdamW`` -> ``FusedAdamW``, ``torch.amp.GradScaler`` -> ``GradScaler``,
``torch.nn.utils.clip_grad_norm_`` -> ``clip_grad_norm_``.

Data: the reference trains on a character corpus that is not part of the package; a seeded
uniform token stream over the same 65-symbol vocabulary stands in for it.
"""

from __future__ import annotations

import io
import random
import sys
import warnings
from dataclasses import dataclass, replace
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent
REF = ROOT / "baseline" / "_ref"


def _reference():
    if not (REF / "minigpt" / "optim.py").exists():
        pytest.skip("the reference is not installed under baseline/_ref (pip install --no-index "
                    "--no-build-isolation --no-deps --target baseline/_ref <reference checkout>)")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from minigpt import checkpoint, data, model, optim, runtime
    return SimpleNamespace(checkpoint=checkpoint, data=data, model=model, optim=optim,
                           runtime=runtime)


@dataclass(frozen=True)
class Recipe:
    """The values of the reference's configs/tiny_gpu.json (model and train sections)."""
    block_size: int = 128
    n_layer: int = 4
    n_head: int = 4
    n_embd: int = 128
    dropout: float = 0.1
    precision: str = "bf16"
    seed: int = 1337
    batch_size: int = 16
    gradient_accumulation_steps: int = 4
    max_steps: int = 200
    learning_rate: float = 6e-4
    min_learning_rate: float = 6e-5
    warmup_steps: int = 20
    weight_decay: float = 0.01
    beta1: float = 0.9
    beta2: float = 0.95
    adam_eps: float = 1e-8
    grad_clip: float = 1.0
    vocab_size: int = 65


TINY_GPU = Recipe()
# The recipe of the reference's tests/test_resume_consistency.py:84-112 (checkpoint at step 2 of 4)
RESUME = Recipe(block_size=8, n_layer=1, n_head=2, n_embd=16, precision="fp32", batch_size=2,
                gradient_accumulation_steps=2, max_steps=4, learning_rate=1e-3,
                min_learning_rate=1e-4, warmup_steps=1)


def run_loop(R, cfg: Recipe, steps: int, swap: bool, *, model_dtype=torch.float32,
             scaler_enabled: bool | None = None, checkpoint_at: int | None = None,
             resume: bytes | None = None):
    """train.py's loop (lines 343-491, without eval/logging) on the reference's modules."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    rt = R.runtime.RuntimeContext.create("cuda", cfg.precision)
    device = rt.device
    random.seed(cfg.seed)
    rt.manual_seed(cfg.seed)
    tokens = torch.randint(0, cfg.vocab_size, (50_000,), generator=torch.Generator().manual_seed(0))
    batcher = R.data.RandomTokenBatcher(tokens=tokens, batch_size=cfg.batch_size,
                                        block_size=cfg.block_size, device=device,
                                        seed=cfg.seed + 1)
    model = R.model.MiniGPT(R.model.MiniGPTConfig(
        vocab_size=cfg.vocab_size, block_size=cfg.block_size, n_layer=cfg.n_layer,
        n_head=cfg.n_head, n_embd=cfg.n_embd, dropout=cfg.dropout)).to(device)
    model.to(model_dtype)
    groups = R.optim.build_adamw_param_groups(model, cfg.weight_decay)
    AdamW = FusedAdamW if swap else torch.optim.AdamW
    Scaler = GradScaler if swap else torch.amp.GradScaler
    clip = clip_grad_norm_ if swap else torch.nn.utils.clip_grad_norm_
    optimizer = AdamW(groups, lr=cfg.learning_rate, betas=(cfg.beta1, cfg.beta2),
                      eps=cfg.adam_eps, fused=rt.capabilities.supports_fused_adamw)
    enabled = (rt.precision == "fp16") if scaler_enabled is None else scaler_enabled
    scaler = Scaler(device.type, enabled=enabled, init_scale=2.0 ** 12)
    start = 0
    if resume is not None:  # train.py:371-383
        ckpt = torch.load(io.BytesIO(resume), map_location="cpu", weights_only=False)
        model.load_state_dict(R.model.migrate_model_state_dict(ckpt["model_state"]))
        R.optim.load_optimizer_state(optimizer, ckpt["optimizer_state"], model)
        R.optim.load_grad_scaler_state(scaler, ckpt["scaler_state"])
        R.checkpoint.restore_rng_state(ckpt)
        batcher.generator.set_state(ckpt["train_batcher_state"].cpu())
        start = int(ckpt["step"])
    model.train()
    trace = {"loss": [], "norm": [], "scale": [], "lr": []}
    saved = None
    for step in range(start, steps):
        lr = R.optim.cosine_lr(step=step, base_lr=cfg.learning_rate,
                               min_lr=cfg.min_learning_rate, warmup_steps=cfg.warmup_steps,
                               max_steps=cfg.max_steps)
        R.optim.set_optimizer_lr(optimizer, lr)
        optimizer.zero_grad(set_to_none=True)
        loss_sum = torch.zeros((), dtype=torch.float32, device=device)
        for _ in range(cfg.gradient_accumulation_steps):
            x, y = batcher.get_batch()
            with rt.autocast():
                logits = model(x)
                loss = R.model.next_token_cross_entropy(logits, y)
                loss_for_backward = loss / cfg.gradient_accumulation_steps
            scaler.scale(loss_for_backward).backward()
            loss_sum += loss.detach().float()
        scaler.unscale_(optimizer)
        grad_norm = clip(model.parameters(), cfg.grad_clip)
        scaler.step(optimizer)
        scaler.update()
        trace["loss"].append(float(loss_sum) / cfg.gradient_accumulation_steps)
        trace["norm"].append(float(grad_norm))
        trace["scale"].append(scaler.get_scale() if scaler.is_enabled() else 1.0)
        trace["lr"].append(lr)
        if checkpoint_at is not None and step + 1 == checkpoint_at:
            payload = R.checkpoint.build_checkpoint_payload(
                model=model, optimizer=optimizer, scaler=scaler, step=step + 1, config={},
                best_val_loss=None)
            payload["train_batcher_state"] = batcher.generator.get_state()
            buf = io.BytesIO()
            torch.save(payload, buf)
            saved = buf.getvalue()
    return SimpleNamespace(model=model, optimizer=optimizer, scaler=scaler, trace=trace,
                           saved=saved)


def completed_steps(optimizer) -> int:
    """train.py:162-176 optimizer_completed_steps: state["step"] of the first parameter."""
    for group in optimizer.param_groups:
        for p in group["params"]:
            st = optimizer.state.get(p)
            if st and "step" in st:
                return int(st["step"].item())
    return 0


def _rel(a, b) -> float:
    return max(abs(x - y) / max(abs(y), 1e-12) for x, y in zip(a, b))


def test_tiny_gpu_recipe_with_the_three_line_swap():
    """configs/tiny_gpu.json: bf16 autocast over fp32 parameters, scaler off, four accumulation
    micro-steps, warm-up then cosine lr, 30 optimizer steps.  The swapped arm tracks torch's
    AdamW(fused=True) arm step for step (different but equally rounded fp32 arithmetic)."""
    R = _reference()
    stock = run_loop(R, TINY_GPU, 30, swap=False)
    ours = run_loop(R, TINY_GPU, 30, swap=True)
    assert stock.trace["lr"] == ours.trace["lr"]
    assert _rel(ours.trace["loss"], stock.trace["loss"]) <= 2e-3
    assert _rel(ours.trace["norm"], stock.trace["norm"]) <= 2e-2
    assert completed_steps(ours.optimizer) == completed_steps(stock.optimizer) == 30
    assert ours.trace["loss"][-1] < ours.trace["loss"][0]


def test_fp16_recipe_scaler_sequence_matches_stock():
    """The reference's fp16 mode (train.py:366-370: scaler enabled, init 2**12, fp32 parameters):
    the swapped arm follows the stock arm's loss-scale sequence and skip decisions exactly."""
    R = _reference()
    cfg = replace(TINY_GPU, precision="fp16")
    stock = run_loop(R, cfg, 30, swap=False)
    ours = run_loop(R, cfg, 30, swap=True)
    assert ours.trace["scale"] == stock.trace["scale"]
    assert completed_steps(ours.optimizer) == completed_steps(stock.optimizer)
    assert _rel(ours.trace["loss"], stock.trace["loss"]) <= 2e-3


def _assert_nested_equal(left, right, path="root"):
    """tests/test_resume_consistency.py:23-40 of the reference: exact equality, tensors by
    torch.equal."""
    if isinstance(left, torch.Tensor):
        assert isinstance(right, torch.Tensor) and torch.equal(left, right), path
        return
    if isinstance(left, dict):
        assert isinstance(right, dict) and left.keys() == right.keys(), path
        for k in left:
            _assert_nested_equal(left[k], right[k], f"{path}.{k}")
        return
    if isinstance(left, (list, tuple)):
        assert type(left) is type(right) and len(left) == len(right), path
        for i, (a, b) in enumerate(zip(left, right)):
            _assert_nested_equal(a, b, f"{path}[{i}]")
        return
    assert left == right, f"{path}: {left!r} != {right!r}"


@pytest.mark.parametrize("variant", ["fp32_params", "bf16_params_scaled"])
def test_resume_through_reference_checkpoint_is_bit_exact(variant):
    """tests/test_resume_consistency.py:76-149 of the reference, on a GPU with the swap: four
    steps in one go against two steps, a checkpoint (build_checkpoint_payload, torch.save), a
    fresh process state restored by load_optimizer_state / load_grad_scaler_state /
    restore_rng_state, and two more steps.  Model, optimizer and scaler state must be equal.
    Attention runs on the math backend, whose backward is deterministic.  The second variant
    keeps bf16 parameters (fp32 masters in the checkpoint) with the scaler enabled."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    R = _reference()
    kw = {} if variant == "fp32_params" else {"model_dtype": torch.bfloat16,
                                               "scaler_enabled": True}
    with sdpa_kernel(SDPBackend.MATH):
        cont = run_loop(R, RESUME, 4, swap=True, checkpoint_at=2, **kw)
        resumed = run_loop(R, RESUME, 4, swap=True, resume=cont.saved, **kw)
    assert resumed.trace["loss"] == cont.trace["loss"][2:]
    _assert_nested_equal(cont.model.state_dict(), resumed.model.state_dict(), "model_state")
    _assert_nested_equal(cont.optimizer.state_dict(), resumed.optimizer.state_dict(),
                         "optimizer_state")
    _assert_nested_equal(cont.scaler.state_dict(), resumed.scaler.state_dict(), "scaler_state")
    sd = cont.optimizer.state_dict()
    if variant == "bf16_params_scaled":
        assert all(s["master_param"].dtype == torch.float32 and
                   s["exp_avg"].dtype == torch.float32 for s in sd["state"].values())
    assert completed_steps(resumed.optimizer) == 4


def test_reference_legacy_loader_moment_truncation_is_reported():
    """load_optimizer_state's migration path (src/minigpt/optim.py:124-133,242-251) casts every
    state tensor to the parameter dtype before assigning it.  Under bf16 parameters that rounds
    the fp32 moments to bf16; the optimizer warns when such state reaches it, and stays silent
    for the native format (which load_state_dict keeps in fp32)."""
    R = _reference()
    run = run_loop(R, RESUME, 2, swap=True, model_dtype=torch.bfloat16, scaler_enabled=True)
    model, opt = run.model, run.optimizer
    sd = opt.state_dict()
    # a single-group payload in model parameter order (the pre-v0.3 layout the migration reads)
    ids = {id(p): i for i, p in enumerate(p for g in opt.param_groups for p in g["params"])}
    order = [ids[id(p)] for _, p in model.named_parameters()]
    legacy = {"state": {k: sd["state"][i] for k, i in enumerate(order)},
              "param_groups": [{k: v for k, v in sd["param_groups"][0].items()
                                if k not in ("param_names", "group_name", "params")}
                               | {"params": list(range(len(order)))}]}
    with pytest.warns(RuntimeWarning, match="rounded"):
        R.optim.load_optimizer_state(opt, legacy, model)
        opt.state_dict()  # the optimizer reconciles assigned state here
    with warnings.catch_warnings():
        warnings.simplefilter("error", RuntimeWarning)
        R.optim.load_optimizer_state(opt, sd, model)
        opt.state_dict()


def test_zero_consolidated_state_continues_in_fused_adamw_bit_exactly():
    """ZeroAdamW (one rank) -> consolidated_state_dict() -> FusedAdamW.load_state_dict -> two
    more steps, against ZeroAdamW continuing itself: every state word equal."""
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    from minigpt_train_infra_b200.zero1 import ZeroAdamW
    dev = torch.device("cuda", 0)
    shapes = [(64, 48), (48,), (1000,), (7,)]
    gen = torch.Generator().manual_seed(21)
    w0 = [torch.randn(s, generator=gen) * 0.02 for s in shapes]

    def grads(step):
        g = torch.Generator().manual_seed(300 + step)
        return [(torch.randn(s, generator=g) * 0.1 * 2.0 ** 10).to(torch.bfloat16).to(dev)
                for s in shapes]

    def step_with(opt, params, sc, k):
        for p, g in zip(params, grads(k)):
            p.grad = g
        sc.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        sc.step(opt)
        sc.update()

    pz = [torch.nn.Parameter(w.to(torch.bfloat16).to(dev)) for w in w0]
    zopt = ZeroAdamW([{"params": pz[:1], "weight_decay": 0.1},
                      {"params": pz[1:], "weight_decay": 0.0}], lr=1e-3, betas=(0.9, 0.95))
    zsc = GradScaler("cuda", init_scale=2.0 ** 10)
    zsc.scale(torch.ones((), device=dev))
    for k in range(2):
        step_with(zopt, zopt.managed_params(), zsc, k)
    consolidated = zopt.consolidated_state_dict()
    pf = [torch.nn.Parameter(p.detach().clone()) for p in zopt.managed_params()]
    fopt = FusedAdamW([{"params": pf[:1], "weight_decay": 0.1},
                       {"params": pf[1:], "weight_decay": 0.0}], lr=1e-3, betas=(0.9, 0.95))
    fopt.load_state_dict(consolidated)
    fsc = GradScaler("cuda", init_scale=2.0 ** 10)
    fsc.load_state_dict(zsc.state_dict())
    fsc.scale(torch.ones((), device=dev))  # creates the scale tensor, as scaling a loss does
    for k in range(2, 4):
        step_with(zopt, zopt.managed_params(), zsc, k)
        step_with(fopt, pf, fsc, k)
    torch.cuda.synchronize()
    zsd = zopt.consolidated_state_dict()
    fsd = fopt.state_dict()
    for i in range(len(shapes)):
        for key in ("step", "exp_avg", "exp_avg_sq", "master_param"):
            assert torch.equal(zsd["state"][i][key].cpu(), fsd["state"][i][key].cpu()), (i, key)
    for a, b in zip(zopt.managed_params(), pf):
        assert torch.equal(a, b)
