"""Generate the golden fixtures in this directory from the reference itself.

Run in a container that has the reference checkout (the GPU box does not need it):

    python tests/golden/make_golden.py --reference <path to minigpt-train-infra>

It imports the reference's own modules (``src/minigpt/model.py``, ``optim.py``, ``qwen3.py``)
and drives the reference's optimizer step (``train.py:359-370`` construction, ``:485-491``
step sequence) on CPU through ``oracle/torch_chain.py``.  Outputs:

* ``param_shapes.json`` -- ``(name, shape, group)`` of every trainable tensor of the benchmark
  configurations, from the reference's model classes and ``build_adamw_param_groups``.
* ``tiny_minigpt_fp32.npz`` -- a small MiniGPT (reference class) trained for 10 free-running
  steps with fp32 gradients from its own forward/backward, scaler disabled, clip 1.0 (the
  reference's fp32 configuration).
* ``tiny_minigpt_bf16_scaled.npz`` -- the same model, gradients rounded to bf16 after scaling
  by the loss scale, GradScaler enabled (growth interval 4), +inf injected at step 5 and NaN
  at step 8 to exercise skip-and-backoff and growth.
* ``ragged_bf16_scaled.npz`` -- synthetic tensors of ragged sizes (0, 1, 7, 9, 4097, ...) with
  bf16 gradients, two groups, clipping active, an inf step and a NaN step.

Each ``.npz`` stores the initial masters, every step's gradients and, after every step, the
reference's masters, ``exp_avg``, ``exp_avg_sq``, ``step``, the returned total norm,
``found_inf``, the loss scale and the growth tracker.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle.torch_chain import ChainConfig, ReferenceChain  # noqa: E402

HP = dict(lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_norm=1.0)


def _import_reference(root: Path):
    sys.path.insert(0, str(root / "src"))
    import minigpt.model as model  # noqa: F401
    import minigpt.optim as optim  # noqa: F401
    import minigpt.qwen3 as qwen3  # noqa: F401
    return model, optim, qwen3


def param_shapes(model_mod, optim_mod, qwen3_mod) -> dict:
    MiniGPT, MiniGPTConfig = model_mod.MiniGPT, model_mod.MiniGPTConfig
    out = {}

    def record(name, model):
        groups = optim_mod.build_adamw_param_groups(model, HP["weight_decay"])
        gid = {}
        for gi, g in enumerate(groups):
            for n in g["param_names"]:
                gid[n] = gi
        out[name] = [[n, list(p.shape), gid[n]] for n, p in model.named_parameters()
                     if p.requires_grad]

    with torch.device("meta"):
        record("minigpt_6l_384", MiniGPT(MiniGPTConfig(vocab_size=65, block_size=256, n_layer=6,
                                                       n_head=6, n_embd=384, dropout=0.0)))
        record("gpt2_124m", MiniGPT(MiniGPTConfig(vocab_size=50257, block_size=1024, n_layer=12,
                                                  n_head=12, n_embd=768, dropout=0.0)))
    qwen = {
        "qwen3_1_7b": dict(vocab_size=151936, hidden_size=2048, intermediate_size=6144,
                           num_hidden_layers=28, num_attention_heads=16, num_key_value_heads=8,
                           head_dim=128, max_position_embeddings=40960,
                           tie_word_embeddings=True),
        "qwen3_8b": dict(vocab_size=151936, hidden_size=4096, intermediate_size=12288,
                         num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8,
                         head_dim=128, max_position_embeddings=40960,
                         tie_word_embeddings=False),
    }
    for name, raw in qwen.items():
        cfg = qwen3_mod.Qwen3Config.from_dict(raw)
        record(name, qwen3_mod.Qwen3ForCausalLM(cfg, device="meta"))
    return out


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def _run(chain: ReferenceChain, names, grads_per_step, grad_store):
    """Step ``chain`` over the given gradients; return arrays for the fixture."""
    rec = {"norm": [], "found_inf": [], "scale": [], "tracker": []}
    ws, ms, vs, steps = [], [], [], []
    for grads in grads_per_step:
        out = chain.step([g.float() for g in grads])
        rec["norm"].append(np.nan if out["norm"] is None else out["norm"])
        rec["found_inf"].append(out["found_inf"])
        rec["scale"].append(out.get("scale", 1.0))
        rec["tracker"].append(out.get("tracker", 0))
        ws.append([p.detach().numpy().copy() for p in chain.params])
        st = [chain.state_of(p) for p in chain.params]
        ms.append([s["exp_avg"].numpy().copy() if s else np.zeros(p.shape, np.float32)
                   for s, p in zip(st, chain.params)])
        vs.append([s["exp_avg_sq"].numpy().copy() if s else np.zeros(p.shape, np.float32)
                   for s, p in zip(st, chain.params)])
        steps.append([float(s["step"]) if s else 0.0 for s in st])
    arrays = {}
    for k, v in rec.items():
        arrays[k] = np.asarray(v, dtype=np.float64 if k != "tracker" else np.int64)
    n_steps = len(grads_per_step)
    for i in range(len(names)):
        arrays[f"w/{i}"] = np.stack([ws[s][i] for s in range(n_steps)])
        arrays[f"m/{i}"] = np.stack([ms[s][i] for s in range(n_steps)])
        arrays[f"v/{i}"] = np.stack([vs[s][i] for s in range(n_steps)])
        arrays[f"g/{i}"] = np.stack([grad_store(grads_per_step[s][i]) for s in range(n_steps)])
    arrays["step"] = np.asarray(steps, dtype=np.float32)
    return arrays


def tiny_minigpt(model_mod, optim_mod, bf16_scaled: bool) -> dict:
    MiniGPT, MiniGPTConfig = model_mod.MiniGPT, model_mod.MiniGPTConfig
    torch.manual_seed(1234)
    model = MiniGPT(MiniGPTConfig(vocab_size=65, block_size=16, n_layer=1, n_head=2, n_embd=16,
                                  dropout=0.0))
    groups = optim_mod.build_adamw_param_groups(model, HP["weight_decay"])
    names = [n for g in groups for n in g["param_names"]]
    group_of = [gi for gi, g in enumerate(groups) for _ in g["params"]]
    init = [p.detach().numpy().copy() for g in groups for p in g["params"]]
    scale = 2.0 ** 16
    cfg = ChainConfig(lr=HP["lr"], betas=HP["betas"], eps=HP["eps"], max_norm=HP["max_norm"],
                      scaler_enabled=bf16_scaled, init_scale=scale, growth_interval=4)
    chain = ReferenceChain([g["params"] for g in groups], [g["weight_decay"] for g in groups], cfg)
    gen = torch.Generator().manual_seed(99)
    grads_per_step = []
    arrays_steps = []
    # The reference model runs forward/backward on the chain's own (updated) fp32 params, so the
    # run is free-running: gradients of step s come from the parameters after step s-1.
    by_name = dict(model.named_parameters())
    targets = [by_name[n] for n in names]
    for s in range(10):
        with torch.no_grad():
            for dst, src in zip(targets, chain.params):
                dst.copy_(src)
        model.zero_grad(set_to_none=True)
        x = torch.randint(0, 65, (4, 16), generator=gen)
        y = torch.randint(0, 65, (4, 16), generator=gen)
        loss = model_mod.next_token_cross_entropy(model(x), y)
        (loss * (scale if bf16_scaled else 1.0)).backward()
        grads = [t.grad.detach().clone() for t in targets]
        if bf16_scaled:
            grads = [g.to(torch.bfloat16) for g in grads]
            if s == 4:
                grads[1].view(-1)[5] = float("inf")
            if s == 7:
                grads[-1].view(-1)[0] = float("nan")
        grads_per_step.append(grads)
        arrays_steps.append(_run(chain, names, [grads], _bf16_bits if bf16_scaled else
                                 (lambda g: g.numpy().copy())))
    # merge per-step records
    arrays = {k: np.concatenate([a[k] for a in arrays_steps]) for k in arrays_steps[0]}
    for i, w0 in enumerate(init):
        arrays[f"w0/{i}"] = w0
    arrays["names"] = np.asarray(names)
    arrays["group"] = np.asarray(group_of, dtype=np.int64)
    arrays["wd"] = np.asarray([g["weight_decay"] for g in groups], dtype=np.float64)
    arrays["hp"] = np.asarray([HP["lr"], HP["betas"][0], HP["betas"][1], HP["eps"],
                               HP["max_norm"], scale if bf16_scaled else 1.0, 4.0])
    arrays["grad_dtype"] = np.asarray("bf16" if bf16_scaled else "fp32")
    return arrays


def ragged(model_mod, optim_mod) -> dict:
    shapes = [(0,), (1,), (7,), (9,), (4097,), (33, 65), (3, 5, 7), (100, 24), (8,), (2053,)]
    torch.manual_seed(7)
    init = [torch.randn(s) * 0.02 for s in shapes]
    group_of = [0 if len(s) >= 2 else 1 for s in shapes]
    order = [i for i in range(len(shapes)) if group_of[i] == 0] + \
            [i for i in range(len(shapes)) if group_of[i] == 1]
    scale = 2.0 ** 16
    cfg = ChainConfig(lr=3e-4, betas=(0.9, 0.95), eps=1e-8, max_norm=1.0, scaler_enabled=True,
                      init_scale=scale, growth_interval=3)
    dec = [init[i] for i in order if group_of[i] == 0]
    nod = [init[i] for i in order if group_of[i] == 1]
    chain = ReferenceChain([dec, nod], [0.1, 0.0], cfg)
    gen = torch.Generator().manual_seed(11)
    grads_per_step = []
    for s in range(9):
        gs = [(torch.randn(shapes[i], generator=gen) * 1e-1 * scale).to(torch.bfloat16)
              for i in order]
        if s == 3:
            gs[order.index(4)].view(-1)[17] = float("-inf")
        if s == 6:
            gs[order.index(6)].view(-1)[0] = float("nan")
        grads_per_step.append(gs)
    arrays = _run(chain, [str(i) for i in order], grads_per_step, _bf16_bits)
    for j, i in enumerate(order):
        arrays[f"w0/{j}"] = init[i].numpy().copy()
    arrays["names"] = np.asarray([f"t{i}" for i in order])
    arrays["group"] = np.asarray([group_of[i] for i in order], dtype=np.int64)
    arrays["wd"] = np.asarray([0.1, 0.0])
    arrays["hp"] = np.asarray([3e-4, 0.9, 0.95, 1e-8, 1.0, scale, 3.0])
    arrays["grad_dtype"] = np.asarray("bf16")
    return arrays


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MINIGPT_REFERENCE", ""))
    args = ap.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference <checkout of the reference repository>")
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    model_mod, optim_mod, qwen3_mod = _import_reference(Path(args.reference))
    shapes = param_shapes(model_mod, optim_mod, qwen3_mod)
    (HERE / "param_shapes.json").write_text(json.dumps(shapes, separators=(",", ":")) + "\n")
    np.savez_compressed(HERE / "tiny_minigpt_fp32.npz", **tiny_minigpt(model_mod, optim_mod, False))
    np.savez_compressed(HERE / "tiny_minigpt_bf16_scaled.npz",
                        **tiny_minigpt(model_mod, optim_mod, True))
    np.savez_compressed(HERE / "ragged_bf16_scaled.npz", **ragged(model_mod, optim_mod))
    meta = {"torch": torch.__version__, "numpy": np.__version__,
            "cpu_capability": torch.backends.cpu.get_cpu_capability(),
            "threads": torch.get_num_threads()}
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    print("wrote fixtures:", meta)


if __name__ == "__main__":
    main()
