"""Parameter-shape lists of the benchmark configurations.

Each list is ``[(name, shape, group)]`` in ``named_parameters`` order with the reference's
decay split (group 0 = ``ndim >= 2`` with weight decay, group 1 = the rest), exactly what
``build_adamw_param_groups`` (reference ``src/minigpt/optim.py:15-64``) yields for:

* ``minigpt_6l_384`` -- ``MiniGPT`` (reference ``src/minigpt/model.py:271``) 6 layers, 6 heads,
  384 wide, block 256, vocab 65, tied ``lm_head``: 76 tensors, 10,770,816 params;
* ``gpt2_124m`` -- the same class at 12 layers, 768 wide, block 1024, vocab 50257: 148 tensors,
  124,439,808 params;
* ``qwen3_1_7b`` -- ``Qwen3ForCausalLM`` (reference ``src/minigpt/qwen3.py:708``) 28 layers, hidden
  2048, MLP 6144, 16 q / 8 kv heads of 128, vocab 151936, tied: 310 tensors, 1,720,574,976;
* ``qwen3_8b`` -- 36 layers, hidden 4096, MLP 12288, 32 q / 8 kv heads of 128, untied
  ``lm_head``: 399 tensors, 8,190,735,360 params;
* ``flat_2_28`` -- one tensor of 2**28 elements; ``flat_2_26`` -- 2**26 elements, the small case
  used for profiler captures (about 1.2 GB on the device, still far above the L2).

The lists are written out here (the benchmark box has no reference checkout); a CPU test checks
them against ``tests/golden/param_shapes.json``, which was generated from the reference classes.
"""

from __future__ import annotations

import math


def minigpt(vocab: int, block: int, n_layer: int, n_embd: int) -> list[tuple[str, tuple, int]]:
    c = n_embd
    out = [("token_embedding.weight", (vocab, c), 0), ("position_embedding.weight", (block, c), 0)]
    for i in range(n_layer):
        p = f"blocks.{i}."
        out += [
            (p + "ln_1.weight", (c,), 1), (p + "ln_1.bias", (c,), 1),
            (p + "attn.qkv_proj.weight", (3 * c, c), 0), (p + "attn.qkv_proj.bias", (3 * c,), 1),
            (p + "attn.out_proj.weight", (c, c), 0), (p + "attn.out_proj.bias", (c,), 1),
            (p + "ln_2.weight", (c,), 1), (p + "ln_2.bias", (c,), 1),
            (p + "mlp.fc.weight", (4 * c, c), 0), (p + "mlp.fc.bias", (4 * c,), 1),
            (p + "mlp.proj.weight", (c, 4 * c), 0), (p + "mlp.proj.bias", (c,), 1),
        ]
    out += [("ln_f.weight", (c,), 1), ("ln_f.bias", (c,), 1)]
    return out


def qwen3(vocab: int, hidden: int, inter: int, n_layer: int, n_q: int, n_kv: int, head_dim: int,
          tied: bool) -> list[tuple[str, tuple, int]]:
    h = hidden
    out = [("model.embed_tokens.weight", (vocab, h), 0)]
    for i in range(n_layer):
        p = f"model.layers.{i}."
        out += [
            (p + "self_attn.q_proj.weight", (n_q * head_dim, h), 0),
            (p + "self_attn.k_proj.weight", (n_kv * head_dim, h), 0),
            (p + "self_attn.v_proj.weight", (n_kv * head_dim, h), 0),
            (p + "self_attn.o_proj.weight", (h, n_q * head_dim), 0),
            (p + "self_attn.q_norm.weight", (head_dim,), 1),
            (p + "self_attn.k_norm.weight", (head_dim,), 1),
            (p + "mlp.gate_proj.weight", (inter, h), 0),
            (p + "mlp.up_proj.weight", (inter, h), 0),
            (p + "mlp.down_proj.weight", (h, inter), 0),
            (p + "input_layernorm.weight", (h,), 1),
            (p + "post_attention_layernorm.weight", (h,), 1),
        ]
    out += [("model.norm.weight", (h,), 1)]
    if not tied:
        out += [("lm_head.weight", (vocab, h), 0)]
    return out


WORKLOADS = {
    "minigpt_6l_384": lambda: minigpt(65, 256, 6, 384),
    "gpt2_124m": lambda: minigpt(50257, 1024, 12, 768),
    "qwen3_1_7b": lambda: qwen3(151936, 2048, 6144, 28, 16, 8, 128, True),
    "qwen3_8b": lambda: qwen3(151936, 4096, 12288, 36, 32, 8, 128, False),
    "flat_2_28": lambda: [("flat", (1 << 28,), 0)],
    "flat_2_26": lambda: [("flat", (1 << 26,), 0)],
}


def shapes(name: str) -> list[tuple[str, tuple, int]]:
    try:
        return WORKLOADS[name]()
    except KeyError:
        raise KeyError(f"unknown workload {name!r}; choose from {sorted(WORKLOADS)}") from None


def n_params(name: str) -> int:
    return sum(math.prod(s) for _, s, _ in shapes(name))
