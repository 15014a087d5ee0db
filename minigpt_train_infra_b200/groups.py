"""AdamW parameter grouping with the reference's contract.

Restates ``build_adamw_param_groups`` (reference ``src/minigpt/optim.py:15-64``) so that callers
without the reference package (the benchmark, the GPU tests) group parameters exactly as the
training loop does: trainable tensors with ``ndim >= 2`` go to ``"decay"`` with the given weight
decay, the rest to ``"no_decay"`` with 0.0, in ``named_parameters`` order, each group carrying
``param_names`` and ``group_name``; a parameter seen twice, or a trainable parameter left out,
raises ``ValueError``.  The reference's own function works unchanged with ``FusedAdamW``.
"""

from __future__ import annotations

from typing import Any

import torch


def build_adamw_param_groups(model: torch.nn.Module, weight_decay: float) -> list[dict[str, Any]]:
    if weight_decay < 0:
        raise ValueError("weight_decay must be non-negative")
    decay, no_decay, decay_names, no_decay_names = [], [], [], []
    seen: set[int] = set()
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if id(p) in seen:
            raise ValueError(f"Model parameter appears more than once: {name}")
        seen.add(id(p))
        if p.ndim >= 2:
            decay.append(p)
            decay_names.append(name)
        else:
            no_decay.append(p)
            no_decay_names.append(name)
    expected = {id(p) for p in model.parameters() if p.requires_grad}
    if seen != expected:
        raise ValueError("Optimizer parameter grouping did not cover every trainable model "
                         "parameter exactly once")
    return [
        {"params": decay, "param_names": decay_names, "group_name": "decay",
         "weight_decay": weight_decay},
        {"params": no_decay, "param_names": no_decay_names, "group_name": "no_decay",
         "weight_decay": 0.0},
    ]
