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
    members: dict[str, tuple[list, list]] = {"decay": ([], []), "no_decay": ([], [])}
    owner: dict[int, str] = {}
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        if id(p) in owner:
            raise ValueError(f"Model parameter appears more than once: {name}")
        owner[id(p)] = name
        tensors, names = members["decay" if p.ndim >= 2 else "no_decay"]
        tensors.append(p)
        names.append(name)
    if set(owner) != {id(p) for p in model.parameters() if p.requires_grad}:
        raise ValueError("Optimizer parameter grouping did not cover every trainable model "
                         "parameter exactly once")
    # key order and values as the reference writes them (they end up in checkpoints)
    return [{"params": members[g][0], "param_names": members[g][1], "group_name": g,
             "weight_decay": weight_decay if g == "decay" else 0.0}
            for g in ("decay", "no_decay")]
