"""B200-native fused mixed-precision optimizer step for the MiniGPT training loop.

Public surface (drop-ins for the reference's ``train.py:359-370,485-491``):

* :class:`FusedAdamW` -- ``torch.optim.AdamW`` replacement (``optim.py``);
* :class:`GradScaler` -- ``torch.amp.GradScaler`` replacement (``amp.py``);
* :func:`clip_grad_norm_` -- ``torch.nn.utils.clip_grad_norm_`` replacement (``clip.py``);
* :class:`ZeroAdamW` -- ZeRO-1 sharded variant over ``torch.distributed`` NCCL (``zero1.py``);
* :func:`build_adamw_param_groups` -- the reference's decay/no-decay grouping (``groups.py``).

The arithmetic runs in hand-written sm_100a kernels behind the C ABI of
``include/b200_optim.h`` (``csrc/``), loaded with ctypes from ``lib/libb200_optim.so``.
"""

from .amp import GradScaler
from .clip import clip_grad_norm_
from .groups import build_adamw_param_groups
from .optim import FusedAdamW

__all__ = ["FusedAdamW", "GradScaler", "clip_grad_norm_", "build_adamw_param_groups",
           "ZeroAdamW"]


def __getattr__(name):
    if name == "ZeroAdamW":
        from .zero1 import ZeroAdamW
        return ZeroAdamW
    raise AttributeError(name)
