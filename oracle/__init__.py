"""CPU oracle for the fused mixed-precision optimizer step.

TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import, call or execute anything in this package, and only
as the checker (or, for ``bench.py``, as the timed CPU baseline).  The product path in
``minigpt_train_infra_b200`` never imports it and has no CPU fallback.

Modules:

* ``adamw_oracle`` -- numpy restatement of the arithmetic that the reference's training step
  (``train.py:485-491``) runs through PyTorch: ``GradScaler.unscale_``, ``clip_grad_norm_``,
  single-tensor ``AdamW`` and ``GradScaler.update``, plus the bf16 parameter copy and the ZeRO-1
  shard arithmetic that the build adds.
* ``torch_chain`` -- the reference's own CPU call sequence (torch ``AdamW(foreach=False,
  fused=False)``, ``torch.amp.GradScaler("cpu")``, ``torch.nn.utils.clip_grad_norm_``) driven
  on host tensors; this is what the reference executes on a CPU and what ``bench.py --impl
  reference`` times.
Parity pin: ``tests/golden/make_golden.py`` imports the reference (``src/minigpt``) in the
build container, runs its optimizer chain on CPU and commits the outputs as fixtures; the CPU
test suite checks this oracle against them.
"""
