"""One rank of the "a rank leaves between steps" test (run as a child process by
``test_zero1_gpu.py``; not a test module itself).

    python zero_leave_worker.py <rank> <world> <port> <out_dir> <timeout_s>

Every rank runs ZeroAdamW steps over NCCL (no peer memory), with the rendezvous store passed to
ZeroAdamW as its membership store.  After two completed steps the last rank announces that it
leaves (``announce_leave``), takes part in a barrier with the others -- nothing of any rank in
flight -- destroys its process group and exits 0.  The other ranks start a third step, whose
membership check must raise before any collective or kernel is issued; the rank records the
error and exits 3.  Progress lines go to ``<out_dir>/rank<r>.log`` so the parent can see where
it stopped.
"""

from __future__ import annotations

import datetime
import faulthandler
import os
import sys
import time

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [HERE, os.path.dirname(HERE)]


def main() -> None:
    rank, world, port, out_dir, timeout_s = (int(sys.argv[1]), int(sys.argv[2]),
                                             int(sys.argv[3]), sys.argv[4], float(sys.argv[5]))
    from minigpt_train_infra_b200 import GradScaler, ZeroAdamW, clip_grad_norm_
    log = open(os.path.join(out_dir, f"rank{rank}.log"), "w", buffering=1)

    def note(msg: str) -> None:
        log.write(f"{time.time():.3f} {msg}\n")

    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0,
                          timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s), device_id=device)
    gen = torch.Generator().manual_seed(5)
    shapes = [(256, 128), (128,), (4097,)]
    params = [torch.nn.Parameter((torch.randn(s, generator=gen) * 0.02).to(torch.bfloat16)
                                 .to(device)) for s in shapes]
    opt = ZeroAdamW(params, lr=1e-3, betas=(0.9, 0.95), peer_memory=False,
                    membership_store=store)
    scaler = GradScaler("cuda", init_scale=2.0 ** 10)
    scaler.scale(torch.ones((), device=device))
    for step in range(3):
        if step == 2 and rank == world - 1:
            note("left")
            log.close()
            dist.destroy_process_group()
            return
        note(f"step {step} start")
        if step == 2:  # where the rank is stuck if the check does not end the step
            faulthandler.dump_traceback_later(timeout_s + 40, exit=False, file=log)
        try:
            for p in opt.managed_params():
                p.grad.copy_(torch.randn(p.shape, generator=gen).to(torch.bfloat16).to(device)
                             * 64)
            scaler.unscale_(opt)
            clip_grad_norm_(opt.managed_params(), 1.0)
            scaler.step(opt)
            scaler.update()
            torch.cuda.synchronize()
        except Exception as e:  # the collective's timeout, raised in this thread
            note(f"step {step} error {type(e).__name__}: {' '.join(str(e).split())[:400]}")
            log.close()
            os._exit(3)  # the process group is unusable; leave without touching it
        note(f"step {step} done")
        if step == 1:
            if rank == world - 1:
                opt.announce_leave()
                note("announced")
            dist.barrier()  # every rank between steps, nothing in flight
            torch.cuda.synchronize()
            note("barrier done")
    note("all steps done")
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
