"""Benchmark of the fused mixed-precision optimizer step (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload qwen3_8b] [--impl ours]

One "step" is the reference's optimizer step (train.py:485-491) through this package's public
API: ``GradScaler.unscale_`` -> ``clip_grad_norm_`` -> ``GradScaler.step`` -> ``update`` over
the whole parameter list of the workload, with the optimizer state resident in HBM.  At N=1 it
is :class:`FusedAdamW`; at N>1 (torchrun, one rank per GPU, NCCL) it is the ZeRO-1
:class:`ZeroAdamW`, each rank updating its contiguous 1/N shard.

Printed by rank 0: one JSON line with ``value`` = Gparams/s of the timed steps (device time,
max over ranks), the roofline of the AdamW kernel, the end-to-end number through host buffers,
the CPU baseline (the reference's torch CPU chain on the host cores), clocks and launch count.
``--impl reference`` times only the reference's CPU chain, on rank 0.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from minigpt_train_infra_b200 import workloads  # noqa: E402

METRIC = "fused AdamW step Gparams/s and HBM GB/s vs peak at 1/2/4/8 B200"
L2_BYTES = 126 * 2 ** 20
ADAMW_BYTES = 28   # read g(2)+w,m,v(12); write w,m,v(12)+bf16 param(2)
STATS_BYTES = 2    # read g
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes per parameter of one adamw_kernel launch, from an ncu capture of the flat 2**26
# workload (dram__bytes_read.sum + dram__bytes_write.sum = 940.43 MB + 882.66 MB over 2**26
# params).  The full workload is too large to capture under the profiler's size rule, so the
# per-parameter figure of the small capture is scaled by the params per launch.
NCU_TRAFFIC_BYTES_PER_PARAM = (940.429824e6 + 882.656768e6) / 2 ** 26
LR, BETAS, EPS, WD, CLIP = 3e-4, (0.9, 0.95), 1e-8, 0.1, 1.0
SCALES = {"qwen3_8b": 2.0 ** 15}
GRAD_STD = {"flat_2_28": 1e-2, "flat_2_26": 1e-2}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ------------------------------------------------------------------------------------------
# peaks and clocks
# ------------------------------------------------------------------------------------------

def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """NVML samples of SM clock and throttle reasons while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x10: "sync_boost"}

    def __init__(self, device_index: int, period: float = 0.05):
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            uuid = None
            try:
                uuid = torch.cuda.get_device_properties(device_index).uuid
            except Exception:
                pass
            self._h = None
            if uuid is not None:
                try:
                    self._h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
                except Exception:
                    self._h = None
            if self._h is None:
                vis = os.environ.get("CUDA_VISIBLE_DEVICES")
                idx = int(vis.split(",")[device_index]) if vis else device_index
                self._h = pynvml.nvmlDeviceGetHandleByIndex(idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._ok = True
        except Exception as e:  # NVML missing: report no clock data rather than fail
            log("clock sampling unavailable:", e)
        self.period = period
        self._t = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                r = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self._stop.wait(self.period)

    def __enter__(self):
        if self._ok:
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._ok:
            self._t.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ------------------------------------------------------------------------------------------
# workload setup
# ------------------------------------------------------------------------------------------

def make_model_params(shape_list, device) -> tuple[list, list]:
    params, groups = [], []
    for _, shape, g in shape_list:
        params.append(torch.nn.Parameter(torch.empty(shape, dtype=torch.bfloat16, device=device)))
        groups.append(g)
    return params, groups


def fill_seeded(t: torch.Tensor, seed: int, std: float, absval: bool = False) -> None:
    """Seeded N(0, std) (or |N(0,1)|*std) fill, generated on the device tensor by tensor."""
    gen = torch.Generator(device=t.device).manual_seed(seed)
    flat = t.view(-1)
    step = 1 << 28
    for k, s in enumerate(range(0, flat.numel(), step)):
        part = flat[s:s + step]
        tmp = torch.empty(part.numel(), dtype=torch.float32, device=t.device)
        tmp.normal_(0.0, 1.0, generator=gen)
        if absval:
            tmp.abs_()
        tmp.mul_(std)
        part.copy_(tmp)
        del tmp


def seed_state(opt, params, step0: float = 999.0) -> None:
    """Config-2 state: master ~ N(0,0.02), m ~ N(0,1e-3), v = |N(0,1)|*1e-6, step 999."""
    store = opt._ensure_store()
    opt._sync_state()
    fill_seeded(store.master, 1, 0.02)
    fill_seeded(store.exp_avg, 2, 1e-3)
    fill_seeded(store.exp_avg_sq, 3, 1e-6, absval=True)
    store.steps.fill_(step0)
    with torch.no_grad():
        for slot, p in enumerate(store.params):
            mp = store.views[slot].get("master_param")
            if mp is not None:
                p.copy_(mp)


def make_grads(params, scale: float, std: float, seed: int = 7) -> list[torch.Tensor]:
    grads = []
    for i, p in enumerate(params):
        g = torch.empty_like(p)
        fill_seeded(g, seed * 1000 + i, std * scale)
        grads.append(g)
    return grads


# ------------------------------------------------------------------------------------------
# CPU baseline: the reference's torch CPU chain on a bounded sample of the same workload
# ------------------------------------------------------------------------------------------

def cpu_sample_shapes(shape_list, min_params: int = 1 << 27) -> list:
    """The workload's tensors from the first 2-D weight on, until >= min_params (bounded)."""
    out, tot = [], 0
    for item in shape_list:
        n = math.prod(item[1])
        if tot >= min_params:
            break
        if n > 4 * min_params and tot == 0 and len(shape_list) > 1:
            continue  # skip a vocabulary matrix so the sample stays bounded
        out.append(item)
        tot += n
    return out


def run_cpu_baseline(shape_list, scale: float, std: float, steps: int = 3, warmup: int = 1):
    from oracle.torch_chain import ChainConfig, ReferenceChain, time_reference_chain
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample = cpu_sample_shapes(shape_list)
    n = sum(math.prod(s) for _, s, _ in sample)
    gen = torch.Generator().manual_seed(11)
    dec = [torch.randn(s, generator=gen) * 0.02 for _, s, g in sample if g == 0]
    nod = [torch.randn(s, generator=gen) * 0.02 for _, s, g in sample if g == 1]
    cfg = ChainConfig(lr=LR, betas=BETAS, eps=EPS, max_norm=CLIP, init_scale=scale)
    chain = ReferenceChain([dec, nod], [WD, 0.0], cfg)
    order = [s for _, s, g in sample if g == 0] + [s for _, s, g in sample if g == 1]
    grads = [(torch.randn(s, generator=gen) * std * scale).to(torch.bfloat16) for s in order]
    times = time_reference_chain(chain, grads, steps=steps, warmup=warmup)
    med = statistics.median(times)
    cpu_name = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu_name = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {
        "value": n / med / 1e9, "unit": "Gparams/s", "cores": torch.get_num_threads(),
        "kind": "reference",
        "sample": (f"{len(sample)} tensors / {n:,} params of the workload (its first layers), "
                   f"median of {steps} steps after {warmup} warm-up; torch {torch.__version__} "
                   f"CPU AdamW(foreach=False,fused=False)+GradScaler('cpu')+clip_grad_norm_ in "
                   f"the order of train.py:485-491, bf16 grads upcast and bf16 param copy "
                   f"included; CPU: {cpu_name}"),
        "seconds_per_step": med,
    }


# ------------------------------------------------------------------------------------------
# parity leg: one more step through the public API, after the timed steps, checked against the
# oracle.  The oracle is the checker here, never the thing timed.
# ------------------------------------------------------------------------------------------

PARITY_SAMPLES = 4096


def _owned_slices(opt, ws: int) -> list[dict]:
    """Every tensor range this rank updates, as flat 1-D views of its state, gradient and bf16
    parameter, with its step slot and hyper-parameter group."""
    out = []
    if ws > 1:
        g = opt.geom
        for slot, lo, hi in g.local_ranges():
            if hi <= lo:
                continue
            la, lb = lo - g.lo, hi - g.lo
            out.append({"slot": slot, "group": opt._slot_group[slot], "flat_lo": lo,
                        "master": opt.master[la:lb], "exp_avg": opt.exp_avg[la:lb],
                        "exp_avg_sq": opt.exp_avg_sq[la:lb], "grad": opt.flat_grad[lo:hi],
                        "param": opt.flat_param[lo:hi], "steps": opt.steps})
        return out
    store = opt._store
    gid = {id(p): gi for gi, grp in enumerate(opt.param_groups) for p in grp["params"]}
    for slot, p in enumerate(store.params):
        v = store.views[slot]
        out.append({"slot": slot, "group": gid[id(p)], "flat_lo": None,
                    "master": v["master_param"].view(-1), "exp_avg": v["exp_avg"].view(-1),
                    "exp_avg_sq": v["exp_avg_sq"].view(-1), "grad": p.grad.view(-1),
                    "param": p.detach().view(-1), "steps": store.steps})
    return out


def _bits16(t: torch.Tensor):
    return t.contiguous().view(torch.int16).cpu().numpy().view("uint16")


def _piecewise_int_sum(t: torch.Tensor, piece: int = 1 << 27) -> int:
    """Exact integer sum of a tensor's words, in pieces (no full-size int64 temporary)."""
    dt = torch.int16 if t.element_size() == 2 else torch.int32
    flat = t.view(dt).view(-1)
    return sum(int(flat[a:a + piece].sum(dtype=torch.int64)) for a in range(0, flat.numel(), piece))


def _fp64_norm(grads, inv_scale: float, piece: int = 1 << 26) -> float:
    """The statistics' two-level norm with the sums in fp64: fp32(sqrt(sum x^2)) per tensor, then
    the norm of those, x = fp32(g * inv_scale)."""
    import numpy as np
    from oracle import adamw_oracle as O
    norms = []
    for g in grads:
        flat = g.reshape(-1)
        acc = 0.0
        for a in range(0, flat.numel(), piece):
            x = (flat[a:a + piece].float() * inv_scale).double()
            acc += float((x * x).sum())
        norms.append(np.float32(math.sqrt(acc)))
    return float(O.total_norm(norms))


def _state_checksum(opt, ws: int) -> list[int]:
    """Exact checksums of every state word this rank owns, its step counters and its copy of the
    bf16 parameters."""
    if ws > 1:
        bufs = [opt.master, opt.exp_avg, opt.exp_avg_sq, opt.steps, opt.flat_param]
    else:
        st = opt._store
        bufs = [st.master, st.exp_avg, st.exp_avg_sq, st.steps] + [p.detach() for p in st.params]
    return [_piecewise_int_sum(b) for b in bufs]


def parity_check(opt, scaler, step_params, ws: int, rank: int, seed: int = 0) -> dict:
    """Two more steps through the public API (unscale_ -> clip_grad_norm_ -> step -> update, and
    the bf16 parameter exchange at N>1), checked against the oracle:

    * a clean step: on every rank, PARITY_SAMPLES seeded elements of every tensor range the rank
      owns (all of a shorter range) -- master, exp_avg and exp_avg_sq bit-exact against the
      oracle fed the kernel's global norm; at N>1 every rank's copy of the bf16 parameters at
      every rank's samples bit-exact against the oracle's bf16 rounding (the gathered
      parameters), and each rank's own bf16 shard equal to bf16(master) word for word; rank 0
      checks the global norm against an fp64 norm of the whole gradient (within 2 ulp);
    * a step with +inf at one element of the last rank's range: found_inf is 1 on every rank,
      every state word, step counter and bf16 parameter is unchanged on every rank, and the loss
      scale is halved.

    Returns the summary on rank 0 (None elsewhere).  Every rank issues the same collectives."""
    import numpy as np
    from minigpt_train_infra_b200 import clip_grad_norm_
    from oracle import adamw_oracle as O
    dist = torch.distributed if ws > 1 else None
    device = scaler._scale.device
    sync = torch.cuda.synchronize if device.type == "cuda" else (lambda: None)
    slices = _owned_slices(opt, ws)
    gen = torch.Generator().manual_seed(1000 * seed + 17 * rank + 1)
    before = []
    for sl in slices:
        n = sl["master"].numel()
        k = min(n, PARITY_SAMPLES)
        ix = torch.randint(0, n, (k,), generator=gen).to(device)
        before.append({"ix": ix, "w": sl["master"][ix].cpu().numpy(),
                       "m": sl["exp_avg"][ix].cpu().numpy(),
                       "v": sl["exp_avg_sq"][ix].cpu().numpy(), "g": _bits16(sl["grad"][ix]),
                       "step": float(sl["steps"][sl["slot"]])})
    scale0 = float(scaler.get_scale())
    sync()

    def api_step():
        scaler.unscale_(opt)
        norm = clip_grad_norm_(step_params, CLIP)
        found = next(iter(scaler._per_optimizer_states[id(opt)]["found_inf_per_device"]
                          .values())).clone()
        scaler.step(opt)
        scaler.update()
        if ws > 1 and opt.defer_param_gather:
            opt.gather_params()
        sync()
        return float(norm), float(found)

    norm, found = api_step()
    norm32 = np.float32(norm)
    inv = O.inv_scale_of(scale0)
    coef = O.clip_coefficient(norm32, CLIP)
    groups = opt.param_groups
    mism = 0
    max_ulp = 0
    checked = 0
    expect_pos, expect_bits = [], []
    for sl, b in zip(slices, before):
        grp = groups[sl["group"]]
        hp = O.GroupHP(grp["lr"], grp["betas"][0], grp["betas"][1], grp["eps"],
                       grp["weight_decay"])
        g = (O.unscale(O.bf16_bits_to_f32(b["g"]), inv) * coef).astype(np.float32)
        w2, m2, v2 = O.adamw_update(b["w"], b["m"], b["v"], g, hp, b["step"] + 1.0)
        for key, want in (("master", w2), ("exp_avg", m2), ("exp_avg_sq", v2)):
            got = sl[key][b["ix"]].cpu().numpy()
            d = np.abs(got.view(np.int32).astype(np.int64) - want.view(np.int32).astype(np.int64))
            mism += int(np.count_nonzero(d))
            max_ulp = max(max_ulp, int(d.max()) if d.size else 0)
        pbits = O.f32_to_bf16_bits(w2)
        mism += int(np.count_nonzero(_bits16(sl["param"][b["ix"]]) != pbits))
        checked += len(b["w"])
        if sl["flat_lo"] is not None:
            expect_pos.append(b["ix"].cpu().numpy() + sl["flat_lo"])
            expect_bits.append(pbits)
    gathered_checked = gathered_mism = shard_mism = 0
    if ws > 1:
        # each rank's own bf16 shard is bf16(master), word for word ...
        own = opt.flat_param[opt.geom.lo:opt.geom.hi]
        for a in range(0, own.numel(), 1 << 27):
            shard_mism += int((own[a:a + (1 << 27)].view(torch.int16) !=
                               opt.master[a:a + (1 << 27)].to(torch.bfloat16).view(torch.int16))
                              .sum())
        # ... and every rank holds every rank's updated bf16 values at the sampled positions
        mine = (np.concatenate(expect_pos) if expect_pos else np.zeros(0, np.int64),
                np.concatenate(expect_bits) if expect_bits else np.zeros(0, np.uint16))
        allv = [None] * ws
        dist.all_gather_object(allv, mine)
        for pos, bits in allv:
            if len(pos) == 0:
                continue
            got = _bits16(opt.flat_param[torch.from_numpy(pos).to(device)])
            gathered_mism += int(np.count_nonzero(got != bits))
            gathered_checked += len(pos)
    norm_ref = None
    if rank == 0:
        grads = [p.grad for p in step_params]
        norm_ref = _fp64_norm(grads, float(inv))
    norm_ulp = None if norm_ref is None else abs(float(norm32) - norm_ref) / float(
        np.spacing(norm32))

    # the skip: +inf at one element of the last rank's range
    sums0 = _state_checksum(opt, ws)
    inj = None
    if rank == ws - 1:
        sl = slices[-1]
        pos = min(17, sl["grad"].numel() - 1)
        inj = (sl["grad"], pos, sl["grad"][pos].clone())
        sl["grad"][pos] = float("inf")
    scale1 = float(scaler.get_scale())
    _, found_skip = api_step()
    scale2 = float(scaler.get_scale())
    sums1 = _state_checksum(opt, ws)
    if inj is not None:
        inj[0][inj[1]] = inj[2]
        sync()
    local = torch.tensor([mism, max_ulp, checked, gathered_checked, gathered_mism, shard_mism,
                          found_skip != 1.0, sums0 != sums1, scale2 != scale1 * 0.5,
                          found != 0.0], dtype=torch.float64, device=device)
    if ws > 1:
        parts = [torch.empty_like(local) for _ in range(ws)]
        dist.all_gather(parts, local)
        tot = torch.stack(parts).cpu().numpy()
    else:
        tot = local.cpu().numpy()[None, :]
    if rank != 0:
        return None
    ok = bool(tot[:, [0, 4, 5, 6, 7, 8, 9]].sum() == 0 and norm_ulp is not None and
              norm_ulp <= 2.0)
    return {
        "ok": ok,
        "samples_checked": int(tot[:, 2].sum()),
        "state_words_checked": int(3 * tot[:, 2].sum()),
        "state_words_mismatched": int(tot[:, 0].sum()),
        "max_ulp_diff": int(tot[:, 1].max()),
        "gathered_bf16_checked": int(tot[:, 3].sum()),
        "gathered_bf16_mismatched": int(tot[:, 4].sum()),
        "own_shard_bf16_vs_master_mismatched": int(tot[:, 5].sum()),
        "norm": {"kernel": float(norm32), "fp64_reference": norm_ref,
                 "ulp_diff": None if norm_ulp is None else round(norm_ulp, 3)},
        "clean_step_found_inf_zero_on_every_rank": bool(tot[:, 9].sum() == 0),
        "skip": {"inf_on_rank": ws - 1, "found_inf_on_every_rank": bool(tot[:, 6].sum() == 0),
                 "state_and_steps_unchanged_on_every_rank": bool(tot[:, 7].sum() == 0),
                 "scale_halved_on_every_rank": bool(tot[:, 8].sum() == 0),
                 "scale": [scale1, scale2]},
        "how": (f"{PARITY_SAMPLES} seeded samples of every owned tensor range per rank, after "
                "the timed steps; oracle fed the kernel's global norm; bit-exact compare"),
    }


# ------------------------------------------------------------------------------------------
# our arm
# ------------------------------------------------------------------------------------------

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def make_zero_opt(groups, pg, rank: int, std: float, scale: float, peer_memory: bool,
                  defer_param_gather: bool):
    """ZeroAdamW over ``groups`` with the seeded state of the benchmark: each rank's shard of
    master ~ N(0,0.02), m ~ N(0,1e-3), v = |N(0,1)|*1e-6 (rank-specific seeds), step 999, and the
    same bf16 gradients N(0,std)*scale on every rank."""
    from minigpt_train_infra_b200 import ZeroAdamW
    opt = ZeroAdamW(groups, lr=LR, betas=BETAS, eps=EPS, process_group=pg,
                    defer_param_gather=defer_param_gather, peer_memory=peer_memory)
    fill_seeded(opt.master, 1 + 101 * rank, 0.02)
    fill_seeded(opt.exp_avg, 2 + 101 * rank, 1e-3)
    fill_seeded(opt.exp_avg_sq, 3 + 101 * rank, 1e-6, absval=True)
    opt.steps.fill_(999.0)
    with torch.no_grad():
        opt.owned_param_shard().copy_(opt.master)
    if peer_memory:
        # the fused broadcast writes tensor ranges only from the first step on; start every
        # rank's copy equal with one ordinary all-gather
        torch.distributed.all_gather_into_tensor(opt.flat_param, opt.owned_param_shard(),
                                                 group=pg)
    opt.gather_params()
    fill_seeded(opt.flat_grad, 7, std * scale)
    return opt


def run_ours(args) -> None:
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    pg = None
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)
        pg = dist.group.WORLD
    from minigpt_train_infra_b200 import FusedAdamW, GradScaler, clip_grad_norm_
    name = args.workload
    shape_list = workloads.shapes(name)
    P = workloads.n_params(name)
    scale = SCALES.get(name, 2.0 ** 16)
    std = GRAD_STD.get(name, 1e-3)
    t0 = time.time()
    params, gids = make_model_params(shape_list, device)
    groups = [{"params": [p for p, g in zip(params, gids) if g == 0], "weight_decay": WD},
              {"params": [p for p, g in zip(params, gids) if g == 1], "weight_decay": 0.0}]
    groups = [g for g in groups if g["params"]]
    if ws > 1:
        opt = make_zero_opt(groups, pg, rank, std, scale, peer_memory=args.peer_memory,
                            defer_param_gather=True)
        grads = opt.make_flat_grads_()
        step_params = opt.managed_params()
        params = step_params
    else:
        opt = FusedAdamW(groups, lr=LR, betas=BETAS, eps=EPS, capturable=args.graph)
        seed_state(opt, params)
        grads = make_grads(params, scale, std)
        step_params = params
    scaler = GradScaler("cuda", init_scale=scale, growth_interval=2000, backoff_factor=0.5)
    for p, g in zip(params, grads):
        p.grad = g
    scaler.scale(torch.ones((), device=device))  # creates the scale tensor, as loss scaling does
    torch.cuda.synchronize()
    log(f"[rank {rank}] setup {time.time() - t0:.1f}s, {P:,} params, "
        f"mem {torch.cuda.memory_allocated() / 2**30:.1f} GiB")

    def one_step(ev=None):
        """One step; ``ev`` = 2 events (start, end) for the timed steps, or 4 (start, after the
        statistics pass, after the update, end) for the per-kernel breakdown."""
        if ev is not None:
            ev[0].record()
        scaler.unscale_(opt)
        clip_grad_norm_(step_params, CLIP)
        if ev is not None and len(ev) == 4:
            ev[1].record()
        scaler.step(opt)
        if ev is not None and len(ev) == 4:
            ev[2].record()
        scaler.update()
        if ev is not None:
            ev[-1].record()

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    # Workloads whose per-step footprint (bf16 grad + bf16 param + fp32 master/m/v = 16 B per
    # owned parameter) is under 4x the 126 MB L2 get L2 flushed before every timed step (a
    # 256 MB write outside the step's events); larger ones stream far more than L2 holds.
    P_own = opt.local_numel() if ws > 1 else P
    footprint = 16 * P_own
    flush_buf = torch.empty(64 << 20, dtype=torch.float32, device=device) \
        if footprint < 4 * L2_BYTES else None

    def flush_l2():
        if flush_buf is not None:
            flush_buf.zero_()

    eager_phases = None
    if args.graph and ws == 1:
        # a replay cannot be split into its kernels with events, so the per-kernel times (and the
        # roofline) come from eager steps of the same kernels, timed here before the capture
        k = max(3, min(args.steps, 10))
        pev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(k)]
        for e in pev:
            flush_l2()
            one_step(e)
        torch.cuda.synchronize()
        eager_phases = [statistics.mean(e[i].elapsed_time(e[i + 1]) for e in pev)
                        for i in range(3)]
        # the whole step captured once; each timed step stages hyper-parameters and replays
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            scaler.unscale_(opt)
            clip_grad_norm_(step_params, CLIP)
            scaler.step(opt)
            scaler.update()
        torch.cuda.synchronize()

        def one_step(ev=None):  # noqa: F811 -- the timed step becomes a replay
            if ev is not None:
                ev[0].record()
            opt.prepare_replay()
            graph.replay()
            if ev is not None:
                ev[-1].record()
    if pg is not None:
        torch.distributed.barrier()
    # the timed steps record a start and an end event only (the host records no more than a
    # caller would); the per-kernel split comes from separate steps of the same kernels below
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        if pg is not None:
            torch.distributed.barrier()
            torch.cuda.synchronize()
        for i in range(args.steps):
            flush_l2()
            one_step(evs[i])
        torch.cuda.synchronize()
    if flush_buf is None:
        total_ms = evs[0][0].elapsed_time(evs[-1][1])
    else:  # the flushes between steps are not step time
        total_ms = sum(e[0].elapsed_time(e[1]) for e in evs)
    if eager_phases is not None:
        stats_ms, adamw_ms, upd_ms = eager_phases
    else:
        k = max(3, min(args.steps, 10))
        pev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(k)]
        for e in pev:
            flush_l2()
            one_step(e)
        torch.cuda.synchronize()
        stats_ms, adamw_ms, upd_ms = [statistics.mean(e[i].elapsed_time(e[i + 1]) for e in pev)
                                      for i in range(3)]
    if pg is not None:
        t = torch.tensor([total_ms, stats_ms, adamw_ms, upd_ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        total_ms, stats_ms, adamw_ms, upd_ms = [float(x) for x in t.tolist()]
    ms_per_step = total_ms / args.steps
    value = P * args.steps / (total_ms / 1e3) / 1e9
    allgather = None
    if ws > 1 and args.peer_memory:
        allgather = fused_broadcast_report(opt, P, ws, ms_per_step, adamw_ms)
    elif ws > 1:
        allgather = time_allgather(args, opt, one_step, device, P, ws)
    P_local = opt.local_numel() if ws > 1 else P
    peak, peak_kind = hbm_peak()
    achieved = ADAMW_BYTES * P_local / (adamw_ms / 1e3) / 1e9
    n_plans = len(opt._plans or [])
    launches_per_step = (n_plans + (1 if n_plans > 1 else 0)) + n_plans + 1
    if ws > 1:
        launches_per_step += 1  # finalize of the exchanged partials

    # parity: two more steps through the same API after the timed ones, checked by the oracle
    leg = "single_gpu" if ws == 1 else ("zero1_peer_memory" if args.peer_memory else
                                        "zero1_nccl_allgather")
    parity = {leg: parity_check(opt, scaler, step_params, ws, rank)}

    # end-to-end through the public API with host-resident gradients
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, opt, scaler, step_params, params, grads, device, P, pg)

    # N>1: the full step with the bf16 all-gather fused into the update, timed and checked in
    # the same run (the NCCL leg's buffers are released first: both do not fit at once)
    peer_leg = None
    if ws > 1 and not args.peer_memory and not args.no_peer_leg:
        del opt, grads, step_params, params, scaler
        opt = None
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        peer_leg = run_peer_leg(args, shape_list, P, scale, std, device, pg, ws, rank)
        parity["zero1_peer_memory"] = peer_leg.pop("parity")

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_baseline(shape_list, scale, std)
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 3), "unit": "Gparams/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded on device: master~N(0,0.02), m~N(0,1e-3), v=|N(0,1)|*1e-6,"
                    f" bf16 grads~N(0,{std})*{scale:g})",
            "config": {
                "workload": f"{name}: {len(shape_list)} tensors, {P:,} params (BASELINE config "
                            f"{ {'minigpt_6l_384': 1, 'flat_2_28': 2, 'gpt2_124m': 3, 'qwen3_1_7b': 4, 'qwen3_8b': 5}.get(name, '?') })",
                "params": P, "params_per_rank": P_local,
                "parallelism": "single GPU" if ws == 1 else f"zero1 over {ws} GPUs",
                "timed": "unscale_+clip_grad_norm_+step+update per step" +
                         ((" (sharded update with the bf16 all-gather fused into it as peer "
                           "stores)" if args.peer_memory else
                           " (sharded update; bf16 all-gather reported under allgather)")
                          if ws > 1 else ""),
                "l2": (f"flushed before every timed step (256 MB write outside the step's "
                       f"events): the step's {footprint / 1e6:.0f} MB footprint is under 4x the "
                       "126 MB L2") if flush_buf is not None else
                      ("no flush: every step streams the whole optimizer state "
                       f"({footprint / 1e9:.1f} GB per rank, {footprint / L2_BYTES:.0f}x the "
                       "126 MB L2)"),
                "hp": {"lr": LR, "betas": BETAS, "eps": EPS, "weight_decay": WD, "clip": CLIP,
                       "loss_scale": scale},
            },
            "kernels_ms_source": ("eager steps of the same kernels before the capture"
                                  if eager_phases is not None else
                                  "eager steps of the same kernels after the timed steps, with "
                                  "an event between the statistics pass, the update and the "
                                  "scaler update"),
            "kernels_ms": {"grad_stats": round(stats_ms, 4), "adamw": round(adamw_ms, 4),
                           "scaler_update": round(upd_ms, 4)},
            "hbm_gbs": round((ADAMW_BYTES + STATS_BYTES) * P_local / (ms_per_step / 1e3) / 1e9, 1),
            "hbm_frac": round((ADAMW_BYTES + STATS_BYTES) * P_local / (ms_per_step / 1e3) / 1e9
                              / peak, 4),
            "roofline": {"bound": "hbm", "kernel": "b2o adamw_kernel", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": f"{peak_kind} copy bandwidth",
                         "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "bytes_per_param": ADAMW_BYTES, "params_per_launch": P_local,
                         "traffic": round(NCU_TRAFFIC_BYTES_PER_PARAM * P_local),
                         "traffic_source": "ncu dram read+write bytes per param of the 2**26 "
                                           "capture x params per launch"},
            "clocks": clocks.summary(),
            "gpu_launches": launches_per_step * args.steps,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        if ws > 1:
            line["allgather"] = allgather
            line["full_step"] = {"zero1_nccl_allgather": allgather}
            if peer_leg is not None:
                line["full_step"]["zero1_peer_memory"] = peer_leg
        line["parity"] = {"ok": all(v is not None and v["ok"] for v in parity.values()),
                          **parity}
        emit_result(line)
    if pg is not None:
        if opt is not None and hasattr(opt, "close"):
            opt.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def _nvlink_bound(P_padded: int, P_local: int, ws: int) -> dict:
    """Lower bound of a full ZeRO-1 step at N ranks: every rank must receive the other ranks'
    updated bf16 shards, 2 * P * (N-1)/N bytes over its NVLink at the measured 770 GB/s per
    direction, and must stream its own shard's 30 bytes per parameter through HBM."""
    peak, _ = hbm_peak()
    recv = 2 * P_padded * (ws - 1) / ws
    nvlink_ms = recv / 770e9 * 1e3
    hbm_ms = (ADAMW_BYTES + STATS_BYTES) * P_local / (peak * 1e9) * 1e3
    return {"recv_bytes_per_rank": int(recv), "nvlink_ms": round(nvlink_ms, 3),
            "hbm_ms": round(hbm_ms, 3), "bound_ms": round(max(nvlink_ms, hbm_ms), 3),
            "bound": "nvlink" if nvlink_ms >= hbm_ms else "hbm"}


def run_peer_leg(args, shape_list, P: int, scale: float, std: float, device, pg, ws: int,
                 rank: int) -> dict:
    """The ZeRO-1 step with the bf16 all-gather fused into the update (``peer_memory=True``):
    the AdamW kernel stores every updated bf16 value into every rank's parameter buffer over
    NVLink (TMA bulk stores of staged 4 KB chunks, 16-byte stores for ragged ones), then a
    one-element all-reduce orders the ranks.
    Timed as the full step -- statistics, norm exchange, update with broadcast, ordering, scaler
    update -- with CUDA events, max over ranks; then checked by the parity leg."""
    import torch.distributed as dist
    from minigpt_train_infra_b200 import GradScaler, clip_grad_norm_
    params, gids = make_model_params(shape_list, device)
    groups = [{"params": [p for p, g in zip(params, gids) if g == 0], "weight_decay": WD},
              {"params": [p for p, g in zip(params, gids) if g == 1], "weight_decay": 0.0}]
    groups = [g for g in groups if g["params"]]
    opt = make_zero_opt(groups, pg, rank, std, scale, peer_memory=True,
                        defer_param_gather=False)
    opt.make_flat_grads_()
    step_params = opt.managed_params()
    scaler = GradScaler("cuda", init_scale=scale, growth_interval=2000, backoff_factor=0.5)
    scaler.scale(torch.ones((), device=device))

    def one_step():
        scaler.unscale_(opt)
        clip_grad_norm_(step_params, CLIP)
        scaler.step(opt)
        scaler.update()

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        one_step()
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / args.steps], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    bound = _nvlink_bound(opt.geom.padded, opt.local_numel(), ws)
    out = {"ms": round(ms, 4), "gparams_s": round(P / (ms / 1e3) / 1e9, 3), **bound,
           "frac_of_bound": round(bound["bound_ms"] / ms, 4),
           "note": "statistics + norm exchange + AdamW with the bf16 broadcast fused in (bulk "
                   "stores of staged chunks to legacy CUDA IPC mappings) + ordering all-reduce + "
                   "scaler update, per step; max over ranks"}
    out["parity"] = parity_check(opt, scaler, step_params, ws, rank, seed=1)
    opt.close()
    return out


def fused_broadcast_report(opt, P, ws, ms_per_step, adamw_ms):
    """With peer memory the update kernel stores every updated bf16 shard element into all ranks'
    parameter buffers, so the timed step already holds the whole all-gather; this reports its
    NVLink rate.  Each rank sends (and receives) 2 bytes x its shard x (N-1) peers."""
    sent = 2 * opt.local_numel() * (ws - 1)
    gbs = sent / (adamw_ms / 1e3) / 1e9
    return {"ms": None, "fused_into_update": True, "send_bytes_per_rank": int(sent),
            "gbs_per_rank": round(gbs, 1), "nvlink_peak_gbs": 770.0,
            "frac_of_nvlink": round(gbs / 770.0, 4),
            "full_step_ms": round(ms_per_step, 4),
            "full_step_gparams_s": round(P / (ms_per_step / 1e3) / 1e9, 3),
            "note": "AdamW kernel stores bf16 results to every peer's parameters over NVLink "
                    "(legacy CUDA IPC mappings, plain st.global); gbs_per_rank = peer bytes sent / "
                    "AdamW kernel time; full_step_* = the timed step itself"}


def time_allgather(args, opt, one_step, device, P, ws):
    """The bf16 parameter all-gather of ZeRO-1, timed on its own and after each update."""
    import torch.distributed as dist
    k = args.steps
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    dist.barrier()
    ev[0].record()
    for _ in range(k):
        opt.gather_params()
    ev[1].record()
    torch.cuda.synchronize()
    dist.barrier()
    ev[2].record()
    for _ in range(k):
        one_step()
        opt.gather_params()
    ev[3].record()
    torch.cuda.synchronize()
    t = torch.tensor([ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ag_ms, full_ms = (float(x) / k for x in t.tolist())
    recv = 2 * opt.geom.padded * (ws - 1) / ws  # bytes each rank receives per gather
    bound = _nvlink_bound(opt.geom.padded, opt.local_numel(), ws)
    return {"ms": round(ag_ms, 4), "recv_bytes_per_rank": int(recv),
            "full_step_bound_ms": bound["bound_ms"], "full_step_bound": bound["bound"],
            "full_step_frac_of_bound": round(bound["bound_ms"] / full_ms, 4),
            "gbs_per_rank": round(recv / (ag_ms / 1e3) / 1e9, 1),
            "nvlink_peak_gbs": 770.0,
            "frac_of_nvlink": round(recv / (ag_ms / 1e3) / 1e9 / 770.0, 4),
            "full_step_ms": round(full_ms, 4),
            "full_step_gparams_s": round(P / (full_ms / 1e3) / 1e9, 3),
            "note": "in-place NCCL all_gather_into_tensor of the bf16 shards; value above times "
                    "the sharded update (stats + norm-partial exchange + AdamW + scaler update), "
                    "full_step_* times update + this gather back to back"}


def run_e2e(args, opt, scaler, step_params, params, grads, device, P, pg):
    """Same metric through the public API with host-resident inputs: every step's gradients are
    copied from pinned host memory, and every step's result (norm, found_inf, scale) is read back
    to the host before the next step starts.

    The host-to-device copy of step k+1 runs on a copy stream into a device staging buffer while
    step k computes (one staging buffer: the copy waits until the previous staging contents were
    moved into the gradient tensors).  The first step's copy happens before the timed region and
    one extra copy (for the step after the last) inside it, so the region holds exactly one copy
    per timed step."""
    from minigpt_train_infra_b200 import clip_grad_norm_
    steps = max(2, min(args.steps, args.e2e_steps))
    if pg is not None:
        # under ZeRO-1 a rank's step consumes only the gradients of its own shard
        grads = [opt.flat_grad[opt.geom.lo:opt.geom.hi]]
    host = [torch.empty(g.shape, dtype=g.dtype, pin_memory=True) for g in grads]
    for h, g in zip(host, grads):
        h.copy_(g)
    staging = [torch.empty_like(g) for g in grads]
    res_host = torch.empty(3, dtype=torch.float32, pin_memory=True)
    h2d = sum(g.numel() * g.element_size() for g in grads)
    if pg is not None:
        h2d *= torch.distributed.get_world_size()
    main = torch.cuda.current_stream(device)
    copy = torch.cuda.Stream(device)
    staged = torch.cuda.Event()
    free = torch.cuda.Event()

    def h2d_async():
        copy.wait_event(free)
        with torch.cuda.stream(copy):
            for st, h in zip(staging, host):
                st.copy_(h, non_blocking=True)
        staged.record(copy)

    def step():
        main.wait_event(staged)
        for g, st in zip(grads, staging):
            g.copy_(st, non_blocking=True)
        free.record(main)
        h2d_async()  # the next step's inputs, overlapping this step's kernels
        scaler.unscale_(opt)
        norm = clip_grad_norm_(step_params, CLIP)
        found = next(iter(scaler._per_optimizer_states[id(opt)]["found_inf_per_device"].values()))
        scaler.step(opt)
        res = torch.stack([norm.float(), found.float(), scaler._scale.float()])
        scaler.update()
        res_host.copy_(res, non_blocking=True)
        main.synchronize()

    free.record(main)
    h2d_async()
    step()
    if pg is not None:
        torch.distributed.barrier()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    for _ in range(steps):
        step()
    main.wait_event(staged)  # the extra copy issued by the last step is inside the region too
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1)
    if pg is not None:
        t = torch.tensor([ms], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    del host, staging
    return {"value": round(P * steps / (ms / 1e3) / 1e9, 3), "unit": "Gparams/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": 12 * (torch.distributed.get_world_size() if pg else 1),
            "steps": steps, "ms_per_step": round(ms / steps, 3),
            "pipelining": "step k+1's host-to-device copy overlaps step k's kernels"}


def run_torch_cuda(args) -> None:
    """torch's own CUDA path for the same workload, as the reference runs it on a GPU
    (train.py:359-370 with fused=True: fp32 params and grads, AdamW(fused=True), GradScaler,
    clip_grad_norm_).  An extra measurement for comparison, not the reference arm."""
    ws, rank, local = dist_env()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    name = args.workload
    shape_list = workloads.shapes(name)
    P = workloads.n_params(name)
    scale = SCALES.get(name, 2.0 ** 16)
    std = GRAD_STD.get(name, 1e-3)
    params = [torch.nn.Parameter(torch.empty(s, device=device)) for _, s, _ in shape_list]
    for i, p in enumerate(params):
        fill_seeded(p.data, 1000 + i, 0.02)
        g = torch.empty_like(p)
        fill_seeded(g, 7000 + i, std * scale)
        p.grad = g
    groups = [{"params": [p for p, (_, _, g) in zip(params, shape_list) if g == 0],
               "weight_decay": WD},
              {"params": [p for p, (_, _, g) in zip(params, shape_list) if g == 1],
               "weight_decay": 0.0}]
    groups = [g for g in groups if g["params"]]
    opt = torch.optim.AdamW(groups, lr=LR, betas=BETAS, eps=EPS, fused=True)
    scaler = torch.amp.GradScaler("cuda", init_scale=scale)
    scaler.scale(torch.ones((), device=device))

    def one_step():
        scaler.unscale_(opt)
        torch.nn.utils.clip_grad_norm_(params, CLIP)
        scaler.step(opt)
        scaler.update()

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        one_step()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    emit_result({"metric": METRIC, "impl": "torch-cuda", "value": round(P / (ms / 1e3) / 1e9, 3),
                 "unit": "Gparams/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                 "ms_per_step": round(ms, 4), "higher_is_better": True, "dtype": "f32",
                 "config": {"workload": name, "params": P,
                            "path": f"torch {torch.__version__} AdamW(fused=True) + GradScaler + "
                                    "clip_grad_norm_, fp32 params and grads"}})


def run_dp_step(args) -> None:
    """The complete data-parallel ZeRO-1 step, N ranks with different local gradients:
    gradient reduce-scatter -> statistics -> norm exchange -> AdamW -> bf16 parameter gather,
    either with NCCL collectives around the kernels (``--dp-step nccl``) or with the fused
    peer-memory kernels (``--dp-step fused``).  Prints its own JSON line (the default run is
    run_ours)."""
    import datetime
    import torch.distributed as dist
    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    from minigpt_train_infra_b200 import GradScaler, ZeroAdamW, clip_grad_norm_
    name = args.workload
    shape_list = workloads.shapes(name)
    P = workloads.n_params(name)
    scale = SCALES.get(name, 2.0 ** 16)
    std = GRAD_STD.get(name, 1e-3)
    params, gids = make_model_params(shape_list, device)
    groups = [{"params": [p for p, g in zip(params, gids) if g == 0], "weight_decay": WD},
              {"params": [p for p, g in zip(params, gids) if g == 1], "weight_decay": 0.0}]
    groups = [g for g in groups if g["params"]]
    fused = args.dp_step == "fused"
    opt = ZeroAdamW(groups, lr=LR, betas=BETAS, eps=EPS, process_group=dist.group.WORLD,
                    reduce_grads=True, peer_memory=fused)
    fill_seeded(opt.master, 1 + 101 * rank, 0.02)
    fill_seeded(opt.exp_avg, 2 + 101 * rank, 1e-3)
    fill_seeded(opt.exp_avg_sq, 3 + 101 * rank, 1e-6, absval=True)
    opt.steps.fill_(999.0)
    with torch.no_grad():
        opt.owned_param_shard().copy_(opt.master)
    opt.gather_params()
    local_grads = torch.empty_like(opt.flat_grad)
    fill_seeded(local_grads, 7 + 1000 * rank, std * scale)  # this rank's own micro-batch grads
    scaler = GradScaler("cuda", init_scale=scale, growth_interval=2000, backoff_factor=0.5)
    scaler.scale(torch.ones((), device=device))
    step_params = opt.managed_params()

    def one_step():
        opt.flat_grad.copy_(local_grads)  # backward's output: fresh local grads every step
        scaler.unscale_(opt)
        clip_grad_norm_(step_params, CLIP)
        scaler.step(opt)
        scaler.update()

    def timed(fn, k):
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(k):
            fn()
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / k], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        one_step()
    step_ms = timed(one_step, args.steps)
    copy_ms = timed(lambda: opt.flat_grad.copy_(local_grads), args.steps)
    ms = step_ms - copy_ms
    # Every rank must receive the other ranks' gradients for its shard (reduce-scatter) and the
    # other ranks' updated bf16 shards (gather): 2 x 2 bytes x P x (N-1)/N over NVLink, whoever
    # moves them; at the measured 770 GB/s per direction that bounds the step from below.
    recv = 4 * P * (ws - 1) / ws
    nvlink = {"bound": "nvlink", "recv_bytes_per_rank": int(recv),
              "achieved": round(recv / (ms / 1e3) / 1e9, 1), "peak": 770.0, "unit": "GB/s",
              "frac": round(recv / (ms / 1e3) / 1e9 / 770.0, 4),
              "peak_kind": "measured peer copy bandwidth per direction"}
    if rank == 0:
        emit_result({
            "metric": "ZeRO-1 data-parallel step incl. grad reduce-scatter and param gather",
            "impl": f"dp-{args.dp_step}", "value": round(P / (ms / 1e3) / 1e9, 3),
            "unit": "Gparams/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "dtype": "f32",
            "config": {"workload": name, "params": P,
                       "collectives": ("fused peer-memory kernels (reduce-scatter+stats, "
                                       "AdamW+bf16 broadcast)") if fused else
                       "NCCL reduce_scatter_tensor + all_gather_into_tensor around the kernels",
                       "note": "the timed loop copies fresh local grads each step (a stand-in "
                               "for backward); that copy is timed separately and subtracted",
                       "grad_copy_ms": round(copy_ms, 4)},
            "roofline": nvlink})
    opt.close()
    dist.barrier()
    dist.destroy_process_group()


def run_reference(args) -> None:
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    name = args.workload
    shape_list = workloads.shapes(name)
    scale = SCALES.get(name, 2.0 ** 16)
    std = GRAD_STD.get(name, 1e-3)
    steps = max(1, min(args.steps, 5))
    warmup = max(1, min(args.warmup, 2))
    cpu = run_cpu_baseline(shape_list, scale, std, steps=steps, warmup=warmup)
    line = {
        "metric": METRIC, "impl": "reference", "value": round(cpu["value"], 4),
        "unit": "Gparams/s", "n_gpus": ws, "steps": steps, "warmup": warmup,
        "ms_per_step": round(cpu["seconds_per_step"] * 1e3, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": f"{name}: bounded sample (see cpu_baseline.sample)",
                   "parallelism": "host CPU, rank 0 only"},
        "cpu_baseline": {**{k: cpu[k] for k in ("unit", "cores", "kind", "sample")},
                         "value": round(cpu["value"], 4)},
        "e2e": {"value": round(cpu["value"], 4), "unit": "Gparams/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    emit_result(line)


_RESULT_FD = None


def emit_result(line: dict) -> None:
    """Write the one result line to the real stdout (everything else goes to stderr)."""
    data = (json.dumps(line) + "\n").encode()
    fd = _RESULT_FD if _RESULT_FD is not None else 1
    os.write(fd, data)


def _stdout_to_stderr() -> None:
    """Libraries (NCCL's version banner, for one) print to stdout; keep stdout for the result
    line only by pointing file descriptor 1 at stderr and remembering the original."""
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


def main() -> None:
    _stdout_to_stderr()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1,
                    help="GPUs of this node (N>1 under torchrun: one rank per GPU, ZeRO-1)")
    ap.add_argument("--steps", type=int, default=10, help="timed steps")
    ap.add_argument("--warmup", type=int, default=3, help="untimed steps before them")
    ap.add_argument("--workload", default="qwen3_8b", choices=sorted(workloads.WORKLOADS),
                    help="parameter-shape list (default: the Qwen3-8B-shaped configuration)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "torch-cuda"],
                    help="ours: this package; reference: the reference's CPU chain on the host "
                         "cores (rank 0); torch-cuda: torch's own fused CUDA AdamW path")
    ap.add_argument("--e2e-steps", type=int, default=3,
                    help="steps of the end-to-end measurement with host-resident gradients")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true",
                    help="skip the CPU baseline leg (N=1)")
    ap.add_argument("--peer-memory", action="store_true",
                    help="N>1: store the updated bf16 shards into every rank's parameters from "
                         "the update kernel (fused all-gather over NVLink peer memory)")
    ap.add_argument("--no-peer-leg", action="store_true",
                    help="N>1: skip the second leg that times and checks the step with the bf16 "
                         "all-gather fused into the update over peer memory")
    ap.add_argument("--graph", action="store_true",
                    help="N=1: capture the step in a CUDA graph and time its replays")
    ap.add_argument("--dp-step", choices=["nccl", "fused"], default=None,
                    help="time the full data-parallel ZeRO-1 step instead (N>1, torchrun)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        log("note: fewer than 3 warm-up steps")
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "torch-cuda":
        run_torch_cuda(args)
    elif args.dp_step is not None:
        run_dp_step(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
