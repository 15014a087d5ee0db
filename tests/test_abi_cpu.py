"""The C-ABI library loads on a machine without a GPU, exports exactly the symbols of
``include/b200_optim.h``, and its host-only planner validates and chunks tensor tables."""

from __future__ import annotations

import re
from pathlib import Path

import numpy as np
import pytest

from minigpt_train_infra_b200 import _build, _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "b200_optim.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(b2o_[a-z0-9_]+)\s*\(", text))


def test_header_and_binding_agree():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.b2o_abi_version() == _lib.ABI_VERSION
    assert lib.b2o_status_string(0) == b"ok"


def test_built_for_sm100a_only():
    assert "arch=compute_100a,code=sm_100a" in " ".join(_build.ARCH)
    assert "--use_fast_math" not in _build.NVCC_FLAGS


def _table(entries):
    t = np.zeros(len(entries), dtype=_lib.TENSOR_DTYPE)
    for i, e in enumerate(entries):
        t[i] = e
    return t


def _plan(t, chunk_elems=64, n_groups=2, n_slots=None, grad_dtype=_lib.BF16):
    lib = _lib.load()
    n_slots = len(t) if n_slots is None else n_slots
    n = np.zeros(1, np.int64)
    st = lib.b2o_plan_chunks(_lib.ptr(t), len(t), n_groups, n_slots, chunk_elems, grad_dtype,
                             None, 0, _lib.ptr(n))
    if st != 0:
        return st, None
    c = np.zeros(int(n[0]), dtype=_lib.CHUNK_DTYPE)
    st = lib.b2o_plan_chunks(_lib.ptr(t), len(t), n_groups, n_slots, chunk_elems, grad_dtype,
                             _lib.ptr(c) if c.size else None, c.size, _lib.ptr(n))
    return st, c


A = 0x10000  # a 16-byte-aligned fake device address


def test_planner_chunks_cover_every_element_once():
    sizes = [0, 1, 7, 64, 65, 1000, 4096]
    t = _table([(A, A, A, A, A, n, i % 2, i, 0, 0, 0, 0) for i, n in enumerate(sizes)])
    st, c = _plan(t, chunk_elems=64)
    assert st == 0
    for i, n in enumerate(sizes):
        mine = c[c["tensor"] == i]
        assert t["chunk_count"][i] == len(mine) == (n + 63) // 64
        if len(mine):
            assert t["chunk_begin"][i] == np.nonzero(c["tensor"] == i)[0][0]
        covered = np.zeros(n, bool)
        for b, e in zip(mine["begin"], mine["end"]):
            assert not covered[b:e].any()
            covered[b:e] = True
        assert covered.all()
    assert (t["flags"] & _lib.FLAG_VECTOR).all()


def test_planner_flags_misaligned_tensors_for_the_scalar_path():
    t = _table([(A + 2, A, A, A, A, 100, 0, 0, 0, 0, 0, 0),
                (A, A + 2, A, A, A, 100, 0, 1, 0, 0, 0, 0),
                (A, 0, A + 4, A, A, 100, 0, 2, 0, 0, 0, 0),
                (A, 0, A, A, A, 100, 0, 3, 0, 0, 0, 0)])
    st, _ = _plan(t)
    assert st == 0
    assert list(t["flags"] & _lib.FLAG_VECTOR) == [0, 0, 0, 1]


@pytest.mark.parametrize("bad", ["slot_twice", "slot_range", "group_range", "null", "neg"])
def test_planner_rejects_inconsistent_tables(bad):
    rows = [(A, A, A, A, A, 10, 0, 0, 0, 0, 0, 0), (A, A, A, A, A, 10, 1, 1, 0, 0, 0, 0)]
    if bad == "slot_twice":
        rows[1] = (A, A, A, A, A, 10, 1, 0, 0, 0, 0, 0)
    elif bad == "slot_range":
        rows[1] = (A, A, A, A, A, 10, 1, 5, 0, 0, 0, 0)
    elif bad == "group_range":
        rows[1] = (A, A, A, A, A, 10, 2, 1, 0, 0, 0, 0)
    elif bad == "null":
        rows[1] = (0, A, A, A, A, 10, 1, 1, 0, 0, 0, 0)
    elif bad == "neg":
        rows[1] = (A, A, A, A, A, -1, 1, 1, 0, 0, 0, 0)
    st, _ = _plan(_table(rows))
    assert st == -5  # B2O_ERR_TABLE


def test_planner_rejects_bad_arguments():
    t = _table([(A, A, A, A, A, 10, 0, 0, 0, 0, 0, 0)])
    assert _plan(t, chunk_elems=12)[0] == -1   # not a multiple of 8
    assert _plan(t, n_groups=17)[0] == -1      # more than B2O_MAX_GROUPS
    assert _plan(t, grad_dtype=7)[0] == -1
    lib = _lib.load()
    n = np.zeros(1, np.int64)
    c = np.zeros(1, dtype=_lib.CHUNK_DTYPE)
    t2 = _table([(A, A, A, A, A, 1000, 0, 0, 0, 0, 0, 0)])
    assert lib.b2o_plan_chunks(_lib.ptr(t2), 1, 1, 1, 64, 0, _lib.ptr(c), 1, _lib.ptr(n)) == -2


def test_workspace_size_formula():
    lib = _lib.load()
    assert lib.b2o_workspace_bytes(10, 3) == 64 + 8 * 10 + 8 * 4
    assert lib.b2o_workspace_bytes(-1, 3) == 0


def test_launching_entry_points_reject_bad_arguments_without_a_gpu():
    """Argument checks run before any CUDA call, so they are testable on a CPU-only host."""
    lib = _lib.load()
    g = np.zeros(1, dtype=_lib.GROUP_DTYPE)
    assert lib.b2o_grad_stats(None, 0, None, 0, 0, 0, None, None, None, 0, None, None, None) == -1
    assert lib.b2o_adamw_step(None, 0, None, 0, _lib.ptr(g), 1, 0, 0, None, None, None, None,
                              0.0, None, None, None) == -1
    assert lib.b2o_finalize_norm(None, 1, 1, None, None, None) == -1
    assert lib.b2o_scaler_update(None, None, None, 2.0, 0.5, 2000, None) == -1
    assert lib.b2o_adamw_step_dev(None, 0, None, 0, None, 1, 0, 0, None, None, None, None, 0.0,
                                  None, None) == -1
    peers = _lib.ptr_array([A, A])
    t = np.zeros(1, dtype=_lib.TENSOR_DTYPE)
    ws = np.zeros(64, dtype=np.uint8)
    # more ranks than one node holds, or a null peer, is rejected before any CUDA call
    assert lib.b2o_reduce_scatter_stats(_lib.ptr_array([A] * 9), 9, A, 1.0, _lib.ptr(t), 1, None,
                                        0, 1, None, _lib.ptr(ws), None, None) == -1
    assert lib.b2o_reduce_scatter_stats(_lib.ptr_array([A, 0]), 2, A, 1.0, _lib.ptr(t), 1, None,
                                        0, 1, None, _lib.ptr(ws), None, None) == -1
    assert lib.b2o_adamw_step_bcast(_lib.ptr(t), 1, None, 0, _lib.ptr(g), 1, 0, None, None, None,
                                    None, 0.0, peers, 2, 2, A, _lib.ptr(ws), None) == -1
    for fn in ("b2o_peer_free", "b2o_peer_close"):
        assert getattr(lib, fn)(None) == -1
    assert lib.b2o_peer_alloc(0, None) == -1
    assert lib.b2o_peer_export(None, None) == -1
    assert lib.b2o_peer_import(None, None) == -1


@pytest.mark.parametrize("seed", range(8))
def test_planner_random_tables(seed):
    """Random tables: every element of every tensor is in exactly one chunk of its own tensor,
    chunks are contiguous per tensor and in table order, no chunk is longer than chunk_elems,
    and the vector flag is set exactly when every non-null pointer is 16-byte aligned."""
    rng = np.random.default_rng(seed)
    n = int(rng.integers(1, 40))
    chunk = int(8 * rng.integers(1, 64))
    rows, aligned = [], []
    for i in range(n):
        numel = int(rng.choice([0, 1, 7, 8, 9, int(rng.integers(1, 5000))]))
        offs = [int(rng.choice([0, 0, 0, 2, 4, 8])) for _ in range(5)]
        fp32_param = bool(rng.integers(0, 2))
        ptrs = [A + 0x100000 * (i + 1) + o for o in offs]
        if fp32_param:
            ptrs[1] = 0
        rows.append((*ptrs, numel, int(rng.integers(0, 3)), i, 0, 0, 0, 0))
        aligned.append(all(p % 16 == 0 for p in ptrs if p))
    t = _table(rows)
    perm = rng.permutation(n)  # slots need not follow table order
    t["slot"] = perm
    st, c = _plan(t, chunk_elems=chunk, n_groups=3, n_slots=n)
    assert st == 0
    pos = 0
    for i in range(n):
        cnt = int(t["chunk_count"][i])
        assert int(t["chunk_begin"][i]) == pos
        mine = c[pos:pos + cnt]
        assert (mine["tensor"] == i).all()
        if cnt:
            assert mine["begin"][0] == 0 and mine["end"][-1] == rows[i][5]
            assert (mine["end"][:-1] == mine["begin"][1:]).all()
            assert ((mine["end"] - mine["begin"]) <= chunk).all()
            assert ((mine["end"] - mine["begin"]) > 0).all()
        else:
            assert rows[i][5] == 0
        assert bool(t["flags"][i] & _lib.FLAG_VECTOR) == aligned[i]
        pos += cnt
    assert pos == len(c)
