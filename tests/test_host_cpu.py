"""Host-side logic that needs no GPU: parameter grouping, workload shape lists, argument checks."""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from minigpt_train_infra_b200 import build_adamw_param_groups, workloads
from minigpt_train_infra_b200.optim import validate_adamw_args

SHAPES = json.loads((Path(__file__).resolve().parent / "golden" / "param_shapes.json").read_text())


class _Named(torch.nn.Module):
    """A module whose named_parameters() reproduce a (name, shape) list in order."""

    def __init__(self, items):
        super().__init__()
        self._names = []
        for name, shape, _ in items:
            mod = self
            parts = name.split(".")
            for part in parts[:-1]:
                if not hasattr(mod, part):
                    mod.add_module(part, torch.nn.Module())
                mod = getattr(mod, part)
            mod.register_parameter(parts[-1], torch.nn.Parameter(torch.empty(shape, device="meta")))


@pytest.mark.parametrize("config", sorted(SHAPES))
def test_workload_shapes_match_reference_models(config):
    """workloads.py restates the reference models' parameter lists; the fixture holds the lists
    generated from the reference classes themselves (tests/golden/make_golden.py)."""
    mine = [[n, list(s), g] for n, s, g in workloads.shapes(config)]
    assert mine == SHAPES[config]


@pytest.mark.parametrize("config", ["minigpt_6l_384", "gpt2_124m"])
def test_param_groups_match_reference_grouping(config):
    model = _Named(SHAPES[config])
    groups = build_adamw_param_groups(model, 0.1)
    assert [g["group_name"] for g in groups] == ["decay", "no_decay"]
    assert [g["weight_decay"] for g in groups] == [0.1, 0.0]
    want = {n: g for n, _, g in SHAPES[config]}
    for gi, g in enumerate(groups):
        assert all(want[n] == gi for n in g["param_names"])
        assert len(g["params"]) == len(g["param_names"])
    assert sum(len(g["params"]) for g in groups) == len(SHAPES[config])


def test_param_groups_reject_duplicates_and_negative_decay():
    lin = torch.nn.Linear(3, 3)

    class Tied(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.a = lin
            self.b = torch.nn.Linear(3, 3)
            self.b.weight = lin.weight

    groups = build_adamw_param_groups(Tied(), 0.1)  # named_parameters() deduplicates ties
    assert sum(len(g["params"]) for g in groups) == 3
    with pytest.raises(ValueError):
        build_adamw_param_groups(lin, -1.0)


@pytest.mark.parametrize("bad", [
    dict(lr=-1.0), dict(eps=-1.0), dict(betas=(1.0, 0.9)), dict(betas=(0.9, -0.1)),
    dict(weight_decay=-0.1), dict(chunk_elems=12)])
def test_adamw_argument_checks(bad):
    args = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, amsgrad=False,
                maximize=False, differentiable=False, chunk_elems=None)
    args.update(bad)
    with pytest.raises(ValueError):
        validate_adamw_args(**args)


def test_unsupported_variants_raise():
    args = dict(lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, amsgrad=True,
                maximize=False, differentiable=False, chunk_elems=None)
    with pytest.raises(NotImplementedError):
        validate_adamw_args(**args)


def test_tracked_state_records_every_mutation():
    """``optimizer.state`` of the fused optimizers remembers any write from outside, so a
    loader's assignments are copied into the flat buffers at the next step."""
    import copy
    import pickle

    from minigpt_train_infra_b200.optim import _TrackedState
    st = _TrackedState()
    assert st.dirty
    key = object()
    mutations = [
        lambda s: s.__setitem__(key, {"step": 1}),
        lambda s: s.__delitem__(key),
        lambda s: s.clear(),
        lambda s: s.pop(key, None),
        lambda s: s.update({key: {}}),
        lambda s: s.setdefault(key, {}),
        lambda s: s[object()],            # defaultdict insertion of a missing key
        lambda s: s.popitem(),
    ]
    for mutate in mutations:
        st[key] = {}
        st.dirty = False
        mutate(st)
        assert st.dirty
    st.dirty = False
    _ = st.get(key), key in st, len(st), list(st.items())  # reads do not mark it
    assert not st.dirty
    # pickling and deep copies give torch's plain mapping back
    assert type(pickle.loads(pickle.dumps(_TrackedState({1: {"a": 2}})))) is dict
    assert copy.deepcopy(_TrackedState({1: {"a": 2}})) == {1: {"a": 2}}
