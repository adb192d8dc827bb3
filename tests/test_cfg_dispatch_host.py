"""Per-conditioning CFG dispatch on the CPU (dgx_monarch_b200/cfg_dispatch.py):
the fold decision, the cond groups and the length rule against the verdicts
the reference's adapters/cfg_dispatch.py gave on the same inputs
(tests/golden/, make_golden.py section (o)), and the dispatch itself -- each
rank runs only its group, the gathered list equals one GPU's list in cond
order, a rank with nothing to do still joins the gather -- with the ranks'
stacks gathered on the host."""
from __future__ import annotations

import importlib.util
import json
from pathlib import Path

import pytest
import torch

HERE = Path(__file__).resolve().parent
GOLDEN = json.loads((HERE / "golden" / "golden.json").read_text())
_spec = importlib.util.spec_from_file_location("make_golden", HERE / "golden" / "make_golden.py")
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)


@pytest.mark.parametrize("entry", GOLDEN["cond_fold"], ids=lambda e: str(e["case"])[:70])
def test_fold_decision_matches_the_reference(entry):
    from dgx_monarch_b200.cfg_dispatch import conds_fold

    slots = make_golden.build_cond_slots(entry["case"])
    assert conds_fold(slots, torch.zeros(2, 3), entry["case"].get("key")) is entry["folds"]


def test_cond_groups_and_length_rule_match_the_reference():
    from dgx_monarch_b200.cfg_dispatch import cond_group_bounds, cross_attn_pair_folds

    for e in GOLDEN["cond_groups"]:
        assert list(cond_group_bounds(e["count"], e["world"], e["rank"])) == e["bounds"]
    for e in GOLDEN["cross_attn_folds"]:
        assert cross_attn_pair_folds(e["a"], e["b"]) is e["folds"]


class _Toy:
    """A stand-in for stock _calc_cond_batch: zeros per slot, then each entry
    adds x * weight + its token count; it records which conds it ran."""

    def __init__(self):
        self.seen = []

    def __call__(self, conds, x_in, *rest):
        out = [torch.zeros_like(x_in) for _ in conds]
        for i, slot in enumerate(conds):
            for item in slot or []:
                tokens = item["model_conds"]["c_crossattn"].cond.shape[1]
                self.seen.append((i, tokens))
                out[i] = out[i] + x_in * item["weight"] + float(tokens)
        return out


def _slots(*tokens):
    slots = make_golden.build_cond_slots({"slots": [[{"tokens": t}] for t in tokens]})
    for n, slot in enumerate(slots):
        slot[0]["weight"] = float(n + 2)
    return slots


def _run_all_ranks(conds, world):
    """Every rank's dispatch; the gather completed from all ranks' stacks."""
    from dgx_monarch_b200.cfg_dispatch import CondDispatch

    x = torch.arange(6.0).reshape(2, 3)
    stacks, seen = [], []
    for rank in range(world):
        sent = {}

        def gather(local, sent=sent):
            sent["local"] = local
            return torch.cat([local] * world)

        toy = _Toy()
        CondDispatch(world=world, rank=rank, gather=gather)(toy, conds, x)
        stacks.append(sent.get("local"))
        seen.append(toy.seen)
    full = torch.cat(stacks) if all(s is not None for s in stacks) else None
    outs = [CondDispatch(world=world, rank=r, gather=lambda local: full)(_Toy(), conds, x)
            for r in range(world)]
    return outs, stacks, seen, _Toy()(conds, x)


def test_two_conds_that_never_fold_run_one_per_rank():
    outs, stacks, seen, want = _run_all_ranks(_slots(7, 11), 2)
    assert seen == [[(0, 7)], [(1, 11)]]
    for out in outs:
        assert len(out) == 2 and all(torch.equal(a, b) for a, b in zip(out, want))


def test_three_conds_on_two_ranks_keep_the_order_and_pad():
    outs, stacks, seen, want = _run_all_ranks(_slots(7, 11, 13), 2)
    assert seen == [[(0, 7), (1, 11)], [(2, 13)]]
    assert stacks[0].shape[0] == 2 and stacks[1].shape[0] == 2
    assert torch.equal(stacks[1][1], torch.zeros_like(stacks[1][1]))
    for out in outs:
        assert len(out) == 3 and all(torch.equal(a, b) for a, b in zip(out, want))


def test_a_rank_with_nothing_to_do_joins_the_gather():
    outs, stacks, seen, want = _run_all_ranks(_slots(7, 11), 3)
    assert seen == [[(0, 7)], [(1, 11)], []]
    assert stacks[2].shape[0] == 1 and torch.equal(stacks[2][0], torch.zeros_like(stacks[2][0]))
    for out in outs:
        assert all(torch.equal(a, b) for a, b in zip(out, want))


def test_folding_or_single_conds_take_the_batch_path_without_a_gather():
    from dgx_monarch_b200.cfg_dispatch import CondDispatch

    def no_gather(local):
        raise AssertionError("no collective on the batch path")

    x = torch.arange(6.0).reshape(2, 3)
    for conds in (_slots(9, 9), [_slots(7)[0], None]):
        toy = _Toy()
        d = CondDispatch(world=2, rank=1, gather=no_gather)
        out = d(toy, conds, x)
        assert d.last_path == "slice"
        assert all(torch.equal(a, b) for a, b in zip(out, _Toy()(conds, x)))


def test_the_dispatch_flag_is_set_only_inside_the_rank_call():
    from dgx_monarch_b200.cfg_dispatch import CondDispatch, dispatch_in_progress

    inside = []

    def executor(conds, x):
        inside.append(dispatch_in_progress())
        return _Toy()(conds, x)

    x = torch.zeros(2, 3)
    CondDispatch(world=2, rank=0, gather=lambda local: torch.cat([local, local]))(executor, _slots(7, 11), x)
    assert inside == [True] and not dispatch_in_progress()
