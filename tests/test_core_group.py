"""The real C++ group state machine, driven with a fake libnccl, checked
against the GroupFallback model: scripted cases plus random traces whose
every step is compared with the model's transition."""
import random

import pytest

from scc26_nccl_shim_b200 import _core as c
from scc26_nccl_shim_b200.models import tla_models as m


def run(script, n=2, result=0):
    return c.group_script(script, n, result)


def events(lines):
    """(forwarded ids, custom id sets, real starts, real ends, return codes)"""
    fwd, custom, rs, re_, rcs = [], [], 0, 0, []
    for l in lines:
        t = l.split()
        if t[0] == "F":
            fwd.append(int(t[1]))
        elif t[0] == "C":
            custom.append([int(x) for x in t[1:]])
        elif t[0] == "RS":
            rs += 1
        elif t[0] == "RE":
            re_ += 1
        elif t[0] == "R":
            rcs.append(int(t[1]))
    return fwd, custom, rs, re_, rcs


def test_exact_pair_runs_custom():
    fwd, custom, rs, re_, rcs = events(run("S A0 A1 E"))
    assert custom == [[1, 2]] and fwd == [] and rs == 1 and re_ == 1 and set(rcs) == {0}


def test_exact_clique_of_four():
    fwd, custom, *_ = events(run("S A2 A0 A3 A1 E", n=4))
    assert custom == [[1, 2, 3, 4]] and fwd == []


def test_unsupported_op_flushes_prefix_in_order():
    fwd, custom, *_ = events(run("S A0 U A1 E"))
    assert custom == [] and fwd == [1, 2]


def test_unsupported_first():
    fwd, custom, *_ = events(run("S U A0 A1 E"))
    assert custom == [] and fwd == [1, 2]


def test_extra_call_flushes():
    fwd, custom, *_ = events(run("S A0 A1 A0 E"))
    assert custom == [] and fwd == [1, 2, 3]


def test_mixed_kinds_flush():
    fwd, custom, *_ = events(run("S A0 G1 E"))
    assert custom == [] and fwd == [1, 2]


def test_gate_failure_flushes():
    fwd, custom, *_ = events(run("S A0 B1 E"))  # B: misaligned -> fails the call gate
    assert custom == [] and fwd == [1, 2]


def test_duplicate_rank_replays_at_end():
    fwd, custom, *_ = events(run("S A0 A0 E"))
    assert custom == [] and fwd == [1, 2]


def test_nested_group_goes_passthrough():
    lines = run("S A0 S A1 E E")
    fwd, custom, rs, re_, _ = events(lines)
    assert custom == [] and fwd == [1, 2] and rs == 2 and re_ == 2


def test_runner_fallback_replays_in_order():
    fwd, custom, *_ = events(run("S A1 A0 E", result=1))
    assert custom == [] and fwd == [1, 2]


def test_runner_error_returns_unhandled_cuda_error_without_replay():
    fwd, custom, rs, re_, rcs = events(run("S A0 A1 E", result=2))
    assert fwd == [] and custom == [] and rcs[-1] == 1 and re_ == 1


def test_ungrouped_calls_forward():
    fwd, custom, rs, re_, _ = events(run("A0 A1"))
    assert fwd == [1, 2] and rs == 0 and re_ == 0


def test_one_rank_clique_runs_ungrouped():
    fwd, custom, *_ = events(run("A0", n=1))
    assert custom == [[1]] and fwd == []


def test_simulate_end_flushes_and_pops():
    fwd, custom, rs, re_, _ = events(run("S A0 I A1 A0", n=2))
    assert fwd == [1, 2, 3] and custom == []


def test_real_group_calls_balanced():
    for script in ["S A0 A1 E", "S A0 U A1 E", "S S E E", "S A0 S U E A1 E"]:
        _, _, rs, re_, _ = events(run(script))
        assert rs == re_, script


def model_replay(ops, n):
    """Expected forwarded ids and custom flag from the GroupFallback model."""
    state = ((), (), (), False, False, False, False)
    ids = {}
    next_id = 1
    for op in ops:
        if op != "unsupported":
            ids[len(state[0])] = next_id
            next_id += 1
        state = m.group_receive(state, op, n)
    state = m.group_end(state, n)
    seen, fwd, _, _, _, _, custom = state
    # Map forwarded model calls back to call ids (unsupported ops have none).
    pos = {i: ids.get(i) for i in range(len(seen))}
    fwd_ids = []
    k = 0
    for i, op in enumerate(seen):
        if k < len(fwd) and fwd[k] == op:
            if pos[i] is not None:
                fwd_ids.append(pos[i])
            k += 1
    return fwd_ids, custom


@pytest.mark.parametrize("n", [2, 3, 4])
def test_random_traces_match_model(n):
    rng = random.Random(n)
    ops_names = m.group_fallback_ops(n)
    for _ in range(400):
        k = rng.randrange(0, n + 3)
        ops = [rng.choice(ops_names) for _ in range(k)]
        script = "S " + " ".join("U" if o == "unsupported" else f"A{o[4:]}" for o in ops) + " E"
        fwd, custom, rs, re_, _ = events(run(script, n=n))
        want_fwd, want_custom = model_replay(ops, n)
        assert bool(custom) == want_custom, (script, custom)
        assert fwd == want_fwd, (script, fwd, want_fwd)
        # OrderedPrefix on the real trace: forwarded ids increase
        assert fwd == sorted(fwd)
        assert rs == 1 and re_ == 1
