"""The GroupFallback and HostLaneReuse models (generalized to N ranks):
good configurations satisfy their invariants, broken ones must violate them
(mutation checks of the models themselves)."""
import os

import pytest

from scc26_nccl_shim_b200.models import tla_models as m

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("n,calls", [(2, 5), (2, 6), (3, 6), (4, 6)])
def test_group_fallback_holds(n, calls):
    r = m.check_group_fallback(nranks=n, max_calls=calls)
    assert r.ok, (r.violation, r.trace)


@pytest.mark.parametrize("n", [2, 3])
def test_group_fallback_broken_violates_ordered_prefix(n):
    r = m.check_group_fallback(nranks=n, max_calls=5, skip_unsupported_flush=True)
    assert not r.ok and r.violation == "OrderedPrefix"


@pytest.mark.parametrize("pieces,lanes", [(5, 4), (9, 4), (13, 4), (7, 2)])
def test_host_lane_reuse_copy_holds(pieces, lanes):
    assert m.check_host_lane_reuse(pieces=pieces, lanes=lanes).ok


@pytest.mark.parametrize("pieces,lanes", [(5, 4), (9, 4), (7, 2)])
def test_host_lane_reuse_copy_broken(pieces, lanes):
    r = m.check_host_lane_reuse(pieces=pieces, lanes=lanes, skip_reuse_wait=True)
    assert not r.ok and r.violation == "CorrectOutputs"


@pytest.mark.parametrize("sources,dests", [(2, 2), (3, 3), (1, 3)])
def test_host_lane_reuse_fold_holds(sources, dests):
    assert m.check_host_lane_reuse(pieces=6, lanes=2, sources=sources, dests=dests).ok


@pytest.mark.parametrize("sources,dests", [(2, 2), (1, 3)])
def test_host_lane_reuse_fold_broken(sources, dests):
    r = m.check_host_lane_reuse(pieces=6, lanes=2, sources=sources, dests=dests,
                                skip_reuse_wait=True)
    assert not r.ok


@pytest.mark.parametrize("n,rounds,depth", [(2, 4, 2), (3, 4, 2), (3, 5, 1), (4, 3, 2)])
def test_push_reduce_holds(n, rounds, depth):
    """The push-reduce engine's progress words: no owner reads a scratch slot
    that a sender already refilled, and no reachable deadlock."""
    r = m.check_push_reduce(nranks=n, rounds=rounds, depth=depth)
    assert r.ok, (r.violation, r.trace)


@pytest.mark.parametrize("n", [2, 3])
def test_push_reduce_broken_reads_stale(n):
    r = m.check_push_reduce(nranks=n, rounds=4, depth=2, skip_consumed_wait=True)
    assert not r.ok and r.violation == "NoStaleRead"


@pytest.mark.parametrize("n,rounds,bufs,in_first", [(2, 4, 3, True), (2, 6, 3, True), (3, 4, 3, True),
                                                     (2, 4, 3, False), (3, 4, 3, False), (3, 4, 2, False)])
def test_nvls_allreduce_holds(n, rounds, bufs, in_first):
    """The NVLS AllReduce's copier/mover progress words with three round
    buffers (the kernel's), in the kernel's order (copy-out of round s-2
    before copy-in of round s) and in the swapped order. The kernel's order
    is also safe with two buffers (A(s) reuses a buffer only after every
    rank's B(s-2), which the wait before C(s-2) already needs)."""
    r = m.check_nvls_allreduce(nranks=n, rounds=rounds, bufs=bufs, in_first=in_first)
    assert r.ok, (r.violation, r.trace)


@pytest.mark.parametrize("n,rounds", [(2, 4), (3, 3)])
def test_nvls_allreduce_ahead_with_a_buffer_per_round(n, rounds):
    """Every copy-in first, then the copy-outs: safe with a buffer per
    round, and refuted when the buffers are fewer than the rounds."""
    r = m.check_nvls_allreduce(nranks=n, rounds=rounds, bufs=rounds, ahead=True)
    assert r.ok, (r.violation, r.trace)
    r = m.check_nvls_allreduce(nranks=n, rounds=rounds, bufs=rounds - 1, ahead=True)
    assert not r.ok and r.violation == "RoundsInOrder"


@pytest.mark.parametrize("n", [2, 3])
def test_nvls_allreduce_copy_in_first_needs_three_buffers(n):
    """Copying round s in before round s-2 is out overwrites round s-2's
    reduced data when there are only two buffers."""
    r = m.check_nvls_allreduce(nranks=n, rounds=4, bufs=2, in_first=True)
    assert not r.ok and r.violation == "RoundsInOrder"


@pytest.mark.parametrize("n", [2, 3])
def test_nvls_allreduce_broken_mover_waits_own_copier_only(n):
    r = m.check_nvls_allreduce(nranks=n, rounds=4, mover_waits_all=False)
    assert not r.ok and r.violation == "RoundsInOrder"


@pytest.mark.parametrize("n,steps", [(2, 3), (3, 3), (4, 3), (5, 2)])
def test_broadcast_chain_holds(n, steps):
    """The push chain's progress words: a rank forwards only pieces it has
    received, every output ends with every piece, no deadlock."""
    r = m.check_broadcast_chain(nranks=n, steps=steps)
    assert r.ok, (r.violation, r.trace)


def test_broadcast_chain_broken_forwards_early():
    r = m.check_broadcast_chain(nranks=3, steps=2, skip_wait=True)
    assert not r.ok and r.violation == "ForwardedArrived"


@pytest.mark.parametrize("n,calls,two", [(2, 3, False), (2, 3, True), (3, 3, True), (3, 2, False)])
def test_oneshot_barrier_holds(n, calls, two):
    """The low-latency engine's arrive/depart barriers: every rank reads
    every input of the current call, and every output slice a rank consumes
    holds the previous call, across consecutive calls, one-shot and
    two-shot alike; no deadlock."""
    r = m.check_oneshot_barrier(nranks=n, calls=calls, two=two)
    assert r.ok, (r.violation, r.trace)


@pytest.mark.parametrize("two", [False, True])
def test_oneshot_barrier_broken_without_either_wait(two):
    for kw in ({"skip_arrive": True}, {"skip_depart": True}):
        r = m.check_oneshot_barrier(nranks=2, calls=2, two=two, **kw)
        assert not r.ok and r.violation == "CallsInStep", (kw, two)


def test_tla_sources_present():
    for f in ["GroupFallbackN.tla", "HostLaneReuseN.tla", "GroupFallbackN.cfg",
              "GroupFallbackN-broken.cfg", "HostLaneReuseN.cfg", "HostLaneReuseN-broken.cfg",
              "PushReduceN.tla", "PushReduceN.cfg", "PushReduceN-broken.cfg",
              "NvlsAllReduceN.tla", "NvlsAllReduceN.cfg", "NvlsAllReduceN-broken.cfg",
              "BroadcastChainN.tla", "BroadcastChainN.cfg", "BroadcastChainN-broken.cfg",
              "OneShotBarrierN.tla", "OneShotBarrierN.cfg", "OneShotBarrierN-broken.cfg"]:
        assert os.path.exists(os.path.join(REPO, "tla", f)), f


def _cfgs():
    d = os.path.join(REPO, "tla")
    return sorted(f for f in os.listdir(d) if f.endswith(".cfg"))


def test_every_spec_has_a_good_and_a_broken_cfg():
    names = _cfgs()
    assert len(names) == 2 * len(m.SPECS), names
    for spec in m.SPECS:
        assert f"{spec}.cfg" in names and f"{spec}-broken.cfg" in names, spec


@pytest.mark.parametrize("cfg", _cfgs())
def test_committed_cfg_checked_with_its_own_constants(cfg):
    """Each committed configuration runs the checker with the constants it
    states; the constants, invariants and deadlock setting must agree with
    the spec file and the checker. Good configurations hold; broken ones
    are refuted on one of their own invariants (or a deadlock)."""
    c, r = m.check_cfg(os.path.join(REPO, "tla", cfg))
    if cfg.endswith("-broken.cfg"):
        assert not r.ok, cfg
        assert r.violation in c.invariants or (r.violation == "Deadlock" and c.check_deadlock)
    else:
        assert r.ok, (cfg, r.violation, r.trace)


def test_cfg_parser_rejects_drift(tmp_path):
    """A configuration whose constants drift from the spec is rejected."""
    src = open(os.path.join(REPO, "tla", "PushReduceN.cfg")).read()
    (tmp_path / "PushReduceN.tla").write_text(open(os.path.join(REPO, "tla", "PushReduceN.tla")).read())
    (tmp_path / "PushReduceN.cfg").write_text(src.replace("D = 2", "Depth = 2"))
    with pytest.raises(ValueError):
        m.check_cfg(str(tmp_path / "PushReduceN.cfg"))
    (tmp_path / "PushReduceN.cfg").write_text(src.replace("NoStaleRead", "NoSuchInvariant"))
    with pytest.raises(ValueError):
        m.check_cfg(str(tmp_path / "PushReduceN.cfg"))
