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


def test_tla_sources_present():
    for f in ["GroupFallbackN.tla", "HostLaneReuseN.tla", "GroupFallbackN.cfg",
              "GroupFallbackN-broken.cfg", "HostLaneReuseN.cfg", "HostLaneReuseN-broken.cfg"]:
        assert os.path.exists(os.path.join(REPO, "tla", f)), f
