"""Explicit-state checkers of the two protocol models, generalized to N ranks.

The TLA+ sources are in tla/ (GroupFallbackN.tla, HostLaneReuseN.tla, with
good and deliberately broken configurations). TLC needs a JRE, which this
image does not have; these checkers enumerate the same state spaces
breadth-first with the same initial states, actions and invariants, and the
tests also replay random traces of the real C++ group state machine against
GroupFallback's transitions.

GroupFallback (one outer group): calls arrive one at a time (a rank's
collective or an unsupported operation) and End closes the group. Receive
buffers a rank call while not passthrough and fewer than N are pending;
otherwise (passthrough, an unsupported op, or N already pending) the pending
prefix and the call are forwarded in order and the group goes passthrough.
End runs the clique when nothing went passthrough and the pending calls are
exactly one call per rank; otherwise it forwards the pending calls.
Invariants: OrderedPrefix, PendingBound, BufferedOrder, Complete. The broken
variant forwards an unsupported op without flushing the pending prefix.

HostLaneReuse (one host-staged range): piece k uses lane (k-1) % Lanes.
Produce(k, q): source rank q's D2H of piece k into its bounce buffer; in
order per (q, lane) stream, and (unless SkipReuseWait) only after every H2D
of piece k-Lanes finished (LaneFree). Fold(k): after all sources produced
piece k, the host writes the lane's output buffer (reads each bounce).
Consume(k, r): destination r's H2D of piece k, after Fold(k), in order per
(r, lane) stream. Invariants: CorrectOutputs (every consumed piece reads the
value folded from piece k's own inputs) and ProducedBeforeConsumed. The
broken variant skips the LaneFree wait.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass


@dataclass
class Result:
    ok: bool
    states: int
    violation: str | None = None
    trace: list | None = None


def _bfs(init, actions, invariants, max_states=2_000_000):
    seen = {init: None}
    q = deque([init])
    while q:
        s = q.popleft()
        for name, inv in invariants:
            if not inv(s):
                trace = []
                cur = s
                while cur is not None:
                    trace.append(cur)
                    cur = seen[cur]
                return Result(False, len(seen), name, list(reversed(trace)))
        for t in actions(s):
            if t not in seen:
                seen[t] = s
                if len(seen) > max_states:
                    raise RuntimeError("state space too large")
                q.append(t)
    return Result(True, len(seen))


# --------------------------------------------------------------------------
# GroupFallback
# --------------------------------------------------------------------------

def group_fallback_ops(nranks: int) -> tuple:
    return tuple(f"rank{i}" for i in range(nranks)) + ("unsupported",)


def group_receive(state, op, nranks, skip_unsupported_flush=False):
    seen, fwd, pend, pt, uns, ended, custom = state
    seen = seen + (op,)
    uns = uns or op == "unsupported"
    if op == "unsupported" and skip_unsupported_flush:
        return (seen, fwd + (op,), pend, pt, uns, ended, custom)
    if pt or op == "unsupported" or len(pend) == nranks:
        return (seen, fwd + pend + (op,), (), True, uns, ended, custom)
    return (seen, fwd, pend + (op,), pt, uns, ended, custom)


def is_clique(calls, nranks) -> bool:
    return len(calls) == nranks and set(calls) == {f"rank{i}" for i in range(nranks)}


def group_end(state, nranks):
    seen, fwd, pend, pt, uns, ended, custom = state
    run = (not pt) and is_clique(pend, nranks)
    return (seen, fwd if run else fwd + pend, (), pt, uns, True, run)


def check_group_fallback(nranks=2, max_calls=5, skip_unsupported_flush=False) -> Result:
    ops = group_fallback_ops(nranks)
    init = ((), (), (), False, False, False, False)

    def actions(s):
        seen, _, _, _, _, ended, _ = s
        if ended:
            return
        if len(seen) < max_calls:
            for op in ops:
                yield group_receive(s, op, nranks, skip_unsupported_flush)
        yield group_end(s, nranks)

    def ordered_prefix(s):
        seen, fwd = s[0], s[1]
        return len(fwd) <= len(seen) and fwd == seen[:len(fwd)]

    def pending_bound(s):
        return len(s[2]) <= nranks

    def buffered_order(s):
        seen, fwd, pend, _, _, ended, _ = s
        return ended or fwd + pend == seen

    def complete(s):
        seen, fwd, _, _, uns, ended, custom = s
        if not ended:
            return True
        if custom:
            return is_clique(seen, nranks) and not uns and fwd == ()
        return fwd == seen

    invs = [("OrderedPrefix", ordered_prefix), ("PendingBound", pending_bound),
            ("BufferedOrder", buffered_order), ("Complete", complete)]
    if skip_unsupported_flush:
        invs = [("OrderedPrefix", ordered_prefix)]
    return _bfs(init, actions, invs)


# --------------------------------------------------------------------------
# HostLaneReuse (N sources folded on the host, M destinations)
# --------------------------------------------------------------------------

def check_host_lane_reuse(pieces=5, lanes=4, sources=1, dests=1, skip_reuse_wait=False,
                          fold=None) -> Result:
    """State: produced[k][q], folded[k], consumed[k][r], bounce[q][lane],
    out[lane], output[k][r]. Values are piece numbers (0 = empty)."""
    fold = sources > 1 if fold is None else fold
    K = pieces

    def lane(k):
        return (k - 1) % lanes

    init = (frozenset(), frozenset(), frozenset(),
            tuple(tuple(0 for _ in range(lanes)) for _ in range(sources)),
            tuple(0 for _ in range(lanes)), tuple(tuple(0 for _ in range(dests)) for _ in range(K)))

    def lane_free(consumed, k):
        # Every destination's H2D of piece k-lanes finished.
        return k <= lanes or all((k - lanes, r) in consumed for r in range(dests))

    def actions(s):
        produced, folded, consumed, bounce, out, output = s
        for k in range(1, K + 1):
            L = lane(k)
            for q in range(sources):
                if (k, q) in produced:
                    continue
                if k > lanes and (k - lanes, q) not in produced:
                    continue  # in-order D2H stream of (q, lane)
                if not skip_reuse_wait and not lane_free(consumed, k):
                    continue
                nb = tuple(tuple(k if (qq == q and ll == L) else bounce[qq][ll] for ll in range(lanes))
                           for qq in range(sources))
                yield (produced | {(k, q)}, folded, consumed, nb, out, output)
            if fold and k not in folded and all((k, q) in produced for q in range(sources)):
                if k > lanes and (k - lanes) not in folded:
                    continue  # in-order host stream of the lane
                # The fold reads every source's bounce; the result is the
                # piece number only if every bounce still holds piece k.
                v = k if all(bounce[q][L] == k for q in range(sources)) else -1
                nout = tuple(v if ll == L else out[ll] for ll in range(lanes))
                yield (produced, folded | {k}, consumed, bounce, nout, output)
            for r in range(dests):
                if (k, r) in consumed:
                    continue
                ready = (k in folded) if fold else all((k, q) in produced for q in range(sources))
                if not ready:
                    continue
                if k > lanes and (k - lanes, r) not in consumed:
                    continue  # in-order H2D stream of (r, lane)
                val = out[L] if fold else bounce[0][L]
                nout = tuple(tuple(val if (kk == k - 1 and rr == r) else output[kk][rr]
                                   for rr in range(dests)) for kk in range(K))
                yield (produced, folded, consumed | {(k, r)}, bounce, out, nout)

    def correct_outputs(s):
        consumed, output = s[2], s[5]
        return all(output[k - 1][r] == k for (k, r) in consumed)

    def produced_before_consumed(s):
        produced, consumed = s[0], s[2]
        return all(all((k, q) in produced for q in range(sources)) for (k, _) in consumed)

    return _bfs(init, actions, [("CorrectOutputs", correct_outputs),
                                ("ProducedBeforeConsumed", produced_before_consumed)])
