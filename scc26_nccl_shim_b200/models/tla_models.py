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

PushReduce (one block index of the push-reduce engine, exec/pushred.cu):
N ranks, R rounds, D scratch rounds per (sender, owner). Sender s, round j:
Write(s) stores its pieces into every owner's slot (s, j % D) once every
owner consumed round j - D (unless SkipConsumedWait), then Publish(s) sets
filled[q][s] = j + 1 for every owner. Owner q: Wait(q) until every sender's
filled reached j + 1, Read(q) reads the N - 1 slots (non-atomically with
respect to senders: a sender may write between Wait and Read), Consume(q)
sets consumed[s][q] = j + 1. Invariants: NoStaleRead (every slot an owner
reads holds the round it expects) and no deadlock (every reachable state
without a successor has all ranks past round R). The broken variant skips
the consumed wait and must read a slot that was already overwritten.

NvlsAllReduce (one block index of the NVLS AllReduce, exec/nvls.cu): each
rank has B round buffers of N slices. Copier of rank r, step s: if s >= 2,
wait until every rank's mover published s - 1 (B(s-2) done everywhere),
then C(s-2) reads its own buffer (s-2) % B, all slices; if s < R, A(s)
writes its input round s into buffer s % B (all slices); publish s + 1.
Mover of rank r, step s < R: wait until every rank's copier published s + 1
(A(s) done everywhere), ReadB reads slice r of buffer s % B on every rank
(the switch's ld_reduce), WriteB writes the reduced slice r into every
rank's buffer s % B (the multicast store), publish s + 1. Invariants:
every ld_reduce reads round s inputs, every copy-out reads round s results,
no deadlock. Broken variants: two buffers instead of three, or a mover that
waits only for its own copier.

BroadcastChain (one block index of the push chain, exec/ring.cu): ranks
0 -> 1 -> ... -> N-1 (rank 0 the root), S steps. The root stores piece k
into rank 1's output and publishes flag[1] = k + 1. Rank r in 1..N-2 waits
until flag[r] >= k + 1 (unless SkipWait), reads piece k from its own output,
stores it into rank r+1's output and publishes flag[r+1] = k + 1. Invariants:
every forwarded piece had arrived (ForwardedArrived), no deadlock, and at
the end every output holds every piece.
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
    checked: tuple = ()          # names of the invariants this run checked
    deadlock_checked: bool = False


def _bfs(init, actions, invariants, max_states=2_000_000, done=None, only=None):
    """Breadth-first over every reachable state. With `done`, a state with no
    successor that is not done is reported as the violation "Deadlock".
    `only` restricts the check to the named invariants (a configuration's
    INVARIANTS list); naming one the model does not have is an error."""
    if only is not None:
        have = {name for name, _ in invariants}
        missing = [x for x in only if x not in have]
        if missing:
            raise ValueError(f"the model has no invariant {missing}")
        invariants = [(name, inv) for name, inv in invariants if name in only]
    seen = {init: None}
    q = deque([init])
    names = tuple(name for name, _ in invariants)
    dl = done is not None

    def trace_to(s):
        trace = []
        cur = s
        while cur is not None:
            trace.append(cur)
            cur = seen[cur]
        return list(reversed(trace))

    while q:
        s = q.popleft()
        for name, inv in invariants:
            if not inv(s):
                return Result(False, len(seen), name, trace_to(s), names, dl)
        succ = 0
        for t in actions(s):
            succ += 1
            if t not in seen:
                seen[t] = s
                if len(seen) > max_states:
                    raise RuntimeError("state space too large")
                q.append(t)
        if done is not None and succ == 0 and not done(s):
            return Result(False, len(seen), "Deadlock", trace_to(s), names, dl)
    return Result(True, len(seen), checked=names, deadlock_checked=dl)


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


def check_group_fallback(nranks=2, max_calls=5, skip_unsupported_flush=False, only=None) -> Result:
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
    return _bfs(init, actions, invs, only=only)


# --------------------------------------------------------------------------
# HostLaneReuse (N sources folded on the host, M destinations)
# --------------------------------------------------------------------------

def check_host_lane_reuse(pieces=5, lanes=4, sources=1, dests=1, skip_reuse_wait=False,
                          fold=None, only=None) -> Result:
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
                                ("ProducedBeforeConsumed", produced_before_consumed)], only=only)


# --------------------------------------------------------------------------
# PushReduce (progress words of the push-reduce engine)
# --------------------------------------------------------------------------

def check_push_reduce(nranks=3, rounds=4, depth=2, skip_consumed_wait=False, only=None) -> Result:
    """State: sj[s] (sender round), sphase[s] (0 write, 1 publish), rj[q]
    (owner round), rphase[q] (0 wait, 1 read, 2 consume), filled[q][s],
    consumed[s][q], slot[q][s][d] (round number held, -1 empty), stale
    (an owner read a wrong round)."""
    N, R, D = nranks, rounds, depth
    init = (tuple([0] * N), tuple([0] * N), tuple([0] * N), tuple([0] * N),
            tuple(tuple([0] * N) for _ in range(N)), tuple(tuple([0] * N) for _ in range(N)),
            tuple(tuple(tuple([-1] * D) for _ in range(N)) for _ in range(N)), False)

    def setv(t, i, v):
        return t[:i] + (v,) + t[i + 1:]

    def actions(st):
        sj, sph, rj, rph, filled, consumed, slot, stale = st
        for s in range(N):
            j = sj[s]
            if j >= R:
                continue
            if sph[s] == 0:
                if not skip_consumed_wait and j >= D and \
                        not all(consumed[s][q] >= j - D + 1 for q in range(N) if q != s):
                    continue
                ns = tuple(tuple(tuple(j if (qq != s and ss == s and d == j % D) else slot[qq][ss][d]
                                       for d in range(D)) for ss in range(N)) for qq in range(N))
                yield (sj, setv(sph, s, 1), rj, rph, filled, consumed, ns, stale)
            else:
                nf = tuple(tuple(j + 1 if (qq != s and ss == s) else filled[qq][ss] for ss in range(N))
                           for qq in range(N))
                yield (setv(sj, s, j + 1), setv(sph, s, 0), rj, rph, nf, consumed, slot, stale)
        for q in range(N):
            j = rj[q]
            if j >= R:
                continue
            if rph[q] == 0:
                if all(filled[q][s] >= j + 1 for s in range(N) if s != q):
                    yield (sj, sph, rj, setv(rph, q, 1), filled, consumed, slot, stale)
            elif rph[q] == 1:
                bad = any(slot[q][s][j % D] != j for s in range(N) if s != q)
                yield (sj, sph, rj, setv(rph, q, 2), filled, consumed, slot, stale or bad)
            else:
                nc = tuple(tuple(j + 1 if (ss != q and qq == q) else consumed[ss][qq] for qq in range(N))
                           for ss in range(N))
                yield (sj, sph, setv(rj, q, j + 1), setv(rph, q, 0), filled, nc, slot, stale)

    def done(st):
        return all(x >= R for x in st[0]) and all(x >= R for x in st[2])

    return _bfs(init, actions, [("NoStaleRead", lambda st: not st[7])], done=done, only=only)


# --------------------------------------------------------------------------
# NvlsAllReduce (progress words of the NVLS AllReduce kernel)
# --------------------------------------------------------------------------

def check_nvls_allreduce(nranks=2, rounds=4, bufs=3, mover_waits_all=True, in_first=False, ahead=False,
                         only=None) -> Result:
    """State: cs[r], cph[r] (copier step and phase), ms[r], mph[r] (mover
    step, 0 wait, 1 read, 2 write+publish), cflag[r], mflag[r],
    buf[r][b][q] = (round, 0 input | 1 reduced) or None, bad.

    Copier step s (the kernel's order): phase 0 waits for every rank's B(s-2)
    and copies round s-2 out (C(s-2)); phase 1 copies round s in (A(s)) and
    publishes s+1. With `in_first` the phases swap (copy-in of round s, then
    copy-out of round s-2): an order that holds in this model but failed the
    pipeline-edge stress on the GPU, so the kernel does not use it. With
    `ahead` (the kernel's NCCL_B200_NVLS_AHEAD, for a buffer per round) the
    copier copies every round in first (steps 0..R-1), then copies round
    s - R out at step s >= R after every rank's B(s - R)."""
    N, R, B = nranks, rounds, bufs
    empty = tuple(tuple(tuple(None for _ in range(N)) for _ in range(B)) for _ in range(N))
    init = (tuple([0] * N), tuple([0] * N), tuple([0] * N), tuple([0] * N),
            tuple([0] * N), tuple([0] * N), empty, False)

    def setv(t, i, v):
        return t[:i] + (v,) + t[i + 1:]

    def setbuf(buf, ranks, b, slices, val):
        return tuple(tuple(tuple(val if (r in ranks and bb == b and q in slices) else buf[r][bb][q]
                                 for q in range(N)) for bb in range(B)) for r in range(N))

    def copy_out(st, r, s_, nxt_cs, nxt_cph):
        """C(s-2) after every rank's B(s-2); None while waiting."""
        cs, cph, ms, mph, cflag, mflag, buf, bad = st
        if s_ < 2:
            return (nxt_cs, nxt_cph, ms, mph, cflag, mflag, buf, bad)
        if not all(mflag[q] >= s_ - 1 for q in range(N)):
            return None
        i = s_ - 2
        wrong = any(buf[r][i % B][q] != (i, 1) for q in range(N))
        return (nxt_cs, nxt_cph, ms, mph, cflag, mflag, buf, bad or wrong)

    def copy_in(st, r, s_, nxt_cs, nxt_cph):
        """A(s) into buffer s%B, then publish s+1."""
        cs, cph, ms, mph, cflag, mflag, buf, bad = st
        nb = setbuf(buf, {r}, s_ % B, set(range(N)), (s_, 0)) if s_ < R else buf
        return (nxt_cs, nxt_cph, ms, mph, setv(cflag, r, s_ + 1), mflag, nb, bad)

    def ahead_step(st, r):
        cs, cph, ms, mph, cflag, mflag, buf, bad = st
        s_ = cs[r]
        if s_ < R:  # copy round s in, publish s+1
            nb = setbuf(buf, {r}, s_ % B, set(range(N)), (s_, 0))
            return (setv(cs, r, s_ + 1), cph, ms, mph, setv(cflag, r, s_ + 1), mflag, nb, bad)
        i = s_ - R  # copy round i out after every rank's B(i)
        if not all(mflag[q] >= i + 1 for q in range(N)):
            return None
        wrong = any(buf[r][i % B][q] != (i, 1) for q in range(N))
        return (setv(cs, r, s_ + 1), cph, ms, mph, cflag, mflag, buf, bad or wrong)

    def actions(st):
        cs, cph, ms, mph, cflag, mflag, buf, bad = st
        for r in range(N):
            s_ = cs[r]
            if ahead:
                if s_ < 2 * R:
                    nxt = ahead_step(st, r)
                    if nxt is not None:
                        yield nxt
            elif s_ < R + 2:
                first, second = (copy_in, copy_out) if in_first else (copy_out, copy_in)
                if cph[r] == 0:
                    nxt = first(st, r, s_, cs, setv(cph, r, 1))
                else:
                    nxt = second(st, r, s_, setv(cs, r, s_ + 1), setv(cph, r, 0))
                if nxt is not None:
                    yield nxt
            s_ = ms[r]
            if s_ < R:
                if mph[r] == 0:
                    ready = all(cflag[q] >= s_ + 1 for q in range(N)) if mover_waits_all else \
                        cflag[r] >= s_ + 1
                    if ready:
                        yield (cs, cph, ms, setv(mph, r, 1), cflag, mflag, buf, bad)
                elif mph[r] == 1:
                    wrong = any(buf[q][s_ % B][r] != (s_, 0) for q in range(N))
                    yield (cs, cph, ms, setv(mph, r, 2), cflag, mflag, buf, bad or wrong)
                else:
                    nb = setbuf(buf, set(range(N)), s_ % B, {r}, (s_, 1))
                    yield (cs, cph, setv(ms, r, s_ + 1), setv(mph, r, 0), cflag, setv(mflag, r, s_ + 1),
                           nb, bad)

    def done(st):
        return all(x >= (2 * R if ahead else R + 2) for x in st[0]) and all(x >= R for x in st[2])

    return _bfs(init, actions, [("RoundsInOrder", lambda st: not st[7])], done=done, only=only)


# --------------------------------------------------------------------------
# BroadcastChain (progress words of the Broadcast push chain)
# --------------------------------------------------------------------------

def check_broadcast_chain(nranks=4, steps=3, skip_wait=False, only=None) -> Result:
    """State: k[r] (next step of rank r), ph[r] (0 wait, 1 read, 2 write),
    flag[r], got[r] (bitmask of pieces in rank r's output), bad."""
    N, S = nranks, steps
    full = (1 << S) - 1
    init = (tuple([0] * N), tuple([0] * N), tuple([0] * N), tuple([full] + [0] * (N - 1)), False)

    def setv(t, i, v):
        return t[:i] + (v,) + t[i + 1:]

    def actions(st):
        k, ph, flag, got, bad = st
        for r in range(N - 1):  # the last rank only receives
            j = k[r]
            if j >= S:
                continue
            if ph[r] == 0:
                if r == 0 or skip_wait or flag[r] >= j + 1:
                    yield (k, setv(ph, r, 1), flag, got, bad)
            elif ph[r] == 1:
                yield (k, setv(ph, r, 2), flag, got, bad or not (got[r] >> j) & 1)
            else:
                ng = setv(got, r + 1, got[r + 1] | (((got[r] >> j) & 1) << j))
                yield (setv(k, r, j + 1), setv(ph, r, 0), setv(flag, r + 1, j + 1), ng, bad)

    def done(st):
        return all(x >= S for x in st[0][:N - 1])

    def complete(st):
        return not done(st) or all(g == full for g in st[3])

    return _bfs(init, actions, [("ForwardedArrived", lambda st: not st[4]),
                                ("AllPiecesDelivered", complete)], done=done, only=only)


# --------------------------------------------------------------------------
# OneShotBarrierN (arrive/depart barriers of the low-latency engine)
# --------------------------------------------------------------------------

def check_oneshot_barrier(nranks=3, calls=3, two=True, skip_arrive=False, skip_depart=False,
                          only=None) -> Result:
    """State: c[r] (call), ph[r] (0 produce, 1 data, 2 depart, 3 leave),
    arr[r], dep[r] (published epochs), inp[r] (call whose input rank r's
    buffer holds), out[r][s] (call whose result slice s of rank r's output
    holds), bad."""
    N, C = nranks, calls
    init = (tuple([0] * N), tuple([0] * N), tuple([0] * N), tuple([0] * N), tuple([-1] * N),
            tuple(tuple([-1] * N) for _ in range(N)), False)

    def setv(t, i, v):
        return t[:i] + (v,) + t[i + 1:]

    def actions(st):
        c, ph, arr, dep, inp, out, bad = st
        for r in range(N):
            if c[r] >= C:
                continue
            k = c[r]
            if ph[r] == 0:
                wrong = k > 0 and any(x != k - 1 for x in out[r])
                yield (c, setv(ph, r, 1), setv(arr, r, k + 1), dep, setv(inp, r, k), out, bad or wrong)
            elif ph[r] == 1:
                if skip_arrive or all(a >= k + 1 for a in arr):
                    wrong = any(x != k for x in inp)
                    if two:
                        nout = tuple(setv(out[q], r, k) for q in range(N))
                    else:
                        nout = setv(out, r, tuple([k] * N))
                    yield (c, setv(ph, r, 2), arr, dep, inp, nout, bad or wrong)
            elif ph[r] == 2:
                yield (c, setv(ph, r, 3), arr, setv(dep, r, k + 1), inp, out, bad)
            else:
                if skip_depart or all(d >= k + 1 for d in dep):
                    yield (setv(c, r, k + 1), setv(ph, r, 0), arr, dep, inp, out, bad)

    def done(st):
        return all(x >= C for x in st[0])

    return _bfs(init, actions, [("CallsInStep", lambda st: not st[6])], done=done, only=only)


# --------------------------------------------------------------------------
# The committed TLC configurations drive the checkers
# --------------------------------------------------------------------------

# Spec module -> (checker, {cfg constant: checker keyword}).
SPECS = {
    "GroupFallbackN": (check_group_fallback, {"N": "nranks", "MaxCalls": "max_calls",
                                              "SkipUnsupportedFlush": "skip_unsupported_flush"}),
    "HostLaneReuseN": (check_host_lane_reuse, {"Pieces": "pieces", "Lanes": "lanes", "S": "sources",
                                               "D": "dests", "SkipReuseWait": "skip_reuse_wait"}),
    "PushReduceN": (check_push_reduce, {"N": "nranks", "R": "rounds", "D": "depth",
                                        "SkipConsumedWait": "skip_consumed_wait"}),
    "NvlsAllReduceN": (check_nvls_allreduce, {"N": "nranks", "R": "rounds", "B": "bufs",
                                              "MoverWaitsAll": "mover_waits_all", "InFirst": "in_first",
                                              "Ahead": "ahead"}),
    "BroadcastChainN": (check_broadcast_chain, {"N": "nranks", "S": "steps", "SkipWait": "skip_wait"}),
    "OneShotBarrierN": (check_oneshot_barrier, {"N": "nranks", "C": "calls", "Two": "two",
                                                "SkipArrive": "skip_arrive", "SkipDepart": "skip_depart"}),
}


@dataclass
class Cfg:
    constants: dict
    invariants: list
    check_deadlock: bool
    specification: str


def _value(tok: str):
    if tok in ("TRUE", "FALSE"):
        return tok == "TRUE"
    return int(tok)


def parse_cfg(text: str) -> Cfg:
    """The subset of TLC's configuration language the committed files use:
    SPECIFICATION, CONSTANT(S) name = value, INVARIANT(S) names, CHECK_DEADLOCK."""
    consts, invs, deadlock, spec = {}, [], True, ""
    section = None
    for raw in text.splitlines():
        line = raw.split("\\*")[0].strip()
        if not line:
            continue
        head, _, rest = line.partition(" ")
        if head in ("CONSTANT", "CONSTANTS"):
            section, line = "const", rest.strip()
        elif head in ("INVARIANT", "INVARIANTS"):
            section, line = "inv", rest.strip()
        elif head == "SPECIFICATION":
            spec, section = rest.strip(), None
            continue
        elif head == "CHECK_DEADLOCK":
            deadlock, section = _value(rest.strip()), None
            continue
        if not line:
            continue
        if section == "const":
            name, eq, val = line.partition("=")
            if not eq:
                raise ValueError(f"constant without a value: {raw!r}")
            consts[name.strip()] = _value(val.strip())
        elif section == "inv":
            invs.extend(line.split())
        else:
            raise ValueError(f"unrecognized line: {raw!r}")
    return Cfg(consts, invs, deadlock, spec)


def parse_tla(text: str) -> tuple:
    """(module name, declared constants, names of the defined operators)."""
    import re
    m = re.search(r"-+\s*MODULE\s+(\w+)", text)
    decl = re.search(r"^CONSTANTS?\s+([^\n]+)", text, re.M)
    consts = [c.strip() for c in decl.group(1).split(",")] if decl else []
    defs = set(re.findall(r"^(\w+)(?:\([^)]*\))?\s*==", text, re.M))
    return (m.group(1) if m else None), consts, defs


def check_cfg(cfg_path: str) -> tuple:
    """Run the checker of a committed configuration with exactly its
    constants. Verifies first that the configuration and its spec agree with
    the checker: the same constants as the spec declares, invariants the spec
    defines and the checker checks, and the same deadlock setting.
    Returns (Cfg, Result)."""
    import os
    cfg_text = open(cfg_path).read()
    cfg = parse_cfg(cfg_text)
    base = os.path.basename(cfg_path)
    module = base.split(".")[0].replace("-broken", "")
    tla_path = os.path.join(os.path.dirname(cfg_path), module + ".tla")
    name, declared, defined = parse_tla(open(tla_path).read())
    if name != module:
        raise ValueError(f"{tla_path}: module {name}, expected {module}")
    checker, kw = SPECS[module]
    if set(cfg.constants) != set(declared) or set(declared) != set(kw):
        raise ValueError(f"{base}: constants {sorted(cfg.constants)}, spec declares {declared}, "
                         f"checker maps {sorted(kw)}")
    if cfg.specification not in defined:
        raise ValueError(f"{base}: SPECIFICATION {cfg.specification} is not defined in {module}.tla")
    for inv in cfg.invariants:
        if inv not in defined:
            raise ValueError(f"{base}: invariant {inv} is not defined in {module}.tla")
    res = checker(**{kw[k]: v for k, v in cfg.constants.items()}, only=list(cfg.invariants))
    if set(res.checked) != set(cfg.invariants):
        raise ValueError(f"{base}: the checker checked {res.checked}, the configuration lists "
                         f"{cfg.invariants}")
    if res.deadlock_checked != cfg.check_deadlock:
        raise ValueError(f"{base}: CHECK_DEADLOCK {cfg.check_deadlock}, checker "
                         f"{res.deadlock_checked}")
    return cfg, res
