"""Explicit-state model checks (CPU only) of the synchronisation protocols of the kernels:
the tensor-parallel exchange protocols of okc_b200/csrc/tp_comm.cu, and (at the end of the
file) the mbarrier shared-memory ring of the attention and tcgen05 GEMM kernels.

Both kernels synchronise per CTA index: CTA c of a rank only exchanges flags with CTA c of the
other ranks, so one CTA index is modelled, on W ranks, over E consecutive calls.  Every
interleaving of the ranks' steps is explored (breadth-first over the reachable states); the
model asserts the two safety properties the kernels rely on and that no reachable state is
stuck before every rank has finished:

  * a rank reads only data of the current call (a receive slot or a peer's partial written in
    the same call: neither stale nor already overwritten by the peer's next call);
  * when a rank's call completes, every slice of its output holds the current call's result,
    and no slice is overwritten by a peer's next call before this rank consumed it (the
    consumer of the output runs in stream order between two calls).

A step that publishes a flag is atomic with the data written before it (the kernels' release:
barrier, fence.acq_rel.sys, relaxed flag store; the waiter's acquire load).  Stream order on a
rank: the call's data writes happen after its griddepcontrol.wait, i.e. after the previous
call and the consumer of its output completed.  Planted protocol mistakes (in the model) are
detected, which shows the check has teeth.
"""

from collections import deque

import pytest


def _explore(W, E, program):
    """BFS over (per-rank (call, pc), memory).  `program(W, r[, e])` returns the step list of rank
    r for a call: each step is (kind, arg) interpreted by _step.  Returns None or a violation."""
    init = (tuple((1, 0) for _ in range(W)), ())
    progs = {(r, e): _prog(program, W, r, e) for r in range(W) for e in range(1, E + 1)}
    seen = {init}
    dq = deque([init])
    while dq:
        pcs, mem_t = dq.popleft()
        mem = dict(mem_t)
        moved = False
        for r in range(W):
            e, pc = pcs[r]
            if e > E:
                continue
            res = _step(progs[r, e][pc], r, e, W, mem)
            if res is None:  # blocked
                continue
            if isinstance(res, str):
                return res
            moved = True
            pc2, e2 = pc + 1, e
            if pc2 == len(progs[r, e]):
                pc2, e2 = 0, e + 1
            npcs = list(pcs)
            npcs[r] = (e2, pc2)
            st = (tuple(npcs), tuple(sorted(res.items())))
            if st not in seen:
                seen.add(st)
                dq.append(st)
        if not moved and any(e <= E for e, _ in pcs):
            return f"stuck: {pcs}"
    return None


def _prog(program, W, r, e):
    # program(W, r) is the same for every call; program(W, r, e) may differ per call
    return program(W, r, e) if program.__code__.co_argcount == 3 else program(W, r)


def _step(step, r, e, W, mem):
    """Applies one step of rank r in call e; returns the new memory, None if blocked, or a
    violation message."""
    kind, arg = step
    m = dict(mem)
    g = lambda k: m.get(k, 0)  # noqa: E731
    if kind == "write":        # data store: key template with r / q substituted
        m[arg(r)] = e
    elif kind == "check_eq":   # read that must see this call's data
        for key in arg(r):
            if g(key) != e:
                return f"rank {r} call {e}: read {key} = {g(key)}"
    elif kind == "signal":     # release: flag words of the other ranks
        for key in arg(r):
            m[key] = e
    elif kind == "wait":       # acquire: every listed flag >= e
        if any(g(key) < e for key in arg(r)):
            return None
    return m


def fused_oproj_program(W, r, *, wait_push=True, wait_exit=True, out_before_wait=False):
    """tp_oproj_kernel, one CTA index: push the other ranks' slices into their receive slots,
    raise their push flags, wait for this rank's W-1 push flags, reduce (read the slots), store
    the output slice into every rank, raise exit flags, wait for the peers' exit flags; then the
    stream's consumer reads the whole output."""
    others = [q for q in range(W) if q != r]
    push = [("write", (lambda q: lambda r: ("recv", q, r))(s)) for s in others]
    sig_push = [("signal", lambda r: [("push", q, r) for q in range(W) if q != r])]
    wpush = [("wait", lambda r: [("push", r, q) for q in range(W) if q != r])] if wait_push else []
    read = [("check_eq", lambda r: [("recv", r, q) for q in range(W) if q != r])]
    out = [("write", (lambda q: lambda r: ("out", q, r))(q)) for q in range(W)]
    sig_exit = [("signal", lambda r: [("exit", q, r) for q in range(W) if q != r])]
    wexit = [("wait", lambda r: [("exit", r, q) for q in range(W) if q != r])] if wait_exit else []
    consume = [("check_eq", lambda r: [("out", r, s) for s in range(W)])]
    if out_before_wait:
        return push + sig_push + out + wpush + read + sig_exit + wexit + consume
    return push + sig_push + wpush + read + out + sig_exit + wexit + consume


def _renamed(steps, prefix):
    """The same steps on flag words of another namespace (each kernel has its own flag range
    and per-CTA epochs); data keys (receive slots, partials, outputs) are shared."""
    out = []
    for kind, arg in steps:
        if kind in ("signal", "wait"):
            out.append((kind, (lambda a: lambda r: [(prefix,) + k for k in a(r)])(arg)))
        else:
            out.append((kind, arg))
    return out


def exchange_program(W, r, *, entry=True, wait_exit=True):
    """tp_allreduce_kernel, one CTA index: the producer (the O projection's GEMM) writes this
    rank's partial, entry flags, wait for the peers' entry flags, read every rank's partial
    (peer loads), store the output slice into every rank, exit flags, wait; then consume."""
    part = [("write", lambda r: ("part", r))]
    sig_entry = [("signal", lambda r: [("entry", q, r) for q in range(W) if q != r])] if entry else []
    wentry = [("wait", lambda r: [("entry", r, q) for q in range(W) if q != r])] if entry else []
    read = [("check_eq", lambda r: [("part", q) for q in range(W)])]
    out = [("write", (lambda q: lambda r: ("out", q, r))(q)) for q in range(W)]
    sig_exit = [("signal", lambda r: [("exit", q, r) for q in range(W) if q != r])]
    wexit = [("wait", lambda r: [("exit", r, q) for q in range(W) if q != r])] if wait_exit else []
    consume = [("check_eq", lambda r: [("out", r, s) for s in range(W)])]
    return part + sig_entry + wentry + read + out + sig_exit + wexit + consume


@pytest.mark.parametrize("W,E", [(2, 3), (3, 2)])
def test_fused_oproj_protocol_is_safe_and_live(W, E):
    assert _explore(W, E, fused_oproj_program) is None


@pytest.mark.parametrize("W,E", [(2, 3), (3, 2)])
def test_exchange_protocol_is_safe_and_live(W, E):
    assert _explore(W, E, exchange_program) is None


@pytest.mark.parametrize("mistake,expect", [
    (dict(wait_push=False), "read ('recv'"),          # reduce before the slices arrived
    (dict(wait_exit=False), "read ('out'"),           # complete before the peers' rows landed
    (dict(out_before_wait=True), "read ('out'"),      # write a peer's output before it reached this call
])
def test_planted_fused_protocol_mistakes_are_found(mistake, expect):
    err = _explore(2, 2, lambda W, r: fused_oproj_program(W, r, **mistake))
    assert err is not None and expect in err, err


@pytest.mark.parametrize("mistake,expect", [
    (dict(entry=False), "read ('part'"),              # pull a partial the peer has not written yet
    (dict(wait_exit=False), "read ("),                # complete (and rewrite the partial) too early
])
def test_planted_exchange_protocol_mistakes_are_found(mistake, expect):
    err = _explore(2, 2, lambda W, r: exchange_program(W, r, **mistake))
    assert err is not None and expect in err, err


@pytest.mark.parametrize("W,E", [(2, 4), (3, 2)])
def test_fused_and_exchange_alternating_on_one_group(W, E):
    """One exchange group (one output buffer) used by both kernels in turn, as the layer's
    fused O projection and the expert-parallel MoE's exchange would share it."""
    def prog(W, r, e):
        if e % 2:
            return _renamed(fused_oproj_program(W, r), "f")
        return _renamed(exchange_program(W, r), "x")
    assert _explore(W, E, prog) is None


def test_planted_mistake_in_alternating_use_is_found():
    def prog(W, r, e):
        if e % 2:
            return _renamed(fused_oproj_program(W, r), "f")
        return _renamed(exchange_program(W, r, wait_exit=False), "x")
    err = _explore(2, 3, prog)
    assert err is not None and "read (" in err, err


# ------------------------------------------------------------------------------------------
# The shared-memory ring of the attention and tcgen05 GEMM kernels (mbarrier full/empty pairs).
# Producer: for unit i, slot s = i % NS with phase bit ph (flips when s wraps): wait
# empty[s] with parity ph ^ 1, arm full[s] (expect_tx), issue the copy; the copy lands
# asynchronously and completes full[s]'s phase.  Consumers (C warps; empty[s] expects C
# arrivals): wait full[s] with parity ph, read the slot, arrive on empty[s].  Before exiting the
# producer waits on the full barriers of its last min(issued, NS) units, walking the slots
# backwards (attention.cu / gemm_tc.cu drain loops).  try_wait.parity(P) succeeds once the
# barrier's completed-phase count has parity != P (the phase with parity P is complete).

def _ring_explore(NS, N, C, drain=True, parity_ok=True, aborts=True, empty_count=None):
    """All interleavings of one producer, C consumers and the asynchronous copy completions
    over N units, including aborts: a consumer may give up at any point (a wait that timed out)
    and set the abort flag, after which the producer stops issuing (its own bounded empty-wait
    gives up too) and drains.  Checked: a consumer reads only the unit it waited for; a copy
    never lands in a slot a consumer has not released; no copy is in flight when the CTA exits
    (producer drained, every consumer finished or gave up); and nothing is stuck (with aborts
    off this is the liveness of the protocol itself: a wait that never ends is a hang)."""
    # state: producer (issued, stage, ph, stopped, drained), abort flag, consumers (unit, stage,
    # ph, gone), full (completed phases, armed), empty (completed phases, arrivals), copies in
    # flight ((unit, slot), ...), slot contents
    init = (0, 0, 0, False, 0, False, tuple((0, 0, 0, False) for _ in range(C)),
            tuple((0, 0) for _ in range(NS)), tuple((0, 0) for _ in range(NS)), (), tuple(-1 for _ in range(NS)))
    ec = C if empty_count is None else empty_count  # arrivals that complete an empty phase
    seen = {init}
    dq = deque([init])
    while dq:
        st = dq.popleft()
        pi, ps, pph, stopped, dk, ab, cons, full, empty, fly, slot = st
        looping = pi < N and not stopped
        n_drain = min(pi, NS) if drain else 0
        nxt = []
        if looping:
            want = (pph ^ 1) if parity_ok else pph
            if empty[ps][0] % 2 != want:  # issue unit pi into slot ps
                f = list(full)
                f[ps] = (f[ps][0], 1)
                ns, nph = ps + 1, pph
                if ns == NS:
                    ns, nph = 0, pph ^ 1
                nxt.append((pi + 1, ns, nph, stopped, dk, ab, cons, tuple(f), empty, fly + ((pi, ps),), slot))
            if ab:  # the abort flag is seen (or the bounded empty-wait gives up)
                nxt.append((pi, ps, pph, True, dk, ab, cons, full, empty, fly, slot))
        elif dk < n_drain:  # drain: the k-th slot back from the next one to issue
            sd, ph = ps, pph
            for _ in range(dk + 1):
                sd -= 1
                if sd < 0:
                    sd, ph = NS - 1, ph ^ 1
            if full[sd][0] % 2 != ph:
                nxt.append((pi, ps, pph, stopped, dk + 1, ab, cons, full, empty, fly, slot))
        for k, (u, sl_) in enumerate(fly):  # a copy lands
            for ci, (ciu, _, _, gone) in enumerate(cons):
                if not gone and ciu < u - NS + 1:
                    return f"unit {u} landed in slot {sl_} before consumer {ci} released unit {u - NS}"
            f = list(full)
            f[sl_] = (f[sl_][0] + 1, 0)  # armed arrival + bytes complete: the phase completes
            sl = list(slot)
            sl[sl_] = u
            nxt.append((pi, ps, pph, stopped, dk, ab, cons, tuple(f), empty, fly[:k] + fly[k + 1:], tuple(sl)))
        for ci, (u, sc, ph, gone) in enumerate(cons):
            if gone or u >= N:
                continue
            if aborts:
                c2 = list(cons)
                c2[ci] = (u, sc, ph, True)  # gives up: sets the abort flag and leaves
                nxt.append((pi, ps, pph, stopped, dk, True, tuple(c2), full, empty, fly, slot))
            if full[sc][0] % 2 == ph:
                continue
            if slot[sc] != u:
                return f"consumer {ci} read slot {sc} holding unit {slot[sc]} for unit {u}"
            e = list(empty)
            ph_e, arr = e[sc]
            arr += 1
            e[sc] = (ph_e + 1, 0) if arr == ec else (ph_e, arr)
            ns, nph = sc + 1, ph
            if ns == NS:
                ns, nph = 0, ph ^ 1
            c2 = list(cons)
            c2[ci] = (u + 1, ns, nph, False)
            nxt.append((pi, ps, pph, stopped, dk, ab, tuple(c2), full, tuple(e), fly, slot))
        producer_done = not looping and dk == n_drain
        consumers_done = all(g or u >= N for u, _, _, g in cons)
        if producer_done and consumers_done and fly:
            return f"CTA exits with copies in flight {fly}"
        if not nxt and not (producer_done and consumers_done):
            return f"stuck: producer {pi} stopped={stopped} drained={dk}, consumers {cons}"
        for t in nxt:
            if t not in seen:
                seen.add(t)
                dq.append(t)
    return None


@pytest.mark.parametrize("NS,N,C", [(2, 5, 1), (3, 6, 1), (3, 5, 2), (2, 4, 3)])
def test_mbarrier_ring_is_safe_and_drains(NS, N, C):
    assert _ring_explore(NS, N, C, aborts=False) is None  # safety and liveness
    assert _ring_explore(NS, N, C) is None                # safety and a clean exit under aborts


def test_planted_ring_mistakes_are_found():
    # the wrong parity on the empty barrier: the producer waits for a phase that never comes
    assert "stuck" in (_ring_explore(2, 4, 1, parity_ok=False, aborts=False) or "")
    # empty barriers that expect fewer arrivals than there are consumer warps: a slot is
    # refilled while a consumer has not read it yet
    err = _ring_explore(2, 4, 2, aborts=False, empty_count=1) or ""
    assert "landed in slot" in err or "read slot" in err, err
    # no drain: after an abort the CTA can exit with copies still landing in its shared memory
    assert "in flight" in (_ring_explore(2, 4, 1, drain=False) or "")
