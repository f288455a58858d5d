"""Explicit-state model check of the tensor-parallel exchange protocols of
okc_b200/csrc/tp_comm.cu (CPU only).

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
