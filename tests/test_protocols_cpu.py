"""Flag protocols of the peer-memory kernels, checked on an emulated
flag/counter model (``protocol_sim``) under many random interleavings of the
ranks: no rank reads a buffer before its producer's data is there or after a
later producer has overwritten it, and no schedule deadlocks.

Each model restates, per rank, the order of kernel launches, flag channels,
sequence numbers and buffer choices that the host code issues
(``parallel/peer_dp.py`` for the ZeRO step, ``parallel/tp_fused.py`` for
tensor + sequence parallelism, whose sequence bookkeeping is the real
``TPComm.next_seq`` / ``parts_index``, ``parallel/ep_fused.py`` for expert
parallelism, ``parallel/context_parallel.py`` for context parallelism), and
the loads and stores each kernel makes (``csrc/zero_comm.cu``,
``csrc/tp_comm.cu``, ``csrc/gemm.cu``, ``csrc/ep_comm.cu``,
``csrc/cp_comm.cu``).  A variant with a protocol step removed must be
caught.
"""

import pytest

from protocol_sim import ProtocolError, explore

# ------------------------------------------------------------------ ZeRO step


def zero_rank(r: int, W: int, steps: int, publish: bool = True):
    """One rank of the fused data-parallel step over ``steps`` steps: the
    forward/backward reads every shard of the local bf16 compute copy and
    writes every shard of the local fp32 gradient; ``zero_rs`` (flag slot 0)
    reads shard r of every peer's gradient and writes the mean into the local
    shard; after the norm all-reduce ``zero_adamw_ag`` stores the updated
    shard r into every peer's compute copy; ``zero_publish`` (slot 1) is the
    barrier before anyone's next forward."""
    for t in range(1, steps + 1):
        for s in range(W):
            yield ("read", ("comp", s), ("w", t - 1))          # forward / backward
        for s in range(W):
            yield ("write", r, ("grad", s), ("g", r, t))
        for p in range(W):                                    # zero_rs: signal, wait
            yield ("signal", p, "zero0", r, t)
        yield ("wait", "zero0", range(W), t)
        for p in range(W):
            yield ("read_peer", p, ("grad", r), ("g", p, t))
        yield ("write", r, ("grad", r), ("mean", t))
        yield ("collective", f"norm{t}")                      # squared norm all-reduce
        yield ("read", ("grad", r), ("mean", t))              # zero_adamw_ag
        for p in range(W):
            yield ("write", p, ("comp", r), ("w", t))
        if publish:                                           # zero_publish
            for p in range(W):
                yield ("signal", p, "zero1", r, t)
            yield ("wait", "zero1", range(W), t)


def _zero_ranks(W, steps, publish=True):
    def make():
        ranks = [zero_rank(r, W, steps, publish) for r in range(W)]
        return ranks

    return make


def _init_zero(W):
    # initial compute copy: version 0 everywhere (written before the first step)
    def gen(r):
        for s in range(W):
            yield ("write", r, ("comp", s), ("w", 0))
        yield ("collective", "init")
    return gen


def _with_init(W, body):
    init = _init_zero(W)

    def make():
        out = []
        for r, g in enumerate(body()):
            def chain(r=r, g=g):
                yield from init(r)
                yield from g
            out.append(chain())
        return out
    return make


@pytest.mark.parametrize("W", [2, 4, 8])
def test_zero_step_protocol(W):
    explore(_with_init(W, _zero_ranks(W, 3)), schedules=150)


def test_zero_step_without_publish_barrier_races():
    """Without the publish barrier a fast rank's next forward reads a compute
    shard that a slow peer has not stored yet."""
    with pytest.raises(ProtocolError):
        explore(_with_init(4, _zero_ranks(4, 3, publish=False)), schedules=150)


def zero_ep_rank(r: int, W: int, EP: int, steps: int, expert_peers_only: bool = True,
                 skip_empty: bool = False):
    """One rank of the fused data-parallel step with an expert span
    (``PeerDataParallel`` under expert parallelism): ranks r with the same
    r % EP hold the same experts.  The dense shard is reduced in two calls
    (the pieces before and after the expert span; flag epochs 2t-1 and 2t);
    the expert span is sharded over the X = W / EP ranks holding the same
    experts, with its own flag words (``xzero0``) and the subset of the peer
    pointers, and its AdamW stores only into those ranks' compute copies
    (``expert_peers_only``); one publish barrier over all W ranks.
    ``skip_empty``: rank 0 leaves out its second (empty) dense call, with
    its own epoch count, which the peers' waits must expose."""
    X = W // EP
    blk = r % EP
    members = [p for p in range(W) if p % EP == blk]
    xr = members.index(r)
    for t in range(1, steps + 1):
        for s in range(W):
            yield ("read", ("comp", s), ("w", t - 1))
        for j in range(X):
            yield ("read", ("xcomp", j), ("xw", blk, t - 1))
        for s in range(W):
            yield ("write", r, ("grad", s), ("g", r, t))
        for j in range(X):
            yield ("write", r, ("xgrad", j), ("xg", r, t))
        calls = (t,) if (skip_empty and r == 0) else (2 * t - 1, 2 * t)
        for call in calls:                                    # dense pieces
            for p in range(W):
                yield ("signal", p, "zero0", r, call)
            yield ("wait", "zero0", range(W), call)
            if call == calls[0]:
                for p in range(W):
                    yield ("read_peer", p, ("grad", r), ("g", p, t))
                yield ("write", r, ("grad", r), ("mean", t))
        for p in members:                                     # expert span
            yield ("signal", p, "xzero0", xr, t)
        yield ("wait", "xzero0", range(X), t)
        for p in members:
            yield ("read_peer", p, ("xgrad", xr), ("xg", p, t))
        yield ("write", r, ("xgrad", xr), ("xmean", t))
        yield ("collective", f"norm{t}")
        yield ("read", ("grad", r), ("mean", t))
        for p in range(W):
            yield ("write", p, ("comp", r), ("w", t))
        yield ("read", ("xgrad", xr), ("xmean", t))
        for p in (members if expert_peers_only else range(W)):
            yield ("write", p, ("xcomp", xr), ("xw", blk, t))
        for p in range(W):
            yield ("signal", p, "zero1", r, t)
        yield ("wait", "zero1", range(W), t)


def _zero_ep(W, EP, steps, expert_peers_only=True, skip_empty=False):
    def make():
        out = []
        for r in range(W):
            def chain(r=r):
                for s in range(W):
                    yield ("write", r, ("comp", s), ("w", 0))
                for j in range(W // EP):
                    yield ("write", r, ("xcomp", j), ("xw", r % EP, 0))
                yield ("collective", "init")
                yield from zero_ep_rank(r, W, EP, steps, expert_peers_only, skip_empty)
            out.append(chain())
        return out
    return make


@pytest.mark.parametrize("W,EP", [(2, 2), (4, 2), (8, 2), (8, 4)])
def test_zero_step_with_expert_span_protocol(W, EP):
    explore(_zero_ep(W, EP, 3), schedules=120)


def test_zero_step_uneven_dense_calls_are_caught():
    """A rank that skips its empty dense piece (and so counts its flag
    epochs differently) leaves its peers waiting or reading early."""
    with pytest.raises(ProtocolError):
        explore(_zero_ep(4, 2, 3, skip_empty=True), schedules=60)


def test_zero_step_expert_update_to_every_rank_is_caught():
    """Storing the updated expert shard into every data-parallel rank, not
    only the ranks holding the same experts, overwrites other experts."""
    with pytest.raises(ProtocolError):
        explore(_zero_ep(4, 2, 2, expert_peers_only=False), schedules=60)


# -------------------------------------------------------- tensor parallel

AG_FWD, RS_FWD, AG_BWD, RS_BWD = 0, 1, 2, 3


def _comm(W, r):
    from nano_qwen_b200.parallel.tp_fused import TPComm
    c = object.__new__(TPComm)
    c.world, c.rank, c.seq, c.count = W, r, [0, 0, 0, 0], 0
    return c


def tp_rank(r: int, W: int, layers: int, steps: int, ping_pong: int = 2, norm_waits: bool = True,
            close_step: bool = True):
    """One rank of fused TP+SP training (``block_forward`` and the autograd
    backward of its functions) over ``steps`` steps.  Buffers: x_full per
    (layer, norm) (persistent, read again by the weight-gradient GEMMs),
    ``parts_fwd`` / ``parts_bwd`` / ``dy_full`` rotating over ``ping_pong``
    copies chosen by sequence number, planes indexed by the writing rank."""
    from nano_qwen_b200.parallel.tp_fused import parts_index
    comm = _comm(W, r)

    def signal_all(ch, seq):
        for p in range(W):
            yield ("signal", p, ch, r, seq)

    def rs_write(kind, ch):            # gemm_rs: row tiles to their owners, then the grid flag
        seq = comm.next_seq(ch)
        for q in range(W):
            yield ("write", q, (kind, seq % ping_pong, r), (kind, r, seq))
        yield from signal_all(ch, seq)

    def rs_read(kind, ch, seq):        # tp_norm: wait for every source, read every plane
        if norm_waits:
            yield ("wait", ch, range(W), seq)
        for p in range(W):
            yield ("read", (kind, seq % ping_pong, p), (kind, p, seq))

    def ag_write(key, ch, seq):        # tp_norm: this rank's rows into every rank's buffer
        for q in range(W):
            yield ("write", q, key + (r,), (key, r, seq))
        yield from signal_all(ch, seq)

    def ag_read(key, ch, seq):         # gemm_ag: producer waits per owner, reads all rows
        yield ("wait", ch, range(W), seq)
        for p in range(W):
            yield ("read", key + (p,), (key, p, seq))

    for t in range(steps):
        ag_seqs = {}
        # ---- forward
        have_parts = False
        for layer in range(layers):
            for n in (0, 1):
                if have_parts:
                    _, pseq = parts_index(comm)
                    yield from rs_read("pf", RS_FWD, pseq)
                s = comm.next_seq(AG_FWD)
                key = ("x", layer, n)
                ag_seqs[(layer, n)] = s
                yield from ag_write(key, AG_FWD, s)
                yield from ag_read(key, AG_FWD, comm.seq[AG_FWD])   # q|k|v or gate|up
                yield from rs_write("pf", RS_FWD)                    # o_proj or down_proj
                have_parts = True
        _, pseq = parts_index(comm)
        yield from rs_read("pf", RS_FWD, pseq)                       # final norm
        # ---- backward: final norm (gathers dy for the last down_proj)
        s = comm.next_seq(AG_BWD)
        yield from ag_write(("dy", s % ping_pong), AG_BWD, s)
        for layer in reversed(range(layers)):
            for n in (1, 0):
                s = comm.seq[AG_BWD]                                 # row-parallel dgrad/wgrad
                yield from ag_read(("dy", s % ping_pong), AG_BWD, s)
                yield from rs_write("pb", RS_BWD)                    # column-parallel dgrad
                key = ("x", layer, n)                                # its weight gradient
                for p in range(W):
                    yield ("read", key + (p,), (key, p, ag_seqs[(layer, n)]))
                yield from rs_read("pb", RS_BWD, comm.seq[RS_BWD])   # norm backward
                if not (layer == 0 and n == 0):                      # fed by partials: gather dy
                    s = comm.next_seq(AG_BWD)
                    yield from ag_write(("dy", s % ping_pong), AG_BWD, s)
        # replicated-gradient all-reduce and the norm all-reduce close the step
        if close_step:
            yield ("collective", f"grads{t}")


def _tp_ranks(W, layers, steps, ping_pong=2, norm_waits=True, close_step=True):
    return lambda: [tp_rank(r, W, layers, steps, ping_pong, norm_waits, close_step)
                    for r in range(W)]


@pytest.mark.parametrize("W", [2, 4, 8])
def test_tensor_parallel_protocol(W):
    explore(_tp_ranks(W, layers=3, steps=2), schedules=60)


def test_tensor_parallel_single_buffer_is_also_ordered():
    """The partial / gradient buffers alternate between two copies, but the
    protocol does not depend on it: a rank's next reduce-scatter store comes
    after its all-gather wait on every rank's norm, which has finished
    reading the previous partials.  (The second copy is kept as slack.)"""
    explore(_tp_ranks(4, layers=3, steps=2, ping_pong=1), schedules=60)


def test_tensor_parallel_norm_without_wait_races():
    """A norm that sums the partials without waiting for every source's
    reduce-scatter flag reads a plane that is not there yet."""
    with pytest.raises(ProtocolError):
        explore(_tp_ranks(4, layers=3, steps=2, norm_waits=False), schedules=60)


def test_tensor_parallel_steps_are_ordered_by_the_gradient_all_reduce():
    """The gathered activations of a layer are read again by its
    weight-gradient GEMM; the next step's all-gather into them is held back
    only by the collectives that close a step (replicated-gradient and norm
    all-reduces).  Without them a fast rank overwrites a slow rank's x_full."""
    with pytest.raises(ProtocolError):
        explore(_tp_ranks(4, layers=2, steps=3, close_step=False), schedules=100)


# -------------------------------------------------------- expert parallel

CH_COUNTS, CH_DISPATCH, CH_OUT, CH_DOUT, CH_DX = 0, 1, 2, 3, 4


def ep_rank(r: int, W: int, routes, steps: int, dx_buffers: int = 2):
    """One rank of fused expert parallelism (``parallel/ep_fused.py``) over
    ``steps`` steps of len(routes) MoE layers; ``routes[l][s][q]`` is True
    when source s has (token, expert) pairs on owner q's experts in layer l.
    Per layer: the counts exchange (every rank's table, all-rank wait), the
    dispatch (P2P stores into the owners' per-layer receive buffers, then the
    grid flag to every rank), the gate|up GEMM whose tiles wait only for the
    sources whose rows they read, the outputs in the shared ``y_out`` buffer
    pulled by the sources' combine (all-rank wait).  Backward: the weighted
    output gradient pushed into the owners' shared ``dy_recv``, the dgrad
    GEMM's per-source waits, the weight gradients re-reading ``dy_recv`` and
    the receive buffer, the input gradient staged in ``dx_recv`` (one copy
    per layer parity) and pulled by the sources (all-rank wait)."""
    seq = [0] * 5
    L = len(routes)

    def nxt(ch):
        seq[ch] += 1
        return seq[ch]

    def signal_all(ch, s):
        for p in range(W):
            yield ("signal", p, ch, r, s)

    for t in range(steps):
        for layer in range(L):
            rt = routes[layer]
            s0 = nxt(CH_COUNTS)
            for p in range(W):
                yield ("write", p, ("counts", r), ("cnt", layer, r, t))
            yield from signal_all(CH_COUNTS, s0)
            yield ("wait", CH_COUNTS, range(W), s0)
            for p in range(W):
                yield ("read", ("counts", p), ("cnt", layer, p, t))   # layout + table copy
            s1 = nxt(CH_DISPATCH)
            for q in range(W):
                if rt[r][q]:
                    yield ("write", q, ("recv", layer, r), ("x", layer, r, t))
            yield from signal_all(CH_DISPATCH, s1)
            senders = [s for s in range(W) if rt[s][r]]
            if senders:
                yield ("wait", CH_DISPATCH, senders, s1)
            for s in senders:
                yield ("read", ("recv", layer, s), ("x", layer, s, t))
            s2 = nxt(CH_OUT)
            yield ("write", r, ("yout",), ("y", layer, r, t))
            yield from signal_all(CH_OUT, s2)
            yield ("wait", CH_OUT, range(W), s2)
            for q in range(W):
                if rt[r][q]:
                    yield ("read_peer", q, ("yout",), ("y", layer, q, t))
        for layer in reversed(range(L)):
            rt = routes[layer]
            s3 = nxt(CH_DOUT)
            for q in range(W):
                if rt[r][q]:
                    yield ("write", q, ("dyr", r), ("dy", layer, r, t))
            yield from signal_all(CH_DOUT, s3)
            senders = [s for s in range(W) if rt[s][r]]
            if senders:
                yield ("wait", CH_DOUT, senders, s3)
            for s in senders:
                yield ("read", ("dyr", s), ("dy", layer, s, t))        # dgrad, then weight grads
                yield ("read", ("recv", layer, s), ("x", layer, s, t))
            s4 = nxt(CH_DX)
            slot = layer % dx_buffers
            yield ("write", r, ("dxr", slot), ("dx", layer, r, t))
            yield from signal_all(CH_DX, s4)
            yield ("wait", CH_DX, range(W), s4)
            for q in range(W):
                if rt[r][q]:
                    yield ("read_peer", q, ("dxr", slot), ("dx", layer, q, t))
        yield ("collective", f"grads{t}")      # dense-gradient all-reduce closes the step


def _routes(W, L, seed, density=0.5):
    import random
    g = random.Random(seed)
    return [[[g.random() < density for _ in range(W)] for _ in range(W)] for _ in range(L)]


@pytest.mark.parametrize("W", [2, 4, 8])
def test_expert_parallel_protocol(W):
    for k in range(6):
        routes = _routes(W, 4, k, density=0.3 + 0.1 * k)
        explore(lambda: [ep_rank(r, W, routes, 2) for r in range(W)], schedules=40)


def test_expert_parallel_single_dx_buffer_races():
    """With one ``dx_recv`` buffer an owner that no source waits on can
    overwrite it with the next (earlier) layer's input gradient while a
    source still pulls the current layer's rows: source 0 routes to owner 1
    in layer 1 but not in layer 0, so owner 1's layer-0 dgrad does not wait
    for it."""
    routes = [[[True, False], [True, True]],      # layer 0: 0 -> 0 only; 1 -> both
              [[True, True], [True, True]]]       # layer 1: everyone -> everyone
    with pytest.raises(ProtocolError):
        explore(lambda: [ep_rank(r, 2, routes, 1, dx_buffers=1) for r in range(2)], schedules=200)
    explore(lambda: [ep_rank(r, 2, routes, 1, dx_buffers=2) for r in range(2)], schedules=200)


# -------------------------------------------------------- context parallel


def cp_rank(r: int, W: int, layers: int, steps: int, dkv_buffers: int = 2):
    """One rank of context parallelism on the peer-memory kernels
    (``parallel/context_parallel.py``, ``csrc/cp_comm.cu``): per layer the
    rank stores its k|v rows into every rank's per-layer gathered buffer and
    releases channel 0; its attention waits, per key block, for the owner's
    flag (with the zigzag split every rank's later chunk sees every owner).
    Backward: the rank's fp32 dk|dv partial for every key goes into its own
    buffer (alternating by sequence number), channel 1 is released, and the
    gather waits for every rank before summing the rows of its own tokens
    from every rank's partial; the backward also re-reads the gathered k|v."""
    seq = [0, 0]
    for t in range(steps):
        for layer in range(layers):
            seq[0] += 1
            s0 = seq[0]
            for q in range(W):
                yield ("write", q, ("kv", layer, r), ("kv", layer, r, t))
            for q in range(W):
                yield ("signal", q, 0, r, s0)
            for o in range(W):
                yield ("wait", 0, [o], s0)
                yield ("read", ("kv", layer, o), ("kv", layer, o, t))
        for layer in reversed(range(layers)):
            for o in range(W):
                yield ("read", ("kv", layer, o), ("kv", layer, o, t))
            seq[1] += 1
            s1 = seq[1]
            slot = s1 % dkv_buffers
            yield ("write", r, ("dkv", slot), ("dkv", layer, r, t))
            for q in range(W):
                yield ("signal", q, 1, r, s1)
            yield ("wait", 1, range(W), s1)
            for q in range(W):
                yield ("read_peer", q, ("dkv", slot), ("dkv", layer, q, t))
        yield ("collective", f"grads{t}")


@pytest.mark.parametrize("W", [2, 4, 8])
def test_context_parallel_protocol(W):
    explore(lambda: [cp_rank(r, W, 3, 2) for r in range(W)], schedules=80)


def test_context_parallel_single_dkv_buffer_races():
    """The dk|dv partial buffers must alternate: with one buffer a fast rank
    writes the next layer's partial while a slow rank still sums this
    layer's rows from it."""
    with pytest.raises(ProtocolError):
        explore(lambda: [cp_rank(r, 4, 3, 2, dkv_buffers=1) for r in range(4)], schedules=150)


# ------------------------------------------- ZeRO step with overlapped RS


def zero_overlap_rank(r: int, W: int, spans: int, steps: int, side_waits_block: bool = True):
    """``PeerDataParallel.attach_overlap``: as each block's backward ends, the
    main stream records an event and the side (communication) stream runs
    ``zero_rs`` over that block's gradient span (flag slot 0, the sequence
    number of the call, the same order on every rank); after the backward the
    main stream waits for the side stream, reduces what remains (span
    ``spans``: embedding, norms) itself, and runs the norm all-reduce,
    ``zero_adamw_ag`` and ``zero_publish`` as in the plain step.  Returns the
    (rank, main) and (rank, side) actors."""
    calls = {"n": 0}
    shared = {"epoch": 0}

    def rs(span, seq):
        for p in range(W):
            yield ("signal", p, "zero0", r, seq)
        yield ("wait", "zero0", range(W), seq)
        for p in range(W):
            yield ("read_peer", p, ("grad", span, r), ("g", p, span, shared["t"]))
        yield ("write", r, ("grad", span, r), ("mean", span, shared["t"]))

    def main():
        for t in range(1, steps + 1):
            shared["t"] = t
            for sp in range(spans + 1):
                for s in range(W):
                    yield ("read", ("comp", sp, s), ("w", t - 1))     # forward
            for sp in reversed(range(spans + 1)):                      # backward, last block first
                for s in range(W):
                    yield ("write", r, ("grad", sp, s), ("g", r, sp, t))
                if sp < spans:
                    yield ("record", ("block", t, sp))
            yield ("wait_event", ("side_done", t))
            base = shared["epoch"]
            yield from rs(spans, base + spans + 1)                    # the remainder, on main
            shared["epoch"] = base + spans + 1
            yield ("collective", f"norm{t}")
            for sp in range(spans + 1):
                yield ("read", ("grad", sp, r), ("mean", sp, t))
                for p in range(W):
                    yield ("write", p, ("comp", sp, r), ("w", t))
            for p in range(W):
                yield ("signal", p, "zero1", r, t)
            yield ("wait", "zero1", range(W), t)

    def side():
        for t in range(1, steps + 1):
            base = (t - 1) * (spans + 1)
            for k, sp in enumerate(reversed(range(spans))):           # hooks fire in backward order
                if side_waits_block:
                    yield ("wait_event", ("block", t, sp))
                yield from rs(sp, base + k + 1)
            yield ("record", ("side_done", t))

    return [(r, main()), (r, side())]


def _overlap(W, spans, steps, side_waits_block=True):
    def make():
        init = _init_zero_spans(W, spans)
        out = []
        for r in range(W):
            (rm, m), (rs_, sd) = zero_overlap_rank(r, W, spans, steps, side_waits_block)

            def chain(r=r, m=m):
                yield from init(r)
                yield from m

            def side_after_init(r=r, sd=sd):
                yield ("wait_event", "init")
                yield from sd
            out += [(r, chain()), (r, side_after_init())]
        return out
    return make


def _init_zero_spans(W, spans):
    def gen(r):
        for sp in range(spans + 1):
            for s in range(W):
                yield ("write", r, ("comp", sp, s), ("w", 0))
        yield ("collective", "init")
        yield ("record", "init")
    return gen


@pytest.mark.parametrize("W", [2, 4])
def test_zero_step_overlapped_reduce_scatter_protocol(W):
    explore(_overlap(W, spans=3, steps=2), schedules=150)


def test_overlapped_reduce_scatter_needs_the_block_event():
    """A side-stream reduce-scatter that does not wait for its block's
    backward reads a peer's gradient before the peer has written it."""
    with pytest.raises(ProtocolError):
        explore(_overlap(4, spans=3, steps=2, side_waits_block=False), schedules=150)
