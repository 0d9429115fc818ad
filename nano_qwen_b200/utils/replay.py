"""Deterministic-replay check: run one training step twice from the same state
and compare everything it produced.

Race detection without a sanitizer (compute-sanitizer is not available on the
target GPU pool): a kernel with a race, a missing barrier or an unordered
read of a buffer that another kernel still writes produces results that change
from run to run.  ``replay_step`` snapshots the engine's complete state
(fp32 master, bf16 compute copy, gradients, Adam moments, step counters,
scheduler), runs ``train_step`` on a batch, restores the snapshot, runs it
again and reports, per parameter, whether the two updates are bit-identical
and the largest difference.

Expected nondeterminism is narrow and bounded: the attention backward adds
the dQ partials of different key blocks with TMA bulk add-reductions, the
embedding backward scatters rows with fp32 atomics and the cross-entropy adds
its per-row losses with atomics, so those sums can round differently from run
to run (relative differences around 1e-7).  Everything else is deterministic: the forward pass,
the GEMMs (one CTA owns each output tile, fixed K order) and the optimizer.
"""

from __future__ import annotations

from typing import Dict, List

import torch


def _snapshot(engine) -> Dict[str, object]:
    st = engine.store
    opt = engine.optimizer
    snap = {"master": st.master.clone(), "grad": st.grad.clone(),
            "compute": st.compute.clone() if st.compute is not None else None,
            "m": opt.exp_avg.clone(), "v": opt.exp_avg_sq.clone(), "step": opt.step_count,
            "sched": engine.scheduler.state_dict(),
            "groups": [dict(g) for g in opt.param_groups]}
    return snap


@torch.no_grad()
def _restore(engine, snap) -> None:
    st = engine.store
    opt = engine.optimizer
    st.master.copy_(snap["master"])
    st.grad.copy_(snap["grad"])
    if snap["compute"] is not None:
        st.compute.copy_(snap["compute"])
    opt.exp_avg.copy_(snap["m"])
    opt.exp_avg_sq.copy_(snap["v"])
    opt.step_count = snap["step"]
    engine.scheduler.load_state_dict(snap["sched"])
    for g, sg in zip(opt.param_groups, snap["groups"]):
        g.update({k: v for k, v in sg.items() if k != "params"})


def replay_step(engine, micro_batches: List[dict]) -> dict:
    """Two runs of ``engine.train_step(micro_batches)`` from one state.

    Returns ``{"loss_equal", "loss": (a, b), "identical": [names],
    "differs": {name: max_abs_diff}}`` and leaves the engine in the state
    after the second run."""
    snap = _snapshot(engine)
    out_a = engine.train_step(micro_batches)
    loss_a = float(out_a["loss"])
    after_a = engine.store.master.clone()
    _restore(engine, snap)
    out_b = engine.train_step(micro_batches)
    loss_b = float(out_b["loss"])
    after_b = engine.store.master
    identical, differs = [], {}
    for n, p in zip(engine.store.names, engine.store.params):
        o = engine.store.offsets[id(p)]
        a = after_a[o:o + p.numel()]
        b = after_b[o:o + p.numel()]
        if torch.equal(a, b):
            identical.append(n)
        else:
            differs[n] = float((a - b).abs().max())
    return {"loss_equal": loss_a == loss_b, "loss": (loss_a, loss_b), "identical": identical,
            "differs": differs}


@torch.no_grad()
def replay_forward(model, input_ids: torch.Tensor) -> bool:
    """True when two forward passes give bit-identical logits."""
    a = model(input_ids)["logits"]
    b = model(input_ids)["logits"]
    return bool(torch.equal(a, b))
