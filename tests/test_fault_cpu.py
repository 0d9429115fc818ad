"""Host-side failure detection: watchdog, fault injector (no GPU involved)."""

import time

import pytest


def test_step_watchdog_reports_overrun():
    from nano_qwen_b200.utils.fault import StepWatchdog
    seen = []
    wd = StepWatchdog(0.2, handler=lambda s, t: seen.append(s))
    with wd.step(7):
        time.sleep(0.5)
    with pytest.raises(TimeoutError):
        wd.check()
    assert seen == [7]
    with wd.step(8):
        pass
    wd.check()  # no new overrun
    wd.close()


def test_fault_injector_raise_and_silent():
    from nano_qwen_b200.utils.fault import FaultInjector

    class HB:
        silent = False

    inj = FaultInjector(rank=1, spec="1:3:raise")
    inj.maybe_fail(2)
    with pytest.raises(RuntimeError):
        inj.maybe_fail(3)
    FaultInjector(rank=0, spec="1:3:raise").maybe_fail(3)  # other rank: nothing happens
    hb = HB()
    FaultInjector(rank=2, spec="2:5:silent").maybe_fail(5, hb)
    assert hb.silent


def test_zigzag_indices_balance():
    from nano_qwen_b200.parallel.context_parallel import zigzag_indices
    cp, S = 4, 64
    parts = [zigzag_indices(S, cp, r) for r in range(cp)]
    allpos = sorted(int(i) for p in parts for i in p)
    assert allpos == list(range(S))
    # causal work (sum of positions + 1) is the same on every rank
    work = [int((p + 1).sum()) for p in parts]
    assert max(work) == min(work)
