"""Failure detection on one GPU: a bounded device wait that runs out returns
an error status through the device error word, and the context stays usable.

Nothing here faults, traps or hangs the GPU: the wait is on a local flag that
nothing sets, with the peer-flag limit lowered to 50 ms, so the kernel gives
up, records ``kErrTimeoutPeer`` and returns."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_flag_wait_runs_out_and_reports():
    from nano_qwen_b200.ops import ext
    from nano_qwen_b200.utils.fault import (DeviceWaitTimeout, check_device_errors, get_wait_limits,
                                            set_wait_limits)
    E = ext()
    torch.cuda.synchronize()
    E.error_flag_clear()
    old_mbar, old_peer = get_wait_limits()
    assert old_mbar == pytest.approx(2.0) and old_peer == pytest.approx(20.0)
    # the expert-parallel flag block of a one-rank "group": channel 0, rank 0
    flags = torch.zeros(4 * 8, dtype=torch.int32, device="cuda")
    counts = torch.zeros(8, dtype=torch.int32, device="cuda")
    try:
        set_wait_limits(peer_s=0.05)
        assert get_wait_limits()[1] == pytest.approx(0.05)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        E.ep_wait([flags.data_ptr()], [counts.data_ptr()], 0, 0, 1)  # flag never reaches 1
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        ms = e0.elapsed_time(e1)
        assert 45.0 <= ms < 1000.0, f"wait lasted {ms:.1f} ms on the device"
        assert wall < 5.0
        assert E.error_flag_read() == 6  # kErrTimeoutPeer
        with pytest.raises(DeviceWaitTimeout, match="peer flag wait timed out"):
            check_device_errors()
        assert E.error_flag_read() == 0  # cleared by check_device_errors
        # the context is still usable: publish the flag, and the same wait passes at once
        E.ep_signal([flags.data_ptr()], [counts.data_ptr()], 0, 0, 1)
        E.ep_wait([flags.data_ptr()], [counts.data_ptr()], 0, 0, 1)
        torch.cuda.synchronize()
        assert E.error_flag_read() == 0
        x = torch.randn(256, 256, device="cuda", dtype=torch.bfloat16)
        assert torch.isfinite(x @ x).all()
    finally:
        set_wait_limits(old_mbar, old_peer)
        E.error_flag_clear()
    assert get_wait_limits() == pytest.approx((old_mbar, old_peer))
