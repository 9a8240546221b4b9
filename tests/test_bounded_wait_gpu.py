"""The failure path of the bounded device-side waits on one GPU
(rxla_b200_bounded_wait_check with rxla_b200_set_wait_timeout and
rxla_b200_device_status): a wait that nothing satisfies — a fresh mbarrier,
the wait of every TMA ring here, or a device flag, the peer all-reduce's
wait — gives up after the budget, records RXLA_B200_DEADLINE_EXCEEDED and
returns, and the context keeps running work.  The two-rank form, a peer that
skips an all-reduce, is tests/test_tp_gpu.py's
test_bounded_wait_runs_out_and_reports_deadline_exceeded."""
import ctypes

import pytest
import torch

from rxla_b200 import _lib

pytestmark = pytest.mark.gpu

BUDGET_NS = 50_000_000  # 50 ms


def _timed_wait(kind, flag_ptr, target):
    lib = _lib.load()
    torch.cuda.synchronize()
    lib.rxla_b200_device_status(1)  # start from a clear status word
    _lib.call("rxla_b200_set_wait_timeout", BUDGET_NS)
    try:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        e0.record()
        _lib.call("rxla_b200_bounded_wait_check", kind, ctypes.c_void_p(flag_ptr),
                  ctypes.c_uint64(target), s)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3, lib.rxla_b200_device_status(1)  # read and clear
    finally:
        _lib.call("rxla_b200_set_wait_timeout", 4_000_000_000)


def _gpu_answers():
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    return float((x * 2).sum().item()) == float(1023 * 1024)


def test_mbarrier_wait_runs_out_and_the_kernel_returns(cuda):
    sec, status = _timed_wait(0, None, 0)
    print(f"mbarrier wait gave up after {sec * 1e3:.1f} ms")
    assert status == _lib.DEADLINE_EXCEEDED
    assert 0.045 <= sec < 1.0
    assert _gpu_answers()


def test_flag_wait_runs_out_then_passes_once_the_flag_is_set(cuda):
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    sec, status = _timed_wait(1, flag.data_ptr(), 1)
    print(f"flag wait gave up after {sec * 1e3:.1f} ms")
    assert status == _lib.DEADLINE_EXCEEDED
    assert 0.045 <= sec < 1.0
    flag.fill_(1)
    sec, status = _timed_wait(1, flag.data_ptr(), 1)
    assert status == 0
    assert sec < 0.01
    assert _gpu_answers()
