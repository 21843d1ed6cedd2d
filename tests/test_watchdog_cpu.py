"""CPU: the host-side watchdog that guards vk_gemm_sharded's NCCL all-gather (no GPU, no NCCL).

A fake completion query stands in for the gather: one that never reports "done" (a rank that never
joins) must end in VK_ERR_NCCL after the deadline with exactly one abort (ncclCommAbort on the real
path); one that reports a failure must abort at once; one that completes must not abort."""
import ctypes
import time

import pytest

vk = pytest.importorskip("vibekernel_b200")


def _run(deadline_ms, done_after, fail_at=0):
    aborted = ctypes.c_int32(-1)
    polls = ctypes.c_int64(0)
    t0 = time.perf_counter()
    rc = vk.lib.vk_debug_watchdog(deadline_ms, done_after, fail_at, ctypes.byref(aborted), ctypes.byref(polls))
    return rc, aborted.value, polls.value, time.perf_counter() - t0


def test_never_done_aborts_after_deadline():
    rc, aborted, polls, dt = _run(200, -1)
    assert rc == vk.VK_ERR_NCCL and aborted == 1
    assert 0.2 <= dt < 5.0 and polls > 1
    assert "did not complete within 200 ms" in vk.last_error()


def test_failure_aborts_immediately():
    rc, aborted, polls, dt = _run(10_000, -1, fail_at=3)
    assert rc == vk.VK_ERR_NCCL and aborted == 1 and polls == 3 and dt < 1.0
    assert "failed" in vk.last_error()


@pytest.mark.parametrize("done_after", [0, 1, 50])
def test_completion_does_not_abort(done_after):
    rc, aborted, polls, dt = _run(10_000, done_after)
    assert rc == vk.VK_OK and aborted == 0 and polls == done_after + 1 and dt < 1.0


def test_gather_timeout_option():
    vk.set_option("gather_timeout_ms", 1234)
    with pytest.raises(vk.VkError):
        vk.set_option("gather_timeout_ms", 0)
    vk.set_option("gather_timeout_ms", 60000)
