"""Failure detection on the GPU without a GPU fault (the reference's analogue:
the command-buffer error check after waitUntilCompleted,
Sources/ImarelloDirect/DirectDiTStep.swift:968-970).

* A bounded device wait is made to run out: aex_selftest_wait launches one
  kernel that waits on a barrier nothing arrives on, with a 1 ms limit instead
  of the library's 2 s; the kernel records a device status and returns. The
  next aex_sync reports AEX_ERR_DEVICE, clears the status, and the context
  keeps working (a fused attention call afterwards is checked).
* aex_sync's host-side deadline: a bounded GPU busy kernel (torch.cuda._sleep,
  a fixed cycle count of about half a second) keeps the stream busy past a
  20 ms deadline, so aex_sync returns AEX_ERR_TIMEOUT; an unbounded aex_sync
  afterwards returns AEX_OK once the kernel has finished."""
import pytest
import torch

from aestrix_b200 import _lib, attention

pytestmark = pytest.mark.gpu


def test_bounded_wait_expiry_is_reported_and_context_survives(cuda_ctx):
    L = _lib.lib()
    s = torch.cuda.Stream()
    assert cuda_ctx.device_status() == 0
    cuda_ctx.check(L.aex_selftest_wait(cuda_ctx.handle, 1000, s.cuda_stream))
    rc = L.aex_sync(cuda_ctx.handle, s.cuda_stream, 10000)
    assert rc == _lib.AEX_ERR_DEVICE
    assert b"device status 7" in L.aex_last_error_string(cuda_ctx.handle)
    assert cuda_ctx.device_status() == 0  # aex_sync cleared it
    # the context still runs work correctly
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 256, 2, 128, generator=g).to(torch.bfloat16).cuda() for _ in range(3))
    out = attention.joint_attention(q, k, v, ctx=cuda_ctx, stream=s)
    ref = torch.softmax((q.float().transpose(1, 2) @ k.float().transpose(1, 2).transpose(-1, -2)) / 128 ** 0.5, -1) @ \
        v.float().transpose(1, 2)
    cuda_ctx.sync(s.cuda_stream)
    err = (out.float().transpose(1, 2) - ref).abs().max().item()
    assert err <= 2e-2, err
    assert cuda_ctx.device_status() == 0


def test_selftest_wait_rejects_out_of_range_limits(cuda_ctx):
    L = _lib.lib()
    assert L.aex_selftest_wait(cuda_ctx.handle, 0, None) == _lib.AEX_ERR_INVALID_ARG
    assert L.aex_selftest_wait(cuda_ctx.handle, 2_000_000, None) == _lib.AEX_ERR_INVALID_ARG


def test_sync_deadline_returns_timeout(cuda_ctx):
    L = _lib.lib()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        torch.cuda._sleep(1_000_000_000)  # ~0.5 s of device time at ~2 GHz, then the kernel ends
    rc = L.aex_sync(cuda_ctx.handle, s.cuda_stream, 20)
    assert rc == _lib.AEX_ERR_TIMEOUT
    assert b"still busy" in L.aex_last_error_string(cuda_ctx.handle)
    assert L.aex_sync(cuda_ctx.handle, s.cuda_stream, 0) == _lib.AEX_OK
    assert cuda_ctx.device_status() == 0
