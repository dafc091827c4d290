"""Failure detection on the device, the counterpart of the reference's drain and timeout tests
(board_package/tests/test_drain.py:23-159, runtime/memcpy.py:289-312): a bounded wait that nothing completes runs
out, the kernel returns with a watchdog code instead of hanging, the host reports it as the reference's TimeoutError,
the runtime's own deadline fires while the kernel still waits, and the context stays usable for the next launch.

The wait that runs out is the probe's (tempo_wait_probe): an mbarrier nobody arrives on, with a limit of 50 ms to
1 s. Nothing here faults or traps the GPU."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

PROBE_CODE = 6


@pytest.fixture(scope="module")
def rt():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tempo_compiler_b200 import runtime
    runtime.minitpuSetDevice("minitpu")
    return runtime


def _probe(arrive: int, limit_s: float, stream=None) -> None:
    from tempo_compiler_b200 import lib
    lib.call("tempo_wait_probe", arrive, int(limit_s * 1e9), stream)


def test_a_wait_that_runs_out_is_reported_and_drain_says_so(rt) -> None:
    _probe(0, 0.05)
    assert rt.minitpuDrain(timeout=5.0) is False       # the watchdog expiry, read and cleared by the drain
    assert rt.minitpuDrain(timeout=5.0) is True        # nothing left: the next drain is clean


def test_the_runtime_deadline_fires_while_the_kernel_still_waits(rt) -> None:
    from tempo_compiler_b200 import lib
    _probe(0, 1.0)
    with pytest.raises(TimeoutError, match="did not finish"):
        lib.call("tempo_sync", 0.05)
    with pytest.raises(TimeoutError, match="bounded wait"):
        lib.call("tempo_sync", 5.0)
    code = ctypes.c_int32(-1)
    lib.call("tempo_watchdog", ctypes.byref(code))
    assert code.value == 0


def test_a_completed_wait_sets_no_code(rt) -> None:
    _probe(1, 1.0)
    assert rt.minitpuDrain(timeout=5.0) is True


def test_the_watchdog_names_the_probe_on_another_stream(rt) -> None:
    from tempo_compiler_b200 import ops
    stream = torch.cuda.current_stream()
    _probe(0, 0.02, stream.cuda_stream)
    torch.cuda.synchronize()
    assert ops.watchdog() == PROBE_CODE
    assert ops.watchdog() == 0                         # read once, cleared


def test_the_context_stays_usable_after_an_expiry(rt) -> None:
    from tempo_compiler_b200 import ops
    _probe(0, 0.05)
    assert rt.minitpuDrain(timeout=5.0) is False
    x = torch.randn((64, 768), device="cuda").to(torch.bfloat16)
    gamma = torch.ones(768, device="cuda", dtype=torch.bfloat16)
    beta = torch.zeros(768, device="cuda", dtype=torch.bfloat16)
    out = ops.layernorm(x, gamma, beta)
    ref = torch.nn.functional.layer_norm(x.float(), (768,), eps=1e-5)
    torch.cuda.synchronize()
    assert ops.watchdog() == 0
    assert float((out.float() - ref).abs().max()) < 0.05
    words = np.arange(16, dtype=np.uint32)
    region = rt.minitpuHostAlloc(64)
    region.view[:16] = words
    address = rt.minitpuMalloc(64)
    try:
        rt.minitpuMemcpy(address, region, 64, rt.MemcpyKind.HostToDevice)
        region.view[:16] = 0
        rt.minitpuMemcpy(region, address, 64, rt.MemcpyKind.DeviceToHost)
        np.testing.assert_array_equal(region.view[:16], words)
    finally:
        rt.minitpuFree(address)
        rt.minitpuHostReset()


def test_the_probe_refuses_a_limit_past_ten_seconds(rt) -> None:
    with pytest.raises(ValueError):
        _probe(0, 11.0)
    with pytest.raises(ValueError):
        _probe(0, 0.0)
