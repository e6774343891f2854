"""GPU: failure detection of the bounded device-side waits, and per-call
precision.

Every pipeline wait of the contraction kernels gives up after a time limit,
records a code in the device status word and returns, so a producer that
never arrives turns into AGPU_ERR_TIMEOUT on the next agpu_synchronize /
agpu_read instead of a hung GPU.  agpu_selftest_wait_timeout makes such a
wait run out on purpose: one warp waits ~1 ms on an mbarrier that nothing
arrives on (no TMA, no tensor cores, no tensor memory).  The tests check the
status the host reads, that the status word is cleared, and that the next
contraction on the same device is still correct.
"""
from __future__ import annotations

import threading

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SELFTEST_CODE = 0x7E57  # AGPU_SELFTEST_WAIT_CODE


def _matmul_ok(dev, orc, n=256, tol=1e-3, seed=5):
    r = np.random.default_rng(seed)
    a = r.uniform(-1, 1, n * n).astype(np.float32)
    b = r.uniform(-1, 1, n * n).astype(np.float32)
    c = dev.read(dev.matmul(dev.upload(a), dev.upload(b), n, n, n))
    err = orc.rel_fro(c, orc.matmul(a, b, n, n, n))
    assert err <= tol, f"matmul after the expired wait: rel_fro {err}"


def test_expired_wait_reports_timeout_then_device_recovers(dev, orc):
    from any_gpu import AnyGpuError
    dev.synchronize()
    dev.selftest_wait_timeout(1000)
    with pytest.raises(AnyGpuError) as e:
        dev.synchronize()
    assert e.value.status == 6, e.value
    assert f"0x{SELFTEST_CODE:x}" in str(e.value)
    dev.synchronize()  # the status word was cleared by the read-back
    _matmul_ok(dev, orc)


def test_expired_wait_reported_by_read(dev, orc):
    from any_gpu import AnyGpuError
    buf = dev.upload(np.arange(16, dtype=np.float32))
    dev.selftest_wait_timeout(500)
    with pytest.raises(AnyGpuError) as e:
        dev.read(buf)
    assert e.value.status == 6
    assert np.array_equal(dev.read(buf), np.arange(16, dtype=np.float32))
    _matmul_ok(dev, orc, n=512)


def test_expired_wait_on_caller_stream(dev, orc):
    import torch
    from any_gpu import AnyGpuError
    s = torch.cuda.Stream()
    dev.selftest_wait_timeout(300, stream=s.cuda_stream)
    s.synchronize()
    with pytest.raises(AnyGpuError) as e:
        dev.synchronize()
    assert e.value.status == 6
    dev.synchronize()
    _matmul_ok(dev, orc)


def test_selftest_rejects_limits_out_of_range(dev):
    from any_gpu import AnyGpuError
    for bad in (0, 1_000_001):
        with pytest.raises(AnyGpuError) as e:
            dev.selftest_wait_timeout(bad)
        assert e.value.status == 2
    dev.synchronize()


def test_thread_precision_is_per_call_and_per_thread(dev, orc):
    """agpu_set_thread_precision: 3xTF32 inside the block on this thread only;
    the device's own setting and a concurrent thread keep TF32."""
    from any_gpu import GpuDevice, _lib
    n = 512
    r = np.random.default_rng(11)
    a = r.uniform(-1, 1, n * n).astype(np.float32)
    b = r.uniform(-1, 1, n * n).astype(np.float32)
    want = (a.reshape(n, n).astype(np.float64) @ b.reshape(n, n).astype(np.float64)).reshape(-1)
    ga, gb = dev.upload(a), dev.upload(b)

    def err():
        c = dev.read(dev.matmul(ga, gb, n, n, n))
        return orc.rel_fro(c, want)

    other = {}

    def worker():
        other["mode"] = _lib.load().agpu_get_thread_precision()
        other["err"] = err()

    assert dev.get_precision() == "tf32"
    e_tf32 = err()
    with GpuDevice.precision("tf32x3"):
        assert dev.get_precision() == "tf32"  # device setting untouched
        e_x3 = err()
        t = threading.Thread(target=worker)
        t.start()
        t.join()
    e_after = err()
    assert e_x3 <= 1e-5, e_x3
    assert e_tf32 > 1e-5 and e_after > 1e-5, (e_tf32, e_after)
    assert other["mode"] == -1
    assert other["err"] > 1e-5, other


def test_wait_flags_expires_without_a_signal(dev, orc):
    """The end-of-step wait of the copy-engine gathers: a flag no peer ever
    sets makes agpu_wait_flags give up after its limit and report
    AGPU_ERR_TIMEOUT (code 0x5157) -- a peer that died shows up as an error,
    not a hung GPU -- and the device stays usable."""
    import ctypes as C

    import torch
    from any_gpu import AnyGpuError, _lib
    lib = _lib.load()
    flags = torch.zeros(3, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    assert lib.agpu_wait_flags(dev.handle, C.c_void_p(flags.data_ptr()), 3, 1, 2000, None) == 0
    with pytest.raises(AnyGpuError) as e:
        dev.synchronize()
    assert e.value.status == 6 and "0x5157" in str(e.value)
    dev.synchronize()
    _matmul_ok(dev, orc)


def test_signal_then_wait_flags_round_trip(dev):
    """agpu_signal_peers stores the step into each flag word (here local ones
    standing in for the peers' slots) and agpu_wait_flags returns once every
    word has reached it; serial-number compare across the 2^32 wrap."""
    import ctypes as C

    import torch
    from any_gpu import _lib
    lib = _lib.load()
    flags = torch.zeros(4, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    slots = (C.c_void_p * 4)(*[flags.data_ptr() + 4 * i for i in range(4)])
    for value in (1, 2, 0xFFFFFFFF, 0):  # the last two wrap
        assert lib.agpu_signal_peers(dev.handle, slots, 4, value, None) == 0
        assert lib.agpu_wait_flags(dev.handle, C.c_void_p(flags.data_ptr()), 4, value, 1_000_000,
                                   None) == 0
        dev.synchronize()
    assert flags.cpu().tolist() == [0, 0, 0, 0]
    assert lib.agpu_wait_flags(dev.handle, C.c_void_p(flags.data_ptr()), 33, 1, 10, None) == 2
    assert lib.agpu_signal_peers(dev.handle, slots, 17, 1, None) == 2
