"""GPU: the allocation-free group norm entry point.

agpu_group_norm_noalloc serves callers that may not allocate device memory
themselves (a process that owns all device memory through its own arena, a
foreign host that passes only device pointers and a stream, a latency-
critical loop).  Its scratch is a fixed array inside the library, so this
test checks that two calls in a row, with different shapes, match the
regular group norm entry point, and that a shape beyond the fixed scratch is
rejected.  The file is named so that pytest collects it last.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(dev, X, G, B, Y, n, c, s, g, eps, swish):
    from any_gpu import _check, _lib
    _check(_lib.load().agpu_group_norm_noalloc(
        C.c_void_p(X.device_ptr), C.c_void_p(G.device_ptr), C.c_void_p(B.device_ptr),
        C.c_void_p(Y.device_ptr), n, c, s, g, C.c_float(eps), int(swish),
        C.c_void_p(dev.stream)))


def test_group_norm_noalloc_matches_group_norm(dev, orc):
    shapes = [(2, 64, 1024, 32, False),  # 2048-element groups: one chunk each
              (3, 12, 37, 4, True),       # ragged spatial, fused swish
              (1, 4, 300000, 2, False)]   # 600k-element groups -> 74 chunks each
    r = np.random.default_rng(2024)
    for n, c, s, g, swish in shapes:
        x = r.standard_normal(n * c * s).astype(np.float32)
        gamma = (1 + 0.1 * r.standard_normal(c)).astype(np.float32)
        beta = (0.1 * r.standard_normal(c)).astype(np.float32)
        X, G, B = dev.upload(x), dev.upload(gamma), dev.upload(beta)
        fn = dev.group_norm_swish if swish else dev.group_norm
        want = dev.read(fn(X, G, B, n, c, s, g, 1e-5))
        for _ in range(2):  # two calls in a row share the fixed scratch
            Y = dev.alloc(n * c * s)
            _noalloc(dev, X, G, B, Y, n, c, s, g, 1e-5, swish)
            got = dev.read(Y)
            assert orc.rel_fro(got, want) <= 1e-5


def test_group_norm_noalloc_rejects_oversized_scratch(dev):
    from any_gpu import AnyGpuError
    X = dev.alloc(4)
    # 65535 groups x 2 chunks of 8192 elements = 131070 partials > 65536
    with pytest.raises(AnyGpuError) as e:
        _noalloc(dev, X, X, X, X, 65535, 1, 16384, 1, 1e-5, False)
    assert e.value.status == 7
    with pytest.raises(AnyGpuError) as e:
        _noalloc(dev, X, X, X, X, 1, 5, 4, 2, 1e-5, False)
    assert e.value.status == 1
