"""Failure detection on the device without a GPU fault: every device-side wait
in the library is bounded, gives up after its limit, records a code in the
context's device error word and returns, so that lt_sync reports
LT_ETIMEOUT and the context stays usable.

lt_selftest_wait runs the library's own wait helpers (the grid barrier of
the persistent kernels, the mbarrier wait of every TMA tile) in a two-CTA
kernel with a short test limit; kinds 1 and 2 wait for one arrival more
than ever comes.  The reference has no device timeouts: on a GPU error its
forward loop falls back to the CPU (src/model/gemma4/forward.zig:456-480).
"""
from __future__ import annotations

import time

import numpy as np
import pytest

from test_gpu_parity import dev, empty, host

pytestmark = pytest.mark.gpu

LIMIT_US = 20_000  # 20 ms: the test-only limit (the kernels' own is 2 s)


def _argmax_works(ctx):
    x = np.zeros(5000, np.float32)
    x[1234] = 3.0
    out = empty(1, "int32")
    ctx.argmax(dev(x), 5000, 1, out)
    ctx.sync()
    assert int(host(out)[0]) == 1234


def test_grid_barrier_that_completes(ctx, pkg):
    lib = pkg.load_library()
    assert lib.lt_selftest_wait(ctx.ptr, 0, 1_000_000) == 0
    ctx.sync()


@pytest.mark.parametrize("kind", [1, 2], ids=["grid_barrier", "mbarrier"])
def test_wait_that_runs_out_returns_timeout(ctx, pkg, kind):
    lib = pkg.load_library()
    t0 = time.perf_counter()
    assert lib.lt_selftest_wait(ctx.ptr, kind, LIMIT_US) == 0  # asynchronous: the launch itself succeeds
    with pytest.raises(pkg.LtError) as err:
        ctx.sync()
    assert err.value.status == 5, err.value  # LT_ETIMEOUT
    assert time.perf_counter() - t0 < 10.0
    ctx.sync()  # the error word was read and cleared
    _argmax_works(ctx)  # the context is still usable
    # and the barrier counters kept their invariant: a complete barrier still completes
    assert lib.lt_selftest_wait(ctx.ptr, 0, 1_000_000) == 0
    ctx.sync()


def test_selftest_rejects_bad_arguments(ctx, pkg):
    lib = pkg.load_library()
    assert lib.lt_selftest_wait(ctx.ptr, 3, LIMIT_US) == 1
    assert lib.lt_selftest_wait(ctx.ptr, 1, 0) == 1
    assert lib.lt_selftest_wait(ctx.ptr, 1, 3_000_000) == 1
    ctx.sync()
