"""Failure detection on the GPU without a GPU fault: a bounded device wait that nothing will
satisfy gives up after its limit, the call reports K3C_ETIMEOUT, and the CUDA context stays
usable for the next call (the waits in every pipelined kernel use the same helpers with a
~2 s limit)."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", [0, 1])
def test_bounded_wait_gives_up_and_reports(k3, kind):
    L = k3.lib()
    t0 = time.perf_counter()
    rc = L.k3c_selftest_wait(kind, 50.0, None)
    dt = time.perf_counter() - t0
    assert rc == -4, L.k3c_last_error()                     # K3C_ETIMEOUT
    assert b"gave up" in L.k3c_last_error()
    assert 0.04 < dt < 5.0


def test_satisfied_wait_returns_ok_and_context_is_usable(k3, ora):
    import torch
    L = k3.lib()
    assert L.k3c_selftest_wait(0, 20.0, None) == -4
    assert L.k3c_selftest_wait(2, 20.0, None) == 0
    g = k3.synth.rng(5)
    packed, scales = k3.synth.mxfp4_matrix(g, 8, 64)
    got = k3.mxfp4_dequant(torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda()).cpu().numpy()
    want = ora.mxfp4_dequant(packed, scales)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_selftest_rejects_bad_arguments(k3):
    L = k3.lib()
    assert L.k3c_selftest_wait(3, 10.0, None) == -1
    assert L.k3c_selftest_wait(0, 5000.0, None) == -1
