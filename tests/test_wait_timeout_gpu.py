"""The bounded on-device waits: every mbarrier wait of the tensor-core
kernels gives up after a limit, raises TL_FLAG_TIMEOUT in the device status
word, frees its TMEM and returns, so a lost arrival becomes an error the
host reads instead of a hung GPU.  tl_check_wait_timeout runs that path on
an mbarrier nothing arrives at, with a limit of a few milliseconds; the GPU
stays usable (a tensor-core GEMM, which allocates TMEM, runs right after)."""
import ctypes

import numpy as np
import pytest

from oracle import ops
from templit_b200 import capi
from tests.helpers import Dev

pytestmark = pytest.mark.gpu


def test_wait_gives_up_and_reports():
    dev = Dev()
    lib = dev.lib
    flags = ctypes.c_uint32()
    capi.check(lib.tl_device_status(ctypes.byref(flags), dev.stream), lib, "status")  # clear
    waited = dev.torch.zeros(1, dtype=dev.torch.int32, device=dev.dev)
    capi.check(lib.tl_check_wait_timeout(5_000_000, ctypes.c_void_p(waited.data_ptr()),
                                         dev.stream), lib, "wait check")
    capi.check(lib.tl_device_status(ctypes.byref(flags), dev.stream), lib, "status")
    assert flags.value & capi.TL_FLAG_TIMEOUT
    us = int(dev.host(waited)[0])
    assert 5_000 <= us < 1_000_000, us  # gave up after the limit, not never
    # the status word was cleared by the read; TMEM was freed: a tensor-core
    # GEMM (which allocates TMEM) runs and is right
    capi.check(lib.tl_device_status(ctypes.byref(flags), dev.stream), lib, "status")
    assert flags.value == 0
    r = np.random.default_rng(0)
    a = r.standard_normal((512, 384)).astype(np.float32)
    b = r.standard_normal((384, 256)).astype(np.float32)
    got = dev.gemm(a, b)
    want = ops.gemm(a, b)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-3
    assert lib.tl_check_wait_timeout(2_000_000_000, ctypes.c_void_p(waited.data_ptr()),
                                     dev.stream) == capi.TL_ERR_RANGE
