"""The allocation-free reduction entry point, tl_reduce_noalloc.

For callers that cannot allocate device memory when they need a reduction
(code inside a CUDA stream capture, hosts whose device memory is owned by
another allocator, foreign-language callers without a CUDA allocator), the
library offers tl_reduce without a workspace argument: its partial sums
live in a fixed 4 MiB array inside the library.  This checks, through the C
ABI, that it returns what tl_reduce (caller workspace) returns, on two calls
in a row that reuse the shared array, and that it refuses reductions too big
for the array.  Collected last (file name) so a failure here cannot hide
other tests; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from templit_b200 import capi
from tests.helpers import Dev

pytestmark = pytest.mark.gpu


def run_noalloc(dev, x, out_shape, op=capi.TL_REDUCE_SUM):
    tx = dev.t(x)
    out = dev.empty(out_shape)
    dev.call("tl_reduce_noalloc", op, dev.p(tx), capi.shape_arr(x.shape), x.ndim, dev.p(out),
             capi.shape_arr(out_shape), len(out_shape), dev.stream)
    return dev.host(out)


@pytest.mark.parametrize("shape,out_shape", [
    ((12288, 1536), (1536,)),        # split columns: partials in the shared array
    ((64, 192, 384), (64, 192, 1)),  # rows, no partials
    ((4_000_000,), (1,)),            # split rows: partials again, different layout
])
def test_noalloc_matches_workspace_reduce_two_calls_in_a_row(shape, out_shape):
    dev = Dev()
    rng = np.random.default_rng(42)
    for call in range(2):
        x = rng.standard_normal(shape).astype(np.float32)
        want = dev.reduce("sum", x, out_shape)
        got = run_noalloc(dev, x, out_shape)
        # same plan, same kernels: the results agree to the last bit; the
        # tolerance of the other reduction tests (1e-6 of sum |x|) is the bound
        scale = np.abs(x).sum() if len(out_shape) == 1 and out_shape[0] == 1 else \
            np.abs(x).max() * x.size / max(1, int(np.prod(out_shape)))
        np.testing.assert_allclose(got, want, rtol=0, atol=1e-6 * scale + 1e-6,
                                   err_msg=f"call {call}")
        np.testing.assert_array_equal(got, want)


def test_noalloc_max_and_size_limit():
    dev = Dev()
    x = np.random.default_rng(1).standard_normal((64, 6, 192, 192)).astype(np.float32)
    np.testing.assert_array_equal(run_noalloc(dev, x, (64, 6, 192, 1), capi.TL_REDUCE_MAX),
                                  x.max(axis=-1, keepdims=True))
    lib = capi.cuda_lib()
    assert lib.tl_reduce_noalloc_max_workspace() == 4 << 20
    # [64, 606204] -> [606204]: two split planes of 606,204 partials = 4.85 MB > 4 MiB
    big = (ctypes.c_uint32 * 2)(64, 606204)
    small = (ctypes.c_uint32 * 1)(606204)
    need = lib.tl_reduce_workspace_size(big, 2, small, 1)
    assert need > lib.tl_reduce_noalloc_max_workspace()
    t = dev.empty((64, 606204))
    o = dev.empty((606204,))
    rc = lib.tl_reduce_noalloc(capi.TL_REDUCE_SUM, dev.p(t), big, 2, dev.p(o), small, 1,
                               dev.stream)
    assert rc == capi.TL_ERR_RANGE
    assert b"4 MiB" in lib.tl_last_error()
