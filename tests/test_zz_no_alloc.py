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
    # the planner keeps every split plan well inside the built-in array (its
    # partial planes are bounded by the threads it wants in flight), so the
    # TL_ERR_RANGE guard is never reached by a valid reduction
    for shape, out in [((64, 606204), (606204,)), ((64, 606205), (606205,)),
                       ((1, 1 << 27), (1, 1)), ((4096, 3, 7), (1, 3, 1)), ((12288, 384), (1, 384))]:
        a = (ctypes.c_uint32 * len(shape))(*shape)
        b = (ctypes.c_uint32 * len(out))(*out)
        need = lib.tl_reduce_workspace_size(a, len(shape), b, len(out))
        assert need <= lib.tl_reduce_noalloc_max_workspace(), (shape, need)
