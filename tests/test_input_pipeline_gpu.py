"""Training input pipeline: tlg_loader_* draws the
same batches as the reference's own Dataset::load_tokens + Loader::get_batch
(src/model_utils/dataset.cpp, loader.cpp, compiled into the host oracle)
from the same token file and seed - bit-exact - into pinned memory, and a
training step fed from it equals one fed the same batch from numpy."""
import ctypes

import numpy as np
import pytest

from templit_b200 import capi
from tests.test_gpt_gpu import CudaGPT, config, oracle

pytestmark = pytest.mark.gpu


def token_file(tmp_path, n=20000, seed=0):
    rng = np.random.default_rng(seed)
    tokens = rng.integers(0, 2048, n).astype(np.uint32)
    tokens[rng.integers(0, n, 40)] = 256  # end-of-text marks (the split looks for one)
    path = tmp_path / "tokens.bin"
    tokens.tofile(path)
    return path


class Loader:
    def __init__(self, path, fraction, validation, batch, seq, seed):
        self.lib = capi.gpt_lib()
        self.h = ctypes.c_void_p()
        self.shape = (batch, seq)
        capi.check(self.lib.tlg_loader_create(str(path).encode(), fraction, int(validation),
                                              batch, seq, seed, ctypes.byref(self.h)),
                   self.lib, "loader")

    def next(self):
        x, y = capi.U32P(), capi.U32P()
        capi.check(self.lib.tlg_loader_next(self.h, ctypes.byref(x), ctypes.byref(y)), self.lib,
                   "next")
        n = self.shape[0] * self.shape[1]
        return (np.ctypeslib.as_array(x, (n,)).reshape(self.shape).copy(),
                np.ctypeslib.as_array(y, (n,)).reshape(self.shape).copy(), x, y)

    def close(self):
        self.lib.tlg_loader_destroy(self.h)


@pytest.mark.parametrize("validation,seed", [(False, 1), (True, 2)])
def test_batches_equal_the_reference_loader(tmp_path, validation, seed):
    cg = oracle()
    path = token_file(tmp_path)
    want_x, want_y = cg.loader_batches(path, 0.95, validation, 4, 32, seed, 6)
    ld = Loader(path, 0.95, validation, 4, 32, seed)
    try:
        for i in range(6):
            x, y, _, _ = ld.next()
            np.testing.assert_array_equal(x, want_x[i])
            np.testing.assert_array_equal(y, want_y[i])
    finally:
        ld.close()


def test_step_fed_from_the_pipeline(tmp_path):
    path = token_file(tmp_path, seed=3)
    ld = Loader(path, 0.95, False, 4, 64, 7)
    a, b = CudaGPT(config(4, 64, seed=8)), CudaGPT(config(4, 64, seed=8))
    try:
        for _ in range(3):
            x, y, px, py = ld.next()
            capi.check(a.lib.tlg_set_batch(a.h, px, py), a.lib, "set_batch")  # pinned
            b.set_batch(x, y)
            assert a.train_step() == b.train_step()
    finally:
        ld.close()
        a.close()
        b.close()


def test_bad_files_are_rejected(tmp_path):
    lib = capi.gpt_lib()
    h = ctypes.c_void_p()
    odd = tmp_path / "odd.bin"
    odd.write_bytes(bytes([1, 2, 3]))
    assert lib.tlg_loader_create(str(odd).encode(), 0.95, 0, 2, 8, 1, ctypes.byref(h)) != 0
    assert b"invalid token dataset size" in lib.tlg_last_error()
    assert lib.tlg_loader_create(str(tmp_path / "none.bin").encode(), 0.95, 0, 2, 8, 1,
                                 ctypes.byref(h)) != 0
