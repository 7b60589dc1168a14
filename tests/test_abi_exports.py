"""The drop-in boundary on CPU: the built shared libraries load without a
GPU and export every entry point their headers declare (include/*.h).
No compute calls here."""
import ctypes
import os
import re

import pytest

from templit_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions(header):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(tlg?_[a-z0-9_]+)\s*\(",
                       text, flags=re.M)
    return sorted(set(names))


def test_cuda_header_declarations_are_bound():
    names = declared_functions("templit_cuda.h")
    assert len(names) > 40
    assert set(names) == set(capi.CUDA_ABI), set(names) ^ set(capi.CUDA_ABI)


def test_cuda_library_exports_every_declared_symbol():
    path = capi.library_path("libtemplit_cuda.so")
    assert os.path.exists(path), "run make -C templit_b200"
    lib = ctypes.CDLL(path)
    for name in declared_functions("templit_cuda.h"):
        assert hasattr(lib, name), name
    assert lib.tl_version() == 1


def test_gpt_header_declarations_are_bound():
    assert set(declared_functions("templit_gpt.h")) == set(capi.GPT_ABI)


def test_gpt_library_exports_every_declared_symbol():
    path = capi.library_path("libtemplit_gpt.so")
    if not os.path.exists(path):
        pytest.skip("GPT library not built in this checkout")
    capi.cuda_lib()
    lib = ctypes.CDLL(path)
    for name in declared_functions("templit_gpt.h"):
        assert hasattr(lib, name), name


def test_runtime_library_is_built():
    assert os.path.exists(capi.library_path("libtemplit_runtime.so"))


def test_errors_without_gpu_are_reported_not_raised():
    lib = capi.cuda_lib()
    # argument validation happens before any device call
    rc = lib.tl_transpose(None, capi.shape_arr([4]), 1, 0, 1, None, None)
    assert rc == capi.TL_ERR_INVALID
    assert b"rank" in lib.tl_last_error()
    rc = lib.tl_binary(capi.TL_ADD, None, capi.shape_arr([2, 3]), 2, None, capi.shape_arr([4]), 1,
                       None, capi.shape_arr([2, 3]), 2, None)
    assert rc == capi.TL_ERR_INVALID and b"broadcast" in lib.tl_last_error()
    assert lib.tl_argmax(None, 0, None, None, 0, None) == capi.TL_ERR_INVALID
    assert lib.tl_adamw(None, None, None, None, None, None, None, None, None, 1e-8, 0, 4,
                        None) == capi.TL_ERR_INVALID


def test_struct_layouts_match_the_headers(tmp_path):
    """The ctypes mirrors of the C structs have the C compiler's size and
    field offsets (a missing field would let the library read past the
    caller's struct)."""
    structs = {"tl_gemm_desc": capi.TlGemmDesc, "tl_param_slot": capi.TlParamSlot,
               "tlg_config": capi.TlgConfig, "tl_attn_view": capi.TlAttnView,
               "tl_attn_desc": capi.TlAttnDesc, "tl_flash_desc": capi.TlFlashDesc}
    lines = ['#include <stddef.h>', '#include <stdio.h>', '#include "templit_cuda.h"',
             '#include "templit_gpt.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines.append("  return 0;\n}")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    cuda_inc = "/usr/local/cuda/include"
    rc = os.system(f"gcc -I{ROOT}/include -I{cuda_inc} {src} -o {exe} 2> {tmp_path}/err.txt")
    if rc != 0:
        pytest.skip("no C compiler for the layout check: " + open(f"{tmp_path}/err.txt").read())
    got = dict(line.rsplit(" ", 1) for line in os.popen(str(exe)).read().splitlines())
    for cname, py in structs.items():
        assert int(got[f"{cname} size"]) == ctypes.sizeof(py), cname
        for field, _ in py._fields_:
            assert int(got[f"{cname} {field}"]) == getattr(py, field).offset, (cname, field)
