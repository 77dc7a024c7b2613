"""The C-ABI library (libvitb200.so) on a machine without a GPU: it loads,
exports exactly what include/vitb200.h declares, its ctypes structs match the C
layout, workspace queries are pure host arithmetic, and bad arguments are
rejected with a status code before any device work."""
import ctypes
import os
import re
import subprocess

import pytest

from vit_cuda import _lib
from vit_cuda._lib import BlockParams, VitParams, lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "vitb200.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vitb200_[a-z0-9_]+)\s*\(", text)))


def test_library_loads():
    assert os.path.exists(_lib.LIB_PATH)
    assert lib.vitb200_version() >= 100


def test_exports_match_header():
    declared = header_functions()
    assert declared, "no declarations parsed"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in vitb200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = sorted({ln.split()[-1] for ln in out.splitlines()
                       if " T " in ln and ln.split()[-1].startswith("vitb200_")})
    assert exported == declared
    assert sorted(_lib.exported_names()) == declared


def test_status_strings():
    for code in (0, -1, -2, -3, -4, -5, -6):
        s = _lib.status_string(code)
        assert s and s != "unknown status"
    assert _lib.status_string(-99) == "unknown status"


def test_struct_layout_matches_c(tmp_path):
    """Compile a tiny C program against the header and compare sizeof/offsetof
    with the ctypes mirrors."""
    fields = [f for f, _ in VitParams._fields_]
    bfields = [f for f, _ in BlockParams._fields_]
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "vitb200.h"', "int main(void){",
           'printf("%zu %zu\\n", sizeof(vitb200_vit_params), sizeof(vitb200_block_params));']
    for f in fields:
        src.append(f'printf("%zu\\n", offsetof(vitb200_vit_params, {f}));')
    for f in bfields:
        src.append(f'printf("%zu\\n", offsetof(vitb200_block_params, {f}));')
    src.append("return 0;}")
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", os.path.join(REPO, "include"), str(c), "-o", str(exe)],
                   check=True)
    vals = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    vals = [int(v) for v in vals]
    assert vals[0] == ctypes.sizeof(VitParams)
    assert vals[1] == ctypes.sizeof(BlockParams)
    offs = vals[2:]
    assert offs[:len(fields)] == [getattr(VitParams, f).offset for f in fields]
    assert offs[len(fields):] == [getattr(BlockParams, f).offset for f in bfields]


def test_workspace_queries_are_host_only():
    assert lib.vitb200_gemm_workspace_bytes(100, 768, 3072) >= 2 * 4 * (100 + 3072) * 768
    assert lib.vitb200_gemm_workspace_bytes(-1, 8, 8) == 0
    # K is padded to a multiple of 4 for the TMA row stride
    assert lib.vitb200_gemm_workspace_bytes(1, 5, 1) >= 2 * 4 * 2 * 8
    assert lib.vitb200_mlp_workspace_bytes(10, 768, 3072) > lib.vitb200_gemm_workspace_bytes(
        10, 768, 3072)
    assert lib.vitb200_patch_embed_workspace_bytes(2, 3, 224, 224, 768) >= 2 * 4 * 392 * 768


def test_vit_workspace_query_validates_params():
    p = VitParams(depth=12, embed_dim=768, num_heads=12, mlp_dim=3072, patch=16, in_chans=3,
                  img_h=224, img_w=224, num_classes=1000, ln_eps=1e-6, attn_scale=0.125)
    # null weight pointers: the query refuses (returns 0)
    assert lib.vitb200_vit_workspace_bytes(ctypes.byref(p), 2) == 0


@pytest.mark.parametrize("call", [
    lambda: lib.vitb200_gemm(None, None, None, None, None, -1, 4, 4, 0, None, 0, None),
    lambda: lib.vitb200_gemm(1, 1, None, None, 1, 4, 4, 4, _lib.EPI_BIAS, None, 0, None),
    lambda: lib.vitb200_gemm(1, 1, 1, None, 1, 4, 4, 4, 99, None, 0, None),
    lambda: lib.vitb200_gemm_pairs(None, None, None, None, None, 0, None, 4, 6, 4, 0, None),
    lambda: lib.vitb200_split_tf32(1, 4, 8, 8, 1, 6, None),
    lambda: lib.vitb200_layernorm(None, None, None, None, 4, 768, 1e-6, None),
    lambda: lib.vitb200_attention(1, 1, 1, 1, 1, 10, 12, 700, 768, 768, 768, 0.125, None, 0,
                                  None),
    lambda: lib.vitb200_pos_encoding(None, 1, 1, 1, 1, 196, 768, None),
    lambda: lib.vitb200_patch_embed(1, 1, None, 1, 1, 3, 200, 224, 768, None, 0, None),
    lambda: lib.vitb200_classifier(1, 1, None, 1, 1, 197, 768, 10, None, 0, None),
    lambda: lib.vitb200_vit_forward(None, 1, 1, 1, None, 0, None),
])
def test_bad_arguments_rejected_without_gpu(call):
    assert call() == _lib.E_INVALID_ARG


def test_diagnostic_entries_without_gpu():
    v, d = ctypes.c_int(-1), ctypes.c_int(-1)
    for shape in ((0, 768, 768), (197, -1, 768), (197, 768, 0)):
        assert lib.vitb200_gemm_plan(*shape, 1, ctypes.byref(v), ctypes.byref(d)) == \
            _lib.E_INVALID_ARG
    assert (v.value, d.value) == (-1, -1)
    assert lib.vitb200_check_wait_timeout(2, None) == _lib.E_INVALID_ARG
    old = lib.vitb200_set_split_k(0)
    try:
        assert lib.vitb200_set_split_k(1) == 0
        assert lib.vitb200_set_split_k(1) == 1
    finally:
        lib.vitb200_set_split_k(old)


def test_workspace_too_small_rejected_without_gpu():
    assert lib.vitb200_gemm(1, 1, None, None, 1, 4, 8, 4, _lib.EPI_NONE, 1, 16,
                            None) == _lib.E_WORKSPACE


def test_qkv_width_not_multiple_of_32_is_unsupported():
    assert lib.vitb200_qkv(1, 1, 1, 1, 4, 40, None, 0, None) == _lib.E_UNSUPPORTED


def test_preprocess_argument_checks():
    """vitb200_preprocess validates before touching the device."""
    import ctypes
    from vit_cuda import _lib
    m = (ctypes.c_float * 3)(0.5, 0.5, 0.5)
    s = (ctypes.c_float * 3)(0.2, 0.2, 0.2)
    bad_s = (ctypes.c_float * 3)(0.2, 0.0, 0.2)
    f = _lib.lib.vitb200_preprocess
    assert f(None, 0, 10, 10, 300, 256, 224, m, s, None, None) == 0           # empty batch
    assert f(None, 1, 10, 10, 299, 256, 224, m, s, None, None) == _lib.E_INVALID_ARG  # stride
    assert f(None, 1, 10, 10, 300, 256, 224, m, s, None, None) == _lib.E_INVALID_ARG  # null
    assert f(None, -1, 10, 10, 300, 256, 224, m, s, None, None) == _lib.E_INVALID_ARG
    assert f(None, 1, 10, 10, 300, 256, 224, m, None, None, None) == _lib.E_INVALID_ARG
    p = ctypes.c_void_p(16)
    assert f(p, 1, 10, 10, 300, 200, 224, m, s, p, None) == _lib.E_UNSUPPORTED  # crop > resize
    assert f(p, 1, 10, 10, 300, 256, 224, m, bad_s, p, None) == _lib.E_INVALID_ARG
