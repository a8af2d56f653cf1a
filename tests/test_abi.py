"""The drop-in boundary without a GPU: both libraries load, export every entry point their headers declare, and the
host-side checks of the reference's operator interface (engine/h3-core/src/ops.rs:299-324, 405-461) hold."""
import os
import re
import subprocess

import pytest
import torch

from sycl_minimax_h3_b200 import native, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header: str) -> list[str]:
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"\b(h3s\w*|h3sage\w*)\s*\(", text)


def exported(lib_path: str) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], check=True, capture_output=True, text=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


@pytest.fixture(scope="module", autouse=True)
def built():
    from sycl_minimax_h3_b200 import build

    build.build()


@pytest.mark.parametrize("header,lib", [("h3cuda.h", native.CUDA_LIB), ("h3sage.h", native.SAGE_LIB)])
def test_every_declared_symbol_is_exported(header, lib):
    names = declared(header)
    assert len(names) >= 4
    missing = set(names) - exported(lib)
    assert not missing, f"{lib} lacks {sorted(missing)}"


def test_bindings_cover_the_headers():
    assert {n for n, _, _ in native.CUDA_SYMBOLS} == set(declared("h3cuda.h"))
    assert {n for n, _, _ in native.SAGE_SYMBOLS} == set(declared("h3sage.h"))


def test_libraries_load_with_every_symbol():
    native.lib()
    native.sage_lib()


def test_reference_attention_symbols_present():
    """The attention entry points of the reference's kernels/h3sycl.h:190-197 and kernels/sage.cpp:28-32."""
    names = exported(native.CUDA_LIB)
    for n in ("h3s_attention", "h3s_attention_batch", "h3s_open", "h3s_create", "h3s_alloc", "h3s_wait", "h3s_last_error"):
        assert n in names
    assert {"h3sage_attention", "h3sage_error"} <= exported(native.SAGE_LIB)


def test_sage_plugin_is_not_linked_into_the_host_library():
    """libh3cuda.so finds libh3sage.so at run time beside itself (kernels/h3sycl.cpp:1683-1701), not at link time."""
    out = subprocess.run(["readelf", "-d", native.CUDA_LIB], check=True, capture_output=True, text=True).stdout
    assert "libh3sage" not in out


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_without_a_gpu_open_fails_cleanly():
    L = native.lib()
    assert L.h3s_open() is None
    assert native.last_error()


def test_rows_bounds_like_the_reference():
    t = torch.zeros(10, 3 * 2 * 8, dtype=torch.float16)
    q, k, v = ops.Rows.qkv(t, 2, 8)
    assert q.stride == 48 and k.offset == 16 and v.offset == 32
    bad = ops.Rows(t, 40, 48, 10, 2, 8)               # the last row would run past the buffer
    with pytest.raises(native.H3Error, match="do not fit"):
        bad.ptr()
    with pytest.raises(native.H3Error, match="do not fit"):
        ops.Rows(t, 0, 15, 10, 2, 8).ptr()            # stride shorter than a row


def test_attention_layout_checks_before_any_device_work():
    t = torch.zeros(10, 48, dtype=torch.float16)
    q, k, v = ops.Rows.qkv(t, 2, 8)
    with pytest.raises(native.H3Error, match="same layout"):
        ops.attention(q, ops.Rows(t, 16, 48, 9, 2, 8), v, torch.zeros(10, 16, dtype=torch.float16))
    with pytest.raises(native.H3Error, match="out"):
        ops.attention(q, k, v, torch.zeros(9, 16, dtype=torch.float16))
    with pytest.raises(native.H3Error, match="equal sequences"):
        ops.attention_batch(q, k, v, 3, torch.zeros(10, 16, dtype=torch.float16))
    with pytest.raises(native.H3Error):
        native.dt_code(torch.int32)
