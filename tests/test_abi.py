"""The C-ABI library: it loads, exports every declared symbol, and fails with a
status (never an abort) on bad arguments.  No GPU needed."""
import ctypes
import subprocess

import pytest

import bramha_b200 as bb
from bramha_b200 import _lib


def test_library_exports_every_header_symbol():
    L = bb.lib()
    syms = bb.header_symbols()
    assert len(syms) >= 21
    for s in syms:
        assert hasattr(L, s), s
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    assert set(syms) <= exported
    # nothing else leaks out of the library except the ABI (C++ internals are hidden)
    ours = {s for s in exported if s.startswith("bramha")}
    assert ours == set(syms)


def test_every_header_symbol_has_a_binding():
    assert set(bb.header_symbols()) == set(_lib._SIGNATURES)


def test_abi_version():
    assert bb.lib().bramha_cuda_abi_version() == 1


def test_null_arguments_return_status_not_abort():
    L = bb.lib()
    assert L.bramha_cuda_init(0, None) == -1
    assert "null" in bb.last_error()
    assert L.bramha_cuda_destroy(None) == -1
    assert L.bramha_cuda_gemv(None, None, None, 1, None) == -1
    assert L.bramha_cuda_clear(None) == -1
    assert L.bramha_cuda_weight_info(None, None, None, None, None) == -1


def test_init_without_usable_device_is_an_error_status():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    ctx = ctypes.c_void_p()
    rc = bb.lib().bramha_cuda_init(0, ctypes.byref(ctx))
    assert rc in (-3, -5) and not ctx.value
    assert bb.last_error()


def test_get_cuda_plane_respects_bramha_cpu(monkeypatch):
    from bramha_b200 import plane
    monkeypatch.setenv("BRAMHA_CPU", "1")
    assert plane.get_cuda_plane(0) is None


def test_static_archive_links_into_a_host_program(tmp_path):
    """libbramha_cuda.a (the static form a Rust build step links) holds the
    whole ABI: a C program that names every header symbol links against it
    alone (plus the CUDA runtime) and runs; without a GPU, init reports an
    error status."""
    import os
    from bramha_b200 import build as b
    if not os.path.exists(b.STATIC_LIB):
        b.build()
    syms = bb.header_symbols()
    src = tmp_path / "prog.c"
    refs = "\n".join(f"    (void*)&{s}," for s in syms)
    src.write_text(
        '#include <stdio.h>\n#include "bramha_cuda.h"\n'
        f"static void* all[] = {{\n{refs}\n}};\n"
        "int main(void) {\n"
        "    bramha_ctx* ctx = 0;\n"
        "    int v = bramha_cuda_abi_version();\n"
        "    int rc = bramha_cuda_init(0, 0);\n"
        '    printf("%d %d %d\\n", v, rc, (int)(sizeof(all) / sizeof(all[0])));\n'
        "    (void)ctx;\n    return 0;\n}\n")
    exe = tmp_path / "prog"
    cuda = "/usr/local/cuda"
    r = subprocess.run(["g++", "-x", "c", str(src), "-x", "none", "-I", os.path.join(b.ROOT, "include"),
                        b.STATIC_LIB, f"-L{cuda}/lib64", "-lcudart_static", "-lrt", "-ldl", "-lpthread",
                        "-lstdc++", "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, out.stderr
    v, rc, n = map(int, out.stdout.split())
    assert v == 1 and rc == -1 and n == len(syms)
