"""CPU: the C-ABI library loads, exports every symbol the header declares, and
rejects bad arguments on the host before any launch (no compute calls here)."""

from __future__ import annotations

import ctypes as C
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = ROOT / "include" / "ssd_verify.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ssd_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_verify_path():
    names = declared_functions()
    for must in ("ssd_verify_greedy", "ssd_verify_sample", "ssd_page_rollback", "ssd_page_allocate",
                 "ssd_page_free", "ssd_kv_write", "ssd_paged_verify_attention", "ssd_linear",
                 "ssd_gemma_forward"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from ssd_b200 import _lib

    so = _lib.lib()
    names = declared_functions()
    missing = [n for n in names if not hasattr(so, n)]
    assert not missing, missing
    # the ctypes table binds exactly the declared set
    assert sorted(_lib.SIGNATURES) == names
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (ssd_[a-z0-9_]+)", out))
    assert set(names) <= exported


def test_status_strings_and_version():
    from ssd_b200 import _lib

    so = _lib.lib()
    assert so.ssd_status_string(0) == b"ok"
    assert so.ssd_status_string(5) == b"workspace too small"
    assert so.ssd_abi_version() >> 16 == 1


def test_host_side_argument_checks():
    from ssd_b200 import _lib

    so = _lib.lib()
    # rejected before any CUDA call, so these run without a GPU
    assert so.ssd_verify_greedy(None, None, None, None, None, None, None, None, 0, 0, 4, 10) == 1
    assert so.ssd_verify_sample(None, None, None, None, None, None, 1.0, 1.0, 0.5, 0, None, None, None, None, 0,
                                1, 4, 10) == 1
    assert so.ssd_verify_sample(None, 1, 1, 1, 1, 1, 0.0, 1.0, 0.5, 0, 1, 1, None, 1, 1 << 30, 1, 4, 10) == 1
    assert so.ssd_linear(None, None, None, 0, None, 0, 1, 8, 8, None, 0) == 1
    assert so.ssd_linear(None, 1, 1, 0, 1, 3, 1, 7, 8, None, 0) == 1          # GeGLU needs even N
    assert so.ssd_linear(None, 1, 1, 0, 1, 0, 4096, 8, 8, None, 0) == 4       # M over the limit
    assert so.ssd_paged_verify_attention(None, 1, 1, 0, 2, 4, 16, 3, 64, 0, 1, 4, 1, None, 1, 0.1,
                                         1, 5, 4, 64, None, 0) == 1           # Hq % Hkv != 0
    assert so.ssd_page_rollback(None, None, None, 4, None, None, None, 8, None, None, None, 16, 0) == 0  # B = 0
    assert so.ssd_page_rollback(None, None, None, 4, None, None, None, 8, None, None, None, 16, 1) == 1
    assert so.ssd_gemma_forward(None, None, None) == 1


def test_workspace_sizes_are_host_computable():
    from ssd_b200 import _lib

    so = _lib.lib()
    assert so.ssd_verify_greedy_workspace_size(8, 4, 256000) > 0
    assert so.ssd_verify_sample_workspace_size(8, 4, 256000) > 0
    assert so.ssd_paged_attention_workspace_size(8, 5, 16, 16, 256, 4096) > 0
    assert so.ssd_linear_workspace_size(5, 3072, 24576) > 0
    assert so.ssd_linear_max_m() >= 16


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    from ssd_b200 import _lib

    monkeypatch.setattr(_lib, "_LIB", None)
    monkeypatch.setenv("SSD_B200_LIB", str(tmp_path / "nope.so"))
    with pytest.raises(_lib.SSDError):
        _lib.lib()
    monkeypatch.setattr(_lib, "_LIB", None)


def test_ctypes_structs_match_the_header(tmp_path):
    """The ctypes mirrors of the header's structs have the C compiler's size and field offsets."""
    from ssd_b200 import _lib

    structs = {"ssd_comm": _lib.CommC, "ssd_gemma_weights": _lib.GemmaWeightsC, "ssd_gemma_batch": _lib.GemmaBatchC}
    lines = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in py._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-o", str(exe), str(src)], check=True, capture_output=True)
    got = {}
    for line in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.splitlines():
        cname, field, value = line.split()
        got[(cname, field)] = int(value)
    for cname, py in structs.items():
        assert got[(cname, "size")] == C.sizeof(py), cname
        for field, _ in py._fields_:
            assert got[(cname, field)] == getattr(py, field).offset, (cname, field)
