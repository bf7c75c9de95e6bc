"""The C-ABI library loads on a machine without a GPU and exports exactly the
entry points include/torchnative_b200.h declares, with the signatures the
ctypes binding uses. No compute call is made here."""

import os
import re

import pytest

from torchnative_b200 import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "torchnative_b200.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"^TN_API\s+[\w\s\*]*?\b(tn_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    from torchnative_b200 import build

    build.build()
    return _native.lib()


def test_header_declares_the_boundary():
    names = declared()
    for must in ("tn_q4_0_linear", "tn_q4_0_dequantize", "tn_q4_0_quantize", "tn_q8_0_quantize",
                 "tn_sdpa_flash_attention", "tn_last_error", "tn_alloc", "tn_free"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared():
        assert hasattr(lib, name), name


def test_binding_covers_every_declared_symbol():
    assert sorted(_native.SIGNATURES) == declared()


def test_runtime_calls_that_need_no_device(lib):
    assert lib.tn_abi_version() == 1
    assert lib.tn_status_name(1) == b"TN_ERR_NOT_IMPLEMENTED"
    assert _native.counters()["q4_linear_calls"] >= 0


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(_native, "LIB_PATH", str(tmp_path / "nope.so"))
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(_native.NativeLibraryMissing):
        _native.lib()


def _c_layout(tmp_path, ctype: str, names):
    """sizeof and offsetof of a header struct, from a C probe compiled here."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    src = tmp_path / f"probe_{ctype}.c"
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"torchnative_b200.h\"\nint main(void) {\n"
                   f"  printf(\"size %zu\\n\", sizeof({ctype}));\n"
                   + "".join(f"  printf(\"{n} %zu\\n\", offsetof({ctype}, {n}));\n" for n in names)
                   + "  return 0;\n}\n")
    exe = tmp_path / f"probe_{ctype}"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    return {k: int(v) for k, v in (line.split() for line in out.splitlines())}


@pytest.mark.parametrize("ctype,mirror", [("tn_counters", "Counters"), ("tn_tp_link", "TpLink"),
                                          ("tn_llama_q4_model", "LlamaQ4Model"),
                                          ("tn_llama_decode_layout", "DecodeLayout")])
def test_struct_bindings_match_the_header(tmp_path, ctype, mirror):
    """The ctypes mirrors of the header's structs have the C size and every
    field at the C offset (a field added on one side only would shift every
    field read after it)."""
    import ctypes

    cls = getattr(_native, mirror)
    names = [n for n, _ in cls._fields_]
    got = _c_layout(tmp_path, ctype, names)
    assert got["size"] == ctypes.sizeof(cls)
    for n in names:
        assert got[n] == getattr(cls, n).offset, n
