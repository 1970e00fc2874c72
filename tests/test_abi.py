"""The C-ABI library builds, loads without a GPU and exports exactly what the header declares.

No compute is called here (no GPU in the CPU suite): only symbol presence, the
ABI version and agreement between the header prototypes and the ctypes
signatures the host layer binds.
"""
import ctypes
import re
from pathlib import Path

import pytest

from conftest import REPO

HEADER = REPO / "include" / "moss_tts_b200.h"


def header_prototypes():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for m in re.finditer(r"\bint\s+(mt_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a.strip() for a in m.group(2).split(",") if a.strip() and a.strip() != "void"]
        kinds = []
        for a in args:
            if a.startswith("int*"):
                kinds.append("ip")
            elif a.startswith("long long*"):
                kinds.append("llp")
            elif a.startswith("const mt_tp_exchange*"):
                kinds.append("p")
            elif "*" in a:
                kinds.append("p")
            elif a.startswith("float"):
                kinds.append("f")
            elif a.startswith("int"):
                kinds.append("i")
            else:
                raise AssertionError(f"unexpected parameter type: {a}")
        protos[m.group(1)] = kinds
    return protos


@pytest.fixture(scope="module")
def lib():
    from moss_tts._runtime import native
    import sys
    sys.path.insert(0, str(REPO / "moss-tts-optimized_b200"))
    import build  # noqa: F401  (the in-tree build script)
    build.build()
    native.library.cache_clear()
    return native.library()


def test_header_declares_the_entry_points():
    protos = header_prototypes()
    assert {"mt_w4a16_linear", "mt_dequant_w4", "mt_attention_decode", "mt_heads_greedy",
            "mt_embedding_sum", "mt_rmsnorm", "mt_qk_rope_kv", "mt_bf16_linear",
            "mt_silu_mul", "mt_abi_version"} <= set(protos)


def test_library_exports_every_declared_symbol(lib):
    for name in header_prototypes():
        assert hasattr(lib, name), name


def test_ctypes_signatures_match_header():
    from moss_tts._runtime import native
    kind = {ctypes.c_void_p: "p", ctypes.c_int: "i", ctypes.c_float: "f", ctypes.POINTER(ctypes.c_int): "ip",
            ctypes.POINTER(ctypes.c_longlong): "llp"}
    protos = header_prototypes()
    assert set(native.SIGNATURES) == set(protos)
    for name, (args, res) in native.SIGNATURES.items():
        assert [kind[a] for a in args] == protos[name], name
        assert res is ctypes.c_int


def test_abi_version_callable_without_gpu(lib):
    assert lib.mt_abi_version() == 1


def test_library_has_no_torch_dependency():
    from moss_tts._runtime import native
    deps = Path("/proc/self/maps").read_text()  # loaded above; check the file itself
    data = native.LIB_PATH.read_bytes()
    assert b"libtorch" not in data and b"libc10" not in data
    assert deps  # maps readable
