"""The C-ABI library loads on a machine without a GPU and exports every
function include/chimera_b200.h declares (no compute calls here)."""
import ctypes as C
import os
import re

from chimera_b200 import capi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header):
    src = open(os.path.join(ROOT, "include", header)).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(chm_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    lib = C.CDLL(capi.LIB_PATH)
    names = declared("chimera_b200.h")
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_table_covers_header():
    assert set(declared("chimera_b200.h")) <= set(capi.EXPORTS)


def test_version_string():
    assert capi.lib().chm_version().startswith(b"chimera_b200")


def test_sharded_library_exports_its_header():
    """lib/libchimera_nccl.so (the document-sharded search over NCCL) loads
    and exports every function include/chimera_b200_sharded.h declares."""
    lib = capi.nccl_lib()
    names = declared("chimera_b200_sharded.h")
    assert "chm_search_sharded" in names and len(names) >= 6
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
