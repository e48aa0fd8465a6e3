"""The C-ABI library loads and exports every entry point the header declares
(no GPU needed: only argument validation runs)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "ddtree_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"DDT_API\s+[\w\s\*]+?\b(ddt_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("ddt_tree_build", "ddt_tree_attention", "ddt_tree_accept", "ddt_kv_compact", "ddt_eagle3_accept"):
        assert name in syms


def test_library_exports_every_declared_symbol():
    from ddtree_eagle3_patch_b200 import _lib
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert sorted(_lib.exported_symbols()) == declared_symbols()


def test_library_exports_nothing_else():
    import subprocess
    from ddtree_eagle3_patch_b200 import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    text_syms = sorted(line.split()[-1] for line in out.splitlines() if " T " in line)
    assert text_syms == declared_symbols()


def test_abi_version_and_validation_errors():
    from ddtree_eagle3_patch_b200 import _lib
    lib = _lib.load()
    assert lib.ddt_abi_version() == 1
    # argument validation happens before any CUDA call
    assert lib.ddt_tree_attention(None, None, 0, None) == 1
    assert b"null" in lib.ddt_last_error()
    assert lib.ddt_tree_build(None, 0, 15, 100, 100, 8, None, 0, None, None, 0, None) == 1
    assert lib.ddt_kv_compact(None, 4, 8, 256, 0, 256, 0, 10, None, None, 4, None) == 1
    a = _lib.AttentionArgs(q=16, k=16, v=16, out=16, visibility=16, head_dim=64, n_tokens=1, hq=1, hkv=1,
                           kv_rows=1, vis_words=1, scale=1.0)
    assert lib.ddt_tree_attention(ctypes.byref(a), None, 0, None) == 3   # unsupported head_dim
    a.head_dim = 128
    a.hq, a.hkv = 3, 2
    assert lib.ddt_tree_attention(ctypes.byref(a), None, 0, None) == 1   # hq % hkv
    assert lib.ddt_tree_attention_window(ctypes.byref(a), None, None, 0, None) == 1   # key_lo is null
    assert b"key_lo" in lib.ddt_last_error()


def test_workspace_sizes_are_positive():
    from ddtree_eagle3_patch_b200 import _lib
    lib = _lib.load()
    assert lib.ddt_tree_build_workspace_size(15, 151936, 64) >= 256
    assert lib.ddt_tree_accept_workspace_size(65, 151936) >= 256


def test_product_code_has_no_oracle_dependency():
    pkg = ROOT / "ddtree_eagle3_patch_b200"
    for f in pkg.rglob("*.py"):
        t = f.read_text()
        assert "oracle" not in t.replace("oracle/", ""), f


@pytest.mark.parametrize("mod", ["ddtree", "eagle3", "attention", "kernels"])
def test_modules_import_without_gpu(mod):
    __import__(f"ddtree_eagle3_patch_b200.{mod}")
