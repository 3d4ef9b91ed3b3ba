"""CPU tests of the C-ABI boundary: the shared library loads, exports every
entry point include/tabinfer_b200.h declares, the ctypes table matches the
header, and the oracle is not reachable from the product package."""
import ctypes
import os
import re
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "tabinfer_b200", "libtabinfer_b200.so")


def _header_names():
    from tabinfer_b200 import _lib
    return _lib.header_symbols()


def test_library_exists_and_loads():
    assert os.path.exists(LIB), "build first: python -c 'import __graft_entry__ as g; g.build()'"
    ctypes.CDLL(LIB)


def test_every_header_symbol_is_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = set(line.split()[-1] for line in out.splitlines() if " T " in line)
    missing = [n for n in _header_names() if n not in exported]
    assert not missing, missing


def test_ctypes_table_matches_header():
    from tabinfer_b200 import _lib
    assert sorted(_lib.SIGNATURES) == sorted(_header_names())


def test_header_arg_counts_match_ctypes_table():
    from tabinfer_b200 import _lib
    txt = open(os.path.join(REPO, "include", "tabinfer_b200.h")).read()
    for m in re.finditer(r"TB_API\s+[\w\s\*]+?\b(tb_\w+)\s*\(([^;]*?)\);", txt, re.S):
        name, args = m.group(1), m.group(2).strip()
        n = 0 if args in ("", "void") else args.count(",") + 1
        assert len(_lib.SIGNATURES[name]) == n, name


def test_version_and_null_context_are_safe():
    from tabinfer_b200._lib import LIB as lib
    assert lib.tb_version() >= 100
    assert lib.tb_last_error(None) == b"null context"
    assert lib.tb_ctx_destroy(None) == 0
    assert lib.tb_gemv_int4_q8(None, None, None, None, None, None, 1, 32, 1, 0) == 1


def test_product_does_not_import_the_oracle():
    pkg = os.path.join(REPO, "tabinfer_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                src = open(os.path.join(root, f)).read()
                assert "oracle" not in re.sub(r"#.*|//.*", "", src).replace("oracle/", ""), f


@pytest.mark.skipif(os.environ.get("CUDA_VISIBLE_DEVICES") == "", reason="no devices")
def test_context_create_fails_cleanly_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present; covered by -m gpu tests")
    from tabinfer_b200._lib import LIB as lib
    h = ctypes.c_void_p()
    assert lib.tb_ctx_create(0, ctypes.byref(h)) != 0
    assert not h.value
