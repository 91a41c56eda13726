"""The reference's own Python bindings (tinygiant/_lib.py:26-76) against this library,
without a GPU: the committed prototype table lists every function that loader
registers, this library exports each of them, and, where the reference checkout is
present, the unmodified loader loads this library and registers exactly that table."""
import ctypes
import json
from pathlib import Path

import pytest

from tests.conftest import ROOT

TABLE = json.loads((ROOT / "tests" / "golden" / "ref_bindings.json").read_text())["functions"]
REF = Path("/root/reference")


def test_table_symbols_exported():
    from tinygiant_b200._lib import find_library
    lib = ctypes.CDLL(str(find_library()))
    missing = [n for n in TABLE if not hasattr(lib, n)]
    assert not missing, f"the reference's loader registers symbols this library lacks: {missing}"
    assert "tg_transformer_layer" in TABLE and len(TABLE) >= 13


@pytest.mark.skipif(not (REF / "tinygiant" / "_lib.py").exists(), reason="reference checkout not present")
def test_stock_loader_loads_this_library():
    import importlib.util
    spec = importlib.util.spec_from_file_location("mk", ROOT / "tests" / "golden" / "make_ref_bindings.py")
    mk = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mk)
    table = mk.registered_table(REF, ROOT / "tinygiant_b200" / "libtinygiant.so")
    assert table == TABLE
