"""Write tests/golden/ref_bindings.json: the prototype table that the reference's own
loader, tinygiant/_lib.py:26-76 (load_tinygiant_lib), registers on a library.

Run in a container that holds the reference checkout (its path is the first argument,
default /root/reference).  The loader module is imported unmodified from there and
called on this repository's libtinygiant.so; every function it registered is read
back from the loaded library (ctypes keeps each looked-up function in the library
object's __dict__) with its argtypes and restype.  The GPU test
tests/test_gpu_ref_bindings.py registers exactly this table, so it runs where the
reference checkout does not exist.

    python tests/golden/make_ref_bindings.py [/path/to/reference]
"""
from __future__ import annotations

import importlib.util
import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent / "ref_bindings.json"


def load_reference_loader(ref_root: Path):
    spec = importlib.util.spec_from_file_location("reference_tinygiant_lib", ref_root / "tinygiant" / "_lib.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ctype_name(t) -> str:
    return "None" if t is None else t.__name__


def registered_table(ref_root: Path, so_path: Path) -> dict:
    mod = load_reference_loader(ref_root)
    lib = mod.load_tinygiant_lib(str(so_path))
    if lib is None:
        raise RuntimeError("the reference loader returned None")
    table = {}
    for name, fn in sorted(vars(lib).items()):
        if name.startswith("tg_"):
            table[name] = {"restype": ctype_name(fn.restype), "argtypes": [ctype_name(a) for a in fn.argtypes]}
    return table


def main() -> None:
    ref_root = Path(sys.argv[1]) if len(sys.argv) > 1 else Path("/root/reference")
    so = ROOT / "tinygiant_b200" / "libtinygiant.so"
    table = registered_table(ref_root, so)
    doc = {"source": "tinygiant/_lib.py:26-76 (load_tinygiant_lib), recorded by tests/golden/make_ref_bindings.py",
           "functions": table}
    OUT.write_text(json.dumps(doc, indent=1) + "\n")
    print(f"{OUT}: {len(table)} functions")


if __name__ == "__main__":
    main()
