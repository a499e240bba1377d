"""Records how the reference's Python host binds and calls the library, so the
GPU tests can drive the new library through exactly that binding without the
reference tree (which is absent where the GPU tests run).

Reads benchmark_pytorch_final.py from the reference checkout (its path is the
first argument, or FMHA_BWD_REFERENCE_TREE) with the `ast` module -- nothing
is executed and no source text is stored -- and writes reference_host.json
beside this script:

  library        the path handed to ctypes.CDLL (benchmark_pytorch_final.py:30)
  function       the entry point it binds, and its argtypes (:32-37)
  call_args      the argument expressions of the call in
                 custom_flash_attn_backward, in order (:47-52)
  zero_filled    the outputs the host zero-fills before the call (:43-45)
  seed           torch.manual_seed in benchmark_size (:87)
  result_keys    the keys of the dict benchmark_size returns (:129-136)
  configs        the (batch, heads, M, N, K_dim) list of __main__ (:146-151)
  sha256         of the script, to notice a changed reference

Run from the repository root:
    python tests/golden/make_reference_host.py <reference checkout>
"""
from __future__ import annotations

import ast
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "reference_host.json")
SCRIPT = "benchmark_pytorch_final.py"


def _call_name(node: ast.AST) -> str:
    return ast.unparse(node.func) if isinstance(node, ast.Call) else ""


def extract(source: str) -> dict:
    tree = ast.parse(source)
    rec: dict = {}
    for node in ast.walk(tree):
        # lib = ctypes.CDLL('<path>')
        if isinstance(node, ast.Call) and _call_name(node) == "ctypes.CDLL":
            rec["library"] = ast.literal_eval(node.args[0])
        # lib.<fn>.argtypes = [...]
        if isinstance(node, ast.Assign) and isinstance(node.targets[0], ast.Attribute) \
                and node.targets[0].attr == "argtypes":
            fn = node.targets[0].value
            rec["function"] = fn.attr
            rec["argtypes"] = [ast.unparse(e) for e in node.value.elts]
    for fn in (n for n in tree.body if isinstance(n, ast.FunctionDef)):
        if fn.name == "custom_flash_attn_backward":
            for node in ast.walk(fn):
                if isinstance(node, ast.Call) and _call_name(node) == f"lib.{rec['function']}":
                    rec["call_args"] = [ast.unparse(a) for a in node.args]
                if isinstance(node, ast.Assign) and isinstance(node.value, ast.Call) \
                        and _call_name(node.value) == "torch.zeros_like":
                    rec.setdefault("zero_filled", []).append(node.targets[0].id)
        if fn.name == "benchmark_size":
            for node in ast.walk(fn):
                if isinstance(node, ast.Call) and _call_name(node) == "torch.manual_seed":
                    rec["seed"] = ast.literal_eval(node.args[0])
                if isinstance(node, ast.Return) and isinstance(node.value, ast.Dict):
                    rec["result_keys"] = [ast.literal_eval(k) for k in node.value.keys]
    for node in ast.walk(tree):
        if isinstance(node, ast.Assign) and isinstance(node.targets[0], ast.Name) \
                and node.targets[0].id == "configs":
            rec["configs"] = [list(ast.literal_eval(e)) for e in node.value.elts]
    return rec


def main() -> None:
    tree = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FMHA_BWD_REFERENCE_TREE")
    if not tree:
        raise SystemExit("usage: make_reference_host.py <reference checkout>")
    path = os.path.join(tree, SCRIPT)
    with open(path, "rb") as f:
        raw = f.read()
    rec = extract(raw.decode())
    rec["script"] = SCRIPT
    rec["sha256"] = hashlib.sha256(raw).hexdigest()
    with open(OUT, "w") as f:
        json.dump(rec, f, indent=1)
        f.write("\n")
    print(json.dumps(rec))


if __name__ == "__main__":
    main()
