"""Build the reference's own WKV-7 kernels for the CPU into ``oracle/_ref/``.

The reference's only native code is two Metal kernel bodies that
``rwkv_mlx/kernels/wkv7_metal.py`` generates as Python f-strings
(``_make_forward_source`` at :20-92, ``_make_backward_source`` at :95-215) and
hands to ``mx.fast.metal_kernel`` (:223-247).  MLX and Metal are not available
here, so this script:

1. parses that file with ``ast`` and evaluates only ``_CHUNK_LEN`` and the two
   source-generator functions (pure string builders; nothing else from the file
   is executed and ``mlx`` is never imported);
2. wraps each generated body in the C++ Metal stand-in (``oracle/metal_shim.hpp``)
   with the signature ``mx.fast.metal_kernel`` would give it (input/output names
   and dtypes from ``wkv7_metal.py:228-247`` and ``:270-279`` / ``:307-318``);
3. compiles the result with g++ into ``oracle/_ref/`` (git-ignored; it travels to
   the GPU box with the rest of the tree, which needs no reference sources).

The reference checkout is read from ``$RWKV_MLX_REFERENCE`` (default: a directory
named ``reference`` beside this repository).  Run: ``python oracle/build_ref.py``.  Outputs:
``oracle/_ref/manifest.json`` plus one ``.so`` per (kernel, dtype).
"""

from __future__ import annotations

import ast
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from oracle.metal_cpu import build_kernel  # noqa: E402

REF_ROOT = Path(os.environ.get("RWKV_MLX_REFERENCE", str(HERE.parent.parent / "reference")))
REF_FILE = REF_ROOT / "rwkv_mlx" / "kernels" / "wkv7_metal.py"
OUT = HERE / "_ref"

FWD_IN = ["r", "w", "k", "v", "a", "b", "wkv_H", "wkv_T"]
FWD_OUT = ["y", "s_out", "sa_out"]
BWD_IN = ["r", "w", "k", "v", "a", "b", "dy", "s", "sa", "wkv_H", "wkv_T"]
BWD_OUT = ["dr", "dw_out", "dk_out", "dv_out", "da_out", "db_out"]


def extract_sources(ref_file: Path = REF_FILE, head_size: int = 64):
    tree = ast.parse(ref_file.read_text())
    keep = []
    for node in tree.body:
        if isinstance(node, ast.Assign) and any(
            isinstance(t, ast.Name) and t.id == "_CHUNK_LEN" for t in node.targets
        ):
            keep.append(node)
        elif isinstance(node, ast.FunctionDef) and node.name in (
            "_make_forward_source",
            "_make_backward_source",
        ):
            keep.append(node)
    ns: dict = {}
    exec(compile(ast.Module(body=keep, type_ignores=[]), str(ref_file), "exec"), ns)
    return ns["_make_forward_source"](head_size), ns["_make_backward_source"](head_size), ns["_CHUNK_LEN"]


def build(out_dir: Path = OUT) -> dict:
    fwd_src, bwd_src, chunk = extract_sources()
    manifest = {"chunk_len": chunk, "head_size": 64, "source": str(REF_FILE), "kernels": {}}
    for tname, T in (("f32", np.float32), ("f16", np.float16)):
        f = build_kernel(fwd_src, FWD_IN, [T] * 6 + [np.uint32] * 2, FWD_OUT,
                         [T, np.float32, np.float32], T, out_dir, f"wkv7_fwd_{tname}")
        b = build_kernel(bwd_src, BWD_IN, [T] * 7 + [np.float32] * 2 + [np.uint32] * 2, BWD_OUT,
                         [T] * 6, T, out_dir, f"wkv7_bwd_{tname}")
        manifest["kernels"][f"fwd_{tname}"] = f.name
        manifest["kernels"][f"bwd_{tname}"] = b.name
    (out_dir / "manifest.json").write_text(json.dumps(manifest, indent=1))
    return manifest


if __name__ == "__main__":
    if not REF_FILE.exists():
        print(f"reference not present ({REF_FILE}); nothing to build")
        sys.exit(0)
    print(json.dumps(build(), indent=1))
