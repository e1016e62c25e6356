"""Packs this build as a CUDA solution of the benchmark harness, and unpacks one.

The reference packs its solution with ``scripts/pack_solution.py:34-83``: ``config.toml`` names the
solution, its definition and author, the language and the entry point, and the source files of
the language's directory become a Solution JSON (``name``, ``definition``, ``author``, ``spec``
with ``language``, ``target_hardware`` and ``entry_point``, and ``sources`` as path/content
pairs). Here the sources are the CUDA C ABI (``include/fmoe.h``, ``flashinfer_b200/csrc``), the
Python host code that loads it and the slot module ``binding.py``; loading the unpacked solution
compiles the CUDA sources with nvcc for sm_100a and registers ``flashinfer.kernel``.

``python -m flashinfer_b200.solution [-o solution.json]`` writes the JSON.
"""
from __future__ import annotations

import json
import os
from typing import Dict, List, Optional

try:
    import tomllib
except ImportError:  # Python < 3.11
    import tomli as tomllib

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
ROOT = os.path.dirname(PKG)
CONFIG = os.path.join(HERE, "config.toml")

# Python modules of the package the slot needs (the operator, its C-ABI binding, the build and
# the TVM-FFI registration); every CUDA source and header of csrc; the public header.
PY_MODULES = ["__init__.py", "_lib.py", "build.py", "moe.py", "tvm_binding.py"]


def load_config(path: str = CONFIG) -> dict:
    with open(path, "rb") as f:
        return tomllib.load(f)


def source_files() -> List[str]:
    """Repository-relative paths of the packed sources (binding.py is packed at the root)."""
    files = [os.path.join("flashinfer_b200", m) for m in PY_MODULES]
    csrc = os.path.join(PKG, "csrc")
    files += sorted(os.path.join("flashinfer_b200", "csrc", f) for f in os.listdir(csrc)
                    if f.endswith((".cu", ".h", ".cuh")))
    files.append(os.path.join("include", "fmoe.h"))
    return files


def pack(output: Optional[str] = None, config: str = CONFIG) -> dict:
    """The Solution JSON of this build (written to ``output`` when given)."""
    cfg = load_config(config)
    sol, bld = cfg["solution"], cfg["build"]
    if bld["language"] != "cuda":
        raise ValueError(f"unsupported language {bld['language']!r}: this build is a CUDA solution")
    sources = [{"path": "binding.py", "content": open(os.path.join(HERE, "binding.py")).read()}]
    for rel in source_files():
        sources.append({"path": rel, "content": open(os.path.join(ROOT, rel)).read()})
    solution = {
        "name": sol["name"], "definition": sol["definition"], "author": sol["author"],
        "spec": {"language": bld["language"], "target_hardware": ["cuda"],
                 "entry_point": bld["entry_point"], "destination_passing_style": True},
        "sources": sources,
    }
    if output is not None:
        with open(output, "w") as f:
            json.dump(solution, f, indent=2)
    return solution


def unpack(solution: Dict, dest: str) -> str:
    """Writes a Solution's sources under ``dest``; returns the entry module's path."""
    for src in solution["sources"]:
        path = os.path.normpath(os.path.join(dest, src["path"]))
        if not path.startswith(os.path.normpath(dest) + os.sep):
            raise ValueError(f"source path {src['path']!r} leaves the destination")
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "w") as f:
            f.write(src["content"])
    module = solution["spec"]["entry_point"].split("::")[0]
    return os.path.join(dest, module)


def main():
    import argparse
    ap = argparse.ArgumentParser(description="Pack this build as a CUDA solution JSON")
    ap.add_argument("-o", "--output", default="solution.json")
    args = ap.parse_args()
    sol = pack(args.output)
    print(f"Solution packed: {args.output}  ({sol['name']}, {sol['definition']}, "
          f"{sol['spec']['language']}, {len(sol['sources'])} sources)")


if __name__ == "__main__":
    main()
