"""Pack a definition's solution into a self-contained solution.json.

Replaces the reference's `scripts/pack_solution.py` (lines 34-84 of the
reference project), which packs a solution folder through flashinfer-bench's
`pack_solution_from_files`.  The record has the fields the reference README
documents for a solution (README.md:235-248 and :265-278): name, definition,
author, spec {language, target_hardware, entry_point, dependencies,
destination_passing_style} and sources.  Each source is written as
{"path": ..., "content": ...}; the README elides the entries ("[...]"), so
that shape is the one flashinfer-bench's packer is assumed to produce.

The builders take no custom compile flags (reference FAQ.md:59-61), so the
packed solution is a Python solution that compiles its own CUDA: its sources
are this library's CUDA files, C header and Python modules in the
repository's layout, plus a `kernel.py` whose import builds libgdn_b200.so
for sm_100a with nvcc (once per extracted copy) and binds `run` to the
package's value-returning entry point for the definition.

    python track-c-gdn_b200/pack.py --definition gdn_decode_qk4_v8_d128_k_last -o solution.json
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path
from typing import Dict, List, Optional, Union

try:
    import tomllib
except ImportError:  # pragma: no cover - Python < 3.11
    import tomli as tomllib

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
PACKAGE = HERE.name

DEFINITIONS = {
    "gdn_decode_qk4_v8_d128_k_last": "decode",
    "gdn_prefill_qk4_v8_d128_k_last": "prefill",
}

# the packed kernel.py: build on first import, then bind the package's run
_KERNEL_PY = '''"""Solution entry point for definition {definition} (packed by pack.py).

Importing this file compiles the library's sm_100a CUDA with nvcc on first use
(into the package directory of this extracted copy) and binds `run` to the
value-returning entry point with the reference's signature.
"""
import importlib
import importlib.util
import sys
from pathlib import Path

_ROOT = Path(__file__).resolve().parent
if str(_ROOT) not in sys.path:
    sys.path.insert(0, str(_ROOT))
_spec = importlib.util.spec_from_file_location("_gdn_pack_build", _ROOT / "{package}" / "build.py")
_build = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_build)
_build.build()
_gdn = importlib.import_module("{package}")

run = _gdn.{module}.run
'''


def library_sources() -> List[Path]:
    """Files a packed solution carries, relative to the repository root."""
    pkg = REPO / PACKAGE
    files = sorted((pkg / "csrc").glob("*.cu")) + sorted((pkg / "csrc").glob("*.cuh"))
    files += sorted((REPO / "include").glob("*.h"))
    files += [pkg / n for n in ("__init__.py", "_native.py", "build.py", "decode.py",
                                "prefill.py", "shard.py")]
    return [f.relative_to(REPO) for f in files]


def solution_config(definition: str) -> Dict:
    cfg = HERE / "solutions" / definition / "config.toml"
    with open(cfg, "rb") as f:
        return tomllib.load(f)


def pack_solution(definition: str, name: Optional[str] = None, author: Optional[str] = None,
                  language: str = "python") -> Dict:
    """The solution record for `definition` (a dict ready for json.dump)."""
    if definition not in DEFINITIONS:
        raise ValueError(f"unknown definition {definition!r}; one of {sorted(DEFINITIONS)}")
    cfg = solution_config(definition)
    sol, build = cfg["solution"], cfg["build"]
    sources = [{"path": "kernel.py",
                "content": _KERNEL_PY.format(definition=definition, package=PACKAGE,
                                             module=DEFINITIONS[definition])}]
    for rel in library_sources():
        sources.append({"path": rel.as_posix(), "content": (REPO / rel).read_text()})
    return {
        "name": name or sol["name"],
        "definition": definition,
        "author": author or sol["author"],
        "spec": {
            "language": language,
            "target_hardware": ["cuda"],
            "entry_point": build["entry_point"],
            "dependencies": [],
            "destination_passing_style": bool(build.get("destination_passing_style", False)),
        },
        "sources": sources,
    }


def extract_solution(solution: Union[Dict, str, Path], dest: Union[str, Path]) -> Path:
    """Write a solution's sources under `dest` (the inverse of pack_solution)."""
    if not isinstance(solution, dict):
        solution = json.loads(Path(solution).read_text())
    dest = Path(dest)
    for src in solution["sources"]:
        rel = Path(src["path"])
        if rel.is_absolute() or ".." in rel.parts:
            raise ValueError(f"unsafe source path {src['path']!r}")
        out = dest / rel
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(src["content"])
    return dest


def main() -> None:
    ap = argparse.ArgumentParser(description="Pack a GDN solution into solution.json")
    ap.add_argument("--definition", required=True, choices=sorted(DEFINITIONS))
    ap.add_argument("-o", "--output", type=Path, default=Path("solution.json"))
    ap.add_argument("--name")
    ap.add_argument("--author")
    ap.add_argument("--language", default="python")
    args = ap.parse_args()
    sol = pack_solution(args.definition, args.name, args.author, args.language)
    args.output.write_text(json.dumps(sol, indent=2))
    print(f"solution packed: {args.output} ({sol['name']}, {len(sol['sources'])} sources)")


if __name__ == "__main__":
    main()
