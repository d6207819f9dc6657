"""Write this package as a flashinfer-bench contest submission.

    python -m <package>.submission --op gdn_decode --out <dir> [--name N --author A]

The contest harness (reference README.md:60-110, FAQ.md:46-62, 144-168) packs a solution
from ``config.toml`` plus the source files under ``solution/<language>/`` (or takes a
``solution.json``), builds it from source on an sm_100a machine without network,
and calls the entry point named in ``config.toml`` in destination-passing style.  This
writes, for one operator:

* ``config.toml`` — ``[solution]`` name / definition / author, ``[build]`` language
  "python", entry point ``kernel.py::kernel`` and ``destination_passing_style = true``
  (the reference's build section, gdn_prefill/config.toml:6-8, and the flag its packer
  forwards, gdn_prefill/scripts/pack_solution.py:56-62);
* ``solution/python/kernel.py`` — compiles the bundled CUDA sources for sm_100a with nvcc
  on first import (no prebuilt binary is shipped) and binds ``kernel`` to the
  exact-arity DPS function (11 parameters for decode, 12 for prefill, 13 for multi-token
  decode);
* ``solution/python/gdn_b200/`` — this package's host code, CUDA sources and C ABI header;
* ``solution.json`` (the name the reference's packer writes by default) — the same files
  as a Solution document (name, definition, author, description, spec {language,
  target_hardware, entry_point, destination_passing_style, dependencies}, sources [{path,
  content}]), following flashinfer-bench's Solution and BuildSpec fields.
"""
from __future__ import annotations

import argparse
import json
import pathlib
from typing import Dict

PKG = pathlib.Path(__file__).resolve().parent
REPO = PKG.parent

OPS = {
    "gdn_decode": ("decode_kernel", "gdn_decode_qk16_v32_d128_k_last"),
    "gdn_prefill": ("prefill_kernel", "gdn_prefill_qk16_v32_d128_k_last"),
    "gdn_mtp": ("mtp_kernel", "gdn_mtp_qk16_v32_d128_k_last"),
}
PY_FILES = ("__init__.py", "_lib.py", "_checks.py", "decode.py", "prefill.py", "mtp.py",
            "sharding.py", "workloads.py", "build.py")

KERNEL_PY = '''"""flashinfer-bench entry point for {op}: B200 (sm_100a) Gated DeltaNet kernels.

The CUDA sources in gdn_b200/csrc are compiled for sm_100a by nvcc the first time this
module is imported (into gdn_b200/libgdn_b200.so); `kernel` is the destination-passing
entry point with the definition's exact parameter list.
"""
import importlib.util
import pathlib
import sys

_HERE = pathlib.Path(__file__).resolve().parent
if str(_HERE) not in sys.path:
    sys.path.insert(0, str(_HERE))

# build first, from the script itself (importing the package loads the library)
_spec = importlib.util.spec_from_file_location("_gdn_b200_build", _HERE / "gdn_b200" / "build.py")
_build = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(_build)
_build.build(quiet=True)

import gdn_b200 as _gdn  # noqa: E402

kernel = _gdn.{fn}
'''


def bundle() -> Dict[str, str]:
    """Relative path -> text of every file the submission carries."""
    files = {f"gdn_b200/{name}": (PKG / name).read_text() for name in PY_FILES}
    for src in sorted((PKG / "csrc").iterdir()):
        if src.suffix in (".cu", ".cuh", ".h"):
            files[f"gdn_b200/csrc/{src.name}"] = src.read_text()
    header = REPO / "include" / "gdn_b200.h"
    if not header.exists():
        header = PKG / "include" / "gdn_b200.h"
    files["gdn_b200/include/gdn_b200.h"] = header.read_text()
    return files


def write(out: pathlib.Path, op: str, name: str, author: str, definition: str = "") -> dict:
    if op not in OPS:
        raise ValueError(f"op must be one of {sorted(OPS)}")
    fn, default_def = OPS[op]
    definition = definition or default_def
    out = pathlib.Path(out)
    src_dir = out / "solution" / "python"
    files = {"kernel.py": KERNEL_PY.format(op=op, fn=fn), **bundle()}
    for rel, text in files.items():
        path = src_dir / rel
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(text)
    (out / "config.toml").write_text(
        "[solution]\n"
        f'name = "{name}"\n'
        f'definition = "{definition}"\n'
        f'author = "{author}"\n\n'
        "[build]\n"
        'language = "python"\n'
        'entry_point = "kernel.py::kernel"\n'
        "destination_passing_style = true\n")
    doc = {
        "name": name,
        "definition": definition,
        "author": author,
        "description": f"{op}: hand-written sm_100a CUDA (tcgen05 / TMEM / TMA) built from "
                       "source at load time; destination-passing entry point.",
        "spec": {"language": "python", "target_hardware": ["cuda"],
                 "entry_point": "kernel.py::kernel", "destination_passing_style": True,
                 "dependencies": []},
        "sources": [{"path": rel, "content": text} for rel, text in sorted(files.items())],
    }
    (out / "solution.json").write_text(json.dumps(doc, indent=2))
    return doc


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", choices=sorted(OPS), required=True)
    ap.add_argument("--out", type=pathlib.Path, required=True)
    ap.add_argument("--name", default="gdn-b200")
    ap.add_argument("--author", default="gdn-b200")
    ap.add_argument("--definition", default="")
    a = ap.parse_args()
    doc = write(a.out, a.op, a.name, a.author, a.definition)
    print(f"wrote {a.out} ({len(doc['sources'])} sources, definition {doc['definition']})")


if __name__ == "__main__":
    main()
