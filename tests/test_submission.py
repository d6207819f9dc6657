"""CPU: the flashinfer-bench submission writer (config.toml, solution/python, solution.json)."""
import ast
import importlib.util
import json
import pathlib

import pytest

from conftest import load_pkg


@pytest.mark.parametrize("op,fn", [("gdn_decode", "decode_kernel"),
                                   ("gdn_prefill", "prefill_kernel"), ("gdn_mtp", "mtp_kernel")])
def test_submission_tree(tmp_path, op, fn):
    pkg = load_pkg()
    mod = __import__("importlib").import_module(pkg.__name__ + ".submission")
    doc = mod.write(tmp_path, op, "team-x", "me")
    cfg = (tmp_path / "config.toml").read_text()
    assert 'language = "python"' in cfg and 'entry_point = "kernel.py::kernel"' in cfg
    assert "destination_passing_style = true" in cfg
    assert f'definition = "{doc["definition"]}"' in cfg
    src = tmp_path / "solution" / "python"
    tree = ast.parse((src / "kernel.py").read_text())
    assigns = [n for n in tree.body if isinstance(n, ast.Assign)
               and any(getattr(t, "id", None) == "kernel" for t in n.targets)]
    assert assigns and ast.unparse(assigns[0].value) == f"_gdn.{fn}"
    paths = {s["path"] for s in doc["sources"]}
    pkg_dir = pathlib.Path(pkg.__file__).parent
    for cu in (pkg_dir / "csrc").glob("*.cu"):
        assert f"gdn_b200/csrc/{cu.name}" in paths
    assert "gdn_b200/include/gdn_b200.h" in paths and "kernel.py" in paths
    assert not any(p.endswith((".so", ".o", ".cubin", ".fatbin")) for p in paths)
    packed = json.loads((tmp_path / "solution.json").read_text())
    assert packed["spec"]["entry_point"] == "kernel.py::kernel"
    assert packed["spec"]["destination_passing_style"] is True
    assert packed["spec"]["language"] == "python" and len(packed["sources"]) == len(paths)
    # the bundled build script finds the bundled header (no repository around it)
    spec = importlib.util.spec_from_file_location("_bundled_build", src / "gdn_b200" / "build.py")
    bmod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bmod)
    assert bmod.INCLUDE == src / "gdn_b200" / "include"
