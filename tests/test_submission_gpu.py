"""GPU: a written flashinfer-bench submission builds from its bundled sources and its
`kernel` entry point matches the oracle (decode, 11-parameter DPS form)."""
import importlib.util
import inspect
import os
import sys

import pytest
import torch

from conftest import load_pkg
from gpu_util import assert_parity, oracle_decode, to

pytestmark = pytest.mark.gpu


def test_decode_submission_builds_and_runs(cuda, tmp_path, monkeypatch):
    pkg = load_pkg()
    mod = __import__("importlib").import_module(pkg.__name__ + ".submission")
    mod.write(tmp_path, "gdn_decode", "t", "a")
    monkeypatch.setenv("GDN_B200_BUILD_DIR", str(tmp_path / "_obj"))
    src = tmp_path / "solution" / "python"
    monkeypatch.syspath_prepend(str(src))
    spec = importlib.util.spec_from_file_location("_submitted_kernel", src / "kernel.py")
    km = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(km)
    assert (src / "gdn_b200" / "libgdn_b200.so").exists()
    assert len(inspect.signature(km.kernel).parameters) == 11
    inp = pkg.workloads.decode_inputs(3, hq=2, hv=4, seed=71)
    d = to(inp, cuda)
    out = torch.empty_like(d["v"])
    ns = torch.empty_like(d["state"])
    o, s = km.kernel(d["q"], d["k"], d["v"], d["state"], d["A_log"], d["a"], d["dt_bias"],
                     d["b"], d["scale"], out, ns)
    torch.cuda.synchronize()
    ro, rs = oracle_decode(inp, False)
    assert_parity(o, s, ro, rs, what="submission")
    sys.modules.pop("gdn_b200", None)
