"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once, in a container that has both the reference repository and the
``flashinfer-python`` package installed (neither is needed to *use* the
fixtures)::

    python tests/golden/make_golden.py --reference-root <path to reference checkout>

Sources of truth, executed here, never copied:

* ``flashinfer.trace.templates.gdn._gdn_decode_reference`` and
  ``_gdn_prefill_reference`` (flashinfer-python, installed) -- the
  flashinfer-bench definition reference the reference repository is scored
  against.
* ``gdn_decode/solution/triton/kernel.py`` from the reference repository
  itself, run on the CPU by the Triton interpreter (``TRITON_INTERPRET=1``)
  with one explicit tile configuration (its autotuner needs a GPU).  The
  reference prefill Triton kernel is NOT used: under the Triton 3.6
  interpreter its bf16 ``tl.dot`` is wrong, and its ``log_gamma`` clamp
  (``gdn_prefill/solution/triton/kernel.py:166``) departs from the recurrence
  under strong decay, so the definition reference is the prefill truth.

Each fixture is an ``.npz`` holding the inputs and the expected outputs.
bf16 tensors are stored as their raw uint16 bit patterns.
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import os
import pathlib
import sys

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))


def _pkg_workloads():
    spec = importlib.util.spec_from_file_location(
        "_gdn_workloads",
        REPO / "mlsys26-flashinfer-ai-kernel-generation-contest_b200" / "workloads.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def _np(x: torch.Tensor):
    if x.dtype == torch.bfloat16:
        return x.contiguous().view(torch.int16).numpy().view(np.uint16)
    return x.contiguous().numpy()


def _save(name: str, tensors: dict, meta: dict):
    arrs = {}
    for key, val in tensors.items():
        if val is None:
            continue
        arrs[key] = _np(val)
        arrs[key + "__dtype"] = np.array(str(val.dtype).replace("torch.", ""))
    for key, val in meta.items():
        arrs["meta__" + key] = np.array(val)
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **arrs)
    print(f"wrote {path.relative_to(REPO)} ({path.stat().st_size // 1024} KiB)")


def _reference_triton_decode(reference_root: pathlib.Path):
    path = reference_root / "gdn_decode" / "solution" / "triton" / "kernel.py"
    spec = importlib.util.spec_from_file_location("_ref_gdn_decode_triton", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference_triton_decode(mod, inp):
    """Launch the reference decode kernel body once with a fixed tile config."""
    q, k, v, state = inp["q"], inp["k"], inp["v"], inp["state"]
    B, T, HQ, D = q.shape
    HV = v.shape[2]
    out = torch.empty(B, T, HV, D, dtype=torch.bfloat16)
    new_state = torch.empty_like(state)
    fn = mod.gdn_decode_kernel.fn  # bypass the autotuner
    bv = 32
    grid = (B, HV, (D // bv) * T)
    fn[grid](
        q, k, v, state, inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], out, new_state,
        *q.stride(), *k.stride(), *v.stride(), *state.stride(),
        *inp["a"].stride(), *inp["b"].stride(), *out.stride(), *new_state.stride(),
        inp["scale"], HV // HQ, D, HEAD_SIZE=D, BLOCK_V=bv, BLOCK_K=128,
    )
    return out, new_state


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-root", required=True, type=pathlib.Path)
    args = ap.parse_args()
    from flashinfer.trace.templates.gdn import (_gdn_decode_reference, _gdn_mtp_reference,
                                                 _gdn_prefill_reference)

    W = _pkg_workloads()
    ref_triton = _reference_triton_decode(args.reference_root)

    # ---- decode, GVA 2 q/k heads -> 4 v heads, raw (un-normalised) q/k ----
    inp = W.decode_inputs(2, hq=2, hv=4, seed=11)
    o, s = _gdn_decode_reference(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"],
                                 inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
    o_t, s_t = run_reference_triton_decode(ref_triton, inp)
    _save("decode_gva", {**{k_: v_ for k_, v_ in inp.items() if k_ != "scale"},
                         "out": o, "new_state": s, "out_triton": o_t, "new_state_triton": s_t},
          {"scale": inp["scale"], "source": "flashinfer 0.6.11.post2 _gdn_decode_reference; "
                                            "reference gdn_decode Triton kernel (interpreter)"})

    # ---- decode, state=None and scale=0 (defaults), L2-normalised fp32 q/k ----
    inp = W.decode_inputs(3, hq=1, hv=2, seed=12, with_state=False)
    qn = inp["q"].float()
    qn = qn * torch.rsqrt((qn * qn).sum(-1, keepdim=True) + 1e-6)
    kn = inp["k"].float()
    kn = kn * torch.rsqrt((kn * kn).sum(-1, keepdim=True) + 1e-6)
    o, s = _gdn_decode_reference(qn, kn, inp["v"], None, inp["A_log"], inp["a"],
                                 inp["dt_bias"], inp["b"], 0.0)
    _save("decode_nostate_l2", {**{k_: v_ for k_, v_ in inp.items()
                                   if k_ not in ("scale", "state")},
                                "out": o, "new_state": s},
          {"scale": 0.0, "use_qk_l2norm": 1,
           "source": "flashinfer 0.6.11.post2 _gdn_decode_reference on host-normalised q/k"})

    # ---- prefill varlen with an empty sequence and a non-zero initial state ----
    lens = [7, 0, 70]
    inp = W.prefill_inputs(lens, hq=1, hv=2, seed=13)
    qn = inp["q"].float()
    qn = qn * torch.rsqrt((qn * qn).sum(-1, keepdim=True) + 1e-6)
    kn = inp["k"].float()
    kn = kn * torch.rsqrt((kn * kn).sum(-1, keepdim=True) + 1e-6)
    o, s = _gdn_prefill_reference(qn, kn, inp["v"], inp["state"], inp["A_log"], inp["a"],
                                  inp["dt_bias"], inp["b"], inp["cu_seqlens"], inp["scale"])
    _save("prefill_varlen_l2", {**{k_: v_ for k_, v_ in inp.items() if k_ != "scale"},
                                "out": o, "new_state": s},
          {"scale": inp["scale"], "use_qk_l2norm": 1,
           "source": "flashinfer 0.6.11.post2 _gdn_prefill_reference on host-normalised q/k"})

    # ---- prefill, zero initial state, raw q/k (short: raw k grows the state fast) ----
    lens = [64, 33]
    inp = W.prefill_inputs(lens, hq=2, hv=4, seed=14, with_state=False)
    o, s = _gdn_prefill_reference(inp["q"], inp["k"], inp["v"], None, inp["A_log"], inp["a"],
                                  inp["dt_bias"], inp["b"], inp["cu_seqlens"], None)
    _save("prefill_nostate_raw", {**{k_: v_ for k_, v_ in inp.items()
                                     if k_ not in ("scale", "state")},
                                  "out": o, "new_state": s},
          {"scale": 0.0, "use_qk_l2norm": 0,
           "source": "flashinfer 0.6.11.post2 _gdn_prefill_reference"})

    # ---- multi-token decode: GVA 1 -> 2, pool of 4, three rows, raw q/k, rollback buffer ----
    inp = W.mtp_inputs(3, 3, 4, hq=1, hv=2, seed=15, indices=[3, 0, 2])
    inter = torch.zeros(4, 3, 2, 128, 128, dtype=torch.float32)
    o, s = _gdn_mtp_reference(inp["q"], inp["k"], inp["v"], inp["state"], inp["state_indices"],
                              inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"],
                              intermediate_states_buffer=inter)
    _save("mtp_gva_inter", {**{k_: v_ for k_, v_ in inp.items() if k_ != "scale"},
                            "out": o, "final_state": s, "intermediate": inter},
          {"scale": inp["scale"], "use_qk_l2norm": 0,
           "source": "flashinfer 0.6.11.post2 _gdn_mtp_reference"})

    # ---- multi-token decode: int64 indices, default scale, host-normalised q/k ----
    inp = W.mtp_inputs(2, 3, 2, hq=1, hv=2, seed=16, indices=[1, 0],
                       index_dtype=torch.int64)
    qn = inp["q"].float()
    qn = qn * torch.rsqrt((qn * qn).sum(-1, keepdim=True) + 1e-6)
    kn = inp["k"].float()
    kn = kn * torch.rsqrt((kn * kn).sum(-1, keepdim=True) + 1e-6)
    o, s = _gdn_mtp_reference(qn, kn, inp["v"], inp["state"], inp["state_indices"],
                              inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], 0.0)
    _save("mtp_l2", {**{k_: v_ for k_, v_ in inp.items() if k_ != "scale"},
                     "out": o, "final_state": s},
          {"scale": 0.0, "use_qk_l2norm": 1,
           "source": "flashinfer 0.6.11.post2 _gdn_mtp_reference on host-normalised q/k"})


if __name__ == "__main__":
    main()
