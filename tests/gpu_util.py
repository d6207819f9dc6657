"""Helpers shared by the GPU parity tests (CUDA path vs the CPU oracle)."""
import torch

from oracle import gdn_oracle as O

OUT_ATOL = 2e-2      # bf16 outputs: flashinfer rule, 100% of elements must match
OUT_RTOL = 2e-2
STATE_REL = 1e-3     # fp32 final state: ||dS|| / ||S_ref||
CONTEST_TOL = 1e-2   # the contest's own atol = rtol bar, also checked on outputs


def to(d, dev):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in d.items()}


def oracle_decode(inp, l2):
    q, k = (O.l2norm(inp["q"]), O.l2norm(inp["k"])) if l2 else (inp["q"], inp["k"])
    return O.decode(q, k, inp["v"], inp.get("state"), inp["A_log"], inp["a"], inp["dt_bias"],
                    inp["b"], inp.get("scale"))


def oracle_prefill(inp, l2):
    q, k = (O.l2norm(inp["q"]), O.l2norm(inp["k"])) if l2 else (inp["q"], inp["k"])
    return O.prefill(q, k, inp["v"], inp.get("state"), inp["A_log"], inp["a"], inp["dt_bias"],
                     inp["b"], inp["cu_seqlens"], inp.get("scale"))


def assert_parity(out, new_state, ref_out, ref_state, *, state_rel=STATE_REL, out_tol=OUT_ATOL,
                  what=""):
    out = out.cpu()
    new_state = new_state.cpu()
    ok, frac, max_abs, max_rel = O.flashinfer_allclose(out, ref_out, out_tol, out_tol)
    assert ok, f"{what} output mismatch: matched {frac:.6f}, max abs {max_abs:.3e}"
    err = O.state_rel_err(new_state, ref_state)
    assert err <= state_rel, f"{what} state rel err {err:.3e} > {state_rel:.1e}"
    assert torch.isfinite(new_state).all()
    return err, max_abs
