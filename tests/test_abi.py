"""CPU: the C-ABI library loads, exports what include/*.h declares, and rejects bad
arguments before touching a GPU; the host mirror validates like the reference."""
import ctypes
import re

import pytest
import torch

from conftest import REPO, load_pkg

HEADERS = sorted((REPO / "include").glob("*.h"))


def declared_functions():
    names = []
    for h in HEADERS:
        text = h.read_text()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(gdn_\w+)\s*\(", text, flags=re.M):
            names.append(m.group(1))
    return sorted(set(names))


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("gdn_decode_launch", "gdn_prefill_launch", "gdn_prefill_workspace_size"):
        assert required in names


def test_library_exports_every_declared_symbol():
    pkg = load_pkg()
    lib = ctypes.CDLL(str(pkg.LIB_PATH))
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"
    # and the Python binding knows every one of them
    from importlib import import_module
    binding = import_module(pkg.__name__ + "._lib")
    assert set(binding.SIGNATURES) == set(declared_functions())


def test_status_strings():
    pkg = load_pkg()
    assert pkg.LIB.gdn_b200_version() >= 100
    assert pkg.LIB.gdn_status_string(0) == b"GDN_OK"
    assert pkg.LIB.gdn_status_string(-4) == b"GDN_ERR_WORKSPACE"


def _decode_call(lib, **kw):
    args = dict(q=None, k=None, v=None, state=None, A_log=None, a=None, dt_bias=None, b=None,
                scale=0.0, out=None, ns=None, batch=1, hq=16, hk=16, hv=32, d=128, l2=0,
                stream=None)
    args.update(kw)
    return lib.gdn_decode_launch(*args.values())


def test_decode_argument_checks_return_before_launch():
    lib = load_pkg().LIB
    assert _decode_call(lib, batch=0) == 0                      # no-op
    assert _decode_call(lib, d=64) == -2                        # unsupported head size
    assert _decode_call(lib, hk=8) == -2                        # HK != HQ
    assert _decode_call(lib, hv=24) == -2                       # HV % HQ != 0
    assert _decode_call(lib, batch=-1) == -1
    assert _decode_call(lib) == -1                              # null pointers
    fake = 0x1000
    assert _decode_call(lib, q=fake + 2, k=fake, v=fake, A_log=fake, a=fake, dt_bias=fake,
                        b=fake, out=fake, ns=fake) == -1        # misaligned q


def test_prefill_argument_checks_return_before_launch():
    lib = load_pkg().LIB
    call = lambda **kw: lib.gdn_prefill_launch(*{**dict(  # noqa: E731
        q=None, k=None, v=None, state=None, A_log=None, a=None, dt_bias=None, b=None, cu=None,
        cu64=0, scale=0.0, out=None, ns=None, T=10, N=1, hq=16, hk=16, hv=32, d=128, l2=0,
        ws=None, wsb=0, stream=None), **kw}.values())
    assert call(N=0) == 0
    assert call(d=256) == -2
    assert call() == -1
    assert call(T=-1) == -1
    fake = 0x1000
    ptrs = dict(q=fake, k=fake, v=fake, A_log=fake, a=fake, dt_bias=fake, b=fake, cu=fake,
                out=fake, ns=fake)
    size = lib.gdn_prefill_workspace_size_variant(3, 4096, 1, 16, 32, 128)
    assert size > 0
    # a workspace that is not 16-byte aligned is refused before anything is launched
    vcall = lambda **kw: lib.gdn_prefill_launch_variant(3, *{**dict(  # noqa: E731
        q=None, k=None, v=None, state=None, A_log=None, a=None, dt_bias=None, b=None, cu=None,
        cu64=0, scale=0.0, out=None, ns=None, T=4096, N=1, hq=16, hk=16, hv=32, d=128, l2=1,
        ws=None, wsb=0, stream=None), **kw}.values())
    assert vcall(**ptrs, ws=fake + 8, wsb=size) == -1
    assert vcall(**ptrs, ws=fake, wsb=size - 1) == -4  # too small


def test_host_rejects_cpu_tensors_and_bad_dtypes():
    pkg = load_pkg()
    W = pkg.workloads
    inp = W.decode_inputs(1, hq=1, hv=2)
    with pytest.raises(ValueError, match="CUDA"):
        pkg.gdn_decode(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"],
                       inp["dt_bias"], inp["b"], inp["scale"])
    with pytest.raises(TypeError):
        pkg.gdn_decode([1], inp["k"], inp["v"], None, inp["A_log"], inp["a"], inp["dt_bias"],
                       inp["b"], 0.0)


def test_dps_entry_point_arity_matches_reference():
    """flashinfer-bench checks the DPS parameter count: 11 (decode) / 12 (prefill)."""
    import inspect
    pkg = load_pkg()
    assert len(inspect.signature(pkg.decode_kernel).parameters) == 11
    assert len(inspect.signature(pkg.prefill_kernel).parameters) == 12
    assert list(inspect.signature(pkg.prefill_kernel).parameters)[8] == "cu_seqlens"


def test_strided_entry_points_refuse_overlapping_or_unaligned_rows():
    """The strided entry points check the row strides before anything is launched: rows
    of one tensor must not overlap and q/k rows must stay 8-byte aligned."""
    lib = load_pkg().LIB
    fake = 0x1000
    dense = dict(qs=16 * 128, ks=16 * 128, vs=32 * 128, as_=32, bs=32, os=32 * 128)

    def dcall(**kw):
        s = {**dense, **kw}
        return lib.gdn_decode_launch_strided(fake, fake, fake, None, fake, fake, fake, fake, 0.0,
                                             fake, fake, 4, 16, 16, 32, 128, 0, s["qs"], s["ks"],
                                             s["vs"], s["as_"], s["bs"], s["os"], None)

    def pcall(**kw):
        s = {**dense, **kw}
        return lib.gdn_prefill_launch_strided(0, fake, fake, fake, None, fake, fake, fake, fake,
                                              fake, 0, 0.0, fake, fake, 100, 1, 16, 16, 32, 128,
                                              1, s["qs"], s["ks"], s["vs"], s["as_"], s["bs"],
                                              s["os"], None, 0, None)

    for call in (dcall, pcall):
        assert call(qs=16 * 128 - 8) == -1   # q rows overlap
        assert call(vs=31 * 128) == -1       # v rows overlap
        assert call(os=32 * 128 - 1) == -1  # output rows overlap
        assert call(as_=31) == -1            # a rows overlap
        assert call(ks=16 * 128 + 2) == -1   # k rows lose their 8-byte alignment


def test_row_stride_of_views():
    pkg = load_pkg()
    from importlib import import_module
    C = import_module(pkg.__name__ + "._checks")
    fused = torch.zeros(10, 2 * 16 * 128 + 32 * 128, dtype=torch.bfloat16)
    q = fused[:, :16 * 128].view(10, 16, 128)
    v = fused[:, 2 * 16 * 128:].view(10, 32, 128)
    assert C.row_stride(q) == fused.stride(0) and C.row_stride(v) == fused.stride(0)
    assert C.row_stride(torch.zeros(10, 16, 128)) == 16 * 128
    assert C.row_stride(q.transpose(1, 2)) is None          # heads not dense: copied
    x, rs = C.rows_in(q.transpose(1, 2))
    assert x.is_contiguous() and rs == 16 * 128
    odd = torch.zeros(10, 16 * 128 + 2, dtype=torch.bfloat16)[:, :16 * 128].view(10, 16, 128)
    assert C.row_stride(odd, 4) is None and C.row_stride(odd) == 16 * 128 + 2


def test_selftest_argument_checks_return_before_launch():
    lib = load_pkg().LIB
    assert lib.gdn_selftest_bounded_wait(0, 0, None, None) == -1          # no polls
    assert lib.gdn_selftest_bounded_wait((1 << 24) + 1, 0, None, None) == -1
    assert lib.gdn_selftest_bounded_wait(16, 0, 0x1002, None) == -1       # misaligned


def test_segmented_argument_checks_return_before_launch():
    lib = load_pkg().LIB
    fake = 0x10000

    def call(T=256, hq=2, hk=2, hv=4, hd=128, segments=2, ns=fake, qs=256):
        return lib.gdn_prefill_segmented_launch(
            fake, fake, fake, None, fake, fake, fake, fake, 0.0, fake, ns, T, hq, hk, hv, hd, 1,
            segments, None, qs, 256, 512, 4, 4, fake, 1 << 30, None)
    assert call(T=-1) == -1                      # GDN_ERR_INVALID_ARGUMENT
    assert call(segments=-1) == -1
    assert call(ns=None) == -1
    assert call(ns=fake + 4) == -1               # new_state not 16-byte aligned
    assert call(hk=4) == -2                      # GDN_ERR_UNSUPPORTED
    assert call(hd=64) == -2
    assert call(qs=128) == -1                    # q rows overlap
    # sizes need no device: S = min(segments, chunks); one segment has no scratch rows
    size = lib.gdn_prefill_segmented_workspace_size
    assert size(0, 4, 2, None) == 0
    assert size(256, 4, 2, None) > size(256, 4, 1, None) > 0
    assert size(256, 4, 64, None) == size(256, 4, 4, None)   # capped at the 4 chunks
    import ctypes
    arr = lambda *x: (ctypes.c_int * len(x))(*x)  # noqa: E731
    assert size(256, 4, 2, arr(0, 128, 256)) == size(256, 4, 2, None)
    assert size(256, 4, 2, arr(0, 192, 256)) < size(256, 4, 2, None)   # fewer scratch rows
    for bad in (arr(0, 100, 256), arr(0, 256, 256), arr(64, 128, 256), arr(0, 128, 255)):
        assert size(256, 4, 2, bad) == 0
        assert lib.gdn_prefill_segmented_launch(
            fake, fake, fake, None, fake, fake, fake, fake, 0.0, fake, fake, 256, 2, 2, 4, 128,
            1, 2, bad, 256, 256, 512, 4, 4, fake, 1 << 30, None) == -1
