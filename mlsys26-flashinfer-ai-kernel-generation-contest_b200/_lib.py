"""ctypes binding of the in-tree C-ABI library ``libgdn_b200.so`` (see include/gdn_b200.h).

There is deliberately no fallback: if the library is missing the import fails
with instructions to build it, and a failing launch raises.
"""
from __future__ import annotations

import ctypes
import pathlib

_PKG = pathlib.Path(__file__).resolve().parent
LIB_PATH = _PKG / "libgdn_b200.so"

GDN_OK = 0
GDN_ERR_INVALID_ARGUMENT = -1
GDN_ERR_UNSUPPORTED = -2
GDN_ERR_LAUNCH = -3
GDN_ERR_WORKSPACE = -4
GDN_ERR_TOO_LARGE = -5

# Every symbol include/gdn_b200.h declares, with its ctypes signature.
_vp, _i, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_size_t
_ll = ctypes.c_longlong
SIGNATURES = {
    "gdn_b200_version": (_i, []),
    "gdn_status_string": (ctypes.c_char_p, [_i]),
    "gdn_decode_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp,
                               _i, _i, _i, _i, _i, _i, _vp]),
    "gdn_mtp_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _f, _vp, _vp, _vp,
                            _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "gdn_decode_launch_strided": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp,
                                       _i, _i, _i, _i, _i, _i, _ll, _ll, _ll, _ll, _ll, _ll,
                                       _vp]),
    "gdn_decode_launch_bf16state": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp,
                                         _i, _i, _i, _i, _i, _i, _vp]),
    "gdn_mtp_launch_bf16state": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _f, _vp,
                                      _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "gdn_prefill_workspace_size": (_sz, [_i, _i, _i, _i, _i]),
    "gdn_prefill_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _f, _vp, _vp,
                                _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "gdn_prefill_launch_recurrent": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _f,
                                          _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "gdn_prefill_launch_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _f,
                                        _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "gdn_prefill_workspace_size_variant": (_sz, [_i, _i, _i, _i, _i, _i]),
    "gdn_prefill_launch_variant": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _f,
                                        _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "gdn_prefill_launch_strided": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _f,
                                        _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _ll, _ll, _ll, _ll,
                                        _ll, _ll, _vp, _sz, _vp]),
    "gdn_prefill_workspace_size_ext": (_sz, [_i, _i, _i, _i, _i, _i, _i, _i, _i]),
    "gdn_prefill_launch_ext": (_i, [_i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _vp, _vp, _vp, _vp,
                                    _vp, _i, _f, _vp, _vp, _vp, _vp, ctypes.c_longlong, _i, _i,
                                    _i, _i, _i, _i, _i, _i, _vp, _sz, _vp]),
    "gdn_segment_outputs_launch": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "gdn_segment_chain_launch": (_i, [_vp, _i, _i, _vp, _vp, _i, _i, _vp]),
    "gdn_segment_chain_all_launch": (_i, [_vp, _i, _vp, _vp, _i, _i, _vp]),
    "gdn_prefill_segments_auto": (_i, [_i, _i]),
    "gdn_prefill_segment_plan": (_i, [_i, _i, _i, _i, _vp, _i]),
    "gdn_prefill_segmented_workspace_size": (_sz, [_i, _i, _i, _vp]),
    "gdn_prefill_segmented_launch": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp,
                                          _i, _i, _i, _i, _i, _i, _i, _vp, _ll, _ll, _ll, _ll,
                                          _ll, _vp, _sz, _vp]),
    "gdn_device_error": (_i, [_i]),
    "gdn_selftest_bounded_wait": (_i, [ctypes.c_uint, _i, _vp, _vp]),
}

# Prefill kernel selection (gdn_prefill_launch_variant).
GDN_PREFILL_AUTO = 0
GDN_PREFILL_RECURRENT = 1
GDN_PREFILL_FUSED = 2
GDN_PREFILL_SPLIT = 3


def _load() -> ctypes.CDLL:
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python __graft_entry__.py` or "
            f"`python {_PKG.name}/build.py` (needs nvcc with sm_100a support)")
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()


class GDNError(RuntimeError):
    """A C-ABI entry point returned a non-zero status."""

    def __init__(self, where: str, status: int):
        name = LIB.gdn_status_string(status).decode()
        super().__init__(f"{where} failed: {name} ({status})")
        self.status = status


def check(where: str, status: int) -> None:
    if status != GDN_OK:
        raise GDNError(where, status)


def device_error(clear: bool = True) -> int:
    """Synchronise the current device and return the kernels' device-side error bits
    (0 = none; 1 = a TMA wait ran out; 2 = a tensor-core wait ran out; 8 = a streaming
    stage was never released; 16 = the self-test's wait ran out)."""
    return int(LIB.gdn_device_error(int(bool(clear))))
