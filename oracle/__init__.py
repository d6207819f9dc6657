"""Test-infrastructure oracle (CPU) for the GDN hot path; never on the product path."""
from .gdn_oracle import (  # noqa: F401
    decode,
    flashinfer_allclose,
    gates,
    l2norm,
    prefill,
    state_rel_err,
)
