"""CPU oracle package (test infrastructure only; never on the product path)."""
from .dynconv_oracle import (  # noqa: F401
    headwise_bwd,
    headwise_fwd,
    lowrank_bwd,
    lowrank_fwd,
    shift_future,
    shift_past,
)
