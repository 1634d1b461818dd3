from .fused_tied_crossentropy import (
    TiedCEStats,
    fused_tied_crossentropy_backward,
    fused_tied_crossentropy_forward,
)

__all__ = ["TiedCEStats", "fused_tied_crossentropy_forward", "fused_tied_crossentropy_backward"]
