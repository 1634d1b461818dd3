from .cross_entropy import CrossEntropyLoss, tied_cross_entropy
from .sampled_cross_entropy import SampledCrossEntropyLoss, sample_negative_indices

__all__ = ["CrossEntropyLoss", "SampledCrossEntropyLoss", "sample_negative_indices", "tied_cross_entropy"]
