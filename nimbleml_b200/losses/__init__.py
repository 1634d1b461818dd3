from .cross_entropy import CrossEntropyLoss, tied_cross_entropy

__all__ = ["CrossEntropyLoss", "tied_cross_entropy"]
