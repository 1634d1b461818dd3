"""Bindings that run the reference NimbleML package's own tied-CE path on this library's kernels."""
