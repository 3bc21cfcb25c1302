def _autoload():
    """torch.backends entry point (called by torch at import time)."""
    import fp4_fp8_for_torch_mps  # noqa: F401
