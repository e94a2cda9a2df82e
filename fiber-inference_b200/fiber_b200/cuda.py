"""Device API bindings (filled in with libfiber_cuda.so)."""
__all__ = []
