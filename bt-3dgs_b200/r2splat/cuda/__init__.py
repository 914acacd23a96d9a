"""Lazy access to the compiled sm_100a library (see ``_backend``)."""

from ._wrapper import is_cuda_extension_available

__all__ = ["is_cuda_extension_available"]
