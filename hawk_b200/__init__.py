"""hawk_b200: a B200-native (sm_100a) device execution path for hawk kernels."""

from .errors import HawkError

__all__ = ["HawkError"]
