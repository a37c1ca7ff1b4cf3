"""Model-side ops of the hot path: the Rosa mixer and the KS3 weight container."""

from .rosa import RosaMixer, _match_payload_sign
from .ks3 import KS3

__all__ = ["RosaMixer", "_match_payload_sign", "KS3"]
