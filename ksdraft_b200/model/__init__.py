"""Model-side ops of the hot path: the Rosa mixer and the vocab-sharded LM head."""

from .rosa import RosaMixer, _match_payload_sign

__all__ = ["RosaMixer", "_match_payload_sign"]
