"""Agent sessions with stable logical ids that move between serving
instances (balancing, scale-down, failure) without the client noticing
(reference ``connex/agents/__init__.py``)."""
from .session import HEADER, KVMover, ReprefillMover, Session, SessionProxy

__all__ = ["HEADER", "KVMover", "ReprefillMover", "Session", "SessionProxy"]
