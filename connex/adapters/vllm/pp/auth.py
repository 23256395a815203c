"""Authenticated control frames (reference ``connex/adapters/vllm/pp/auth.py``).

Control messages between pipeline stages may carry pickled objects, and
unpickling runs code; every frame therefore carries an HMAC-SHA256 tag over
its payload under a secret shared by the deployment's stages, and a frame
whose tag does not verify is dropped before anything is unpickled.

Secret: ``CONNEX_PP_SECRET`` (value) or ``CONNEX_PP_SECRET_FILE`` (a file
holding it, surrounding whitespace ignored), at least 16 bytes.
``CONNEX_PP_AUTH=off`` disables the check (trusted test networks only);
with neither, :func:`load_secret` refuses.

Frame layout: ``b"CXA1" + HMAC-SHA256(secret, payload)[:16] + payload``.  The
tag covers the payload only, so a captured frame can be replayed; the step
protocol tolerates duplicates (each step carries its epoch and sequence).
"""
from __future__ import annotations

import hashlib
import hmac
import logging
import os
from typing import Mapping, Optional

log = logging.getLogger("connex.pp.auth")

MAGIC = b"CXA1"
TAG_LEN = 16
MIN_SECRET = 16


class AuthError(RuntimeError):
    pass


def load_secret(env: Optional[Mapping[str, str]] = None) -> Optional[bytes]:
    """The shared secret, or None when authentication is switched off."""
    env = os.environ if env is None else env
    if env.get("CONNEX_PP_AUTH", "on").strip().lower() in ("off", "0", "no", "false"):
        return None
    val = env.get("CONNEX_PP_SECRET")
    path = env.get("CONNEX_PP_SECRET_FILE")
    if not val and path:
        try:
            with open(path, "rb") as f:
                val = f.read().strip()
        except OSError as ex:
            raise AuthError(f"CONNEX_PP_SECRET_FILE={path}: {ex}") from ex
    if not val:
        raise AuthError("control frames are authenticated: set CONNEX_PP_SECRET or CONNEX_PP_SECRET_FILE to the "
                        "same secret on every stage, or CONNEX_PP_AUTH=off on a trusted network")
    key = val.encode() if isinstance(val, str) else bytes(val)
    if len(key) < MIN_SECRET:
        raise AuthError(f"CONNEX_PP_SECRET needs at least {MIN_SECRET} bytes")
    return key


class FrameAuth:
    """``seal`` / ``open`` frames with ``key`` (None: pass-through)."""

    def __init__(self, key: Optional[bytes]):
        self.key = key
        self.rejected = 0
        if key is None:
            log.warning("CONNEX_PP_AUTH=off: control frames are not authenticated")

    def _tag(self, payload) -> bytes:
        return hmac.new(self.key, payload, hashlib.sha256).digest()[:TAG_LEN]

    def seal(self, payload: bytes) -> bytes:
        return payload if self.key is None else MAGIC + self._tag(payload) + payload

    def open(self, frame) -> Optional[memoryview]:
        """The payload of a frame whose tag verifies, else None."""
        view = memoryview(frame)
        if self.key is None:
            return view
        head = len(MAGIC) + TAG_LEN
        if len(view) < head or bytes(view[:len(MAGIC)]) != MAGIC:
            self.rejected += 1
            return None
        payload = view[head:]
        if not hmac.compare_digest(bytes(view[len(MAGIC):head]), self._tag(payload)):
            self.rejected += 1
            return None
        return payload
