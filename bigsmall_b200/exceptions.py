"""Exception types.

``BigSmallVersionError`` keeps the reference's constructor and message shape
(BigSmall ``bigsmall/exceptions.py:11-27``) so callers that catch it keep
working.  ``BsGpuError`` and ``BsCorruptError`` carry the C-ABI status code
(and, for device-side stream errors, the per-tensor device status word).
"""
from __future__ import annotations


class BigSmallVersionError(Exception):
    """A container or codec needs a newer release than this one."""

    def __init__(self, required: str, installed: str, *, detail: str | None = None):
        self.required = required
        self.installed = installed
        msg = (
            f"This file requires bigsmall >= {required} (you have {installed}).\n"
            "Run: pip install --upgrade bigsmall"
        )
        if detail:
            msg += f"\n({detail})"
        super().__init__(msg)


class BsGpuError(RuntimeError):
    """A libbsgpu call failed (status code in ``.status``)."""

    def __init__(self, status: int, message: str, device_status=None):
        self.status = status
        self.device_status = device_status
        super().__init__(message)


class BsCorruptError(ValueError):
    """A compressed stream is malformed (bad magic, truncated, corrupt words,
    count mismatch).  A ValueError, like the reference's decoders raise."""

    def __init__(self, status: int, message: str, device_status=None):
        self.status = status
        self.device_status = device_status
        super().__init__(message)
