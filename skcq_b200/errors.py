"""Error types (the convention of skcq/errors.py:4-22).

``ValueError`` / ``RuntimeError`` are bugs and are left to crash.
``InfrastructureError`` marks failures of the machinery around the
computation, which job loops catch at their boundary and may retry.
``DeviceTimeoutError`` is the one raised by this package: a kernel's bounded
wait ran out (a pipeline partner did not arrive within about two seconds, as
when the GPU is preempted or overloaded). The kernel returned and the CUDA
context stays usable, so the job can be run again.
"""

from __future__ import annotations


class InfrastructureError(Exception):
    """An infrastructure failure; ``context`` carries what the job was."""

    def __init__(self, message: str = "", *, context: dict[str, object] | None = None) -> None:
        super().__init__(message)
        self.context = context or {}
        self.message = message


class DeviceTimeoutError(InfrastructureError):
    """A device-side bounded wait gave up (device error code in ``code``)."""

    def __init__(self, message: str, code: int) -> None:
        super().__init__(message, context={"device_code": code})
        self.code = code


# device error codes of a bounded wait that ran out (include/skcq_b200.h)
WAIT_TIMEOUT_CODES = frozenset(range(11, 20)) | frozenset(range(51, 60)) | {90}
