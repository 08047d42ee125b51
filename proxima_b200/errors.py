"""ProximaError and its variants, as crates/proxima-core/src/error.rs:37-160 defines them.

The C ABI returns one status code per variant; ``raise_for_status`` turns a
status plus the pxc_error payload back into the matching exception.
"""
from __future__ import annotations


class ProximaError(Exception):
    """Base of every error the library raises (ProximaError)."""

    def is_caller_error(self) -> bool:
        """crates/proxima-core/src/error.rs:204-213."""
        return isinstance(self, (DimensionMismatch, UnknownId, DuplicateId, NonFinite, Configuration))


class DimensionMismatch(ProximaError):
    def __init__(self, expected: int, actual: int):
        super().__init__(f"dimension mismatch: index holds {expected}-dimensional vectors, got {actual}")
        self.expected, self.actual = expected, actual


class UnknownId(ProximaError):
    def __init__(self, id: int):
        super().__init__(f"unknown vector id {id}")
        self.id = id


class DuplicateId(ProximaError):
    def __init__(self, id: int):
        super().__init__(f"duplicate vector id {id}")
        self.id = id


class Capacity(ProximaError):
    def __init__(self, what: str, limit: int):
        super().__init__(f"capacity exceeded: {what} limit is {limit}")
        self.what, self.limit = what, limit


class NonFinite(ProximaError):
    def __init__(self, index: int, value: float = float("nan")):
        super().__init__(f"vector component {index} is not finite ({value})")
        self.index, self.value = index, value


class Corruption(ProximaError):
    def __init__(self, structure: str, detail: str):
        super().__init__(f"corrupt {structure}: {detail}")
        self.structure, self.detail = structure, detail


class Configuration(ProximaError):
    def __init__(self, parameter: str, value, reason: str):
        super().__init__(f"invalid configuration: {parameter} = {value} ({reason})")
        self.parameter, self.value, self.reason = parameter, value, reason


class Internal(ProximaError):
    def __init__(self, location: str, detail: str):
        super().__init__(f"internal invariant violated in {location}: {detail}")
        self.location, self.detail = location, detail


class Io(ProximaError):
    def __init__(self, operation: str, path: str, detail: str):
        super().__init__(f"{operation} failed on {path}: {detail}")


class DeviceTimeout(Internal):
    """A bounded device-side wait gave up (PXC_TIMEOUT); maps to Internal."""


def raise_for_status(status: int, a: int, b: int, parameter: str, detail: str) -> None:
    if status == 1:
        raise DimensionMismatch(a, b)
    if status == 2:
        raise UnknownId(a)
    if status == 3:
        raise DuplicateId(a)
    if status == 4:
        raise Capacity(detail, a)
    if status == 5:
        raise NonFinite(a)
    if status == 6:
        raise Corruption(parameter or "device mirror", detail)
    if status == 7:
        raise Configuration(parameter, a, detail)
    if status == 11:
        raise DeviceTimeout("device wait", detail)
    if status == 10:
        raise Internal("cuda", detail)
    raise Internal("libproxima_cuda", f"status {status}: {detail}")
