"""Error types and numerical tolerance tiers.

Parity: the reference's `RingError` and `ToleranceTier` (rust/src/error.rs:14-77). The tier
constants are kept identical because the correctness suite reports against them.
"""

from __future__ import annotations

import dataclasses
import enum


class RingError(Exception):
    """Base class for every framework error."""


class InvalidChunkSum(RingError):
    def __init__(self, actual: int, expected: int):
        super().__init__(f"sum(seq_chunk_len)={actual} does not match global_seq_len={expected}")
        self.actual = actual
        self.expected = expected


class InvalidDomain(RingError):
    def __init__(self, domain_id: str):
        super().__init__(f"domain {domain_id} has invalid seq_chunk_len or block_size")
        self.domain_id = domain_id


class InvalidCli(RingError):
    pass


class ProtocolError(RingError):
    pass


class CapacityError(RingError):
    """KV byte admission / reservation failure."""


class Overloaded(RingError):
    """The coordinator's queue is at its limit; the HTTP API answers 503 (retry later)."""


class AdmissionError(RingError):
    """The coordinator rejected a request before any rank ran it (e.g. a prompt shorter than
    the number of ranks). The HTTP API answers 400, as for a `CapacityError`."""


class KernelError(RingError):
    """A device kernel reported a failure through the runtime status word."""


class PeerTimeout(KernelError):
    """A bounded device- or host-side wait on a peer rank ran out."""


class NativeExtensionMissing(RingError):
    """The compiled sm_100a extension is not importable on a machine that has a GPU."""


@dataclasses.dataclass(frozen=True)
class Tolerance:
    max_abs_err: float
    mean_abs_err: float
    max_rel_err: float


class ToleranceTier(enum.Enum):
    STRICT = "strict"
    RELAXED = "relaxed"
    END_TO_END = "end-to-end"

    @classmethod
    def parse(cls, s: str) -> "ToleranceTier":
        table = {
            "strict": cls.STRICT, "s": cls.STRICT,
            "relaxed": cls.RELAXED, "r": cls.RELAXED,
            "end-to-end": cls.END_TO_END, "e2e": cls.END_TO_END, "e": cls.END_TO_END,
        }
        try:
            return table[s]
        except KeyError:
            raise InvalidCli(f"unknown tolerance tier: {s}") from None

    def tolerance(self) -> Tolerance:
        return {
            ToleranceTier.STRICT: Tolerance(1e-5, 1e-6, 1e-5),
            ToleranceTier.RELAXED: Tolerance(1e-4, 1e-5, 1e-4),
            ToleranceTier.END_TO_END: Tolerance(1e-3, 1e-4, 1e-3),
        }[self]
