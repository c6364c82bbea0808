"""Coordinator <-> worker control protocol and the control plane that carries it.

Parity: rust/src/distributed/protocol.rs:14-192 (`WorkerCommand`, `WorkerResponse`,
`validate_stationary_continuation`, `validate_stationary_decode`) and the 16-byte worker handshake
{domain_id, capacity_mb} (protocol.rs:301-345, runtime.rs:99-106). The command and response set is
kept so a reference user finds the same verbs; the NIXL exchange commands are dropped (peer memory
is mapped once at start-up through CUDA IPC, see the domain runtime).

Transport: the reference frames bincode messages over QUIC streams (protocol.rs:194-553). Here all
ranks live in one torchrun job, so the control plane is torch.distributed on a gloo group: rank 0
(the coordinator) broadcasts each command to every rank, every rank executes it SPMD, and rank 0
gathers the responses. Messages are dataclasses; `encode`/`decode` turn them into the native
codec's binary frames (csrc/host/protocol.cpp), which is what the control group carries.
"""

from __future__ import annotations

import dataclasses
import struct
from datetime import timedelta
from typing import Any, List, Optional, Sequence

import numpy as np

from ..errors import ProtocolError
from ..host import lib


# --------------------------------------------------------------------------- commands
@dataclasses.dataclass
class Prefill:
    request_id: int
    prompt: List[int]                    # full prompt (every rank extracts its own positions)
    chunks: List[int]
    strategy: str = "vanilla"
    decode_horizon: int = 128
    capacity_tickets: Optional[List[int]] = None
    keep_kv: bool = False
    want_logits: bool = True             # ship the first token's logits to every rank


@dataclasses.dataclass
class Decode:
    request_id: int
    token: int


@dataclasses.dataclass
class DecodeBatch:
    request_tokens: List[Any]            # [(request_id, token)]
    want_logits: bool = True             # False: greedy rows only, no rank needs the logits


@dataclasses.dataclass
class StationaryContinuation:
    request_id: int
    tokens: List[int]
    position_ids: List[int]
    capacity_tickets: List[int]
    starter_domain: int = 0
    decode_horizon: int = 128            # decode tokens the continued request may still take
    want_logits: bool = True             # ship the next token's logits to every rank


@dataclasses.dataclass
class StationaryDecode:
    request_id: int
    token: int
    position: int
    capacity_tickets: List[int]
    starter_domain: int
    token_offset: int
    decode_horizon: int


@dataclasses.dataclass
class SyncGlobalSeqLen:
    request_id: int
    len: int


@dataclasses.dataclass
class ReleaseRequest:
    request_id: int


@dataclasses.dataclass
class Shutdown:
    pass


# --------------------------------------------------------------------------- responses
@dataclasses.dataclass
class PrefillDone:
    request_id: int
    token: int
    global_seq_len: int
    logits: Optional[List[float]] = None


@dataclasses.dataclass
class DecodeDone:
    request_id: int
    token: int


@dataclasses.dataclass
class DecodeBatchDone:
    request_tokens: List[Any]


@dataclasses.dataclass
class StationaryContinuationDone:
    request_id: int
    token: Optional[int] = None


@dataclasses.dataclass
class Ack:
    request_id: int = -1


@dataclasses.dataclass
class Error:
    request_id: int
    message: str


COMMANDS = {c.__name__: c for c in (Prefill, Decode, DecodeBatch, StationaryContinuation,
                                     StationaryDecode, SyncGlobalSeqLen, ReleaseRequest, Shutdown)}
RESPONSES = {c.__name__: c for c in (PrefillDone, DecodeDone, DecodeBatchDone,
                                      StationaryContinuationDone, Ack, Error)}
# wire type ids of the native codec (csrc/host/protocol.cpp): commands 1-8, responses 64-69
TYPE_IDS = {Prefill: 1, Decode: 2, DecodeBatch: 3, StationaryContinuation: 4, StationaryDecode: 5,
            SyncGlobalSeqLen: 6, ReleaseRequest: 7, Shutdown: 8, PrefillDone: 64, DecodeDone: 65,
            DecodeBatchDone: 66, StationaryContinuationDone: 67, Ack: 68, Error: 69}
_BY_ID = {v: k for k, v in TYPE_IDS.items()}
# array fields that stay numpy int64 arrays after decoding (prompt-sized); the other arrays
# become lists
_BULK = {(Prefill, "prompt"), (StationaryContinuation, "tokens"),
         (StationaryContinuation, "position_ids")}


def encode(msg) -> bytes:
    """One binary frame: [u32 payload bytes][u8 version][u8 type][fields], little endian, built
    by the native codec; token arrays travel as raw int64."""
    tid = TYPE_IDS.get(type(msg))
    if tid is None:
        raise ProtocolError(f"not a protocol message: {type(msg).__name__}")
    return lib().encode_frame(tid, [getattr(msg, f.name) for f in dataclasses.fields(msg)])


def decode(frame: bytes):
    """Inverse of `encode`; a short, partial, trailing-byte, wrong-version or unknown-type frame
    raises ProtocolError."""
    tid, values = lib().decode_frame(bytes(frame))
    cls = _BY_ID[tid]
    out = []
    for f, v in zip(dataclasses.fields(cls), values):
        if isinstance(v, np.ndarray) and (cls, f.name) not in _BULK:
            v = v.tolist()
        out.append(v)
    return cls(*out)


def as_plain(msg) -> dict:
    """The message's fields with arrays as lists (for comparisons and logs)."""
    return {f.name: (v.tolist() if isinstance(v, np.ndarray) else v)
            for f in dataclasses.fields(msg) for v in [getattr(msg, f.name)]}


def _check_schemas() -> None:
    for cls, tid in TYPE_IDS.items():
        kinds = lib().message_schema(tid)
        if len(kinds) != len(dataclasses.fields(cls)):
            raise ProtocolError(f"{cls.__name__}: {len(dataclasses.fields(cls))} fields, native "
                                f"schema {kinds!r}")


# --------------------------------------------------------------------------- validators
def validate_stationary_continuation(domains: int, tokens: Sequence[int],
                                     position_ids: Sequence[int], capacity_tickets: Sequence[int],
                                     starter_domain: int) -> None:
    if domains == 0:
        raise ProtocolError("stationary continuation requires at least one domain")
    if len(tokens) == 0:
        raise ProtocolError("stationary continuation requires a non-empty segment")
    if len(tokens) != len(position_ids):
        raise ProtocolError(f"stationary continuation segment/position length mismatch: "
                            f"{len(tokens)} vs {len(position_ids)}")
    if len(capacity_tickets) != domains:
        raise ProtocolError(f"stationary continuation tickets/domains mismatch: "
                            f"{len(capacity_tickets)} vs {domains}")
    if all(t == 0 for t in capacity_tickets):
        raise ProtocolError("stationary continuation tickets must not be all zero")
    if starter_domain >= domains or starter_domain < 0:
        raise ProtocolError(f"stationary continuation starter {starter_domain} out of {domains} domains")


def validate_stationary_decode(domains: int, capacity_tickets: Sequence[int], starter_domain: int,
                               token_offset: int, decode_horizon: int) -> None:
    if domains == 0:
        raise ProtocolError("stationary decode requires at least one domain")
    if len(capacity_tickets) != domains:
        raise ProtocolError(f"stationary decode tickets/domains mismatch: "
                            f"{len(capacity_tickets)} vs {domains}")
    if all(t == 0 for t in capacity_tickets):
        raise ProtocolError("stationary decode tickets must not be all zero")
    if starter_domain >= domains or starter_domain < 0:
        raise ProtocolError(f"stationary decode starter {starter_domain} out of {domains} domains")
    if decode_horizon == 0:
        raise ProtocolError("stationary decode horizon must be non-zero")
    if token_offset >= decode_horizon:
        raise ProtocolError(f"stationary decode token_offset {token_offset} out of horizon "
                            f"{decode_horizon}")


# --------------------------------------------------------------------------- handshake
HANDSHAKE = struct.Struct("<QQ")  # {domain_id u64, capacity_mb u64}: 16 bytes


def pack_handshake(domain_id: int, capacity_mb: int) -> bytes:
    return HANDSHAKE.pack(int(domain_id), int(capacity_mb) & ((1 << 64) - 1))


def unpack_handshake(b: bytes):
    if len(b) != HANDSHAKE.size:
        raise ProtocolError(f"handshake must be {HANDSHAKE.size} bytes, got {len(b)}")
    return HANDSHAKE.unpack(b)


# --------------------------------------------------------------------------- control plane
class ControlPlane:
    """Broadcast commands from rank 0 and gather responses over a gloo process group.

    Every rank must take the same sequence of collective steps; the group's timeout bounds how
    long a rank waits for a peer that died (the reference's HCP_QUIC_TIMEOUT_SECS)."""

    def __init__(self, group=None, rank: int = 0, world: int = 1):
        self.group = group
        self.rank = rank
        self.world = world

    @staticmethod
    def make_group(timeout_s: int = 600):
        import torch.distributed as dist
        return dist.new_group(backend="gloo", timeout=timedelta(seconds=timeout_s))

    def broadcast(self, cmd=None):
        if self.world == 1:
            return cmd
        import torch.distributed as dist
        box = [encode(cmd) if self.rank == 0 else None]
        dist.broadcast_object_list(box, src=0, group=self.group)
        return decode(box[0])

    def gather(self, resp) -> Optional[list]:
        if self.world == 1:
            return [resp]
        import torch.distributed as dist
        out = [None] * self.world if self.rank == 0 else None
        dist.gather_object(encode(resp), out, dst=0, group=self.group)
        return [decode(b) for b in out] if self.rank == 0 else None

    def all_gather(self, obj) -> list:
        if self.world == 1:
            return [obj]
        import torch.distributed as dist
        out = [None] * self.world
        dist.all_gather_object(out, obj, group=self.group)
        return out
