"""Wire messages of the compression session (role of
kvsfuse-vllm0.30.0/mooncake/compression/protocol.py:12-96).

Requests (consumer -> producer): :class:`SessionOpen`, :class:`ChunkPull`,
:class:`SessionAbort`.  Responses: :class:`SessionOpened`,
:class:`ChunkReady`, :class:`SessionAbortAck`.  All are msgspec tagged
structs, so one decoder per direction recognises the type from the payload.

Differences from the reference, which addresses RDMA-registered memory:
the consumer's metadata carries CUDA IPC handles of its frame arena and of
its publish flags, and a pull names ``slot_id`` plus ``slot_offset`` inside
that arena; ``flag_index`` is the u32 publish flag the producer's kernel
release-stores when the chunk's frames have landed.  A consumer that
exports no arena (a peer on another node) receives each chunk's payload
inline in its ``ChunkReady``.
"""
from __future__ import annotations

from typing import Optional, Union

import msgspec

ReqId = str
TransferId = str


class XferMetadata(msgspec.Struct, omit_defaults=True):
    """What the consumer tells the producer when it opens a session."""

    remote_hostname: str
    remote_port: int
    remote_tp_size: int
    remote_tp_rank: int
    # transfer_id -> (consumer request id, block ids per KV-cache group)
    req_blocks: dict[str, tuple[str, list[list[int]]]]
    arena_ipc_handle: bytes = b""
    flags_ipc_handle: bytes = b""
    arena_bytes: int = 0
    slot_bytes: int = 0
    num_slots: int = 0
    block_size: int = 16
    registered_layer_names: list[str] = msgspec.field(default_factory=list)
    registered_layer_indices: list[int] = msgspec.field(default_factory=list)
    num_tokens: int = 0
    logical_blocks_per_chunk: int = 1


class SessionOpen(msgspec.Struct, tag=True, frozen=True):
    metadata: XferMetadata
    nonce: str = ""


class SessionOpened(msgspec.Struct, tag=True, frozen=True):
    logical_block_count: int
    total_chunks: int
    error: Optional[str] = None


class ChunkPull(msgspec.Struct, tag=True, frozen=True):
    transfer_id: TransferId
    d_req_id: ReqId
    chunk_id: int
    slot_id: int
    slot_offset: int
    flag_index: int
    nonce: str = ""


class ChunkReady(msgspec.Struct, tag=True, frozen=True):
    chunk_id: int
    data_bytes: int      # uncompressed bytes the chunk represents
    payload_bytes: int   # bytes written into the slot
    aux_bytes: int = 0
    error: Optional[str] = None
    # the payload itself, when the consumer exported no arena the producer
    # can write (peers on different nodes): the reply carries the slot's bytes
    inline: bytes = b""


class SessionAbort(msgspec.Struct, tag=True, frozen=True):
    transfer_id: TransferId
    d_req_id: ReqId
    reason: str
    nonce: str = ""


class SessionAbortAck(msgspec.Struct, tag=True, frozen=True):
    transfer_id: TransferId
    d_req_id: ReqId
    nonce: str
    error: Optional[str] = None


Request = Union[SessionOpen, ChunkPull, SessionAbort]
Response = Union[SessionOpened, ChunkReady, SessionAbortAck]

_enc = msgspec.msgpack.Encoder()
_req_dec = msgspec.msgpack.Decoder(Request)
_resp_dec = msgspec.msgpack.Decoder(Response)


def encode_message(msg) -> bytes:
    return _enc.encode(msg)


def decode_request(data: bytes) -> Request:
    return _req_dec.decode(data)


def decode_response(data: bytes) -> Response:
    return _resp_dec.decode(data)
