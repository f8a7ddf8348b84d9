"""Chunked compression-session protocol between a prefill (producer) and a
decode (consumer) worker: the role of the reference's Mooncake compression
session (kvsfuse-vllm0.30.0/mooncake/compression/{protocol,state,tokens}.py,
session_ipc.py, session_process.py), re-designed for one NVSwitch node.

The consumer owns receive slots in CUDA-IPC-exported device memory; a pull
names a slot by id and byte offset inside the exported arena (not a raw
RDMA address), and the producer's fused encode kernel stores the chunk's
frames straight into that slot over NVLink.  The control plane is ZeroMQ
with msgspec-encoded tagged messages; the state machines live in
:mod:`.service`, optionally in a helper process (:mod:`.process`).
"""
from .protocol import (ChunkPull, ChunkReady, SessionAbort, SessionAbortAck, SessionOpen, SessionOpened,
                       XferMetadata, decode_request, decode_response, encode_message)
from .state import (ConsumerSession, ProducerSession, ReceiveSlot, ReceiveSlotState, SessionState,
                    IllegalTransition)
from .tokens import chunk_token_counts, suffix_token_counts

__all__ = ["ChunkPull", "ChunkReady", "SessionAbort", "SessionAbortAck", "SessionOpen", "SessionOpened",
           "XferMetadata", "decode_request", "decode_response", "encode_message", "ConsumerSession",
           "ProducerSession", "ReceiveSlot", "ReceiveSlotState", "SessionState", "IllegalTransition",
           "chunk_token_counts", "suffix_token_counts"]
