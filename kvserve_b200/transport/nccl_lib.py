"""Minimal ctypes binding of the NCCL point-to-point API (the library that
PyTorch bundles), enough for a 2-rank producer/consumer communicator:
``ncclGetUniqueId``, ``ncclCommInitRank``, ``ncclSend``, ``ncclRecv``,
``ncclCommDestroy``.  Used by the uncompressed/modular baseline transport;
the product hand-off does not use NCCL for KV."""
from __future__ import annotations

import ctypes
import glob
import os
from typing import Optional

import torch

_DTYPES = {torch.uint8: 1, torch.int8: 0, torch.int32: 2, torch.int64: 4, torch.float16: 6, torch.float32: 7,
           torch.float64: 8, torch.bfloat16: 9}


class NcclUniqueId(ctypes.Structure):
    _fields_ = [("internal", ctypes.c_byte * 128)]


def _find_lib() -> str:
    env = os.environ.get("KVSERVE_NCCL_LIB")
    if env:
        return env
    try:
        import nvidia.nccl
        base = list(nvidia.nccl.__path__)[0]
        cands = glob.glob(os.path.join(base, "lib", "libnccl.so*"))
        if cands:
            return cands[0]
    except ImportError:
        pass
    return "libnccl.so.2"


class NcclLib:
    _instance: Optional["NcclLib"] = None

    def __init__(self, path: Optional[str] = None):
        self.lib = ctypes.CDLL(path or _find_lib())
        L = self.lib
        L.ncclGetUniqueId.argtypes = [ctypes.POINTER(NcclUniqueId)]
        L.ncclCommInitRank.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, NcclUniqueId, ctypes.c_int]
        L.ncclSend.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                               ctypes.c_void_p]
        L.ncclRecv.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                               ctypes.c_void_p]
        L.ncclCommDestroy.argtypes = [ctypes.c_void_p]
        L.ncclGetErrorString.argtypes = [ctypes.c_int]
        L.ncclGetErrorString.restype = ctypes.c_char_p

    @classmethod
    def get(cls) -> "NcclLib":
        if cls._instance is None:
            cls._instance = NcclLib()
        return cls._instance

    def _check(self, rc: int) -> None:
        if rc != 0:
            raise RuntimeError(f"NCCL error {rc}: {self.lib.ncclGetErrorString(rc).decode()}")

    def unique_id(self) -> bytes:
        uid = NcclUniqueId()
        self._check(self.lib.ncclGetUniqueId(ctypes.byref(uid)))
        return bytes(bytearray(uid.internal))

    def comm_init(self, nranks: int, uid_bytes: bytes, rank: int) -> int:
        uid = NcclUniqueId()
        ctypes.memmove(uid.internal, uid_bytes, len(uid_bytes))
        comm = ctypes.c_void_p()
        self._check(self.lib.ncclCommInitRank(ctypes.byref(comm), nranks, uid, rank))
        return comm.value

    def send(self, t: torch.Tensor, peer: int, comm: int, stream: int) -> None:
        self._check(self.lib.ncclSend(ctypes.c_void_p(t.data_ptr()), t.numel(), _DTYPES[t.dtype], peer,
                                      ctypes.c_void_p(comm), ctypes.c_void_p(stream)))

    def recv(self, t: torch.Tensor, peer: int, comm: int, stream: int) -> None:
        self._check(self.lib.ncclRecv(ctypes.c_void_p(t.data_ptr()), t.numel(), _DTYPES[t.dtype], peer,
                                      ctypes.c_void_p(comm), ctypes.c_void_p(stream)))

    def destroy(self, comm: int) -> None:
        if comm:
            self.lib.ncclCommDestroy(ctypes.c_void_p(comm))
