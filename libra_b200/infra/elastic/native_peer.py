"""ctypes front end of the native ``peer_xfer`` library (``libra_b200/native``).

Role of the reference's ``infra/elastic/native_rdma.py`` (``NativeRDMAFileTransfer
:34-229`` builds the verbs helper, runs server/client subprocesses and ships a
serialized payload; gradient client/server on top ``:232-365``).  On one
NVSwitch box the native service moves buffers directly: a receiver registers
destination buffers, a sender exports its buffer (CUDA IPC handle or POSIX
shared memory) and pushes it as a copy or an element-wise add, which the
receiver's GPU executes by reading the peer memory over NVLink.  Unlike the
reference helper, a push is a request/response, so lockstep gradient exchange
works over it.
"""

from __future__ import annotations

import ctypes
import os
import secrets
import threading
from dataclasses import dataclass
from typing import Dict, Optional, Sequence

import torch

from libra_b200.infra.elastic.hybrid_pool import GradientPayload

LIB_PATH = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(__file__))), "native", "libpeer_xfer.so")

KIND_HOST, KIND_DEVICE = 0, 1
OP_COPY, OP_ADD = 0, 1
DTYPE_F32, DTYPE_BF16 = 0, 1
ERRORS = {1: "connect", 2: "auth", 3: "unknown buffer", 4: "range", 5: "map", 6: "cuda", 7: "timeout", 8: "protocol"}
_DTYPE_CODES = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16}


class LpxHandle(ctypes.Structure):
    _pack_ = 1
    _fields_ = [("kind", ctypes.c_int32), ("device", ctypes.c_int32), ("bytes", ctypes.c_uint64),
                ("offset", ctypes.c_uint64), ("pid", ctypes.c_int64), ("local_ptr", ctypes.c_uint64),
                ("ipc", ctypes.c_char * 64), ("shm_name", ctypes.c_char * 64)]


class PeerXferError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"peer_xfer error {code} ({ERRORS.get(code, '?')}): {message}")
        self.code = code


_LIB = None
_LIB_LOCK = threading.Lock()


def library(path: str = LIB_PATH):
    """Load the native library (raises with a build hint when absent)."""
    global _LIB
    with _LIB_LOCK:
        if _LIB is None:
            if not os.path.exists(path):
                raise RuntimeError(f"{path} is not built; run `make -C libra_b200/native`")
            lib = ctypes.CDLL(path)
            P, H = ctypes.c_void_p, ctypes.POINTER(LpxHandle)
            sig = {"lpx_last_error": (ctypes.c_char_p, []),
                   "lpx_host_alloc": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(P), H]),
                   "lpx_host_free": (ctypes.c_int, [P, ctypes.c_uint64, ctypes.c_char_p, ctypes.c_int]),
                   "lpx_export_device": (ctypes.c_int, [P, ctypes.c_uint64, H]),
                   "lpx_server_create": (P, [ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p]),
                   "lpx_server_port": (ctypes.c_int, [P]),
                   "lpx_server_register": (ctypes.c_int, [P, ctypes.c_char_p, P, ctypes.c_uint64, ctypes.c_int,
                                                          ctypes.c_int]),
                   "lpx_server_stats": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_longlong),
                                                       ctypes.POINTER(ctypes.c_longlong)]),
                   "lpx_server_destroy": (ctypes.c_int, [P]),
                   "lpx_push": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p, H,
                                               ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_double])}
            for name, (res, args) in sig.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            _LIB = lib
    return _LIB


def available() -> bool:
    try:
        library()
        return True
    except (RuntimeError, OSError):
        return False


def _check(rc: int) -> None:
    if rc != 0:
        raise PeerXferError(rc, library().lpx_last_error().decode("utf-8", "replace"))


class HostBuffer:
    """Host memory in POSIX shared memory, exportable to a peer_xfer server."""

    def __init__(self, nbytes: int, name: Optional[str] = None):
        self.name = name or f"/libra_pxf_{os.getpid()}_{secrets.token_hex(6)}"
        self.nbytes = int(nbytes)
        self.handle = LpxHandle()
        ptr = ctypes.c_void_p()
        _check(library().lpx_host_alloc(self.name.encode(), self.nbytes, ctypes.byref(ptr), ctypes.byref(self.handle)))
        self._ptr = ptr.value

    def tensor(self, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """A CPU tensor view of the shared memory (valid until ``close``)."""
        arr = (ctypes.c_uint8 * self.nbytes).from_address(self._ptr)
        return torch.frombuffer(arr, dtype=torch.uint8).view(dtype)

    def close(self) -> None:
        if self._ptr:
            library().lpx_host_free(ctypes.c_void_p(self._ptr), self.nbytes, self.name.encode(), 1)
            self._ptr = None


def export_tensor(t: torch.Tensor) -> LpxHandle:
    """Export a CUDA tensor's bytes (CUDA IPC handle of its allocation + offset)."""
    if not t.is_cuda or not t.is_contiguous():
        raise ValueError("export_tensor needs a contiguous CUDA tensor")
    h = LpxHandle()
    _check(library().lpx_export_device(ctypes.c_void_p(t.data_ptr()), t.numel() * t.element_size(), ctypes.byref(h)))
    return h


class PeerXferServer:
    def __init__(self, host: str = "127.0.0.1", port: int = 0, token: Optional[str] = None):
        self.host = host
        self.token = token if token is not None else secrets.token_hex(16)
        lib = library()
        self._srv = lib.lpx_server_create(host.encode(), int(port), self.token.encode())
        if not self._srv:
            raise PeerXferError(1, lib.lpx_last_error().decode())
        self.port = lib.lpx_server_port(self._srv)
        self._keep: Dict[str, torch.Tensor] = {}

    def register(self, name: str, t: torch.Tensor) -> None:
        if not t.is_contiguous() or t.dtype not in _DTYPE_CODES:
            raise ValueError("destination must be a contiguous fp32 or bf16 tensor")
        dev = t.device.index if t.is_cuda else -1
        _check(library().lpx_server_register(self._srv, name.encode(), ctypes.c_void_p(t.data_ptr()),
                                             t.numel() * t.element_size(), dev, _DTYPE_CODES[t.dtype]))
        self._keep[name] = t

    def stats(self) -> Dict[str, int]:
        a, b = ctypes.c_longlong(), ctypes.c_longlong()
        _check(library().lpx_server_stats(self._srv, ctypes.byref(a), ctypes.byref(b)))
        return {"served": a.value, "failed": b.value}

    def close(self) -> None:
        if self._srv:
            library().lpx_server_destroy(self._srv)
            self._srv = None
            self._keep.clear()


def push(host: str, port: int, token: str, dst_name: str, src: LpxHandle, *, nbytes: Optional[int] = None,
         dst_offset: int = 0, op: int = OP_COPY, timeout_s: float = 30.0) -> None:
    n = int(src.bytes - src.offset) if nbytes is None else int(nbytes)
    _check(library().lpx_push(host.encode(), int(port), token.encode(), dst_name.encode(), ctypes.byref(src),
                              int(dst_offset), n, int(op), float(timeout_s)))


@dataclass
class NativePeerEndpoint:
    host: str
    port: int
    token: str


class NativePeerGradientLane:
    """Hybrid replica -> core replica gradient lane over peer_xfer.

    The core side registers one accumulation buffer per (replica, tensor
    index); a hybrid replica pushes each gradient tensor with OP_ADD, so the
    core's buffer ends up holding the sum of every pushed contribution.  The
    core adds that buffer into its own gradient before the core DP reduction
    (the placement ``InterReplicaGradientDomain`` prescribes) and zeroes it.
    """

    def __init__(self, server: PeerXferServer):
        self.server = server
        self.buffers: Dict[str, torch.Tensor] = {}

    @property
    def endpoint(self) -> NativePeerEndpoint:
        return NativePeerEndpoint(self.server.host, self.server.port, self.server.token)

    @staticmethod
    def buffer_name(replica_id: str, index: int) -> str:
        return f"{replica_id}/{index}"[:63]

    def register_replica(self, replica_id: str, like: Sequence[torch.Tensor]) -> None:
        for i, t in enumerate(like):
            buf = torch.zeros_like(t, memory_format=torch.contiguous_format)
            name = self.buffer_name(replica_id, i)
            self.server.register(name, buf)
            self.buffers[name] = buf

    def drain_into(self, replica_id: str, grads: Sequence[torch.Tensor]) -> None:
        for i, g in enumerate(grads):
            buf = self.buffers[self.buffer_name(replica_id, i)]
            g.add_(buf.to(g.dtype))
            buf.zero_()

    @staticmethod
    def send(endpoint: NativePeerEndpoint, payload: GradientPayload, timeout_s: float = 30.0) -> None:
        if payload.zero_placeholder:
            return
        for i, t in enumerate(payload.tensors):
            if t.is_cuda:
                src = export_tensor(t.contiguous())
                push(endpoint.host, endpoint.port, endpoint.token, NativePeerGradientLane.buffer_name(
                    payload.replica_id, i), src, op=OP_ADD, timeout_s=timeout_s)
            else:
                hb = HostBuffer(t.numel() * t.element_size())
                try:
                    hb.tensor(t.dtype)[: t.numel()].copy_(t.reshape(-1))
                    push(endpoint.host, endpoint.port, endpoint.token, NativePeerGradientLane.buffer_name(
                        payload.replica_id, i), hb.handle, op=OP_ADD, timeout_s=timeout_s)
                finally:
                    hb.close()
