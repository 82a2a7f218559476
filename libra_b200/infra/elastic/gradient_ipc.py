"""Cross-process gradient transport for elastic hybrid replicas (TCP).

Role of the reference's ``infra/elastic/gradient_ipc.py:43-310``: a hybrid
replica sends its ``GradientPayload`` to the core trainer's gradient server
and, in lockstep mode, blocks until the server publishes the post-reduce
``GradientUpdate`` for that (replica, step, membership epoch), which comes
back on the same connection.

Wire format (own design; no pickling of network input): every frame is an
8-byte big-endian length followed by the bytes.  The first frame is a JSON
header (payload metadata, one ``{"dtype", "shape"}`` entry per tensor and an
HMAC-SHA256 of the header body under the shared authkey); each tensor follows
as one frame of its raw little-endian bytes.  The receiver answers one byte
(1 = accepted, 0 = rejected), then, if requested, the update in the same
format.  This is the CPU-testable fallback lane; on one box the fast lane is
the peer-memory transport in ``hybrid_pool.PeerMemoryTransport`` and the
native ``peer_xfer`` library.
"""

from __future__ import annotations

import hashlib
import hmac
import json
import socket
import struct
import threading
import time
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch

from libra_b200.infra.elastic.hybrid_pool import GradientPayload

_LEN = struct.Struct("!Q")
_ACK, _NACK = b"\x01", b"\x00"
PROTOCOL_VERSION = 1
MAX_HEADER_BYTES = 1 << 20

_DTYPES: Dict[str, torch.dtype] = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16,
                                   "float64": torch.float64, "int64": torch.int64, "int32": torch.int32,
                                   "uint8": torch.uint8, "int8": torch.int8, "bool": torch.bool}
_NAMES = {v: k for k, v in _DTYPES.items()}


@dataclass(frozen=True)
class GradientEndpoint:
    host: str
    port: int
    authkey: str = ""

    def to_dict(self) -> Dict[str, object]:
        return {"host": self.host, "port": self.port, "authkey": self.authkey}


@dataclass(frozen=True)
class GradientUpdate:
    """Post-reduce gradient returned to one hybrid replica lane."""

    replica_id: str
    tensors: Tuple[torch.Tensor, ...]
    step: int
    state_version: int
    membership_epoch: int


# ------------------------------------------------------------------------------- framing
def _recv_exact(sock: socket.socket, n: int) -> bytes:
    buf = bytearray(n)
    view = memoryview(buf)
    got = 0
    while got < n:
        k = sock.recv_into(view[got:])
        if k == 0:
            raise ConnectionError("connection closed mid-frame")
        got += k
    return bytes(buf)


def _send_frame(sock: socket.socket, data: bytes) -> None:
    sock.sendall(_LEN.pack(len(data)))
    sock.sendall(data)


def _recv_frame(sock: socket.socket, limit: Optional[int] = None) -> bytes:
    (n,) = _LEN.unpack(_recv_exact(sock, _LEN.size))
    if limit is not None and n > limit:
        raise ValueError(f"frame of {n} bytes exceeds limit {limit}")
    return _recv_exact(sock, n)


def _tensor_bytes(t: torch.Tensor) -> Tuple[Dict[str, object], bytes]:
    t = t.detach().to("cpu").contiguous()
    if t.dtype not in _NAMES:
        raise TypeError(f"unsupported tensor dtype {t.dtype}")
    raw = t.view(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
    return {"dtype": _NAMES[t.dtype], "shape": list(t.shape)}, raw


def _tensor_from(desc: Dict[str, object], raw: bytes) -> torch.Tensor:
    dtype = _DTYPES[str(desc["dtype"])]
    shape = [int(s) for s in desc["shape"]]
    numel = 1
    for s in shape:
        numel *= s
    if numel == 0:
        return torch.empty(shape, dtype=dtype)
    elem = torch.empty((), dtype=dtype).element_size()
    if len(raw) != numel * elem:
        raise ValueError(f"tensor frame has {len(raw)} bytes, expected {numel * elem}")
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dtype).reshape(shape).clone()


def _sign(body: bytes, key: str) -> str:
    return hmac.new(key.encode("utf-8"), body, hashlib.sha256).hexdigest()


def _send_message(sock: socket.socket, meta: Dict[str, object], tensors, key: str) -> None:
    descs, blobs = [], []
    for t in tensors:
        d, b = _tensor_bytes(t)
        descs.append(d)
        blobs.append(b)
    body = json.dumps({**meta, "protocol": PROTOCOL_VERSION, "tensors": descs}, sort_keys=True).encode("utf-8")
    _send_frame(sock, json.dumps({"body": body.decode("utf-8"), "mac": _sign(body, key)}).encode("utf-8"))
    for b in blobs:
        _send_frame(sock, b)


def _recv_message(sock: socket.socket, key: str, max_tensor_bytes: int) -> Tuple[Dict[str, object], List[torch.Tensor]]:
    outer = json.loads(_recv_frame(sock, MAX_HEADER_BYTES).decode("utf-8"))
    body = str(outer["body"]).encode("utf-8")
    if not hmac.compare_digest(_sign(body, key), str(outer.get("mac", ""))):
        raise PermissionError("gradient message failed authentication")
    meta = json.loads(body)
    if int(meta.get("protocol", -1)) != PROTOCOL_VERSION:
        raise ValueError(f"unsupported gradient protocol {meta.get('protocol')}")
    tensors = [_tensor_from(d, _recv_frame(sock, max_tensor_bytes)) for d in meta["tensors"]]
    return meta, tensors


# ------------------------------------------------------------------------------- client
class ElasticGradientClient:
    def __init__(self, endpoint: GradientEndpoint, timeout: float = 300.0, max_tensor_bytes: int = 1 << 36):
        self.endpoint, self.timeout, self.max_tensor_bytes = endpoint, timeout, max_tensor_bytes

    def send(self, payload: GradientPayload, *, expect_update: bool = False) -> Optional[GradientUpdate]:
        meta = {"kind": "payload", "replica_id": payload.replica_id, "target_core_id": payload.target_core_id,
                "zero_placeholder": bool(payload.zero_placeholder), "replica_rank": int(payload.replica_rank),
                "replica_world_size": int(payload.replica_world_size), "step": int(payload.step),
                "state_version": int(payload.state_version), "membership_epoch": int(payload.membership_epoch),
                "expect_update": bool(expect_update)}
        with socket.create_connection((self.endpoint.host, self.endpoint.port), timeout=self.timeout) as sock:
            sock.settimeout(self.timeout)
            _send_message(sock, meta, payload.tensors, self.endpoint.authkey)
            if _recv_exact(sock, 1) != _ACK:
                raise ConnectionError("gradient server rejected the payload")
            if not expect_update:
                return None
            umeta, tensors = _recv_message(sock, self.endpoint.authkey, self.max_tensor_bytes)
            return GradientUpdate(str(umeta["replica_id"]), tuple(tensors), int(umeta["step"]),
                                  int(umeta["state_version"]), int(umeta["membership_epoch"]))


# ------------------------------------------------------------------------------- server
class ElasticGradientServer:
    """Background receiver; ``on_payload`` runs on the connection's thread."""

    def __init__(self, *, host: str = "127.0.0.1", port: int = 0, authkey: str = "",
                 on_payload: Callable[[GradientPayload], None], update_timeout: float = 300.0,
                 max_tensor_bytes: int = 1 << 36):
        self.host, self.port, self.authkey = host, int(port), authkey
        self.on_payload = on_payload
        self.update_timeout = float(update_timeout)
        self.max_tensor_bytes = max_tensor_bytes
        self._sock: Optional[socket.socket] = None
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self._received = 0
        self._rejected = 0
        self._handlers: set = set()
        self._hlock = threading.Lock()
        self._cond = threading.Condition()
        self._updates: Dict[Tuple[str, int, int], GradientUpdate] = {}

    @property
    def endpoint(self) -> GradientEndpoint:
        if self._sock is None:
            raise RuntimeError("ElasticGradientServer is not started")
        host, port = self._sock.getsockname()[:2]
        return GradientEndpoint(self.host if self.host not in ("", "0.0.0.0") else host, int(port), self.authkey)

    @property
    def received_count(self) -> int:
        return self._received

    @property
    def rejected_count(self) -> int:
        return self._rejected

    def start(self) -> GradientEndpoint:
        if self._sock is not None:
            return self.endpoint
        s = socket.socket(socket.AF_INET, socket.SOCK_STREAM)
        s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
        s.bind((self.host, self.port))
        s.listen()
        s.settimeout(0.25)
        self._sock = s
        self._thread = threading.Thread(target=self._serve, name="elastic-gradient-server", daemon=True)
        self._thread.start()
        return self.endpoint

    def close(self) -> None:
        self._stop.set()
        with self._cond:
            self._cond.notify_all()
        if self._sock is not None:
            try:
                self._sock.close()
            except OSError:
                pass
        if self._thread is not None:
            self._thread.join(timeout=2.0)
        with self._hlock:
            handlers = list(self._handlers)
        for h in handlers:
            h.join(timeout=2.0)
        self._sock, self._thread = None, None

    def publish_update(self, update: GradientUpdate) -> None:
        with self._cond:
            self._updates[(update.replica_id, int(update.step), int(update.membership_epoch))] = update
            self._cond.notify_all()

    def _serve(self) -> None:
        while not self._stop.is_set():
            try:
                conn, _ = self._sock.accept()
            except socket.timeout:
                continue
            except OSError:
                break
            t = threading.Thread(target=self._handle, args=(conn,), daemon=True)
            with self._hlock:
                self._handlers.add(t)
            t.start()

    def _handle(self, conn: socket.socket) -> None:
        try:
            with conn:
                conn.settimeout(max(self.update_timeout, 1.0))
                try:
                    meta, tensors = _recv_message(conn, self.authkey, self.max_tensor_bytes)
                    payload = GradientPayload(str(meta["replica_id"]), str(meta["target_core_id"]), tuple(tensors),
                                              bool(meta["zero_placeholder"]), int(meta["replica_rank"]),
                                              int(meta["replica_world_size"]), int(meta["step"]),
                                              int(meta["state_version"]), int(meta["membership_epoch"]))
                    self.on_payload(payload)
                    self._received += 1
                    update = self._wait_update(payload) if meta.get("expect_update") else None
                except Exception:
                    self._rejected += 1
                    try:
                        conn.sendall(_NACK)
                    except OSError:
                        pass
                    return
                conn.sendall(_ACK)
                if update is not None:
                    _send_message(conn, {"kind": "update", "replica_id": update.replica_id, "step": update.step,
                                         "state_version": update.state_version,
                                         "membership_epoch": update.membership_epoch}, update.tensors, self.authkey)
        finally:
            with self._hlock:
                self._handlers.discard(threading.current_thread())

    def _wait_update(self, p: GradientPayload) -> GradientUpdate:
        key = (p.replica_id, int(p.step), int(p.membership_epoch))
        deadline = time.monotonic() + max(self.update_timeout, 0.0)
        with self._cond:
            while key not in self._updates and not self._stop.is_set():
                left = deadline - time.monotonic()
                if left <= 0:
                    raise TimeoutError(f"no post-reduce update published for {key}")
                self._cond.wait(timeout=min(left, 0.25))
            if key not in self._updates:
                raise RuntimeError("gradient server closed before the update was published")
            return self._updates.pop(key)
