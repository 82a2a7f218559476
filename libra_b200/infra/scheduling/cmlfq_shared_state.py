"""Box-wide C-MLFQ load counters in one shared memory-mapped table.

When several trainer ranks route requests to the same rollout instances, the
least-connections choice must see every rank's in-flight requests, not only
its own (the reference keeps one JSON snapshot per rank on a shared
filesystem and sums them, ``infra/scheduling/cmlfq_shared_state.py``).  On a
single box the processes can share memory directly, so this module keeps one
fixed-size table in a file that every process maps:

* the file ``<dir>/cmlfq_load.bin`` holds a header and ``SLOTS`` rows; a row is
  ``[pid, heartbeat (seconds), count per instance column]``;
* each process claims one row for its lifetime (an ``O_EXCL`` claim file per
  row) and is the only writer of that row, so updates need no lock: an
  increment is one aligned 32-bit store into shared memory;
* instance ids map to columns through ``<dir>/cmlfq_load.columns.json``, which
  grows under an ``fcntl`` lock when a process meets a new id;
* a reader sums the rows whose owner is alive: the pid still exists on this
  host and the heartbeat (refreshed by a daemon thread) is younger than the
  TTL, so the counts of a crashed process stop counting at once, or after the
  TTL when the pid has been reused.

Reading costs one pass over a few KB of mapped memory; nothing is parsed or
rewritten per request.  The table is local to one machine (a memory map over a
network filesystem is not coherent between hosts).
"""

from __future__ import annotations

import atexit
import errno
import fcntl
import json
import mmap
import os
import struct
import threading
import time
from pathlib import Path
from typing import Dict, List

MAGIC = 0x4C4D4C51  # "QLML"
SLOTS = 64           # writer processes per table
COLUMNS = 256        # distinct rollout instances
_HEADER = struct.Struct("<IIII")            # magic, version, slots, columns
_ROW_HEAD = struct.Struct("<qd")            # pid, heartbeat
_ROW_BYTES = _ROW_HEAD.size + 4 * COLUMNS
_FILE_BYTES = _HEADER.size + SLOTS * _ROW_BYTES


def _pid_alive(pid: int) -> bool:
    if pid <= 0:
        return False
    try:
        os.kill(pid, 0)
    except OSError as exc:
        return exc.errno == errno.EPERM
    return True


class SharedCMLFQLoadState:
    """One process's view of the box-wide table; ``increment`` / ``decrement``
    touch only this process's row, ``aggregate`` sums the live rows."""

    def __init__(self, directory: str, ttl_s: float = 60.0, heartbeat_interval_s: float = 10.0, writer_id: str = ""):
        self.directory = Path(directory)
        self.directory.mkdir(parents=True, exist_ok=True)
        self.writer_id = writer_id or f"rank_{os.environ.get('RANK', '0')}"
        self.heartbeat_interval_s = max(0.05, float(heartbeat_interval_s))
        self.ttl_s = max(2.0 * self.heartbeat_interval_s, float(ttl_s))
        self._table = self.directory / "cmlfq_load.bin"
        self._columns_path = self.directory / "cmlfq_load.columns.json"
        self._mm = self._map_table()
        self._columns: Dict[str, int] = {}
        self._slot, self._claim = self._claim_slot()
        self._base = _HEADER.size + self._slot * _ROW_BYTES
        self._pid = os.getpid()
        self._mm[self._base:self._base + _ROW_BYTES] = bytes(_ROW_BYTES)
        self._stamp()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._beat, daemon=True, name=f"cmlfq-load-{self.writer_id}")
        self._thread.start()
        atexit.register(self.close)

    # ------------------------------------------------------------------ table and rows
    def _map_table(self) -> mmap.mmap:
        fd = os.open(self._table, os.O_RDWR | os.O_CREAT, 0o644)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX)
            try:
                if os.fstat(fd).st_size < _FILE_BYTES:
                    os.ftruncate(fd, _FILE_BYTES)
                    os.pwrite(fd, _HEADER.pack(MAGIC, 1, SLOTS, COLUMNS), 0)
            finally:
                fcntl.flock(fd, fcntl.LOCK_UN)
            mm = mmap.mmap(fd, _FILE_BYTES)
        finally:
            os.close(fd)
        magic, _, slots, cols = _HEADER.unpack_from(mm, 0)
        if magic != MAGIC or slots != SLOTS or cols != COLUMNS:
            raise RuntimeError(f"{self._table} is not a C-MLFQ load table of this layout")
        return mm

    def _claim_slot(self):
        for slot in range(SLOTS):
            claim = self.directory / f"cmlfq_load.slot{slot}"
            try:
                fd = os.open(claim, os.O_CREAT | os.O_EXCL | os.O_WRONLY, 0o644)
            except FileExistsError:
                try:
                    owner = int(claim.read_text().split()[0])
                except (OSError, ValueError, IndexError):
                    owner = -1
                if owner > 0 and _pid_alive(owner):
                    continue
                try:  # the previous owner died: take the row over
                    claim.unlink()
                    fd = os.open(claim, os.O_CREAT | os.O_EXCL | os.O_WRONLY, 0o644)
                except OSError:
                    continue
            with os.fdopen(fd, "w") as fh:
                fh.write(f"{os.getpid()} {self.writer_id}\n")
            return slot, claim
        raise RuntimeError(f"all {SLOTS} rows of {self._table} are held by live processes")

    def _stamp(self) -> None:
        _ROW_HEAD.pack_into(self._mm, self._base, self._pid, time.time())

    def _beat(self) -> None:
        while not self._stop.wait(self.heartbeat_interval_s):
            self._stamp()

    def _column(self, instance_id: str) -> int:
        col = self._columns.get(instance_id)
        if col is not None:
            return col
        fd = os.open(self._columns_path, os.O_RDWR | os.O_CREAT, 0o644)
        try:
            fcntl.flock(fd, fcntl.LOCK_EX)
            raw = os.read(fd, 1 << 20)
            names: List[str] = json.loads(raw) if raw.strip() else []
            if instance_id not in names:
                if len(names) >= COLUMNS:
                    raise RuntimeError(f"more than {COLUMNS} rollout instances in one C-MLFQ load table")
                names.append(instance_id)
                data = json.dumps(names).encode()
                os.ftruncate(fd, 0)
                os.pwrite(fd, data, 0)
        finally:
            fcntl.flock(fd, fcntl.LOCK_UN)
            os.close(fd)
        self._columns = {n: i for i, n in enumerate(names)}
        return self._columns[instance_id]

    def _cell(self, col: int) -> int:
        return self._base + _ROW_HEAD.size + 4 * col

    # ------------------------------------------------------------------ API
    def increment(self, instance_id: str) -> None:
        off = self._cell(self._column(instance_id))
        (n,) = struct.unpack_from("<i", self._mm, off)
        struct.pack_into("<i", self._mm, off, n + 1)

    def decrement(self, instance_id: str) -> None:
        off = self._cell(self._column(instance_id))
        (n,) = struct.unpack_from("<i", self._mm, off)
        struct.pack_into("<i", self._mm, off, max(0, n - 1))

    def aggregate(self) -> Dict[str, int]:
        try:
            names = json.loads(self._columns_path.read_text(encoding="utf-8") or "[]")
        except (OSError, ValueError):
            names = list(self._columns)
        now = time.time()
        totals = [0] * len(names)
        for slot in range(SLOTS):
            base = _HEADER.size + slot * _ROW_BYTES
            pid, beat = _ROW_HEAD.unpack_from(self._mm, base)
            if pid <= 0 or now - beat > self.ttl_s or not _pid_alive(pid):
                continue
            counts = struct.unpack_from(f"<{len(names)}i", self._mm, base + _ROW_HEAD.size)
            for i, n in enumerate(counts):
                totals[i] += max(0, n)
        return {name: n for name, n in zip(names, totals) if n > 0}

    def close(self) -> None:
        if getattr(self, "_stop", None) is None or self._stop.is_set():
            return
        self._stop.set()
        try:
            self._mm[self._base:self._base + _ROW_BYTES] = bytes(_ROW_BYTES)
            self._mm.flush()
        except ValueError:  # already unmapped
            pass
        try:
            self._claim.unlink()
        except OSError:
            pass
