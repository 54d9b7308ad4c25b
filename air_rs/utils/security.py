"""Memory-safety helpers for multi-tenant serving (reference ``src/strix/security.rs``:
OwnerToken, BoundsCheckedPtr, ShardedRwLock, SecurityAuditLog ring buffer, SecureAllocator
that zeroes memory before freeing it).

* ``BoundsCheckedRegion`` guards views into a shared device buffer (e.g. a KV pool) by
  owner and range; violations are recorded in the audit log and raise.
* ``SecureAllocator`` hands out device tensors per owner and zero-fills them on release.
* ``SecurityAuditLog`` keeps the last N events; each entry carries an HMAC-SHA256 chained
  over the previous one (keyed per process), so a log excerpt can be checked for tampering.
* ``Engine(secure_kv=True)`` zeroes the KV blocks a finished request returns to the pool.
"""
from __future__ import annotations

import hashlib
import hmac
import itertools
import json
import os
import threading
import time
from dataclasses import dataclass, field

import torch


@dataclass(frozen=True)
class OwnerToken:
    session_id: int


class BoundsError(RuntimeError):
    pass


@dataclass
class AuditEvent:
    kind: str
    detail: dict
    t: float = field(default_factory=time.time)
    mac: str = ""


class SecurityAuditLog:
    def __init__(self, capacity: int = 1024, key: bytes | None = None):
        self.capacity = max(16, capacity)
        self.events: list[AuditEvent] = []
        self.write_pos = 0
        self.total_logged = 0
        self._key = key or os.urandom(32)
        self._prev = b"\0" * 32
        self._lock = threading.Lock()

    def _mac(self, prev: bytes, ev: AuditEvent) -> bytes:
        body = json.dumps([ev.kind, ev.detail, ev.t], sort_keys=True, default=str).encode()
        return hmac.new(self._key, prev + body, hashlib.sha256).digest()

    def log(self, kind: str, **detail) -> AuditEvent:
        ev = AuditEvent(kind, detail)
        with self._lock:
            mac = self._mac(self._prev, ev)
            ev.mac = mac.hex()
            self._prev = mac
            if len(self.events) < self.capacity:
                self.events.append(ev)
            else:
                self.events[self.write_pos] = ev
            self.write_pos = (self.write_pos + 1) % self.capacity
            self.total_logged += 1
        return ev

    def __len__(self):
        return len(self.events)

    def ordered(self) -> list[AuditEvent]:
        """Events oldest first (the ring may have wrapped)."""
        if len(self.events) < self.capacity:
            return list(self.events)
        return self.events[self.write_pos:] + self.events[: self.write_pos]

    def verify(self, events: list[AuditEvent] | None = None) -> bool:
        """Check the HMAC chain across consecutive events (oldest first)."""
        evs = events if events is not None else self.ordered()
        for a, b in zip(evs, evs[1:]):
            if not hmac.compare_digest(self._mac(bytes.fromhex(a.mac), b).hex(), b.mac):
                return False
        return True


class BoundsCheckedRegion:
    """A [offset, offset + size) window of a flat buffer owned by one session."""

    def __init__(self, buf: torch.Tensor, offset: int, size: int, owner: OwnerToken, log: SecurityAuditLog | None = None):
        if offset < 0 or offset + size > buf.numel():
            raise BoundsError(f"region {offset}..{offset + size} outside a buffer of {buf.numel()}")
        self.buf, self.offset, self.size, self.owner, self.log = buf, offset, size, owner, log

    def view(self, start: int, length: int, owner: OwnerToken) -> torch.Tensor:
        if owner != self.owner:
            if self.log is not None:
                self.log.log("owner_violation", expected=self.owner.session_id, actual=owner.session_id)
            raise BoundsError(f"session {owner.session_id} does not own this region")
        if start < 0 or length < 0 or start + length > self.size:
            if self.log is not None:
                self.log.log("bounds_violation", offset=start, len=length, size=self.size)
            raise BoundsError(f"access {start}..{start + length} outside a region of {self.size}")
        return self.buf.view(-1)[self.offset + start: self.offset + start + length]


class SecureAllocator:
    """Device allocations tagged with their owner; released memory is zero-filled first."""

    def __init__(self, device="cpu", log: SecurityAuditLog | None = None):
        self.device = torch.device(device)
        self.log = log or SecurityAuditLog()
        self._live: dict[int, tuple[torch.Tensor, OwnerToken]] = {}
        self._ids = itertools.count(1)

    def allocate(self, shape, dtype, owner: OwnerToken) -> tuple[int, torch.Tensor]:
        t = torch.zeros(shape, dtype=dtype, device=self.device)
        h = next(self._ids)
        self._live[h] = (t, owner)
        self.log.log("allocated", handle=h, bytes=t.numel() * t.element_size(), owner=owner.session_id)
        return h, t

    def secure_free(self, handle: int, owner: OwnerToken):
        t, own = self._live.get(handle, (None, None))
        if t is None:
            raise KeyError(f"unknown allocation {handle}")
        if own != owner:
            self.log.log("owner_violation", handle=handle, expected=own.session_id, actual=owner.session_id)
            raise BoundsError("free by a session that does not own the allocation")
        t.zero_()
        del self._live[handle]
        self.log.log("zeroed_and_freed", handle=handle, bytes=t.numel() * t.element_size(), owner=owner.session_id)

    def active_allocations(self) -> int:
        return len(self._live)


class ShardedRwLock:
    """Readers lock one of N shards (chosen by key); a writer takes them all."""

    def __init__(self, n: int = 8):
        self._locks = [threading.Lock() for _ in range(max(1, n))]

    def read(self, key: int, fn):
        with self._locks[hash(key) % len(self._locks)]:
            return fn()

    def write(self, fn):
        for lk in self._locks:
            lk.acquire()
        try:
            return fn()
        finally:
            for lk in reversed(self._locks):
                lk.release()

    def shard_count(self) -> int:
        return len(self._locks)


def zero_kv_blocks(kv: torch.Tensor, blocks: list[int]):
    """Zero-fill whole KV blocks of a pool [L, num_blocks, ...] (one launch)."""
    if blocks:
        kv.index_fill_(1, torch.tensor(blocks, dtype=torch.long, device=kv.device), 0)
