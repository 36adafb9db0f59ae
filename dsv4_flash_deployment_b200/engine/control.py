"""Control channels of the multi-rank serving front: rank 0 broadcasts one
control message per step and gathers every rank's reply.

* :class:`GlooControl`: ``broadcast_object_list`` / ``gather_object`` on a CPU
  (gloo) process group; works across nodes.
* :class:`ShmControl`: one shared file on tmpfs for the ranks of one node
  (native ``csrc/host/ctl_ring.cpp``): the message and the replies are pickled
  into shared memory and the ranks wait on sequence words with futex, so a
  round trip costs tens of microseconds instead of the gloo group's
  milliseconds.  A rank that died is reported by the next wait within a few
  milliseconds (its process id is checked between 1 ms sleeps); a rank that
  stalls makes the wait fail at ``timeout_s``.

Both raise :class:`ControlError` on a failed round trip; the engine front
turns that into an unhealthy server.
"""

from __future__ import annotations

import ctypes
import os
import pickle
import uuid

import torch.distributed as dist


class ControlError(RuntimeError):
    pass


class GlooControl:
    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)

    def broadcast(self, msg=None):
        box = [msg if self.rank == 0 else None]
        try:
            dist.broadcast_object_list(box, src=0, group=self.group)
        except Exception as e:  # noqa: BLE001  (gloo raises RuntimeError / DistBackendError)
            raise ControlError(f"control broadcast failed: {e}") from e
        return box[0]

    def gather(self, reply) -> list | None:
        out = [None] * self.world if self.rank == 0 else None
        try:
            dist.gather_object(reply, out, dst=0, group=self.group)
        except Exception as e:  # noqa: BLE001
            raise ControlError(f"control gather failed: {e}") from e
        return out

    def close(self) -> None:
        pass


_CODES = {-1: "deadline passed", -2: "message larger than its area", -3: "channel closed by rank 0",
          -4: "peer process is gone", -5: "bad arguments"}


def _lib():
    from ..ops.host import lib

    L = lib()
    if not getattr(L, "_ctl_declared", False):
        vp, i64, u64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_int
        L.dsv4_ctl_open.argtypes = [ctypes.c_char_p, c_int, c_int, u64, u64]
        L.dsv4_ctl_open.restype = vp
        L.dsv4_ctl_close.argtypes = [vp, c_int, ctypes.c_char_p]
        L.dsv4_ctl_close.restype = None
        L.dsv4_ctl_bcast_ptr.argtypes = [vp]
        L.dsv4_ctl_bcast_ptr.restype = vp
        L.dsv4_ctl_reply_ptr.argtypes = [vp, c_int]
        L.dsv4_ctl_reply_ptr.restype = vp
        L.dsv4_ctl_bcast.argtypes = [vp, ctypes.c_char_p, u64]
        L.dsv4_ctl_bcast.restype = c_int
        L.dsv4_ctl_recv.argtypes = [vp, i64]
        L.dsv4_ctl_recv.restype = i64
        L.dsv4_ctl_reply.argtypes = [vp, ctypes.c_char_p, u64]
        L.dsv4_ctl_reply.restype = c_int
        L.dsv4_ctl_gather.argtypes = [vp, i64, ctypes.POINTER(i64), ctypes.POINTER(c_int)]
        L.dsv4_ctl_gather.restype = c_int
        L._ctl_declared = True
    return L


class ShmControl:
    """Broadcast / gather through a shared file (one node).  ``path`` is created by
    rank 0 (any stale file is replaced) and must be on tmpfs; the other ranks open
    it afterwards.  :meth:`create` does the rendezvous over a process group."""

    def __init__(self, path: str, rank: int, world: int, bcast_bytes: int = 256 << 20,
                 reply_bytes: int = 32 << 20, timeout_s: float = 600.0):
        self.path, self.rank, self.world = path, rank, world
        self.timeout_ms = int(timeout_s * 1000)
        self.L = _lib()
        self.h = self.L.dsv4_ctl_open(path.encode(), rank, world, bcast_bytes, reply_bytes)
        if not self.h:
            raise ControlError(f"cannot open the control file {path} (rank {rank} of {world})")
        self._lens = (ctypes.c_int64 * world)()

    @staticmethod
    def remove_stale(directory: str = "/dev/shm") -> list[str]:
        """Removes control files left by a rank 0 that died without closing them
        (named ``dsv4_ctl_<pid>_<tag>``; a file is stale when that process is gone)."""
        import glob

        gone = []
        for path in glob.glob(os.path.join(directory, "dsv4_ctl_*_*")):
            try:
                pid = int(os.path.basename(path).split("_")[2])
            except (IndexError, ValueError):
                continue
            if pid == os.getpid():
                continue
            try:
                os.kill(pid, 0)
                continue                    # its creator is alive
            except ProcessLookupError:
                pass
            except PermissionError:
                continue                    # another user's live process
            try:
                os.remove(path)
                gone.append(path)
            except OSError:
                pass
        return gone

    @classmethod
    def create(cls, group=None, directory: str = "/dev/shm", timeout_s: float = 600.0, **kw) -> "ShmControl":
        """Rank 0 creates the file and broadcasts its path over ``group``; every rank
        opens it; a barrier orders the opens before the first message."""
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        box = [os.path.join(directory, f"dsv4_ctl_{os.getpid()}_{uuid.uuid4().hex[:8]}") if rank == 0 else None]
        ch = None
        if rank == 0:
            cls.remove_stale(directory)
            ch = cls(box[0], 0, world, timeout_s=timeout_s, **kw)
        dist.broadcast_object_list(box, src=0, group=group)
        if rank != 0:
            ch = cls(box[0], rank, world, timeout_s=timeout_s, **kw)
        dist.barrier(group=group)
        return ch

    def _check(self, rc: int, what: str, peer: int | None = None) -> None:
        if rc < 0:
            who = f" (rank {peer})" if peer is not None else ""
            raise ControlError(f"control {what} failed{who}: {_CODES.get(rc, rc)}")

    def broadcast(self, msg=None):
        if self.rank == 0:
            b = pickle.dumps(msg, protocol=pickle.HIGHEST_PROTOCOL)
            self._check(self.L.dsv4_ctl_bcast(self.h, b, len(b)), "broadcast")
            return msg
        n = self.L.dsv4_ctl_recv(self.h, self.timeout_ms)
        self._check(n, "receive", 0)
        return pickle.loads(ctypes.string_at(self.L.dsv4_ctl_bcast_ptr(self.h), n))

    def gather(self, reply) -> list | None:
        if self.rank != 0:
            b = pickle.dumps(reply, protocol=pickle.HIGHEST_PROTOCOL)
            self._check(self.L.dsv4_ctl_reply(self.h, b, len(b)), "reply")
            return None
        bad = ctypes.c_int(-1)
        rc = self.L.dsv4_ctl_gather(self.h, self.timeout_ms, self._lens, ctypes.byref(bad))
        self._check(rc, "gather", bad.value)
        return [reply] + [pickle.loads(ctypes.string_at(self.L.dsv4_ctl_reply_ptr(self.h, r), self._lens[r]))
                          for r in range(1, self.world)]

    def close(self) -> None:
        if self.h:
            self.L.dsv4_ctl_close(self.h, 1 if self.rank == 0 else 0, self.path.encode())
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001  (interpreter shutdown)
            pass


def make_control(kind: str, group=None, timeout_s: float = 600.0):
    """``kind`` "shm" (one node, shared memory) or "gloo" (the process group)."""
    if kind == "shm":
        return ShmControl.create(group, timeout_s=timeout_s)
    if kind == "gloo":
        return GlooControl(group)
    raise ValueError(f"unknown control channel {kind!r}")
