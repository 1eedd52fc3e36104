"""Host control plane between rank 0 and the tensor-parallel workers.

Same shape as the reference (``llmserve/engine/model_runner.py:87-115``: rank 0 pickles
``(method, args)`` into POSIX shared memory and the workers replay the call), with the failure
handling the reference lacks:

* every wait is bounded: a worker that sees no call for ``idle_timeout`` checks that rank 0 is
  still alive and exits if it is gone (no orphaned GPU processes);
* workers acknowledge each call and report exceptions through their status slot, so rank 0 can
  raise a clear error instead of blocking;
* the wait is a spin-then-sleep poll on a sequence counter (tens of microseconds per call);
* a call is published only after every worker acknowledged the previous one (one payload slot).

Layout of the segment: ``[0:8)`` call sequence number, ``[8:16)`` payload length,
``[64 + 16*w, +16)`` worker ``w``'s (acknowledged sequence, status), error text of worker ``w``
at ``2048 + 256*w``, payload from 4096.
"""
import os
import pickle
import struct
import time
from multiprocessing.shared_memory import SharedMemory

HEADER = 4096
STATUS_OK, STATUS_ERROR = 0, 1


class RpcTimeout(RuntimeError):
    pass


class RpcChannel:

    def __init__(self, name: str, num_workers: int, create: bool, size: int = 1 << 22, ack_timeout_s: float = 120.0):
        self.name = name
        self.ack_timeout_s = ack_timeout_s
        self.num_workers = num_workers
        if create:
            try:
                stale = SharedMemory(name=name)
                stale.close()
                stale.unlink()
            except FileNotFoundError:
                pass
            self.shm = SharedMemory(name=name, create=True, size=size)
            self.shm.buf[:HEADER] = bytes(HEADER)
        else:
            self.shm = SharedMemory(name=name)
        self.owner = create
        self.seq = 0

    # ---- rank 0 ------------------------------------------------------------------------------
    def send(self, method: str, *args):
        """Publish one call.  The payload area is single-slot, so the previous call must have been
        taken by every worker first: without this wait a worker that is still busy (or asleep in
        its poll back-off) when two calls are sent in a row would skip the earlier one, and the
        ranks' collective sequences would diverge.  Rank 0 runs its own part of every call it
        sends before sending the next, so the wait cannot deadlock."""
        if self.seq:
            self.wait_acks(self.ack_timeout_s)
        data = pickle.dumps((method, args), protocol=pickle.HIGHEST_PROTOCOL)
        if HEADER + len(data) > self.shm.size:
            raise ValueError(f"RPC payload of {len(data)} bytes exceeds the channel size")
        self.shm.buf[HEADER:HEADER + len(data)] = data
        struct.pack_into("<Q", self.shm.buf, 8, len(data))
        self.seq += 1
        struct.pack_into("<Q", self.shm.buf, 0, self.seq)

    def worker_status(self, w: int) -> tuple[int, int, str]:
        ack, status = struct.unpack_from("<QQ", self.shm.buf, 64 + 16 * w)
        msg = ""
        if status == STATUS_ERROR:
            off = HEADER // 2 + 256 * w
            msg = bytes(self.shm.buf[off:off + 256]).split(b"\0", 1)[0].decode(errors="replace")
        return ack, status, msg

    def check_workers(self):
        for w in range(self.num_workers):
            _, status, msg = self.worker_status(w)
            if status == STATUS_ERROR:
                raise RuntimeError(f"tensor-parallel worker {w + 1} failed: {msg}")

    def wait_acks(self, timeout_s: float):
        # acknowledgements normally follow within tens of microseconds (a worker acks as soon as it
        # has queued its kernels), so spin first and only then back off to sleeps
        start = time.monotonic()
        deadline = start + timeout_s
        while True:
            self.check_workers()
            if min((self.worker_status(w)[0] for w in range(self.num_workers)), default=self.seq) >= self.seq:
                return
            now = time.monotonic()
            if now > deadline:
                raise RpcTimeout(f"workers did not acknowledge call {self.seq} within {timeout_s}s")
            if now - start > 0.005:
                time.sleep(0.0002)

    # ---- workers -----------------------------------------------------------------------------
    def recv(self, worker: int, idle_timeout_s: float, parent_pid: int):
        # busy-poll while calls are likely to follow (a decode step is a few milliseconds), then
        # back off to short sleeps
        spin_until = time.monotonic() + 0.05
        sleep_s = 0.00002
        last_check = time.monotonic()
        while True:
            seq = struct.unpack_from("<Q", self.shm.buf, 0)[0]
            if seq > self.seq:
                n = struct.unpack_from("<Q", self.shm.buf, 8)[0]
                method, args = pickle.loads(bytes(self.shm.buf[HEADER:HEADER + n]))
                self.seq = seq
                return method, args
            now = time.monotonic()
            if now > spin_until:
                time.sleep(sleep_s)
                sleep_s = min(sleep_s * 2, 0.0002)
            if now - last_check > idle_timeout_s:
                last_check = now
                if not _alive(parent_pid):
                    raise RpcTimeout("rank 0 exited; worker shutting down")

    def ack(self, worker: int, ok: bool = True, message: str = ""):
        if not ok:
            off = HEADER // 2 + 256 * worker
            raw = message.encode(errors="replace")[:255] + b"\0"
            self.shm.buf[off:off + len(raw)] = raw
        struct.pack_into("<QQ", self.shm.buf, 64 + 16 * worker, self.seq, STATUS_OK if ok else STATUS_ERROR)

    def close(self):
        try:
            self.shm.close()
            if self.owner:
                self.shm.unlink()
        except FileNotFoundError:
            pass


def _alive(pid: int) -> bool:
    try:
        os.kill(pid, 0)
        return True
    except OSError:
        return False
