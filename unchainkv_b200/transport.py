"""GPU-to-GPU transport of splitzip streams over NVLink / NVSwitch.

The reference ships each compressed layer as a framed TCP message (a header
with the layer, block count, raw and encoded sizes and codec, then the
stream; src/unchain_kv/tcp_data.py:615-652, native/unchain_kv/kvq_tcp.cc:224-270),
after a device-to-host copy on the sender and before a host-to-device copy
on the receiver (vllm_connector.py:3406, 5134).

Here the sender's stream buffers are opened in the receiving process over
CUDA IPC, and the receiver's decode reads the streams straight from the
sender's HBM over NVLink and scatters them into its own paged cache: the
transfer is the decode's own loads, with no receive buffer and no copy.
The frame's metadata needs no wire: the mode byte and sizes are in the
stream, and each side knows its jobs.

Order is kept on the CUDA streams by small NCCL messages, never by the
hosts.  Step k uses buffer slot k % slots.  Each step every rank issues one
group of point-to-point operations:

  sender:    send ready(k)     and receive free(k - 1)
  receiver:  receive ready(k)  and send free(k - 1)

so the receiver's decode of step k follows the sender's encode of step k,
and the sender's encode into a slot follows the receiver's decode of the
slot's previous step (it waits for that step's free token, received one
step earlier).  Grouping the two directions keeps the NCCL streams of the
pair from waiting on each other in a cycle.  ``finish`` drains the last free
token.

``TokenSchedule`` is the ordering alone (any backend, so the CPU tests run
it over gloo); ``StreamTransport`` adds the buffers.
"""

from __future__ import annotations

import ctypes


class TokenSchedule:
    """The ready / free token exchange of one sender -> receiver pair."""

    def __init__(self, sender: int, receiver: int, rank: int, device=None, group=None):
        import torch

        if sender == receiver:
            raise ValueError("sender and receiver must differ")
        self.sender, self.receiver, self.group = sender, receiver, group
        self.role = "sender" if rank == sender else "receiver" if rank == receiver else None
        kw = {"dtype": torch.int64, "device": device}
        self._ready = torch.zeros(1, **kw)
        self._free = torch.zeros(1, **kw)
        self._step = -1  # last step exchanged
        self._freed = -1  # last step whose free token the sender has received
        self.last_ready = -1  # receiver: value of the last ready token (the sender's step)

    def _exchange(self, ops):
        import torch.distributed as dist

        if ops:
            for work in dist.batch_isend_irecv(ops):
                work.wait()

    def step(self, k: int) -> None:
        """Sender: after enqueuing step k's encode.  Receiver: before
        enqueuing step k's decode (and after step k - 1's)."""
        import torch.distributed as dist

        if k != self._step + 1:
            raise ValueError(f"steps must be consecutive: expected {self._step + 1}, got {k}")
        ops = []
        if self.role == "sender":
            self._ready.fill_(k)
            ops.append(dist.P2POp(dist.isend, self._ready, self.receiver, self.group))
            if k > 0:
                ops.append(dist.P2POp(dist.irecv, self._free, self.receiver, self.group))
        elif self.role == "receiver":
            ops.append(dist.P2POp(dist.irecv, self._ready, self.sender, self.group))
            if k > 0:
                self._free.fill_(k - 1)
                ops.append(dist.P2POp(dist.isend, self._free, self.sender, self.group))
        self._exchange(ops)
        if self.role == "sender" and k > 0:
            self._freed = k - 1
        self._step = k

    def received_step(self) -> int:
        """Receiver: the step number the last ready token carried (host read,
        synchronises; for checks)."""
        return int(self._ready.item())

    def freed_step(self) -> int:
        """Sender: the step number the last free token carried (host read)."""
        return int(self._free.item())

    def finish(self) -> None:
        """Drain the last free token (both roles)."""
        import torch.distributed as dist

        if self._step < 0 or self.role is None:
            return
        ops = []
        if self.role == "sender":
            ops.append(dist.P2POp(dist.irecv, self._free, self.receiver, self.group))
        else:
            self._free.fill_(self._step)
            ops.append(dist.P2POp(dist.isend, self._free, self.sender, self.group))
        self._exchange(ops)
        if self.role == "sender":
            self._freed = self._step


class StreamTransport:
    """``slots`` stream buffers of ``capacity`` bytes on the sender's GPU,
    opened on the receiver's; call on every rank of ``group`` (ranks other
    than the pair take no part in the tokens)."""

    def __init__(self, capacity: int, sender: int, receiver: int, slots: int = 2, group=None):
        import torch
        import torch.distributed as dist

        from . import splitzip_cuda as S

        self.lib = S._require_lib()
        self.capacity, self.slots = int(capacity), int(slots)
        rank = dist.get_rank()
        device = torch.device("cuda", torch.cuda.current_device())
        self.tokens = TokenSchedule(sender, receiver, rank, device, group)
        self.role = self.tokens.role
        self._own, self._peer = [], []
        handles = None
        if self.role == "sender":
            for _ in range(self.slots):
                ptr = self.lib.kvq_splitzip_ipc_alloc(self.capacity)
                if not ptr:
                    raise RuntimeError("stream buffer: " + self.lib.kvq_splitzip_last_error().decode())
                self._own.append(int(ptr))
            handles = []
            for ptr in self._own:
                h = (ctypes.c_ubyte * 64)()
                if self.lib.kvq_splitzip_ipc_get_handle(ptr, h) != 64:
                    raise RuntimeError("IPC handle: " + self.lib.kvq_splitzip_last_error().decode())
                handles.append(bytes(h))
        box = [handles]
        dist.broadcast_object_list(box, src=sender, group=group)
        if self.role == "receiver":
            for raw in box[0]:
                h = (ctypes.c_ubyte * 64).from_buffer_copy(raw)
                ptr = self.lib.kvq_splitzip_ipc_open(h)
                if not ptr:
                    raise RuntimeError("IPC open: " + self.lib.kvq_splitzip_last_error().decode())
                self._peer.append(int(ptr))

    def buffer(self, k: int) -> int:
        """Address (in this process) of step k's slot: the sender's own
        buffer, or the same memory opened on the receiver."""
        slots = self._own if self.role == "sender" else self._peer
        return slots[k % self.slots]

    def step(self, k: int) -> None:
        self.tokens.step(k)

    def finish(self) -> None:
        self.tokens.finish()

    def close(self) -> None:
        """Release the buffers (after ``finish`` on both sides)."""
        import torch

        torch.cuda.synchronize()
        for ptr in self._peer:
            self.lib.kvq_splitzip_ipc_close(ptr)
        self._peer = []
        for ptr in self._own:
            self.lib.kvq_splitzip_ipc_free(ptr)
        self._own = []


def peer_job(kv_layer, block_ids, stream_ptr: int, stream_bytes: int, tables=None, block_start: int = 0,
             block_count: int | None = None):
    """A decode job whose stream is at a raw device address (e.g. a peer's
    buffer opened by ``StreamTransport``)."""
    from . import splitzip_cuda as S

    class _At:
        def __init__(self, ptr, size):
            self._ptr, self._size = ptr, size

        def data_ptr(self):
            return self._ptr

        def numel(self):
            return self._size

    return S.make_job(kv_layer, block_ids, _At(stream_ptr, stream_bytes), stream_bytes, tables, block_start,
                      block_count)
