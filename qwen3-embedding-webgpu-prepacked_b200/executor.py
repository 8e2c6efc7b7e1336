"""A micro-batch split by request across the GPUs of one box.

The reference serves a micro-batch on one WebGPU device and, for long inputs,
splits a batch of 16 on the host into native batches of 4
(src/main.ts:308-320). Here the requests of one micro-batch are divided
among N devices instead:

* ``ShardPlan`` assigns requests to ranks by LPT on their kept (q, k) pairs
  (``sharding.lpt_shard``) and resolves the AUTO attention mode once, on the
  whole micro-batch's longest request (ops.ts:328). A rank whose own
  requests are all short would otherwise pick the sparse rule where the
  reference, seeing the whole batch, picks full causal.
* ``ShardExecutor`` runs one rank's share, layer by layer: its requests' rows
  are scattered from a host ``qkv`` buffer into a packed device batch
  (one copy per run of adjacent rows), the prologue and attention run on
  that batch, and the output rows are written back to their places in a
  host output buffer. The host output buffer, shared by all ranks, is the
  gather: every request lands at its own rows, in request order, with no
  collective on the data path.
* ``DeviceBackend`` is the device half (libqwa through its C ABI), pipelined
  over layers: the upload of layer l+1 and the download of layer l-1 run on
  their own streams while layer l computes.
* ``MultiDeviceExecutor`` drives N devices from one process with one host
  thread per device, which is how a host binding (the N-API addon) would
  use the library.

``SharedHostBuffer`` is page-locked host memory that several processes can
map (a file under /dev/shm), used when ranks are processes (torchrun).
"""
from __future__ import annotations

import mmap
import os
import threading
from typing import List, Optional, Sequence, Tuple

import numpy as np

from . import sharding

Q_HEADS, KV_HEADS, HEAD_DIM, QKV_WIDTH = 16, 8, 128, 4096
MODE_AUTO, MODE_FULL, MODE_SPARSE = 0, 1, 2


class ShardPlan:
    """Request-to-rank assignment of one micro-batch and the row maps it implies."""

    def __init__(self, lengths: Sequence[int], world: int, mode: int = MODE_AUTO):
        if world < 1:
            raise ValueError("world must be >= 1")
        if mode not in (MODE_AUTO, MODE_FULL, MODE_SPARSE):
            raise ValueError("mode must be AUTO, FULL or SPARSE")
        self.lengths = [int(x) for x in lengths]
        if any(x < 0 for x in self.lengths):
            raise ValueError("request lengths must be >= 0")
        self.world = world
        self.mode = mode
        # AUTO is resolved here, on the whole batch, so every rank applies the
        # rule the single-device call would (ops.ts:328)
        self.resolved_mode = (MODE_SPARSE if sharding.resolve_sparse(mode, self.lengths)
                              else MODE_FULL)
        self.assignment = sharding.lpt_shard(self.lengths, world, self.resolved_mode)
        self.cu = [0] + np.cumsum(self.lengths, dtype=np.int64).astype(int).tolist()

    @property
    def total_tokens(self) -> int:
        return self.cu[-1]

    def requests(self, rank: int) -> List[int]:
        return self.assignment[rank]

    def local_lengths(self, rank: int) -> List[int]:
        return [self.lengths[i] for i in self.assignment[rank]]

    def local_cu(self, rank: int) -> List[int]:
        return [0] + np.cumsum(self.local_lengths(rank), dtype=np.int64).astype(int).tolist()

    def local_tokens(self, rank: int) -> int:
        return self.local_cu(rank)[-1]

    def kept_pairs(self, rank: int) -> int:
        sparse = self.resolved_mode == MODE_SPARSE
        return sum(sharding.kept_pairs(n, sparse) for n in self.local_lengths(rank))

    def row_ranges(self, rank: int) -> List[Tuple[int, int, int]]:
        """(global first row, local first row, rows) of each run of rows that
        are adjacent both in the micro-batch and in this rank's packed batch."""
        out: List[List[int]] = []
        local = 0
        for i in self.assignment[rank]:
            g, n = self.cu[i], self.lengths[i]
            if n == 0:
                continue
            if out and out[-1][0] + out[-1][2] == g and out[-1][1] + out[-1][2] == local:
                out[-1][2] += n
            else:
                out.append([g, local, n])
            local += n
        return [tuple(r) for r in out]


class ShardExecutor:
    """One rank's share of a micro-batch through ``layers`` layers.

    ``backend`` provides ``stage_in(buf, ranges, host_qkv)``,
    ``compute(buf, local_cu, weights, mode, prefix, window)``,
    ``stage_out(buf, ranges, host_out)`` and ``finish()``; ``DeviceBackend``
    is the product's. A backend may overlap the three stages across layers
    (it owns ``buffers`` device buffer sets); the executor only fixes their
    order per layer."""

    def __init__(self, plan: ShardPlan, rank: int, backend, prefix: int = 176,
                 window: int = 432):
        self.plan, self.rank, self.backend = plan, rank, backend
        self.ranges = plan.row_ranges(rank)
        self.local_cu = plan.local_cu(rank)
        self.prefix, self.window = prefix, window

    def run(self, host_inputs: Sequence, host_outputs: Sequence, weights: Sequence):
        """host_inputs[l]: [T, 4096] f16 host rows of the whole micro-batch;
        host_outputs[l]: [T, 16, 128] f16 host rows; weights[l]: the layer's
        (q_weight, k_weight) as the backend expects them. Writes this rank's
        requests' rows of every host_outputs[l]."""
        if not (len(host_inputs) == len(host_outputs) == len(weights)):
            raise ValueError("host_inputs, host_outputs and weights differ in length")
        if not self.ranges:
            return self.backend.finish()
        nbuf = self.backend.buffers
        for layer, (hin, hout, w) in enumerate(zip(host_inputs, host_outputs, weights)):
            b = layer % nbuf
            self.backend.stage_in(b, self.ranges, hin)
            self.backend.compute(b, self.local_cu, w, self.plan.resolved_mode, self.prefix,
                                 self.window)
            self.backend.stage_out(b, self.ranges, hout)
        return self.backend.finish()


class DeviceBackend:
    """libqwa on one CUDA device: packed per-rank buffers, a compute stream
    and copy streams in each direction, ordered by events (PCIe is full
    duplex, so uploads, kernels and downloads of consecutive layers overlap).

    Host buffers must be page-locked (``torch.Tensor.pin_memory`` or a
    registered ``SharedHostBuffer``) for the copies to be asynchronous."""

    def __init__(self, device: int, tokens: int, buffers: int = 2, ctx=None):
        import torch

        from . import attention
        self.torch = torch
        self.attn = attention
        self.device = torch.device("cuda", device)
        self.tokens = tokens
        self.buffers = buffers
        # a context of its own: a qwa_ctx is not thread-safe, and two
        # executors may share a device
        self._own_ctx = ctx is None
        self.ctx = ctx if ctx is not None else attention.Context(self.device.index)
        n = max(tokens, 1)
        with torch.cuda.device(self.device):
            f16 = dict(dtype=torch.float16, device=self.device)
            self.dev_in = [torch.empty(n, QKV_WIDTH, **f16) for _ in range(buffers)]
            self.q = torch.empty(n, Q_HEADS, HEAD_DIM, **f16)
            self.k = torch.empty(n, KV_HEADS, HEAD_DIM, **f16)
            self.dev_out = [torch.empty(n, Q_HEADS, HEAD_DIM, **f16) for _ in range(buffers)]
            self.stream = torch.cuda.Stream(self.device)
            self.h2d = torch.cuda.Stream(self.device)
            self.d2h = torch.cuda.Stream(self.device)
        self._in_free: List[Optional[object]] = [None] * buffers
        self._out_free: List[Optional[object]] = [None] * buffers
        self._last = None

    def _event(self):
        return self.torch.cuda.Event()

    def stage_in(self, b: int, ranges, host_qkv) -> None:
        torch = self.torch
        with torch.cuda.device(self.device), torch.cuda.stream(self.h2d):
            if self._in_free[b] is not None:
                self.h2d.wait_event(self._in_free[b])
            for g, l0, n in ranges:
                self.dev_in[b][l0:l0 + n].copy_(host_qkv[g:g + n], non_blocking=True)
            ready = self._event()
            ready.record(self.h2d)
        self.stream.wait_event(ready)

    def compute(self, b: int, local_cu, weights, mode: int, prefix: int, window: int) -> None:
        torch = self.torch
        qw, kw = weights
        if self._out_free[b] is not None:
            self.stream.wait_event(self._out_free[b])
        with torch.cuda.device(self.device):
            self.attn.prefill_attention_layer(self.dev_in[b], qw, kw, local_cu, mode, prefix,
                                              window, q_buf=self.q, k_buf=self.k,
                                              out=self.dev_out[b], stream=self.stream,
                                              ctx=self.ctx)
            done = self._event()
            done.record(self.stream)
        self._in_free[b] = done

    def stage_out(self, b: int, ranges, host_out) -> None:
        torch = self.torch
        with torch.cuda.device(self.device), torch.cuda.stream(self.d2h):
            self.d2h.wait_event(self._in_free[b])
            for g, l0, n in ranges:
                host_out[g:g + n].copy_(self.dev_out[b][l0:l0 + n], non_blocking=True)
            freed = self._event()
            freed.record(self.d2h)
        self._out_free[b] = freed
        self._last = freed

    def finish(self):
        """Make the compute stream wait for the last download; returns that
        stream (synchronise it, or record an event on it, to know that this
        rank's rows are on the host)."""
        if self._last is not None:
            self.stream.wait_event(self._last)
        return self.stream

    def check(self) -> None:
        """Synchronise and raise if a kernel recorded a device-side timeout."""
        self.ctx.check(self.stream)

    def close(self) -> None:
        if self._own_ctx:
            self.ctx.close()


class MultiDeviceExecutor:
    """One micro-batch over several devices from one process: one host thread
    per device, each running its ``ShardExecutor``; outputs land in one host
    buffer in request order."""

    def __init__(self, lengths: Sequence[int], devices: Sequence[int], mode: int = MODE_AUTO,
                 prefix: int = 176, window: int = 432, buffers: int = 2):
        if not devices:
            raise ValueError("devices must not be empty")
        self.plan = ShardPlan(lengths, len(devices), mode)
        self.devices = list(devices)
        self.backends = [DeviceBackend(d, self.plan.local_tokens(r), buffers)
                         for r, d in enumerate(self.devices)]
        self.shards = [ShardExecutor(self.plan, r, be, prefix, window)
                       for r, be in enumerate(self.backends)]
        self._weights = None

    def set_weights(self, weights: Sequence) -> None:
        """Per-layer (q_weight, k_weight) as host float32 arrays of 128; copied
        to every device once."""
        import torch
        per_dev = []
        for be in self.backends:
            per_dev.append([(torch.as_tensor(np.asarray(qw, np.float32)).to(be.device),
                             torch.as_tensor(np.asarray(kw, np.float32)).to(be.device))
                            for qw, kw in weights])
        self._weights = per_dev

    def run(self, host_inputs: Sequence, host_outputs: Sequence) -> None:
        """Every layer's host qkv in, every layer's host output filled; returns
        once all rows are on the host. Raises the first device error."""
        if self._weights is None:
            raise RuntimeError("set_weights() first")
        errors: List[BaseException] = []

        def work(r: int) -> None:
            try:
                self.shards[r].run(host_inputs, host_outputs, self._weights[r])
                self.backends[r].check()
            except BaseException as e:  # noqa: BLE001 -- re-raised on the caller's thread
                errors.append(e)

        threads = [threading.Thread(target=work, args=(r,)) for r in range(len(self.shards))]
        for t in threads:
            t.start()
        for t in threads:
            t.join()
        if errors:
            raise errors[0]

    def close(self) -> None:
        for be in self.backends:
            be.close()


class SharedHostBuffer:
    """A host array that several processes map from one file (under
    /dev/shm, so it lives in RAM), optionally page-locked for the device
    copies with cudaHostRegister. ``tensor`` is a torch view of it.

    The creating process sizes the file; the others open it after a barrier."""

    def __init__(self, path: str, shape: Sequence[int], dtype=np.float16, create: bool = False,
                 pin: bool = True):
        import torch
        self.path = path
        self.shape = tuple(int(x) for x in shape)
        nbytes = int(np.prod(self.shape)) * np.dtype(dtype).itemsize
        self.nbytes = nbytes
        if create:
            with open(path, "wb") as f:
                f.truncate(max(nbytes, 1))
        self._file = open(path, "r+b")
        self._map = mmap.mmap(self._file.fileno(), max(nbytes, 1))
        self.array = np.frombuffer(self._map, dtype=dtype, count=int(np.prod(self.shape))
                                   ).reshape(self.shape)
        self.tensor = torch.from_numpy(self.array)
        self._registered = False
        if pin and nbytes and torch.cuda.is_available():
            err = torch.cuda.cudart().cudaHostRegister(self.tensor.data_ptr(), nbytes, 0)
            if int(err) != 0:
                raise RuntimeError(f"cudaHostRegister failed ({int(err)}) for {path}")
            self._registered = True

    @staticmethod
    def fits(nbytes: int, directory: str = "/dev/shm") -> bool:
        try:
            st = os.statvfs(directory)
        except OSError:
            return False
        return st.f_bavail * st.f_frsize > nbytes * 1.1

    def close(self, unlink: bool = False) -> None:
        import torch
        if self._registered:
            torch.cuda.cudart().cudaHostUnregister(self.tensor.data_ptr())
            self._registered = False
        self.tensor = None
        self.array = None
        try:
            self._map.close()
        except BufferError:
            pass  # a view is still alive; the mapping goes with the process
        self._file.close()
        if unlink:
            try:
                os.unlink(self.path)
            except FileNotFoundError:
                pass
