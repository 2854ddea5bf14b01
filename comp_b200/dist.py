"""Row-sharded decode GEMV over the GPUs of one node (one process per GPU, torch.distributed).

The reference has no multi-GPU path. Output rows are independent (src/komp/kernels.py:55-56, 94), so a layer's rows
are partitioned across ranks: rank r holds rows [row0_r, row0_r + rows_r) of WQ/WS, resident in its HBM. Every rank
holds the same f32 activations (the decode hidden state is replicated) and quantizes them locally -- quantization is
deterministic, so every rank gets the same q8 bytes and no activation broadcast is needed. After the local GEMV the
output slices are all-gathered so every rank holds the full Y [M][N], ready to be the next layer's input. A row's
result does not depend on which rank computes it: the sharded Y is bit-identical to the single-GPU Y.

Exchange paths:
  "p2p"   fused into the GEMV kernel (b2q_gemv_allgather): every output value is sent to each peer as one 64-bit
          (flag, value) word store into its receive buffer (CUDA IPC mappings over NVLink), and each CTA collects its
          slice of the peers' rows with bounded polls -- no fences, no grid-wide barrier. One launch per layer,
          graph-capturable. The returned Y is this layer's output buffer: call t's result stays valid until the
          layer's next call. Given a pinned host `out`, the kernel stores Y there instead (b2q_host_device_pointer).
Host buffers: x may be a pinned CPU tensor (copied to the GPU by a kernel, b2q_stage_pinned) and `out` a pinned CPU
tensor, so a decode loop that keeps its activations on the host needs no memcpy around the layer.
  "nccl"  host.quant_gemv, then torch.distributed.all_gather_into_tensor of equal-size padded slices.
"""

import ctypes

import torch
import torch.distributed as dist

from . import _lib, host

SPIN_LIMIT = 1 << 26  # polls of one receive entry (~1-3 s) before the kernel reports a timeout


def partition(n, nranks, align=4):
    """[(row0, rows)] per rank: equal slices of ceil(n / nranks) rows rounded up to `align`, the last ones shorter
    (possibly empty). Non-empty slices start at rank * slice_rows(n, nranks)."""
    if nranks < 1:
        raise ValueError("nranks must be >= 1")
    per = slice_rows(n, nranks, align)
    out = []
    for r in range(nranks):
        a = min(n, r * per)
        b = min(n, a + per)
        out.append((a, b - a))
    return out


def slice_rows(n, nranks, align=4):
    """Rows per (padded) slice: every rank's slice of the gathered output has this many rows."""
    per = -(-n // nranks)
    return -(-per // align) * align


def assemble(gathered, world, m, per, n):
    """[world*m][per] slices as all-gathered (rank-major) -> Y [m][n]."""
    return gathered.view(world, m, per).permute(1, 0, 2).reshape(m, world * per)[:, :n]


class _PeerMapped:
    """A device buffer of this rank plus the peer-mapped pointers of the same buffer on every rank (CUDA IPC)."""

    def __init__(self, t, group):
        lib = _lib.load()
        self.t = t
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_uint64(0)
        _lib.call("b2q_ipc_get_handle", t.data_ptr(), handle, ctypes.byref(off))
        mine = (bytes(handle.raw), int(off.value))
        world = dist.get_world_size(group)
        rank = dist.get_rank(group)
        allh = [None] * world
        dist.all_gather_object(allh, mine, group=group)
        self.ptrs, self.opened = [], []
        for q, (h, o) in enumerate(allh):
            if q == rank:
                self.ptrs.append(t.data_ptr())
                continue
            base = ctypes.c_void_p()
            rc = lib.b2q_ipc_open_handle(ctypes.create_string_buffer(h, 64), ctypes.byref(base))
            if rc != 0:
                raise _lib.B2QError(rc, _lib.last_error())
            self.opened.append(base.value)
            self.ptrs.append(base.value + o)

    def close(self):
        for b in self.opened:
            _lib.load().b2q_ipc_close_handle(b)
        self.opened = []


class RowShardedGemv:
    """One quantized layer, row-sharded over `group` (default: the world group).

    wq/ws: this rank's rows of the split planes (CUDA tensors; rows given by partition(n, world)[rank]), n/k: the
    full layer's shape. __call__(x f32 [M][K], M <= 4 for "p2p") -> Y f32 [M][N], the full output, on every rank.
    Every rank must make the same calls in the same order.
    """

    def __init__(self, fmt, wq, ws, n, k, group=None, exchange="p2p", max_m=4):
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange {exchange!r}: expected 'p2p' or 'nccl'")
        self.fmt, self.n, self.k, self.group, self.max_m = fmt, n, k, group, max_m
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.row0, self.rows = partition(n, self.world)[self.rank]
        if wq.shape[0] != self.rows or ws.shape[0] != self.rows:
            raise ValueError(f"rank {self.rank}: expected {self.rows} rows (from row {self.row0}), got "
                             f"{wq.shape[0]}/{ws.shape[0]}")
        self.wq, self.ws = wq, ws
        self.per = slice_rows(n, self.world)
        self.dev = wq.device
        # the fused exchange needs every rank to own rows (it runs the barrier); tiny layers use NCCL
        if exchange == "p2p" and (self.world == 1 or any(r == 0 for _, r in partition(n, self.world))):
            exchange = "nccl"
        self.exchange = exchange
        self._calls = 0
        if exchange == "p2p":
            self._init_p2p()

    # ---- fused P2P exchange ----
    def _init_p2p(self):
        dev = self.dev
        with torch.cuda.device(dev):
            self.y = torch.zeros((self.max_m, self.n), dtype=torch.float32, device=dev)
            self.rx_stride = self.max_m * self.n
            # 64-bit entries: low 32 bits the value's bits, high 32 bits the flag
            self.rx = torch.zeros((2, self.rx_stride), dtype=torch.int64, device=dev)
            self.done = torch.zeros(1, dtype=torch.int64, device=dev)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
            torch.cuda.synchronize(dev)
            self._rxmap = _PeerMapped(self.rx, self.group)
            self._rxpeers = torch.tensor(self._rxmap.ptrs, dtype=torch.int64, device=dev)
        dist.barrier(group=self.group)

    def _p2p(self, x, out=None):
        m = x.shape[0]
        if m > self.max_m:
            raise ValueError(f"p2p exchange: M={m} > max_m={self.max_m}")
        self._calls += 1
        with host._on(self.dev):
            if out is None:
                yp = self.y.data_ptr()
            else:  # the kernel stores the whole Y (its rows and the peers') straight into the pinned buffer
                dp = ctypes.c_void_p()
                _lib.call("b2q_host_device_pointer", out.data_ptr(), ctypes.byref(dp))
                yp = dp.value
            _lib.call("b2q_gemv_allgather", host.FMT_ID[self.fmt], self.wq.data_ptr(), self.wq.stride(0),
                      self.ws.data_ptr(), x.data_ptr(), x.stride(0), yp, self.rx.data_ptr(),
                      self._rxpeers.data_ptr(), self.rx_stride, self.done.data_ptr(), self.status.data_ptr(),
                      self.row0, self.rows, self.n, self.k, m, self.rank, self.world, SPIN_LIMIT,
                      torch.cuda.current_stream(self.dev).cuda_stream)
        return self.y[:m] if out is None else out

    def _stage(self, x):
        """Pinned host x [M][K] -> this layer's device staging buffer, copied by a kernel through x's device mapping
        (b2q_stage_pinned: the following GEMV starts its weight stream while x arrives)."""
        if not x.is_pinned() or x.stride(1) != 1:
            raise ValueError("x on the host must be a pinned CPU tensor (tensor.pin_memory()) with unit column stride")
        m = x.shape[0]
        if getattr(self, "_xs", None) is None or self._xs.shape[0] < m:
            self._xs = torch.empty((max(m, self.max_m), self.k), dtype=torch.float32, device=self.dev)
        with host._on(self.dev):
            _lib.call("b2q_stage_pinned", x.data_ptr(), x.stride(0), self._xs.data_ptr(), m, self.k,
                      torch.cuda.current_stream(self.dev).cuda_stream)
        return self._xs[:m]

    def status_code(self):
        """0, or 1 if a receive poll timed out (synchronizes)."""
        return int(self.status.item()) if self.exchange == "p2p" else 0

    def reset(self):
        """Restores the fused exchange after a timed-out call (status_code() == 1), when a late value may still sit
        in a receive buffer: every rank waits for its own work, the ranks meet, each zeroes its receive buffer, call
        counter and status, and the ranks meet again before anyone calls the layer. Collective: every rank calls it."""
        if self.exchange != "p2p":
            return
        torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.dev):
            self.rx.zero_()
            self.done.zero_()
            self.status.zero_()
            torch.cuda.synchronize(self.dev)
        dist.barrier(group=self.group)

    # ---- NCCL exchange ----
    def local(self, x):
        """This rank's output slice [M][rows] (no exchange), on the same single-launch schedule as the fused exchange
        (split=False), so that both exchanges give the unsharded split=False Y bit for bit."""
        return host.quant_gemv(self.fmt, self.wq, self.ws, x, self.rows, self.k, split=False)

    def _nccl(self, x):
        m = x.shape[0]
        part = torch.zeros((m, self.per), dtype=torch.float32, device=x.device)
        if self.rows:
            part[:, : self.rows] = self.local(x)
        gathered = torch.empty((self.world * m, self.per), dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(gathered, part, group=self.group)
        return assemble(gathered, self.world, m, self.per, self.n)

    def __call__(self, x, out=None):
        """Y [M][N] on every rank. x: f32 [M][K] on this rank's GPU, or a pinned CPU tensor (then a kernel copies it to
        the GPU). out: optional pinned CPU f32 [M][N] that receives Y (the fused exchange stores into it directly; the
        NCCL exchange copies into it); it is complete once the current stream is synchronized. Returns out if given."""
        if x.dtype != torch.float32 or x.dim() != 2 or x.shape[1] != self.k:
            raise ValueError(f"x must be float32 [M][{self.k}], got {x.dtype} {tuple(x.shape)}")
        m = x.shape[0]
        if out is not None and (out.device.type != "cpu" or not out.is_pinned() or out.dtype != torch.float32 or
                                tuple(out.shape) != (m, self.n) or not out.is_contiguous()):
            raise ValueError(f"out must be a contiguous pinned CPU float32 [{m}][{self.n}] tensor")
        x = self._stage(x) if x.device.type == "cpu" else host._rows_aligned(x)
        if self.exchange == "p2p":
            return self._p2p(x, out)
        y = self._nccl(x)
        if out is None:
            return y
        out.copy_(y, non_blocking=True)
        return out

    def close(self):
        """Unmaps the peers' buffers (collective: every rank calls it, after its last use of the layer)."""
        if self.exchange == "p2p" and getattr(self, "_rxmap", None) is not None:
            torch.cuda.synchronize(self.dev)
            dist.barrier(group=self.group)
            self._rxmap.close()
            self._rxmap = None
