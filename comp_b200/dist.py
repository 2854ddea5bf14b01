"""Row-sharded decode GEMV over the GPUs of one node (one process per GPU, torch.distributed).

The reference has no multi-GPU path. Output rows are independent (src/komp/kernels.py:55-56, 94), so a layer's rows
are partitioned across ranks: rank r holds rows [row0_r, row0_r + rows_r) of WQ/WS, resident in its HBM. Every rank
holds the same f32 activations (the decode hidden state is replicated) and quantizes them locally -- quantization is
deterministic, so every rank gets the same q8 bytes and no activation broadcast is needed. After the local GEMV the
output slices are all-gathered so every rank holds the full Y [M][N], ready to be the next layer's input.

Exchange paths:
  "nccl"  torch.distributed.all_gather_into_tensor of equal-size padded slices (NCCL over NVLink/NVSwitch).
  "p2p"   fused in the GEMV kernel: each CTA stores its output rows straight into every peer's Y (CUDA IPC
          mappings over NVLink), and the last CTA runs a flag barrier with bounded waits (b2q_gemv_allgather).
"""

import torch
import torch.distributed as dist

from . import host


def partition(n, nranks, align=4):
    """[(row0, rows)] per rank: equal slices of ceil(n / nranks) rows rounded up to `align`, the last one shorter
    (possibly empty). Slice starts are multiples of `align`."""
    if nranks < 1:
        raise ValueError("nranks must be >= 1")
    per = -(-n // nranks)
    per = -(-per // align) * align
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


class RowShardedGemv:
    """One quantized layer, row-sharded over `group` (default: the world group).

    wq/ws: this rank's rows of the split planes (CUDA tensors), n/k: the full layer's shape.
    __call__(x f32 [M][K]) -> Y f32 [M][N] (the full output, on every rank).
    """

    def __init__(self, fmt, wq, ws, n, k, group=None, exchange="nccl"):
        if exchange not in ("nccl",):
            raise ValueError(f"exchange {exchange!r} is not available (expected 'nccl')")
        self.fmt, self.n, self.k, self.group, self.exchange = fmt, n, k, group, exchange
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.row0, self.rows = partition(n, self.world)[self.rank]
        if wq.shape[0] != self.rows or ws.shape[0] != self.rows:
            raise ValueError(f"rank {self.rank}: expected {self.rows} rows (from row {self.row0}), got "
                             f"{wq.shape[0]}/{ws.shape[0]}")
        self.wq, self.ws = wq, ws
        self.per = slice_rows(n, self.world)

    def local(self, x):
        """This rank's output slice [M][rows] (no exchange)."""
        return host.quant_gemv(self.fmt, self.wq, self.ws, x, self.rows, self.k)

    def __call__(self, x):
        m = x.shape[0]
        dev = x.device
        part = torch.zeros((m, self.per), dtype=torch.float32, device=dev)
        if self.rows:
            part[:, : self.rows] = self.local(x)
        gathered = torch.empty((self.world, m, self.per), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(gathered, part, group=self.group)
        return gathered.permute(1, 0, 2).reshape(m, self.world * self.per)[:, : self.n]
