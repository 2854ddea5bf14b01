"""GGUF weight ingest: a Q4_0 / TQ2_0 / Q8_0 / IQ4_NL / Q4_K tensor of a GGUF file -> the GEMV's split planes in GPU
memory.

The tensor's bytes are copied to the GPU as stored (ggml blocks, row after row) and cut into WQ / WS there
(`host.split_device`, the on-device form of `host.split`, src/komp/host.py:16-22). GGUF lists a 2-D weight's shape as
[k, n] (values per row first); the file is read with gguf-py (`gguf.GGUFReader`, memory-mapped).
"""

import numpy as np
import torch

from . import host

GGUF_TYPES = {"Q4_0": "q4_0", "TQ2_0": "tq2_0", "Q8_0": "q8_0", "IQ4_NL": "iq4_nl", "Q4_K": "q4_k"}


def tensor_info(reader, name):
    """(fmt, n, k, raw uint8 [n][bytes per row]) of tensor `name` in an open gguf.GGUFReader."""
    for t in reader.tensors:
        if t.name == name:
            kind = t.tensor_type.name
            if kind not in GGUF_TYPES:
                raise ValueError(f"{name}: GGUF type {kind}, expected one of {sorted(GGUF_TYPES)}")
            shape = [int(s) for s in t.shape]
            if len(shape) != 2:
                raise ValueError(f"{name}: {len(shape)}-D tensor, expected a 2-D weight")
            k, n = shape
            return GGUF_TYPES[kind], n, k, np.asarray(t.data)
    raise KeyError(f"no tensor {name!r} in the GGUF file")


def load_split(path, name, device="cuda", ldwq=None):
    """-> (fmt, WQ, WS, n, k): tensor `name` of the GGUF file at `path`, split on `device` (a CUDA device)."""
    import gguf

    reader = gguf.GGUFReader(path)
    fmt, n, k, raw = tensor_info(reader, name)
    # staged through pinned host memory: the memory-mapped tensor is read once, and the upload is one DMA copy
    staging = torch.empty(raw.nbytes, dtype=torch.uint8, pin_memory=True)
    staging.numpy()[:] = np.ascontiguousarray(raw).reshape(-1)
    blocks = staging.to(device)
    wq, ws = host.split_device(fmt, blocks, n, k, ldwq=ldwq)
    return fmt, wq, ws, n, k
