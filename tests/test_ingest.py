"""GGUF ingest (comp_b200.gguf_io): a Q4_0 / TQ2_0 / Q8_0 tensor written with gguf-py is read back as the same ggml block
bytes with KURN's (n, k); host.split of those bytes is the reference's plane cut (src/komp/host.py:16-22). The
on-device cut (host.split_device, b2q_split_blocks) is checked against host.split in tests/test_gpu_parity.py."""

import numpy as np
import pytest
import torch

from comp_b200 import gguf_io, host
from oracle import ref

gguf = pytest.importorskip("gguf")


def _write(path, tensors):
    w = gguf.GGUFWriter(str(path), "llama")
    for name, fmt, raw, n, k in tensors:
        arr = np.frombuffer(raw, dtype=np.uint8).reshape(n, -1)
        w.add_tensor(name, arr, raw_dtype=getattr(gguf.GGMLQuantizationType, fmt.upper()))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_gguf_tensor_round_trip_and_split(tmp_path):
    rng = np.random.default_rng(61)
    specs = [("blk.0.ffn_down.weight", "q4_0", 37, 416), ("blk.0.ffn_gate.weight", "tq2_0", 5, 768),
             ("output.weight", "q4_0", 64, 4096), ("blk.0.ffn_up.weight", "q8_0", 11, 1024),
             ("blk.0.attn_k.weight", "iq4_nl", 7, 512)]
    tensors = [(name, fmt, ref.weight_blocks(fmt, rng, n, k), n, k) for name, fmt, n, k in specs]
    path = tmp_path / "t.gguf"
    _write(path, tensors)
    reader = gguf.GGUFReader(str(path))
    for name, fmt, raw, n, k in tensors:
        f, rn, rk, data = gguf_io.tensor_info(reader, name)
        assert (f, rn, rk) == (fmt, n, k)
        assert np.ascontiguousarray(data).tobytes() == raw
        wq, ws = host.split(fmt, data.tobytes(), n, k)
        blocks = np.frombuffer(raw, dtype=np.uint8).reshape(n, -1, host.FORMATS[fmt]["nbytes"])
        fm = host.FORMATS[fmt]
        assert np.array_equal(wq, blocks[:, :, fm["qoff"]:fm["qoff"] + fm["qbytes"]].reshape(n, -1))
        assert np.array_equal(ws.view(np.uint8).reshape(n, -1, 2), blocks[:, :, fm["soff"]:fm["soff"] + 2])
    with pytest.raises(KeyError):
        gguf_io.tensor_info(reader, "missing.weight")


def test_gguf_rejects_other_types(tmp_path):
    path = tmp_path / "f.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_tensor("tok_embd.weight", np.zeros((4, 32), dtype=np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ValueError, match="expected one of"):
        gguf_io.tensor_info(gguf.GGUFReader(str(path)), "tok_embd.weight")


def test_split_device_needs_cuda_tensors():
    raw = torch.zeros(18 * 4, dtype=torch.uint8)
    with pytest.raises(RuntimeError, match="CUDA"):
        host.split_device("q4_0", raw, 4, 32)
    with pytest.raises(ValueError):
        host.split_device("q4_0", raw, 4, 33)
