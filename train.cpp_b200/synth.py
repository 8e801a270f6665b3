"""Seeded synthetic inputs for the quantized-weight hot path, and a minimal GGUF v3 writer.

There is no dataset or checkpoint behind the workloads: every input is drawn here from a seeded
numpy PCG64 generator with the distributions the benchmark configurations specify:

  * block scale d: uniform in [1e-3, 1e-2], rounded to fp16 (round to nearest even)
  * block minimum m (Q4_1, Q5_1): uniform in [-0.05, 0.05], rounded to fp16
  * nibbles (qs) and Q5 high bits (qh): uniform random bytes / 32-bit words
  * Q8_0 quants: uniform int8 in [-128, 127]
  * activations / upstream gradients: N(0, 1) and N(0, 1e-2) (sigma = 1e-2) as float32

Block layouts follow GGUF's legacy formats (train.cpp src/io/trc_gguf.cpp:320-417): little-endian,
32 weights per block, fp16 fields first.

The GGUF writer emits the on-disk format train.cpp's reader parses (src/io/trc_gguf.cpp:521-654):
magic "GGUF", version 3, tensor and KV counts, KV pairs, tensor infos (name, n_dims, ne[], type,
offset), zero padding to the alignment (32), then the data segment. train.cpp's own writer cannot
store quantized tensors (include/traincpp/trc_gguf.h:150), so synthetic quantized files are made here.
"""
from __future__ import annotations

import struct
from pathlib import Path
from typing import Iterable

import numpy as np

QK = 32
TYPE_Q4_0, TYPE_Q4_1, TYPE_Q5_0, TYPE_Q5_1, TYPE_Q8_0 = 2, 3, 6, 7, 8
TYPE_F32 = 0
BLOCK_BYTES = {TYPE_Q4_0: 18, TYPE_Q4_1: 20, TYPE_Q5_0: 22, TYPE_Q5_1: 24, TYPE_Q8_0: 34}
TYPE_BY_NAME = {"q4_0": TYPE_Q4_0, "q4_1": TYPE_Q4_1, "q5_0": TYPE_Q5_0, "q5_1": TYPE_Q5_1, "q8_0": TYPE_Q8_0}


def _f16_bits(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float32).astype(np.float16).view(np.uint16)


def random_blocks(qtype: int, n_blocks: int, seed: int, d_range=(1e-3, 1e-2), m_range=(-0.05, 0.05)) -> np.ndarray:
    """n_blocks packed blocks (uint8 array of n_blocks * block_bytes) drawn per the configs."""
    rng = np.random.Generator(np.random.PCG64(seed))
    bb = BLOCK_BYTES[qtype]
    out = np.empty((n_blocks, bb), dtype=np.uint8)
    d = _f16_bits(rng.uniform(d_range[0], d_range[1], n_blocks))
    out[:, 0:2] = d.view(np.uint8).reshape(n_blocks, 2)
    if qtype == TYPE_Q4_0:
        out[:, 2:18] = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    elif qtype == TYPE_Q4_1:
        m = _f16_bits(rng.uniform(m_range[0], m_range[1], n_blocks))
        out[:, 2:4] = m.view(np.uint8).reshape(n_blocks, 2)
        out[:, 4:20] = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    elif qtype == TYPE_Q5_0:
        out[:, 2:6] = rng.integers(0, 256, (n_blocks, 4), dtype=np.uint8)
        out[:, 6:22] = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    elif qtype == TYPE_Q5_1:
        m = _f16_bits(rng.uniform(m_range[0], m_range[1], n_blocks))
        out[:, 2:4] = m.view(np.uint8).reshape(n_blocks, 2)
        out[:, 4:8] = rng.integers(0, 256, (n_blocks, 4), dtype=np.uint8)
        out[:, 8:24] = rng.integers(0, 256, (n_blocks, 16), dtype=np.uint8)
    elif qtype == TYPE_Q8_0:
        out[:, 2:34] = rng.integers(-128, 128, (n_blocks, 32), dtype=np.int8).view(np.uint8)
    else:
        raise ValueError(f"not a legacy quantized type: {qtype}")
    return out.reshape(-1)


def random_blocks_torch(qtype: int, n_blocks: int, generator, device) -> "torch.Tensor":
    """random_blocks' distributions drawn on the device with a seeded torch generator (for the
    multi-GB whole-model workload; the bytes differ from the numpy draw). Returns a uint8 tensor
    of n_blocks * block_bytes."""
    import torch

    bb = BLOCK_BYTES[qtype]
    out = torch.empty((n_blocks, bb), dtype=torch.uint8, device=device)

    def f16_bytes(lo: float, hi: float) -> "torch.Tensor":
        x = torch.rand(n_blocks, generator=generator, device=device, dtype=torch.float32) * (hi - lo) + lo
        return x.to(torch.float16).view(torch.uint8).view(n_blocks, 2)

    def rand_bytes(n: int) -> "torch.Tensor":
        return torch.randint(0, 256, (n_blocks, n), generator=generator, device=device, dtype=torch.uint8)

    out[:, 0:2] = f16_bytes(1e-3, 1e-2)
    if qtype == TYPE_Q4_0:
        out[:, 2:18] = rand_bytes(16)
    elif qtype == TYPE_Q4_1:
        out[:, 2:4] = f16_bytes(-0.05, 0.05)
        out[:, 4:20] = rand_bytes(16)
    elif qtype == TYPE_Q5_0:
        out[:, 2:22] = rand_bytes(20)
    elif qtype == TYPE_Q5_1:
        out[:, 2:4] = f16_bytes(-0.05, 0.05)
        out[:, 4:24] = rand_bytes(20)
    elif qtype == TYPE_Q8_0:
        out[:, 2:34] = rand_bytes(32)  # every byte value is an int8 in [-128, 127]
    else:
        raise ValueError(f"not a legacy quantized type: {qtype}")
    return out.view(-1)


def normal(shape, seed: int, sigma: float = 1.0) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(seed))
    return (rng.standard_normal(size=shape, dtype=np.float32) * np.float32(sigma)).astype(np.float32)


# ------------------------------------------------------------------ workloads of the configs

def llama7b_tensors() -> list[tuple[str, int, tuple[int, int]]]:
    """The whole-model configuration: 32 layers, d=4096, ffn=11008, vocab=32000, no biases.
    Attention Q/K/V/O are Q8_0, MLP gate/up/down Q4_0, token embedding and output head Q5_1.
    Returns (name, type, ne) in file order; ne follows ggml (ne0 = row length)."""
    d, ffn, vocab = 4096, 11008, 32000
    t: list[tuple[str, int, tuple[int, int]]] = [("token_embd.weight", TYPE_Q5_1, (d, vocab))]
    for layer in range(32):
        p = f"blk.{layer}."
        for n in ("attn_q", "attn_k", "attn_v", "attn_output"):
            t.append((p + n + ".weight", TYPE_Q8_0, (d, d)))
        t.append((p + "ffn_gate.weight", TYPE_Q4_0, (d, ffn)))
        t.append((p + "ffn_up.weight", TYPE_Q4_0, (d, ffn)))
        t.append((p + "ffn_down.weight", TYPE_Q4_0, (ffn, d)))
    t.append(("output.weight", TYPE_Q5_1, (d, vocab)))
    return t


def lpt_shards(sizes, n_shards: int):
    """Byte-balanced tensor partition (see sharding.lpt_shards)."""
    from sharding import lpt_shards as _lpt

    return _lpt(list(sizes), n_shards)


# ------------------------------------------------------------------ GGUF v3 writer

def _gguf_str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str | Path, tensors: list[tuple[str, int, tuple[int, ...], bytes | np.ndarray]],
               alignment: int = 32) -> None:
    """Writes a GGUF v3 file holding the given (name, type, ne, raw bytes) tensors, no KV pairs."""
    infos = bytearray()
    offset = 0
    offsets = []
    for name, ttype, ne, data in tensors:
        offsets.append(offset)
        nbytes = len(data) if isinstance(data, (bytes, bytearray)) else data.nbytes
        infos += _gguf_str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<q", n) for n in ne)
        infos += struct.pack("<IQ", ttype, offset)
        offset += (nbytes + alignment - 1) // alignment * alignment
    header = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), 0)
    with open(path, "wb") as f:
        f.write(header)
        f.write(infos)
        pos = len(header) + len(infos)
        f.write(b"\0" * ((alignment - pos % alignment) % alignment))
        for (name, ttype, ne, data), off in zip(tensors, offsets):
            raw = bytes(data) if isinstance(data, (bytes, bytearray)) else data.tobytes()
            f.write(raw)
            f.write(b"\0" * ((alignment - len(raw) % alignment) % alignment))
