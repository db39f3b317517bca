"""numpy restatement of the `.sme` model container and of the weight
conversion the library performs when it loads one.

TEST INFRASTRUCTURE ONLY: used by tests/ to write model files of any size,
to read them independently of the library's C++ parser, and to form the
expected int4 weights.  The product path never imports it.

  write_sme   follows convert_model.py:8-67 (quantize_matrix, save_sme_model):
              2-D tensors with more than 16 rows become int8 rows with the row
              factor rs = 127 / max|w| (1 for an all-zero row) and
              q = clip(round(w * rs), -128, 127) in float32; everything else
              is stored as f32.  The output is pinned byte for byte against a
              file written by the reference's own save_sme_model
              (tests/golden/tiny_llama.sme, made by
              tests/golden/make_sme_fixture.py).
  read_sme    follows load_sme_model (server/main.cpp:112-228): offsets advance
              by the element count; a repeated name replaces the earlier
              tensor.
  sme_values  the weight values the loader forms: q / rs in float32 for int8
              rows (the writer's definition, model/README.md:41-52), the f32
              data otherwise, times a folded RMSNorm weight per column.
"""
from __future__ import annotations

import json
import struct

import numpy as np


def quantize_rows(w: np.ndarray):
    w = np.asarray(w, np.float32)
    q = np.zeros(w.shape, np.int8)
    rs = []
    for i in range(w.shape[0]):
        row = w[i]
        m = np.max(np.abs(row))
        s = np.float32(1.0) if m == 0 else np.float32(127.0) / m
        rs.append(s)
        q[i] = np.clip(np.round(row * s), -128, 127).astype(np.int8)
    return q, np.array(rs, np.float32)


def write_sme(config: dict, vocab, tensors: dict) -> bytes:
    out = [b"SME_MODEL"]
    cfg = json.dumps(config).encode("utf-8")
    out += [struct.pack("<I", len(cfg)), cfg, struct.pack("<I", len(vocab))]
    for tok in vocab:
        b = tok.encode("utf-8")
        out += [struct.pack("<I", len(b)), b]
    out.append(struct.pack("<I", len(tensors)))
    for name, data in tensors.items():
        nb = name.encode("utf-8")
        out += [struct.pack("<I", len(nb)), nb, struct.pack("<I", len(data.shape))]
        out += [struct.pack("<I", d) for d in data.shape]
        quant = 1 if len(data.shape) == 2 and data.shape[0] > 16 else 0
        out.append(struct.pack("B", quant))
        if quant:
            q, rs = quantize_rows(data)
            qb = q.tobytes()
            out += [struct.pack("<I", len(qb)), rs.tobytes(), qb]
        else:
            fb = np.asarray(data, np.float32).tobytes()
            out += [struct.pack("<I", len(fb)), fb]
    return b"".join(out)


class Truncated(ValueError):
    pass


def read_sme(buf: bytes) -> dict:
    """dict(config=str, vocab=[bytes], tensors={name: dict(dims, quantized,
    data_bytes, scales, data)}); Truncated / ValueError on a bad file."""
    at = 0

    def take(n):
        nonlocal at
        if n > len(buf) - at:
            raise Truncated(f"need {n} bytes at {at}")
        b = buf[at:at + n]
        at += n
        return b

    def u32():
        return struct.unpack("<I", take(4))[0]

    if len(buf) < 9 or buf[:9] != b"SME_MODEL":
        raise ValueError("magic header mismatch")
    at = 9
    config = take(u32()).decode("utf-8", "replace")
    vocab = [take(u32()) for _ in range(u32())]
    tensors = {}
    for _ in range(u32()):
        name = take(u32()).decode("utf-8", "replace")
        dims = tuple(u32() for _ in range(u32()))
        quant = take(1)[0] == 1
        data_bytes = u32()
        n = int(np.prod(dims, dtype=np.uint64)) if dims else 1
        if quant:
            scales = np.frombuffer(take(4 * dims[0]), np.float32)
            data = np.frombuffer(take(n), np.int8)
        else:
            scales = None
            data = np.frombuffer(take(4 * n), np.float32)
        tensors[name] = dict(dims=dims, quantized=quant, data_bytes=data_bytes, scales=scales, data=data)
    return dict(config=config, vocab=vocab, tensors=tensors)


def sme_values(t: dict, fold=None) -> np.ndarray:
    """[rows, K] float32 values of a 2-D tensor as the loader forms them."""
    rows, K = t["dims"]
    if t["quantized"]:
        v = t["data"].reshape(rows, K).astype(np.float32) / t["scales"][:, None]
    else:
        v = t["data"].reshape(rows, K).astype(np.float32)
    if fold is not None:
        v = v * np.asarray(fold, np.float32)[None, :]
    return np.ascontiguousarray(v, np.float32)
