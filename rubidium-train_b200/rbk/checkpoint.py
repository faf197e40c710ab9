"""Checkpoint files of rubidium-train models, read and written on the host.

Layout (little-endian), as written by rbk_model_save (include/rbk.h):

    "RBN2" | V T D H L FF (int32) | char map [256] (int32) |
    FP16 weights in the reference's tensor order            (src/model.cu:585-624)
    "RBKX" | version (int32) | elements per family (int64) | scaler (8 x 4 bytes) |
    FP32 masters | Adam m | Adam v, each in the same tensor order

The first part is the reference's own RBN2 file (its save/load pass device
pointers to fwrite / fread, and it keeps no optimizer state); the "RBKX" block
after it is optional.  Tensors are stored as rows * cols elements without the
device arena's padding.  This module needs no GPU: it inspects, converts or
prepares files (e.g. a reference-layout file from FP16 weights).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field

import numpy as np

# per-layer order of the reference's save() (src/model.cu:607-614)
FILE_LAYER_ORDER = ["ln1_w", "ln1_b", "ln2_w", "ln2_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo",
                    "w1", "b1", "w2", "b2"]
EXT_VERSION = 1
SCALER_FIELDS = ["scale", "unskipped", "interval", "skipped", "applied_steps", "overflow_steps", "status", "pad"]


def file_tensors(V, T, D, H, L, FF):
    """[(name, rows, cols)] in file order; names as in rbk.model.param_table."""
    def shape(n):
        return {"wq": (D, D), "wk": (D, D), "wv": (D, D), "wo": (D, D), "w1": (FF, D), "w2": (D, FF),
                "b1": (1, FF)}.get(n, (1, D))
    out = [("token_emb", V, D), ("pos_emb", T, D)]
    for l in range(L):
        out += [(f"layers.{l}.{n}",) + shape(n) for n in FILE_LAYER_ORDER]
    out += [("ln_f_w", 1, D), ("ln_f_b", 1, D), ("lm_w", V, D), ("lm_b", 1, V)]
    return out


@dataclass
class Checkpoint:
    config: tuple                      # (V, T, D, H, L, FF)
    char_map: np.ndarray               # int32 [256]
    weights16: dict                    # name -> float16 array [rows, cols] (vectors: [cols])
    scaler: dict | None = None         # extension block, when present
    masters: dict = field(default_factory=dict)
    adam_m: dict = field(default_factory=dict)
    adam_v: dict = field(default_factory=dict)

    @property
    def has_optimizer_state(self) -> bool:
        return self.scaler is not None


def _shaped(a, r, c):
    return a.reshape(r, c) if r > 1 else a


def read(path) -> Checkpoint:
    with open(path, "rb") as f:
        data = f.read()
    if len(data) < 4 + 24 + 1024 or data[:4] != b"RBN2":
        raise ValueError(f"{path}: not an RBN2 checkpoint")
    cfg = struct.unpack_from("<6i", data, 4)
    cmap = np.frombuffer(data, "<i4", 256, 28).copy()
    pos = 28 + 1024
    tens = file_tensors(*cfg)

    def family(dtype, pos):
        out = {}
        es = np.dtype(dtype).itemsize
        for name, r, c in tens:
            n = r * c
            if pos + n * es > len(data):
                raise ValueError(f"{path}: file is truncated")
            out[name] = _shaped(np.frombuffer(data, dtype, n, pos).copy(), r, c)
            pos += n * es
        return out, pos

    w16, pos = family("<f2", pos)
    ck = Checkpoint(cfg, cmap, w16)
    if pos == len(data):
        return ck
    if data[pos:pos + 4] != b"RBKX":
        raise ValueError(f"{path}: unknown data after the FP16 weights")
    ver, ne = struct.unpack_from("<iq", data, pos + 4)
    if ver != EXT_VERSION:
        raise ValueError(f"{path}: extension version {ver}")
    if ne != sum(r * c for _, r, c in tens):
        raise ValueError(f"{path}: element count {ne} does not match the config")
    sc = struct.unpack_from("<fiiiiiii", data, pos + 16)
    ck.scaler = dict(zip(SCALER_FIELDS, sc))
    pos += 16 + 32
    ck.masters, pos = family("<f4", pos)
    ck.adam_m, pos = family("<f4", pos)
    ck.adam_v, pos = family("<f4", pos)
    if pos != len(data):
        raise ValueError(f"{path}: trailing bytes after the extension block")
    return ck


def write(path, ck: Checkpoint):
    """Write `ck`; the extension block only when ck.scaler is set."""
    tens = file_tensors(*ck.config)
    cmap = np.zeros(256, "<i4") if ck.char_map is None else np.asarray(ck.char_map, "<i4")
    with open(path, "wb") as f:
        f.write(b"RBN2")
        f.write(struct.pack("<6i", *ck.config))
        f.write(cmap.tobytes())
        for name, r, c in tens:
            f.write(np.asarray(ck.weights16[name], "<f2").reshape(r * c).tobytes())
        if ck.scaler is None:
            return
        f.write(b"RBKX")
        f.write(struct.pack("<iq", EXT_VERSION, sum(r * c for _, r, c in tens)))
        s = ck.scaler
        f.write(struct.pack("<fiiiiiii", *(s.get(k, 0) for k in SCALER_FIELDS)))
        for fam in (ck.masters, ck.adam_m, ck.adam_v):
            for name, r, c in tens:
                f.write(np.asarray(fam[name], "<f4").reshape(r * c).tobytes())
