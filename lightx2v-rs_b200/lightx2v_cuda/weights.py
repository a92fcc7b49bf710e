"""Quantized checkpoints straight to device weights, without an f32 round trip.

The reference stores a quantized linear `X` in safetensors
(crates/lightx2v-core/src/export.rs:1-17, written by `quantize_dit`
:41-121) as
    X.weight.q8   I8 [out, in]        X.weight.scale  F32 [out, in/group]
    X.weight.q4   U8 [out, in/2]      X.weight.scale, X.weight.zero  F16 [out, in/group]
                  (element 2i in the low nibble)
    X.weight.fp8  U8 [out, in]        X.weight.scale  F32 [out, in/group]
and reads it back with `SafetensorsDir::stored` (weights.rs:146-208) into
the `Q8` / `Q4` / `Fp8E4M3` structs that `Backend::weight_q8 / q4 / fp8`
take. `SafetensorsDir.stored` below does the same, with the same shape and
dtype checks, and `upload_stored` hands the codes and scales to the device as
stored (the library transposes the scales and packs Q4 on upload).

The reader is a small self-contained safetensors parser (8-byte
little-endian header length, JSON header, raw little-endian data, files
mapped read-only), so that BF16 tensors need no numpy bf16 type.
"""
from __future__ import annotations

import json
import os

import numpy as np

from .quant import Fp8E4M3, Q4, Q8

_NP = {"F32": np.float32, "F16": np.float16, "I8": np.int8, "U8": np.uint8, "BF16": np.uint16,
       "I32": np.int32, "I64": np.int64, "F64": np.float64}


class WeightsError(ValueError):
    """A missing or malformed tensor (the reference's `Error::Weights`)."""


class SafetensorsDir:
    """All `*.safetensors` under a directory (or one file), mapped read-only."""

    def __init__(self, path: str):
        files = ([os.path.join(path, f) for f in sorted(os.listdir(path)) if f.endswith(".safetensors")]
                 if os.path.isdir(path) else [path])
        self._index = {}
        for f in files:
            mm = np.memmap(f, dtype=np.uint8, mode="r")
            n = int(np.frombuffer(mm[:8].tobytes(), "<u8")[0])
            header = json.loads(mm[8:8 + n].tobytes())
            base = 8 + n
            for name, meta in header.items():
                if name == "__metadata__":
                    continue
                lo, hi = meta["data_offsets"]
                self._index[name] = (meta["dtype"], list(meta["shape"]), mm[base + lo:base + hi])

    def contains(self, name: str) -> bool:
        return name in self._index

    def raw(self, name: str):
        """(dtype, shape, little-endian bytes) of a tensor."""
        if name not in self._index:
            raise WeightsError(f"missing tensor `{name}`")
        return self._index[name]

    def get_f32(self, name: str) -> np.ndarray:
        """The tensor as f32 (exact for F16 and BF16 sources)."""
        dt, shape, data = self.raw(name)
        if dt == "BF16":
            bits = np.frombuffer(data, "<u2").astype(np.uint32) << 16
            return bits.view(np.float32).reshape(shape).copy()
        if dt not in ("F32", "F16", "F64"):
            raise WeightsError(f"`{name}` is {dt}, not a float tensor")
        return np.frombuffer(data, np.dtype(_NP[dt]).newbyteorder("<")).astype(np.float32).reshape(shape)

    def stored(self, key: str):
        """The linear `key` (no `.weight`) as Q8 / Q4 / Fp8E4M3 if it is stored
        quantized, else None (weights.rs:146-208)."""
        def bad(msg):
            return WeightsError(f"`{key}`: {msg}")

        q8, q4, fp8 = f"{key}.weight.q8", f"{key}.weight.q4", f"{key}.weight.fp8"
        if self.contains(q8):
            dt, shape, data = self.raw(q8)
            if dt != "I8" or len(shape) != 2:
                raise bad(f"q8 is {dt} {shape}")
            scales = self.get_f32(f"{key}.weight.scale")
            if scales.ndim != 2 or scales.shape[0] != shape[0] or shape[1] % scales.shape[1] != 0:
                raise bad(f"scale {list(scales.shape)} for codes {shape}")
            return Q8(np.frombuffer(data, np.int8).copy(), scales.reshape(-1).copy(), shape[0], shape[1],
                      shape[1] // scales.shape[1])
        if self.contains(q4):
            dt, shape, data = self.raw(q4)
            if dt != "U8" or len(shape) != 2:
                raise bad(f"q4 is {dt} {shape}")
            rows, cols = shape[0], 2 * shape[1]
            scales = self.get_f32(f"{key}.weight.scale")
            zeros = self.get_f32(f"{key}.weight.zero")
            if scales.shape != zeros.shape or scales.ndim != 2 or scales.shape[0] != rows or cols % scales.shape[1]:
                raise bad(f"scale {list(scales.shape)} / zero {list(zeros.shape)} for codes {shape}")
            return Q4.from_packed(np.frombuffer(data, np.uint8), scales.reshape(-1), zeros.reshape(-1), rows, cols)
        if self.contains(fp8):
            dt, shape, data = self.raw(fp8)
            if dt != "U8" or len(shape) != 2:
                raise bad(f"fp8 is {dt} {shape}")
            scales = self.get_f32(f"{key}.weight.scale")
            if scales.ndim != 2 or scales.shape[0] != shape[0] or shape[1] % scales.shape[1] != 0:
                raise bad(f"scale {list(scales.shape)} for codes {shape}")
            return Fp8E4M3(np.frombuffer(data, np.uint8).copy(), scales.reshape(-1).copy(), shape[0], shape[1],
                           shape[1] // scales.shape[1])
        return None

    def has_linear(self, key: str) -> bool:
        return any(self.contains(f"{key}.weight{s}") for s in ("", ".q8", ".q4", ".fp8"))


def upload_stored(be, w):
    """A stored quantized linear as a device weight (no f32 round trip)."""
    if isinstance(w, Q8):
        return be.weight_q8(w)
    if isinstance(w, Q4):
        return be.weight_q4(w)
    if isinstance(w, Fp8E4M3):
        return be.weight_fp8(w)
    raise TypeError(type(w))


def write_quantized(path: str, linears: dict, metadata: dict | None = None) -> None:
    """Write quantized linears `{key: Q8 | Q4 | Fp8E4M3}` in the reference's
    layout (export.rs:59-121): codes, F32 scales (Q8 / FP8) or F16 scale and
    zero (Q4), one safetensors file."""
    tensors = []
    for key, w in linears.items():
        name = f"{key}.weight"
        ng = w.cols // w.group
        if isinstance(w, Q8):
            tensors.append((f"{name}.q8", "I8", [w.rows, w.cols], np.asarray(w.q, np.int8).tobytes()))
            tensors.append((f"{name}.scale", "F32", [w.rows, ng], np.asarray(w.scales, "<f4").tobytes()))
        elif isinstance(w, Q4):
            tensors.append((f"{name}.q4", "U8", [w.rows, w.cols // 2], w.packed().tobytes()))
            tensors.append((f"{name}.scale", "F16", [w.rows, ng], np.asarray(w.scales, "<f2").tobytes()))
            tensors.append((f"{name}.zero", "F16", [w.rows, ng], np.asarray(w.zeros, "<f2").tobytes()))
        elif isinstance(w, Fp8E4M3):
            tensors.append((f"{name}.fp8", "U8", [w.rows, w.cols], np.asarray(w.q, np.uint8).tobytes()))
            tensors.append((f"{name}.scale", "F32", [w.rows, ng], np.asarray(w.scales, "<f4").tobytes()))
        else:
            raise TypeError(type(w))
    header, off = {}, 0
    for name, dt, shape, data in tensors:
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(data)]}
        off += len(data)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * (-len(hb) % 8)
    with open(path, "wb") as f:
        f.write(np.array([len(hb)], "<u8").tobytes())
        f.write(hb)
        for _, _, _, data in tensors:
            f.write(data)
