"""INT4 weights on disk: quantise a safetensors checkpoint into the layout
``gemm_int4`` reads, and load it back.

The reference's model loader only stubs safetensors (src/runtime/model_loader.cpp:57-85)
and its header documents, without producing, the INT4 format (include/clove/kernels/
gemm.cuh:67-87). This module closes that gap:

* ``quantize_checkpoint(src, dst)`` reads every tensor of ``src``; each 2-D floating
  point weight ``[rows, K]`` whose name matches ``include`` and whose K is a multiple
  of 128 is packed on the GPU by ``clove_quantize_int4`` into three tensors,
  ``<name>.q4`` (codes ``[rows, K/2]`` uint8, element 2j in the high nibble of byte j),
  ``<name>.q4_scale`` and ``<name>.q4_zero`` (``[rows, K/128]`` fp16); every other
  tensor is copied unchanged. The file records the format in its metadata
  (``clove.int4`` = ``group128-kpacked-hi-even``).
* ``load_int4(path, name)`` returns ``(codes, scales, zeros)`` on the GPU, ready for
  ``gemm_int4`` as either operand.

Safetensors is read and written directly (an 8-byte little-endian header length, a
JSON header of ``{name: {dtype, shape, data_offsets}}`` plus optional
``__metadata__``, then the raw little-endian tensor bytes), so no extra package is
needed. Command line: ``python -m clove_compute_b200.quantize IN OUT [--include RE]``.
"""
from __future__ import annotations

import argparse
import json
import re
import struct

import numpy as np

INT4_FORMAT = "group128-kpacked-hi-even"

_DTYPES = {  # safetensors dtype -> numpy dtype (BF16 is carried as raw uint16)
    "F64": np.float64, "F32": np.float32, "F16": np.float16, "BF16": np.uint16,
    "I64": np.int64, "I32": np.int32, "I16": np.int16, "I8": np.int8,
    "U64": np.uint64, "U32": np.uint32, "U16": np.uint16, "U8": np.uint8, "BOOL": np.bool_,
}
_NAMES = {np.dtype(np.float64): "F64", np.dtype(np.float32): "F32", np.dtype(np.float16): "F16",
          np.dtype(np.int64): "I64", np.dtype(np.int32): "I32", np.dtype(np.int16): "I16",
          np.dtype(np.int8): "I8", np.dtype(np.uint64): "U64", np.dtype(np.uint32): "U32",
          np.dtype(np.uint16): "U16", np.dtype(np.uint8): "U8", np.dtype(np.bool_): "BOOL"}


class Tensor:
    """One safetensors entry: its dtype name, shape and raw bytes."""

    def __init__(self, dtype: str, shape, data: bytes):
        self.dtype, self.shape, self.data = dtype, tuple(int(x) for x in shape), data

    def numpy(self) -> np.ndarray:
        return np.frombuffer(self.data, dtype=_DTYPES[self.dtype]).reshape(self.shape)

    @staticmethod
    def from_numpy(a: np.ndarray, dtype: str | None = None) -> "Tensor":
        a = np.asarray(a)  # (np.ascontiguousarray would turn a 0-d array into 1-d)
        return Tensor(dtype or _NAMES[a.dtype], a.shape, a.tobytes(order="C"))


def read_safetensors(path: str):
    """(tensors {name: Tensor} in file order, metadata {str: str})."""
    with open(path, "rb") as f:
        raw = f.read()
    if len(raw) < 8:
        raise ValueError(f"{path}: too short for a safetensors header")
    (n,) = struct.unpack("<Q", raw[:8])
    if 8 + n > len(raw):
        raise ValueError(f"{path}: header length {n} runs past the file")
    header = json.loads(raw[8:8 + n].decode("utf-8"))
    meta = header.pop("__metadata__", {}) or {}
    base = 8 + n
    out = {}
    for name, h in header.items():
        b, e = h["data_offsets"]
        if h["dtype"] not in _DTYPES:
            raise ValueError(f"{path}: {name}: unsupported dtype {h['dtype']}")
        count = int(np.prod(h["shape"], dtype=np.int64)) if h["shape"] else 1
        if not 0 <= b <= e <= len(raw) - base or e - b != count * np.dtype(_DTYPES[h["dtype"]]).itemsize:
            raise ValueError(f"{path}: {name}: data offsets {b}..{e} do not match its shape")
        out[name] = Tensor(h["dtype"], h["shape"], raw[base + b:base + e])
    return out, meta


def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """tensors: {name: Tensor}; metadata: {str: str}."""
    header, off = {}, 0
    for name, t in tensors.items():
        header[name] = {"dtype": t.dtype, "shape": list(t.shape),
                        "data_offsets": [off, off + len(t.data)]}
        off += len(t.data)
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hb = json.dumps(header, separators=(",", ":")).encode("utf-8")
    hb += b" " * (-len(hb) % 8)  # keep the data 8-byte aligned
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for t in tensors.values():
            f.write(t.data)


def _to_fp16(t: Tensor) -> np.ndarray:
    a = t.numpy()
    if t.dtype == "BF16":  # bf16 bits are the high half of an fp32
        a = (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float16)


def selects(name: str, t: Tensor, include: str) -> bool:
    """Whether quantize_checkpoint packs this tensor."""
    return (t.dtype in ("F32", "F16", "BF16") and len(t.shape) == 2 and t.shape[1] > 0
            and t.shape[1] % 128 == 0 and t.shape[0] > 0 and re.search(include, name) is not None)


def quantize_checkpoint(src: str, dst: str, include: str = r".", device: str = "cuda") -> list:
    """Writes dst with every selected weight packed to INT4 on the GPU; returns the
    names that were packed."""
    import torch
    from . import api
    tensors, meta = read_safetensors(src)
    out, packed = {}, []
    for name, t in tensors.items():
        if not selects(name, t, include):
            out[name] = t
            continue
        W = torch.from_numpy(_to_fp16(t)).to(device)
        codes, scales, zeros = api.quantize_int4(W)
        torch.cuda.synchronize()
        out[name + ".q4"] = Tensor.from_numpy(codes.cpu().numpy())
        out[name + ".q4_scale"] = Tensor.from_numpy(scales.cpu().numpy())
        out[name + ".q4_zero"] = Tensor.from_numpy(zeros.cpu().numpy())
        packed.append(name)
    meta = dict(meta)
    meta["clove.int4"] = INT4_FORMAT
    write_safetensors(dst, out, meta)
    return packed


def load_int4(path: str, name: str, device: str = "cuda"):
    """(codes, scales, zeros) of one packed weight, as CUDA tensors."""
    import torch
    tensors, meta = read_safetensors(path)
    if meta.get("clove.int4") != INT4_FORMAT:
        raise ValueError(f"{path} does not hold clove INT4 weights ({meta.get('clove.int4')!r})")
    parts = [tensors[name + s].numpy() for s in (".q4", ".q4_scale", ".q4_zero")]
    return tuple(torch.from_numpy(np.array(p)).to(device) for p in parts)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="Pack a safetensors checkpoint's 2-D weights to "
                                             "clove INT4 (group 128, K-packed) on the GPU.")
    ap.add_argument("src")
    ap.add_argument("dst")
    ap.add_argument("--include", default=r".", help="regex on tensor names (default: all)")
    a = ap.parse_args(argv)
    names = quantize_checkpoint(a.src, a.dst, a.include)
    print(f"packed {len(names)} tensor(s) into {a.dst}")


if __name__ == "__main__":
    main()
