"""Safetensors fuel checkpoints: zero-copy reading (native mmap reader) and writing.

    tensors = load_dir("/path/to/fuel")          # every *.safetensors (or the index)
    save_dir(tensors, "/path/to/fuel", shard_bytes=4 << 30)

Reading maps each file once through ``rocket_b200._rt.SafetensorsFile`` (C++:
header JSON parse, offset / size validation, mmap) and wraps every tensor's
bytes as a CPU torch tensor without copying; the mapping lives as long as any
tensor viewing it.  Writing is the offline path (fuel packing): the header is
JSON padded with spaces to an 8-byte boundary, tensors follow in name order.

Behavioural counterpart of the reference's Checkpoint reader
(engines/glm5-moe-nvfp4-2b/src/safetensors.h:25-83) and its fuel packing scripts
(scripts/fuels/pack-resident-weights.py).
"""
from __future__ import annotations

import json
import os
import struct

import torch

_TO_TORCH = {
    "F64": torch.float64, "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16,
    "I64": torch.int64, "I32": torch.int32, "I16": torch.int16, "I8": torch.int8, "U8": torch.uint8,
    "BOOL": torch.bool, "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2,
}
_FROM_TORCH = {v: k for k, v in _TO_TORCH.items()}
INDEX = "model.safetensors.index.json"


def load_file(path: str) -> dict[str, torch.Tensor]:
    """All tensors of one .safetensors file as zero-copy CPU tensors (read-only memory:
    clone before writing to one)."""
    import warnings

    from .. import _rt
    f = _rt.SafetensorsFile(path)
    out = {}
    for name in f.keys():
        dtype, shape, begin, end = f.info(name)
        if dtype not in _TO_TORCH:
            raise ValueError(f"{path}: {name}: unsupported dtype {dtype}")
        if end == begin:
            out[name] = torch.empty(shape, dtype=_TO_TORCH[dtype])
            continue
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")  # the mapping is read-only by design
            t = torch.frombuffer(f.bytes(name), dtype=torch.uint8)
        out[name] = t.view(_TO_TORCH[dtype]).reshape(shape)
    return out


def metadata(path: str) -> dict[str, str]:
    from .. import _rt
    return dict(_rt.SafetensorsFile(path).metadata())


def save_file(tensors: dict[str, torch.Tensor], path: str, meta: dict[str, str] | None = None):
    header: dict = {}
    if meta:
        header["__metadata__"] = {str(k): str(v) for k, v in meta.items()}
    off = 0
    names = sorted(tensors)
    blobs = []
    for n in names:
        t = tensors[n].detach().contiguous().cpu()
        if t.dtype not in _FROM_TORCH:
            raise ValueError(f"{n}: unsupported dtype {t.dtype}")
        b = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[n] = {"dtype": _FROM_TORCH[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * (-len(h) % 8)
    tmp = path + ".tmp"
    with open(tmp, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)))
        fh.write(h)
        for b in blobs:
            fh.write(b)
    os.replace(tmp, path)


def save_dir(tensors: dict[str, torch.Tensor], d: str, shard_bytes: int = 4 << 30, meta: dict | None = None):
    """Shards of at most ~shard_bytes plus a model.safetensors.index.json weight map."""
    os.makedirs(d, exist_ok=True)
    shards, cur, size = [], {}, 0
    for n in sorted(tensors):
        nb = tensors[n].numel() * tensors[n].element_size()
        if cur and size + nb > shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[n] = tensors[n]
        size += nb
    if cur or not shards:
        shards.append(cur)
    wmap = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(d, fn), meta)
        wmap.update({n: fn for n in sh})
    with open(os.path.join(d, INDEX), "w") as fh:
        json.dump({"metadata": dict(meta or {}), "weight_map": wmap}, fh, indent=1, sort_keys=True)


def load_dir(d: str) -> dict[str, torch.Tensor]:
    """Every tensor of a fuel directory (through the index when present)."""
    idx = os.path.join(d, INDEX)
    if os.path.exists(idx):
        with open(idx) as fh:
            files = sorted(set(json.load(fh)["weight_map"].values()))
    else:
        files = sorted(f for f in os.listdir(d) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {d}")
    out: dict[str, torch.Tensor] = {}
    for fn in files:
        part = load_file(os.path.join(d, fn))
        dup = set(part) & set(out)
        if dup:
            raise ValueError(f"tensor(s) in more than one shard: {sorted(dup)[:3]}")
        out.update(part)
    return out
