"""Offline fuel materialization: a bf16 / fp32 checkpoint -> an NVFP4 fuel directory.

    rep = materialize(src_dir, out_dir, cfg)            # weight_format of the fuel decides
    bad = verify(out_dir)                                # [] when every shard's digest matches

Each linear weight whose part (experts, shared, dense, attention, lm_head,
eh_proj) the fuel's ``weight_format`` marks ``nvfp4`` is written as the NVFP4
triplet (``.weight`` U8 [N, K/2], ``.weight_scale`` E4M3 [N, K/16],
``.weight_scale_2`` F32), one marked ``fp8`` as FP8-row (``.weight`` F8_E4M3 [N, K],
``.weight_scale`` F32 [N]); the remaining floating-point tensors are cast to bf16
except those the engine keeps in fp32 (router bias, DeltaNet A_log / dt_bias).
The quantization and the file writing are native (``_rt.materialize_nvfp4``,
multi-threaded C++); the report carries the worst relative quantization error
and a 256-bit digest per shard (also written to ``checksums.txt``).

Counterpart of the reference's overlay materializer and checksum tooling
(scripts/numerics/materialize-nvfp4-overlay.cc, scripts/fuels/build-checksums-blake3.py).
"""
from __future__ import annotations

import json
import os
import re

from .safetensors_io import INDEX

_FP32_KEEP = re.compile(r"(\.router\.bias|\.A_log|\.dt_bias)$")


def part_of(name: str) -> str | None:
    """Weight-format part of a linear named `name` (without '.weight'), None if not a linear."""
    if ".moe.experts." in name:
        return "experts"
    if ".moe.shared" in name and not name.endswith("shared_gate"):
        return "shared"
    if ".mlp." in name:
        return "dense"
    if ".attn." in name and not name.endswith("_norm"):
        return "attention"
    if ".dn." in name and name.rsplit(".", 1)[-1] in ("in_proj_qkvz", "in_proj_ba", "out_proj"):
        return "attention"
    if name == "lm_head":
        return "lm_head"
    if name.endswith("eh_proj"):
        return "eh_proj"
    return None


def _inputs(src: str) -> list[str]:
    if os.path.isfile(src):
        return [src]
    idx = os.path.join(src, INDEX)
    if os.path.exists(idx):
        with open(idx) as fh:
            files = sorted(set(json.load(fh)["weight_map"].values()))
    else:
        files = sorted(f for f in os.listdir(src) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {src}")
    return [os.path.join(src, f) for f in files]


def plan(inputs: list[str], weight_format: dict) -> tuple[set, set, set]:
    """(linear names to store as NVFP4, as FP8-row, tensor names to cast to bf16)."""
    from .. import _rt
    quant, fp8, cast = set(), set(), set()
    for p in inputs:
        f = _rt.SafetensorsFile(p)
        for n in f.keys():
            dtype, shape, _, _ = f.info(n)
            if dtype not in ("F32", "F16", "BF16"):
                continue
            if n.endswith(".weight") and len(shape) == 2:
                part = part_of(n[:-len(".weight")])
                fmt = weight_format.get(part, "bf16") if part else "bf16"
                if fmt == "nvfp4" and shape[1] % 16 == 0:
                    quant.add(n[:-len(".weight")])
                    continue
                if fmt == "fp8":
                    fp8.add(n[:-len(".weight")])
                    continue
            if dtype != "BF16" and not _FP32_KEEP.search(n) and not n.endswith(".weight_scale_2"):
                cast.add(n)
    return quant, fp8, cast


def materialize(src: str, out_dir: str, weight_format: dict, shard_bytes: int = 4 << 30, threads: int = 0,
                meta: dict | None = None) -> dict:
    from .. import _rt
    inputs = _inputs(src)
    quant, fp8, cast = plan(inputs, weight_format)
    m = {"format": "rocket_b200-fuel", "weight_format": json.dumps(weight_format, sort_keys=True)}
    m.update({str(k): str(v) for k, v in (meta or {}).items()})
    return _rt.materialize_nvfp4(inputs, out_dir, quant, cast, shard_bytes, threads, m, fp8)


def verify(out_dir: str) -> list[str]:
    from .. import _rt
    return list(_rt.verify_checksums(out_dir))
