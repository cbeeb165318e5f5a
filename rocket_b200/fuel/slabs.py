"""Rank-local expert slabs: pack once offline, preload with one sequential read.

    pack_expert_slabs(tensors, cfg, out_dir, world=8)               # offline
    load_expert_slabs(model, path)                                   # at engine start

A slab holds one EP rank's routed experts (and the shared experts every rank
keeps) for every MoE layer, already in the engine layout: per expert a slot of
six pieces -- fused gate|up (w13) packed e2m1, its scale atoms in the tcgen05
layout, its per-row tensor scales, then the same three for the down projection
(w2).  Slots start on 64 KiB boundaries, so the loader reads the file in large
4 KiB-aligned O_DIRECT requests straight into a ring of pinned buffers and
copies each slot's pieces to their place in the stacked device weights while the
next buffers are being read (native reader: ``_rt.SlabReader``).  Each slot
carries a 256-bit digest checked in the reader threads before its bytes are
copied to the device: a damaged slab refuses to load.

File: ``RKTSLAB1`` magic, u64 header length, JSON header, zero padding to a
64 KiB boundary, slots.  The header records the fuel, rank / world, expert order
and, per layer, the slot names, offsets, piece extents and digests.

Counterpart of the reference's expert slab packing and preload
(scripts/fuels/pack-expert-slabs.py:1-10 -- 64 KiB-aligned rank-local slots;
engines/glm5-moe-nvfp4-2b/src/weights.cu:777-925 preload_expert_slab, pinned
double-buffered O_DIRECT -> H2D; :928 preload_owned_experts).
"""
from __future__ import annotations

import json
import os
import struct

import torch

MAGIC = b"RKTSLAB1"
ALIGN = 64 << 10
PIECES = ("w13.packed", "w13.sf", "w13.g", "w2.packed", "w2.sf", "w2.g")


def _up(x: int, a: int = ALIGN) -> int:
    return (x + a - 1) // a * a


def slab_name(rank: int, world: int) -> str:
    return f"experts.rank{rank}-of-{world}.slab"


def moe_prefixes(cfg, tensors=None) -> list[str]:
    pre = [f"layers.{i}" for i in range(cfg.num_layers) if cfg.is_moe_layer(i)]
    if cfg.num_experts and cfg.mtp_layers and (tensors is None or "mtp.0.layer.moe.router.weight" in tensors):
        pre.append("mtp.0.layer")
    return pre


def slot_names(cfg, pre: str, rank: int, world: int, expert_order=None) -> list[str]:
    """Expert linears rank `rank` holds for layer `pre`, in the engine's stacking order."""
    E = cfg.num_experts
    order = list(expert_order) if expert_order is not None else list(range(E))
    El = E // world
    names = [f"{pre}.moe.experts.{order[e]}" for e in range(rank * El, (rank + 1) * El)]
    names += ([f"{pre}.moe.shared"] if cfg.num_shared_experts == 1 else
              [f"{pre}.moe.shared.{s}" for s in range(cfg.num_shared_experts)])
    return names


def _slot_pieces(t: dict, name: str) -> list[bytes]:
    from ..models import weights as W
    from . import nvfp4 as nv
    w13 = W.fuse_w13(W.triplet_of(t, name + ".gate_proj"), W.triplet_of(t, name + ".up_proj"))
    w2 = W.triplet_of(t, name + ".down_proj")
    out = []
    for tr in (w13, w2):
        out.append(tr.packed.contiguous().numpy().tobytes())
        out.append(nv.swizzle_sf(tr.sf.contiguous()).numpy().tobytes())
        out.append(tr.gscale.float().contiguous().numpy().tobytes())
    return out


def pack_expert_slabs(t: dict, cfg, out_dir: str, world: int, expert_order=None, fuel: str = "") -> list[str]:
    """Write one slab per EP rank; returns the paths."""
    from .. import _rt
    if cfg.num_experts % world:
        raise ValueError(f"{cfg.num_experts} experts do not split over {world} ranks")
    os.makedirs(out_dir, exist_ok=True)
    paths = []
    for r in range(world):
        layers, blobs, off = [], [], 0
        for pre in moe_prefixes(cfg, t):
            slots = []
            for nm in slot_names(cfg, pre, r, world, expert_order):
                pcs = _slot_pieces(t, nm)
                rel, ext = 0, {}
                for key, b in zip(PIECES, pcs):
                    ext[key] = [rel, len(b)]
                    rel += len(b)
                body = b"".join(pcs)
                slots.append({"name": nm, "offset": off, "bytes": len(body), "pieces": ext,
                              "digest": _rt.digest_hex(body)})
                blobs.append((off, body))
                off = _up(off + len(body))
            layers.append({"prefix": pre, "slots": slots})
        header = {"version": 1, "fuel": fuel, "rank": r, "world": world,
                  "expert_order": list(expert_order) if expert_order is not None else list(range(cfg.num_experts)),
                  "d_model": cfg.d_model, "layers": layers}
        h = json.dumps(header, separators=(",", ":")).encode()
        base = _up(16 + len(h))
        # offsets in the header are relative to the data start; store it for the reader
        header["data_start"] = base
        h = json.dumps(header, separators=(",", ":")).encode()
        if _up(16 + len(h)) != base:  # the extra field pushed the header over a boundary
            base = _up(16 + len(h))
            header["data_start"] = base
            h = json.dumps(header, separators=(",", ":")).encode()
        p = os.path.join(out_dir, slab_name(r, world))
        with open(p + ".tmp", "wb") as f:
            f.write(MAGIC + struct.pack("<Q", len(h)) + h)
            f.write(b"\0" * (base - 16 - len(h)))
            pos = 0
            for o, body in blobs:
                if o > pos:
                    f.write(b"\0" * (o - pos))
                f.write(body)
                pos = o + len(body)
            end = _up(pos, 4096)
            if end > pos:
                f.write(b"\0" * (end - pos))   # the last O_DIRECT request stays 4 KiB-aligned
        os.replace(p + ".tmp", p)
        paths.append(p)
    return paths


def read_header(path: str) -> dict:
    with open(path, "rb") as f:
        head = f.read(16)
        if len(head) < 16 or head[:8] != MAGIC:
            raise ValueError(f"{path}: not an expert slab")
        (n,) = struct.unpack("<Q", head[8:])
        return json.loads(f.read(n))


def _buffers(n_buf: int, nbytes: int, pinned: bool):
    bufs = []
    for _ in range(n_buf):
        raw = torch.empty(nbytes + 4096, dtype=torch.uint8, pin_memory=pinned)
        a = (-raw.data_ptr()) % 4096   # O_DIRECT wants a 4 KiB-aligned destination
        bufs.append((raw, raw[a:a + nbytes]))
    return bufs


def read_slab(path: str, targets: dict, ring_bytes: int = 256 << 20, n_buf: int = 3, threads: int = 4,
              verify: bool = True, direct: bool = True) -> dict:
    """Copy every slot of the slab into `targets`: {layer prefix: {piece: flat uint8 tensor
    holding the stacked weights}} (CPU or CUDA; the slots of a layer are laid out back to
    back in each piece tensor, in slot order).  Returns read statistics."""
    from .. import _rt
    hdr = read_header(path)
    base = hdr["data_start"]
    slots = []   # (file offset, bytes, digest, prefix, pieces, index within layer)
    for L in hdr["layers"]:
        if L["prefix"] not in targets:
            continue
        for j, s in enumerate(L["slots"]):
            slots.append((base + s["offset"], s["bytes"], s["digest"] if verify else "", L["prefix"], s["pieces"], j))
    # running destination offsets: slot j of a layer lands after slots 0..j-1 of that layer
    dst_off = {}
    for _, _, _, pre, pcs, j in slots:
        for k, (_, n) in pcs.items():
            dst_off.setdefault((pre, k), []).append(n)
    starts = {key: [sum(v[:i]) for i in range(len(v))] for key, v in dst_off.items()}
    for pre in targets:
        for k, tgt in targets[pre].items():
            need = sum(dst_off.get((pre, k), []))
            if need != tgt.numel():
                raise ValueError(f"{path}: {pre} {k}: slab holds {need} bytes, the engine expects {tgt.numel()}")
    # group file-contiguous slots into requests of at most ring_bytes (whole slots)
    reqs, cur = [], []
    for s in slots:
        if cur and (s[0] + s[1] - cur[0][0] > ring_bytes or s[0] != _up(cur[-1][0] + cur[-1][1])):
            reqs.append(cur)
            cur = []
        cur.append(s)
    if cur:
        reqs.append(cur)
    span = max((r[-1][0] + r[-1][1] - r[0][0] for r in reqs), default=0)
    buf_bytes = _up(max(span, 1), 4096)
    cuda_dst = any(t.is_cuda for d in targets.values() for t in d.values())
    bufs = _buffers(min(n_buf, max(1, len(reqs))), buf_bytes, pinned=cuda_dst)
    events = [None] * len(bufs)
    rd = _rt.SlabReader(path, threads, direct)
    inflight = []

    def issue(i):
        b = i % len(bufs)
        if events[b] is not None:
            events[b].synchronize()   # the device copies out of this buffer are done
        r = reqs[i]
        o0 = r[0][0]
        n = _up(r[-1][0] + r[-1][1] - o0, 4096)
        n = min(n, rd.file_size() - o0)
        checks = [(s[0] - o0, s[1], s[2]) for s in r]
        inflight.append((i, b, rd.submit(bufs[b][1].data_ptr(), o0, n, checks)))

    for i in range(min(len(bufs), len(reqs))):
        issue(i)
    nxt = len(inflight)
    while inflight:
        i, b, tk = inflight.pop(0)
        bad = rd.wait(tk)
        r = reqs[i]
        if bad >= 0:
            raise ValueError(f"{path}: slot {r[bad][3]}[{r[bad][5]}] failed its digest check")
        buf = bufs[b][1]
        o0 = r[0][0]
        for off, _, _, pre, pcs, j in r:
            for k, (rel, n) in pcs.items():
                d0 = starts[(pre, k)][j]
                src = buf[off - o0 + rel:off - o0 + rel + n]
                targets[pre][k][d0:d0 + n].copy_(src, non_blocking=cuda_dst)
        if cuda_dst:
            ev = torch.cuda.Event()
            ev.record()
            events[b] = ev
        if nxt < len(reqs):
            issue(nxt)
            nxt += 1
    if cuda_dst:
        torch.cuda.current_stream().synchronize()
    return {"bytes": int(rd.bytes_read()), "requests": len(reqs), "direct_reads": int(rd.direct_reads()),
            "slots": len(slots)}


def engine_targets(weights_by_prefix: dict) -> dict:
    """{prefix: (w13 NvFp4Weight, w2 NvFp4Weight)} -> read_slab targets (flat byte views)."""
    out = {}
    for pre, (w13, w2) in weights_by_prefix.items():
        d = {}
        for tag, w in (("w13", w13), ("w2", w2)):
            d[f"{tag}.packed"] = w.packed.view(-1).view(torch.uint8)
            d[f"{tag}.sf"] = w.sf.view(-1).view(torch.uint8)
            d[f"{tag}.g"] = w.gscale.view(-1).view(torch.uint8)
        out[pre] = d
    return out
