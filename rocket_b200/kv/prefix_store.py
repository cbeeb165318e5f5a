"""Persistent prefix tier: KV pages of prompt prefixes on NVMe / local disk.

    tier = PrefixTier(engine, "/nvme/rkt-prefix", max_bytes=200 << 30)
    engine.attach_prefix_tier(tier)

After a prompt is prefilled its sealed (full, hashed) pages are written to the
native ``PrefixStore`` (C++: 64 KiB-aligned segments, append-only manifest,
torn-tail recovery, 256-bit checksums) keyed by the page's chained token hash
and a fingerprint of the model / shard / page geometry.  Before a new request is
admitted, the leading blocks of its prompt that the GPU index lacks are read back
(checksums verified), imported into the KV manager as cached pages and copied
host -> device, so the prefix-cache hit path serves them.  Under tensor
parallelism every rank stores its own head shard and the ranks agree on the
restored block count with an all-reduce(min) first, so their KV managers stay
identical (the reference's sync_prefix_boundary,
engines/glm5-moe-nvfp4-2b/src/coding_bench_main.cu:379-404).

A corrupt record reads as a miss: the blocks from there on are recomputed.
Hybrid (DeltaNet) models keep recurrent state that pages cannot rebuild, so
they use session checkpoints instead (``engine.save_session``).

Counterpart of the reference's NVMe prefix store path
(engines/glm5-moe-nvfp4-2b/src/kv/nvme_prefix_store.h, model.cu:807-873).
"""
from __future__ import annotations

import hashlib

import torch


def fingerprint(model, extra: str = "") -> int:
    c = model.cfg
    s = (f"{c.name}|{c.num_layers}|{c.d_model}|{c.num_q_heads}|{c.num_kv_heads}|{c.head_dim}|{c.vocab_size}|"
         f"tp{model.par.tp}:{model.par.tp_rank}|page{model.page_size}|kv{model.k_cache.dtype}|"
         f"layers{model.k_cache.shape[0]}|{extra}")
    return int.from_bytes(hashlib.blake2b(s.encode(), digest_size=8).digest(), "little") & ((1 << 63) - 1)


class PrefixTier:
    def __init__(self, engine, directory: str, max_bytes: int = 64 << 30, segment_bytes: int = 256 << 20,
                 direct_io: bool = False, max_restore_blocks: int = 4096):
        from .. import _rt
        self.engine = engine
        self.store = _rt.PrefixStore(directory, max_bytes, segment_bytes, direct_io)
        m = engine.model
        caches = m.page_caches()
        self.fp = fingerprint(m, f"parts{len(caches)}")
        # one record part per page cache ([layers, pages, ...] -> the page's [layers, ...] slice)
        self.shapes = [(tuple(c.shape[:1]) + tuple(c.shape[2:]), c.dtype) for c in caches]
        self.max_restore = max_restore_blocks
        self._stage = [torch.empty(sh, dtype=dt).pin_memory() for sh, dt in self.shapes]
        self.saved = 0
        self.restored = 0

    # ------------------------------------------------------------------ save
    def save(self, rid: int):
        """Write every sealed page of sequence `rid` that the store lacks."""
        m, kv = self.engine.model, self.engine.kv
        caches = m.page_caches()
        for key, page in kv.sealed_blocks(rid):
            if self.store.contains(key, self.fp):
                continue
            for h, c in zip(self._stage, caches):
                h.copy_(c[:, page])
            if self.store.put(key, self.fp, [h.view(torch.uint8).numpy() for h in self._stage]):
                self.saved += 1

    # ------------------------------------------------------------------ restore
    def restore(self, prompt: list[int]) -> int:
        """Import the prompt's leading blocks the GPU index lacks; returns how many."""
        m, kv, par = self.engine.model, self.engine.kv, self.engine.par
        ps = m.page_size
        usable = (len(prompt) - 1) // ps  # the KV manager always leaves >= 1 token to compute
        keys = kv.block_keys(prompt[:usable * ps])[: self.max_restore]
        n0 = kv.cached_prefix_blocks(keys)
        # phase 1: how many consecutive blocks this rank can read (checksums verified)
        staged = []
        for key in keys[n0:]:
            hs = [torch.empty(sh, dtype=dt).pin_memory() for sh, dt in self.shapes]
            if not self.store.get_into(key, self.fp, [h.view(torch.uint8).numpy() for h in hs]):
                break
            staged.append((key, hs))
        n = len(staged)
        if par.world > 1:  # every rank restores the same count
            t = torch.tensor([n], dtype=torch.int64, device=m.dev)
            import torch.distributed as dist
            dist.all_reduce(t, op=dist.ReduceOp.MIN)
            n = int(t.item())
        # phase 2: import and copy host -> device
        done = 0
        caches = m.page_caches()
        for key, hs in staged[:n]:
            page = kv.import_block(key)
            if page < 0:
                break
            for h, c in zip(hs, caches):
                c[:, page].copy_(h, non_blocking=True)
            done += 1
        torch.cuda.current_stream(m.dev).synchronize()
        self.restored += done
        return done

    def stats(self) -> dict:
        d = dict(self.store.stats())
        d.update(saved_blocks=self.saved, restored_blocks=self.restored)
        return d


class SessionStore:
    """Checkpoint / resume of whole running sequences (detach a request, restore it in
    another engine or after a restart): its token history, committed KV pages (every
    attention layer, the MTP head's included), DeltaNet recurrent + conv state of its
    slot, and its pending drafts.  Records live in a PrefixStore keyed by a hash of
    the token history and the model fingerprint.

    Counterpart of the reference's kv_checkpoint / kv_open_shared / kv_detach /
    kv_resume (engines/glm5-moe-nvfp4-2b/src/model.h:155-190, model.cu:758-873) and the
    Qwen state transactions (engines/qwen38-flash-next-nvfp4-2b/src/qwen38_slab/
    state_txn.py:229).
    """

    def __init__(self, engine, directory: str, max_bytes: int = 64 << 30):
        from .. import _rt
        self.engine = engine
        self.store = _rt.PrefixStore(directory, max_bytes, 256 << 20, False)
        self.fp = fingerprint(engine.model, "session")

    @staticmethod
    def key_of(tokens: list[int]) -> int:
        import struct
        b = struct.pack(f"<{len(tokens)}i", *tokens)
        return int.from_bytes(hashlib.blake2b(b, digest_size=8).digest(), "little") & ((1 << 63) - 1)

    def _parts(self, req) -> list:
        """This rank's state of a running request as byte arrays: metadata JSON, K pages,
        V pages (+ DeltaNet recurrent and conv state of its slot)."""
        import json

        import numpy as np
        eng = self.engine
        m, kv = eng.model, eng.kv
        tokens = list(req.prompt) + list(req.output)
        n = req.computed  # tokens whose KV is committed
        pages = list(kv.pages(req.rid))[: -(-n // m.page_size)]
        idx = torch.tensor(pages, dtype=torch.long, device=m.dev)
        caches = m.page_caches()
        meta = {"prompt_len": len(req.prompt), "tokens": tokens, "computed": n, "drafts": list(req.drafts),
                "max_new_tokens": req.max_new_tokens, "stop_ids": list(req.stop_ids), "n_caches": len(caches)}
        parts = [np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)]
        parts += [c.index_select(1, idx).cpu().reshape(-1).view(torch.uint8).numpy() for c in caches]
        if eng.hybrid:
            slot = eng.slot_of[req.rid]
            b = m.dn_buf
            parts.append(b.state[:, slot].cpu().reshape(-1).view(torch.uint8).numpy())
            parts.append(b.conv_state[:, slot].cpu().reshape(-1).view(torch.uint8).numpy())
        return parts

    def save(self, req) -> int:
        """Checkpoint a running (decoding) request; returns its key."""
        parts = self._parts(req)
        key = self.key_of(list(req.prompt) + list(req.output))
        self.store.erase(key, self.fp)
        self.store.put(key, self.fp, parts)
        return key

    def save_txn(self, req, session: str, txn) -> str:
        """Collective checkpoint of `req` under tensor parallelism: every rank's shard
        commits atomically through a kv.state_txn.DistributedTxn (all ranks call)."""
        return txn.checkpoint(session, self._parts(req))

    def resume_txn(self, session: str, txn, max_new_tokens: int | None = None):
        """Collective restore of a session saved with save_txn (all ranks call)."""
        _, bufs = txn.restore(session)
        return self._install(bufs, max_new_tokens)

    def resume(self, key: int, max_new_tokens: int | None = None):
        """Re-open a checkpointed sequence in this engine; returns the Request (decoding)."""
        import numpy as np
        sizes = self.store.sizes(key, self.fp)
        if not sizes:
            raise KeyError(f"no session {key}")
        bufs = [np.empty(s, dtype=np.uint8) for s in sizes]
        if not self.store.get_into(key, self.fp, bufs):
            raise IOError(f"session {key} failed its checksum")
        return self._install(bufs, max_new_tokens)

    def _install(self, bufs, max_new_tokens):
        import json

        from ..engine.scheduler import Request, Status
        eng = self.engine
        m, kv = eng.model, eng.kv
        meta = json.loads(bufs[0].tobytes())
        tokens, n = meta["tokens"], meta["computed"]
        P = meta["prompt_len"]
        r = Request(tokens[:P], max_new_tokens or meta["max_new_tokens"], tuple(meta["stop_ids"]))
        r.output = tokens[P:]
        kv.open(r.rid, [])
        kv.append(r.rid, tokens[:n])
        pages = list(kv.pages(r.rid))
        idx = torch.tensor(pages, dtype=torch.long, device=m.dev)
        caches = m.page_caches()
        if meta.get("n_caches", 2) != len(caches):
            raise ValueError("session was saved by a model with a different cache layout")
        for j, c in enumerate(caches):
            if c.numel() == 0:  # MLA has no V cache
                continue
            shp = (c.shape[0], len(pages)) + tuple(c.shape[2:])
            c.index_copy_(1, idx, torch.from_numpy(bufs[1 + j]).view(c.dtype).view(shp).to(m.dev))
        slot = eng.free_slots.pop()
        eng.slot_of[r.rid] = slot
        if eng.hybrid:
            b = m.dn_buf
            o = 1 + len(caches)
            st = torch.from_numpy(bufs[o]).view(torch.float32).view(b.state[:, slot].shape)
            cs = torch.from_numpy(bufs[o + 1]).view(b.conv_state.dtype).view(b.conv_state[:, slot].shape)
            b.state[:, slot].copy_(st.to(m.dev))
            b.conv_state[:, slot].copy_(cs.to(m.dev))
        r.computed = n
        r.drafts = list(meta["drafts"])
        r.status = Status.DECODE
        r.t_first = r.arrival
        eng.sched.running.append(r)
        if m.dev.type == "cuda":
            torch.cuda.current_stream(m.dev).synchronize()
        return r
