"""Expert slabs: offline packing, the native O_DIRECT ring reader, digest refusal (CPU)."""
import os

import pytest
import torch

from rocket_b200.config import load_fuel
from rocket_b200.fuel import slabs
from rocket_b200.models import init_fuel_tensors
from rocket_b200.models import weights as W

rt = pytest.importorskip("rocket_b200._rt")


@pytest.fixture(scope="module")
def fuel():
    cfg = load_fuel("tiny-moe").model
    return cfg, {k: v for k, v in init_fuel_tensors(cfg, 0).items() if not k.startswith("master.")}


def _expected(cfg, t, rank, world, order):
    out = {}
    for pre in slabs.moe_prefixes(cfg, t):
        names = slabs.slot_names(cfg, pre, rank, world, order)
        w13 = W.stack_nvfp4([W.fuse_w13(W.triplet_of(t, n + ".gate_proj"), W.triplet_of(t, n + ".up_proj"))
                             for n in names], "cpu")
        w2 = W.stack_nvfp4([W.triplet_of(t, n + ".down_proj") for n in names], "cpu")
        out[pre] = (w13, w2)
    return out


def _empty(cfg, t, world):
    out = {}
    n_e = cfg.num_experts // world + cfg.num_shared_experts
    for pre in slabs.moe_prefixes(cfg, t):
        out[pre] = (W.empty_nvfp4(2 * cfg.moe_intermediate, cfg.d_model, n_e, "cpu"),
                    W.empty_nvfp4(cfg.d_model, cfg.moe_intermediate, n_e, "cpu"))
    return out


@pytest.mark.parametrize("direct,ring", [(True, 256 << 20), (False, 100 << 10)])
def test_pack_and_read_back(tmp_path, fuel, direct, ring):
    cfg, t = fuel
    world = 2
    order = list(range(cfg.num_experts))[::-1]
    paths = slabs.pack_expert_slabs(t, cfg, str(tmp_path), world, order, fuel="tiny-moe")
    assert [os.path.basename(p) for p in paths] == [slabs.slab_name(r, world) for r in range(world)]
    for r, p in enumerate(paths):
        hdr = slabs.read_header(p)
        assert hdr["rank"] == r and hdr["expert_order"] == order and hdr["data_start"] % slabs.ALIGN == 0
        for L in hdr["layers"]:
            assert all(s["offset"] % slabs.ALIGN == 0 for s in L["slots"])
        got = _empty(cfg, t, world)
        st = slabs.read_slab(p, slabs.engine_targets(got), ring_bytes=ring, direct=direct, threads=3)
        assert st["slots"] == sum(len(L["slots"]) for L in hdr["layers"])
        if ring < (1 << 20):
            assert st["requests"] > len(hdr["layers"])   # a small ring: many requests, buffers reused
        exp = _expected(cfg, t, r, world, order)
        for pre in exp:
            for a, b in zip(got[pre], exp[pre]):
                assert torch.equal(a.packed, b.packed), pre
                assert torch.equal(a.sf, b.sf), pre
                assert torch.equal(a.gscale, b.gscale), pre


def test_damaged_slot_is_refused(tmp_path, fuel):
    cfg, t = fuel
    p = slabs.pack_expert_slabs(t, cfg, str(tmp_path), 1)[0]
    hdr = slabs.read_header(p)
    s = hdr["layers"][0]["slots"][2]
    with open(p, "r+b") as f:
        f.seek(hdr["data_start"] + s["offset"] + 17)
        b = f.read(1)
        f.seek(-1, 1)
        f.write(bytes([b[0] ^ 1]))
    with pytest.raises(ValueError, match="digest"):
        slabs.read_slab(p, slabs.engine_targets(_empty(cfg, t, 1)))
    # without verification the bytes load (the damage is then the caller's choice)
    slabs.read_slab(p, slabs.engine_targets(_empty(cfg, t, 1)), verify=False)


def test_reader_tickets_and_tail(tmp_path):
    data = os.urandom(3 * 4096 + 123)
    p = str(tmp_path / "f.bin")
    with open(p, "wb") as f:
        f.write(data)
    rd = rt.SlabReader(p, 2, True)
    raw = torch.empty(5 * 4096, dtype=torch.uint8)
    a = (-raw.data_ptr()) % 4096
    buf = raw[a:a + 4 * 4096]
    tk = rd.submit(buf.data_ptr(), 0, len(data), [(0, 4096, rt.digest_hex(data[:4096])),
                                                  (4096, 100, "0" * 64)])
    assert rd.wait(tk) == 1          # the second check has a wrong digest
    assert bytes(buf[:len(data)].numpy()) == data
    with pytest.raises(Exception):
        rd.submit(buf.data_ptr(), 4096, len(data), [])   # past the end of the file
