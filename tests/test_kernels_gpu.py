"""sm_100a kernels against plain PyTorch fp32 restatements of the same op.

Reference-test idea: engines/glm5-moe-nvfp4-2b/tests/test_kernels.cu:1-3 (CPU
math written from the model's arithmetic, not from the kernel it checks).
"""
import math

import pytest
import torch

from rocket_b200 import ops
from rocket_b200.fuel import nvfp4 as nv

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_err(a, b):
    a = a.float().cpu()
    b = b.float().cpu()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("m", [1, 5, 32, 77, 200, 300])
def test_linear_bf16(m):
    torch.manual_seed(m)
    n, k = 384, 512
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) * 0.05).bfloat16()
    out = ops.linear_bf16(x, w)
    ref = x.float() @ w.float().t()
    assert rel_err(out, ref) < 1e-2
    ops.check_errors()


def test_linear_bf16_f32_and_residual():
    torch.manual_seed(0)
    m, n, k = 40, 256, 1024
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) * 0.05).bfloat16()
    res = torch.randn(m, n, device=DEV).bfloat16()
    o32 = ops.linear_bf16(x, w, epi=ops.EPI_STORE_F32)
    ref = x.float() @ w.float().t()
    assert o32.dtype == torch.float32 and rel_err(o32, ref) < 1e-4
    o = ops.linear_bf16(x, w, epi=ops.EPI_RESIDUAL_BF16, residual=res)
    assert rel_err(o, ref + res.float()) < 1e-2


@pytest.mark.parametrize("rows,k", [(3, 256), (130, 512), (64, 5120)])
def test_quantize_nvfp4_matches_cpu_restatement(rows, k):
    torch.manual_seed(rows)
    x = (torch.randn(rows, k, device=DEV) * 3).bfloat16()
    q = ops.NvFp4Act(rows, k, DEV)
    ops.quantize_rows(x, q)
    p_ref, sf_ref, g_ref = nv.quantize_rows_nvfp4_reference(x.float().cpu())
    assert torch.equal(q.packed[:rows].cpu(), p_ref)
    sf_dev = nv.unswizzle_sf(q.sf.cpu()[: nv.sf_swizzled_bytes(q.rows, k)], q.rows, k)[:rows]
    assert torch.equal(sf_dev, sf_ref)
    assert torch.allclose(q.row_scale[:rows].cpu(), g_ref)


def _nvfp4_weight(n, k, experts=1, seed=0, std=0.02):
    g = torch.Generator().manual_seed(seed)
    trip, deq = [], []
    for _ in range(experts):
        w = torch.randn(n, k, generator=g) * std
        p, s, gs = nv.quantize_nvfp4(w)
        trip.append((p, s, gs))
        deq.append(nv.dequantize_nvfp4(p, s, gs))
    return ops.NvFp4Weight.from_triplets(trip, DEV), deq


def _deq_act(q: ops.NvFp4Act, rows, k, sf_rows=128):
    """Dequantize the GPU's NVFP4 rows; scale atoms hold `sf_rows` rows each."""
    sf_all = q.sf.cpu().long()
    kt = k // 64
    r = torch.arange(rows).view(-1, 1)
    s = torch.arange(k // 16).view(1, -1)
    rr = r % sf_rows
    off = ((r // sf_rows) * kt + s // 4) * 512 + (rr % 32) * 16 + (rr // 32) * 4 + s % 4
    sf = sf_all[off].to(torch.uint8)
    return nv.dequantize_nvfp4(q.packed[:rows].cpu(), sf, 1.0) * q.row_scale[:rows].cpu().unsqueeze(1)


@pytest.mark.parametrize("m", [1, 17, 32, 100, 256, 300])
def test_linear_nvfp4(m):
    torch.manual_seed(m)
    n, k = 256, 1024
    w, deq = _nvfp4_weight(n, k, seed=m)
    x = torch.randn(m, k, device=DEV).bfloat16()
    q = ops.NvFp4Act(m, k, DEV)
    ops.quantize_rows(x, q)
    out = ops.linear_nvfp4(q, m, w, epi=ops.EPI_STORE_F32)
    ref = _deq_act(q, m, k) @ deq[0].t()
    assert rel_err(out, ref) < 1e-4
    ops.check_errors()


def test_linear_nvfp4_swiglu():
    torch.manual_seed(3)
    m, inter, k = 20, 128, 512
    w, deq = _nvfp4_weight(2 * inter, k, seed=3)
    x = torch.randn(m, k, device=DEV).bfloat16()
    q = ops.NvFp4Act(m, k, DEV)
    ops.quantize_rows(x, q)
    h = ops.linear_nvfp4(q, m, w, epi=ops.EPI_SWIGLU)
    acc = _deq_act(q, m, k) @ deq[0].t()          # [m, 256]: tile rows [64 gate | 64 up] x 2
    acc = acc.view(m, 2, 2, 64)
    ref = (torch.nn.functional.silu(acc[:, :, 0]) * acc[:, :, 1]).reshape(m, 128)
    assert h.shape == (m, 128) and rel_err(h, ref) < 1e-2


def test_grouped_moe_pipeline():
    """router top-k -> plan -> dispatch quantize -> grouped GEMM -> combine."""
    torch.manual_seed(7)
    T, E, K, topk, d, inter = 50, 16, 4, 4, 512, 256
    w13, deq13 = _nvfp4_weight(2 * inter, d, experts=E + 1, seed=1)
    w2, deq2 = _nvfp4_weight(d, inter, experts=E + 1, seed=2)
    x = torch.randn(T, d, device=DEV).bfloat16()
    logits = torch.randn(T, E, device=DEV)
    bn = 32
    plan = ops.MoePlan(T, topk + 1, E + 1, bn, DEV)
    ops.router_topk(logits, E, topk, 1, False, True, 1.0, None, -1, plan, T)
    ops.moe_plan(plan)
    xq = ops.NvFp4Act(plan.max_rows, d, DEV)
    ops.moe_dispatch_quantize(x, T, plan, xq)
    h = torch.zeros(plan.max_rows, inter, dtype=torch.bfloat16, device=DEV)
    ops.grouped_nvfp4(xq, w13, h, ops.EPI_SWIGLU, plan, bn)
    hq = ops.NvFp4Act(plan.max_rows, inter, DEV)
    ops.quantize_assigned(h, T, plan, hq)
    y = torch.zeros(plan.max_rows, d, dtype=torch.bfloat16, device=DEV)
    ops.grouped_nvfp4(hq, w2, y, ops.EPI_STORE_BF16, plan, bn)
    out = torch.empty(T, d, dtype=torch.bfloat16, device=DEV)
    ops.moe_combine(y, plan, T, x, out)
    torch.cuda.synchronize()
    ops.check_errors()

    # reference: same routing, dequantized weights, the GPU's own quantized activations
    ids = plan.ids[:T].cpu()
    wts = plan.weights[:T].cpu()
    p = torch.softmax(logits.cpu(), -1)
    top = torch.topk(p, topk, -1)
    assert torch.equal(ids[:, :topk].sort(-1).values, top.indices.int().sort(-1).values)
    assert torch.allclose(wts[:, :topk].sum(-1), torch.ones(T), atol=1e-5)
    pos = plan.pos[:T * (topk + 1)].cpu().view(T, topk + 1)
    xdq = _deq_act(xq, plan.max_rows, d, plan.sf_rows)
    ref = x.float().cpu().clone()
    for t in range(T):
        for j in range(topk + 1):
            e = int(ids[t, j])
            r = int(pos[t, j])
            a = xdq[r] @ deq13[e].t()
            a = a.view(-1, 2, 64)
            hh = (torch.nn.functional.silu(a[:, 0]) * a[:, 1]).reshape(inter)
            hh = hh.bfloat16().float()
            hp, hs, hg = nv.quantize_rows_nvfp4_reference(hh.unsqueeze(0))
            hd = nv.dequantize_nvfp4(hp, hs, 1.0) * hg.unsqueeze(1)
            yy = (hd @ deq2[e].t())[0]
            ref[t] += float(wts[t, j]) * yy.bfloat16().float()
    assert rel_err(out, ref) < 2e-2


@pytest.mark.parametrize("sigmoid", [False, True])
def test_router_topk(sigmoid):
    torch.manual_seed(11)
    T, E, k = 33, 160, 8
    logits = torch.randn(T, 256, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1
    plan = ops.MoePlan(T, k, E, 32, DEV)
    ops.router_topk(logits, E, k, 0, sigmoid, True, 2.5, bias if sigmoid else None, -1, plan, T)
    l = logits[:, :E].cpu()
    if sigmoid:
        s = torch.sigmoid(l)
        sel = torch.topk(s + bias.cpu(), k, -1).indices
        w = torch.gather(s, 1, sel)
    else:
        s = torch.softmax(l, -1)
        sel = torch.topk(s, k, -1).indices
        w = torch.gather(s, 1, sel)
    w = w / w.sum(-1, keepdim=True) * 2.5
    assert torch.equal(plan.ids[:T].cpu().long(), sel)
    assert torch.allclose(plan.weights[:T].cpu(), w, atol=1e-5)
    counts = torch.bincount(sel.flatten(), minlength=E)
    assert torch.equal(plan.counts.cpu().long(), counts)


def test_rmsnorm():
    torch.manual_seed(0)
    x = torch.randn(37, 5120, device=DEV).bfloat16()
    w = torch.randn(5120, device=DEV).bfloat16()
    out = ops.rmsnorm(x, w, 1e-6)
    xf = x.float()
    ref = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert rel_err(out, ref) < 1e-2


def _ref_attention(q, k, v, causal_offset, scale):
    # q [Tq, H, D]; k, v [Tk, Hkv, D]
    Tq, H, D = q.shape
    Hkv = k.shape[1]
    G = H // Hkv
    kk = k.repeat_interleave(G, 1).float()
    vv = v.repeat_interleave(G, 1).float()
    s = torch.einsum("qhd,khd->hqk", q.float(), kk) * scale
    qi = torch.arange(Tq).unsqueeze(1) + causal_offset
    ki = torch.arange(k.shape[0]).unsqueeze(0)
    s = s.masked_fill(ki > qi, float("-inf"))
    p = torch.softmax(s, -1)
    return torch.einsum("hqk,khd->qhd", p, vv)


def _kv_store(x, kv, scale):
    """What a cache of dtype `kv` holds for values x, and what it decodes back to."""
    if kv == "fp8":
        q = (x.float() / scale).to(torch.float8_e4m3fn)
        return q, q.float() * scale
    return x, x.float()


@pytest.mark.parametrize("D,Hq,Hkv", [(128, 12, 1), (128, 96, 8), (64, 8, 2), (256, 16, 2)])
@pytest.mark.parametrize("splits", [1, 3])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
@pytest.mark.parametrize("block_n", [0, 128])
def test_paged_attention_prefill_and_decode(D, Hq, Hkv, splits, kv, block_n):
    if kv == "fp8" and D > 128:
        pytest.skip("fp8 KV supports head_dim <= 128")
    if block_n and (D != 128 or kv != "bf16"):
        pytest.skip("the key-block choice applies to bf16 head_dim 128")
    torch.manual_seed(D + Hq)
    page = 64
    ks_, vs_ = (0.5, 2.0) if kv == "fp8" else (1.0, 1.0)
    kd = torch.float8_e4m3fn if kv == "fp8" else torch.bfloat16
    # two sequences: one chunked-prefill (prefix 100 + 70 new), one decode (300 ctx + 1 new)
    seqs = [(100, 70), (300, 1)]
    num_pages = 32
    kc = torch.zeros(num_pages, Hkv, page, D, dtype=kd, device=DEV)
    vc = torch.zeros(num_pages, Hkv, D, page, dtype=kd, device=DEV)
    perm = torch.randperm(num_pages).tolist()
    max_pages = 8
    bt = torch.zeros(len(seqs), max_pages, dtype=torch.int32)
    qs, ks, vs = [], [], []
    q_start, q_len, kv_len = [], [], []
    t0 = 0
    for si, (prefix, new) in enumerate(seqs):
        L = prefix + new
        k, k_ref = _kv_store(torch.randn(L, Hkv, D).bfloat16(), kv, ks_)
        v, v_ref = _kv_store(torch.randn(L, Hkv, D).bfloat16(), kv, vs_)
        q = torch.randn(new, Hq, D).bfloat16()
        npg = (L + page - 1) // page
        for pi in range(npg):
            pg = perm.pop()
            bt[si, pi] = pg
            lo, hi = pi * page, min(L, (pi + 1) * page)
            kc[pg, :, : hi - lo] = k[lo:hi].transpose(0, 1).to(DEV)
            vc[pg, :, :, : hi - lo] = v[lo:hi].permute(1, 2, 0).to(DEV)
        qs.append(q)
        ks.append(k_ref)
        vs.append(v_ref)
        q_start.append(t0)
        q_len.append(new)
        kv_len.append(L)
        t0 += new
    q_all = torch.cat(qs).to(DEV)
    out = torch.zeros_like(q_all)
    w_seq, w_tok0 = ops.attention_work(q_len, Hq, Hkv)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    T = q_all.shape[0]
    ws_o = torch.empty(splits, T * Hq, D, device=DEV) if splits > 1 else None
    ws_ml = torch.empty(splits, T * Hq, 2, device=DEV) if splits > 1 else None
    ops.attention(q_all, out, kc, vc, Hq, Hkv, D, bt.to(DEV), i32(q_start), i32(q_len), i32(kv_len), i32(w_seq),
                  i32(w_tok0), i32([len(w_seq)]), len(w_seq), num_splits=splits, ws_o=ws_o, ws_ml=ws_ml,
                  k_scale=ks_, v_scale=vs_, block_n=block_n)
    torch.cuda.synchronize()
    ops.check_errors()
    scale = 1.0 / math.sqrt(D)
    for si, (prefix, new) in enumerate(seqs):
        ref = _ref_attention(qs[si], ks[si], vs[si], prefix, scale)
        got = out[q_start[si]:q_start[si] + new].cpu()
        assert rel_err(got, ref) < 2e-2, (si, rel_err(got, ref))


@pytest.mark.parametrize("kv", ["bf16", "fp8"])
@pytest.mark.parametrize("T", [7, 300])
def test_qk_rope_kv_write(kv, T):
    """Per-token path (decode-sized) and the prefill path whose V rows go through the
    tile transpose kernel (300 tokens over shuffled pages, some rows not written)."""
    torch.manual_seed(5)
    Hq, Hkv, D, page = 8, 2, 128, 64
    rot = 64
    kd = torch.float8_e4m3fn if kv == "fp8" else torch.bfloat16
    ks_, vs_ = (0.5, 0.25) if kv == "fp8" else (1.0, 1.0)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device=DEV).bfloat16()
    inv = ops.rope_inv_freq(rot, 1e6, DEV)
    q_out = torch.empty(T, Hq, D, dtype=torch.bfloat16, device=DEV)
    if T == 7:
        pos = torch.tensor([0, 1, 2, 63, 64, 65, 500], dtype=torch.int32, device=DEV)
        slots = torch.tensor([0, 1, 2, 63, 64, 65, 200], dtype=torch.int32, device=DEV)
        n_pages = 4
    else:
        p = torch.arange(T) + 20  # a chunk that starts mid-page
        n_pages = (int(p[-1]) // page) + 2
        perm = torch.randperm(n_pages)
        sl = perm[p // page] * page + p % page
        sl[::37] = -1  # rows whose KV is not written
        pos, slots = p.int().to(DEV), sl.int().to(DEV)
    kc = torch.zeros(n_pages, Hkv, page, D, dtype=kd, device=DEV)
    vc = torch.zeros(n_pages, Hkv, D, page, dtype=kd, device=DEV)
    ops.qk_rope_kv(qkv, T, Hq, Hkv, D, rot, False, pos, inv, q_out, k_cache=kc, v_cache=vc, slot_mapping=slots,
                   page_size=page, k_scale=ks_, v_scale=vs_)
    tol = 7e-2 if kv == "fp8" else 1e-2  # e4m3 keeps 3 mantissa bits
    x = qkv.float().cpu()
    q = x[:, : Hq * D].view(T, Hq, D)
    k = x[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = x[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    ang = pos.cpu().float().unsqueeze(1) * inv.cpu().unsqueeze(0)  # [T, rot/2]
    cos, sin = torch.cos(ang).unsqueeze(1), torch.sin(ang).unsqueeze(1)

    def rope(t):
        a, b = t[..., : rot // 2], t[..., rot // 2: rot]
        return torch.cat([a * cos - b * sin, b * cos + a * sin, t[..., rot:]], -1)

    assert rel_err(q_out.cpu(), rope(q)) < 1e-2
    kr = rope(k)
    kcc, vcc = kc.float().cpu(), vc.float().cpu()
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        assert rel_err(kcc[s // page, :, s % page] * ks_, kr[t]) < tol
        assert rel_err(vcc[s // page, :, :, s % page] * vs_, v[t]) < tol


def test_lm_head_argmax():
    torch.manual_seed(9)
    m, V, k = 19, 1000, 512
    Vp = 1024
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = torch.zeros(Vp, k, device=DEV).bfloat16()
    w[:V] = (torch.randn(V, k, device=DEV) * 0.05).bfloat16()
    keys = torch.zeros(m, dtype=torch.int64, device=DEV)
    ids = torch.empty(m, dtype=torch.int32, device=DEV)
    ops.lm_head_argmax(x, w, keys, ids, V)
    ref = (x.float() @ w[:V].float().t()).argmax(-1)
    # allow near-ties to differ, values must agree
    logits = x.float() @ w[:V].float().t()
    got_v = logits.gather(1, ids.long().unsqueeze(1)).squeeze(1)
    ref_v = logits.gather(1, ref.unsqueeze(1)).squeeze(1)
    assert torch.allclose(got_v, ref_v, atol=1e-2)
    assert int(keys.abs().sum()) == 0  # finalize resets the keys


@pytest.mark.parametrize("Hq,Hkv", [(12, 1), (96, 8), (16, 2), (8, 2)])
@pytest.mark.parametrize("splits", [1, 2, 5])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_paged_attention_decode_kernel(Hq, Hkv, splits, kv):
    """Pure decode batch (q_len == 1): the keys-on-M decode kernel."""
    torch.manual_seed(Hq * 7 + splits)
    D, page = 128, 64
    ks_, vs_ = (0.25, 1.5) if kv == "fp8" else (1.0, 1.0)
    kd = torch.float8_e4m3fn if kv == "fp8" else torch.bfloat16
    ctxs = [1, 63, 64, 65, 300, 1000]
    num_pages = sum((c + page - 1) // page for c in ctxs) + 1
    kc = torch.zeros(num_pages, Hkv, page, D, dtype=kd, device=DEV)
    vc = torch.zeros(num_pages, Hkv, D, page, dtype=kd, device=DEV)
    max_pages = 16
    bt = torch.zeros(len(ctxs), max_pages, dtype=torch.int32)
    nxt = 0
    qs, ks, vs = [], [], []
    for si, L in enumerate(ctxs):
        k, k_ref = _kv_store(torch.randn(L, Hkv, D).bfloat16(), kv, ks_)
        v, v_ref = _kv_store(torch.randn(L, Hkv, D).bfloat16(), kv, vs_)
        for pi in range((L + page - 1) // page):
            bt[si, pi] = nxt
            lo, hi = pi * page, min(L, (pi + 1) * page)
            kc[nxt, :, : hi - lo] = k[lo:hi].transpose(0, 1).to(DEV)
            vc[nxt, :, :, : hi - lo] = v[lo:hi].permute(1, 2, 0).to(DEV)
            nxt += 1
        qs.append(torch.randn(1, Hq, D).bfloat16())
        ks.append(k_ref)
        vs.append(v_ref)
    q_all = torch.cat(qs).to(DEV)
    out = torch.zeros_like(q_all)
    S = len(ctxs)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    ws_o = torch.empty(splits, S * Hq, D, device=DEV) if splits > 1 else None
    ws_ml = torch.empty(splits, S * Hq, 2, device=DEV) if splits > 1 else None
    ops.attention(q_all, out, kc, vc, Hq, Hkv, D, bt.to(DEV), i32(list(range(S))), i32([1] * S), i32(ctxs),
                  i32(list(range(S))), i32([0] * S), i32([S]), S, num_splits=splits, ws_o=ws_o, ws_ml=ws_ml,
                  decode=True, k_scale=ks_, v_scale=vs_)
    torch.cuda.synchronize()
    ops.check_errors()
    # fp8: the decode kernel also rounds the query rows and P to e4m3 (fp8 MMAs)
    tol = 5e-2 if kv == "fp8" else 2e-2
    for si, L in enumerate(ctxs):
        ref = _ref_attention(qs[si], ks[si], vs[si], L - 1, 1.0 / math.sqrt(D))
        assert rel_err(out[si:si + 1].cpu(), ref) < tol, (si, rel_err(out[si:si + 1].cpu(), ref))


@pytest.mark.parametrize("splits", [1, 2])
@pytest.mark.parametrize("kv", ["bf16", "fp8"])
def test_paged_attention_decode_many_items_and_max_jumps(splits, kv):
    """64 sequences x 8 kv heads (several work items per persistent CTA, so the next
    item's Q is staged while the current one drains) with mixed contexts, and keys whose
    scores jump far past the running max mid-sequence (the O rescale path)."""
    torch.manual_seed(4242 + splits)
    D, page, Hq, Hkv = 128, 64, 96, 8
    ks_, vs_ = (0.25, 1.5) if kv == "fp8" else (1.0, 1.0)
    kd = torch.float8_e4m3fn if kv == "fp8" else torch.bfloat16
    g = torch.Generator().manual_seed(7)
    ctxs = torch.randint(1, 700, (64,), generator=g).tolist()
    num_pages = sum((c + page - 1) // page for c in ctxs) + 1
    kc = torch.zeros(num_pages, Hkv, page, D, dtype=kd, device=DEV)
    vc = torch.zeros(num_pages, Hkv, D, page, dtype=kd, device=DEV)
    max_pages = 16
    bt = torch.zeros(len(ctxs), max_pages, dtype=torch.int32)
    nxt = 0
    qs, ks, vs = [], [], []
    for si, L in enumerate(ctxs):
        k = torch.randn(L, Hkv, D)
        if L > 300 and si % 2 == 0:
            k[260:300] *= 6.0  # scores jump by far more than 2^8 in the third key block
        k, k_ref = _kv_store((k * (0.5 if kv == "fp8" else 1.0)).bfloat16(), kv, ks_)
        v, v_ref = _kv_store(torch.randn(L, Hkv, D).bfloat16(), kv, vs_)
        for pi in range((L + page - 1) // page):
            bt[si, pi] = nxt
            lo, hi = pi * page, min(L, (pi + 1) * page)
            kc[nxt, :, : hi - lo] = k[lo:hi].transpose(0, 1).to(DEV)
            vc[nxt, :, :, : hi - lo] = v[lo:hi].permute(1, 2, 0).to(DEV)
            nxt += 1
        qs.append(torch.randn(1, Hq, D).bfloat16())
        ks.append(k_ref)
        vs.append(v_ref)
    q_all = torch.cat(qs).to(DEV)
    out = torch.zeros_like(q_all)
    S = len(ctxs)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    ws_o = torch.empty(splits, S * Hq, D, device=DEV) if splits > 1 else None
    ws_ml = torch.empty(splits, S * Hq, 2, device=DEV) if splits > 1 else None
    for _ in range(2):  # run twice: the same bits (no state carried between launches)
        ops.attention(q_all, out, kc, vc, Hq, Hkv, D, bt.to(DEV), i32(list(range(S))), i32([1] * S), i32(ctxs),
                      i32(list(range(S))), i32([0] * S), i32([S]), S, num_splits=splits, ws_o=ws_o, ws_ml=ws_ml,
                      decode=True, k_scale=ks_, v_scale=vs_)
        torch.cuda.synchronize()
        first = out.clone() if _ == 0 else first
    ops.check_errors()
    assert torch.equal(first, out)
    # fp8: Q and P are e4m3 in the decode MMAs; with the boosted keys P is peaked, so its
    # 3-bit mantissa rounding shows (bf16 stays at the usual bound)
    tol = 8e-2 if kv == "fp8" else 2e-2
    for si, L in enumerate(ctxs):
        ref = _ref_attention(qs[si], ks[si], vs[si], L - 1, 1.0 / math.sqrt(D))
        assert rel_err(out[si:si + 1].cpu(), ref) < tol, (si, L, rel_err(out[si:si + 1].cpu(), ref))


@pytest.mark.parametrize("m,n,k,splits", [(64, 5120, 12288, 8), (7, 256, 5120, 16), (200, 384, 2048, 3)])
def test_linear_bf16_split_k(m, n, k, splits):
    torch.manual_seed(m + splits)
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) * 0.02).bfloat16()
    res = torch.randn(m, n, device=DEV).bfloat16()
    out = ops.linear_bf16(x, w, epi=ops.EPI_RESIDUAL_BF16, residual=res, splits=splits)
    ref = x.float() @ w.float().t() + res.float()
    assert rel_err(out, ref) < 1e-2
    o32 = ops.linear_bf16(x, w, epi=ops.EPI_STORE_F32, splits=splits)
    assert rel_err(o32, x.float() @ w.float().t()) < 1e-4
    # deterministic: same bits twice
    o32b = ops.linear_bf16(x, w, epi=ops.EPI_STORE_F32, splits=splits)
    assert torch.equal(o32, o32b)


def test_grouped_persistent_many_units():
    """More work units than SMs: every CTA loops over several units (both TMEM accumulators)."""
    torch.manual_seed(21)
    m, n, k = 40, 128 * 160, 512
    w, deq = _nvfp4_weight(n, k, seed=21)
    x = torch.randn(m, k, device=DEV).bfloat16()
    q = ops.NvFp4Act(m, k, DEV)
    ops.quantize_rows(x, q)
    out = ops.linear_nvfp4(q, m, w, epi=ops.EPI_STORE_F32, splits=1)
    ref = _deq_act(q, m, k) @ deq[0].t()
    assert rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("hc,T,d", [(4, 7, 512), (4, 33, 5120), (2, 5, 1024)])
def test_hyper_connection_kernels(hc, T, d):
    """mHC split (coefficients, Sinkhorn, collapse), combine, expand and mean against the
    CPU oracle's fp32 math (models/reference.py hc_pre / hc_post)."""
    from rocket_b200.config import ModelConfig
    from rocket_b200.models.reference import ReferenceModel
    torch.manual_seed(hc * 100 + T)
    nm = 2 * hc + hc * hc
    S = torch.randn(T, hc, d, device=DEV).bfloat16()
    fn = (torch.randn(nm, hc * d) * 0.02).bfloat16()
    base = torch.randn(nm) * 0.5
    scale = torch.tensor([1.0, 0.7, 1.3])
    cfg = ModelConfig(hc_streams=hc, hc_sinkhorn_iters=20, hc_eps=1e-6, norm_eps=1e-6)
    ref = ReferenceModel(cfg, {"s.fn": fn, "s.base": base, "s.scale": scale})
    xr, post_r, cm_r = ref.hc_pre("s", S.float().cpu())
    fnp = torch.zeros(128, hc * d, dtype=torch.bfloat16)
    fnp[:nm] = fn
    mix = ops.linear_bf16(S.view(T, -1), fnp.to(DEV), epi=ops.EPI_STORE_F32)
    coef = torch.empty(T, hc + hc * hc, device=DEV)
    x = torch.empty(T, d, device=DEV, dtype=torch.bfloat16)
    ops.hc_split(hc, S, mix, base.to(DEV), scale.to(DEV), coef, x, T, 1e-6, 1e-6, 20)
    assert rel_err(coef[:, :hc], post_r) < 1e-4
    assert rel_err(coef[:, hc:].view(T, hc, hc), cm_r) < 1e-3
    assert rel_err(x, xr) < 1e-2
    y = torch.randn(T, d, device=DEV).bfloat16()
    out_r = ref.hc_post(S.float().cpu(), y.float().cpu(), coef[:, :hc].cpu(), coef[:, hc:].view(T, hc, hc).cpu())
    S2 = S.clone()
    ops.hc_combine(hc, S2, y, coef, T)
    assert rel_err(S2, out_r) < 1e-2
    xm = torch.empty(T, d, device=DEV, dtype=torch.bfloat16)
    ops.hc_mean(hc, S2, xm, T)
    assert rel_err(xm, S2.float().mean(1)) < 1e-2
    S3 = torch.empty_like(S)
    ops.hc_expand(hc, S3, xm, T)
    assert torch.equal(S3, xm.unsqueeze(1).expand(T, hc, d))


def test_device_stamp_and_bandwidth_kernels():
    """%globaltimer stamps bracket a kernel; the bandwidth kernels move the right bytes."""
    st = torch.zeros(2, dtype=torch.int64, device=DEV)
    ops.ext().device_stamp(st, 0)
    torch.cuda._sleep(2_000_000)
    ops.ext().device_stamp(st, 1)
    torch.cuda.synchronize()
    assert st[1] > st[0] > 0
    n = 8 << 20
    b = torch.randint(0, 255, (n,), dtype=torch.uint8, device=DEV)
    a = torch.empty_like(b)
    ops.ext().mem_bw(0, a, b, None, None, n)
    assert torch.equal(a, b)
    x = torch.randn(n // 4, device=DEV)
    y = torch.randn(n // 4, device=DEV)
    z = torch.empty_like(x)
    ops.ext().mem_bw(2, z, x, y, None, n)
    assert torch.allclose(z, x + 3 * y, rtol=1e-5, atol=1e-5)  # the kernel fuses x + 3y into one FMA
    rows = n // 64
    idx = torch.randint(0, rows, (rows,), dtype=torch.int32, device=DEV)
    g = torch.empty_like(b)
    ops.ext().mem_bw(3, g, b, None, idx, n)
    assert torch.equal(g.view(rows, 64), b.view(rows, 64)[idx.long()])
    from rocket_b200 import hwbench
    r = hwbench.bandwidth("copy", 256 << 20, iters=3)
    assert r["gb_s"] > 100


@pytest.mark.parametrize("m,k", [(1, 512), (37, 1024), (200, 4096)])
def test_linear_fp8_rows(m, k):
    """e4m3 x e4m3 tcgen05 GEMM with per-weight-row and per-token scales against fp32 math
    on the dequantized operands (the per-token activation quantizer included)."""
    torch.manual_seed(m + k)
    n = 384
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = torch.randn(n, k, device=DEV) * 0.05
    wq = ops.Fp8Weight.quantize(w)
    xq = ops.Fp8Act(m, k, DEV)
    ops.quantize_rows_fp8(x, xq, m)
    amax = x.float().abs().amax(1)
    assert torch.allclose(xq.row_scale, amax / 448, rtol=1e-6)
    xd = xq.q.float() * xq.row_scale.unsqueeze(1)
    assert rel_err(xd, x) < 0.05
    ref = xd @ wq.dequant().t()
    out = ops.linear_fp8(xq, m, wq)
    assert rel_err(out, ref) < 1e-2
    res = torch.randn(m, n, device=DEV).bfloat16()
    out2 = ops.linear_fp8(xq, m, wq, out=torch.empty(m, n, dtype=torch.bfloat16, device=DEV),
                          epi=ops.EPI_RESIDUAL_BF16, residual=res)
    assert rel_err(out2, ref + res.float()) < 1e-2


@pytest.mark.parametrize("T,E,k,sig,bn", [(64, 160, 8, True, 32), (7, 16, 2, False, 32), (300, 160, 8, True, 128),
                                          (1024, 512, 10, False, 128), (2048, 160, 8, True, 128)])
def test_route_and_plan_equals_router_then_plan(T, E, k, sig, bn):
    """The one-launch router + plan (many routing CTAs, the last one plans) gives the ids,
    weights, segment offsets and block list of router_topk followed by moe_plan
    (expert-parallel slice and shared expert included), and again on a second launch (its
    counts and CTA ticket are left cleared)."""
    torch.manual_seed(T + E)
    logits = torch.randn(T, E + 1, device=DEV)
    bias = torch.randn(E, device=DEV) * 0.1 if sig else None
    e_lo, e_hi = E // 4, E // 2  # this rank's experts
    E_tot = (e_hi - e_lo) + 1
    outs = []
    for fused in (False, True, True):
        plan = ops.MoePlan(T, k + 1, E_tot, bn, DEV) if len(outs) < 2 else plan
        args = (logits, E, k, 1, sig, True, 2.5, bias, E, plan, T)
        if fused:
            ops.route_and_plan(*args, e_lo=e_lo, e_hi=e_hi, shared_local=True)
        else:
            ops.router_topk(*args, e_lo=e_lo, e_hi=e_hi, shared_local=True)
            ops.moe_plan(plan)
        torch.cuda.synchronize()
        nb = int(plan.num_blocks.item())
        outs.append((plan.ids[:T].cpu(), plan.weights[:T].cpu(), plan.offsets.cpu(), plan.cursor.cpu(),
                     plan.blk_expert[:nb].cpu(), plan.blk_row[:nb].cpu(), plan.blk_valid[:nb].cpu(),
                     int(plan.total_rows.item()), int(plan.counts.abs().sum().item())))
    ops.check_errors()
    for b in outs[1:]:
        a = outs[0]
        for x, y in zip(a[:7], b[:7]):
            assert torch.equal(x, y)
        assert a[7] == b[7] and a[8] == 0 and b[8] == 0  # counts left at zero for the next router launch


@pytest.mark.parametrize("splits", [1, 4])
@pytest.mark.parametrize("zc", [False, True])
def test_residual_gemm_with_next_norm_equals_gemm_then_norm(splits, zc):
    """A residual GEMM that also writes the next RMSNorm (folded into the split-K reduce, or
    a second launch when K is not split) gives exactly the GEMM's rows and rmsnorm's output."""
    torch.manual_seed(11 + splits)
    m, n, k = 37, 5120, 1024
    x = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) * 0.03).bfloat16()
    res = torch.randn(m, n, device=DEV).bfloat16()
    nw = (torch.randn(n, device=DEV) * 0.1 + (0.0 if zc else 1.0)).bfloat16()
    ref = ops.linear_bf16(x, w, out=res.clone(), epi=ops.EPI_RESIDUAL_BF16, residual=res.clone(), splits=splits)
    ref_n = ops.rmsnorm(ref, nw, 1e-6, zc)
    out = res.clone()
    xn = torch.zeros(m, n, dtype=torch.bfloat16, device=DEV)
    ops.linear_bf16(x, w, out=out, epi=ops.EPI_RESIDUAL_BF16, residual=out, splits=splits,
                    fused=ops.norm_args(nw, xn, 1e-6, zc))
    torch.cuda.synchronize()
    ops.check_errors()
    assert torch.equal(out, ref)
    assert torch.equal(xn, ref_n)


def test_moe_combine_with_next_norm_equals_combine_then_norm():
    """moe_combine with the next sub-layer's norm: the same combined rows as moe_combine and
    the same normed rows as rmsnorm of them, bit for bit."""
    torch.manual_seed(5)
    T, E, topk, d = 45, 16, 4, 5120
    plan = ops.MoePlan(T, topk + 1, E + 1, 32, DEV)
    logits = torch.randn(T, E, device=DEV)
    ops.router_topk(logits, E, topk, 1, False, True, 1.0, None, -1, plan, T)
    ops.moe_plan(plan)
    x = torch.randn(T, d, device=DEV).bfloat16()
    xq = ops.NvFp4Act(plan.max_rows, d, DEV)
    ops.moe_dispatch_quantize(x, T, plan, xq)  # fills plan.pos
    y = torch.randn(plan.max_rows, d, device=DEV).bfloat16()
    nw = (torch.randn(d, device=DEV) * 0.1 + 1.0).bfloat16()
    ref = ops.moe_combine(y, plan, T, x, torch.empty(T, d, dtype=torch.bfloat16, device=DEV))
    ref_n = ops.rmsnorm(ref, nw, 1e-6)
    out = torch.empty(T, d, dtype=torch.bfloat16, device=DEV)
    xn = torch.zeros(T, d, dtype=torch.bfloat16, device=DEV)
    ops.moe_combine(y, plan, T, x, out, norm=(nw, xn, 1e-6, False))
    torch.cuda.synchronize()
    ops.check_errors()
    assert torch.equal(out, ref)
    assert torch.equal(xn, ref_n)


@pytest.mark.parametrize("kda,Hk,Hv", [(True, 4, 4), (False, 2, 4), (False, 4, 4)])
def test_deltanet_one_token_kernel_equals_scan_then_norm(kda, Hk, Hv):
    """A decode step (one token per sequence) through the fused one-token scan + gated-norm
    kernel: output, recurrent state and conv state bit-equal to the scan and norm launches,
    and the state / output equal to an fp32 restatement of the delta rule on the prep
    kernel's q, k, v and gates.  Sequences 0 and 3 start fresh (position 0)."""
    torch.manual_seed(11)
    S, D, K = 6, 128, 4
    C = 2 * Hk * D + Hv * D
    rows = C + Hv * D + 2 * Hv + (Hv * D - Hv if kda else 0)
    f32 = dict(dtype=torch.float32, device=DEV)
    i32 = lambda a: torch.tensor(a, dtype=torch.int32, device=DEV)
    proj = torch.randn(S, rows, device=DEV).bfloat16()
    conv_w = (torch.randn(C, K, device=DEV) * 0.5).bfloat16()
    conv_state0 = torch.randn(S + 1, K - 1, C, device=DEV).bfloat16()
    state0 = torch.randn(S + 1, Hv, D, D, **f32) * 0.05
    A_log, dt_bias = torch.randn(Hv, **f32) * 0.3, torch.randn(Hv * (D if kda else 1), **f32) * 0.3
    norm_w = (torch.randn(D, device=DEV) * 0.1 + 1.0).bfloat16()
    slots = [4, 0, 2, 5, 1, 3]
    pos = [0, 17, 1, 0, 40, 3]

    def run(one_token):
        bufs = dict(q=torch.zeros(S, Hk, D, **f32), k=torch.zeros(S, Hk, D, **f32), v=torch.zeros(S, Hv, D, **f32),
                    beta=torch.zeros(S, Hv, **f32), g=torch.zeros(S, Hv * (D if kda else 1), **f32))
        cs, st = conv_state0.clone(), state0.clone()
        out = torch.zeros(S, Hv * D, dtype=torch.bfloat16, device=DEV)
        o_raw = torch.zeros(S, Hv, D, **f32)
        ops.ext().gdn(proj, conv_w, cs, A_log, dt_bias, norm_w, bufs["q"], bufs["k"], bufs["v"], bufs["beta"],
                      bufs["g"], st, out, i32(pos), i32(list(range(S))), i32([1] * S), i32(slots), Hk, Hv, K, C,
                      1e-6, S, S, 0, None, None, None, None, None, int(kda), -5.0, int(kda), o_raw, one_token)
        torch.cuda.synchronize()
        ops.check_errors()
        return out, st, cs, bufs

    out1, st1, cs1, b = run(1)
    out0, st0, cs0, b0 = run(0)
    for name in b:
        assert torch.equal(b[name], b0[name]), name
    assert torch.equal(out1, out0)
    assert torch.equal(st1, st0)
    assert torch.equal(cs1, cs0)
    # fp32 restatement of the one-token delta rule + gated RMSNorm on the prep outputs
    ref_out = torch.empty(S, Hv, D, **f32)
    for s in range(S):
        for h in range(Hv):
            hk = h // (Hv // Hk)
            St = torch.zeros(D, D, **f32) if pos[s] == 0 else state0[slots[s], h].clone()  # [j][i]
            kk, qq, vv = b["k"][s, hk], b["q"][s, hk], b["v"][s, h]
            dec = b["g"][s].view(Hv, -1)[h].exp()
            Sd = St * dec
            upd = b["beta"][s, h] * (vv - Sd @ kk)
            Sn = Sd + upd[:, None] * kk[None, :]
            assert torch.allclose(st1[slots[s], h], Sn, rtol=1e-4, atol=1e-5)
            o = Sn @ qq
            z = proj[s, C + h * D:C + (h + 1) * D].float()
            gz = torch.sigmoid(z) if kda else z * torch.sigmoid(z)
            ref_out[s, h] = o * torch.rsqrt(o.pow(2).mean() + 1e-6) * norm_w.float() * gz
    assert torch.allclose(out1.float().view(S, Hv, D), ref_out, rtol=2e-2, atol=2e-2)
