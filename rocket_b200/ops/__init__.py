"""Python face of the sm_100a kernels.

Every function here launches a hand-written kernel from ``rocket_b200._C``.
There is no eager-PyTorch fallback: on a machine without the extension or
without an sm_100 GPU the ops raise.
"""
from __future__ import annotations

import math

import torch

from ..fuel import nvfp4 as _nv

_C = None
_IMPORT_ERROR: Exception | None = None
try:  # the extension is built in-tree by setup.py / __graft_entry__.build()
    from .. import _C as _C  # type: ignore
except Exception as e:  # pragma: no cover - exercised on machines without a build
    _IMPORT_ERROR = e

EPI_STORE_BF16 = 0
EPI_STORE_F32 = 1
EPI_SWIGLU = 2
EPI_MOE_DOWN = 3
EPI_RESIDUAL_BF16 = 4
EPI_ARGMAX = 5
EPI_REDUCE_SCATTER = 6
EPI_COMBINE_PUSH = 7
EPI_AR_PUSH = 8
EPI_COMBINE_ALL = 9


_LAUNCHES = 0


class _Counted:
    """Counts kernel launches issued through the extension (one per call)."""

    def __init__(self, mod):
        self._m = mod

    def __getattr__(self, name):
        f = getattr(self._m, name)

        def call(*a, **k):
            global _LAUNCHES
            _LAUNCHES += 1
            return f(*a, **k)
        return call


_COUNTED = None


def ext():
    global _COUNTED
    if _C is None:
        raise RuntimeError(f"rocket_b200._C is not built or failed to load: {_IMPORT_ERROR!r}; "
                           "run `python setup.py build_ext --inplace`")
    if _COUNTED is None:
        _COUNTED = _Counted(_C)
    return _COUNTED


def launch_count() -> int:
    """Kernels this process launched (or captured) through rocket_b200 ops."""
    return _LAUNCHES


def reset_launch_count():
    global _LAUNCHES
    _LAUNCHES = 0


def available() -> bool:
    return _C is not None and torch.cuda.is_available() and torch.cuda.get_device_capability() >= (10, 0)


_ERR: dict[int, torch.Tensor] = {}


def err_flag(device=None) -> torch.Tensor:
    """Per-device int32 status word the kernels OR error bits into."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _ERR:
        _ERR[idx] = torch.zeros(1, dtype=torch.int32, device=f"cuda:{idx}")
        ext().set_err_flag(_ERR[idx])
    return _ERR[idx]


def check_errors(device=None):
    e = int(err_flag(device).item())
    if e:
        raise RuntimeError(f"device kernel reported error bits 0x{e:x} (1=mbarrier timeout, 2=peer timeout, "
                           f"4=bad shape, 8=TMEM allocation, 16=index out of bounds in a debug build)")


# ----------------------------------------------------------------- weights
class NvFp4Weight:
    """NVFP4 weight prepared for the tcgen05 block-scaled GEMM.

    ``packed`` [E*N, K/2] uint8, ``sf`` scale atoms [E][N/128][K/64][512],
    ``gscale`` [E*N] fp32 tensor scale of every row (rows of a fused gate|up
    weight keep their own tensor's scale).  ``E`` experts share N and K.
    """

    def __init__(self, packed, sf, gscale, n, k, num_experts=1):
        self.packed, self.sf, self.gscale = packed, sf, gscale
        self.n, self.k, self.num_experts = n, k, num_experts

    @staticmethod
    def from_triplets(triplets, device):
        """triplets: list of (packed [N,K/2] u8, sf_linear [N,K/16] u8, global float), one per expert."""
        n = triplets[0][0].shape[0]
        k = triplets[0][0].shape[1] * 2
        packed = torch.cat([t[0] for t in triplets], 0).to(device)
        sf = torch.cat([_nv.swizzle_sf(t[1]) for t in triplets], 0).to(device)
        g = torch.tensor([t[2] for t in triplets], dtype=torch.float32).repeat_interleave(n).to(device)
        return NvFp4Weight(packed, sf, g, n, k, len(triplets))

    def nbytes(self):
        return self.packed.numel() + self.sf.numel() + self.gscale.numel() * 4


class NvFp4Act:
    """Activation rows quantized to NVFP4 (per-row tensor scale)."""

    def __init__(self, rows, k, device):
        self.k = k
        cap = ((rows + 255) // 256) * 256
        self.packed = torch.zeros(cap, k // 2, dtype=torch.uint8, device=device)
        # sized for 32-row scale atoms (the larger of the two layouts)
        self.sf = torch.zeros(cap // 32 * (k // 64) * 512, dtype=torch.uint8, device=device)
        self.row_scale = torch.zeros(cap, dtype=torch.float32, device=device)
        self.rows = cap


class Fp8Weight:
    """e4m3 weight rows [N, K] with one fp32 scale per row (w ~= q * scale[n])."""

    def __init__(self, q, scale):
        self.q, self.scale = q, scale
        self.n, self.k = q.shape

    @staticmethod
    def quantize(w: torch.Tensor, device=None) -> "Fp8Weight":
        """Per-row amax / 448 scales, round-to-nearest e4m3 (saturating)."""
        w = w.float()
        amax = w.abs().amax(dim=1)
        scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
        q = (w / scale.unsqueeze(1)).clamp(-448, 448).to(torch.float8_e4m3fn)
        dev = device if device is not None else w.device
        return Fp8Weight(q.contiguous().to(dev), scale.contiguous().to(dev))

    def dequant(self) -> torch.Tensor:
        return self.q.float() * self.scale.unsqueeze(1)

    def nbytes(self):
        return self.q.numel() + self.scale.numel() * 4


class Fp8Act:
    """Activation rows quantized to e4m3 with one fp32 scale per row."""

    def __init__(self, rows, k, device):
        self.k = k
        self.q = torch.zeros(rows, k, dtype=torch.float8_e4m3fn, device=device)
        self.row_scale = torch.ones(rows, dtype=torch.float32, device=device)
        self.rows = rows


def quantize_rows_fp8(x: torch.Tensor, out: Fp8Act, rows: int | None = None):
    rows = x.shape[0] if rows is None else rows
    ext().quantize_rows_fp8(x, out.q, out.row_scale, rows)
    return out


def linear_fp8(xq: Fp8Act, m: int, w: Fp8Weight, out: torch.Tensor | None = None, epi=None, residual=None, bn=None,
               splits=None, fused=None):
    """out[t, n] = (sum_k q_x[t,k] q_w[n,k]) * s_x[t] * s_w[n] on the e4m3 tensor-core path."""
    epi = EPI_STORE_BF16 if epi is None else epi
    n = w.n
    if out is None:
        dt = torch.float32 if epi == EPI_STORE_F32 else torch.bfloat16
        out = torch.empty(m, n, dtype=dt, device=w.q.device)
    bn = bn or _bn_for(m)
    splits = pick_splits(m, n, w.k // 2, False, bn) if splits is None else splits
    ws = splitk_workspace(w.q.device, splits, m, n) if splits > 1 else None
    ext().gemm(w.q, xq.q, out, epi, n, w.k, m, bn, None, None, w.scale, xq.row_scale, None, residual,
               None, None, None, None, 0, 1, 1 << 30, err_flag(w.q.device), 0, splits, ws, fused)
    _count_second_kernel(splits, epi, fused)
    return out


def quantize_weight_rows(w: torch.Tensor, gscale: torch.Tensor, rows_per_g: int, packed: torch.Tensor,
                         sf: torch.Tensor):
    """Quantize bf16 weight rows [R, K] on the GPU with tensor scale gscale[r // rows_per_g]."""
    ext().quantize_nvfp4(w, w.shape[0], 3, 1, None, None, None, None, packed, sf, None, None, 128, gscale,
                         rows_per_g, None)


def quantize_rows(x: torch.Tensor, out: NvFp4Act, rows: int | None = None):
    rows = x.shape[0] if rows is None else rows
    ext().quantize_nvfp4(x, rows, 0, 1, None, None, None, None, out.packed, out.sf, out.row_scale, None, 128, None, 0,
                         None)
    return out


# ----------------------------------------------------------------- GEMMs
def _bn_for(m: int) -> int:
    """Token tile of the GEMM: 64 for decode-sized batches of 33-64 rows (bf16 / fp8 weights
    get a 64-row variant with more weight stages in flight; NVFP4 uses its 128-row one)."""
    return 32 if m <= 32 else (64 if m <= 64 else (128 if m <= 128 else 256))


_SMS = None
_WS: dict[int, torch.Tensor] = {}


def set_pdl(on: bool):
    """Programmatic dependent launch for the hot kernels: each may be scheduled while its
    predecessor drains and waits for it on the device (griddepcontrol).  CUDA graphs
    keep the mode they were captured with.  Default: ROCKET_PDL=1 in the environment.
    Needs the device-side waits (every build of setup.py compiles them in)."""
    if on and not pdl_supported():
        raise RuntimeError("programmatic dependent launch needs a build with the device-side waits (-DRKT_PDL)")
    ext().set_pdl(bool(on))


def pdl_supported() -> bool:
    return bool(ext().pdl_supported())


def pdl_enabled() -> bool:
    return bool(ext().pdl_enabled())


def num_sms() -> int:
    global _SMS
    if _SMS is None:
        _SMS = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    return _SMS


def pick_splits(m: int, n: int, k: int, nvf4: bool, bn: int | None = None) -> int:
    """Split-K factor for the persistent GEMM: the best SM-wave efficiency of
    (token blocks x weight tiles x splits) units, with >= 4 K-tiles per split
    and the fp32 partials (splits x m x n) kept within 16 MiB so they stay in L2."""
    bn = bn or _bn_for(m)
    units = -(-m // bn) * (n // 128)
    kt = k // (256 if nvf4 else 64)
    sms = num_sms()
    if units >= 4 * sms or kt < 8:
        return 1
    best, best_t = 1, float("inf")
    for s in range(1, min(32, kt // 4) + 1):
        if s > 1 and s * m * n * 4 > (16 << 20):
            break
        u = units * s
        t = (-(-u // sms) * sms) / u + 0.002 * s
        if t < best_t - 1e-9:
            best, best_t = s, t
    return best


def splitk_workspace(device, splits: int, rows: int, n: int) -> torch.Tensor:
    """Per-device fp32 split-K workspace (grown outside graph capture)."""
    dev = torch.device(device)
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    need = splits * rows * n
    ws = _WS.get(idx)
    if ws is None or ws.numel() < need:
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError("split-K workspace must be sized before CUDA graph capture")
        ws = torch.empty(max(need, 1 << 22), dtype=torch.float32, device=f"cuda:{idx}")
        _WS[idx] = ws
    return ws[:need]


def _count_second_kernel(splits, epi, fused):
    """A split-K GEMM launches its reduce kernel, and a norm with no reduce to fold into
    launches the norm kernel: one more launch behind the single extension call."""
    if splits > 1 or (fused is not None and "norm_w" in fused and epi == EPI_RESIDUAL_BF16):
        global _LAUNCHES
        _LAUNCHES += 1


def norm_args(w, out, eps, zero_centered) -> dict:
    """`fused` entries for an EPI_RESIDUAL_BF16 GEMM that also writes RMSNorm(out) * w
    into `out` (the norm is folded into the split-K reduce when the GEMM splits K)."""
    return {"norm_w": w, "norm_out": out, "norm_eps": float(eps), "norm_zc": int(bool(zero_centered))}


def linear_bf16(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, epi=EPI_STORE_BF16,
                residual=None, bn=None, splits=None, fused=None):
    """out[m, n] = x[m] . w[n] with bf16 operands (w: [N, K], N % 128 == 0)."""
    m, k = x.shape
    n = w.shape[0]
    if out is None:
        dt = torch.float32 if epi == EPI_STORE_F32 else torch.bfloat16
        out = torch.empty(m, n, dtype=dt, device=x.device)
    bn = bn or _bn_for(m)
    splits = pick_splits(m, n, k, False, bn) if splits is None else splits
    ws = splitk_workspace(x.device, splits, m, n) if splits > 1 else None
    ext().gemm(w, x, out, epi, n, k, m, bn, None, None, None, None, None, residual,
               None, None, None, None, 0, 1, 1 << 30, err_flag(x.device), 0, splits, ws, fused)
    _count_second_kernel(splits, epi, fused)
    return out


def linear_nvfp4(xq: NvFp4Act, m: int, w: NvFp4Weight, out: torch.Tensor | None = None, epi=EPI_STORE_BF16,
                 residual=None, bn=None, splits=None, fused=None):
    n = w.n
    if out is None:
        cols = n // 2 if epi == EPI_SWIGLU else n
        dt = torch.float32 if epi == EPI_STORE_F32 else torch.bfloat16
        out = torch.empty(m, cols, dtype=dt, device=xq.packed.device)
    bn = bn or _bn_for(m)
    if splits is None:
        splits = 1 if epi in (EPI_SWIGLU, EPI_ARGMAX, EPI_MOE_DOWN) else pick_splits(m, n, w.k, True, bn)
    ws = splitk_workspace(xq.packed.device, splits, m, n) if splits > 1 else None
    ext().gemm(w.packed, xq.packed, out, epi, n, w.k, m, bn, w.sf, xq.sf, w.gscale, xq.row_scale,
               None, residual, None, None, None, None, 0, 1, 1 << 30, err_flag(xq.packed.device), 0, splits, ws,
               fused)
    _count_second_kernel(splits, epi, fused)
    return out


def grouped_nvfp4(xq: NvFp4Act, w: NvFp4Weight, out: torch.Tensor, epi, plan, bn: int, row_weight=None, fused=None):
    """Grouped (per-expert) NVFP4 GEMM driven by a device-side block list."""
    ext().gemm(w.packed, xq.packed, out, epi, w.n, w.k, 0, bn, w.sf, xq.sf, w.gscale, xq.row_scale, row_weight,
               None, plan.blk_expert, plan.blk_row, plan.blk_valid, plan.num_blocks, plan.max_blocks,
               w.num_experts, 1 << 30, err_flag(xq.packed.device), 0, 1, None, fused)
    return out


def lm_head_keys(x: torch.Tensor, w: torch.Tensor, keys: torch.Tensor, n_valid: int, n_offset: int = 0):
    """Fused lm_head GEMM + per-tile argmax into u64 keys (orderable value, ~global id).
    `keys` must be zero on entry (argmax_finalize leaves them zero)."""
    m, k = x.shape
    ext().gemm(w, x, keys, EPI_ARGMAX, w.shape[0], k, m, _bn_for(m), None, None, None, None, None, None,
               None, None, None, None, 0, 1, n_valid, err_flag(x.device), n_offset, 1, None, None)
    return keys


def argmax_finalize(keys, ids_out, vals_out=None):
    ext().argmax_finalize(keys, keys.shape[0], ids_out, vals_out)
    return ids_out


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor, keys: torch.Tensor, ids_out: torch.Tensor, n_valid: int,
                   vals_out=None):
    """Greedy token: fused lm_head GEMM + per-tile argmax + finalize."""
    lm_head_keys(x, w, keys, n_valid)
    ext().argmax_finalize(keys, x.shape[0], ids_out, vals_out)
    return ids_out


# ----------------------------------------------------------------- MoE plumbing
class MoePlan:
    """Device buffers of one MoE routing plan (sized for `max_tokens`)."""

    def __init__(self, max_tokens: int, k_out: int, e_tot: int, bn: int, device):
        self.k_out, self.e_tot, self.bn = k_out, e_tot, bn
        i32 = dict(dtype=torch.int32, device=device)
        self.ids = torch.zeros(max_tokens, k_out, **i32)
        self.weights = torch.zeros(max_tokens, k_out, dtype=torch.float32, device=device)
        self.counts = torch.zeros(e_tot, **i32)
        self.ticket = torch.zeros(1, **i32)  # CTAs of the router launch that finished (reset by the last)
        self.offsets = torch.zeros(e_tot + 1, **i32)
        self.cursor = torch.zeros(e_tot, **i32)
        self.max_blocks = max_tokens * k_out // bn + e_tot + 1
        self.blk_expert = torch.zeros(self.max_blocks, **i32)
        self.blk_row = torch.zeros(self.max_blocks, **i32)
        self.blk_valid = torch.zeros(self.max_blocks, **i32)
        self.num_blocks = torch.zeros(1, **i32)
        self.total_rows = torch.zeros(1, **i32)
        self.pos = torch.zeros(max_tokens * k_out, **i32)
        # expert segments are aligned to the token tile's scale-atom height
        self.sf_rows = 32 if bn <= 32 else 128
        self.max_rows = max_tokens * k_out + e_tot * self.sf_rows


def router_topk(logits, E, top_k, n_shared, sigmoid, norm_topk, scaling, bias, shared_gate_col, plan: MoePlan, T,
                e_lo=0, e_hi=None, shared_local=True):
    """Top-k routing; under expert parallelism only experts [e_lo, e_hi) stay (rebased)."""
    ext().router_topk(logits[:T], E, top_k, n_shared, sigmoid, norm_topk, scaling, bias, shared_gate_col,
                      e_lo, E if e_hi is None else e_hi, shared_local, plan.ids, plan.weights, plan.counts)


def route_and_plan(logits, E, top_k, n_shared, sigmoid, norm_topk, scaling, bias, shared_gate_col, plan: MoePlan, T,
                   e_lo=0, e_hi=None, shared_local=True):
    """router_topk + moe_plan in one launch: one token per warp over many CTAs, the last CTA
    to finish builds the plan from the (global, atomically accumulated) counts."""
    ext().router_plan(logits[:T], E, top_k, n_shared, sigmoid, norm_topk, scaling, bias, shared_gate_col, e_lo,
                      E if e_hi is None else e_hi, shared_local, plan.ids, plan.weights, plan.counts, plan.ticket,
                      plan.e_tot, plan.bn, plan.offsets, plan.cursor, plan.blk_expert, plan.blk_row, plan.blk_valid,
                      plan.num_blocks, plan.total_rows)


def moe_plan(plan: MoePlan):
    ext().moe_plan(plan.counts, plan.e_tot, plan.bn, plan.offsets, plan.cursor, plan.blk_expert, plan.blk_row,
                   plan.blk_valid, plan.num_blocks, plan.total_rows)


def moe_recount(plan: MoePlan, T):
    """plan.counts from the routing ids of T tokens (after the ids were rewritten)."""
    ext().moe_recount(plan.ids, T * plan.k_out, plan.e_tot, plan.counts)


def moe_dispatch_quantize(x, T, plan: MoePlan, out: NvFp4Act, row_meta=None):
    """Quantize each token row once and copy it into the segment of every expert it routes to;
    `row_meta` (optional, int32 [rows]) receives token << 8 | slot of every written row."""
    ext().quantize_nvfp4(x, T, 2, plan.k_out, plan.ids, plan.weights, plan.cursor, plan.pos, out.packed, out.sf,
                         out.row_scale, None, plan.sf_rows, None, 0, row_meta)


def quantize_assigned(h, T, plan: MoePlan, out: NvFp4Act):
    """Quantize the rows h[pos[a]] of every assignment a (mode 1, in place layout)."""
    ext().quantize_nvfp4(h, T * plan.k_out, 1, 1, None, None, None, plan.pos, out.packed, out.sf, out.row_scale,
                         None, plan.sf_rows, None, 0, None)


def moe_combine(y, plan: MoePlan, T, residual, out, norm=None):
    """out = residual + the weighted expert rows; with `norm` = (w, norm_out, eps,
    zero_centered) the same kernel also writes RMSNorm(out) * w into norm_out."""
    if norm is None:
        ext().moe_combine(y, plan.pos, plan.weights, plan.k_out, T, residual, out, None, None, 0.0, 0)
    else:
        w, no, eps, zc = norm
        ext().moe_combine(y, plan.pos, plan.weights, plan.k_out, T, residual, out, w, no, float(eps), int(bool(zc)))
    return out


# ----------------------------------------------------------------- hyper-connections (mHC)
def hc_split(hc, streams, mix, base, scale, coef, x, T, norm_eps, hc_eps, iters):
    """x[:T] = sum_i pre_i * streams[:, i]; coef[:T] = (post, Sinkhorn comb) from the raw
    mix projection (streams [T, hc, d] bf16, mix [T, >=2hc+hc^2] f32)."""
    ext().hc_split(hc, streams, mix, base, scale, coef, x, T, norm_eps, hc_eps, iters)
    return x


def hc_combine(hc, streams, y, coef, T):
    """streams[t, i] <- post_i * y[t] + sum_j comb[j][i] * streams[t, j] (in place)."""
    ext().hc_combine(hc, streams, y, coef, T)
    return streams


def hc_expand(hc, streams, x, T):
    ext().hc_expand_mean(hc, streams, x, T, 0)
    return streams


def hc_mean(hc, streams, x, T):
    ext().hc_expand_mean(hc, streams, x, T, 1)
    return x


# ----------------------------------------------------------------- norm / rope / embed
def rmsnorm(x, w, eps, zero_centered=False, out=None):
    out = torch.empty_like(x) if out is None else out
    ext().rmsnorm(x, w, eps, zero_centered, out)
    return out


def rope_inv_freq(rot_dim: int, theta: float, device) -> torch.Tensor:
    i = torch.arange(rot_dim // 2, dtype=torch.float64)
    return (1.0 / (theta ** (2 * i / rot_dim))).float().to(device)


def qk_rope_kv(qkv, T, Hq, Hkv, D, rot, has_gate, positions, inv_freq, q_out, gate_out=None, qn_w=None, kn_w=None,
               eps=1e-6, zero_centered=False, k_cache=None, v_cache=None, slot_mapping=None, page_size=64,
               k_scale=1.0, v_scale=1.0):
    """q/k norm + RoPE + paged KV write.  An fp8 (e4m3) cache stores value / scale."""
    ext().qk_rope_kv(qkv, T, Hq, Hkv, D, rot, has_gate, positions, inv_freq, qn_w, kn_w, eps, zero_centered, q_out,
                     gate_out, k_cache, v_cache, slot_mapping, page_size, k_scale, v_scale)


def embed(ids, table, out, vocab_lo=0):
    ext().embed(ids, table, vocab_lo, out)
    return out


def attention(q, out, k_cache, v_cache, Hq, Hkv, D, block_table, q_start, q_len, kv_len, w_seq, w_tok0, num_work,
              grid_work, gate=None, num_splits=1, ws_o=None, ws_ml=None, page_size=64, scale=None, decode=False,
              k_scale=1.0, v_scale=1.0, block_n=0):
    """Paged GQA attention; fp8 (e4m3) caches are widened in shared memory (value = byte * scale)."""
    scale = 1.0 / math.sqrt(D) if scale is None else scale
    ext().attention(q, out, gate, k_cache, v_cache, Hq, Hkv, D, page_size, block_table, q_start, q_len, kv_len,
                    w_seq, w_tok0, num_work, grid_work, scale, num_splits, ws_o, ws_ml, err_flag(q.device), decode,
                    k_scale, v_scale, block_n)
    if num_splits > 1:  # the split-K merge is a second kernel
        global _LAUNCHES
        _LAUNCHES += 1
    return out


def attention_work(q_lens, Hq, Hkv):
    """Host-side work list: one item per (sequence, block of 128//G query tokens)."""
    G = Hq // Hkv
    tpb = 128 // G
    w_seq, w_tok0 = [], []
    for s, ql in enumerate(q_lens):
        for t0 in range(0, ql, tpb):
            w_seq.append(s)
            w_tok0.append(t0)
    return w_seq, w_tok0
