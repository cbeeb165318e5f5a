"""NVFP4 codec: e2m1 values, e4m3 block scales per 16 elements, fp32 tensor scale.

The on-disk triplet for a quantized projection ``p`` is the one the reference
checkpoints use (``engines/glm5-moe-nvfp4-2b/src/nvfp4.h:4-11``)::

    p.weight          uint8         [N, K/2]   packed e2m1, low nibble = column 2j
    p.weight_scale    float8_e4m3   [N, K/16]  one block scale per 16 columns
    p.weight_scale_2  float32       scalar     tensor ("global") scale

and ``w[n, k] = e2m1(nibble) * e4m3(block_scale[n, k // 16]) * global``.
The global scale is ``amax / (448 * 6)`` so that the largest block scale lands
at the top of the e4m3 range.

Block scales are stored row-major on disk.  The tcgen05 block-scaled MMA wants
them in 512-byte atoms of 128 rows x 4 scales, byte offset inside an atom
``(r % 32) * 16 + (r // 32) * 4 + s``, atoms ordered (row_tile, k_tile) with
k fastest (the layout the reference documents at ``src/nvfp4.h:38-62``).  That
is the layout ``tcgen05.cp.32x128b.warpx4`` moves into tensor memory so that
TMEM lane ``l``, column ``c``, byte ``s`` holds the scale of row ``l%32 + 32c``.
:func:`swizzle_sf` / :func:`unswizzle_sf` convert between the two.

Rounding is round-to-nearest-even for both codes, with e4m3 saturating at 448
and e2m1 at 6, written from the format definitions.
"""
from __future__ import annotations

import torch

E2M1_VALUES = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=torch.float32)
FP4_MAX = 6.0
E4M3_MAX = 448.0
SF_VEC = 16


def e2m1_encode(x: torch.Tensor) -> torch.Tensor:
    """Round fp32 values to the nearest e2m1 code (ties to even code), saturating at 6.

    Returns uint8 codes in [0, 15]: bit 3 is the sign, bits 0-2 index
    ``E2M1_VALUES``.
    """
    a = x.abs().float()
    # Midpoints between consecutive magnitudes; at a tie the even code wins,
    # so the comparison is <= where the lower code is even, < where it is odd.
    code = torch.zeros_like(a, dtype=torch.uint8)
    code = torch.where(a > 0.25, 1, code)
    code = torch.where(a >= 0.75, 2, code)
    code = torch.where(a > 1.25, 3, code)
    code = torch.where(a >= 1.75, 4, code)
    code = torch.where(a > 2.5, 5, code)
    code = torch.where(a >= 3.5, 6, code)
    code = torch.where(a > 5.0, 7, code)
    code = code.to(torch.uint8)
    sign = (x < 0) & (code > 0)
    return code | (sign.to(torch.uint8) << 3)


def e2m1_decode(code: torch.Tensor) -> torch.Tensor:
    mag = E2M1_VALUES.to(code.device)[(code & 7).long()]
    return torch.where((code & 8) != 0, -mag, mag)


def e4m3_encode(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> e4m3fn bits (uint8), RNE, saturating at +-448."""
    x = x.float().clamp(-E4M3_MAX, E4M3_MAX)
    return x.to(torch.float8_e4m3fn).view(torch.uint8)


def e4m3_decode(bits: torch.Tensor) -> torch.Tensor:
    return bits.view(torch.float8_e4m3fn).float()


def pack_nibbles(codes: torch.Tensor) -> torch.Tensor:
    """[..., K] uint8 codes -> [..., K/2] bytes, low nibble = even column."""
    lo = codes[..., 0::2]
    hi = codes[..., 1::2]
    return (lo | (hi << 4)).to(torch.uint8)


def unpack_nibbles(packed: torch.Tensor) -> torch.Tensor:
    lo = packed & 0xF
    hi = packed >> 4
    return torch.stack([lo, hi], dim=-1).flatten(-2)


def quantize_nvfp4(w: torch.Tensor, global_scale: float | None = None):
    """Quantize a 2-D tensor [N, K] to the NVFP4 triplet.

    Returns ``(packed uint8 [N, K/2], block_scale uint8(e4m3) [N, K/16], global fp32)``.
    ``global_scale`` defaults to ``amax / (448 * 6)``.
    """
    assert w.dim() == 2 and w.shape[1] % SF_VEC == 0, w.shape
    w = w.float()
    n, k = w.shape
    if global_scale is None:
        amax = w.abs().max().item()
        global_scale = amax / (E4M3_MAX * FP4_MAX) if amax > 0 else 1.0
    g = torch.tensor(global_scale, dtype=torch.float32)
    blocks = w.view(n, k // SF_VEC, SF_VEC)
    bamax = blocks.abs().amax(dim=-1)
    sf_bits = e4m3_encode(bamax / FP4_MAX / g)
    sf = e4m3_decode(sf_bits)
    denom = (sf * g).unsqueeze(-1)
    q = torch.where(denom > 0, blocks / torch.where(denom > 0, denom, torch.ones_like(denom)),
                    torch.zeros_like(blocks))
    codes = e2m1_encode(q).view(n, k)
    return pack_nibbles(codes), sf_bits, float(global_scale)


def dequantize_nvfp4(packed: torch.Tensor, sf_bits: torch.Tensor, global_scale: float) -> torch.Tensor:
    n = packed.shape[0]
    k = packed.shape[1] * 2
    vals = e2m1_decode(unpack_nibbles(packed)).view(n, k // SF_VEC, SF_VEC)
    sf = e4m3_decode(sf_bits).unsqueeze(-1)
    return (vals * sf * float(global_scale)).view(n, k)


# --- tcgen05 scale-factor atom layout -------------------------------------

def sf_swizzled_bytes(rows: int, k: int) -> int:
    k_sf = k // SF_VEC
    return ((rows + 127) // 128) * ((k_sf + 3) // 4) * 512


def sf_offset(rows_idx: torch.Tensor, sf_idx: torch.Tensor, k_tiles: int) -> torch.Tensor:
    """Byte offset of scale (row, s) in the atom layout (see module docstring)."""
    atom = (rows_idx // 128) * k_tiles + (sf_idx // 4)
    r = rows_idx % 128
    return atom * 512 + (r % 32) * 16 + (r // 32) * 4 + (sf_idx % 4)


def swizzle_sf(sf_linear: torch.Tensor) -> torch.Tensor:
    """Row-major [rows, K/16] uint8 scales -> flat atom layout (zero padded)."""
    rows, k_sf = sf_linear.shape
    k_tiles = (k_sf + 3) // 4
    out = torch.zeros(sf_swizzled_bytes(rows, k_sf * SF_VEC), dtype=torch.uint8, device=sf_linear.device)
    r = torch.arange(rows, device=sf_linear.device).view(-1, 1).expand(rows, k_sf)
    s = torch.arange(k_sf, device=sf_linear.device).view(1, -1).expand(rows, k_sf)
    out[sf_offset(r, s, k_tiles).reshape(-1)] = sf_linear.reshape(-1)
    return out


def unswizzle_sf(sf_swz: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    k_sf = k // SF_VEC
    k_tiles = (k_sf + 3) // 4
    r = torch.arange(rows, device=sf_swz.device).view(-1, 1).expand(rows, k_sf)
    s = torch.arange(k_sf, device=sf_swz.device).view(1, -1).expand(rows, k_sf)
    return sf_swz[sf_offset(r, s, k_tiles).reshape(-1)].view(rows, k_sf)


def quantize_rows_nvfp4_reference(x: torch.Tensor):
    """CPU restatement of the activation quantizer the GPU kernel implements.

    Each row gets its own tensor scale ``amax_row / (448 * 6)``, then the NVFP4
    procedure above.  Returns ``(packed [M, K/2], sf_linear [M, K/16], row_scale [M])``.
    """
    x = x.float()
    m, k = x.shape
    amax = x.abs().amax(dim=1)
    g = torch.where(amax > 0, amax / (E4M3_MAX * FP4_MAX), torch.ones_like(amax))
    blocks = x.view(m, k // SF_VEC, SF_VEC)
    bamax = blocks.abs().amax(dim=-1)
    sf_bits = e4m3_encode(bamax / FP4_MAX / g.unsqueeze(1))
    sf = e4m3_decode(sf_bits)
    denom = (sf * g.unsqueeze(1)).unsqueeze(-1)
    q = torch.where(denom > 0, blocks / torch.where(denom > 0, denom, torch.ones_like(denom)),
                    torch.zeros_like(blocks))
    codes = e2m1_encode(q).view(m, k)
    return pack_nibbles(codes), sf_bits, g
