"""NVFP4 codec against values written from the format definitions."""
import torch

from rocket_b200.fuel import nvfp4 as nv


def test_e2m1_roundtrip_exact_values():
    vals = torch.tensor([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0])
    for sgn in (1.0, -1.0):
        codes = nv.e2m1_encode(vals * sgn)
        assert torch.equal(nv.e2m1_decode(codes), vals * sgn if sgn > 0 else torch.where(vals == 0, vals, -vals))


def test_e2m1_ties_to_even_and_saturation():
    x = torch.tensor([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 100.0, 0.26, 0.74])
    got = nv.e2m1_decode(nv.e2m1_encode(x))
    want = torch.tensor([0.0, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, 0.5, 0.5])
    assert torch.equal(got, want)


def test_e4m3_saturates():
    bits = nv.e4m3_encode(torch.tensor([1000.0, -1000.0, 448.0, 0.0]))
    assert nv.e4m3_decode(bits).tolist() == [448.0, -448.0, 448.0, 0.0]


def test_quantize_dequantize_error_bound():
    torch.manual_seed(0)
    w = torch.randn(64, 256) * 0.02
    packed, sf, g = nv.quantize_nvfp4(w)
    assert packed.shape == (64, 128) and sf.shape == (64, 16)
    assert abs(g - w.abs().max().item() / 2688) < 1e-12
    wd = nv.dequantize_nvfp4(packed, sf, g)
    # e2m1 step is at most 1/3 of a block's max (between 4 and 6) -> half-step error
    blk = w.view(64, 16, 16).abs().amax(-1, keepdim=True)
    err = (wd - w).view(64, 16, 16).abs()
    # half an e2m1 step (1/6 of the block max) plus the e4m3 rounding of the scale
    assert torch.all(err <= blk * 0.2 + 1e-6)
    rel = (wd - w).norm() / w.norm()
    assert rel < 0.12


def test_nibble_order_low_is_even_column():
    codes = torch.tensor([[1, 2, 3, 4]], dtype=torch.uint8)
    p = nv.pack_nibbles(codes)
    assert p.tolist() == [[0x21, 0x43]]
    assert torch.equal(nv.unpack_nibbles(p), codes)


def test_sf_swizzle_roundtrip_and_atom_layout():
    rows, k = 256, 512
    sf = torch.randint(0, 255, (rows, k // 16), dtype=torch.uint8)
    swz = nv.swizzle_sf(sf)
    assert swz.numel() == nv.sf_swizzled_bytes(rows, k)
    assert torch.equal(nv.unswizzle_sf(swz, rows, k), sf)
    # row 33, scale 5: atom (0, 1), in-atom (33%32)*16 + (33//32)*4 + 1
    k_tiles = (k // 16) // 4
    assert swz[1 * 512 + 1 * 16 + 1 * 4 + 1] == sf[33, 5]
    assert swz[(1 * k_tiles + 0) * 512 + 0] == sf[128, 0]


def test_row_quantizer_reference_matches_tensor_quantizer_per_row():
    torch.manual_seed(1)
    x = torch.randn(8, 128)
    packed, sf, g = nv.quantize_rows_nvfp4_reference(x)
    for r in range(8):
        p2, s2, g2 = nv.quantize_nvfp4(x[r:r + 1])
        assert torch.equal(packed[r:r + 1], p2) and torch.equal(sf[r:r + 1], s2)
        assert abs(g[r].item() - g2) < 1e-9
