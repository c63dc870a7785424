"""MatMulNBits weight image (CPU): decoding the image the way the kernel's
dequant warps do gives, for every real weight, the reference's dequantised
value ((float)q - (float)zp) * (float)scale (templates/matmul_nbits_op.c.j2:
5-54) rounded once to fp16, and exactly 0 for every padding row/column."""
import numpy as np
import pytest

from emx_onnx_cgen_b200.plan import (nbits_dequant_from_image, nbits_weight_image, unpack_nbits,
                                     unpack_nbits_zero_points)


def _random_part(rng, n, k, block, with_zp, with_bias):
    n_blocks = -(-k // block)
    b = rng.integers(0, 256, (n, n_blocks, block // 2), dtype=np.uint8)
    scales = rng.uniform(0.005, 0.02, (n, n_blocks)).astype(np.float16)
    zp = rng.integers(0, 256, (n, (n_blocks + 1) // 2), dtype=np.uint8) if with_zp else None
    bias = rng.standard_normal(n).astype(np.float32) if with_bias else None
    q = unpack_nbits(b, n, block)
    zpu = unpack_nbits_zero_points(zp, n, n_blocks)
    return (q, zpu, scales, bias), (b, scales, zp)


def _expected(q, zpu, scales, block, k):
    kk = np.arange(k)
    blk = kk // block
    deq = (q[:, :k].astype(np.float32) - zpu[:, blk].astype(np.float32)) * scales[:, blk].astype(np.float32)
    return deq.astype(np.float16)


@pytest.mark.parametrize("n,k,block,with_zp,with_bias", [
    (96, 64, 32, False, False),
    (160, 128, 32, True, True),
    (130, 200, 16, True, False),
    (256, 256, 64, False, True),
    (40, 384, 128, True, False),
])
def test_plain_image_decodes_to_reference_dequant(n, k, block, with_zp, with_bias):
    rng = np.random.default_rng(n * 7 + k)
    part, _ = _random_part(rng, n, k, block, with_zp, with_bias)
    img, bias, n_tiles, k_steps, groups = nbits_weight_image([part], k, block, fused=False)
    assert img.nbytes == n_tiles * k_steps * (4096 + 512 * groups)
    deq = nbits_dequant_from_image(img, n_tiles, k_steps, groups)
    exp = _expected(part[0], part[1], part[2], block, k)
    np.testing.assert_array_equal(deq[:n, :k].view(np.uint16), exp.view(np.uint16))
    # padding rows and the columns past the last block are exactly 0 (columns
    # K .. n_blocks*block of a partial last block meet zero activations)
    assert not np.any(deq[n:].astype(np.float32))
    assert not np.any(deq[:n, (-(-k // block)) * block:].astype(np.float32))
    if with_bias:
        np.testing.assert_array_equal(bias[:n], part[3])
        assert not np.any(bias[n:])
    else:
        assert bias is None


@pytest.mark.parametrize("n,k,block", [(96, 64, 32), (160, 128, 32), (200, 96, 16)])
def test_fused_image_interleaves_gate_and_up(n, k, block):
    rng = np.random.default_rng(n + k)
    gate, _ = _random_part(rng, n, k, block, True, False)
    up, _ = _random_part(rng, n, k, block, False, False)
    img, bias, n_tiles, k_steps, groups = nbits_weight_image([gate, up], k, block, fused=True)
    assert n_tiles == -(-n // 64) and bias is None
    deq = nbits_dequant_from_image(img, n_tiles, k_steps, groups).reshape(n_tiles, 2, 64, -1)
    eg = _expected(gate[0], gate[1], gate[2], block, k)
    eu = _expected(up[0], up[1], up[2], block, k)
    got_g = deq[:, 0].reshape(n_tiles * 64, -1)
    got_u = deq[:, 1].reshape(n_tiles * 64, -1)
    np.testing.assert_array_equal(got_g[:n, :k].view(np.uint16), eg.view(np.uint16))
    np.testing.assert_array_equal(got_u[:n, :k].view(np.uint16), eu.view(np.uint16))
    assert not np.any(got_g[n:].astype(np.float32)) and not np.any(got_u[n:].astype(np.float32))


def test_unpack_matches_reference_nibble_order():
    # byte 0x21 holds k=0 -> 1 (low nibble) and k=1 -> 2 (high nibble)
    b = np.array([[[0x21, 0x43]]], np.uint8)
    assert unpack_nbits(b, 1, 4).tolist() == [[1, 2, 3, 4]]
    zp = np.array([[0x5A]], np.uint8)
    assert unpack_nbits_zero_points(zp, 1, 2).tolist() == [[10, 5]]
