"""CPU oracle of the block-record <-> BC6H bridge (no GPU).

The reference's BLOCK_FEATURES path (train.cu:316-458) trains float BC6 records and decodes
them with its float BC6 decode (train.cu:161-182, pinned by the golden vectors of
test_oracle_golden.py); the bridge connects those records with the integer BC6H codec.
Properties checked here:
- bitstream -> records -> bitstream decodes to the same texels, for every mode (random raw
  blocks, reserved modes and wrapping deltas included) and bit for bit for blocks our encoder
  writes;
- each record's float decode is within one fp16 ulp of the block's integer decode;
- records -> bitstream -> records -> bitstream is idempotent in decoded texels.
"""
import numpy as np
import pytest

from tests.model_utils import realistic_blocks

MODE_BITS = [10, 7, 11, 11, 11, 9, 8, 8, 8, 6]
PARTS = [0xCCCC, 0x8888, 0xEEEE, 0xECC8, 0xC880, 0xFEEC, 0xFEC8, 0xEC80, 0xC800, 0xFFEC, 0xFE80, 0xE800, 0xFFE8,
         0xFF00, 0xFFF0, 0xF000, 0xF710, 0x008E, 0x7100, 0x08CE, 0x008C, 0x7310, 0x3100, 0x8CCE, 0x088C, 0x3110,
         0x6666, 0x366C, 0x17E8, 0x0FF0, 0x718E, 0x399C]


def _float_decode(O, rec):
    """16 x 3 texels of one record through the oracle's float decode (train.cu:240-261)."""
    part = int(rec[28:29].view(np.int32)[0]) & 31
    mode = int(rec[29:30].view(np.int32)[0])
    b = MODE_BITS[mode if 0 <= mode <= 9 else 0]
    out = np.zeros((16, 3), np.float32)
    for px in range(16):
        r = (PARTS[part] >> px) & 1
        out[px] = O.bc6f_decode(rec[6 * r:6 * r + 3], rec[6 * r + 3:6 * r + 6], b, float(rec[12 + px]))
    return out


def _blocks_to_texels(O, blocks):
    return O.bc6h_decode_blocks(blocks, False)


def test_random_blocks_round_trip_to_the_same_texels(oracle):
    O = oracle
    rng = np.random.default_rng(5)
    raw = rng.integers(0, 256, (2048, 16), dtype=np.uint8)
    # 2048 blocks as a 4 x 4 x 384-channel surface: one triple per block
    w = h = 4
    ch = 3 * raw.shape[0]
    rec = O.bc6f_from_bc6h(raw.reshape(-1), w, h, ch)
    back = O.bc6f_to_bc6h(rec, w, h, ch).reshape(-1, 16)
    modes = {O.bc6h_mode_index(b) for b in raw}
    assert {-1, 0, 9, 10, 13} <= modes  # reserved, two-region and one-region modes all present
    assert np.array_equal(_blocks_to_texels(O, raw), _blocks_to_texels(O, back))


def test_encoder_blocks_round_trip_bit_exact(oracle):
    O = oracle
    rng = np.random.default_rng(6)
    C, H, W = 8, 32, 48
    lat = O.smooth_latents(rng, (C, H, W))
    blocks = O.bc6h_encode_surface(lat, "planar", 4.0)
    rec = O.bc6f_from_bc6h(blocks, W, H, C)
    assert np.array_equal(O.bc6f_to_bc6h(rec, W, H, C), blocks)


def test_record_float_decode_matches_integer_decode(oracle):
    O = oracle
    rng = np.random.default_rng(7)
    C, H, W = 6, 16, 16
    lat = O.smooth_latents(rng, (C, H, W))
    blocks = O.bc6h_encode_surface(lat, "planar", 4.0)
    rec = O.bc6f_from_bc6h(blocks, W, H, C).reshape(H // 4, W // 4, 2, 32)
    tex = _blocks_to_texels(O, blocks).reshape(2, H // 4, W // 4, 16, 3).view(np.float16).astype(np.float32)
    for by in range(H // 4):
        for bx in range(W // 4):
            for t in range(2):
                f = _float_decode(O, rec[by, bx, t])
                i = tex[t, by, bx]
                assert np.all(np.abs(f - i) <= 2.0 ** -10 * np.abs(i) + 1e-7), (by, bx, t)


def test_records_to_blocks_is_idempotent(oracle):
    O = oracle
    rng = np.random.default_rng(8)
    W = H = 16
    C = 12
    rec = realistic_blocks(rng, W, H, C)
    # a few records outside the trained range: negative / large pixel indices, far endpoints
    r2 = rec.reshape(-1, 32)
    r2[0, 12:28] = np.linspace(-0.1, 0.3, 16)
    r2[1, :12] *= 3.0
    b1 = O.bc6f_to_bc6h(rec, W, H, C)
    b2 = O.bc6f_to_bc6h(O.bc6f_from_bc6h(b1, W, H, C), W, H, C)
    assert np.array_equal(_blocks_to_texels(O, b1), _blocks_to_texels(O, b2))


def test_quantized_records_stay_close(oracle):
    """Trained-like records lose only the format's precision (3-bit indices, mode
    endpoint precision) when quantized."""
    O = oracle
    rng = np.random.default_rng(9)
    W = H = 16
    C = 6
    rec = realistic_blocks(rng, W, H, C).reshape(H // 4, W // 4, 2, 32)
    tex = _blocks_to_texels(O, O.bc6f_to_bc6h(rec.reshape(-1), W, H, C)).reshape(2, H // 4, W // 4, 16, 3)
    tex = tex.view(np.float16).astype(np.float32)
    rel = []
    for by in range(H // 4):
        for bx in range(W // 4):
            for t in range(2):
                f = _float_decode(O, rec[by, bx, t])
                rel.append(np.abs(f - tex[t, by, bx]) / np.abs(f))
    rel = np.array(rel)
    assert np.median(rel) < 0.03 and rel.max() < 0.25
