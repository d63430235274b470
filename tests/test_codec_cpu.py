"""BC6H codec on the CPU: the format tables, the oracle's decoder against an independent
decoder (Pillow's BC6H, 8-bit output), and encoder properties."""
import numpy as np
import pytest


def test_format_tables_are_consistent():
    from neural_textures_b200 import bc6h_format as F
    F.check_tables()
    # the reference's partition table and 2-region endpoint precisions (train.cu:20-34)
    assert F.PARTITIONS[:4] == [0xCCCC, 0x8888, 0xEEEE, 0xECC8]
    assert [m[2] for m in F.MODES[:10]] == [10, 7, 11, 11, 11, 9, 8, 8, 8, 6]


def test_weight_tables_follow_the_rounding_formula():
    # the CUDA decoder computes the weights as round(64 i / (n - 1)) instead of loading them
    from neural_textures_b200 import bc6h_format as F
    assert F.WEIGHTS3 == [(128 * i + 7) // 14 for i in range(8)]
    assert F.WEIGHTS4 == [(128 * i + 15) // 30 for i in range(16)]


def test_generated_header_is_current():
    import os
    from neural_textures_b200 import bc6h_format as F
    from tests.conftest import ROOT
    with open(os.path.join(ROOT, "include", "neural_textures", "bc6h_format.h")) as f:
        assert f.read() == F.emit_header(), "regenerate with python -m neural_textures_b200.bc6h_format"


def _random_blocks(rng, n, mode_index=None):
    from neural_textures_b200 import bc6h_format as F
    blocks = rng.integers(0, 256, (n, 16), dtype=np.uint8)
    if mode_index is not None:
        val, mbits = F.MODES[mode_index][0], F.MODES[mode_index][1]
        mask = (1 << mbits) - 1
        blocks[:, 0] = (blocks[:, 0] & np.uint8(0xFF ^ mask)) | np.uint8(val)
    return blocks


@pytest.mark.parametrize("signed", [False])
def test_oracle_decoder_matches_pillow(oracle, signed):
    """Pillow decodes BC6H to 8-bit (clamp to [0, 1], x 255, truncated): every texel whose
    oracle value lies in (0, 1) must agree within one 8-bit step, for every mode.  UF16 only
    (the format the codec writes): Pillow's SF16 output disagrees with the specification's
    sign handling on blocks whose transformed endpoints wrap, so SF16 is pinned against the
    GPU's own BC6H texture decoder instead (tests/test_gpu_codec.py)."""
    from PIL import Image
    rng = np.random.default_rng(1 if signed else 0)
    checked = 0
    for mi in range(14):
        blocks = _random_blocks(rng, 200, mi)
        ours = oracle.bc6h_decode_blocks(blocks, signed).view(np.float16).astype(np.float64)
        for b in range(blocks.shape[0]):
            assert oracle.bc6h_mode_index(blocks[b]) == mi
            pil = np.array(Image.frombytes("RGB", (4, 4), blocks[b].tobytes(), "bcn", 6,
                                           "BC6HS" if signed else "BC6H"), np.int32).reshape(16, 3)
            v = ours[b]
            sel = (v > 0) & (v < 1)
            want = np.floor(np.clip(v, 0, 1) * 255)
            assert np.all(np.abs(pil[sel] - want[sel]) <= 1), (mi, b)
            checked += int(sel.sum())
    assert checked > 5000


def test_reserved_modes_decode_to_zero(oracle):
    for val in (0x13, 0x17, 0x1B, 0x1F):
        blk = np.full(16, 0xA5, np.uint8)
        blk[0] = (blk[0] & np.uint8(0xE0)) | np.uint8(val)
        assert oracle.bc6h_mode_index(blk) == -1
        assert np.all(oracle.bc6h_decode_blocks(blk, False) == 0)


def test_encoder_round_trip_and_determinism(oracle):
    rng = np.random.default_rng(3)
    x = oracle.smooth_latents(rng, (6, 64, 64))
    b1 = oracle.bc6h_encode_surface(x)
    b2 = oracle.bc6h_encode_surface(x, threads=1)
    np.testing.assert_array_equal(b1, b2)
    d = oracle.bc6h_decode_surface(b1, x.shape)
    err = d.view(np.float16).astype(np.float64) - x.view(np.float16).astype(np.float64)
    assert np.sqrt((err ** 2).mean()) < 0.2
    assert np.abs(err).max() < 2.0
    # every two-region mode and several one-region modes occur on this data
    modes = {oracle.bc6h_mode_index(b) for b in b1.reshape(-1, 16)}
    assert len(modes) >= 6


def test_constant_blocks_are_nearly_exact(oracle):
    for v in (-3.5, -1.0, -0.25, 0.0, 0.3, 1.7, 3.9):
        x = np.full((3, 4, 4), np.float16(v)).view(np.uint16)
        d = oracle.bc6h_decode_surface(oracle.bc6h_encode_surface(x), x.shape)
        assert np.abs(d.view(np.float16).astype(np.float64) - v).max() <= 4e-3


def test_planar_and_interleaved_layouts_agree(oracle):
    rng = np.random.default_rng(5)
    x = oracle.smooth_latents(rng, (5, 20, 28))
    inter = np.ascontiguousarray(np.transpose(x, (1, 2, 0)))
    np.testing.assert_array_equal(oracle.bc6h_encode_surface(x),
                                  oracle.bc6h_encode_surface(inter, layout="interleaved"))


def test_ragged_surface_replicates_edges(oracle):
    rng = np.random.default_rng(6)
    x = oracle.smooth_latents(rng, (2, 9, 7))
    b = oracle.bc6h_encode_surface(x)
    assert b.size == 1 * 3 * 2 * 16
    d = oracle.bc6h_decode_surface(b, x.shape)
    err = d.view(np.float16).astype(np.float64) - x.view(np.float16).astype(np.float64)
    assert np.abs(err).max() < 2.0
