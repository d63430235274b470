"""BC6H codec on the GPU: encode and decode bit-exact against the CPU oracle, raw decode of
random blocks of every mode (signed and unsigned) bit-exact against the oracle, and the
decoder against the B200's own BC6H texture decoder."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SHAPES = [
    ((3, 64, 64), "planar"),
    ((16, 128, 96), "planar"),
    ((5, 37, 23), "planar"),      # ragged: partial blocks, missing third channel
    ((1, 4, 4), "planar"),
    ((40, 24, 8), "interleaved"),  # [H][W][C] latent-grid layout, C = 8
    ((20, 12, 12), "interleaved"),
]


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(cuda).view(torch.float16)


@pytest.mark.parametrize("shape,layout", SHAPES)
def test_encode_decode_bit_exact(cuda, oracle, shape, layout):
    import torch
    import neural_textures_b200 as nt
    from neural_textures_b200 import api
    rng = np.random.default_rng(hash(shape) % 1000)
    if layout == "planar":
        x = oracle.smooth_latents(rng, shape)
    else:
        x = np.ascontiguousarray(np.transpose(oracle.smooth_latents(rng, (shape[2], shape[0], shape[1])), (1, 2, 0)))
    t = _dev(x, cuda)
    blocks = api.bc6h_encode(t, layout=layout)
    torch.cuda.synchronize()
    ref_blocks = oracle.bc6h_encode_surface(x, layout=layout)
    np.testing.assert_array_equal(blocks.cpu().numpy(), ref_blocks)
    out = torch.zeros_like(t)
    api.bc6h_decode(blocks, out, layout=layout)
    torch.cuda.synchronize()
    ref = oracle.bc6h_decode_surface(ref_blocks, x.shape, layout=layout)
    np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)


@pytest.mark.parametrize("bias", [4.0, 0.5, 3.3, 1e-3])
def test_decode_bias_bit_exact(cuda, oracle, bias):
    """Decode with several biases (fp16-exact or not), whole blocks (the palette decode) and a
    ragged surface (the per-texel decode), bit for bit against the oracle."""
    import torch
    from neural_textures_b200 import api
    rng = np.random.default_rng(11)
    for shape in ((6, 64, 32), (3, 21, 10)):
        x = oracle.smooth_latents(rng, shape)
        ref_blocks = oracle.bc6h_encode_surface(x, bias=bias)
        blocks = torch.from_numpy(ref_blocks).to(cuda)
        out = torch.zeros(shape, dtype=torch.float16, device=cuda)
        api.bc6h_decode(blocks, out, bias=bias)
        torch.cuda.synchronize()
        ref = oracle.bc6h_decode_surface(ref_blocks, shape, bias=bias)
        np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)


@pytest.mark.parametrize("signed", [0, 1])
def test_raw_decode_all_modes_bit_exact(cuda, oracle, signed):
    import torch
    from neural_textures_b200 import _native
    rng = np.random.default_rng(10 + signed)
    blocks = rng.integers(0, 256, (14 * 512 + 64, 16), dtype=np.uint8)
    from neural_textures_b200 import bc6h_format as F
    for mi in range(14):
        val, mbits = F.MODES[mi][0], F.MODES[mi][1]
        sl = slice(mi * 512, (mi + 1) * 512)
        blocks[sl, 0] = (blocks[sl, 0] & np.uint8(0xFF ^ ((1 << mbits) - 1))) | np.uint8(val)
    d_blocks = torch.from_numpy(blocks).to(cuda)
    out = torch.zeros(blocks.shape[0] * 48, dtype=torch.int16, device=cuda)
    _native.check(_native.load().nt_bc6h_decode_raw(d_blocks.data_ptr(), blocks.shape[0], signed, out.data_ptr(),
                                                     None))
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16).reshape(-1, 16, 3)
    np.testing.assert_array_equal(got, oracle.bc6h_decode_blocks(blocks, bool(signed)))


def test_surface_decode_all_modes_bit_exact(cuda, oracle):
    """Random bitstreams of every mode (reserved mode values included) decoded into a planar
    surface of whole blocks, the per-block palette path, bit for bit against the oracle's
    surface decode (bias 4, UF16)."""
    import torch
    from neural_textures_b200 import api
    from neural_textures_b200 import bc6h_format as F
    rng = np.random.default_rng(23)
    bw, bh = 64, 113  # 7,232 blocks of one channel triple
    blocks = rng.integers(0, 256, (bw * bh, 16), dtype=np.uint8)
    for mi in range(14):
        val, mbits = F.MODES[mi][0], F.MODES[mi][1]
        sl = slice(mi * 512, (mi + 1) * 512)
        blocks[sl, 0] = (blocks[sl, 0] & np.uint8(0xFF ^ ((1 << mbits) - 1))) | np.uint8(val)
    shape = (3, 4 * bh, 4 * bw)
    out = torch.zeros(shape, dtype=torch.float16, device=cuda)
    api.bc6h_decode(torch.from_numpy(blocks.reshape(-1)).to(cuda), out)
    torch.cuda.synchronize()
    ref = oracle.bc6h_decode_surface(blocks.reshape(-1), shape)
    np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), ref)


@pytest.mark.parametrize("signed", [0, 1])
def test_decoder_matches_texture_hardware(cuda, oracle, signed):
    """Upload random blocks of every mode into a BC6H CUDA array and fetch them through the
    texture unit: every texel must equal the decoder's half value exactly."""
    import ctypes as C
    import torch
    from neural_textures_b200 import _native
    from neural_textures_b200 import bc6h_format as F
    rng = np.random.default_rng(20 + signed)
    bw, bh = 64, 14
    blocks = rng.integers(0, 256, (bh, bw, 16), dtype=np.uint8)
    for mi in range(14):  # one block row per mode
        val, mbits = F.MODES[mi][0], F.MODES[mi][1]
        blocks[mi, :, 0] = (blocks[mi, :, 0] & np.uint8(0xFF ^ ((1 << mbits) - 1))) | np.uint8(val)
    d_blocks = torch.from_numpy(blocks.reshape(-1)).to(cuda)
    rgba = np.zeros((bh * 4, bw * 4, 4), np.float32)
    _native.check(_native.load().nt_bc6h_decode_hardware(d_blocks.data_ptr(), bw, bh, signed,
                                                          rgba.ctypes.data_as(C.POINTER(C.c_float))))
    ours = oracle.bc6h_decode_blocks(blocks.reshape(-1, 16), bool(signed)).view(np.float16).astype(np.float32)
    ours = ours.reshape(bh, bw, 4, 4, 3).transpose(0, 2, 1, 3, 4).reshape(bh * 4, bw * 4, 3)
    bad = ~np.isclose(rgba[..., :3], ours, rtol=0, atol=0, equal_nan=True)
    assert not bad.any(), f"{int(bad.sum())} texel channels differ; first at {np.argwhere(bad)[:4].tolist()}"


def test_codec_rejects_bad_arguments(cuda):
    import ctypes as C
    from neural_textures_b200 import _native
    L = _native.load()
    s = _native.NtBc6hSurface()
    assert L.nt_bc6h_encode(C.byref(s), None, 4.0, None) == 1
    assert L.nt_bc6h_blocks_bytes(4096, 4096, 16) == 6 * 1024 * 1024 * 16
