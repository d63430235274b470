"""Host-side mirror of the reference's training / decode interface over the C ABI.

mavenkim2/neural_textures exposes train.h:158-161 (InvokeOptimizeNetwork,
InvokeOptimizeFeatures, InvokeTraining, InvokeInference) taking a KernelParams by value,
and tests/forward_pass_test.h:6 (RunForwardPassTest).  The same entry points are exported
here under the same names (plus snake_case aliases); they take an NtKernelParams built from
device buffers and raise NtError when the library rejects a call, as the reference's
driver raises std::runtime_error from CheckCuda (main.cpp:103-110).

NeuralTexture owns the device buffers of one material (what the reference's driver
allocates in main.cpp:657-793) using torch only as the allocator; every computation runs
in libnt_b200.so.
"""
from __future__ import annotations

import contextlib
import ctypes as C
import enum
import functools
import math
import os

import numpy as np

from . import _native as N
from ._native import NtError, NtKernelParams, check, load


class TrainingKernelType(enum.IntEnum):
    """train.h:22-27"""
    UNCONSTRAINED = N.NT_TRAIN_UNCONSTRAINED
    BLOCK_FEATURES = N.NT_TRAIN_BLOCK_FEATURES
    FINALIZE = N.NT_TRAIN_FINALIZE


def _device_guard(device):
    """Make `device` current for calls into the library (its kernels launch on the current
    device, so a material on another GPU must select its own)."""
    if device is None or getattr(device, "type", None) != "cuda":
        return contextlib.nullcontext()
    import torch
    return torch.cuda.device(device)


def _on_device(fn):
    @functools.wraps(fn)
    def wrapped(self, *args, **kwargs):
        with _device_guard(self.device):
            return fn(self, *args, **kwargs)
    return wrapped


def _stream(stream) -> int | None:
    if stream is None:
        return None
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


def InvokeTraining(params: NtKernelParams, type=TrainingKernelType.UNCONSTRAINED, stream=None):
    """train.h:160 -- fused sample / forward / loss / backward, accumulating gradients."""
    check(load().nt_invoke_training(C.byref(params), int(type), _stream(stream)))


def InvokeOptimizeNetwork(params: NtKernelParams, stream=None):
    """train.h:158 -- Adam over the network weights and biases (consumes and zeroes grads)."""
    check(load().nt_invoke_optimize_network(C.byref(params), _stream(stream)))


def InvokeOptimizeFeatures(params: NtKernelParams, type=TrainingKernelType.UNCONSTRAINED, stream=None):
    """train.h:159 -- Adam over both latent grids (consumes and zeroes grads)."""
    check(load().nt_invoke_optimize_features(C.byref(params), int(type), _stream(stream)))


def InvokeOptimizeAll(params: NtKernelParams, stream=None):
    """Network + latent Adam in one launch."""
    check(load().nt_invoke_optimize_all(C.byref(params), _stream(stream)))


def InvokeInference(params: NtKernelParams, stream=None):
    """train.h:161 -- decode every texel centre into params.inference_output."""
    check(load().nt_invoke_inference(C.byref(params), _stream(stream)))


def TrainStep(params: NtKernelParams, stream=None):
    """One training step as the reference driver issues it (main.cpp:1071-1076)."""
    check(load().nt_train_step(C.byref(params), _stream(stream)))


def RunForwardPassTest() -> bool:
    """tests/forward_pass_test.h:6 -- the 12 -> 16 -> 16 known-answer test on the device."""
    return bool(load().nt_run_forward_pass_test())


invoke_training = InvokeTraining
invoke_optimize_network = InvokeOptimizeNetwork
invoke_optimize_features = InvokeOptimizeFeatures
invoke_optimize_all = InvokeOptimizeAll
invoke_inference = InvokeInference
train_step = TrainStep
run_forward_pass_test = RunForwardPassTest


def launch_count() -> int:
    return int(load().nt_launch_count())


# ---------------------------------------------------------------------------------------
# BC6H latent block codec

def bc6h_surface(t, layout: str = "planar") -> N.NtBc6hSurface:
    """Describe an fp16 device tensor as a codec surface: `planar` [C][H][W] or
    `interleaved` [H][W][C] (the latent-grid layout)."""
    s = N.NtBc6hSurface()
    s.data = t.data_ptr()
    if layout == "planar":
        C_, H, W = t.shape
        s.channel_stride, s.row_stride, s.texel_stride = t.stride()
    elif layout == "interleaved":
        H, W, C_ = t.shape
        s.row_stride, s.texel_stride, s.channel_stride = t.stride()
    else:
        raise ValueError(f"unknown layout {layout!r}")
    s.width, s.height, s.channels = W, H, C_
    return s


def bc6h_blocks_bytes(width: int, height: int, channels: int) -> int:
    return int(load().nt_bc6h_blocks_bytes(width, height, channels))


def bc6h_encode(t, layout: str = "planar", bias: float = 4.0, blocks=None, stream=None):
    """Encode an fp16 surface to BC6H UF16 blocks of (value + bias); returns uint8 blocks."""
    import torch
    s = bc6h_surface(t, layout)
    nbytes = bc6h_blocks_bytes(s.width, s.height, s.channels)
    if blocks is None:
        blocks = torch.empty(nbytes, dtype=torch.uint8, device=t.device)
    check(load().nt_bc6h_encode(C.byref(s), blocks.data_ptr(), bias, _stream(stream)))
    return blocks


def bc6h_decode(blocks, out, layout: str = "planar", bias: float = 4.0, stream=None):
    """Decode blocks into the fp16 tensor `out` (its shape selects the surface)."""
    s = bc6h_surface(out, layout)
    check(load().nt_bc6h_decode(blocks.data_ptr(), C.byref(s), bias, _stream(stream)))
    return out


def mip_chain_texels(width: int, height: int, num_mips: int) -> int:
    """Texels of a num_mips-level chain (level m: max(w >> m, 1) x max(h >> m, 1))."""
    return int(load().nt_mip_chain_texels(width, height, num_mips))


def bc6f_records_floats(width: int, height: int, channels: int) -> int:
    return int(load().nt_bc6f_records_floats(width, height, channels))


def bc6f_from_bc6h(blocks, width: int, height: int, channels: int, records=None, stream=None):
    """BC6H blocks (bc6h_encode's layout) -> float BC6 block records (fp32 device tensor,
    [height/4][width/4][ceil(channels/3)][32]), the BLOCK_FEATURES latent layout."""
    import torch
    n = bc6f_records_floats(width, height, channels)
    if n == 0:
        raise ValueError(f"block records need width and height multiples of 4, got {width} x {height}")
    if records is None:
        records = torch.empty(n, dtype=torch.float32, device=blocks.device)
    check(load().nt_bc6f_from_bc6h(blocks.data_ptr(), width, height, channels, records.data_ptr(), _stream(stream)))
    return records


def bc6f_to_bc6h(records, width: int, height: int, channels: int, blocks=None, stream=None):
    """Float BC6 block records -> BC6H UF16 blocks (uint8 device tensor, bc6h_encode's layout)."""
    import torch
    if blocks is None:
        blocks = torch.empty(bc6h_blocks_bytes(width, height, channels), dtype=torch.uint8, device=records.device)
    check(load().nt_bc6f_to_bc6h(records.data_ptr(), width, height, channels, blocks.data_ptr(), _stream(stream)))
    return blocks


# ---------------------------------------------------------------------------------------
# reference textures (train.h:69-77, main.cpp:558-637)

def box_chain_f32(level0: np.ndarray, num_mips: int) -> np.ndarray:
    """fp32 chain (levels one after another) of [h][w][c] level 0: 2x2 box average per level,
    source texels clamped to the level below (the rule of nt_build_mips, in fp32)."""
    levels = [np.ascontiguousarray(level0, np.float32)]
    for _ in range(1, max(int(num_mips), 1)):
        a = levels[-1]
        h, w = a.shape[:2]
        dh, dw = max(h >> 1, 1), max(w >> 1, 1)
        ys0, xs0 = np.minimum(2 * np.arange(dh), h - 1), np.minimum(2 * np.arange(dw), w - 1)
        ys1, xs1 = np.minimum(ys0 + 1, h - 1), np.minimum(xs0 + 1, w - 1)
        p = lambda ys, xs: a[ys][:, xs]
        levels.append(((p(ys0, xs0) + p(ys0, xs1)) + (p(ys1, xs0) + p(ys1, xs1))) * np.float32(0.25))
    return np.concatenate([l.reshape(-1) for l in levels])


class ReferenceTexture:
    """A reference texture (train.h:69-77): a CUDA texture object over an fp32 mip chain with
    the reference's descriptor (nt_reference_texture_create).  `chain` holds the levels one after
    another, [h_m][w_m][c] with c = channels (4 for 3 channels); host (numpy) or device (torch)."""

    def __init__(self, chain, width: int, height: int, channels: int, num_mips: int = 1, loss_weight: float = 1.0,
                 device=None):
        import torch
        host = isinstance(chain, np.ndarray)
        data = np.ascontiguousarray(chain, np.float32) if host else chain.contiguous()
        self.device = torch.device(device if device is not None else
                                   ("cuda" if host else data.device))  # the texture lives on this GPU
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.desc = N.NtReferenceTexture()
        with _device_guard(self.device):
            check(load().nt_reference_texture_create(data.ctypes.data if host else data.data_ptr(), width, height,
                                                     channels, num_mips, loss_weight, C.byref(self.desc)))

    @classmethod
    def from_image(cls, image: np.ndarray, num_mips: int = 1, loss_weight: float = 1.0, device=None):
        """From an fp32 [h][w][channels] image (1 .. 4 channels; RGB is padded with alpha 1, as
        main.cpp:547 does), its chain built with the box filter."""
        img = np.asarray(image, np.float32)
        if img.ndim == 2:
            img = img[:, :, None]
        h, w, ch = img.shape
        if ch == 3:
            img = np.concatenate([img, np.ones((h, w, 1), np.float32)], axis=2)
        return cls(box_chain_f32(img, num_mips), w, h, ch, num_mips, loss_weight, device=device)

    def sample(self, uv, lod: float = 0.0, stream=None):
        """SampleReferenceTextureTrilinear (train.cu:78-103) at device coordinates uv [n][2] ->
        [n][4] float32 (channels past num_channels are 0)."""
        import torch
        uv = uv.contiguous()
        out = torch.empty((uv.shape[0], 4), dtype=torch.float32, device=uv.device)
        with _device_guard(self.device):
            check(load().nt_reference_texture_sample(C.byref(self.desc), uv.data_ptr(), uv.shape[0], lod,
                                                     out.data_ptr(), _stream(stream)))
        return out

    def close(self):
        if getattr(self, "desc", None) is not None and self.desc.texture:
            with _device_guard(self.device):
                check(load().nt_reference_texture_destroy(C.byref(self.desc)))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ---------------------------------------------------------------------------------------
# on-disk format (nt_checkpoint_write / _index / _read: named, typed, checksummed sections)

_CKPT_DTYPES = {np.dtype(np.float16): N.NT_DTYPE_F16, np.dtype(np.float32): N.NT_DTYPE_F32,
                np.dtype(np.uint8): N.NT_DTYPE_U8, np.dtype(np.int32): N.NT_DTYPE_I32}
_CKPT_NUMPY = {v: k for k, v in _CKPT_DTYPES.items()}


def checkpoint_write(path, sections: dict):
    """Write host arrays (float16, float32, uint8 or int32; up to 4 dimensions) as named
    sections; the file is replaced atomically."""
    arrs = [(str(k), np.asarray(v, order="C")) for k, v in sections.items()]  # keeps 0-d arrays 0-d
    tab = (N.NtCheckpointSection * max(len(arrs), 1))()
    for i, (name, a) in enumerate(arrs):
        if a.dtype not in _CKPT_DTYPES or a.ndim > 4:
            raise ValueError(f"section {name!r}: dtype {a.dtype} with {a.ndim} dimensions is not storable")
        e = tab[i]
        e.name = name.encode()
        e.dtype = _CKPT_DTYPES[a.dtype]
        e.ndim = a.ndim
        for d in range(a.ndim):
            e.shape[d] = a.shape[d]
        e.bytes = a.nbytes
        e.data = a.ctypes.data
    check(load().nt_checkpoint_write(os.fsencode(str(path)), tab, len(arrs)))


def checkpoint_index(path) -> dict:
    """{name: (numpy dtype, shape)} of a checkpoint file."""
    L = load()
    n = C.c_int32(0)
    check(L.nt_checkpoint_index(os.fsencode(str(path)), None, 0, C.byref(n)))
    tab = (N.NtCheckpointSection * max(n.value, 1))()
    check(L.nt_checkpoint_index(os.fsencode(str(path)), tab, n.value, C.byref(n)))
    return {tab[i].name.decode(): (_CKPT_NUMPY[tab[i].dtype], tuple(tab[i].shape[:tab[i].ndim]))
            for i in range(n.value)}


def checkpoint_read(path, name: str | None = None):
    """One section as a numpy array, or all of them as a dict (checksums verified)."""
    idx = checkpoint_index(path)
    names = [name] if name is not None else list(idx)
    out = {}
    for nm in names:
        if nm not in idx:
            raise KeyError(f"{path} has no section {nm!r}")
        dt, shape = idx[nm]
        a = np.empty(shape, dt)
        check(load().nt_checkpoint_read(os.fsencode(str(path)), nm.encode(), a.ctypes.data if a.nbytes else None,
                                        a.nbytes))
        out[nm] = a
    return out[name] if name is not None else out


# ---------------------------------------------------------------------------------------
# parameter initialisation (host, seeded)

PAD_IN = (32, 64, 64)
PAD_OUT = (64, 64, 16)


def he_normal_weights(seed: int, cout: int) -> list[np.ndarray]:
    """He-normal N(0, 2 / fan_in) weights in the padded column-major fp16 layout
    (W[out * padIn + in]); padded rows / columns are zero.  Returned as fp16 arrays."""
    rng = np.random.default_rng(seed)
    out = []
    for l in range(3):
        W = np.zeros((PAD_OUT[l], PAD_IN[l]), np.float32)
        active_out = 64 if l < 2 else cout
        fan = PAD_IN[l]
        W[:active_out, :fan] = rng.standard_normal((active_out, fan)) * math.sqrt(2.0 / fan)
        out.append(W.astype(np.float16).reshape(-1))
    return out


def zero_padded_inputs(W0: np.ndarray, n_inputs: int) -> np.ndarray:
    """Zero layer-0 weights of the padded inputs (>= n_inputs)."""
    W = W0.reshape(64, 32).copy()
    W[:, n_inputs:] = 0
    return W.reshape(-1)


class NeuralTexture:
    """Device state of one material: two fp16 latent grids, the 32 -> 64 -> 64 -> cout
    network, fp32 gradients and Adam moments for everything, and the fp16 target."""

    def __init__(self, image_w: int, image_h: int, grid_sizes=((512, 512), (256, 256)),
                 latent_channels: int = 8, output_channels: int = 8, device="cuda",
                 lattice=None, latent_lr: float = 1e-2, network_lr: float = 5e-3,
                 beta1: float = 0.9, beta2: float = 0.99, eps: float = 1e-8, num_mips=(1, 1),
                 target_num_mips: int = 1):
        import torch
        self.torch = torch
        self.device = torch.device(device)
        self.image_w, self.image_h = image_w, image_h
        self.C, self.cout = latent_channels, output_channels
        self.grid_sizes = [tuple(g) for g in grid_sizes]
        self.num_mips = [max(int(n), 1) for n in num_mips]
        self.target_num_mips = max(int(target_num_mips), 1)
        self.lod = 0.0  # mip coordinate of every sample (NtKernelParams.lod)
        f16, f32 = torch.float16, torch.float32
        z = lambda shape, dt: torch.zeros(shape, dtype=dt, device=self.device)
        # each grid is a mip chain (level 0 first); grids[g] views level 0 as [h][w][C]
        self.grid_chains = [z(mip_chain_texels(w, h, n) * self.C, f16)
                            for (w, h), n in zip(self.grid_sizes, self.num_mips)]
        self.grids = [c[:w * h * self.C].view(h, w, self.C) for c, (w, h) in zip(self.grid_chains, self.grid_sizes)]
        shaped = lambda c, g: c.view(g.shape) if c.numel() == g.numel() else c
        self.ggrads = [shaped(z(c.numel(), f32), g) for c, g in zip(self.grid_chains, self.grids)]
        self.gm1 = [shaped(z(c.numel(), f32), g) for c, g in zip(self.grid_chains, self.grids)]
        self.gm2 = [shaped(z(c.numel(), f32), g) for c, g in zip(self.grid_chains, self.grids)]
        self.W = [z(PAD_OUT[l] * PAD_IN[l], f16) for l in range(3)]
        self.b = [z(64, f16), z(64, f16), z(self.cout, f16)]
        self.gW = [z(w.shape, f32) for w in self.W]
        self.mW = [z(w.shape, f32) for w in self.W]
        self.vW = [z(w.shape, f32) for w in self.W]
        self.gb = [z(b.shape, f32) for b in self.b]
        self.mb = [z(b.shape, f32) for b in self.b]
        self.vb = [z(b.shape, f32) for b in self.b]
        self.target_chain = z(mip_chain_texels(image_w, image_h, self.target_num_mips) * self.cout, f16)
        self.target = self.target_chain[:image_w * image_h * self.cout].view(image_h, image_w, self.cout)
        self.loss_accum = z(1, f32)
        # tile counter of the training kernel (NtKernelParams.workspace; zero between calls)
        self.workspace = z(int(load().nt_workspace_bytes()) // 4, torch.int32)
        if lattice is None:
            lattice = (image_w, image_h)
        self.lattice = tuple(lattice)
        self.latent_adam = (beta1, beta2, latent_lr, eps)
        self.network_adam = (beta1, beta2, network_lr, eps)
        self.channel_weights = [1.0] * self.cout
        self.seed = 0
        self.step = 0
        self.latent_format = N.NT_LATENT_GRID_F16
        self.blocks = None  # BC6 block-feature records per grid (fp32), when latent_format is 1
        self.reference_textures = []  # ReferenceTexture list: replaces `target` when non-empty

    def use_blocks(self, records):
        """Switch the latents to BC6 block features: `records` holds, per grid, the fp32
        records (ceil(C / 3) triples of 32 floats per 4x4 block, nt_capi.h latent_format).
        Gradients and Adam moments of the records are allocated here, zeroed."""
        torch = self.torch
        as_dev = lambda r: (r.to(self.device, torch.float32).contiguous() if isinstance(r, torch.Tensor) else
                            torch.as_tensor(np.ascontiguousarray(r, np.float32)).to(self.device))
        self.blocks = [as_dev(r) for r in records]
        self.ggrads = [torch.zeros_like(b) for b in self.blocks]
        self.gm1 = [torch.zeros_like(b) for b in self.blocks]
        self.gm2 = [torch.zeros_like(b) for b in self.blocks]
        self.latent_format = N.NT_LATENT_BC6_BLOCKS

    def _shift_latent_inputs(self, delta: float):
        """Layer-1 bias += delta * (sum of W1's latent columns): compensates latent inputs that
        move by -delta (layer-1 inputs 0 .. 2C - 1 are the two grids' channels)."""
        torch = self.torch
        W1 = self.W[0].view(PAD_OUT[0], PAD_IN[0]).float()
        b1 = self.b[0].float() + delta * W1[:, :2 * self.C].sum(dim=1)
        self.b[0].copy_(b1.to(torch.float16))

    @_on_device
    def to_blocks(self, bias: float = 4.0, stream=None):
        """Switch from fp16 grids to BC6 block features for compression-aware fine-tuning
        (the reference's UNCONSTRAINED -> BLOCK_FEATURES schedule, main.cpp:1046-1061): each grid
        is encoded as BC6H UF16 blocks of (value + bias) and the blocks become block records
        (nt_bc6f_from_bc6h).  The records decode to value + bias, so the layer-1 bias absorbs
        -bias x W1's latent columns and the network output stays that of the encoded grids."""
        if max(self.num_mips) > 1:
            raise ValueError("to_blocks converts single-level grids (num_mips 1)")
        blocks = [bc6h_encode(g, "interleaved", bias, stream=stream) for g in self.grids]
        recs = [bc6f_from_bc6h(b, w, h, self.C, stream=stream) for b, (w, h) in zip(blocks, self.grid_sizes)]
        self._shift_latent_inputs(-bias)
        self.use_blocks(recs)
        self.block_bias = bias

    @_on_device
    def export_bc6h(self, stream=None):
        """BC6H blocks of the block records (nt_bc6f_to_bc6h), one uint8 tensor per grid; they
        hold value + self.block_bias, as bc6h_encode(..., bias=self.block_bias) would."""
        if self.latent_format != N.NT_LATENT_BC6_BLOCKS:
            raise RuntimeError("export_bc6h needs block features (call to_blocks first)")
        return [bc6f_to_bc6h(r, w, h, self.C, stream=stream) for r, (w, h) in zip(self.blocks, self.grid_sizes)]

    @_on_device
    def from_bc6h(self, blocks, bias: float | None = None, stream=None):
        """Back to fp16 grids: decode BC6H blocks (value + bias) into the grids, undo the
        layer-1 shift of to_blocks and train / decode grids from here on."""
        torch = self.torch
        bias = getattr(self, "block_bias", 4.0) if bias is None else bias
        for g, bl in zip(self.grids, blocks):
            bc6h_decode(bl, g, "interleaved", bias, stream=stream)
        if self.latent_format == N.NT_LATENT_BC6_BLOCKS:
            self._shift_latent_inputs(bias)
        f32 = torch.float32
        self.ggrads = [torch.zeros(g.shape, dtype=f32, device=self.device) for g in self.grids]
        self.gm1 = [torch.zeros_like(g) for g in self.ggrads]
        self.gm2 = [torch.zeros_like(g) for g in self.ggrads]
        self.blocks = None
        self.latent_format = N.NT_LATENT_GRID_F16

    # -- initialisation -------------------------------------------------------------------
    @_on_device
    def init(self, seed: int = 0, target_seed: int | None = None, pbr_normals: bool = False,
             stream=None):
        torch = self.torch
        L = load()
        for i, g in enumerate(self.grid_chains):  # per-index hash: level 0 does not depend on the chain
            check(L.nt_init_latents(g.data_ptr(), g.numel(), seed * 7919 + i + 1, _stream(stream)))
        Ws = he_normal_weights(seed, self.cout)
        Ws[0] = zero_padded_inputs(Ws[0], 2 * self.C + 8)
        for l in range(3):
            self.W[l].copy_(torch.from_numpy(Ws[l]).to(self.device))
            self.b[l].zero_()
        ts = seed if target_seed is None else target_seed
        check(L.nt_generate_target(self.target.data_ptr(), self.image_w, self.image_h, self.cout,
                                   ts, int(pbr_normals), _stream(stream)))
        self.build_target_mips(stream)
        for t in self.ggrads + self.gm1 + self.gm2 + self.gW + self.mW + self.vW + self.gb + self.mb + self.vb:
            t.zero_()
        self.step = 0

    # -- mip chains -----------------------------------------------------------------------------
    def mip_level(self, g: int, m: int, chain=None):
        """[h_m][w_m][C] view of level m of grid g's chain (or of a same-layout chain: gradients,
        moments)."""
        w, h = self.grid_sizes[g]
        c = (self.grid_chains[g] if chain is None else chain).reshape(-1)
        off = mip_chain_texels(w, h, m) if m > 0 else 0
        lw, lh = max(w >> m, 1), max(h >> m, 1)
        return c[off * self.C:(off + lw * lh) * self.C].view(lh, lw, self.C)

    def target_level(self, m: int):
        off = mip_chain_texels(self.image_w, self.image_h, m) if m > 0 else 0
        lw, lh = max(self.image_w >> m, 1), max(self.image_h >> m, 1)
        return self.target_chain[off * self.cout:(off + lw * lh) * self.cout].view(lh, lw, self.cout)

    @_on_device
    def build_target_mips(self, stream=None):
        """Levels 1 .. target_num_mips - 1 of the target from level 0 (nt_build_mips)."""
        check(load().nt_build_mips(self.target_chain.data_ptr(), self.image_w, self.image_h, self.cout,
                                   self.target_num_mips, _stream(stream)))

    @_on_device
    def build_latent_mips(self, stream=None):
        """Latent levels 1 .. n - 1 from level 0 (box filter), e.g. after training level 0."""
        for c, (w, h), n in zip(self.grid_chains, self.grid_sizes, self.num_mips):
            check(load().nt_build_mips(c.data_ptr(), w, h, self.C, n, _stream(stream)))

    # -- checkpoints ------------------------------------------------------------------------------
    @_on_device
    def save(self, path, optimizer: bool = True, latents: str = "native", bias: float = 4.0,
             target: bool = False):
        """Write the material to a checkpoint file (nt_checkpoint_write).  Sections: meta.i32 /
        meta.f32 (sizes, chains, latent format, step, seed, lod, Adam constants, loss weights),
        net.W0..2 / net.b0..2 (fp16), latent0 / latent1 (fp16 chains or fp32 block records; with
        latents="bc6h", BC6H blocks of value + bias from nt_bc6h_encode), with optimizer=True the
        Adam moments (adam.*), with target=True the target chain.  Gradients are not stored: every
        optimiser step consumes them."""
        torch = self.torch
        h = lambda t: t.detach().cpu().contiguous().numpy()
        blocks_fmt = self.latent_format == N.NT_LATENT_BC6_BLOCKS
        if latents not in ("native", "bc6h"):
            raise ValueError("latents must be 'native' or 'bc6h'")
        bc6h = latents == "bc6h"
        if bc6h and (blocks_fmt or max(self.num_mips) > 1):
            raise ValueError("latents='bc6h' stores single-level fp16 grids")
        torch.cuda.synchronize(self.device)
        meta = [1, self.image_w, self.image_h, self.C, self.cout, self.lattice[0], self.lattice[1],
                *self.grid_sizes[0], *self.grid_sizes[1], *self.num_mips, self.target_num_mips,
                int(self.latent_format), int(self.step), int(self.seed), int(bc6h), int(optimizer), int(target)]
        metaf = [self.lod, *self.latent_adam, *self.network_adam, bias, getattr(self, "block_bias", 4.0),
                 *([float(c) for c in self.channel_weights] + [0.0] * (16 - len(self.channel_weights)))]
        sec = {"meta.i32": np.array(meta, np.int32), "meta.f32": np.array(metaf, np.float32)}
        for l in range(3):
            sec[f"net.W{l}"] = h(self.W[l])
            sec[f"net.b{l}"] = h(self.b[l])
        for g in range(2):
            if blocks_fmt:
                sec[f"latent{g}"] = h(self.blocks[g])
            elif bc6h:
                sec[f"latent{g}.bc6h"] = h(bc6h_encode(self.grids[g], "interleaved", bias))
            else:
                sec[f"latent{g}"] = h(self.grid_chains[g])
        if optimizer:
            for l in range(3):
                sec[f"adam.mW{l}"], sec[f"adam.vW{l}"] = h(self.mW[l]), h(self.vW[l])
                sec[f"adam.mb{l}"], sec[f"adam.vb{l}"] = h(self.mb[l]), h(self.vb[l])
            for g in range(2):
                sec[f"adam.m{g}"], sec[f"adam.v{g}"] = h(self.gm1[g]).reshape(-1), h(self.gm2[g]).reshape(-1)
        if target:
            sec["target"] = h(self.target_chain)
        checkpoint_write(path, sec)

    @classmethod
    def load(cls, path, device="cuda"):
        """A material from a checkpoint file written by save (checksums verified)."""
        import torch
        sec = checkpoint_read(path)
        m = [int(x) for x in sec["meta.i32"]]
        if m[0] != 1:
            raise ValueError(f"{path}: material layout {m[0]} is not supported")
        (_, iw, ih, Cc, cout, lw, lh, g0w, g0h, g1w, g1h, nm0, nm1, tnm, fmt, step, seed, bc6h, has_opt,
         has_target) = m[:20]
        f = [float(x) for x in sec["meta.f32"]]
        tex = cls(iw, ih, grid_sizes=((g0w, g0h), (g1w, g1h)), latent_channels=Cc, output_channels=cout,
                  device=device, lattice=(lw, lh), latent_lr=f[3], network_lr=f[7], beta1=f[5], beta2=f[6],
                  eps=f[8], num_mips=(nm0, nm1), target_num_mips=tnm)
        tex.latent_adam = tuple(f[1:5])
        tex.network_adam = tuple(f[5:9])
        tex.lod, tex.step, tex.seed = f[0], step, seed
        tex.block_bias = f[10]
        tex.channel_weights = f[11:11 + cout]
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(tex.device)
        for l in range(3):
            tex.W[l].copy_(d(sec[f"net.W{l}"]))
            tex.b[l].copy_(d(sec[f"net.b{l}"]))
        if fmt == N.NT_LATENT_BC6_BLOCKS:
            tex.use_blocks([d(sec["latent0"]), d(sec["latent1"])])
        for g in range(2):
            if fmt == N.NT_LATENT_BC6_BLOCKS:
                continue
            if bc6h:
                bc6h_decode(d(sec[f"latent{g}.bc6h"]), tex.grids[g], "interleaved", f[9])
            else:
                tex.grid_chains[g].copy_(d(sec[f"latent{g}"]))
        if has_opt:
            for l in range(3):
                tex.mW[l].copy_(d(sec[f"adam.mW{l}"]))
                tex.vW[l].copy_(d(sec[f"adam.vW{l}"]))
                tex.mb[l].copy_(d(sec[f"adam.mb{l}"]))
                tex.vb[l].copy_(d(sec[f"adam.vb{l}"]))
            for g in range(2):
                tex.gm1[g].view(-1).copy_(d(sec[f"adam.m{g}"]))
                tex.gm2[g].view(-1).copy_(d(sec[f"adam.v{g}"]))
        if has_target:
            tex.target_chain.copy_(d(sec["target"]))
        return tex

    def load_host(self, grids, W, b, target=None):
        """Upload host fp16 arrays (grids [h][w][C], padded W, b, optional target)."""
        torch = self.torch
        for g, src in zip(self.grids, grids):
            g.copy_(torch.from_numpy(np.ascontiguousarray(src)).view(torch.float16).reshape(g.shape))
        for dst, src in zip(self.W, W):
            dst.copy_(torch.from_numpy(np.ascontiguousarray(src)).view(torch.float16).reshape(dst.shape))
        for dst, src in zip(self.b, b):
            dst.copy_(torch.from_numpy(np.ascontiguousarray(src)).view(torch.float16).reshape(dst.shape))
        if target is not None:
            self.target.copy_(torch.from_numpy(np.ascontiguousarray(target)).view(torch.float16)
                              .reshape(self.target.shape))

    # -- parameter block --------------------------------------------------------------------
    def params(self, step: int | None = None, inference_output=None, mse_accum=None,
               loss_accum: bool = True) -> NtKernelParams:
        p = NtKernelParams()
        for i in range(2):
            f = p.features[i]
            f.grid = (self.blocks[i] if self.latent_format == N.NT_LATENT_BC6_BLOCKS else self.grids[i]).data_ptr()
            f.gradients = self.ggrads[i].data_ptr()
            f.moment1 = self.gm1[i].data_ptr()
            f.moment2 = self.gm2[i].data_ptr()
            f.width, f.height = self.grid_sizes[i]
            f.num_mips = self.num_mips[i]
        p.latent_channels, p.output_channels = self.C, self.cout
        for l in range(3):
            p.network_weights[l] = self.W[l].data_ptr()
            p.network_weight_gradients[l] = self.gW[l].data_ptr()
            p.network_weight_moment1[l] = self.mW[l].data_ptr()
            p.network_weight_moment2[l] = self.vW[l].data_ptr()
            p.network_biases[l] = self.b[l].data_ptr()
            p.network_bias_gradients[l] = self.gb[l].data_ptr()
            p.network_bias_moment1[l] = self.mb[l].data_ptr()
            p.network_bias_moment2[l] = self.vb[l].data_ptr()
        (p.network_adam.beta1, p.network_adam.beta2, p.network_adam.learning_rate,
         p.network_adam.epsilon) = self.network_adam
        (p.feature_adam.beta1, p.feature_adam.beta2, p.feature_adam.learning_rate,
         p.feature_adam.epsilon) = self.latent_adam
        p.target = self.target.data_ptr()
        for c in range(self.cout):
            p.channel_loss_weights[c] = self.channel_weights[c]
        if inference_output is not None:
            p.inference_output = inference_output.data_ptr()
            p.inference_output_dtype = (N.NT_DTYPE_F32 if inference_output.dtype == self.torch.float32
                                        else N.NT_DTYPE_F16)
        if mse_accum is not None:
            p.inference_mse_accum = mse_accum.data_ptr()
        p.image_width, p.image_height = self.image_w, self.image_h
        p.lattice_width, p.lattice_height = self.lattice
        p.sample_stride_x = self.image_w / self.lattice[0]
        p.sample_stride_y = self.image_h / self.lattice[1]
        p.num_samples = self.lattice[0] * self.lattice[1]
        p.step = self.step if step is None else step
        p.latent_format = self.latent_format
        p.lod = self.lod
        p.target_num_mips = self.target_num_mips
        if len(self.reference_textures) > N.NT_MAX_REFERENCE_TEXTURES:
            raise ValueError(f"at most {N.NT_MAX_REFERENCE_TEXTURES} reference textures")
        for i, rt in enumerate(self.reference_textures):
            p.reference_textures[i] = rt.desc
        p.num_reference_textures = len(self.reference_textures)
        p.seed = self.seed
        if loss_accum:
            p.loss_accum = self.loss_accum.data_ptr()
        p.workspace = self.workspace.data_ptr()
        p.workspace_bytes = self.workspace.numel() * 4
        return p

    # -- operations ---------------------------------------------------------------------------
    @_on_device
    def train_step(self, stream=None, params: NtKernelParams | None = None):
        TrainStep(params or self.params(), stream)
        self.step += 1

    @_on_device
    def decode(self, dtype=None, stream=None, out=None):
        torch = self.torch
        if out is None:
            out = torch.empty((self.image_h * self.image_w, self.cout),
                              dtype=dtype or torch.float16, device=self.device)
        InvokeInference(self.params(inference_output=out), stream)
        return out

    def host_model(self):
        """fp16 copies (numpy uint16 bit patterns) of grids, weights and biases."""
        torch = self.torch
        to16 = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()
        return ([to16(g) for g in self.grids], [to16(w) for w in self.W], [to16(b) for b in self.b])
