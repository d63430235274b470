"""ctypes binding of the CPU oracle (oracle/nt_oracle.c) and of the reference-extract library.

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm, as the checker; the product package never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libnt_oracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libnt_ref.so")

_lib = None
_ref = None

u16p = C.POINTER(C.c_uint16)
f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int32)


def build(force: bool = False) -> str:
    """Compile the oracle with make (gcc, OpenMP)."""
    if force or not os.path.exists(LIB_PATH) or _stale():
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def _stale() -> bool:
    t = os.path.getmtime(LIB_PATH)
    for f in ("nt_oracle.c", "nt_oracle_codec.c", "nt_oracle.h",
              os.path.join("..", "include", "neural_textures", "bc6h_format.h")):
        if os.path.getmtime(os.path.join(HERE, f)) > t:
            return True
    return False


def build_ref(reference_root: str | None = None) -> str | None:
    """Build oracle/_ref from the reference sources in `reference_root` (else the directory
    named by $NT_REFERENCE_ROOT).  Returns None, building nothing, when neither names a
    checkout of the reference (GPU hosts carry no reference sources)."""
    root = reference_root or os.environ.get("NT_REFERENCE_ROOT")
    if not root or not os.path.exists(os.path.join(root, "train.cu")):
        return None
    subprocess.run([os.path.join(HERE, "build_ref.sh"), root], check=True,
                   stdout=subprocess.DEVNULL)
    return REF_LIB_PATH


class Sampler(C.Structure):
    _fields_ = [("image_w", C.c_int32), ("image_h", C.c_int32),
                ("lattice_w", C.c_int32), ("lattice_h", C.c_int32),
                ("stride_x", C.c_float), ("stride_y", C.c_float),
                ("offset_x", C.c_int32), ("offset_y", C.c_int32),
                ("step", C.c_int32), ("seed", C.c_uint32)]


class Model(C.Structure):
    _fields_ = [("channels", C.c_int32), ("cout", C.c_int32),
                ("gw", C.c_int32 * 2), ("gh", C.c_int32 * 2),
                ("grid", u16p * 2), ("blocks", f32p * 2), ("W", u16p * 3), ("b", u16p * 3),
                ("grid_b", u16p * 2), ("gw_b", C.c_int32 * 2), ("gh_b", C.c_int32 * 2), ("mip_t", C.c_float * 2)]


class RefTexture(C.Structure):
    _fields_ = [("chain", f32p), ("w", C.c_int32), ("h", C.c_int32), ("channels", C.c_int32),
                ("num_mips", C.c_int32), ("loss_weight", C.c_float)]


class TrainArgs(C.Structure):
    _fields_ = [("target", u16p), ("channel_weights", f32p), ("sampler", Sampler),
                ("finalize", C.c_int32), ("target_w", C.c_int32), ("target_h", C.c_int32),
                ("target_b", u16p), ("target_w_b", C.c_int32), ("target_h_b", C.c_int32),
                ("target_t", C.c_float), ("ggrid_b", f32p * 2), ("ref", C.POINTER(RefTexture)),
                ("num_ref", C.c_int32), ("lod", C.c_float)]


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        L.nto_f2h.restype = C.c_uint16
        L.nto_f2h.argtypes = [C.c_float]
        L.nto_h2f.restype = C.c_float
        L.nto_h2f.argtypes = [C.c_uint16]
        L.nto_rng_seed.restype = C.c_uint32
        L.nto_rng_seed.argtypes = [C.c_uint32, C.c_uint32, C.c_uint32]
        L.nto_rng_next.restype = C.c_uint32
        L.nto_rng_next.argtypes = [C.POINTER(C.c_uint32)]
        L.nto_rng_uniform.restype = C.c_float
        L.nto_rng_uniform.argtypes = [C.POINTER(C.c_uint32)]
        L.nto_sample_uv_array.argtypes = [C.POINTER(Sampler), f32p]
        L.nto_catmull_rom_weights.argtypes = [C.c_float, f32p]
        L.nto_wrap.restype = C.c_int32
        L.nto_wrap.argtypes = [C.c_int32, C.c_int32]
        L.nto_sample_grid.argtypes = [u16p, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                      C.c_float, f32p, i32p, f32p, f32p]
        L.nto_posenc.argtypes = [C.c_float, C.c_float, f32p]
        L.nto_decode.argtypes = [C.POINTER(Model), C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                 u16p, C.POINTER(C.c_double), C.c_int32]
        L.nto_decode_range.argtypes = [C.POINTER(Model), C.c_int32, C.c_int32, C.c_int64,
                                       C.c_int64, C.c_void_p, C.c_int32, C.c_int32]
        L.nto_set_texture_filter_mode.argtypes = [C.c_int32]
        L.nto_ref_trilinear.argtypes = [C.POINTER(RefTexture), C.c_float, C.c_float, C.c_float, f32p]
        L.nto_ref_expected.argtypes = [C.POINTER(RefTexture), C.c_int32, C.c_float, C.c_float, C.c_float, f32p, f32p]
        L.nto_mip_select.argtypes = [C.c_int32, C.c_float, C.POINTER(C.c_int32), C.POINTER(C.c_int32),
                                     C.POINTER(C.c_float)]
        L.nto_mip_dim.restype = C.c_int32
        L.nto_mip_dim.argtypes = [C.c_int32, C.c_int32]
        L.nto_mip_offset.restype = C.c_int64
        L.nto_mip_offset.argtypes = [C.c_int32, C.c_int32, C.c_int32]
        L.nto_build_mips.argtypes = [u16p, C.c_int32, C.c_int32, C.c_int32, C.c_int32]
        L.nto_train_pass.restype = C.c_double
        L.nto_train_pass.argtypes = [C.POINTER(Model), C.POINTER(TrainArgs), f32p * 3, f32p * 3,
                                     f32p * 2, C.c_int32]
        L.nto_train_pass_range.restype = C.c_double
        L.nto_train_pass_range.argtypes = [C.POINTER(Model), C.POINTER(TrainArgs), C.c_int64,
                                           C.c_int64, f32p * 3, f32p * 3, f32p * 2, C.c_int32]
        L.nto_adam_bias_correction.argtypes = [C.c_float, C.c_float, C.c_int32, f32p, f32p]
        for name, wt in (("nto_adam_f16", u16p), ("nto_adam_f32", f32p)):
            getattr(L, name).argtypes = [wt, f32p, f32p, f32p, C.c_int64, C.c_float, C.c_float,
                                         C.c_float, C.c_float, C.c_float, C.c_float]
        L.nto_target_params.argtypes = [C.c_uint32, C.c_int32, C.c_int32, i32p, i32p, f32p, f32p]
        L.nto_generate_target.argtypes = [u16p, C.c_int32, C.c_int32, C.c_int32, C.c_uint32,
                                          C.c_int32, C.c_int32]
        L.nto_fwdtest_generate.argtypes = [u16p] * 5
        L.nto_fwdtest_reference.argtypes = [u16p] * 5 + [f32p]
        _lib = L
    return _lib


def ref_lib():
    """The library compiled from the reference's own source lines, or None if unavailable."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB_PATH):
            if build_ref() is None:
                return None
        R = C.CDLL(REF_LIB_PATH)
        R.ref_fwdtest.argtypes = [u16p] * 5 + [f32p]
        R.ref_rng.argtypes = [C.c_uint32, C.c_int, C.POINTER(C.c_uint32), f32p]
        R.ref_wrap.restype = C.c_int
        R.ref_wrap.argtypes = [C.c_int, C.c_int]
        R.ref_clamp.restype = C.c_float
        R.ref_clamp.argtypes = [C.c_float, C.c_float, C.c_float]
        R.ref_catmull_rom.argtypes = [C.c_float, C.c_float, f32p, f32p]
        R.ref_adam_f16.argtypes = [u16p, f32p, f32p, C.c_float, C.c_float, C.c_float, C.c_float,
                                   C.c_float, C.c_int]
        R.ref_adam_f32.argtypes = [f32p, f32p, f32p, C.c_float, C.c_float, C.c_float, C.c_float,
                                   C.c_float, C.c_int]
        R.ref_decompress_bc6.argtypes = [f32p, f32p, C.c_int, C.c_float, f32p]
        _ref = R
    return _ref


# ---------------------------------------------------------------------------------------
# numpy helpers

def _p(a: np.ndarray, t):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(t)


def f2h(a) -> np.ndarray:
    """fp32 -> fp16 bits (uint16) with the oracle's rounding (same as numpy's)."""
    return np.asarray(a, dtype=np.float32).astype(np.float16).view(np.uint16)


def h2f(a) -> np.ndarray:
    return np.asarray(a, dtype=np.uint16).view(np.float16).astype(np.float32)


@dataclass
class OracleModel:
    """Host copy of a model: fp16 bit arrays (uint16)."""
    channels: int
    cout: int
    grids: list          # 2 x uint16 [h][w][C]
    W: list              # 3 x uint16 padded column-major
    b: list              # 3 x uint16
    blocks: list | None = None       # 2 x float32 BC6 block features (then grids are unused)
    block_sizes: list | None = None  # 2 x (w, h) texels of the block grids
    mips: list | None = None         # 2 x list of levels (uint16 [h_m][w_m][C]); level 0 = grids[g]
    lod: float = 0.0                 # mip coordinate of every sample (with mips)

    def levels(self, g):
        """(m0, m1, t) of grid g at self.lod (nto_mip_select)."""
        return mip_select(len(self.mips[g]) if self.mips else 1, self.lod)

    def ctype(self) -> Model:
        m = Model()
        m.channels = self.channels
        m.cout = self.cout
        for g in range(2):
            if self.blocks is not None:
                m.gw[g], m.gh[g] = self.block_sizes[g]
                m.blocks[g] = _p(self.blocks[g], f32p)
            elif self.mips is not None:
                m0, m1, t = self.levels(g)
                a, b = self.mips[g][m0], self.mips[g][m1]
                m.gh[g], m.gw[g] = a.shape[0], a.shape[1]
                m.grid[g] = _p(a, u16p)
                if t > 0:
                    m.gh_b[g], m.gw_b[g] = b.shape[0], b.shape[1]
                    m.grid_b[g] = _p(b, u16p)
                    m.mip_t[g] = t
            else:
                m.gh[g], m.gw[g] = self.grids[g].shape[0], self.grids[g].shape[1]
                m.grid[g] = _p(self.grids[g], u16p)
        for l in range(3):
            m.W[l] = _p(self.W[l], u16p)
            m.b[l] = _p(self.b[l], u16p)
        return m


def make_sampler(image_w, image_h, lattice_w, lattice_h, step=0, seed=0, stride_x=None,
                 stride_y=None, offset_x=0, offset_y=0) -> Sampler:
    s = Sampler()
    s.image_w, s.image_h = image_w, image_h
    s.lattice_w, s.lattice_h = lattice_w, lattice_h
    s.stride_x = float(image_w) / lattice_w if stride_x is None else stride_x
    s.stride_y = float(image_h) / lattice_h if stride_y is None else stride_y
    s.offset_x, s.offset_y = offset_x, offset_y
    s.step, s.seed = step, seed
    return s


def sample_uv(sampler: Sampler) -> np.ndarray:
    n = sampler.lattice_w * sampler.lattice_h
    out = np.zeros((n, 2), np.float32)
    lib().nto_sample_uv_array(C.byref(sampler), _p(out, f32p))
    return out


def decode(model: OracleModel, w: int, h: int, out_f32: bool = False, threads: int = 1):
    out = np.zeros((h * w, model.cout), np.float32 if out_f32 else np.uint16)
    m = model.ctype()
    sse = C.c_double(0.0)
    lib().nto_decode(C.byref(m), w, h, out.ctypes.data, int(out_f32), None, C.byref(sse), threads)
    return out


def decode_range(model: OracleModel, w: int, h: int, first: int, count: int, threads: int = 1):
    out = np.zeros((count, model.cout), np.uint16)
    m = model.ctype()
    lib().nto_decode_range(C.byref(m), w, h, first, count, out.ctypes.data, 0, threads)
    return out


def ref_textures(defs):
    """ctypes array of reference textures from [(chain float32, w, h, channels, num_mips,
    loss_weight)] (the chains must stay alive while the array is used)."""
    arr = (RefTexture * max(len(defs), 1))()
    for i, (chain, w, h, ch, nm, lw) in enumerate(defs):
        arr[i].chain = _p(chain, f32p)
        arr[i].w, arr[i].h, arr[i].channels, arr[i].num_mips, arr[i].loss_weight = w, h, ch, nm, lw
    return arr


def ref_sample(defs, uv: np.ndarray, lod: float, filter_mode: int = 1) -> np.ndarray:
    """SampleReferenceTextureTrilinear (train.cu:78-103) of the first texture at uv ([n][2]) ->
    [n][4]; emulated bilinear weights: 0 exact, 1 nearest 1/256, 2 truncated to 1/256."""
    L = lib()
    L.nto_set_texture_filter_mode(filter_mode)
    arr = ref_textures(defs)
    out = np.zeros((len(uv), 4), np.float32)
    for i, (u, v) in enumerate(np.asarray(uv, np.float32)):
        L.nto_ref_trilinear(arr, float(u), float(v), lod, _p(out[i], f32p))
    L.nto_set_texture_filter_mode(1)
    return out


def mip_select(num_mips: int, lod: float):
    m0, m1, t = C.c_int32(), C.c_int32(), C.c_float()
    lib().nto_mip_select(num_mips, lod, C.byref(m0), C.byref(m1), C.byref(t))
    return m0.value, m1.value, t.value


def mip_chain_levels(w: int, h: int, n: int):
    """[(w_m, h_m, texel offset)] of an n-level chain."""
    L = lib()
    return [(L.nto_mip_dim(w, m), L.nto_mip_dim(h, m), L.nto_mip_offset(w, h, m)) for m in range(n)]


def build_mips(level0: np.ndarray, n: int) -> list:
    """fp16 bit chain (list of [h_m][w_m][c] uint16 levels) built from level 0 (nto_build_mips)."""
    h, w, c = level0.shape
    lv = mip_chain_levels(w, h, n)
    total = lv[-1][2] + lv[-1][0] * lv[-1][1]
    chain = np.zeros(total * c, np.uint16)
    chain[:w * h * c] = level0.reshape(-1)
    lib().nto_build_mips(_p(chain, u16p), w, h, c, n)
    return [chain[o * c:(o + lw * lh) * c].reshape(lh, lw, c) for (lw, lh, o) in lv]


def train_pass(model: OracleModel, target: np.ndarray, sampler: Sampler, channel_weights=None,
               finalize: bool = False, threads: int = 1, first: int = 0, count: int | None = None,
               target_mips: list | None = None, ref_textures_defs=None):
    """One training pass.  Returns (sse, gW[3], gb[3], ggrid[2]) with fresh fp32 grads; with
    model.mips, ggrid[g] is the list of per-level gradients of grid g's chain.  target_mips
    (list of levels, level 0 = target) is sampled at model.lod."""
    m = model.ctype()
    a = TrainArgs()
    if target_mips is not None:
        t0, t1, tt = mip_select(len(target_mips), model.lod)
        target = target_mips[t0]
        a.target_h, a.target_w = target.shape[0], target.shape[1]
        if tt > 0:
            tb = target_mips[t1]
            a.target_b = _p(tb, u16p)
            a.target_h_b, a.target_w_b = tb.shape[0], tb.shape[1]
            a.target_t = tt
    if target is not None:
        a.target = _p(target, u16p)
    refs = None
    if ref_textures_defs:  # reference textures replace the target (train.cu:105-157)
        refs = ref_textures(ref_textures_defs)
        a.ref = C.cast(refs, C.POINTER(RefTexture))
        a.num_ref = len(ref_textures_defs)
        a.lod = model.lod
    cw = None
    if channel_weights is not None:
        cw = np.ascontiguousarray(channel_weights, np.float32)
        a.channel_weights = _p(cw, f32p)
    a.sampler = sampler
    a.finalize = int(finalize)
    gW = [np.zeros(x.shape, np.float32) for x in model.W]
    gb = [np.zeros(64, np.float32), np.zeros(64, np.float32), np.zeros(model.cout, np.float32)]
    if model.mips is not None:
        chains = [[np.zeros(lv.shape, np.float32) for lv in model.mips[g]] for g in range(2)]
        sel = [model.levels(g) for g in range(2)]
        pg = (f32p * 2)(*[_p(chains[g][sel[g][0]], f32p) for g in range(2)])
        for g in range(2):
            if sel[g][2] > 0:
                a.ggrid_b[g] = _p(chains[g][sel[g][1]], f32p)
        gg = chains
    else:
        gg = ([np.zeros(bl.shape, np.float32) for bl in model.blocks] if model.blocks is not None
              else [np.zeros(g.shape, np.float32) for g in model.grids])
        pg = (f32p * 2)(*[_p(x, f32p) for x in gg])
    pW = (f32p * 3)(*[_p(x, f32p) for x in gW])
    pb = (f32p * 3)(*[_p(x, f32p) for x in gb])
    if count is None:
        sse = lib().nto_train_pass(C.byref(m), C.byref(a), pW, pb, pg, threads)
    else:
        sse = lib().nto_train_pass_range(C.byref(m), C.byref(a), first, count, pW, pb, pg,
                                         threads)
    return sse, gW, gb, gg


def bias_correction(beta1, beta2, step):
    b1, b2 = C.c_float(), C.c_float()
    lib().nto_adam_bias_correction(beta1, beta2, step, C.byref(b1), C.byref(b2))
    return b1.value, b2.value


def adam_f16(w, g, m, v, lr, beta1, beta2, eps, step):
    """In-place Adam on fp16 bits w (uint16) with fp32 g, m, v (train.cu:521-588)."""
    bc1, bc2 = bias_correction(beta1, beta2, step)
    lib().nto_adam_f16(_p(w, u16p), _p(g, f32p), _p(m, f32p), _p(v, f32p), w.size, lr, beta1,
                       beta2, eps, bc1, bc2)


def adam_f32(w, g, m, v, lr, beta1, beta2, eps, step):
    bc1, bc2 = bias_correction(beta1, beta2, step)
    lib().nto_adam_f32(_p(w, f32p), _p(g, f32p), _p(m, f32p), _p(v, f32p), w.size, lr, beta1,
                       beta2, eps, bc1, bc2)


def generate_target(w, h, channels, seed, pbr_normals=False, threads=1) -> np.ndarray:
    out = np.zeros((h, w, channels), np.uint16)
    lib().nto_generate_target(_p(out, u16p), w, h, channels, seed, int(pbr_normals), threads)
    return out


def fwdtest():
    """(inputs, w0, w1, b0, b1, expected) of the forward-pass known-answer test."""
    inputs = np.zeros(32 * 12, np.uint16)
    w0 = np.zeros(256, np.uint16)
    w1 = np.zeros(256, np.uint16)
    b0 = np.zeros(16, np.uint16)
    b1 = np.zeros(16, np.uint16)
    out = np.zeros(32 * 16, np.float32)
    L = lib()
    L.nto_fwdtest_generate(*[_p(x, u16p) for x in (inputs, w0, w1, b0, b1)])
    L.nto_fwdtest_reference(*[_p(x, u16p) for x in (inputs, w0, w1, b0, b1)], _p(out, f32p))
    return inputs, w0, w1, b0, b1, out


# ---------------------------------------------------------------------------------------
# seeded model construction (shared by tests and bench)

def he_normal_weights(rng: np.random.Generator, cout: int):
    """fp16 padded column-major weights, He-normal N(0, 2 / fan_in) on the active block."""
    shapes = [(64, 32, 32), (64, 64, 64), (16, 64, 64)]  # (padOut, padIn, fan_in)
    Ws = []
    for l, (po, pi, fan) in enumerate(shapes):
        W = np.zeros((po, pi), np.float32)
        active_out = 64 if l < 2 else cout
        W[:active_out, :fan] = rng.standard_normal((active_out, fan)) * np.sqrt(2.0 / fan)
        Ws.append(f2h(W).reshape(-1).copy())
    return Ws


def zero_input_rows(W0: np.ndarray, n_inputs: int) -> np.ndarray:
    """Zero the padded input rows of layer 0 (inputs >= n_inputs)."""
    W = W0.reshape(64, 32).copy()
    W[:, n_inputs:] = 0
    return W.reshape(-1)


# ---------------------------------------------------------------------------------------
# BC6H codec

_u8p = C.POINTER(C.c_uint8)


def _codec_lib():
    L = lib()
    if not getattr(L, "_codec_bound", False):
        L.nto_bc6f_decode.argtypes = [f32p, f32p, C.c_int32, C.c_float, f32p]
        L.nto_bc6h_mode_index.restype = C.c_int
        L.nto_bc6h_mode_index.argtypes = [_u8p]
        L.nto_bc6h_decode_block.argtypes = [_u8p, C.c_int, u16p]
        L.nto_bc6h_encode_block.argtypes = [u16p, _u8p]
        L.nto_bc6h_encode_surface.argtypes = [u16p, C.c_int32, C.c_int32, C.c_int32, C.c_int64, C.c_int64,
                                              C.c_int64, C.c_float, _u8p, C.c_int32]
        L.nto_bc6h_decode_surface.argtypes = [_u8p, C.c_int32, C.c_int32, C.c_int32, C.c_int64, C.c_int64,
                                              C.c_int64, C.c_float, u16p, C.c_int32]
        L.nto_bc6f_from_bc6h_block.argtypes = [_u8p, f32p]
        L.nto_bc6f_to_bc6h_block.argtypes = [f32p, _u8p]
        L.nto_bc6f_from_bc6h_surface.argtypes = [_u8p, C.c_int32, C.c_int32, C.c_int32, f32p]
        L.nto_bc6f_to_bc6h_surface.argtypes = [f32p, C.c_int32, C.c_int32, C.c_int32, _u8p]
        L._codec_bound = True
    return L


def bc6h_decode_blocks(blocks: np.ndarray, is_signed: bool) -> np.ndarray:
    """[n][16] uint8 blocks -> [n][16][3] fp16 bit patterns."""
    L = _codec_lib()
    blocks = np.ascontiguousarray(blocks, np.uint8).reshape(-1, 16)
    out = np.zeros((blocks.shape[0], 16, 3), np.uint16)
    for i in range(blocks.shape[0]):
        L.nto_bc6h_decode_block(blocks[i].ctypes.data_as(_u8p), int(is_signed), out[i].ctypes.data_as(u16p))
    return out


def bc6h_mode_index(block: np.ndarray) -> int:
    return _codec_lib().nto_bc6h_mode_index(np.ascontiguousarray(block, np.uint8).ctypes.data_as(_u8p))


def _strides(shape, layout):
    if layout == "planar":
        C_, H, W = shape
        return W, H, C_, H * W, W, 1
    H, W, C_ = shape
    return W, H, C_, 1, W * C_, C_


def bc6h_encode_surface(data: np.ndarray, layout="planar", bias=4.0, threads=8) -> np.ndarray:
    """fp16 bits (uint16) surface -> uint8 blocks (same layout conventions as the C ABI)."""
    L = _codec_lib()
    data = np.ascontiguousarray(data, np.uint16)
    W, H, C_, cs, rs, ts = _strides(data.shape, layout)
    nb = ((C_ + 2) // 3) * ((H + 3) // 4) * ((W + 3) // 4)
    blocks = np.zeros(nb * 16, np.uint8)
    L.nto_bc6h_encode_surface(data.ctypes.data_as(u16p), W, H, C_, cs, rs, ts, bias, blocks.ctypes.data_as(_u8p),
                              threads)
    return blocks


def bc6h_decode_surface(blocks: np.ndarray, shape, layout="planar", bias=4.0, threads=8) -> np.ndarray:
    L = _codec_lib()
    out = np.zeros(shape, np.uint16)
    W, H, C_, cs, rs, ts = _strides(shape, layout)
    blocks = np.ascontiguousarray(blocks, np.uint8)
    L.nto_bc6h_decode_surface(blocks.ctypes.data_as(_u8p), W, H, C_, cs, rs, ts, bias, out.ctypes.data_as(u16p),
                              threads)
    return out


def smooth_latents(rng: np.random.Generator, shape, std=0.5, clip=4.0, corr=8) -> np.ndarray:
    """BASELINE config 3 inputs: Gaussian values (mean 0, std 0.5) with corr x corr
    box-correlated smoothness (wrap), clipped to +-clip; fp16 bit patterns."""
    n = rng.standard_normal(shape)
    for ax in (-1, -2):
        acc = np.zeros_like(n)
        for k in range(corr):
            acc += np.roll(n, k, axis=ax)
        n = acc
    n = n / n.std() * std
    return np.clip(n, -clip, clip).astype(np.float16).view(np.uint16)


def bc6f_decode(e0, e1, bits: int, x: float) -> np.ndarray:
    """BC6 float decode of one texel (train.cu:161-182): 3 channels."""
    a = np.ascontiguousarray(e0, np.float32)
    b = np.ascontiguousarray(e1, np.float32)
    out = np.zeros(3, np.float32)
    _codec_lib().nto_bc6f_decode(_p(a, f32p), _p(b, f32p), int(bits), float(x), _p(out, f32p))
    return out


def bc6f_from_bc6h(blocks: np.ndarray, w: int, h: int, channels: int) -> np.ndarray:
    """BC6H blocks [triple][h/4][w/4] x 16 B -> float BC6 records [h/4][w/4][triple][32]."""
    blocks = np.ascontiguousarray(blocks, np.uint8)
    out = np.zeros((h // 4) * (w // 4) * ((channels + 2) // 3) * 32, np.float32)
    _codec_lib().nto_bc6f_from_bc6h_surface(blocks.ctypes.data_as(_u8p), w, h, channels, _p(out, f32p))
    return out


def bc6f_to_bc6h(records: np.ndarray, w: int, h: int, channels: int) -> np.ndarray:
    """Float BC6 records -> BC6H blocks (layouts as bc6f_from_bc6h)."""
    records = np.ascontiguousarray(records, np.float32)
    out = np.zeros((h // 4) * (w // 4) * ((channels + 2) // 3) * 16, np.uint8)
    _codec_lib().nto_bc6f_to_bc6h_surface(_p(records, f32p), w, h, channels, out.ctypes.data_as(_u8p))
    return out


def random_blocks(rng, w: int, h: int, channels: int) -> np.ndarray:
    """Seeded BC6 block features for a w x h grid: endpoints U(-1, 1), pixel indices U(0, 1),
    random partition (0..31) and mode (0..9); float32 [blocks * triples * 32]."""
    T = (channels + 2) // 3
    nb = (w // 4) * (h // 4) * T
    p = np.zeros((nb, 32), np.float32)
    p[:, :12] = rng.uniform(-1, 1, (nb, 12))
    p[:, 12:28] = rng.uniform(0, 1, (nb, 16))
    p[:, 28].view(np.int32)[:] = rng.integers(0, 32, nb)
    p[:, 29].view(np.int32)[:] = rng.integers(0, 10, nb)
    return p.reshape(-1)
