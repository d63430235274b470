"""Shared builders for the parity tests: one seeded material, uploaded to the device through
the product API and handed unchanged (fp16 bit patterns) to the CPU oracle."""
from __future__ import annotations

import numpy as np


def make_texture(image, grids, C, cout, lattice=None, seed=0, device="cuda:0", **kw):
    import neural_textures_b200 as nt
    tex = nt.NeuralTexture(image[0], image[1], grid_sizes=grids, latent_channels=C, output_channels=cout,
                           device=device, lattice=lattice, **kw)
    tex.init(seed=seed)
    # non-zero biases exercise the bias paths (the reference initialises them to zero)
    rng = np.random.default_rng(seed + 99)
    import torch
    for l, n in enumerate((64, 64, cout)):
        tex.b[l].copy_(torch.from_numpy((rng.standard_normal(n) * 0.1).astype(np.float16)).to(tex.device))
    return tex


def oracle_model(O, tex):
    grids, W, b = tex.host_model()
    return O.OracleModel(channels=tex.C, cout=tex.cout, grids=grids, W=W, b=b)


def target_host(tex):
    import torch
    return tex.target.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a))


def max_rel(a, b, floor=1.0):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), floor)))
