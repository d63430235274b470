"""Torch restatement of the CPU oracle's training step, for long runs at BASELINE size.

TEST INFRASTRUCTURE ONLY.  The product never imports this module; only tests/ do.  It
restates, tensor-wide, exactly what oracle/nt_oracle.c does per sample, so that the 2,000-step
loss criterion can be checked at BASELINE config-1 size (1024^2 material, 262,144 samples per
step) in seconds on the device instead of the half hour the C oracle needs.  It is pinned to
the C oracle on one pass and one Adam update by tests/test_torch_oracle_cpu.py (CPU).

Each piece follows the C oracle, which follows the reference (mavenkim2/neural_textures):
  sample_uv      nto_sample_uv        train.cu:37-58 (xorshift32), :827-844 (jittered lattice)
  sample_grid    nto_sample_grid      filter/catmull_rom.h:46-59 weights, train.cu:65-69 wrap;
                                      row sums first, then the weighted sum of rows
  posenc         nto_posenc           2 frequencies x (u, v) x (sin, cos), double, then fp16
  forward        nto_forward_sample   mlp.h:18-40 per layer, fp16 at the tensor-core operands
  loss/backward  backward_sample      train.cu:876-888 loss, mlp.h:222-257 per layer; 2 w err
                                      rounded to fp16, 1 / numSamples applied in fp32
  scatter        scatter_latent       train.cu:460-509 with the 16 Catmull-Rom taps
  adam           nto_adam_f16         train.cu:521-543, :566-588 (zero-gradient skip, zeroing)
Differences from the C oracle: the per-layer sums are fp32 matrix products (the C oracle
sums in double) and gradient sums run in a different order, so results agree to fp32
rounding, not bit for bit.
"""
from __future__ import annotations

import math

import numpy as np

PAD_IN = (32, 64, 64)
PAD_OUT = (64, 64, 16)
M32 = 0xFFFFFFFF


def _r16(x):
    return x.half().float()


class TorchTrainer:
    """A material as float32 tensors that hold fp16 values (latents, weights, biases), with fp32
    gradients and Adam moments, trained by `step`."""

    def __init__(self, grids, W, b, target, C, cout, image, lattice, latent_adam, network_adam,
                 channel_weights=None, seed=0, device="cpu"):
        import torch
        self.torch = torch
        self.dev = torch.device(device)
        f = lambda a: torch.from_numpy(np.asarray(a, np.uint16).view(np.float16).astype(np.float32)).to(self.dev)
        self.grids = [f(g) for g in grids]                     # [h][w][C]
        self.W = [f(w).view(PAD_OUT[l], PAD_IN[l]) for l, w in enumerate(W)]
        self.b = [f(x) for x in b]
        self.target = f(target)                                # [H][W][cout]
        self.C, self.cout = C, cout
        self.image = tuple(image)
        self.lattice = tuple(lattice)
        self.seed = seed
        self.latent_adam = latent_adam                         # (beta1, beta2, lr, eps)
        self.network_adam = network_adam
        cw = [1.0] * cout if channel_weights is None else list(channel_weights)
        self.cw = torch.tensor(cw, dtype=torch.float32, device=self.dev)
        z = torch.zeros_like
        self.mW, self.vW = [z(w) for w in self.W], [z(w) for w in self.W]
        self.mb, self.vb = [z(x) for x in self.b], [z(x) for x in self.b]
        self.mg, self.vg = [z(g) for g in self.grids], [z(g) for g in self.grids]

    # ---- sampling ---------------------------------------------------------------------
    def sample_uv(self, step):
        """nto_sample_uv for every lattice cell (train.cu:827-844)."""
        torch = self.torch
        lw, lh = self.lattice
        iw, ih = self.image
        n = lw * lh
        idx = torch.arange(n, dtype=torch.int64, device=self.dev)
        s = idx ^ ((step * 747796405 + 2891336453) & M32) ^ ((self.seed * 0x9E3779B9) & M32)
        s = torch.where(s == 0, torch.ones_like(s), s)

        def nxt(x):
            x = x ^ ((x << 13) & M32)
            x = x ^ (x >> 17)
            x = x ^ ((x << 5) & M32)
            return x

        s = nxt(s)
        jx = (s & 0xFFFFFF).float() * (1.0 / 16777216.0) - 0.5
        s = nxt(s)
        jy = (s & 0xFFFFFF).float() * (1.0 / 16777216.0) - 0.5
        ix = (idx % lw).float()
        iy = (idx // lw).float()
        sx = torch.tensor(float(iw) / lw, dtype=torch.float32, device=self.dev)
        sy = torch.tensor(float(ih) / lh, dtype=torch.float32, device=self.dev)
        px = ((ix + 0.5) + jx) * sx
        py = ((iy + 0.5) + jy) * sy
        px = px.clamp(0.5, float(iw) - 0.5)
        py = py.clamp(0.5, float(ih) - 0.5)
        return px / float(iw), py / float(ih)

    def _taps(self, u, size):
        """Base texel and Catmull-Rom weights along one axis (filter/catmull_rom.h:46-59)."""
        torch = self.torch
        sp = u * float(size)
        fl = torch.floor(sp - 0.5)
        fr = sp - (fl + 0.5)
        w0 = fr * (fr * (fr * -0.5 + 1.0) - 0.5)
        w1 = fr * fr * (fr * 1.5 - 2.5) + 1.0
        w2 = fr * (fr * (fr * -1.5 + 2.0) + 0.5)
        w3 = fr * fr * (fr * 0.5 - 0.5)
        base = fl.long()
        idx = torch.stack([torch.remainder(base - 1 + i, size) for i in range(4)], 1)
        return idx, torch.stack([w0, w1, w2, w3], 1)

    def sample_grid(self, grid, u, v):
        """nto_sample_grid: (values [n][C], flat tap indices [n][4][4], tap weights [n][4][4])."""
        h, w, C = grid.shape
        xi, wx = self._taps(u, w)
        yi, wy = self._taps(v, h)
        flat = yi[:, :, None] * w + xi[:, None, :]              # [n][row j][col i]
        vals = grid.reshape(-1, C)[flat.reshape(-1)].view(-1, 4, 4, C)
        rows = (vals * wx[:, None, :, None]).sum(2)             # row sums over i
        out = (rows * wy[:, :, None]).sum(1)
        return out, flat, wy[:, :, None] * wx[:, None, :]

    def posenc(self, u, v):
        torch = self.torch
        cols = []
        for k in range(2):
            m = float(2 << k)
            au = math.pi * (m * u).double()
            av = math.pi * (m * v).double()
            cols += [torch.sin(au), torch.cos(au), torch.sin(av), torch.cos(av)]
        return torch.stack(cols, 1).float()

    # ---- one pass ---------------------------------------------------------------------
    def train_pass(self, step, scatter=True):
        """Forward, loss and backward of every lattice sample at `step`.  Returns (sse, gW,
        gb, ggrids) with the 1 / numSamples scale applied, like nto_train_pass."""
        torch = self.torch
        u, v = self.sample_uv(step)
        n = u.numel()
        C, cout = self.C, self.cout
        feats, taps = [], []
        for g in self.grids:
            val, flat, wt = self.sample_grid(g, u, v)
            feats.append(_r16(val))
            taps.append((flat, wt))
        x = torch.zeros((n, 32), dtype=torch.float32, device=self.dev)
        x[:, :2 * C] = torch.cat(feats, 1)
        x[:, 2 * C:2 * C + 8] = _r16(self.posenc(u, v))
        W1, W2, W3 = self.W
        h1 = _r16(torch.relu(x @ W1.t() + self.b[0]))
        h2 = _r16(torch.relu(h1 @ W2.t() + self.b[1]))
        y = _r16(h2 @ W3[:cout].t() + self.b[2])
        t, _, _ = self.sample_grid(self.target, u, v)
        err = y - t
        sse = float((self.cw.double() * err.double() ** 2).sum())
        dy = _r16(2.0 * self.cw * err)
        dh2 = torch.where(h2 > 0, _r16(dy @ W3[:cout]), torch.zeros_like(h2))
        dh1 = torch.where(h1 > 0, _r16(dh2 @ W2), torch.zeros_like(h1))
        dx = dh1 @ W1
        scale = 1.0 / float(n)
        gW = [torch.zeros_like(w) for w in self.W]
        gW[2][:cout] = (dy.t() @ h2) * scale
        gW[1][:] = (dh2.t() @ h1) * scale
        gW[0][:] = (dh1.t() @ x) * scale
        gb = [dh1.sum(0) * scale, dh2.sum(0) * scale, dy.sum(0) * scale]
        gg = [torch.zeros_like(g) for g in self.grids]
        if scatter:
            for gi, (flat, wt) in enumerate(taps):
                d = dx[:, gi * C:(gi + 1) * C]
                vals = (wt.reshape(n, 16, 1) * d[:, None, :]) * scale
                gg[gi].view(-1, C).index_add_(0, flat.reshape(-1), vals.reshape(-1, C))
        return sse, gW, gb, gg

    # ---- Adam -------------------------------------------------------------------------
    def _adam(self, w, g, m, v, lr, b1, b2, eps, step):
        torch = self.torch
        t = max(int(step), 1)
        bc1 = np.float32(1.0) - np.float32(np.power(np.float32(b1), np.float32(t)))
        bc2 = np.float32(1.0) - np.float32(np.power(np.float32(b2), np.float32(t)))
        b1t = torch.tensor(b1, dtype=torch.float32, device=self.dev)
        b2t = torch.tensor(b2, dtype=torch.float32, device=self.dev)
        m1 = b1t * m + (1.0 - b1t) * g
        m2 = b2t * v + ((1.0 - b2t) * g) * g
        upd = w - lr * (m1 / float(bc1)) / (torch.sqrt(m2 / float(bc2)) + eps)
        live = g != 0
        m.copy_(torch.where(live, m1, m))
        v.copy_(torch.where(live, m2, v))
        w.copy_(torch.where(live, _r16(upd), w))

    def step(self, step):
        """One training step as the reference driver runs it (main.cpp:1071-1077): the pass,
        then Adam on the network and the latents.  Returns the pass's sum of squared errors."""
        sse, gW, gb, gg = self.train_pass(step)
        b1, b2, lr, eps = self.network_adam
        for l in range(3):
            self._adam(self.W[l], gW[l], self.mW[l], self.vW[l], lr, b1, b2, eps, step)
            self._adam(self.b[l], gb[l], self.mb[l], self.vb[l], lr, b1, b2, eps, step)
        b1, b2, lr, eps = self.latent_adam
        for gi in range(2):
            self._adam(self.grids[gi], gg[gi], self.mg[gi], self.vg[gi], lr, b1, b2, eps, step)
        return sse
