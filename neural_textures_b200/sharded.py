"""Row-sharded training of one material over several GPUs (BASELINE config 4b).

The reference trains one material on one device (main.cpp:1071-1077).  Here a material
too large for one GPU's share of work is split into bands of lattice rows, one per rank;
each rank stores, for every latent grid and for the target, only the band of rows its
samples reach, plus HALO rows on each side:

    stored rows of a grid = [halo above | owned band | halo below]

A training step on rank r is
  1. the training pass over its lattice rows (nt_invoke_training with lattice_row0 /
     lattice_rows and per-source row_origin / stored_rows);
  2. the gradients its samples left in the halo rows go to the neighbours that own those
     rows (two point-to-point phases over NCCL: halo above -> rank r - 1, halo below ->
     rank r + 1), which add them to their bands;
  3. one allreduce (sum) of the MLP weight and bias gradients, kept in one flat buffer;
  4. Adam over the MLP (identical on every rank) and over the owned band of each grid;
  5. the updated band edges go back to the neighbours' halo rows.
So the result equals the single-GPU step up to the order of floating-point additions.
Every rank posts the same collectives in the same order.

The exchanges come in two forms: DistComm runs them over torch.distributed (NCCL on GPUs,
gloo on CPU), LocalShards runs several shards in one process (tests on one GPU).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _native as N
from ._native import check, load
from .api import PAD_IN, PAD_OUT, _device_guard, _on_device, _stream, he_normal_weights, zero_padded_inputs

HALO = 3  # filter reach beyond a band: taps at -2.5 .. +1.5 rows of the band's sample range


@dataclass(frozen=True)
class Band:
    """Rows of one source (height `height`) held by one rank."""
    height: int
    lo: int        # first owned row
    hi: int        # one past the last owned row
    halo: int      # halo rows above and below (0: unsharded)

    @property
    def origin(self) -> int:
        return (self.lo - self.halo) % self.height

    @property
    def stored(self) -> int:
        return self.hi - self.lo + 2 * self.halo

    @property
    def owned(self) -> int:
        return self.hi - self.lo

    def stored_rows_of_full(self) -> np.ndarray:
        """Full row index of every stored row."""
        return (self.origin + np.arange(self.stored)) % self.height


def lattice_band(rank: int, world: int, lattice_h: int) -> tuple[int, int]:
    return rank * lattice_h // world, (rank + 1) * lattice_h // world


def source_band(rank: int, world: int, lattice_h: int, height: int) -> Band:
    """Rows of a source of `height` rows that the samples of rank's lattice band reach.

    Sample rows of lattice band [a, b) lie in [a, b) * height / lattice_h of the source (the
    sample stride is image_h / lattice_h and a source of height h spans the image), so the
    owned rows are that range rounded to the nearest row; consecutive ranks' bands then
    partition the source."""
    a, b = lattice_band(rank, world, lattice_h)
    rnd = lambda x: (2 * x * height + lattice_h) // (2 * lattice_h)
    lo, hi = rnd(a), rnd(b)
    if world == 1:
        return Band(height, 0, height, 0)
    if hi - lo < 2 * HALO or hi - lo + 2 * HALO > height:  # the halo adds at both band edges must not overlap
        raise ValueError(f"rank {rank}: band of {hi - lo} rows of a {height}-row source cannot be sharded "
                         f"{world} ways with a {HALO}-row halo (a band needs at least {2 * HALO} rows)")
    return Band(height, lo, hi, HALO)


class ShardedTexture:
    """Device state of one rank's band of a material: stored rows of both latent grids (fp16)
    with fp32 gradients and Adam moments, the stored rows of the target, and a full copy of
    the network (its gradients in one flat fp32 buffer, the allreduce operand)."""

    def __init__(self, rank: int, world: int, image_w: int, image_h: int, grid_sizes, latent_channels: int,
                 output_channels: int, lattice, device="cuda", latent_lr: float = 1e-2, network_lr: float = 5e-3,
                 beta1: float = 0.9, beta2: float = 0.99, eps: float = 1e-8):
        import torch
        self.torch = torch
        self.rank, self.world = rank, world
        self.device = torch.device(device)
        self.image_w, self.image_h = image_w, image_h
        self.C, self.cout = latent_channels, output_channels
        self.grid_sizes = [tuple(g) for g in grid_sizes]
        self.lattice = tuple(lattice)
        self.lat_band = lattice_band(rank, world, self.lattice[1])
        self.bands = [source_band(rank, world, self.lattice[1], h) for (_, h) in self.grid_sizes]
        self.tband = source_band(rank, world, self.lattice[1], image_h)
        f16, f32 = torch.float16, torch.float32
        z = lambda shape, dt: torch.zeros(shape, dtype=dt, device=self.device)
        self.grids = [z((b.stored, w, self.C), f16) for b, (w, _) in zip(self.bands, self.grid_sizes)]
        self.ggrads = [z(g.shape, f32) for g in self.grids]
        self.gm1 = [z(g.shape, f32) for g in self.grids]
        self.gm2 = [z(g.shape, f32) for g in self.grids]
        self.target = z((self.tband.stored, image_w, self.cout), f16)
        self.W = [z(PAD_OUT[l] * PAD_IN[l], f16) for l in range(3)]
        self.b = [z(64, f16), z(64, f16), z(self.cout, f16)]
        # network gradients: one flat buffer (each piece 16-byte aligned), views per layer
        sizes = [w.numel() for w in self.W] + [b.numel() for b in self.b]
        offs, o = [], 0
        for n in sizes:
            offs.append(o)
            o += (n + 3) // 4 * 4
        self.net_grad = z(o, f32)
        self.gW = [self.net_grad[offs[l]:offs[l] + sizes[l]] for l in range(3)]
        self.gb = [self.net_grad[offs[3 + l]:offs[3 + l] + sizes[3 + l]] for l in range(3)]
        self.mW = [z(w.shape, f32) for w in self.W]
        self.vW = [z(w.shape, f32) for w in self.W]
        self.mb = [z(b.shape, f32) for b in self.b]
        self.vb = [z(b.shape, f32) for b in self.b]
        self.loss_accum = z(1, f32)
        self.workspace = z(int(load().nt_workspace_bytes()) // 4, torch.int32)  # the training pass's tile counter
        self.latent_adam = (beta1, beta2, latent_lr, eps)
        self.network_adam = (beta1, beta2, network_lr, eps)
        self.channel_weights = [1.0] * self.cout
        self.seed = 0
        self.step = 0

    # -- initialisation: the same material as NeuralTexture.init(seed), cut to the stored rows --
    @_on_device
    def init(self, seed: int = 0, target_seed: int | None = None, pbr_normals: bool = False, stream=None):
        torch = self.torch
        L = load()
        for i, (band, (w, h)) in enumerate(zip(self.bands, self.grid_sizes)):
            full = torch.empty((h, w, self.C), dtype=torch.float16, device=self.device)
            check(L.nt_init_latents(full.data_ptr(), full.numel(), seed * 7919 + i + 1, _stream(stream)))
            rows = torch.from_numpy(band.stored_rows_of_full()).to(self.device)
            self.grids[i].copy_(full.index_select(0, rows))
            del full
        Ws = he_normal_weights(seed, self.cout)
        Ws[0] = zero_padded_inputs(Ws[0], 2 * self.C + 8)
        for l in range(3):
            self.W[l].copy_(torch.from_numpy(Ws[l]).to(self.device))
            self.b[l].zero_()
        full = torch.empty((self.image_h, self.image_w, self.cout), dtype=torch.float16, device=self.device)
        ts = seed if target_seed is None else target_seed
        check(L.nt_generate_target(full.data_ptr(), self.image_w, self.image_h, self.cout, ts, int(pbr_normals),
                                   _stream(stream)))
        rows = torch.from_numpy(self.tband.stored_rows_of_full()).to(self.device)
        self.target.copy_(full.index_select(0, rows))
        del full
        for t in self.ggrads + self.gm1 + self.gm2 + self.mW + self.vW + self.mb + self.vb + [self.net_grad]:
            t.zero_()
        self.step = 0

    # -- parameter blocks ------------------------------------------------------------------------
    def _common(self, p: N.NtKernelParams):
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
        p.image_width, p.image_height = self.image_w, self.image_h
        p.lattice_width, p.lattice_height = self.lattice
        p.sample_stride_x = self.image_w / self.lattice[0]
        p.sample_stride_y = self.image_h / self.lattice[1]
        p.num_samples = self.lattice[0] * self.lattice[1]
        p.step = self.step
        p.seed = self.seed

    def train_params(self) -> N.NtKernelParams:
        """Training pass over this rank's lattice rows; sources addressed by full row.  Built
        once (every buffer keeps its address) and updated with the step; refresh_params()
        rebuilds it after a hyper-parameter change."""
        p = self.__dict__.get("_train_p")
        if p is None:
            p = self._train_p = self._build_train_params()
        p.step = self.step
        return p

    def adam_params(self) -> N.NtKernelParams:
        """Adam over the network and the owned band of each grid (halo rows excluded)."""
        p = self.__dict__.get("_adam_p")
        if p is None:
            p = self._adam_p = self._build_adam_params()
        p.step = self.step
        return p

    def refresh_params(self):
        for k in ("_train_p", "_adam_p", "_adam_split"):
            self.__dict__.pop(k, None)

    def _adam_rows(self, rows, network: bool) -> N.NtKernelParams:
        """Adam over band rows [r0, r1) of each grid (rows[i] for grid i, relative to the band),
        with or without the network."""
        p = N.NtKernelParams()
        self._common(p)
        for i in range(2):
            band, f = self.bands[i], p.features[i]
            r0, r1 = rows[i]
            s0 = band.halo + r0
            f.grid = self.grids[i][s0:].data_ptr()
            f.gradients = self.ggrads[i][s0:].data_ptr()
            f.moment1 = self.gm1[i][s0:].data_ptr()
            f.moment2 = self.gm2[i][s0:].data_ptr()
            f.width, f.height = self.grid_sizes[i][0], r1 - r0
        p.target = self.target.data_ptr()
        return p

    def adam_split(self):
        """Adam of a multi-rank step in three parts: (interior, first edge + network, last edge).
        Halo gradients from the neighbours only reach the first and last HALO rows of each band,
        so the interior rows can be updated while the exchange is in flight; Adam is elementwise,
        so the parts give exactly the full update.  None when a band is too thin to split."""
        sp = self.__dict__.get("_adam_split", 0)
        if sp == 0:
            sp = None
            owned = [self.bands[i].owned for i in range(2)]
            e = [min(self.bands[i].halo, owned[i]) for i in range(2)]
            if all(o > 2 * ei for o, ei in zip(owned, e)):
                sp = (self._adam_rows([(e[i], owned[i] - e[i]) for i in range(2)], False),
                      self._adam_rows([(0, e[i]) for i in range(2)], True),
                      self._adam_rows([(owned[i] - e[i], owned[i]) for i in range(2)], False))
            self._adam_split = sp
        if sp is not None:
            for p in sp:
                p.step = self.step
        return sp

    def _build_train_params(self) -> N.NtKernelParams:
        p = N.NtKernelParams()
        self._common(p)
        for i in range(2):
            f = p.features[i]
            f.grid, f.gradients = self.grids[i].data_ptr(), self.ggrads[i].data_ptr()
            f.moment1, f.moment2 = self.gm1[i].data_ptr(), self.gm2[i].data_ptr()
            f.width, f.height = self.grid_sizes[i]
            p.row_origin[i] = self.bands[i].origin
            p.stored_rows[i] = self.bands[i].stored if self.world > 1 else 0
        p.row_origin[2] = self.tband.origin
        p.stored_rows[2] = self.tband.stored if self.world > 1 else 0
        p.target = self.target.data_ptr()
        for c in range(self.cout):
            p.channel_loss_weights[c] = self.channel_weights[c]
        p.lattice_row0 = self.lat_band[0]
        p.lattice_rows = self.lat_band[1] - self.lat_band[0]
        p.loss_accum = self.loss_accum.data_ptr()
        p.workspace = self.workspace.data_ptr()
        p.workspace_bytes = self.workspace.numel() * 4
        return p

    def _build_adam_params(self) -> N.NtKernelParams:
        p = N.NtKernelParams()
        self._common(p)
        for i in range(2):
            band, f = self.bands[i], p.features[i]
            h0 = band.halo
            f.grid = self.grids[i][h0:].data_ptr()
            f.gradients = self.ggrads[i][h0:].data_ptr()
            f.moment1 = self.gm1[i][h0:].data_ptr()
            f.moment2 = self.gm2[i][h0:].data_ptr()
            f.width, f.height = self.grid_sizes[i][0], band.owned
        p.target = self.target.data_ptr()
        return p

    # -- views -------------------------------------------------------------------------------------
    def band_view(self, tensors, i: int):
        b = self.bands[i]
        return tensors[i][b.halo:b.halo + b.owned]

    def halo_above(self, tensors, i: int):
        return tensors[i][:self.bands[i].halo]

    def halo_below(self, tensors, i: int):
        b = self.bands[i]
        return tensors[i][b.halo + b.owned:]

    def band_first(self, tensors, i: int):
        b = self.bands[i]
        return tensors[i][b.halo:2 * b.halo]

    def band_last(self, tensors, i: int):
        b = self.bands[i]
        return tensors[i][b.owned:b.owned + b.halo]

    # -- the step ------------------------------------------------------------------------------------
    @_on_device
    def train_pass(self, stream=None):
        check(load().nt_invoke_training(C.byref(self.train_params()), N.NT_TRAIN_UNCONSTRAINED, _stream(stream)))

    @_on_device
    def adam(self, stream=None):
        check(load().nt_invoke_optimize_all(C.byref(self.adam_params()), _stream(stream)))


# ---- communication -----------------------------------------------------------------------------------

class DistComm:
    """Exchanges over torch.distributed (one process per rank).  A process group created with
    ProcessGroupNCCL.Options(is_high_priority_stream=True) lets the exchanges run beside the
    interior Adam of train_step instead of queueing behind its CTAs."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group

    def exchange(self, sends, recvs):
        """One batched group: sends [(tensor, dst)], recvs [(tensor, src)].  Every rank posts
        its operations in the same order, so the k-th send to a peer meets that peer's k-th
        receive from this rank (which keeps two ranks, where both neighbours are the same
        peer, unambiguous)."""
        self.wait(self.exchange_async(sends, recvs))

    def exchange_async(self, sends, recvs):
        """exchange() without the wait: returns the works (wait() orders the current stream after them)."""
        dist = self.dist
        ops = [dist.P2POp(dist.isend, t, d, self.group) for t, d in sends]
        ops += [dist.P2POp(dist.irecv, t, s, self.group) for t, s in recvs]
        return list(dist.batch_isend_irecv(ops))

    def allreduce(self, t):
        self.dist.all_reduce(t, group=self.group)

    def allreduce_async(self, t):
        return [self.dist.all_reduce(t, group=self.group, async_op=True)]

    @staticmethod
    def wait(works):
        for w in works:
            w.wait()


class _Packed:
    """One contiguous buffer holding the same rows of both grids (flat views), so that each
    neighbour gets one message per exchange instead of one per grid."""

    def __init__(self, views):
        assert all(v.is_contiguous() for v in views), "band and halo rows must be contiguous row ranges"
        self.views = [v.view(-1) for v in views]
        sizes = [v.numel() for v in self.views]
        self.buf = views[0].new_empty(sum(sizes))
        self.parts = list(self.buf.split(sizes))

    def pack(self, torch):
        torch.cat(self.views, out=self.buf)

    def unpack_add(self, torch):
        torch._foreach_add_(self.views, self.parts)

    def unpack_copy(self, torch):
        torch._foreach_copy_(self.views, self.parts)


def _plan(shard):
    """Per-rank exchange buffers, built once: packed halo gradients to send up / down, packed
    receives for the band edges, and the same for the latent rows."""
    pl = shard.__dict__.get("_xplan")
    if pl is not None:
        return pl
    g, lat = shard.ggrads, shard.grids
    both = lambda f, t: [f(t, 0), f(t, 1)]
    pl = shard._xplan = {
        # gradients: my halo above belongs to the rank above (its last rows), my halo below to
        # the rank below (its first rows)
        "g_up": _Packed(both(shard.halo_above, g)), "g_dn": _Packed(both(shard.halo_below, g)),
        "g_last": _Packed(both(shard.band_last, g)), "g_first": _Packed(both(shard.band_first, g)),
        "g_halos": both(shard.halo_above, g) + both(shard.halo_below, g),
        # latents: my first rows fill the upper rank's halo below, my last rows the lower rank's halo above
        "l_first": _Packed(both(shard.band_first, lat)), "l_last": _Packed(both(shard.band_last, lat)),
        "l_below": _Packed(both(shard.halo_below, lat)), "l_above": _Packed(both(shard.halo_above, lat)),
    }
    return pl


def start_gradient_exchange(shard, comm):
    """Packs the halo gradients and posts their exchange (dn's halo above = my last rows, up's
    halo below = my first rows); returns the works to pass to finish_gradient_exchange."""
    torch = shard.torch
    r, n = shard.rank, shard.world
    up, dn = (r - 1) % n, (r + 1) % n
    pl = _plan(shard)
    pl["g_up"].pack(torch)
    pl["g_dn"].pack(torch)
    return comm.exchange_async([(pl["g_up"].buf, up), (pl["g_dn"].buf, dn)],
                               [(pl["g_last"].buf, dn), (pl["g_first"].buf, up)])


def finish_gradient_exchange(shard, comm, works):
    """Waits for the exchange, adds the received gradients to the band edges, clears the halos."""
    torch = shard.torch
    comm.wait(works)
    pl = _plan(shard)
    pl["g_last"].unpack_add(torch)
    pl["g_first"].unpack_add(torch)
    torch._foreach_zero_(pl["g_halos"])


def exchange_gradients(shard, comm):
    """Halo gradients -> owners (added to their bands); halo gradients cleared."""
    if shard.world == 1:
        return
    finish_gradient_exchange(shard, comm, start_gradient_exchange(shard, comm))


def exchange_latents(shard, comm):
    """Updated band edges -> the neighbours' halo rows."""
    r, n = shard.rank, shard.world
    if n == 1:
        return
    torch = shard.torch
    up, dn = (r - 1) % n, (r + 1) % n
    pl = _plan(shard)
    pl["l_first"].pack(torch)
    pl["l_last"].pack(torch)
    comm.exchange([(pl["l_first"].buf, up), (pl["l_last"].buf, dn)],
                  [(pl["l_below"].buf, dn), (pl["l_above"].buf, up)])
    pl["l_below"].unpack_copy(torch)
    pl["l_above"].unpack_copy(torch)


def train_step(shard: ShardedTexture, comm, stream=None):
    """One data-parallel step of the sharded material (every rank calls it).  With several
    ranks, Adam over the band interiors runs while the halo-gradient exchange and the
    network-gradient allreduce are in flight; the band edges and the network follow them."""
    with _device_guard(shard.device):
        _train_step(shard, comm, stream)


def _train_step(shard, comm, stream):
    shard.train_pass(stream)
    if shard.world == 1:
        shard.adam(stream)
        shard.step += 1
        return
    split = shard.adam_split()
    works = start_gradient_exchange(shard, comm)
    works_net = comm.allreduce_async(shard.net_grad)
    if split is None:
        finish_gradient_exchange(shard, comm, works)
        comm.wait(works_net)
        shard.adam(stream)
    else:
        L, s = load(), _stream(stream)
        check(L.nt_invoke_optimize_features(C.byref(split[0]), N.NT_TRAIN_UNCONSTRAINED, s))  # interior
        finish_gradient_exchange(shard, comm, works)
        comm.wait(works_net)
        check(L.nt_invoke_optimize_all(C.byref(split[1]), s))  # network + first edge rows
        check(L.nt_invoke_optimize_features(C.byref(split[2]), N.NT_TRAIN_UNCONSTRAINED, s))  # last edge rows
    exchange_latents(shard, comm)
    shard.step += 1


class LocalShards:
    """All ranks of a sharded material in one process (several bands on one device): the
    same exchanges as DistComm, done with copies.  Used to test the sharded step against
    the unsharded one on a single GPU."""

    def __init__(self, shards: list[ShardedTexture]):
        self.shards = shards

    def step(self, stream=None):
        self.gradients(stream)
        self.apply(stream)

    def gradients(self, stream=None):
        """Training passes, halo gradients to their owners, network gradients summed."""
        sh = self.shards
        n = len(sh)
        for s in sh:
            s.train_pass(stream)
        for i in range(2):
            above = [s.halo_above(s.ggrads, i).clone() for s in sh]
            below = [s.halo_below(s.ggrads, i).clone() for s in sh]
            for r, s in enumerate(sh):
                s.band_last(s.ggrads, i).add_(above[(r + 1) % n])
                s.band_first(s.ggrads, i).add_(below[(r - 1) % n])
                s.halo_above(s.ggrads, i).zero_()
                s.halo_below(s.ggrads, i).zero_()
        total = sum(s.net_grad for s in sh)
        for s in sh:
            s.net_grad.copy_(total)

    def apply(self, stream=None):
        """Adam on every band and the network, then the halo rows refreshed."""
        sh = self.shards
        n = len(sh)
        for s in sh:
            s.adam(stream)
        for i in range(2):
            first = [s.band_first(s.grids, i).clone() for s in sh]
            last = [s.band_last(s.grids, i).clone() for s in sh]
            for r, s in enumerate(sh):
                s.halo_below(s.grids, i).copy_(first[(r + 1) % n])
                s.halo_above(s.grids, i).copy_(last[(r - 1) % n])
        for s in sh:
            s.step += 1

    def gather(self, tensors_of, i: int):
        """Full-height tensor of grid i assembled from the owned bands."""
        return self.shards[0].torch.cat([s.band_view(tensors_of(s), i) for s in self.shards], 0)


def dist_train_step(shards: list[ShardedTexture], streams=None):
    """One step of every shard of a material, driven from this thread through
    nt_dist_train_step: the training passes, then per shard one kernel that adds the
    neighbours' halo gradients to its band edges and runs Adam on the network with the sum
    of all shards' network gradients (read from their memory), Adam over the band, and one
    kernel that refreshes its halo rows from the neighbours' updated bands.  The shards may
    share a device or sit on several; `streams` (one per shard) defaults to each device's
    current stream."""
    torch = shards[0].torch
    n = len(shards)
    arr = (N.NtShard * n)()
    for r, s in enumerate(shards):
        arr[r].params = s.train_params()
        for i in range(2):
            arr[r].halo_rows[i] = s.bands[i].halo
        dev = s.device.index if s.device.index is not None else torch.cuda.current_device()
        arr[r].device = dev
        arr[r].stream = (streams[r] if streams is not None else torch.cuda.current_stream(dev).cuda_stream)
    check(load().nt_dist_train_step(arr, n))
    for s in shards:
        s.step += 1


class NcclComm:
    """One rank's communicator of the C ABI's NCCL path (include/nt_capi.h nt_nccl_*): a process
    (or host thread) per GPU, the halo exchanges and the network-gradient sum over NCCL, the
    step queued on the shard's stream by nt_nccl_train_step.  The exchange workspace is a torch
    buffer on the shard's device."""

    @staticmethod
    def unique_id() -> bytes:
        buf = (C.c_ubyte * N.NT_NCCL_UNIQUE_ID_BYTES)()
        check(load().nt_nccl_unique_id(buf))
        return bytes(buf)

    def __init__(self, uid: bytes, world: int, rank: int, device: int):
        self.world, self.rank, self.device = world, rank, device
        buf = (C.c_ubyte * N.NT_NCCL_UNIQUE_ID_BYTES).from_buffer_copy(uid)
        h = C.c_void_p()
        check(load().nt_nccl_comm_create(buf, world, rank, device, C.byref(h)))
        self.handle = h
        self.workspace = None

    def shard_of(self, shard: ShardedTexture, stream=None) -> N.NtShard:
        torch = shard.torch
        s = N.NtShard()
        s.params = shard.train_params()
        for i in range(2):
            s.halo_rows[i] = shard.bands[i].halo
        s.device = self.device
        s.stream = stream if stream is not None else torch.cuda.current_stream(shard.device).cuda_stream
        return s

    def train_step(self, shard: ShardedTexture, stream=None):
        """One step of this rank's band (every rank calls it); advances shard.step."""
        torch = shard.torch
        s = self.shard_of(shard, stream)
        need = int(load().nt_nccl_workspace_bytes(C.byref(s)))
        if self.workspace is None or self.workspace.numel() < need:
            self.workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=shard.device)
        check(load().nt_nccl_train_step(self.handle, C.byref(s), self.workspace.data_ptr(), self.workspace.numel()))
        shard.step += 1

    def wait(self, timeout_ms: int = 60000):
        """Bounded wait for the last step (NT_ERR_TIMEOUT / NT_ERR_NCCL abort the communicator)."""
        check(load().nt_nccl_comm_wait(self.handle, int(timeout_ms)))

    def close(self):
        if self.handle is not None:
            check(load().nt_nccl_comm_destroy(self.handle))
            self.handle = None
