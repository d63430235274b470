"""Row-sharded training over NCCL between real GPUs (one process per GPU).

Each rank trains its band of a small material with the NCCL halo exchanges and network
allreduce, and also runs the unsharded step of the same material on its own GPU; after
the steps its owned rows must match the unsharded result (same tolerances as the
single-GPU shard test).  Skipped when fewer than two GPUs are visible."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import numpy as np
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    ok = False
    try:
        import neural_textures_b200 as nt
        from neural_textures_b200.sharded import DistComm, ShardedTexture, train_step
        args = ((256, 256), ((128, 128), (64, 64)), 8, 8, (128, 128))
        image, grids, Cc, cout, lattice = args
        ref = nt.NeuralTexture(*image, grid_sizes=grids, latent_channels=Cc, output_channels=cout, lattice=lattice,
                               device=dev)
        ref.init(seed=7)
        sh = ShardedTexture(rank, world, *image, grids, Cc, cout, lattice, device=dev)
        sh.init(seed=7)
        comm = DistComm()
        for _ in range(3):
            ref.train_step()
            train_step(sh, comm)
        torch.cuda.synchronize(dev)
        ok = True
        for i in range(2):
            b = sh.bands[i]
            got = sh.band_view(sh.grids, i).float().cpu().numpy()
            exp = ref.grids[i][b.lo:b.hi].float().cpu().numpy()
            diff = np.abs(got - exp)
            ok = ok and bool(np.mean(diff > 1e-3) < 0.01 and diff.max() <= 6e-2 + 1e-3)
        w = [torch.zeros_like(sh.W[0]) for _ in range(world)]
        dist.all_gather(w, sh.W[0])
        ok = ok and all(torch.equal(w[0], x) for x in w)  # the network stays replicated
    finally:
        q.put((rank, ok))
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def test_nccl_sharded_steps_match_unsharded(cuda):
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(res.values()), res
