"""Row-sharded training through the C ABI's NCCL path (nt_nccl_*, one process per GPU) against
the unsharded step: each rank steps its band with nt_nccl_train_step (halo exchanges and the
network-gradient sum over NCCL), waits with the bounded nt_nccl_comm_wait, and also runs the
unsharded step of the same material on its GPU; after the steps its owned rows must match
the unsharded result (the tolerances of the other sharded tests) and the network must be
identical on every rank.  Skipped with fewer than two GPUs."""
import hashlib
import os

import pytest

pytestmark = pytest.mark.gpu

CASES = [  # image, grids, C, cout, lattice
    ((256, 256), ((128, 128), (64, 64)), 8, 8, (128, 128)),
    ((192, 256), ((96, 128), (48, 64)), 12, 12, (96, 128)),
]


def _worker(rank, world, uid, case, q):
    import numpy as np
    import torch
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    ok, digest, msg = False, "", ""
    comm = None
    try:
        import neural_textures_b200 as nt
        from neural_textures_b200.sharded import NcclComm, ShardedTexture
        image, grids, Cc, cout, lattice = CASES[case]
        ref = nt.NeuralTexture(*image, grid_sizes=grids, latent_channels=Cc, output_channels=cout, lattice=lattice,
                               device=dev)
        ref.init(seed=7)
        sh = ShardedTexture(rank, world, *image, grids, Cc, cout, lattice, device=dev)
        sh.init(seed=7)
        comm = NcclComm(uid, world, rank, rank)
        for _ in range(3):
            ref.train_step()
            comm.train_step(sh)
            comm.wait(60000)
        torch.cuda.synchronize(dev)
        ok = True
        for i in range(2):
            b = sh.bands[i]
            got = sh.band_view(sh.grids, i).float().cpu().numpy()
            exp = ref.grids[i][b.lo:b.hi].float().cpu().numpy()
            diff = np.abs(got - exp)
            ok = ok and bool(np.mean(diff > 1e-3) < 0.01 and diff.max() <= 6e-2 + 1e-3)
            # the halo rows hold the neighbours' updated band edges
            rows = b.stored_rows_of_full()
            full = ref.grids[i].float().cpu().numpy()[rows]
            hd = np.abs(sh.grids[i].float().cpu().numpy() - full)
            ok = ok and bool(np.mean(hd > 1e-3) < 0.01 and hd.max() <= 6e-2 + 1e-3)
        digest = hashlib.sha256(b"".join(w.cpu().numpy().tobytes() for w in sh.W + sh.b)).hexdigest()
        msg = f"steps {sh.step}"
    except Exception as e:  # reported to the parent
        msg = repr(e)
    finally:
        if comm is not None:
            comm.close()
        q.put((rank, ok, digest, msg))


@pytest.mark.parametrize("case", range(len(CASES)))
def test_nccl_capi_steps_match_unsharded(cuda, case):
    import torch
    import torch.multiprocessing as mp
    from neural_textures_b200.sharded import NcclComm
    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs two GPUs")
    uid = NcclComm.unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, ok, digest, msg = q.get(timeout=300)
        res[r] = (ok, digest, msg)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(v[0] for v in res.values()), res
    assert len({v[1] for v in res.values()}) == 1, res  # the network stays replicated
