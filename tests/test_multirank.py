"""The N>1 path on CPU: two gloo ranks shard a batch the way bench.py does (even split, each
rank's inputs = its slice of the global batch, no collective on the data path), run their
shard through the C port oracle, and the gathered result equals a single-process run of the
whole batch; the timing reduction takes the max over ranks."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import datetime

    import torch
    import torch.distributed as dist

    import bench
    import oracle
    from spinn_b200 import ennf, netdef
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        gb = 4
        start, stop = bench.shard_bounds(gb, rank, world)
        g = netdef.resnet(50, batch=stop - start, image=32, num_classes=10, seed=7, width=8)
        x = netdef.image_batch(start, stop - start, 32, seed=11)
        y = oracle.PortOracle().run_model(ennf.convert(g), x)
        y = torch.from_numpy(list(y.values())[0].reshape(stop - start, -1).copy())
        parts = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(parts, y)
        tmax = bench.reduce_max(float(rank + 1), dist)
        if rank == 0:
            np.save(os.path.join(out_dir, "gathered.npy"), torch.cat(parts).numpy())
            np.save(os.path.join(out_dir, "tmax.npy"), np.array([tmax]))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_matches_single_process(tmp_path):
    import sys
    sys.path.insert(0, ROOT)
    import bench
    import oracle
    from spinn_b200 import ennf, netdef
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    gathered = np.load(tmp_path / "gathered.npy")
    g = netdef.resnet(50, batch=4, image=32, num_classes=10, seed=7, width=8)
    x = netdef.image_batch(0, 4, 32, seed=11)
    full = list(oracle.PortOracle().run_model(ennf.convert(g), x).values())[0].reshape(4, -1)
    assert np.allclose(gathered, full, rtol=1e-5, atol=1e-5 * np.abs(full).max())
    assert float(np.load(tmp_path / "tmax.npy")[0]) == 2.0
    assert bench.shard_bounds(256, 3, 8) == (96, 128)
    with pytest.raises(ValueError):
        bench.shard_bounds(256, 0, 3)


def test_image_batch_slices_are_consistent():
    from spinn_b200 import netdef
    full = netdef.image_batch(0, 6, 16, seed=1)
    assert np.array_equal(full[2:5], netdef.image_batch(2, 3, 16, seed=1))
