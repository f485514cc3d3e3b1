"""Host-side checks of the tcgen05 planner and of the stream-K work split, through the
library's diagnostic exports (no GPU needed: both are the same host/device code the launches
use).

Stream-K: worker w of G owns k-blocks [w T / G, (w + 1) T / G) of the T = tiles x k-blocks
laid out tile after tile; a tile split between workers is finished by the worker holding its
first k-blocks, which adds the tail parts of the workers after it.  The invariants below are
what the kernel relies on: every k-block belongs to exactly one piece, a tail part is always a
worker's first piece and a head part its last (so no worker waits on another while it still
owes work), and a head's contributors are exactly the tail parts of its tile, in k order.
"""
import ctypes
import random

import pytest

SMS = 148


@pytest.fixture(scope="module")
def L():
    from spinn_b200 import lib
    return lib.lib()


@pytest.fixture(autouse=True)
def _no_forced_tiles(monkeypatch):
    monkeypatch.delenv("SPINN_TC_TILES", raising=False)


def _pieces(L, tiles, kb, w, G):
    out = (ctypes.c_int * 4)()
    res = []
    i = 0
    while True:
        rc = L.spinn_cuda_diag_streamk_piece(tiles, kb, w, G, i, out)
        assert rc in (0, 1), rc
        if rc == 0:
            return res
        res.append(tuple(out))
        i += 1


def _check_split(L, tiles, kb, G):
    owner = {}
    heads = {}
    tails = {}
    for w in range(G):
        ps = _pieces(L, tiles, kb, w, G)
        assert ps, "every worker has work when T >= G"
        for i, (t, k0, k1, kind) in enumerate(ps):
            assert 0 <= t < tiles and 0 <= k0 < k1 <= kb
            assert kind == (1 if k0 > 0 else 2 if k1 < kb else 0)
            if kind == 1:
                assert i == 0, "a tail part is only ever a worker's first piece"
                tails[w] = (t, k0, k1)
            if kind == 2:
                assert i == len(ps) - 1, "a head part is only ever a worker's last piece"
                heads[t] = (w, k1)
            for k in range(k0, k1):
                assert (t, k) not in owner
                owner[(t, k)] = w
    assert len(owner) == tiles * kb
    for t, (w, k1) in heads.items():
        got = []
        j = w + 1
        while L.spinn_cuda_diag_streamk_contributes(tiles, kb, j, G, t):
            tt, a, b = tails[j]
            assert tt == t
            got.extend(range(a, b))
            j += 1
        assert got == list(range(k1, kb)), (tiles, kb, G, t)
    for j, (t, _, _) in tails.items():
        assert t in heads and heads[t][0] < j


def test_streamk_split_resnet_shapes(L):
    # 14x14 3x3 at 64 / 128 / 256 images on 74 pairs, the 7x7 512-channel 3x3 at 256
    for tiles, kb, G in ((49, 36, 74), (98, 36, 74), (196, 36, 74), (98, 72, 74), (25, 36, 74)):
        _check_split(L, tiles, kb, G)


def test_streamk_split_random(L):
    rng = random.Random(7)
    done = 0
    while done < 300:
        tiles, kb, G = rng.randint(1, 400), rng.randint(1, 80), rng.randint(1, SMS)
        if tiles * kb < G:
            continue
        _check_split(L, tiles, kb, G)
        done += 1


def test_streamk_split_rejects_too_few_kblocks(L):
    from spinn_b200 import lib
    out = (ctypes.c_int * 4)()
    assert L.spinn_cuda_diag_streamk_piece(2, 3, 0, 7, 0, out) == lib.EINVAL


def _plan(L, m, n, k, cb=32, res=False, taps=1, sk=True):
    out = (ctypes.c_int * 7)()
    assert L.spinn_cuda_diag_tile_plan(m, n, k, cb, int(res), SMS, taps, int(sk), out) == 0
    return dict(zip(("bn", "pair", "bk", "ms", "wr", "ksplit", "sk"), tuple(out)))


def test_planner_takes_streamk_for_short_last_waves(L):
    # the 7x7 512-channel 3x3 layer at 256 images: 98 pair tiles of 72 k-blocks on 74 slots
    p = _plan(L, 256 * 49, 512, 4608, taps=9)
    assert p["sk"] == 1 and p["ksplit"] == 1, p
    assert _plan(L, 256 * 49, 512, 4608, taps=9, sk=False)["sk"] == 0
    # the 14x14 3x3 layer at 128 images (1.32 waves of pairs)
    assert _plan(L, 128 * 196, 256, 2304, taps=9)["sk"] == 1


def test_planner_keeps_whole_tiles_elsewhere(L):
    # 14x14 3x3 at 64 images (one partial wave: stream-K's fixed cost is not repaid)
    assert _plan(L, 64 * 196, 256, 2304, taps=9)["sk"] == 0
    # the stem at 256 images: many waves, C = 3 padded to 4 (channel blocks of 4), 49 taps
    p = _plan(L, 256 * 112 * 112, 64, 4 * 49, cb=4, taps=49)
    assert p["sk"] == 0, p
    # a fused residual never runs stream-K
    assert _plan(L, 32 * 196, 1024, 256, res=True)["sk"] == 0


def test_planner_forced_streamk(L, monkeypatch):
    monkeypatch.setenv("SPINN_TC_TILES", "256,1,2,64,1,0,1")
    p = _plan(L, 2 * 784, 200, 2304, taps=9)
    assert (p["bn"], p["pair"], p["bk"], p["sk"]) == (256, 2, 64, 1), p
    monkeypatch.setenv("SPINN_TC_TILES", "0,0,0,0,0,0,-1")
    assert _plan(L, 256 * 49, 512, 4608, taps=9)["sk"] == 0


def test_planner_rejects_bad_arguments(L):
    from spinn_b200 import lib
    out = (ctypes.c_int * 7)()
    assert L.spinn_cuda_diag_tile_plan(0, 64, 64, 32, 0, SMS, 1, 1, out) == lib.EINVAL
    assert L.spinn_cuda_diag_tile_plan(64, 64, 64, 12, 0, SMS, 1, 1, out) == lib.EINVAL
