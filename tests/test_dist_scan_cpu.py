"""The sharded exact scan's host logic (sparsl_b200/dist_scan.py) on CPU:
world size 2 and 3 over gloo, each rank's run computed by the oracle's
sequential fold (src/scan.rs:298-313 restated).  The concatenated output must
equal the single sequential fold bit for bit, whether the guessed entry
states are right at once (contracting maps), wrong and repaired in one round
(a planted bad guess), or wrong on every rank with no contraction at all (a
cascade of repair rounds)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _comb(p, q):
    """(q.a * p.a, q.a * p.b + q.b) in f32, two roundings (scan.rs:127-132)."""
    a = np.float32(q[0]) * np.float32(p[0])
    b = np.float32(q[0]) * np.float32(p[1]) + np.float32(q[1])
    return np.array([a, b], np.float32)


class OracleRun:
    def __init__(self, O, x, plant=None):
        self.O, self.x, self.n, self.plant = O, x, len(x), plant
        self.out = None

    def tail(self, h):
        return self.x[-h:]

    def table(self, k):
        v = np.arange(8, dtype=np.uint32).view(np.float32)
        for a in self.x[k:, 0]:
            v = v * np.float32(a)
        b = v.view(np.uint32)
        return int(sum((int(x) if x <= 7 else 8) << (4 * m) for m, x in enumerate(b)))

    def settle(self):
        a, i = np.float32(self.x[0, 0]), 1
        while i < self.n and int(np.array([a]).view(np.uint32)[0]) > 7:
            a = np.float32(self.x[i, 0]) * a
            i += 1
        return a, i

    def fold(self, prefix):
        st = self.O.scan_sequential(np.ascontiguousarray(prefix))[-1].copy()
        if self.plant is not None:
            st = st + np.float32(self.plant)  # a deliberately wrong guess
        return st

    def _scan(self, entry):
        x2 = self.x.copy()
        if entry is not None:
            x2[0] = _comb(entry, self.x[0])
        return self.O.scan_sequential(x2)

    def scan(self, entry):
        self.out = self._scan(entry)

    def exit_state(self):
        return self.out[-1].copy()

    def rejoin(self, entry):
        exact = self._scan(entry)
        same = np.all(exact.view(np.uint32) == self.out.view(np.uint32), axis=1)
        k = int(np.argmax(same)) if same.any() else self.n
        self.out[:k] = exact[:k]
        return k


def _data(kind, n):
    r = np.random.default_rng(17)
    x = np.empty((n, 2), np.float32)
    if kind == "contracting":  # the config-2 distribution
        x[:, 0] = r.uniform(0.9, 1.0, n)
        x[:, 1] = r.standard_normal(n)
    else:  # a = 1: no contraction, every guess is off
        x[:, 0] = 1.0
        x[:, 1] = r.uniform(-1, 1, n)
    return x.astype(np.float32)


def _rank_main(rank, world, port, kind, n, plant_rank, halo, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import bench
    import oracle as O
    from sparsl_b200 import dist_scan

    dist = bench.Dist()
    try:
        x = _data(kind, n)
        lo, hi = rank * n // world, (rank + 1) * n // world
        run = OracleRun(O, x[lo:hi].copy(), plant=1.0 if rank == plant_rank else None)
        st = dist_scan.sharded_scan(run, rank, world, dist_scan.process_group_all_gather(dist.pg, world), halo=halo)
        q.put((rank, run.out.tobytes(), st.rounds, st.rewritten, st.entry_exact))
    finally:
        dist.close()


@pytest.mark.parametrize("world,kind,n,plant_rank,halo", [
    (2, "contracting", 40_000, -1, 2048),
    (3, "contracting", 30_001, 2, 2048),     # rank 2's guess is planted wrong: one repair round
    (3, "flat", 3_000, -1, 256),             # no contraction: a cascade of repairs
    (3, "contracting", 900, -1, 2048),       # halo covers the whole prefix: exact guesses
])
def test_sharded_scan_equals_sequential(world, kind, n, plant_rank, halo):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, kind, n, plant_rank, halo, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    want = O.scan_sequential(_data(kind, n))
    got = np.concatenate([np.frombuffer(b, np.float32).reshape(-1, 2) for _, b, _, _, _ in res])
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    rounds = {r for _, _, r, _, _ in res}
    assert len(rounds) == 1, "every rank takes the same number of exchange rounds"
    if plant_rank >= 0:
        assert res[plant_rank][3] > 0 and not res[plant_rank][4]
    if kind == "flat":
        assert rounds.pop() >= 1
    if kind == "contracting" and plant_rank < 0:
        # the offset chain's guess contracts onto the trajectory and the
        # multiplier arrives exactly through the tables: no repair at all
        assert all(e for *_, e in res) and res[0][2] == 0
