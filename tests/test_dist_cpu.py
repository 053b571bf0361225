"""The multi-rank network tick's host-side logic on CPU, world size 2 over gloo.

Each rank owns a contiguous row block of a recurrent network.  Per tick it runs
the fused spike-SpMV + LIF over its rows (here with the oracle), packs its
slice of the spike vector, and the ranks all-gather the packed words -- the
exchange the CUDA path does with one in-place ncclAllGather.  Row-local sums
make the global trace independent of the number of ranks, so it must equal the
single-process recurrent run bit for bit.  Also covers bench.py's plumbing
(barrier, max over ranks, id broadcast, trace gather) and its row-block split.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT

N, DEG, STEPS = 2048, 48, 12


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _network():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    rng = O.Rng(0xD157)
    csr = O.random_csr(N, N, DEG, rng)
    w = O.random_vec(csr.nnz, 0.6, rng)
    v0 = O.random_vec(N, 1.0, rng)
    t0 = np.full(N, 0.45, np.float32)
    xs0 = O.pack_spikes((np.random.default_rng(5).random(N) < 0.05).astype(np.uint8))
    return O, csr, w, v0, t0, xs0


def _rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    import torch
    import bench

    dist = bench.Dist()
    try:
        O, csr, w, v0, t0, xs0 = _network()
        local = N // world
        r0 = rank * local
        rp = (csr.row_ptr[r0:r0 + local + 1] - csr.row_ptr[r0]).astype(np.uint32)
        blk = O.Csr(rp, csr.col[csr.row_ptr[r0]:csr.row_ptr[r0 + local]], N)
        wl = w[csr.row_ptr[r0]:csr.row_ptr[r0 + local]]
        v, t, sp, xs = v0[r0:r0 + local].copy(), t0[r0:r0 + local].copy(), np.zeros(local, np.uint8), xs0.copy()
        trace = []
        for _ in range(STEPS):
            O.fused_spikes_lif(blk, wl, xs, v, t, sp, 0.95, 0.0, 0.0)
            mine = torch.from_numpy(O.pack_spikes(sp).view(np.int32).copy())
            parts = [torch.zeros_like(mine) for _ in range(world)]
            dist.pg.all_gather(parts, mine)
            xs = torch.cat(parts).numpy().view(np.uint32).copy()
            trace.append(int(sum(bin(int(x)).count("1") for x in xs)))
        # bench.py plumbing
        dist.barrier()
        assert dist.max(float(rank + 1)) == float(world)
        blob = dist.bcast_bytes(b"id-bytes" if rank == 0 else None)
        assert blob == b"id-bytes"
        traces = dist.gather(trace)
        q.put((rank, trace, all(tr == traces[0] for tr in traces), v.tobytes(), t.tobytes()))
    finally:
        dist.close()


def test_two_rank_network_tick_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    O, csr, w, v0, t0, xs0 = _network()
    vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(N, np.uint8), xs0.copy()
    want = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, STEPS)
    for rank, trace, same, vb, tb in res:
        assert same, "ranks disagree on the global spike trace"
        assert trace == list(want)
        local = N // world
        assert np.frombuffer(vb, np.float32).view(np.uint32).tolist() == \
            vw[rank * local:(rank + 1) * local].view(np.uint32).tolist()


@pytest.mark.parametrize("local,fan", [(4_194_304, 1024), (2_097_152, 1024), (524_288, 1024), (1000, 7)])
def test_row_blocks_respect_the_u32_offset_limit(local, fan):
    sys.path.insert(0, ROOT)
    import bench

    blocks = bench.net_blocks(local, fan)
    assert blocks[0][0] == 0 and sum(n for _, n in blocks) == local
    for (off, n), nxt in zip(blocks, blocks[1:] + [(local, 0)]):
        assert off + n == nxt[0]
        assert n * fan <= 1 << 31
        assert off % 32 == 0


# bench.py's CPU check of the sharded network: each rank draws its rows from
# the workload definition, splits them into row blocks, and runs
# bench.cpu_net_ticks (oracle ticks + gloo all-gather of the packed words).
WL_N, WL_FAN, WL_SEED, WL_TICKS = 4096, 96, 0xC0FFEE, 6


def _wl_rank_main(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import bench
    import oracle as O

    dist = bench.Dist()
    try:
        local = WL_N // world
        row0 = rank * local
        host = []
        for off, k in ((0, local // 2), (local // 2, local - local // 2)):
            col, w = O.wl_fixed_fanin(WL_SEED, row0 + off, k, WL_N, WL_FAN, 0.4)
            rp = (np.arange(k + 1, dtype=np.uint64) * WL_FAN).astype(np.uint32)
            host.append((rp, col, w, row0 + off))
        v, th, s0 = O.wl_lif_state(WL_SEED ^ 1, 0, WL_N, 0.0, 1.0, 1.0, 0.05)
        trace, vv, tt, pk, _ = bench.cpu_net_ticks(O, dist, host, WL_N, v[row0:row0 + local].copy(),
                                                   th[row0:row0 + local].copy(), O.pack_spikes(s0), WL_TICKS)
        q.put((rank, trace.tolist(), vv.tobytes(), tt.tobytes(), pk.tobytes()))
    finally:
        dist.close()


def test_bench_cpu_check_over_two_ranks_matches_one_process():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_wl_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # One process: the whole network as one CSR, the reference's recurrent ticks.
    col, w = O.wl_fixed_fanin(WL_SEED, 0, WL_N, WL_N, WL_FAN, 0.4)
    rp = (np.arange(WL_N + 1, dtype=np.uint64) * WL_FAN).astype(np.uint32)
    v, th, s0 = O.wl_lif_state(WL_SEED ^ 1, 0, WL_N, 0.0, 1.0, 1.0, 0.05)
    xs = O.pack_spikes(s0)
    want = O.recurrent_steps(O.Csr(rp, col, WL_N), w, xs, v, th, np.zeros(WL_N, np.uint8), 0.95, 0.0, 0.0, WL_TICKS,
                             par=True)
    assert want.sum() > 0, "the test network should spike"
    local = WL_N // world
    for rank, trace, vb, tb, pb in res:
        assert trace == want.tolist()
        assert np.frombuffer(vb, np.uint32).tolist() == v[rank * local:(rank + 1) * local].view(np.uint32).tolist()
        assert np.frombuffer(tb, np.uint32).tolist() == th[rank * local:(rank + 1) * local].view(np.uint32).tolist()
        assert np.frombuffer(pb, np.uint32).tolist() == xs.tolist()
