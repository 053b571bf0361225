"""The CPU oracle against the reference's own golden vectors and known answers.

These pin the restatement before anything is compared with it.  Every value
below is transcribed from the reference's tests (tests/golden/reference_goldens.json
cites each source line).
"""
import json
import os

import numpy as np
import pytest

from conftest import SHAPES, assert_bits_equal

GOLD = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "reference_goldens.json")))


def test_chacha12_reproduces_reference_golden_stream(O):
    g = GOLD["rng_golden"]
    rng = O.Rng(int(g["seed"], 16))
    assert [rng.next_u64() for _ in range(8)] == [int(v, 16) for v in g["first_u64"]]


def test_rng_split_u64_across_refill_and_determinism(O):
    # 63 u32 draws leave one word in the buffer; the next u64 straddles a refill.
    a, b = O.Rng(42), O.Rng(42)
    for _ in range(63):
        assert a.next_u32() == b.next_u32()
    x = a.next_u64()
    lo = b.next_u32()
    hi = b.next_u32()
    assert x == (hi << 32) | lo
    assert O.Rng(1).next_u64() != O.Rng(2).next_u64()


def test_cpu_fingerprint_matches_reference_golden(O):
    """tests/golden.rs:77 -- SpMV + fused LIF over SHAPES, FNV-1a of the bits."""
    assert O.golden_fingerprint() == int(GOLD["cpu_fingerprint"]["fnv1a_64"], 16)


def test_half_exhaustive_round_trips(O):
    """src/half.rs:231-265: all 65536 binary16 and bfloat16 patterns."""
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    wide = O.f16_bits_to_f32(allbits)
    back = O.f32_to_f16_bits(wide)
    nan = ((allbits & 0x7C00) == 0x7C00) & ((allbits & 0x03FF) != 0)
    assert np.array_equal(back[~nan], allbits[~nan])
    assert np.all((back[nan] & 0x7C00) == 0x7C00) and np.all((back[nan] & 0x03FF) != 0)
    wb = O.bf16_bits_to_f32(allbits)
    bb = O.f32_to_bf16_bits(wb)
    nanb = ((allbits & 0x7F80) == 0x7F80) & ((allbits & 0x007F) != 0)
    assert np.array_equal(bb[~nanb], allbits[~nanb])
    assert np.all((bb[nanb] & 0x7F80) == 0x7F80) and np.all((bb[nanb] & 0x007F) != 0)


def test_half_known_answers(O):
    for v, want in GOLD["half_cases"]["f16"]:
        assert int(O.f32_to_f16_bits(np.array([v], np.float32))[0]) == int(want, 16)
    for v, want in GOLD["half_cases"]["f16_roundtrip"]:
        got = O.f16_bits_to_f32(O.f32_to_f16_bits(np.array([v], np.float32)))[0]
        assert got == np.float32(want)
    tiny = np.float32(2.0 ** -24)
    assert int(O.f32_to_f16_bits(np.array([tiny]))[0]) == 1
    assert int(O.f32_to_f16_bits(np.array([tiny * np.float32(0.4)]))[0]) == 0
    assert int(O.f32_to_f16_bits(np.array([-tiny * np.float32(0.4)]))[0]) == 0x8000
    # bfloat16 ties to even, and f32::MAX rounds past the largest finite value.
    assert O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.array([1 + 2.0 ** -8], np.float32)))[0] == 1.0
    assert np.isinf(O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.array([np.finfo(np.float32).max])))[0])


def test_spike_layout_is_lsb_first(O):
    s = np.zeros(40, np.uint8)
    s[[0, 31, 32]] = 1
    w = O.pack_spikes(s)
    assert [int(x) for x in w] == [int(v, 16) for v in GOLD["spike_layout"]["words"]]
    w33 = O.pack_spikes(np.ones(33, np.uint8))
    assert [int(x) for x in w33] == [int(v, 16) for v in GOLD["spike_layout"]["all_true_33"]]


def test_fma_counterexample_rounds_twice(O):
    """mod.rs:517-521: separate rounding gives exactly 0.0 (a fused FMA does not)."""
    c = GOLD["fma_counterexample"]
    v = np.array([c["v"]], np.float32)
    th = np.array([10.0], np.float32)
    sp = np.zeros(1, np.uint8)
    O.lif_integrate(v, th, np.array([c["current"]], np.float32), sp, np.float32(c["decay"]), 0.0, 0.0)
    assert v[0] == np.float32(0.0)


def _leak_steps(O, n, seed):
    rng = O.Rng(seed)
    out = np.zeros((n, 2), np.float32)
    for i in range(n):
        tau = np.float32(2.0) + np.float32(rng.next_f32()) * np.float32(8.0)
        inp = np.float32(rng.next_f32()) * np.float32(2.0) - np.float32(1.0)
        alpha = np.float32(1.0) / tau
        out[i] = (np.float32(1.0) - alpha, alpha * inp)
    return out


def test_scan_counting_doubling_and_cycle_known_answers(O):
    """tests/scan_backend.rs:322-419."""
    for n in (1, 1023, 1024, 1025, 5000, 60000):
        got = O.scan_sequential(np.tile(np.array([1.0, 1.0], np.float32), (n, 1)))
        assert np.array_equal(got[:, 1], np.arange(1, n + 1, dtype=np.float32))
        assert np.all(got[:, 0] == 1.0)
    got = O.scan_sequential(np.tile(np.array([2.0, 0.0], np.float32), (100, 1)))
    assert np.array_equal(got[:, 0], np.float32(2.0) ** np.arange(1, 101, dtype=np.float32))
    cyc = np.array([[2.0, 1.0], [0.5, 0.5], [1.0, 1.0]], np.float32)
    xs = cyc[np.arange(4 * 1024 + 33) % 3]
    want = O.scan_sequential(xs)
    assert np.all(np.isfinite(want[:, 0])) and np.all(want[:, 0] != 0)


def test_scan_first_prefix_is_copied(O):
    got = O.scan_sequential(np.array([[np.inf, -0.0]], np.float32))
    assert_bits_equal(got, np.array([[np.inf, -0.0]], np.float32))


@pytest.mark.parametrize("n", [0, 1, 2, 16, 255, 256, 257, 512, 1000, 4096])
def test_chunked_scan_matches_sequential(O, n):
    """src/scan.rs:410-433 for every chunk size the reference exercises."""
    xs = _leak_steps(O, n, 0x5CA10000 + n)
    want = O.scan_sequential(xs)
    for cs in (1, 3, 7, 64, 128, 256):
        assert_bits_equal(O.scan_chunked(xs, cs), want, f"chunk={cs} n={n}")


def test_parallel_arms_are_bit_identical(O):
    """tests/honesty.rs:99-249: CPU parallel == CPU sequential."""
    rng = O.Rng(0xB0B)
    for nrows, ncols, deg in [(257, 128, 16), (1000, 1000, 64), (2048, 512, 3)]:
        csr = O.random_csr(nrows, ncols, deg, rng)
        w = O.random_vec(csr.nnz, 1.0, rng)
        x = O.random_vec(ncols, 1.0, rng)
        y0 = O.random_vec(nrows, 1.0, rng)
        ys, yp = y0.copy(), y0.copy()
        O.spmv(csr, w, x, ys, par=False)
        O.spmv(csr, w, x, yp, par=True)
        assert_bits_equal(yp, ys)
        xm = O.random_vec(ncols * 5, 1.0, rng)
        ms, mp = np.zeros(nrows * 5, np.float32), np.zeros(nrows * 5, np.float32)
        O.spmm(csr, w, xm, 5, ms)
        O.spmm(csr, w, xm, 5, mp, par=True)
        assert_bits_equal(mp, ms)


def test_partitions_keep_hub_rows_alone(O):
    """mod.rs:2662-2700: a hub row is its own first part; leaves balance."""
    import ctypes

    hub, leaves = 12000, 3000
    row_ptr = np.array([0, hub] + [hub + i + 1 for i in range(leaves)], np.uint32)
    out = np.zeros(16, np.uint64)
    n = O.lib().or_nnz_balanced_partitions(row_ptr, len(row_ptr) - 1, 8, out)
    parts = out[: 2 * n].reshape(-1, 2)
    assert n == 8 and tuple(parts[0]) == (0, 1)
    leaf = [int(row_ptr[e] - row_ptr[s]) for s, e in parts[1:]]
    assert max(leaf) - min(leaf) <= 1 and sum(leaf) == leaves
    del ctypes


def test_validate_csr_check_order(O):
    """The first failing check in mod.rs:2116-2182 order is reported."""
    assert O.validate_csr([], [], 0, 0)[0] == "EmptyRowPtr"
    assert O.validate_csr([1, 1], [0], 1, 1)[0] == "NonZeroStart"
    assert O.validate_csr([0, 2, 1], [0, 0], 1, 1)[0] == "NotMonotonic"
    assert O.validate_csr([0, 2], [0], 1, 1)[0] == "NnzMismatch"
    assert O.validate_csr([0, 1], [0], 2, 1)[0] == "NcolsMismatch"
    assert O.validate_csr([0, 2], [0, 5], 2, 2)[0] == "ColumnOutOfRange"
    assert O.validate_csr([0, 2], [1, 0], 2, 2)[0] == "RowUnsorted"
    code, sh = O.validate_csr([0, 2, 3], [0, 1, 1], 2, 2)
    assert code == "Ok" and (sh.nrows, sh.ncols, sh.nnz, sh.max_row_nnz) == (2, 2, 3, 2)


def test_csc_is_stable(O):
    """sparse.rs:720-749: entries of one column keep CSR order."""
    csr = O.Csr.from_adjacency([[1, 2], [0], [0, 1]])
    cp, row, eidx = O.csc_from_csr(csr, csr.ncols)
    assert list(cp) == [0, 2, 4, 5]
    assert list(row) == [1, 2, 0, 2, 0] and list(eidx) == [2, 3, 0, 4, 1]


@pytest.mark.parametrize("shape", SHAPES)
def test_oracle_fused_matches_unfused_order(O, shape):
    """fused == row_dot then lif_step, bit for bit (mod.rs:2503-2545)."""
    nrows, ncols, deg = shape
    rng = O.Rng(0x5EED + nrows)
    csr = O.random_csr(nrows, ncols, deg, rng)
    w = O.random_vec(csr.nnz, 1.0, rng)
    x = O.random_vec(ncols, 1.0, rng)
    v = O.random_vec(nrows, 0.5, rng)
    th = np.abs(O.random_vec(nrows, 0.5, rng))
    cur = np.zeros(nrows, np.float32)
    O.spmv(csr, w, x, cur)
    v1, t1, s1 = v.copy(), th.copy(), np.zeros(nrows, np.uint8)
    O.lif_integrate(v1, t1, cur, s1, 0.9, 0.0, 0.1)
    v2, t2, s2 = v.copy(), th.copy(), np.zeros(nrows, np.uint8)
    O.fused_lif(csr, w, x, v2, t2, s2, 0.9, 0.0, 0.1)
    assert_bits_equal(v2, v1)
    assert_bits_equal(t2, t1)
    assert np.array_equal(s1, s2)


def test_workload_definition_series_and_streams(O):
    """The benchmark workload's host definition: the ln / cos series agree
    with libm to a few ulp, row streams are the reference Rng's, and the
    multi-block network tick equals recurrent_steps on one CSR."""
    import math

    r = np.random.default_rng(3)
    for u in r.random(2000):
        x = 1.0 - u
        assert abs(O.wl_log(x) - math.log(x)) <= 4e-16 * max(1.0, abs(math.log(x)))
        assert abs(O.wl_cos2pi(u) - math.cos(2 * math.pi * u)) <= 2e-15
    assert O.wl_log(1.0) == 0.0 and O.wl_cos2pi(0.0) == 1.0
    seed, row0, nrows, ncols, fan = 0x77, 5, 4, 1 << 31, 100
    col, w = O.wl_fixed_fanin(seed, row0, nrows, ncols, fan, 0.03)
    for i in range(nrows):
        rr = row0 + i
        rng = O.Rng(seed ^ ((rr * 0x9E3779B97F4A7C15) & (2 ** 64 - 1)))
        want = np.sort(np.array([rng.gen_index(ncols) for _ in range(fan)], np.uint32))
        assert np.array_equal(col[i * fan:(i + 1) * fan], want)
        wr = O.Rng((seed ^ 0x5EED5EED5EED5EED) ^ ((rr * 0x9E3779B97F4A7C15) & (2 ** 64 - 1)))
        for k in range(fan):
            u1, u2 = wr.next_f64(), wr.next_f64()
            z = math.sqrt(-2.0 * O.wl_log(1.0 - u1)) * O.wl_cos2pi(u2)
            assert np.float32(np.float64(np.float32(0.03)) * z) == w[i * fan + k]
    v, th, sp = O.wl_lif_state(9, 32, 64, 0.0, 1.0, 1.0, 0.5)
    for i in range(64):
        rng = O.Rng(9 ^ (((32 + i) * 0x9E3779B97F4A7C15) & (2 ** 64 - 1)))
        f0, f1 = rng.next_f32(), rng.next_f32()
        assert v[i] == np.float32(f0) and sp[i] == (f1 < np.float32(0.5))
    # multi-block ticks == one CSR's recurrent steps
    n, fan = 2048, 40
    col, w = O.wl_fixed_fanin(11, 0, n, n, fan, 0.5)
    rp = (np.arange(n + 1, dtype=np.uint64) * fan).astype(np.uint32)
    v0, t0, s0 = O.wl_lif_state(12, 0, n, 0.0, 1.0, 1.0, 0.05)
    xs, v, t = O.pack_spikes(s0), v0.copy(), t0.copy()
    want = O.recurrent_steps(O.Csr(rp, col, n), w, xs, v, t, np.zeros(n, np.uint8), 0.9, 0.0, 0.0, 7)
    blocks = [((rp[:1025] - rp[0]).astype(np.uint32), col[:1024 * fan], w[:1024 * fan]),
              ((rp[1024:] - rp[1024]).astype(np.uint32), col[1024 * fan:], w[1024 * fan:])]
    xs2, v2, t2 = O.pack_spikes(s0), v0.copy(), t0.copy()
    got = O.net_ticks(blocks, n, xs2, v2, t2, np.zeros(n, np.uint8), 0.9, 0.0, 0.0, 7)
    assert got.tolist() == want.tolist() and want.sum() > 0
    assert np.array_equal(v2.view(np.uint32), v.view(np.uint32)) and np.array_equal(xs2, xs)
