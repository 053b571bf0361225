"""The TMA-pipelined row fold (operators whose rows all have the same length)
against the oracle and against the generic row-fold kernel, bit for bit."""
import numpy as np
import pytest

from conftest import assert_bits_equal

import sparsl_b200 as S

pytestmark = pytest.mark.gpu


def _uniform(O, nrows, ncols, L, seed):
    r = np.random.default_rng(seed)
    col = np.sort(r.integers(0, ncols, size=(nrows, L), dtype=np.uint32), axis=1).reshape(-1)
    rp = (np.arange(nrows + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = r.uniform(-1, 1, nrows * L).astype(np.float32)
    return O.Csr(rp, col, ncols), w


def _prepare(dev, csr, w, precision, generic):
    op = dev.prepare_with(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w, precision)
    if generic:
        op.force_plain_row_fold()
        assert not op.layouts() & 1
    return op


@pytest.mark.parametrize("nrows,ncols,L", [(1, 64, 8), (31, 100, 32), (33, 1000, 40), (129, 4096, 64),
                                           (1000, 1000, 96), (5000, 70000, 512), (300, 5000, 1024)])
@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_uniform_rows_spmv_and_fused_bit_exact(O, cuda_device, nrows, ncols, L, precision):
    csr, w = _uniform(O, nrows, ncols, L, nrows * 7 + L)
    wq = O.quantise(int(precision), w)
    op = _prepare(cuda_device, csr, w, precision, generic=False)
    ref = _prepare(cuda_device, csr, w, precision, generic=True)
    r = np.random.default_rng(L)
    x = r.uniform(-1, 1, ncols).astype(np.float32)
    y0 = r.uniform(-1, 1, nrows).astype(np.float32)
    got, gen = y0.copy(), y0.copy()
    op.spmv(x, got)
    ref.spmv(x, gen)
    want = O.spmv(csr, wq, x, y0.copy())
    assert_bits_equal(got, want, "spmv vs oracle")
    assert_bits_equal(gen, want, "generic path vs oracle")
    s = (r.random(ncols) < 0.3).astype(np.uint8)
    pk = O.pack_spikes(s)
    got = y0.copy()
    op.spmv_spikes(pk, got)
    assert_bits_equal(got, O.spmv_spikes(csr, wq, pk, y0.copy()), "spmv_spikes")
    v0 = r.uniform(-1, 1, nrows).astype(np.float32)
    t0 = np.abs(r.uniform(-1, 1, nrows)).astype(np.float32)
    v, t, sp = v0.copy(), t0.copy(), np.zeros(nrows, np.bool_)
    op.fused_spmv_spikes_lif(pk, v, t, sp, S.LifParams.new(0.9, 0.0, 0.1))
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(nrows, np.uint8)
    O.fused_spikes_lif(csr, wq, pk, vw, tw, sw, 0.9, 0.0, 0.1)
    assert_bits_equal(v, vw, "fused v")
    assert_bits_equal(t, tw, "fused theta")
    assert np.array_equal(sp.astype(np.uint8), sw)


@pytest.mark.parametrize("n,L", [(4096, 64), (32768, 512), (262144, 512), (60_000, 64), (600_000, 64)])
def test_uniform_recurrent_network_bit_exact(O, cuda_device, n, L):
    """The fixed fan-in network tick (trace, state, device-compacted indices).
    600,000 rows read the spike vector through the shared-memory summary and
    launch 16 warps per CTA (18,750 tiles: whichever of 12, 14, 16 leaves the
    fewest tiles on the busiest warp); the others launch 12."""
    r = np.random.default_rng(n)
    col = np.sort(r.integers(0, n, size=(n, L), dtype=np.uint32), axis=1).reshape(-1)
    rp = (np.arange(n + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = (r.standard_normal(n * L) * 0.05).astype(np.float32)
    csr = O.Csr(rp, col, n)
    v0 = r.random(n).astype(np.float32)
    t0 = np.ones(n, np.float32)
    pk0 = O.pack_spikes((r.random(n) < 0.02).astype(np.uint8))
    op = cuda_device.prepare(S.Csr(rp, col, n), n, w)
    op.write_x_spikes(pk0)
    op.write_lif_state(v0, t0)
    steps = 6
    op.fused_spmv_spikes_lif_recurrent_steps(S.LifParams.new(0.95, 0.0, 0.0), steps)
    vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(n, np.uint8), pk0.copy()
    trace = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, steps, par=True)
    assert np.array_equal(op.spike_trace(), trace)
    v, t, sp = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.bool_)
    op.sync_lif_state(v, t, sp)
    assert_bits_equal(v, vw)
    assert np.array_equal(op.sync_x_spikes(), xw)
    assert np.array_equal(op.spike_indices(), np.flatnonzero(sw).astype(np.uint32))


def test_uniform_rows_with_non_finite_weights(O, cuda_device):
    """inf * cleared spike is NaN on the TMA path too (spikes_backend.rs:48-89)."""
    csr, w = _uniform(O, 64, 256, 32, 5)
    w[3] = np.inf
    w[40] = np.nan
    s = np.ones(256, np.uint8)
    s[csr.col[3]] = 0
    pk = O.pack_spikes(s)
    op = cuda_device.prepare(S.Csr(csr.row_ptr, csr.col, 256), 256, w)
    got = np.zeros(64, np.float32)
    op.spmv_spikes(pk, got)
    want = O.spmv_spikes(csr, w, pk, np.zeros(64, np.float32))
    assert_bits_equal(got, want)
    assert np.isnan(got[0]) and np.isnan(got[1])


@pytest.mark.parametrize("ncols,density", [(600_000, 0.01), (600_000, 0.6), (5_000_000, 0.001),
                                           (20_000_000, 0.05)])
@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16])
def test_uniform_rows_spike_operand_beyond_shared_memory(O, cuda_device, ncols, density, precision):
    """Spike bitmasks too large for shared memory are gathered through a
    per-CTA summary of nonzero column groups; results stay bit-exact at every
    density, including non-finite weights on cleared spikes."""
    nrows, L = 3000, 40
    csr, w = _uniform(O, nrows, ncols, L, ncols % 1000 + L)
    w[5] = np.inf
    w[L * 7 + 3] = np.nan
    wq = O.quantise(int(precision), w)
    op = _prepare(cuda_device, csr, w, precision, generic=False)
    r = np.random.default_rng(ncols)
    s = (r.random(ncols) < density).astype(np.uint8)
    s[csr.col[5]] = 0
    pk = O.pack_spikes(s)
    y0 = r.uniform(-1, 1, nrows).astype(np.float32)
    got = y0.copy()
    op.spmv_spikes(pk, got)
    want = O.spmv_spikes(csr, wq, pk, y0.copy())
    assert_bits_equal(got, want, "spmv_spikes")
    assert np.isnan(got[0]) and np.isnan(got[7])


def test_uniform_recurrent_network_spike_operand_beyond_shared_memory(O, cuda_device):
    """The compacting network tick with a bitmask gathered through the summary."""
    n, L = 600_000, 16
    r = np.random.default_rng(77)
    col = np.sort(r.integers(0, n, size=(n, L), dtype=np.uint32), axis=1).reshape(-1)
    rp = (np.arange(n + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = (r.standard_normal(n * L) * 0.4).astype(np.float32)
    csr = O.Csr(rp, col, n)
    v0 = r.random(n).astype(np.float32)
    t0 = np.full(n, 0.8, np.float32)
    pk0 = O.pack_spikes((r.random(n) < 0.05).astype(np.uint8))
    op = cuda_device.prepare(S.Csr(rp, col, n), n, w)
    vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(n, np.uint8), pk0.copy()
    trace = []
    op.write_x_spikes(pk0)
    op.write_lif_state(v0, t0)
    for steps in (3, 4):  # two calls: the second reuses the ticket counters and flags
        op.fused_spmv_spikes_lif_recurrent_steps(S.LifParams.new(0.95, 0.0, 0.0), steps)
        trace += list(O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, steps, par=True))
        assert np.array_equal(op.spike_trace(), trace[-steps:])
        assert np.array_equal(op.spike_indices(), np.flatnonzero(sw).astype(np.uint32))
    assert sum(trace) > 1000
    v, t, sp = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.bool_)
    op.sync_lif_state(v, t, sp)
    assert_bits_equal(v, vw)
    assert_bits_equal(t, tw)
    assert np.array_equal(op.sync_x_spikes(), xw)


@pytest.mark.parametrize("generic", [False, True])
def test_f16_weights_every_binary16_pattern(O, cuda_device, generic):
    """Every one of the 65,536 binary16 patterns as a weight, through the TMA
    path and the generic path: each row folds one pattern followed by +0
    entries against x = 1, so y is the widened weight (NaN patterns compare as
    NaN, -0 becomes +0 exactly as in the reference's fold)."""
    pats = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    wide = O.f16_bits_to_f32(pats)
    nrows, L = 65536, 8
    col = np.tile(np.arange(L, dtype=np.uint32), nrows)
    rp = (np.arange(nrows + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = np.zeros((nrows, L), np.float32)
    w[:, 0] = wide
    w = w.reshape(-1)
    csr = O.Csr(rp, col, L)
    op = _prepare(cuda_device, csr, w, S.WeightPrecision.F16, generic=generic)
    x = np.ones(L, np.float32)
    got = np.zeros(nrows, np.float32)
    op.spmv(x, got)
    want = O.spmv(csr, O.quantise(int(S.WeightPrecision.F16), w), x, np.zeros(nrows, np.float32))
    assert_bits_equal(got, want, f"all binary16 patterns generic={generic}")


def test_recurrent_index_list_over_several_compaction_rounds(O, cuda_device):
    """The ascending spike index list of a tick on the TMA path comes from a
    separate one-block compaction over the packed words: 300,007 cells are
    9,376 words (two rounds of 8,192) with a ragged last word."""
    n, L = 300_007, 16
    r = np.random.default_rng(300)
    col = np.sort(r.integers(0, n, size=(n, L), dtype=np.uint32), axis=1).reshape(-1)
    rp = (np.arange(n + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = (r.standard_normal(n * L) * 0.4).astype(np.float32)
    csr = O.Csr(rp, col, n)
    v0 = r.random(n).astype(np.float32)
    t0 = np.full(n, 0.8, np.float32)
    pk0 = O.pack_spikes((r.random(n) < 0.05).astype(np.uint8))
    op = cuda_device.prepare(S.Csr(rp, col, n), n, w)
    assert op.layouts() & 1, "uniform rows take the TMA path"
    op.write_x_spikes(pk0)
    op.write_lif_state(v0, t0)
    vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(n, np.uint8), pk0.copy()
    steps = 4
    op.fused_spmv_spikes_lif_recurrent_steps(S.LifParams.new(0.95, 0.0, 0.0), steps)
    trace = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, steps, par=True)
    assert np.array_equal(op.spike_trace(), trace)
    idx = op.spike_indices()
    assert np.array_equal(idx, np.flatnonzero(sw).astype(np.uint32))
    assert sum(trace) > 1000 and (idx.size == 0 or idx[-1] < n)


@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_uniform_rows_dense_fused_lif_bit_exact(O, cuda_device, precision):
    """The dense-x fused LIF (fused_spmv_lif, mod.rs:1609-1636) on the TMA path:
    one CTA per SM with x cached in L1, the LIF epilogue on every row."""
    nrows, ncols, L = 20_003, 60_000, 64
    csr, w = _uniform(O, nrows, ncols, L, 2024)
    wq = O.quantise(int(precision), w)
    op = _prepare(cuda_device, csr, w, precision, generic=False)
    assert op.layouts() & 1
    r = np.random.default_rng(9)
    x = r.uniform(-1, 1, ncols).astype(np.float32)
    v0 = r.uniform(-1, 1, nrows).astype(np.float32)
    t0 = np.abs(r.uniform(-1, 1, nrows)).astype(np.float32)
    v, t, sp = v0.copy(), t0.copy(), np.zeros(nrows, np.bool_)
    op.fused_spmv_lif(x, v, t, sp, S.LifParams.new(0.9, 0.0, 0.1))
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(nrows, np.uint8)
    O.fused_lif(csr, wq, x, vw, tw, sw, 0.9, 0.0, 0.1, par=True)
    assert_bits_equal(v, vw, "v")
    assert_bits_equal(t, tw, "theta")
    assert np.array_equal(sp.astype(np.uint8), sw) and 0 < sw.sum() < nrows
