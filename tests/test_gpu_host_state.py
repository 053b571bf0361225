"""The slice calls with their outputs and state in pinned host memory.

When v, theta and the spike bytes are pinned host memory that the GPU can
address (sparsl_host_alloc), the tick's epilogue reads and writes them in
place over PCIe instead of staging them through device copies.  Checked bit
for bit against the oracle on the three engines a tick can take (the TMA
stream for uniform rows, the ordered fold for skewed rows, the plain row
fold), with a dense and a spike operand, a ragged last tile, and a mix of
pinned and pageable buffers (which takes the copying route).  Likewise y of
the forward SpMV and spike SpMV, accumulated in place by every engine."""
import numpy as np
import pytest

from conftest import assert_bits_equal

import sparsl_b200 as S

pytestmark = pytest.mark.gpu

PARAMS = S.LifParams.new(0.9, 0.0, 0.1)


class _Pinned:
    """A pinned copy of `like` (sparsl_b200.HostBuffer)."""

    def __init__(self, like):
        self.h = S.HostBuffer(like.size, like.dtype)
        self.a = self.h.array
        self.a[:] = like

    def free(self):
        del self.a, self.h


def _skewed(O, nrows, ncols, seed):
    r = np.random.default_rng(seed)
    lens = np.minimum(r.zipf(1.5, nrows), min(2500, ncols))
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(ncols, k, replace=False)) for k in lens]).astype(np.uint32)
    return O.Csr(rp.astype(np.uint32), col, ncols)


PANELS, ELL, ORDERED = 16, 1, 64  # SPARSL_LAYOUT_X_PANELS, _ELL, _ORDERED_COPY


def _uniform(O, nrows, ncols, L, seed):
    """Rows of exactly L sorted random columns (the TMA stream's and the
    panels' operators)."""
    r = np.random.default_rng(seed)
    col = np.sort(r.integers(0, ncols, size=(nrows, L), dtype=np.uint32), axis=1).reshape(-1)
    rp = (np.arange(nrows + 1, dtype=np.uint64) * L).astype(np.uint32)
    return O.Csr(rp, col, ncols)


def _operator(O, dev, kind, nrows, ncols, seed, L=48):
    """kind: "uniform" (equal rows), "skewed" (Zipf lengths: the ordered
    fold) or "plain" (equal rows forced onto the plain row fold)."""
    rng = O.Rng(seed)
    csr = _skewed(O, nrows, ncols, seed) if kind == "skewed" else _uniform(O, nrows, ncols, L, seed)
    w = O.random_vec(csr.nnz, 0.5, rng)
    op = dev.prepare(S.Csr(csr.row_ptr, csr.col, ncols), ncols, w)
    if kind == "plain":
        op.force_plain_row_fold()
    lay = op.layouts()
    assert bool(lay & ELL) == (kind == "uniform")
    assert bool(lay & ORDERED) == (kind == "skewed")
    return csr, w, op


@pytest.mark.parametrize("kind", ["uniform", "skewed", "plain"])
@pytest.mark.parametrize("nrows", [4096, 1031])
def test_pinned_state_matches_oracle(O, cuda_device, kind, nrows):
    ncols = 3000
    csr, w, op = _operator(O, cuda_device, kind, nrows, ncols, 0x5A + nrows)
    r = np.random.default_rng(nrows)
    v0 = r.uniform(-0.5, 0.8, nrows).astype(np.float32)
    t0 = r.uniform(0.2, 0.6, nrows).astype(np.float32)
    x = r.uniform(0, 0.05, ncols).astype(np.float32)
    packed = O.pack_spikes((r.random(ncols) < 0.3).astype(np.uint8))
    for operand in ("dense", "spikes"):
        hv, ht, hs = _Pinned(v0), _Pinned(t0), _Pinned(np.zeros(nrows, np.uint8))
        try:
            vw, tw, sw = v0.copy(), t0.copy(), np.zeros(nrows, np.uint8)
            # two ticks in a row on the same pinned buffers
            for _ in range(2):
                if operand == "dense":
                    op.fused_spmv_lif(x, hv.a, ht.a, hs.a, PARAMS)
                    O.fused_lif(csr, w, x, vw, tw, sw, 0.9, 0.0, 0.1)
                else:
                    op.fused_spmv_spikes_lif(packed, hv.a, ht.a, hs.a, PARAMS)
                    O.fused_spikes_lif(csr, w, packed, vw, tw, sw, 0.9, 0.0, 0.1)
                assert_bits_equal(hv.a, vw, f"{kind} {operand} v")
                assert_bits_equal(ht.a, tw, f"{kind} {operand} theta")
                assert np.array_equal(hs.a, sw), f"{kind} {operand} spikes"
            assert sw.any() and not sw.all(), "the case should spike in some rows only"
        finally:
            for h in (hv, ht, hs):
                h.free()


def test_pinned_and_pageable_mixed(O, cuda_device):
    """Pinned v and theta with pageable spike bytes: the call copies, and the
    result is the same."""
    nrows, ncols = 2048, 2000
    csr, w, op = _operator(O, cuda_device, "uniform", nrows, ncols, 0x77)
    r = np.random.default_rng(3)
    v0 = r.uniform(-0.5, 0.8, nrows).astype(np.float32)
    t0 = r.uniform(0.2, 0.6, nrows).astype(np.float32)
    x = r.uniform(0, 0.05, ncols).astype(np.float32)
    hv, ht = _Pinned(v0), _Pinned(t0)
    try:
        sp = np.zeros(nrows, np.uint8)
        op.fused_spmv_lif(x, hv.a, ht.a, sp, PARAMS)
        vw, tw, sw = v0.copy(), t0.copy(), np.zeros(nrows, np.uint8)
        O.fused_lif(csr, w, x, vw, tw, sw, 0.9, 0.0, 0.1)
        assert_bits_equal(hv.a, vw, "v")
        assert_bits_equal(ht.a, tw, "theta")
        assert np.array_equal(sp, sw)
    finally:
        hv.free()
        ht.free()


@pytest.mark.parametrize("kind,nrows,ncols,L", [
    ("uniform", 3000, 3000, 48),    # x in shared-memory panels; spikes on the TMA stream
    ("uniform", 1031, 230_000, 16), # x past the panels: the TMA stream for both
    ("skewed", 4096, 3000, 0),      # the ordered fold
    ("plain", 1031, 3000, 48),      # the plain row fold
])
def test_pinned_y_spmv_matches_oracle(O, cuda_device, kind, nrows, ncols, L):
    """y += A x and y += A s into a pinned y, accumulated in place over PCIe
    by every engine a forward product can take."""
    csr, w, op = _operator(O, cuda_device, kind, nrows, ncols, 0x99 + nrows, L)
    assert bool(op.layouts() & PANELS) == (kind == "uniform" and ncols == 3000)
    r = np.random.default_rng(nrows)
    y0 = r.uniform(-1, 1, nrows).astype(np.float32)
    y0[::7] = -0.0
    x = r.uniform(-1, 1, ncols).astype(np.float32)
    packed = O.pack_spikes((r.random(ncols) < 0.3).astype(np.uint8))
    hy = _Pinned(y0)
    try:
        want = y0.copy()
        for _ in range(2):
            op.spmv(x, hy.a)
            O.spmv(csr, w, x, want)
            assert_bits_equal(hy.a, want, f"{kind} spmv")
        op.spmv_spikes(packed, hy.a)
        O.spmv_spikes(csr, w, packed, want)
        assert_bits_equal(hy.a, want, f"{kind} spmv_spikes")
    finally:
        hy.free()
