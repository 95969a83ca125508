"""The DedupCount codec oracle (models/dedup/) on CPU.  The reference has no
tests of this codec, so the restatement is pinned by (1) hand-computed cases
in independent numpy float32 arithmetic, (2) the reference's fallbacks for
short sandbags and out-of-range indices (`.get(i).copied().unwrap_or(0)`),
(3) the compress -> decompress round trip and (4) the global-table path,
which must reproduce the local one bit for bit when the prefix digits agree."""
import numpy as np
import pytest

from oracle import oracle as O

F = np.float32


def numpy_decompress(prefixes, tails, count, pd, td, avg, pidx, tidx, signs):
    """decompressor.rs:7-27 in numpy float32 (independent of the C oracle)."""
    out = np.empty(count, np.float32)
    ps, div = F(10.0) ** pd, F(10.0) ** (pd + td)
    for i in range(count):
        p = int(pidx[i]) if i < len(pidx) else 0
        t = int(tidx[i]) if i < len(tidx) else 0
        prefix = F(prefixes[p] if p < len(prefixes) else 0) / ps
        tail = F(tails[t] if t < len(tails) else 0)
        v = F(prefix + tail / div)
        v = F(v + F(avg))
        sb = int(signs[i // 8]) if i // 8 < len(signs) else 0
        out[i] = -v if (sb >> (i % 8)) & 1 else v
    return out


def test_decompress_all_hand_case(oracle):
    t = O.DedupTensor([3, 0, 12], [5, 120, 999], 5, 2, 3, 0.00005)
    s = O.Sandbag([0, 1, 2, 0, 2], [0, 1, 2, 2, 0], [0b01010], 5)
    got = O.dedup_decompress_all(t, s)
    want = numpy_decompress(t.prefixes, t.tail_values, 5, 2, 3, t.avg_precision_lost, s.prefix_idx, s.tail_idx,
                            s.sign_bits)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # element 1: prefix 0 + 120 / 1e5 + 5e-5, sign bit 1 set
    assert got[1] == -(F(0.0) + F(120) / F(1e5) + F(0.00005))


def test_decompress_all_fallbacks(oracle):
    # count beyond the sandbag arrays, indices past the tables, missing sign bytes
    t = O.DedupTensor([7, 2], [11, 40000], 20, 1, 4, -1e-6)
    s = O.Sandbag([0, 1, 5, 1, 0, 9, 1], [1, 0, 1, 7, 1], [0xFF], 20)
    got = O.dedup_decompress_all(t, s)
    want = numpy_decompress(t.prefixes, t.tail_values, 20, 1, 4, t.avg_precision_lost, s.prefix_idx, s.tail_idx,
                            s.sign_bits)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # i >= 8: sign byte missing -> positive; i >= 7: both indices read 0
    assert got[10] == F(F(F(7) / F(10)) + F(11) / F(1e5)) + F(t.avg_precision_lost)


@pytest.mark.parametrize("pd,rounds", [(2, 2), (1, 3), (3, 0)])
def test_compress_round_trip(oracle, pd, rounds):
    rng = np.random.default_rng(pd * 10 + rounds)
    w = (rng.standard_normal(40000) * 0.02).astype(np.float32)
    t, s = O.dedup_compress(w, pd, rounds)
    assert t.tail_digits == 7 - pd - rounds
    assert t.prefix_counts.sum() == w.size and t.tail_counts.sum() == w.size
    assert np.all(np.diff(t.tail_values.astype(np.int64)) > 0)  # unique tails ascending
    d = O.dedup_decompress_all(t, s)
    # each truncation round moves a tail by < 1 unit of the kept digit, and the
    # average loss is added back: error within 10^-(pd+td) plus that average
    bound = 10.0 ** -(pd + t.tail_digits) + abs(t.avg_precision_lost) + 1e-7
    if rounds == 0 and pd == 3:  # 4 tail digits kept as u16 (< 65536): no wrap
        bound = 1e-7 + 1e-7
    assert np.max(np.abs(d - w)) <= bound
    big = np.abs(w) > 2 * bound
    assert np.array_equal(np.sign(d[big]), np.sign(w[big]))


def test_global_table_reproduces_local(oracle):
    rng = np.random.default_rng(3)
    chunks = [O.dedup_compress((rng.standard_normal(5000) * s).astype(np.float32), 2, 2) for s in (0.02, 0.05)]
    g = O.dedup_global_table_new([c[0] for c in chunks])
    assert g.prefix_digits == 2
    assert np.all(np.diff(g.prefixes) > 0)
    for t, s in chunks:
        local = O.dedup_decompress_all(t, s)
        glob = O.dedup_decompress_all_global(t, s, g)
        assert np.array_equal(local.view(np.uint32), glob.view(np.uint32))


def test_remap_path_runs_and_rejects_what_panics(oracle):
    rng = np.random.default_rng(4)
    chunks = [O.dedup_compress((rng.standard_normal(3000) * 0.03).astype(np.float32), 2, 2) for _ in range(2)]
    g = O.dedup_global_table_new([c[0] for c in chunks])
    t, s = chunks[1]
    remap = O.dedup_build_chunk_remap(g, t)
    assert remap.size == t.tail_values.size
    out = O.dedup_decompress_with_remap(g, s, t, remap)
    assert out.size == s.count and np.all(np.isfinite(out))
    short = O.Sandbag(s.prefix_idx[:10], s.tail_idx, s.sign_bits, s.count)
    with pytest.raises(IndexError):
        O.dedup_decompress_with_remap(g, short, t, remap)
