"""The CPU oracle against known answers from the reference's own tests and
against independent computations (numpy).  CPU only."""
import numpy as np
import pytest


def test_pack_known_answers(oracle):
    # tests/test_ops.py:8-11 of the reference: [0,1,2,3]*4 round trip;
    # word value 0xE4E4E4E4.
    v = np.array([0, 1, 2, 3] * 4, np.uint8)
    p = oracle.pack_2bit(v)
    assert p.tolist() == [np.int32(-454761244)]
    assert (oracle.unpack_2bit(p, 16) == v).all()
    # tests/test_ops.py:15-18
    v4 = np.array([0, 3, 7, 15, 1, 8, 12, 4], np.uint8)
    p4 = oracle.pack_4bit(v4)
    assert p4[0] == np.int32(np.uint32(0x4C81F730).view(np.int32))
    assert (oracle.unpack_4bit(p4, 8) == v4).all()
    # core/quantize.cu:557-617 (native self-test): i%4 and 2*i patterns
    assert (oracle.unpack_2bit(oracle.pack_2bit(np.arange(16, dtype=np.uint8) % 4), 16)
            == np.arange(16) % 4).all()
    assert (oracle.unpack_4bit(oracle.pack_4bit(np.arange(8, dtype=np.uint8) * 2), 8)
            == np.arange(8) * 2).all()


def test_pack_masks_high_bits_and_partial_unpack(oracle):
    v = np.arange(32, dtype=np.uint8) * 7
    p = oracle.pack_2bit(v)
    assert (oracle.unpack_2bit(p, 32) == (v & 3)).all()
    assert (oracle.unpack_2bit(p, 20) == (v & 3)[:20]).all()
    p4 = oracle.pack_4bit(v)
    assert (oracle.unpack_4bit(p4, 27) == (v & 15)[:27]).all()


def test_fp16_conversions_exhaustive(oracle):
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle.f16_bits_to_f32(int(b)) for b in bits], np.float32)
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all()
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(20000) * np.exp(rng.uniform(-20, 12, 20000))).astype(np.float32)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16_bits(float(v)) for v in x], np.uint16)
    assert (got == want).all()


def test_group_stats_vs_numpy(oracle):
    # core/quantize.cu:619-685 checks the stats kernel against a CPU loop on
    # a 64x64 U(-1, 1) matrix; here the oracle against numpy on ragged shapes.
    rng = np.random.default_rng(42)
    for M, K in ((64, 64), (17, 100), (3, 4104)):
        w = rng.uniform(-1, 1, (M, K)).astype(np.float16)
        mn, mx = oracle.group_stats(w)
        ng = (K + 15) // 16
        for g in range(ng):
            blk = w[:, g * 16:(g + 1) * 16].astype(np.float32)
            assert mn[g] == blk.min() and mx[g] == blk.max()


def test_sensitivity_is_serial_fp32(oracle):
    rng = np.random.default_rng(7)
    M, K = 33, 48
    w = (rng.standard_normal((M, K)) * 0.02).astype(np.float16)
    h = np.exp(rng.standard_normal(K) * 1.5).astype(np.float32)
    h[::5] = 1e-10
    s = oracle.sensitivity(w, h)
    for g in range(K // 16):
        acc = np.float32(0)
        for r in range(M):
            for c in range(g * 16, g * 16 + 16):
                x = np.float32(w[r, c]) * np.float32(w[r, c])
                acc = np.float32(acc + (x / h[c] if h[c] > np.float32(1e-8) else x))
        assert acc == s[g]


def test_select_matches_sort(oracle):
    rng = np.random.default_rng(1)
    s = rng.random(256).astype(np.float32)
    gp = oracle.select(s, 0.1)
    top = np.argsort(-s, kind="stable")[:25]
    assert gp.sum() == 25 and gp[top].all()
    # ratio > 1 is clamped to all groups
    assert oracle.select(s, 2.0).sum() == 256


def test_quantize_roundtrip_small(oracle):
    rng = np.random.default_rng(0)
    w = (rng.standard_normal((64, 80)) * 0.02).astype(np.float16)
    q = oracle.quantize(w, 0.2, np.ones(80, np.float32))
    assert q["group_precision"].sum() == 1  # int(0.2 * 5)
    d = oracle.dequantize(q)
    assert d.shape == w.shape
    # all-2-bit groups of gaussian weights: error bounded by about one scale
    err = np.abs(d.astype(np.float32) - w.astype(np.float32))
    assert err.mean() < 0.02


def test_outliers_on_shifted_groups(oracle):
    # groups entirely above zero clamp the zero point and produce outliers
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((8, 32)) * 0.02 + np.r_[np.zeros(16), np.full(16, 0.2)]).astype(np.float16)
    q = oracle.quantize(w, 0.0)
    rp = q["outlier_row_ptrs"]
    assert rp[-1] == q["outlier_values"].size > 0
    assert (q["outlier_col_indices"] >= 16).all()
    for r in range(8):
        cols = q["outlier_col_indices"][rp[r]:rp[r + 1]]
        assert (np.diff(cols) > 0).all()
        assert (q["outlier_values"][rp[r]:rp[r + 1]] == w[r, cols]).all()
