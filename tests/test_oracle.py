"""The oracle pinned against the reference's own outputs (tests/golden) and
against independent float64 / pure-Python restatements."""

import numpy as np
import pytest

import oracle
from oracle import features as F


def test_sorted_backward_inputs_match_reference(golden):
    g = golden("sorted_backward_inputs.npz")
    for name in g["names"]:
        got = oracle.sorted_backward_inputs(g[f"{name}_idx"], int(g[f"{name}_T"]))
        for arr, key in zip(got, ["sorted_bid", "seg_feat", "seg_count", "seg_start"]):
            np.testing.assert_array_equal(arr, g[f"{name}_{key}"], err_msg=f"{name}/{key}")


def test_quantisation_matches_reference(golden):
    q = golden("quantize_ft.npz")
    s = float(q["ft_quantized_one"])
    ps = float(q["psqt_scale"])
    np.testing.assert_array_equal(oracle.quantize(q["weight"], s, np.int16), q["q_weight"])
    np.testing.assert_array_equal(oracle.quantize(q["bias"], s, np.int16), q["q_bias"])
    np.testing.assert_array_equal(oracle.quantize(q["psqt"], ps, np.int32), q["q_psqt"])


def test_export_weights_match_reference(golden):
    e = golden("export_weights.npz")
    np.testing.assert_array_equal(oracle.halfka_export_weights(e["weight"], e["virtual"]), e["export"])


def test_halfka_index_table_matches_reference(golden):
    table = golden("halfka_idx.npz")["table"]
    pov, ksq, sq, pid = np.meshgrid(np.arange(2), np.arange(64), np.arange(64), np.arange(12), indexing="ij")
    got = np.vectorize(F.halfka_feature_index)(pov, ksq, sq, pid)
    np.testing.assert_array_equal(got, table)


def test_composed_sizes_match_reference(golden):
    c = golden("composed_sizes.npz")
    assert F.feature_set_sizes("Full_Threats+HalfKAv2_hm^") == (int(c["num_inputs"]), int(c["max_active"]))
    assert F.HALFKA_INPUTS == int(c["halfka_inputs"])
    assert F.FULL_THREATS_INPUTS == int(c["threat_inputs"])


def test_threat_table_total_is_reference_constant():
    # feature_extraction.rs:826 asserts the offsets add up to FULL_THREATS_INPUTS
    assert F.THREAT_TOTAL == 60720


def _forward_py(idx, W, bias):
    out = np.empty((idx.shape[0], W.shape[1]), np.float32)
    for b in range(idx.shape[0]):
        acc = bias.copy()
        for f in idx[b]:
            if f != -1:
                acc = (acc + W[f]).astype(np.float32)
        out[b] = acc
    return out


def test_oracle_forward_is_sequential_fp32():
    rng = np.random.default_rng(0)
    idx = rng.integers(-1, 50, size=(40, 9)).astype(np.int32)
    W = rng.standard_normal((50, 13)).astype(np.float32)
    bias = rng.standard_normal(13).astype(np.float32)
    np.testing.assert_array_equal(oracle.ft_forward(idx, W, bias), _forward_py(idx, W, bias))


def test_oracle_forward_rejects_bad_index():
    with pytest.raises(ValueError):
        oracle.ft_forward(np.array([[0, 7]], np.int32), np.zeros((5, 4), np.float32), np.zeros(4, np.float32))


def test_oracle_backward_sequential_and_close_to_float64():
    rng = np.random.default_rng(1)
    T, C, B, K = 30, 7, 64, 6
    idx = np.full((B, K), -1, np.int32)
    for b in range(B):
        n = rng.integers(0, K + 1)
        idx[b, :n] = rng.permutation(T)[:n]
    g = rng.standard_normal((B, C)).astype(np.float32)
    dW, dB = oracle.ft_backward(idx, g, T)
    # exact: ascending-position sequential fp32 sum per feature
    ref = np.zeros((T, C), np.float32)
    for f in range(T):
        acc = np.zeros(C, np.float32)
        for b in range(B):
            if f in idx[b]:
                acc = (acc + g[b]).astype(np.float32)
        ref[f] = acc
    np.testing.assert_array_equal(dW, ref)
    np.testing.assert_allclose(dB, g.astype(np.float64).sum(0), rtol=1e-6, atol=1e-6)


def test_oracle_backward_accumulates_touched_rows_only():
    idx = np.array([[1, -1], [1, 2]], np.int32)
    g = np.ones((2, 3), np.float32)
    dW = np.full((4, 3), 5.0, np.float32)
    dB = np.full(3, 1.0, np.float32)
    oracle.ft_backward(idx, g, 4, dW, dB)
    np.testing.assert_array_equal(dW[0], [5, 5, 5])
    np.testing.assert_array_equal(dW[1], [7, 7, 7])
    np.testing.assert_array_equal(dW[2], [6, 6, 6])
    np.testing.assert_array_equal(dW[3], [5, 5, 5])
    np.testing.assert_array_equal(dB, [3, 3, 3])


def test_quantized_forward_wraps_int16():
    wq = np.array([[30000, -30000, 1, 0, 0, 0, 0, 0]], np.int16)
    pq = np.array([[2**31 - 1, 0, 0, 0]], np.int32)
    bias = np.array([10000, -10000, 0, 0, 0, 0, 0, 0], np.int16)
    idx = np.array([[0, 0, -1]], np.int32)
    acc, ps = oracle.ft_quantized_forward(idx, wq, pq, bias, map_training=False)
    expect = ((bias.astype(np.int64) + 2 * wq[0].astype(np.int64) + 2**15) % 2**16 - 2**15).astype(np.int16)
    np.testing.assert_array_equal(acc[0], expect)
    assert ps[0, 0] == np.int32(-2)


def test_halfka_export_row_map():
    rows = np.arange(24576)
    m = oracle.halfka_export_rows(rows)
    assert m.max() == 22527 and m.min() == 0
    # planes 0..9 map one to one
    keep = (rows % 768) // 64 < 10
    assert len(np.unique(m[keep])) == keep.sum()
