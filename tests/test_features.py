"""Native position generator + feature-index encoder vs the Python oracle and
the reference's own known answers (src/rust/feature_extraction.rs:853-881,
src/rust/pipeline.rs:1337-1384, 1669-1681)."""

import numpy as np
import pytest

from oracle import features as F
from stockfish_trainer_b200 import positions as P

# pipeline.rs:1345-1350
REFERENCE_FENS = [
    "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1",
    "r1bq1rk1/pp2bppp/2n2n2/2pp4/2P5/2NP1NP1/PP2PPBP/R1BQ1RK1 w - - 0 9",
    "8/2k5/8/2p5/2P5/2K5/8/8 w - - 0 1",
    "r3k2r/pppq1ppp/2npbn2/3Np3/2B1P3/2N5/PPP2PPP/R1BQ1RK1 b kq - 2 10",
]
FEATURE_SETS = ["HalfKAv2_hm^", "Full_Threats", "Full_Threats+HalfKAv2_hm^"]


def _assert_valid_row(row, count, num_inputs):
    # pipeline.rs:1669-1681
    assert np.all((row[:count] >= 0) & (row[:count] < num_inputs))
    assert np.all(row[count:] == -1)
    assert len(np.unique(row[:count])) == count


def test_threat_table_total():
    assert P.threat_table_total() == 60720


def test_feature_set_sizes_match_reference():
    # feature_extraction.rs:857-868
    assert P.feature_set_info("Full_Threats+HalfKAv2_hm^")[1:] == (60720 + 24576, 128 + 32)
    assert P.feature_set_info("HalfKAv2_hm^")[1:] == (24576, 32)


def test_startpos_has_32_halfka_features_per_side():
    # feature_extraction.rs:870-880
    board, _ = F.parse_fen(REFERENCE_FENS[0])
    w, b, wc, bc = P.encode(np.array([board], np.uint8), "HalfKAv2_hm^")
    assert wc[0] == 32 and bc[0] == 32


@pytest.mark.parametrize("fs", FEATURE_SETS)
def test_reference_fens_match_oracle_and_are_valid(fs):
    boards = np.array([F.parse_fen(f)[0] for f in REFERENCE_FENS], np.uint8)
    w, b, wc, bc = P.encode(boards, fs)
    n_inputs = P.feature_set_info(fs)[1]
    for i in range(len(REFERENCE_FENS)):
        for color, arr, cnt in ((0, w, wc), (1, b, bc)):
            row, count = F.encode(boards[i], color, fs)
            np.testing.assert_array_equal(arr[i], np.array(row, np.int32))
            assert cnt[i] == count
            _assert_valid_row(arr[i], count, n_inputs)


@pytest.mark.parametrize("fs", FEATURE_SETS)
def test_random_positions_match_oracle(fs):
    boards, _ = P.generate_positions(150, seed=11)
    w, b, wc, bc = P.encode(boards, fs)
    n_inputs = P.feature_set_info(fs)[1]
    for i in range(len(boards)):
        for color, arr, cnt in ((0, w, wc), (1, b, bc)):
            row, count = F.encode(boards[i], color, fs)
            np.testing.assert_array_equal(arr[i], np.array(row, np.int32))
            _assert_valid_row(arr[i], count, n_inputs)


def test_generator_is_deterministic_and_sliceable():
    b1, s1 = P.generate_positions(500, seed=3)
    b2, s2 = P.generate_positions(500, seed=3)
    np.testing.assert_array_equal(b1, b2)
    np.testing.assert_array_equal(s1, s2)
    b3, s3 = P.generate_positions(100, seed=3, first=200)
    np.testing.assert_array_equal(b1[200:300], b3)
    np.testing.assert_array_equal(s1[200:300], s3)
    b4, _ = P.generate_positions(500, seed=4)
    assert not np.array_equal(b1, b4)


def test_generator_distribution():
    boards, stm = P.generate_positions(4000, seed=9)
    for bd in boards:
        assert np.sum(bd == 10) == 1 and np.sum(bd == 11) == 1  # one king per side
        n_other = np.sum(bd < 10)
        assert 0 <= n_other <= 30
        pawn_sq = np.nonzero((bd == 0) | (bd == 1))[0]
        assert np.all((pawn_sq >= 8) & (pawn_sq <= 55))
    assert set(np.unique(stm)) <= {0, 1}
    counts = np.sum(boards < 10, axis=1)
    assert abs(counts.mean() - 15) < 0.6  # U{0..30}


def test_threat_counts_fit_reference_layout():
    boards, _ = P.generate_positions(20000, seed=5)
    _, _, wc, bc = P.encode(boards, "Full_Threats")
    assert wc.max() <= 128 and bc.max() <= 128
    assert 20 < wc.mean() < 30


def test_encode_rejects_position_without_king():
    board = np.full((1, 64), 12, np.uint8)
    with pytest.raises(RuntimeError):
        P.encode(board, "HalfKAv2_hm^")


def test_host_encoder_rejects_invalid_positions():
    """A perspective without its king, or any pawn on a back rank (the
    reference's threat table has no slot for such pawns), is rejected: the
    batch reports INVALID_ARGUMENT and the rejected rows are all -1, the
    others intact."""
    from stockfish_trainer_b200 import _native

    boards = np.array([F.parse_fen(f)[0] for f in REFERENCE_FENS], np.uint8)
    bad = boards.copy()
    bad[1][bad[1] == 11] = 12          # position 1: no black king
    bad[2][60] = 0                     # position 2: a white pawn on e8
    good_w, good_b, _, _ = P.encode(boards, "Full_Threats+HalfKAv2_hm^")
    with pytest.raises(_native.NativeError):
        P.encode(bad, "Full_Threats+HalfKAv2_hm^")
    K = 160
    w = np.empty((4, K), np.int32)
    b = np.empty((4, K), np.int32)
    rc = _native.load().nnue_encode_features(bad.ctypes.data, 4, 2, w.ctypes.data, b.ctypes.data, None, None, 0)
    assert rc == _native.NNUE_ERR_INVALID_ARGUMENT
    assert np.all(b[1] == -1) and (w[1] >= 0).sum() > 0  # only black lacks its king
    assert np.all(w[2] == -1) and np.all(b[2] == -1)
    np.testing.assert_array_equal(w[[0, 3]], good_w[[0, 3]])
    np.testing.assert_array_equal(b[[0, 3]], good_b[[0, 3]])


def test_oracle_position_generator_matches_native():
    """oracle/positions.py restates the package's seeded generator: the same
    boards and side to move for any (seed, first) slice, including positions
    redrawn for exceeding 128 threat features."""
    from oracle import positions as OP

    for seed, first, n in ((2024, 0, 300), (7, 123_456, 200), (2**63 + 5, 10**9, 100)):
        nb, ns = P.generate_positions(n, seed=seed, first=first)
        ob, os_ = OP.generate_positions(n, seed=seed, first=first)
        np.testing.assert_array_equal(ob, nb)
        np.testing.assert_array_equal(os_, ns)


def test_oracle_synthetic_batch_matches_native_in_worker_processes():
    """The bench's CPU legs build their inputs with the oracle encoder in
    spawned worker processes; the rows equal the native encoder's."""
    from oracle import positions as OP

    fs = "Full_Threats+HalfKAv2_hm^"
    ow, ob, os_ = OP.synthetic_batch(256, fs, seed=99, first=4096, processes=2)
    nw, nb, ns = P.synthetic_batch(256, fs, seed=99, first=4096)
    np.testing.assert_array_equal(ow, nw)
    np.testing.assert_array_equal(ob, nb)
    np.testing.assert_array_equal(os_, ns)
