"""Device feature encoder (nnue_ft_encode_features) vs the host encoder.

Both run the same encoding functions (feature_encode.h, a restatement of
src/rust/feature_extraction.rs pinned by test_features.py against the
reference's known answers and the Python oracle), so the index rows and
counts must be identical, including the -1 tails and rejected positions."""

import numpy as np
import pytest
import torch

from oracle import features as F
from stockfish_trainer_b200 import _native
from stockfish_trainer_b200 import positions as P

pytestmark = pytest.mark.gpu

FEATURE_SETS = ["HalfKAv2_hm^", "Full_Threats", "Full_Threats+HalfKAv2_hm^"]

FENS = [
    "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1",
    "r1bq1rk1/pp2bppp/2n2n2/2pp4/2P5/2NP1NP1/PP2PPBP/R1BQ1RK1 w - - 0 9",
    "8/2k5/8/2p5/2P5/2K5/8/8 w - - 0 1",
    "r3k2r/pppq1ppp/2npbn2/3Np3/2B1P3/2N5/PPP2PPP/R1BQ1RK1 b kq - 2 10",
]


def _device_encode(board_dev, n, fs, dev):
    fid, _, K = P.feature_set_info(fs)
    w = torch.empty(n, K, dtype=torch.int32, device=dev)
    b = torch.empty(n, K, dtype=torch.int32, device=dev)
    wc = torch.empty(n, dtype=torch.int32, device=dev)
    bc = torch.empty(n, dtype=torch.int32, device=dev)
    _native.call("nnue_ft_encode_features", board_dev.data_ptr(), n, fid, w.data_ptr(), b.data_ptr(),
                 wc.data_ptr(), bc.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    return w.cpu().numpy(), b.cpu().numpy(), wc.cpu().numpy(), bc.cpu().numpy()


@pytest.mark.parametrize("fs", FEATURE_SETS)
@pytest.mark.parametrize("n", [1, 63, 20000 + 37])
def test_device_encoder_matches_host_encoder(cuda, fs, n):
    board, _ = P.generate_positions(n, seed=77)
    host = P.encode(board, fs)
    dev = _device_encode(torch.from_numpy(board).to(cuda), n, fs, cuda)
    for h, d in zip(host, dev):
        np.testing.assert_array_equal(d, h)
    assert _native.device_errors() == 0


@pytest.mark.parametrize("fs", FEATURE_SETS)
def test_device_encoder_reference_fens_and_unaligned_boards(cuda, fs):
    boards = np.array([F.parse_fen(f)[0] for f in FENS] * 17, np.uint8)  # 68 positions: two blocks
    host = P.encode(boards, fs)
    # boards at an odd byte offset: the kernel's byte-wise staging path
    buf = torch.empty(boards.size + 1, dtype=torch.uint8, device=cuda)
    buf[1:] = torch.from_numpy(boards.reshape(-1)).to(cuda)
    view = buf[1:]
    assert view.data_ptr() % 16 != 0
    dev = _device_encode(view, boards.shape[0], fs, cuda)
    for h, d in zip(host, dev):
        np.testing.assert_array_equal(d, h)
    assert _native.device_errors() == 0


def test_device_encoder_rejects_like_the_host(cuda):
    boards = np.array([F.parse_fen(f)[0] for f in FENS], np.uint8)
    boards[1][boards[1] == 11] = 12  # no black king
    boards[2][60] = 0                # a white pawn on e8
    K = 160
    hw = np.empty((4, K), np.int32)
    hb = np.empty((4, K), np.int32)
    hwc = np.empty(4, np.int32)
    hbc = np.empty(4, np.int32)
    rc = _native.load().nnue_encode_features(boards.ctypes.data, 4, 2, hw.ctypes.data, hb.ctypes.data,
                                              hwc.ctypes.data, hbc.ctypes.data, 0)
    assert rc == _native.NNUE_ERR_INVALID_ARGUMENT
    _native.device_errors()
    dw, db, dwc, dbc = _device_encode(torch.from_numpy(boards).to(cuda), 4, "Full_Threats+HalfKAv2_hm^", cuda)
    assert _native.device_errors() == _native.DEVERR_BAD_POSITION
    np.testing.assert_array_equal(dw, hw)
    np.testing.assert_array_equal(db, hb)
    np.testing.assert_array_equal(dwc, hwc)
    np.testing.assert_array_equal(dbc, hbc)
    assert np.all(db[1] == -1) and dbc[1] == 0
    assert np.all(dw[2] == -1) and np.all(db[2] == -1)


def test_device_encoder_empty_batch_and_argument_errors(cuda):
    lib = _native.load()
    assert lib.nnue_ft_encode_features(None, 0, 2, None, None, None, None, None) == _native.NNUE_OK
    assert lib.nnue_ft_encode_features(None, 4, 3, None, None, None, None, None) == _native.NNUE_ERR_INVALID_ARGUMENT
    assert lib.nnue_ft_encode_features(None, 4, 2, None, None, None, None, None) == _native.NNUE_ERR_INVALID_ARGUMENT


def test_encode_device_wrapper(cuda):
    board, _ = P.generate_positions(3000, seed=9)
    w, b = P.encode_device(torch.from_numpy(board).to(cuda), "Full_Threats+HalfKAv2_hm^")
    hw, hb, _, _ = P.encode(board, "Full_Threats+HalfKAv2_hm^")
    np.testing.assert_array_equal(w.cpu().numpy(), hw)
    np.testing.assert_array_equal(b.cpu().numpy(), hb)
    with pytest.raises(ValueError):
        P.encode_device(torch.from_numpy(board), "Full_Threats+HalfKAv2_hm^")


@pytest.mark.parametrize("fs", FEATURE_SETS)
def test_device_encoder_matches_python_oracle(cuda, fs):
    """Device rows against the independent Python restatement of the
    reference's feature functions (oracle/features.py), not only against the
    host encoder that shares the device encoder's source: the reference FENs
    and 400 seeded positions."""
    board, _ = P.generate_positions(400, seed=4242)
    boards = np.concatenate([np.array([F.parse_fen(f)[0] for f in FENS], np.uint8), board])
    dw, db, dwc, dbc = _device_encode(torch.from_numpy(boards).to(cuda), boards.shape[0], fs, cuda)
    assert _native.device_errors() == 0
    for i in range(boards.shape[0]):
        for color, rows, counts in ((F.WHITE, dw, dwc), (F.BLACK, db, dbc)):
            row, count = F.encode(boards[i], color, fs)
            np.testing.assert_array_equal(rows[i], np.array(row, np.int32))
            assert counts[i] == count
