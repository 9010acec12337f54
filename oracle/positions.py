"""ORACLE -- TEST INFRASTRUCTURE ONLY.

Seeded synthetic positions and their index rows, computed without the
product library: a pure-Python restatement of the package's position
generator (``stockfish_trainer_b200/csrc/features.cpp``:
``nnue_generate_positions``) feeding the Python restatement of the
reference's feature functions (``oracle/features.py``, which follows
``src/rust/feature_extraction.rs``).  ``tests/test_features.py`` checks that
both give the same boards and rows as the package's native encoder.

The bench's CPU legs (the reference arm and the CPU baseline) build their
inputs here, so the processes that time the CPU restatement never load the
product's shared library.

Position i of a seed depends only on (seed, first + i):
* the stream is splitmix64 (Steele, Lea & Flood, "Fast splittable
  pseudorandom number generators", OOPSLA 2014), started at
  seed * 0xD1B54A32D192ED03 + (first + i) * 0x9E3779B97F4A7C15 (mod 2^64);
* a draw in [0, n) is the high 32 bits of a splitmix64 output times n,
  shifted right by 32 (multiply-shift range reduction);
* the white king takes a uniform square, the black king a uniform other one;
  then n ~ U{0..30} pieces: type uniform over pawn..queen, colour uniform,
  square uniform among empty squares (pawns on ranks 2-7 only); side to move
  uniform; a position whose threat features exceed 128 for either side is
  redrawn from the continuing stream.
"""

from __future__ import annotations

import multiprocessing as mp
import os

import numpy as np

from . import features as F

MASK64 = (1 << 64) - 1
GOLDEN_GAMMA = 0x9E3779B97F4A7C15
SEED_MIX = 0xD1B54A32D192ED03


class _SplitMix64:
    def __init__(self, state: int):
        self.s = state & MASK64

    def next(self) -> int:
        self.s = (self.s + GOLDEN_GAMMA) & MASK64
        z = self.s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK64
        return z ^ (z >> 31)

    def uniform(self, n: int) -> int:
        return ((self.next() >> 32) * n) >> 32


def _draw(rng: _SplitMix64) -> tuple[list[int], int]:
    board = [F.EMPTY] * 64
    wk = rng.uniform(64)
    bk = rng.uniform(63)
    if bk >= wk:
        bk += 1
    board[wk] = F.KING * 2 + F.WHITE
    board[bk] = F.KING * 2 + F.BLACK
    for _ in range(rng.uniform(31)):
        pt = rng.uniform(5)
        color = rng.uniform(2)
        while True:
            sq = 8 + rng.uniform(48) if pt == F.PAWN else rng.uniform(64)
            if board[sq] == F.EMPTY:
                break
        board[sq] = pt * 2 + color
    stm = rng.uniform(2)
    return board, stm


def _position(seed: int, index: int) -> tuple[list[int], int]:
    rng = _SplitMix64(((seed & MASK64) * SEED_MIX + index * GOLDEN_GAMMA) & MASK64)
    while True:
        board, stm = _draw(rng)
        if all(len(F.full_threat_indices(board, c)) <= F.FULL_THREATS_MAX_ACTIVE for c in (F.WHITE, F.BLACK)):
            return board, stm


def _chunk(args):
    seed, first, n, feature_set = args
    _, K = F.feature_set_sizes(feature_set) if feature_set else (0, 0)
    boards = np.empty((n, 64), np.uint8)
    stm = np.empty(n, np.uint8)
    white = np.empty((n, K), np.int32)
    black = np.empty((n, K), np.int32)
    for i in range(n):
        board, s = _position(seed, first + i)
        boards[i] = board
        stm[i] = s
        if feature_set:
            white[i] = F.encode(board, F.WHITE, feature_set)[0]
            black[i] = F.encode(board, F.BLACK, feature_set)[0]
    return boards, stm, white, black


def _spawn_safe() -> bool:
    """A spawned worker re-imports the parent's main module; a main module
    read from standard input cannot be re-imported, so no pool then."""
    import sys

    main = sys.modules.get("__main__")
    return bool(getattr(main, "__file__", None) or getattr(main, "__spec__", None))


def _run(seed: int, first: int, n: int, feature_set: str | None, processes: int):
    processes = max(1, min(processes or (os.cpu_count() or 1), max(1, n // 64)))
    if not _spawn_safe():
        processes = 1
    bounds = [first + n * p // processes for p in range(processes + 1)]
    jobs = [(seed, bounds[p], bounds[p + 1] - bounds[p], feature_set) for p in range(processes)]
    if processes == 1:
        parts = [_chunk(jobs[0])]
    else:
        # spawn: safe whether or not the caller has already touched a GPU
        with mp.get_context("spawn").Pool(processes) as pool:
            parts = pool.map(_chunk, jobs)
    return tuple(np.concatenate([p[j] for p in parts]) for j in range(4))


def generate_positions(n: int, seed: int = 0, first: int = 0, processes: int = 1):
    """Boards [n, 64] uint8 and side to move [n] uint8."""
    boards, stm, _, _ = _run(seed, first, n, None, processes)
    return boards, stm


def synthetic_batch(n: int, feature_set: str, seed: int = 0, first: int = 0, processes: int = 0):
    """(white [n, K], black [n, K], side to move [n]) for n seeded positions,
    encoded by the oracle's feature functions; ``processes`` = 0 uses every
    core."""
    _, stm, white, black = _run(seed, first, n, feature_set, processes)
    return white, black, stm
