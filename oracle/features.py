"""ORACLE -- TEST INFRASTRUCTURE ONLY.

Pure-Python restatement of the feature-index functions of
rgodha24/stockfish-trainer (``src/rust/feature_extraction.rs``).  It checks
the package's native index encoder on small position sets; it is never used
by the product path.

The reference computes indices with the ``sfbinpack 0.6.2`` crate's board and
attack helpers (crates.io, not vendored in the reference).  Only standard
chess attack sets are taken from it (``attacks::piece_attacks``,
``attacks::pawn``); they are rewritten here from the rules of chess.

Board encoding used throughout this repository: a length-64 sequence indexed
by square (a1 = 0, b1 = 1, ..., h8 = 63) holding a piece id
``ordinal(type) * 2 + color`` (types pawn..king = 0..5, white = 0, black = 1),
or ``EMPTY`` (12).  The same id order as the reference's ``PIECE_TABLE``
(feature_extraction.rs:36-49).
"""

from __future__ import annotations

EMPTY = 12
WHITE, BLACK = 0, 1
PAWN, KNIGHT, BISHOP, ROOK, QUEEN, KING = range(6)

HALFKA_INPUTS = 24_576  # feature_extraction.rs:10
HALFKA_MAX_ACTIVE = 32  # :11
FULL_THREATS_INPUTS = 60_720  # :12
FULL_THREATS_MAX_ACTIVE = 128  # :13

MASK64 = (1 << 64) - 1
A_FILE = 0x0101_0101_0101_0101  # :18
H_FILE = 0x8080_8080_8080_8080  # :19

# feature_extraction.rs:21-25
KING_BUCKETS = [
    -1, -1, -1, -1, 31, 30, 29, 28, -1, -1, -1, -1, 27, 26, 25, 24,
    -1, -1, -1, -1, 23, 22, 21, 20, -1, -1, -1, -1, 19, 18, 17, 16,
    -1, -1, -1, -1, 15, 14, 13, 12, -1, -1, -1, -1, 11, 10, 9, 8,
    -1, -1, -1, -1, 7, 6, 5, 4, -1, -1, -1, -1, 3, 2, 1, 0,
]  # fmt: skip
# feature_extraction.rs:27-35
NUM_VALID_TARGETS = [6, 6, 10, 10, 8, 8, 8, 8, 10, 10, 0, 0]
THREAT_MAP = [
    [0, 1, -1, 2, -1, -1],
    [0, 1, 2, 3, 4, -1],
    [0, 1, 2, 3, -1, -1],
    [0, 1, 2, 3, -1, -1],
    [0, 1, 2, 3, 4, -1],
    [-1, -1, -1, -1, -1, -1],
]


def piece_type(pid: int) -> int:
    return pid >> 1


def piece_color(pid: int) -> int:
    return pid & 1


def _bits(bb: int):
    """Squares of a bitboard in ascending order (Bitboard::iter / pop)."""
    while bb:
        low = bb & -bb
        yield low.bit_length() - 1
        bb ^= low


def _popcount(bb: int) -> int:
    return bin(bb).count("1")


def _on_board(f: int, r: int) -> bool:
    return 0 <= f < 8 and 0 <= r < 8


def _step_attacks(sq: int, steps) -> int:
    f0, r0 = sq % 8, sq // 8
    bb = 0
    for df, dr in steps:
        f, r = f0 + df, r0 + dr
        if _on_board(f, r):
            bb |= 1 << (r * 8 + f)
    return bb


def _slide_attacks(sq: int, occ: int, dirs) -> int:
    f0, r0 = sq % 8, sq // 8
    bb = 0
    for df, dr in dirs:
        f, r = f0 + df, r0 + dr
        while _on_board(f, r):
            s = r * 8 + f
            bb |= 1 << s
            if occ >> s & 1:
                break
            f, r = f + df, r + dr
    return bb


_KNIGHT_STEPS = [(1, 2), (2, 1), (2, -1), (1, -2), (-1, -2), (-2, -1), (-2, 1), (-1, 2)]
_KING_STEPS = [(1, 0), (1, 1), (0, 1), (-1, 1), (-1, 0), (-1, -1), (0, -1), (1, -1)]
_DIAG = [(1, 1), (1, -1), (-1, 1), (-1, -1)]
_ORTH = [(1, 0), (-1, 0), (0, 1), (0, -1)]


def piece_attacks(pt: int, sq: int, occ: int) -> int:
    """Standard attack set of a non-pawn piece type (sfbinpack attacks::piece_attacks)."""
    if pt == KNIGHT:
        return _step_attacks(sq, _KNIGHT_STEPS)
    if pt == KING:
        return _step_attacks(sq, _KING_STEPS)
    if pt == BISHOP:
        return _slide_attacks(sq, occ, _DIAG)
    if pt == ROOK:
        return _slide_attacks(sq, occ, _ORTH)
    if pt == QUEEN:
        return _slide_attacks(sq, occ, _DIAG + _ORTH)
    raise ValueError(pt)


def pawn_attacks(color: int, sq: int) -> int:
    """Squares a pawn of ``color`` on ``sq`` attacks (sfbinpack attacks::pawn)."""
    dr = 1 if color == WHITE else -1
    return _step_attacks(sq, [(-1, dr), (1, dr)])


# --- HalfKAv2_hm --------------------------------------------------------------


def orient_mask(color: int, ksq: int) -> int:
    """feature_extraction.rs:745-752."""
    return (7 if (ksq & 7) < 4 else 0) ^ (56 if color == BLACK else 0)


def halfka_feature_index(color: int, ksq: int, sq: int, pid: int) -> int:
    """feature_extraction.rs:677-685."""
    m = orient_mask(color, ksq)
    piece_index = piece_type(pid) * 2 + int(piece_color(pid) != color)
    bucket = KING_BUCKETS[ksq ^ m]
    return (sq ^ m) + piece_index * 64 + bucket * 768


def king_square(board, color: int) -> int:
    kid = KING * 2 + color
    for sq in range(64):
        if board[sq] == kid:
            return sq
    raise ValueError("position has no king of colour %d" % color)


def halfka_indices(board, color: int) -> list[int]:
    """fill_halfka_feature_indices_sparse, feature_extraction.rs:391-404."""
    ksq = king_square(board, color)
    return [
        halfka_feature_index(color, ksq, sq, board[sq])
        for sq in range(64)
        if board[sq] != EMPTY
    ]


# --- Full_Threats ------------------------------------------------------------


def _build_threat_table():
    """threat_feature_calc, feature_extraction.rs:788-832."""
    table = [[0] * 66 for _ in range(12)]
    piece_offset = 0
    for color in (WHITE, BLACK):
        for pt in range(6):
            pi = 2 * pt + color
            table[pi][65] = piece_offset
            square_offset = 0
            for frm in range(64):
                table[pi][frm] = square_offset
                if pt != PAWN:
                    square_offset += _popcount(piece_attacks(pt, frm, 0))
                elif 8 <= frm <= 55:
                    push = frm + 8 if color == WHITE else frm - 8
                    square_offset += _popcount(pawn_attacks(color, frm) | (1 << push))
            table[pi][64] = square_offset
            piece_offset += NUM_VALID_TARGETS[pi] * square_offset
    return table, piece_offset


THREAT_TABLE, THREAT_TOTAL = _build_threat_table()


def full_threat_orient_mask(color: int, ksq: int) -> int:
    """feature_extraction.rs:758-765."""
    return (7 if (ksq & 7) >= 4 else 0) ^ (56 if color == BLACK else 0)


def full_threat_index(persp: int, attacker: int, frm: int, to: int, attacked: int, ksq: int) -> int:
    """feature_extraction.rs:687-739."""
    enemy = piece_color(attacker) != piece_color(attacked)
    m = full_threat_orient_mask(persp, ksq)
    frm ^= m
    to ^= m
    if persp == BLACK:
        attacker ^= 1
        attacked ^= 1
    at, dt = piece_type(attacker), piece_type(attacked)
    mapped = THREAT_MAP[at][dt]
    if mapped < 0 or (at == dt and (enemy or at != PAWN) and frm < to):
        return -1
    if at == PAWN:
        ac = piece_color(attacker)
        push = frm + 8 if ac == WHITE else frm - 8
        attack_mask = pawn_attacks(ac, frm) | (1 << push)
    else:
        attack_mask = piece_attacks(at, frm, 0)
    ai = attacker  # piece_index(): type * 2 + colour == the piece id
    row = THREAT_TABLE[ai]
    return (
        row[65]
        + (piece_color(attacked) * (NUM_VALID_TARGETS[ai] // 2) + mapped) * row[64]
        + row[frm]
        + _popcount(((1 << to) - 1) & attack_mask)
    )


def _bb(board, pid: int) -> int:
    bb = 0
    for sq in range(64):
        if board[sq] == pid:
            bb |= 1 << sq
    return bb


def full_threat_indices(board, persp: int) -> list[int]:
    """fill_full_threat_feature_indices_sparse, feature_extraction.rs:581-675."""
    occupied = 0
    for sq in range(64):
        if board[sq] != EMPTY:
            occupied |= 1 << sq
    pawns = _bb(board, PAWN * 2 + WHITE) | _bb(board, PAWN * 2 + BLACK)
    ksq = king_square(board, persp)
    out: list[int] = []

    def push(attacker, frm, to):
        idx = full_threat_index(persp, attacker, frm, to, board[to], ksq)
        if idx >= 0:
            out.append(idx)

    for color in (persp, 1 - persp):
        for pt in range(6):
            attacker = pt * 2 + color
            piece_bb = _bb(board, attacker)
            if pt == PAWN:
                if color == WHITE:  # :767-786
                    left = ((piece_bb & ~H_FILE) << 9) & MASK64
                    right = ((piece_bb & ~A_FILE) << 7) & MASK64
                    fwd = (piece_bb << 8) & MASK64
                    dl, dr_, df = -9, -7, -8
                else:
                    left = (piece_bb & ~A_FILE) >> 9
                    right = (piece_bb & ~H_FILE) >> 7
                    fwd = piece_bb >> 8
                    dl, dr_, df = 9, 7, 8
                for to in _bits(left & occupied):
                    push(attacker, to + dl, to)
                for to in _bits(right & occupied):
                    push(attacker, to + dr_, to)
                for to in _bits(fwd & pawns):
                    push(attacker, to + df, to)
            else:
                for frm in _bits(piece_bb):
                    for to in _bits(piece_attacks(pt, frm, occupied) & occupied):
                        push(attacker, frm, to)
    return out


# --- Composition (FeatureSet::fill_feature_indices_sparse, :213-241) ---------

FEATURE_SETS = {
    "HalfKAv2_hm": [("HalfKAv2_hm", HALFKA_INPUTS, HALFKA_MAX_ACTIVE)],
    "Full_Threats": [("Full_Threats", FULL_THREATS_INPUTS, FULL_THREATS_MAX_ACTIVE)],
    "Full_Threats+HalfKAv2_hm": [
        ("Full_Threats", FULL_THREATS_INPUTS, FULL_THREATS_MAX_ACTIVE),
        ("HalfKAv2_hm", HALFKA_INPUTS, HALFKA_MAX_ACTIVE),
    ],
}


def feature_set_sizes(name: str) -> tuple[int, int]:
    comps = FEATURE_SETS[name.replace("^", "")]
    return sum(c[1] for c in comps), sum(c[2] for c in comps)


def encode(board, color: int, feature_set: str) -> tuple[list[int], int]:
    """Indices for one perspective, compacted, -1 padded (:213-241, :457-460)."""
    comps = FEATURE_SETS[feature_set.replace("^", "")]
    total_inputs, max_active = feature_set_sizes(feature_set)
    board = [int(x) for x in board]  # plain ints: no fixed-width overflow
    row: list[int] = []
    offset = 0
    for name, inputs, comp_max in comps:
        vals = halfka_indices(board, color) if name == "HalfKAv2_hm" else full_threat_indices(board, color)
        if len(vals) > comp_max:
            raise ValueError(f"{name}: {len(vals)} active features exceed {comp_max}")
        row.extend(v + offset for v in vals)
        offset += inputs
    count = len(row)
    return row + [-1] * (max_active - count), count


def parse_fen(fen: str) -> tuple[list[int], int]:
    """Board + side to move (0 white, 1 black) from a FEN string."""
    fields = fen.split()
    board = [EMPTY] * 64
    letters = "pnbrqk"
    for i, rank_str in enumerate(fields[0].split("/")):
        r = 7 - i
        f = 0
        for ch in rank_str:
            if ch.isdigit():
                f += int(ch)
                continue
            pt = letters.index(ch.lower())
            color = WHITE if ch.isupper() else BLACK
            board[r * 8 + f] = pt * 2 + color
            f += 1
    stm = WHITE if len(fields) < 2 or fields[1] == "w" else BLACK
    return board, stm
