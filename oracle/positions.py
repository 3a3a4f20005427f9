"""TEST INFRASTRUCTURE ONLY: seeded chess positions and their network inputs, through the reference's own C++
chess core (oracle/_ref/libchesscore.so, built by oracle/Makefile from mayfly/chess/cpp/chess_core.cpp).

Only the fixture generator (tests/golden/make_golden.py) and the tests use this module. The product never
imports it; the bench reads the committed position fixtures as data.

What it restates:
  * the inputs MCTS._prepare builds for a batch (mayfly/chess/mcts.py:1004-1058, cpp/export_ts.py:73-86
    encode, cpp/export_ts.py:101-117 make_batches): ids (B, 64) int64, cast (B, 4) float32, hm (B,) int64,
    ep (B,) int64, and I (B, wide) int64 / M (B, wide) bool, the legal moves' policy indices padded to the
    batch's widest row, in python-chess's legal-move order (chess_core.cpp:550-563 legal_moves);
  * the encoder itself is chess_core.cpp:582-612 encode (mayfly_movegen.encode), which
    encode.py:11-35 board_to_ids/clock_and_ep and encode.py:73-100 encode_keys equal.

Random playouts: numpy Generator(PCG64(seed)); per board a ply count drawn uniformly from [0, max_plies], then
uniformly random legal moves from the initial position. A move that would leave the side to move with no legal
reply ends the playout one ply earlier, so every position has at least one legal move (the reference's own
generator demands the same, cudanet/test_cudanet.py:121-155).
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_ref", "libchesscore.so")
START_FEN = "rnbqkbnr/pppppppp/8/8/8/8/PPPPPPPP/RNBQKBNR w KQkq - 0 1"
MAX_MOVES = 256

_lib = None


def lib():
    """The chess core, loaded once. Raises if oracle/_ref was not built (make -C oracle)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(f"{LIB_PATH} missing: build it with `make -C oracle`")
        L = ctypes.CDLL(LIB_PATH)
        vp, i32, i64p = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_int64)
        L.cc_pos_size.restype = i32
        L.cc_init.restype = None
        L.cc_parse_fen.argtypes = [ctypes.c_char_p, vp]
        L.cc_parse_fen.restype = i32
        L.cc_legal.argtypes = [vp, ctypes.POINTER(ctypes.c_int), i64p, i32, ctypes.POINTER(ctypes.c_int)]
        L.cc_legal.restype = i32
        L.cc_push.argtypes = [vp, i32]
        L.cc_push.restype = None
        L.cc_encode.argtypes = [vp, i64p, ctypes.POINTER(ctypes.c_float), i64p, i64p]
        L.cc_encode.restype = None
        L.cc_halfmove.argtypes = [vp]
        L.cc_halfmove.restype = i32
        L.cc_turn.argtypes = [vp]
        L.cc_turn.restype = i32
        L.cc_key.argtypes = [vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int)]
        L.cc_key.restype = None
        L.cc_init()
        _lib = L
    return _lib


class Position:
    """One chess_core Pos (an opaque block), with legal moves, push and the network encoding."""

    def __init__(self, fen=START_FEN):
        L = lib()
        self.buf = ctypes.create_string_buffer(L.cc_pos_size())
        if not L.cc_parse_fen(fen.encode("ascii"), self.buf):
            raise ValueError(f"bad FEN {fen!r}")

    def copy(self):
        p = Position.__new__(Position)
        p.buf = ctypes.create_string_buffer(self.buf.raw, len(self.buf))
        return p

    def legal(self):
        """(move codes, policy indices) of the legal moves, python-chess order."""
        codes = (ctypes.c_int * MAX_MOVES)()
        idx = (ctypes.c_int64 * MAX_MOVES)()
        flags = ctypes.c_int(0)
        n = lib().cc_legal(self.buf, codes, idx, MAX_MOVES, ctypes.byref(flags))
        if n < 0 or n > MAX_MOVES:
            raise RuntimeError("chess_core move generator overflow")
        return list(codes[:n]), list(idx[:n])

    def push(self, code):
        lib().cc_push(self.buf, int(code))

    def key(self):
        """The transposition key (chess_core make_key = Board._transposition_key()): ten uint64 words in
        encode.py's _KEY10 order and the legal en passant square (-1 for None)."""
        k = np.zeros(10, np.uint64)
        ep = ctypes.c_int(0)
        lib().cc_key(self.buf, k.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), ctypes.byref(ep))
        return k, int(ep.value)

    def halfmove(self):
        return int(lib().cc_halfmove(self.buf))

    def encode(self):
        ids = np.zeros(64, np.int64)
        cast = np.zeros(4, np.float32)
        hm = ctypes.c_int64(0)
        ep = ctypes.c_int64(0)
        lib().cc_encode(self.buf, ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                        cast.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), ctypes.byref(hm), ctypes.byref(ep))
        return ids, cast, int(hm.value), int(ep.value)


def random_playouts(n, seed, max_plies):
    """n Positions from seeded uniform-random legal playouts of 0..max_plies plies (see the module docstring)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = []
    for _ in range(n):
        p = Position()
        plies = int(rng.integers(0, max_plies + 1))
        for _ in range(plies):
            codes, _ = p.legal()
            nxt = p.copy()
            nxt.push(codes[int(rng.integers(0, len(codes)))])
            if not nxt.legal()[0]:
                break           # mate or stalemate next: stop one ply earlier
            p = nxt
        out.append(p)
    return out


def key_batch(positions):
    """(keys uint64 (B, 10), ep int64 (B,) with -1 for None, clock int64 (B,)): what encode_keys reads."""
    B = len(positions)
    keys = np.zeros((B, 10), np.uint64)
    ep = np.zeros(B, np.int64)
    clock = np.zeros(B, np.int64)
    for i, p in enumerate(positions):
        keys[i], ep[i] = p.key()
        clock[i] = p.halfmove()
    return keys, ep, clock


def encode_batch(positions):
    """The network inputs for a list of Positions, I/M padded to the widest row (export_ts.make_batches)."""
    B = len(positions)
    ids = np.zeros((B, 64), np.int64)
    cast = np.zeros((B, 4), np.float32)
    hm = np.zeros(B, np.int64)
    ep = np.zeros(B, np.int64)
    rows = []
    for i, p in enumerate(positions):
        ids[i], cast[i], hm[i], ep[i] = p.encode()
        rows.append(p.legal()[1])
    widths = np.array([len(r) for r in rows], np.int32)
    wide = int(widths.max())
    I = np.zeros((B, wide), np.int64)
    M = np.zeros((B, wide), bool)
    for i, r in enumerate(rows):
        I[i, :len(r)] = r
        M[i, :len(r)] = True
    return dict(ids=ids, cast=cast, hm=hm, ep=ep, I=I, M=M, widths=widths)
