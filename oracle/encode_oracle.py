"""TEST INFRASTRUCTURE ONLY: a numpy restatement of the reference's batch encoder from transposition keys.

mayfly/chess/encode.py:73-100 encode_keys (with _castle_bits, encode.py:54-70) turns a batch of python-chess
Board._transposition_key() tuples and halfmove clocks into the network's inputs: ids (B, 64) int64 in the side
to move's frame (0 empty, 1..6 the mover's P N B R Q K, 7..12 the opponent's), cast (B, 4) float32 (own
kingside, own queenside, their kingside, their queenside), hm (B,) int64 = min(clock, 100) and ep (B,) int64
(legal en passant square + 1 in the mover's frame, 0 for none). This module restates it on arrays:

    keys   uint64 (B, 10)  pawns, knights, bishops, rooks, queens, kings, white, black, turn (1 white), castling
    ep_sq  int64 (B,)      the key's legal en passant square, -1 for None
    clock  int64 (B,)      the halfmove clock

It is the checker of the GPU encoder (cudanet_encode_keys) and is pinned to the reference's own encode_keys
through tests/golden/keys_seed1.npz (made by tests/golden/make_golden.py, which runs encode.py itself). Only
tests use it; the product never imports it.
"""
import numpy as np

RANK1 = np.uint64(0xFF)
RANK8 = np.uint64(0xFF) << np.uint64(56)


def castle_bits(keys, black):
    """encode.py:54-70 _castle_bits: a right needs a king of that colour on its back rank and a castling-rights
    bit on that rank above the king (kingside) or below it (queenside); 64-bit wrap-around arithmetic as numpy's."""
    kings, cr = keys[:, 5], keys[:, 9]
    K = np.stack([kings & keys[:, 6] & RANK1, kings & keys[:, 7] & RANK8], 1)
    C = np.stack([cr & RANK1, cr & RANK8], 1)
    one = np.uint64(1)
    with np.errstate(over="ignore"):
        ok = K != 0
        ks = ok & ((C & ~((K << one) - one)) != 0)
        qs = ok & ((C & (K - one)) != 0)
    r = np.arange(keys.shape[0])
    mover = black.astype(np.intp)
    other = 1 - mover
    return np.stack([ks[r, mover], qs[r, mover], ks[r, other], qs[r, other]], 1).astype(np.float32)


def encode_keys(keys, ep_sq, clock):
    """encode.py:73-100 encode_keys on arrays: (ids, cast, hm, ep) exactly as the reference returns them."""
    keys = np.ascontiguousarray(keys, np.uint64).reshape(-1, 10)
    B = keys.shape[0]
    ep_sq = np.asarray(ep_sq, np.int64).reshape(B)
    clock = np.asarray(clock, np.int64).reshape(B)
    white = keys[:, 8] != 0
    black = ~white
    bb = np.empty((B, 7), np.uint64)
    bb[:, :6] = keys[:, :6]
    bb[:, 6] = np.where(white, keys[:, 7], keys[:, 6])          # the side not to move
    sq = np.arange(64, dtype=np.uint64)
    # the mover's square s reads the board's square s ^ 56 when black is to move (encode.py:90 byteswap)
    src = np.where(black[:, None], sq[None, :] ^ np.uint64(56), sq[None, :])                   # (B, 64)
    bits = ((bb[:, :, None] >> src[:, None, :]) & np.uint64(1)).astype(np.uint8)               # (B, 7, 64)
    w6 = np.arange(1, 7, dtype=np.uint8).reshape(1, 6, 1)
    ids = ((bits[:, :6] * w6).sum(1, dtype=np.uint8) + 6 * bits[:, 6]).astype(np.int64)
    cast = castle_bits(keys, black)
    hm = np.minimum(clock, 100)
    ep = np.where(ep_sq >= 0, np.where(black, ep_sq ^ 56, ep_sq) + 1, 0).astype(np.int64)
    return ids, cast, hm, ep
