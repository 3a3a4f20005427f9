"""Batches of network inputs from a compact position set (the committed, seeded random-playout fixtures).

A position set (.npz) holds, for N positions already encoded as mayfly/chess/cpp/chess_core.cpp:582-612 encode
and legal_moves (:550-563) produce them:
    ids    uint8 [N, 64]   piece ids 0..12 in the side to move's frame
    cast   uint8 [N, 4]    castling rights (own K, own Q, their K, their Q), 0/1
    hm     uint8 [N]       halfmove clock bucket min(clock, 100)
    ep     uint8 [N]       legal en passant square + 1, 0 for none
    widths uint16 [N]      number of legal moves
    moves  uint16 [sum(widths)]  every position's legal moves' policy indices, python-chess order, concatenated
make_batch turns a slice of it into what MCTS._prepare builds (mayfly/chess/mcts.py:1004-1058,
cpp/export_ts.py:101-117 make_batches): ids int64 (B, 64), cast float32 (B, 4), hm int64 (B,), ep int64 (B,),
I int64 (B, wide) and M bool (B, wide), padded to the batch's widest row.
"""
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


class PositionSet:
    def __init__(self, path):
        z = np.load(path)
        self.ids = z["ids"]
        self.cast = z["cast"]
        self.hm = z["hm"]
        self.ep = z["ep"]
        self.widths = z["widths"].astype(np.int64)
        self.moves = z["moves"]
        self.offsets = np.concatenate([[0], np.cumsum(self.widths)])
        self.n = int(self.ids.shape[0])

    def __len__(self):
        return self.n

    def batch(self, start, B):
        """Positions start .. start+B-1 (cycling) as one padded batch dict."""
        idx = (np.arange(B) + start) % self.n
        widths = self.widths[idx]
        wide = int(widths.max())
        I = np.zeros((B, wide), np.int64)
        M = np.zeros((B, wide), bool)
        for r, j in enumerate(idx):
            w = int(self.widths[j])
            I[r, :w] = self.moves[self.offsets[j]:self.offsets[j] + w]
            M[r, :w] = True
        return dict(ids=self.ids[idx].astype(np.int64), cast=self.cast[idx].astype(np.float32),
                    hm=self.hm[idx].astype(np.int64), ep=self.ep[idx].astype(np.int64), I=I, M=M,
                    widths=widths.astype(np.int32))


def pack(batch):
    """The compact arrays of a padded batch dict (the inverse of PositionSet.batch), for np.savez."""
    widths = np.asarray(batch["widths"], np.int64)
    moves = np.concatenate([batch["I"][r, :w] for r, w in enumerate(widths)]).astype(np.uint16)
    return dict(ids=batch["ids"].astype(np.uint8), cast=batch["cast"].astype(np.uint8),
                hm=batch["hm"].astype(np.uint8), ep=batch["ep"].astype(np.uint8),
                widths=widths.astype(np.uint16), moves=moves)
