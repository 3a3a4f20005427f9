// TEST INFRASTRUCTURE ONLY. A flat C interface over the reference's own C++ chess core
// (mayfly/chess/cpp/chess_core.{h,cpp}), compiled from the reference's sources by oracle/Makefile into
// oracle/_ref/libchesscore.so. Only tests/golden/make_golden.py (fixture generation) and the tests load it.
// It is the position and encoding oracle: python-chess is not installed, and chess_core is the reference's
// port of python-chess's move generator (legal moves in python-chess order with their policy indices) and of
// the batch encoder mayfly_movegen.encode.
//
// Positions are opaque byte blocks of cc_pos_size() bytes owned by the caller.
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "chess_core.h"

using mayfly::Pos;

extern "C" {

// sizeof(mayfly::Pos), so Python can allocate a block for one position
int cc_pos_size() { return (int)sizeof(Pos); }

// chess_core.h:49 init_tables, once before anything else
void cc_init() { mayfly::init_tables(); }

// chess_core.cpp:511 parse_fen. Returns 1 on success, 0 on a malformed FEN.
int cc_parse_fen(const char* fen, void* out)
{
    Pos p;
    if (!mayfly::parse_fen(std::string(fen), p)) return 0;
    std::memcpy(out, &p, sizeof(Pos));
    return 1;
}

// chess_core.cpp:550 legal_moves on the position's transposition key (chess_core.cpp make_key): the move
// codes and the policy index of each (moves.py move_to_idx), in python-chess order. Writes at most cap of
// each, returns the number of legal moves, or -1 on a generator overflow.
int cc_legal(const void* pos, int* codes, int64_t* idx, int cap, int* flags)
{
    Pos p;
    std::memcpy(&p, pos, sizeof(Pos));
    std::vector<int> c;
    std::vector<int64_t> i;
    int f = 0;
    if (!mayfly::legal_moves(mayfly::make_key(p), c, i, f)) return -1;
    const int n = (int)c.size();
    for (int k = 0; k < n && k < cap; ++k) {
        codes[k] = c[(size_t)k];
        idx[k] = i[(size_t)k];
    }
    if (flags) *flags = f;
    return n;
}

// chess_core.cpp:464 push (python-chess Board.push), in place
void cc_push(void* pos, int code)
{
    Pos p;
    std::memcpy(&p, pos, sizeof(Pos));
    mayfly::push(p, code);
    std::memcpy(pos, &p, sizeof(Pos));
}

// chess_core.cpp:582 encode: ids[64], cast[4], hm (capped at 100) and ep (legal ep square + 1, 0 for none),
// all in the side to move's frame
void cc_encode(const void* pos, int64_t* ids, float* cast, int64_t* hm, int64_t* ep)
{
    Pos p;
    std::memcpy(&p, pos, sizeof(Pos));
    mayfly::encode(mayfly::make_key(p), p.hm, ids, cast, hm, ep);
}

// the halfmove clock and the side to move (1 white, 0 black) of a position
int cc_halfmove(const void* pos)
{
    Pos p;
    std::memcpy(&p, pos, sizeof(Pos));
    return p.hm;
}

int cc_turn(const void* pos)
{
    Pos p;
    std::memcpy(&p, pos, sizeof(Pos));
    return p.turn;
}

// chess_core.cpp make_key: python-chess's Board._transposition_key() (chess_core.h:15-27) as the ten 64-bit words
// encode.py:48 packs (pawns, knights, bishops, rooks, queens, kings, white, black, turn 1/0, clean castling
// rights) and the legal en passant square (-1 for None)
void cc_key(const void* pos, uint64_t* k10, int* ep)
{
    Pos p;
    std::memcpy(&p, pos, sizeof(Pos));
    const mayfly::Key k = mayfly::make_key(p);
    const uint64_t v[10] = {k.P, k.N, k.B, k.R, k.Q, k.K, k.W, k.Bk, (uint64_t)(k.turn ? 1 : 0), k.castle};
    std::memcpy(k10, v, sizeof(v));
    *ep = k.ep;
}

}  // extern "C"
