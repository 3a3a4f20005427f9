// The batch encoder from transposition keys, on the GPU.
//
// mayfly/chess/encode.py:73-100 encode_keys (with _castle_bits, encode.py:54-70), the reference's fast path
// for MCTS._prepare, decodes a batch of python-chess Board._transposition_key() tuples and halfmove clocks with
// numpy into the network's inputs. chess_core.cpp:582-612 encode is the same thing in C++ for one position.
// Here each (board, square) is one thread, so a batch's encoding is one launch that reads 96 bytes a board
// (instead of the 548 bytes of encoded inputs a board crossing PCIe) and writes the evaluator's input slots.
//
// Inputs per board b:
//   keys[10 b .. 10 b + 9]   pawns, knights, bishops, rooks, queens, kings, white, black (64-bit boards,
//                            bit s = square s, a1 = 0), turn (nonzero: white to move), clean castling rights
//   ep_sq[b]                 the key's legal en passant square, negative for None
//   clock[b]                 the halfmove clock
// Outputs, exactly encode_keys' values:
//   ids[64 b + s]   in the side to move's frame (square s reads board square s ^ 56 when black is to move):
//                   sum over piece types t of t * [bit of type t] + 6 * [bit of the side not to move]
//   cast[4 b + j]   own kingside, own queenside, their kingside, their queenside: a king of that colour on its
//                   back rank and a castling-rights bit on that rank above it (kingside) or below it
//                   (queenside), in 64-bit wrap-around arithmetic (a king on h8 has no square above it)
//   hm[b]           min(clock, 100)
//   ep[b]           (the square, mirrored when black is to move) + 1, or 0 for None
#pragma once
#include <cstdint>

#include "ptx.cuh"

namespace mf {

constexpr int kEncodeBoardsPerBlock = 4;   // 4 boards x 64 squares = 256 threads

__global__ void __launch_bounds__(64 * kEncodeBoardsPerBlock)
encode_keys_kernel(const uint64_t* __restrict__ keys, const int64_t* __restrict__ ep_sq,
                   const int64_t* __restrict__ clock, int B, int64_t* __restrict__ ids, float* __restrict__ cast,
                   int64_t* __restrict__ hm, int64_t* __restrict__ ep)
{
    griddep_wait();   // the keys may come from an earlier kernel's output
    const int b = blockIdx.x * kEncodeBoardsPerBlock + static_cast<int>(threadIdx.x >> 6);
    const int s = threadIdx.x & 63;
    if (b < B) {
        const uint64_t* k = keys + 10 * static_cast<size_t>(b);
        const bool white = k[8] != 0;
        const int src = white ? s : (s ^ 56);
        const uint64_t opp = white ? k[7] : k[6];
        int id = 0;
#pragma unroll
        for (int t = 0; t < 6; ++t) id += (t + 1) * static_cast<int>((k[t] >> src) & 1u);
        id += 6 * static_cast<int>((opp >> src) & 1u);
        ids[64 * static_cast<size_t>(b) + s] = id;
        if (s < 4) {
            constexpr uint64_t kRank1 = 0xFFull, kRank8 = 0xFFull << 56;
            const int side = (s < 2) == white ? 0 : 1;   // 0 white, 1 black; s 0, 1 the mover's, 2, 3 the other's
            const uint64_t king = side == 0 ? (k[5] & k[6] & kRank1) : (k[5] & k[7] & kRank8);
            const uint64_t rights = k[9] & (side == 0 ? kRank1 : kRank8);
            bool r = false;
            if (king) r = (s & 1) == 0 ? (rights & ~((king << 1) - 1)) != 0 : (rights & (king - 1)) != 0;
            cast[4 * static_cast<size_t>(b) + s] = r ? 1.0f : 0.0f;
        } else if (s == 4) {
            const int64_t c = clock[b];
            hm[b] = c < 100 ? c : 100;
        } else if (s == 5) {
            const int64_t e = ep_sq[b];
            ep[b] = e >= 0 ? (white ? e : (e ^ 56)) + 1 : 0;
        }
    }
    griddep_launch();
}

}  // namespace mf
