// Attention per (board, head) on the 5th-generation tensor cores (head width 64): the same arithmetic as
// attention_kernel (trunk.cuh; chess_net.py:159-161 SDPA, cudanet/kernels_trunk.cu:385-509), with both products
// as tcgen05.mma and the scores and outputs in tensor memory.
//
// Per item (board b, head h), with the 65 tokens of board b as rows 0..64:
//   S [128 x 80]  = Q K^T        A = Q tile (rows 0..79 from TMA, 80..127 zero), B = K tile (80 keys), K-major
//   P             = 2^(S * scale * log2 e - row max), keys 65..79 masked to 0 (bf16 or f16, in shared memory)
//   O [128 x 64]  = P V          A = P (K = 80 keys), B = the V tile read MN-major (its natural layout)
//   att row r     = O[r] / sum(P[r]), r < 65
// One CTA per SM, persistent over items blockIdx.x, + gridDim.x, ...; a ring of four Q/K/V tile sets keeps the
// loads several items ahead, and two compute slots (a P tile and tensor-memory columns for S and O) let the MMAs
// and the softmax of neighbouring items overlap:
//   warp 0       one thread TMA-loads Q, K, V of item n into load slot n % 4 (boxes of 64 columns x 80 rows)
//   warp 1       one thread issues S(n), then P(n-1) V(n-1); commits signal S ready, O ready, tiles free
//   warps 2..5   group 0, items of slot 0; warps 6..9 group 1, slot 1: thread = tensor-memory lane = query row:
//                the row's 80 scores come in with tcgen05.ld, the softmax runs in registers with no shuffles,
//                P goes to shared memory in the 128-byte-swizzled layout the second MMA reads, then the row of O
//                comes back, is normalised and stored.
// Every wait is bounded and every decision of a group is taken by its leader and broadcast, as in gemm.cuh.
#pragma once
#include "trunk.cuh"

namespace mf {

struct AttTcCfg {
    static constexpr int DH = 64;
#ifndef MF_ATT_LS
#define MF_ATT_LS 4
#endif
#ifndef MF_ATT_CS
#define MF_ATT_CS 2
#endif
    static constexpr int LS = MF_ATT_LS;                     // load slots (Q, K, V tile sets)
    static constexpr int CS = MF_ATT_CS;                     // compute slots (P tile, S and O columns), one
                                                             // softmax group of 4 warps each
    static constexpr int KEYS = 80;                          // 65 keys padded to a multiple of 16
    static constexpr uint32_t Q_BYTES = 128 * 128;           // 128 rows x 64 x 16-bit
    static constexpr uint32_t KV_BYTES = KEYS * 128;
    static constexpr uint32_t Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + KV_BYTES;
    static constexpr uint32_t LOAD_SLOT = V_OFF + KV_BYTES;  // 36 KB, a multiple of 1024
    static constexpr uint32_t P_CHUNK = 128 * 128;           // keys 0..63; a second chunk holds keys 64..79
    static constexpr uint32_t P_SLOT = 2 * P_CHUNK;
    static constexpr uint32_t P_BASE = LS * LOAD_SLOT;
    static constexpr uint32_t LOAD_BYTES = 3 * KEYS * 128;
    static constexpr size_t SMEM = 1024 + (size_t)P_BASE + CS * (size_t)P_SLOT + 256;
    static constexpr int THREADS = 64 + 128 * CS;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t T_STRIDE = CS == 2 ? 256 : 160;   // per compute slot: S (80 columns) at
    static constexpr uint32_t O_COL = CS == 2 ? 128 : 96;       // T_STRIDE * slot, O (64) at + O_COL
    static_assert(CS * T_STRIDE <= TMEM_COLS, "tensor memory per compute slot");
    static_assert(LOAD_SLOT % 1024 == 0 && K_OFF % 1024 == 0 && V_OFF % 1024 == 0 && P_BASE % 1024 == 0,
                  "swizzled tiles start on 1024-byte boundaries");
    static_assert(SMEM <= 232448, "shared memory over the per-block limit");
};

template <typename T, typename TO>
__global__ void __launch_bounds__(AttTcCfg::THREADS, 1)
attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, TO* __restrict__ att, int B, int heads, int d,
                    float scale, float mul, uint32_t* err)
{
    using C = AttTcCfg;
    constexpr int LS = C::LS, S = C::CS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + C::P_BASE + S * C::P_SLOT);   // [LS] Q, K, V landed
    uint64_t* empty = full + LS;    // [LS] the load slot's tiles are read (the P V commit)
    uint64_t* sfull = empty + LS;   // [CS] S in tensor memory
    uint64_t* pready = sfull + S;   // [CS] P in shared memory (the group's 4 warps)
    uint64_t* ofull = pready + S;   // [CS] O in tensor memory
    uint64_t* tfree = ofull + S;    // [CS] the compute slot's tensor-memory columns are read (the group's 4 warps)
    uint64_t* mma_done = tfree + S;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile uint32_t* ok = tmem_slot + 1;   // per group: its leader's broadcast

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = B * heads;
    const int my = (int)blockIdx.x < items ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    // Q rows 80..127 are never loaded: zero them once (the MMA reads all 128 rows; their results are unused)
    for (int i = threadIdx.x; i < LS * 48 * 8; i += blockDim.x) {
        const int sl = i / 384, rem = i % 384;
        *reinterpret_cast<uint4*>(base + sl * C::LOAD_SLOT + C::Q_OFF + (80 + rem / 8) * 128 + (rem % 8) * 16) =
            make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int i = 0; i < LS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < S; ++i) {
            mbar_init(&sfull[i], 1);
            mbar_init(&pready[i], 4);
            mbar_init(&ofull[i], 1);
            mbar_init(&tfree[i], 4);
        }
        mbar_init(mma_done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmQKV);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();   // qkv and att belong to the earlier kernels until they complete
    if (threadIdx.x == 0) griddep_launch();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t issued = 0, issued_par = 0;
            for (int n = 0; n < my; ++n) {
                const int slot = n % LS, use = n / LS;
                if (use > 0 && !mbar_wait(&empty[slot], (use - 1) & 1, err, kErrSmemEmpty)) break;
                const int item = (int)blockIdx.x + n * (int)gridDim.x;
                const int b = item / heads, h = item - b * heads;
                uint8_t* sb = base + slot * C::LOAD_SLOT;
                mbar_arrive_expect_tx(&full[slot], C::LOAD_BYTES);
                tma_load_2d(sb + C::Q_OFF, &tmQKV, &full[slot], h * C::DH, b * kTokens);
                tma_load_2d(sb + C::K_OFF, &tmQKV, &full[slot], d + h * C::DH, b * kTokens);
                tma_load_2d(sb + C::V_OFF, &tmQKV, &full[slot], 2 * d + h * C::DH, b * kTokens);
                issued |= 1u << slot;
                issued_par = (issued_par & ~(1u << slot)) | ((uint32_t)(use & 1) << slot);
            }
            for (int sl = 0; sl < LS; ++sl)
                if (issued & (1u << sl)) mbar_wait(&full[sl], (issued_par >> sl) & 1, err, kErrTmaFull);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = Operand<T>::idesc(128, C::KEYS);
            constexpr uint32_t idO = Operand<T>::idesc(128, C::DH) | (1u << 16);   // B (V) MN-major
            for (int n = 0; n <= my; ++n) {
                if (n < my) {
                    const int slot = n % S, use = n / S, ls = n % LS;
                    if (!mbar_wait(&full[ls], (n / LS) & 1, err, kErrTmaFull)) break;
                    if (use > 0 && !mbar_wait(&tfree[slot], (use - 1) & 1, err, kErrTmemEmpty)) break;
                    tc_fence_after();
                    const uint32_t sb = smem_u32(base + ls * C::LOAD_SLOT);
#pragma unroll
                    for (int k = 0; k < C::DH / 16; ++k)
                        umma_f16(tmem + C::T_STRIDE * slot, sdesc_sw128(sb + C::Q_OFF + 32u * k),
                                 sdesc_sw128(sb + C::K_OFF + 32u * k), idS, k > 0 ? 1u : 0u);
                    umma_commit(&sfull[slot]);
                }
                if (n >= 1) {
                    const int m = n - 1, slot = m % S, use = m / S, ls = m % LS;
                    if (!mbar_wait(&pready[slot], use & 1, err, kErrTmaFull)) break;
                    tc_fence_after();
                    const uint32_t sb = smem_u32(base + ls * C::LOAD_SLOT);
                    const uint32_t pb = smem_u32(base + C::P_BASE + slot * C::P_SLOT);
                    // K = 80 keys: steps 0..3 in P's first chunk (32 bytes a step), step 4 in the second; V's
                    // step is 16 keys = two 8-row swizzle atoms = 2048 bytes
#pragma unroll
                    for (int k = 0; k < C::KEYS / 16; ++k) {
                        const uint32_t pa = pb + (k < 4 ? 32u * k : C::P_CHUNK);
                        umma_f16(tmem + C::T_STRIDE * slot + C::O_COL, sdesc_sw128(pa), sdesc_sw128(sb + C::V_OFF + 2048u * k),
                                 idO, k > 0 ? 1u : 0u);
                    }
                    umma_commit(&ofull[slot]);
                    umma_commit(&empty[ls]);
                }
            }
            // every MMA issued has completed before tensor memory is freed
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, err, kErrTmemFull);
        }
    } else {
        // ---------------------------------------------------------------- softmax and output (two groups)
        const int grp = (warp - 2) >> 2;                 // group g takes the items of compute slot g
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;             // tensor-memory lane = query row
        const bool leader = threadIdx.x == 64 + 128 * grp;
        const uint32_t bar_id = 1 + grp;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const float sl2 = scale * 1.4426950408889634f;
        for (int n = grp; n < my; n += S) {
            const int slot = grp, use = n / S;
            const int item = (int)blockIdx.x + n * (int)gridDim.x;
            const int b = item / heads, h = item - b * heads;
            if (leader) ok[grp] = mbar_wait(&sfull[slot], use & 1, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(bar_id, 128);
            if (!ok[grp]) break;
            tc_fence_after();
            // this row's 80 scores
            float sc[C::KEYS];
            {
                uint32_t r0[32], r1[32], r2[16];
                const uint32_t ts = t_lane + C::T_STRIDE * slot;
                tmem_ld_32x32b_x32(ts, r0);
                tmem_ld_32x32b_x32(ts + 32, r1);
                tmem_ld_32x32b_x16(ts + 64, r2);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    sc[j] = __uint_as_float(r0[j]);
                    sc[32 + j] = __uint_as_float(r1[j]);
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) sc[64 + j] = __uint_as_float(r2[j]);
            }
            float mx = sc[0];
#pragma unroll
            for (int j = 1; j < kTokens; ++j) mx = fmaxf(mx, sc[j]);
            const float mc = mx * sl2;
            float sum = 0.f;
            uint32_t pk[C::KEYS / 2];
#pragma unroll
            for (int j = 0; j < C::KEYS; j += 2) {
                const float p0 = j < kTokens ? ex2_approx(fmaf(sc[j], sl2, -mc)) : 0.f;
                const float p1 = j + 1 < kTokens ? ex2_approx(fmaf(sc[j + 1], sl2, -mc)) : 0.f;
                sum += p0 + p1;
                pk[j / 2] = pack2<T>(p0, p1);
            }
            // P row into the slot's P tile: keys 0..63 in chunk 0 (8 units of 16 bytes), 64..79 in chunk 1
            uint8_t* pb = base + C::P_BASE + slot * C::P_SLOT;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                *reinterpret_cast<uint4*>(pb + swz<128>(row, u)) =
                    make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
#pragma unroll
            for (int u = 0; u < 2; ++u)
                *reinterpret_cast<uint4*>(pb + C::P_CHUNK + swz<128>(row, u)) =
                    make_uint4(pk[32 + 4 * u], pk[33 + 4 * u], pk[34 + 4 * u], pk[35 + 4 * u]);
            fence_proxy_async_smem();   // the MMA (async proxy) reads what these generic stores wrote
            __syncwarp();
            if (lane == 0) mbar_arrive(&pready[slot]);

            if (leader) ok[grp] = mbar_wait(&ofull[slot], use & 1, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(bar_id, 128);
            if (!ok[grp]) break;
            tc_fence_after();
            uint32_t o0[32], o1[32];
            tmem_ld_32x32b_x32(t_lane + C::T_STRIDE * slot + C::O_COL, o0);
            tmem_ld_32x32b_x32(t_lane + C::T_STRIDE * slot + C::O_COL + 32u, o1);
            tmem_ld_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tfree[slot]);   // S and O of this slot are read
            if (row < kTokens) {
                const float inv = 1.f / sum;
                const size_t orow = (size_t)b * kTokens + row;
                if constexpr (is_e4m3<TO>) {
                    const float m = inv * mul;
                    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(att) + orow * d + (size_t)h * C::DH);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        const uint32_t* src = u < 2 ? o0 + 16 * u : o1 + 16 * (u - 2);
                        uint32_t w[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            w[i] = pack_e4m3x4(__uint_as_float(src[4 * i]) * m, __uint_as_float(src[4 * i + 1]) * m,
                                               __uint_as_float(src[4 * i + 2]) * m, __uint_as_float(src[4 * i + 3]) * m);
                        dst[u] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                } else {
                    uint4* dst = reinterpret_cast<uint4*>(att + orow * d + (size_t)h * C::DH);
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const uint32_t* src = u < 4 ? o0 + 8 * u : o1 + 8 * (u - 4);
                        dst[u] = make_uint4(pack2<T>(__uint_as_float(src[0]) * inv, __uint_as_float(src[1]) * inv),
                                            pack2<T>(__uint_as_float(src[2]) * inv, __uint_as_float(src[3]) * inv),
                                            pack2<T>(__uint_as_float(src[4]) * inv, __uint_as_float(src[5]) * inv),
                                            pack2<T>(__uint_as_float(src[6]) * inv, __uint_as_float(src[7]) * inv));
                    }
                }
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace mf
