// Attention per (board, head) on the 5th-generation tensor cores (head width 64): the same arithmetic as
// attention_kernel (trunk.cuh; chess_net.py:159-161 SDPA, cudanet/kernels_trunk.cu:385-509), with both products
// as tcgen05.mma and the scores and outputs in tensor memory.
//
// Per item (board b, head h), with the 65 tokens of board b as rows 0..64:
//   S [128 x 80] = Q K^T       A = Q tile (rows 0..79 from TMA, 80..127 zero), B = K tile (keys 0..79), K-major
//                  (rows past 64 are padding: the warp of rows 96..127 skips them)
//   P            = 2^(S * scale * log2 e - row max), keys 65..79 masked to 0, rounded to the 16-bit type
//   O [128 x 64] = P[:, 0:64] V[0:64] + P[:, 64] V[64]
//                  the first term a tcgen05.mma (A = P in the Q tile's place, B = the V tile read MN-major, its
//                  natural layout), the second, the last live key, a rank-1 update on the CUDA cores
//   att row r    = O[r] / sum(P[r]), r < 65
// One CTA per SM, persistent over items blockIdx.x, + gridDim.x, ...:
//   warp 0       one thread TMA-loads Q, K, V of item n into load slot n % LS (boxes of 64 columns x 80 rows)
//   warp 1       one thread issues S(n) into tensor-memory slot n % 4, then P(n-1) V(n-1) into the same
//                columns as S(n-1) (read by then); commits signal S ready and O ready
//   warps 2..9   two groups of 4 warps, group g the items n = g mod 2; thread = tensor-memory lane = query row.
//                A group writes P(i), then finishes item i-1 (its O is ready by then): the row's 80 scores come
//                in with tcgen05.ld and the softmax runs in registers, P goes over the item's Q tile (free once S
//                is done) in the 128-byte-swizzled layout the second MMA reads; the row of O is normalised and
//                stored, and the load slot and tensor-memory slot are handed back.
// Every wait is bounded and every decision of a group is taken by its leader and broadcast, as in gemm.cuh.
#pragma once
#include "trunk.cuh"

namespace mf {

struct AttTcCfg {
    static constexpr int DH = 64;
    static constexpr int LS = 6;                             // load slots (Q, K, V tile sets)
    static constexpr int TS = 4;                             // tensor-memory slots (two per softmax group)
    static constexpr int KEYS = 80;                          // 65 keys padded to a multiple of 16
    static constexpr uint32_t Q_BYTES = 128 * 128;           // 128 rows x 64 x 16-bit; P[:, 0:64] afterwards
    static constexpr uint32_t KV_BYTES = KEYS * 128;
    static constexpr uint32_t Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + KV_BYTES;
    static constexpr uint32_t LOAD_SLOT = V_OFF + KV_BYTES;  // 36 KB, a multiple of 1024
    static constexpr uint32_t LOAD_BYTES = 3 * KEYS * 128;
    static constexpr size_t SMEM = 1024 + LS * (size_t)LOAD_SLOT + 256;
    static constexpr int THREADS = 64 + 256;
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t T_STRIDE = 128;                // slot t: S at 128 t (80 columns), then O there (64)
    static_assert(LOAD_SLOT % 1024 == 0 && K_OFF % 1024 == 0 && V_OFF % 1024 == 0, "1024-byte aligned tiles");
    static_assert(TS * T_STRIDE <= TMEM_COLS && SMEM <= 232448, "resources");
};

template <typename T, typename TO>
__global__ void __launch_bounds__(AttTcCfg::THREADS, 1)
attention_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, TO* __restrict__ att, int B, int heads, int d,
                    float scale, float mul, uint32_t* err)
{
    using C = AttTcCfg;
    constexpr int LS = C::LS, TS = C::TS;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + LS * C::LOAD_SLOT);   // [LS] Q, K, V landed
    uint64_t* empty = full + LS;     // [LS] the load slot is finished with (its group's 4 warps)
    uint64_t* sfull = empty + LS;    // [TS] S in tensor memory
    uint64_t* pready = sfull + TS;   // [TS] P in shared memory (the group's 4 warps)
    uint64_t* ofull = pready + TS;   // [TS] O in tensor memory
    uint64_t* tfree = ofull + TS;    // [TS] the slot's columns are read (the group's 4 warps)
    uint64_t* mma_done = tfree + TS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile uint32_t* ok = tmem_slot + 1;   // [2 groups x 2]: the leaders' broadcasts

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = B * heads;
    const int my = (int)blockIdx.x < items ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    // Q rows 80..127 are never loaded: zero them once (the MMA reads all 128 rows; their results are unused;
    // P overwrites them with the probabilities of those rows, finite too)
    for (int i = threadIdx.x; i < LS * 48 * 8; i += blockDim.x) {
        const int sl = i / 384, rem = i % 384;
        *reinterpret_cast<uint4*>(base + sl * C::LOAD_SLOT + C::Q_OFF + (80 + rem / 8) * 128 + (rem % 8) * 16) =
            make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int i = 0; i < LS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 4);
        }
        for (int i = 0; i < TS; ++i) {
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
                const int ls = n % LS, use = n / LS;
                if (use > 0 && !mbar_wait(&empty[ls], (use - 1) & 1, err, kErrSmemEmpty)) break;
                const int item = (int)blockIdx.x + n * (int)gridDim.x;
                const int b = item / heads, h = item - b * heads;
                uint8_t* sb = base + ls * C::LOAD_SLOT;
                mbar_arrive_expect_tx(&full[ls], C::LOAD_BYTES);
                tma_load_2d(sb + C::Q_OFF, &tmQKV, &full[ls], h * C::DH, b * kTokens);
                tma_load_2d(sb + C::K_OFF, &tmQKV, &full[ls], d + h * C::DH, b * kTokens);
                tma_load_2d(sb + C::V_OFF, &tmQKV, &full[ls], 2 * d + h * C::DH, b * kTokens);
                issued |= 1u << ls;
                issued_par = (issued_par & ~(1u << ls)) | ((uint32_t)(use & 1) << ls);
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
                    const int ts = n % TS, ls = n % LS;
                    if (!mbar_wait(&full[ls], (n / LS) & 1, err, kErrTmaFull)) break;
                    if (n >= TS && !mbar_wait(&tfree[ts], (n / TS - 1) & 1, err, kErrTmemEmpty)) break;
                    tc_fence_after();
                    const uint32_t sb = smem_u32(base + ls * C::LOAD_SLOT);
#pragma unroll
                    for (int k = 0; k < C::DH / 16; ++k)
                        umma_f16(tmem + C::T_STRIDE * ts, sdesc_sw128(sb + C::Q_OFF + 32u * k),
                                 sdesc_sw128(sb + C::K_OFF + 32u * k), idS, k > 0 ? 1u : 0u);
                    umma_commit(&sfull[ts]);
                }
                if (n >= 1) {
                    const int m = n - 1, ts = m % TS, ls = m % LS;
                    if (!mbar_wait(&pready[ts], (m / TS) & 1, err, kErrTmaFull)) break;
                    tc_fence_after();
                    const uint32_t sb = smem_u32(base + ls * C::LOAD_SLOT);
                    // keys 0..63: P over the Q tile (32 bytes a 16-key step), V's step 16 keys = 2048 bytes
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        umma_f16(tmem + C::T_STRIDE * ts, sdesc_sw128(sb + C::Q_OFF + 32u * k),
                                 sdesc_sw128(sb + C::V_OFF + 2048u * k), idO, k > 0 ? 1u : 0u);
                    umma_commit(&ofull[ts]);
                }
            }
            // every MMA issued has completed before tensor memory is freed
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, err, kErrTmemFull);
        }
    } else {
        // ---------------------------------------------------------------- softmax and output (two groups)
        const int grp = (warp - 2) >> 2;                 // group g takes the items n = g mod 2
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;             // tensor-memory lane = query row
        // rows 96..127 are padding: their warp only keeps the handshakes (the MMA reads their P rows, which hold
        // finite leftovers, and their O rows are never stored)
        const bool live = quarter < 3;
        const bool leader = threadIdx.x == 64 + 128 * grp;
        const uint32_t bar_id = 1 + grp;
        const uint32_t t_lane = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
        const float sl2 = scale * 1.4426950408889634f;
        float inv_prev = 0.f, p64_prev = 0.f;           // the pending item's 1 / sum and P[row, 64]
        int prev = -1;                                   // the pending item (its O not yet read)

        // item m's O row: + P[row, 64] V[64], / sum, stored; then its slots handed back
        auto finish = [&](int m, float inv, float p64) -> bool {
            const int ts = m % TS, ls = m % LS;
            if (leader) ok[2 * grp + 1] = mbar_wait(&ofull[ts], (m / TS) & 1, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(bar_id, 128);
            if (!ok[2 * grp + 1]) return false;
            if (!live) {
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&tfree[ts]);
                    mbar_arrive(&empty[ls]);
                }
                return true;
            }
            tc_fence_after();
            uint32_t o0[32], o1[32];
            tmem_ld_32x32b_x32(t_lane + C::T_STRIDE * ts, o0);
            tmem_ld_32x32b_x32(t_lane + C::T_STRIDE * ts + 32u, o1);
            tmem_ld_wait();
            tc_fence_before();
            // V[64] (row 64 of the V tile: swizzle row 64 % 8 = 0, so its 16-byte units are in order)
            const uint4* v64 = reinterpret_cast<const uint4*>(base + ls * C::LOAD_SLOT + C::V_OFF + 64 * 128);
            float o[C::DH];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint4 q = v64[u];
                const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int c = 8 * u + 2 * i;
                    const uint32_t* src = c < 32 ? o0 + c : o1 + (c - 32);
                    o[c] = fmaf(p64, to_f32<T>(reinterpret_cast<const T*>(&w[i])[0]), __uint_as_float(src[0])) * inv;
                    o[c + 1] =
                        fmaf(p64, to_f32<T>(reinterpret_cast<const T*>(&w[i])[1]), __uint_as_float(src[1])) * inv;
                }
            }
            fence_proxy_async_smem();   // the TMA refill of the load slot comes after these reads
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tfree[ts]);   // the slot's columns are read
                mbar_arrive(&empty[ls]);   // and the load slot (P, V[64]) too
            }
            if (row < kTokens) {
                const int item = (int)blockIdx.x + m * (int)gridDim.x;
                const int b = item / heads, h = item - b * heads;
                const size_t orow = (size_t)b * kTokens + row;
                if constexpr (is_e4m3<TO>) {
                    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(att) + orow * d + (size_t)h * C::DH);
#pragma unroll
                    for (int u = 0; u < 4; ++u) {
                        uint32_t w[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i)
                            w[i] = pack_e4m3x4(o[16 * u + 4 * i] * mul, o[16 * u + 4 * i + 1] * mul,
                                               o[16 * u + 4 * i + 2] * mul, o[16 * u + 4 * i + 3] * mul);
                        dst[u] = make_uint4(w[0], w[1], w[2], w[3]);
                    }
                } else {
                    uint4* dst = reinterpret_cast<uint4*>(att + orow * d + (size_t)h * C::DH);
#pragma unroll
                    for (int u = 0; u < 8; ++u)
                        dst[u] = make_uint4(pack2<T>(o[8 * u], o[8 * u + 1]), pack2<T>(o[8 * u + 2], o[8 * u + 3]),
                                            pack2<T>(o[8 * u + 4], o[8 * u + 5]), pack2<T>(o[8 * u + 6], o[8 * u + 7]));
                }
            }
            return true;
        };

        bool good = true;
        for (int n = grp; n < my && good; n += 2) {
            const int ts = n % TS, ls = n % LS;
            if (leader) ok[2 * grp] = mbar_wait(&sfull[ts], (n / TS) & 1, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(bar_id, 128);
            if (!ok[2 * grp]) break;
            if (!live) {
                __syncwarp();
                if (lane == 0) mbar_arrive(&pready[ts]);
                if (prev >= 0) good = finish(prev, 0.f, 0.f);
                prev = n;
                continue;
            }
            tc_fence_after();
            // this row's 80 scores
            float sc[C::KEYS];
            {
                uint32_t r0[32], r1[32], r2[16];
                const uint32_t tsa = t_lane + C::T_STRIDE * ts;
                tmem_ld_32x32b_x32(tsa, r0);
                tmem_ld_32x32b_x32(tsa + 32, r1);
                tmem_ld_32x32b_x16(tsa + 64, r2);
                tmem_ld_wait();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    sc[j] = __uint_as_float(r0[j]);
                    sc[32 + j] = __uint_as_float(r1[j]);
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) sc[64 + j] = __uint_as_float(r2[j]);
            }
            // row max over the 65 live keys (eight independent chains), then the exponentials and their sum
            float m8[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) m8[i] = sc[i];
#pragma unroll
            for (int j = 8; j < 64; ++j) m8[j & 7] = fmaxf(m8[j & 7], sc[j]);
            m8[0] = fmaxf(m8[0], sc[64]);
            const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                   fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
            const float mc = mx * sl2;
            float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            uint32_t pk[32];
#pragma unroll
            for (int j = 0; j < 64; j += 2) {
                const float p0 = ex2_approx(fmaf(sc[j], sl2, -mc));
                const float p1 = ex2_approx(fmaf(sc[j + 1], sl2, -mc));
                // P goes to the MMA rounded to the 16-bit type; the sum is of the f32 probabilities
                pk[j / 2] = pack2<T>(p0, p1);
                s8[(j / 2) & 7] += p0 + p1;
            }
            const float p64 = ex2_approx(fmaf(sc[64], sl2, -mc));
            const float sum = ((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])) + p64;
            // P[:, 0:64] over the Q tile (free: S is done)
            uint8_t* pb = base + ls * C::LOAD_SLOT + C::Q_OFF;
#pragma unroll
            for (int u = 0; u < 8; ++u)
                *reinterpret_cast<uint4*>(pb + swz<128>(row, u)) =
                    make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
            fence_proxy_async_smem();   // the MMA (async proxy) reads what these generic stores wrote
            tc_fence_before();          // and overwrites the S columns this thread has read
            __syncwarp();
            if (lane == 0) mbar_arrive(&pready[ts]);
            // the previous item's O is ready by now
            if (prev >= 0) good = finish(prev, inv_prev, p64_prev);
            prev = n;
            inv_prev = 1.f / sum;
            p64_prev = p64;
        }
        if (good && prev >= 0) finish(prev, inv_prev, p64_prev);
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------ four groups
// The same arithmetic with four softmax groups, group n % 4 taking item n and finishing it before it takes the
// next: S(n) -> softmax -> P over the Q tile -> (PV(n) on the tensor cores) -> O(n) normalised and stored ->
// slots handed back. Four items are in flight instead of two. A group is the 3 warps whose tensor-memory lane
// quarters hold the 65 live query rows (rows 0..95; rows 96..127 are padding, so no warp reads them): warps
// 4g, 4g + 1, 4g + 2 of the 16 (512 threads); warp 3 issues the TMA loads, warp 7 owns tensor memory and
// issues the MMAs, warps 11 and 15 have no role. With 16 warps a thread may hold 128 registers, so a row's 80
// scores come out of tensor memory in one pass (three loads, one wait), and its 64 outputs in another. Item n's
// scores and output live in tensor-memory slot n % NS (NS = 5 slots of 96 columns, S taking 80 and O 64 of
// them): one more slot than groups, so the S product of a group's next item runs while the group still works on
// its current one. The MMA thread issues whichever of the next S (its load landed, its slot free) and the next
// PV (its P written) is ready first, polling with mbarrier.test_wait (which never suspends the thread on one
// barrier while the other is ready); it gives up after the wait limit with no progress.
struct AttTc4Cfg {
    static constexpr int DH = 64;
    static constexpr int LS = 6;
    static constexpr int G = 4;                              // softmax groups
    static constexpr int GW = 3;                             // warps a group (lane quarters 0..2)
    static constexpr int NS = 5;                             // tensor-memory slots
    static constexpr int KEYS = 80;
    static constexpr uint32_t Q_BYTES = 128 * 128;
    static constexpr uint32_t KV_BYTES = KEYS * 128;
    static constexpr uint32_t Q_OFF = 0, K_OFF = Q_BYTES, V_OFF = K_OFF + KV_BYTES;
    static constexpr uint32_t LOAD_SLOT = V_OFF + KV_BYTES;
    static constexpr uint32_t LOAD_BYTES = 3 * KEYS * 128;
    static constexpr size_t SMEM = 1024 + LS * (size_t)LOAD_SLOT + 512;
    static constexpr int THREADS = 512;
    static constexpr int LOAD_WARP = 3, MMA_WARP = 7;        // warps of lane quarter 3, which holds no live row
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr uint32_t T_STRIDE = 96;
    static_assert(LOAD_SLOT % 1024 == 0 && K_OFF % 1024 == 0 && V_OFF % 1024 == 0, "1024-byte aligned tiles");
    static_assert(NS * T_STRIDE <= TMEM_COLS && T_STRIDE >= KEYS && NS > G && SMEM <= 232448, "resources");
    static_assert((2 * LS + 3 * NS + G + 1) * 8 + 4 + 8 * G <= 512, "barriers");
    static_assert(G * 4 * 32 == THREADS && GW * 32 > kTokens, "warp roles");
};

template <typename T, typename TO>
__global__ void __launch_bounds__(AttTc4Cfg::THREADS, 1)
attention_tc4_kernel(const __grid_constant__ CUtensorMap tmQKV, TO* __restrict__ att, int B, int heads, int d,
                     float scale, float mul, uint32_t* err, int rev)
{
    using C = AttTc4Cfg;
    constexpr int LS = C::LS, G = C::G, NS = C::NS, GW = C::GW;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(base + LS * C::LOAD_SLOT);   // [LS] Q, K, V landed
    uint64_t* empty = full + LS;     // [LS] the load slot is finished with (its group's warps)
    uint64_t* sfull = empty + LS;    // [NS] S in the tensor-memory slot
    uint64_t* ofull = sfull + NS;    // [NS] O in the slot
    uint64_t* tfree = ofull + NS;    // [NS] the slot is read (its group's warps)
    uint64_t* pready = tfree + NS;   // [G] the group's P in shared memory (its warps)
    uint64_t* mma_done = pready + G;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
    volatile uint32_t* ok = tmem_slot + 1;   // [G x 2]: the leaders' broadcasts

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int quarter = warp & 3;
    const int items = B * heads;
    const int my = (int)blockIdx.x < items ? (items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    for (int i = threadIdx.x; i < LS * 48 * 8; i += blockDim.x) {
        const int sl = i / 384, rem = i % 384;
        *reinterpret_cast<uint4*>(base + sl * C::LOAD_SLOT + C::Q_OFF + (80 + rem / 8) * 128 + (rem % 8) * 16) =
            make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int i = 0; i < LS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], GW);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(&sfull[i], 1);
            mbar_init(&ofull[i], 1);
            mbar_init(&tfree[i], GW);
        }
        for (int i = 0; i < G; ++i) mbar_init(&pready[i], GW);
        mbar_init(mma_done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmQKV);
    }
    if (warp == C::MMA_WARP) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    griddep_wait();
    if (threadIdx.x == 0) griddep_launch();

    if (warp == C::LOAD_WARP) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t issued = 0, issued_par = 0;
            for (int n = 0; n < my; ++n) {
                const int ls = n % LS, use = n / LS;
                if (use > 0 && !mbar_wait(&empty[ls], (use - 1) & 1, err, kErrSmemEmpty)) break;
                const int item = (int)blockIdx.x + n * (int)gridDim.x;
                const int bf = item / heads, h = item - bf * heads;
                const int b = rev ? B - 1 - bf : bf;   // rev: boards in descending order
                uint8_t* sb = base + ls * C::LOAD_SLOT;
                mbar_arrive_expect_tx(&full[ls], C::LOAD_BYTES);
                tma_load_2d(sb + C::Q_OFF, &tmQKV, &full[ls], h * C::DH, b * kTokens);
                tma_load_2d(sb + C::K_OFF, &tmQKV, &full[ls], d + h * C::DH, b * kTokens);
                tma_load_2d(sb + C::V_OFF, &tmQKV, &full[ls], 2 * d + h * C::DH, b * kTokens);
                issued |= 1u << ls;
                issued_par = (issued_par & ~(1u << ls)) | ((uint32_t)(use & 1) << ls);
            }
            for (int sl = 0; sl < LS; ++sl)
                if (issued & (1u << sl)) mbar_wait(&full[sl], (issued_par >> sl) & 1, err, kErrTmaFull);
        }
    } else if (warp == C::MMA_WARP) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idS = Operand<T>::idesc(128, C::KEYS);
            constexpr uint32_t idO = Operand<T>::idesc(128, C::DH) | (1u << 16);   // B (V) MN-major
            int ns = 0, np = 0;                    // the next S and the next PV to issue
            uint64_t t0 = globaltimer();
            uint32_t idle = 0;
            while (np < my) {
                bool progressed = false;
                if (ns < my && ns < np + NS) {
                    const int ls = ns % LS, ts = ns % NS;
                    if (mbar_test_wait(&full[ls], (ns / LS) & 1) &&
                        (ns < NS || mbar_test_wait(&tfree[ts], (ns / NS - 1) & 1))) {
                        tc_fence_after();
                        const uint32_t sb = smem_u32(base + ls * C::LOAD_SLOT);
#pragma unroll
                        for (int k = 0; k < C::DH / 16; ++k)
                            umma_f16(tmem + C::T_STRIDE * ts, sdesc_sw128(sb + C::Q_OFF + 32u * k),
                                     sdesc_sw128(sb + C::K_OFF + 32u * k), idS, k > 0 ? 1u : 0u);
                        umma_commit(&sfull[ts]);
                        ++ns;
                        progressed = true;
                    }
                }
                if (np < ns) {
                    const int ls = np % LS, g = np % G, ts = np % NS;
                    if (mbar_test_wait(&pready[g], (np / G) & 1)) {
                        tc_fence_after();
                        const uint32_t sb = smem_u32(base + ls * C::LOAD_SLOT);
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            umma_f16(tmem + C::T_STRIDE * ts, sdesc_sw128(sb + C::Q_OFF + 32u * k),
                                     sdesc_sw128(sb + C::V_OFF + 2048u * k), idO, k > 0 ? 1u : 0u);
                        umma_commit(&ofull[ts]);
                        ++np;
                        progressed = true;
                    }
                }
                if (progressed) {
                    idle = 0;
                } else if ((++idle & 1023u) == 0) {
                    const uint64_t now = globaltimer();
                    if (idle == 1024u) t0 = now;          // the start of this stretch without progress
                    else if (now - t0 > kWaitLimitNs) {
                        set_error(err, kErrTmaFull);
                        break;
                    }
                }
            }
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, err, kErrTmemFull);
        }
    } else if (quarter < GW) {
        // ---------------------------------------------------------------- softmax and output (four groups)
        const int grp = warp >> 2;
        const int row = quarter * 32 + lane;
        const bool leader = threadIdx.x == 128 * grp;
        const uint32_t bar_id = 1 + grp;
        const float sl2 = scale * 1.4426950408889634f;
        for (int n = grp; n < my; n += G) {
            const int ls = n % LS, ts = n % NS;
            const uint32_t par = (n / NS) & 1;   // the phase of item n's tensor-memory slot
            const uint32_t t_row = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + C::T_STRIDE * ts;
            if (leader) ok[2 * grp] = mbar_wait(&sfull[ts], par, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(bar_id, 32 * GW);
            if (!ok[2 * grp]) break;
            tc_fence_after();
            float p64, sum;
            {
                // the row's 80 scores in one pass: keys 0..63, then 64.. (key 64 the last live one)
                uint32_t ra[32], rb[32], r16[16];   // keys 0..31, 32..63, 64..79
                tmem_ld_32x32b_x32(t_row, ra);
                tmem_ld_32x32b_x32(t_row + 32, rb);
                tmem_ld_32x32b_x16(t_row + 64, r16);
                tmem_ld_wait();
                const float s64 = __uint_as_float(r16[0]);
                float m4[4] = {s64, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    m4[j & 3] = fmaxf(m4[j & 3], __uint_as_float(ra[j]));
                    m4[j & 3] = fmaxf(m4[j & 3], __uint_as_float(rb[j]));
                }
                const float mc = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;
                // exponentials, their sum, P (rounded to T) over the Q tile
                uint8_t* pb = base + ls * C::LOAD_SLOT + C::Q_OFF;
                float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    uint32_t pk[16];
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const uint32_t* rh = hh == 0 ? ra : rb;
                        const float p0 = ex2_approx(fmaf(__uint_as_float(rh[j]), sl2, -mc));
                        const float p1 = ex2_approx(fmaf(__uint_as_float(rh[j + 1]), sl2, -mc));
                        pk[j / 2] = pack2<T>(p0, p1);
                        s4[(j / 2) & 3] += p0 + p1;
                    }
#pragma unroll
                    for (int u = 0; u < 4; ++u)
                        *reinterpret_cast<uint4*>(pb + swz<128>(row, 4 * hh + u)) =
                            make_uint4(pk[4 * u], pk[4 * u + 1], pk[4 * u + 2], pk[4 * u + 3]);
                }
                p64 = ex2_approx(fmaf(s64, sl2, -mc));
                sum = ((s4[0] + s4[1]) + (s4[2] + s4[3])) + p64;
            }
            fence_proxy_async_smem();   // the MMA (async proxy) reads what these generic stores wrote
            tc_fence_before();          // and overwrites the S columns this thread has read
            __syncwarp();
            if (lane == 0) mbar_arrive(&pready[grp]);
            if (leader) ok[2 * grp + 1] = mbar_wait(&ofull[ts], par, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(bar_id, 32 * GW);
            if (!ok[2 * grp + 1]) break;
            tc_fence_after();
            {
                const float inv = (is_e4m3<TO> ? mul : 1.f) / sum;   // e4m3: att * mul, folded into 1 / sum
                const uint4* v64 = reinterpret_cast<const uint4*>(base + ls * C::LOAD_SLOT + C::V_OFF + 64 * 128);
                const int item = (int)blockIdx.x + n * (int)gridDim.x;
                const int bf = item / heads, h = item - bf * heads;
                const int b = rev ? B - 1 - bf : bf;
                const size_t orow = (size_t)b * kTokens + row;
                uint32_t ra[32], rb[32];   // output columns 0..31, 32..63
                tmem_ld_32x32b_x32(t_row, ra);
                tmem_ld_32x32b_x32(t_row + 32, rb);
                tmem_ld_wait();
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) {   // 16 output columns at a time
                    float o[16];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint4 q = v64[2 * qq + u];
                        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int c = 8 * u + 2 * i;
                            o[c] = fmaf(p64, to_f32<T>(reinterpret_cast<const T*>(&w[i])[0]),
                                        __uint_as_float((qq < 2 ? ra : rb)[16 * (qq & 1) + c])) * inv;
                            o[c + 1] = fmaf(p64, to_f32<T>(reinterpret_cast<const T*>(&w[i])[1]),
                                            __uint_as_float((qq < 2 ? ra : rb)[16 * (qq & 1) + c + 1])) * inv;
                        }
                    }
                    if (row < kTokens) {
                        if constexpr (is_e4m3<TO>) {
                            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(att) + orow * d +
                                                                  (size_t)h * C::DH + 16 * qq);
                            uint32_t w[4];
#pragma unroll
                            for (int i = 0; i < 4; ++i)
                                w[i] = pack_e4m3x4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                            dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                        } else {
                            uint4* dst = reinterpret_cast<uint4*>(att + orow * d + (size_t)h * C::DH + 16 * qq);
#pragma unroll
                            for (int u = 0; u < 2; ++u)
                                dst[u] = make_uint4(pack2<T>(o[8 * u], o[8 * u + 1]), pack2<T>(o[8 * u + 2], o[8 * u + 3]),
                                                    pack2<T>(o[8 * u + 4], o[8 * u + 5]),
                                                    pack2<T>(o[8 * u + 6], o[8 * u + 7]));
                        }
                    }
                }
                tc_fence_before();
                fence_proxy_async_smem();   // the TMA refill of the load slot comes after these reads
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&tfree[ts]);
                mbar_arrive(&empty[ls]);
            }
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == C::MMA_WARP) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace mf
