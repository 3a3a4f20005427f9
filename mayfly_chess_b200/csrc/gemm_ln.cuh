// The residual products fused with the LayerNorm that follows them:
//
//   X = X + (A W^T + bias)           (f32 residual stream, in place; the out projection or the second FFN product)
//   H = LN(X) * g + b                 (16-bit, the next product's input: LN2 after the out projection, the next
//                                      layer's LN1 after the FFN)
//
// mayfly/chess/chess_net.py:162-164 (x += out_proj(..); h = norm2(x); ...; x += linear2(..); next layer's
// h = norm1(x)), which the reference runs as a cuBLASLt product with a residual epilogue and then a LayerNorm
// kernel (cudanet/cudanet.cpp:491-550, kernels_trunk.cu:135-191). A LayerNorm needs a whole row (d = 1024 = 4 x
// 256 columns), so a cluster of NCL = d / 256 CTAs computes one 128-row block: CTA rank r owns columns
// 256 r .. 256 r + 255. Each CTA
//   1. runs the residual epilogue of its 128 x 256 tile (TMA-staged, as gemm_tc_kernel's kEpiResidual) and
//      accumulates, per row, the mean and sum of squared deviations of its 256 new values (two passes over each
//      32-value chunk in registers, chunks merged with Chan's pairwise formula);
//   2. publishes those per-row partial statistics in its shared memory and arrives on every cluster CTA's
//      `stats_ready` barrier; once all NCL arrivals are in, each thread reads the NCL partials of its row through
//      distributed shared memory and merges them: mean and biased variance of the whole row, as F.layer_norm;
//   3. reads its 256 columns of the new X back from tensor memory (the epilogue wrote them over the
//      accumulator's columns in step 1), normalises them and stores H with TMA.
// The residual chunks' loads run up to three staging buffers ahead, across tiles, so the next tile's first X
// chunks arrive while this tile is being normalised.
// The MMA side is gemm_tc_kernel's (one CTA, M = 128, N = 256, tcgen05.mma.cta_group::1, TMA ring, two TMEM
// accumulators). Every wait is bounded; the final cluster barrier keeps every CTA's shared memory alive until
// the other CTAs are done reading it.
#pragma once
#include "gemm.cuh"

namespace mf {

template <int NCL> struct ResLnCfg {
    static constexpr int BM = 128, BN = 256, BK = 64;
    static constexpr int CHUNK_COLS = 32;                 // f32 staging chunk: 128 rows x 128 bytes
    static constexpr int NC = BN / CHUNK_COLS;            // 8 residual chunks per tile
    static constexpr uint32_t CHUNK_BYTES = 128 * 128;
    static constexpr int NBUF = 4;
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t STATS_BYTES = 2 * 128 * 8;   // float2 [tile parity][row]
    static constexpr int STAGES = (224 * 1024 - NBUF * (int)CHUNK_BYTES - (int)STATS_BYTES) / (int)STAGE_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * BN;
    static constexpr size_t SMEM =
        1024 + (size_t)STAGES * STAGE_BYTES + (size_t)NBUF * CHUNK_BYTES + STATS_BYTES + 256;
    static constexpr int THREADS = 64 + 128;
    static_assert(STAGES >= 3, "pipeline too shallow");
    static_assert(SMEM <= 232448, "shared memory over the per-block limit");
};

// Chan, Golub, LeVeque: merge (n_a, mean_a, M2_a) with a part of n_b values (mean_b, M2_b).
__device__ __forceinline__ void chan_merge(float& n_a, float& mean_a, float& m2_a, float n_b, float mean_b,
                                           float m2_b)
{
    const float n = n_a + n_b;
    const float delta = mean_b - mean_a;
    mean_a = mean_a + delta * (n_b / n);
    m2_a = m2_a + m2_b + delta * delta * (n_a * n_b / n);
    n_a = n;
}

__device__ __forceinline__ float2 ld_shared_cluster_f2(uint32_t addr)
{
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
    return v;
}

template <typename T, int NCL>
__global__ void __cluster_dims__(NCL, 1, 1) __launch_bounds__(ResLnCfg<NCL>::THREADS, 1)
gemm_tc_resln_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmH, int M, int K,
                     const float* __restrict__ bias, const float* __restrict__ ln_g,
                     const float* __restrict__ ln_b, float eps, uint32_t* err)
{
    using C = ResLnCfg<NCL>;
    constexpr int BN = C::BN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + C::STAGES * C::A_BYTES;
    uint8_t* sC = sB + C::STAGES * C::B_BYTES;
    float2* stats = reinterpret_cast<float2*>(sC + C::NBUF * C::CHUNK_BYTES);   // [2][128]
    uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(stats) + C::STATS_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* mma_done = tempty + 2;
    uint64_t* xfull = mma_done + 1;          // NBUF
    uint64_t* stats_ready = xfull + C::NBUF; // 2 (tile parity)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(stats_ready + 2);
    volatile uint32_t* epi_ok = tmem_slot + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = NCL > 1 ? (int)cluster_ctarank() : 0;     // this CTA's 256-column block
    const int cluster = (int)blockIdx.x / NCL, num_clusters = (int)gridDim.x / NCL;
    const int m_tiles = (M + C::BM - 1) / C::BM;
    const int my_tiles = cluster < m_tiles ? (m_tiles - 1 - cluster) / num_clusters + 1 : 0;
    const int k_iters = K / C::BK;
    const int colb = rank * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
            mbar_init(&stats_ready[b], NCL);
        }
        mbar_init(mma_done, 1);
        for (int b = 0; b < C::NBUF; ++b) mbar_init(&xfull[b], 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmH);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    if constexpr (NCL > 1) cluster_sync();   // every CTA's barriers exist before any other CTA arrives on them
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    griddep_wait();   // A, X and H belong to the earlier kernels until they complete
    if (threadIdx.x == 0) griddep_launch();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0 && k_iters > 0) {
            int stage = 0;
            uint32_t phase = 0, issued = 0, issued_par = 0;
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                const int m_blk = cluster + it * num_clusters;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, kErrSmemEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * C::BK, m_blk * C::BM);
                    tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * C::BK, colb);
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            for (int s = 0; s < C::STAGES; ++s)
                if (issued & (1u << s)) mbar_wait(&full[s], (issued_par >> s) & 1u, err, kErrTmaFull);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && k_iters > 0) {
            constexpr uint32_t idesc = Operand<T>::idesc(128, BN);
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err, kErrTmemEmpty)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&full[stage], phase, err, kErrTmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
                    for (int k = 0; k < C::BK / 16; ++k)
                        umma_f16(d_tmem, sdesc_sw128(a_addr + 32u * k), sdesc_sw128(b_addr + 32u * k), idesc,
                                 (kb | k) != 0 ? 1u : 0u);
                    umma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, err, kErrTmemFull);
        }
    } else if (k_iters > 0) {
        // ---------------------------------------------------------------- epilogue (warps 2..5)
        // Per tile, 12 uses of the 4 staging buffers ("slots", buffer = global slot % 4): slots 0..7 are the
        // 32-column chunks of X (TMA-loaded, updated, stored back), slots 8..11 the 64-column units of H (written,
        // stored). X loads are issued 3 slots ahead, across tile boundaries, as soon as a buffer's last store has
        // been read. The new X also goes back into the accumulator's tensor-memory columns, where the
        // normalisation reads it.
        constexpr int XS = C::NC, SLOTS = C::NC + C::BN / 64;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const bool leader = threadIdx.x == 64;
        const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        const int total_slots = my_tiles * SLOTS;
        uint32_t xpar = 0;        // leader: bit b = parity of the next wait on xfull[b]
        int pending = 0;          // leader: bit b = a load into buffer b is in flight and not yet waited for
        int issued = 0;           // leader: slots below this have had their load (if any) issued
        int acc = 0;
        uint32_t acc_phase = 0;
        bool ok = true;

        auto issue_loads_upto = [&](int last) {   // leader: X loads of slots issued .. last
            for (; issued <= last && issued < total_slots; ++issued) {
                const int local = issued % SLOTS;
                if (local >= XS) continue;
                const int b = issued % C::NBUF;
                const int r0 = (cluster + (issued / SLOTS) * num_clusters) * C::BM;
                mbar_arrive_expect_tx(&xfull[b], C::CHUNK_BYTES);
                tma_load_2d(sC + b * C::CHUNK_BYTES, &tmX, &xfull[b], colb + local * C::CHUNK_COLS, r0);
                pending |= 1 << b;
            }
        };
        auto wait_x = [&](int b) -> bool {        // leader
            const bool r = mbar_wait(&xfull[b], (xpar >> b) & 1u, err, kErrTmaFull);
            xpar ^= 1u << b;
            pending &= ~(1 << b);
            return r;
        };
        // the next tile's X is pulled into L2 a tile ahead, so the staged loads hit L2
        auto prefetch_tile = [&](int it) {   // leader
            if (it < my_tiles)
                for (int c = 0; c < XS; ++c)
                    tma_prefetch_l2_2d(&tmX, colb + c * C::CHUNK_COLS, (cluster + it * num_clusters) * C::BM);
        };
        if (leader) {
            prefetch_tile(0);
            issue_loads_upto(C::NBUF - 2);
        }

        for (int it = 0; it < my_tiles && ok; ++it) {
            const int row0 = (cluster + it * num_clusters) * C::BM;
            const int base = it * SLOTS;
            if (leader) prefetch_tile(it + 1);
            if (leader) *epi_ok = mbar_wait(&tfull[acc], acc_phase, err, kErrTmemFull) ? 1u : 0u;
            named_barrier(1, 128);
            if (!*epi_ok) break;
            tc_fence_after();
            const uint32_t t_acc = t_lane + static_cast<uint32_t>(acc * BN);

            // ------------------------------------------------ phase 1: X += acc + bias, row statistics
            float n_a = 0.f, mean_a = 0.f, m2_a = 0.f;
            for (int c = 0; c < XS; ++c) {
                const int slot = base + c;
                uint8_t* buf = sC + (slot % C::NBUF) * C::CHUNK_BYTES;
                const int col0 = colb + c * C::CHUNK_COLS;
                float v[32];
                {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(c * C::CHUNK_COLS), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                }
                add_bias32<32>(v, 0, bias, col0, colb + BN);
                if (leader) *epi_ok = wait_x(slot % C::NBUF) ? 1u : 0u;
                named_barrier(1, 128);
                if (!*epi_ok) {
                    ok = false;
                    break;
                }
                float s = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float4* p = reinterpret_cast<float4*>(buf + swz<128>(row, j));
                    float4 x = *p;
                    x.x += v[4 * j + 0];
                    x.y += v[4 * j + 1];
                    x.z += v[4 * j + 2];
                    x.w += v[4 * j + 3];
                    *p = x;
                    v[4 * j + 0] = x.x;
                    v[4 * j + 1] = x.y;
                    v[4 * j + 2] = x.z;
                    v[4 * j + 3] = x.w;
                    s += (x.x + x.y) + (x.z + x.w);
                }
                {
                    uint32_t r[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
                    tmem_st_32x32b_x32(t_acc + static_cast<uint32_t>(c * C::CHUNK_COLS), r);
                }
                const float mean_b = s * (1.0f / 32.0f);
                float m2_b = 0.f;
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float dv = v[i] - mean_b;
                    m2_b = fmaf(dv, dv, m2_b);
                }
                if (c == 0) {
                    n_a = 32.f;
                    mean_a = mean_b;
                    m2_a = m2_b;
                } else {
                    chan_merge(n_a, mean_a, m2_a, 32.f, mean_b, m2_b);
                }
                fence_proxy_async_smem();
                named_barrier(1, 128);
                if (leader) {
                    tma_store_2d(&tmX, buf, col0, row0);
                    bulk_commit();
                    bulk_wait_read<1>();          // the previous slot's buffer is free
                    issue_loads_upto(slot + C::NBUF - 1);
                }
            }
            if (!ok) break;
            tmem_st_wait();   // the new X is in tensor memory before it is read back

            // ------------------------------------------------ phase 2: the whole row's statistics
            const int par = it & 1;
            stats[par * 128 + row] = make_float2(mean_a, m2_a);
            fence_cluster();   // the write is visible cluster-wide before the leader's arrivals announce it
            named_barrier(1, 128);
            if (leader) {
                if constexpr (NCL > 1) {
                    const uint32_t sr = smem_u32(&stats_ready[par]);
                    for (int c = 0; c < NCL; ++c) mbar_arrive_cluster(mapa_shared(sr, (uint32_t)c));
                } else {
                    mbar_arrive(&stats_ready[par]);
                }
                *epi_ok = mbar_wait(&stats_ready[par], (it >> 1) & 1u, err, kErrCluster) ? 1u : 0u;
            }
            named_barrier(1, 128);
            if (!*epi_ok) {
                ok = false;
                break;
            }
            fence_cluster();   // the other CTAs' statistics, announced to the leader, are visible to this thread
            float n_t = 0.f, mean_t = 0.f, m2_t = 0.f;
            const uint32_t my_stat = smem_u32(&stats[par * 128 + row]);
#pragma unroll
            for (int c = 0; c < NCL; ++c) {
                const float2 p = NCL > 1 ? ld_shared_cluster_f2(mapa_shared(my_stat, (uint32_t)c))
                                         : stats[par * 128 + row];
                if (c == 0) {
                    n_t = (float)BN;
                    mean_t = p.x;
                    m2_t = p.y;
                } else {
                    chan_merge(n_t, mean_t, m2_t, (float)BN, p.x, p.y);
                }
            }
            const float mean = mean_t;
            const float rstd = rsqrtf(m2_t / n_t + eps);

            // ------------------------------------------------ phase 3: H = LN(X), 64 columns per slot
            for (int u = 0; u < BN / 64; ++u) {
                const int slot = base + XS + u;
                uint8_t* buf = sC + (slot % C::NBUF) * C::CHUNK_BYTES;
                const int c0 = colb + u * 64;
                float x[64];
                {
                    uint32_t r[32];
                    tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(u * 64), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) x[i] = __uint_as_float(r[i]);
                    tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(u * 64 + 32), r);
                    tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 32; ++i) x[32 + i] = __uint_as_float(r[i]);
                }
                if (u == BN / 64 - 1) {
                    // this warp is done with the accumulator: hand it back to the MMA thread
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[acc]);
                }
                const float4* g4 = reinterpret_cast<const float4*>(ln_g + c0);
                const float4* bb4 = reinterpret_cast<const float4*>(ln_b + c0);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float4 g = __ldg(g4 + j), bb = __ldg(bb4 + j);
                    x[4 * j + 0] = (x[4 * j + 0] - mean) * rstd * g.x + bb.x;
                    x[4 * j + 1] = (x[4 * j + 1] - mean) * rstd * g.y + bb.y;
                    x[4 * j + 2] = (x[4 * j + 2] - mean) * rstd * g.z + bb.z;
                    x[4 * j + 3] = (x[4 * j + 3] - mean) * rstd * g.w + bb.w;
                }
                if (leader) bulk_wait_read<C::NBUF - 1>();   // this slot's buffer was read by its last store
                named_barrier(1, 128);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    uint4 q;
                    q.x = pack2<T>(x[8 * j + 0], x[8 * j + 1]);
                    q.y = pack2<T>(x[8 * j + 2], x[8 * j + 3]);
                    q.z = pack2<T>(x[8 * j + 4], x[8 * j + 5]);
                    q.w = pack2<T>(x[8 * j + 6], x[8 * j + 7]);
                    *reinterpret_cast<uint4*>(buf + swz<128>(row, j)) = q;
                }
                fence_proxy_async_smem();
                named_barrier(1, 128);
                if (leader) {
                    tma_store_2d(&tmH, buf, c0, row0);
                    bulk_commit();
                    bulk_wait_read<1>();
                    issue_loads_upto(slot + C::NBUF - 1);   // the next tile's first X chunks
                }
            }
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
        if (leader) {
            bulk_wait_all();
            // loads issued but never waited for (only after a failure) land before the CTA leaves
            for (int b = 0; b < C::NBUF; ++b)
                if (pending & (1 << b)) mbar_wait(&xfull[b], (xpar >> b) & 1u, err, kErrTmaFull);
        }
    }

    __syncwarp();
    tc_fence_before();
    if constexpr (NCL > 1) cluster_sync();   // no CTA leaves while another may still read its statistics
    else __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace mf
