// The trunk's and the heads' matrix products on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[M, N] = A[M, K] * W[N, K]^T  (+ epilogue), A and W 16-bit (f16 or bf16), K-major, f32 accumulation.
//
// These are the five products of mayfly/chess/cudanet/cudanet_spec.h:94-101 (qkv, out, ff1, ff2, heads), which
// the reference runs through cuBLASLt (cudanet/gemm.cpp:209-231) or mma.sync (cudanet/kernels_gemm.cu:99-302).
// Epilogues (kEpi*), each the arithmetic of the reference's product plus what follows it:
//   kEpiBias      C (16-bit) = acc + bias                            qkv (gemm.h F16_BIAS)
//   kEpiBiasGelu  C (16-bit) = gelu_erf(acc + bias)                  ff1 + the GELU pass (kernels_trunk.cu:528-549)
//   kEpiResidual  X (f32)   = X + (acc + bias), in place             out and ff2 (gemm.h F32_BIAS_RESIDUAL)
//   kEpiF32       C (f32)   = acc + bias                             heads
//
// Design (one CTA per SM, persistent over output tiles of 128 x BN):
//   warp 0      one thread issues TMA tile loads (128-byte swizzle) of A and W into a STAGES-deep ring
//   warp 1      allocates tensor memory (2 accumulators of BN f32 columns); one thread issues tcgen05.mma
//               (M=128, N=BN, K=16 per instruction) and tcgen05.commit to release ring stages / accumulators
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31, one row per
//               thread), bias / GELU / residual, store; then hand the accumulator back to the MMA warp
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1. Tiles run M-block-major
// (all N blocks of an M block back to back), so an A block is read from HBM once and the weights stay in L2.
// Out-of-range rows (M tail) and columns (N tail) are zero-filled by TMA and skipped by the epilogue.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"

namespace mf {

enum Epi : int { kEpiBias = 0, kEpiBiasGelu = 1, kEpiResidual = 2, kEpiF32 = 3 };

template <typename T> struct Fmt;
template <> struct Fmt<__half> { static constexpr uint32_t v = 0; };
template <> struct Fmt<__nv_bfloat16> { static constexpr uint32_t v = 1; };

template <int BN> struct GemmCfg {
    static constexpr int BM = 128;
    static constexpr int BK = 64;                       // 64 x 16-bit = one 128-byte swizzle row
    static constexpr int STAGES = BN == 256 ? 4 : (BN == 128 ? 6 : 8);
    static constexpr uint32_t A_BYTES = BM * BK * 2;
    static constexpr uint32_t B_BYTES = BN * BK * 2;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr size_t SMEM = 1024 + STAGES * (size_t)STAGE_BYTES + 256;
    static constexpr int THREADS = 192;
};

__device__ __forceinline__ float gelu_erf(float x)
{
    // F.gelu(approximate="none"): x * 0.5 * (1 + erf(x / sqrt(2)))
    return x * 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b)
{
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// The epilogue of 32 consecutive columns col0..col0+31 of one row, r[] holding the raw f32 accumulators.
// out and bias are 16-byte aligned (checked by the host); vector accesses are used only when every row of
// out is 16-byte aligned too (ldc a multiple of 16 bytes), scalar ones otherwise and on the N tail.
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_chunk(const uint32_t (&r)[32], int row, int col0, int N, int ldc,
                                               const float* __restrict__ bias, void* __restrict__ out)
{
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
    const bool full = col0 + 32 <= N;
    if (full) {
        const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = __ldg(b4 + i);
            v[4 * i + 0] += b.x;
            v[4 * i + 1] += b.y;
            v[4 * i + 2] += b.z;
            v[4 * i + 3] += b.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (col0 + i < N) v[i] += __ldg(bias + col0 + i);
    }
    if constexpr (EPI == kEpiBiasGelu) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = gelu_erf(v[i]);
    }
    if constexpr (EPI == kEpiBias || EPI == kEpiBiasGelu) {
        T* o = reinterpret_cast<T*>(out) + (size_t)row * ldc + col0;
        if (full && (ldc % 8) == 0) {   // 16-byte stores need 16-byte aligned rows
            uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                uint4 q;
                q.x = pack2<T>(v[8 * i + 0], v[8 * i + 1]);
                q.y = pack2<T>(v[8 * i + 2], v[8 * i + 3]);
                q.z = pack2<T>(v[8 * i + 4], v[8 * i + 5]);
                q.w = pack2<T>(v[8 * i + 6], v[8 * i + 7]);
                o4[i] = q;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < N) o[i] = static_cast<T>(v[i]);
        }
    } else if constexpr (EPI == kEpiResidual) {
        float* x = reinterpret_cast<float*>(out) + (size_t)row * ldc + col0;
        if (full && (ldc % 4) == 0) {
            float4* x4 = reinterpret_cast<float4*>(x);
            float4 old[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) old[i] = x4[i];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                old[i].x += v[4 * i + 0];
                old[i].y += v[4 * i + 1];
                old[i].z += v[4 * i + 2];
                old[i].w += v[4 * i + 3];
                x4[i] = old[i];
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < N) x[i] += v[i];
        }
    } else {  // kEpiF32
        float* o = reinterpret_cast<float*>(out) + (size_t)row * ldc + col0;
        if (full && (ldc % 4) == 0) {
            float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
            for (int i = 0; i < 8; ++i) o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if (col0 + i < N) o[i] = v[i];
        }
    }
}

template <typename T, int BN, int EPI>
__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N,
               int K, const float* __restrict__ bias, void* __restrict__ out, int ldc, uint32_t* err)
{
    using C = GemmCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_BYTES);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* mma_done = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (M + C::BM - 1) / C::BM;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_iters = K / C::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(mma_done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0 && k_iters > 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;       // bit s: stage s was loaded at least once
            uint32_t issued_par = 0;   // bit s: parity of the last load into stage s
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int m_blk = tile / n_tiles, n_blk = tile % n_tiles;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1u, err, kErrSmemEmpty)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(sA + stage * C::A_BYTES, &tmA, &full[stage], kb * C::BK, m_blk * C::BM);
                    tma_load_2d(sB + stage * C::B_BYTES, &tmB, &full[stage], kb * C::BK, n_blk * BN);
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // every copy this thread started has landed before the CTA can leave (immediate when the MMA warp
            // consumed them all; bounded when something upstream failed)
            for (int s = 0; s < C::STAGES; ++s)
                if (issued & (1u << s)) mbar_wait(&full[s], (issued_par >> s) & 1u, err, kErrTmaFull);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && k_iters > 0) {
            constexpr uint32_t idesc = idesc_f16(Fmt<T>::v, 128, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
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
            // every MMA this thread issued has completed before tensor memory is freed
            umma_commit(mma_done);
            mbar_wait(mma_done, 0, err, kErrTmemFull);
        }
    } else {
        // ---------------------------------------------------------------- epilogue (warps 2..5)
        const int quarter = warp & 3;
        const int row_in_tile = quarter * 32 + lane;
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles && k_iters > 0; tile += gridDim.x) {
            const int m_blk = tile / n_tiles, n_blk = tile % n_tiles;
            if (!mbar_wait(&tfull[acc], acc_phase, err, kErrTmemFull)) break;
            tc_fence_after();
            const int row = m_blk * C::BM + row_in_tile;
            const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                   static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                const int col0 = n_blk * BN + c;
                if (col0 >= N) break;   // whole warp agrees: col0 does not depend on the lane
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_row + static_cast<uint32_t>(c), r);
                tmem_ld_wait();
                if (row < M) epilogue_chunk<T, EPI>(r, row, col0, N, ldc, bias, out);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[acc]);
            acc ^= 1;
            if (acc == 0) acc_phase ^= 1u;
        }
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

}  // namespace mf
