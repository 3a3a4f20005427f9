// The trunk's and the heads' matrix products on the 5th-generation tensor cores (tcgen05, sm_100a).
//
//   C[M, N] = A[M, K] * W[N, K]^T  (+ epilogue), A and W 16-bit (f16 or bf16, kind::f16) or e4m3 (the FP8
//   path, kind::f8f6f4, the accumulator scaled per column in the epilogue), K-major, f32 accumulation.
//
// These are the five products of mayfly/chess/cudanet/cudanet_spec.h:94-101 (qkv, out, ff1, ff2, heads), which
// the reference runs through cuBLASLt (cudanet/gemm.cpp:209-231) or mma.sync (cudanet/kernels_gemm.cu:99-302).
// Epilogues (kEpi*), each the arithmetic of the reference's product plus what follows it:
//   kEpiBias      C (16-bit) = acc + bias                            qkv (gemm.h F16_BIAS)
//   kEpiBiasGelu  C (16-bit) = gelu(acc + bias), exact-erf GELU      ff1 + the GELU pass (kernels_trunk.cu:528-549)
//   kEpiResidual  X (f32)   = X + (acc + bias), in place             out and ff2 (gemm.h F32_BIAS_RESIDUAL)
//   kEpiF32       C (f32)   = acc + bias                             heads
// and for the FP8 path (no reference counterpart; acc scaled per column first):
//   kEpiGeluE4m3  C (e4m3)  = e4m3(gelu(acc + bias) / scale)         ff1, writing ff2's input
//   kEpiResidual16 X (bf16) = bf16(X + bf16(acc + bias)), in place   out and ff2 on a bf16 residual stream
//
// Two kernels, both persistent over output tiles with one CTA per SM:
//   gemm_tc_kernel       one CTA per 128 x BN tile (BN 64, 128 or 256): tcgen05.mma.cta_group::1, M=128.
//   gemm_tc_pair_kernel  a cluster of 2 CTAs per 256 x 256 tile: tcgen05.mma.cta_group::2, M=256, issued by the
//                        leader CTA. Each CTA loads its 128 rows of A and 128 of the 256 rows of W, so a CTA moves
//                        a third less operand data per FLOP than with 128 x 256 alone, and a 32 KB stage buys a
//                        deeper ring. Each CTA holds and drains its own 128 rows of the accumulator.
// Warp roles (both kernels):
//   warp 0      one thread issues TMA tile loads (128-byte swizzle) of A and W into a STAGES-deep ring
//   warp 1      allocates tensor memory (2 accumulators of BN f32 columns); one thread (the leader CTA's, for a
//               pair) issues the MMAs (K=16 each) and tcgen05.commit to release ring stages / accumulators
//   warps 2..   epilogue, 1, 2 or 4 groups of 4 warps (GemmCfg::EG), one output row per thread per group:
//               tcgen05.ld of the accumulator (warp w reads TMEM lanes 32*(w%4)..+31; the groups split a tile's
//               column chunks), bias / GELU / residual, then the row goes into a 128-row staging chunk in shared
//               memory (128-byte rows with the 128-byte swizzle, or 64-byte rows with the 64-byte swizzle for the
//               4-group epilogues) and one thread stores the chunk with a TMA tensor store (coalesced,
//               asynchronous); for the FP8 bias epilogue, lane 0 of each warp stores the warp's own 32 rows. The residuals stage v = acc + bias alone (f32, or rounded to bf16 for the bf16
//               stream) and add it into X with a TMA reduction (cp.reduce.async.bulk.tensor .add, done at L2, in
//               X's type: f32, or bf16 rounded to nearest): X is never read into the SM, and the shared-memory
//               traffic per tile halves against a read-modify-write through the staging chunk.
// The two accumulators let the epilogue of tile i overlap the MMAs of tile i+1. Tiles run M-block-major (all
// N blocks of an M block back to back), so an A block is read from HBM once and the weights stay in L2.
// Out-of-range rows and columns (M and N tails) are zero-filled by TMA loads and clipped by TMA stores.
// No load uses multicast.
//
// Every wait is bounded (ptx.cuh). Epilogue decisions are made by one thread and broadcast through shared
// memory at a named barrier, so the epilogue warps always take the same path and never strand one another at a
// barrier. Before a CTA leaves, its own TMA loads have landed and the MMAs that write its tensor memory have
// completed.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "ptx.cuh"

// Epilogue groups and staging buffers per group of the f32 residual (added into X by TMA reductions).
#ifndef MF_REDUCE_EG
#define MF_REDUCE_EG 2
#endif
#ifndef MF_REDUCE_NBUF
#define MF_REDUCE_NBUF 1
#endif
// The FP8 bias epilogue (qkv): 64-byte staging rows in four groups (1) or 128-byte rows (0), and its staging
// buffers per group.
#ifndef MF_F8_BIAS_NARROW
#define MF_F8_BIAS_NARROW 1
#endif
#ifndef MF_F8_BIAS_NBUF
#define MF_F8_BIAS_NBUF 1
#endif
#ifndef MF_EPI_BATCH
#define MF_EPI_BATCH 1
#endif

namespace mf {

enum Epi : int { kEpiBias = 0, kEpiBiasGelu = 1, kEpiResidual = 2, kEpiF32 = 3, kEpiGeluE4m3 = 4, kEpiResidual16 = 5 };

// Rows of one epilogue TMA store (or reduce-add), the height of the output tensor map's box: 128 (one thread of
// a group stores the group's whole staging chunk, after a barrier of the group's 4 warps), or 32 for the FP8
// bias epilogue (each warp stores the 32 rows it wrote, no barrier between the warps per chunk: 2-4% faster on
// the FP8 qkv product, slower on the 16-bit products and the residuals' reduce-adds, measured).
__host__ __device__ constexpr int store_rows(int epi, bool f8) { return epi == kEpiBias && f8 ? 32 : 128; }

// Operand types: 16-bit (kind::f16) or e4m3 (kind::f8f6f4). A stage row is always 128 bytes (the swizzle atom),
// so an FP8 stage holds 128 elements of K and each MMA instruction 32 (16 for 16-bit); the byte sizes, smem
// descriptors and the 32-byte step per instruction are the same.
template <typename T> struct Operand;
template <> struct Operand<__half> {
    static constexpr bool F8 = false;
    __host__ __device__ static constexpr uint32_t idesc(uint32_t M, uint32_t N) { return idesc_f16(0, M, N); }
};
template <> struct Operand<__nv_bfloat16> {
    static constexpr bool F8 = false;
    __host__ __device__ static constexpr uint32_t idesc(uint32_t M, uint32_t N) { return idesc_f16(1, M, N); }
};
template <> struct Operand<__nv_fp8_e4m3> {
    static constexpr bool F8 = true;
    __host__ __device__ static constexpr uint32_t idesc(uint32_t M, uint32_t N) { return idesc_e4m3(M, N); }
};

template <typename TI>
__device__ __forceinline__ void umma_issue(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    if constexpr (Operand<TI>::F8) umma_f8(d, a, b, idesc, acc);
    else umma_f16(d, a, b, idesc, acc);
}

template <typename TI>
__device__ __forceinline__ void umma_issue_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc)
{
    if constexpr (Operand<TI>::F8) umma_f8_pair(d, a, b, idesc, acc);
    else umma_f16_pair(d, a, b, idesc, acc);
}

// The epilogue's per-product constants: FP8 products scale the accumulator column by column
// (colscale[c] = input scale x weight scale of output channel c) and the e4m3 output divides by its own scale.
struct EpiArgs {
    const float* bias;
    const float* colscale;   // nullptr: no scaling (16-bit operands)
    float out_scale_inv;     // kEpiGeluE4m3 only
    int rev;                 // 1: the M blocks in descending order (the output is the same)
};

// PAIR: the CTA-pair kernel, where a CTA loads BN/2 rows of W per stage and a pair covers 256 rows of M.
// F8: e4m3 operands (128 elements of K per stage instead of 64; the same bytes).
template <int BN, int EPI, bool PAIR = false, bool F8 = false> struct GemmCfg {
    static constexpr int BM = 128;                      // rows of A and of the output per CTA
    static constexpr int BK = F8 ? 128 : 64;            // elements of K per stage: one 128-byte swizzle row
    static constexpr int KSTEPS = 4;                    // MMA instructions per stage (K = 16 or 32 each, 32 bytes)
    static constexpr int B_ROWS = PAIR ? BN / 2 : BN;   // rows of W per CTA per stage
    // the residuals are added into X by a TMA reduction at L2 (f32 adds for the f32 stream, bf16 adds of the
    // bf16-rounded v for the bf16 stream), so X is neither read into the SM nor staged
    static constexpr bool REDUCE = EPI == kEpiResidual || EPI == kEpiResidual16;
    static constexpr bool IS_F8 = F8;
    static constexpr bool HEAVY = EPI == kEpiBiasGelu || EPI == kEpiGeluE4m3;   // GELU's erf per element
    static constexpr int OUT_BYTES = (EPI == kEpiResidual || EPI == kEpiF32) ? 4 : (EPI == kEpiGeluE4m3 ? 1 : 2);
    // one staging chunk: 128 rows x ROW_BYTES (64-byte rows for the GELU epilogues, whose four groups each take
    // a narrow chunk at a time, and for the FP8 bias and bf16-residual epilogues, which have half the mainloop
    // time of a 16-bit tile to hide in: four groups on narrower chunks measured 2.7% faster on the FP8 qkv
    // product, no faster on the 16-bit one; 128-byte rows otherwise)
    static constexpr bool F8_BIAS = EPI == kEpiBias && F8;
    static constexpr bool NARROW = (F8_BIAS && MF_F8_BIAS_NARROW) || EPI == kEpiResidual16;
    static constexpr int ROW_BYTES = (HEAVY || NARROW) ? 64 : 128;
    static constexpr int STORE_ROWS = store_rows(EPI, F8);   // 32: per-warp stores
    static constexpr int CHUNK_COLS = ROW_BYTES / OUT_BYTES;
    static constexpr int NC = BN / CHUNK_COLS;           // staging chunks per tile
    static constexpr uint32_t CHUNK_BYTES = 128 * ROW_BYTES;
    // Epilogue groups: 4 warps each, one per TMEM lane quarter, splitting a tile's chunks round-robin. Four
    // groups where the per-element work is heavy (GELU's erf: more warps to hide its latency and share its
    // issue slots) and for the narrow chunks, two where the chunks are many. The f32 residual stages only
    // acc + bias for its TMA reductions: two groups of one buffer (measured best of 1 x 2, 2 x 1, 2 x 2 and
    // 4 x 1).
    static constexpr int EG = EPI == kEpiResidual ? ((NC % MF_REDUCE_EG == 0) ? MF_REDUCE_EG : 1)
                              : ((HEAVY || NARROW) && NC % 4 == 0) ? 4 : (NC % 2 == 0 ? 2 : 1);
    // the FP8 bias epilogue with several chunks a group (MF_EPI_BATCH): one staging buffer per chunk, so a group
    // writes all its chunks of a tile before one proxy fence and one barrier, then stores them
    static constexpr bool BATCH = MF_EPI_BATCH && F8_BIAS && NC / EG > 1;
    static constexpr int NBUF = BATCH ? NC / EG
                                : EPI == kEpiResidual ? MF_REDUCE_NBUF
                                : F8_BIAS ? MF_F8_BIAS_NBUF : (EG >= 2 ? 1 : 2);   // staging buffers a group
    static constexpr uint32_t A_BYTES = BM * 128;
    static constexpr uint32_t B_BYTES = B_ROWS * 128;
    static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES_FIT = (224 * 1024 - EG * NBUF * (int)CHUNK_BYTES) / (int)STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
    static constexpr size_t SMEM =
        1024 + (size_t)STAGES * STAGE_BYTES + (size_t)EG * NBUF * CHUNK_BYTES + 256;
    static constexpr int THREADS = 64 + 128 * EG;
    static_assert(STAGES >= 3, "pipeline too shallow");
    static_assert(SMEM <= 232448, "shared memory over the per-block limit");
    static_assert(BN % CHUNK_COLS == 0 && NC >= 1, "tile width must hold whole staging chunks");
    static_assert(!PAIR || BN == 256, "the pair kernel covers 256 columns");
};

// ------------------------------------------------------------------------------------------------ GELU
// Packed f32 pairs: sm_100's f32x2 arithmetic does two IEEE round-to-nearest f32 operations per instruction
// (the GELU epilogues are issue-bound, so halving their FMA-class instructions matters).
__device__ __forceinline__ uint64_t pk2(float a, float b)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ float2 upk2(uint64_t r)
{
    float2 f;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(f.x), "=f"(f.y) : "l"(r));
    return f;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b)
{
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ float rcp_approx(float x)
{
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float ex2_approx_f(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// s * gelu(x) for the exact-erf GELU (F.gelu(approximate="none") = x * Phi(x), Phi the standard normal CDF).
// With a = |x| and q(a) = Phi(-a) = erfc(a / sqrt(2)) / 2, x * Phi(x) = relu(x) - a q(a) for either sign of x
// (no cancellation: the negative side is -a q directly). log2 q(a) is smooth on [0, 10], so
// q(a) = 2^P(u), u = a / 5 - 1, with P the degree-8 polynomial csrc/gelu_poly.py fits to log2 Phi(-a) (least
// squares on Chebyshev nodes, relative error of q below 2.5e-5 over [0, 10] in f32 arithmetic); a is clamped to
// 10, where q = 7.6e-24 (GELU is then x, or below 1e-21 in magnitude). One 2^x on the special-function unit per
// value and no division; the polynomial runs two lanes per instruction (f32x2). The output scale s (e4m3
// outputs) rides in the constant term: s q = 2^(P + log2 s), and s relu(x) = relu(s x) for s > 0.
struct GeluK {
    uint64_t c0, c1, c2, c3, c4, c5, c6, c7, c8, mu, m1, s;
    __device__ __forceinline__ explicit GeluK(float scale)
    {
        const float l2s = scale == 1.0f ? 0.0f : log2f(scale);
        c0 = pk2(-2.173420143e+01f + l2s, -2.173420143e+01f + l2s);
        c1 = pk2(-3.741247559e+01f, -3.741247559e+01f);
        c2 = pk2(-1.744393730e+01f, -1.744393730e+01f);
        c3 = pk2(-3.288443387e-01f, -3.288443387e-01f);
        c4 = pk2(1.906916946e-01f, 1.906916946e-01f);
        c5 = pk2(-9.975451976e-02f, -9.975451976e-02f);
        c6 = pk2(6.548856944e-02f, 6.548856944e-02f);
        c7 = pk2(-5.716544390e-02f, -5.716544390e-02f);
        c8 = pk2(2.371014841e-02f, 2.371014841e-02f);
        mu = pk2(-0.2f, -0.2f);      // u = (-a) * (-1/5) - 1
        m1 = pk2(-1.0f, -1.0f);
        s = pk2(scale, scale);
    }
};

// s * gelu of both lanes of x2 (SCALED: s != 1)
template <bool SCALED = false>
__device__ __forceinline__ float2 gelu_pair(uint64_t x2, const GeluK& K)
{
    const float2 x = upk2(x2);
    const uint64_t na = pk2(fmaxf(-fabsf(x.x), -10.0f), fmaxf(-fabsf(x.y), -10.0f));   // -a, a clamped to 10
    const uint64_t u = fma2(na, K.mu, K.m1);
    uint64_t p = fma2(u, K.c8, K.c7);
    p = fma2(u, p, K.c6);
    p = fma2(u, p, K.c5);
    p = fma2(u, p, K.c4);
    p = fma2(u, p, K.c3);
    p = fma2(u, p, K.c2);
    p = fma2(u, p, K.c1);
    p = fma2(u, p, K.c0);                                                 // log2(s q)
    const float2 lp = upk2(p);
    const uint64_t sq = pk2(ex2_approx_f(lp.x), ex2_approx_f(lp.y));      // s q
    float2 xs = x;
    if constexpr (SCALED) xs = upk2(mul2(x2, K.s));
    return upk2(fma2(na, sq, pk2(fmaxf(xs.x, 0.f), fmaxf(xs.y, 0.f))));  // s relu(x) - s a q
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

// v[off + i] += bias[col0 + i], i < 32; vector loads when the whole run is inside N (bias is 16-byte aligned)
template <int NV>
__device__ __forceinline__ void add_bias32(float (&v)[NV], int off, const float* __restrict__ bias, int col0, int N)
{
    if (col0 + 32 <= N) {
        const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 b = __ldg(b4 + i);
            v[off + 4 * i + 0] += b.x;
            v[off + 4 * i + 1] += b.y;
            v[off + 4 * i + 2] += b.z;
            v[off + 4 * i + 3] += b.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (col0 + i < N) v[off + i] += __ldg(bias + col0 + i);
    }
}

// v[off + i] = v[off + i] * colscale[col0 + i] + bias[col0 + i], i < 32 (the FP8 products)
template <int NV>
__device__ __forceinline__ void scale_bias32(float (&v)[NV], int off, const float* __restrict__ colscale,
                                             const float* __restrict__ bias, int col0, int N)
{
    if (col0 + 32 <= N) {
        const float4* s4 = reinterpret_cast<const float4*>(colscale + col0);
        const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float4 sc = __ldg(s4 + i), b = __ldg(b4 + i);
            const float2 lo = upk2(fma2(pk2(v[off + 4 * i + 0], v[off + 4 * i + 1]), pk2(sc.x, sc.y), pk2(b.x, b.y)));
            const float2 hi = upk2(fma2(pk2(v[off + 4 * i + 2], v[off + 4 * i + 3]), pk2(sc.z, sc.w), pk2(b.z, b.w)));
            v[off + 4 * i + 0] = lo.x;
            v[off + 4 * i + 1] = lo.y;
            v[off + 4 * i + 2] = hi.x;
            v[off + 4 * i + 3] = hi.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (col0 + i < N) v[off + i] = fmaf(v[off + i], __ldg(colscale + col0 + i), __ldg(bias + col0 + i));
    }
}

// four floats to four e4m3 bytes (round to nearest even, saturating to +-448), first value in the lowest byte
__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d)
{
    const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
    const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
    return lo | (hi << 16);
}

// byte offset of 16-byte unit j of row r in a swizzled staging chunk of ROW_BYTES-byte rows, what a TMA tensor
// map with CU_TENSOR_MAP_SWIZZLE_128B (128-byte rows: unit ^= row % 8) or _64B (64-byte rows: unit ^= (row / 2)
// % 4) reads and writes; the chunk base is 1024-byte aligned
template <int ROW_BYTES> __device__ __forceinline__ uint32_t swz(int r, int j)
{
    if constexpr (ROW_BYTES == 128) return (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4));
    else return (uint32_t)(r * 64 + ((j ^ ((r >> 1) & 3)) << 4));
}

__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// The shared-memory carve-up common to both kernels.
template <typename C> struct SmemLayout {
    uint8_t *sA, *sB, *sC;
    uint64_t *full, *empty, *tfull, *tempty, *mma_done;
    uint32_t* tmem_slot;
    volatile uint32_t* epi_ok;   // per epilogue group: the leader's broadcast flag

    __device__ __forceinline__ explicit SmemLayout(uint8_t* smem_raw)
    {
        uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
        sA = smem;
        sB = smem + C::STAGES * C::A_BYTES;
        sC = sB + C::STAGES * C::B_BYTES;                                // EG x NBUF staging chunks
        full = reinterpret_cast<uint64_t*>(sC + C::EG * C::NBUF * C::CHUNK_BYTES);
        empty = full + C::STAGES;
        tfull = empty + C::STAGES;
        tempty = tfull + 2;
        mma_done = tempty + 2;
        tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
        epi_ok = tmem_slot + 1;
    }
};

// The epilogue warps' loop over this CTA's tiles (warps 2 .. 2 + 4*EG - 1). Tile `it` of this CTA has its
// output origin at (origin_row(it), origin_col(it)); when a warp has read its last accumulator columns of a
// tile it calls release(acc) on lane 0 (an arrive on the barrier the MMA thread waits on).
// T is the 16-bit output type (kEpiBias / kEpiBiasGelu); the FP8 products (C::F8) scale each column first.
template <typename T, int EPI, typename C, typename RowFn, typename ColFn, typename ReleaseFn>
__device__ __forceinline__ void epilogue_loop(const SmemLayout<C>& L, const CUtensorMap* tmC, uint32_t tmem_base,
                                              int my_tiles, RowFn origin_row, ColFn origin_col, ReleaseFn release,
                                              const EpiArgs& ep, int M, int N, uint32_t* err)
{
    const float* __restrict__ bias = ep.bias;
    const float* __restrict__ colscale = ep.colscale;
    griddep_wait();   // the output (and residual) buffers are the earlier kernels' until they complete
    constexpr int BN = C::NC * C::CHUNK_COLS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = (warp - 2) >> 2;                      // epilogue group: chunks grp, grp + EG, ...
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;                  // row of the tile this thread owns
    const bool leader = threadIdx.x == 64 + 128 * grp;    // issues the group's TMA traffic
    const uint32_t bar_id = 1 + grp;
    constexpr int CPG = C::NC / C::EG;                    // chunks per tile for one group
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    uint8_t* gbuf = L.sC + grp * C::NBUF * C::CHUNK_BYTES;

    // the bias slice of the next tile is pulled into L1 a tile ahead (8 x 128-byte lines for 256 columns), so
    // the epilogue's bias reads do not wait on L2 (and the column scales, for FP8 products)
    const int gtid = (int)threadIdx.x - 64 - 128 * grp;
    auto prefetch_bias = [&](int it) {
        if (it < my_tiles && gtid < BN / 32) {
            const int c = origin_col(it) + 32 * gtid;
            if (c < N) {
                asm volatile("prefetch.global.L1 [%0];" ::"l"(bias + c));
                if constexpr (C::IS_F8) asm volatile("prefetch.global.L1 [%0];" ::"l"(colscale + c));
            }
        }
    };
    prefetch_bias(0);

    int acc = 0;
    uint32_t acc_phase = 0;
    int g = 0;        // this group's chunks done
    for (int it = 0; it < my_tiles; ++it) {
        const int row0 = origin_row(it), colb = origin_col(it);
        prefetch_bias(it + 1);
        if (leader) L.epi_ok[grp] = mbar_wait(&L.tfull[acc], acc_phase, err, kErrTmemFull) ? 1u : 0u;
        named_barrier(bar_id, 128);
        if (!L.epi_ok[grp]) break;
        tc_fence_after();
        const uint32_t t_acc = t_lane + static_cast<uint32_t>(acc * BN);
        for (int ci = 0; ci < CPG; ++ci, ++g) {
            const int c = grp + ci * C::EG;
            const int b = g % C::NBUF;
            uint8_t* buf = gbuf + b * C::CHUNK_BYTES;
            const int col0 = colb + c * C::CHUNK_COLS;
            // this chunk's row in registers, 32 accumulator columns at a time: f32 values (f32 outputs, 32 columns
            // a chunk) or the row's output bytes already packed (16-bit and e4m3 outputs)
            constexpr int LOADS = C::CHUNK_COLS / 32;
            constexpr int QW = C::ROW_BYTES / 4;
            float v[32];
            uint32_t q[QW];
#pragma unroll
            for (int p = 0; p < LOADS; ++p) {
                uint32_t r[32];
                tmem_ld_32x32b_x32(t_acc + static_cast<uint32_t>(c * C::CHUNK_COLS + 32 * p), r);
                tmem_ld_wait();
                if (ci == CPG - 1 && p == LOADS - 1) {
                    // this warp is done with the accumulator: hand it back to the MMA thread
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) release(acc);
                }
                constexpr int off = 0;
#pragma unroll
                for (int i = 0; i < 32; ++i) v[off + i] = __uint_as_float(r[i]);
                if constexpr (C::IS_F8) scale_bias32(v, off, colscale, bias, col0 + 32 * p, N);
                else add_bias32(v, off, bias, col0 + 32 * p, N);
                if constexpr (EPI == kEpiBiasGelu) {
                    const GeluK K(1.0f);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float2 g = gelu_pair(pk2(v[2 * i], v[2 * i + 1]), K);
                        q[16 * p + i] = pack2<T>(g.x, g.y);
                    }
                } else if constexpr (EPI == kEpiGeluE4m3) {
                    const GeluK K(ep.out_scale_inv);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float2 g0 = gelu_pair<true>(pk2(v[4 * i], v[4 * i + 1]), K);
                        const float2 g1 = gelu_pair<true>(pk2(v[4 * i + 2], v[4 * i + 3]), K);
                        q[8 * p + i] = pack_e4m3x4(g0.x, g0.y, g1.x, g1.y);
                    }
                } else if constexpr (EPI == kEpiBias) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) q[16 * p + i] = pack2<T>(v[2 * i], v[2 * i + 1]);
                } else if constexpr (EPI == kEpiResidual16) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) q[16 * p + i] = pack2<__nv_bfloat16>(v[2 * i], v[2 * i + 1]);
                }
            }
            // the staging buffer (per-warp stores: this warp's rows of it) must no longer be read by its last store;
            // batched: once a tile, before the first chunk, for all of the group's buffers
            constexpr bool WARP_STORE = C::STORE_ROWS == 32;
            if (!C::BATCH || ci == 0) {
                constexpr int AHEAD = C::BATCH ? 0 : C::NBUF - 1;
                if constexpr (WARP_STORE) {
                    if (lane == 0) bulk_wait_read<AHEAD>();
                    __syncwarp();
                } else {
                    if (leader) bulk_wait_read<AHEAD>();
                    named_barrier(bar_id, 128);
                }
            }
            constexpr int RB = C::ROW_BYTES;
            if constexpr (C::OUT_BYTES == 4) {
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    *reinterpret_cast<float4*>(buf + swz<RB>(row, j)) =
                        make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < QW / 4; ++j)
                    *reinterpret_cast<uint4*>(buf + swz<RB>(row, j)) =
                        make_uint4(q[4 * j], q[4 * j + 1], q[4 * j + 2], q[4 * j + 3]);
            }
            if (C::BATCH && ci < CPG - 1) continue;   // batched: the fence and the stores after the last chunk
            fence_proxy_async_smem();
            constexpr int NST = C::BATCH ? CPG : 1;   // chunks this fence covers: ci - NST + 1 .. ci
            if constexpr (WARP_STORE) {
                __syncwarp();
                const int wrow = row0 + quarter * 32;   // this warp's first output row
                if (lane == 0 && wrow < M) {
#pragma unroll
                    for (int k = 0; k < NST; ++k) {
                        const int cc = grp + (ci - NST + 1 + k) * C::EG;
                        tma_store_2d(tmC, gbuf + ((g - NST + 1 + k) % C::NBUF) * C::CHUNK_BYTES + quarter * 32 * RB,
                                     colb + cc * C::CHUNK_COLS, wrow);
                    }
                    bulk_commit();
                }
            } else {
                named_barrier(bar_id, 128);
                if (leader) {
#pragma unroll
                    for (int k = 0; k < NST; ++k) {
                        const int cc = grp + (ci - NST + 1 + k) * C::EG;
                        uint8_t* sb = gbuf + ((g - NST + 1 + k) % C::NBUF) * C::CHUNK_BYTES;
                        if constexpr (C::REDUCE) tma_reduce_add_2d(tmC, sb, colb + cc * C::CHUNK_COLS, row0);   // X += v
                        else tma_store_2d(tmC, sb, colb + cc * C::CHUNK_COLS, row0);
                    }
                    bulk_commit();
                }
            }
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
    }
    if (C::STORE_ROWS == 32 ? lane == 0 : leader) bulk_wait_all();
}

// ------------------------------------------------------------------------------------------------ one CTA
// TI: the operands' type (f16, bf16 or e4m3); T: the 16-bit output type of kEpiBias / kEpiBiasGelu.
template <typename TI, typename T, int BN, int EPI>
__global__ void __launch_bounds__(GemmCfg<BN, EPI, false, Operand<TI>::F8>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, int M, int N, int K, const EpiArgs ep, uint32_t* err)
{
    using C = GemmCfg<BN, EPI, false, Operand<TI>::F8>;
    extern __shared__ uint8_t smem_raw[];
    const SmemLayout<C> L(smem_raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (M + C::BM - 1) / C::BM;
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_iters = K / C::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&L.full[s], 1);
            mbar_init(&L.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&L.tfull[b], 1);
            mbar_init(&L.tempty[b], 4 * C::EG);
        }
        mbar_init(L.mma_done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc(L.tmem_slot, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *L.tmem_slot;
    if (threadIdx.x == 0) griddep_launch();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0 && k_iters > 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0;       // bit s: stage s was loaded at least once
            uint32_t issued_par = 0;   // bit s: parity of the last load into stage s
            bool ok = true;
            // the weight tiles of this CTA's first stages depend on no earlier kernel: they load while that
            // kernel finishes; A (an earlier kernel's output) only after griddep_wait
            const int pre = (int)blockIdx.x < num_tiles ? (k_iters < C::STAGES ? k_iters : C::STAGES) : 0;
            for (int kb = 0; kb < pre; ++kb) {
                mbar_arrive_expect_tx(&L.full[kb], C::STAGE_BYTES);
                tma_load_2d(L.sB + kb * C::B_BYTES, &tmB, &L.full[kb], kb * C::BK, ((int)blockIdx.x % n_tiles) * BN);
            }
            griddep_wait();
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                const int m_fwd = tile / n_tiles, n_blk = tile % n_tiles;
                const int m_blk = ep.rev ? m_tiles - 1 - m_fwd : m_fwd;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&L.empty[stage], phase ^ 1u, err, kErrSmemEmpty)) {
                        ok = false;
                        break;
                    }
                    const bool early = tile == (int)blockIdx.x && kb < pre;   // weights already in flight
                    if (!early) mbar_arrive_expect_tx(&L.full[stage], C::STAGE_BYTES);
                    tma_load_2d(L.sA + stage * C::A_BYTES, &tmA, &L.full[stage], kb * C::BK, m_blk * C::BM);
                    if (!early) tma_load_2d(L.sB + stage * C::B_BYTES, &tmB, &L.full[stage], kb * C::BK, n_blk * BN);
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
                if (issued & (1u << s)) mbar_wait(&L.full[s], (issued_par >> s) & 1u, err, kErrTmaFull);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0 && k_iters > 0) {
            constexpr uint32_t idesc = Operand<TI>::idesc(128, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                if (!mbar_wait(&L.tempty[acc], acc_phase ^ 1u, err, kErrTmemEmpty)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&L.full[stage], phase, err, kErrTmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(L.sA + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(L.sB + stage * C::B_BYTES);
#pragma unroll
                    for (int k = 0; k < C::KSTEPS; ++k)
                        umma_issue<TI>(d_tmem, sdesc_sw128(a_addr + 32u * k), sdesc_sw128(b_addr + 32u * k), idesc,
                                       (kb | k) != 0 ? 1u : 0u);
                    umma_commit(&L.empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                umma_commit(&L.tfull[acc]);
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
            // every MMA this thread issued has completed before tensor memory is freed
            umma_commit(L.mma_done);
            mbar_wait(L.mma_done, 0, err, kErrTmemFull);
        }
    } else if (k_iters > 0) {
        const int my_tiles =
            (int)blockIdx.x < num_tiles ? (num_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
        epilogue_loop<T, EPI, C>(
            L, &tmC, tmem_base, my_tiles,
            [&](int it) {
                const int m_fwd = ((int)blockIdx.x + it * (int)gridDim.x) / n_tiles;
                return (ep.rev ? m_tiles - 1 - m_fwd : m_fwd) * C::BM;
            },
            [&](int it) { return (((int)blockIdx.x + it * (int)gridDim.x) % n_tiles) * BN; },
            [&](int acc) { mbar_arrive(&L.tempty[acc]); }, ep, M, N, err);
    }

    __syncwarp();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1) tmem_dealloc(tmem_base, C::TMEM_COLS);
}

// ------------------------------------------------------------------------------------------------ CTA pair
// A cluster of two CTAs computes a 256 x 256 tile. Rank 0 (the leader) owns the ring's `full` barriers (both
// CTAs' loads complete there), the accumulator's `tempty` barriers (both CTAs' epilogue warps arrive there) and
// issues every MMA; each CTA's `empty` and `tfull` barriers are signalled by the leader's commits.
template <typename TI, typename T, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GemmCfg<256, EPI, true, Operand<TI>::F8>::THREADS, 1)
gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, int M, int N, int K, const EpiArgs ep, uint32_t* err)
{
    constexpr int BN = 256;
    using C = GemmCfg<BN, EPI, true, Operand<TI>::F8>;
    extern __shared__ uint8_t smem_raw[];
    const SmemLayout<C> L(smem_raw);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool lead = rank == 0;
    const int pair = (int)blockIdx.x >> 1, num_pairs = (int)gridDim.x >> 1;
    const int m_tiles = (M + 2 * C::BM - 1) / (2 * C::BM);
    const int n_tiles = (N + BN - 1) / BN;
    const int num_tiles = m_tiles * n_tiles;
    const int k_iters = K / C::BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&L.full[s], 1);
            mbar_init(&L.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&L.tfull[b], 1);
            mbar_init(&L.tempty[b], 2 * 4 * C::EG);   // the epilogue warps of both CTAs
        }
        mbar_init(L.mma_done, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(L.tmem_slot, C::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync();   // both CTAs' barriers exist before either signals the other's
    tc_fence_after();
    const uint32_t tmem_base = *L.tmem_slot;
    if (threadIdx.x == 0) griddep_launch();

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer (both CTAs)
        if (lane == 0 && k_iters > 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_par = 0;
            bool ok = true;
            // this CTA's half of the first stages' weight tiles loads before griddep_wait (as in gemm_tc_kernel)
            const int pre = pair < num_tiles ? (k_iters < C::STAGES ? k_iters : C::STAGES) : 0;
            for (int kb = 0; kb < pre; ++kb) {
                if (lead) mbar_arrive_expect_tx(&L.full[kb], 2 * C::STAGE_BYTES);
                tma_load_2d_pair(L.sB + kb * C::B_BYTES, &tmB, mapa_shared(smem_u32(&L.full[kb]), 0), kb * C::BK,
                                 (pair % n_tiles) * BN + (int)rank * C::B_ROWS);
            }
            griddep_wait();
            for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
                const int m_fwd = tile / n_tiles, n_blk = tile % n_tiles;
                const int m_blk = ep.rev ? m_tiles - 1 - m_fwd : m_fwd;
                const int a_row = m_blk * 2 * C::BM + (int)rank * C::BM;
                const int b_row = n_blk * BN + (int)rank * C::B_ROWS;
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&L.empty[stage], phase ^ 1u, err, kErrSmemEmpty)) {
                        ok = false;
                        break;
                    }
                    const bool early = tile == pair && kb < pre;   // weights already in flight
                    if (lead && !early) mbar_arrive_expect_tx(&L.full[stage], 2 * C::STAGE_BYTES);
                    const uint32_t full_lead = mapa_shared(smem_u32(&L.full[stage]), 0);
                    tma_load_2d_pair(L.sA + stage * C::A_BYTES, &tmA, full_lead, kb * C::BK, a_row);
                    if (!early) tma_load_2d_pair(L.sB + stage * C::B_BYTES, &tmB, full_lead, kb * C::BK, b_row);
                    issued |= 1u << stage;
                    issued_par = (issued_par & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // this CTA's copies have landed before it can leave: the leader sees them on its `full` barriers;
            // the other CTA learns it from its `empty` barriers (a stage is released only after both halves
            // landed and were read)
            for (int s = 0; s < C::STAGES; ++s)
                if (issued & (1u << s)) {
                    if (lead) mbar_wait(&L.full[s], (issued_par >> s) & 1u, err, kErrTmaFull);
                    else mbar_wait(&L.empty[s], (issued_par >> s) & 1u, err, kErrSmemEmpty);
                }
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer (leader only)
        if (lead && lane == 0 && k_iters > 0) {
            constexpr uint32_t idesc = Operand<TI>::idesc(256, BN);
            int stage = 0;
            uint32_t phase = 0;
            int acc = 0;
            uint32_t acc_phase = 0;
            bool ok = true;
            for (int tile = pair; tile < num_tiles && ok; tile += num_pairs) {
                if (!mbar_wait(&L.tempty[acc], acc_phase ^ 1u, err, kErrTmemEmpty)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
                for (int kb = 0; kb < k_iters; ++kb) {
                    if (!mbar_wait(&L.full[stage], phase, err, kErrTmaFull)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(L.sA + stage * C::A_BYTES);
                    const uint32_t b_addr = smem_u32(L.sB + stage * C::B_BYTES);
#pragma unroll
                    for (int k = 0; k < C::KSTEPS; ++k)
                        umma_issue_pair<TI>(d_tmem, sdesc_sw128(a_addr + 32u * k), sdesc_sw128(b_addr + 32u * k),
                                            idesc, (kb | k) != 0 ? 1u : 0u);
                    const uint32_t e = smem_u32(&L.empty[stage]);
                    umma_commit_pair(e);                    // this CTA's stage
                    umma_commit_pair(mapa_shared(e, 1));    // the other CTA's stage
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                const uint32_t tf = smem_u32(&L.tfull[acc]);
                umma_commit_pair(tf);
                umma_commit_pair(mapa_shared(tf, 1));
                acc ^= 1;
                if (acc == 0) acc_phase ^= 1u;
            }
            // every MMA issued has completed (both CTAs' tensor memory) before either frees it
            umma_commit_pair(smem_u32(L.mma_done));
            mbar_wait(L.mma_done, 0, err, kErrTmemFull);
        }
    } else if (k_iters > 0) {
        const int my_tiles = pair < num_tiles ? (num_tiles - 1 - pair) / num_pairs + 1 : 0;
        const uint32_t tempty_lead0 = mapa_shared(smem_u32(&L.tempty[0]), 0);
        const uint32_t tempty_lead1 = mapa_shared(smem_u32(&L.tempty[1]), 0);
        epilogue_loop<T, EPI, C>(
            L, &tmC, tmem_base, my_tiles,
            [&](int it) {
                const int m_fwd = (pair + it * num_pairs) / n_tiles;
                return (ep.rev ? m_tiles - 1 - m_fwd : m_fwd) * 2 * C::BM + (int)rank * C::BM;
            },
            [&](int it) { return ((pair + it * num_pairs) % n_tiles) * BN; },
            [&](int acc) { mbar_arrive_cluster(acc ? tempty_lead1 : tempty_lead0); }, ep, M, N, err);
    }

    __syncwarp();
    tc_fence_before();
    cluster_sync();   // the leader's MMAs are done and no CTA signals the other any more
    tc_fence_after();
    if (warp == 1) tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
}

}  // namespace mf
