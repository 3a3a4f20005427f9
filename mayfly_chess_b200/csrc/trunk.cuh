// The bandwidth-bound kernels of the forward pass: the embedding fused with the first LayerNorm, LayerNorm,
// attention per (board, head), the final LayerNorm of the CLS rows, and the search's reduction of the heads.
// Row r of every activation is token r % 65 of board r / 65 (token 0 is CLS), as in
// mayfly/chess/cudanet/cudanet_spec.h:68-80.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <type_traits>

#include "gemm.cuh"

namespace mf {

constexpr int kTokens = 65;
constexpr int kPieces = 13;
constexpr int kHmBuckets = 102;

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

template <typename T> constexpr bool is_e4m3 = std::is_same<T, __nv_fp8_e4m3>::value;

// Four values to p in the activation type T: 16-bit (8 bytes), or e4m3 (4 bytes) after multiplying by `mul`
// (the reciprocal of the consumer's static input scale; the 16-bit types ignore it).
template <typename T> __device__ __forceinline__ void store4(T* p, float a, float b, float c, float d, float mul)
{
    if constexpr (is_e4m3<T>) {
        *reinterpret_cast<uint32_t*>(p) = pack_e4m3x4(a * mul, b * mul, c * mul, d * mul);
    } else {
        uint2 q;
        q.x = pack2<T>(a, b);
        q.y = pack2<T>(c, d);
        *reinterpret_cast<uint2*>(p) = q;
    }
}

// LayerNorm of one row held by one warp (V float4 per lane, lane owns float4s lane, lane+32, ...): biased
// variance from a second pass over (x - mean) in registers, rstd = rsqrt(var + eps), as F.layer_norm in fp32.
template <typename T, int V>
__device__ __forceinline__ void ln_row_store(const float4 (&v)[V], int d, const float* __restrict__ g,
                                             const float* __restrict__ b, T* __restrict__ y, float eps, float mul)
{
    const int lane = threadIdx.x & 31;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = warp_sum(s) / static_cast<float>(d);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const float a = v[i].x - mean, bb = v[i].y - mean, c = v[i].z - mean, e = v[i].w - mean;
        q += (a * a + bb * bb) + (c * c + e * e);
    }
    const float rstd = rsqrtf(warp_sum(q) / static_cast<float>(d) + eps);
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
    for (int i = 0; i < V; ++i) {
        const int c4 = lane + 32 * i;
        const float4 gg = __ldg(g4 + c4), bb = __ldg(b4 + c4);
        store4<T>(y + 4 * c4, (v[i].x - mean) * rstd * gg.x + bb.x, (v[i].y - mean) * rstd * gg.y + bb.y,
                  (v[i].z - mean) * rstd * gg.z + bb.z, (v[i].w - mean) * rstd * gg.w + bb.w, mul);
    }
}

// The residual stream x: f32, or bf16 on the FP8 path. Four consecutive values at p (16 or 8 bytes).
template <typename XT> __device__ __forceinline__ float4 load_x4(const XT* p)
{
    if constexpr (std::is_same<XT, float>::value) {
        return *reinterpret_cast<const float4*>(p);
    } else {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
    }
}

// stores v in XT and returns the value stored (v itself for f32, its bf16 rounding otherwise)
template <typename XT> __device__ __forceinline__ float4 store_x4(XT* p, float4 v)
{
    if constexpr (std::is_same<XT, float>::value) {
        *reinterpret_cast<float4*>(p) = v;
        return v;
    } else {
        uint2 u;
        u.x = pack2<__nv_bfloat16>(v.x, v.y);
        u.y = pack2<__nv_bfloat16>(v.z, v.w);
        *reinterpret_cast<uint2*>(p) = u;
        return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
    }
}

// ------------------------------------------------------------------------------------------------ embed + LN1
// mayfly/chess/chess_net.py:182-192 (cudanet/kernels_trunk.cu:74-122 embed), then layer 0's norm1:
//   x[b*65]     = cls + (cast_b + cast_w . cast[b]) + hm_emb[hm[b]]
//   x[b*65+1+s] = piece[ids[b*64+s]] + pos[s] (+ ep_mark when ep[b] > 0 and s == ep[b] - 1)
//   h = LN(x; g, beta)
// One warp per row, rows = B * 65. ids and hm are clamped to their tables (a bad input cannot read out of
// bounds), as the reference kernel does. d = 128 * V. h is 16-bit, or e4m3 of h * mul (the FP8 path); x is
// f32, or bf16 (the FP8 path), and h is the norm of x as stored.
// One row (a whole warp): the body of embed_ln_kernel.
template <typename T, int V, typename XT = float>
__device__ __forceinline__ void embed_ln_row(
    int row, const int64_t* __restrict__ ids, const float* __restrict__ cast, const int64_t* __restrict__ hm,
    const int64_t* __restrict__ ep, const float* __restrict__ piece, const float* __restrict__ pos,
    const float* __restrict__ cls, const float* __restrict__ cast_w, const float* __restrict__ cast_b,
    const float* __restrict__ hm_emb, const float* __restrict__ ep_mark, const float* __restrict__ g,
    const float* __restrict__ beta, XT* __restrict__ x, T* __restrict__ h, float eps, float mul)
{
    constexpr int d = 128 * V;
    const int lane = threadIdx.x & 31;
    const int b = row / kTokens, t = row % kTokens;
    float4 v[V];
    if (t == 0) {
        const float c0 = cast[4 * b + 0], c1 = cast[4 * b + 1], c2 = cast[4 * b + 2], c3 = cast[4 * b + 3];
        long long hi = hm[b];
        hi = hi < 0 ? 0 : (hi >= kHmBuckets ? kHmBuckets - 1 : hi);
        const float4* cl4 = reinterpret_cast<const float4*>(cls);
        const float4* cb4 = reinterpret_cast<const float4*>(cast_b);
        const float4* he4 = reinterpret_cast<const float4*>(hm_emb + (size_t)hi * d);
        const float4* cw4 = reinterpret_cast<const float4*>(cast_w);   // row c of cast_w [d, 4] is cw4[c]
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int c4 = lane + 32 * i;
            const float4 w0 = __ldg(cw4 + 4 * c4 + 0), w1 = __ldg(cw4 + 4 * c4 + 1);
            const float4 w2 = __ldg(cw4 + 4 * c4 + 2), w3 = __ldg(cw4 + 4 * c4 + 3);
            const float4 bb = __ldg(cb4 + c4), cl = __ldg(cl4 + c4), he = __ldg(he4 + c4);
            const float l0 = bb.x + (w0.x * c0 + w0.y * c1 + w0.z * c2 + w0.w * c3);
            const float l1 = bb.y + (w1.x * c0 + w1.y * c1 + w1.z * c2 + w1.w * c3);
            const float l2 = bb.z + (w2.x * c0 + w2.y * c1 + w2.z * c2 + w2.w * c3);
            const float l3 = bb.w + (w3.x * c0 + w3.y * c1 + w3.z * c2 + w3.w * c3);
            v[i] = make_float4(cl.x + l0 + he.x, cl.y + l1 + he.y, cl.z + l2 + he.z, cl.w + l3 + he.w);
        }
    } else {
        const int s = t - 1;
        long long p = ids[(size_t)b * 64 + s];
        p = p < 0 ? 0 : (p >= kPieces ? kPieces - 1 : p);
        const long long e = ep[b];
        const bool mark = e > 0 && (long long)s == e - 1;
        const float4* pc4 = reinterpret_cast<const float4*>(piece + (size_t)p * d);
        const float4* ps4 = reinterpret_cast<const float4*>(pos + (size_t)s * d);
        const float4* em4 = reinterpret_cast<const float4*>(ep_mark);
#pragma unroll
        for (int i = 0; i < V; ++i) {
            const int c4 = lane + 32 * i;
            const float4 a = __ldg(pc4 + c4), q = __ldg(ps4 + c4);
            float4 r = make_float4(a.x + q.x, a.y + q.y, a.z + q.z, a.w + q.w);
            if (mark) {
                const float4 m = __ldg(em4 + c4);
                r = make_float4(r.x + m.x, r.y + m.y, r.z + m.z, r.w + m.w);
            }
            v[i] = r;
        }
    }
    XT* xr = x + (size_t)row * d;
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = store_x4<XT>(xr + 4 * (lane + 32 * i), v[i]);
    ln_row_store<T, V>(v, d, g, beta, h + (size_t)row * d, eps, mul);
}

template <typename T, int V, typename XT = float>
__global__ void __launch_bounds__(256) embed_ln_kernel(
    const int64_t* __restrict__ ids, const float* __restrict__ cast, const int64_t* __restrict__ hm,
    const int64_t* __restrict__ ep, const float* __restrict__ piece, const float* __restrict__ pos,
    const float* __restrict__ cls, const float* __restrict__ cast_w, const float* __restrict__ cast_b,
    const float* __restrict__ hm_emb, const float* __restrict__ ep_mark, const float* __restrict__ g,
    const float* __restrict__ beta, XT* __restrict__ x, T* __restrict__ h, int rows, float eps, float mul)
{
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;   // whole warp
    embed_ln_row<T, V, XT>(row, ids, cast, hm, ep, piece, pos, cls, cast_w, cast_b, hm_emb, ep_mark, g, beta, x, h,
                           eps, mul);
}

// ------------------------------------------------------------------------------------------------ LayerNorm
// h[r] = LN(x[r]) for rows r = row0 + i * row_stride, i < n (row_stride 65 picks the CLS rows for the final
// norm, chess_net.py:194 / cudanet/kernels_heads.cu:64-86). Output rows are dense: h row i. One warp per row.
// h is 16-bit, or e4m3 of h * mul (the FP8 path); x is f32, or bf16 (the FP8 path).
// Output row i (a whole warp): the body of layernorm_kernel.
template <typename T, int V, typename XT = float>
__device__ __forceinline__ void ln_row(int i, const XT* __restrict__ x, const float* __restrict__ g,
                                       const float* __restrict__ b, T* __restrict__ h, int row_stride, float eps,
                                       float mul)
{
    constexpr int d = 128 * V;
    const int lane = threadIdx.x & 31;
    const XT* xr = x + (size_t)i * row_stride * d;
    float4 v[V];
#pragma unroll
    for (int k = 0; k < V; ++k) v[k] = load_x4<XT>(xr + 4 * (lane + 32 * k));
    ln_row_store<T, V>(v, d, g, b, h + (size_t)i * d, eps, mul);
}

// rev: the rows in descending order (rows the producer of x wrote last, still in L2, come first)
template <typename T, int V, typename XT = float>
__global__ void __launch_bounds__(256) layernorm_kernel(const XT* __restrict__ x, const float* __restrict__ g,
                                                        const float* __restrict__ b, T* __restrict__ h, int n,
                                                        int row_stride, float eps, float mul, int rev)
{
    griddep_wait();
    griddep_launch();
    const int i = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (i >= n) return;
    ln_row<T, V, XT>(rev ? n - 1 - i : i, x, g, b, h, row_stride, eps, mul);
}

// ------------------------------------------------------------------------------------------------ attention
// softmax(q k^T / sqrt(DH)) v over all 65 tokens of one board for one head (chess_net.py:159-161 SDPA, no
// mask; cudanet/kernels_trunk.cu:385-509 attention_mma). qkv [rows, 3*d] holds q, k, v column blocks; head j
// owns columns j*DH..j*DH+DH-1 of each. att [rows, d] gets the heads concatenated.
//
// A persistent kernel: each CTA (5 warps) runs (board, head) items blockIdx.x, + gridDim.x, ... (heads of a
// board on neighbouring CTAs). One thread streams each item's Q, K and V tiles (80 rows x DH from row 65*b,
// three TMA loads with the 128-byte swizzle, or 64-byte for DH = 32) into one of two buffers while the warps
// compute the previous item, so loads and math overlap. Rows 65..79 of a tile are the next board's rows (or
// zeros past the end): finite values whose queries are discarded and whose keys are masked (P = 0 there).
// Warp w owns query rows 16w..16w+15; S = Q K^T and O = P V run on mma.sync m16n8k16 with f32 accumulation
// (ldmatrix addresses follow the swizzle, which keeps them free of bank conflicts); the softmax runs on the S
// fragments in registers (row max and sum across the 4 lanes of a quad by shuffles); P is rounded to the
// 16-bit type for the second product and O is divided by the f32 row sum at the end.
// The output type TO is T, or e4m3 of O * mul (the FP8 path: the out-projection's input).
template <typename T> struct MmaName;
template <> struct MmaName<__half> {
    static __device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
    {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <> struct MmaName<__nv_bfloat16> {
    static __device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1)
    {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// 2^x by the special-function unit (ex2.approx.ftz.f32); 2^-inf = 0
__device__ __forceinline__ float ex2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr int kAttRows = 80;     // 65 tokens padded to 5 tiles of 16
#ifndef MF_ATT_BUFFERS
#define MF_ATT_BUFFERS 2
#endif
constexpr int kAttBuffers = MF_ATT_BUFFERS;   // Q/K/V tile sets per CTA: 2 streams the next item during the math
constexpr int kAttWarps = 5;

template <int DH> struct AttCfg {
    static constexpr int ROWB = DH * 2;                                  // bytes of a 16-bit tile row
    static constexpr uint32_t TILE = kAttRows * ROWB;                    // one of Q, K, V
    static constexpr uint32_t SET = 3 * TILE;                            // one item's tiles
    static constexpr size_t SMEM = 1024 + kAttBuffers * (size_t)SET + 64;   // the sets + barriers
    static_assert(DH == 64 || DH == 32, "head width 32 or 64");
};

// byte offset of 16-byte chunk c of row r in a tile written by TMA with the 128-byte (DH 64) or 64-byte (DH 32)
// swizzle
template <int DH> __device__ __forceinline__ uint32_t att_off(int r, int c)
{
    if constexpr (DH == 64) return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
    else return (uint32_t)(r * 64 + ((c ^ ((r >> 1) & 3)) << 4));
}

// The item loop of the mma.sync attention over items first, first + stride, ... < B * heads, run by every thread
// of the CTA (warps from kAttWarps on only take part in the barriers). Shared memory at `base` holds NB Q/K/V
// tile sets and `full` their NB barriers; thread 0 issues the loads. n counts the items this CTA computed before
// the call (the barriers' phases continue from it) and the count after the call is returned; issued counts the
// items whose loads thread 0 started.
template <typename T, typename TO, int DH, int NB>
__device__ __forceinline__ int attention_mma_items(uint8_t* base, uint64_t* full, volatile uint32_t* ok_flag,
                                                   const CUtensorMap* tmQKVp, TO* __restrict__ att, int B,
                                                   int heads, int d, float scale, float mul, uint32_t* err,
                                                   int first, int stride, int n, int& issued)
{
    using C = AttCfg<DH>;
    static_assert(kTokens == 65 && kAttRows == 80, "the softmax below hard-codes which key tiles are live");
    constexpr int NT = kAttRows / 8;          // 10 key tiles of 8
    constexpr int DT = DH / 8;                // output column tiles of 8
    constexpr int CH = DH * 2 / 16;           // 16-byte chunks per 16-bit row
    const CUtensorMap& tmQKV = *tmQKVp;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int items = B * heads;
    auto issue = [&](int item, int buf) {
        const int b = item / heads, h = item - b * heads;
        uint8_t* s = base + buf * C::SET;
        mbar_arrive_expect_tx(&full[buf], C::SET);
#pragma unroll
        for (int which = 0; which < 3; ++which)
            tma_load_2d(s + which * C::TILE, &tmQKV, &full[buf], which * d + h * DH, b * kTokens);
    };
    if (tid == 0 && first < items) {
        issue(first, n % NB);
        ++issued;
    }

    const int g = lane >> 2, t = lane & 3;
    const int q0 = warp * 16;
    const float sl2 = scale * 1.4426950408889634f;
    for (int item = first; item < items; item += stride, ++n) {
        const int buf = n % NB;
        if (tid == 0) {
            if (NB == 2 && item + stride < items) {
                issue(item + stride, buf ^ 1);   // that buffer's last reader finished before the last barrier
                ++issued;
            }
            *ok_flag = mbar_wait(&full[buf], (n / NB) & 1, err, kErrTmaFull) ? 1u : 0u;
        }
        __syncthreads();
        if (!*ok_flag) break;
        if (warp < kAttWarps) {
            const uint8_t* sQ = base + buf * C::SET;
            const uint8_t* sK = sQ + C::TILE;
            const uint8_t* sV = sK + C::TILE;
            const int b = item / heads, h = item - b * heads;

            // S = Q K^T for this warp's 16 rows and keys 0..71 (key tile 9, keys 72..79, is all padding: P = 0)
            constexpr int NT_LIVE = (kTokens + 7) / 8;   // 9 key tiles hold the 65 live keys
            float s[NT][4];
#pragma unroll
            for (int nn = 0; nn < NT; ++nn) s[nn][0] = s[nn][1] = s[nn][2] = s[nn][3] = 0.f;
#pragma unroll
            for (int k0 = 0; k0 < DH; k0 += 16) {
                uint32_t a[4];
                ldsm_x4(smem_u32(sQ + att_off<DH>(q0 + (lane & 15), (k0 >> 3) + (lane >> 4))), a[0], a[1], a[2], a[3]);
#pragma unroll
                for (int nn = 0; nn < NT_LIVE; nn += 2) {
                    // keys nn*8 .. nn*8+15: matrices (keys 0-7, k0), (keys 0-7, k0+8), (keys 8-15, k0), (keys 8-15, k0+8)
                    const int key = nn * 8 + (lane & 7) + ((lane >> 4) << 3);
                    const int kc = (k0 >> 3) + ((lane >> 3) & 1);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(smem_u32(sK + att_off<DH>(key, kc)), b0, b1, b2, b3);
                    MmaName<T>::mma(s[nn], a, b0, b1);
                    if (nn + 1 < NT_LIVE) MmaName<T>::mma(s[nn + 1], a, b2, b3);
                }
            }

            // softmax over keys 0..64 of rows g and g+8 (each row spread over the quad's 4 lanes), in base 2:
            // exp(x * scale - m) = 2^(x * c - m * c), c = scale * log2(e), one FMA per score before the hardware 2^x
            // (ex2.approx, relative error near 2^-22, far below the 16-bit rounding P gets next). Key tiles 0..7 are
            // all live, tile 8 holds key 64 (lane t = 0, j = 0) and padding, tile 9 is padding: P = 0 there.
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int nn = 0; nn < 8; ++nn) {
                mx0 = fmaxf(mx0, fmaxf(s[nn][0], s[nn][1]));
                mx1 = fmaxf(mx1, fmaxf(s[nn][2], s[nn][3]));
            }
            if (t == 0) {
                mx0 = fmaxf(mx0, s[8][0]);
                mx1 = fmaxf(mx1, s[8][2]);
            }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            const float mc0 = mx0 * sl2, mc1 = mx1 * sl2;
            float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
            for (int nn = 0; nn < 8; ++nn) {
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    s[nn][j] = ex2_approx(fmaf(s[nn][j], sl2, -mc0));
                    s[nn][2 + j] = ex2_approx(fmaf(s[nn][2 + j], sl2, -mc1));
                    sum0 += s[nn][j];
                    sum1 += s[nn][2 + j];
                }
            }
            s[8][0] = t == 0 ? ex2_approx(fmaf(s[8][0], sl2, -mc0)) : 0.f;
            s[8][2] = t == 0 ? ex2_approx(fmaf(s[8][2], sl2, -mc1)) : 0.f;
            s[8][1] = s[8][3] = 0.f;
            sum0 += s[8][0];
            sum1 += s[8][2];
#pragma unroll
            for (int j = 0; j < 4; ++j) s[9][j] = 0.f;
            sum0 += __shfl_xor_sync(0xffffffffu, sum0, 1);
            sum0 += __shfl_xor_sync(0xffffffffu, sum0, 2);
            sum1 += __shfl_xor_sync(0xffffffffu, sum1, 1);
            sum1 += __shfl_xor_sync(0xffffffffu, sum1, 2);

            // O = P V: P's fragments are S's accumulators (keys 16kk..16kk+15 = key tiles 2kk, 2kk+1)
            float o[DT][4];
#pragma unroll
            for (int nn = 0; nn < DT; ++nn) o[nn][0] = o[nn][1] = o[nn][2] = o[nn][3] = 0.f;
#pragma unroll
            for (int kk = 0; kk < kAttRows / 16; ++kk) {
                uint32_t a[4];
                a[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
                a[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
                a[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
                a[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
                for (int nn = 0; nn < DT; nn += 2) {
                    // V rows (keys) 16kk.., transposed: matrices (keys 0-7, cols nn*8), (keys 8-15, cols nn*8),
                    // (keys 0-7, cols nn*8+8), (keys 8-15, cols nn*8+8)
                    const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                    const int vc = nn + (lane >> 4);
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4_t(smem_u32(sV + att_off<DH>(key, vc)), b0, b1, b2, b3);
                    MmaName<T>::mma(o[nn], a, b0, b1);
                    MmaName<T>::mma(o[nn + 1], a, b2, b3);
                }
            }

            // normalise, stage this warp's rows in its own rows of the Q tile (no other warp reads them; the
            // tile is not refilled before the barrier that ends this item), store
            const float inv0 = 1.f / sum0, inv1 = 1.f / sum1;
            uint8_t* st = base + buf * C::SET;
            const size_t row0 = (size_t)b * kTokens;
            __syncwarp();
            if constexpr (is_e4m3<TO>) {
                // e4m3 rows of DH bytes at a pitch of DH + 16 bytes, inside the warp's own 16 rows of the Q tile
                constexpr int PB = DH + 16;
                constexpr int CH8 = DH / 16;
                static_assert(16 * PB <= 16 * C::ROWB, "staging stays inside the warp's rows");
                uint8_t* wst = st + q0 * C::ROWB;
                const float m0 = inv0 * mul, m1 = inv1 * mul;
#pragma unroll
                for (int nn = 0; nn < DT; ++nn) {
                    *reinterpret_cast<uint16_t*>(wst + g * PB + nn * 8 + 2 * t) = static_cast<uint16_t>(
                        __nv_cvt_float2_to_fp8x2(make_float2(o[nn][0] * m0, o[nn][1] * m0), __NV_SATFINITE, __NV_E4M3));
                    *reinterpret_cast<uint16_t*>(wst + (g + 8) * PB + nn * 8 + 2 * t) = static_cast<uint16_t>(
                        __nv_cvt_float2_to_fp8x2(make_float2(o[nn][2] * m1, o[nn][3] * m1), __NV_SATFINITE, __NV_E4M3));
                }
                __syncwarp();
                for (int i = lane; i < 16 * CH8; i += 32) {
                    const int lr = i / CH8, c = i % CH8;
                    if (q0 + lr < kTokens)
                        *(reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(att) + (row0 + q0 + lr) * d +
                                                   (size_t)h * DH) + c) =
                            *reinterpret_cast<const uint4*>(wst + lr * PB + c * 16);
                }
            } else {
#pragma unroll
                for (int nn = 0; nn < DT; ++nn) {
                    *reinterpret_cast<uint32_t*>(st + att_off<DH>(q0 + g, nn) + 4 * t) =
                        pack2<T>(o[nn][0] * inv0, o[nn][1] * inv0);
                    *reinterpret_cast<uint32_t*>(st + att_off<DH>(q0 + g + 8, nn) + 4 * t) =
                        pack2<T>(o[nn][2] * inv1, o[nn][3] * inv1);
                }
                __syncwarp();
                for (int i = lane; i < 16 * CH; i += 32) {
                    const int r = q0 + i / CH, c = i % CH;
                    if (r < kTokens)
                        *(reinterpret_cast<uint4*>(att + (row0 + r) * d + (size_t)h * DH) + c) =
                            *reinterpret_cast<const uint4*>(st + att_off<DH>(r, c));
                }
            }
        }
        fence_proxy_async_smem();   // this thread's shared-memory reads and writes of the buffer come before
        __syncthreads();            // the TMA writes that refill it next
        if (NB == 1 && tid == 0 && item + stride < items) {
            issue(item + stride, 0);
            ++issued;
        }
    }
    return n;
}

template <typename T, typename TO, int DH>
__global__ void __launch_bounds__(kAttWarps * 32) attention_kernel(const __grid_constant__ CUtensorMap tmQKV,
                                                                   TO* __restrict__ att, int B, int heads, int d,
                                                                   float scale, float mul, uint32_t* err)
{
    using C = AttCfg<DH>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int NB = kAttBuffers;
    uint64_t* full = reinterpret_cast<uint64_t*>(base + NB * C::SET);
    volatile uint32_t* ok_flag = reinterpret_cast<volatile uint32_t*>(full + 2);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < NB; ++i) mbar_init(&full[i], 1);
        fence_barrier_init();
        tma_prefetch_desc(&tmQKV);
    }
    __syncthreads();
    griddep_wait();   // qkv and att belong to the earlier kernels until they complete
    if (tid == 0) griddep_launch();
    int issued = 0;   // items whose loads thread 0 started (thread 0's count)
    const int n = attention_mma_items<T, TO, DH, NB>(base, full, ok_flag, &tmQKV, att, B, heads, d, scale, mul, err,
                                                     blockIdx.x, gridDim.x, 0, issued);
    // the loads thread 0 started have landed before the CTA leaves (only after a failed wait are any pending)
    if (tid == 0)
        for (int k = n; k < issued; ++k) mbar_wait(&full[k % NB], (k / NB) & 1, err, kErrTmaFull);
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }


// ------------------------------------------------------------------------------------------------ CLS attention
// The last layer needs attention for the CLS query only (the heads read the CLS row alone, chess_net.py:194):
// att_cls[b, head] = softmax(q_cls k^T / sqrt(DH)) v over the 65 keys of board b. One warp per (board, head):
// lane j scores keys j, j + 32 and j + 64 (q broadcast to every lane in registers, each key row read whole),
// the softmax is a warp reduction, then lane j accumulates output dims 2j, 2j + 1 over the 65 keys (each key's
// probability broadcast by a shuffle). att_cls [B, d] is dense; TO is T, or e4m3 of att * mul (the FP8 path).
// One (board, head) item (a whole warp): the body of attention_cls_kernel.
template <typename T, typename TO, int DH>
__device__ __forceinline__ void attention_cls_item(int item, const T* __restrict__ qkv, TO* __restrict__ att,
                                                   int heads, int d, float scale, float mul)
{
    static_assert(DH == 64 || DH == 32, "head width 32 or 64");
    const int lane = threadIdx.x & 31;
    const int b = item / heads, h = item - b * heads;
    const size_t ld = 3 * (size_t)d;
    const T* q = qkv + (size_t)b * kTokens * ld + (size_t)h * DH;   // token 0's q
    const T* kb = q + d;                                              // token 0's k; token t at + t * ld
    const T* vb = q + 2 * (size_t)d;

    float qf[DH];
#pragma unroll
    for (int c = 0; c < DH / 8; ++c) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(q) + c);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            qf[8 * c + 2 * i] = to_f32<T>(reinterpret_cast<const T*>(&w[i])[0]);
            qf[8 * c + 2 * i + 1] = to_f32<T>(reinterpret_cast<const T*>(&w[i])[1]);
        }
    }
    const float sl2 = scale * 1.4426950408889634f;
    float sc[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int key = lane + 32 * j;
        sc[j] = -INFINITY;
        if (key < kTokens) {
            const uint4* kr = reinterpret_cast<const uint4*>(kb + (size_t)key * ld);
            float acc = 0.f;
#pragma unroll
            for (int c = 0; c < DH / 8; ++c) {
                const uint4 u = __ldg(kr + c);
                const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    acc = fmaf(qf[8 * c + 2 * i], to_f32<T>(reinterpret_cast<const T*>(&w[i])[0]), acc);
                    acc = fmaf(qf[8 * c + 2 * i + 1], to_f32<T>(reinterpret_cast<const T*>(&w[i])[1]), acc);
                }
            }
            sc[j] = acc * sl2;
        }
    }
    const float mx = warp_max(fmaxf(fmaxf(sc[0], sc[1]), sc[2]));
    float p[3], sum = 0.f;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        p[j] = ex2_approx(sc[j] - mx);   // 2^-inf = 0 for the keys past 64
        sum += p[j];
    }
    sum = warp_sum(sum);
    float o0 = 0.f, o1 = 0.f;
    const bool owns = 2 * lane < DH;   // lane j: output dims 2j, 2j + 1
    for (int key = 0; key < kTokens; ++key) {
        const float pk = __shfl_sync(0xffffffffu, p[key >> 5], key & 31);
        if (owns) {
            const uint32_t w = __ldg(reinterpret_cast<const uint32_t*>(vb + (size_t)key * ld) + lane);
            o0 = fmaf(pk, to_f32<T>(reinterpret_cast<const T*>(&w)[0]), o0);
            o1 = fmaf(pk, to_f32<T>(reinterpret_cast<const T*>(&w)[1]), o1);
        }
    }
    if (!owns) return;
    const float inv = 1.f / sum;
    const size_t oc = (size_t)b * d + (size_t)h * DH + 2 * lane;
    if constexpr (is_e4m3<TO>) {
        *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(att) + oc) = static_cast<uint16_t>(
            __nv_cvt_float2_to_fp8x2(make_float2(o0 * inv * mul, o1 * inv * mul), __NV_SATFINITE, __NV_E4M3));
    } else {
        *reinterpret_cast<uint32_t*>(att + oc) = pack2<T>(o0 * inv, o1 * inv);
    }
}

template <typename T, typename TO, int DH>
__global__ void __launch_bounds__(256) attention_cls_kernel(const T* __restrict__ qkv, TO* __restrict__ att,
                                                            int B, int heads, int d, float scale, float mul)
{
    griddep_wait();
    griddep_launch();
    const int item = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= B * heads) return;   // whole warp
    attention_cls_item<T, TO, DH>(item, qkv, att, heads, d, scale, mul);
}

// ------------------------------------------------------------------------------------------------ calibration
// out = max(out, max |p[i]|) over i < n (out holds the f32 bits: non-negative floats order like their bits).
// Records the ranges of the four product inputs in a 16-bit pass, from which the FP8 path's static input
// scales are set.
template <typename T>
__global__ void __launch_bounds__(256) absmax_kernel(const T* __restrict__ p, size_t n, unsigned int* __restrict__ out)
{
    float m = 0.f;
    griddep_wait();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(to_f32<T>(p[i])));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));
}

// ------------------------------------------------------------------------------------------------ heads_post
// The search's reduction of the two heads at each row's legal moves (mcts.py:1152-1164 _collect,
// cpp/export_ts.py:147-156 post, cudanet/kernels_heads.cu:88-143 heads_post):
//   p_k = policy[I_k], q_k = sigmoid(qvalue[I_k]); w = softmax(p over legal k)
//   val = 2 * sum_k w_k q_k - 1;  pol_k = p_k, qv_k = 2 q_k - 1 on legal slots, 0 on padding
// A row with no legal slot gets val = -1. logits [B, 2*moves] f32 (policy, then qvalue). One warp per board.
// Policy indices outside 0..moves-1 are clamped (a bad input cannot read out of bounds).
__device__ __forceinline__ void heads_post_board(int b, const float* __restrict__ logits,
                                                 const int64_t* __restrict__ I, const uint8_t* __restrict__ Mk,
                                                 int wide, int moves, float* __restrict__ pol,
                                                 float* __restrict__ val, float* __restrict__ qv)
{
    const int lane = threadIdx.x & 31;
    const float* lp = logits + (size_t)b * 2 * moves;
    const float* lq = lp + moves;
    const size_t base = (size_t)b * wide;
    float mx = -INFINITY;
    for (int k = lane; k < wide; k += 32) {
        if (Mk[base + k]) {
            long long j = I[base + k];
            j = j < 0 ? 0 : (j >= moves ? moves - 1 : j);
            const float p = lp[j];
            pol[base + k] = p;
            qv[base + k] = (1.0f / (1.0f + expf(-lq[j]))) * 2.0f - 1.0f;
            mx = fmaxf(mx, p);
        } else {
            pol[base + k] = 0.0f;
            qv[base + k] = 0.0f;
        }
    }
    mx = warp_max(mx);
    float s = 0.f, acc = 0.f;
    for (int k = lane; k < wide; k += 32) {
        if (Mk[base + k]) {
            long long j = I[base + k];
            j = j < 0 ? 0 : (j >= moves ? moves - 1 : j);
            const float e = expf(lp[j] - mx);
            s += e;
            acc += e * (1.0f / (1.0f + expf(-lq[j])));
        }
    }
    s = warp_sum(s);
    acc = warp_sum(acc);
    if (lane == 0) val[b] = s > 0.f ? (acc / s) * 2.0f - 1.0f : -1.0f;
}

__global__ void __launch_bounds__(256) heads_post_kernel(const float* __restrict__ logits,
                                                         const int64_t* __restrict__ I,
                                                         const uint8_t* __restrict__ Mk, int B, int wide,
                                                         int moves, float* __restrict__ pol,
                                                         float* __restrict__ val, float* __restrict__ qv)
{
    griddep_wait();
    const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (b >= B) return;
    heads_post_board(b, logits, I, Mk, wide, moves, pol, val, qv);
}

}  // namespace mf
