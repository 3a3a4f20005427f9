// The evaluator's host runtime and its C ABI (include/cudanet_b200.h).
//
// One Net owns, on one device: the weights (one allocation, tensors at their 256-aligned file offsets), every
// activation buffer for max_batch positions, one stream, a CUDA graph of the whole forward per batch size
// (captured on its first use), pinned host staging for two batches in flight, and a device error word that
// the kernels' bounded waits write. This is the role of the reference's CudaNet
// (mayfly/chess/cudanet/cudanet.h:15-59, cudanet/cudanet.cpp:144-770), re-designed for sm_100a:
//   * the products are this library's tcgen05 GEMMs (gemm.cuh), not cuBLASLt, fed by TMA tensor maps made
//     once per buffer;
//   * GELU and the residual adds are GEMM epilogues, the first LayerNorm is fused into the embedding;
//   * kernels are compiled ahead of time for sm_100a (no NVRTC, no runtime library loading).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <mutex>
#include <set>
#include <stdexcept>
#include <string>
#include <tuple>
#include <type_traits>
#include <vector>

#include "../../include/cudanet_b200.h"
#include "attention_tc.cuh"
#include "encode.cuh"
#include "gemm_ln.cuh"
#include "json_min.h"
#include "trunk.cuh"

namespace mf {

// ------------------------------------------------------------------------------------------------ errors
static void check_rt(cudaError_t e, const char* what, int line)
{
    if (e != cudaSuccess)
        throw std::runtime_error(std::string("cudanet_b200: ") + what + " failed (line " + std::to_string(line) +
                                 "): " + cudaGetErrorString(e));
}
#define RT(call) check_rt((call), #call, __LINE__)

static const char* err_site_name(uint32_t site)
{
    switch (site) {
        case kErrTmaFull: return "a tensor-core product waited too long for a TMA tile";
        case kErrSmemEmpty: return "a TMA load waited too long for a free shared-memory stage";
        case kErrTmemFull: return "an epilogue waited too long for its accumulator";
        case kErrTmemEmpty: return "a tensor-core product waited too long for a free accumulator";
        case kErrArgs: return "a kernel was launched with arguments it cannot handle";
        case kErrCluster: return "a CTA waited too long for its cluster's row statistics";
        default: return "unknown device error";
    }
}

// ------------------------------------------------------------------------------------------------ TMA maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled()
{
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (!fn) throw std::runtime_error("cudanet_b200: the driver has no cuTensorMapEncodeTiled");
    return fn;
}

// A row-major matrix [outer, inner] with row pitch `pitch` elements, tiles of box_inner x box_outer with the
// 128-byte swizzle (box_inner * element size = 128 bytes: the layout sdesc_sw128 and the epilogue's staging
// describe) or, with swz64, the 64-byte swizzle (64-byte box rows: the GELU epilogues' staging). Reads past the
// extents are zero, writes past them are dropped. U8 carries e4m3 bytes.
enum class MapType { F16, BF16, F32, U8 };

static uint64_t map_elem_bytes(MapType type) { return type == MapType::F32 ? 4 : type == MapType::U8 ? 1 : 2; }

static CUtensorMap make_map(const void* base, MapType type, uint64_t inner, uint64_t outer, uint64_t pitch,
                            uint32_t box_inner, uint32_t box_outer, bool swz64 = false)
{
    const uint64_t es = map_elem_bytes(type);
    if ((reinterpret_cast<uintptr_t>(base) & 15) || (pitch * es) % 16)
        throw std::runtime_error("cudanet_b200: a TMA operand or its row pitch is not 16-byte aligned");
    if (box_inner * es != (swz64 ? 64u : 128u))
        throw std::runtime_error("cudanet_b200: TMA box rows must be 128 bytes (64 with the 64-byte swizzle)");
    CUtensorMap m;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {pitch * es};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = type == MapType::F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : type == MapType::BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                   : type == MapType::U8   ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const CUresult r = encode_tiled()(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                      CU_TENSOR_MAP_INTERLEAVE_NONE,
                                      swz64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        throw std::runtime_error("cudanet_b200: cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return m;
}

static MapType type16(bool bf16) { return bf16 ? MapType::BF16 : MapType::F16; }

// A K-major operand [rows, K]: 16-bit (tiles of 64 x box_rows) or e4m3 (U8, tiles of 128 x box_rows).
static CUtensorMap operand_map(const void* base, MapType type, uint64_t K, uint64_t rows, uint32_t box_rows)
{
    return make_map(base, type, K, rows, K, static_cast<uint32_t>(128 / map_elem_bytes(type)), box_rows);
}

// The output (and, for the residuals, the input) of a product: [M, N] with pitch ldc, 16-bit (`t16`) for
// kEpiBias / kEpiBiasGelu, f32 for kEpiResidual / kEpiF32, e4m3 for kEpiGeluE4m3, bf16 for kEpiResidual16;
// boxes of one epilogue store (GemmCfg::ROW_BYTES wide: 64-byte rows for the GELU epilogues, the bf16 residual
// and the bias epilogue of an FP8 product, `f8`; store_rows(epi, f8) rows high). The residuals' maps take TMA
// reduce-adds into X.
static CUtensorMap output_map(void* base, int epi, MapType t16, int M, int N, int ldc, bool f8 = false)
{
    const uint32_t rows = static_cast<uint32_t>(store_rows(epi, f8));
    if (epi == kEpiResidual || epi == kEpiF32) return make_map(base, MapType::F32, N, M, ldc, 32, rows);
    if (epi == kEpiGeluE4m3) return make_map(base, MapType::U8, N, M, ldc, 64, rows, true);
    if (epi == kEpiBiasGelu) return make_map(base, t16, N, M, ldc, 32, rows, true);
    if (epi == kEpiResidual16) return make_map(base, MapType::BF16, N, M, ldc, 32, rows, true);
    if (epi == kEpiBias && f8 && MF_F8_BIAS_NARROW) return make_map(base, t16, N, M, ldc, 32, rows, true);
    return make_map(base, t16, N, M, ldc, 64, rows);
}

// ------------------------------------------------------------------------------------------------ launchers
// MAYFLY_CUDANET_PDL=0 launches without programmatic dependent launch (each kernel then starts only after the
// previous one has completed); the default lets each kernel's prologue, and a product's first weight tiles,
// overlap the previous kernel's tail (griddep_wait in the kernels keeps the data dependencies).
static bool pdl_on()
{
    static bool on = [] {
        const char* e = std::getenv("MAYFLY_CUDANET_PDL");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    return on;
}

template <typename... KArgs, typename... Args>
static void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_on() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    RT(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

template <typename TI, typename T, int BN, int EPI>
static void launch_gemm_bn(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M, int N, int K,
                           const EpiArgs& ep, uint32_t* err, int num_sms, cudaStream_t s)
{
    using C = GemmCfg<BN, EPI, false, Operand<TI>::F8>;
    // the shared-memory opt-in, once per instantiation and device (the first launch of a batch size is eager,
    // never inside a graph capture)
    static bool attr[64] = {};
    int dev = 0;
    RT(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_b200: device index out of range");
    if (!attr[dev]) {
        RT(cudaFuncSetAttribute(gemm_tc_kernel<TI, T, BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)C::SMEM));
        attr[dev] = true;
    }
    const int tiles = ((M + C::BM - 1) / C::BM) * ((N + BN - 1) / BN);
    const int grid = std::min(tiles, num_sms);
    launch_k(gemm_tc_kernel<TI, T, BN, EPI>, dim3(grid), dim3(C::THREADS), C::SMEM, s, ma, mb, mc, M, N, K, ep, err);
}

// The CTA-pair kernel: 256 x 256 tiles, as many clusters as can be resident at once (a persistent grid must
// never wait for a cluster slot).
template <typename TI, typename T, int EPI>
static void launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M, int N,
                             int K, const EpiArgs& ep, uint32_t* err, cudaStream_t s)
{
    using C = GemmCfg<256, EPI, true, Operand<TI>::F8>;
    static int max_pairs[64] = {};
    int dev = 0;
    RT(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_b200: device index out of range");
    if (!max_pairs[dev]) {
        RT(cudaFuncSetAttribute(gemm_tc_pair_kernel<TI, T, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)C::SMEM));
        int sms = 0;
        RT(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = C::SMEM;
        int clusters = 0;
        RT(cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_pair_kernel<TI, T, EPI>, &cfg));
        if (clusters < 1) throw std::runtime_error("cudanet_b200: no CTA pair fits on this device");
        max_pairs[dev] = clusters;
    }
    const int tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const int pairs = std::min(tiles, max_pairs[dev]);
    launch_k(gemm_tc_pair_kernel<TI, T, EPI>, dim3(2 * pairs), dim3(C::THREADS), C::SMEM, s, ma, mb, mc, M, N, K, ep,
             err);
}

// X += A W^T + bias, then H = LN(X) (gemm_ln.cuh): one cluster of d / 256 CTAs per 128-row block, as many
// clusters as can be resident.
template <typename T, int NCL>
static void launch_gemm_resln_ncl(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mx,
                                  const CUtensorMap& mh, int M, int K, const float* bias, const float* g,
                                  const float* b, uint32_t* err, cudaStream_t s)
{
    using C = ResLnCfg<NCL>;
    static int max_clusters[64] = {};
    int dev = 0;
    RT(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_b200: device index out of range");
    if (!max_clusters[dev]) {
        RT(cudaFuncSetAttribute(gemm_tc_resln_kernel<T, NCL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)C::SMEM));
        int sms = 0;
        RT(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(sms / NCL * NCL));
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = C::SMEM;
        int clusters = 0;
        RT(cudaOccupancyMaxActiveClusters(&clusters, gemm_tc_resln_kernel<T, NCL>, &cfg));
        if (clusters < 1) throw std::runtime_error("cudanet_b200: no LayerNorm cluster fits on this device");
        max_clusters[dev] = clusters;
    }
    const int m_tiles = (M + 127) / 128;
    const int clusters = std::min(m_tiles, max_clusters[dev]);
    launch_k(gemm_tc_resln_kernel<T, NCL>, dim3(clusters * NCL), dim3(C::THREADS), C::SMEM, s, ma, mb, mx, mh, M, K,
             bias, g, b, 1e-5f, err);
}

template <typename T>
static void launch_gemm_resln(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mx,
                              const CUtensorMap& mh, int M, int N, int K, const float* bias, const float* g,
                              const float* b, uint32_t* err, cudaStream_t s)
{
    if (K % 64 || K <= 0) throw std::runtime_error("cudanet_b200: GEMM K must be a positive multiple of 64");
    if (M < 1) throw std::runtime_error("cudanet_b200: GEMM with an empty output");
    if ((reinterpret_cast<uintptr_t>(bias) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(b)) & 15)
        throw std::runtime_error("cudanet_b200: bias and LayerNorm vectors must be 16-byte aligned");
    switch (N) {
        case 256: launch_gemm_resln_ncl<T, 1>(ma, mb, mx, mh, M, K, bias, g, b, err, s); break;
        case 512: launch_gemm_resln_ncl<T, 2>(ma, mb, mx, mh, M, K, bias, g, b, err, s); break;
        case 1024: launch_gemm_resln_ncl<T, 4>(ma, mb, mx, mh, M, K, bias, g, b, err, s); break;
        default: throw std::runtime_error("cudanet_b200: the fused LayerNorm product needs N in {256, 512, 1024}");
    }
}

// The epilogues each operand type has: 16-bit products bias / bias+GELU (16-bit out), residual, f32; FP8
// products bias (16-bit out), residual (f32 or bf16), f32, and bias+GELU with e4m3 out.
template <typename TI, int EPI, int BN> constexpr bool epi_supported()
{
    if constexpr (Operand<TI>::F8) return EPI != kEpiBiasGelu;
    else return EPI != kEpiGeluE4m3 && EPI != kEpiResidual16;
}

template <typename TI, typename T, int BN, int EPI>
static void launch_gemm_bn_if(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M, int N,
                              int K, const EpiArgs& ep, uint32_t* err, int num_sms, cudaStream_t s)
{
    if constexpr (epi_supported<TI, EPI, BN>()) launch_gemm_bn<TI, T, BN, EPI>(ma, mb, mc, M, N, K, ep, err, num_sms, s);
    else throw std::runtime_error("cudanet_b200: this epilogue is not built for this operand type and tile");
}

template <typename TI, typename T, int BN>
static void launch_gemm_epi(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M,
                            int N, int K, const EpiArgs& ep, uint32_t* err, int num_sms, cudaStream_t s)
{
    switch (epi) {
        case kEpiBias: launch_gemm_bn_if<TI, T, BN, kEpiBias>(ma, mb, mc, M, N, K, ep, err, num_sms, s); break;
        case kEpiBiasGelu: launch_gemm_bn_if<TI, T, BN, kEpiBiasGelu>(ma, mb, mc, M, N, K, ep, err, num_sms, s); break;
        case kEpiResidual: launch_gemm_bn_if<TI, T, BN, kEpiResidual>(ma, mb, mc, M, N, K, ep, err, num_sms, s); break;
        case kEpiF32: launch_gemm_bn_if<TI, T, BN, kEpiF32>(ma, mb, mc, M, N, K, ep, err, num_sms, s); break;
        case kEpiGeluE4m3: launch_gemm_bn_if<TI, T, BN, kEpiGeluE4m3>(ma, mb, mc, M, N, K, ep, err, num_sms, s); break;
        case kEpiResidual16:
            launch_gemm_bn_if<TI, T, BN, kEpiResidual16>(ma, mb, mc, M, N, K, ep, err, num_sms, s);
            break;
        default: throw std::runtime_error("cudanet_b200: unknown epilogue");
    }
}

template <typename TI, typename T, int EPI>
static void launch_gemm_pair_if(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M, int N,
                                int K, const EpiArgs& ep, uint32_t* err, cudaStream_t s)
{
    if constexpr (epi_supported<TI, EPI, 256>()) launch_gemm_pair<TI, T, EPI>(ma, mb, mc, M, N, K, ep, err, s);
    else throw std::runtime_error("cudanet_b200: this epilogue is not built for this operand type");
}

// Tile choice: kPairTile (a CTA pair per 256 x 256 tile) when there are at least as many pair tiles as pairs
// fit and the epilogue is light next to the MMAs (bias-only, f32 outputs, the residuals' TMA reductions, or
// K >= 2048), or, for the 16-bit GELU epilogue, when every pair gets at least four tiles (measured on a B200 in
// the graph pass: ff1 on pairs +1.3% positions/s for the bf16 pass at B = 1,024 and 4,096, though its eager
// per-step time reads a little slower: the single-CTA kernel is bound by shared-memory bandwidth near two thirds
// of the tensor rate, a pair near four fifths; the FP8 ff1, whose MMAs take half as long, stays single, its
// GELU epilogue exposed on pairs: -1% to +0.8% across runs), else the widest single-CTA
// tile that still gives two thirds of the SMs a tile. A launch costs ~10 us however small it is, so at small M
// fewer, wider tiles win while most SMs are busy (measured, back-to-back launches: M = 4,160, the out product
// 14.4 us with 132 tiles of 256 against 18.2 with 264 of 128; ff2 20.5 against 28.3); below that the weights
// stream through too few SMs.
constexpr int kPairTile = 2;

// MAYFLY_CUDANET_TILE: "pair" or "single" forces the CTA-pair or the single-CTA kernels, anything else (the
// default) chooses per product.
static int tile_mode()
{
    static int mode = [] {
        const char* e = std::getenv("MAYFLY_CUDANET_TILE");
        if (e && std::strcmp(e, "pair") == 0) return 1;
        if (e && std::strcmp(e, "single") == 0) return 2;
        return 0;
    }();
    return mode;
}

static int pick_bn(int M, int N, int K, int epi, int num_sms)
{
    const int mode = tile_mode();
    const bool light = epi == kEpiBias || epi == kEpiF32 || epi == kEpiResidual || epi == kEpiResidual16 || K >= 2048;
    const int pair_tiles = ((M + 255) / 256) * ((N + 255) / 256);
    const bool gelu16 = epi == kEpiBiasGelu;
    if (mode == 1 || (mode == 0 && (light ? pair_tiles >= num_sms / 2 : gelu16 && pair_tiles >= 2 * num_sms)))
        return kPairTile;
    const int m_tiles = (M + 127) / 128;
    for (int bn : {256, 128})
        if (3 * m_tiles * ((N + bn - 1) / bn) >= 2 * num_sms) return bn;
    return 64;
}

// rows of W in one TMA box for a tile choice
static uint32_t w_box_rows(int bn) { return bn == kPairTile ? 128u : static_cast<uint32_t>(bn); }

// C = epilogue(A W^T) with A, W of type TI (f16, bf16 or e4m3) and T the 16-bit output type of kEpiBias.
template <typename TI, typename T>
static void launch_gemm(int epi, int bn, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M,
                        int N, int K, const EpiArgs& ep, uint32_t* err, int num_sms, cudaStream_t s)
{
    constexpr int bk = Operand<TI>::F8 ? 128 : 64;
    if (K % bk || K <= 0)
        throw std::runtime_error("cudanet_b200: GEMM K must be a positive multiple of " + std::to_string(bk));
    if (M < 1 || N < 1) throw std::runtime_error("cudanet_b200: GEMM with an empty output");
    if (!ep.bias || (reinterpret_cast<uintptr_t>(ep.bias) & 15))
        throw std::runtime_error("cudanet_b200: bias missing or not 16-byte aligned");
    if (Operand<TI>::F8 && (!ep.colscale || (reinterpret_cast<uintptr_t>(ep.colscale) & 15)))
        throw std::runtime_error("cudanet_b200: FP8 column scales missing or not 16-byte aligned");
    if (bn == kPairTile) {
        switch (epi) {
            case kEpiBias: launch_gemm_pair_if<TI, T, kEpiBias>(ma, mb, mc, M, N, K, ep, err, s); break;
            case kEpiBiasGelu: launch_gemm_pair_if<TI, T, kEpiBiasGelu>(ma, mb, mc, M, N, K, ep, err, s); break;
            case kEpiResidual: launch_gemm_pair_if<TI, T, kEpiResidual>(ma, mb, mc, M, N, K, ep, err, s); break;
            case kEpiF32: launch_gemm_pair_if<TI, T, kEpiF32>(ma, mb, mc, M, N, K, ep, err, s); break;
            case kEpiGeluE4m3: launch_gemm_pair_if<TI, T, kEpiGeluE4m3>(ma, mb, mc, M, N, K, ep, err, s); break;
            case kEpiResidual16: launch_gemm_pair_if<TI, T, kEpiResidual16>(ma, mb, mc, M, N, K, ep, err, s); break;
            default: throw std::runtime_error("cudanet_b200: unknown epilogue");
        }
    } else if (bn == 256) launch_gemm_epi<TI, T, 256>(epi, ma, mb, mc, M, N, K, ep, err, num_sms, s);
    else if (bn == 128) launch_gemm_epi<TI, T, 128>(epi, ma, mb, mc, M, N, K, ep, err, num_sms, s);
    else if (bn == 64) launch_gemm_epi<TI, T, 64>(epi, ma, mb, mc, M, N, K, ep, err, num_sms, s);
    else throw std::runtime_error("cudanet_b200: tile choice must be 2 (CTA pair), 64, 128 or 256");
}

// h = LN(x) in T (16-bit, or e4m3 of h * mul), x f32 or bf16 (XT)
template <typename T, typename XT = float>
static void launch_layernorm(const XT* x, const float* g, const float* b, T* h, int n, int d, int row_stride,
                             float mul, cudaStream_t s, int rev = 0)
{
    const dim3 grid((n + 7) / 8), block(256);
    switch (d) {
        case 256: launch_k(layernorm_kernel<T, 2, XT>, grid, block, 0, s, x, g, b, h, n, row_stride, 1e-5f, mul, rev);
            break;
        case 512: launch_k(layernorm_kernel<T, 4, XT>, grid, block, 0, s, x, g, b, h, n, row_stride, 1e-5f, mul, rev);
            break;
        case 1024: launch_k(layernorm_kernel<T, 8, XT>, grid, block, 0, s, x, g, b, h, n, row_stride, 1e-5f, mul, rev);
            break;
        default: throw std::runtime_error("cudanet_b200: width must be 256, 512 or 1024");
    }
}

// The TMA map attention reads qkv [rows, 3d] through: boxes of one head's DH columns x 80 rows.
static CUtensorMap qkv_map(const void* qkv, bool bf16, int rows, int d, int heads)
{
    const int dh = d / heads;
    if (dh != 64 && dh != 32) throw std::runtime_error("cudanet_b200: head width must be 32 or 64");
    return make_map(qkv, type16(bf16), static_cast<uint64_t>(3 * d), static_cast<uint64_t>(rows),
                    static_cast<uint64_t>(3 * d), static_cast<uint32_t>(dh), kAttRows, dh == 32);
}

template <typename T, typename TO, int DH>
static void launch_attention_dh(const CUtensorMap& map, TO* att, int B, int d, int heads, float mul, uint32_t* err,
                                cudaStream_t s)
{
    using C = AttCfg<DH>;
    static int per_sm[64] = {};
    static int sms[64] = {};
    int dev = 0;
    RT(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_b200: device index out of range");
    if (!per_sm[dev]) {
        RT(cudaFuncSetAttribute(attention_kernel<T, TO, DH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)C::SMEM));
        // the whole unified L1 / shared array as shared memory: three CTAs (two buffer sets each) per SM
        RT(cudaFuncSetAttribute(attention_kernel<T, TO, DH>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared));
        int k = 0;
        RT(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, attention_kernel<T, TO, DH>, kAttWarps * 32, C::SMEM));
        if (k < 1) throw std::runtime_error("cudanet_b200: the attention kernel does not fit on this device");
        RT(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
        per_sm[dev] = k;
    }
    const int items = B * heads;
    const int grid = std::min(items, per_sm[dev] * sms[dev]);
    const float scale = 1.0f / std::sqrt(static_cast<float>(DH));
    launch_k(attention_kernel<T, TO, DH>, dim3(grid), dim3(kAttWarps * 32), C::SMEM, s, map, att, B, heads, d, scale,
             mul, err);
}

// Which attention kernel runs head width 64 (attention_tc.cuh has two tensor-memory kernels: two softmax groups
// with a finished item pending per group, and four groups that finish each item before the next, over five
// tensor-memory slots). Measured on a B200, the four-group kernel is the fastest for both output types: 2.36 ms
// per 1,024-position bf16 pass against 2.59 for the mma.sync kernel and 2.90 for the two-group one, and 8.46
// against 8.96 ms (two-group) per 4,096-position FP8 pass. Forcing: MAYFLY_CUDANET_ATT_TC=0 the mma.sync kernel,
// 1 the two-group kernel, 4 the four-group kernel.
static int att_tc_env()
{
    const char* e = std::getenv("MAYFLY_CUDANET_ATT_TC");
    if (e && std::strcmp(e, "1") == 0) return 1;
    if (e && std::strcmp(e, "4") == 0) return 4;
    if (e && std::strcmp(e, "0") == 0) return 0;
    return -1;
}

static int att_tc_mode()
{
    static int mode = att_tc_env();
    return mode;
}

template <typename T, typename TO>
static void launch_attention_tc4(const CUtensorMap& map, TO* att, int B, int d, int heads, float mul, uint32_t* err,
                                 cudaStream_t s, int rev = 0)
{
    using C = AttTc4Cfg;
    static bool attr[64] = {};
    static int sms[64] = {};
    int dev = 0;
    RT(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_b200: device index out of range");
    if (!attr[dev]) {
        RT(cudaFuncSetAttribute(attention_tc4_kernel<T, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
        RT(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
        attr[dev] = true;
    }
    const int items = B * heads;
    const float scale = 1.0f / std::sqrt(static_cast<float>(C::DH));
    launch_k(attention_tc4_kernel<T, TO>, dim3(std::min(items, sms[dev])), dim3(C::THREADS), C::SMEM, s, map, att, B,
             heads, d, scale, mul, err, rev);
}

// the tcgen05 attention (attention_tc.cuh): one CTA per SM, persistent over the (board, head) items
template <typename T, typename TO>
static void launch_attention_tc(const CUtensorMap& map, TO* att, int B, int d, int heads, float mul, uint32_t* err,
                                cudaStream_t s)
{
    using C = AttTcCfg;
    static bool attr[64] = {};
    static int sms[64] = {};
    int dev = 0;
    RT(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_b200: device index out of range");
    if (!attr[dev]) {
        RT(cudaFuncSetAttribute(attention_tc_kernel<T, TO>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
        RT(cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev));
        attr[dev] = true;
    }
    const int items = B * heads;
    const float scale = 1.0f / std::sqrt(static_cast<float>(C::DH));
    launch_k(attention_tc_kernel<T, TO>, dim3(std::min(items, sms[dev])), dim3(C::THREADS), C::SMEM, s, map, att, B,
             heads, d, scale, mul, err);
}

// att = attention(qkv) in TO (T, or e4m3 of att * mul); map from qkv_map over at least B * 65 rows. rev: the
// boards in descending order, where the kernel supports it (the four-group kernel); the output is the same.
template <typename T, typename TO>
static void launch_attention(const CUtensorMap& map, TO* att, int B, int d, int heads, float mul, uint32_t* err,
                             cudaStream_t s, int mode_override = -2, int rev = 0)
{
    if (B < 1 || heads < 1 || d % heads) throw std::runtime_error("cudanet_b200: bad attention sizes");
    const int dh = d / heads;
    const int mode = mode_override != -2 ? mode_override : att_tc_mode();
    const int pick = mode >= 0 ? mode : 4;
    if (dh == 64 && pick == 4) launch_attention_tc4<T, TO>(map, att, B, d, heads, mul, err, s, rev);
    else if (dh == 64 && pick == 1) launch_attention_tc<T, TO>(map, att, B, d, heads, mul, err, s);
    else if (dh == 64) launch_attention_dh<T, TO, 64>(map, att, B, d, heads, mul, err, s);
    else if (dh == 32) launch_attention_dh<T, TO, 32>(map, att, B, d, heads, mul, err, s);
    else throw std::runtime_error("cudanet_b200: head width must be 32 or 64");
}

// att_cls [B, d] = attention of the CLS query of every board (TO: T, or e4m3 of att * mul)
template <typename T, typename TO>
static void launch_attention_cls(const T* qkv, TO* att, int B, int d, int heads, float mul, cudaStream_t s)
{
    if (B < 1 || heads < 1 || d % heads) throw std::runtime_error("cudanet_b200: bad attention sizes");
    const int dh = d / heads;
    const dim3 grid((B * heads + 7) / 8), block(256);
    const float scale = 1.0f / std::sqrt(static_cast<float>(dh));
    if (dh == 64) launch_k(attention_cls_kernel<T, TO, 64>, grid, block, 0, s, qkv, att, B, heads, d, scale, mul);
    else if (dh == 32) launch_k(attention_cls_kernel<T, TO, 32>, grid, block, 0, s, qkv, att, B, heads, d, scale, mul);
    else throw std::runtime_error("cudanet_b200: head width must be 32 or 64");
}

// ------------------------------------------------------------------------------------------------ weights
struct Arch {
    int d = 0, layers = 0, heads = 0, ff = 0, tokens = 0, moves = 0;
};

// F16 and BF16 run every product in that type; E4M3 runs the four layer products on e4m3 operands (the heads
// and every 16-bit activation in bf16).
enum class Prec { F16, BF16, E4M3 };

struct TensorEntry {
    std::string dtype;
    std::vector<long long> shape;
    size_t offset = 0, nbytes = 0;
};

// The FP8 products of one layer: per product (qkv, out, ff1, ff2) the offset of its column scales in
// Weights::colscale (input scale x weight scale of each output channel) and the reciprocal of its input scale.
struct F8Layer {
    size_t cs[4];
    float inv_in[4];
};

// The weight file (mayfly/chess/cudanet/cudanet_spec.h:35-55; version 2 adds bf16 and e4m3 matrices), parsed,
// checked (magic, version, numbers, every tensor with its dtype, shape, offset and size) and uploaded in one
// device allocation (cudanet/weights.cpp:264 is the reference's reader).
struct Weights {
    Arch a;
    Prec prec = Prec::BF16;
    std::string fingerprint, source;
    void* base = nullptr;
    size_t bytes = 0;
    std::map<std::string, TensorEntry> t;
    float* colscale = nullptr;      // e4m3 files: every product's column scales, one device allocation
    std::vector<F8Layer> f8;

    ~Weights()
    {
        if (base) cudaFree(base);
        if (colscale) cudaFree(colscale);
    }

    [[noreturn]] static void fail(const std::string& path, const std::string& why)
    {
        throw std::runtime_error("cudanet_b200 weights " + path + ": " + why);
    }

    static int whole(const std::string& path, const JVal* v, const char* what)
    {
        if (!v || v->kind != JVal::Num || v->num != std::floor(v->num)) fail(path, std::string("no integer ") + what);
        return static_cast<int>(v->num);
    }

    void load(const std::string& path)
    {
        std::ifstream f(path, std::ios::binary);
        if (!f) fail(path, "cannot open");
        std::vector<char> raw((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
        if (raw.size() < 12 || std::memcmp(raw.data(), "MFCNW001", 8) != 0) fail(path, "bad magic (not MFCNW001)");
        uint32_t n = 0;
        std::memcpy(&n, raw.data() + 8, 4);
        if (12ull + n > raw.size()) fail(path, "header runs past the end");
        const std::string js(raw.data() + 12, n);
        const JVal h = JParser(js).parse();
        const int version = whole(path, h.get("version"), "version");
        if (version != 1 && version != 2) fail(path, "unknown version (this reader knows 1 and 2)");
        a.d = whole(path, h.get("d"), "d");
        a.layers = whole(path, h.get("layers"), "layers");
        a.heads = whole(path, h.get("heads"), "heads");
        a.ff = whole(path, h.get("ff"), "ff");
        a.tokens = whole(path, h.get("tokens"), "tokens");
        a.moves = whole(path, h.get("moves"), "moves");
        if (const JVal* fp = h.get("fingerprint")) fingerprint = fp->str;
        if (const JVal* src = h.get("source")) source = src->str;
        std::string prec_name = version == 1 ? "f16" : "bf16";
        if (const JVal* p = h.get("precision")) prec_name = p->str;
        if (prec_name == "f16") prec = Prec::F16;
        else if (prec_name == "bf16") prec = Prec::BF16;
        else if (prec_name == "e4m3") prec = Prec::E4M3;
        else fail(path, "precision " + prec_name + " is not supported by this build (f16, bf16, e4m3)");
        check_arch(path);

        const JVal* ts = h.get("tensors");
        if (!ts || ts->kind != JVal::Arr) fail(path, "no tensor list");
        const size_t start = (12ull + n + 255) / 256 * 256;
        size_t end = 0;
        for (const JVal& e : ts->arr) {
            const JVal* nm = e.get("name");
            if (!nm || nm->kind != JVal::Str) fail(path, "a tensor without a name");
            TensorEntry te;
            const JVal* dt = e.get("dtype");
            te.dtype = dt ? dt->str : "";
            const JVal* sh = e.get("shape");
            if (!sh || sh->kind != JVal::Arr) fail(path, nm->str + ": no shape");
            size_t count = 1;
            for (const JVal& s : sh->arr) {
                if (s.kind != JVal::Num || s.num < 0) fail(path, nm->str + ": bad shape");
                te.shape.push_back(static_cast<long long>(s.num));
                count *= static_cast<size_t>(s.num);
            }
            const JVal* off = e.get("offset");
            const JVal* nb = e.get("nbytes");
            if (!off || !nb) fail(path, nm->str + ": no offset or nbytes");
            te.offset = static_cast<size_t>(off->num);
            te.nbytes = static_cast<size_t>(nb->num);
            size_t es = 0;
            if (te.dtype == "f16" || te.dtype == "bf16") es = 2;
            else if (te.dtype == "f32") es = 4;
            else if (te.dtype == "e4m3") es = 1;
            else fail(path, nm->str + ": dtype " + te.dtype + " (f16, bf16, e4m3 or f32 only)");
            if (te.offset % 256) fail(path, nm->str + ": offset not 256-aligned");
            if (te.nbytes != count * es) fail(path, nm->str + ": nbytes does not match dtype and shape");
            if (start + te.offset + te.nbytes > raw.size()) fail(path, nm->str + ": runs past the end of the file");
            end = std::max(end, te.offset + te.nbytes);
            t[nm->str] = te;
        }
        check_tensors(path);
        bytes = (end + 255) / 256 * 256;
        RT(cudaMalloc(&base, bytes));
        RT(cudaMemcpy(base, raw.data() + start, std::min(bytes, raw.size() - start), cudaMemcpyHostToDevice));
        if (prec == Prec::E4M3) derive_f8(path, raw, start);
    }

    // e4m3 files: W[o, :] ~= w_scale[o] * e4m3 and a product's input x ~= act_scale * e4m3 (static, per layer
    // and product), so a product's f32 accumulator times act_scale * w_scale[o] is its value in column o.
    void derive_f8(const std::string& path, const std::vector<char>& raw, size_t start)
    {
        auto host = [&](const std::string& name) {
            const TensorEntry& e = t.at(name);
            std::vector<float> v(e.nbytes / 4);
            std::memcpy(v.data(), raw.data() + start + e.offset, e.nbytes);
            for (float x : v)
                if (!(x > 0.f) || !std::isfinite(x)) fail(path, name + ": scales must be positive and finite");
            return v;
        };
        static const char* const kMat[4] = {"qkv_w", "out_w", "ff1_w", "ff2_w"};
        std::vector<float> all;
        for (int i = 0; i < a.layers; ++i) {
            const std::string p = "L" + std::to_string(i) + ".";
            const std::vector<float> act = host(p + "act_scale");
            F8Layer fl;
            for (int j = 0; j < 4; ++j) {
                const std::vector<float> ws = host(p + kMat[j] + "_scale");
                fl.cs[j] = all.size();
                for (float w : ws) all.push_back(act[static_cast<size_t>(j)] * w);
                while (all.size() % 64) all.push_back(0.f);   // every product's scales 256-byte aligned
                fl.inv_in[j] = 1.0f / act[static_cast<size_t>(j)];
            }
            f8.push_back(fl);
        }
        RT(cudaMalloc(&colscale, all.size() * 4));
        RT(cudaMemcpy(colscale, all.data(), all.size() * 4, cudaMemcpyHostToDevice));
    }

    void check_arch(const std::string& path) const
    {
        char msg[256];
        std::snprintf(msg, sizeof msg, "d=%d layers=%d heads=%d ff=%d tokens=%d moves=%d", a.d, a.layers, a.heads,
                      a.ff, a.tokens, a.moves);
        const bool ok = (a.d == 256 || a.d == 512 || a.d == 1024) && a.layers >= 1 && a.heads >= 1 &&
                        a.d % a.heads == 0 && (a.d / a.heads == 32 || a.d / a.heads == 64) && a.ff >= 64 &&
                        a.ff % 64 == 0 && a.tokens == kTokens && a.moves >= 1;
        if (!ok)
            fail(path, std::string(msg) +
                           ": this build needs d in {256, 512, 1024}, head width 32 or 64, ff a multiple of 64 and "
                           "65 tokens");
    }

    void check_tensors(const std::string& path) const
    {
        const std::string m16 = prec == Prec::F16 ? "f16" : "bf16";
        const std::string mat = prec == Prec::E4M3 ? "e4m3" : m16;   // the layers' four matrices
        const long long d = a.d, ff = a.ff, mv = a.moves;
        std::vector<std::pair<std::string, std::pair<std::string, std::vector<long long>>>> want = {
            {"piece", {"f32", {13, d}}}, {"pos", {"f32", {64, d}}},   {"cls", {"f32", {d}}},
            {"cast_w", {"f32", {d, 4}}}, {"cast_b", {"f32", {d}}},    {"hm", {"f32", {102, d}}},
            {"ep_mark", {"f32", {d}}},   {"ln_g", {"f32", {d}}},      {"ln_b", {"f32", {d}}},
            {"heads_w", {m16, {2 * mv, d}}}, {"heads_b", {"f32", {2 * mv}}}};
        for (int i = 0; i < a.layers; ++i) {
            const std::string p = "L" + std::to_string(i) + ".";
            want.push_back({p + "n1_g", {"f32", {d}}});
            want.push_back({p + "n1_b", {"f32", {d}}});
            want.push_back({p + "qkv_w", {mat, {3 * d, d}}});
            want.push_back({p + "qkv_b", {"f32", {3 * d}}});
            want.push_back({p + "out_w", {mat, {d, d}}});
            want.push_back({p + "out_b", {"f32", {d}}});
            want.push_back({p + "n2_g", {"f32", {d}}});
            want.push_back({p + "n2_b", {"f32", {d}}});
            want.push_back({p + "ff1_w", {mat, {ff, d}}});
            want.push_back({p + "ff1_b", {"f32", {ff}}});
            want.push_back({p + "ff2_w", {mat, {d, ff}}});
            want.push_back({p + "ff2_b", {"f32", {d}}});
            if (prec == Prec::E4M3) {
                want.push_back({p + "qkv_w_scale", {"f32", {3 * d}}});
                want.push_back({p + "out_w_scale", {"f32", {d}}});
                want.push_back({p + "ff1_w_scale", {"f32", {ff}}});
                want.push_back({p + "ff2_w_scale", {"f32", {d}}});
                want.push_back({p + "act_scale", {"f32", {4}}});   // inputs of qkv, out, ff1, ff2
            }
        }
        for (const auto& w : want) {
            auto it = t.find(w.first);
            if (it == t.end()) fail(path, w.first + " missing");
            if (it->second.dtype != w.second.first) fail(path, w.first + ": dtype " + it->second.dtype + ", needs " + w.second.first);
            if (it->second.shape != w.second.second) fail(path, w.first + ": shape differs from the architecture");
        }
    }

    template <typename P = void> const P* ptr(const std::string& name) const
    {
        auto it = t.find(name);
        if (it == t.end()) throw std::runtime_error("cudanet_b200 weights: no tensor named " + name);
        return reinterpret_cast<const P*>(static_cast<const char*>(base) + it->second.offset);
    }
};

// ------------------------------------------------------------------------------------------------ the net
constexpr int kMaxWide = 256;              // widest I / M row (chess has at most 218 legal moves)
constexpr int kDefaultMaxBatch = 1024;
constexpr int kMaxBatchLimit = 16384;
constexpr size_t kOutHeader = 256;         // the error word, then the outputs at this offset

enum ProfOp { kPEmbed, kPLn1, kPQkv, kPAtt, kPOut, kPLn2, kPFf1, kPGelu, kPFf2, kPCls, kPHeads, kProfOps };
static const char* const kProfNames = "embed,ln1,qkv,attention,out,ln2,ff1,gelu,ff2,cls_ln,heads,graph_pass";

struct InLayout {
    size_t ids, hm, ep, cast, I, M, total;
};

// Offsets of the inputs in the staging block: ids, hm, ep and cast depend on B alone, so a graph per B stays
// valid whatever wide is (cudanet/cudanet.cpp:107-119 in_layout).
static InLayout in_layout(int B, int wide)
{
    const size_t b = static_cast<size_t>(B), w = static_cast<size_t>(wide);
    InLayout l;
    l.ids = 0;
    l.hm = l.ids + 8 * b * 64;
    l.ep = l.hm + 8 * b;
    l.cast = l.ep + 8 * b;
    l.I = l.cast + 4 * b * 4;
    l.M = l.I + 8 * b * w;
    l.total = l.M + b * w;
    return l;
}

struct LayerW {
    const float *n1_g, *n1_b, *qkv_b, *out_b, *n2_g, *n2_b, *ff1_b, *ff2_b;
    const void *qkv_w, *out_w, *ff1_w, *ff2_w;
    // e4m3 files: the products' column scales and the reciprocals of their static input scales
    const float *qkv_cs = nullptr, *out_cs = nullptr, *ff1_cs = nullptr, *ff2_cs = nullptr;
    float inv_qkv = 1.f, inv_out = 1.f, inv_ff1 = 1.f, inv_ff2 = 1.f;
};

class Net {
public:
    Net(const std::string& path, int device) { init(path, device); }
    ~Net() { release(); }

    std::mutex mu;

    int max_batch() const { return max_batch_; }
    const std::string& fingerprint() const { return w_.fingerprint; }
    const char* precision() const
    {
        return w_.prec == Prec::F16 ? "f16" : w_.prec == Prec::BF16 ? "bf16" : "e4m3";
    }

    void begin(int B, int wide, const int64_t* ids, const float* cast, const int64_t* hm, const int64_t* ep,
               const int64_t* I, const uint8_t* M, bool queued, bool want_logits);
    // begin from transposition keys: the keys cross PCIe and encode_keys_kernel fills the input slots
    void begin_keys(int B, int wide, const uint64_t* keys, const int64_t* ep_sq, const int64_t* clock,
                    const int64_t* I, const uint8_t* M, bool queued, bool want_logits);
    void end(float* pol, float* val, float* qv, float* logits);
    void evaluate_device(int B, int wide, const int64_t* ids, const float* cast, const int64_t* hm,
                         const int64_t* ep, const int64_t* I, const uint8_t* M, float* pol, float* val, float* qv,
                         cudaStream_t s);
    void check(cudaStream_t s);
    std::vector<double> profile(int B, int reps);
    std::vector<float> calibrate(int B, const int64_t* ids, const float* cast, const int64_t* hm, const int64_t* ep);

private:
    int device_ = 0;
    int max_batch_ = 0;
    int num_sms_ = 148;
    Weights w_;
    std::vector<LayerW> L_;
    size_t rows_pad_ = 0, cls_pad_ = 0;
    float* x_ = nullptr;
    void *h_ = nullptr, *qkv_ = nullptr, *att_ = nullptr, *ff_ = nullptr, *cls_ = nullptr;
    float* logits_ = nullptr;
    uint8_t* d_in_ = nullptr;
    uint8_t* d_out_ = nullptr;
    uint8_t* h_in_[2] = {nullptr, nullptr};
    uint8_t* h_out_[2] = {nullptr, nullptr};
    float* h_logits_[2] = {nullptr, nullptr};
    cudaStream_t stream_ = nullptr;
    cudaEvent_t done_[2] = {nullptr, nullptr};
    std::map<int, cudaGraphExec_t> graphs_;
    bool use_graph_ = true;
    CUtensorMap map_h_, map_att_, map_ff_, map_cls_, map_qkv_;
    std::map<std::pair<const void*, int>, CUtensorMap> wmaps_;
    std::map<std::tuple<const void*, int, int, int, int>, CUtensorMap> omaps_;   // (out, epi + 16 f8, M, N, ldc)

    struct Fly {
        int B, wide, slot;
        bool queued, logits;
    };
    size_t key_off_ = 0;   // the key block (96 bytes a board) in the staging buffers, after the encoded inputs
    int begin_checks(int B, int wide, bool queued);
    void begin_run(int B, int wide, int slot, bool queued, bool want_logits);
    Fly fly_[2];
    int fly_n_ = 0;

    // calibration: while set, the 16-bit pass records max |.| of the four products' inputs per layer here
    unsigned int* amax_ = nullptr;

    int att_mode_ = -1;   // MAYFLY_CUDANET_ATT_TC when the handle was made (-1: the evaluator's choice)
    bool alt_order_ = true;   // alternate the row order along the kernel chain (MAYFLY_CUDANET_ORDER=fwd: off)
    std::set<int> no_graph_;   // batch sizes whose capture failed: run eagerly

    // profiling marks
    bool prof_on_ = false;
    std::vector<cudaEvent_t> prof_ev_;
    std::vector<int> prof_op_;
    size_t prof_n_ = 0;

    uint32_t* err_word() const { return reinterpret_cast<uint32_t*>(d_out_); }
    bool bf16() const { return w_.prec != Prec::F16; }   // the 16-bit type is bf16 (also in e4m3 files)
    bool f8() const { return w_.prec == Prec::E4M3; }

    void init(const std::string& path, int device);
    void release();
    const CUtensorMap& wmap(const void* W, MapType type, int N, int K, int bn);
    // out = epilogue(A W^T); W is e4m3 when w_f8 (A then is too, and ep carries the column scales)
    void gemm(int epi, const CUtensorMap& ma, const void* W, bool w_f8, int M, int N, int K, const EpiArgs& ep,
              void* out, int ldc, cudaStream_t s);
    void amax(int slot, const void* p, size_t n, cudaStream_t s);
    void forward_f8(int B, cudaStream_t s);
    // x += A W^T + bias, then h = LN(x; g, b), in one cluster kernel (gemm_ln.cuh)
    void gemm_resln(const CUtensorMap& ma, const void* W, int M, int K, const float* bias, const float* g,
                    const float* b, cudaStream_t s);
    void forward_kernels(int B, cudaStream_t s);
    void forward(int B, cudaStream_t s);
    void capture(int B);
    void mark(int op, cudaStream_t s);
    void check_batch(int B) const
    {
        if (B >= 1 && B <= max_batch_) return;
        std::string msg = "cudanet_b200: batch size " + std::to_string(B) + " outside 1.." + std::to_string(max_batch_);
        if (B > max_batch_ && max_batch_ < kMaxBatchLimit) msg += " (env MAYFLY_CUDANET_MAX_BATCH sets the limit)";
        throw std::runtime_error(msg);
    }
    template <typename T> void forward_t(int B, cudaStream_t s);
};

static int pick_max_batch()
{
    const char* e = std::getenv("MAYFLY_CUDANET_MAX_BATCH");
    if (!e || !*e) return kDefaultMaxBatch;
    char* end = nullptr;
    const long v = std::strtol(e, &end, 10);
    if (*end || v < 1 || v > kMaxBatchLimit)
        throw std::runtime_error(std::string("cudanet_b200: MAYFLY_CUDANET_MAX_BATCH=") + e + " is not in 1.." +
                                 std::to_string(kMaxBatchLimit));
    return static_cast<int>(v);
}

void Net::init(const std::string& path, int device)
{
    device_ = device;
    max_batch_ = pick_max_batch();
    int ndev = 0;
    RT(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev)
        throw std::runtime_error("cudanet_b200: device " + std::to_string(device) + " not present (" +
                                 std::to_string(ndev) + " devices)");
    RT(cudaSetDevice(device_));
    cudaDeviceProp prop;
    RT(cudaGetDeviceProperties(&prop, device_));
    if (prop.major != 10)
        throw std::runtime_error(std::string("cudanet_b200: device ") + prop.name + " is sm_" +
                                 std::to_string(prop.major) + std::to_string(prop.minor) +
                                 "; this library is built for sm_100a (B200)");
    num_sms_ = prop.multiProcessorCount;
    try {
        w_.load(path);
        const Arch& a = w_.a;
        for (int i = 0; i < a.layers; ++i) {
            const std::string p = "L" + std::to_string(i) + ".";
            LayerW l;
            l.n1_g = w_.ptr<float>(p + "n1_g");
            l.n1_b = w_.ptr<float>(p + "n1_b");
            l.qkv_w = w_.ptr(p + "qkv_w");
            l.qkv_b = w_.ptr<float>(p + "qkv_b");
            l.out_w = w_.ptr(p + "out_w");
            l.out_b = w_.ptr<float>(p + "out_b");
            l.n2_g = w_.ptr<float>(p + "n2_g");
            l.n2_b = w_.ptr<float>(p + "n2_b");
            l.ff1_w = w_.ptr(p + "ff1_w");
            l.ff1_b = w_.ptr<float>(p + "ff1_b");
            l.ff2_w = w_.ptr(p + "ff2_w");
            l.ff2_b = w_.ptr<float>(p + "ff2_b");
            if (f8()) {
                const F8Layer& f = w_.f8[static_cast<size_t>(i)];
                l.qkv_cs = w_.colscale + f.cs[0];
                l.out_cs = w_.colscale + f.cs[1];
                l.ff1_cs = w_.colscale + f.cs[2];
                l.ff2_cs = w_.colscale + f.cs[3];
                l.inv_qkv = f.inv_in[0];
                l.inv_out = f.inv_in[1];
                l.inv_ff1 = f.inv_in[2];
                l.inv_ff2 = f.inv_in[3];
            }
            L_.push_back(l);
        }
        const size_t d = a.d, ff = a.ff;
        rows_pad_ = (static_cast<size_t>(max_batch_) * kTokens + 127) / 128 * 128;
        cls_pad_ = (static_cast<size_t>(max_batch_) + 127) / 128 * 128;
        RT(cudaMalloc(&x_, rows_pad_ * d * 4));
        RT(cudaMalloc(&h_, rows_pad_ * d * 2));
        RT(cudaMalloc(&qkv_, rows_pad_ * 3 * d * 2));
        RT(cudaMalloc(&att_, rows_pad_ * d * 2));
        RT(cudaMalloc(&ff_, rows_pad_ * ff * 2));
        RT(cudaMalloc(&cls_, cls_pad_ * d * 2));
        RT(cudaMalloc(&logits_, cls_pad_ * 2 * a.moves * 4));
        RT(cudaMemset(x_, 0, rows_pad_ * d * 4));
        RT(cudaMemset(h_, 0, rows_pad_ * d * 2));
        RT(cudaMemset(qkv_, 0, rows_pad_ * 3 * d * 2));
        RT(cudaMemset(att_, 0, rows_pad_ * d * 2));
        RT(cudaMemset(ff_, 0, rows_pad_ * ff * 2));
        RT(cudaMemset(cls_, 0, cls_pad_ * d * 2));
        key_off_ = (in_layout(max_batch_, kMaxWide).total + 255) & ~size_t(255);
        const size_t in_bytes = key_off_ + 96 * static_cast<size_t>(max_batch_);
        const size_t out_bytes = kOutHeader + 4 * static_cast<size_t>(max_batch_) * (2 * kMaxWide + 1);
        RT(cudaMalloc(&d_in_, in_bytes));
        RT(cudaMalloc(&d_out_, out_bytes));
        RT(cudaMemset(d_in_, 0, in_bytes));
        RT(cudaMemset(d_out_, 0, out_bytes));
        for (int s = 0; s < 2; ++s) {
            RT(cudaMallocHost(&h_in_[s], in_bytes));
            RT(cudaMallocHost(&h_out_[s], out_bytes));
            RT(cudaMallocHost(&h_logits_[s], static_cast<size_t>(max_batch_) * 2 * a.moves * 4));
            RT(cudaEventCreateWithFlags(&done_[s], cudaEventDisableTiming));
        }
        RT(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        // the products' activation inputs: 16-bit, or e4m3 (the same buffers, 1 byte an element)
        const MapType act = f8() ? MapType::U8 : type16(bf16());
        map_h_ = operand_map(h_, act, d, rows_pad_, 128);
        map_att_ = operand_map(att_, act, d, rows_pad_, 128);
        map_ff_ = operand_map(ff_, act, ff, rows_pad_, 128);
        map_cls_ = operand_map(cls_, type16(bf16()), d, cls_pad_, 128);
        map_qkv_ = qkv_map(qkv_, bf16(), static_cast<int>(rows_pad_), a.d, a.heads);
        const char* g = std::getenv("MAYFLY_CUDANET_GRAPH");
        use_graph_ = !(g && std::strcmp(g, "0") == 0);
        att_mode_ = att_tc_env();
        {
            const char* e = std::getenv("MAYFLY_CUDANET_ORDER");
            alt_order_ = !(e && std::strcmp(e, "fwd") == 0);
        }
        RT(cudaStreamSynchronize(stream_));
    } catch (...) {
        release();
        throw;
    }
}

void Net::release()
{
    cudaSetDevice(device_);
    if (stream_) cudaStreamSynchronize(stream_);
    for (auto& kv : graphs_) cudaGraphExecDestroy(kv.second);
    graphs_.clear();
    for (cudaEvent_t e : prof_ev_) cudaEventDestroy(e);
    prof_ev_.clear();
    void* dev[] = {x_, h_, qkv_, att_, ff_, cls_, logits_, d_in_, d_out_};
    for (void* p : dev)
        if (p) cudaFree(p);
    x_ = nullptr;
    h_ = qkv_ = att_ = ff_ = cls_ = nullptr;
    logits_ = nullptr;
    d_in_ = d_out_ = nullptr;
    for (int s = 0; s < 2; ++s) {
        if (h_in_[s]) cudaFreeHost(h_in_[s]);
        if (h_out_[s]) cudaFreeHost(h_out_[s]);
        if (h_logits_[s]) cudaFreeHost(h_logits_[s]);
        if (done_[s]) cudaEventDestroy(done_[s]);
        h_in_[s] = h_out_[s] = nullptr;
        h_logits_[s] = nullptr;
        done_[s] = nullptr;
    }
    if (stream_) cudaStreamDestroy(stream_);
    stream_ = nullptr;
}

const CUtensorMap& Net::wmap(const void* W, MapType type, int N, int K, int bn)
{
    const auto key = std::make_pair(W, bn);
    auto it = wmaps_.find(key);
    if (it != wmaps_.end()) return it->second;
    return wmaps_[key] = operand_map(W, type, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                     static_cast<uint32_t>(bn));
}

void Net::gemm(int epi, const CUtensorMap& ma, const void* W, bool w_f8, int M, int N, int K, const EpiArgs& ep,
               void* out, int ldc, cudaStream_t s)
{
    const int bn = pick_bn(M, N, K, epi, num_sms_);
    const CUtensorMap& mb = wmap(W, w_f8 ? MapType::U8 : type16(bf16()), N, K, static_cast<int>(w_box_rows(bn)));
    const auto okey = std::make_tuple(static_cast<const void*>(out), epi + (w_f8 ? 16 : 0), M, N, ldc);
    auto it = omaps_.find(okey);
    if (it == omaps_.end())
        it = omaps_.emplace(okey, output_map(out, epi, type16(bf16()), M, N, ldc, w_f8)).first;
    if (w_f8)
        launch_gemm<__nv_fp8_e4m3, __nv_bfloat16>(epi, bn, ma, mb, it->second, M, N, K, ep, err_word(), num_sms_, s);
    else if (bf16())
        launch_gemm<__nv_bfloat16, __nv_bfloat16>(epi, bn, ma, mb, it->second, M, N, K, ep, err_word(), num_sms_, s);
    else
        launch_gemm<__half, __half>(epi, bn, ma, mb, it->second, M, N, K, ep, err_word(), num_sms_, s);
}

void Net::amax(int slot, const void* p, size_t n, cudaStream_t s)
{
    if (!amax_) return;
    if (bf16())
        launch_k(absmax_kernel<__nv_bfloat16>, dim3(4 * num_sms_), dim3(256), 0, s,
                 static_cast<const __nv_bfloat16*>(p), n, amax_ + slot);
    else
        launch_k(absmax_kernel<__half>, dim3(4 * num_sms_), dim3(256), 0, s, static_cast<const __half*>(p), n,
                 amax_ + slot);
}

void Net::gemm_resln(const CUtensorMap& ma, const void* W, int M, int K, const float* bias, const float* g,
                     const float* b, cudaStream_t s)
{
    const int d = w_.a.d;
    const CUtensorMap& mb = wmap(W, type16(bf16()), d, K, 256);
    const auto xkey = std::make_tuple(static_cast<const void*>(x_), static_cast<int>(kEpiResidual), M, d, d);
    auto ix = omaps_.find(xkey);
    if (ix == omaps_.end()) ix = omaps_.emplace(xkey, output_map(x_, kEpiResidual, type16(bf16()), M, d, d)).first;
    const auto hkey = std::make_tuple(static_cast<const void*>(h_), static_cast<int>(kEpiBias), M, d, d);
    auto ih = omaps_.find(hkey);
    if (ih == omaps_.end()) ih = omaps_.emplace(hkey, output_map(h_, kEpiBias, type16(bf16()), M, d, d)).first;
    if (bf16())
        launch_gemm_resln<__nv_bfloat16>(ma, mb, ix->second, ih->second, M, d, K, bias, g, b, err_word(), s);
    else
        launch_gemm_resln<__half>(ma, mb, ix->second, ih->second, M, d, K, bias, g, b, err_word(), s);
}

// MAYFLY_CUDANET_FUSE_LN=1 fuses each LayerNorm into the residual product before it (gemm_ln.cuh). Off by
// default: on a B200 the fused kernels' epilogues (a whole-row statistics exchange per tile) cost more than the
// separate LayerNorm passes they save (measured 23.1 vs 22.3 ms per 1,024-position pass).
static bool fuse_ln()
{
    static bool on = [] {
        const char* e = std::getenv("MAYFLY_CUDANET_FUSE_LN");
        return e && std::strcmp(e, "1") == 0;
    }();
    return on;
}

// The heads read the CLS row alone (chess_net.py:194), so after the last layer's qkv product the pass computes
// the CLS rows only: attention for the CLS query, then out, LN2 and the FFN on B rows (the residual stream's
// CLS rows through a 65-row pitch). Exact; MAYFLY_CUDANET_CLS_ONLY=0 runs the whole last layer instead.
static bool cls_only()
{
    static bool on = [] {
        const char* e = std::getenv("MAYFLY_CUDANET_CLS_ONLY");
        return !(e && std::strcmp(e, "0") == 0);
    }();
    return on;
}

void Net::mark(int op, cudaStream_t s)
{
    if (!prof_on_) return;
    if (prof_n_ >= prof_ev_.size()) {
        cudaEvent_t e;
        RT(cudaEventCreate(&e));
        prof_ev_.push_back(e);
        prof_op_.push_back(0);
    }
    RT(cudaEventRecord(prof_ev_[prof_n_], s));
    prof_op_[prof_n_] = op;
    ++prof_n_;
}

// The embedding fused with layer 0's first LayerNorm: x (XT: f32, or bf16) and h (T: 16-bit, or e4m3 of h * mul).
template <typename T, typename XT = float>
static void launch_embed_ln(const Weights& w, const LayerW& l0, const uint8_t* d_in, int B, XT* x, T* h,
                            float mul, cudaStream_t s)
{
    const int rows = B * kTokens;
    const InLayout lay = in_layout(B, 1);
    const int64_t* ids = reinterpret_cast<const int64_t*>(d_in + lay.ids);
    const int64_t* hm = reinterpret_cast<const int64_t*>(d_in + lay.hm);
    const int64_t* ep = reinterpret_cast<const int64_t*>(d_in + lay.ep);
    const float* cast = reinterpret_cast<const float*>(d_in + lay.cast);
    const dim3 grid((rows + 7) / 8), block(256);
    const float *piece = w.ptr<float>("piece"), *pos = w.ptr<float>("pos"), *cls = w.ptr<float>("cls"),
                *cast_w = w.ptr<float>("cast_w"), *cast_b = w.ptr<float>("cast_b"), *hm_emb = w.ptr<float>("hm"),
                *ep_mark = w.ptr<float>("ep_mark");
    switch (w.a.d) {
        case 256:
            launch_k(embed_ln_kernel<T, 2, XT>, grid, block, 0, s, ids, cast, hm, ep, piece, pos, cls, cast_w, cast_b,
                     hm_emb, ep_mark, l0.n1_g, l0.n1_b, x, h, rows, 1e-5f, mul);
            break;
        case 512:
            launch_k(embed_ln_kernel<T, 4, XT>, grid, block, 0, s, ids, cast, hm, ep, piece, pos, cls, cast_w, cast_b,
                     hm_emb, ep_mark, l0.n1_g, l0.n1_b, x, h, rows, 1e-5f, mul);
            break;
        default:
            launch_k(embed_ln_kernel<T, 8, XT>, grid, block, 0, s, ids, cast, hm, ep, piece, pos, cls, cast_w, cast_b,
                     hm_emb, ep_mark, l0.n1_g, l0.n1_b, x, h, rows, 1e-5f, mul);
    }
    RT(cudaGetLastError());
}

template <typename T> void Net::forward_t(int B, cudaStream_t s)
{
    const Arch& a = w_.a;
    const int rows = B * kTokens, d = a.d, ff = a.ff;
    const size_t nd = static_cast<size_t>(rows) * d, nf = static_cast<size_t>(rows) * ff;
    T* h = static_cast<T*>(h_);
    mark(kPEmbed, s);
    launch_embed_ln<T>(w_, L_[0], d_in_, B, x_, h, 1.f, s);
    const bool fuse = fuse_ln() && !amax_;
    // Each kernel of the chain walks its rows in the opposite order to the kernel that wrote its input, so it
    // starts on what is still in L2 (the producer's last rows); the outputs do not depend on the order.
    int dir = 0;
    auto flip = [&] { return alt_order_ ? (dir ^= 1) : 0; };
    for (int i = 0; i < a.layers; ++i) {
        const LayerW& l = L_[static_cast<size_t>(i)];
        const bool last = i + 1 == a.layers;
        mark(kPLn1, s);
        if (i > 0 && !fuse) launch_layernorm<T>(x_, l.n1_g, l.n1_b, h, rows, d, 1, 1.f, s, flip());
        amax(4 * i + 0, h, nd, s);
        mark(kPQkv, s);
        gemm(kEpiBias, map_h_, l.qkv_w, false, rows, 3 * d, d, EpiArgs{l.qkv_b, nullptr, 1.f, flip()}, qkv_, 3 * d,
             s);
        mark(kPAtt, s);
        if (last && cls_only() && !amax_) {
            // the CLS rows only (cls_only): dense [B, ...] operands in att_, h_, ff_; x's CLS rows at pitch 65 d
            const int xp = kTokens * d;
            launch_attention_cls<T, T>(static_cast<const T*>(qkv_), static_cast<T*>(att_), B, d, a.heads, 1.f, s);
            mark(kPOut, s);
            gemm(kEpiResidual, map_att_, l.out_w, false, B, d, d, EpiArgs{l.out_b, nullptr, 1.f}, x_, xp, s);
            mark(kPLn2, s);
            launch_layernorm<T>(x_, l.n2_g, l.n2_b, h, B, d, kTokens, 1.f, s);
            mark(kPFf1, s);
            gemm(kEpiBiasGelu, map_h_, l.ff1_w, false, B, ff, d, EpiArgs{l.ff1_b, nullptr, 1.f}, ff_, ff, s);
            mark(kPFf2, s);
            gemm(kEpiResidual, map_ff_, l.ff2_w, false, B, d, ff, EpiArgs{l.ff2_b, nullptr, 1.f}, x_, xp, s);
            continue;
        }
        launch_attention<T, T>(map_qkv_, static_cast<T*>(att_), B, d, a.heads, 1.f, err_word(), s, att_mode_,
                               flip());
        amax(4 * i + 1, att_, nd, s);
        mark(kPOut, s);
        if (fuse) {
            flip();
            gemm_resln(map_att_, l.out_w, rows, d, l.out_b, l.n2_g, l.n2_b, s);   // x += out; h = LN2(x)
        } else {
            gemm(kEpiResidual, map_att_, l.out_w, false, rows, d, d, EpiArgs{l.out_b, nullptr, 1.f, flip()}, x_, d,
                 s);
            mark(kPLn2, s);
            launch_layernorm<T>(x_, l.n2_g, l.n2_b, h, rows, d, 1, 1.f, s, flip());
        }
        amax(4 * i + 2, h, nd, s);
        mark(kPFf1, s);
        gemm(kEpiBiasGelu, map_h_, l.ff1_w, false, rows, ff, d, EpiArgs{l.ff1_b, nullptr, 1.f, flip()}, ff_, ff, s);
        amax(4 * i + 3, ff_, nf, s);
        mark(kPFf2, s);
        if (fuse && !last) {
            const LayerW& n = L_[static_cast<size_t>(i + 1)];
            flip();
            gemm_resln(map_ff_, l.ff2_w, rows, ff, l.ff2_b, n.n1_g, n.n1_b, s);   // x += ff; h = next LN1(x)
        } else {
            gemm(kEpiResidual, map_ff_, l.ff2_w, false, rows, d, ff, EpiArgs{l.ff2_b, nullptr, 1.f, flip()}, x_, d,
                 s);
        }
    }
    mark(kPCls, s);
    launch_layernorm<T>(x_, w_.ptr<float>("ln_g"), w_.ptr<float>("ln_b"), static_cast<T*>(cls_), B, d, kTokens, 1.f,
                        s);
    mark(kPHeads, s);
    gemm(kEpiF32, map_cls_, w_.ptr("heads_w"), false, B, 2 * a.moves, d,
         EpiArgs{w_.ptr<float>("heads_b"), nullptr, 1.f}, logits_, 2 * a.moves, s);
    mark(kPHeads, s);
}

// The FP8 pass: each layer product's input is written as e4m3 of x / act_scale by its producer (the
// LayerNorms, attention, ff1's GELU epilogue) and the product scales its f32 accumulator per column; q, k, v
// and the heads' input stay bf16, and so does the residual stream x (the FP8 configuration's bf16
// activations: the residual adds are f32 sums rounded once to bf16, and x is read and written at half the
// bytes of the 16-bit pass's f32 stream).
void Net::forward_f8(int B, cudaStream_t s)
{
    using T = __nv_bfloat16;
    using F8 = __nv_fp8_e4m3;
    const Arch& a = w_.a;
    const int rows = B * kTokens, d = a.d, ff = a.ff;
    F8* h = static_cast<F8*>(h_);
    T* x = reinterpret_cast<T*>(x_);
    mark(kPEmbed, s);
    launch_embed_ln<F8, T>(w_, L_[0], d_in_, B, x, h, L_[0].inv_qkv, s);
    int dir = 0;   // the row order of each kernel, opposite to its input's producer (as in forward_t)
    auto flip = [&] { return alt_order_ ? (dir ^= 1) : 0; };
    for (int i = 0; i < a.layers; ++i) {
        const LayerW& l = L_[static_cast<size_t>(i)];
        mark(kPLn1, s);
        if (i > 0) launch_layernorm<F8, T>(x, l.n1_g, l.n1_b, h, rows, d, 1, l.inv_qkv, s, flip());
        mark(kPQkv, s);
        gemm(kEpiBias, map_h_, l.qkv_w, true, rows, 3 * d, d, EpiArgs{l.qkv_b, l.qkv_cs, 1.f, flip()}, qkv_, 3 * d,
             s);
        mark(kPAtt, s);
        if (i + 1 == a.layers && cls_only()) {
            // the CLS rows only, as in forward_t
            const int xp = kTokens * d;
            launch_attention_cls<T, F8>(static_cast<const T*>(qkv_), static_cast<F8*>(att_), B, d, a.heads, l.inv_out,
                                        s);
            mark(kPOut, s);
            gemm(kEpiResidual16, map_att_, l.out_w, true, B, d, d, EpiArgs{l.out_b, l.out_cs, 1.f}, x, xp, s);
            mark(kPLn2, s);
            launch_layernorm<F8, T>(x, l.n2_g, l.n2_b, h, B, d, kTokens, l.inv_ff1, s);
            mark(kPFf1, s);
            gemm(kEpiGeluE4m3, map_h_, l.ff1_w, true, B, ff, d, EpiArgs{l.ff1_b, l.ff1_cs, l.inv_ff2}, ff_, ff, s);
            mark(kPFf2, s);
            gemm(kEpiResidual16, map_ff_, l.ff2_w, true, B, d, ff, EpiArgs{l.ff2_b, l.ff2_cs, 1.f}, x, xp, s);
            continue;
        }
        launch_attention<T, F8>(map_qkv_, static_cast<F8*>(att_), B, d, a.heads, l.inv_out, err_word(), s, att_mode_,
                                flip());
        mark(kPOut, s);
        gemm(kEpiResidual16, map_att_, l.out_w, true, rows, d, d, EpiArgs{l.out_b, l.out_cs, 1.f, flip()}, x, d, s);
        mark(kPLn2, s);
        launch_layernorm<F8, T>(x, l.n2_g, l.n2_b, h, rows, d, 1, l.inv_ff1, s, flip());
        mark(kPFf1, s);
        gemm(kEpiGeluE4m3, map_h_, l.ff1_w, true, rows, ff, d, EpiArgs{l.ff1_b, l.ff1_cs, l.inv_ff2, flip()}, ff_, ff,
             s);
        mark(kPFf2, s);
        gemm(kEpiResidual16, map_ff_, l.ff2_w, true, rows, d, ff, EpiArgs{l.ff2_b, l.ff2_cs, 1.f, flip()}, x, d, s);
    }
    mark(kPCls, s);
    launch_layernorm<T, T>(x, w_.ptr<float>("ln_g"), w_.ptr<float>("ln_b"), static_cast<T*>(cls_), B, d, kTokens, 1.f,
                           s);
    mark(kPHeads, s);
    gemm(kEpiF32, map_cls_, w_.ptr("heads_w"), false, B, 2 * a.moves, d,
         EpiArgs{w_.ptr<float>("heads_b"), nullptr, 1.f}, logits_, 2 * a.moves, s);
    mark(kPHeads, s);
}

void Net::forward_kernels(int B, cudaStream_t s)
{
    if (f8()) forward_f8(B, s);
    else if (bf16()) forward_t<__nv_bfloat16>(B, s);
    else forward_t<__half>(B, s);
}

void Net::capture(int B)
{
    RT(cudaStreamSynchronize(stream_));
    RT(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    cudaGraph_t g = nullptr;
    try {
        forward_kernels(B, stream_);
    } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    RT(cudaStreamEndCapture(stream_, &g));
    cudaGraphExec_t e = nullptr;
    const cudaError_t err = cudaGraphInstantiate(&e, g, 0);
    cudaGraphDestroy(g);
    check_rt(err, "cudaGraphInstantiate", __LINE__);
    graphs_[B] = e;
}

// The whole pass for B rows on stream s: the graph when there is one, else eager (the first use of B runs
// eager, which also makes every launch's one-time set-up happen outside a capture, then captures).
void Net::forward(int B, cudaStream_t s)
{
    auto it = graphs_.find(B);
    if (it != graphs_.end()) {
        RT(cudaGraphLaunch(it->second, s));
        return;
    }
    forward_kernels(B, s);
    if (!use_graph_ || no_graph_.count(B)) return;
    RT(cudaStreamSynchronize(s));
    try {
        capture(B);
    } catch (const std::exception& ex) {
        std::fprintf(stderr, "cudanet_b200: CUDA graph capture failed at B=%d, eager for this batch size: %.300s\n",
                     B, ex.what());
        no_graph_.insert(B);
        cudaGetLastError();
    }
}

// The checks every begin makes; returns the staging slot the batch takes.
int Net::begin_checks(int B, int wide, bool queued)
{
    check_batch(B);
    if (wide < 1 || wide > kMaxWide)
        throw std::runtime_error("cudanet_b200: wide " + std::to_string(wide) + " outside 1.." +
                                 std::to_string(kMaxWide));
    if (fly_n_ == 2) throw std::runtime_error("cudanet_b200: begin with two batches already in flight");
    if (fly_n_ && !queued) throw std::runtime_error("cudanet_b200: evaluate while a batch is in flight");
    return fly_n_ ? 1 - fly_[0].slot : 0;
}

void Net::begin(int B, int wide, const int64_t* ids, const float* cast, const int64_t* hm, const int64_t* ep,
                const int64_t* I, const uint8_t* M, bool queued, bool want_logits)
{
    if (!ids || !cast || !hm || !ep || !I || !M) throw std::runtime_error("cudanet_b200: a null input pointer");
    const int slot = begin_checks(B, wide, queued);
    RT(cudaSetDevice(device_));
    const size_t b = static_cast<size_t>(B), wd = static_cast<size_t>(wide);
    const InLayout lay = in_layout(B, wide);
    uint8_t* hin = h_in_[slot];
    std::memcpy(hin + lay.ids, ids, 8 * b * 64);
    std::memcpy(hin + lay.hm, hm, 8 * b);
    std::memcpy(hin + lay.ep, ep, 8 * b);
    std::memcpy(hin + lay.cast, cast, 4 * b * 4);
    std::memcpy(hin + lay.I, I, 8 * b * wd);
    std::memcpy(hin + lay.M, M, b * wd);
    RT(cudaMemcpyAsync(d_in_, hin, lay.total, cudaMemcpyHostToDevice, stream_));
    begin_run(B, wide, slot, queued, want_logits);
}

void Net::begin_keys(int B, int wide, const uint64_t* keys, const int64_t* ep_sq, const int64_t* clock,
                     const int64_t* I, const uint8_t* M, bool queued, bool want_logits)
{
    if (!keys || !ep_sq || !clock || !I || !M) throw std::runtime_error("cudanet_b200: a null input pointer");
    const int slot = begin_checks(B, wide, queued);
    RT(cudaSetDevice(device_));
    const size_t b = static_cast<size_t>(B), wd = static_cast<size_t>(wide);
    const InLayout lay = in_layout(B, wide);
    uint8_t* hin = h_in_[slot];
    std::memcpy(hin + key_off_, keys, 80 * b);
    std::memcpy(hin + key_off_ + 80 * b, ep_sq, 8 * b);
    std::memcpy(hin + key_off_ + 88 * b, clock, 8 * b);
    std::memcpy(hin + lay.I, I, 8 * b * wd);
    std::memcpy(hin + lay.M, M, b * wd);
    RT(cudaMemcpyAsync(d_in_ + key_off_, hin + key_off_, 96 * b, cudaMemcpyHostToDevice, stream_));
    RT(cudaMemcpyAsync(d_in_ + lay.I, hin + lay.I, lay.total - lay.I, cudaMemcpyHostToDevice, stream_));
    const uint8_t* kd = d_in_ + key_off_;
    launch_k(encode_keys_kernel, dim3((B + kEncodeBoardsPerBlock - 1) / kEncodeBoardsPerBlock),
             dim3(64 * kEncodeBoardsPerBlock), 0, stream_, reinterpret_cast<const uint64_t*>(kd),
             reinterpret_cast<const int64_t*>(kd + 80 * b), reinterpret_cast<const int64_t*>(kd + 88 * b), B,
             reinterpret_cast<int64_t*>(d_in_ + lay.ids), reinterpret_cast<float*>(d_in_ + lay.cast),
             reinterpret_cast<int64_t*>(d_in_ + lay.hm), reinterpret_cast<int64_t*>(d_in_ + lay.ep));
    begin_run(B, wide, slot, queued, want_logits);
}

// The pass, the search's reduction and the copies back, once the inputs are in d_in_ (stream order).
void Net::begin_run(int B, int wide, int slot, bool queued, bool want_logits)
{
    const size_t b = static_cast<size_t>(B), wd = static_cast<size_t>(wide);
    const InLayout lay = in_layout(B, wide);
    forward(B, stream_);
    const int64_t* I_d = reinterpret_cast<const int64_t*>(d_in_ + lay.I);
    const uint8_t* M_d = d_in_ + lay.M;
    float* pol_d = reinterpret_cast<float*>(d_out_ + kOutHeader);
    float* val_d = pol_d + b * wd;
    float* qv_d = val_d + b;
    launch_k(heads_post_kernel, dim3((B + 7) / 8), dim3(256), 0, stream_, static_cast<const float*>(logits_), I_d, M_d,
             B, wide, w_.a.moves, pol_d, val_d, qv_d);
    RT(cudaMemcpyAsync(h_out_[slot], d_out_, kOutHeader + 4 * b * (2 * wd + 1), cudaMemcpyDeviceToHost, stream_));
    if (want_logits)
        RT(cudaMemcpyAsync(h_logits_[slot], logits_, 4 * b * 2 * w_.a.moves, cudaMemcpyDeviceToHost, stream_));
    RT(cudaEventRecord(done_[slot], stream_));
    fly_[fly_n_++] = Fly{B, wide, slot, queued, want_logits};
}

void Net::end(float* pol, float* val, float* qv, float* logits)
{
    if (!fly_n_) throw std::runtime_error("cudanet_b200: end with no batch in flight");
    const Fly f = fly_[0];
    fly_[0] = fly_[1];
    fly_n_--;
    RT(cudaSetDevice(device_));
    RT(cudaEventSynchronize(done_[f.slot]));
    const uint8_t* hout = h_out_[f.slot];
    uint32_t errw = 0;
    std::memcpy(&errw, hout, 4);
    if (errw) {
        // the context is still usable: clear the word for the next batch and report this one as failed
        RT(cudaMemsetAsync(d_out_, 0, 4, stream_));
        RT(cudaStreamSynchronize(stream_));
        throw std::runtime_error(std::string("cudanet_b200: device error: ") + err_site_name(errw >> 8));
    }
    const size_t b = static_cast<size_t>(f.B), wd = static_cast<size_t>(f.wide);
    const float* o = reinterpret_cast<const float*>(hout + kOutHeader);
    if (pol) std::memcpy(pol, o, 4 * b * wd);
    if (val) std::memcpy(val, o + b * wd, 4 * b);
    if (qv) std::memcpy(qv, o + b * wd + b, 4 * b * wd);
    if (logits && f.logits) std::memcpy(logits, h_logits_[f.slot], 4 * b * 2 * w_.a.moves);
}

void Net::evaluate_device(int B, int wide, const int64_t* ids, const float* cast, const int64_t* hm,
                          const int64_t* ep, const int64_t* I, const uint8_t* M, float* pol, float* val, float* qv,
                          cudaStream_t s)
{
    check_batch(B);
    if (wide < 1 || wide > kMaxWide)
        throw std::runtime_error("cudanet_b200: wide " + std::to_string(wide) + " outside 1.." +
                                 std::to_string(kMaxWide));
    if (fly_n_) throw std::runtime_error("cudanet_b200: evaluate_device while a batch is in flight");
    RT(cudaSetDevice(device_));
    const size_t b = static_cast<size_t>(B);
    const InLayout lay = in_layout(B, 1);
    RT(cudaMemcpyAsync(d_in_ + lay.ids, ids, 8 * b * 64, cudaMemcpyDeviceToDevice, s));
    RT(cudaMemcpyAsync(d_in_ + lay.hm, hm, 8 * b, cudaMemcpyDeviceToDevice, s));
    RT(cudaMemcpyAsync(d_in_ + lay.ep, ep, 8 * b, cudaMemcpyDeviceToDevice, s));
    RT(cudaMemcpyAsync(d_in_ + lay.cast, cast, 16 * b, cudaMemcpyDeviceToDevice, s));
    if (graphs_.find(B) == graphs_.end() && use_graph_) {
        // the first use of B: make the graph on the handle's stream, ordered after the copies above
        cudaEvent_t ev;
        RT(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
        RT(cudaEventRecord(ev, s));
        RT(cudaStreamWaitEvent(stream_, ev, 0));
        forward(B, stream_);
        RT(cudaEventRecord(ev, stream_));
        RT(cudaStreamWaitEvent(s, ev, 0));
        RT(cudaEventDestroy(ev));
    } else {
        forward(B, s);
    }
    launch_k(heads_post_kernel, dim3((B + 7) / 8), dim3(256), 0, s, static_cast<const float*>(logits_), I, M, B, wide,
             w_.a.moves, pol, val, qv);
}

void Net::check(cudaStream_t s)
{
    RT(cudaSetDevice(device_));
    if (s) RT(cudaStreamSynchronize(s));
    RT(cudaStreamSynchronize(stream_));
    RT(cudaDeviceSynchronize());
    uint32_t errw = 0;
    RT(cudaMemcpy(&errw, d_out_, 4, cudaMemcpyDeviceToHost));
    if (errw) {
        RT(cudaMemset(d_out_, 0, 4));
        throw std::runtime_error(std::string("cudanet_b200: device error: ") + err_site_name(errw >> 8));
    }
}

// Runs the 16-bit pass eagerly on B positions and returns, per layer, max |.| of the inputs of its four
// products (qkv, out, ff1, ff2): the ranges an e4m3 weight file's static input scales are set from.
std::vector<float> Net::calibrate(int B, const int64_t* ids, const float* cast, const int64_t* hm, const int64_t* ep)
{
    check_batch(B);
    if (!ids || !cast || !hm || !ep) throw std::runtime_error("cudanet_calibrate: a null input pointer");
    if (f8()) throw std::runtime_error("cudanet_calibrate: needs a 16-bit weight file (this one is e4m3)");
    if (fly_n_) throw std::runtime_error("cudanet_calibrate: a batch is in flight");
    RT(cudaSetDevice(device_));
    const size_t b = static_cast<size_t>(B);
    const InLayout lay = in_layout(B, 1);
    uint8_t* hin = h_in_[0];
    std::memcpy(hin + lay.ids, ids, 8 * b * 64);
    std::memcpy(hin + lay.hm, hm, 8 * b);
    std::memcpy(hin + lay.ep, ep, 8 * b);
    std::memcpy(hin + lay.cast, cast, 4 * b * 4);
    RT(cudaMemcpyAsync(d_in_, hin, lay.I, cudaMemcpyHostToDevice, stream_));
    const size_t n = 4 * static_cast<size_t>(w_.a.layers);
    RT(cudaMalloc(&amax_, n * sizeof(unsigned int)));
    std::vector<unsigned int> bits(n, 0);
    try {
        RT(cudaMemsetAsync(amax_, 0, n * sizeof(unsigned int), stream_));
        forward_kernels(B, stream_);
        RT(cudaMemcpyAsync(bits.data(), amax_, n * sizeof(unsigned int), cudaMemcpyDeviceToHost, stream_));
        RT(cudaStreamSynchronize(stream_));
    } catch (...) {
        cudaStreamSynchronize(stream_);
        cudaFree(amax_);
        amax_ = nullptr;
        throw;
    }
    cudaFree(amax_);
    amax_ = nullptr;
    check(nullptr);
    std::vector<float> out(n);
    std::memcpy(out.data(), bits.data(), n * sizeof(float));
    return out;
}

std::vector<double> Net::profile(int B, int reps)
{
    check_batch(B);
    if (reps < 1) reps = 1;
    if (fly_n_) throw std::runtime_error("cudanet_b200: profile while a batch is in flight");
    RT(cudaSetDevice(device_));
    // an empty board in every row: ids, hm, ep and cast all zero
    RT(cudaMemsetAsync(d_in_, 0, in_layout(B, 1).I, stream_));
    forward_kernels(B, stream_);   // warm-up
    std::vector<double> ms(kProfOps + 1, 0.0);
    for (int r = 0; r < reps; ++r) {
        prof_n_ = 0;
        prof_on_ = true;
        try {
            forward_kernels(B, stream_);
        } catch (...) {
            prof_on_ = false;
            throw;
        }
        prof_on_ = false;
        RT(cudaEventSynchronize(prof_ev_[prof_n_ - 1]));
        for (size_t i = 1; i < prof_n_; ++i) {
            float t = 0.f;
            RT(cudaEventElapsedTime(&t, prof_ev_[i - 1], prof_ev_[i]));
            ms[static_cast<size_t>(prof_op_[i - 1])] += t;
        }
    }
    forward(B, stream_);   // makes the graph if there is none yet
    cudaEvent_t e0, e1;
    RT(cudaEventCreate(&e0));
    RT(cudaEventCreate(&e1));
    for (int r = 0; r < reps; ++r) {
        RT(cudaEventRecord(e0, stream_));
        forward(B, stream_);
        RT(cudaEventRecord(e1, stream_));
        RT(cudaEventSynchronize(e1));
        float t = 0.f;
        RT(cudaEventElapsedTime(&t, e0, e1));
        ms[kProfOps] += t;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    for (double& v : ms) v /= reps;
    check(nullptr);
    return ms;
}

// ------------------------------------------------------------------------------------------------ C ABI glue
static void put(char* err, int err_len, const char* msg)
{
    if (!err || err_len <= 0) return;
    size_t n = std::strlen(msg);
    if (n > static_cast<size_t>(err_len - 1)) n = static_cast<size_t>(err_len - 1);
    std::memcpy(err, msg, n);
    err[n] = 0;
}

template <typename F> static int guarded(char* err, int err_len, const char* what, F&& fn)
{
    put(err, err_len, "");
    try {
        return fn();
    } catch (const std::exception& e) {
        put(err, err_len, e.what());
    } catch (...) {
        put(err, err_len, what);
    }
    return -1;
}

// ------------------------------------------------------------------------------------------------ no-alloc product
// Some callers cannot call cudaMalloc at all: a search thread that has reserved the whole GPU memory budget up
// front, or code that must not take the implicit device-wide synchronisation a cudaMalloc/cudaFree pair costs
// while other batches are in flight. cudanet_k_gemm allocates its device error word on every call, so they
// cannot use it. cudanet_k_gemm_noalloc runs the same product with that scratch in this file-scope array
// instead: 256 bytes on every GPU that loads the library, held until the process exits. A call uses the first
// 4-byte word (the kernel's bounded-wait error report), whatever M, N and K are.
constexpr size_t kNoAllocScratchBytes = 256;
constexpr size_t kNoAllocBytesPerCall = sizeof(uint32_t);
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocScratchBytes / sizeof(uint32_t)];

// The array's device address on the current device, looked up once per device (host code must not hand the
// symbol itself to a kernel: on the host it is only a stand-in for the device copy). The address belongs to the
// device's context as it was at the lookup: a process that resets a device (cudaDeviceReset) must not call the
// entry point on that device afterwards.
static uint32_t* noalloc_scratch(int dev)
{
    static std::mutex mu;
    static uint32_t* addr[64] = {};
    if (dev < 0 || dev >= 64) throw std::runtime_error("cudanet_k_gemm_noalloc: device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p)
            throw std::runtime_error(std::string("cudanet_k_gemm_noalloc: cudaGetSymbolAddress failed: ") +
                                     cudaGetErrorString(e));
        addr[dev] = static_cast<uint32_t*>(p);
    }
    return addr[dev];
}

// One attention launch of the unit-test entry points: its own error word, a map over exactly B * 65 rows.
template <typename T, typename TO>
static void attention_once(const void* qkv, void* att, int B, int d, int heads, float mul, cudaStream_t s,
                           const char* who, int kernel = -1)
{
    if (B < 1 || heads < 1 || d % heads) throw std::runtime_error(std::string(who) + ": bad sizes");
    if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(att)) & 15)
        throw std::runtime_error(std::string(who) + ": qkv and att must be 16-byte aligned");
    const CUtensorMap map = qkv_map(qkv, std::is_same<T, __nv_bfloat16>::value, B * kTokens, d, heads);
    uint32_t* errw = nullptr;
    RT(cudaMalloc(&errw, 4));
    RT(cudaMemset(errw, 0, 4));
    try {
        if (kernel >= 0 && d / heads != 64) throw std::runtime_error(std::string(who) + ": head width must be 64");
        if (kernel == 1) launch_attention_tc<T, TO>(map, static_cast<TO*>(att), B, d, heads, mul, errw, s);
        else if (kernel == 4) launch_attention_tc4<T, TO>(map, static_cast<TO*>(att), B, d, heads, mul, errw, s);
        else if (kernel == 0) launch_attention_dh<T, TO, 64>(map, static_cast<TO*>(att), B, d, heads, mul, errw, s);
        else if (kernel == -1) launch_attention<T, TO>(map, static_cast<TO*>(att), B, d, heads, mul, errw, s);
        else throw std::runtime_error(std::string(who) + ": kernel must be -1, 0, 1 or 4");
        RT(cudaStreamSynchronize(s));
    } catch (...) {
        cudaFree(errw);
        throw;
    }
    uint32_t e = 0;
    RT(cudaMemcpy(&e, errw, 4, cudaMemcpyDeviceToHost));
    cudaFree(errw);
    if (e) throw std::runtime_error(std::string(who) + ": device error: " + err_site_name(e >> 8));
}

}  // namespace mf

using mf::Net;

extern "C" {

CUDANET_API void* cudanet_create(const char* weights_path, int device, char* err, int err_len)
{
    mf::put(err, err_len, "");
    if (!weights_path) {
        mf::put(err, err_len, "cudanet_create: no weights path");
        return nullptr;
    }
    try {
        return new Net(std::string(weights_path), device);
    } catch (const std::exception& e) {
        mf::put(err, err_len, e.what());
    } catch (...) {
        mf::put(err, err_len, "cudanet_create: unknown exception");
    }
    return nullptr;
}

CUDANET_API int cudanet_evaluate(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                                 const int64_t* hm, const int64_t* ep, const int64_t* I, const uint8_t* M,
                                 float* pol, float* val, float* qv, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_evaluate: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_evaluate: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->begin(B, wide, ids, cast, hm, ep, I, M, false, false);
        n->end(pol, val, qv, nullptr);
        return 0;
    });
}

CUDANET_API int cudanet_evaluate_keys(void* handle, int B, int wide, const uint64_t* keys, const int64_t* ep_sq,
                                      const int64_t* clock, const int64_t* I, const uint8_t* M, float* pol,
                                      float* val, float* qv, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_evaluate_keys: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_evaluate_keys: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->begin_keys(B, wide, keys, ep_sq, clock, I, M, false, false);
        n->end(pol, val, qv, nullptr);
        return 0;
    });
}

CUDANET_API int cudanet_begin_keys(void* handle, int B, int wide, const uint64_t* keys, const int64_t* ep_sq,
                                   const int64_t* clock, const int64_t* I, const uint8_t* M, char* err,
                                   int err_len)
{
    return mf::guarded(err, err_len, "cudanet_begin_keys: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_begin_keys: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->begin_keys(B, wide, keys, ep_sq, clock, I, M, true, false);
        return 0;
    });
}

CUDANET_API int cudanet_encode_keys(const uint64_t* keys, const int64_t* ep_sq, const int64_t* clock, int B,
                                    int64_t* ids, float* cast, int64_t* hm, int64_t* ep, void* stream, char* err,
                                    int err_len)
{
    return mf::guarded(err, err_len, "cudanet_encode_keys: unknown exception", [&] {
        if (B < 0) throw std::runtime_error("cudanet_encode_keys: negative batch");
        if (B == 0) return 0;
        if (!keys || !ep_sq || !clock || !ids || !cast || !hm || !ep)
            throw std::runtime_error("cudanet_encode_keys: a null pointer");
        mf::launch_k(mf::encode_keys_kernel,
                     dim3(static_cast<unsigned>((B + mf::kEncodeBoardsPerBlock - 1) / mf::kEncodeBoardsPerBlock)),
                     dim3(64 * mf::kEncodeBoardsPerBlock), 0, static_cast<cudaStream_t>(stream), keys, ep_sq, clock,
                     B, ids, cast, hm, ep);
        return 0;
    });
}

CUDANET_API int cudanet_evaluate_logits(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                                        const int64_t* hm, const int64_t* ep, const int64_t* I,
                                        const uint8_t* M, float* pol, float* val, float* qv, float* logits,
                                        char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_evaluate_logits: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_evaluate_logits: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->begin(B, wide, ids, cast, hm, ep, I, M, false, true);
        n->end(pol, val, qv, logits);
        return 0;
    });
}

CUDANET_API int cudanet_begin(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                              const int64_t* hm, const int64_t* ep, const int64_t* I, const uint8_t* M, char* err,
                              int err_len)
{
    return mf::guarded(err, err_len, "cudanet_begin: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_begin: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->begin(B, wide, ids, cast, hm, ep, I, M, true, false);
        return 0;
    });
}

CUDANET_API int cudanet_end(void* handle, float* pol, float* val, float* qv, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_end: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_end: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->end(pol, val, qv, nullptr);
        return 0;
    });
}

CUDANET_API int cudanet_fingerprint(void* handle, char* buf, int buf_len)
{
    if (!handle) {
        mf::put(buf, buf_len, "");
        return -1;
    }
    const std::string& fp = static_cast<Net*>(handle)->fingerprint();
    mf::put(buf, buf_len, fp.c_str());
    return static_cast<int>(fp.size());
}

CUDANET_API int cudanet_max_batch(void* handle) { return handle ? static_cast<Net*>(handle)->max_batch() : -1; }

CUDANET_API int cudanet_precision(void* handle, char* buf, int buf_len)
{
    if (!handle) {
        mf::put(buf, buf_len, "");
        return -1;
    }
    const char* p = static_cast<Net*>(handle)->precision();
    mf::put(buf, buf_len, p);
    return static_cast<int>(std::strlen(p));
}

CUDANET_API int cudanet_profile(void* handle, int B, int reps, double* ms, int n, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_profile: unknown exception", [&] {
        if (!handle || !ms) throw std::runtime_error("cudanet_profile: null handle or output");
        Net* net = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(net->mu);
        const std::vector<double> got = net->profile(B, reps);
        const int k = static_cast<int>(got.size()) < n ? static_cast<int>(got.size()) : n;
        for (int i = 0; i < k; ++i) ms[i] = got[static_cast<size_t>(i)];
        return k;
    });
}

CUDANET_API int cudanet_profile_names(char* buf, int buf_len)
{
    mf::put(buf, buf_len, mf::kProfNames);
    return static_cast<int>(std::strlen(mf::kProfNames));
}

CUDANET_API void cudanet_destroy(void* handle)
{
    try {
        delete static_cast<Net*>(handle);
    } catch (...) {
    }
}

CUDANET_API int cudanet_evaluate_device(void* handle, int B, int wide, const int64_t* ids, const float* cast,
                                        const int64_t* hm, const int64_t* ep, const int64_t* I,
                                        const uint8_t* M, float* pol, float* val, float* qv, void* stream,
                                        char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_evaluate_device: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_evaluate_device: null handle");
        if (!ids || !cast || !hm || !ep || !I || !M || !pol || !val || !qv)
            throw std::runtime_error("cudanet_evaluate_device: a null pointer");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->evaluate_device(B, wide, ids, cast, hm, ep, I, M, pol, val, qv, static_cast<cudaStream_t>(stream));
        return 0;
    });
}

CUDANET_API int cudanet_check(void* handle, void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_check: unknown exception", [&] {
        if (!handle) throw std::runtime_error("cudanet_check: null handle");
        Net* n = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(n->mu);
        n->check(static_cast<cudaStream_t>(stream));
        return 0;
    });
}

CUDANET_API int cudanet_calibrate(void* handle, int B, const int64_t* ids, const float* cast, const int64_t* hm,
                                  const int64_t* ep, float* amax, int n, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_calibrate: unknown exception", [&] {
        if (!handle || !amax) throw std::runtime_error("cudanet_calibrate: null handle or output");
        Net* net = static_cast<Net*>(handle);
        std::lock_guard<std::mutex> lock(net->mu);
        const std::vector<float> got = net->calibrate(B, ids, cast, hm, ep);
        if (n < static_cast<int>(got.size()))
            throw std::runtime_error("cudanet_calibrate: the output holds " + std::to_string(n) + " floats, needs " +
                                     std::to_string(got.size()));
        std::memcpy(amax, got.data(), got.size() * sizeof(float));
        return static_cast<int>(got.size());
    });
}

CUDANET_API int cudanet_k_gemm(int dtype, int epi, int bn, const void* A, const void* W, const float* bias, void* C,
                               int M, int N, int K, int ldc, void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_gemm: unknown exception", [&] {
        if (dtype != 0 && dtype != 1) throw std::runtime_error("cudanet_k_gemm: dtype must be 0 (f16) or 1 (bf16)");
        if (M < 1 || N < 1 || K < 64) throw std::runtime_error("cudanet_k_gemm: bad sizes");
        int dev = 0;
        mf::RT(cudaGetDevice(&dev));
        int sms = 0;
        mf::RT(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        if (bn == 0) bn = mf::pick_bn(M, N, K, epi, sms);
        if ((reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(bias)) & 15)
            throw std::runtime_error("cudanet_k_gemm: C and bias must be 16-byte aligned");
        const long long ob = (epi == 2 || epi == 3) ? 4 : 2;
        if ((ldc * ob) % 16 || (N * ob) % 16)
            throw std::runtime_error("cudanet_k_gemm: C's rows and row pitch must be multiples of 16 bytes");
        if (ldc < N) throw std::runtime_error("cudanet_k_gemm: ldc < N");
        const bool b16 = dtype == 1;
        if (epi < 0 || epi > 3) throw std::runtime_error("cudanet_k_gemm: epi must be 0..3");
        const mf::MapType t = mf::type16(b16);
        const CUtensorMap ma = mf::operand_map(A, t, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 128);
        const CUtensorMap mb = mf::operand_map(W, t, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                               mf::w_box_rows(bn));
        const CUtensorMap mc = mf::output_map(C, epi, t, M, N, ldc);
        const mf::EpiArgs ep{bias, nullptr, 1.f};
        uint32_t* errw = nullptr;
        mf::RT(cudaMalloc(&errw, 4));
        mf::RT(cudaMemset(errw, 0, 4));
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        try {
            if (b16) mf::launch_gemm<__nv_bfloat16, __nv_bfloat16>(epi, bn, ma, mb, mc, M, N, K, ep, errw, sms, s);
            else mf::launch_gemm<__half, __half>(epi, bn, ma, mb, mc, M, N, K, ep, errw, sms, s);
            mf::RT(cudaStreamSynchronize(s));
        } catch (...) {
            cudaFree(errw);
            throw;
        }
        uint32_t e = 0;
        mf::RT(cudaMemcpy(&e, errw, 4, cudaMemcpyDeviceToHost));
        cudaFree(errw);
        if (e) throw std::runtime_error(std::string("cudanet_k_gemm: device error: ") + mf::err_site_name(e >> 8));
        return 0;
    });
}

CUDANET_API int cudanet_k_gemm_noalloc(int dtype, int epi, int bn, const void* A, const void* W, const float* bias,
                                       void* C, int M, int N, int K, int ldc, void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_gemm_noalloc: unknown exception", [&] {
        if (dtype != 0 && dtype != 1)
            throw std::runtime_error("cudanet_k_gemm_noalloc: dtype must be 0 (f16) or 1 (bf16)");
        if (M < 1 || N < 1 || K < 64) throw std::runtime_error("cudanet_k_gemm_noalloc: bad sizes");
        if (epi < 0 || epi > 3) throw std::runtime_error("cudanet_k_gemm_noalloc: epi must be 0..3");
        if (mf::kNoAllocBytesPerCall > mf::kNoAllocScratchBytes)
            throw std::runtime_error("cudanet_k_gemm_noalloc: the call needs more scratch than the static " +
                                     std::to_string(mf::kNoAllocScratchBytes) + " bytes");
        int dev = 0;
        mf::RT(cudaGetDevice(&dev));
        uint32_t* errw = mf::noalloc_scratch(dev);   // the first call on a device looks the address up
        int sms = 0;
        mf::RT(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        if (bn == 0) bn = mf::pick_bn(M, N, K, epi, sms);
        if ((reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(bias)) & 15)
            throw std::runtime_error("cudanet_k_gemm_noalloc: C and bias must be 16-byte aligned");
        const long long ob = (epi == 2 || epi == 3) ? 4 : 2;
        if ((ldc * ob) % 16 || (N * ob) % 16)
            throw std::runtime_error("cudanet_k_gemm_noalloc: C's rows and row pitch must be multiples of 16 bytes");
        if (ldc < N) throw std::runtime_error("cudanet_k_gemm_noalloc: ldc < N");
        const bool b16 = dtype == 1;
        const mf::MapType t = mf::type16(b16);
        const CUtensorMap ma = mf::operand_map(A, t, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 128);
        const CUtensorMap mb = mf::operand_map(W, t, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                               mf::w_box_rows(bn));
        const CUtensorMap mc = mf::output_map(C, epi, t, M, N, ldc);
        const mf::EpiArgs ep{bias, nullptr, 1.f};
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        // the word keeps the last call's value: clear it for this call, in stream order
        mf::RT(cudaMemsetAsync(errw, 0, mf::kNoAllocBytesPerCall, s));
        if (b16) mf::launch_gemm<__nv_bfloat16, __nv_bfloat16>(epi, bn, ma, mb, mc, M, N, K, ep, errw, sms, s);
        else mf::launch_gemm<__half, __half>(epi, bn, ma, mb, mc, M, N, K, ep, errw, sms, s);
        uint32_t e = 0;
        mf::RT(cudaMemcpyAsync(&e, errw, sizeof e, cudaMemcpyDeviceToHost, s));
        mf::RT(cudaStreamSynchronize(s));
        if (e)
            throw std::runtime_error(std::string("cudanet_k_gemm_noalloc: device error: ") + mf::err_site_name(e >> 8));
        return 0;
    });
}

CUDANET_API int cudanet_k_gemm_resln(int dtype, const void* A, const void* W, const float* bias, float* X,
                                     const float* g, const float* b, void* H, int M, int N, int K, void* stream,
                                     char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_gemm_resln: unknown exception", [&] {
        if (dtype != 0 && dtype != 1) throw std::runtime_error("cudanet_k_gemm_resln: dtype must be 0 (f16) or 1 (bf16)");
        if (M < 1 || K < 64) throw std::runtime_error("cudanet_k_gemm_resln: bad sizes");
        if ((reinterpret_cast<uintptr_t>(X) | reinterpret_cast<uintptr_t>(H)) & 15)
            throw std::runtime_error("cudanet_k_gemm_resln: X and H must be 16-byte aligned");
        const bool b16 = dtype == 1;
        const mf::MapType t = mf::type16(b16);
        const CUtensorMap ma = mf::operand_map(A, t, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 128);
        const CUtensorMap mb = mf::operand_map(W, t, static_cast<uint64_t>(K), static_cast<uint64_t>(N), 256);
        const CUtensorMap mx = mf::output_map(X, mf::kEpiResidual, t, M, N, N);
        const CUtensorMap mh = mf::output_map(H, mf::kEpiBias, t, M, N, N);
        uint32_t* errw = nullptr;
        mf::RT(cudaMalloc(&errw, 4));
        mf::RT(cudaMemset(errw, 0, 4));
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        try {
            if (b16) mf::launch_gemm_resln<__nv_bfloat16>(ma, mb, mx, mh, M, N, K, bias, g, b, errw, s);
            else mf::launch_gemm_resln<__half>(ma, mb, mx, mh, M, N, K, bias, g, b, errw, s);
            mf::RT(cudaStreamSynchronize(s));
        } catch (...) {
            cudaFree(errw);
            throw;
        }
        uint32_t e = 0;
        mf::RT(cudaMemcpy(&e, errw, 4, cudaMemcpyDeviceToHost));
        cudaFree(errw);
        if (e) throw std::runtime_error(std::string("cudanet_k_gemm_resln: device error: ") + mf::err_site_name(e >> 8));
        return 0;
    });
}

CUDANET_API int cudanet_k_attention(int dtype, const void* qkv, void* att, int B, int d, int heads, void* stream,
                                    char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_attention: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (dtype == 1)
            mf::attention_once<__nv_bfloat16, __nv_bfloat16>(qkv, att, B, d, heads, 1.f, s, "cudanet_k_attention");
        else if (dtype == 0)
            mf::attention_once<__half, __half>(qkv, att, B, d, heads, 1.f, s, "cudanet_k_attention");
        else
            throw std::runtime_error("cudanet_k_attention: dtype must be 0 (f16) or 1 (bf16)");
        return 0;
    });
}

CUDANET_API int cudanet_k_attention_tc(int dtype, const void* qkv, void* att, int B, int d, int heads, void* stream,
                                       char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_attention_tc: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (dtype == 1)
            mf::attention_once<__nv_bfloat16, __nv_bfloat16>(qkv, att, B, d, heads, 1.f, s, "cudanet_k_attention_tc",
                                                             1);
        else if (dtype == 0)
            mf::attention_once<__half, __half>(qkv, att, B, d, heads, 1.f, s, "cudanet_k_attention_tc", 1);
        else
            throw std::runtime_error("cudanet_k_attention_tc: dtype must be 0 (f16) or 1 (bf16)");
        return 0;
    });
}

CUDANET_API int cudanet_k_attention_kernel(int dtype, int e4m3_out, int kernel, const void* qkv, void* att, int B,
                                           int d, int heads, float mul, void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_attention_kernel: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        const char* who = "cudanet_k_attention_kernel";
        if (e4m3_out && dtype == 1)
            mf::attention_once<__nv_bfloat16, __nv_fp8_e4m3>(qkv, att, B, d, heads, mul, s, who, kernel);
        else if (e4m3_out)
            throw std::runtime_error("cudanet_k_attention_kernel: e4m3 outputs take bf16 qkv (dtype 1)");
        else if (dtype == 1)
            mf::attention_once<__nv_bfloat16, __nv_bfloat16>(qkv, att, B, d, heads, 1.f, s, who, kernel);
        else if (dtype == 0)
            mf::attention_once<__half, __half>(qkv, att, B, d, heads, 1.f, s, who, kernel);
        else
            throw std::runtime_error("cudanet_k_attention_kernel: dtype must be 0 (f16) or 1 (bf16)");
        return 0;
    });
}

CUDANET_API int cudanet_k_attention_cls(int dtype, const void* qkv, void* att, int B, int d, int heads, void* stream,
                                        char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_attention_cls: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if ((reinterpret_cast<uintptr_t>(qkv) | reinterpret_cast<uintptr_t>(att)) & 15)
            throw std::runtime_error("cudanet_k_attention_cls: qkv and att must be 16-byte aligned");
        if (dtype == 1)
            mf::launch_attention_cls<__nv_bfloat16, __nv_bfloat16>(static_cast<const __nv_bfloat16*>(qkv),
                                                                   static_cast<__nv_bfloat16*>(att), B, d, heads, 1.f, s);
        else if (dtype == 0)
            mf::launch_attention_cls<__half, __half>(static_cast<const __half*>(qkv), static_cast<__half*>(att), B, d,
                                                     heads, 1.f, s);
        else
            throw std::runtime_error("cudanet_k_attention_cls: dtype must be 0 (f16) or 1 (bf16)");
        mf::RT(cudaStreamSynchronize(s));
        return 0;
    });
}

CUDANET_API int cudanet_k_layernorm(int dtype, const float* x, const float* g, const float* b, void* h, int n,
                                    int d, int row_stride, void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_layernorm: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (n < 1 || row_stride < 1) throw std::runtime_error("cudanet_k_layernorm: bad sizes");
        if (dtype == 1)
            mf::launch_layernorm<__nv_bfloat16>(x, g, b, static_cast<__nv_bfloat16*>(h), n, d, row_stride, 1.f, s);
        else if (dtype == 0)
            mf::launch_layernorm<__half>(x, g, b, static_cast<__half*>(h), n, d, row_stride, 1.f, s);
        else
            throw std::runtime_error("cudanet_k_layernorm: dtype must be 0 (f16) or 1 (bf16)");
        mf::RT(cudaStreamSynchronize(s));
        return 0;
    });
}

// ------------------------------------------------------------------------------------------------ FP8 pieces
CUDANET_API int cudanet_k_gemm_f8(int epi, int bn, const void* A, const void* W, const float* colscale,
                                  const float* bias, float out_scale_inv, void* C, int M, int N, int K, int ldc,
                                  void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_gemm_f8: unknown exception", [&] {
        if (epi != mf::kEpiBias && epi != mf::kEpiResidual && epi != mf::kEpiF32 && epi != mf::kEpiGeluE4m3 &&
            epi != mf::kEpiResidual16)
            throw std::runtime_error("cudanet_k_gemm_f8: epi must be 0 (bf16 out), 2 (f32 residual), 3 (f32), 4 "
                                     "(GELU, e4m3 out) or 5 (bf16 residual)");
        if (M < 1 || N < 1 || K < 128) throw std::runtime_error("cudanet_k_gemm_f8: bad sizes");
        int dev = 0;
        mf::RT(cudaGetDevice(&dev));
        int sms = 0;
        mf::RT(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        if (bn == 0) bn = mf::pick_bn(M, N, K, epi, sms);
        if ((reinterpret_cast<uintptr_t>(C) | reinterpret_cast<uintptr_t>(bias) |
             reinterpret_cast<uintptr_t>(colscale)) & 15)
            throw std::runtime_error("cudanet_k_gemm_f8: C, bias and colscale must be 16-byte aligned");
        const long long ob = (epi == mf::kEpiResidual || epi == mf::kEpiF32) ? 4 : epi == mf::kEpiGeluE4m3 ? 1 : 2;
        if ((ldc * ob) % 16 || (N * ob) % 16)
            throw std::runtime_error("cudanet_k_gemm_f8: C's rows and row pitch must be multiples of 16 bytes");
        if (ldc < N) throw std::runtime_error("cudanet_k_gemm_f8: ldc < N");
        const CUtensorMap ma = mf::operand_map(A, mf::MapType::U8, static_cast<uint64_t>(K), static_cast<uint64_t>(M), 128);
        const CUtensorMap mb = mf::operand_map(W, mf::MapType::U8, static_cast<uint64_t>(K), static_cast<uint64_t>(N),
                                               mf::w_box_rows(bn));
        const CUtensorMap mc = mf::output_map(C, epi, mf::MapType::BF16, M, N, ldc, true);
        const mf::EpiArgs ep{bias, colscale, out_scale_inv};
        uint32_t* errw = nullptr;
        mf::RT(cudaMalloc(&errw, 4));
        mf::RT(cudaMemset(errw, 0, 4));
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        try {
            mf::launch_gemm<__nv_fp8_e4m3, __nv_bfloat16>(epi, bn, ma, mb, mc, M, N, K, ep, errw, sms, s);
            mf::RT(cudaStreamSynchronize(s));
        } catch (...) {
            cudaFree(errw);
            throw;
        }
        uint32_t e = 0;
        mf::RT(cudaMemcpy(&e, errw, 4, cudaMemcpyDeviceToHost));
        cudaFree(errw);
        if (e) throw std::runtime_error(std::string("cudanet_k_gemm_f8: device error: ") + mf::err_site_name(e >> 8));
        return 0;
    });
}

CUDANET_API int cudanet_k_attention_f8(const void* qkv, void* att, int B, int d, int heads, float mul, void* stream,
                                       char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_attention_f8: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        mf::attention_once<__nv_bfloat16, __nv_fp8_e4m3>(qkv, att, B, d, heads, mul, s, "cudanet_k_attention_f8");
        return 0;
    });
}

CUDANET_API int cudanet_k_layernorm_f8(int x_dtype, const void* x, const float* g, const float* b, void* h, int n,
                                       int d, int row_stride, float mul, void* stream, char* err, int err_len)
{
    return mf::guarded(err, err_len, "cudanet_k_layernorm_f8: unknown exception", [&] {
        const cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (n < 1 || row_stride < 1) throw std::runtime_error("cudanet_k_layernorm_f8: bad sizes");
        auto* hp = static_cast<__nv_fp8_e4m3*>(h);
        if (x_dtype == 0)
            mf::launch_layernorm<__nv_fp8_e4m3, float>(static_cast<const float*>(x), g, b, hp, n, d, row_stride, mul, s);
        else if (x_dtype == 1)
            mf::launch_layernorm<__nv_fp8_e4m3, __nv_bfloat16>(static_cast<const __nv_bfloat16*>(x), g, b, hp, n, d,
                                                               row_stride, mul, s);
        else
            throw std::runtime_error("cudanet_k_layernorm_f8: x_dtype must be 0 (f32) or 1 (bf16)");
        mf::RT(cudaStreamSynchronize(s));
        return 0;
    });
}

}  // extern "C"
