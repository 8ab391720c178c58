// gemm_q8.cu -- host side of the Q8_0 tensor-core GEMM: argument checks, TMA tensor maps, tile
// selection and launch of gemm_q8_tc_kernel (gemm_q8.cuh).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "backend.hpp"
#include "gemm_q8_2sm.cuh"

namespace sdvk {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 3-D tiled tensor map: dims {d0 (contiguous), d1, d2}, byte strides for d1 and d2.
int make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
             uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw, const LaunchEnv& env,
             const char* what) {
    auto fn = encode_fn();
    if (!fn) return fail(env, SDVK_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    if (d2 <= 1) {
        d2 = 1;
        s2 = s1 * d1;
    }
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(env, SDVK_E_SHAPE, std::string("tensor map rejected: ") + what);
    return SDVK_OK;
}

CUtensorMapDataType tma_type(int dt) {
    return dt == SDVK_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                          : dt == SDVK_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// K == 0: the product is empty, so C = bias (or 0), or C += bias when accumulating.
__global__ void gemm_k0_fill(float* c, const float* bias, uint32_t rows, uint32_t cols, uint64_t ld, uint64_t sb,
                             uint32_t batch, bool bias_per_row, bool accumulate) {
    const uint64_t n = (uint64_t)rows * cols * batch;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t z = i / ((uint64_t)rows * cols), rc = i % ((uint64_t)rows * cols);
        const uint32_t r = (uint32_t)(rc / cols), cc = (uint32_t)(rc % cols);
        const float b = bias ? bias[bias_per_row ? r : cc] : 0.0f;
        float* dst = c + z * sb + (uint64_t)r * ld + cc;
        *dst = accumulate ? *dst + b : b;
    }
}

bool set_smem_attr(const void* kern, int bytes, int device) {
    static std::mutex mu;
    static uint64_t done[64] = {};
    static const void* keys[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < 64; ++i) {
        if (keys[i] == kern) {
            if (done[i] & (1ull << device)) return true;
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
                return false;
            done[i] |= 1ull << device;
            return true;
        }
        if (!keys[i]) {
            keys[i] = kern;
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
                return false;
            done[i] = 1ull << device;
            return true;
        }
    }
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
}

template <class TA, int BN, bool NN, class TC>
int launch(const GemmQ8Desc& d, const LaunchEnv& env) {
    using Cfg = GemmQ8Config<TA, BN>;
    const int es = sizeof(TA), ces = sizeof(TC);
    CUtensorMap tmA, tmW, tmC;
    int rc;
    if (!NN) {
        rc = make_map(&tmA, tma_type(d.x_dtype), d.x, d.K, d.xrows, d.batch, d.ldx * es, d.sx * es, Cfg::kBK,
                      Cfg::kBM, CU_TENSOR_MAP_SWIZZLE_128B, env, "activation");
    } else {
        // N-major activation; 32-bit elements need the 32-byte-atom swizzle the tensor core reads
        // for MN-major tf32 operands.
        rc = make_map(&tmA, tma_type(d.x_dtype), d.x, d.xrows, d.K, d.batch, d.ldx * es, d.sx * es, Cfg::kBK,
                      Cfg::kBK, es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B, env,
                      "activation");
    }
    if (rc) return rc;
    rc = make_map(&tmW, CU_TENSOR_MAP_DATA_TYPE_UINT8, d.wq, d.K, d.wrows, d.sw ? d.batch : 1, d.ldw, d.sw,
                  Cfg::kBK, BN, CU_TENSOR_MAP_SWIZZLE_NONE, env, "weight");
    if (rc) return rc;
    if (!NN) {
        rc = make_map(&tmC, tma_type(d.c_dtype), d.c, d.wrows, d.xrows, d.batch, d.ldc * ces, d.sc * ces, 32, 32,
                      ces == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, env, "output");
    } else {
        rc = make_map(&tmC, tma_type(d.c_dtype), d.c, d.xrows, d.wrows, d.batch, d.ldc * ces, d.sc * ces, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_NONE, env, "output");
    }
    if (rc) return rc;

    GemmQ8Params p{};
    p.wq = d.wq;
    p.ws = d.ws;
    p.bias = d.bias;
    p.xrows = d.xrows;
    p.wrows = d.wrows;
    p.K = d.K;
    p.batch = d.batch;
    p.ldw = d.ldw;
    p.sW = d.sw;
    p.tiles_x = (d.xrows + Cfg::kBM - 1) / Cfg::kBM;
    p.tiles_w = (d.wrows + BN - 1) / BN;
    p.num_tiles = p.tiles_x * p.tiles_w * d.batch;
    p.k_stages = (d.K + Cfg::kBK - 1) / Cfg::kBK;
    p.accumulate = d.accumulate ? 1u : 0u;
    p.sbias = d.sbias;
    p.err = env.err_dev;
    p.timeout_ns = env.timeout_ns;
    p.c = d.c;
    p.ldc = d.ldc;
    p.sc = d.sc;

    auto kern = gemm_q8_tc_kernel<TA, BN, NN, TC>;
    if (!set_smem_attr(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, env.device))
        return fail(env, SDVK_E_CUDA, "cudaFuncSetAttribute(max dynamic smem) failed");
    const uint32_t grid = std::min<uint32_t>(p.num_tiles, (uint32_t)env.num_sms);
    kern<<<grid, Cfg::kThreads, Cfg::kSmemBytes, env.stream>>>(tmA, tmW, tmC, p);
    return cuda_check(env, cudaGetLastError(), "gemm_q8_tc_kernel launch");
}


// CTA-pair variant: 256 (weight rows) x BNX (activation rows) tiles on two SMs (cta_group::2).
template <class TA, int BNX, bool NN, class TC>
int launch_pair(const GemmQ8Desc& d, const LaunchEnv& env) {
    using Cfg = Gemm2Config<TA, BNX>;
    const int es = sizeof(TA), ces = sizeof(TC);
    CUtensorMap tmX, tmC;
    int rc;
    if (!NN) {
        rc = make_map(&tmX, tma_type(d.x_dtype), d.x, d.K, d.xrows, d.batch, d.ldx * es, d.sx * es, Cfg::kBK,
                      Cfg::kBXC, CU_TENSOR_MAP_SWIZZLE_128B, env, "activation");
    } else {
        rc = make_map(&tmX, tma_type(d.x_dtype), d.x, d.xrows, d.K, d.batch, d.ldx * es, d.sx * es, Cfg::kBK,
                      Cfg::kBK, es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B, env,
                      "activation");
    }
    if (rc) return rc;
    // no weight map: the dequantisers load the raw weights with 16-byte loads (gemm_q8 checked
    // the 16-byte base and the 32-element strides they rely on)
    if (!NN && d.geglu) {  // 16 output columns per 32 weight rows: [32 x][16] f16 tiles
        rc = make_map(&tmC, tma_type(d.c_dtype), d.c, d.wrows / 2, d.xrows, d.batch, d.ldc * ces, d.sc * ces, 16, 32,
                      CU_TENSOR_MAP_SWIZZLE_NONE, env, "output");
    } else if (!NN) {  // the accumulator transposed: [32 x][32 w] tiles
        rc = make_map(&tmC, tma_type(d.c_dtype), d.c, d.wrows, d.xrows, d.batch, d.ldc * ces, d.sc * ces, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_NONE, env, "output");
    } else {  // [32 w][32 x] swizzled rows
        rc = make_map(&tmC, tma_type(d.c_dtype), d.c, d.xrows, d.wrows, d.batch, d.ldc * ces, d.sc * ces, 32, 32,
                      ces == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B, env, "output");
    }
    if (rc) return rc;
    GemmQ8Params p{};
    p.wq = d.wq;
    p.ws = d.ws;
    p.bias = d.bias;
    p.xrows = d.xrows;
    p.wrows = d.wrows;
    p.K = d.K;
    p.batch = d.batch;
    p.ldw = d.ldw;
    p.sW = d.sw;
    p.geglu = d.geglu ? 1u : 0u;
    p.weights_static = d.weights_static ? 1u : 0u;
    p.tiles_x = (d.xrows + Cfg::kBNX - 1) / Cfg::kBNX;
    p.tiles_w = (d.wrows + 2 * Cfg::kBW - 1) / (2 * Cfg::kBW);
    p.num_tiles = p.tiles_x * p.tiles_w * d.batch;
    p.k_stages = (d.K + Cfg::kBK - 1) / Cfg::kBK;
    p.accumulate = d.accumulate ? 1u : 0u;
    p.sbias = d.sbias;
    p.err = env.err_dev;
    p.timeout_ns = env.timeout_ns;
    p.c = d.c;
    p.ldc = d.ldc;
    p.sc = d.sc;
    auto kern = gemm_q8_tc2_kernel<TA, BNX, NN, TC>;
    if (!set_smem_attr(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, env.device))
        return fail(env, SDVK_E_CUDA, "cudaFuncSetAttribute(max dynamic smem) failed");
    const uint32_t clusters = std::min<uint32_t>(p.num_tiles, (uint32_t)env.num_sms / 2);
    // Programmatic stream serialisation: this grid's prologue may overlap the previous kernel's
    // tail; the kernel waits (griddepcontrol.wait) before its first global access.
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(2 * clusters);
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = env.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_check(env, cudaLaunchKernelEx(&cfg, kern, tmX, tmC, p), "gemm_q8_tc2_kernel launch");
}

// Pair-tile width (tensor-core N = activation rows): the candidate minimising waves x per-tile
// cost, where a tile costs its N plus a fixed share (the 256 weight rows' dequantisation and the
// per-tile overheads do not shrink with N).  NN stages activations as 64-column blocks per CTA,
// so its widths are 128 and 256.
int pick_pair_bn(const GemmQ8Desc& d, int num_sms, bool nn) {
    const int clusters = num_sms / 2;
    const uint64_t wt = (d.wrows + 255) / 256;
    int best = 256;
    uint64_t best_cost = ~0ull;
    for (int bn : {256, 224, 192, 160, 128}) {
        if (nn && bn % 128) continue;
        const uint64_t tiles = wt * ((d.xrows + bn - 1) / bn) * d.batch;
        const uint64_t waves = (tiles + clusters - 1) / clusters;
        const uint64_t cost = waves * (uint64_t)(bn + 256);
        if (cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    return best;
}

// Kernel choice: the CTA-pair kernel when the problem fills at least about half of the SM pairs
// with 256 x 256 tiles, or when a launch-time model says it is at least 10% faster: below about
// half the pairs the single-CTA tiles (128 x 128 or 128 x 256) give more parallelism, but a
// single-CTA stage dequantises twice the weight rows per SM, and over a long K (the batch-1
// feed-forward output, K = 5120: 58.6 us single-CTA against 39.0 us as 20 pair tiles, measured
// back to back on the B200) the per-stage cost decides.
// SDVK_GEMM_VARIANT=1sm|2sm forces one of them; SDVK_GEMM_PAIR_BN forces the pair tile width.
// Modelled launch time in units of 0.64 ns (a 256 x 256 pair k-stage = 512, about 0.33 us when
// the clusters are not all busy; a 128 x 256 single-CTA stage about 0.62 us = 960), plus each
// kernel's fill and drain (about 12.9 us pair, 8.7 us single-CTA), from back-to-back launches of
// the 1024 x 1280 x {1280, 5120} projections.
uint64_t modelled_pair(const GemmQ8Desc& d, int num_sms, int bn, int es) {
    const uint64_t clusters = (uint64_t)num_sms / 2, ks = (d.K + 128 / es - 1) / (128 / es);
    const uint64_t tiles = ((d.wrows + 255) / 256) * ((d.xrows + bn - 1) / bn) * d.batch;
    return 20000 + (tiles + clusters - 1) / clusters * ks * (uint64_t)(bn + 256);
}
uint64_t modelled_single(const GemmQ8Desc& d, int num_sms, int es) {
    const uint64_t bn = d.wrows <= 128 ? 128 : 256, ks = (d.K + 128 / es - 1) / (128 / es);
    const uint64_t tiles = ((d.xrows + 127) / 128) * ((d.wrows + bn - 1) / bn) * d.batch;
    return 13500 + (tiles + num_sms - 1) / num_sms * ks * (bn == 256 ? 960 : 600);
}

int variant_override() {
    const char* e = getenv("SDVK_GEMM_VARIANT");
    return (e && e[0] == '1') ? 1 : (e && e[0] == '2') ? 2 : 0;
}

template <class TA, bool NN, class TC>
int launch_bn(const GemmQ8Desc& d, const LaunchEnv& env) {
    const uint64_t pair_tiles = (uint64_t)((d.xrows + 255) / 256) * ((d.wrows + 255) / 256) * d.batch;
    const int forced = variant_override();
    // the GEGLU epilogue exists in the CTA-pair kernel only
    const int pick = pick_pair_bn(d, env.num_sms, NN);
    const bool fills = pair_tiles * 4 >= (uint64_t)env.num_sms;
    const bool faster = !fills && d.wrows > 128 &&
                        modelled_pair(d, env.num_sms, pick, sizeof(TA)) * 10 < modelled_single(d, env.num_sms, sizeof(TA)) * 9;
    const bool pair = d.geglu || forced == 2 || (forced == 0 && d.wrows > 128 && (fills || faster));
    if (pair) {
        const char* e = getenv("SDVK_GEMM_PAIR_BN");
        int bn = e ? atoi(e) : pick;
        if constexpr (NN) {
            return bn == 128 ? launch_pair<TA, 128, NN, TC>(d, env) : launch_pair<TA, 256, NN, TC>(d, env);
        } else {
            if (bn == 224) return launch_pair<TA, 224, NN, TC>(d, env);
            if (bn == 192) return launch_pair<TA, 192, NN, TC>(d, env);
            if (bn == 160) return launch_pair<TA, 160, NN, TC>(d, env);
            if (bn == 128) return launch_pair<TA, 128, NN, TC>(d, env);
            return launch_pair<TA, 256, NN, TC>(d, env);
        }
    }
    if (d.wrows <= 128) return launch<TA, 128, NN, TC>(d, env);
    return launch<TA, 256, NN, TC>(d, env);
}

template <class TA, bool NN>
int launch_c(const GemmQ8Desc& d, const LaunchEnv& env) {
    if (d.c_dtype == SDVK_F32) return launch_bn<TA, NN, float>(d, env);
    return launch_bn<TA, NN, __half>(d, env);
}

template <bool NN>
int launch_a(const GemmQ8Desc& d, const LaunchEnv& env) {
    switch (d.x_dtype) {
        case SDVK_F16: return launch_c<__half, NN>(d, env);
        case SDVK_BF16: return launch_c<__nv_bfloat16, NN>(d, env);
        default: return launch_c<float, NN>(d, env);
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

bool pdl_enabled() {
    const char* e = getenv("SDVK_PDL");
    return !(e && e[0] == '0');
}

// GEGLU interleave of an ff.net.0.proj weight [2F][K] (rows 0..F-1 = a, F..2F-1 = gate): output row
// r = 32j + t holds a row 16j + t for t < 16 and gate row 16j + t - 16 otherwise, with its scales and
// bias, so that each 32-column accumulator chunk of the GEMM holds 16 (a, gate) column pairs.
__global__ void geglu_interleave_kernel(const int8_t* __restrict__ q, const float* __restrict__ s,
                                        const float* __restrict__ bias, uint32_t F, uint32_t K, int8_t* q_out,
                                        float* s_out, float* bias_out) {
    const uint32_t r = blockIdx.x, t = r & 31, j = r >> 5;
    const uint32_t src = t < 16 ? 16 * j + t : F + 16 * j + (t - 16);
    const uint4* qs = reinterpret_cast<const uint4*>(q + (uint64_t)src * K);
    uint4* qd = reinterpret_cast<uint4*>(q_out + (uint64_t)r * K);
    for (uint32_t i = threadIdx.x; i < K / 16; i += blockDim.x) qd[i] = qs[i];
    for (uint32_t i = threadIdx.x; i < K / 32; i += blockDim.x) s_out[(uint64_t)r * (K / 32) + i] = s[(uint64_t)src * (K / 32) + i];
    if (bias && bias_out && threadIdx.x == 0) bias_out[r] = bias[src];
}

int geglu_interleave(const int8_t* q, const float* s, const float* bias, uint32_t F, uint32_t K, int8_t* q_out,
                     float* s_out, float* bias_out, const LaunchEnv& env) {
    if (!q || !s || !q_out || !s_out || (bias && !bias_out)) return fail(env, SDVK_E_ARG, "null pointer");
    if (F == 0 || F % 16 || K % 32 || !aligned16(q) || !aligned16(q_out))
        return fail(env, SDVK_E_SHAPE, "GEGLU interleave needs F % 16 == 0, K % 32 == 0, 16-byte aligned rows");
    geglu_interleave_kernel<<<2 * F, 128, 0, env.stream>>>(q, s, bias, F, K, q_out, s_out, bias_out);
    return cuda_check(env, cudaGetLastError(), "geglu_interleave_kernel launch");
}

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return encode_fn(); }
int tiled_map_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw, const LaunchEnv& env,
                 const char* what) {
    return make_map(m, dt, base, d0, d1, d2, s1, s2, b0, b1, sw, env, what);
}
CUtensorMapDataType tma_dtype(int dt) { return tma_type(dt); }
bool kernel_smem_attr(const void* kern, int bytes, int device) { return set_smem_attr(kern, bytes, device); }

int gemm_q8(const GemmQ8Desc& d, const LaunchEnv& env) {
    if (!d.x || !d.wq || !d.ws || !d.c) return fail(env, SDVK_E_ARG, "null pointer");
    if (d.x_dtype != SDVK_F32 && d.x_dtype != SDVK_F16 && d.x_dtype != SDVK_BF16)
        return fail(env, SDVK_E_ARG, "activation dtype must be F32, F16 or BF16");
    if (d.c_dtype != SDVK_F32 && d.c_dtype != SDVK_F16) return fail(env, SDVK_E_ARG, "output dtype must be F32 or F16");
    if (d.accumulate && d.c_dtype != SDVK_F32) return fail(env, SDVK_E_ARG, "accumulate requires an F32 output");
    if (d.batch == 0 || d.xrows == 0 || d.wrows == 0) return SDVK_OK;
    if (d.K % 32) return fail(env, SDVK_E_SHAPE, "K must be a multiple of 32 (whole Q8_0 blocks)");
    if (d.ldw % 32 || d.sw % 32 || d.ldw < d.K) return fail(env, SDVK_E_SHAPE, "weight strides must be multiples of 32");
    const int es = dtype_size(d.x_dtype), ces = dtype_size(d.c_dtype);
    const uint64_t xmin = d.nn ? d.xrows : d.K, cmin = d.nn ? d.xrows : d.geglu ? d.wrows / 2 : d.wrows;
    if (d.ldx < xmin || d.ldc < cmin) return fail(env, SDVK_E_SHAPE, "row stride smaller than the row");
    if (!aligned16(d.x) || !aligned16(d.c) || !aligned16(d.wq))
        return fail(env, SDVK_E_SHAPE, "operands must be 16-byte aligned");
    if ((d.ldx * es) % 16 || (d.ldc * ces) % 16 || (d.batch > 1 && ((d.sx * es) % 16 || (d.sc * ces) % 16)))
        return fail(env, SDVK_E_SHAPE, "row/batch strides must be multiples of 16 bytes");
    if (d.geglu && (d.nn || d.c_dtype != SDVK_F16 || d.accumulate || d.wrows % 32 || d.ldc < d.wrows / 2 || d.K == 0))
        return fail(env, SDVK_E_SHAPE, "the GEGLU epilogue needs NT, an F16 output, 32 | rows and K > 0");
    if (d.K == 0) {
        if (d.accumulate && !d.bias) return SDVK_OK;
        if (d.c_dtype != SDVK_F32) return fail(env, SDVK_E_SHAPE, "K == 0 needs an F32 output");
        const uint32_t rows = d.nn ? d.wrows : d.xrows, cols = d.nn ? d.xrows : d.wrows;
        gemm_k0_fill<<<256, 256, 0, env.stream>>>(static_cast<float*>(d.c), d.bias, rows, cols, d.ldc, d.sc, d.batch,
                                                   d.nn, d.accumulate);
        return cuda_check(env, cudaGetLastError(), "gemm_k0_fill launch");
    }
    return d.nn ? launch_a<true>(d, env) : launch_a<false>(d, env);
}

}  // namespace sdvk
