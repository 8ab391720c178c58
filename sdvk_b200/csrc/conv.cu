// conv.cu -- the UNet's 3x3 convolutions with Q8_0 weights: im2col + the Q8_0 NN GEMM, the
// reference's structure (conv3RawInto and conv3s2, sdvkgen.cpp:1133-1175; im2col.comp and
// im2col_s2.comp; gemmNnQ8 with ldc = P; biasAddCh).
//
// x [batch][cin][H][W] (channel-major), weight [cout][cin*9] with k = c*9 + ky*3 + kx, output
// [batch][cout][OH][OW].  Stride 1 pads 1 on every side; stride 2 gives OH = H/2, OW = W/2 with either
// the symmetric pad-1 ring (off = -1, the UNet downsamplers) or padding on the right/bottom only
// (off = 0, the VAE encoder's Downsample2D).  The column matrix col[k][p] (p over a band of output rows)
// goes to a caller-provided workspace in the GEMM's activation type, in bands of output rows that fit
// it; the GEMM writes the band's output columns with the row stride OH*OW and adds the bias in its
// epilogue.
//
// The implicit-GEMM form (conv_tc2.cuh) never materialises col: TMA im2col loads read the input
// windows from a channels-last fp16 copy of x, and the weights are a tap-major fp16 repack of the
// Q8_0 payload.  sdvk_conv3x3_q8 takes it for fp16 inputs whose shape it handles when the workspace
// holds the two (x channels-last, then the repacked weights); the UNet keeps both resident.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "backend.hpp"
#include "conv_tc2.cuh"
#include "ptx.cuh"

namespace sdvk {
namespace {

constexpr int kColThreads = 256;

// grid (ceil(np / (256 * 8)), K, images): thread = 8 consecutive output positions p of column-matrix row k,
// col[k][p] = x[c][oh*stride + ky + off][ow*stride + kx + off] (0 outside), stored with 16-byte
// vector stores (rows of col ld elements apart, ld % 8 == 0; positions in [np, round_up(np, 8)) are
// written with values the GEMM never reads).
template <class T>
__global__ void __launch_bounds__(kColThreads) im2col3x3_kernel(const T* __restrict__ x, T* __restrict__ col,
                                                                uint32_t H, uint32_t W, uint32_t OW, uint32_t row0,
                                                                uint32_t np, uint64_t ld, uint32_t stride, int off,
                                                                uint64_t xbs, uint64_t cbs) {
    grid_dependency_wait();
    grid_launch_dependents();
    x += blockIdx.z * xbs;  // image z: its input, and its column matrix cbs elements further on
    col += blockIdx.z * cbs;
    const uint32_t k = blockIdx.y;
    const uint32_t p0 = (blockIdx.x * kColThreads + threadIdx.x) * 8;
    if (p0 >= np) return;
    const uint32_t c = k / 9, r = k - c * 9, ky = r / 3, kx = r - ky * 3;
    uint32_t oh = row0 + p0 / OW, ow = p0 % OW;
    const T* xc = x + (uint64_t)c * H * W;
    T v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int ih = (int)(oh * stride + ky) + off, iw = (int)(ow * stride + kx) + off;
        v[j] = (ih >= 0 && ih < (int)H && iw >= 0 && iw < (int)W) ? xc[(uint64_t)ih * W + iw] : T(0.0f);
        if (++ow == OW) ow = 0, ++oh;
    }
    T* dst = col + (uint64_t)k * ld + p0;
    if constexpr (sizeof(T) == 2) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = (uint32_t)__builtin_bit_cast(uint16_t, v[2 * j]) |
                   ((uint32_t)__builtin_bit_cast(uint16_t, v[2 * j + 1]) << 16);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// 8 consecutive values of T from a 16-byte aligned address, widened to float
template <class T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] = (float)__builtin_bit_cast(T, (uint16_t)(u[j] & 0xFFFFu));
            v[2 * j + 1] = (float)__builtin_bit_cast(T, (uint16_t)(u[j] >> 16));
        }
    }
}

// 8 floats stored as T (exact: every value came from a T) to a 16-byte aligned address
template <class T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = (uint32_t)__builtin_bit_cast(uint16_t, T(v[2 * j])) |
                   ((uint32_t)__builtin_bit_cast(uint16_t, T(v[2 * j + 1])) << 16);
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Row-segment im2col: grid (ceil(rows * OW/8 / 256), cin, images); a thread owns 8 consecutive output
// positions of one output row and one input channel c.  It reads the three input rows it needs once
// (the aligned 8*S values under the segment as 16-byte vectors, plus a one-value halo on either side)
// and writes all nine column-matrix rows k = c*9 + ky*3 + kx for its positions, 16 bytes each.
// Requires OW % 8 == 0, W % 8 == 0 and a 16-byte aligned x (every row and segment start aligned).
template <class T, int S, int OFF>
__global__ void __launch_bounds__(kColThreads) im2col3x3_rows_kernel(const T* __restrict__ x, T* __restrict__ col,
                                                                     uint32_t H, uint32_t W, uint32_t OW,
                                                                     uint32_t row0, uint32_t nrows, uint64_t ld,
                                                                     uint64_t xbs, uint64_t cbs) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t segs = OW / 8, seg = blockIdx.x * kColThreads + threadIdx.x;
    if (seg >= nrows * segs) return;
    const uint32_t c = blockIdx.y, r = seg / segs, ow0 = (seg - r * segs) * 8, oh = row0 + r;
    const T* xc = x + blockIdx.z * xbs + (uint64_t)c * H * W;
    T* dst = col + blockIdx.z * cbs + (uint64_t)c * 9 * ld + (uint64_t)r * OW + ow0;
    const uint32_t a0 = ow0 * S;  // first input column under the segment (8-aligned)
    constexpr int NV = 8 * S + 2;  // v[i] holds input column a0 - 1 + i
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
        const int ih = (int)(oh * S) + ky + OFF;
        float v[NV];
        if (ih >= 0 && ih < (int)H) {
            const T* row = xc + (uint64_t)ih * W;
            v[0] = a0 >= 1 ? (float)row[a0 - 1] : 0.0f;
#pragma unroll
            for (int h = 0; h < S; ++h) {
                float t[8];
                load8(row + a0 + 8 * h, t);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[1 + 8 * h + j] = t[j];
            }
            v[NV - 1] = a0 + 8 * S < W ? (float)row[a0 + 8 * S] : 0.0f;
        } else {
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = 0.0f;
        }
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = v[j * S + kx + OFF + 1];
            store8(dst + (uint64_t)(ky * 3 + kx) * ld, o);
        }
    }
}

// im2col of output rows [row0, row0 + nrows) of `images` images into col (row pitch ld elements; image z
// at x + z*xbs, its columns at col + z*cbs): the row-segment kernel where the shape allows, else the
// per-element one.
template <class T>
int im2col_launch(const T* x, T* col, uint32_t cin, uint32_t H, uint32_t W, uint32_t OW, uint32_t row0,
                  uint32_t nrows, uint64_t ld, uint32_t stride, int off, uint32_t images, uint64_t xbs, uint64_t cbs,
                  const LaunchEnv& env) {
    const bool rows_ok = OW % 8 == 0 && W % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                         (xbs * sizeof(T)) % 16 == 0 && ld % 8 == 0 && (cbs * sizeof(T)) % 16 == 0;
    if (rows_ok) {
        const dim3 grid((nrows * (OW / 8) + kColThreads - 1) / kColThreads, cin, images);
        auto kern = stride == 1 ? im2col3x3_rows_kernel<T, 1, -1>
                                : off == 0 ? im2col3x3_rows_kernel<T, 2, 0> : im2col3x3_rows_kernel<T, 2, -1>;
        return launch_pdl(kern, grid, dim3(kColThreads), 0, env, "im2col3x3_rows_kernel launch", x, col, H, W, OW, row0,
                          nrows, ld, xbs, cbs);
    }
    const uint32_t np = nrows * OW;
    const dim3 grid((np + 8 * kColThreads - 1) / (8 * kColThreads), cin * 9, images);
    return launch_pdl(im2col3x3_kernel<T>, grid, dim3(kColThreads), 0, env, "im2col3x3_kernel launch", x, col, H, W,
                      OW, row0, np, ld, stride, off, xbs, cbs);
}

int im2col_any(const void* x, int x_dtype, void* col, uint32_t cin, uint32_t H, uint32_t W, uint32_t OW,
               uint32_t row0, uint32_t nrows, uint64_t ld, uint32_t stride, int off, uint32_t images, uint64_t xbs,
               uint64_t cbs, const LaunchEnv& env) {
    if (x_dtype == SDVK_F32)
        return im2col_launch(static_cast<const float*>(x), static_cast<float*>(col), cin, H, W, OW, row0, nrows, ld,
                             stride, off, images, xbs, cbs, env);
    if (x_dtype == SDVK_F16)
        return im2col_launch(static_cast<const __half*>(x), static_cast<__half*>(col), cin, H, W, OW, row0, nrows, ld,
                             stride, off, images, xbs, cbs, env);
    return im2col_launch(static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(col), cin, H, W, OW, row0,
                         nrows, ld, stride, off, images, xbs, cbs, env);
}

// ---------------------------------------------------------------- the implicit-GEMM form

PFN_cuTensorMapEncodeIm2col_v12000 im2col_encode_fn() {
    static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
    });
    return fn;
}

// w16[o][(cb*9 + t)*64 + j] = q[o][(cb*64 + j)*9 + t] * scale, both factors as fp16 and one rounded fp16
// multiply: the value the GEMM's dequantiser writes for the same weight (dequant16<__half>).
__global__ void conv_weights_f16_kernel(const int8_t* __restrict__ q, const float* __restrict__ s,
                                        __half* __restrict__ w16, uint32_t cout, uint32_t cin) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t K = cin * 9;
    const uint64_t n = (uint64_t)cout * K;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t o = (uint32_t)(i / K), kp = (uint32_t)(i % K), ks = kp / 64, j = kp % 64, cb = ks / 9,
                       t = ks - cb * 9;
        const uint64_t src = (uint64_t)o * K + (uint64_t)(cb * 64 + j) * 9 + t;
        w16[i] = __hmul(__float2half_rn((float)q[src]), __float2half_rn(s[src >> 5]));
    }
}

// out[b][p][c] = in[b][c][p]: 32 x 32 tiles through shared memory; grid (ceil(P/32), ceil(C/32), B),
// block (32, 8).
__global__ void __launch_bounds__(256) channels_last_kernel(const __half* __restrict__ in, __half* __restrict__ out,
                                                            uint32_t C, uint32_t P) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ __half tile[32][34];
    const uint32_t b = blockIdx.z, c0 = blockIdx.y * 32, p0 = blockIdx.x * 32;
    const __half* src = in + (uint64_t)b * C * P;
    __half* dst = out + (uint64_t)b * C * P;
    for (uint32_t r = threadIdx.y; r < 32; r += 8) {
        const uint32_t c = c0 + r, pp = p0 + threadIdx.x;
        if (c < C && pp < P) tile[r][threadIdx.x] = src[(uint64_t)c * P + pp];
    }
    __syncthreads();
    for (uint32_t r = threadIdx.y; r < 32; r += 8) {
        const uint32_t pp = p0 + r, c = c0 + threadIdx.x;
        if (c < C && pp < P) dst[(uint64_t)pp * C + c] = tile[threadIdx.x][r];
    }
}

// Pair-tile width (tensor-core N = output channels): the candidate with the fewest waves x per-stage
// cycles, where a stage costs the tensor core's 2*BN cycles or the L2 reads of its operands (16 KB of
// windows and BN*64 bytes of weights per CTA, at about 60 bytes per cycle per SM), whichever is longer.
int pick_conv_bn(uint64_t positions, uint32_t cout, int num_sms) {
    if (const char* e = getenv("SDVK_CONV_BN")) return atoi(e);
    const uint64_t clusters = (uint64_t)std::max(1, num_sms / 2), mt = (positions + 255) / 256;
    int best = 256;
    double best_cost = 1e300;
    for (int bn : {256, 192, 160, 128, 64, 32}) {
        const uint64_t tiles = mt * ((cout + bn - 1) / bn), waves = (tiles + clusters - 1) / clusters;
        const double cost = (double)waves * std::max(2.0 * bn, (16384.0 + 64.0 * bn) / 60.0);
        if (cost < best_cost) best_cost = cost, best = bn;
    }
    return best;
}

template <int BN, class TC>
int launch_conv_tc2(const ConvImplicitDesc& d, const LaunchEnv& env) {
    using Cfg = ConvCfg<BN>;
    const uint32_t S = d.stride, OH = S == 1 ? d.H : d.H / 2, OW = S == 1 ? d.W : d.W / 2, P = OH * OW;
    const int lower = S == 1 ? -1 : d.off;
    auto enc = im2col_encode_fn();
    if (!enc) return fail(env, SDVK_E_CUDA, "cuTensorMapEncodeIm2col unavailable");
    // The pixel box holds the window corners of the output positions, (lower + S*o) for o < OW (OH),
    // walked with traversal stride S; the load's offsets pick the tap.
    CUtensorMap tmX, tmW, tmC;
    const cuuint64_t dims[4] = {d.cin, d.W, d.H, d.batch};
    const cuuint64_t strides[3] = {(uint64_t)d.cin * 2, (uint64_t)d.W * d.cin * 2, (uint64_t)d.H * d.W * d.cin * 2};
    const int lo[2] = {lower, lower};
    const int hi[2] = {(int)((OW - 1) * S) + lower - (int)d.W + 1, (int)((OH - 1) * S) + lower - (int)d.H + 1};
    const cuuint32_t estr[4] = {1, S, S, 1};
    CUresult r = enc(&tmX, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<__half*>(d.x), dims, strides, lo, hi, 64,
                     128, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(env, SDVK_E_SHAPE, "tensor map rejected: conv input windows (im2col)");
    const uint64_t K = 9ull * d.cin;
    int rc = tiled_map_3d(&tmW, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, d.w16, K, d.cout, 1, K * 2, 0, 64, BN / 2,
                          CU_TENSOR_MAP_SWIZZLE_128B, env, "conv weights");
    if (rc) return rc;
    const uint64_t ces = sizeof(TC);
    rc = tiled_map_3d(&tmC, tma_dtype(d.y_dtype), d.y, P, d.cout, d.batch, P * ces, (uint64_t)d.cout * P * ces, 32, 32,
                      CU_TENSOR_MAP_SWIZZLE_NONE, env, "conv output");
    if (rc) return rc;
    ConvParams p{};
    p.bias = d.bias;
    p.sbias = d.bias ? d.sbias : 0;
    p.P = P;
    p.OW = OW;
    p.batch = d.batch;
    p.cout = d.cout;
    p.stride = (int)S;
    p.lower = lower;
    p.k_stages = 9 * d.cin / 64;
    p.tiles_n = (d.cout + BN - 1) / BN;
    const uint64_t tiles = ((uint64_t)d.batch * P + 255) / 256 * p.tiles_n;
    if (tiles > 0x7FFFFFFFull) return fail(env, SDVK_E_SHAPE, "convolution too large");
    p.num_tiles = (uint32_t)tiles;
    p.accumulate = d.accumulate ? 1u : 0u;
    p.err = env.err_dev;
    p.timeout_ns = env.timeout_ns;
    auto kern = conv3x3_tc2_kernel<BN, TC>;
    if (!kernel_smem_attr(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, env.device))
        return fail(env, SDVK_E_CUDA, "cudaFuncSetAttribute(max dynamic smem) failed");
    const uint32_t clusters = std::min<uint32_t>(p.num_tiles, (uint32_t)env.num_sms / 2);
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
    return cuda_check(env, cudaLaunchKernelEx(&cfg, kern, tmX, tmW, tmC, p), "conv3x3_tc2_kernel launch");
}

template <class TC>
int launch_conv_bn(const ConvImplicitDesc& d, int bn, const LaunchEnv& env) {
    switch (bn) {
        case 32: return launch_conv_tc2<32, TC>(d, env);
        case 64: return launch_conv_tc2<64, TC>(d, env);
        case 128: return launch_conv_tc2<128, TC>(d, env);
        case 160: return launch_conv_tc2<160, TC>(d, env);
        case 192: return launch_conv_tc2<192, TC>(d, env);
        case 256: return launch_conv_tc2<256, TC>(d, env);
        default: return fail(env, SDVK_E_ARG, "conv tile width must be 32, 64, 128, 160, 192 or 256");
    }
}

// Shared argument checks of both forms (the explicit one's order: pointers, dtypes, stride, padding).
int check_conv(const void* x, int x_dtype, const void* w, const void* y, int y_dtype, bool accumulate, uint32_t stride,
               int& off, const LaunchEnv& env) {
    if (!x || !w || !y) return fail(env, SDVK_E_ARG, "null pointer");
    if (accumulate && y_dtype != SDVK_F32) return fail(env, SDVK_E_ARG, "an accumulating conv needs an F32 output");
    if (x_dtype != SDVK_F16 && x_dtype != SDVK_BF16 && x_dtype != SDVK_F32)
        return fail(env, SDVK_E_ARG, "conv input must be F16, BF16 or F32");
    if (y_dtype != SDVK_F16 && y_dtype != SDVK_F32) return fail(env, SDVK_E_ARG, "conv output must be F16 or F32");
    if (stride != 1 && stride != 2) return fail(env, SDVK_E_SHAPE, "conv stride must be 1 or 2");
    if (stride == 1) off = -1;
    if (off != -1 && off != 0) return fail(env, SDVK_E_SHAPE, "conv padding offset must be -1 or 0");
    return SDVK_OK;
}

}  // namespace

bool conv_implicit_ok(uint32_t batch, uint32_t cin, uint32_t H, uint32_t W, uint32_t stride) {
    if (const char* e = getenv("SDVK_CONV_IMPLICIT"))
        if (e[0] == '0') return false;
    if ((stride != 1 && stride != 2) || batch == 0 || cin == 0 || cin % 64 || H == 0 || W == 0) return false;
    const uint64_t OH = stride == 1 ? H : H / 2, OW = stride == 1 ? W : W / 2, P = OH * OW;
    if (P == 0 || P % 128 || P > 0xFFFFFFFFull || H > 0x7FFFFFFF || W > 0x7FFFFFFF) return false;
    // Inputs under 128 KB go the explicit way: CUTLASS adjusts im2col tensor maps of such small
    // tensors on drivers up to 13.1, and nothing here needs the implicit form at that size.
    return (uint64_t)batch * cin * H * W * 2 >= (128u << 10);
}

int conv_weights_f16(const int8_t* q, const float* s, uint32_t cout, uint32_t cin, __half* w16, const LaunchEnv& env) {
    if (!q || !s || !w16) return fail(env, SDVK_E_ARG, "null pointer");
    if (cin % 64) return fail(env, SDVK_E_SHAPE, "the repacked conv weights need cin % 64 == 0");
    const uint64_t n = (uint64_t)cout * cin * 9;
    if (n == 0) return SDVK_OK;
    return launch_pdl(conv_weights_f16_kernel, dim3((uint32_t)std::min<uint64_t>((n + 255) / 256, 148ull * 16)),
                      dim3(256), 0, env, "conv_weights_f16_kernel launch", q, s, w16, cout, cin);
}

int to_channels_last_f16(const __half* x, __half* y, uint32_t batch, uint32_t C, uint32_t P, const LaunchEnv& env) {
    if (!x || !y) return fail(env, SDVK_E_ARG, "null pointer");
    if (batch == 0 || C == 0 || P == 0) return SDVK_OK;
    if (batch > 65535 || (C + 31) / 32 > 65535) return fail(env, SDVK_E_SHAPE, "too many images or channels");
    return launch_pdl(channels_last_kernel, dim3((P + 31) / 32, (C + 31) / 32, batch), dim3(32, 8), 0, env,
                      "channels_last_kernel launch", x, y, C, P);
}

int conv3x3_implicit(const ConvImplicitDesc& d, const LaunchEnv& env) {
    int off = d.off;
    if (int rc = check_conv(d.x, SDVK_F16, d.w16, d.y, d.y_dtype, d.accumulate, d.stride, off, env)) return rc;
    if (d.batch == 0 || d.cout == 0 || d.H == 0 || d.W == 0) return SDVK_OK;
    if (d.batch > 0x7FFFFFFFu || d.cout > 0xFFFFu * 256)
        return fail(env, SDVK_E_SHAPE, "too many images or output channels");
    if (!conv_implicit_ok(d.batch, d.cin, d.H, d.W, d.stride))
        return fail(env, SDVK_E_SHAPE,
                    "the implicit conv needs cin % 64 == 0, OH*OW % 128 == 0 and an input of at least 128 KB");
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (!a16(d.x) || !a16(d.w16) || !a16(d.y)) return fail(env, SDVK_E_SHAPE, "operands must be 16-byte aligned");
    ConvImplicitDesc e = d;
    e.off = off;
    const uint32_t OH = d.stride == 1 ? d.H : d.H / 2, OW = d.stride == 1 ? d.W : d.W / 2;
    const int bn = pick_conv_bn((uint64_t)d.batch * OH * OW, d.cout, env.num_sms);
    if (d.y_dtype == SDVK_F32) return launch_conv_bn<float>(e, bn, env);
    return launch_conv_bn<__half>(e, bn, env);
}

uint64_t conv3x3_workspace(uint32_t cin, uint32_t H, uint32_t W, uint32_t stride, int dtype) {
    if (stride != 1 && stride != 2) return 0;
    const uint32_t OH = stride == 1 ? H : H / 2, OW = stride == 1 ? W : W / 2;
    return (uint64_t)cin * 9 * OH * OW * dtype_size(dtype);
}

int conv3x3_q8(const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias, void* y, int y_dtype,
               uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H, uint32_t W, uint32_t stride, int off,
               void* workspace, uint64_t ws_bytes, const LaunchEnv& env) {
    if (int rc = check_conv(x, x_dtype, q, y, y_dtype, false, stride, off, env)) return rc;
    if (!s) return fail(env, SDVK_E_ARG, "null pointer");
    // The implicit form when the input is fp16, the shape is one it takes and the workspace holds x
    // channels-last and the repacked weights; the explicit form otherwise.
    const uint64_t xb = ((uint64_t)batch * cin * H * W * 2 + 255) & ~uint64_t(255), wb = (uint64_t)cout * cin * 9 * 2;
    if (x_dtype == SDVK_F16 && cout > 0 && conv_implicit_ok(batch, cin, H, W, stride) && workspace &&
        (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0 && ws_bytes >= xb + wb &&
        (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0) {
        __half* xcl = static_cast<__half*>(workspace);
        __half* w16 = reinterpret_cast<__half*>(static_cast<uint8_t*>(workspace) + xb);
        if (int rc = to_channels_last_f16(static_cast<const __half*>(x), xcl, batch, cin, H * W, env)) return rc;
        if (int rc = conv_weights_f16(q, s, cout, cin, w16, env)) return rc;
        ConvImplicitDesc d{xcl, w16, bias, 0, false, y, y_dtype, batch, cin, cout, H, W, stride, off};
        return conv3x3_implicit(d, env);
    }
    return conv3x3_q8_ex(x, x_dtype, q, s, bias, 0, false, y, y_dtype, batch, cin, cout, H, W, stride, off, workspace,
                         ws_bytes, env);
}

int conv3x3_q8_ex(const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias, uint64_t bias_stride,
                  bool accumulate, void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H,
                  uint32_t W, uint32_t stride, int off, void* workspace, uint64_t ws_bytes, const LaunchEnv& env) {
    if (int rc = check_conv(x, x_dtype, q, y, y_dtype, accumulate, stride, off, env)) return rc;
    if (!s) return fail(env, SDVK_E_ARG, "null pointer");
    if (batch == 0 || cout == 0 || H == 0 || W == 0) return SDVK_OK;
    const uint32_t K = cin * 9;
    if (cin == 0 || K % 32) return fail(env, SDVK_E_SHAPE, "conv needs cin*9 % 32 == 0 (whole Q8_0 blocks)");
    const uint32_t OH = stride == 1 ? H : H / 2, OW = stride == 1 ? W : W / 2;
    if (OH == 0 || OW == 0) return SDVK_OK;
    const uint64_t P = (uint64_t)OH * OW, es = dtype_size(x_dtype);
    // Bands of output rows: a band's column matrix (pitch rows*OW elements, a multiple of 8 so that
    // the GEMM's TMA rows and every band's output columns start 16-byte aligned) must fit the
    // workspace.  The last band may be shorter; it keeps the pitch.
    const uint64_t row_bytes = (uint64_t)K * OW * es;
    uint32_t rows = (uint32_t)std::min<uint64_t>(OH, workspace ? ws_bytes / row_bytes : 0);
    while (rows > 0 && ((uint64_t)rows * OW) % 8 && rows < OH) --rows;
    if (rows < OH && ((uint64_t)rows * OW) % 8) rows = 0;
    if (rows == 0 || (reinterpret_cast<uintptr_t>(workspace) & 15u))
        return fail(env, SDVK_E_ARG, "conv workspace too small for one aligned band of output rows, or misaligned");
    const uint64_t pitch = (uint64_t)rows * OW;
    const uint64_t xs = (uint64_t)cin * H * W * es, ys = (uint64_t)cout * P * dtype_size(y_dtype);
    if (rows == OH && batch > 1 && ws_bytes / ((uint64_t)K * P * es) >= batch && P % 8 == 0) {
        // Every image's column matrix fits: one im2col launch over the images and one batched GEMM
        // (image z's columns at z*K*P, its output at z*cout*P, its bias at z*bias_stride).
        const uint64_t xbe = (uint64_t)cin * H * W, cbe = (uint64_t)K * P;
        int rc = im2col_any(x, x_dtype, workspace, cin, H, W, OW, 0u, OH, P, stride, off, batch, xbe, cbe, env);
        if (rc) return rc;
        GemmQ8Desc d{};
        d.x = workspace;
        d.x_dtype = x_dtype;
        d.ldx = P;
        d.sx = cbe;
        d.wq = q;
        d.ws = s;
        d.ldw = K;
        d.bias = bias;
        d.sbias = bias ? bias_stride : 0;
        d.c = y;
        d.c_dtype = y_dtype;
        d.ldc = P;
        d.sc = (uint64_t)cout * P;
        d.xrows = (uint32_t)P;
        d.wrows = cout;
        d.K = K;
        d.batch = batch;
        d.nn = true;
        d.accumulate = accumulate;
        return gemm_q8(d, env);
    }
    for (uint32_t bi = 0; bi < batch; ++bi) {
        const uint8_t* xb = static_cast<const uint8_t*>(x) + bi * xs;
        uint8_t* yb = static_cast<uint8_t*>(y) + bi * ys;
        for (uint32_t r0 = 0; r0 < OH; r0 += rows) {
            const uint32_t rr = std::min(rows, OH - r0), np = rr * OW;
            int rc = im2col_any(xb, x_dtype, workspace, cin, H, W, OW, r0, rr, pitch, stride, off, 1u, 0, 0, env);
            if (rc) return rc;
            GemmQ8Desc d{};
            d.x = workspace;
            d.x_dtype = x_dtype;
            d.ldx = pitch;
            d.wq = q;
            d.ws = s;
            d.ldw = K;
            d.bias = bias ? bias + (uint64_t)bi * bias_stride : nullptr;
            d.accumulate = accumulate;
            d.c = yb + (uint64_t)r0 * OW * dtype_size(y_dtype);
            d.c_dtype = y_dtype;
            d.ldc = P;
            d.xrows = np;
            d.wrows = cout;
            d.K = K;
            d.batch = 1;
            d.nn = true;
            if ((rc = gemm_q8(d, env))) return rc;
        }
    }
    return SDVK_OK;
}

}  // namespace sdvk
