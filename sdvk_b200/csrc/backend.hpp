// backend.hpp -- internal interface between the C ABI (sdvk_abi.cu) and the kernel launchers.
#pragma once

#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <utility>

#include "../../include/sdvk_cuda.h"

namespace sdvk {

// What every launcher needs from the context.
struct LaunchEnv {
    cudaStream_t stream;
    uint32_t* err_dev;    // device error word the kernels OR their error codes into
    uint64_t timeout_ns;  // deadline of every bounded wait inside a kernel
    int device;
    int num_sms;
    std::string* msg;     // error text for sdvk_last_error
    int precision;        // SDVK_PRECISION_REFERENCE or SDVK_PRECISION_FAST
    cudaStream_t side;    // the context's second stream, for work that overlaps the main stream
    cudaEvent_t fork, join;
};

// One Q8_0 GEMM in kernel terms: x = activation operand, w = quantised weight operand.
//   nn == false: C[z][x][w] = sum_k X[z][x][k] * W[w][k]      (X row stride ldx)
//   nn == true:  C[z][w][x] = sum_k W[z][w][k] * X[z][k][x]   (X row stride ldx along k)
struct GemmQ8Desc {
    const void* x;
    int x_dtype;
    uint64_t ldx, sx;
    const int8_t* wq;
    const float* ws;
    uint64_t ldw, sw;
    const float* bias;  // per w row, or null
    uint64_t sbias;     // bias batch stride (elements; 0 = one bias for every batch)
    void* c;
    int c_dtype;
    uint64_t ldc, sc;
    uint32_t xrows, wrows, K, batch;
    bool nn;
    bool accumulate;
    bool geglu;  // NT, f16 output: GEGLU-interleaved weight rows, output [rows][wrows / 2]
    // The weights (payload and scales) are parameters that the kernel launched just before this GEMM
    // does not write, so the CTA-pair kernel's weight roles may start before that kernel completes.
    bool weights_static;
};

int gemm_q8(const GemmQ8Desc& d, const LaunchEnv& env);
int geglu_interleave(const int8_t* q, const float* s, const float* bias, uint32_t F, uint32_t K, int8_t* q_out,
                     float* s_out, float* bias_out, const LaunchEnv& env);
// cuTensorMapEncodeTiled from the driver (null if unavailable), and the per-device dynamic
// shared-memory opt-in for a kernel (done once per kernel and device).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();
bool kernel_smem_attr(const void* kern, int bytes, int device);
// 3-D tiled tensor map {d0 (contiguous), d1, d2} with byte strides s1, s2 and box {b0, b1, 1}
// (SDVK_E_SHAPE if the driver rejects it), and the TMA element type of an SDVK dtype.
int tiled_map_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                 uint64_t s1, uint64_t s2, uint32_t b0, uint32_t b1, CUtensorMapSwizzle sw, const LaunchEnv& env,
                 const char* what);
CUtensorMapDataType tma_dtype(int dt);
int attention(const sdvk_attn_desc& d, const LaunchEnv& env);
int layernorm(const float* x, const float* gamma, const float* beta, void* y, int y_dtype, uint32_t rows, uint32_t d,
              uint64_t ldx, uint64_t ldy, float eps, const LaunchEnv& env);
int geglu(const void* h, void* y, uint32_t rows, uint32_t F, uint64_t ldh, uint64_t ldy, const LaunchEnv& env);
uint64_t block_workspace_bytes(const sdvk_block_desc& d);
int transformer_block(const sdvk_block_desc& d, void* ws, uint64_t ws_bytes, const LaunchEnv& env);
// The block with the cross-attention's K|V already projected by the caller: kv_pre [batch][Tctx][ld_kv]
// fp16 holding this block's K at columns 0..C-1 and V at C..2C-1 (no K|V GEMM, no side-stream fork).
int transformer_block_ex(const sdvk_block_desc& d, const __half* kv_pre, uint64_t ld_kv, void* ws, uint64_t ws_bytes,
                         const LaunchEnv& env);
int static_scratch(int device, void** ptr, const LaunchEnv& env);
int cfg_combine(const float* cond, const float* uncond, float* out, uint64_t n, float cfg, float rescale,
                const LaunchEnv& env);
int comm_unique_id(void* id);
int comm_create(int nranks, int rank, const void* id, uint32_t timeout_ms, sdvk_comm** out, const LaunchEnv& env);
int comm_destroy(sdvk_comm* c);
int comm_abort(sdvk_comm* c);
int allgather(sdvk_comm* c, const void* send, void* recv, uint64_t count, int dtype, uint32_t timeout_ms,
              const LaunchEnv& env);
int comm_wait(sdvk_comm* c, uint32_t timeout_ms, const LaunchEnv& env);
uint64_t sampler_workspace(int num_sms);
int sampler_step(const sdvk_sampler_step_desc& d, void* ws, uint64_t ws_bytes, const LaunchEnv& env);
int sampler_scale(const float* x, float* out, uint64_t n, float sigma, const LaunchEnv& env);
int check_finite(const void* x, int dtype, uint64_t n, uint32_t* flag_dev, const LaunchEnv& env);

// ingest.cu: GGUF Q8_0 blocks -> (int8 payload, fp32 scales); GroupNorm (+SiLU).
int q8_0_ingest(const void* blocks, uint64_t rows, uint64_t cols, int8_t* q, uint64_t ldq, float* scales,
                const LaunchEnv& env);
uint64_t groupnorm_workspace(uint32_t batch, uint32_t C, uint32_t P, uint32_t G);
// conv.cu: 3x3 convolution with Q8_0 weights (im2col + NN GEMM).
uint64_t conv3x3_workspace(uint32_t cin, uint32_t H, uint32_t W, uint32_t stride, int dtype);
int conv3x3_q8(const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias, void* y, int y_dtype,
               uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H, uint32_t W, uint32_t stride, int off,
               void* workspace, uint64_t ws_bytes, const LaunchEnv& env);
// The same convolution with image b's bias at bias + b * bias_stride (the UNet's conv bias plus that
// image's time-embedding projection) and, with accumulate, y += conv(x) (F32 y: the residual add).
int conv3x3_q8_ex(const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias, uint64_t bias_stride,
                  bool accumulate, void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H,
                  uint32_t W, uint32_t stride, int off, void* workspace, uint64_t ws_bytes, const LaunchEnv& env);
// The implicit-GEMM form (conv_tc2.cuh): x channels-last fp16 [batch][H][W][cin], w16 the weights
// repacked by conv_weights_f16, y channel-major [batch][cout][OH][OW] in F16 or F32 (F32 to
// accumulate), image b's bias at bias + b * sbias.
struct ConvImplicitDesc {
    const __half* x;
    const __half* w16;
    const float* bias;
    uint64_t sbias;
    bool accumulate;
    void* y;
    int y_dtype;
    uint32_t batch, cin, cout, H, W, stride;
    int off;
};
// Whether conv3x3_implicit takes this shape: cin % 64 == 0, OH*OW % 128 == 0, stride 1 or 2, an input of
// at least 128 KB, and SDVK_CONV_IMPLICIT is not 0.
bool conv_implicit_ok(uint32_t batch, uint32_t cin, uint32_t H, uint32_t W, uint32_t stride);
// w16[o][(cb*9 + tap)*64 + j] = fp16(q[o][(cb*64 + j)*9 + tap] * scale), [cout][cin*9]
int conv_weights_f16(const int8_t* q, const float* s, uint32_t cout, uint32_t cin, __half* w16, const LaunchEnv& env);
int conv3x3_implicit(const ConvImplicitDesc& d, const LaunchEnv& env);
// [batch][C][P] fp16 -> [batch][P][C] fp16
int to_channels_last_f16(const __half* x, __half* y, uint32_t batch, uint32_t C, uint32_t P, const LaunchEnv& env);
int groupnorm(const float* x, const float* gamma, const float* beta, float* y, uint32_t batch, uint32_t C, uint32_t P,
              uint32_t G, float eps, uint32_t act, void* workspace, uint64_t ws_bytes, const LaunchEnv& env);
// The same GroupNorm with y in F32 or F16 (the UNet feeds the F16 form to its convolutions); with
// channels_last, y is F16 [batch][P][C] (C % 32 == 0) holding the same values.
int groupnorm_ex(const float* x, const float* gamma, const float* beta, void* y, int y_dtype, uint32_t batch,
                 uint32_t C, uint32_t P, uint32_t G, float eps, uint32_t act, void* workspace, uint64_t ws_bytes,
                 const LaunchEnv& env, bool channels_last = false);

// unet.cu: the SDXL UNet pass over the kernels above.
int unet_plan(const sdvk_unet_desc& d, sdvk_unet** out, const LaunchEnv& env);
int unet_create(const sdvk_unet_desc& d, sdvk_unet** out, const LaunchEnv& env);
int unet_destroy(sdvk_unet* u);
int unet_init_random(sdvk_unet* u, uint64_t seed, const LaunchEnv& env);
int unet_prepare(sdvk_unet* u, const LaunchEnv& env);
int unet_forward(sdvk_unet* u, const float* x, const float* timesteps, const float* adm, const void* ctx, int ctx_dtype,
                 float* out, const LaunchEnv& env);
uint64_t unet_flops(const sdvk_unet* u);
uint64_t unet_launches(const sdvk_unet* u);
uint64_t unet_workspace_bytes(const sdvk_unet* u);
uint64_t unet_parameter_bytes(const sdvk_unet* u);
int unet_tensor(const sdvk_unet* u, uint32_t i, sdvk_unet_tensor_info* out);
uint32_t unet_tensor_count(const sdvk_unet* u);
int unet_tensor_layout(const sdvk_unet* u, uint32_t i, sdvk_unet_param_layout* out);

// table.cu: the rest of the reference's kernel table, with its push-constant blocks (sdvkgen.cpp:901-907
// for Pg and Pnd, the ew2 block of mul2 :1003-1019).
struct TablePg {
    uint32_t M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, pad;
};
struct TablePnd {
    uint32_t n, d0, d1, d2, d3, os0, os1, os2, os3, ss0, ss1, ss2, ss3, mode;
    float scale;
};
struct TablePew2 {
    uint32_t n, d0, d1, d2, d3, as0, as1, as2, as3, bs0, bs1, bs2, bs3, mode;
};
int table_add2(float* c, const float* a, const float* b, uint32_t n, const LaunchEnv& env);
int table_copy_nd(float* d, const float* s, const TablePnd& p, const LaunchEnv& env);
int table_ew2(float* c, const float* a, const float* b, const TablePew2& p, const LaunchEnv& env);
int table_unary(const float* x, float* y, uint32_t n, uint32_t mode, const LaunchEnv& env);
int table_bias_add(float* x, const float* b, uint32_t C, uint32_t P, const LaunchEnv& env);
int table_upsample2x(const float* x, float* y, uint32_t C, uint32_t H, uint32_t W, const LaunchEnv& env);
// stride2 = false: im2col (a = row0, b = rows); true: im2col_s2 (a = OH, b = OW, off)
int table_im2col(const float* x, float* col, uint32_t C, uint32_t H, uint32_t W, uint32_t a, uint32_t b, int off,
                 bool stride2, const LaunchEnv& env);
int table_gemm_fp32(bool nt, const float* A, const float* B, float* C, const TablePg& p, uint32_t batch,
                    const LaunchEnv& env);
int table_softmax(const float* x, float* y, uint32_t rows, uint32_t cols, const LaunchEnv& env);
int table_causal_mask(float* s, uint32_t batch, uint32_t rows, uint32_t cols, const LaunchEnv& env);

inline int dtype_size(int dt) { return dt == SDVK_F32 ? 4 : (dt == SDVK_F16 || dt == SDVK_BF16) ? 2 : 0; }

inline int fail(const LaunchEnv& env, int code, const std::string& what) {
    if (env.msg) *env.msg = what;
    return code;
}

inline int cuda_check(const LaunchEnv& env, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return SDVK_OK;
    return fail(env, SDVK_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Programmatic dependent launch (SDVK_PDL=0 turns it off): a kernel launched this way may start
// its prologue while the previous kernel on the stream finishes; every kernel launched through
// launch_pdl touches global memory only after griddepcontrol.wait (grid_dependency_wait), which
// returns once the previous grid has completed and its writes are visible.
bool pdl_enabled();

template <class... KArgs, class... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, const LaunchEnv& env, const char* what,
               Args&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = env.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_check(env, cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...), what);
}

}  // namespace sdvk
