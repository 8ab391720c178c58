// sampler.cu -- the sampler step on the device: the reference's per-evaluation host loop of the
// generation pass (src/Modules/Diffusion/sdvkgen.cpp:3759-4021) without the host round trip.
// Per model evaluation, in the reference's order and rounding:
//   evalGuided   non-finite check of the model outputs (:3819-3823), the guidance combine
//                res = u + cfg * (c - u) (:3825-3826) and the optional spread rescale (:3829-3844)
//   x0FromEps    eps- or v-prediction x0 estimate (:3770-3776)
//   finishX0     dynamic threshold at the 99.5th percentile of |x0| (:3779-3784) and the inpaint
//                mask blend toward the init latent (:3788-3793)
//   the update   Euler, Euler a, Heun, LMS, DPM2, DPM2 a, DPM++ 2M, DPM++ 2S a, DDIM (:3859-4019),
//                and the next evaluation's scaled model input x / sqrt(sigma^2 + 1) (:3808-3809)
// Every fp32 operation is separately rounded (explicit _rn intrinsics: no contraction into FMA)
// and mixed float/double expressions keep the reference's types, so the results equal the host
// loop's bit for bit; only the rescale's double-precision sums are added in another order (a
// fixed tree), which can move a result by an ulp.  The scalar coefficients (sigma_up, sigma_down,
// expm1(-h), the DPM++ ratios) are computed on the host in the reference's expressions.
//
// Launches per evaluation: the guide pass (non-finite check, combine, x0) and the update pass, with
// the rescale's two statistics passes and the threshold's one-CTA select between them when those
// options are on.  Each elementwise pass gives one latent element to a thread (the SDXL 1024^2
// latent is 4 x 128 x 128 = 65536 floats, 256 CTAs), so a pass is one memory round trip; the
// whole-array statistics go through per-CTA partial sums in a small context workspace, reduced in a
// fixed order so every run and every CTA gets the same value.  A non-finite model output sets a bit
// in the context's error word, which the update pass reads: the latent is left as it was and the
// next synchronising call reports SDVK_E_NOT_FINITE.
#include <algorithm>
#include <cmath>

#include "backend.hpp"
#include "ptx.cuh"

namespace sdvk {
namespace {

constexpr int kPassThreads = 256;   // the elementwise passes
constexpr int kSelThreads = 1024;   // the threshold's radix select

struct SampParams {
    uint64_t n;
    // guidance and x0 of this evaluation
    const float* eps_c;
    const float* eps_u;   // null: guidance off
    const float* x_eval;  // the latent this evaluation's model input was scaled from
    float cfg, rescale;
    float sig;            // this evaluation's sigma (x0FromEps)
    float s2;             // sig * sig + 1
    float neg_sig_root;   // -sig / sqrt(s2)  (v-prediction)
    int vpred, dynthresh;
    uint64_t q;           // dynthresh: the order statistic's index, (n - 1) * 0.995
    const float* mask;
    uint64_t mask_cells;
    const float* init_lat;
    float* x0;            // out: this evaluation's finished x0
    float* thr_out;
    // the update
    int kind, phase, last;
    float* lat;
    float* x_tmp;
    const float* x0v;     // phase 1: the step's first x0
    float* x0_prev;
    float* lms0;
    const float* lms1;
    const float* lms2;
    const float* lms3;
    int lms_count;
    float cf0, cf1, cf2, cf3;
    const float* noise;
    float a, b, c;        // per-sampler coefficients (see the host side)
    double em1;           // DPM++: expm1(-h)
    float c0, c1;         // DPM++ with history
    int have_prev;
    float* x_model;
    float model_inv;
    uint32_t* err;
    double* ws;           // 3 x G partial sums, then the threshold
};

__device__ __forceinline__ float fadd(float x, float y) { return __fadd_rn(x, y); }
__device__ __forceinline__ float fsub(float x, float y) { return __fsub_rn(x, y); }
__device__ __forceinline__ float fmul(float x, float y) { return __fmul_rn(x, y); }
__device__ __forceinline__ float fdiv(float x, float y) { return __fdiv_rn(x, y); }

// x0FromEps (sdvkgen.cpp:3770-3776)
__device__ __forceinline__ float x0_from_eps(const SampParams& p, float x, float e) {
    return p.vpred ? fadd(fmul(e, p.neg_sig_root), fdiv(x, p.s2)) : fsub(x, fmul(p.sig, e));
}

// finishX0's per-element part (sdvkgen.cpp:3786-3795)
__device__ __forceinline__ float finish_x0(const SampParams& p, uint64_t k, float v, float thr) {
    if (p.dynthresh) v = fdiv(fminf(fmaxf(v, -thr), thr), thr);
    if (p.mask) {
        const float m = p.mask[k % p.mask_cells];
        v = fadd(fmul(m, v), fmul(fsub(1.0f, m), p.init_lat[k]));
    }
    return v;
}

// The update of one element from the evaluation's x0 (sdvkgen.cpp:3859-4019).  Writes the step's
// outputs for index k.
__device__ __forceinline__ void update_elem(const SampParams& p, uint64_t k, float x0) {
    const float lat = p.lat[k];
    float out;
    bool to_tmp = false;
    if (p.last) {
        out = p.phase == 0 ? x0 : p.x0v[k];
    } else {
        switch (p.kind) {
            case SDVK_SAMPLER_EULER_A:  // lat + (lat - x0) * (ratio - 1) + noise * sigma_up
                out = fadd(fadd(lat, fmul(fsub(lat, x0), p.a)), fmul(p.noise[k], p.b));
                break;
            case SDVK_SAMPLER_HEUN:
                if (p.phase == 0) {  // x_tmp = lat + (lat - x0) / sigma * dt
                    out = fadd(lat, fmul(fdiv(fsub(lat, x0), p.a), p.b));
                    to_tmp = true;
                } else {  // lat + 0.5 * ((lat - x0v) / sigma + (x_tmp - x0b) / sigma_next) * dt
                    const float d1 = fdiv(fsub(lat, p.x0v[k]), p.a);
                    const float d2 = fdiv(fsub(p.x_tmp[k], x0), p.b);
                    out = fadd(lat, fmul(fmul(0.5f, fadd(d1, d2)), p.c));
                }
                break;
            case SDVK_SAMPLER_LMS: {  // derivative history, newest first; lat + dt * sum cf[j] d[j]
                const float d = fdiv(fsub(lat, x0), p.a);
                p.lms0[k] = d;
                float acc = fadd(0.0f, fmul(p.cf0, d));
                if (p.lms_count > 1) acc = fadd(acc, fmul(p.cf1, p.lms1[k]));
                if (p.lms_count > 2) acc = fadd(acc, fmul(p.cf2, p.lms2[k]));
                if (p.lms_count > 3) acc = fadd(acc, fmul(p.cf3, p.lms3[k]));
                out = fadd(lat, fmul(p.b, acc));
                break;
            }
            case SDVK_SAMPLER_DPM2:
            case SDVK_SAMPLER_DPM2_A:
                if (p.phase == 0) {  // x_tmp = lat + (lat - x0) / sigma * half_step
                    out = fadd(lat, fmul(fdiv(fsub(lat, x0), p.a), p.b));
                    to_tmp = true;
                } else {  // lat + (x_tmp - x0b) / sigma_mid * step [+ noise * sigma_up]
                    out = fadd(lat, fmul(fdiv(fsub(p.x_tmp[k], x0), p.a), p.b));
                    if (p.kind == SDVK_SAMPLER_DPM2_A) out = fadd(out, fmul(p.noise[k], p.c));
                }
                break;
            case SDVK_SAMPLER_DPMPP_2M:
            case SDVK_SAMPLER_DPMPP_2S_A: {  // ratio * lat - expm1(-h) * x0d, the difference in double
                const float x0d = p.have_prev ? fsub(fmul(p.c0, x0), fmul(p.c1, p.x0_prev[k])) : x0;
                out = (float)__dsub_rn((double)fmul(p.a, lat), __dmul_rn(p.em1, (double)x0d));
                if (p.kind == SDVK_SAMPLER_DPMPP_2S_A) out = fadd(out, fmul(p.noise[k], p.b));
                p.x0_prev[k] = x0;
                break;
            }
            case SDVK_SAMPLER_DDIM:  // x0 + ratio * (lat - x0)
                out = fadd(x0, fmul(p.a, fsub(lat, x0)));
                break;
            default:  // Euler: lat + (lat - x0) / sigma * dt
                out = fadd(lat, fmul(fdiv(fsub(lat, x0), p.a), p.b));
                break;
        }
    }
    if (to_tmp) p.x_tmp[k] = out;
    else p.lat[k] = out;
    if (p.x_model) p.x_model[k] = fmul(out, p.model_inv);
}

// The passes run over the whole GPU, one element per thread (grid-stride beyond G x 256).  The
// whole-array steps sit between launches: the rescale's sums are per-CTA partials that every CTA of
// the next pass reduces in the same fixed order, and the threshold's order statistic is one CTA's
// radix select.
__device__ __forceinline__ uint64_t elem0() { return (uint64_t)blockIdx.x * kPassThreads + threadIdx.x; }
__device__ __forceinline__ uint64_t elem_step() { return (uint64_t)gridDim.x * kPassThreads; }

// Sum of the G partials [part + i * stride], the same fixed order in every CTA (each lane of warp 0
// adds a strided subset in sequence, then a fixed butterfly); the result in every thread.
__device__ double reduce_partials(const double* part, uint32_t G, double* red) {
    if (threadIdx.x < 32) {
        double a = 0.0;
        for (uint32_t i = threadIdx.x; i < G; i += 32) a = __dadd_rn(a, part[i]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) a = __dadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (threadIdx.x == 0) red[0] = a;
    }
    __syncthreads();
    const double r = red[0];
    __syncthreads();
    return r;
}

// Block sum of two doubles (fixed shuffle tree, then the warps' totals in a fixed tree), to thread 0.
__device__ void block_sum2_to0(double& a, double& b, double* red) {
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        a = __dadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        b = __dadd_rn(b, __shfl_xor_sync(0xffffffffu, b, o));
    }
    if (lane == 0) red[warp] = a, red[8 + warp] = b;
    __syncthreads();
    if (threadIdx.x == 0) {
        a = red[0], b = red[8];
        for (int w = 1; w < kPassThreads / 32; ++w) a = __dadd_rn(a, red[w]), b = __dadd_rn(b, red[8 + w]);
    }
    __syncthreads();
}

// Pass 1: finiteness, the guidance combine, then x0 (or, with rescale, the combine and its sums).
__global__ void __launch_bounds__(kPassThreads) samp_guide_kernel(const SampParams p) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ double red[16];
    const bool guided = p.eps_u != nullptr;
    const bool rescale = guided && p.rescale > 0.0f;
    bool bad = false;
    double msum = 0.0, u2 = 0.0;
    for (uint64_t k = elem0(); k < p.n; k += elem_step()) {
        const float c = p.eps_c[k];
        const float u = guided ? p.eps_u[k] : 0.0f;
        bad |= !isfinite(c) || (guided && !isfinite(u));
        const float r = guided ? fadd(u, fmul(p.cfg, fsub(c, u))) : c;
        if (rescale) {
            p.x0[k] = r;
            msum = __dadd_rn(msum, (double)r);
            u2 = __dadd_rn(u2, __dmul_rn((double)u, (double)u));
        } else {
            const float x0 = x0_from_eps(p, p.x_eval[k], r);
            p.x0[k] = p.dynthresh ? x0 : finish_x0(p, k, x0, 1.0f);
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(p.err, kErrNotFinite);  // the update skips
    if (rescale) {
        block_sum2_to0(msum, u2, red);
        if (threadIdx.x == 0) p.ws[blockIdx.x] = msum, p.ws[gridDim.x + blockIdx.x] = u2;
    }
}

// Rescale, pass 2: the mean from the partial sums, then this CTA's share of sum (res - mean)^2.
__global__ void __launch_bounds__(kPassThreads) samp_rescale_stats_kernel(const SampParams p) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ double red[16];
    const double m = reduce_partials(p.ws, gridDim.x, red) / (double)p.n;
    double s2 = 0.0, unused = 0.0;
    for (uint64_t k = elem0(); k < p.n; k += elem_step()) {
        const double d = __dsub_rn((double)p.x0[k], m);
        s2 = __dadd_rn(s2, __dmul_rn(d, d));
    }
    block_sum2_to0(s2, unused, red);
    if (threadIdx.x == 0) p.ws[2 * gridDim.x + blockIdx.x] = s2;
}

// Rescale, pass 3: er = (res - m) * (su / sg) + m, res = rescale * er + (1 - rescale) * res, then x0.
__global__ void __launch_bounds__(kPassThreads) samp_rescale_apply_kernel(const SampParams p) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ double red[16];
    const uint32_t G = gridDim.x;
    const double m = reduce_partials(p.ws, G, red) / (double)p.n;
    const double u2 = reduce_partials(p.ws + G, G, red);
    const double s2 = reduce_partials(p.ws + 2 * G, G, red);
    const double su = sqrt(u2 / (double)p.n);
    const double sg = __dadd_rn(sqrt(s2 / (double)p.n), 1e-6);
    const double f = su / sg;
    const double keep = 1.0 - (double)p.rescale;
    for (uint64_t k = elem0(); k < p.n; k += elem_step()) {
        const float r = p.x0[k];
        const float er = (float)__dadd_rn(__dmul_rn(__dsub_rn((double)r, m), f), m);
        const float rr = (float)__dadd_rn((double)fmul(p.rescale, er), __dmul_rn(keep, (double)r));
        const float x0 = x0_from_eps(p, p.x_eval[k], rr);
        p.x0[k] = p.dynthresh ? x0 : finish_x0(p, k, x0, 1.0f);
    }
}

// Dynamic threshold: the q-th smallest |x0| by a 4 x 8-bit radix select on its bits, one CTA;
// thr = max(that, 1) into the workspace's last slot.
__global__ void __launch_bounds__(kSelThreads) samp_select_kernel(const SampParams p, uint32_t G) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sel[2];
    const uint32_t tid = threadIdx.x;
    uint32_t prefix = 0, pmask = 0;
    uint64_t rank = p.q;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (uint32_t i = tid; i < 256; i += kSelThreads) hist[i] = 0;
        __syncthreads();
        for (uint64_t k = tid; k < p.n; k += kSelThreads) {
            const uint32_t bits = __float_as_uint(p.x0[k]) & 0x7fffffffu;
            if ((bits & pmask) == prefix) atomicAdd(&hist[(bits >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t bin = 0;
            uint64_t below = 0;
            while (bin < 255 && below + hist[bin] <= rank) below += hist[bin++];
            sel[0] = bin;
            sel[1] = (uint32_t)(rank - below);
        }
        __syncthreads();
        prefix |= sel[0] << shift;
        pmask |= 255u << shift;
        rank = sel[1];
        __syncthreads();
    }
    if (tid == 0) reinterpret_cast<float*>(p.ws + 3 * G)[0] = fmaxf(__uint_as_float(prefix), 1.0f);
}

// Last pass: the threshold and inpaint blend (when deferred), then the sampler update.  Nothing is
// written after a non-finite model output (the context's error word says so until it is collected).
__global__ void __launch_bounds__(kPassThreads) samp_update_kernel(const SampParams p, uint32_t G) {
    grid_dependency_wait();
    grid_launch_dependents();
    if (*reinterpret_cast<volatile uint32_t*>(p.err) & kErrNotFinite) return;
    const float thr = p.dynthresh ? reinterpret_cast<const float*>(p.ws + 3 * G)[0] : 1.0f;
    if (p.thr_out && blockIdx.x == 0 && threadIdx.x == 0) *p.thr_out = thr;
    for (uint64_t k = elem0(); k < p.n; k += elem_step()) {
        float x0 = p.x0[k];
        if (p.dynthresh) {
            x0 = finish_x0(p, k, x0, thr);
            p.x0[k] = x0;
        }
        update_elem(p, k, x0);
    }
}

// The next evaluation's model input alone: x * 1/sqrt(sigma^2 + 1) (sdvkgen.cpp:3808-3809).
__global__ void __launch_bounds__(256) sampler_scale_kernel(const float* __restrict__ x, float* __restrict__ out,
                                                            uint64_t n, float inv) {
    grid_dependency_wait();
    grid_launch_dependents();
    for (uint64_t k = blockIdx.x * 256ull + threadIdx.x; k < n; k += (uint64_t)gridDim.x * 256)
        out[k] = __fmul_rn(x[k], inv);
}

// ancestralSigma (sdvkgen.cpp:2809-2813), in float as the reference computes it.
float ancestral_sigma(float s_down, float sigma, float eta) {
    if (sigma <= 0.0f) return 0.0f;
    const float inside = s_down * s_down * (sigma * sigma - s_down * s_down) / (sigma * sigma);
    return eta * std::sqrt(std::max(0.0f, inside));
}

float model_inv(float sigma) { return 1.0f / std::sqrt(sigma * sigma + 1.0f); }

}  // namespace

uint32_t sampler_grid(uint64_t n, int num_sms) {
    return (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>((n + kPassThreads - 1) / kPassThreads, 4ull * num_sms));
}

uint64_t sampler_workspace(int num_sms) { return (3ull * 4 * std::max(num_sms, 1) + 2) * sizeof(double); }

int sampler_step(const sdvk_sampler_step_desc& d, void* ws, uint64_t ws_bytes, const LaunchEnv& env) {
    if (d.n == 0) return SDVK_OK;
    if (!ws || ws_bytes < sampler_workspace(env.num_sms)) return fail(env, SDVK_E_ARG, "sampler step: workspace");
    if (!d.eps_c || !d.lat || !d.x0) return fail(env, SDVK_E_ARG, "sampler step: null eps_c, lat or x0");
    if (d.kind < SDVK_SAMPLER_EULER || d.kind > SDVK_SAMPLER_DDIM) return fail(env, SDVK_E_ARG, "unknown sampler kind");
    const bool two_eval =
        d.kind == SDVK_SAMPLER_HEUN || d.kind == SDVK_SAMPLER_DPM2 || d.kind == SDVK_SAMPLER_DPM2_A;
    if (d.phase != 0 && !(d.phase == 1 && two_eval))
        return fail(env, SDVK_E_ARG, "sampler step: phase 1 exists for Heun, DPM2 and DPM2 a only");
    if (d.mask && (!d.init_lat || d.mask_cells == 0)) return fail(env, SDVK_E_ARG, "mask needs init_lat and cells");
    if (!(d.sigma > 0.0f)) return fail(env, SDVK_E_ARG, "sampler step: sigma must be positive");
    const bool last = d.sigma_next <= 0.0f;
    if (d.phase == 1 && last) return fail(env, SDVK_E_ARG, "sampler step: the last step has no second evaluation");
    const bool ancestral = d.kind == SDVK_SAMPLER_EULER_A || d.kind == SDVK_SAMPLER_DPM2_A ||
                           d.kind == SDVK_SAMPLER_DPMPP_2S_A;
    const bool dpmpp = d.kind == SDVK_SAMPLER_DPMPP_2M || d.kind == SDVK_SAMPLER_DPMPP_2S_A;
    if (!last) {
        if (ancestral && !d.noise && (d.kind != SDVK_SAMPLER_DPM2_A || d.phase == 1))
            return fail(env, SDVK_E_ARG, "ancestral sampler step needs noise");
        if (two_eval && !d.x_tmp) return fail(env, SDVK_E_ARG, "two-evaluation sampler needs x_tmp");
        if (d.phase == 1 && !d.x0v) return fail(env, SDVK_E_ARG, "phase 1 needs the first evaluation's x0");
        if (dpmpp && !d.x0_prev) return fail(env, SDVK_E_ARG, "DPM++ sampler needs x0_prev");
        if (d.kind == SDVK_SAMPLER_LMS) {
            if (d.lms_count < 1 || d.lms_count > 4) return fail(env, SDVK_E_ARG, "LMS history count must be 1..4");
            for (int j = 0; j < d.lms_count; ++j)
                if (!d.lms[j]) return fail(env, SDVK_E_ARG, "LMS history buffer missing");
        }
    }
    SampParams p{};
    p.n = d.n;
    p.eps_c = d.eps_c;
    p.eps_u = d.eps_u;
    p.cfg = d.cfg;
    p.rescale = d.rescale;
    p.vpred = d.vpred != 0;
    p.dynthresh = d.dynthresh != 0;
    p.q = (uint64_t)((double)(d.n - 1) * 0.995);
    p.mask = d.mask;
    p.mask_cells = d.mask_cells;
    p.init_lat = d.init_lat;
    p.x0 = d.x0;
    p.thr_out = d.thr;
    p.kind = d.kind;
    p.phase = d.phase;
    p.last = last;
    p.lat = d.lat;
    p.x_tmp = d.x_tmp;
    p.x0v = d.x0v;
    p.x0_prev = d.x0_prev;
    p.noise = d.noise;
    p.err = env.err_dev;
    // the evaluation's latent and sigma, and the per-sampler coefficients, in the reference's float
    // and double expressions
    const float sigma = d.sigma, sn = d.sigma_next, dt = sn - sigma;
    const float eta = d.eta > 0 ? d.eta : 1.0f;
    float eval_sigma = sigma, next_sigma = sn;  // the sigma of this evaluation; of the next one
    p.x_eval = d.phase == 0 ? d.lat : d.x_tmp;
    if (!last) {
        switch (d.kind) {
            case SDVK_SAMPLER_EULER_A: {
                const float up = ancestral_sigma(sn, sigma, eta);
                const float down = std::sqrt(std::max(0.0f, sn * sn - up * up));
                const float ratio = down / sigma;
                p.a = ratio - 1.0f;
                p.b = up;
                break;
            }
            case SDVK_SAMPLER_HEUN:
                if (d.phase == 0) p.a = sigma, p.b = dt;
                else p.a = sigma, p.b = sn, p.c = dt, eval_sigma = sn;
                break;
            case SDVK_SAMPLER_LMS: {
                static const float coeff[4][4] = {
                    {1.0f, 0.0f, 0.0f, 0.0f},
                    {3.0f / 2.0f, -1.0f / 2.0f, 0.0f, 0.0f},
                    {23.0f / 12.0f, -16.0f / 12.0f, 5.0f / 12.0f, 0.0f},
                    {55.0f / 24.0f, -59.0f / 24.0f, 37.0f / 24.0f, -9.0f / 24.0f},
                };
                const float* cf = coeff[d.lms_count - 1];
                p.cf0 = cf[0], p.cf1 = cf[1], p.cf2 = cf[2], p.cf3 = cf[3];
                p.lms0 = d.lms[0], p.lms1 = d.lms[1], p.lms2 = d.lms[2], p.lms3 = d.lms[3];
                p.lms_count = d.lms_count;
                p.a = sigma, p.b = dt;
                break;
            }
            case SDVK_SAMPLER_DPM2: {
                const float mid = sigma + 0.5f * dt;
                if (d.phase == 0) p.a = sigma, p.b = 0.5f * dt, next_sigma = mid;
                else p.a = mid, p.b = dt, eval_sigma = mid;
                break;
            }
            case SDVK_SAMPLER_DPM2_A: {
                const float up = std::min(sn, ancestral_sigma(sn, sigma, eta));
                const float down = std::sqrt(std::max(0.0f, sn * sn - up * up));
                const float ddown = down - sigma;
                const float mid = sigma + 0.5f * ddown;
                if (d.phase == 0) p.a = sigma, p.b = 0.5f * ddown, next_sigma = mid;
                else p.a = mid, p.b = ddown, p.c = up, eval_sigma = mid;
                break;
            }
            case SDVK_SAMPLER_DPMPP_2M:
            case SDVK_SAMPLER_DPMPP_2S_A: {
                float up = 0.0f, num = sn;
                if (d.kind == SDVK_SAMPLER_DPMPP_2S_A) {
                    up = std::min(sn, ancestral_sigma(sn, sigma, eta));
                    num = std::sqrt(std::max(0.0f, sn * sn - up * up));
                }
                const double t_now = -std::log((double)sigma), t_next = -std::log((double)sn);
                const double h = t_next - t_now;
                p.a = num / sigma;
                p.b = up;
                p.em1 = std::expm1(-h);
                p.have_prev = d.have_prev != 0;
                if (p.have_prev) {
                    const double t_prev = -std::log((double)d.sigma_prev);
                    const double r = (t_now - t_prev) / h;
                    p.c0 = (float)(1.0 + 1.0 / (2.0 * r));
                    p.c1 = (float)(1.0 / (2.0 * r));
                }
                break;
            }
            case SDVK_SAMPLER_DDIM:
                p.a = sn / sigma;
                break;
            default:
                p.a = sigma, p.b = dt;
                break;
        }
    }
    {  // x0FromEps's scalars for this evaluation's sigma
        const float s2 = eval_sigma * eval_sigma + 1.0f;
        const float root = std::sqrt(s2);
        p.sig = eval_sigma;
        p.s2 = s2;
        p.neg_sig_root = -eval_sigma / root;
    }
    if (!p.x_eval) return fail(env, SDVK_E_ARG, "sampler step: phase 1 needs x_tmp");
    if (d.x_model && !last) {
        p.x_model = d.x_model;
        p.model_inv = model_inv(next_sigma);
    }
    p.ws = static_cast<double*>(ws);
    const uint32_t G = sampler_grid(d.n, env.num_sms);
    if (int rc = launch_pdl(samp_guide_kernel, dim3(G), dim3(kPassThreads), 0, env, "samp_guide_kernel launch", p))
        return rc;
    if (d.eps_u && d.rescale > 0.0f) {
        if (int rc = launch_pdl(samp_rescale_stats_kernel, dim3(G), dim3(kPassThreads), 0, env,
                                "samp_rescale_stats_kernel launch", p))
            return rc;
        if (int rc = launch_pdl(samp_rescale_apply_kernel, dim3(G), dim3(kPassThreads), 0, env,
                                "samp_rescale_apply_kernel launch", p))
            return rc;
    }
    if (p.dynthresh) {
        if (int rc = launch_pdl(samp_select_kernel, dim3(1), dim3(kSelThreads), 0, env, "samp_select_kernel launch",
                                p, G))
            return rc;
    }
    return launch_pdl(samp_update_kernel, dim3(G), dim3(kPassThreads), 0, env, "samp_update_kernel launch", p, G);
}

int sampler_scale(const float* x, float* out, uint64_t n, float sigma, const LaunchEnv& env) {
    if (n == 0) return SDVK_OK;
    if (!x || !out) return fail(env, SDVK_E_ARG, "null pointer");
    const uint64_t blocks = std::min<uint64_t>((n + 255) / 256, 4ull * env.num_sms);
    return launch_pdl(sampler_scale_kernel, dim3((uint32_t)blocks), dim3(256), 0, env, "sampler_scale_kernel launch",
                      x, out, n, model_inv(sigma));
}

}  // namespace sdvk
