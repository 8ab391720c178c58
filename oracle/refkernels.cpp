// refkernels.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h for who may load it and why).
//
// CPU restatements of the remaining kernels of the reference's kernel table that its UNet walker,
// its sampler loop and its attention fallback dispatch (src/Modules/GPU/vk_engine.cpp:51-125):
// the elementwise, layout and convolution-helper shaders plus the fp32 GEMMs.  Each function keeps
// its shader's 32-bit unsigned index arithmetic and its per-element operation order; like
// oracle.cpp this file is compiled with -ffp-contract=off, with fmaf() exactly where a shader
// accumulates `acc += a * b`.  File paths are relative to the sdvk project root.
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "oracle.h"

extern "C" {

// add2.comp:11-14 -- c[i] = a[i] + b[i] for i < n.
void orc_add2_shader(float* c, const float* a, const float* b, uint32_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) c[i] = a[i] + b[i];
}

// bias_add.comp:11-14 -- x[i] += b[i / P] over a [C][P] tensor, in place.
void orc_bias_add_shader(float* x, const float* b, uint32_t C, uint32_t P) {
    const uint32_t n = C * P;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) x[i] += b[(uint32_t)i / P];
}

// copy_nd.comp:20-30 -- i decomposes over d0..d3 (c0 fastest); dst[sum c*os] = scale * src[sum c*ss]
// (mode 0) or += (mode 1).  Source and destination may alias element for element (the reference's
// in-place scale), so each i reads before it writes.
void orc_copy_nd_shader(float* d, const float* s, const orc_pnd* p) {
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)p->n; ++ii) {
        const uint32_t i = (uint32_t)ii;
        const uint32_t c0 = i % p->d0;
        uint32_t t = i / p->d0;
        const uint32_t c1 = t % p->d1;
        t /= p->d1;
        const uint32_t c2 = t % p->d2;
        t /= p->d2;
        const uint32_t c3 = t;
        const uint32_t so = p->ss0 * c0 + p->ss1 * c1 + p->ss2 * c2 + p->ss3 * c3;
        const uint32_t dof = p->os0 * c0 + p->os1 * c1 + p->os2 * c2 + p->os3 * c3;
        const float v = p->scale * s[so];
        if (p->mode == 0u) d[dof] = v;
        else d[dof] += v;
    }
}

// ew2.comp:19-28 -- c[i] = a[ai] + b[bi] (mode 0) or a[ai] * b[bi] (mode 1), c contiguous.
void orc_ew2_shader(float* c, const float* a, const float* b, const orc_pew2* p) {
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)p->n; ++ii) {
        const uint32_t i = (uint32_t)ii;
        const uint32_t c0 = i % p->d0;
        uint32_t t = i / p->d0;
        const uint32_t c1 = t % p->d1;
        t /= p->d1;
        const uint32_t c2 = t % p->d2;
        t /= p->d2;
        const uint32_t c3 = t;
        const uint32_t ai = p->as0 * c0 + p->as1 * c1 + p->as2 * c2 + p->as3 * c3;
        const uint32_t bi = p->bs0 * c0 + p->bs1 * c1 + p->bs2 * c2 + p->bs3 * c3;
        c[i] = (p->mode == 0u) ? (a[ai] + b[bi]) : (a[ai] * b[bi]);
    }
}

// unary_fwd.comp:11-36 -- mode 0 tanh-GELU (stable tanh from one exponential), 1 sigmoid, 2 SiLU,
// 3 quick GELU (x * sigmoid(1.702 x)), otherwise erf GELU with Abramowitz & Stegun 7.1.26.  The
// GLSL literals are single precision.
void orc_unary_shader(const float* x, float* y, uint32_t n, uint32_t mode) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        const float v = x[i];
        float r;
        if (mode == 0u) {
            const float t = 0.7978845608028654f * (v + 0.044715f * v * v * v);
            const float e = std::exp(-2.0f * std::fabs(t));
            float th = (1.0f - e) / (1.0f + e);
            if (t < 0.0f) th = -th;
            r = 0.5f * v * (1.0f + th);
        } else if (mode == 1u) {
            r = 1.0f / (1.0f + std::exp(-v));
        } else if (mode == 2u) {
            r = v / (1.0f + std::exp(-v));
        } else if (mode == 3u) {
            r = v / (1.0f + std::exp(-1.702f * v));
        } else {
            const float xs = v * 0.70710678118654752440f;
            const float ax = std::fabs(xs);
            const float t = 1.0f / (1.0f + 0.3275911f * ax);
            const float poly =
                (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
            const float e = 1.0f - poly * std::exp(-ax * ax);
            const float erf = xs >= 0.0f ? e : -e;
            r = 0.5f * v * (1.0f + erf);
        }
        y[i] = r;
    }
}

// upsample2x.comp:12-19 -- nearest 2x, [C][H][W] -> [C][2H][2W].
void orc_upsample2x_shader(const float* x, float* y, uint32_t C, uint32_t H, uint32_t W) {
    const uint32_t W2 = W * 2u, H2 = H * 2u, n = C * W2 * H2;
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        const uint32_t i = (uint32_t)ii;
        const uint32_t c = i / (W2 * H2);
        const uint32_t r = i - c * (W2 * H2);
        const uint32_t oh = r / W2;
        const uint32_t ow = r - oh * W2;
        y[i] = x[(c * H + oh / 2u) * W + ow / 2u];
    }
}

// im2col.comp:12-28 -- 3x3, stride 1, pad 1, output rows row0 .. row0+rows-1 of a [C][H][W] input:
// col[k * P + p], k = c*9 + ky*3 + kx, P = rows * W.
void orc_im2col_shader(const float* x, float* col, uint32_t C, uint32_t H, uint32_t W, uint32_t row0, uint32_t rows) {
    const uint32_t P = rows * W, n = C * 9u * P;
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        const uint32_t i = (uint32_t)ii;
        const uint32_t k = i / P, p = i - k * P;
        const uint32_t c = k / 9u, r = k - c * 9u;
        const uint32_t ky = r / 3u, kx = r - ky * 3u;
        const uint32_t oh = row0 + p / W, ow = p % W;
        const int ih = (int)oh + (int)ky - 1, iw = (int)ow + (int)kx - 1;
        float v = 0.0f;
        if (ih >= 0 && ih < (int)H && iw >= 0 && iw < (int)W) v = x[(c * H + (uint32_t)ih) * W + (uint32_t)iw];
        col[i] = v;
    }
}

// im2col_s2.comp:15-31 -- 3x3, stride 2 into OH x OW outputs; off = -1 pads all sides by one,
// off = 0 pads only the right/bottom edge.
void orc_im2col_s2_shader(const float* x, float* col, uint32_t C, uint32_t H, uint32_t W, uint32_t OH, uint32_t OW,
                          int32_t off) {
    const uint32_t P = OH * OW, n = C * 9u * P;
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        const uint32_t i = (uint32_t)ii;
        const uint32_t k = i / P, p = i - k * P;
        const uint32_t c = k / 9u, rr = k - c * 9u;
        const uint32_t ky = rr / 3u, kx = rr - ky * 3u;
        const uint32_t oh = p / OW, ow = p - oh * OW;
        const int ih = (int)(oh * 2u) + (int)ky + off, iw = (int)(ow * 2u) + (int)kx + off;
        float v = 0.0f;
        if (ih >= 0 && ih < (int)H && iw >= 0 && iw < (int)W) v = x[(c * H + (uint32_t)ih) * W + (uint32_t)iw];
        col[i] = v;
    }
}

// gemm_nt.comp:23-75 and gemm_nn.comp:27-84 -- fp32 C[M,N] (=|+=) A . B^T (NT) or A . B (NN),
// batched over z = 0..batch-1 with element strides sA/sB/sC.  Per output one shader thread sums
// acc += a * b over k ascending (BK = 16 tiles, k inside a tile ascending: one sequence).
// NT reads B at bo + n*K + k whatever ldb says (gemm_nt.comp:52); NN reads B at bo + k*ldb + n.
void orc_gemm_fp32_shader(int nt, const float* A, const float* B, float* C, const orc_pg* p, uint32_t batch) {
    const uint32_t M = p->M, N = p->N, K = p->K;
    const uint32_t lda = p->lda ? p->lda : K;
    const uint32_t ldb = nt ? K : (p->ldb ? p->ldb : N);
    const uint32_t ldc = p->ldc ? p->ldc : N;
    const uint32_t MB = 4, NB = 32;
    const uint32_t mblk = (M + MB - 1) / MB, nblk = (N + NB - 1) / NB;
#pragma omp parallel
    {
        std::vector<float> w((size_t)(K ? K : 1) * NB);
#pragma omp for collapse(3) schedule(dynamic)
        for (int64_t z = 0; z < (int64_t)batch; ++z)
            for (int64_t nb = 0; nb < (int64_t)nblk; ++nb)
                for (int64_t mb = 0; mb < (int64_t)mblk; ++mb) {
                    const uint32_t zo = (uint32_t)z, n0 = (uint32_t)nb * NB, m0 = (uint32_t)mb * MB;
                    const uint32_t nc = std::min(NB, N - n0), mr = std::min(MB, M - m0);
                    const uint32_t ao = zo * p->sA, bo = zo * p->sB, co = zo * p->sC;
                    for (uint32_t k = 0; k < K; ++k)
                        for (uint32_t j = 0; j < NB; ++j) {
                            float v = 0.0f;
                            if (j < nc) v = nt ? B[bo + (n0 + j) * ldb + k] : B[bo + k * ldb + n0 + j];
                            w[(size_t)k * NB + j] = v;
                        }
                    float acc[MB][NB];
                    for (uint32_t i = 0; i < MB; ++i)
                        for (uint32_t j = 0; j < NB; ++j) acc[i][j] = 0.0f;
                    for (uint32_t k = 0; k < K; ++k) {
                        const float* wk = &w[(size_t)k * NB];
                        for (uint32_t i = 0; i < mr; ++i) {
                            const float a = A[ao + (m0 + i) * lda + k];
                            for (uint32_t j = 0; j < NB; ++j) acc[i][j] = fmaf(a, wk[j], acc[i][j]);
                        }
                    }
                    for (uint32_t i = 0; i < mr; ++i)
                        for (uint32_t j = 0; j < nc; ++j) {
                            float* dst = C + co + (m0 + i) * ldc + n0 + j;
                            if (p->mode == 0u) *dst = acc[i][j];
                            else *dst += acc[i][j];
                        }
                }
    }
}

// softmax_fwd.comp:13-38 -- one 256-lane workgroup per row: the row max, then lane t sums
// exp(x - m) over j = t, t + 256, ... in order, a tree over the 256 partials (stride 128 .. 1),
// y = exp(x - m) * (1 / sum).  x and y may be the same buffer (attnCore's in-place call).
void orc_softmax_shader(const float* x, float* y, uint32_t rows, uint32_t cols) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        const float* xr = x + (size_t)r * cols;
        float* yr = y + (size_t)r * cols;
        float mx = -3.0e38f;
        for (uint32_t j = 0; j < cols; ++j) mx = std::max(mx, xr[j]);
        float red[256];
        for (uint32_t t = 0; t < 256; ++t) {
            float s = 0.0f;
            for (uint32_t j = t; j < cols; j += 256) s += std::exp(xr[j] - mx);
            red[t] = s;
        }
        for (uint32_t st = 128; st > 0; st >>= 1)
            for (uint32_t t = 0; t < st; ++t) red[t] += red[t + st];
        const float ir = 1.0f / red[0];
        for (uint32_t j = 0; j < cols; ++j) yr[j] = std::exp(xr[j] - mx) * ir;
    }
}

// causal_mask.comp:10-15 -- s[b][r][c] = -3e38 where c > r.
void orc_causal_mask_shader(float* s, uint32_t batch, uint32_t rows, uint32_t cols) {
    const uint32_t n = batch * rows * cols;
#pragma omp parallel for schedule(static)
    for (int64_t ii = 0; ii < (int64_t)n; ++ii) {
        const uint32_t i = (uint32_t)ii;
        const uint32_t r = (i / cols) % rows, c = i % cols;
        if (c > r) s[i] = -3.0e38f;
    }
}

// ------------------------------------------------------------------------------------------
// buildEuler and sigmaAt (src/Modules/Diffusion/sdvkgen.cpp:2723-2765, :2715-2721): the scaled-linear beta
// schedule, alpha_bar in double, optional zero-terminal-SNR rescale, sigma per training step in
// fp32, and the "leading" (steps_offset = offset) or "trailing" timestep spacing.  Writes steps
// timesteps and steps + 1 sigmas (the last 0); returns the initial noise sigma.
static float orc_sigma_at(const std::vector<float>& sigmaOf, float t, int numTrain) {
    if (t <= 0) return sigmaOf[0];
    if (t >= numTrain - 1) return sigmaOf[numTrain - 1];
    int i0 = (int)t;
    float fr = t - (float)i0;
    return sigmaOf[i0] * (1.0f - fr) + sigmaOf[i0 + 1] * fr;
}

float orc_euler_schedule(int steps, int trailing, int numTrain, int offset, int zsnr, float* timesteps, float* sigmas) {
    std::vector<float> betas(numTrain);
    for (int i = 0; i < numTrain; i++) {
        const float b0 = 0.00085f, b1 = 0.012f;
        const float v = std::sqrt(b0) + (std::sqrt(b1) - std::sqrt(b0)) * (float)i / (float)(numTrain - 1);
        betas[i] = v * v;
    }
    std::vector<double> ab(numTrain);
    double run = 1.0;
    for (int i = 0; i < numTrain; i++) {
        run *= (1.0 - betas[i]);
        ab[i] = run;
    }
    if (zsnr) {
        const double a0 = std::sqrt(ab[0]), aT = std::sqrt(ab[numTrain - 1]);
        for (int i = 0; i < numTrain; i++) {
            const double sc = (std::sqrt(ab[i]) - aT) * (a0 / (a0 - aT));
            ab[i] = sc * sc;
        }
        ab[numTrain - 1] = std::pow(2.0, -24.0);
    }
    std::vector<float> sigmaOf(numTrain);
    for (int i = 0; i < numTrain; i++) sigmaOf[i] = (float)std::sqrt((1.0 - ab[i]) / ab[i]);
    if (trailing) {
        const float stepRatio = (float)numTrain / (float)steps;
        for (int i = 0; i < steps; i++) timesteps[i] = std::floor((float)numTrain - (float)i * stepRatio + 0.5f) - 1.0f;
    } else {
        const int stepRatio = numTrain / steps;
        for (int i = 0; i < steps; i++) timesteps[steps - 1 - i] = (float)std::lround((float)i * stepRatio) + (float)offset;
    }
    for (int i = 0; i < steps; i++) sigmas[i] = orc_sigma_at(sigmaOf, timesteps[i], numTrain);
    sigmas[steps] = 0.0f;
    float mx = 0.0f;
    for (int i = 0; i <= steps; i++) mx = std::max(mx, sigmas[i]);
    return trailing ? mx : std::sqrt(mx * mx + 1.0f);
}

// ------------------------------------------------------------------------------------------
// The seeded parameters of sdvk_unet_init_random (sdvk_b200/csrc/unet.cu), rebuilt on the host so
// the reference's own loader can read the same UNet from a GGUF.  SplitMix64 finaliser per element;
// every step is integer arithmetic or a correctly rounded IEEE operation except the Box-Muller
// log/cos, which are evaluated in double and rounded to fp32 and then binary16 (a faithful libm
// lands on the device's binary16 value except with probability about 2^-40 per scale).
static inline uint64_t unet_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// payload bytes first .. first + n - 1 of the arena
void orc_unet_rand_q8(uint64_t seed, uint64_t first, uint64_t n, int8_t* out) {
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < (int64_t)n; ++k) {
        const uint64_t i = first + (uint64_t)k;
        out[k] = (int8_t)((int)(unet_mix64(seed ^ (i * 0xD1B54A32D192ED03ull)) % 255u) - 127);
    }
}

// scales first .. first + n - 1, counted from the first Q8 tensor's scales
void orc_unet_rand_scale(uint64_t seed, uint64_t first, uint64_t n, float* out) {
    const uint64_t key = seed ^ 0x5CA1Eull;
    const double sigma = (double)0.02f;
#pragma omp parallel for schedule(static)
    for (int64_t k = 0; k < (int64_t)n; ++k) {
        const uint64_t i = first + (uint64_t)k;
        const uint64_t h = unet_mix64(key ^ (i * 0x8CB92BA72F3D8DD7ull));
        const double u1 = ((double)(h >> 40) + 1.0) * (1.0 / 16777217.0);
        const double u2 = (double)((h >> 16) & 0xFFFFFF) * (1.0 / 16777216.0);
        const double g = std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
        const float v = (float)(std::fabs(g) * sigma / 127.0);
        uint16_t hb;
        orc_f32_to_f16(&v, &hb, 1);
        orc_f16_to_f32(&hb, &out[k], 1);
    }
}

// F32 tensor number t of the table: init 0 ones, 1 zeros, 2 uniform [-0.02, 0.02]
void orc_unet_rand_f32(uint64_t seed, uint32_t t, int init, uint64_t n, float* out) {
    const uint64_t key = seed + 1000003ull * t;
    const float v = init == 0 ? 1.0f : init == 1 ? 0.0f : 0.02f;
    for (uint64_t e = 0; e < n; ++e) {
        if (init != 2) {
            out[e] = v;
        } else {
            const uint64_t h = unet_mix64(key ^ (e * 0xA24BAED4963EE407ull));
            out[e] = v * (2.0f * (float)(h >> 40) * (1.0f / 16777216.0f) - 1.0f);
        }
    }
}

}  // extern "C"
