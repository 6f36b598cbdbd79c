// troncons_b200 — the attention side of a gpt-oss layer at batch 1: Q8_0 GEMV, RMSNorm, YaRN
// rotation, KV-cache write, attention of one position with sinks and the sliding window (the
// reference's passe.cuh kernels gemv_q8_0, rmsnorm, rope_yarn, ecrire_kv, attention, launched by
// `Noyaux` in trc-noyaux/src/lib.rs:291-381).
//
// Each kernel keeps the reference's arithmetic order, element by element, so that its outputs
// are bit-identical to the reference kernels' on the same GPU (the same CUDA math functions,
// called, not restated); the memory side is this library's own:
//   k_gemv_q8_0   persistent warps stage rows of 34-byte blocks (C/32 of them, rows 2-aligned
//                 only) with coalesced 16-byte cp.async into shared memory, the next row while
//                 the current one is multiplied; x is staged once per block;
//                 lane l then takes blocks l, l + 32, ... : s = sum_i q_i x_i (fmaf chain, i in
//                 order), acc = fmaf(d, s, acc); xor butterfly 16 .. 1; + bias (passe.cuh:57-97);
//   k_rmsnorm     per thread, the f64 fma chain of squares over i = t, t + 256, ...; fixed tree
//                 over 256; y = x r w in f64 rounded once (passe.cuh:250-272);
//   k_rope_yarn   NEOX halves, YaRN inv_freq and concentration in f64 (the published YaRN
//                 formula, passe.cuh:146-169, 280-301);
//   k_ecrire_kv   f32 -> f16 round-to-nearest-even into the position's case (passe.cuh:305-314);
//   k_attention   one query head per block: scores (fmaf chain over d, then x 1/sqrt(d)), max with
//                 the head's sink, exp, z = tree sum + exp(sink - m), values by 4 groups of
//                 positions j = g mod 4 in order, ((g0 + g1) + (g2 + g3)) / z (passe.cuh:316-371).
#include <cuda_fp16.h>

#include "commun.cuh"
#include "noyaux.h"

namespace tb {

__device__ __forceinline__ float f16_f32(uint32_t bits) { return __half2float(__ushort_as_half(static_cast<unsigned short>(bits))); }

// ------------------------------------------------------------------ Q8_0 GEMV

constexpr uint32_t Q8_BLOC = 34;       // f16 d, then 32 x i8 (ggml's block_q8_0)
constexpr uint32_t Q8_WARPS = 8;

// Shared bytes of the padded x (one word per 32), rounded to 16 so the row buffers stay aligned.
__host__ __device__ __forceinline__ uint32_t q8_x_octets(uint32_t C) { return (4u * (C + C / 32u) + 15u) & ~15u; }

__host__ __device__ __forceinline__ uint32_t q8_tampon(uint32_t C) {
    return ((C / 32u) * Q8_BLOC + 16u + 15u) & ~15u;  // a row plus its 16-byte misalignment
}

// Copies a row's bytes [debut, debut + octets) of W (16-aligned) into `ligne` as 16-byte chunks
// from the boundary at or below `debut`, asynchronously (cp.async; bytes past the matrix read 0).
__device__ __forceinline__ void q8_charger_ligne(uint8_t* ligne, const uint8_t* W, uint64_t debut, uint32_t octets,
                                                 uint64_t fin_mat, uint32_t voie) {
    const uint64_t a0 = debut & ~uint64_t(15);
    const uint32_t n16 = uint32_t((debut - a0) + octets + 15u) / 16u;
    for (uint32_t i = voie; i < n16; i += 32u) {
        const uint64_t a = a0 + 16u * i;
        const uint64_t reste = a >= fin_mat ? 0u : fin_mat - a;
        const uint32_t utiles = reste < 16u ? uint32_t(reste) : 16u;
        cp_async16(ligne + 16u * i, utiles ? W + a : W, utiles);
    }
}

// J tokens at once (x [J][C], y [J][R]): each row is staged once and multiplied by the J vectors,
// each token's sums in the single-token order (the same bits as J separate launches).
template <int J>
__global__ void __launch_bounds__(Q8_WARPS * 32) k_gemv_q8_0(const uint8_t* __restrict__ W, const float* __restrict__ x,
                                                           const float* __restrict__ biais, float* __restrict__ y,
                                                           uint32_t R, uint32_t C) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const uint32_t voie = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t B = C / 32u, octets = B * Q8_BLOC, tampon = q8_tampon(C);
    const uint32_t xp = q8_x_octets(C) / 4u;                            // floats per staged token
    float* xs = reinterpret_cast<float*>(dyn);                          // [J][C + C / 32 (+ pad)]
    uint8_t* lignes = dyn + J * q8_x_octets(C) + warp * 2u * tampon;  // two row buffers per warp
    const uint64_t fin_mat = uint64_t(R) * octets;
    const uint32_t pas = gridDim.x * Q8_WARPS;
    uint32_t r = blockIdx.x * Q8_WARPS + warp;
    // The weights are an input of the call: the first row is requested before the wait.
    if (r < R) q8_charger_ligne(lignes, W, uint64_t(r) * octets, octets, fin_mat, voie);
    cp_async_commit();
    attendre_amont();
    liberer_aval();
    // x padded by one word per 32 (xs[c + c / 32]): lane l reads x[32 b + i] for b = l, l + 32,
    // ..., so unpadded all 32 lanes would hit one shared-memory bank.
    for (uint32_t t = threadIdx.x; t < J * (C / 4u); t += blockDim.x) {
        const uint32_t jt = t / (C / 4u), tt = t - jt * (C / 4u);
        const float4 v = __ldg(reinterpret_cast<const float4*>(x + uint64_t(jt) * C) + tt);
        const uint32_t c = 4u * tt, o = jt * xp + c + c / 32u;
        xs[o] = v.x;
        xs[o + 1] = v.y;
        xs[o + 2] = v.z;
        xs[o + 3] = v.w;
    }
    __syncthreads();
    for (uint32_t n = 0; r < R; r += pas, ++n) {
        // The next row goes into the other buffer while this one is multiplied.
        const uint32_t rs = r + pas;
        if (rs < R) q8_charger_ligne(lignes + ((n + 1u) & 1u) * tampon, W, uint64_t(rs) * octets, octets, fin_mat, voie);
        cp_async_commit();
        cp_async_wait<1>();
        __syncwarp();
        const uint8_t* ligne = lignes + (n & 1u) * tampon;
        const uint64_t debut = uint64_t(r) * octets;
        const uint32_t dec = uint32_t(debut - (debut & ~uint64_t(15)));
        float acc[J];
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = 0.0f;
        for (uint32_t b = voie; b < B; b += 32u) {
            const uint16_t* blk = reinterpret_cast<const uint16_t*>(ligne + dec + b * Q8_BLOC);
            const float d = f16_f32(blk[0]);
            const float* xv = xs + 33u * b;
            float s[J];
#pragma unroll
            for (int j = 0; j < J; ++j) s[j] = 0.0f;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const uint32_t w = blk[1 + t];
                const float q0 = float(int8_t(w & 0xFFu)), q1 = float(int8_t(w >> 8));
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    s[j] = fmaf(q0, xv[j * xp + 2 * t], s[j]);
                    s[j] = fmaf(q1, xv[j * xp + 2 * t + 1], s[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < J; ++j) acc[j] = fmaf(d, s[j], acc[j]);
        }
#pragma unroll
        for (int j = 0; j < J; ++j) {
#pragma unroll
            for (int dd = 16; dd > 0; dd >>= 1) acc[j] += __shfl_xor_sync(0xFFFFFFFFu, acc[j], dd);
            if (voie == 0) y[uint64_t(j) * R + r] = biais != nullptr ? acc[j] + biais[r] : acc[j];
        }
        __syncwarp();  // this buffer is refilled two rows from now
    }
    cp_async_wait<0>();
}

// ------------------------------------------------------------------ RMSNorm

__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ x, const float* __restrict__ w, float* y,
                                                 uint32_t n, float eps) {
    __shared__ double part[256];
    attendre_amont();
    liberer_aval();
    const uint32_t t = threadIdx.x;
    const float* xr = x + uint64_t(blockIdx.x) * n;
    float* yr = y + uint64_t(blockIdx.x) * n;
    double s = 0.0;
    for (uint32_t i = t; i < n; i += 256u) {
        const double v = xr[i];
        s = fma(v, v, s);
    }
    part[t] = s;
    __syncthreads();
#pragma unroll
    for (uint32_t k = 128; k > 0; k >>= 1) {
        if (t < k) part[t] += part[t + k];
        __syncthreads();
    }
    const double r = 1.0 / sqrt(part[0] / double(n) + double(eps));
    // y may be x: each thread writes only the elements it read itself.
    for (uint32_t i = t; i < n; i += 256u) yr[i] = float(double(xr[i]) * r * double(w[i]));
}

// ------------------------------------------------------------------ YaRN rotation

// YaRN (Peng et al., 2023) for pair i of a head of dimension d: frequency base^(2i/d); the
// ramp between the pair indices where a rotation makes beta_fast and beta_slow turns over the
// original context decides between the interpolated 1/(s f) and the extrapolated 1/f; the
// attention concentration is 0.1 ln(s) + 1. `variante` 1 rounds the ramp's ends (floor / ceil,
// clamped), as llama.cpp does.
__device__ inline double yarn_inv_freq(const ParamsRope& p, uint32_t i, double& concentration) {
    const uint32_t demi = p.dim_tete / 2u;
    const double freq = pow(p.base, double(2u * i) / double(p.dim_tete));
    if (p.facteur <= 1.0) {
        concentration = 1.0;
        return 1.0 / freq;
    }
    concentration = 0.1 * log(p.facteur) + 1.0;
    const double deux_pi = 6.283185307179586476925286766559;
    double bas = double(demi) * log(p.ctx_origine / (p.beta_rapide * deux_pi)) / log(p.base);
    double haut = double(demi) * log(p.ctx_origine / (p.beta_lent * deux_pi)) / log(p.base);
    if (p.variante == 1u) {
        bas = fmax(floor(bas), 0.0);
        haut = fmin(ceil(haut), double(p.dim_tete - 1u));
    }
    const double interpolation = 1.0 / (p.facteur * freq);
    const double extrapolation = 1.0 / freq;
    const double rampe = fmin(fmax((double(i) - bas) / (haut - bas), 0.0), 1.0);
    const double masque = 1.0 - rampe;
    return interpolation * (1.0 - masque) + extrapolation * masque;
}

__global__ void __launch_bounds__(64) k_rope_yarn(float* __restrict__ q, float* __restrict__ k, uint32_t tetes_q,
                                                  uint32_t tetes_k, uint32_t position, ParamsRope p) {
    attendre_amont();
    liberer_aval();
    const uint32_t demi = p.dim_tete / 2u, i = threadIdx.x;
    if (i >= demi || blockIdx.x >= tetes_q + tetes_k) return;
    double m;
    const double inv = yarn_inv_freq(p, i, m);
    double s, c;
    sincos(double(position) * inv, &s, &c);
    c *= m;
    s *= m;
    float* v = blockIdx.x < tetes_q ? q + uint64_t(blockIdx.x) * p.dim_tete : k + uint64_t(blockIdx.x - tetes_q) * p.dim_tete;
    const double a = v[i], b = v[i + demi];
    v[i] = float(a * c - b * s);
    v[i + demi] = float(b * c + a * s);
}

// ------------------------------------------------------------------ KV cache

__global__ void __launch_bounds__(256) k_ecrire_kv(const float* __restrict__ k, const float* __restrict__ v,
                                                   uint16_t* __restrict__ cache_k, uint16_t* __restrict__ cache_v,
                                                   uint32_t dkv, uint32_t case_kv) {
    attendre_amont();
    liberer_aval();
    const uint32_t i = blockIdx.x * 256u + threadIdx.x;
    if (i >= dkv) return;
    const uint64_t o = uint64_t(case_kv) * dkv + i;
    cache_k[o] = __half_as_ushort(__float2half_rn(k[i]));
    cache_v[o] = __half_as_ushort(__float2half_rn(v[i]));
}

// ------------------------------------------------------------------ attention of one position

constexpr uint32_t ATT_FILS = 256;
constexpr uint32_t ATT_DIM = 64;

template <bool MAX>
__device__ __forceinline__ float arbre_bloc(float* part, float v) {
    const uint32_t t = threadIdx.x;
    part[t] = v;
    __syncthreads();
#pragma unroll
    for (uint32_t k = ATT_FILS / 2; k > 0; k >>= 1) {
        if (t < k) part[t] = MAX ? fmaxf(part[t], part[t + k]) : part[t] + part[t + k];
        __syncthreads();
    }
    const float r = part[0];
    __syncthreads();
    return r;
}

__global__ void __launch_bounds__(ATT_FILS) k_attention(const float* __restrict__ q, const uint16_t* __restrict__ cache_k,
                                                        const uint16_t* __restrict__ cache_v, const float* __restrict__ puits,
                                                        float* __restrict__ sortie, ParamsAttention p) {
    extern __shared__ float scores[];
    __shared__ float qs[ATT_DIM];
    __shared__ float part[ATT_FILS];
    __shared__ float groupes[4][ATT_DIM];
    attendre_amont();
    liberer_aval();
    const uint32_t t = threadIdx.x, h = blockIdx.x;
    const uint32_t hk = h / (p.tetes / p.tetes_kv);
    const uint32_t dkv = p.tetes_kv * ATT_DIM;
    const uint32_t n = p.fin - p.debut;
    if (t < ATT_DIM) qs[t] = q[uint64_t(h) * ATT_DIM + t];
    __syncthreads();
    for (uint32_t j = t; j < n; j += ATT_FILS) {
        const uint32_t pos = p.debut + j;
        const uint32_t c = p.anneau ? pos % p.anneau : pos;
        const uint4* kr = reinterpret_cast<const uint4*>(cache_k + uint64_t(c) * dkv + uint64_t(hk) * ATT_DIM);
        uint4 w[8];
#pragma unroll
        for (int b = 0; b < 8; ++b) w[b] = kr[b];
        float s = 0.0f;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const uint32_t mots[4] = {w[b].x, w[b].y, w[b].z, w[b].w};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                s = fmaf(qs[8 * b + 2 * u], f16_f32(mots[u] & 0xFFFFu), s);
                s = fmaf(qs[8 * b + 2 * u + 1], f16_f32(mots[u] >> 16), s);
            }
        }
        scores[j] = s * p.echelle;
    }
    __syncthreads();
    float m = -INFINITY;
    for (uint32_t j = t; j < n; j += ATT_FILS) m = fmaxf(m, scores[j]);
    const float puits_h = puits[h];
    m = fmaxf(arbre_bloc<true>(part, m), puits_h);
    float z = 0.0f;
    for (uint32_t j = t; j < n; j += ATT_FILS) {
        const float e = expf(scores[j] - m);
        scores[j] = e;
        z += e;
    }
    z = arbre_bloc<false>(part, z) + expf(puits_h - m);
    const uint32_t dd = t & (ATT_DIM - 1u), g = t / ATT_DIM;
    const uint16_t* vcol = cache_v + uint64_t(hk) * ATT_DIM + dd;
    float a = 0.0f;
    uint32_t j = g;
    // Eight positions' values loaded before their (ordered) fmaf chain.
    for (; j + 28u < n; j += 32u) {
        float vv[8];
#pragma unroll
        for (uint32_t u = 0; u < 8u; ++u) {
            const uint32_t pos = p.debut + j + 4u * u;
            const uint32_t c = p.anneau ? pos % p.anneau : pos;
            vv[u] = f16_f32(vcol[uint64_t(c) * dkv]);
        }
#pragma unroll
        for (uint32_t u = 0; u < 8u; ++u) a = fmaf(scores[j + 4u * u], vv[u], a);
    }
    for (; j < n; j += 4u) {
        const uint32_t pos = p.debut + j;
        const uint32_t c = p.anneau ? pos % p.anneau : pos;
        a = fmaf(scores[j], f16_f32(vcol[uint64_t(c) * dkv]), a);
    }
    groupes[g][dd] = a;
    __syncthreads();
    if (t < ATT_DIM)
        sortie[uint64_t(h) * ATT_DIM + t] = ((groupes[0][t] + groupes[1][t]) + (groupes[2][t] + groupes[3][t])) / z;
}

// ------------------------------------------------------------------ launchers

template <int J>
static cudaError_t lancer_q8_0_j(const void* w, const float* x, const float* biais, float* y, uint32_t R, uint32_t C,
                                 cudaStream_t flux) {
    const size_t smem = J * q8_x_octets(C) + Q8_WARPS * 2u * q8_tampon(C);
    cudaError_t e = assurer_smem(reinterpret_cast<const void*>(k_gemv_q8_0<J>), int(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t par_sm = std::max<uint32_t>(1u, std::min<uint32_t>(4u, uint32_t(200000 / smem)));
    const uint32_t blocs = std::min<uint32_t>((R + Q8_WARPS - 1) / Q8_WARPS, uint32_t(sms) * par_sm);
    return lancer_pdl(k_gemv_q8_0<J>, dim3(blocs), dim3(Q8_WARPS * 32), smem, flux, static_cast<const uint8_t*>(w), x,
                      biais, y, R, C);
}

cudaError_t lancer_gemv_q8_0(const void* w, const float* x, const float* biais, float* y, uint32_t R, uint32_t C,
                             cudaStream_t flux) {
    return lancer_q8_0_j<1>(w, x, biais, y, R, C, flux);
}

// n tokens (x [n][C], y [n][R]) by launches of up to Q8_LOT_MAX tokens.
cudaError_t lancer_gemv_q8_0_lot(const void* w, const float* x, const float* biais, float* y, uint32_t R, uint32_t C,
                                 uint32_t n, cudaStream_t flux) {
    for (uint32_t j0 = 0; j0 < n; j0 += Q8_LOT_MAX) {
        const uint32_t m = std::min(Q8_LOT_MAX, n - j0);
        const float* xj = x + uint64_t(j0) * C;
        float* yj = y + uint64_t(j0) * R;
        cudaError_t e;
        switch (m) {
            case 1: e = lancer_q8_0_j<1>(w, xj, biais, yj, R, C, flux); break;
            case 2: e = lancer_q8_0_j<2>(w, xj, biais, yj, R, C, flux); break;
            case 3: e = lancer_q8_0_j<3>(w, xj, biais, yj, R, C, flux); break;
            case 4: e = lancer_q8_0_j<4>(w, xj, biais, yj, R, C, flux); break;
            case 5: e = lancer_q8_0_j<5>(w, xj, biais, yj, R, C, flux); break;
            case 6: e = lancer_q8_0_j<6>(w, xj, biais, yj, R, C, flux); break;
            case 7: e = lancer_q8_0_j<7>(w, xj, biais, yj, R, C, flux); break;
            default: e = lancer_q8_0_j<8>(w, xj, biais, yj, R, C, flux); break;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t lancer_rmsnorm(const float* x, const float* w, float* y, uint32_t n, uint32_t lignes, float eps,
                           cudaStream_t flux) {
    return lancer_pdl(k_rmsnorm, dim3(lignes), dim3(256), 0, flux, x, w, y, n, eps);
}

cudaError_t lancer_rope_yarn(float* q, float* k, uint32_t tetes_q, uint32_t tetes_k, uint32_t position, const ParamsRope& p,
                             cudaStream_t flux) {
    return lancer_pdl(k_rope_yarn, dim3(tetes_q + tetes_k), dim3(p.dim_tete / 2u), 0, flux, q, k, tetes_q, tetes_k, position, p);
}

cudaError_t lancer_ecrire_kv(const float* k, const float* v, uint16_t* ck, uint16_t* cv, uint32_t dkv, uint32_t case_kv,
                             cudaStream_t flux) {
    return lancer_pdl(k_ecrire_kv, dim3((dkv + 255) / 256), dim3(256), 0, flux, k, v, ck, cv, dkv, case_kv);
}

cudaError_t lancer_attention(const float* q, const uint16_t* ck, const uint16_t* cv, const float* puits, float* sortie,
                             const ParamsAttention& p, cudaStream_t flux) {
    const size_t smem = 4u * (p.fin - p.debut);
    cudaError_t e = assurer_smem(reinterpret_cast<const void*>(k_attention), int(smem));
    if (e != cudaSuccess) return e;
    return lancer_pdl(k_attention, dim3(p.tetes), dim3(ATT_FILS), smem, flux, q, ck, cv, puits, sortie, p);
}

}  // namespace tb
