// troncons_b200 — the attention side of a gpt-oss layer at batch 1: Q8_0 GEMV, RMSNorm, YaRN
// rotation, KV-cache write, attention of one position with sinks and the sliding window (the
// reference's passe.cuh kernels gemv_q8_0, rmsnorm, rope_yarn, ecrire_kv, attention, launched by
// `Noyaux` in trc-noyaux/src/lib.rs:291-381).
//
// The Q8_0 GEMV, RMSNorm, rotation and KV write keep the reference's arithmetic order, element by
// element, so that their outputs are bit-identical to the reference kernels' on the same GPU (the
// same CUDA math functions, called, not restated); the memory side is this library's own:
//   k_gemv_q8_0   persistent warps stage rows of 34-byte blocks (C/32 of them, rows 2-aligned
//                 only) with coalesced 16-byte cp.async into shared memory, the next row while
//                 the current one is multiplied; x is staged once per block;
//                 lane l then takes blocks l, l + 32, ... : s = sum_i q_i x_i (fmaf chain, i in
//                 order), acc = fmaf(d, s, acc); xor butterfly 16 .. 1; + bias (passe.cuh:57-97);
//   k_rmsnorm     per thread, the f64 fma chain of squares over i = t, t + 256, ...; fixed tree
//                 over 256; y = x r w in f64 rounded once (passe.cuh:250-272);
//   k_rope_yarn   NEOX halves, YaRN inv_freq and concentration in f64 (the published YaRN
//                 formula, passe.cuh:146-169, 280-301);
//   k_ecrire_kv   f32 -> f16 round-to-nearest-even into the position's case (passe.cuh:305-314).
// The attention itself (k_attention) is this library's own design, split over positions and
// merged within a thread-block cluster: the same function (passe.cuh:316-371), another order of
// the f32 sums, so it agrees with the reference's kernel and an f64 evaluation within 1e-5 of
// max|out| rather than bit for bit.
#include <cooperative_groups.h>
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

// The layer's Q8_0 GEMVs that share an input in one launch (DescQ8Couche): q, k and v on
// RMSNorm(x) (the norm recomputed by every block from x, in k_rmsnorm's order: thread t's f64 fma
// chain over i = t, t + 256, ..., the fixed tree over 256, then each element rounded once), or the
// output projection with the residual add folded in; or, for J tokens at once (x [J][C], matrix m's
// y [J][lignes[m]]), q, k and v on the batch's normed rows. Rows as in k_gemv_q8_0<J>, matrix
// after matrix: the same bits as k_rmsnorm and separate k_gemv_q8_0 launches (then k_combiner),
// with the small k and v projections (512 rows each) riding in the q projection's launch instead
// of each paying a launch's ramp on 64 blocks.
static_assert(Q8_WARPS * 32 == 256, "the in-block RMSNorm follows k_rmsnorm's 256 threads");

template <int J>
__global__ void __launch_bounds__(Q8_WARPS * 32) k_q8_0_couche(DescQ8Couche d) {
    extern __shared__ __align__(16) uint8_t dyn[];
    __shared__ double part[256];
    const uint32_t t = threadIdx.x, voie = t & 31u, warp = t >> 5;
    const uint32_t C = d.C, B = C / 32u, octets = B * Q8_BLOC, tampon = q8_tampon(C);
    const uint32_t xp = q8_x_octets(C) / 4u;  // floats per staged token
    float* xs = reinterpret_cast<float*>(dyn);
    uint8_t* lignes = dyn + J * q8_x_octets(C) + warp * 2u * tampon;
    uint32_t R = 0;
    for (uint32_t m = 0; m < d.n; ++m) R += d.lignes[m];
    auto charger = [&](uint8_t* tampon_l, uint32_t r) {
        uint32_t m = 0;
        while (r >= d.lignes[m]) r -= d.lignes[m++];
        q8_charger_ligne(tampon_l, static_cast<const uint8_t*>(d.w[m]), uint64_t(r) * octets, octets,
                         uint64_t(d.lignes[m]) * octets, voie);
    };
    const uint32_t pas = gridDim.x * Q8_WARPS;
    uint32_t r = blockIdx.x * Q8_WARPS + warp;
    // The weights are an input of the call: the first row is requested before the wait.
    if (r < R) charger(lignes, r);
    cp_async_commit();
    attendre_amont();
    liberer_aval();
    if (J == 1 && d.norme != nullptr) {
        double s = 0.0;
        for (uint32_t i = t; i < C; i += 256u) {
            const double v = d.x[i];
            s = fma(v, v, s);
        }
        part[t] = s;
        __syncthreads();
#pragma unroll
        for (uint32_t k = 128; k > 0; k >>= 1) {
            if (t < k) part[t] += part[t + k];
            __syncthreads();
        }
        const double rn = 1.0 / sqrt(part[0] / double(C) + double(d.eps));
        for (uint32_t i = t; i < C; i += 256u) {
            const float h = float(double(d.x[i]) * rn * double(d.norme[i]));
            xs[i + i / 32u] = h;
            if (blockIdx.x == 0 && d.h != nullptr) d.h[i] = h;
        }
    } else {
        for (uint32_t i = t; i < J * C; i += 256u) {
            const uint32_t jt = i / C, c = i - jt * C;
            xs[jt * xp + c + c / 32u] = d.x[i];
        }
    }
    __syncthreads();
    for (uint32_t n = 0; r < R; r += pas, ++n) {
        const uint32_t rs = r + pas;
        if (rs < R) charger(lignes + ((n + 1u) & 1u) * tampon, rs);
        cp_async_commit();
        cp_async_wait<1>();
        __syncwarp();
        uint32_t m = 0, rl = r;
        while (rl >= d.lignes[m]) rl -= d.lignes[m++];
        const uint8_t* ligne = lignes + (n & 1u) * tampon;
        const uint64_t debut = uint64_t(rl) * octets;
        const uint32_t dec = uint32_t(debut - (debut & ~uint64_t(15)));
        float acc[J];
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = 0.0f;
        for (uint32_t b = voie; b < B; b += 32u) {
            const uint16_t* blk = reinterpret_cast<const uint16_t*>(ligne + dec + b * Q8_BLOC);
            const float dq = f16_f32(blk[0]);
            const float* xv = xs + 33u * b;
            float s[J];
#pragma unroll
            for (int j = 0; j < J; ++j) s[j] = 0.0f;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                const uint32_t w = blk[1 + k];
                const float q0 = float(int8_t(w & 0xFFu)), q1 = float(int8_t(w >> 8));
#pragma unroll
                for (int j = 0; j < J; ++j) {
                    s[j] = fmaf(q0, xv[j * xp + 2 * k], s[j]);
                    s[j] = fmaf(q1, xv[j * xp + 2 * k + 1], s[j]);
                }
            }
#pragma unroll
            for (int j = 0; j < J; ++j) acc[j] = fmaf(dq, s[j], acc[j]);
        }
#pragma unroll
        for (int j = 0; j < J; ++j) {
#pragma unroll
            for (int dd = 16; dd > 0; dd >>= 1) acc[j] += __shfl_xor_sync(0xFFFFFFFFu, acc[j], dd);
            if (voie == 0) {
                const float y = d.biais[m] != nullptr ? acc[j] + d.biais[m][rl] : acc[j];
                d.y[m][uint64_t(j) * d.lignes[m] + rl] = y;
                if (J == 1 && d.residu != nullptr) d.residu[rl] = __fadd_rn(d.residu[rl], y);
            }
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

// The rotation and the KV write in one launch: blocks of q heads rotate as k_rope_yarn; a block of
// kv head h rotates k's head h, then writes its f16 rounding (k_ecrire_kv's) into the position's
// case of cache_k, and v's head h into cache_v. Element for element the same bits as the two
// launches (q and k also keep their rotated f32 values).
__global__ void __launch_bounds__(64) k_rope_kv(float* __restrict__ q, float* __restrict__ k, const float* __restrict__ v,
                                                uint16_t* __restrict__ cache_k, uint16_t* __restrict__ cache_v,
                                                uint32_t tetes_q, uint32_t tetes_k, uint32_t position, uint32_t case_kv,
                                                ParamsRope p) {
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
    const bool est_k = blockIdx.x >= tetes_q;
    const uint32_t h = est_k ? blockIdx.x - tetes_q : blockIdx.x;
    float* t = (est_k ? k : q) + uint64_t(h) * p.dim_tete;
    const double a = t[i], b = t[i + demi];
    const float r0 = float(a * c - b * s), r1 = float(b * c + a * s);
    t[i] = r0;
    t[i + demi] = r1;
    if (est_k) {
        const uint64_t o = uint64_t(case_kv) * tetes_k * p.dim_tete + uint64_t(h) * p.dim_tete;
        const float* vh = v + uint64_t(h) * p.dim_tete;
        cache_k[o + i] = __half_as_ushort(__float2half_rn(r0));
        cache_k[o + i + demi] = __half_as_ushort(__float2half_rn(r1));
        cache_v[o + i] = __half_as_ushort(__float2half_rn(vh[i]));
        cache_v[o + i + demi] = __half_as_ushort(__float2half_rn(vh[i + demi]));
    }
}

// ------------------------------------------------------------------ attention of one position

// Attention of one position, split over positions and merged inside a thread-block cluster.
//
// Grid (S, tetes_kv), clusters of S blocks along x: block (s, hk) takes the s-th slice of the
// positions for the G = tetes / tetes_kv query heads that share key/value head hk, so that each
// key and value row is read from HBM once for all G heads. A block stages up to ATT_TRANCHE
// positions at a time (their key rows, padded to 144 bytes against bank conflicts, and value
// rows) with 16-byte cp.async, computes the G scores of each position (fmaf chain over d, then
// x 1/sqrt(d)), and keeps per head a running maximum m, sum z and value accumulator a over its
// slices (online softmax: a and z rescaled by exp(m_old - m_new) when the maximum grows). The S
// blocks then merge through distributed shared memory: block r merges heads h = r, r + S, ...
// with the head's sink: M = max(sink, m_0 .. m_{S-1}), f_s = exp(m_s - M),
// z = sum_s z_s f_s + exp(sink - M), out = (sum_s a_s f_s) / z, sums in slice order. The result
// is deterministic for a given (n, S); it differs from a single-pass softmax by f32 rounding
// (passe.cuh:316-371 defines the function: sinks, ring of cases, 1/sqrt(d) scale).
constexpr uint32_t ATT_FILS = 256;
constexpr uint32_t ATT_DIM = 64;
constexpr uint32_t ATT_TRANCHE = 128;         // positions staged at once
constexpr uint32_t ATT_K_PAS = 144;           // bytes per staged key row (128 + 16 of padding)
constexpr uint32_t ATT_V_PAS = 128;           // bytes per staged value row
constexpr uint32_t ATT_G_MAX = 64;            // query heads per key/value head
constexpr uint32_t ATT_GRAPPE_MAX = 16;

__host__ __device__ constexpr uint32_t att_smem(uint32_t G) {
    return ATT_TRANCHE * (ATT_K_PAS + ATT_V_PAS)   // key and value rows
           + 4u * G * ATT_DIM                        // q
           + 4u * G * ATT_TRANCHE                    // scores, then exp(score - m)
           + 4u * G * (ATT_DIM + 3u);                // per head: a[64], m, z, rescale factor
}

__global__ void __launch_bounds__(ATT_FILS) k_attention(const float* __restrict__ q, const uint16_t* __restrict__ cache_k,
                                                        const uint16_t* __restrict__ cache_v, const float* __restrict__ puits,
                                                        float* __restrict__ sortie, ParamsAttention p) {
    extern __shared__ __align__(16) uint8_t att_mem[];
    namespace cg = cooperative_groups;
    cg::cluster_group grappe = cg::this_cluster();
    const uint32_t G = p.tetes / p.tetes_kv;
    uint8_t* k_lignes = att_mem;
    uint8_t* v_lignes = k_lignes + ATT_TRANCHE * ATT_K_PAS;
    float* qs = reinterpret_cast<float*>(v_lignes + ATT_TRANCHE * ATT_V_PAS);
    float* sc = qs + G * ATT_DIM;
    float* acc = sc + G * ATT_TRANCHE;   // [G][64]
    float* mx = acc + G * ATT_DIM;       // [G]
    float* zs = mx + G;                  // [G]
    float* fac = zs + G;                 // [G]

    const uint32_t t = threadIdx.x, voie = t & 31u, w = t >> 5;
    const uint32_t S = gridDim.x, s = blockIdx.x, hk = blockIdx.y;
    const uint32_t dkv = p.tetes_kv * ATT_DIM;
    const uint32_t n = p.fin - p.debut;
    const uint32_t par = (n + S - 1) / S;
    const uint32_t j0 = min(n, s * par), j1 = min(n, j0 + par);

    attendre_amont();
    liberer_aval();
    for (uint32_t i = t; i < G * ATT_DIM; i += ATT_FILS) {
        qs[i] = q[uint64_t(hk) * G * ATT_DIM + i];
        acc[i] = 0.0f;
    }
    for (uint32_t g = t; g < G; g += ATT_FILS) {
        mx[g] = -INFINITY;
        zs[g] = 0.0f;
    }

    for (uint32_t a0 = j0; a0 < j1; a0 += ATT_TRANCHE) {
        const uint32_t m = min(ATT_TRANCHE, j1 - a0);
        __syncthreads();  // the previous slice's rows and scores are no longer read
        // Key and value rows of positions a0 .. a0 + m - 1: 8 chunks of 16 bytes per row each.
        for (uint32_t i = t; i < 16u * m; i += ATT_FILS) {
            const uint32_t j = i >> 4, c16 = i & 7u;
            const uint32_t pos = p.debut + a0 + j;
            const uint32_t cas = p.anneau ? pos % p.anneau : pos;
            const uint64_t src = uint64_t(cas) * dkv + uint64_t(hk) * ATT_DIM + 8u * c16;
            if (i & 8u)
                cp_async16(v_lignes + j * ATT_V_PAS + 16u * c16, cache_v + src, 16u);
            else
                cp_async16(k_lignes + j * ATT_K_PAS + 16u * c16, cache_k + src, 16u);
        }
        cp_async_commit();
        cp_async_wait<0>();
        __syncthreads();
        // Scores: thread t takes position t mod 128 for heads t / 128, t / 128 + 2, ...
        {
            const uint32_t j = t % ATT_TRANCHE;
            if (j < m) {
                float kf[ATT_DIM];
                const uint4* kr = reinterpret_cast<const uint4*>(k_lignes + j * ATT_K_PAS);
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const uint4 u = kr[b];
                    const uint32_t mots[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&mots[c]));
                        kf[8 * b + 2 * c] = f.x;
                        kf[8 * b + 2 * c + 1] = f.y;
                    }
                }
                for (uint32_t g = t / ATT_TRANCHE; g < G; g += ATT_FILS / ATT_TRANCHE) {
                    const float* qg = qs + g * ATT_DIM;
                    float v = 0.0f;
#pragma unroll
                    for (int d = 0; d < int(ATT_DIM); ++d) v = fmaf(qg[d], kf[d], v);
                    sc[g * ATT_TRANCHE + j] = v * p.echelle;
                }
            }
        }
        __syncthreads();
        // Per head (warp w takes heads w, w + 8, ...): the slice's maximum, the new running
        // maximum, exp(score - m) in place, the slice's sum, the rescale of the running values.
        for (uint32_t g = w; g < G; g += ATT_FILS / 32u) {
            float* sg = sc + g * ATT_TRANCHE;
            float mt = -INFINITY;
            for (uint32_t j = voie; j < m; j += 32u) mt = fmaxf(mt, sg[j]);
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xFFFFFFFFu, mt, d));
            const float ancien = mx[g];
            const float nouveau = fmaxf(ancien, mt);
            float somme = 0.0f;
            for (uint32_t j = voie; j < m; j += 32u) {
                const float e = expf(sg[j] - nouveau);
                sg[j] = e;
                somme += e;
            }
#pragma unroll
            for (int d = 16; d > 0; d >>= 1) somme += __shfl_xor_sync(0xFFFFFFFFu, somme, d);
            __syncwarp();
            if (voie == 0) {
                const float f = expf(ancien - nouveau);  // 0 on the first slice (ancien = -inf)
                fac[g] = f;
                zs[g] = fmaf(zs[g], f, somme);
                mx[g] = nouveau;
            }
        }
        __syncthreads();
        // Values: thread (w, voie) accumulates dimensions 2 voie, 2 voie + 1 of heads w, w + 8, ...
        for (uint32_t g = w; g < G; g += ATT_FILS / 32u) {
            const float* eg = sc + g * ATT_TRANCHE;
            float a0v = 0.0f, a1v = 0.0f;
            const uint32_t* vr = reinterpret_cast<const uint32_t*>(v_lignes) + voie;
#pragma unroll 4
            for (uint32_t j = 0; j < m; ++j) {
                const uint32_t mot = vr[j * (ATT_V_PAS / 4u)];
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&mot));
                const float e = eg[j];
                a0v = fmaf(e, f.x, a0v);
                a1v = fmaf(e, f.y, a1v);
            }
            float* ag = acc + g * ATT_DIM + 2u * voie;
            const float f = fac[g];
            ag[0] = fmaf(ag[0], f, a0v);
            ag[1] = fmaf(ag[1], f, a1v);
        }
    }
    __syncthreads();
    grappe.sync();  // every block's (m, z, a) is written and visible to the cluster
    // Block r merges heads r, r + S, ...: 64 threads per head, four heads at a time.
    for (uint32_t g = s + S * (t / ATT_DIM); g < G; g += S * (ATT_FILS / ATT_DIM)) {
        const uint32_t d = t % ATT_DIM;
        const uint32_t h = hk * G + g;
        const float puits_h = puits[h];
        float M = puits_h;
        for (uint32_t b = 0; b < S; ++b) M = fmaxf(M, *grappe.map_shared_rank(mx + g, b));
        float z = 0.0f, o = 0.0f;
        for (uint32_t b = 0; b < S; ++b) {
            const float f = expf(*grappe.map_shared_rank(mx + g, b) - M);
            z = fmaf(*grappe.map_shared_rank(zs + g, b), f, z);
            o = fmaf(*grappe.map_shared_rank(acc + g * ATT_DIM + d, b), f, o);
        }
        z += expf(puits_h - M);
        sortie[uint64_t(h) * ATT_DIM + d] = o / z;
    }
    grappe.sync();  // no block leaves while another may still read its shared memory
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

template <int J>
static cudaError_t lancer_q8_0_couche_j(const DescQ8Couche& d, uint32_t R, cudaStream_t flux) {
    const size_t smem = J * q8_x_octets(d.C) + Q8_WARPS * 2u * q8_tampon(d.C);
    cudaError_t e = assurer_smem(reinterpret_cast<const void*>(k_q8_0_couche<J>), int(smem));
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t par_sm = std::max<uint32_t>(1u, std::min<uint32_t>(4u, uint32_t(200000 / smem)));
    const uint32_t blocs = std::min<uint32_t>((R + Q8_WARPS - 1) / Q8_WARPS, uint32_t(sms) * par_sm);
    return lancer_pdl(k_q8_0_couche<J>, dim3(blocs), dim3(Q8_WARPS * 32), smem, flux, d);
}

cudaError_t lancer_q8_0_couche(const DescQ8Couche& d, cudaStream_t flux, uint32_t jetons) {
    if (d.n == 0 || d.n > 3 || d.C % 32u != 0 || jetons == 0) return cudaErrorInvalidValue;
    if ((d.norme != nullptr || d.residu != nullptr) && jetons != 1) return cudaErrorInvalidValue;
    if (d.residu != nullptr && d.n != 1) return cudaErrorInvalidValue;
    uint32_t R = 0;
    for (uint32_t m = 0; m < d.n; ++m) R += d.lignes[m];
    if (R == 0) return cudaSuccess;
    // batches by launches of up to Q8_LOT_MAX tokens
    for (uint32_t j0 = 0; j0 < jetons; j0 += Q8_LOT_MAX) {
        const uint32_t n = std::min(Q8_LOT_MAX, jetons - j0);
        DescQ8Couche dj = d;
        dj.x = d.x + uint64_t(j0) * d.C;
        for (uint32_t m = 0; m < d.n; ++m) dj.y[m] = d.y[m] + uint64_t(j0) * d.lignes[m];
        cudaError_t e;
        switch (n) {
            case 1: e = lancer_q8_0_couche_j<1>(dj, R, flux); break;
            case 2: e = lancer_q8_0_couche_j<2>(dj, R, flux); break;
            case 3: e = lancer_q8_0_couche_j<3>(dj, R, flux); break;
            case 4: e = lancer_q8_0_couche_j<4>(dj, R, flux); break;
            case 5: e = lancer_q8_0_couche_j<5>(dj, R, flux); break;
            case 6: e = lancer_q8_0_couche_j<6>(dj, R, flux); break;
            case 7: e = lancer_q8_0_couche_j<7>(dj, R, flux); break;
            default: e = lancer_q8_0_couche_j<8>(dj, R, flux); break;
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

cudaError_t lancer_rope_kv(float* q, float* k, const float* v, uint16_t* ck, uint16_t* cv, uint32_t tetes_q,
                           uint32_t tetes_k, uint32_t position, uint32_t case_kv, const ParamsRope& p, cudaStream_t flux) {
    if (p.dim_tete == 0 || p.dim_tete % 2u != 0 || p.dim_tete > 128u) return cudaErrorInvalidValue;
    return lancer_pdl(k_rope_kv, dim3(tetes_q + tetes_k), dim3(p.dim_tete / 2u), 0, flux, q, k, v, ck, cv, tetes_q, tetes_k,
                      position, case_kv, p);
}

cudaError_t lancer_ecrire_kv(const float* k, const float* v, uint16_t* ck, uint16_t* cv, uint32_t dkv, uint32_t case_kv,
                             cudaStream_t flux) {
    return lancer_pdl(k_ecrire_kv, dim3((dkv + 255) / 256), dim3(256), 0, flux, k, v, ck, cv, dkv, case_kv);
}

cudaError_t lancer_attention(const float* q, const uint16_t* ck, const uint16_t* cv, const float* puits, float* sortie,
                             const ParamsAttention& p, cudaStream_t flux) {
    const uint32_t G = p.tetes / p.tetes_kv;
    if (G == 0 || G > ATT_G_MAX || p.dim_tete != ATT_DIM) return cudaErrorInvalidValue;
    const uint32_t n = p.fin - p.debut;
    const size_t smem = att_smem(G);
    cudaError_t e = assurer_smem(reinterpret_cast<const void*>(k_attention), int(smem));
    if (e != cudaSuccess) return e;
    static bool grappe16 = [] {
        return cudaFuncSetAttribute(reinterpret_cast<const void*>(k_attention),
                                    cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess;
    }();
    // Slices of at least 32 positions, at most 16 (or 8 where clusters of 16 are refused) per head.
    uint32_t S = std::max(1u, std::min(grappe16 ? ATT_GRAPPE_MAX : 8u, (n + 31u) / 32u));
    for (;;) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S, p.tetes_kv);
        cfg.blockDim = dim3(ATT_FILS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = flux;
        cudaLaunchAttribute at[2];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        at[1].id = cudaLaunchAttributeClusterDimension;
        at[1].val.clusterDim.x = S;
        at[1].val.clusterDim.y = 1;
        at[1].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 2;
        e = cudaLaunchKernelEx(&cfg, k_attention, q, ck, cv, puits, sortie, p);
        if (e == cudaSuccess || S <= 8) return e;
        (void)cudaGetLastError();  // a cluster of 16 refused here: halve it
        grappe16 = false;
        S = 8;
    }
}

}  // namespace tb
