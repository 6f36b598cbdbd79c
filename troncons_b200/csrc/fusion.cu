// troncons_b200 — the fused MoE layer: rANS decoding of the routed experts' parts fused into
// the MXFP4 GEMV, then SwiGLU, the down projection and the weighted combine.
//
// The reference runs, per layer and routed expert, decoder_echelles + decoder_codes into an
// SoA slot in VRAM, then gemv_mxfp4 x3, swiglu_oai, and combiner over the k experts
// (trc-modele/src/lib.rs:533-553, trc-ordo/src/lib.rs:1328-1367). Here, on the caller's stream:
//   1. k_moe_delta   DELTA_j of the k routed experts -> the delta byte of every block, into the
//                    workspace (259,200 bytes per matrix: it stays in L2);
//   2. k_moe_codes   (gate, up) one warp per CODES_CTX tile decodes a macro-step (8 blocks, one
//                    word per lane, table chosen by the block's scale class) into registers and
//                    multiplies it against 2x staged in shared memory, in four stages placed
//                    between the four sub-steps of the next macro-step's decode; the block's
//                    scale = median + delta - 128. The codes never leave the SM. Rows are closed
//                    where they end and at every segment end (256 blocks), giving per-(row,
//                    segment) partials;
//   3. k_moe_swiglu  gate and up rows = fold of their partials + bias; h = SwiGLU (f64);
//   4. k_moe_codes   (down) the same on h;
//   5. k_moe_combiner down rows + bias, then residual += ((w0 s0 + w1 s1) + ...), no FMA.
// The raw path (`brut`) replaces 1-2 and 4 by k_moe_brut, a row-centric GEMV on CODES_BRUTS /
// ECHELLES_BRUTES writing the same partials, so compressed and raw parts give the same bits.
// Integrity counters go to controle[4 i ..] of active expert i (format errors included).
#include <cuda_bf16.h>

#include "commun.cuh"
#include "mxfp4.cuh"
#include "noyaux.h"

namespace tb {

Espace plan_espace(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t k) {
    Espace e{};
    uint64_t p = 0;
    for (int j = 0; j < 3; ++j) {
        const uint64_t nb = uint64_t(lignes[j]) * (colonnes[j] / 32u);
        e.ek[j] = p;
        p = al256(p + nb * k);
    }
    for (int j = 0; j < 3; ++j) {
        e.K[j] = parts_par_ligne(colonnes[j] / 32u);
        e.parts[j] = p;
        p = al256(p + 4ull * lignes[j] * e.K[j] * k);
    }
    e.h = p;
    p = al256(p + 4ull * lignes[0] * k);
    e.total = p;
    return e;
}

struct ArgsMoe {
    Couche c;
    uint8_t* espace;
    Espace plan;
    uint32_t j0;  // first matrix of this launch (0: gate and up; 2: down)
};

// The part of active expert i, if it is addressable.
__device__ __forceinline__ bool partie_de(const Couche& c, uint32_t i, const uint8_t*& partie, uint64_t& taille) {
    const uint32_t e = c.indices[i];
    if (e >= c.experts) return false;
    partie = reinterpret_cast<const uint8_t*>(c.parties[e]);
    taille = c.parties_octets[e];
    return partie != nullptr && taille >= 64 && (reinterpret_cast<uintptr_t>(partie) & 15u) == 0;
}

constexpr uint32_t DELTA_WARPS = 4;
constexpr uint32_t MOE_WARPS = 4;

// ------------------------------------------------------------------ 1. DELTA -> scales, classes

__global__ void __launch_bounds__(DELTA_WARPS * 32) k_moe_delta(ArgsMoe a) {
    __shared__ uint32_t lut[M];
    __shared__ __align__(16) uint16_t anneaux[DELTA_WARPS][ANNEAU_ALLOC];
    attendre_amont();  // first kernel of the layer: every input may come from the previous kernel
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t j = blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], B = c.colonnes[j] / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fd;
    EnteteRans h;
    const bool bon = partie_de(c, i, partie, taille) && trouver_flux(partie, taille, SORTE_DELTA, j, fd) &&
                     lire_entete(fd, nblocs, h);
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const uint32_t warp0 = blockIdx.x * DELTA_WARPS;
    if (warp0 >= h.T) return;
    const uint32_t* src = c.luts + (uint64_t(j) * 4u) * M;
    for (uint32_t t = threadIdx.x; t < M; t += blockDim.x) lut[t] = src[t];
    __syncthreads();
    const uint32_t lut_s = adresse_partagee(lut);
    uint8_t* delta = a.espace + a.plan.ek[j] + uint64_t(i) * nblocs;
    const uint32_t nmacro = h.P / 128u;
    uint32_t hors_l = 0, pointeur = 0;
    Decodeur d;
    for (uint32_t t = warp0 + (threadIdx.x >> 5); t < h.T; t += gridDim.x * DELTA_WARPS) {
        d.debut(h, t, voie, anneaux[threadIdx.x >> 5]);
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        // Word w = 32 m + lane is the delta of blocks 4w .. 4w + 3, stored as it comes.
        for (uint32_t m = m0; m < m1; ++m) {
            d.avancer();
            const uint32_t mot = d.macro(lut_s);
            const uint32_t b0 = 4u * (m * 32u + voie);
            if (b0 + 3u < nblocs) {
                *reinterpret_cast<uint32_t*>(delta + b0) = mot;
            } else {
                for (uint32_t k = 0; k < 4; ++k)
                    if (b0 + k < nblocs) delta[b0 + k] = uint8_t(mot >> (8u * k));
            }
        }
        d.bilan(hors_l, pointeur);
        d.terminer();
    }
    verser_controle(controle, voie, hors_l, pointeur);
}

// ------------------------------------------------------------------ shared-memory x2 = 2 x

__device__ __forceinline__ void charger_x2(float* x2s, const void* x, uint32_t bf16, uint32_t C) {
    if (bf16) {
        const uint16_t* xb = static_cast<const uint16_t*>(x);
        for (uint32_t t = threadIdx.x; t < C; t += blockDim.x) x2s[t] = 2.0f * __uint_as_float(uint32_t(xb[t]) << 16);
    } else {
        const float* xf = static_cast<const float*>(x);
        for (uint32_t t = threadIdx.x; t < C; t += blockDim.x) x2s[t] = 2.0f * xf[t];
    }
}

// ------------------------------------------------------------------ 2/4. CODES_CTX decoded into the GEMV

// The GEMV of one decoded macro-step (8 blocks, one word per lane) into the row partials: the
// block's sum (quad tree), scaled and accumulated on the current row or the next; rows closed
// where they end, and the row in progress closed at the segment's (or the tile's) end.
struct GemvTuile {
    float acc, acc_s;     // current row r, next row
    uint32_t r, fin_r;    // warp-uniform: current row, first block of the next row
    uint32_t med_r, med_s;  // medians of rows r and r + 1 (clamped to the last row)
    uint32_t R, B, K, voie, q;
    float* parts;
    const float4* x2s4;
    const uint8_t* med;   // row medians (shared memory)

    __device__ __forceinline__ void debut(uint32_t m0) {
        acc = 0.0f;
        acc_s = 0.0f;
        r = (8u * m0) / B;
        fin_r = (r + 1u) * B;
        med_r = med[min(r, R - 1u)];
        med_s = med[min(r + 1u, R - 1u)];
    }

    // The block's scale: its row's median + delta - 128 (mod 256); the row is r or r + 1.
    __device__ __forceinline__ float echelle(uint32_t bloc, uint32_t delta) const {
        const uint32_t e = ((bloc < fin_r ? med_r : med_s) + delta - 128u) & 255u;
        return echelle_e8m0(e);
    }

    // Branch-free part: the block's scaled contribution.
    __device__ __forceinline__ void accumuler(uint32_t mot, uint32_t bloc, uint32_t b, uint32_t delta, bool valide) {
        float s = produit_quad(mot, x2s4[8u * b + q], x2s4[8u * b + 4u + q]);
        s = somme_quad(s);
        const float sc = echelle(bloc, delta);
        const bool cour = bloc < fin_r;
        acc = (valide && cour) ? fmaf(s, sc, acc) : acc;
        acc_s = (valide && !cour) ? fmaf(s, sc, acc_s) : acc_s;
    }

    // The same, in four stages to interleave with the four sub-steps of the next decode.
    struct Etapes {
        float lo[4], hi[4];
        float4 xa, xb;
        float p;
    };
    template <int K>
    __device__ __forceinline__ void etape(Etapes& e, uint32_t mot, uint32_t bloc, uint32_t b, uint32_t ekv, bool valide) {
        if constexpr (K == 0) {
            e.xa = x2s4[8u * b + q];
            e.xb = x2s4[8u * b + 4u + q];
            e2m1_mot(mot, e.lo, e.hi);
        } else if constexpr (K == 1) {
            float p = 0.0f;
            p = fmaf(e.lo[0], e.xa.x, p);
            p = fmaf(e.hi[0], e.xb.x, p);
            p = fmaf(e.lo[1], e.xa.y, p);
            p = fmaf(e.hi[1], e.xb.y, p);
            p = fmaf(e.lo[2], e.xa.z, p);
            p = fmaf(e.hi[2], e.xb.z, p);
            p = fmaf(e.lo[3], e.xa.w, p);
            p = fmaf(e.hi[3], e.xb.w, p);
            e.p = p;
        } else if constexpr (K == 2) {
            e.p = somme_quad(e.p);
        } else {
            const float sc = echelle(bloc, ekv);
            const bool cour = bloc < fin_r;
            acc = (valide && cour) ? fmaf(e.p, sc, acc) : acc;
            acc_s = (valide && !cour) ? fmaf(e.p, sc, acc_s) : acc_s;
        }
    }

    // Row and segment closing after macro-step m (warp-uniform branches).
    __device__ __forceinline__ void fermer(uint32_t m, uint32_t m1) {
        const uint32_t seg = m / SEGMENT_MACRO;
        if (fin_r <= 8u * m + 8u) {  // row r ends in this macro-step
            const float P = arbre8(acc);
            if (voie == 0 && r < R) parts[uint64_t(r) * K + (seg - (r * B) / SEGMENT_BLOCS)] = P;
            acc = acc_s;
            acc_s = 0.0f;
            ++r;
            fin_r += B;
            med_r = med_s;
            med_s = med[min(r + 1u, R - 1u)];
        }
        if ((m + 1u) % SEGMENT_MACRO == 0 || m + 1u == m1) {  // segment (or tile) ends
            if (r * B < 8u * m + 8u && r < R) {
                const float P = arbre8(acc);
                if (voie == 0) parts[uint64_t(r) * K + (seg - (r * B) / SEGMENT_BLOCS)] = P;
            }
            acc = 0.0f;
        }
    }
};

// Shared bytes for the row medians of the largest matrix (16-aligned so that 2x stays aligned).
__host__ __device__ __forceinline__ uint32_t medianes_octets(const Couche& c) {
    return (max(c.lignes[0], c.lignes[2]) + 15u) & ~15u;
}

__global__ void __launch_bounds__(MOE_WARPS * 32, 1) k_moe_codes(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fc;
    EnteteRans h;
    Flux fm;
    const bool bon = B >= 8u && partie_de(c, i, partie, taille) && trouver_flux(partie, taille, SORTE_CODES_CTX, j, fc) &&
                     trouver_flux(partie, taille, SORTE_MEDIANES, j, fm) && fm.produits == R && fm.longueur >= R &&
                     R <= 8192u && lire_entete(fc, nblocs * 16u, h) && (h.N % SEGMENT_MACRO) == 0;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const uint32_t warp0 = blockIdx.x * MOE_WARPS;
    if (warp0 >= h.T) return;
    uint32_t* lut = reinterpret_cast<uint32_t*>(dyn);                                  // [3][M]
    uint16_t* anneaux = reinterpret_cast<uint16_t*>(dyn + 3u * M * 4u);                 // [W][ANNEAU_ALLOC]
    uint8_t* med = dyn + 3u * M * 4u + MOE_WARPS * ANNEAU_ALLOC * 2u;                    // [medianes_octets]
    float* x2s = reinterpret_cast<float*>(med + medianes_octets(c));
    {
        const uint4* src = reinterpret_cast<const uint4*>(c.luts + (uint64_t(j) * 4u + 1u) * M);
        uint4* dst = reinterpret_cast<uint4*>(lut);
        for (uint32_t t = threadIdx.x; t < 3u * M / 4u; t += blockDim.x) dst[t] = src[t];
    }
    for (uint32_t t = threadIdx.x; t < R; t += blockDim.x) med[t] = fm.p[t];
    if (j < 2) charger_x2(x2s, c.x, c.x_bf16, C);
    // Everything above reads inputs the layer's first kernel waited for; the scales and classes
    // (and h for the down projection) come from the previous kernel.
    attendre_amont();
    liberer_aval();
    if (j == 2) charger_x2(x2s, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const uint32_t lut_s = adresse_partagee(lut);
    const uint8_t* __restrict__ ek = a.espace + a.plan.ek[j] + uint64_t(i) * nblocs;  // delta bytes
    GemvTuile gv;
    gv.R = R;
    gv.B = B;
    gv.K = a.plan.K[j];
    gv.voie = voie;
    gv.q = voie & 3u;
    gv.parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * gv.K;
    gv.x2s4 = reinterpret_cast<const float4*>(x2s);
    gv.med = med;
    const uint32_t nmacro = h.P / 128u;
    const uint32_t g = voie >> 2;
    uint32_t hors_l = 0, pointeur = 0;
    Decodeur d;
    for (uint32_t t = warp0 + (threadIdx.x >> 5); t < h.T; t += gridDim.x * MOE_WARPS) {
        d.debut(h, t, voie, anneaux + (threadIdx.x >> 5) * ANNEAU_ALLOC);
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        gv.debut(m0);
        // This lane's block at macro-step m is 8 m + g, column block b; its delta read two
        // macro-steps ahead (class -> table; with the median -> scale); the GEMV of macro-step
        // m - 1 runs in stages between the sub-steps of macro-step m.
        uint32_t bloc = 8u * m0 + g;
        uint32_t b = bloc % B;
        uint32_t ek0 = bloc < nblocs ? uint32_t(__ldg(ek + bloc)) : 0u;
        uint32_t ek1 = (m0 + 1u < m1 && bloc + 8u < nblocs) ? uint32_t(__ldg(ek + bloc + 8u)) : 0u;
        uint32_t mot_p, bloc_p, b_p, ek_p;
        {
            const uint32_t ctx = bloc < nblocs ? (ek0 < 128u ? 0u : (ek0 == 128u ? 1u : 2u)) : 0u;
            const uint32_t ek2 = (m0 + 2u < m1 && bloc + 16u < nblocs) ? uint32_t(__ldg(ek + bloc + 16u)) : 0u;
            d.avancer();
            mot_p = d.macro(lut_s + ctx * (M * 4u));
            bloc_p = bloc;
            b_p = b;
            ek_p = ek0;
            bloc += 8u;
            b += 8u;
            b -= b >= B ? B : 0u;
            ek0 = ek1;
            ek1 = ek2;
        }
        for (uint32_t m = m0 + 1; m < m1; ++m) {
            const uint32_t ctx = bloc < nblocs ? (ek0 < 128u ? 0u : (ek0 == 128u ? 1u : 2u)) : 0u;
            const uint32_t ek2 = (m + 2u < m1 && bloc + 16u < nblocs) ? uint32_t(__ldg(ek + bloc + 16u)) : 0u;
            d.avancer();
            GemvTuile::Etapes et;
            const bool valide_p = bloc_p < nblocs;
            const uint32_t mot = d.macro(lut_s + ctx * (M * 4u), [&](auto k) {
                gv.etape<decltype(k)::value>(et, mot_p, bloc_p, b_p, ek_p, valide_p);
            });
            gv.fermer(m - 1u, m1);
            mot_p = mot;
            bloc_p = bloc;
            b_p = b;
            ek_p = ek0;
            bloc += 8u;
            b += 8u;
            b -= b >= B ? B : 0u;
            ek0 = ek1;
            ek1 = ek2;
        }
        gv.accumuler(mot_p, bloc_p, b_p, ek_p, bloc_p < nblocs);
        gv.fermer(m1 - 1u, m1);
        d.bilan(hors_l, pointeur);
        d.terminer();
    }
    verser_controle(controle, voie, hors_l, pointeur);
}

// ------------------------------------------------------------------ raw parts: row-centric

__global__ void __launch_bounds__(MOE_WARPS * 32) k_moe_brut(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fe, fc;
    const bool bon = B > 0 && partie_de(c, i, partie, taille) && trouver_flux(partie, taille, SORTE_ECHELLES_BRUTES, j, fe) &&
                     trouver_flux(partie, taille, SORTE_CODES_BRUTS, j, fc) && fe.produits == nblocs &&
                     fe.longueur >= nblocs && fc.produits == 16u * nblocs && fc.longueur >= 16u * nblocs;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    float* x2s = reinterpret_cast<float*>(dyn);
    if (j < 2)
        charger_x2(x2s, c.x, c.x_bf16, C);
    else
        charger_x2(x2s, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const float4* x2s4 = reinterpret_cast<const float4*>(x2s);
    auto x2f4 = [x2s4](uint32_t t) { return x2s4[t]; };
    const uint32_t K = a.plan.K[j];
    float* parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * K;
    for (uint32_t r = blockIdx.x * MOE_WARPS + (threadIdx.x >> 5); r < R; r += gridDim.x * MOE_WARPS)
        ligne_segments(fc.p, fe.p, x2f4, r, B, voie, parts + uint64_t(r) * K);
}

// ------------------------------------------------------------------ 3. SwiGLU of the gate/up rows

__device__ __forceinline__ float swiglu_f64(float g, float u) {
    const double gv = fmin(double(g), 7.0);
    const double uv = fmin(fmax(double(u), -7.0), 7.0);
    return float(gv / (1.0 + exp(-1.702 * gv)) * (uv + 1.0));
}

__global__ void __launch_bounds__(256) k_moe_swiglu(ArgsMoe a) {
    __shared__ const float* biais[2];
    const Couche& c = a.c;
    const uint32_t i = blockIdx.y;
    if (threadIdx.x < 2) {
        const uint8_t* partie;
        uint64_t taille;
        Flux fb;
        const uint32_t j = threadIdx.x;
        biais[j] = (partie_de(c, i, partie, taille) && trouver_flux(partie, taille, SORTE_BIAIS, j, fb) &&
                    fb.longueur >= 4u * c.lignes[j])
                       ? reinterpret_cast<const float*>(fb.p)
                       : nullptr;
    }
    __syncthreads();
    attendre_amont();
    liberer_aval();
    const uint32_t R = c.lignes[0], r = blockIdx.x * 256u + threadIdx.x;
    if (r >= R) return;
    float* h = reinterpret_cast<float*>(a.espace + a.plan.h) + uint64_t(i) * R;
    if (biais[0] == nullptr || biais[1] == nullptr) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&c.controle[4u * i + CTL_FORMAT], 1u);
        h[r] = 0.0f;
        return;
    }
    const float* p0 = reinterpret_cast<const float*>(a.espace + a.plan.parts[0]) + (uint64_t(i) * R + r) * a.plan.K[0];
    const float* p1 = reinterpret_cast<const float*>(a.espace + a.plan.parts[1]) + (uint64_t(i) * R + r) * a.plan.K[1];
    const float gv = finir_ligne(p0, r, c.colonnes[0] / 32u) + biais[0][r];
    const float uv = finir_ligne(p1, r, c.colonnes[1] / 32u) + biais[1][r];
    h[r] = swiglu_f64(gv, uv);
}

// ------------------------------------------------------------------ 5. down rows, combine

__global__ void __launch_bounds__(256) k_moe_combiner(ArgsMoe a) {
    __shared__ const float* biais[8];
    const Couche& c = a.c;
    if (threadIdx.x < c.k) {
        const uint8_t* partie;
        uint64_t taille;
        Flux fb;
        biais[threadIdx.x] = (partie_de(c, threadIdx.x, partie, taille) && trouver_flux(partie, taille, SORTE_BIAIS, 2, fb) &&
                              fb.longueur >= 4u * c.lignes[2])
                                 ? reinterpret_cast<const float*>(fb.p)
                                 : nullptr;
    }
    __syncthreads();
    attendre_amont();
    liberer_aval();
    const uint32_t R = c.lignes[2], r = blockIdx.x * 256u + threadIdx.x;
    if (r >= R) return;
    const uint32_t B = c.colonnes[2] / 32u, K = a.plan.K[2];
    const float* parts = reinterpret_cast<const float*>(a.espace + a.plan.parts[2]);
    float s = 0.0f;
    for (uint32_t i = 0; i < c.k; ++i) {
        const float b = biais[i] != nullptr ? biais[i][r] : 0.0f;
        const float si = finir_ligne(parts + (uint64_t(i) * R + r) * K, r, B) + b;
        const float p = __fmul_rn(c.poids[i], si);
        s = i == 0 ? p : __fadd_rn(s, p);
    }
    c.residu[r] = __fadd_rn(c.residu[r], s);
}

// ------------------------------------------------------------------ launcher

cudaError_t lancer_moe(const Couche& c, void* espace, cudaStream_t flux, cudaEvent_t const* ev) {
    auto marque = [&](int i) {
        if (ev != nullptr && ev[i] != nullptr) cudaEventRecord(ev[i], flux);
    };
    ArgsMoe a{c, static_cast<uint8_t*>(espace), plan_espace(c.lignes, c.colonnes, c.k), 0};
    const uint32_t nd = c.n_delta ? c.n_delta : 256u, nc = c.n_codes ? c.n_codes : 256u;
    uint32_t td = 1, tc = 1;
    for (int j = 0; j < 3; ++j) {
        const uint64_t nb = uint64_t(c.lignes[j]) * (c.colonnes[j] / 32u);
        td = std::max<uint32_t>(td, uint32_t(((nb + 127) / 128 + nd - 1) / nd));
        tc = std::max<uint32_t>(tc, uint32_t(((16 * nb + 127) / 128 + nc - 1) / nc));
    }
    const uint32_t cmax = std::max(c.colonnes[0], c.colonnes[2]);
    cudaError_t e;
    marque(0);
    if (!c.brut) {
        if ((e = lancer_pdl(k_moe_delta, dim3((td + DELTA_WARPS - 1) / DELTA_WARPS, 3, c.k), dim3(DELTA_WARPS * 32), 0,
                            flux, a)) != cudaSuccess)
            return e;
        const size_t smem = 3u * M * 4u + MOE_WARPS * ANNEAU_ALLOC * 2u + medianes_octets(c) + 4u * cmax;
        if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_codes), int(smem))) != cudaSuccess) return e;
        marque(1);
        const dim3 grille((tc + MOE_WARPS - 1) / MOE_WARPS, 2, c.k);
        if ((e = lancer_pdl(k_moe_codes, grille, dim3(MOE_WARPS * 32), smem, flux, a)) != cudaSuccess) return e;
        marque(2);
        if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, c.k, 1), dim3(256), 0, flux, a)) != cudaSuccess)
            return e;
        marque(3);
        a.j0 = 2;
        if ((e = lancer_pdl(k_moe_codes, dim3(grille.x, 1, c.k), dim3(MOE_WARPS * 32), smem, flux, a)) != cudaSuccess)
            return e;
        marque(4);
    } else {
        const size_t smem = 4u * cmax;
        if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_brut), int(smem))) != cudaSuccess) return e;
        const uint32_t rmax = std::max(c.lignes[0], c.lignes[2]);
        const uint32_t gx = (rmax + MOE_WARPS - 1) / MOE_WARPS;
        marque(1);
        if ((e = lancer_pdl(k_moe_brut, dim3(gx, 2, c.k), dim3(MOE_WARPS * 32), smem, flux, a)) != cudaSuccess) return e;
        marque(2);
        if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, c.k, 1), dim3(256), 0, flux, a)) != cudaSuccess)
            return e;
        marque(3);
        a.j0 = 2;
        if ((e = lancer_pdl(k_moe_brut, dim3(gx, 1, c.k), dim3(MOE_WARPS * 32), smem, flux, a)) != cudaSuccess) return e;
        marque(4);
    }
    if ((e = lancer_pdl(k_moe_combiner, dim3((c.lignes[2] + 255) / 256), dim3(256), 0, flux, a)) != cudaSuccess) return e;
    marque(5);
    return cudaGetLastError();
}

}  // namespace tb
