// troncons_b200 — the fused MoE layer: rANS decoding of the routed experts' parts fused into
// the MXFP4 GEMV, then SwiGLU, the down projection and the weighted combine.
//
// The reference runs, per layer and routed expert, decoder_echelles + decoder_codes into an
// SoA slot in VRAM, then gemv_mxfp4 x3, swiglu_oai, and combiner over the k experts
// (trc-modele/src/lib.rs:533-553, trc-ordo/src/lib.rs:1328-1367). Here, on the caller's stream:
//   1. k_moe_delta   DELTA_j of the k routed experts -> the delta byte of every block, into the
//                    workspace (259,200 bytes per matrix: it stays in L2);
//   2. k_moe_codes   (gate, up) per CODES_CTX tile, a producer warp runs the decode chain (one
//                    word per lane and macro-step, table chosen by the block's scale class) and
//                    hands each 32-macro-step segment of words through shared memory to a
//                    consumer warp, which multiplies it against 2x staged in shared memory; the
//                    block's scale = median + delta - 128. The codes never leave the SM. Rows
//                    are closed where they end and at every segment end (256 blocks), giving
//                    per-(row, segment) partials;
//   3. k_moe_swiglu  gate and up rows = fold of their partials + bias; h = SwiGLU (f64);
//   4. k_moe_codes   (down) the same on h;
//   5. k_moe_combiner down rows + bias, then residual += ((w0 s0 + w1 s1) + ...), no FMA.
// That is the sequential schedule. Given a workspace that holds the down projection's decoded
// words (up to 32 activations), the overlapped schedule runs 2 and 4's decode in ONE launch of
// k_moe_codes_dense (gate/up tiles decoded into their GEMV, down tiles decoded alone into the
// workspace), then 3, then k_moe_bas (the down GEMV on those words, segment by segment, with the
// same closing), then 5: the down chain runs during gate/up. Both give the same bits.
// The raw path (`brut`) replaces 1-2 and 4 by k_moe_brut, a row-centric GEMV on CODES_BRUTS /
// ECHELLES_BRUTES writing the same partials, so compressed and raw parts give the same bits.
// Integrity counters go to controle[4 i ..] of active expert i (format errors included).
#include <cuda_bf16.h>

#include "commun.cuh"
#include "gemv_groupes.cuh"
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
    const uint64_t nb2 = uint64_t(lignes[2]) * (colonnes[2] / 32u);
    e.cd = p;
    p = al256(p + 16ull * nb2 * k);
    e.total_recouvrant = p;
    for (int j = 0; j < 2; ++j) {
        e.cdh[j] = p;
        p = al256(p + 16ull * (uint64_t(lignes[j]) * (colonnes[j] / 32u)) * k);
    }
    e.total_tout = p;
    return e;
}

struct ArgsMoe {
    Couche c;
    uint8_t* espace;
    Espace plan;
    uint32_t j0;     // first matrix of this launch (0: gate and up; 2: down)
    uint32_t seuls;  // 1: the down projection's codes are decoded with gate/up, into the workspace;
                     // 2: all three matrices' codes are (their GEMVs follow, in row groups)
    uint32_t tous;   // k_moe_delta decodes every expert of the layer: activation i = expert i
    uint64_t pre_ek[3];  // with c.deltas: offset of matrix j's delta bytes ([experts][blocks])
};

// Activation i's delta bytes of matrix j (one per block): decoded by this call into the
// workspace, or decoded ahead for every expert of the layer (c.deltas).
__device__ __forceinline__ const uint8_t* deltas_de(const ArgsMoe& a, uint32_t i, uint32_t j, uint32_t nblocs) {
    if (a.c.deltas != nullptr) return a.c.deltas + a.pre_ek[j] + uint64_t(a.c.indices[i]) * nblocs;
    return a.espace + a.plan.ek[j] + uint64_t(i) * nblocs;
}

// Whether activation i's expert is held by this call (others are skipped: no work, no error).
__device__ __forceinline__ bool tenu(const Couche& c, uint32_t i) {
    const uint32_t e = c.indices[i];
    return c.expert_fin == 0 || (e >= c.expert_debut && e < c.expert_fin);
}

// Activation i's input: its token's x.
__device__ __forceinline__ const void* x_de(const Couche& c, uint32_t i) {
    return static_cast<const uint8_t*>(c.x) + uint64_t(i / c.k) * c.colonnes[0] * (c.x_bf16 ? 2u : 4u);
}

// The part of activation i's expert, if it is addressable.
__device__ __forceinline__ bool partie_de(const Couche& c, uint32_t i, const uint8_t*& partie, uint64_t& taille) {
    const uint32_t e = c.indices[i];
    if (e >= c.experts) return false;
    partie = reinterpret_cast<const uint8_t*>(c.parties[e]);
    taille = c.parties_octets[e];
    return partie != nullptr && taille >= 64 && (reinterpret_cast<uintptr_t>(partie) & 15u) == 0;
}

// Copies n 16-byte chunks into shared memory; each thread has up to 8 loads in flight before
// it stores (the prologues are latency-bound: a load at a time would cost one L2 round trip
// per chunk).
__device__ __forceinline__ void copier16(uint4* dst, const uint4* __restrict__ src, uint32_t n) {
    uint32_t t = threadIdx.x;
    const uint32_t pas = blockDim.x;
    for (; t + 7u * pas < n; t += 8u * pas) {
        uint4 v[8];
#pragma unroll
        for (uint32_t k = 0; k < 8u; ++k) v[k] = __ldg(src + t + k * pas);
#pragma unroll
        for (uint32_t k = 0; k < 8u; ++k) dst[t + k * pas] = v[k];
    }
    for (; t < n; t += pas) dst[t] = __ldg(src + t);
}

// A table of M entries s | (f - 1) << 8 | (i - c) << 20 (abi.rs:187-221's layout) restaged as
// {f, i - c} pairs and a byte table of the symbols, for Decodeur::pas_avance2; each thread has up
// to 8 loads of 4 entries in flight before it stores.
__device__ __forceinline__ void restager_lut2(uint2* lut2, uint8_t* symboles, const uint32_t* __restrict__ src) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    const uint32_t pas = blockDim.x;
    auto poser = [&](uint32_t q, const uint4 v) {
        const uint32_t e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
            lut2[4u * q + k] = make_uint2(((e[k] >> 8) & 0xFFFu) + 1u, e[k] >> 20);
            symboles[4u * q + k] = uint8_t(e[k]);
        }
    };
    uint32_t t = threadIdx.x;
    for (; t + 7u * pas < M / 4u; t += 8u * pas) {
        uint4 v[8];
#pragma unroll
        for (uint32_t k = 0; k < 8u; ++k) v[k] = __ldg(s4 + t + k * pas);
#pragma unroll
        for (uint32_t k = 0; k < 8u; ++k) poser(t + k * pas, v[k]);
    }
    for (; t < M / 4u; t += pas) poser(t, __ldg(s4 + t));
}

constexpr uint32_t DELTA_WARPS = 1;  // one DELTA tile per block: each chain alone on its SM
constexpr uint32_t MOE_WARPS = 8;  // k_moe_brut: warps per block (one row at a time each)
constexpr uint32_t BRUT_BLOCS_SM = 3;  // its blocks per SM: the grid is one wave of them

// ------------------------------------------------------------------ 1. DELTA -> scales, classes

// PAIRES: the table restaged as {f, i - c} pairs (39 KB of shared memory per block: the shorter
// chain, for launches whose blocks all fit the SMs at once); otherwise the table as stored (18 KB:
// twice as many blocks per SM when a launch runs in waves, every expert of a layer at once).
template <bool PAIRES>
__global__ void __launch_bounds__(DELTA_WARPS * 32) k_moe_delta(ArgsMoe a) {
    __shared__ __align__(16) uint32_t lut_brute[PAIRES ? 1 : M];
    __shared__ __align__(16) uint2 lut2[PAIRES ? M : 1];
    __shared__ __align__(16) uint8_t symboles[PAIRES ? M : 1];
    __shared__ __align__(16) uint16_t anneaux[DELTA_WARPS][ANNEAU_ALLOC];
    const Couche& c = a.c;
    const uint32_t j = blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u;
    // The LUTs are an input of the layer; the routed experts come from the previous kernel.
    if constexpr (PAIRES)
        restager_lut2(lut2, symboles, c.luts + (uint64_t(j) * 4u) * M);
    else
        copier16(reinterpret_cast<uint4*>(lut_brute), reinterpret_cast<const uint4*>(c.luts + (uint64_t(j) * 4u) * M),
                 M / 4u);
    attendre_amont();
    liberer_aval();
    if (!a.tous && !tenu(c, i)) return;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], B = c.colonnes[j] / 32u, nblocs = R * B;
    const uint8_t* partie = nullptr;
    uint64_t taille = 0;
    Flux fd;
    EnteteRans h;
    bool a_partie;
    if (a.tous) {  // every expert of the layer, in order; one not held here (no part) is skipped
        if (c.parties[i] == 0) return;
        partie = reinterpret_cast<const uint8_t*>(c.parties[i]);
        taille = c.parties_octets[i];
        a_partie = partie != nullptr && taille >= 64 && (reinterpret_cast<uintptr_t>(partie) & 15u) == 0;
    } else {
        a_partie = partie_de(c, i, partie, taille);
    }
    const bool bon = a_partie && trouver_flux_warp(partie, taille, SORTE_DELTA, j, fd) && lire_entete(fd, nblocs, h);
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const uint32_t warp0 = blockIdx.x * DELTA_WARPS;
    if (warp0 >= h.T) return;
    __syncthreads();
    uint8_t* delta = a.espace + a.plan.ek[j] + uint64_t(i) * nblocs;
    const uint32_t nmacro = h.P / 128u;
    uint32_t hors_l = 0, pointeur = 0;
    Decodeur d;
    for (uint32_t t = warp0 + (threadIdx.x >> 5); t < h.T; t += gridDim.x * DELTA_WARPS) {
        d.debut(h, t, voie, anneaux[threadIdx.x >> 5]);
        // one table for every lane: the look-ahead form
        Decodeur::Avance2 av2;
        Decodeur::Avance av;
        if constexpr (PAIRES)
            d.debut_avance2(lut2, av2);
        else
            d.debut_avance(lut_brute, av);
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        // Word w = 32 m + lane is the delta of blocks 4w .. 4w + 3, stored as it comes.
        for (uint32_t m = m0; m < m1; ++m) {
            d.avancer();
            uint32_t mot;
            if constexpr (PAIRES)
                mot = d.macro_avance2(lut2, symboles, av2);
            else
                mot = d.macro_avance(lut_brute, av);
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
// (X2_PAS, x2_octets, x2_indice, charger_x2: mxfp4.cuh)

// ------------------------------------------------------------------ 2/4. CODES_CTX decoded into the GEMV

// The GEMV of decoded macro-steps (8 blocks, one word per lane) into the row partials: the
// block's sum (quad tree), scaled and accumulated on the current row or the next; rows closed
// where they end, and the row in progress closed at the segment's (or the tile's) end.
struct GemvTuile {
    float acc, acc_s;       // current row r, next row
    uint32_t r, fin_r;      // warp-uniform: current row, first block of the next row
    uint32_t med_r, med_s;  // medians of rows r and r + 1 (clamped to the last row)
    uint32_t evt;           // the next macro-step after which a row or a segment closes
    uint32_t R, B, K, voie;
    float* parts;
    const uint8_t* med;     // row medians (shared memory)
    const float* puiss;     // 2^(e - 128) for e = 0..255 (shared memory, echelle_e8m0)

    // The macro-step, from m on, that ends row r, segment m / 32 or the tile.
    __device__ __forceinline__ uint32_t prochain(uint32_t m, uint32_t m1) const {
        return min(min((fin_r - 1u) / 8u, m | (SEGMENT_MACRO - 1u)), m1 - 1u);
    }

    __device__ __forceinline__ void debut(uint32_t m0, uint32_t m1) {
        acc = 0.0f;
        acc_s = 0.0f;
        r = (8u * m0) / B;
        fin_r = (r + 1u) * B;
        med_r = med[min(r, R - 1u)];
        med_s = med[min(r + 1u, R - 1u)];
        evt = prochain(m0, m1);
    }

    // Block `bloc`'s quad sum s, scaled by 2^(median + delta - 256) of its row (r or r + 1).
    __device__ __forceinline__ void accumuler(float s, uint32_t bloc, uint32_t delta, bool valide) {
        const bool cour = bloc < fin_r;
        const float sc = puiss[((cour ? med_r : med_s) + delta - 128u) & 255u];
        acc = (valide && cour) ? fmaf(s, sc, acc) : acc;
        acc_s = (valide && !cour) ? fmaf(s, sc, acc_s) : acc_s;
    }

    // Row and segment closing after macro-step m (warp-uniform): nothing to do before evt.
    __device__ __forceinline__ void fermer(uint32_t m, uint32_t m1) {
        if (m != evt) return;
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
        if (m + 1u < m1) evt = prochain(m + 1u, m1);
    }
};

// The table of block scales: 2^(e - 128) for the 256 E8M0 values (echelle_e8m0's, exactly).
__device__ __forceinline__ void charger_puissances(float* puiss) {
    for (uint32_t t = threadIdx.x; t < 256u; t += blockDim.x) puiss[t] = echelle_e8m0(t);
}

// Decode and multiply run in different warps of a block: MOE_PAIRES producer warps each
// decode one CODES_CTX tile (the bare rANS chain, one word per lane and macro-step, table
// chosen by the block's scale class), writing the words and the blocks' delta bytes into a
// segment buffer in shared memory (one segment = 32 macro-steps, double-buffered); the paired
// consumer warp multiplies each finished segment while the next one decodes. One hand-off per
// segment, through two mbarriers per buffer (full: 32 producer lanes arrive; empty: 32 consumer
// lanes arrive), every wait bounded.
constexpr uint32_t MOE_PAIRES = 4;
constexpr uint32_t SEG_TAMPONS = 2;
constexpr uint32_t SEG_MOTS = SEGMENT_MACRO * 32u;  // words of one segment buffer
constexpr uint32_t SEG_DELTAS = SEGMENT_MACRO * 8u;  // delta bytes of one segment buffer

// Shared bytes for the row medians of the largest matrix (16-aligned so that 2x stays aligned).
__host__ __device__ __forceinline__ uint32_t medianes_octets(const Couche& c) {
    return (max(c.lignes[0], c.lignes[2]) + 15u) & ~15u;
}

// Dynamic shared memory of k_moe_codes: 3 LUTs, the producers' word rings, the segment
// buffers (words, deltas), the medians, 2x, the mbarriers.
struct DispositionCodes {
    uint32_t anneaux, mots, deltas, med, puiss, x2, barrieres, total;
};
__host__ __device__ __forceinline__ DispositionCodes disposition_codes(const Couche& c) {
    DispositionCodes d;
    const uint32_t cmax = max(c.colonnes[0], c.colonnes[2]);
    d.anneaux = 3u * M * 4u;
    d.mots = d.anneaux + MOE_PAIRES * ANNEAU_ALLOC * 2u;
    d.deltas = d.mots + MOE_PAIRES * SEG_TAMPONS * SEG_MOTS * 4u;
    d.med = d.deltas + MOE_PAIRES * SEG_TAMPONS * SEG_DELTAS;
    d.puiss = d.med + medianes_octets(c);
    d.x2 = d.puiss + 1024u;
    d.barrieres = d.x2 + x2_octets(cmax);
    d.total = d.barrieres + MOE_PAIRES * 2u * SEG_TAMPONS * 8u;
    return d;
}

__device__ __forceinline__ uint32_t classe_delta(uint32_t d) { return d < 128u ? 0u : (d == 128u ? 1u : 2u); }

__global__ void __launch_bounds__(MOE_PAIRES * 64, 2) k_moe_codes(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u;
    const uint32_t warp = threadIdx.x >> 5, paire = warp % MOE_PAIRES;
    // The routed experts come from the router: without the DELTA launch between them (deltas
    // decoded ahead), this launch follows the router directly and waits before reading them.
    if (c.deltas != nullptr) attendre_amont();
    if (!tenu(c, i)) return;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fc, fm;
    EnteteRans h;
    const bool bon = B >= 8u && partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_CODES_CTX, j, fc) &&
                     trouver_flux_warp(partie, taille, SORTE_MEDIANES, j, fm) && fm.produits == R && fm.longueur >= R &&
                     R <= 8192u && lire_entete(fc, nblocs * 16u, h) && (h.N % SEGMENT_MACRO) == 0;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const uint32_t warp0 = blockIdx.x * MOE_PAIRES;
    if (warp0 >= h.T) return;
    const DispositionCodes dc = disposition_codes(c);
    uint32_t* lut = reinterpret_cast<uint32_t*>(dyn);
    uint8_t* med = dyn + dc.med;
    float* puiss = reinterpret_cast<float*>(dyn + dc.puiss);
    float* x2s = reinterpret_cast<float*>(dyn + dc.x2);
    uint64_t* barrieres = reinterpret_cast<uint64_t*>(dyn + dc.barrieres);
    charger_puissances(puiss);
    copier16(reinterpret_cast<uint4*>(lut), reinterpret_cast<const uint4*>(c.luts + (uint64_t(j) * 4u + 1u) * M),
             3u * M / 4u);
    if (fm.p + ((R + 15u) & ~15u) <= partie + taille)
        copier16(reinterpret_cast<uint4*>(med), reinterpret_cast<const uint4*>(fm.p), (R + 15u) / 16u);
    else
        for (uint32_t t = threadIdx.x; t < R; t += blockDim.x) med[t] = fm.p[t];
    if (j < 2) charger_x2(x2s, x_de(c, i), c.x_bf16, C);
    if (threadIdx.x < MOE_PAIRES * 2u * SEG_TAMPONS) mbar_init(barrieres + threadIdx.x, 32u);
    const uint32_t paire_t0 = warp0 + paire;
    Decodeur d;
    uint16_t* anneau = reinterpret_cast<uint16_t*>(dyn + dc.anneaux) + paire * ANNEAU_ALLOC;
    // The producer starts its first tile (states, first word chunks): the part is an input of
    // the layer, so this overlaps the previous kernel's tail.
    if (warp < MOE_PAIRES && paire_t0 < h.T) d.debut(h, paire_t0, voie, anneau);
    // Everything above reads inputs the layer's first kernel waited for; the delta bytes (and h
    // for the down projection) come from the previous kernel.
    attendre_amont();
    liberer_aval();
    if (j == 2) charger_x2(x2s, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();

    uint32_t* mots = reinterpret_cast<uint32_t*>(dyn + dc.mots) + paire * SEG_TAMPONS * SEG_MOTS;  // [b][m][lane]
    uint8_t* deltas = dyn + dc.deltas + paire * SEG_TAMPONS * SEG_DELTAS;                          // [b][m][g]
    uint64_t* pleins = barrieres + paire * 2u * SEG_TAMPONS;
    uint64_t* vides = pleins + SEG_TAMPONS;
    const uint32_t nmacro = h.P / 128u;
    const uint32_t g = voie >> 2;
    const uint32_t pas_tuiles = gridDim.x * MOE_PAIRES;
    bool abandon = false;

    if (warp < MOE_PAIRES) {
        // ---------------- producer: the decode chain
        const uint8_t* __restrict__ ek = deltas_de(a, i, j, nblocs);  // delta bytes
        uint32_t hors_l = 0, pointeur = 0, n = 0;
        for (uint32_t t = paire_t0; t < h.T && !abandon; t += pas_tuiles) {
            if (t != paire_t0) d.debut(h, t, voie, anneau);
            const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
            // This lane's block at macro-step m is 8 m + g; its delta read two macro-steps ahead.
            uint32_t bloc = 8u * m0 + g;
            uint32_t e0 = bloc < nblocs ? uint32_t(__ldg(ek + bloc)) : 0u;
            uint32_t e1 = (m0 + 1u < m1 && bloc + 8u < nblocs) ? uint32_t(__ldg(ek + bloc + 8u)) : 0u;
            for (uint32_t s0 = m0; s0 < m1; s0 += SEGMENT_MACRO, ++n) {
                const uint32_t b = n % SEG_TAMPONS;
                if (n >= SEG_TAMPONS && !mbar_attendre(&vides[b], ((n / SEG_TAMPONS) - 1u) & 1u)) {
                    abandon = true;
                    break;
                }
                uint32_t* mb = mots + b * SEG_MOTS;
                uint8_t* db = deltas + b * SEG_DELTAS;
                const uint32_t s1 = min(s0 + SEGMENT_MACRO, m1);
                for (uint32_t m = s0; m < s1; ++m) {
                    const uint32_t ctx = bloc < nblocs ? classe_delta(e0) : 0u;
                    const uint32_t e2 = (m + 2u < m1 && bloc + 16u < nblocs) ? uint32_t(__ldg(ek + bloc + 16u)) : 0u;
                    d.avancer();
                    mb[(m - s0) * 32u + voie] = d.macro(lut + ctx * M);
                    if ((voie & 3u) == 0) db[(m - s0) * 8u + g] = uint8_t(e0);
                    bloc += 8u;
                    e0 = e1;
                    e1 = e2;
                }
                mbar_arrive(&pleins[b]);
            }
            d.bilan(hors_l, pointeur);
            d.terminer();
        }
        verser_controle(controle, voie, hors_l, pointeur);
    } else {
        // ---------------- consumer: the GEMV of each finished segment
        const float4* x2s4 = reinterpret_cast<const float4*>(x2s);
        const uint32_t q = voie & 3u;
        GemvTuile gv;
        gv.R = R;
        gv.B = B;
        gv.K = a.plan.K[j];
        gv.voie = voie;
        gv.parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * gv.K;
        gv.med = med;
        gv.puiss = puiss;
        uint32_t n = 0;
        for (uint32_t t = warp0 + paire; t < h.T && !abandon; t += pas_tuiles) {
            const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
            gv.debut(m0, m1);
            uint32_t bloc = 8u * m0 + g;
            uint32_t bc = bloc % B;  // column block of `bloc` in its row
            for (uint32_t s0 = m0; s0 < m1; s0 += SEGMENT_MACRO, ++n) {
                const uint32_t b = n % SEG_TAMPONS;
                if (!mbar_attendre(&pleins[b], (n / SEG_TAMPONS) & 1u)) {
                    abandon = true;
                    break;
                }
                const uint32_t* mb = mots + b * SEG_MOTS;
                const uint8_t* db = deltas + b * SEG_DELTAS;
                const uint32_t s1 = min(s0 + SEGMENT_MACRO, m1);
                for (uint32_t m = s0; m < s1; m += 8u) {
                    // Eight macro-steps' block sums at once (independent), then their ordered
                    // accumulation with the row and segment closing.
                    float sv[8];
                    uint32_t dv[8];
#pragma unroll
                    for (uint32_t u = 0; u < 8u; ++u) {
                        const bool ok = m + u < s1;
                        const uint32_t mot = ok ? mb[(m + u - s0) * 32u + voie] : 0u;
                        dv[u] = ok ? uint32_t(db[(m + u - s0) * 8u + g]) : 0u;
                        sv[u] = somme_quad(produit_quad(mot, x2s4[X2_PAS * bc + q], x2s4[X2_PAS * bc + 4u + q]));
                        bc += 8u;
                        bc -= bc >= B ? B : 0u;
                    }
#pragma unroll
                    for (uint32_t u = 0; u < 8u; ++u) {
                        if (m + u < s1) {
                            gv.accumuler(sv[u], bloc, dv[u], bloc < nblocs);
                            gv.fermer(m + u, m1);
                            bloc += 8u;
                        }
                    }
                }
                mbar_arrive(&vides[b]);
            }
        }
    }
    if (abandon && voie == 0) atomicAdd(&controle[CTL_ATTENTE], 1u);
}

// Second form of the same launch, for launches with more tiles than the producer / consumer
// form keeps in flight (2 x MOE_PAIRES per SM): one warp per tile both decodes and multiplies,
// DENSE_WARPS warps per block sharing the LUTs, up to two blocks per SM. The product of
// macro-step m - 1 runs in stages between the four sub-steps of macro-step m's decode. Same
// partials, same bits. 11 warps: a config-1 launch (3 x 4 matrices of 127 tiles) is 144 blocks,
// one per SM with at most 11 tiles each, where blocks of 12 were 132, 12 tiles on each of 132
// SMs and 16 SMs idle; the chains run faster with fewer tiles per SM.
constexpr uint32_t DENSE_WARPS = 11;

struct DispositionDense {
    uint32_t anneaux, med, puiss, x2, total;
};
__host__ __device__ __forceinline__ DispositionDense disposition_dense(const Couche& c) {
    DispositionDense d;
    const uint32_t cmax = max(c.colonnes[0], c.colonnes[2]);
    d.anneaux = 3u * M * 4u;
    d.med = d.anneaux + DENSE_WARPS * ANNEAU_ALLOC * 2u;
    d.puiss = d.med + medianes_octets(c);
    d.x2 = d.puiss + 1024u;
    d.total = d.x2 + x2_octets(cmax);
    return d;
}

// A word's quad sum against 2x in three stages: loads and conversions; the fmaf chain; the quad
// tree (the order of produit_quad + somme_quad).
struct ProduitEtage {
    float lo[4], hi[4];
    float4 xa, xb;
    float p;
    template <int K>
    __device__ __forceinline__ void etape(uint32_t mot, const float4* x2s4, uint32_t b, uint32_t q) {
        if constexpr (K == 0) {
            xa = x2s4[X2_PAS * b + q];
            xb = x2s4[X2_PAS * b + 4u + q];
            e2m1_mot(mot, lo, hi);
        } else if constexpr (K == 1) {
            float t = 0.0f;
            t = fmaf(lo[0], xa.x, t);
            t = fmaf(hi[0], xb.x, t);
            t = fmaf(lo[1], xa.y, t);
            t = fmaf(hi[1], xb.y, t);
            t = fmaf(lo[2], xa.z, t);
            t = fmaf(hi[2], xb.z, t);
            t = fmaf(lo[3], xa.w, t);
            t = fmaf(hi[3], xb.w, t);
            p = t;
        } else if constexpr (K == 2) {
            p = somme_quad(p);
        }
    }
};

__global__ void __launch_bounds__(DENSE_WARPS * 32, 2) k_moe_codes_dense(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    if (c.deltas != nullptr) attendre_amont();  // as in k_moe_codes: the routed experts first
    if (!tenu(c, i)) return;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fc, fm;
    EnteteRans h;
    const bool bon = B >= 8u && partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_CODES_CTX, j, fc) &&
                     trouver_flux_warp(partie, taille, SORTE_MEDIANES, j, fm) && fm.produits == R && fm.longueur >= R &&
                     R <= 8192u && lire_entete(fc, nblocs * 16u, h) && (h.N % SEGMENT_MACRO) == 0;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const uint32_t warp0 = blockIdx.x * DENSE_WARPS;
    if (warp0 >= h.T) return;
    const DispositionDense dd = disposition_dense(c);
    uint32_t* lut = reinterpret_cast<uint32_t*>(dyn);
    uint16_t* anneau = reinterpret_cast<uint16_t*>(dyn + dd.anneaux) + warp * ANNEAU_ALLOC;
    uint8_t* med = dyn + dd.med;
    float* puiss = reinterpret_cast<float*>(dyn + dd.puiss);
    float* x2s = reinterpret_cast<float*>(dyn + dd.x2);
    charger_puissances(puiss);
    copier16(reinterpret_cast<uint4*>(lut), reinterpret_cast<const uint4*>(c.luts + (uint64_t(j) * 4u + 1u) * M),
             3u * M / 4u);
    if (fm.p + ((R + 15u) & ~15u) <= partie + taille)
        copier16(reinterpret_cast<uint4*>(med), reinterpret_cast<const uint4*>(fm.p), (R + 15u) / 16u);
    else
        for (uint32_t t = threadIdx.x; t < R; t += blockDim.x) med[t] = fm.p[t];
    const bool seul = (j == 2 && a.seuls != 0u) || a.seuls == 2u;  // decode only (down: h does not exist yet)
    if (j < 2 && !seul) charger_x2(x2s, x_de(c, i), c.x_bf16, C);
    const uint32_t t0 = warp0 + warp;
    Decodeur d;
    if (t0 < h.T) d.debut(h, t0, voie, anneau);  // the part is a layer input: start before the wait
    attendre_amont();
    liberer_aval();
    if (j == 2 && !seul) charger_x2(x2s, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const uint8_t* __restrict__ ek = deltas_de(a, i, j, nblocs);  // delta bytes
    const float4* x2s4 = reinterpret_cast<const float4*>(x2s);
    const uint32_t q = voie & 3u, g = voie >> 2;
    const uint32_t nmacro = h.P / 128u;
    uint32_t hors_l = 0, pointeur = 0;
    if (seul) {
        // The down projection's tiles while gate/up multiply: the words go to the workspace in
        // stream order (word 32 m + lane = bytes 4 (32 m + lane) .. + 3 of the codes); k_moe_bas
        // multiplies them once h exists.
        uint32_t* cd = reinterpret_cast<uint32_t*>(a.espace + (j == 2 ? a.plan.cd : a.plan.cdh[j])) + uint64_t(i) * 4u * nblocs;
        for (uint32_t t = t0; t < h.T; t += gridDim.x * DENSE_WARPS) {
            if (t != t0) d.debut(h, t, voie, anneau);
            const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
            uint32_t bloc = 8u * m0 + g;
            uint32_t e0 = bloc < nblocs ? uint32_t(__ldg(ek + bloc)) : 0u;
            uint32_t e1 = (m0 + 1u < m1 && bloc + 8u < nblocs) ? uint32_t(__ldg(ek + bloc + 8u)) : 0u;
            for (uint32_t m = m0; m < m1; ++m) {
                const uint32_t ctx = bloc < nblocs ? classe_delta(e0) : 0u;
                const uint32_t e2 = (m + 2u < m1 && bloc + 16u < nblocs) ? uint32_t(__ldg(ek + bloc + 16u)) : 0u;
                d.avancer();
                const uint32_t mot = d.macro(lut + ctx * M);
                if (bloc < nblocs) cd[m * 32u + voie] = mot;
                bloc += 8u;
                e0 = e1;
                e1 = e2;
            }
            d.bilan(hors_l, pointeur);
            d.terminer();
        }
        verser_controle(controle, voie, hors_l, pointeur);
        return;
    }
    GemvTuile gv;
    gv.R = R;
    gv.B = B;
    gv.K = a.plan.K[j];
    gv.voie = voie;
    gv.parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * gv.K;
    gv.med = med;
    gv.puiss = puiss;
    for (uint32_t t = t0; t < h.T; t += gridDim.x * DENSE_WARPS) {
        if (t != t0) d.debut(h, t, voie, anneau);
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        gv.debut(m0, m1);
        // This lane's block at macro-step m is 8 m + g, column block b; its delta read two
        // macro-steps ahead.
        uint32_t bloc = 8u * m0 + g;
        uint32_t b = bloc % B;
        uint32_t e0 = bloc < nblocs ? uint32_t(__ldg(ek + bloc)) : 0u;
        uint32_t e1 = (m0 + 1u < m1 && bloc + 8u < nblocs) ? uint32_t(__ldg(ek + bloc + 8u)) : 0u;
        uint32_t mot_p = 0, bloc_p = bloc, b_p = b, e_p = 0;
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t ctx = bloc < nblocs ? classe_delta(e0) : 0u;
            const uint32_t e2 = (m + 2u < m1 && bloc + 16u < nblocs) ? uint32_t(__ldg(ek + bloc + 16u)) : 0u;
            d.avancer();
            uint32_t mot;
            if (m == m0) {
                mot = d.macro(lut + ctx * M);
            } else {
                ProduitEtage pe = {};
                const bool valide_p = bloc_p < nblocs;
                mot = d.macro(lut + ctx * M, [&](auto k) {
                    constexpr int K = decltype(k)::value;
                    if constexpr (K < 3)
                        pe.etape<K>(mot_p, x2s4, b_p, q);
                    else
                        gv.accumuler(pe.p, bloc_p, e_p, valide_p);
                });
                gv.fermer(m - 1u, m1);
            }
            mot_p = mot;
            bloc_p = bloc;
            b_p = b;
            e_p = e0;
            bloc += 8u;
            b += 8u;
            b -= b >= B ? B : 0u;
            e0 = e1;
            e1 = e2;
        }
        gv.accumuler(somme_quad(produit_quad(mot_p, x2s4[X2_PAS * b_p + q], x2s4[X2_PAS * b_p + 4u + q])), bloc_p, e_p,
                     bloc_p < nblocs);
        gv.fermer(m1 - 1u, m1);
        d.bilan(hors_l, pointeur);
        d.terminer();
    }
    verser_controle(controle, voie, hors_l, pointeur);
}

// The decode launch of the overlapped schedule (every tile decode-only, the words stored for the
// row-group GEMVs), with the tiles spread evenly over the SMs. Grid (bx, 3): the bx blocks of
// matrix j (bx = SMs / 3, one block per SM) take the tiles of matrix j of every held activation
// as one list (activation by activation, tile by tile), tile g going to block g mod bx and, in
// it, warp g / bx (round-robin over the blocks first). Each SM then holds ceil(tiles / bx) chains
// or one fewer, whatever the routing, where k_moe_codes_dense's blocks of a fixed width (one
// stream's tiles each) put two blocks, 22 chains, on some SMs once the held activations pass 4:
// an expert-parallel rank's share, batches of tokens. The words and counters are
// k_moe_codes_dense's, tile for tile.
constexpr uint32_t PLAT_WARPS = 22;

__host__ __device__ __forceinline__ uint32_t plat_octets() {
    return 3u * M * 4u + PLAT_WARPS * ANNEAU_ALLOC * 2u + 4u * (RECOUVRE_MAX + 1u);
}

__global__ void __launch_bounds__(PLAT_WARPS * 32, 1) k_moe_codes_plat(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const Couche& c = a.c;
    const uint32_t j = blockIdx.y, voie = threadIdx.x & 31u, warp = threadIdx.x >> 5, W = blockDim.x >> 5;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint32_t na = min(activations(c), RECOUVRE_MAX);
    uint32_t* lut = reinterpret_cast<uint32_t*>(dyn);
    uint16_t* anneau = reinterpret_cast<uint16_t*>(dyn + 3u * M * 4u) + warp * ANNEAU_ALLOC;
    uint32_t* premier = reinterpret_cast<uint32_t*>(dyn + 3u * M * 4u + PLAT_WARPS * ANNEAU_ALLOC * 2u);
    // The routed experts are known at the start unless DELTA was decoded ahead (then the previous
    // kernel is the router's); the delta bytes are read only after the wait.
    bool attendu = false;
    auto attendre = [&] {
        if (!attendu) {
            attendre_amont();
            liberer_aval();
            attendu = true;
        }
    };
    if (c.deltas != nullptr) attendre();
    copier16(reinterpret_cast<uint4*>(lut), reinterpret_cast<const uint4*>(c.luts + (uint64_t(j) * 4u + 1u) * M),
             3u * M / 4u);
    // Tiles of each activation's stream (0 when its expert is not held or its part is malformed:
    // a malformed part counts one format error, from block 0).
    for (uint32_t i = warp; i < na; i += W) {
        uint32_t nt = 0;
        if (tenu(c, i)) {
            const uint8_t* partie;
            uint64_t taille;
            Flux fc, fm;
            EnteteRans h;
            const bool bon = B >= 8u && partie_de(c, i, partie, taille) &&
                             trouver_flux_warp(partie, taille, SORTE_CODES_CTX, j, fc) &&
                             trouver_flux_warp(partie, taille, SORTE_MEDIANES, j, fm) && fm.produits == R &&
                             fm.longueur >= R && R <= 8192u && lire_entete(fc, nblocs * 16u, h) &&
                             (h.N % SEGMENT_MACRO) == 0;
            if (bon)
                nt = h.T;
            else if (voie == 0 && blockIdx.x == 0)
                atomicAdd(&c.controle[4u * i + CTL_FORMAT], 1u);
        }
        if (voie == 0) premier[i + 1u] = nt;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        premier[0] = 0;
        for (uint32_t i = 0; i < na; ++i) premier[i + 1u] += premier[i];
    }
    __syncthreads();
    const uint32_t total = premier[na];
    uint32_t i_cour = RECOUVRE_MAX, hors_l = 0, pointeur = 0;
    for (uint32_t g = blockIdx.x + gridDim.x * warp; g < total; g += gridDim.x * W) {
        uint32_t i = 0;
        while (premier[i + 1u] <= g) ++i;
        const uint32_t t = g - premier[i];
        if (i != i_cour) {
            if (i_cour < RECOUVRE_MAX) {
                verser_controle(c.controle + 4u * i_cour, voie, hors_l, pointeur);
                hors_l = pointeur = 0;
            }
            i_cour = i;
        }
        const uint8_t* partie;
        uint64_t taille;
        Flux fc;
        EnteteRans h;
        partie_de(c, i, partie, taille);
        trouver_flux_warp(partie, taille, SORTE_CODES_CTX, j, fc);
        lire_entete(fc, nblocs * 16u, h);
        Decodeur d;
        d.debut(h, t, voie, anneau);  // the part is a layer input: its first words before the wait
        attendre();
        const uint8_t* __restrict__ ek = deltas_de(a, i, j, nblocs);
        uint32_t* cd = reinterpret_cast<uint32_t*>(a.espace + (j == 2 ? a.plan.cd : a.plan.cdh[j])) + uint64_t(i) * 4u * nblocs;
        const uint32_t g8 = voie >> 2;
        const uint32_t nmacro = h.P / 128u;
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        uint32_t bloc = 8u * m0 + g8;
        uint32_t e0 = bloc < nblocs ? uint32_t(__ldg(ek + bloc)) : 0u;
        uint32_t e1 = (m0 + 1u < m1 && bloc + 8u < nblocs) ? uint32_t(__ldg(ek + bloc + 8u)) : 0u;
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t ctx = bloc < nblocs ? classe_delta(e0) : 0u;
            const uint32_t e2 = (m + 2u < m1 && bloc + 16u < nblocs) ? uint32_t(__ldg(ek + bloc + 16u)) : 0u;
            d.avancer();
            const uint32_t mot = d.macro(lut + ctx * M);
            if (bloc < nblocs) cd[m * 32u + voie] = mot;
            bloc += 8u;
            e0 = e1;
            e1 = e2;
        }
        d.bilan(hors_l, pointeur);
        d.terminer();
    }
    if (i_cour < RECOUVRE_MAX) verser_controle(c.controle + 4u * i_cour, voie, hors_l, pointeur);
    attendre();
}

// ------------------------------------------------------------------ raw parts: row-centric

__global__ void __launch_bounds__(MOE_WARPS * 32, BRUT_BLOCS_SM) k_moe_brut(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, voie = threadIdx.x & 31u;
    if (!tenu(c, i)) return;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fe, fc;
    const bool bon = B > 0 && partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_ECHELLES_BRUTES, j, fe) &&
                     trouver_flux_warp(partie, taille, SORTE_CODES_BRUTS, j, fc) && fe.produits == nblocs &&
                     fe.longueur >= nblocs && fc.produits == 16u * nblocs && fc.longueur >= 16u * nblocs;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    float* x2s = reinterpret_cast<float*>(dyn);
    if (j < 2)
        charger_x2(x2s, x_de(c, i), c.x_bf16, C);
    else
        charger_x2(x2s, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const float4* x2s4 = reinterpret_cast<const float4*>(x2s);
    auto x2f4 = [x2s4](uint32_t t) { return x2s4[x2_indice(t)]; };
    const uint32_t K = a.plan.K[j];
    float* parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * K;
    for (uint32_t r = blockIdx.x * MOE_WARPS + (threadIdx.x >> 5); r < R; r += gridDim.x * MOE_WARPS)
        ligne_segments(fc.p, fe.p, x2f4, r, B, voie, parts + uint64_t(r) * K);
}

// The raw layer's GEMV in row groups (gemv_groupes.cuh): launched when every matrix's shape
// allows it, one block of 8 warps per SM sharing the activation's staged 2x, the same partials
// as k_moe_brut's row walk, bit for bit.
__global__ void __launch_bounds__(128, 3) k_moe_brut_groupes(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, warp = threadIdx.x >> 5;
    if (!tenu(c, i)) return;
    uint32_t* controle = c.controle + 4u * i;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fe, fc;
    const bool bon = B > 0 && partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_ECHELLES_BRUTES, j, fe) &&
                     trouver_flux_warp(partie, taille, SORTE_CODES_BRUTS, j, fc) && fe.produits == nblocs &&
                     fe.longueur >= nblocs && fc.produits == 16u * nblocs && fc.longueur >= 16u * nblocs &&
                     (reinterpret_cast<uintptr_t>(fc.p) & 15u) == 0;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    float4* x2g = reinterpret_cast<float4*>(dyn);
    if (j < 2)
        charger_x2_groupes(x2g, x_de(c, i), c.x_bf16, C);
    else
        charger_x2_groupes(x2g, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const uint32_t W = blockDim.x >> 5;
    const uint32_t K = a.plan.K[j];
    float* parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * K;
    gemv_groupes<true>(fc.p, fe.p, nullptr, x2g, R, B, parts, K, blockIdx.x * W + warp, gridDim.x * W);
}

// ------------------------------------------------------------------ 4'. down, from decoded words

// The down projection's GEMV once h exists, on the words k_moe_codes_dense decoded alongside
// gate/up (workspace, stream order): one warp per segment (32 macro-steps), the product and the
// row / segment closing of the fused kernels (GemvTuile; segments are where tiles close rows
// too), so the partials are those of the fused down launch, bit for bit. Scales from the
// medians and the delta bytes of k_moe_delta.
constexpr uint32_t BAS_WARPS = 8;
constexpr uint32_t BAS_LOT = 16;  // macro-steps loaded before any is used

__host__ __device__ __forceinline__ uint32_t bas_octets(const Couche& c) {
    return medianes_octets(c) + 1024u + x2_octets(c.colonnes[2]);
}

__global__ void __launch_bounds__(BAS_WARPS * 32) k_moe_bas(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const Couche& c = a.c;
    const uint32_t i = blockIdx.z, voie = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    if (!tenu(c, i)) return;
    const uint32_t R = c.lignes[2], C = c.colonnes[2], B = C / 32u, nblocs = R * B;
    const uint32_t nmacro = (nblocs + 7u) / 8u;
    const uint32_t seg0 = blockIdx.x * BAS_WARPS;
    if (seg0 * SEGMENT_MACRO >= nmacro) return;
    const uint8_t* partie;
    uint64_t taille;
    Flux fm;
    const bool bon = partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_MEDIANES, 2, fm) &&
                     fm.produits == R && fm.longueur >= R;
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&c.controle[4u * i + CTL_FORMAT], 1u);
        return;
    }
    uint8_t* med = dyn;
    float* puiss = reinterpret_cast<float*>(dyn + medianes_octets(c));
    float* x2s = reinterpret_cast<float*>(dyn + medianes_octets(c) + 1024u);
    charger_puissances(puiss);
    if (fm.p + ((R + 15u) & ~15u) <= partie + taille)
        copier16(reinterpret_cast<uint4*>(med), reinterpret_cast<const uint4*>(fm.p), (R + 15u) / 16u);
    else
        for (uint32_t t = threadIdx.x; t < R; t += blockDim.x) med[t] = fm.p[t];
    attendre_amont();
    liberer_aval();
    charger_x2(x2s, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const uint32_t seg = seg0 + warp;
    if (seg * SEGMENT_MACRO >= nmacro) return;
    const uint32_t m0 = seg * SEGMENT_MACRO, m1 = min(m0 + SEGMENT_MACRO, nmacro);
    const uint32_t* __restrict__ cd = reinterpret_cast<const uint32_t*>(a.espace + a.plan.cd) + uint64_t(i) * 4u * nblocs;
    const uint8_t* __restrict__ ek = deltas_de(a, i, 2, nblocs);
    const float4* x2s4 = reinterpret_cast<const float4*>(x2s);
    const uint32_t q = voie & 3u, g = voie >> 2;
    GemvTuile gv;
    gv.R = R;
    gv.B = B;
    gv.K = a.plan.K[2];
    gv.voie = voie;
    gv.parts = reinterpret_cast<float*>(a.espace + a.plan.parts[2]) + uint64_t(i) * R * gv.K;
    gv.med = med;
    gv.puiss = puiss;
    gv.debut(m0, m1);
    uint32_t bloc = 8u * m0 + g, b = bloc % B;
    for (uint32_t mb = m0; mb < m1; mb += BAS_LOT) {
        uint32_t mots[BAS_LOT], es[BAS_LOT];
#pragma unroll
        for (uint32_t u = 0; u < BAS_LOT; ++u) {
            const uint32_t bu = bloc + 8u * u;
            const bool v = mb + u < m1 && bu < nblocs;
            mots[u] = v ? __ldg(cd + (mb + u) * 32u + voie) : 0u;
            es[u] = v ? uint32_t(__ldg(ek + bu)) : 0u;
        }
#pragma unroll
        for (uint32_t u = 0; u < BAS_LOT; ++u) {
            const uint32_t m = mb + u;
            if (m >= m1) break;
            const float sq = somme_quad(produit_quad(mots[u], x2s4[X2_PAS * b + q], x2s4[X2_PAS * b + 4u + q]));
            gv.accumuler(sq, bloc, es[u], bloc < nblocs);
            gv.fermer(m, m1);
            bloc += 8u;
            b += 8u;
            b -= b >= B ? B : 0u;
        }
    }
}

// The same down GEMV in row groups (gemv_groupes.cuh), where the shape allows: the words
// k_moe_codes_dense stored are the down matrix's codes in their raw layout (word 32 m + lane =
// bytes 4 (32 m + lane) .. + 3, 16 bytes per block, blocks row-major), so the raw path's GEMV
// reads them as it reads CODES_BRUTS, with each block's scale rebuilt from its row median and
// its delta byte. The partials are k_moe_bas's (and the raw layer's), bit for bit.
// Matrix j = j0 + blockIdx.y: down on h, or (all three decoded first) gate and up on x.
__global__ void __launch_bounds__(128, 3) k_moe_bas_groupes(ArgsMoe a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    const Couche& c = a.c;
    const uint32_t j = a.j0 + blockIdx.y, i = blockIdx.z, warp = threadIdx.x >> 5;
    if (!tenu(c, i)) return;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u, nblocs = R * B;
    const uint8_t* partie;
    uint64_t taille;
    Flux fm;
    // The part and x are layer inputs: the medians are found and x staged before the wait (h and
    // the words come from the previous kernels).
    const bool bon = partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_MEDIANES, j, fm) &&
                     fm.produits == R && fm.longueur >= R;
    float4* x2g = reinterpret_cast<float4*>(dyn);
    if (j < 2) charger_x2_groupes(x2g, x_de(c, i), c.x_bf16, C);
    attendre_amont();
    liberer_aval();
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&c.controle[4u * i + CTL_FORMAT], 1u);
        return;
    }
    if (j == 2) charger_x2_groupes(x2g, reinterpret_cast<const float*>(a.espace + a.plan.h) + uint64_t(i) * C, 0u, C);
    __syncthreads();
    const uint32_t W = blockDim.x >> 5;
    const uint32_t K = a.plan.K[j];
    const uint8_t* cd = a.espace + (j == 2 ? a.plan.cd : a.plan.cdh[j]) + uint64_t(i) * 16u * nblocs;
    float* parts = reinterpret_cast<float*>(a.espace + a.plan.parts[j]) + uint64_t(i) * R * K;
    gemv_groupes<true, true>(cd, deltas_de(a, i, j, nblocs), nullptr, x2g, R, B, parts, K, blockIdx.x * W + warp,
                             gridDim.x * W, fm.p);
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
    const uint32_t i = blockIdx.y, warp = threadIdx.x >> 5;
    // The routed experts were written several kernels back, and the parts are layer inputs:
    // warp j finds BIAIS_j before the wait (the partials come from the previous kernel).
    if (!tenu(c, i)) return;
    if (warp < 2) {
        const uint8_t* partie;
        uint64_t taille;
        Flux fb;
        const bool ok = partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_BIAIS, warp, fb) &&
                        fb.longueur >= 4u * c.lignes[warp];
        if ((threadIdx.x & 31u) == 0) biais[warp] = ok ? reinterpret_cast<const float*>(fb.p) : nullptr;
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

__device__ void echanger(const Couche& c, uint32_t b, uint32_t r, uint32_t R, float s, float* res);

// Token b = blockIdx.y: s = ((w0 s0 + w1 s1) + w2 s2) + ... over its activations held here, in
// slot order, products and sums rounded separately (passe.cuh:611-622); residu[b] += s, or, when
// the call is partial (its experts are one share of an expert-parallel layer), residu[b] = s
// (0 when no activation of the token is held here) for the cross-GPU sum; or, with an exchange,
// the shares of every GPU summed here over peer memory (echanger).
__global__ void __launch_bounds__(256) k_moe_combiner(ArgsMoe a) {
    __shared__ const float* biais[8];
    __shared__ uint32_t tenus;
    const Couche& c = a.c;
    const uint32_t b = blockIdx.y, i0 = b * c.k, warp = threadIdx.x >> 5;
    // Warp u finds slot u's BIAIS_2 before the wait (the routed experts were written several
    // kernels back; the down partials come from the previous kernel).
    if (threadIdx.x == 0) tenus = 0;
    __syncthreads();
    if (warp < c.k) {
        const uint8_t* partie;
        uint64_t taille;
        Flux fb;
        const uint32_t i = i0 + warp;
        const bool t = tenu(c, i);
        const bool ok = t && partie_de(c, i, partie, taille) && trouver_flux_warp(partie, taille, SORTE_BIAIS, 2, fb) &&
                        fb.longueur >= 4u * c.lignes[2];
        if ((threadIdx.x & 31u) == 0) {
            biais[warp] = ok ? reinterpret_cast<const float*>(fb.p) : nullptr;
            if (t) atomicOr(&tenus, 1u << warp);
        }
    }
    __syncthreads();
    attendre_amont();
    liberer_aval();
    const uint32_t R = c.lignes[2], r = blockIdx.x * 256u + threadIdx.x;
    const uint32_t B = c.colonnes[2] / 32u, K = a.plan.K[2];
    const float* parts = reinterpret_cast<const float*>(a.espace + a.plan.parts[2]);
    float s = 0.0f;
    if (r < R) {
        bool premier = true;
        for (uint32_t u = 0; u < c.k; ++u) {
            if (!((tenus >> u) & 1u)) continue;
            const uint32_t i = i0 + u;
            const float bi = biais[u] != nullptr ? biais[u][r] : 0.0f;
            const float si = finir_ligne(parts + (uint64_t(i) * R + r) * K, r, B) + bi;
            const float p = __fmul_rn(c.poids[i], si);
            s = premier ? p : __fadd_rn(s, p);
            premier = false;
        }
    }
    float* res = c.residu + uint64_t(b) * R;
    if (c.ech.monde < 2) {
        if (r < R) res[r] = c.partiel ? s : __fadd_rn(res[r], s);
        return;
    }
    echanger(c, b, r, R, s, res);
}

// ------------------------------------------------------------------ the combine's sum across GPUs

__device__ __forceinline__ void st_release_sys(uint32_t* a, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* a) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// This rank's share s of token b, row r, into its slot on every rank; flags; a bounded wait for
// every rank's flag on this rank's buffer; then the shares summed in rank order (the same bits
// on every rank) and added to the residual. Every thread of the block calls it (barriers).
constexpr uint32_t ECHANGE_ATTENTES_MAX = 1u << 24;  // about 1.5 s with the 100 ns pauses

__device__ void echanger(const Couche& c, uint32_t b, uint32_t r, uint32_t R, float s, float* res) {
    __shared__ uint32_t bon;
    const Echange& e = c.ech;
    const DispositionEchange d = disposition_echange(R, c.jetons, e.monde);
    const uint32_t blk = b * gridDim.x + blockIdx.x;
    if (r < R)
        for (uint32_t q = 0; q < e.monde; ++q)
            reinterpret_cast<float*>(e.tampons[q] + d.slots)[(uint64_t(e.rang) * c.jetons + b) * R + r] = s;
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        uint32_t* attendu = reinterpret_cast<uint32_t*>(e.tampons[e.rang] + d.attendus) + blk;
        const uint32_t seq = *attendu + 1u;
        for (uint32_t q = 0; q < e.monde; ++q)
            st_release_sys(reinterpret_cast<uint32_t*>(e.tampons[q] + d.flags) + uint64_t(e.rang) * d.blocs + blk, seq);
        const uint32_t* mes = reinterpret_cast<const uint32_t*>(e.tampons[e.rang] + d.flags);
        uint32_t ok = 1;
        for (uint32_t q = 0; q < e.monde && ok; ++q) {
            uint32_t n = 0;
            while (ld_acquire_sys(mes + uint64_t(q) * d.blocs + blk) != seq) {
                if (++n >= ECHANGE_ATTENTES_MAX) {
                    ok = 0;
                    break;
                }
                __nanosleep(100);
            }
        }
        if (ok) *attendu = seq;
        bon = ok;
    }
    __syncthreads();
    if (!bon) {
        if (threadIdx.x == 0) atomicAdd(&c.controle[CTL_ATTENTE], 1u);
        return;
    }
    __threadfence();
    if (r < R) {
        const float* sl = reinterpret_cast<const float*>(e.tampons[e.rang] + d.slots);
        float t = sl[uint64_t(b) * R + r];
        for (uint32_t q = 1; q < e.monde; ++q) t = __fadd_rn(t, sl[(uint64_t(q) * c.jetons + b) * R + r]);
        res[r] = __fadd_rn(res[r], t);
    }
}

// ------------------------------------------------------------------ launcher

// One wave of k_moe_brut blocks over `plans` (matrices x activations) grid planes, each warp
// looping over its rows; no more blocks per plane than its rows need.
static uint32_t grille_brut(uint32_t R, uint32_t plans) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t vague = (uint32_t(sms) * BRUT_BLOCS_SM + plans - 1) / plans;
    return std::max(1u, std::min((R + MOE_WARPS - 1) / MOE_WARPS, vague));
}

cudaError_t lancer_moe(const Couche& c, void* espace, uint64_t espace_octets, cudaStream_t flux, cudaEvent_t const* ev) {
    auto marque = [&](int i) {
        if (ev != nullptr && ev[i] != nullptr) cudaEventRecord(ev[i], flux);
    };
    const uint32_t na = activations(c);
    ArgsMoe a{c, static_cast<uint8_t*>(espace), plan_espace(c.lignes, c.colonnes, na), 0, 0, 0, {0, 0, 0}};
    if (c.deltas != nullptr) {
        const Espace pe = plan_espace(c.lignes, c.colonnes, c.experts);
        for (int j = 0; j < 3; ++j) a.pre_ek[j] = pe.ek[j];
    }
    // The down projection's decode overlaps gate/up when the workspace holds its codes; with room
    // for all three matrices' codes (and row-group shapes), every tile decodes only and the three
    // GEMVs follow on the decoded words.
    a.seuls = (!c.brut && na <= RECOUVRE_MAX && espace_octets >= a.plan.total_recouvrant) ? 1u : 0u;
    if (a.seuls && espace_octets >= a.plan.total_tout && groupes_possibles(c.lignes[0], c.colonnes[0] / 32u) &&
        groupes_possibles(c.lignes[2], c.colonnes[2] / 32u))
        a.seuls = 2u;
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
        // DELTA of the routed experts, unless the layer's deltas were decoded ahead.
        int dev = 0, sms = 148;
        if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (c.deltas == nullptr) {
            const dim3 g((td + DELTA_WARPS - 1) / DELTA_WARPS, 3, na);
            e = uint64_t(g.x) * g.y * g.z <= 4ull * uint32_t(sms)
                    ? lancer_pdl(k_moe_delta<true>, g, dim3(DELTA_WARPS * 32), 0, flux, a)
                    : lancer_pdl(k_moe_delta<false>, g, dim3(DELTA_WARPS * 32), 0, flux, a);
            if (e != cudaSuccess) return e;
        }
        // Producer / consumer pairs while the launch's tiles fit them at once (lowest latency per
        // tile); past that, one warp per tile with three times as many tiles in flight.
        const uint64_t places = uint64_t(sms) * 2u * MOE_PAIRES;
        auto codes = [&](uint32_t matrices) -> cudaError_t {
            if (uint64_t(na) * matrices * tc <= places) {
                const size_t smem = disposition_codes(c).total;
                cudaError_t e2 = assurer_smem(reinterpret_cast<const void*>(k_moe_codes), int(smem));
                if (e2 != cudaSuccess) return e2;
                return lancer_pdl(k_moe_codes, dim3((tc + MOE_PAIRES - 1) / MOE_PAIRES, matrices, na),
                                  dim3(MOE_PAIRES * 64), smem, flux, a);
            }
            const size_t smem = disposition_dense(c).total;
            cudaError_t e2 = assurer_smem(reinterpret_cast<const void*>(k_moe_codes_dense), int(smem));
            if (e2 != cudaSuccess) return e2;
            return lancer_pdl(k_moe_codes_dense, dim3((tc + DENSE_WARPS - 1) / DENSE_WARPS, matrices, na),
                              dim3(DENSE_WARPS * 32), smem, flux, a);
        };
        marque(1);
        if (a.seuls == 2u) {
            // every tile decodes only (the three matrices in one launch, the tiles spread evenly
            // over the SMs), then the GEMVs in row groups on the decoded words: gate/up, SwiGLU,
            // down
            const size_t smem = plat_octets();
            if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_codes_plat), int(smem))) != cudaSuccess) return e;
            if ((e = lancer_pdl(k_moe_codes_plat, dim3(std::max(1, sms / 3), 3, 1), dim3(PLAT_WARPS * 32), smem, flux,
                                a)) != cudaSuccess)
                return e;
            marque(2);  // phases: the decode launch alone, then the gate/up GEMV with SwiGLU
            const uint32_t smem_g = x2g_octets(cmax);
            if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_bas_groupes), int(smem_g))) != cudaSuccess) return e;
            auto gx = [&](uint32_t R) { return std::max(1u, ((R + GRP_LIGNES - 1) / GRP_LIGNES + 3u) / 4u); };
            if ((e = lancer_pdl(k_moe_bas_groupes, dim3(gx(c.lignes[0]), 2, na), dim3(128), smem_g, flux, a)) != cudaSuccess)
                return e;
            if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, na, 1), dim3(256), 0, flux, a)) != cudaSuccess)
                return e;
            marque(3);
            a.j0 = 2;
            if ((e = lancer_pdl(k_moe_bas_groupes, dim3(gx(c.lignes[2]), 1, na), dim3(128), smem_g, flux, a)) != cudaSuccess)
                return e;
            marque(4);
        } else if (a.seuls) {
            // gate/up fused with the GEMV, down decoded alone, in one launch; the down GEMV from
            // the decoded words once h exists (k_moe_bas: the same partials).
            const size_t smem = disposition_dense(c).total;
            if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_codes_dense), int(smem))) != cudaSuccess) return e;
            if ((e = lancer_pdl(k_moe_codes_dense, dim3((tc + DENSE_WARPS - 1) / DENSE_WARPS, 3, na),
                                dim3(DENSE_WARPS * 32), smem, flux, a)) != cudaSuccess)
                return e;
            marque(2);
            if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, na, 1), dim3(256), 0, flux, a)) != cudaSuccess)
                return e;
            marque(3);
            if (groupes_possibles(c.lignes[2], c.colonnes[2] / 32u)) {
                const uint32_t smem_b = x2g_octets(c.colonnes[2]);
                if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_bas_groupes), int(smem_b))) != cudaSuccess) return e;
                const uint32_t gx = std::max(1u, ((c.lignes[2] + GRP_LIGNES - 1) / GRP_LIGNES + 3u) / 4u);
                if ((e = lancer_pdl(k_moe_bas_groupes, dim3(gx, 1, na), dim3(128), smem_b, flux, a)) != cudaSuccess) return e;
            } else {
                const size_t smem_b = bas_octets(c);
                if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_bas), int(smem_b))) != cudaSuccess) return e;
                const uint64_t nseg =
                    (uint64_t(c.lignes[2]) * (c.colonnes[2] / 32u) + 8u * SEGMENT_MACRO - 1u) / (8u * SEGMENT_MACRO);
                if ((e = lancer_pdl(k_moe_bas, dim3(uint32_t((nseg + BAS_WARPS - 1) / BAS_WARPS), 1, na),
                                    dim3(BAS_WARPS * 32), smem_b, flux, a)) != cudaSuccess)
                    return e;
            }
            marque(4);
        } else {
            if ((e = codes(2)) != cudaSuccess) return e;
            marque(2);
            if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, na, 1), dim3(256), 0, flux, a)) != cudaSuccess)
                return e;
            marque(3);
            a.j0 = 2;
            if ((e = codes(1)) != cudaSuccess) return e;
            marque(4);
        }
    } else if (groupes_possibles(c.lignes[0], c.colonnes[0] / 32u) && groupes_possibles(c.lignes[2], c.colonnes[2] / 32u)) {
        // Row groups: blocks of 4 warps, one row group per warp, the 2x staged per block.
        const uint32_t smem = x2g_octets(cmax);
        if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_brut_groupes), int(smem))) != cudaSuccess) return e;
        auto gx = [&](uint32_t R) { return std::max(1u, ((R + GRP_LIGNES - 1) / GRP_LIGNES + 3u) / 4u); };
        marque(1);
        if ((e = lancer_pdl(k_moe_brut_groupes, dim3(gx(c.lignes[0]), 2, na), dim3(128), smem, flux, a)) != cudaSuccess)
            return e;
        marque(2);
        if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, na, 1), dim3(256), 0, flux, a)) != cudaSuccess)
            return e;
        marque(3);
        a.j0 = 2;
        if ((e = lancer_pdl(k_moe_brut_groupes, dim3(gx(c.lignes[2]), 1, na), dim3(128), smem, flux, a)) != cudaSuccess)
            return e;
        marque(4);
    } else {
        const size_t smem = x2_octets(cmax);
        if ((e = assurer_smem(reinterpret_cast<const void*>(k_moe_brut), int(smem))) != cudaSuccess) return e;
        const uint32_t rmax = std::max(c.lignes[0], c.lignes[2]);
        const uint32_t gx = grille_brut(rmax, 2u * na);
        marque(1);
        if ((e = lancer_pdl(k_moe_brut, dim3(gx, 2, na), dim3(MOE_WARPS * 32), smem, flux, a)) != cudaSuccess) return e;
        marque(2);
        if ((e = lancer_pdl(k_moe_swiglu, dim3((c.lignes[0] + 255) / 256, na, 1), dim3(256), 0, flux, a)) != cudaSuccess)
            return e;
        marque(3);
        a.j0 = 2;
        if ((e = lancer_pdl(k_moe_brut, dim3(grille_brut(c.lignes[2], na), 1, na), dim3(MOE_WARPS * 32), smem, flux, a)) !=
            cudaSuccess)
            return e;
        marque(4);
    }
    if ((e = lancer_pdl(k_moe_combiner, dim3((c.lignes[2] + 255) / 256, c.jetons), dim3(256), 0, flux, a)) != cudaSuccess) return e;
    marque(5);
    return cudaGetLastError();
}

// The delta bytes of every expert of a layer, decoded ahead into `deltas` (the layout of the
// workspace's delta region for `experts` activations: matrix j at plan_espace(...).ek[j],
// [expert][block]); counters per expert in controle[4 e ..].
uint64_t deltas_octets(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t experts) {
    return plan_espace(lignes, colonnes, experts).parts[0];
}

cudaError_t lancer_predecoder_deltas(const Couche& c, uint8_t* deltas, cudaStream_t flux) {
    ArgsMoe a{c, deltas, plan_espace(c.lignes, c.colonnes, c.experts), 0, 0, 1u, {0, 0, 0}};
    a.c.deltas = nullptr;
    const uint32_t nd = c.n_delta ? c.n_delta : 256u;
    uint32_t td = 1;
    for (int j = 0; j < 3; ++j) {
        const uint64_t nb = uint64_t(c.lignes[j]) * (c.colonnes[j] / 32u);
        td = std::max<uint32_t>(td, uint32_t(((nb + 127) / 128 + nd - 1) / nd));
    }
    cudaError_t e = lancer_pdl(k_moe_delta<false>, dim3((td + DELTA_WARPS - 1) / DELTA_WARPS, 3, c.experts),
                               dim3(DELTA_WARPS * 32), 0, flux, a);
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace tb
