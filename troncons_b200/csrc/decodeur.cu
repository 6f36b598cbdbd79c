// troncons_b200 — decoding a level-0 part into the SoA slot (the reference's decode-then-
// multiply contract, trc-noyaux/noyaux/decodeur.cuh; the spec ARCHITECTURE.md 4.9 and 4.11).
//
// Two launches on the caller's stream, because CODES_CTX's per-lane table is chosen by the
// scale class that DELTA gives (4.9.3: DELTA is always decoded first):
//   k_echelles  grid (X, 3, n), 4 warps: DELTA_j -> scales e = (med[r] + delta - 128) mod 256,
//               BIAIS_j copied bit for bit;
//   k_codes     grid (X, 3, n), 8 warps: CODES_CTX_j with the lane's table kappa(w/4), from the
//               scale just written and the row's median -> codes.
// One warp per tile, tiles strided over the grid, so every grid gives the same bytes; `n`
// experts of a batch are blockIdx.z (their descriptors carry their own part, slot, LUTs and
// counters). Padding blocks past R*B use class 0 (the coder pads delta with 0).
#include "commun.cuh"
#include "noyaux.h"

namespace tb {

struct ArgsDecodage {
    const DescDecodage* descs;  // batch: descriptors (device); single: null
    const uint8_t* partie;
    uint64_t taille;            // part bytes (UINT64_MAX in a batch: the header's useful bytes rule)
    uint8_t* emplacement;
    const uint32_t* luts;
    uint32_t* controle;
    Dims dims;
};

__device__ __forceinline__ void choisir_expert(const ArgsDecodage& a, const uint8_t*& partie, uint64_t& taille,
                                               uint8_t*& emplacement, const uint32_t*& luts, uint32_t*& controle) {
    if (a.descs) {
        const DescDecodage d = a.descs[blockIdx.z];
        partie = reinterpret_cast<const uint8_t*>(d.partie);
        taille = ~uint64_t(0);
        emplacement = reinterpret_cast<uint8_t*>(d.emplacement);
        luts = reinterpret_cast<const uint32_t*>(d.luts);
        controle = reinterpret_cast<uint32_t*>(d.controle);
    } else {
        partie = a.partie;
        taille = a.taille;
        emplacement = a.emplacement;
        luts = a.luts;
        controle = a.controle;
    }
}

constexpr uint32_t ECH_WARPS = 1;  // one DELTA tile per block: each chain alone on its SM
constexpr uint32_t CODES_WARPS = 8;

// Scales of the 4 blocks of a DELTA word: e = (med[r] + delta - 128) mod 256, to the slot.
__device__ __forceinline__ void ecrire_echelles(uint8_t* ech, const uint8_t* med, uint32_t R, uint32_t nblocs,
                                                uint32_t b0, uint32_t mot, const LignesDelta& lg) {
    uint32_t sortie = 0;
#pragma unroll
    for (uint32_t k = 0; k < 4; ++k) {
        const uint32_t rk = lg.rang(k);
        const uint32_t mk = rk < R ? uint32_t(med[rk]) : 0u;
        sortie |= ((mk + ((mot >> (8u * k)) & 255u) - 128u) & 255u) << (8u * k);
    }
    if (b0 + 3u < nblocs) {
        *reinterpret_cast<uint32_t*>(ech + b0) = sortie;
    } else {
        for (uint32_t k = 0; k < 4; ++k)
            if (b0 + k < nblocs) ech[b0 + k] = uint8_t(sortie >> (8u * k));
    }
}

__global__ void __launch_bounds__(ECH_WARPS * 32) k_echelles(ArgsDecodage a) {
    __shared__ uint32_t lut[M];
    __shared__ uint8_t med_s[8192];
    __shared__ __align__(16) uint16_t anneaux[ECH_WARPS][ANNEAU_ALLOC];
    attendre_amont();  // first kernel of the decode: the part may come from the previous kernel
    liberer_aval();
    const uint8_t* partie;
    uint64_t taille;
    uint8_t* emplacement;
    const uint32_t* luts;
    uint32_t* controle;
    choisir_expert(a, partie, taille, emplacement, luts, controle);
    if (partie == nullptr) return;  // a batch entry with no expert (batches sized for their most)
    const uint32_t j = blockIdx.y, voie = threadIdx.x & 31u;
    const uint32_t R = choisir(a.dims.lignes, j), C = choisir(a.dims.colonnes, j);
    const uint32_t B = C / 32u, nblocs = R * B;
    Flux fd, fm, fb;
    EnteteRans h;
    const bool bon = B > 0 && R > 0 && trouver_flux_warp(partie, taille, SORTE_DELTA, j, fd) &&
                     trouver_flux_warp(partie, taille, SORTE_MEDIANES, j, fm) && trouver_flux_warp(partie, taille, SORTE_BIAIS, j, fb) &&
                     fm.produits == R && fm.longueur >= R && fb.produits == 4u * R && fb.longueur >= 4u * R &&
                     lire_entete(fd, nblocs, h);
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const Disposition disp = disposition(a.dims, j);
    uint8_t* mat = emplacement + disp.base;
    {
        const uint32_t* bs = reinterpret_cast<const uint32_t*>(fb.p);
        uint32_t* bd = reinterpret_cast<uint32_t*>(mat + disp.biais);
        for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < R; i += gridDim.x * blockDim.x) bd[i] = bs[i];
    }
    const uint32_t warp0 = blockIdx.x * ECH_WARPS;
    if (warp0 >= h.T) return;  // block-uniform: no tile for this block
    const uint32_t* src = luts + (uint64_t(j) * 4u) * M;
    for (uint32_t i = threadIdx.x; i < M; i += blockDim.x) lut[i] = src[i];
    const uint8_t* med = fm.p;
    if (R <= 8192u) {
        for (uint32_t i = threadIdx.x; i < R; i += blockDim.x) med_s[i] = fm.p[i];
        med = med_s;
    }
    __syncthreads();
    uint8_t* ech = mat + disp.echelles;
    const uint32_t nmacro = h.P / 128u;
    uint32_t hors_l = 0, pointeur = 0;
    Decodeur d;
    for (uint32_t t = warp0 + (threadIdx.x >> 5); t < h.T; t += gridDim.x * ECH_WARPS) {
        d.debut(h, t, voie, anneaux[threadIdx.x >> 5]);
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        // Word w = 32 m + lane carries delta of blocks 4w .. 4w + 3. The scales of macro-step m - 1
        // are written while macro-step m decodes.
        uint32_t b0 = 4u * (m0 * 32u + voie);
        LignesDelta lg;
        lg.debut(b0, B);
        Decodeur::Avance av;
        d.debut_avance(lut, av);  // one table for every lane: the look-ahead form
        d.avancer();
        uint32_t mot_p = d.macro_avance(lut, av);
        for (uint32_t m = m0 + 1; m < m1; ++m) {
            d.avancer();
            uint32_t sortie = 0;
            const uint32_t mot = d.macro_avance(lut, av, [&](auto k) {
                constexpr int K = decltype(k)::value;  // block 4w + K of the previous word
                const uint32_t rk = lg.rang(K);
                const uint32_t mk = rk < R ? uint32_t(med[rk]) : 0u;
                sortie |= ((mk + ((mot_p >> (8u * K)) & 255u) - 128u) & 255u) << (8u * K);
            });
            if (b0 + 3u < nblocs) {
                *reinterpret_cast<uint32_t*>(ech + b0) = sortie;
            } else {
                for (uint32_t k = 0; k < 4; ++k)
                    if (b0 + k < nblocs) ech[b0 + k] = uint8_t(sortie >> (8u * k));
            }
            mot_p = mot;
            b0 += 128u;
            lg.avancer();
        }
        ecrire_echelles(ech, med, R, nblocs, b0, mot_p, lg);
        d.bilan(hors_l, pointeur);
        d.terminer();
    }
    verser_controle(controle, voie, hors_l, pointeur);
}

__global__ void __launch_bounds__(CODES_WARPS * 32) k_codes(ArgsDecodage a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    uint32_t* lut = reinterpret_cast<uint32_t*>(dyn);                            // [3][M]
    uint16_t* anneaux = reinterpret_cast<uint16_t*>(dyn + 3u * M * 4u);           // [8][ANNEAU_ALLOC]
    const uint8_t* partie;
    uint64_t taille;
    uint8_t* emplacement;
    const uint32_t* luts;
    uint32_t* controle;
    choisir_expert(a, partie, taille, emplacement, luts, controle);
    if (partie == nullptr) return;  // a batch entry with no expert (batches sized for their most)
    const uint32_t j = blockIdx.y, voie = threadIdx.x & 31u;
    const uint32_t R = choisir(a.dims.lignes, j), C = choisir(a.dims.colonnes, j);
    const uint32_t B = C / 32u, nblocs = R * B;
    Flux fc, fm;
    EnteteRans h;
    const bool bon = B > 0 && R > 0 && trouver_flux_warp(partie, taille, SORTE_CODES_CTX, j, fc) &&
                     trouver_flux_warp(partie, taille, SORTE_MEDIANES, j, fm) && fm.produits == R && fm.longueur >= R &&
                     lire_entete(fc, nblocs * 16u, h);
    if (!bon) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicAdd(&controle[CTL_FORMAT], 1u);
        return;
    }
    const uint32_t warp0 = blockIdx.x * CODES_WARPS;
    if (warp0 >= h.T) return;
    {
        const uint4* src = reinterpret_cast<const uint4*>(luts + (uint64_t(j) * 4u + 1u) * M);
        uint4* dst = reinterpret_cast<uint4*>(lut);
        for (uint32_t i = threadIdx.x; i < 3u * M / 4u; i += blockDim.x) dst[i] = src[i];
    }
    attendre_amont();  // the scales come from k_echelles
    liberer_aval();
    __syncthreads();
    const Disposition disp = disposition(a.dims, j);
    uint8_t* mat = emplacement + disp.base;
    uint32_t* codes = reinterpret_cast<uint32_t*>(mat);
    const uint8_t* __restrict__ ech = mat + disp.echelles;  // written by k_echelles
    const uint8_t* __restrict__ med = fm.p;
    const uint32_t nmacro = h.P / 128u;
    const uint32_t mots_utiles = nblocs * 4u;
    uint32_t hors_l = 0, pointeur = 0;
    Decodeur d;
    for (uint32_t t = warp0 + (threadIdx.x >> 5); t < h.T; t += gridDim.x * CODES_WARPS) {
        d.debut(h, t, voie, anneaux + (threadIdx.x >> 5) * ANNEAU_ALLOC);
        const uint32_t m0 = t * h.N, m1 = min(m0 + h.N, nmacro);
        // Word w = 32 m + lane belongs to block w / 4 = 8 m + lane / 4; its class needs the
        // block's scale and its row's median, fetched two macro-steps ahead.
        uint32_t bloc = (m0 * 32u + voie) >> 2;
        const uint32_t q8 = 8u / B, r8 = 8u - q8 * B;  // advance of 8 blocks in rows
        uint32_t ligne = bloc / B, reste = bloc - ligne * B;
        auto avancer_ligne = [&](uint32_t& lg, uint32_t& rs) {
            rs += r8;
            lg += q8;
            const bool c = rs >= B;
            rs -= c ? B : 0u;
            lg += c ? 1u : 0u;
        };
        uint32_t l1 = ligne, r1 = reste;
        avancer_ligne(l1, r1);
        const bool v0 = bloc < nblocs, v1 = m0 + 1 < m1 && bloc + 8u < nblocs;
        uint32_t e0 = v0 ? __ldg(ech + bloc) : 0u, md0 = v0 ? __ldg(med + ligne) : 0u;
        uint32_t e1 = v1 ? __ldg(ech + bloc + 8u) : 0u, md1 = v1 ? __ldg(med + l1) : 0u;
        uint32_t l2 = l1, r2 = r1;
        avancer_ligne(l2, r2);
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t ctx = bloc < nblocs ? classe_echelle(e0, md0) : 0u;
            const bool v2 = m + 2u < m1 && bloc + 16u < nblocs;
            const uint32_t e2 = v2 ? __ldg(ech + bloc + 16u) : 0u, md2 = v2 ? __ldg(med + l2) : 0u;
            d.avancer();
            const uint32_t mot = d.macro(lut + ctx * M);
            const uint32_t w = m * 32u + voie;
            if (w < mots_utiles) codes[w] = mot;
            bloc += 8u;
            e0 = e1;
            md0 = md1;
            e1 = e2;
            md1 = md2;
            avancer_ligne(l2, r2);
        }
        d.bilan(hors_l, pointeur);
        d.terminer();
    }
    verser_controle(controle, voie, hors_l, pointeur);
}

// Raw part (file flag bit 2): ECHELLES_BRUTES_j, CODES_BRUTS_j, BIAIS_j copied into the slot.
__global__ void __launch_bounds__(256) k_copier_brut(const uint8_t* partie, uint64_t taille, uint8_t* emplacement, Dims dims,
                                                      uint32_t* controle) {
    attendre_amont();
    liberer_aval();
    copier_brut_matrice(partie, taille, emplacement, dims, blockIdx.y, controle);
}

// ------------------------------------------------------------------ launchers

static uint32_t tuiles_256(uint64_t octets) { return uint32_t(((octets + 127) / 128 + 255) / 256); }

cudaError_t lancer_decodage(const DescDecodage* descs, uint32_t n, const void* partie, uint64_t taille, void* emplacement,
                            const uint32_t* luts, const Dims& dims, uint32_t* controle, cudaStream_t flux) {
    // Grids sized for the tiles trc-codeur writes (N = 256); any other N decodes too (the warps
    // stride over the tiles), only with a different occupancy.
    uint32_t td = 1, tc = 1;
    for (int j = 0; j < 3; ++j) {
        const uint64_t nb = uint64_t(dims.lignes[j]) * (dims.colonnes[j] / 32u);
        td = std::max(td, tuiles_256(nb));
        tc = std::max(tc, tuiles_256(16 * nb));
    }
    ArgsDecodage a{descs, static_cast<const uint8_t*>(partie), taille, static_cast<uint8_t*>(emplacement), luts, controle, dims};
    const uint32_t z = descs ? n : 1u;
    cudaError_t e = lancer_pdl(k_echelles, dim3((td + ECH_WARPS - 1) / ECH_WARPS, 3, z), dim3(ECH_WARPS * 32), 0, flux, a);
    if (e != cudaSuccess) return e;
    const size_t smem = 3u * M * 4u + CODES_WARPS * ANNEAU_ALLOC * 2u;
    if ((e = assurer_smem(reinterpret_cast<const void*>(k_codes), int(smem))) != cudaSuccess) return e;
    return lancer_pdl(k_codes, dim3((tc + CODES_WARPS - 1) / CODES_WARPS, 3, z), dim3(CODES_WARPS * 32), smem, flux, a);
}

cudaError_t lancer_copier_brut(const void* partie, uint64_t taille, void* emplacement, const Dims& dims, uint32_t* controle,
                               cudaStream_t flux) {
    uint64_t n = 1;
    for (int j = 0; j < 3; ++j) n = std::max<uint64_t>(n, uint64_t(dims.lignes[j]) * (dims.colonnes[j] / 32u));
    const uint32_t g = uint32_t(std::min<uint64_t>(std::max<uint64_t>((n + 255) / 256, 1), 296));
    return lancer_pdl(k_copier_brut, dim3(g, 3, 1), dim3(256), 0, flux, static_cast<const uint8_t*>(partie), taille,
                      static_cast<uint8_t*>(emplacement), dims, controle);
}

}  // namespace tb
