/*
 * TEST INFRASTRUCTURE — a seeded synthetic MoE layer built on host cores from the oracle's own
 * encoder, so that the CPU baseline (bench.py `--impl reference`) gets the same layer as the GPU
 * arm without loading the product library.
 *
 *   orc_synth_matrices  the bench workload's weights (gpt-oss-shaped MXFP4 experts): per row
 *                       sigma = 0.02 exp(0.3 n), weights sigma n, per 32-block E8M0 =
 *                       floor(log2 max|w|) - 2, E2M1 nearest with ties to the even code and the
 *                       sign kept, biases 0.01 n rounded to bf16; n from Box-Muller over a
 *                       splitmix64 stream seeded per (seed, matrix, row). It is the workload's
 *                       definition (the same numbers the product's generator draws; a CPU test
 *                       compares the two byte for byte).
 *   orc_comptes_couche  the layer's symbol counts over all its experts: orc_preparer_matrice +
 *                       orc_ajouter_comptes per matrix (trc-codec/src/lib.rs:348-401, as
 *                       bins/trc-codeur/src/coder.rs:207-240 counts a layer).
 *   orc_coder_couche    every expert's level-0 v1.2 part: per matrix MEDIANES, BIAIS, DELTA (one
 *                       table) and CODES_CTX (table chosen by the block's scale class), coded by
 *                       orc_coder_g1 (rans.rs:296-334) and assembled by orc_assembler_partie
 *                       (trc-format/src/lib.rs:882-908); the oracle's encoder is pinned byte for
 *                       byte to the reference bench's encoder.
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

size_t orc_coder_g1(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, size_t n_kappa,
                    const uint16_t* freqs, uint32_t n_tables, uint8_t* out, size_t cap);
size_t orc_assembler_partie(uint16_t couche, uint16_t expert, uint8_t niveau, uint8_t n_matrices, uint32_t n_flux,
                            const uint8_t* descs, const uint32_t* longueurs, const uint32_t* produits,
                            const uint8_t* flux, uint8_t* out, uint32_t* utiles_out);
void orc_preparer_matrice(const uint8_t* blocs, uint32_t R, uint32_t B, int canonique, uint8_t* medianes,
                          uint8_t* delta, uint8_t* qs);
void orc_ajouter_comptes(const uint8_t* delta, size_t pd, const uint8_t* qs, size_t pc, uint64_t* comptes);

/* ------------------------------------------------------------------ the workload's weights */

static uint64_t sm64(uint64_t* s) {
    uint64_t z = (*s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Uniform in (0, 1]: 53 random bits, never 0 (the logarithm below needs it). */
static double uniforme(uint64_t* s) { return (double)((sm64(s) >> 11) + 1) * (1.0 / 9007199254740993.0); }

static double normale(uint64_t* s) {
    const double u = uniforme(s), v = uniforme(s);
    return sqrt(-2.0 * log(u)) * cos(6.283185307179586 * v);
}

/* E2M1 code of v (magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6): nearest, ties to the even code. */
static uint8_t code_e2m1(double v) {
    static const double bornes[7] = {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0};
    const double a = fabs(v);
    uint8_t c = 0;
    while (c < 7 && (a > bornes[c] || (a == bornes[c] && (c & 1)))) ++c;
    return (uint8_t)(c | (signbit(v) ? 8 : 0));
}

static float bf16_pres(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u = (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
    memcpy(&f, &u, 4);
    return f;
}

/* Matrices premier .. premier + n - 1 of `graine`: blocs [n][lignes][colonnes/32][17] (E8M0, then
 * 16 bytes of nibble pairs: low nibble element i, high nibble element i + 16), biais [n][lignes]. */
int orc_synth_matrices(uint64_t graine, uint32_t lignes, uint32_t colonnes, uint32_t premier, uint32_t n,
                       uint8_t* blocs, float* biais, int fils) {
    if (!blocs || !biais || lignes == 0 || colonnes == 0 || colonnes % 32) return -1;
    const uint32_t B = colonnes / 32;
    const int64_t total = (int64_t)n * lignes;
#pragma omp parallel for schedule(static) num_threads(fils > 0 ? fils : omp_get_max_threads())
    for (int64_t t = 0; t < total; ++t) {
        const uint32_t x = (uint32_t)(t / lignes), r = (uint32_t)(t % lignes);
        uint64_t s = graine * 0x9E3779B97F4A7C15ull ^ ((uint64_t)(premier + x) << 32) ^ r;
        sm64(&s);
        const double sigma = 0.02 * exp(0.3 * normale(&s));
        uint8_t* ligne = blocs + ((size_t)x * lignes + r) * B * 17;
        double w[32];
        for (uint32_t b = 0; b < B; ++b) {
            double mx = 0.0;
            for (int i = 0; i < 32; ++i) {
                w[i] = sigma * normale(&s);
                if (fabs(w[i]) > mx) mx = fabs(w[i]);
            }
            int e = mx > 0.0 ? (int)floor(log2(mx)) - 2 : -127;
            if (e < -127) e = -127;
            if (e > 127) e = 127;
            uint8_t* blk = ligne + 17 * b;
            blk[0] = (uint8_t)(e + 127);
            const double inv = ldexp(1.0, -e);
            for (int i = 0; i < 16; ++i)
                blk[1 + i] = (uint8_t)(code_e2m1(w[i] * inv) | (code_e2m1(w[16 + i] * inv) << 4));
        }
        biais[(size_t)x * lignes + r] = bf16_pres((float)(0.01 * normale(&s)));
    }
    return 0;
}

/* ------------------------------------------------------------------ counts and parts */

static size_t al128(size_t x) { return (x + 127) / 128 * 128; }

/* Counts u64[3][4][256] of experts 0 .. n - 1: blocs[j] holds the n experts' matrix j back to
 * back ([n][R_j][B_j][17]). */
void orc_comptes_couche(const uint8_t* const blocs[3], const uint32_t lignes[3], const uint32_t colonnes[3],
                        uint32_t n, int canonique, uint64_t* comptes) {
    memset(comptes, 0, sizeof(uint64_t) * 3 * 4 * 256);
    for (int j = 0; j < 3; ++j) {
        const uint32_t R = lignes[j], B = colonnes[j] / 32;
        const size_t nb = (size_t)R * B, pd = al128(nb), pc = al128(16 * nb);
#pragma omp parallel
        {
            uint64_t local[4 * 256];
            memset(local, 0, sizeof local);
            uint8_t* med = (uint8_t*)malloc(R);
            uint8_t* delta = (uint8_t*)malloc(pd);
            uint8_t* qs = (uint8_t*)malloc(pc);
#pragma omp for schedule(dynamic)
            for (int64_t x = 0; x < (int64_t)n; ++x) {
                orc_preparer_matrice(blocs[j] + (size_t)x * nb * 17, R, B, canonique, med, delta, qs);
                orc_ajouter_comptes(delta, pd, qs, pc, local);
            }
#pragma omp critical
            for (int i = 0; i < 4 * 256; ++i) comptes[(size_t)j * 4 * 256 + i] += local[i];
            free(med);
            free(delta);
            free(qs);
        }
    }
}

/* Level-0 v1.2 parts of experts 0 .. n - 1 (expert numbers premier + x in the headers), each into
 * sorties + x * capacite; octets[x] = the part's length (0: it did not fit or a symbol had no slot
 * in its table). freqs = u16[3][4][256] (DELTA, CODES k = 0, 1, 2 per matrix). */
void orc_coder_couche(const uint8_t* const blocs[3], const float* const biais[3], const uint32_t lignes[3],
                      const uint32_t colonnes[3], uint32_t n, uint32_t premier, const uint16_t* freqs, int canonique,
                      uint32_t n_delta, uint32_t n_codes, uint8_t* sorties, size_t capacite, uint64_t* octets) {
#pragma omp parallel for schedule(dynamic)
    for (int64_t x = 0; x < (int64_t)n; ++x) {
        uint8_t descs[12 * 3];
        uint32_t longueurs[12], produits[12];
        uint8_t* flux[12] = {0};
        int ok = 1;
        for (int j = 0; j < 3 && ok; ++j) {
            const uint32_t R = lignes[j], B = colonnes[j] / 32;
            const size_t nb = (size_t)R * B, pd = al128(nb), pc = al128(16 * nb);
            uint8_t* med = (uint8_t*)malloc(R);
            uint8_t* delta = (uint8_t*)malloc(pd);
            uint8_t* qs = (uint8_t*)malloc(pc);
            uint8_t* kappa = (uint8_t*)malloc(pd);
            orc_preparer_matrice(blocs[j] + (size_t)x * nb * 17, R, B, canonique, med, delta, qs);
            for (size_t i = 0; i < pd; ++i) kappa[i] = delta[i] < 128 ? 0 : (delta[i] == 128 ? 1 : 2);
            const uint16_t* f = freqs + (size_t)j * 4 * 256;
            const size_t cap_d = 2 * pd + 4096 + 132 * (pd / 128 / n_delta + 2);
            const size_t cap_c = 2 * pc + 4096 + 132 * (pc / 128 / n_codes + 2);
            uint8_t* fd = (uint8_t*)malloc(cap_d);
            uint8_t* fc = (uint8_t*)malloc(cap_c);
            const size_t ld = orc_coder_g1(delta, (uint32_t)pd, n_delta, NULL, 0, f, 1, fd, cap_d);
            const size_t lc = orc_coder_g1(qs, (uint32_t)pc, n_codes, kappa, nb, f + 256, 3, fc, cap_c);
            if (ld == 0 || lc == 0 || ld == (size_t)-1 || lc == (size_t)-1) ok = 0;
            const uint8_t sortes[4] = {0x01, 0x02, 0x03, 0x04}, ctx[4] = {0xFF, 0xFF, 0, 0xFF};
            uint8_t* bi = (uint8_t*)malloc(4 * (size_t)R);
            memcpy(bi, biais[j] + (size_t)x * R, 4 * (size_t)R);
            uint8_t* src[4] = {med, bi, fd, fc};
            const uint32_t lg[4] = {R, 4 * R, (uint32_t)ld, (uint32_t)lc};
            const uint32_t pr[4] = {R, 4 * R, (uint32_t)pd, (uint32_t)pc};
            for (int s = 0; s < 4; ++s) {
                const int i = 4 * j + s;
                descs[3 * i] = sortes[s];
                descs[3 * i + 1] = (uint8_t)j;
                descs[3 * i + 2] = ctx[s];
                longueurs[i] = lg[s];
                produits[i] = pr[s];
                flux[i] = src[s];
            }
            free(delta);
            free(qs);
            free(kappa);
        }
        size_t total = 0;
        for (int i = 0; i < 12 && ok; ++i) total += longueurs[i];
        uint8_t* concat = ok ? (uint8_t*)malloc(total ? total : 1) : NULL;
        if (ok) {
            size_t o = 0;
            for (int i = 0; i < 12; ++i) {
                memcpy(concat + o, flux[i], longueurs[i]);
                o += longueurs[i];
            }
            uint32_t utiles = 0;
            const size_t besoin = orc_assembler_partie(0, (uint16_t)(premier + x), 0, 3, 12, descs, longueurs, produits,
                                                       concat, NULL, &utiles);
            if (besoin <= capacite) {
                orc_assembler_partie(0, (uint16_t)(premier + x), 0, 3, 12, descs, longueurs, produits, concat,
                                     sorties + (size_t)x * capacite, &utiles);
                octets[x] = besoin;
            } else {
                octets[x] = 0;
            }
        } else {
            octets[x] = 0;
        }
        free(concat);
        for (int i = 0; i < 12; ++i) free(flux[i]);
    }
}
