/*
 * TEST INFRASTRUCTURE — the MoE layer of the hot path on host cores, built from the oracle's
 * restatements. It is bench.py's CPU baseline (`--impl reference` and `cpu_baseline`): the
 * reference has no runnable CPU engine here (its CPU codec is Rust, absent from this image),
 * so the timed CPU path is this port of it:
 *   router   logits = Wr x + br                       (trc-modele/src/lib.rs:524; passe.cuh:225-233)
 *   top-k    value desc / index asc, f64 softmax       (passe.cuh:455-514)
 *   decode   trc-codec decoder_matrice_v10 per matrix  (trc-codec/src/lib.rs:190-218), parallel
 *            over rANS tiles like the reference verifier parallelises over experts
 *   GEMV     y = W x + b per matrix, f32                (trc-modele/src/lib.rs:533-553)
 *   SwiGLU   clamped, f64                              (passe.cuh:598-605)
 *   combine  residual += sum w_j s_j, no FMA           (passe.cuh:611-622)
 */
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    uint64_t voies_hors_l;
    uint64_t tuiles_mots_faux;
    int64_t premiere_tuile;
} orc_bilan;

int orc_trouver_flux(const uint8_t* partie, size_t n, uint8_t sorte, uint8_t matrice, uint32_t* decalage,
                     uint32_t* longueur, uint32_t* produits);
int orc_flux_valide(const uint8_t* b, size_t n);
int orc_decoder_tuiles(const uint8_t* b, size_t n, const uint8_t* kappa, size_t n_kappa, const uint32_t* luts,
                       uint32_t n_luts, uint32_t t0, uint32_t t1, uint8_t* sortie, orc_bilan* bilan);
void orc_routeur_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices, float* poids);
void orc_swiglu(const float* g, const float* u, float* y, uint32_t n);
void orc_combiner(float* residu, const float* sorties, uint32_t pas, const float* poids, uint32_t n, uint32_t d);

static uint32_t lu32c(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }

typedef struct {
    const uint8_t* partie;
    size_t taille;
    const uint8_t *med, *biais, *fd, *fc;
    uint32_t ld, lc, Td, Tc, Pd, Pc;
    uint8_t *delta, *kappa, *codes, *echelles;
} matrice_cpu;

static float produit_ligne(const uint8_t* codes, const uint8_t* ech, const float* x, uint32_t B) {
    static const float K[16] = {0, 1, 2, 3, 4, 6, 8, 12, -0.0f, -1, -2, -3, -4, -6, -8, -12};
    float s = 0.0f;
    for (uint32_t b = 0; b < B; ++b) {
        const float sc = ldexpf(1.0f, (int)ech[b] - 128);
        float t = 0.0f;
        const uint8_t* q = codes + 16 * (size_t)b;
        const float* xb = x + 32 * (size_t)b;
        for (int i = 0; i < 16; ++i) {
            t += K[q[i] & 15] * xb[i];
            t += K[q[i] >> 4] * xb[16 + i];
        }
        s += sc * t;
    }
    return s;
}

/* One MoE layer for one token. parties[E] / tailles[E]: each expert's level-0 part; luts: the
 * layer's u32[3][4][4096]; lignes/colonnes: the three matrices (gate, up: C0 -> R0; down:
 * R0 -> R2). Returns 0, or a negative value on a format error or a corrupted stream. */
int orc_couche_moe_cpu(const uint8_t* const* parties, const size_t* tailles, uint32_t E, const uint32_t* luts,
                       const uint32_t* lignes, const uint32_t* colonnes, const float* Wr, const float* br,
                       const float* x, uint32_t k, float* residu, uint32_t* idx_out, float* w_out, int n_fils) {
    const uint32_t R = lignes[0], C = colonnes[0], R2 = lignes[2];
    if (k > 8 || lignes[1] != R || colonnes[1] != C || colonnes[2] != R || C % 32 || R % 32) return -1;
    if (n_fils > 0) omp_set_num_threads(n_fils);
    float* logits = (float*)malloc(sizeof(float) * E);
#pragma omp parallel for schedule(static)
    for (uint32_t e = 0; e < E; ++e) {
        float s = 0.0f;
        for (uint32_t c = 0; c < C; ++c) s += Wr[(size_t)e * C + c] * x[c];
        logits[e] = s + br[e];
    }
    uint32_t idx[8];
    float w[8];
    orc_routeur_topk(logits, E, k, idx, w);
    free(logits);
    memcpy(idx_out, idx, 4 * k);
    memcpy(w_out, w, 4 * k);

    matrice_cpu m[24];
    int erreur = 0;
    for (uint32_t i = 0; i < k; ++i) {
        for (uint32_t j = 0; j < 3; ++j) {
            matrice_cpu* a = &m[3 * i + j];
            a->partie = parties[idx[i]];
            a->taille = tailles[idx[i]];
            uint32_t d[4], l[4], p[4];
            for (uint8_t s = 1; s <= 4; ++s)
                if (orc_trouver_flux(a->partie, a->taille, s, (uint8_t)j, &d[s - 1], &l[s - 1], &p[s - 1]) != 0) erreur = -2;
            if (erreur) break;
            a->med = a->partie + d[0];
            a->biais = a->partie + d[1];
            a->fd = a->partie + d[2];
            a->ld = l[2];
            a->fc = a->partie + d[3];
            a->lc = l[3];
            if (orc_flux_valide(a->fd, a->ld) || orc_flux_valide(a->fc, a->lc)) {
                erreur = -3;
                break;
            }
            a->Pd = lu32c(a->fd);
            a->Td = lu32c(a->fd + 8);
            a->Pc = lu32c(a->fc);
            a->Tc = lu32c(a->fc + 8);
            a->delta = (uint8_t*)malloc(a->Pd);
            a->kappa = (uint8_t*)malloc(a->Pd);
            a->codes = (uint8_t*)malloc(a->Pc);
            a->echelles = (uint8_t*)malloc((size_t)lignes[j] * (colonnes[j] / 32));
        }
        if (erreur) break;
    }
    if (erreur) return erreur;
    const uint32_t n_m = 3 * k;
    /* DELTA tiles of every matrix in parallel, then CODES_CTX tiles. */
    uint32_t taches = 0;
    for (uint32_t a = 0; a < n_m; ++a) taches += m[a].Td;
    int faute = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : faute)
    for (uint32_t t = 0; t < taches; ++t) {
        uint32_t a = 0, r = t;
        while (r >= m[a].Td) r -= m[a].Td, ++a;
        orc_bilan bl;
        orc_decoder_tuiles(m[a].fd, m[a].ld, NULL, 0, luts + (size_t)(a % 3) * 4 * 4096, 1, r, r + 1, m[a].delta, &bl);
        faute |= (bl.voies_hors_l || bl.tuiles_mots_faux) ? 1 : 0;
    }
    for (uint32_t a = 0; a < n_m; ++a) {
        const uint32_t Bj = colonnes[a % 3] / 32;
        const size_t nbj = (size_t)lignes[a % 3] * Bj;
        for (size_t i = 0; i < m[a].Pd; ++i) m[a].kappa[i] = m[a].delta[i] < 128 ? 0 : (m[a].delta[i] == 128 ? 1 : 2);
        for (size_t beta = 0; beta < nbj; ++beta) m[a].echelles[beta] = (uint8_t)(m[a].med[beta / Bj] + m[a].delta[beta] - 128);
    }
    taches = 0;
    for (uint32_t a = 0; a < n_m; ++a) taches += m[a].Tc;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : faute)
    for (uint32_t t = 0; t < taches; ++t) {
        uint32_t a = 0, r = t;
        while (r >= m[a].Tc) r -= m[a].Tc, ++a;
        orc_bilan bl;
        orc_decoder_tuiles(m[a].fc, m[a].lc, m[a].kappa, m[a].Pd, luts + (size_t)(a % 3) * 4 * 4096 + 4096, 3, r, r + 1,
                           m[a].codes, &bl);
        faute |= (bl.voies_hors_l || bl.tuiles_mots_faux) ? 1 : 0;
    }
    /* gate, up, SwiGLU, down per expert; rows in parallel. */
    const uint32_t B = C / 32, B2 = R / 32;
    float* g = (float*)malloc(sizeof(float) * R * k);
    float* u = (float*)malloc(sizeof(float) * R * k);
    float* h = (float*)malloc(sizeof(float) * R * k);
    float* s = (float*)malloc(sizeof(float) * R2 * k);
#pragma omp parallel for schedule(static)
    for (uint32_t t = 0; t < 2 * k * R; ++t) {
        const uint32_t i = t / (2 * R), j = (t / R) % 2, r = t % R;
        const matrice_cpu* a = &m[3 * i + j];
        float bias;
        memcpy(&bias, a->biais + 4 * (size_t)r, 4);
        (j == 0 ? g : u)[(size_t)i * R + r] = produit_ligne(a->codes + 16 * (size_t)r * B, a->echelles + (size_t)r * B, x, B) + bias;
    }
    for (uint32_t i = 0; i < k; ++i) orc_swiglu(g + (size_t)i * R, u + (size_t)i * R, h + (size_t)i * R, R);
#pragma omp parallel for schedule(static)
    for (uint32_t t = 0; t < k * R2; ++t) {
        const uint32_t i = t / R2, r = t % R2;
        const matrice_cpu* a = &m[3 * i + 2];
        float bias;
        memcpy(&bias, a->biais + 4 * (size_t)r, 4);
        s[(size_t)i * R2 + r] = produit_ligne(a->codes + 16 * (size_t)r * B2, a->echelles + (size_t)r * B2, h + (size_t)i * R, B2) + bias;
    }
    orc_combiner(residu, s, R2, w, k, R2);
    for (uint32_t a = 0; a < n_m; ++a) {
        free(m[a].delta);
        free(m[a].kappa);
        free(m[a].codes);
        free(m[a].echelles);
    }
    free(g);
    free(u);
    free(h);
    free(s);
    return faute ? -4 : 0;
}

/* Config 0's CPU decode: matrices mats[0 .. n - 1] of one expert's level-0 part decoded into
 * codes[i] (16 R B bytes, canonical when v1.2) and echelles[i] (R B E8M0 bytes), parallel over
 * (matrix, rANS tile) on every host thread: the DELTA tiles of all matrices, then the scales,
 * then the CODES_CTX tiles (trc-codec decoder_matrice_v10, lib.rs:190-218, with rans.rs:388-451
 * per tile). Returns 0, or a negative value on a format error or a corrupted stream. */
int orc_decoder_matrices_cpu(const uint8_t* partie, size_t taille, const uint32_t* luts, const uint32_t* lignes,
                             const uint32_t* colonnes, uint32_t n, const uint32_t* mats, uint8_t* const* codes,
                             uint8_t* const* echelles, int n_fils) {
    if (n == 0 || n > 3) return -1;
    if (n_fils > 0) omp_set_num_threads(n_fils);
    matrice_cpu m[3];
    for (uint32_t a = 0; a < n; ++a) {
        const uint8_t j = (uint8_t)mats[a];
        uint32_t d[4], l[4], p[4];
        for (uint8_t s = 1; s <= 4; ++s)
            if (orc_trouver_flux(partie, taille, s, j, &d[s - 1], &l[s - 1], &p[s - 1]) != 0) return -2;
        m[a].med = partie + d[0];
        m[a].fd = partie + d[2];
        m[a].ld = l[2];
        m[a].fc = partie + d[3];
        m[a].lc = l[3];
        if (orc_flux_valide(m[a].fd, m[a].ld) || orc_flux_valide(m[a].fc, m[a].lc)) return -3;
        m[a].Pd = lu32c(m[a].fd);
        m[a].Td = lu32c(m[a].fd + 8);
        m[a].Pc = lu32c(m[a].fc);
        m[a].Tc = lu32c(m[a].fc + 8);
        if ((size_t)m[a].Pc < 16 * (size_t)lignes[j] * (colonnes[j] / 32)) return -3;
    }
    uint8_t* delta[3];
    uint8_t* kappa[3];
    uint8_t* tampon[3];
    for (uint32_t a = 0; a < n; ++a) {
        delta[a] = (uint8_t*)malloc(m[a].Pd);
        kappa[a] = (uint8_t*)malloc(m[a].Pd);
        tampon[a] = (uint8_t*)malloc(m[a].Pc);
    }
    uint32_t taches = 0;
    for (uint32_t a = 0; a < n; ++a) taches += m[a].Td;
    int faute = 0;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : faute)
    for (uint32_t t = 0; t < taches; ++t) {
        uint32_t a = 0, r = t;
        while (r >= m[a].Td) r -= m[a].Td, ++a;
        orc_bilan bl;
        orc_decoder_tuiles(m[a].fd, m[a].ld, NULL, 0, luts + (size_t)mats[a] * 4 * 4096, 1, r, r + 1, delta[a], &bl);
        faute |= (bl.voies_hors_l || bl.tuiles_mots_faux) ? 1 : 0;
    }
    for (uint32_t a = 0; a < n; ++a) {
        const uint32_t Bj = colonnes[mats[a]] / 32;
        const size_t nbj = (size_t)lignes[mats[a]] * Bj;
        for (size_t i = 0; i < m[a].Pd; ++i) kappa[a][i] = delta[a][i] < 128 ? 0 : (delta[a][i] == 128 ? 1 : 2);
        for (size_t beta = 0; beta < nbj; ++beta) echelles[a][beta] = (uint8_t)(m[a].med[beta / Bj] + delta[a][beta] - 128);
    }
    taches = 0;
    for (uint32_t a = 0; a < n; ++a) taches += m[a].Tc;
#pragma omp parallel for schedule(dynamic, 1) reduction(| : faute)
    for (uint32_t t = 0; t < taches; ++t) {
        uint32_t a = 0, r = t;
        while (r >= m[a].Tc) r -= m[a].Tc, ++a;
        orc_bilan bl;
        orc_decoder_tuiles(m[a].fc, m[a].lc, kappa[a], m[a].Pd, luts + (size_t)mats[a] * 4 * 4096 + 4096, 3, r, r + 1,
                           tampon[a], &bl);
        faute |= (bl.voies_hors_l || bl.tuiles_mots_faux) ? 1 : 0;
    }
    for (uint32_t a = 0; a < n; ++a) {
        memcpy(codes[a], tampon[a], 16 * (size_t)lignes[mats[a]] * (colonnes[mats[a]] / 32));
        free(delta[a]);
        free(kappa[a]);
        free(tampon[a]);
    }
    return faute ? -4 : 0;
}
