/*
 * TEST INFRASTRUCTURE — the CPU oracle of troncons_b200.
 *
 * A plain-C restatement, written from the reference's source text, of the algorithms on the
 * hot path: the `.trc` v1.x part layout, the interleaved 32-lane rANS stream (table
 * normalisation, LUT, coder, normative decoder with its integrity counters), the v1.0/v1.2
 * reconstruction of an MXFP4 expert matrix, empreinte64 (SHA-256, FIPS 180-4), and the
 * single-vector numerics of the MoE layer (router top-k softmax, clamped SwiGLU, combine).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load this library,
 * and only as the checker or as the timed CPU baseline. The product (troncons_b200/) never
 * calls it: its CUDA path fails loudly when its extension is missing.
 *
 * Reference files cited below (paths inside the reference project):
 *   moteur/crates/trc-codec/src/rans.rs      rANS codec
 *   moteur/crates/trc-codec/src/lib.rs       expert reconstruction, v1.2 canonical form
 *   moteur/crates/trc-format/src/lib.rs      part layout, empreinte64, canonical bytes
 *   moteur/crates/trc-noyaux/noyaux/gemv.cuh   device semantics (slot layout, GEMV values)
 *   moteur/crates/trc-reference/src/ops.rs   fp64 router / SwiGLU
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_M 4096u
#define ORC_L 65536u
#define ORC_VOIES 32u
#define ORC_OCTETS_PAR_MACRO 128u

/* ============================================================== SHA-256 (FIPS 180-4) */
/* empreinte64 = first 8 bytes of SHA-256, read little-endian (trc-format/src/lib.rs:111-114). */

typedef struct {
    uint32_t h[8];
    uint64_t n;
    uint8_t bloc[64];
    uint32_t rempli;
} orc_sha256;

static const uint32_t ORC_K256[64] = {
    0x428a2f98, 0x71374491, 0xb5c0fbcf, 0xe9b5dba5, 0x3956c25b, 0x59f111f1, 0x923f82a4, 0xab1c5ed5,
    0xd807aa98, 0x12835b01, 0x243185be, 0x550c7dc3, 0x72be5d74, 0x80deb1fe, 0x9bdc06a7, 0xc19bf174,
    0xe49b69c1, 0xefbe4786, 0x0fc19dc6, 0x240ca1cc, 0x2de92c6f, 0x4a7484aa, 0x5cb0a9dc, 0x76f988da,
    0x983e5152, 0xa831c66d, 0xb00327c8, 0xbf597fc7, 0xc6e00bf3, 0xd5a79147, 0x06ca6351, 0x14292967,
    0x27b70a85, 0x2e1b2138, 0x4d2c6dfc, 0x53380d13, 0x650a7354, 0x766a0abb, 0x81c2c92e, 0x92722c85,
    0xa2bfe8a1, 0xa81a664b, 0xc24b8b70, 0xc76c51a3, 0xd192e819, 0xd6990624, 0xf40e3585, 0x106aa070,
    0x19a4c116, 0x1e376c08, 0x2748774c, 0x34b0bcb5, 0x391c0cb3, 0x4ed8aa4a, 0x5b9cca4f, 0x682e6ff3,
    0x748f82ee, 0x78a5636f, 0x84c87814, 0x8cc70208, 0x90befffa, 0xa4506ceb, 0xbef9a3f7, 0xc67178f2};

static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

static void sha_compresser(orc_sha256* s, const uint8_t* p) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
        w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) | ((uint32_t)p[4 * i + 2] << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
        uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = s->h[0], b = s->h[1], c = s->h[2], d = s->h[3], e = s->h[4], f = s->h[5], g = s->h[6], h = s->h[7];
    for (int i = 0; i < 64; ++i) {
        uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = h + S1 + ch + ORC_K256[i] + w[i];
        uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
        uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + maj;
        h = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    s->h[0] += a; s->h[1] += b; s->h[2] += c; s->h[3] += d;
    s->h[4] += e; s->h[5] += f; s->h[6] += g; s->h[7] += h;
}

static void sha_debut(orc_sha256* s) {
    static const uint32_t h0[8] = {0x6a09e667, 0xbb67ae85, 0x3c6ef372, 0xa54ff53a,
                                   0x510e527f, 0x9b05688c, 0x1f83d9ab, 0x5be0cd19};
    memcpy(s->h, h0, sizeof h0);
    s->n = 0;
    s->rempli = 0;
}

static void sha_ajouter(orc_sha256* s, const uint8_t* p, size_t n) {
    s->n += n;
    while (n > 0) {
        uint32_t k = 64 - s->rempli;
        if (k > n) k = (uint32_t)n;
        memcpy(s->bloc + s->rempli, p, k);
        s->rempli += k;
        p += k;
        n -= k;
        if (s->rempli == 64) {
            sha_compresser(s, s->bloc);
            s->rempli = 0;
        }
    }
}

static void sha_fin(orc_sha256* s, uint8_t out[32]) {
    uint64_t bits = s->n * 8;
    uint8_t un = 0x80, zero = 0;
    sha_ajouter(s, &un, 1);
    while (s->rempli != 56) sha_ajouter(s, &zero, 1);
    uint8_t lg[8];
    for (int i = 0; i < 8; ++i) lg[i] = (uint8_t)(bits >> (56 - 8 * i));
    sha_ajouter(s, lg, 8);
    for (int i = 0; i < 8; ++i) {
        out[4 * i] = (uint8_t)(s->h[i] >> 24);
        out[4 * i + 1] = (uint8_t)(s->h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(s->h[i] >> 8);
        out[4 * i + 3] = (uint8_t)s->h[i];
    }
}

void orc_sha256_octets(const uint8_t* p, size_t n, uint8_t out[32]) {
    orc_sha256 s;
    sha_debut(&s);
    sha_ajouter(&s, p, n);
    sha_fin(&s, out);
}

uint64_t orc_empreinte64(const uint8_t* p, size_t n) {
    uint8_t d[32];
    orc_sha256_octets(p, n, d);
    uint64_t v = 0;
    for (int i = 7; i >= 0; --i) v = (v << 8) | d[i];
    return v;
}

/* ============================================================== rANS table (rans.rs:83-166) */

/* Normalises 256 (geometry 1) or 16 (geometry 2) counts to M = 4096 (rans.rs:83-127):
 * each non-zero count gives max(1, round(c*M/total)); the error is absorbed
 *  - geometry 2: entirely by the largest frequency (last index on ties), if it stays >= 1;
 *  - otherwise one unit at a time over symbols by decreasing frequency (stable order),
 *    never below 1 when removing, only on non-zero symbols when adding.
 * All-zero counts give symbol 0 the whole mass. */
void orc_table_depuis_comptes(const uint64_t* comptes_in, int geometrie, uint16_t* freq_out) {
    const int n = geometrie == 1 ? 256 : 16;
    uint64_t comptes[256];
    uint64_t total = 0;
    for (int i = 0; i < n; ++i) {
        comptes[i] = comptes_in[i];
        total += comptes[i];
    }
    if (total == 0) {
        comptes[0] = 1;
        total = 1;
    }
    int64_t freq[256];
    for (int i = 0; i < n; ++i) {
        freq[i] = 0;
        if (comptes[i] > 0) {
            /* f64 product and division, then round-half-away-from-zero (Rust f64::round). */
            double f = round((double)comptes[i] * 4096.0 / (double)total);
            int64_t fi = (int64_t)f;
            freq[i] = fi < 1 ? 1 : fi;
        }
    }
    int64_t somme = 0;
    for (int i = 0; i < n; ++i) somme += freq[i];
    int fait = 0;
    if (geometrie == 2) {
        /* Iterator::max_by_key returns the LAST maximum. */
        int imax = 0;
        for (int i = 0; i < n; ++i)
            if (freq[i] >= freq[imax]) imax = i;
        int64_t corrige = freq[imax] + (4096 - somme);
        if (corrige >= 1) {
            freq[imax] = corrige;
            fait = 1;
        }
    }
    if (!fait) {
        /* Stable sort of the indices by decreasing frequency. */
        int ordre[256];
        for (int i = 0; i < n; ++i) ordre[i] = i;
        for (int i = 1; i < n; ++i) {
            int v = ordre[i], j = i;
            while (j > 0 && freq[ordre[j - 1]] < freq[v]) {
                ordre[j] = ordre[j - 1];
                --j;
            }
            ordre[j] = v;
        }
        int64_t j = 0;
        while (somme != 4096) {
            int i = ordre[j % n];
            if (somme > 4096 && freq[i] > 1) {
                freq[i] -= 1;
                somme -= 1;
            } else if (somme < 4096 && freq[i] > 0) {
                freq[i] += 1;
                somme += 1;
            }
            ++j;
        }
    }
    for (int i = 0; i < n; ++i) freq_out[i] = (uint16_t)freq[i];
}

/* Decode LUT of a table (rans.rs:146-166; spec ARCHITECTURE.md 4.9.2):
 *   geometry 1: lut[i] = s | (f-1) << 8 | (i - c[s]) << 20
 *   geometry 2: lut[i] = s | f << 4 | (i - c[s]) << 17
 * Returns 0, or -1 when the frequencies do not sum to 4096. */
int orc_lut(const uint16_t* freq, int geometrie, uint32_t* lut) {
    const int n = geometrie == 1 ? 256 : 16;
    uint32_t c = 0;
    for (int s = 0; s < n; ++s) c += freq[s];
    if (c != ORC_M) return -1;
    c = 0;
    for (int s = 0; s < n; ++s) {
        uint32_t f = freq[s];
        for (uint32_t i = c; i < c + f; ++i)
            lut[i] = geometrie == 1 ? ((uint32_t)s | ((f - 1) << 8) | ((i - c) << 20))
                                    : ((uint32_t)s | (f << 4) | ((i - c) << 17));
        c += f;
    }
    return 0;
}

/* ============================================================== rANS coder (rans.rs:296-334) */

static uint32_t lu32(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24); }
static uint32_t lu16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
static void eu32(uint8_t* p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); p[2] = (uint8_t)(v >> 16); p[3] = (uint8_t)(v >> 24); }
static void eu16(uint8_t* p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* Serialized length of a geometry-1 stream (rans.rs:212-214). */
static size_t longueur_flux(uint32_t T, uint32_t W) { return (16 + 4 * (size_t)T + 128 * (size_t)T + 2 * (size_t)W + 15) / 16 * 16; }

/* Encodes `src` (P bytes, P a multiple of 128) with geometry 1 and N macro-steps per tile.
 * Context of byte n: kappa[n/16] when `kappa` is given (per-lane table, CODES_CTX), with 0
 * beyond `n_kappa`; table 0 otherwise (DELTA). `freqs` holds n_tables tables of 256 frequencies.
 * Writes the serialized stream into `out` (capacity `cap`) and returns its length, or 0 when
 * the capacity is too small, or (size_t)-1 when a symbol has frequency 0 in its table.
 * Encoding order: exact reverse of decoding (macro-steps, sub-steps, lanes decreasing), every
 * lane starts at L, the tile's word stack is reversed (rans.rs:296-334). */
size_t orc_coder_g1(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, size_t n_kappa,
                    const uint16_t* freqs, uint32_t n_tables, uint8_t* out, size_t cap) {
    if (P % ORC_OCTETS_PAR_MACRO != 0 || N == 0) return 0;
    const uint32_t n_macro = P / ORC_OCTETS_PAR_MACRO;
    const uint32_t T = (n_macro + N - 1) / N;
    uint32_t* cumul = (uint32_t*)malloc(sizeof(uint32_t) * 256 * n_tables);
    for (uint32_t t = 0; t < n_tables; ++t) {
        uint32_t c = 0;
        for (int s = 0; s < 256; ++s) {
            cumul[256 * t + s] = c;
            c += freqs[256 * t + s];
        }
    }
    uint32_t* debuts = (uint32_t*)malloc(sizeof(uint32_t) * (T ? T : 1));
    uint32_t* etats = (uint32_t*)malloc(sizeof(uint32_t) * 32 * (T ? T : 1));
    size_t cap_mots = (size_t)P + 64, n_mots = 0;
    uint16_t* mots = (uint16_t*)malloc(sizeof(uint16_t) * cap_mots);
    uint16_t* pile = (uint16_t*)malloc(sizeof(uint16_t) * ((size_t)N * 128 + 64));
    size_t res = 0;
    for (uint32_t t = 0; t < T; ++t) {
        const uint32_t m0 = t * N;
        const uint32_t nb = (n_macro - m0) < N ? (n_macro - m0) : N;
        uint64_t x[32];
        for (int l = 0; l < 32; ++l) x[l] = ORC_L;
        size_t np = 0;
        for (int64_t m = (int64_t)nb - 1; m >= 0; --m) {
            for (int k = 3; k >= 0; --k) {
                for (int l = 31; l >= 0; --l) {
                    const size_t n = (((size_t)(m0 + m)) * 32 + (size_t)l) * 4 + (size_t)k;
                    const uint32_t c = kappa ? (n / 16 < n_kappa ? kappa[n / 16] : 0) : 0;
                    const uint32_t s = src[n];
                    const uint64_t f = freqs[256 * c + s];
                    if (f == 0) {
                        res = (size_t)-1;
                        goto fin;
                    }
                    uint64_t xv = x[l];
                    if (xv >= (f << 20)) {
                        pile[np++] = (uint16_t)(xv & 0xFFFF);
                        xv >>= 16;
                    }
                    x[l] = ((xv / f) << 12) + (xv % f) + cumul[256 * c + s];
                }
            }
        }
        debuts[t] = (uint32_t)n_mots;
        for (int l = 0; l < 32; ++l) etats[32 * t + l] = (uint32_t)x[l];
        if (n_mots + np > cap_mots) {
            cap_mots = (n_mots + np) * 2;
            mots = (uint16_t*)realloc(mots, sizeof(uint16_t) * cap_mots);
        }
        for (size_t i = 0; i < np; ++i) mots[n_mots + i] = pile[np - 1 - i];
        n_mots += np;
    }
    {
        const size_t lg = longueur_flux(T, (uint32_t)n_mots);
        if (lg > cap) {
            res = 0;
            goto fin;
        }
        memset(out, 0, lg);
        eu32(out, P);
        eu16(out + 4, N);
        out[6] = 1;
        out[7] = 0;
        eu32(out + 8, T);
        eu32(out + 12, (uint32_t)n_mots);
        size_t p = 16;
        for (uint32_t t = 0; t < T; ++t, p += 4) eu32(out + p, debuts[t]);
        for (uint32_t i = 0; i < 32 * T; ++i, p += 4) eu32(out + p, etats[i]);
        for (size_t i = 0; i < n_mots; ++i, p += 2) eu16(out + p, mots[i]);
        res = lg;
    }
fin:
    free(cumul);
    free(debuts);
    free(etats);
    free(mots);
    free(pile);
    return res;
}

/* ============================================================== rANS decoder (rans.rs:231-451) */

/* Integrity record of a decode (rans.rs:357-382). */
typedef struct {
    uint64_t voies_hors_l;     /* lanes whose final state is not L */
    uint64_t tuiles_mots_faux; /* tiles that did not consume exactly their words */
    int64_t premiere_tuile;    /* first faulty tile, or -1 */
} orc_bilan;

/* Header checks of FluxRans::lire (rans.rs:231-280): returns 0 when the stream is well formed
 * (geometry 1 or 2; P multiple of 128; N > 0; T = ceil((P/128)/N); length covers the payload;
 * zero padding; tile starts non-decreasing, first 0, last <= W; reserved byte zero). */
int orc_flux_valide(const uint8_t* b, size_t n) {
    if (n < 16) return -1;
    const uint32_t P = lu32(b), N = lu16(b + 4), geo = b[6], T = lu32(b + 8), W = lu32(b + 12);
    if (b[7] != 0) return -2;
    if (geo != 1 && geo != 2) return -3;
    if (P % 128 != 0 || N == 0) return -4;
    const uint64_t attendu_t = ((uint64_t)(P / 128) + N - 1) / N;
    if (T != attendu_t) return -5;
    const uint64_t fin = 16 + 4ull * T + 128ull * T + 2ull * W;
    if (fin > n) return -6;
    for (uint64_t i = fin; i < n; ++i)
        if (b[i]) return -7;
    const uint8_t* d = b + 16;
    if (T > 0 && lu32(d) != 0) return -8;
    for (uint32_t t = 1; t < T; ++t)
        if (lu32(d + 4 * (t - 1)) > lu32(d + 4 * t)) return -8;
    if (T > 0 && lu32(d + 4 * (T - 1)) > W) return -8;
    return 0;
}

/* The normative decoder (rans.rs:388-451) on tiles [t0, t1) of a validated stream. `luts`:
 * n_luts LUTs of 4096 entries. Context of symbol n: kappa[n/16] (0 beyond n_kappa) when `kappa`
 * is given, else 0. Writes the tiles' bytes of the P-byte output `sortie` (geometry 1), or ORs
 * their nibbles into it (geometry 2: `sortie` must start zeroed). A missing word reads as 0
 * and is recorded; no stream makes it fail. Tiles are independent, so ranges may run in
 * parallel. */
int orc_decoder_tuiles(const uint8_t* b, size_t n, const uint8_t* kappa, size_t n_kappa, const uint32_t* luts,
                       uint32_t n_luts, uint32_t t0, uint32_t t1, uint8_t* sortie, orc_bilan* bilan) {
    if (orc_flux_valide(b, n) != 0) return -1;
    const uint32_t P = lu32(b), N = lu16(b + 4), g = b[6], T = lu32(b + 8), W = lu32(b + 12);
    const uint32_t spm = g == 1 ? 4 : 8;
    const uint8_t* debuts = b + 16;
    const uint8_t* etats = b + 16 + 4ull * T;
    const uint8_t* mots = b + 16 + 132ull * T;
    const uint32_t n_macro = P / 128;
    if (t1 > T) t1 = T;
    bilan->voies_hors_l = 0;
    bilan->tuiles_mots_faux = 0;
    bilan->premiere_tuile = -1;
    for (uint32_t t = t0; t < t1; ++t) {
        const uint32_t m0 = t * N;
        const uint32_t nb = (n_macro - m0) < N ? (n_macro - m0) : N;
        uint64_t p = lu32(debuts + 4 * t);
        const uint64_t fin = t + 1 < T ? lu32(debuts + 4 * (t + 1)) : W;
        int deborde = 0;
        uint32_t x[32];
        for (int l = 0; l < 32; ++l) x[l] = lu32(etats + 4 * (32 * (size_t)t + l));
        for (uint32_t m = 0; m < nb; ++m) {
            for (uint32_t k = 0; k < spm; ++k) {
                for (uint32_t l = 0; l < 32; ++l) {
                    const size_t w = (size_t)(m0 + m) * 32 + l;
                    const size_t sym = w * spm + k;
                    const uint32_t c = kappa ? (sym / 16 < n_kappa ? kappa[sym / 16] : 0) : 0;
                    if (c >= n_luts) return -2;
                    const uint32_t xv = x[l];
                    const uint32_t e = luts[(size_t)c * ORC_M + (xv & (ORC_M - 1))];
                    uint32_t s, f, bb;
                    if (g == 1) {
                        s = e & 0xFF;
                        f = ((e >> 8) & 0xFFF) + 1;
                        bb = e >> 20;
                    } else {
                        s = e & 0xF;
                        f = (e >> 4) & 0x1FFF;
                        bb = e >> 17;
                    }
                    const uint32_t y = f * (xv >> 12) + bb;
                    if (y < ORC_L) {
                        uint32_t mot = 0;
                        if (p < fin)
                            mot = lu16(mots + 2 * p);
                        else
                            deborde = 1;
                        x[l] = (y << 16) | mot;
                        p += 1;
                    } else {
                        x[l] = y;
                    }
                    if (g == 1)
                        sortie[sym] = (uint8_t)s;
                    else
                        sortie[sym / 2] |= (uint8_t)(s << (4 * (sym % 2)));
                }
            }
        }
        uint64_t hors = 0;
        for (int l = 0; l < 32; ++l) hors += x[l] != ORC_L;
        const int mots_faux = deborde || p != fin;
        if (hors > 0 || mots_faux) {
            bilan->voies_hors_l += hors;
            bilan->tuiles_mots_faux += (uint64_t)mots_faux;
            if (bilan->premiere_tuile < 0) bilan->premiere_tuile = t;
        }
    }
    return 0;
}

/* The whole stream: P bytes into `sortie` (decoder_avec, rans.rs:388-451). */
int orc_decoder(const uint8_t* b, size_t n, const uint8_t* kappa, size_t n_kappa, const uint32_t* luts,
                uint32_t n_luts, uint8_t* sortie, orc_bilan* bilan) {
    if (orc_flux_valide(b, n) != 0) return -1;
    memset(sortie, 0, lu32(b));
    return orc_decoder_tuiles(b, n, kappa, n_kappa, luts, n_luts, 0, lu32(b + 8), sortie, bilan);
}

/* ============================================================== parts (trc-format/src/lib.rs:779-908) */

/* Finds the first stream (sorte, matrice) of a level-0 part after the structural checks of
 * lire_partie (lib.rs:813-866): magic TRC0 / TRC1 by level, reserved bytes zero, stream table
 * inside the useful bytes, stream offsets 16-aligned, non-overlapping and increasing, padding
 * zero. Returns 0 and fills the offset, length and produced bytes, 1 when the stream is absent,
 * a negative value when the part is malformed. */
int orc_trouver_flux(const uint8_t* partie, size_t n, uint8_t sorte, uint8_t matrice, uint32_t* decalage,
                     uint32_t* longueur, uint32_t* produits) {
    if (n < 64) return -1;
    const uint32_t magie = lu32(partie);
    const uint8_t niveau = partie[8];
    if (niveau > 1 || magie != (niveau == 0 ? 0x30435254u : 0x31435254u)) return -2;
    const uint32_t n_matrices = partie[9], n_flux = lu16(partie + 10), utiles = lu32(partie + 12);
    for (int i = 16; i < 64; ++i)
        if (partie[i]) return -3;
    if (utiles > n) return -4;
    const uint64_t fin_table = 64 + 16ull * n_flux;
    if (fin_table > utiles) return -5;
    uint64_t fin_prec = fin_table;
    int trouve = 0;
    for (uint32_t i = 0; i < n_flux; ++i) {
        const uint8_t* e = partie + 64 + 16 * i;
        const uint8_t s = e[0];
        if (!(s == 1 || s == 2 || s == 3 || s == 4 || s == 6 || s == 7 || s == 0x10 || s == 0x11 || s == 0x12)) return -6;
        if (e[3] != 0) return -7;
        if (e[1] >= n_matrices) return -8;
        const uint32_t dec = lu32(e + 4), lon = lu32(e + 8);
        if (dec % 16 != 0 || dec < fin_prec || (uint64_t)dec + lon > utiles) return -9;
        fin_prec = (uint64_t)dec + lon;
        if (!trouve && s == sorte && e[1] == matrice) {
            *decalage = dec;
            *longueur = lon;
            *produits = lu32(e + 12);
            trouve = 1;
        }
    }
    for (size_t i = utiles; i < n; ++i)
        if (partie[i]) return -10;
    return trouve ? 0 : 1;
}

/* Assembles a part (lib.rs:882-908): 64-byte header, stream table, streams aligned to 16,
 * zeros up to a multiple of 4096. `descs` holds per stream {sorte, matrice, contexte}, the
 * stream lengths and produced-bytes fields, and `flux` the stream bytes back to back. Returns
 * the part length (or the needed capacity when `out` is NULL) and sets *utiles. */
size_t orc_assembler_partie(uint16_t couche, uint16_t expert, uint8_t niveau, uint8_t n_matrices, uint32_t n_flux,
                            const uint8_t* descs, const uint32_t* longueurs, const uint32_t* produits,
                            const uint8_t* flux, uint8_t* out, uint32_t* utiles_out) {
    uint64_t p = 64 + 16ull * n_flux;
    for (uint32_t i = 0; i < n_flux; ++i) p = (p + 15) / 16 * 16 + longueurs[i];
    const uint64_t utiles = p;
    const uint64_t total = (utiles + 4095) / 4096 * 4096;
    if (utiles_out) *utiles_out = (uint32_t)utiles;
    if (!out) return (size_t)total;
    memset(out, 0, total);
    eu32(out, niveau == 0 ? 0x30435254u : 0x31435254u);
    eu16(out + 4, couche);
    eu16(out + 6, expert);
    out[8] = niveau;
    out[9] = n_matrices;
    eu16(out + 10, n_flux);
    eu32(out + 12, (uint32_t)utiles);
    p = 64 + 16ull * n_flux;
    const uint8_t* src = flux;
    for (uint32_t i = 0; i < n_flux; ++i) {
        p = (p + 15) / 16 * 16;
        uint8_t* e = out + 64 + 16 * i;
        e[0] = descs[3 * i];
        e[1] = descs[3 * i + 1];
        e[2] = descs[3 * i + 2];
        eu32(e + 4, (uint32_t)p);
        eu32(e + 8, longueurs[i]);
        eu32(e + 12, produits[i]);
        memcpy(out + p, src, longueurs[i]);
        src += longueurs[i];
        p += longueurs[i];
    }
    return (size_t)total;
}

/* ============================================================== expert matrices (trc-codec/src/lib.rs) */

/* Scale class of a delta (lib.rs:48-55). */
static uint8_t classe_echelle(uint8_t d) { return d < 128 ? 0 : (d == 128 ? 1 : 2); }

/* The canonical nibble / byte of v1.2: nibble 8 (-0) becomes 0 (trc-format/src/lib.rs:67-83). */
static uint8_t canoniser_octet(uint8_t o) {
    uint8_t lo = o & 15, hi = o >> 4;
    if (lo == 8) lo = 0;
    if (hi == 8) hi = 0;
    return (uint8_t)(lo | (hi << 4));
}

/* Prepares one matrix for v1.0/v1.2 coding (lib.rs:348-373) from its R*B MXFP4 blocks of 17
 * bytes [e, qs x 16] in beta order: the row medians (tri[B/2] of the row's sorted scales),
 * delta = (e - med + 128) mod 256 padded with zeros to a multiple of 128, and the qs bytes
 * padded to a multiple of 128, canonicalised when `canonique` (v1.2). */
void orc_preparer_matrice(const uint8_t* blocs, uint32_t R, uint32_t B, int canonique, uint8_t* medianes,
                          uint8_t* delta, uint8_t* qs) {
    const size_t nb = (size_t)R * B;
    const size_t pd = (nb + 127) / 128 * 128, pc = (16 * nb + 127) / 128 * 128;
    memset(delta, 0, pd);
    memset(qs, 0, pc);
    uint8_t* tri = (uint8_t*)malloc(B);
    for (uint32_t r = 0; r < R; ++r) {
        const uint8_t* ligne = blocs + (size_t)r * B * 17;
        for (uint32_t b = 0; b < B; ++b) tri[b] = ligne[17 * b];
        /* Insertion sort is enough for a test oracle. */
        for (uint32_t i = 1; i < B; ++i) {
            uint8_t v = tri[i];
            uint32_t j = i;
            while (j > 0 && tri[j - 1] > v) {
                tri[j] = tri[j - 1];
                --j;
            }
            tri[j] = v;
        }
        const uint8_t med = tri[B / 2];
        medianes[r] = med;
        for (uint32_t b = 0; b < B; ++b) {
            const size_t beta = (size_t)r * B + b;
            delta[beta] = (uint8_t)(ligne[17 * b] - med + 128);
            memcpy(qs + 16 * beta, ligne + 17 * b + 1, 16);
        }
    }
    free(tri);
    if (canonique)
        for (size_t i = 0; i < pc; ++i) qs[i] = canoniser_octet(qs[i]);
}

/* Adds a prepared matrix's symbols to a layer's counts (lib.rs:393-401): comptes[0] = delta,
 * comptes[1 + kappa] = code bytes of scale class kappa (padding counted: it is coded). */
void orc_ajouter_comptes(const uint8_t* delta, size_t pd, const uint8_t* qs, size_t pc, uint64_t* comptes /* 4*256 */) {
    for (size_t i = 0; i < pd; ++i) comptes[delta[i]] += 1;
    for (size_t n = 0; n < pc; ++n) {
        const uint8_t k = n / 16 < pd ? classe_echelle(delta[n / 16]) : 0;
        comptes[256 * (1 + k) + qs[n]] += 1;
    }
}

/* Reconstructs matrix j of a level-0 v1.0/v1.2 part (lib.rs:190-218): medians and biases read
 * raw; DELTA decoded with its single table; e[beta] = (med[r] + delta - 128) mod 256; kappa from
 * the decoded delta (padding included); CODES_CTX decoded with the per-lane table kappa(w/4) and
 * truncated to 16*R*B bytes. `luts` = the matrix's 4 LUTs [DELTA, CODES k0, k1, k2]. Returns 0,
 * or a negative value on a format error. The records report lanes off L and bad tiles. */
int orc_decoder_matrice_v10(const uint8_t* partie, size_t n, uint8_t j, uint32_t R, uint32_t B, const uint32_t* luts,
                            uint8_t* codes, uint8_t* echelles, float* biais, orc_bilan* bd, orc_bilan* bc) {
    const size_t nb = (size_t)R * B;
    uint32_t dm, lm, pm, dbi, lbi, pbi, dd, ld, pdd, dc, lc, pcc;
    if (orc_trouver_flux(partie, n, 0x01, j, &dm, &lm, &pm) != 0) return -1;
    if (orc_trouver_flux(partie, n, 0x02, j, &dbi, &lbi, &pbi) != 0) return -1;
    if (orc_trouver_flux(partie, n, 0x03, j, &dd, &ld, &pdd) != 0) return -1;
    if (orc_trouver_flux(partie, n, 0x04, j, &dc, &lc, &pcc) != 0) return -1;
    if (lm != R || pm != R || lbi != 4 * R || pbi != 4 * R) return -2;
    const uint8_t* fd = partie + dd;
    const uint8_t* fc = partie + dc;
    if (orc_flux_valide(fd, ld) != 0 || orc_flux_valide(fc, lc) != 0) return -3;
    const uint32_t Pd = lu32(fd), Pc = lu32(fc);
    if (Pd != pdd || Pc != pcc) return -4;
    if (Pd != (nb + 127) / 128 * 128 || Pc != (16 * nb + 127) / 128 * 128 || fd[6] != 1 || fc[6] != 1) return -5;
    uint8_t* delta = (uint8_t*)malloc(Pd);
    uint8_t* kappa = (uint8_t*)malloc(Pd);
    uint8_t* cod = (uint8_t*)malloc(Pc);
    int r = orc_decoder(fd, ld, NULL, 0, luts, 1, delta, bd);
    if (r == 0) {
        for (size_t i = 0; i < Pd; ++i) kappa[i] = classe_echelle(delta[i]);
        const uint8_t* med = partie + dm;
        for (size_t beta = 0; beta < nb; ++beta) echelles[beta] = (uint8_t)(med[beta / B] + delta[beta] - 128);
        r = orc_decoder(fc, lc, kappa, Pd, luts + ORC_M, 3, cod, bc);
        if (r == 0) memcpy(codes, cod, 16 * nb);
        memcpy(biais, partie + dbi, 4 * (size_t)R);
    }
    free(delta);
    free(kappa);
    free(cod);
    return r == 0 ? 0 : -6;
}

/* SoA slot layout (trc-noyaux/noyaux/commun.cuh:54-92; abi.rs:69-122): codes at 0 (R*B*16),
 * scales at al256(R*B*16), biases at al256(scales + R*B), matrix stride al256(biases + 4R). */
static uint64_t al256(uint64_t x) { return (x + 255) & ~(uint64_t)255; }

void orc_disposition(uint32_t R, uint32_t C, uint64_t* echelles, uint64_t* biais, uint64_t* pas) {
    const uint64_t nb = (uint64_t)R * (C / 32);
    *echelles = al256(nb * 16);
    *biais = al256(*echelles + nb);
    *pas = al256(*biais + 4ull * R);
}

/* Decodes a whole level-0 part (3 matrices) into an SoA slot, the semantics of
 * Noyaux::decoder_expert (noyaux/src/lib.rs:118-136) with the CPU codec: `luts` = the layer's
 * u32[3][4][4096]. controle[0] += lanes off L, controle[2] += tiles with a word-count mismatch,
 * controle[1] = 1 per matrix whose streams are malformed. The slot is left untouched where
 * nothing is decoded. */
int orc_decoder_expert(const uint8_t* partie, size_t n, const uint32_t* luts, const uint32_t* lignes,
                       const uint32_t* colonnes, uint8_t* emplacement, uint32_t controle[4]) {
    uint64_t base = 0;
    for (uint8_t j = 0; j < 3; ++j) {
        const uint32_t R = lignes[j], C = colonnes[j], B = C / 32;
        uint64_t de, db, pas;
        orc_disposition(R, C, &de, &db, &pas);
        orc_bilan bd, bc;
        uint8_t* m = emplacement + base;
        float* bi = (float*)malloc(4 * (size_t)R);
        const int r = orc_decoder_matrice_v10(partie, n, j, R, B, luts + (size_t)j * 4 * ORC_M, m, m + de, bi, &bd, &bc);
        if (r != 0) {
            controle[1] += 1;
        } else {
            memcpy(m + db, bi, 4 * (size_t)R);
            controle[0] += (uint32_t)(bd.voies_hors_l + bc.voies_hors_l);
            controle[2] += (uint32_t)(bd.tuiles_mots_faux + bc.tuiles_mots_faux);
        }
        free(bi);
        base += pas;
    }
    return 0;
}

/* ============================================================== numerics */

/* Exact MXFP4 weight in f64: K[c & 7] * 2^(e - 128), K = {0,1,2,3,4,6,8,12} signed by bit 3
 * (trc-noyaux/noyaux/gemv.cuh:1-12, 25-37; trc-noyaux/tests/carte.rs:379-383). */
static double valeur_mxfp4(uint32_t code, uint32_t e) {
    static const double K[8] = {0, 1, 2, 3, 4, 6, 8, 12};
    const double v = K[code & 7] * ldexp(1.0, (int)e - 128);
    return (code & 8) ? -v : v;
}

/* y = W x + b in f64 from an SoA matrix (codes, scales, f32 biases), x in f64: the host
 * evaluation a kernel is judged against within tolerance. Byte i of a block carries element i
 * (low nibble) and element 16 + i (high nibble) (gemv.cuh:5-7). */
void orc_gemv_f64(const uint8_t* codes, const uint8_t* echelles, const float* biais, const double* x, uint32_t R,
                  uint32_t C, double* y) {
    const uint32_t B = C / 32;
    for (uint32_t r = 0; r < R; ++r) {
        double s = 0.0;
        for (uint32_t b = 0; b < B; ++b) {
            const size_t beta = (size_t)r * B + b;
            const uint32_t e = echelles[beta];
            for (uint32_t t = 0; t < 16; ++t) {
                const uint8_t q = codes[16 * beta + t];
                s += valeur_mxfp4(q & 15, e) * x[32 * b + t];
                s += valeur_mxfp4(q >> 4, e) * x[32 * b + 16 + t];
            }
        }
        y[r] = s + (biais ? (double)biais[r] : 0.0);
    }
}

/* Router top-k (passe.cuh:455-514; ops.rs:123-131): the k largest of E logits, ordered by value
 * decreasing then index increasing (NaN never chosen); weights = softmax of the k chosen in
 * f64 (m = first, exp, sum in order, divide), rounded to f32. */
void orc_routeur_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices, float* poids) {
    uint8_t pris[1024];
    memset(pris, 0, sizeof pris);
    float v[8];
    for (uint32_t r = 0; r < k; ++r) {
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
        for (uint32_t e = 0; e < E; ++e) {
            if (pris[e]) continue;
            const float x = logits[e];
            if (x > bv || (x == bv && e < bi)) {
                bv = x;
                bi = e;
            }
        }
        if (bi != 0xFFFFFFFFu) pris[bi] = 1;
        indices[r] = bi;
        v[r] = bv;
    }
    double ex[8], z = 0.0;
    const double m = v[0];
    for (uint32_t r = 0; r < k; ++r) {
        ex[r] = exp((double)v[r] - m);
        z += ex[r];
    }
    for (uint32_t r = 0; r < k; ++r) poids[r] = (float)(ex[r] / z);
}

/* Clamped SwiGLU of gpt-oss in f64 (passe.cuh:598-605; ops.rs:134-141):
 * g <- min(g, 7); u <- clamp(u, -7, 7); y = g * sigma(1.702 g) * (u + 1), rounded to f32. */
void orc_swiglu(const float* g, const float* u, float* y, uint32_t n) {
    for (uint32_t i = 0; i < n; ++i) {
        const double gv = fmin((double)g[i], 7.0);
        const double uv = fmin(fmax((double)u[i], -7.0), 7.0);
        y[i] = (float)(gv / (1.0 + exp(-1.702 * gv)) * (uv + 1.0));
    }
}

/* residu[i] += ((w0 s0[i] + w1 s1[i]) + w2 s2[i]) + ..., each product and sum rounded to f32
 * separately, no fused multiply-add (passe.cuh:611-622). `poids` NULL means all weights 1. */
void orc_combiner(float* residu, const float* sorties, uint32_t pas, const float* poids, uint32_t n, uint32_t d) {
    for (uint32_t i = 0; i < d; ++i) {
        volatile float s = poids ? poids[0] * sorties[i] : sorties[i];
        for (uint32_t j = 1; j < n; ++j) {
            volatile float p = poids ? poids[j] * sorties[(size_t)j * pas + i] : sorties[(size_t)j * pas + i];
            s = s + p;
        }
        volatile float r = residu[i] + s;
        residu[i] = r;
    }
}
