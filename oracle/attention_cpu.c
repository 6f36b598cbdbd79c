/* TEST INFRASTRUCTURE — CPU restatement of the attention side of a gpt-oss layer, as the
 * reference's kernels compute it (trc-noyaux/noyaux/passe.cuh), for checking troncons_b200's
 * kernels: Q8_0 GEMV (passe.cuh:57-97) in its exact order, RMSNorm (passe.cuh:250-272) with its
 * f64 sums and fixed tree, the YaRN rotation (passe.cuh:146-169, 280-301) with the host's libm,
 * the f16 KV-cache write (passe.cuh:305-314) and the attention of one position with sinks
 * (passe.cuh:316-371) with its reductions in the same order. exp / pow / log / sin / cos are the
 * host C library's: results may differ from the device's by an ulp there; everything else is
 * bit for bit. Compiled with -ffp-contract=off. */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* IEEE binary16 -> binary32, exact (subnormals, infinities and NaN included). */
static float f16_vers_f32(uint16_t h) {
    const uint32_t signe = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u, m = h & 0x3FFu, bits;
    if (e == 0) {
        if (m == 0) {
            bits = signe;
        } else { /* subnormal: normalise */
            int k = -1;
            do {
                ++k;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            bits = signe | ((uint32_t)(127 - 15 - k) << 23) | ((m & 0x3FFu) << 13);
        }
    } else if (e == 31) {
        bits = signe | 0x7F800000u | (m << 13);
    } else {
        bits = signe | ((e + 127u - 15u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* IEEE binary32 -> binary16, round to nearest even (overflow to infinity, subnormals, NaN kept
 * quiet). */
static uint16_t f32_vers_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t signe = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t e = (x >> 23) & 0xFFu, m = x & 0x7FFFFFu;
    if (e == 0xFFu) return (uint16_t)(signe | 0x7C00u | (m ? (0x200u | (m >> 13)) : 0u));
    const int E = (int)e - 127 + 15;
    if (E >= 31) return (uint16_t)(signe | 0x7C00u);
    if (E <= 0) { /* subnormal or zero in binary16 */
        if (E < -10) return signe;
        const uint32_t mant = m | 0x800000u;
        const int dec = 14 - E; /* 14..24 */
        uint32_t q = mant >> dec;
        const uint32_t reste = mant & ((1u << dec) - 1u), moitie = 1u << (dec - 1);
        if (reste > moitie || (reste == moitie && (q & 1u))) ++q;
        return (uint16_t)(signe | q);
    }
    uint32_t q = ((uint32_t)E << 10) | (m >> 13);
    const uint32_t reste = m & 0x1FFFu;
    if (reste > 0x1000u || (reste == 0x1000u && (q & 1u))) ++q; /* may carry into the exponent: right */
    return (uint16_t)(signe | q);
}

void orc_f16_depuis_f32(const float* x, uint16_t* y, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) y[i] = f32_vers_f16(x[i]);
}

void orc_f32_depuis_f16(const uint16_t* x, float* y, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) y[i] = f16_vers_f32(x[i]);
}

/* y = W x (+ b), W Q8_0 (rows of C/32 blocks of 34 bytes: f16 d, 32 x i8). Per lane l of 32:
 * blocks l, l + 32, ...: s = fmaf chain over the 32 codes in order, acc = fmaf(d, s, acc); then
 * the xor butterfly 16, 8, 4, 2, 1; + b. */
void orc_gemv_q8_0(const uint8_t* W, const float* x, const float* biais, uint32_t R, uint32_t C, float* y) {
    const uint32_t B = C / 32;
    const uint64_t octets = (uint64_t)B * 34;
    for (uint32_t r = 0; r < R; ++r) {
        float a[32];
        for (uint32_t l = 0; l < 32; ++l) {
            float acc = 0.0f;
            for (uint32_t b = l; b < B; b += 32) {
                const uint8_t* blk = W + r * octets + (uint64_t)b * 34;
                const float d = f16_vers_f32((uint16_t)(blk[0] | (blk[1] << 8)));
                float s = 0.0f;
                for (uint32_t i = 0; i < 32; ++i) s = fmaf((float)(int8_t)blk[2 + i], x[32 * b + i], s);
                acc = fmaf(d, s, acc);
            }
            a[l] = acc;
        }
        for (uint32_t dd = 16; dd > 0; dd >>= 1) {
            float t[32];
            for (uint32_t l = 0; l < 32; ++l) t[l] = a[l] + a[l ^ dd];
            memcpy(a, t, sizeof a);
        }
        y[r] = biais ? a[0] + biais[r] : a[0];
    }
}

/* RMSNorm of `lignes` vectors of n: per thread t of 256 the f64 fma chain of squares over
 * i = t, t + 256, ...; tree k = 128 .. 1; r = 1 / sqrt(sum / n + eps); y = x r w rounded once. */
void orc_rmsnorm(const float* x, const float* w, float* y, uint32_t n, uint32_t lignes, float eps) {
    for (uint32_t l = 0; l < lignes; ++l) {
        const float* xr = x + (uint64_t)l * n;
        float* yr = y + (uint64_t)l * n;
        double part[256];
        for (uint32_t t = 0; t < 256; ++t) {
            double s = 0.0;
            for (uint32_t i = t; i < n; i += 256) {
                const double v = xr[i];
                s = fma(v, v, s);
            }
            part[t] = s;
        }
        for (uint32_t k = 128; k > 0; k >>= 1)
            for (uint32_t t = 0; t < k; ++t) part[t] += part[t + k];
        const double r = 1.0 / sqrt(part[0] / (double)n + (double)eps);
        for (uint32_t i = 0; i < n; ++i) yr[i] = (float)((double)xr[i] * r * (double)w[i]);
    }
}

typedef struct {
    double base, facteur, ctx_origine, beta_rapide, beta_lent;
    uint32_t dim_tete, variante;
} orc_params_rope;

/* YaRN (Peng et al., 2023): inv_freq of pair i and the attention concentration. */
static double yarn_inv_freq(const orc_params_rope* p, uint32_t i, double* concentration) {
    const uint32_t demi = p->dim_tete / 2;
    const double freq = pow(p->base, (double)(2 * i) / (double)p->dim_tete);
    if (p->facteur <= 1.0) {
        *concentration = 1.0;
        return 1.0 / freq;
    }
    *concentration = 0.1 * log(p->facteur) + 1.0;
    const double deux_pi = 6.283185307179586476925286766559;
    double bas = (double)demi * log(p->ctx_origine / (p->beta_rapide * deux_pi)) / log(p->base);
    double haut = (double)demi * log(p->ctx_origine / (p->beta_lent * deux_pi)) / log(p->base);
    if (p->variante == 1) {
        bas = fmax(floor(bas), 0.0);
        haut = fmin(ceil(haut), (double)(p->dim_tete - 1));
    }
    const double interpolation = 1.0 / (p->facteur * freq);
    const double extrapolation = 1.0 / freq;
    const double rampe = fmin(fmax(((double)i - bas) / (haut - bas), 0.0), 1.0);
    const double masque = 1.0 - rampe;
    return interpolation * (1.0 - masque) + extrapolation * masque;
}

/* NEOX rotation of q (tetes_q heads) and k (tetes_k heads) in place at `position`. */
void orc_rope_yarn(float* q, float* k, uint32_t tetes_q, uint32_t tetes_k, uint32_t position, const orc_params_rope* p) {
    const uint32_t d = p->dim_tete, demi = d / 2;
    for (uint32_t h = 0; h < tetes_q + tetes_k; ++h) {
        float* v = h < tetes_q ? q + (uint64_t)h * d : k + (uint64_t)(h - tetes_q) * d;
        for (uint32_t i = 0; i < demi; ++i) {
            double m;
            const double inv = yarn_inv_freq(p, i, &m);
            const double angle = (double)position * inv;
            const double c = cos(angle) * m, s = sin(angle) * m;
            const double a = v[i], b = v[i + demi];
            v[i] = (float)(a * c - b * s);
            v[i + demi] = (float)(b * c + a * s);
        }
    }
}

void orc_ecrire_kv(const float* k, const float* v, uint16_t* cache_k, uint16_t* cache_v, uint32_t dkv, uint32_t case_kv) {
    for (uint32_t i = 0; i < dkv; ++i) {
        cache_k[(uint64_t)case_kv * dkv + i] = f32_vers_f16(k[i]);
        cache_v[(uint64_t)case_kv * dkv + i] = f32_vers_f16(v[i]);
    }
}

typedef struct {
    uint32_t tetes, tetes_kv, dim_tete, debut, fin, anneau;
    float echelle;
    uint32_t reserve;
} orc_params_attention;

/* Attention of one position (dim_tete 64): per query head h (kv head h / (tetes / tetes_kv)),
 * score_j = (fmaf chain over d of q_d k_jd) * echelle, m = max(max_j score_j, sink_h), e_j =
 * expf(score_j - m), z = (per-thread sums over j = t mod 256, in order; tree over 256) +
 * expf(sink_h - m), out_d = (((g0 + g1) + (g2 + g3))) / z with g the fmaf chains over
 * j = g mod 4 in order. `scores`: room for fin - debut floats. */
void orc_attention(const float* q, const uint16_t* cache_k, const uint16_t* cache_v, const float* puits, float* sortie,
                   const orc_params_attention* p, float* scores) {
    const uint32_t n = p->fin - p->debut, dkv = p->tetes_kv * 64;
    for (uint32_t h = 0; h < p->tetes; ++h) {
        const uint32_t hk = h / (p->tetes / p->tetes_kv);
        const float* qh = q + (uint64_t)h * 64;
        float m = -INFINITY;
        for (uint32_t j = 0; j < n; ++j) {
            const uint32_t pos = p->debut + j, c = p->anneau ? pos % p->anneau : pos;
            const uint16_t* kr = cache_k + (uint64_t)c * dkv + (uint64_t)hk * 64;
            float s = 0.0f;
            for (uint32_t d = 0; d < 64; ++d) s = fmaf(qh[d], f16_vers_f32(kr[d]), s);
            scores[j] = s * p->echelle;
            m = fmaxf(m, scores[j]);
        }
        m = fmaxf(m, puits[h]);
        float part[256];
        for (uint32_t t = 0; t < 256; ++t) {
            float z = 0.0f;
            for (uint32_t j = t; j < n; j += 256) {
                const float e = expf(scores[j] - m);
                scores[j] = e;
                z += e;
            }
            part[t] = z;
        }
        for (uint32_t k = 128; k > 0; k >>= 1)
            for (uint32_t t = 0; t < k; ++t) part[t] = part[t] + part[t + k];
        const float z = part[0] + expf(puits[h] - m);
        for (uint32_t dd = 0; dd < 64; ++dd) {
            float g[4];
            for (uint32_t gi = 0; gi < 4; ++gi) {
                float a = 0.0f;
                for (uint32_t j = gi; j < n; j += 4) {
                    const uint32_t pos = p->debut + j, c = p->anneau ? pos % p->anneau : pos;
                    a = fmaf(scores[j], f16_vers_f32(cache_v[(uint64_t)c * dkv + (uint64_t)hk * 64 + dd]), a);
                }
                g[gi] = a;
            }
            sortie[(uint64_t)h * 64 + dd] = ((g[0] + g[1]) + (g[2] + g[3])) / z;
        }
    }
}
