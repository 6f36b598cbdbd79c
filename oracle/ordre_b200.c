/*
 * TEST INFRASTRUCTURE — a CPU replica of troncons_b200's own floating-point reduction order.
 *
 * The reference fixes its GEMV order by its kernel (trc-noyaux/noyaux/gemv.cuh:14-17, 60-126);
 * troncons_b200 fixes a different order, chosen so that the fused rANS-decode GEMV, the GEMV
 * of a decoded slot and the GEMV of a raw (uncompressed) part all give the same bits. The
 * kernels are judged against the reference within tolerance (trc_oracle.c: orc_gemv_f64) and
 * against this replica bit for bit. Nothing here is product code.
 *
 * The order (f32, fmaf = one rounding):
 *   x2[c]      = 2 * x[c]                                  (exact)
 *   v(code)    = the E2M1 value of a nibble, {0,.5,1,1.5,2,3,4,6} signed by bit 3
 *   p[beta][q] = fmaf chain over k = 0..3 of (low nibble of byte 4q+k, x2[32b+4q+k]),
 *                then (high nibble, x2[32b+16+4q+k]), from +0
 *   s[beta]    = (p0 + p1) + (p2 + p3)
 *   segment g  = blocks [256 g, 256 g + 256)  (32 macro-steps of 8 blocks)
 *   acc[r,g,q] = fmaf chain over the blocks beta of row r in segment g with beta % 8 == q,
 *                ascending, of (s[beta], 2^(e[beta] - 128)), from +0
 *   P[r,g]     = ((a0 + a1) + (a2 + a3)) + ((a4 + a5) + (a6 + a7))
 *   y[r]       = ((P[r,g0] + P[r,g0+1]) + ...) + bias[r]
 * Router logits (f32 weights, row-major): lane l of a warp takes float4 chunks l, l+32, ...,
 * an fmaf chain over .x .y .z .w; then an xor butterfly over distances 16, 8, 4, 2, 1; + bias.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static const float ORD_E2M1[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};

static float ord_valeur(uint32_t c) {
    const float v = ORD_E2M1[c & 7];
    return (c & 8) ? -v : v;
}

/* 2^(e - 128) in f32, exact for every e in [0, 255]. */
static float ord_echelle(uint32_t e) { return ldexpf(1.0f, (int)e - 128); }

static float ord_somme_bloc(const uint8_t* q16, const float* x2b) {
    float p[4];
    for (int qq = 0; qq < 4; ++qq) {
        float a = 0.0f;
        for (int k = 0; k < 4; ++k) {
            const uint8_t o = q16[4 * qq + k];
            a = fmaf(ord_valeur(o & 15), x2b[4 * qq + k], a);
            a = fmaf(ord_valeur(o >> 4), x2b[16 + 4 * qq + k], a);
        }
        p[qq] = a;
    }
    return (p[0] + p[1]) + (p[2] + p[3]);
}

/* y = W x + b in troncons_b200's order. codes: R*B*16 bytes, echelles: R*B, x: f32[C]. */
void ord_gemv(const uint8_t* codes, const uint8_t* echelles, const float* biais, const float* x, uint32_t R,
              uint32_t C, float* y) {
    const uint32_t B = C / 32;
    float x2[65536];
    for (uint32_t c = 0; c < C && c < 65536; ++c) x2[c] = 2.0f * x[c];
    for (uint32_t r = 0; r < R; ++r) {
        const uint64_t b0 = (uint64_t)r * B, b1 = b0 + B;
        float y_r = 0.0f;
        int premier = 1;
        for (uint64_t g = b0 / 256; g * 256 < b1; ++g) {
            const uint64_t lo = b0 > g * 256 ? b0 : g * 256;
            const uint64_t hi = b1 < (g + 1) * 256 ? b1 : (g + 1) * 256;
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (uint64_t beta = lo; beta < hi; ++beta) {
                const float s = ord_somme_bloc(codes + 16 * beta, x2 + 32 * (beta - b0));
                acc[beta % 8] = fmaf(s, ord_echelle(echelles[beta]), acc[beta % 8]);
            }
            const float P = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
            if (premier) {
                y_r = P;
                premier = 0;
            } else {
                y_r = y_r + P;
            }
        }
        y[r] = biais ? y_r + biais[r] : y_r;
    }
}

/* Router logits in troncons_b200's order (C a multiple of 4): per row, the float4 chunks split
 * into 4 quarters of ceil(C/16) chunks; per quarter, 32 lanes' fmaf chains over chunks
 * start + lane + 32 i, an xor butterfly; ((q0 + q1) + (q2 + q3)) + bias. */
void ord_gemv_f32(const float* W, const float* x, const float* biais, uint32_t R, uint32_t C, float* y) {
    const uint32_t C4 = C / 4, Q = (C4 + 3) / 4;
    for (uint32_t r = 0; r < R; ++r) {
        float p[4];
        for (uint32_t q = 0; q < 4; ++q) {
            const uint32_t c0 = q * Q, c1 = c0 + Q < C4 ? c0 + Q : C4;
            float a[32];
            for (uint32_t l = 0; l < 32; ++l) {
                float acc = 0.0f;
                for (uint32_t c = c0 + l; c < c1; c += 32) {
                    const float* w = W + (uint64_t)r * C + 4 * c;
                    const float* xx = x + 4 * c;
                    acc = fmaf(w[0], xx[0], acc);
                    acc = fmaf(w[1], xx[1], acc);
                    acc = fmaf(w[2], xx[2], acc);
                    acc = fmaf(w[3], xx[3], acc);
                }
                a[l] = acc;
            }
            for (uint32_t d = 16; d > 0; d >>= 1) {
                float b[32];
                for (uint32_t l = 0; l < 32; ++l) b[l] = a[l] + a[l ^ d];
                memcpy(a, b, sizeof a);
            }
            p[q] = a[0];
        }
        const float s = (p[0] + p[1]) + (p[2] + p[3]);
        y[r] = biais ? s + biais[r] : s;
    }
}
