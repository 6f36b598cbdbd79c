// troncons_b200 — the whole decode step of a gpt-oss model (the reference's Modele:
// enchasser, debut_couche, fin_couche, sortie; trc-modele/src/lib.rs:476-568), and the seeded
// synthetic weights it is measured on.
//
// The step launches, on the caller's stream: x <- row `jeton` of the Q8_0 embedding (exact);
// per layer, the reference's order kernel for kernel: RMSNorm, q / k / v Q8_0 GEMVs + biases,
// YaRN, the KV write (ring on sliding layers), attention with sinks, the output GEMV, x += o,
// RMSNorm, router logits, top-k softmax, then the fused MoE layer (decode fused into the
// GEMVs, x += sum of the weighted experts) in place of decode-into-slots + GEMVs + combine;
// after the last layer, RMSNorm, the Q8_0 unembedding and the greedy token (argmax, ties to the
// smallest index). The fused layer gives the decode-then-multiply bits (tested), so the logits
// are those of the reference's sequence with this library's GEMV order.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstring>

#include "../../include/troncons_b200.h"
#include "commun.cuh"
#include "noyaux.h"

namespace tb {

// ---------------------------------------------------------------- embedding row, argmax

// Row `ligne` of a Q8_0 matrix of C columns -> f32[C]: d (f16) times q (i8), exact in f32
// (11 + 7 significant bits) (passe.cuh:623-634).
__global__ void __launch_bounds__(256) k_ligne_q8_0(const uint8_t* __restrict__ w, uint32_t ligne, uint32_t C,
                                                   float* __restrict__ y) {
    attendre_amont();
    liberer_aval();
    const uint32_t i = blockIdx.x * 256u + threadIdx.x;
    if (i >= C) return;
    const uint8_t* b = w + (uint64_t(ligne) * (C / 32u) + i / 32u) * 34u;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(b[0] | (b[1] << 8))));
    y[i] = d * float(static_cast<int8_t>(b[2 + (i & 31u)]));
}

// The larger of two candidates in the total order (value descending, index ascending); a NaN is
// never chosen (passe.cuh:636-669).
__device__ __forceinline__ bool meilleur(float x, uint32_t i, float bx, uint32_t bi) {
    if (x != x) return false;
    if (bi == 0xFFFFFFFFu) return true;
    return x > bx || (x == bx && i < bi);
}

// Index of the largest of n floats (ties: smallest index; all NaN: 0xFFFFFFFF): each thread a
// strided run, then a fixed tree (the result does not depend on it: a total order).
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ v, uint32_t n, uint32_t* __restrict__ sortie) {
    __shared__ float pv[1024];
    __shared__ uint32_t pi[1024];
    attendre_amont();
    liberer_aval();
    const uint32_t t = threadIdx.x;
    float bv = 0.0f;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = t; i < n; i += 1024u) {
        const float x = v[i];
        if (meilleur(x, i, bv, bi)) {
            bv = x;
            bi = i;
        }
    }
    pv[t] = bv;
    pi[t] = bi;
    __syncthreads();
    for (uint32_t s = 512; s > 0; s >>= 1) {
        if (t < s && pi[t + s] != 0xFFFFFFFFu && meilleur(pv[t + s], pi[t + s], pv[t], pi[t])) {
            pv[t] = pv[t + s];
            pi[t] = pi[t + s];
        }
        __syncthreads();
    }
    if (t == 0) sortie[0] = pi[0];
}

cudaError_t lancer_ligne_q8_0(const void* w, uint32_t ligne, uint32_t C, float* y, cudaStream_t flux) {
    return lancer_pdl(k_ligne_q8_0, dim3((C + 255) / 256), dim3(256), 0, flux, static_cast<const uint8_t*>(w), ligne, C, y);
}

cudaError_t lancer_argmax(const float* v, uint32_t n, uint32_t* sortie, cudaStream_t flux) {
    return lancer_pdl(k_argmax, dim3(1), dim3(1024), 0, flux, v, n, sortie);
}

// ---------------------------------------------------------------- seeded synthetic weights

// A counter-based generator: splitmix64's finaliser on (seed, stream, counter).
__device__ __forceinline__ uint64_t melange(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
__device__ __forceinline__ uint64_t alea(uint64_t graine, uint64_t flux_id, uint64_t i) {
    return melange(graine * 0x9E3779B97F4A7C15ull ^ melange(flux_id + 0x632BE59BD9B4E019ull) ^ (i * 0xD1B54A32D192ED03ull));
}
__device__ __forceinline__ double uniforme(uint64_t r) { return (double((r >> 11) + 1ull)) * (1.0 / 9007199254740993.0); }
// A standard normal (Box-Muller on two draws).
__device__ __forceinline__ double normale(uint64_t graine, uint64_t flux_id, uint64_t i) {
    const double u1 = uniforme(alea(graine, flux_id, 2 * i)), u2 = uniforme(alea(graine, flux_id, 2 * i + 1));
    return sqrt(-2.0 * log(u1)) * cos(6.283185307179586 * u2);
}

// E2M1 code (sign bit 3) nearest to v in {0, .5, 1, 1.5, 2, 3, 4, 6}, ties to the even code;
// beyond 6, 6.
__device__ __forceinline__ uint32_t e2m1(double v) {
    const double a = fabs(v);
    const double g[8] = {0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0};
    uint32_t c = 7;
    for (uint32_t i = 0; i < 7; ++i) {
        const double m = 0.5 * (g[i] + g[i + 1]);
        if (a < m || (a == m && (i % 2u) == 0u)) {
            c = i;
            break;
        }
    }
    return c | (v < 0.0 ? 8u : 0u);
}

// Matrix `matrice` (a stream id) of R x C MXFP4 weights as 17-byte blocks [e, qs x 16] and f32
// biases: row sigma = 0.02 exp(0.3 N), weights N(0, sigma), E8M0 = floor(log2 max|w|) - 2 (+127),
// E2M1 to nearest (the sign kept: -0 occurs), biases N(0, 0.01) rounded to bf16. One thread per
// 32-block (config 0's distribution).
__global__ void __launch_bounds__(256) k_synth_mxfp4(uint8_t* __restrict__ blocs, float* __restrict__ biais, uint32_t R,
                                                     uint32_t C, uint64_t graine, uint64_t matrice) {
    const uint32_t B = C / 32u;
    const uint64_t b = uint64_t(blockIdx.x) * 256u + threadIdx.x;
    if (b >= uint64_t(R) * B) return;
    const uint32_t r = uint32_t(b / B);
    const double sigma = 0.02 * exp(0.3 * normale(graine, matrice * 4u + 1u, r));
    double w[32], m = 0.0;
    for (uint32_t i = 0; i < 32; ++i) {
        w[i] = sigma * normale(graine, matrice * 4u + 2u, b * 32u + i);
        m = fmax(m, fabs(w[i]));
    }
    int e = m > 0.0 ? int(floor(log2(m))) - 2 + 127 : 0;
    e = e < 1 ? 1 : (e > 254 ? 254 : e);
    const double s = ldexp(1.0, e - 127);
    uint8_t* o = blocs + b * 17u;
    o[0] = uint8_t(e);
    for (uint32_t i = 0; i < 16; ++i) o[1 + i] = uint8_t(e2m1(w[i] / s) | (e2m1(w[16 + i] / s) << 4));
    if (b % B == 0) {
        const float v = float(0.01 * normale(graine, matrice * 4u + 3u, r));
        biais[r] = __bfloat162float(__float2bfloat16(v));
    }
}

// R x C Q8_0 (34-byte blocks: f16 d, 32 x i8): rows of N(0, 0.02) weights quantised per block
// (d = max|w| / 127, q = round(w / d)).
__global__ void __launch_bounds__(256) k_synth_q8_0(uint8_t* __restrict__ w, uint32_t R, uint32_t C, uint64_t graine,
                                                    uint64_t matrice) {
    const uint64_t b = uint64_t(blockIdx.x) * 256u + threadIdx.x;
    if (b >= uint64_t(R) * (C / 32u)) return;
    double v[32], m = 0.0;
    for (uint32_t i = 0; i < 32; ++i) {
        v[i] = 0.02 * normale(graine, matrice * 4u + 2u, b * 32u + i);
        m = fmax(m, fabs(v[i]));
    }
    const __half dh = __float2half(float(m / 127.0));
    const double d = double(__half2float(dh));
    uint8_t* o = w + b * 34u;
    const unsigned short bits = __half_as_ushort(dh);
    o[0] = uint8_t(bits & 0xFFu);
    o[1] = uint8_t(bits >> 8);
    for (uint32_t i = 0; i < 32; ++i) {
        double q = d > 0.0 ? rint(v[i] / d) : 0.0;
        q = q > 127.0 ? 127.0 : (q < -127.0 ? -127.0 : q);
        o[2 + i] = uint8_t(static_cast<int8_t>(q));
    }
}

// n f32 values: moyenne + ecart * N(0, 1).
__global__ void __launch_bounds__(256) k_synth_f32(float* __restrict__ y, uint64_t n, uint64_t graine, uint64_t flux_id,
                                                   float moyenne, float ecart) {
    const uint64_t i = uint64_t(blockIdx.x) * 256u + threadIdx.x;
    if (i < n) y[i] = float(double(moyenne) + double(ecart) * normale(graine, flux_id, i));
}

// The raw part of expert e (9 streams ECHELLES_BRUTES, CODES_BRUTS, BIAIS per matrix;
// trc-codec/src/lib.rs:432-445): the header and stream table (`entete`, identical for every
// expert but its number at bytes 6-7) then each matrix's scales, codes and biases gathered
// from its 17-byte blocks at the table's offsets; zeros elsewhere.
__global__ void __launch_bounds__(256) k_partie_brute(const DescCodage* __restrict__ descs, const uint8_t* __restrict__ entete,
                                                      uint32_t entete_octets, Dims dims, uint64_t taille) {
    const DescCodage& d = descs[blockIdx.y];
    uint8_t* p = reinterpret_cast<uint8_t*>(d.sortie);
    const uint64_t t0 = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x, pas = uint64_t(gridDim.x) * blockDim.x;
    // zeros, then the header (the streams' bytes are written after a grid-wide barrier would be
    // needed; instead every byte is written exactly once: header, streams, and the gaps)
    const uint32_t* dec = reinterpret_cast<const uint32_t*>(entete + 64);  // descriptor i at 64 + 16 i
    for (uint64_t o = t0; o < taille; o += pas) {
        uint8_t v = 0;
        if (o < entete_octets) {
            v = entete[o];
            if (o == 6) v = uint8_t(d.expert);
            if (o == 7) v = uint8_t(d.expert >> 8);
        } else {
            for (uint32_t j = 0; j < 3; ++j) {
                const uint32_t B = dims.colonnes[j] / 32u;
                const uint64_t nb = uint64_t(dims.lignes[j]) * B;
                const uint8_t* blocs = reinterpret_cast<const uint8_t*>(d.blocs[j]);
                const uint64_t de = dec[(3 * j + 0) * 4 + 1], dc = dec[(3 * j + 1) * 4 + 1], db = dec[(3 * j + 2) * 4 + 1];
                if (o >= de && o < de + nb) v = blocs[17u * (o - de)];
                else if (o >= dc && o < dc + 16u * nb) v = blocs[17u * ((o - dc) / 16u) + 1u + (o - dc) % 16u];
                else if (o >= db && o < db + 4ull * dims.lignes[j])
                    v = reinterpret_cast<const uint8_t*>(d.biais[j])[o - db];
            }
        }
        p[o] = v;
    }
}

cudaError_t lancer_synth_mxfp4(uint8_t* blocs, float* biais, uint32_t R, uint32_t C, uint64_t graine, uint64_t matrice,
                               cudaStream_t flux) {
    const uint64_t nb = uint64_t(R) * (C / 32u);
    k_synth_mxfp4<<<uint32_t((nb + 255) / 256), 256, 0, flux>>>(blocs, biais, R, C, graine, matrice);
    return cudaGetLastError();
}

cudaError_t lancer_synth_q8_0(uint8_t* w, uint32_t R, uint32_t C, uint64_t graine, uint64_t matrice, cudaStream_t flux) {
    const uint64_t nb = uint64_t(R) * (C / 32u);
    k_synth_q8_0<<<uint32_t((nb + 255) / 256), 256, 0, flux>>>(w, R, C, graine, matrice);
    return cudaGetLastError();
}

cudaError_t lancer_synth_f32(float* y, uint64_t n, uint64_t graine, uint64_t flux_id, float moyenne, float ecart,
                             cudaStream_t flux) {
    k_synth_f32<<<uint32_t((n + 255) / 256), 256, 0, flux>>>(y, n, graine, flux_id, moyenne, ecart);
    return cudaGetLastError();
}

cudaError_t lancer_parties_brutes(const DescCodage* descs, uint32_t n, const uint8_t* entete, uint32_t entete_octets,
                                  const Dims& dims, uint64_t taille, cudaStream_t flux) {
    k_partie_brute<<<dim3(1184, n), 256, 0, flux>>>(descs, entete, entete_octets, dims, taille);
    return cudaGetLastError();
}

}  // namespace tb

// ---------------------------------------------------------------- the step

namespace {

struct DispositionModele {
    uint64_t x, h, q, k, v, a, o, h2, lr, idx, pw, z, jeton, controle, moe, total;
};

DispositionModele disposition_modele(const trc_modele_config& m) {
    DispositionModele d{};
    const uint64_t dq = uint64_t(m.tetes) * m.dim_tete, dkv = uint64_t(m.tetes_kv) * m.dim_tete;
    uint64_t p = 0;
    auto zone = [&](uint64_t& z, uint64_t n) {
        z = p;
        p = tb::al256(p + n);
    };
    zone(d.x, 4ull * m.d);
    zone(d.h, 4ull * m.d);
    zone(d.q, 4 * dq);
    zone(d.k, 4 * dkv);
    zone(d.v, 4 * dkv);
    zone(d.a, 4 * dq);
    zone(d.o, 4ull * m.d);
    zone(d.h2, 4ull * m.d);
    zone(d.lr, 4ull * m.experts);
    zone(d.idx, 4ull * m.k);
    zone(d.pw, 4ull * m.k);
    zone(d.z, 4ull * m.vocab);
    zone(d.jeton, 16);
    zone(d.controle, 16ull * m.k);
    zone(d.moe, trc_moe_espace_recouvrant_octets(&m.dims, m.k));
    d.total = p;
    return d;
}

// The checks every entry of the step makes (descriptor, shapes, workspace), then the stream's
// device.
int verifier_modele(const trc_modele_config* m, DispositionModele& d, void* flux) {
    if (m == nullptr || m->couches == 0 || m->couches_desc == 0 || m->espace == 0 || m->enchassement == 0)
        return tb::erreur_usage("model: descriptor incomplete");
    if (m->dim_tete != 64 || m->tetes % m->tetes_kv != 0 || m->d % 32 != 0 || m->k == 0 || m->k > 8)
        return tb::erreur_usage("model: attention or routing shape not supported");
    d = disposition_modele(*m);
    if (m->espace_octets < d.total || m->espace % 256 != 0) return tb::erreur_usage("model: workspace too small or misaligned");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    return TRC_OK;
}

#define ESSAI(x)                                       \
    do {                                               \
        if (cudaError_t e_ = (x)) return e_;           \
    } while (0)

// Layer l's attention side for the token in x at `position` (Modele::debut_couche, trc-modele/
// src/lib.rs:476-531): RMSNorm, q / k / v, YaRN, the KV write, attention, x += o; then the
// post-attention RMSNorm into h2, the MoE's input.
cudaError_t etape_attention(const trc_modele_config& m, const DispositionModele& d, uint8_t* esp, uint32_t l,
                            uint32_t position, cudaStream_t f) {
    auto F = [&](uint64_t o) { return reinterpret_cast<float*>(esp + o); };
    auto P = [](uint64_t a) { return reinterpret_cast<const float*>(a); };
    const uint32_t D = m.d, dq = m.tetes * m.dim_tete, dkv = m.tetes_kv * m.dim_tete;
    const trc_modele_couche& c = reinterpret_cast<const trc_modele_couche*>(m.couches_desc)[l];
    tb::ParamsRope rope;
    std::memcpy(&rope, &m.rope, sizeof rope);
    // RMSNorm and the q / k / v projections in one launch (the same bits as four)
    tb::DescQ8Couche qkv{};
    qkv.w[0] = reinterpret_cast<const void*>(c.wq);
    qkv.w[1] = reinterpret_cast<const void*>(c.wk);
    qkv.w[2] = reinterpret_cast<const void*>(c.wv);
    qkv.biais[0] = P(c.bq);
    qkv.biais[1] = P(c.bk);
    qkv.biais[2] = P(c.bv);
    qkv.y[0] = F(d.q);
    qkv.y[1] = F(d.k);
    qkv.y[2] = F(d.v);
    qkv.lignes[0] = dq;
    qkv.lignes[1] = dkv;
    qkv.lignes[2] = dkv;
    qkv.n = 3;
    qkv.C = D;
    qkv.x = F(d.x);
    qkv.norme = P(c.attn_norm);
    qkv.eps = m.eps;
    qkv.h = F(d.h);
    ESSAI(tb::lancer_q8_0_couche(qkv, f));
    const uint32_t case_kv = c.anneau ? position % c.anneau : position;
    ESSAI(tb::lancer_rope_kv(F(d.q), F(d.k), F(d.v), reinterpret_cast<uint16_t*>(c.cache_k),
                             reinterpret_cast<uint16_t*>(c.cache_v), m.tetes, m.tetes_kv, position, case_kv, rope, f));
    tb::ParamsAttention pa{};
    pa.tetes = m.tetes;
    pa.tetes_kv = m.tetes_kv;
    pa.dim_tete = m.dim_tete;
    pa.fin = position + 1;
    pa.debut = c.anneau && pa.fin > c.anneau ? pa.fin - c.anneau : 0;
    pa.anneau = c.anneau;
    pa.echelle = 1.0f / std::sqrt(float(m.dim_tete));
    ESSAI(tb::lancer_attention(F(d.q), reinterpret_cast<const uint16_t*>(c.cache_k),
                               reinterpret_cast<const uint16_t*>(c.cache_v), P(c.puits), F(d.a), pa, f));
    // the output projection with x += o folded in (the same bits as the GEMV, then the combine)
    tb::DescQ8Couche o{};
    o.w[0] = reinterpret_cast<const void*>(c.wo);
    o.biais[0] = P(c.bo);
    o.y[0] = F(d.o);
    o.lignes[0] = D;
    o.n = 1;
    o.C = dq;
    o.x = F(d.a);
    o.residu = F(d.x);
    ESSAI(tb::lancer_q8_0_couche(o, f));
    ESSAI(tb::lancer_rmsnorm(F(d.x), P(c.post_norm), F(d.h2), D, 1, m.eps, f));
    return cudaSuccess;
}

// Layer l's MoE for the token (Modele::fin_couche, lib.rs:533-553): router logits, top-k
// softmax, then the fused layer (x += the weighted experts).
cudaError_t etape_moe(const trc_modele_config& m, const DispositionModele& d, uint8_t* esp, uint32_t l, cudaStream_t f) {
    auto F = [&](uint64_t o) { return reinterpret_cast<float*>(esp + o); };
    auto P = [](uint64_t a) { return reinterpret_cast<const float*>(a); };
    const trc_modele_couche& c = reinterpret_cast<const trc_modele_couche*>(m.couches_desc)[l];
    ESSAI(tb::lancer_gemv_f32(P(c.wr), F(d.h2), 0u, P(c.br), F(d.lr), m.experts, m.d, f));
    ESSAI(tb::lancer_topk(F(d.lr), m.experts, m.k, reinterpret_cast<uint32_t*>(esp + d.idx), F(d.pw), nullptr, 0, f));
    tb::Couche k{};
    k.parties = reinterpret_cast<const uint64_t*>(c.parties);
    k.parties_octets = reinterpret_cast<const uint64_t*>(c.parties_octets);
    k.experts = m.experts;
    k.k = m.k;
    k.luts = reinterpret_cast<const uint32_t*>(c.luts);
    for (int j = 0; j < 3; ++j) {
        k.lignes[j] = m.dims.lignes[j];
        k.colonnes[j] = m.dims.colonnes[j];
    }
    k.indices = reinterpret_cast<const uint32_t*>(esp + d.idx);
    k.poids = F(d.pw);
    k.x = F(d.h2);
    k.x_bf16 = 0;
    k.brut = m.brut ? 1u : 0u;
    k.residu = F(d.x);
    k.controle = reinterpret_cast<uint32_t*>(esp + d.controle);
    k.n_delta = m.n_delta;
    k.n_codes = m.n_codes;
    k.jetons = 1;
    k.deltas = m.brut ? nullptr : reinterpret_cast<const uint8_t*>(c.deltas);
    return tb::lancer_moe(k, esp + d.moe, d.total - d.moe, f);
}

// After the last layer (Modele::sortie, lib.rs:555-568): RMSNorm, the Q8_0 unembedding, the greedy
// token.
cudaError_t etape_sortie(const trc_modele_config& m, const DispositionModele& d, uint8_t* esp, cudaStream_t f) {
    auto F = [&](uint64_t o) { return reinterpret_cast<float*>(esp + o); };
    ESSAI(tb::lancer_rmsnorm(F(d.x), reinterpret_cast<const float*>(m.norme_sortie), F(d.h), m.d, 1, m.eps, f));
    ESSAI(tb::lancer_gemv_q8_0(reinterpret_cast<const void*>(m.sortie), F(d.h), nullptr, F(d.z), m.vocab, m.d, f));
    return tb::lancer_argmax(F(d.z), m.vocab, reinterpret_cast<uint32_t*>(esp + d.jeton), f);
}

// The batch workspace of n sequences' attention sides: f32 rows [n][d] / [n][dq] / [n][dkv].
struct DispositionLot {
    uint64_t h, q, k, v, a, o, total;
};

DispositionLot disposition_lot(const trc_modele_config& m, uint32_t n) {
    DispositionLot d{};
    const uint64_t dq = uint64_t(m.tetes) * m.dim_tete, dkv = uint64_t(m.tetes_kv) * m.dim_tete;
    uint64_t p = 0;
    auto zone = [&](uint64_t& z, uint64_t octets) {
        z = p;
        p = tb::al256(p + octets);
    };
    zone(d.h, 4ull * n * m.d);
    zone(d.q, 4ull * n * dq);
    zone(d.k, 4ull * n * dkv);
    zone(d.v, 4ull * n * dkv);
    zone(d.a, 4ull * n * dq);
    zone(d.o, 4ull * n * m.d);
    d.total = p;
    return d;
}

// Layer l's attention side for n sequences at the same position: what etape_attention does for
// each, with the four Q8_0 GEMVs once for all n tokens (each row of weights read once; every
// token's sums in the single-token order, so each sequence gets etape_attention's bits).
cudaError_t etape_attention_lot(const trc_modele_config* const* seqs, uint32_t n, uint32_t l, uint32_t position,
                                uint8_t* lot, cudaStream_t f) {
    const trc_modele_config& m = *seqs[0];
    const DispositionLot b = disposition_lot(m, n);
    auto L = [&](uint64_t o) { return reinterpret_cast<float*>(lot + o); };
    auto P = [](uint64_t a) { return reinterpret_cast<const float*>(a); };
    auto X = [&](uint32_t i, uint64_t DispositionModele::*z) {
        return reinterpret_cast<float*>(seqs[i]->espace + disposition_modele(*seqs[i]).*z);
    };
    const uint32_t D = m.d, dq = m.tetes * m.dim_tete, dkv = m.tetes_kv * m.dim_tete;
    const trc_modele_couche& c0 = reinterpret_cast<const trc_modele_couche*>(m.couches_desc)[l];
    tb::ParamsRope rope;
    std::memcpy(&rope, &m.rope, sizeof rope);
    for (uint32_t i = 0; i < n; ++i)
        ESSAI(tb::lancer_rmsnorm(X(i, &DispositionModele::x), P(c0.attn_norm), L(b.h) + uint64_t(i) * D, D, 1, m.eps, f));
    // the q / k / v projections of the n tokens in one launch per 8 tokens
    tb::DescQ8Couche qkv{};
    qkv.w[0] = reinterpret_cast<const void*>(c0.wq);
    qkv.w[1] = reinterpret_cast<const void*>(c0.wk);
    qkv.w[2] = reinterpret_cast<const void*>(c0.wv);
    qkv.biais[0] = P(c0.bq);
    qkv.biais[1] = P(c0.bk);
    qkv.biais[2] = P(c0.bv);
    qkv.y[0] = L(b.q);
    qkv.y[1] = L(b.k);
    qkv.y[2] = L(b.v);
    qkv.lignes[0] = dq;
    qkv.lignes[1] = dkv;
    qkv.lignes[2] = dkv;
    qkv.n = 3;
    qkv.C = D;
    qkv.x = L(b.h);
    ESSAI(tb::lancer_q8_0_couche(qkv, f, n));
    for (uint32_t i = 0; i < n; ++i) {
        const trc_modele_couche& c = reinterpret_cast<const trc_modele_couche*>(seqs[i]->couches_desc)[l];
        float* q = L(b.q) + uint64_t(i) * dq;
        float* k = L(b.k) + uint64_t(i) * dkv;
        const uint32_t case_kv = c.anneau ? position % c.anneau : position;
        ESSAI(tb::lancer_rope_kv(q, k, L(b.v) + uint64_t(i) * dkv, reinterpret_cast<uint16_t*>(c.cache_k),
                                 reinterpret_cast<uint16_t*>(c.cache_v), m.tetes, m.tetes_kv, position, case_kv, rope, f));
        tb::ParamsAttention pa{};
        pa.tetes = m.tetes;
        pa.tetes_kv = m.tetes_kv;
        pa.dim_tete = m.dim_tete;
        pa.fin = position + 1;
        pa.debut = c.anneau && pa.fin > c.anneau ? pa.fin - c.anneau : 0;
        pa.anneau = c.anneau;
        pa.echelle = 1.0f / std::sqrt(float(m.dim_tete));
        ESSAI(tb::lancer_attention(q, reinterpret_cast<const uint16_t*>(c.cache_k), reinterpret_cast<const uint16_t*>(c.cache_v),
                                   P(c.puits), L(b.a) + uint64_t(i) * dq, pa, f));
    }
    ESSAI(tb::lancer_gemv_q8_0_lot(reinterpret_cast<const void*>(c0.wo), L(b.a), P(c0.bo), L(b.o), D, dq, n, f));
    for (uint32_t i = 0; i < n; ++i) {
        ESSAI(tb::lancer_combiner(X(i, &DispositionModele::x), L(b.o) + uint64_t(i) * D, D, nullptr, 1, D, f));
        ESSAI(tb::lancer_rmsnorm(X(i, &DispositionModele::x), P(c0.post_norm), X(i, &DispositionModele::h2), D, 1, m.eps, f));
    }
    return cudaSuccess;
}

#undef ESSAI

}  // namespace

extern "C" {

int trc_ligne_q8_0(const void* w, size_t w_octets, uint32_t ligne, uint32_t colonnes, float* y, size_t y_octets, void* flux) {
    if (w == nullptr || y == nullptr || colonnes == 0 || colonnes % 32 != 0 ||
        w_octets < (uint64_t(ligne) + 1) * (colonnes / 32) * 34ull || y_octets < 4ull * colonnes)
        return tb::erreur_usage("ligne_q8_0: views too short or columns not a multiple of 32");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    if (cudaError_t e = tb::lancer_ligne_q8_0(w, ligne, colonnes, y, static_cast<cudaStream_t>(flux))) return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_argmax(const float* v, size_t v_octets, uint32_t n, uint32_t* sortie, size_t sortie_octets, void* flux) {
    if (v == nullptr || sortie == nullptr || n == 0 || v_octets < 4ull * n || sortie_octets < 4)
        return tb::erreur_usage("argmax: views too short");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    if (cudaError_t e = tb::lancer_argmax(v, n, sortie, static_cast<cudaStream_t>(flux))) return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_synth_mxfp4_gpu(uint8_t* blocs, float* biais, uint32_t lignes, uint32_t colonnes, uint64_t graine,
                        uint64_t matrice, void* flux) {
    if (blocs == nullptr || biais == nullptr || lignes == 0 || colonnes == 0 || colonnes % 32 != 0)
        return tb::erreur_usage("synth_mxfp4: buffers or shape");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    if (cudaError_t e = tb::lancer_synth_mxfp4(blocs, biais, lignes, colonnes, graine, matrice, static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_synth_q8_0_gpu(uint8_t* w, uint32_t lignes, uint32_t colonnes, uint64_t graine, uint64_t matrice, void* flux) {
    if (w == nullptr || lignes == 0 || colonnes == 0 || colonnes % 32 != 0) return tb::erreur_usage("synth_q8_0: buffer or shape");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    if (cudaError_t e = tb::lancer_synth_q8_0(w, lignes, colonnes, graine, matrice, static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_synth_f32_gpu(float* y, uint64_t n, uint64_t graine, uint64_t flux_id, float moyenne, float ecart, void* flux) {
    if (y == nullptr || n == 0) return tb::erreur_usage("synth_f32: buffer");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    if (cudaError_t e = tb::lancer_synth_f32(y, n, graine, flux_id, moyenne, ecart, static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_parties_brutes_gpu(const trc_desc_codage* descs, uint32_t n, const trc_dims_expert* dims, const uint8_t* entete,
                           uint32_t entete_octets, uint64_t taille, void* flux) {
    if (descs == nullptr || n == 0 || n > 65535 || dims == nullptr || entete == nullptr || entete_octets < 64 || taille == 0)
        return tb::erreur_usage("parties_brutes: arguments");
    tb::Dims d;
    for (int j = 0; j < 3; ++j) {
        d.lignes[j] = dims->lignes[j];
        d.colonnes[j] = dims->colonnes[j];
    }
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    if (cudaError_t e = tb::lancer_parties_brutes(reinterpret_cast<const tb::DescCodage*>(descs), n, entete, entete_octets, d,
                                                  taille, static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

uint64_t trc_modele_espace_octets(const trc_modele_config* m) {
    if (m == nullptr || m->k == 0) return 0;
    return disposition_modele(*m).total;
}

int trc_modele_sorties(const trc_modele_config* m, uint64_t* logits, uint64_t* jeton, uint64_t* controle) {
    if (m == nullptr) return tb::erreur_usage("model absent");
    const DispositionModele d = disposition_modele(*m);
    if (logits) *logits = m->espace + d.z;
    if (jeton) *jeton = m->espace + d.jeton;
    if (controle) *controle = m->espace + d.controle;
    return TRC_OK;
}

// One token (Modele::enchasser + debut_couche/fin_couche per layer + sortie, trc-modele/src/
// lib.rs:476-568). `sortie` = 0 skips the unembedding (a context token).
int trc_modele_pas(const trc_modele_config* m, uint32_t jeton, uint32_t position, uint32_t sortie, void* flux) {
    DispositionModele d;
    if (int r = verifier_modele(m, d, flux)) return r;
    if (jeton >= m->vocab || position >= m->contexte) return tb::erreur_usage("model: token or position out of range");
    const cudaStream_t f = static_cast<cudaStream_t>(flux);
    uint8_t* esp = reinterpret_cast<uint8_t*>(m->espace);
    cudaError_t e = tb::lancer_ligne_q8_0(reinterpret_cast<const void*>(m->enchassement), jeton, m->d,
                                          reinterpret_cast<float*>(esp + d.x), f);
    for (uint32_t l = 0; l < m->couches && e == cudaSuccess; ++l) {
        e = etape_attention(*m, d, esp, l, position, f);
        if (e == cudaSuccess) e = etape_moe(*m, d, esp, l, f);
    }
    if (e == cudaSuccess && sortie) e = etape_sortie(*m, d, esp, f);
    return e == cudaSuccess ? TRC_OK : tb::erreur_cuda(e);
}

int trc_modele_debut(const trc_modele_config* m, uint32_t jeton, void* flux) {
    DispositionModele d;
    if (int r = verifier_modele(m, d, flux)) return r;
    if (jeton >= m->vocab) return tb::erreur_usage("model: token out of range");
    uint8_t* esp = reinterpret_cast<uint8_t*>(m->espace);
    if (cudaError_t e = tb::lancer_ligne_q8_0(reinterpret_cast<const void*>(m->enchassement), jeton, m->d,
                                              reinterpret_cast<float*>(esp + d.x), static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_modele_attention(const trc_modele_config* m, uint32_t couche, uint32_t position, void* flux) {
    DispositionModele d;
    if (int r = verifier_modele(m, d, flux)) return r;
    if (couche >= m->couches || position >= m->contexte) return tb::erreur_usage("model: layer or position out of range");
    if (cudaError_t e = etape_attention(*m, d, reinterpret_cast<uint8_t*>(m->espace), couche, position,
                                        static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

uint64_t trc_modele_lot_espace_octets(const trc_modele_config* m, uint32_t n) {
    if (m == nullptr || n == 0) return 0;
    return disposition_lot(*m, n).total;
}

int trc_modele_attention_lot(const trc_modele_config* const* sequences, uint32_t n, uint32_t couche, uint32_t position,
                             void* espace, size_t espace_octets, void* flux) {
    if (sequences == nullptr || n == 0 || espace == nullptr) return tb::erreur_usage("model batch: sequences or workspace missing");
    DispositionModele d;
    for (uint32_t i = 0; i < n; ++i)
        if (int r = verifier_modele(sequences[i], d, flux)) return r;
    const trc_modele_config& m = *sequences[0];
    if (couche >= m.couches || position >= m.contexte) return tb::erreur_usage("model batch: layer or position out of range");
    if (espace_octets < disposition_lot(m, n).total || reinterpret_cast<uintptr_t>(espace) % 256 != 0)
        return tb::erreur_usage("model batch: workspace too small or misaligned");
    // one model: the same shapes and the same layer weights (each its own caches and workspace)
    const trc_modele_couche& c0 = reinterpret_cast<const trc_modele_couche*>(m.couches_desc)[couche];
    for (uint32_t i = 1; i < n; ++i) {
        const trc_modele_config& s = *sequences[i];
        const trc_modele_couche& c = reinterpret_cast<const trc_modele_couche*>(s.couches_desc)[couche];
        if (s.d != m.d || s.tetes != m.tetes || s.tetes_kv != m.tetes_kv || s.couches != m.couches ||
            std::memcmp(&s.rope, &m.rope, sizeof m.rope) != 0 || s.eps != m.eps || c.wq != c0.wq || c.wk != c0.wk ||
            c.wv != c0.wv || c.wo != c0.wo || c.bq != c0.bq || c.bk != c0.bk || c.bv != c0.bv || c.bo != c0.bo ||
            c.attn_norm != c0.attn_norm || c.post_norm != c0.post_norm || c.puits != c0.puits || c.anneau != c0.anneau)
            return tb::erreur_usage("model batch: the sequences are not of one model");
        if (c.cache_k == c0.cache_k || s.espace == m.espace) return tb::erreur_usage("model batch: two sequences share a cache or workspace");
    }
    if (cudaError_t e = etape_attention_lot(sequences, n, couche, position, static_cast<uint8_t*>(espace),
                                            static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_modele_moe(const trc_modele_config* m, uint32_t couche, void* flux) {
    DispositionModele d;
    if (int r = verifier_modele(m, d, flux)) return r;
    if (couche >= m->couches) return tb::erreur_usage("model: layer out of range");
    if (cudaError_t e = etape_moe(*m, d, reinterpret_cast<uint8_t*>(m->espace), couche, static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_modele_fin(const trc_modele_config* m, void* flux) {
    DispositionModele d;
    if (int r = verifier_modele(m, d, flux)) return r;
    if (cudaError_t e = etape_sortie(*m, d, reinterpret_cast<uint8_t*>(m->espace), static_cast<cudaStream_t>(flux)))
        return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_modele_etat(const trc_modele_config* m, uint64_t* x, uint64_t* h2) {
    if (m == nullptr || m->espace == 0) return tb::erreur_usage("model absent");
    const DispositionModele d = disposition_modele(*m);
    if (x) *x = m->espace + d.x;
    if (h2) *h2 = m->espace + d.h2;
    return TRC_OK;
}

}  // extern "C"
