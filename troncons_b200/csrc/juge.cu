// troncons_b200 — the quality judge on the GPU: the 16-bit logit entries of llama-perplexity's
// `.kld` files and the per-position KL / first-choice / NLL figures of the reference's trc-juge
// (kld.rs:148-186, stats.rs:24-85), over the whole vocabulary, one block per position.
//
// Entry (kld.rs:1-16): nv = 2 ceil(n / 2) + 4 u16 words: f32 pas, f32 log_p_min, n codes (and
// one zero pad word when n is odd); log p_i ~ pas * code_i + log_p_min, in f32, the product and
// the sum rounded separately (kld.rs:139-142). Coding (kld.rs:148-186), in f64: max, min of the
// row, min raised to max - 16, lse = ln sum exp(l - max), log_p_min = f32(min - max - lse),
// pas = f32((max - min) / 65535), code = round((l - min) / pas) clamped to [0, 65535] when l >
// min, else 0 (all 0 when pas = 0).
//
// Position (stats.rs:41-85): P a coded entry, Q either a coded entry (its log-probabilities
// taken as they are, not renormalised: stats.rs:33-39) or raw logits (f32 or f64, renormalised
// by their log-sum-exp); argmax of each with ties to the first index (NaN never chosen);
// KL(P || Q) = sum over log p_i > -16 of p_i (log p_i - log q_i); NLL of the next token under
// each; dp = q(next) - p(next). All sums in f64, per thread in index order, then a fixed tree:
// the same bits for every launch, within rounding of the reference's serial sums.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "../../include/troncons_b200.h"
#include "noyaux.h"

namespace tb {
namespace {

constexpr uint32_t JUGE_FILS = 512u;
constexpr uint32_t JUGE_WARPS = JUGE_FILS / 32u;

struct Meilleur {
    double v;
    uint32_t i;
};

// a before b: larger value, then smaller index.
__device__ __forceinline__ Meilleur plus_grand(Meilleur a, Meilleur b) {
    return (b.v > a.v || (b.v == a.v && b.i < a.i)) ? b : a;
}

__device__ __forceinline__ Meilleur reduire_meilleur(Meilleur m, Meilleur* tampon) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        Meilleur o;
        o.v = __shfl_xor_sync(0xFFFFFFFFu, m.v, d);
        o.i = __shfl_xor_sync(0xFFFFFFFFu, m.i, d);
        m = plus_grand(m, o);
    }
    const uint32_t w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) tampon[w] = m;
    __syncthreads();
    Meilleur r = tampon[0];
    for (uint32_t k = 1; k < JUGE_WARPS; ++k) r = plus_grand(r, tampon[k]);
    return r;
}

__device__ __forceinline__ double reduire_somme(double s, double* tampon) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, d);
    const uint32_t w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) tampon[w] = s;
    __syncthreads();
    double r = tampon[0];
    for (uint32_t k = 1; k < JUGE_WARPS; ++k) r += tampon[k];
    return r;
}

__device__ __forceinline__ double reduire_max(double v, double* tampon, bool plus_petit) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        const double o = __shfl_xor_sync(0xFFFFFFFFu, v, d);
        v = plus_petit ? fmin(v, o) : fmax(v, o);
    }
    const uint32_t w = threadIdx.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31u) == 0) tampon[w] = v;
    __syncthreads();
    double r = tampon[0];
    for (uint32_t k = 1; k < JUGE_WARPS; ++k) r = plus_petit ? fmin(r, tampon[k]) : fmax(r, tampon[k]);
    return r;
}

__device__ __forceinline__ double lire_logit(const void* q, uint32_t f64, uint64_t i) {
    return f64 ? static_cast<const double*>(q)[i] : double(static_cast<const float*>(q)[i]);
}

// log p_i of an entry: pas * code + log_p_min in f32, product and sum rounded separately.
__device__ __forceinline__ float log_p(float pas, float lpm, uint32_t code) {
    return __fadd_rn(__fmul_rn(pas, float(code)), lpm);
}

__device__ __forceinline__ void entete(const uint16_t* e, float& pas, float& lpm) {
    pas = __uint_as_float(uint32_t(e[0]) | (uint32_t(e[1]) << 16));
    lpm = __uint_as_float(uint32_t(e[2]) | (uint32_t(e[3]) << 16));
}

// One entry per block: row blockIdx.x of `logits` (n values, f32 or f64) -> nv words.
__global__ void __launch_bounds__(JUGE_FILS) k_coder_entrees(const void* __restrict__ logits, uint32_t f64, uint32_t n,
                                                           uint16_t* __restrict__ sortie) {
    __shared__ double tampon[JUGE_WARPS];
    __shared__ float tete[2];
    const uint64_t rang = blockIdx.x;
    const uint32_t paires = (n + 1u) / 2u, nv = 2u * paires + 4u;
    const uint64_t base = rang * n;
    double mx = -INFINITY, mn = INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += JUGE_FILS) {
        const double l = lire_logit(logits, f64, base + i);
        mx = fmax(mx, l);
        mn = fmin(mn, l);
    }
    mx = reduire_max(mx, tampon, false);
    mn = reduire_max(mn, tampon, true);
    mn = fmax(mn, mx - 16.0);
    double s = 0.0;
    for (uint32_t i = threadIdx.x; i < n; i += JUGE_FILS) s += exp(lire_logit(logits, f64, base + i) - mx);
    s = reduire_somme(s, tampon);
    uint16_t* e = sortie + rang * nv;
    if (threadIdx.x == 0) {
        const float lpm = __double2float_rn(mn - mx - log(s));
        const float pas = __double2float_rn((mx - mn) / 65535.0);
        tete[0] = pas;
        tete[1] = lpm;
        const uint32_t pb = __float_as_uint(pas), mb = __float_as_uint(lpm);
        e[0] = uint16_t(pb);
        e[1] = uint16_t(pb >> 16);
        e[2] = uint16_t(mb);
        e[3] = uint16_t(mb >> 16);
    }
    __syncthreads();
    const float pas = tete[0];
    const double inv = 1.0 / double(pas);
    // codes in pairs (one 32-bit store; entries are 4-byte aligned, codes start at word 4)
    uint32_t* paires_sortie = reinterpret_cast<uint32_t*>(e + 4);
    for (uint32_t j = threadIdx.x; j < paires; j += JUGE_FILS) {
        uint32_t c[2] = {0u, 0u};
#pragma unroll
        for (uint32_t k = 0; k < 2; ++k) {
            const uint32_t i = 2u * j + k;
            if (i < n && pas > 0.0f) {
                const double l = lire_logit(logits, f64, base + i);
                if (l > mn) c[k] = uint32_t(fmin(fmax(round((l - mn) * inv), 0.0), 65535.0));
            }
        }
        paires_sortie[j] = c[0] | (c[1] << 16);
    }
}

// One position per block. mode 0: q = coded entries (nv words per position); 1: raw f32
// logits (n per position); 2: raw f64 logits.
__global__ void __launch_bounds__(JUGE_FILS) k_positions(const uint16_t* __restrict__ p, const void* __restrict__ q,
                                                       uint32_t mode, const uint32_t* __restrict__ suivants, uint32_t n,
                                                       trc_juge_position* __restrict__ sortie) {
    __shared__ double tampon[JUGE_WARPS];
    __shared__ Meilleur tampon_m[JUGE_WARPS];
    const uint64_t rang = blockIdx.x;
    const uint32_t paires = (n + 1u) / 2u, nv = 2u * paires + 4u;
    const uint16_t* ep = p + rang * nv;
    float pas_p, lpm_p, pas_q = 0.0f, lpm_q = 0.0f;
    entete(ep, pas_p, lpm_p);
    const uint16_t* eq = mode == 0 ? static_cast<const uint16_t*>(q) + rang * nv : nullptr;
    if (mode == 0) entete(eq, pas_q, lpm_q);
    const uint32_t* cp = reinterpret_cast<const uint32_t*>(ep + 4);
    const uint32_t* cq = mode == 0 ? reinterpret_cast<const uint32_t*>(eq + 4) : nullptr;
    const uint64_t base = rang * n;
    // log q_i (before renormalisation): from the pair word of Q's entry, or the raw logit
    const auto lq = [=](uint32_t j, uint32_t k, uint32_t mot_q) -> double {
        if (mode == 0) return double(log_p(pas_q, lpm_q, k ? (mot_q >> 16) : (mot_q & 0xFFFFu)));
        return lire_logit(q, mode == 2, base + 2ull * j + k);
    };
    // pass 1: argmax of P and of Q
    Meilleur mp{-INFINITY, 0xFFFFFFFFu}, mq{-INFINITY, 0xFFFFFFFFu};
    for (uint32_t j = threadIdx.x; j < paires; j += JUGE_FILS) {
        const uint32_t mot_p = cp[j], mot_q = mode == 0 ? cq[j] : 0u;
#pragma unroll
        for (uint32_t k = 0; k < 2; ++k) {
            const uint32_t i = 2u * j + k;
            if (i >= n) break;
            const double a = double(log_p(pas_p, lpm_p, k ? (mot_p >> 16) : (mot_p & 0xFFFFu)));
            const double b = lq(j, k, mot_q);
            if (a > mp.v) mp = Meilleur{a, i};  // first index within the thread's increasing i
            if (b > mq.v) mq = Meilleur{b, i};
        }
    }
    mp = reduire_meilleur(mp, tampon_m);
    mq = reduire_meilleur(mq, tampon_m);
    if (mp.v == -INFINITY || mp.i == 0xFFFFFFFFu) mp.i = 0;  // nothing above -inf: index 0
    if (mq.v == -INFINITY || mq.i == 0xFFFFFFFFu) mq.i = 0;
    // pass 2 (raw logits): log-sum-exp of Q
    double lse = 0.0;
    if (mode != 0) {
        double s = 0.0;
        for (uint32_t i = threadIdx.x; i < n; i += JUGE_FILS) s += exp(lire_logit(q, mode == 2, base + i) - mq.v);
        s = reduire_somme(s, tampon);
        lse = mq.v + log(s);
    }
    // pass 3: KL(P || Q) over log p_i > -16
    double kl = 0.0;
    for (uint32_t j = threadIdx.x; j < paires; j += JUGE_FILS) {
        const uint32_t mot_p = cp[j], mot_q = mode == 0 ? cq[j] : 0u;
#pragma unroll
        for (uint32_t k = 0; k < 2; ++k) {
            const uint32_t i = 2u * j + k;
            if (i >= n) break;
            const double a = double(log_p(pas_p, lpm_p, k ? (mot_p >> 16) : (mot_p & 0xFFFFu)));
            if (a > -16.0) kl += exp(a) * (a - (lq(j, k, mot_q) - lse));
        }
    }
    kl = reduire_somme(kl, tampon);
    if (threadIdx.x == 0) {
        const uint32_t s = suivants[rang];
        trc_juge_position* r = sortie + rang;
        double nq = NAN, np = NAN;
        if (s < n) {
            const uint32_t mot_p = cp[s / 2u], mot_q = mode == 0 ? cq[s / 2u] : 0u;
            nq = lse - lq(s / 2u, s & 1u, mot_q);
            np = -double(log_p(pas_p, lpm_p, (s & 1u) ? (mot_p >> 16) : (mot_p & 0xFFFFu)));
        }
        r->kl = kl;
        r->nll_q = nq;
        r->nll_p = np;
        r->dp = exp(-nq) - exp(-np);
        r->premier_p = mp.i;
        r->premier_q = mq.i;
        r->meme_premier = mp.i == mq.i ? 1u : 0u;
        r->suivant_valide = s < n ? 1u : 0u;
    }
}

}  // namespace
}  // namespace tb

extern "C" {

int trc_juge_coder(const void* logits, uint32_t f64, size_t logits_octets, uint32_t n_positions, uint32_t n_vocab,
                   uint16_t* sortie, size_t sortie_octets, void* flux) {
    if (logits == nullptr || sortie == nullptr || n_vocab == 0 || n_positions == 0 || f64 > 1)
        return tb::erreur_usage("judge: logits, entries or sizes missing");
    const uint64_t nv = trc_juge_mots_par_entree(n_vocab);
    if (logits_octets < uint64_t(n_positions) * n_vocab * (f64 ? 8u : 4u) || sortie_octets < 2ull * nv * n_positions)
        return tb::erreur_usage("judge: views too short");
    if (reinterpret_cast<uintptr_t>(sortie) % 4 != 0 || reinterpret_cast<uintptr_t>(logits) % (f64 ? 8 : 4) != 0)
        return tb::erreur_usage("judge: misaligned views");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    tb::k_coder_entrees<<<n_positions, tb::JUGE_FILS, 0, static_cast<cudaStream_t>(flux)>>>(logits, f64, n_vocab, sortie);
    if (cudaError_t e = cudaGetLastError()) return tb::erreur_cuda(e);
    return TRC_OK;
}

int trc_juge_positions(const uint16_t* p, size_t p_octets, const void* q, size_t q_octets, uint32_t mode,
                       const uint32_t* suivants, size_t suivants_octets, uint32_t n_positions, uint32_t n_vocab,
                       trc_juge_position* sortie, size_t sortie_octets, void* flux) {
    if (p == nullptr || q == nullptr || suivants == nullptr || sortie == nullptr || n_vocab == 0 || n_positions == 0 ||
        mode > 2)
        return tb::erreur_usage("judge: entries, logits, tokens or sizes missing");
    const uint64_t nv = trc_juge_mots_par_entree(n_vocab);
    const uint64_t q_besoin = mode == 0 ? 2ull * nv * n_positions : uint64_t(n_positions) * n_vocab * (mode == 2 ? 8u : 4u);
    if (p_octets < 2ull * nv * n_positions || q_octets < q_besoin || suivants_octets < 4ull * n_positions ||
        sortie_octets < sizeof(trc_juge_position) * uint64_t(n_positions))
        return tb::erreur_usage("judge: views too short");
    if (reinterpret_cast<uintptr_t>(p) % 4 != 0 || reinterpret_cast<uintptr_t>(q) % (mode == 2 ? 8 : 4) != 0 ||
        reinterpret_cast<uintptr_t>(suivants) % 4 != 0 || reinterpret_cast<uintptr_t>(sortie) % 8 != 0)
        return tb::erreur_usage("judge: misaligned views");
    if (cudaError_t e = tb::aligner_device(flux)) return tb::erreur_cuda(e);
    tb::k_positions<<<n_positions, tb::JUGE_FILS, 0, static_cast<cudaStream_t>(flux)>>>(p, q, mode, suivants, n_vocab, sortie);
    if (cudaError_t e = cudaGetLastError()) return tb::erreur_cuda(e);
    return TRC_OK;
}

uint64_t trc_juge_mots_par_entree(uint32_t n_vocab) { return 2ull * ((uint64_t(n_vocab) + 1u) / 2u) + 4u; }

}  // extern "C"
