// troncons_b200 — the single-vector kernels of the MoE layer, with the reference's semantics
// (trc-noyaux/noyaux/passe.cuh): router top-k with its f64 softmax and host-mapped mailbox,
// clamped SwiGLU in f64, and the in-order weighted combine without FMA contraction.
#include "commun.cuh"
#include "noyaux.h"

namespace tb {

// Better of two (value, index): larger value, then smaller index; a NaN is never better.
__device__ __forceinline__ bool meilleur(float va, uint32_t ia, float vb, uint32_t ib) {
    return va > vb || (va == vb && ia < ib);
}

// One warp. E <= 256, k <= 8: lane l holds logits l, l+32, ..., each round takes the warp's best
// among those not yet taken. Weights: m = the first chosen value, e_r = exp(v_r - m) in f64,
// z = sum in order, w_r = float(e_r / z) (passe.cuh:455-514; ops.rs:123-131).
__global__ void __launch_bounds__(32) k_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices, float* poids,
                                             uint32_t* boite, uint32_t sequence) {
    attendre_amont();
    liberer_aval();
    // Token blockIdx.x of a batch (the mailbox is for a single token).
    logits += uint64_t(blockIdx.x) * E;
    indices += uint64_t(blockIdx.x) * k;
    poids += uint64_t(blockIdx.x) * k;
    const uint32_t voie = threadIdx.x;
    float v[8];
    uint32_t pris = 0;
#pragma unroll
    for (uint32_t i = 0; i < 8; ++i) {
        const uint32_t e = voie + 32u * i;
        v[i] = e < E ? logits[e] : -INFINITY;
        pris |= (e >= E ? 1u : 0u) << i;
    }
    float cv[8];
    uint32_t ci[8];
    for (uint32_t r = 0; r < k; ++r) {
        float bv = -INFINITY;
        uint32_t bi = 0xFFFFFFFFu;
#pragma unroll
        for (uint32_t i = 0; i < 8; ++i)
            if (!((pris >> i) & 1u) && meilleur(v[i], voie + 32u * i, bv, bi)) {
                bv = v[i];
                bi = voie + 32u * i;
            }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, d);
            const uint32_t oi = __shfl_xor_sync(0xFFFFFFFFu, bi, d);
            if (meilleur(ov, oi, bv, bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi != 0xFFFFFFFFu && (bi & 31u) == voie) pris |= 1u << (bi >> 5);
        cv[r] = bv;
        ci[r] = bi;
    }
    if (voie != 0) return;
    double ex[8];
    const double m = cv[0];
    double z = 0.0;
    for (uint32_t r = 0; r < k; ++r) {
        ex[r] = exp(double(cv[r]) - m);
        z += ex[r];
    }
    for (uint32_t r = 0; r < k; ++r) {
        const float w = float(ex[r] / z);
        indices[r] = ci[r];
        poids[r] = w;
        if (boite != nullptr) {
            reinterpret_cast<volatile uint32_t*>(boite)[1 + r] = ci[r];
            reinterpret_cast<volatile uint32_t*>(boite)[1 + k + r] = __float_as_uint(w);
        }
    }
    if (boite != nullptr) {
        __threadfence_system();
        reinterpret_cast<volatile uint32_t*>(boite)[0] = sequence;
    }
}

// Clamped SwiGLU of gpt-oss, element-wise in f64 (passe.cuh:598-605).
__device__ __forceinline__ float swiglu_oai(float g, float u) {
    const double gv = fmin(double(g), 7.0);
    const double uv = fmin(fmax(double(u), -7.0), 7.0);
    return float(gv / (1.0 + exp(-1.702 * gv)) * (uv + 1.0));
}

__global__ void __launch_bounds__(256) k_swiglu(const float* __restrict__ g, const float* __restrict__ u,
                                                float* __restrict__ y, uint32_t n) {
    attendre_amont();
    liberer_aval();
    const uint32_t i = blockIdx.x * 256u + threadIdx.x;
    if (i < n) y[i] = swiglu_oai(g[i], u[i]);
}

// residu[i] += ((w0 s0 + w1 s1) + w2 s2) + ..., no contraction (passe.cuh:611-622).
__global__ void __launch_bounds__(256) k_combiner(float* __restrict__ residu, const float* __restrict__ sorties, uint32_t pas,
                                                  const float* __restrict__ poids, uint32_t n, uint32_t d) {
    attendre_amont();
    liberer_aval();
    const uint32_t i = blockIdx.x * 256u + threadIdx.x;
    if (i >= d || n == 0) return;
    float s = poids != nullptr ? __fmul_rn(poids[0], sorties[i]) : sorties[i];
    for (uint32_t j = 1; j < n; ++j) {
        const float sj = sorties[uint64_t(j) * pas + i];
        s = __fadd_rn(s, poids != nullptr ? __fmul_rn(poids[j], sj) : sj);
    }
    residu[i] = __fadd_rn(residu[i], s);
}

cudaError_t lancer_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices, float* poids, uint32_t* boite,
                        uint32_t sequence, cudaStream_t flux, uint32_t jetons) {
    return lancer_pdl(k_topk, dim3(jetons), dim3(32), 0, flux, logits, E, k, indices, poids, jetons == 1 ? boite : nullptr,
                      sequence);
}

cudaError_t lancer_swiglu(const float* g, const float* u, float* y, uint32_t n, cudaStream_t flux) {
    return lancer_pdl(k_swiglu, dim3((n + 255) / 256), dim3(256), 0, flux, g, u, y, n);
}

cudaError_t lancer_combiner(float* residu, const float* sorties, uint32_t pas, const float* poids, uint32_t n, uint32_t d,
                            cudaStream_t flux) {
    return lancer_pdl(k_combiner, dim3((d + 255) / 256), dim3(256), 0, flux, residu, sorties, pas, poids, n, d);
}

}  // namespace tb
