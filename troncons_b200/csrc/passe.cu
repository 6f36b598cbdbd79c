// troncons_b200 — the single-vector kernels of the MoE layer, with the reference's semantics
// (trc-noyaux/noyaux/passe.cuh): router top-k with its f64 softmax and host-mapped mailbox,
// clamped SwiGLU in f64, and the in-order weighted combine without FMA contraction.
#include "commun.cuh"
#include "noyaux.h"

namespace tb {

// Top-k by rank. One block per token, one thread per expert (E <= 256, rounded up to whole
// warps). Expert e's rank is the number of experts that beat it: a larger value, or the same
// value and a smaller index; a NaN beats nothing and is never ranked, so the order over the
// other logits (-inf included) is total and the experts of rank 0 .. k-1 are the top-k in order
// (passe.cuh:455-514, ops.rs:123-131: value descending, index ascending, NaN never chosen; a slot
// with no candidate left holds index 0xFFFFFFFF and value -inf). Each thread counts its rank over
// the logits staged in shared memory, every thread reading the same word at once (a broadcast).
// Weights: m = the slot-0 value, e_r = exp(v_r - m) in f64, z = e_0 + e_1 + ... in slot order,
// w_r = float(e_r / z). The slots' owners write the outputs and the host-mapped mailbox
// (indices at [1 + r], weight bits at [1 + k + r]); each fences at system scope, and after a
// barrier one thread raises the mailbox's sequence word.
__global__ void __launch_bounds__(256) k_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices,
                                              float* poids, uint32_t* boite, uint32_t sequence) {
    __shared__ float lg[256];
    __shared__ float val_rang[8];
    __shared__ uint32_t idx_rang[8];
    attendre_amont();
    liberer_aval();
    logits += uint64_t(blockIdx.x) * E;
    indices += uint64_t(blockIdx.x) * k;
    poids += uint64_t(blockIdx.x) * k;
    const uint32_t e = threadIdx.x;
    const float v = e < E ? logits[e] : __int_as_float(0x7FC00000);  // padding: a NaN, never ranked
    lg[e] = v;
    if (e < 8) {
        val_rang[e] = -INFINITY;
        idx_rang[e] = 0xFFFFFFFFu;
    }
    __syncthreads();
    if (v == v) {
        uint32_t rang = 0;
        for (uint32_t j = 0; j < E; ++j) {
            const float w = lg[j];
            rang += (w > v || (w == v && j < e)) ? 1u : 0u;
        }
        if (rang < k) {
            val_rang[rang] = v;
            idx_rang[rang] = e;
        }
    }
    __syncthreads();
    if (e < k) {
        const double m = val_rang[0];
        double z = 0.0, mien = 0.0;
        for (uint32_t r = 0; r < k; ++r) {
            const double x = exp(double(val_rang[r]) - m);
            z += x;
            if (r == e) mien = x;
        }
        const float w = float(mien / z);
        indices[e] = idx_rang[e];
        poids[e] = w;
        if (boite != nullptr) {
            volatile uint32_t* b = boite;
            b[1 + e] = idx_rang[e];
            b[1 + k + e] = __float_as_uint(w);
            __threadfence_system();
        }
    }
    __syncthreads();
    if (e == 0 && boite != nullptr) reinterpret_cast<volatile uint32_t*>(boite)[0] = sequence;
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
    const uint32_t fils = (E + 31u) / 32u * 32u;
    return lancer_pdl(k_topk, dim3(jetons), dim3(fils), 0, flux, logits, E, k, indices, poids,
                      jetons == 1 ? boite : nullptr, sequence);
}

cudaError_t lancer_swiglu(const float* g, const float* u, float* y, uint32_t n, cudaStream_t flux) {
    return lancer_pdl(k_swiglu, dim3((n + 255) / 256), dim3(256), 0, flux, g, u, y, n);
}

cudaError_t lancer_combiner(float* residu, const float* sorties, uint32_t pas, const float* poids, uint32_t n, uint32_t d,
                            cudaStream_t flux) {
    return lancer_pdl(k_combiner, dim3((d + 255) / 256), dim3(256), 0, flux, residu, sorties, pas, poids, n, d);
}

}  // namespace tb
