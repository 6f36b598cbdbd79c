// troncons_b200 — the MoE layer over a batch of positions "par flux" (the reference's prefill
// by stream, trc-modele/src/lib.rs:607-717 with trc-ordo/src/lib.rs:782-981): every routed
// expert is decoded ONCE for the batch, then applied to each position routed to it, with the
// same per-position arithmetic as the token-by-token layer, so the result is bit-identical to it
// (the reference's proposition 5: the layer-by-layer order equals the token-by-token order).
//
//   1. k_grouper        the batch's distinct experts (ascending), a slot each, the list of
//                       activations (position x routed slot) of each, the decode batch;
//   2. k_echelles/k_codes (decodeur.cu) each distinct expert into its SoA slot;
//   3. k_gemv_flux      gate and up of every activation on its expert's slot: one warp per row,
//                       the row's code words and scales loaded and converted once for up to 6
//                       activations, each activation's own fixed-order reduction (mxfp4.cuh);
//   4. k_swiglu         (passe.cu) per activation;
//   5. k_gemv_flux      down;
//   6. k_combiner_flux  per position: residual += ((w0 y0 + w1 y1) + ...), no contraction.
// Where the fused layer decodes a routed expert once per activation, this decodes it once per
// batch: the decode work no longer grows with the positions.
#include <cuda_bf16.h>

#include <algorithm>
#include <vector>

#include "commun.cuh"
#include "mxfp4.cuh"
#include "noyaux.h"

namespace tb {

constexpr uint32_t PF_WARPS = 8;
constexpr uint32_t PF_V = 6;       // activations multiplied per weight load (6 staged 2x of 2,880 fit twice per SM)
constexpr uint32_t PF_LOT = 16;    // macro-steps loaded before any is used
constexpr uint32_t NUL32 = 0xFFFFFFFFu;

EspaceParFlux plan_par_flux(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t experts, uint32_t na) {
    EspaceParFlux e{};
    Dims d;
    for (int j = 0; j < 3; ++j) {
        d.lignes[j] = lignes[j];
        d.colonnes[j] = colonnes[j];
    }
    e.taille_slot = 0;
    for (uint32_t j = 0; j < 3; ++j) e.taille_slot += disposition(d, j).pas;
    e.U = std::min(na, experts);
    uint64_t p = 0;
    e.slots = p;
    p = al256(p + e.taille_slot * e.U);
    e.descs = p;
    p = al256(p + sizeof(DescDecodage) * e.U);
    e.nu = p;
    p = al256(p + 4);
    e.ordre = p;
    p = al256(p + 4ull * e.U);
    e.slot_de = p;
    p = al256(p + 4ull * experts);
    e.debut = p;
    p = al256(p + 4ull * (e.U + 1));
    e.liste = p;
    p = al256(p + 4ull * na);
    e.ctl = p;
    p = al256(p + 16ull * e.U);
    e.g = p;
    p = al256(p + 4ull * na * lignes[0]);
    e.u = p;
    p = al256(p + 4ull * na * lignes[1]);
    e.h = p;
    p = al256(p + 4ull * na * lignes[0]);
    e.y = p;
    p = al256(p + 4ull * na * lignes[2]);
    e.total = p;
    return e;
}

struct ArgsParFlux {
    Couche c;
    uint8_t* espace;
    EspaceParFlux p;
    uint32_t j0;
    uint32_t seuil;          // > 0: the experts with at least this many activations are left to the tensor cores
    const uint32_t* petits;  // with seuil: the distinct experts below it (grid z indexes this list)
};

template <typename T>
__device__ __forceinline__ T* zone(const ArgsParFlux& a, uint64_t off) {
    return reinterpret_cast<T*>(a.espace + off);
}

// One block: counts per expert, the distinct experts in ascending order, their lists of
// activations (in any order), the decode descriptors (empty past the last).
// Expert e is held on this device: every expert, or those of the share [expert_debut, expert_fin)
// (the fused layer's rule for an expert-parallel share).
__device__ __forceinline__ bool tient(const Couche& c, uint32_t e) {
    return c.expert_fin == 0 || (e >= c.expert_debut && e < c.expert_fin);
}

__global__ void __launch_bounds__(1024) k_grouper(ArgsParFlux a) {
    __shared__ uint32_t part[1024];
    __shared__ uint32_t base_u, base_a;
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t na = c.jetons * c.k, E = c.experts, U = a.p.U, tid = threadIdx.x;
    uint32_t* cpt = zone<uint32_t>(a, a.p.slot_de);  // counts, then slot of each expert
    uint32_t* debut = zone<uint32_t>(a, a.p.debut);
    uint32_t* ordre = zone<uint32_t>(a, a.p.ordre);
    uint32_t* liste = zone<uint32_t>(a, a.p.liste);
    uint32_t* ctl = zone<uint32_t>(a, a.p.ctl);
    for (uint32_t e = tid; e < E; e += 1024u) cpt[e] = 0;
    for (uint32_t i = tid; i < 4u * U; i += 1024u) ctl[i] = 0;
    __syncthreads();
    for (uint32_t i = tid; i < na; i += 1024u) {
        const uint32_t e = c.indices[i];
        if (e < E && tient(c, e)) atomicAdd(&cpt[e], 1u);
    }
    __syncthreads();
    // exclusive scans over the experts: distinct index u and first activation of each
    if (tid == 0) base_u = base_a = 0;
    __syncthreads();
    for (uint32_t e0 = 0; e0 < E; e0 += 1024u) {
        const uint32_t e = e0 + tid;
        const uint32_t n = e < E ? cpt[e] : 0u;
        const uint32_t v = (n > 0u ? 1u : 0u) | (n << 16);  // distinct flag, count (<= 1,024)
        part[tid] = v;
        __syncthreads();
        for (uint32_t d = 1; d < 1024u; d <<= 1) {
            const uint32_t x = tid >= d ? part[tid - d] : 0u;
            __syncthreads();
            part[tid] += x;
            __syncthreads();
        }
        const uint32_t avant = part[tid] - v;
        if (e < E) {
            if (n > 0u) {
                const uint32_t u = base_u + (avant & 0xFFFFu);
                ordre[u] = e;
                debut[u] = base_a + (avant >> 16);
                cpt[e] = u;
            } else {
                cpt[e] = NUL32;
            }
        }
        __syncthreads();
        if (tid == 1023u) {
            base_u += part[1023] & 0xFFFFu;
            base_a += part[1023] >> 16;
        }
        __syncthreads();
    }
    const uint32_t nu = base_u;
    if (tid == 0) {
        *zone<uint32_t>(a, a.p.nu) = nu;
        debut[nu] = base_a;
    }
    __syncthreads();
    // each activation's place in its expert's list, by a counter per distinct expert (the order
    // within a list is free: every activation's arithmetic is its own, whatever its neighbours)
    uint32_t* rempli = part;  // reused (the scans are done): U <= experts <= 1,024, refused above by the ABI
    rempli[tid] = 0;
    __syncthreads();
    for (uint32_t i = tid; i < na; i += 1024u) {
        const uint32_t e = c.indices[i];
        if (e >= E || !tient(c, e)) continue;
        const uint32_t u = cpt[e];
        liste[debut[u] + atomicAdd(&rempli[u], 1u)] = i;
    }
    DescDecodage* descs = zone<DescDecodage>(a, a.p.descs);
    for (uint32_t u = tid; u < U; u += 1024u) {
        DescDecodage d{0, 0, 0, 0};
        if (u < nu) {
            const uint32_t e = ordre[u];
            const uint64_t pt = c.parties[e];
            if (pt != 0 && c.parties_octets[e] >= 64 && (pt & 15u) == 0) {
                d.partie = pt;
                d.emplacement = uint64_t(a.espace + a.p.slots + a.p.taille_slot * u);
                d.luts = uint64_t(c.luts);
                d.controle = uint64_t(ctl + 4u * u);
            } else {
                ctl[4u * u + CTL_FORMAT] = 1u;  // an absent or misplaced part
            }
        }
        descs[u] = d;
    }
}

// Raw parts: each distinct expert's matrices copied into its slot (the decode's place), matrix
// blockIdx.y of expert blockIdx.z; an absent part was counted by k_grouper.
__global__ void __launch_bounds__(256) k_copier_brut_flux(ArgsParFlux a, Dims dims) {
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t u = blockIdx.z;
    if (u >= *zone<uint32_t>(a, a.p.nu)) return;
    const uint32_t e = zone<uint32_t>(a, a.p.ordre)[u];
    const uint8_t* partie = reinterpret_cast<const uint8_t*>(c.parties[e]);
    if (partie == nullptr || c.parties_octets[e] < 64 || (reinterpret_cast<uintptr_t>(partie) & 15u) != 0) return;
    copier_brut_matrice(partie, c.parties_octets[e], a.espace + a.p.slots + a.p.taille_slot * u, dims, blockIdx.y,
                        zone<uint32_t>(a, a.p.ctl) + 4u * u);
}

// The slots of the batch's distinct experts: decoded from .trc parts, or copied from raw parts.
static cudaError_t remplir_slots(const ArgsParFlux& a, const Dims& dims, cudaStream_t flux) {
    if (a.c.brut) {
        const uint32_t rmax = std::max(dims.lignes[0], dims.lignes[2]);
        const uint32_t g = std::max(1u, std::min(64u, (rmax * 8u + 255u) / 256u));
        return lancer_pdl(k_copier_brut_flux, dim3(g, 3, a.p.U), dim3(256), 0, flux, a, dims);
    }
    return lancer_decodage(reinterpret_cast<const DescDecodage*>(a.espace + a.p.descs), a.p.U, nullptr, 0, nullptr,
                           a.c.luts, dims, nullptr, flux);
}

// The activations of one expert, one matrix: the block stages 2x of up to pf_vecteurs(C)
// activations in shared memory (the fused kernels' padded layout), then each warp walks its rows:
// the row's code words and scales loaded and converted once, applied to every staged activation
// in ligne_segments' order (per-lane fmaf chain, quad tree, scaled fmaf chain per segment and
// quad slot, 8-way tree, segment fold), so each activation gets the slot GEMV's bits + bias.
constexpr uint32_t PF_SMEM = 110u * 1024u;  // two blocks per SM
__host__ __device__ __forceinline__ uint32_t pf_vecteurs(uint32_t C) {
    const uint32_t v = PF_SMEM / x2_octets(C);
    return v < 1u ? 1u : (v > PF_V ? PF_V : v);
}

__global__ void __launch_bounds__(PF_WARPS * 32, 2) k_gemv_flux(ArgsParFlux a) {
    extern __shared__ __align__(16) uint8_t dyn[];
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t u = a.petits != nullptr ? a.petits[blockIdx.z] : blockIdx.z;
    if (u >= *zone<uint32_t>(a, a.p.nu)) return;
    const uint32_t j = a.j0 + blockIdx.y, voie = threadIdx.x & 31u, q = voie & 3u, g = voie >> 2;
    const uint32_t R = c.lignes[j], C = c.colonnes[j], B = C / 32u;
    Dims dims;
    for (int i = 0; i < 3; ++i) {
        dims.lignes[i] = c.lignes[i];
        dims.colonnes[i] = c.colonnes[i];
    }
    const Disposition disp = disposition(dims, j);
    const uint8_t* mat = a.espace + a.p.slots + a.p.taille_slot * u + disp.base;
    const uint8_t* ech = mat + disp.echelles;
    const float* biais = reinterpret_cast<const float*>(mat + disp.biais);
    const uint32_t d0 = zone<uint32_t>(a, a.p.debut)[u], n_act = zone<uint32_t>(a, a.p.debut)[u + 1] - d0;
    if (a.seuil != 0u && n_act >= a.seuil) return;  // this expert's activations go through the tensor cores
    const uint32_t* liste = zone<uint32_t>(a, a.p.liste) + d0;
    float* sortie = zone<float>(a, j == 0 ? a.p.g : j == 1 ? a.p.u : a.p.y);
    const uint32_t V = pf_vecteurs(C), oct = x2_octets(C);
    for (uint32_t v0 = 0; v0 < n_act; v0 += V) {
        const uint32_t nv = min(V, n_act - v0);
        __syncthreads();  // the previous group's rows are done with the staged vectors
        for (uint32_t v = 0; v < nv; ++v) {
            const uint32_t act = liste[v0 + v];
            float* x2s = reinterpret_cast<float*>(dyn + v * oct);
            if (j < 2)
                charger_x2(x2s, static_cast<const uint8_t*>(c.x) + uint64_t(act / c.k) * C * (c.x_bf16 ? 2u : 4u), c.x_bf16, C);
            else
                charger_x2(x2s, a.espace + a.p.h + uint64_t(act) * C * 4u, 0u, C);
        }
        __syncthreads();
        uint32_t act[PF_V];
#pragma unroll
        for (uint32_t v = 0; v < PF_V; ++v) act[v] = v < nv ? liste[v0 + v] : 0u;
        for (uint32_t r = blockIdx.x * PF_WARPS + (threadIdx.x >> 5); r < R; r += gridDim.x * PF_WARPS) {
            const uint64_t b0 = uint64_t(r) * B, b1 = b0 + B;
            const uint64_t ma = b0 >> 3, mb = (b1 - 1) >> 3;
            float acc[PF_V], total[PF_V];
#pragma unroll
            for (uint32_t v = 0; v < PF_V; ++v) acc[v] = total[v] = 0.0f;
            uint64_t seg = ma / SEGMENT_MACRO;
            uint32_t k = 0;
            for (uint64_t mc = ma; mc <= mb; mc += PF_LOT) {
                uint32_t mots[PF_LOT], es[PF_LOT];
#pragma unroll
                for (uint32_t i = 0; i < PF_LOT; ++i) {
                    const uint64_t beta = 8u * (mc + i) + g;
                    const bool v = mc + i <= mb && beta >= b0 && beta < b1;
                    mots[i] = v ? __ldg(reinterpret_cast<const uint32_t*>(mat + 16u * beta) + q) : 0u;
                    es[i] = v ? uint32_t(__ldg(ech + beta)) : 0u;
                }
#pragma unroll
                for (uint32_t i = 0; i < PF_LOT; ++i) {
                    const uint64_t m = mc + i;
                    if (m > mb) break;
                    if (m / SEGMENT_MACRO != seg) {  // the segment closes (ligne_segments' order)
#pragma unroll
                        for (uint32_t v = 0; v < PF_V; ++v) {
                            if (v >= nv) break;  // warp-uniform: the absent activations cost nothing
                            const float P = arbre8(acc[v]);
                            total[v] = k == 0 ? P : total[v] + P;
                            acc[v] = 0.0f;
                        }
                        ++k;
                        seg = m / SEGMENT_MACRO;
                    }
                    const uint64_t beta = 8u * m + g;
                    const bool valide = beta >= b0 && beta < b1;
                    const uint32_t bc = valide ? uint32_t(beta - b0) : 0u;
                    float lo[4], hi[4];
                    e2m1_mot(mots[i], lo, hi);
                    const float sc = echelle_e8m0(es[i]);
                    const uint32_t ia = x2_indice(8u * bc + q), ib = x2_indice(8u * bc + 4u + q);
#pragma unroll
                    for (uint32_t v = 0; v < PF_V; ++v) {
                        if (v >= nv) break;
                        {
                            const float4* x4 = reinterpret_cast<const float4*>(dyn + v * oct);
                            const float4 xa = x4[ia], xb = x4[ib];
                            float p = 0.0f;
                            p = fmaf(lo[0], xa.x, p);
                            p = fmaf(hi[0], xb.x, p);
                            p = fmaf(lo[1], xa.y, p);
                            p = fmaf(hi[1], xb.y, p);
                            p = fmaf(lo[2], xa.z, p);
                            p = fmaf(hi[2], xb.z, p);
                            p = fmaf(lo[3], xa.w, p);
                            p = fmaf(hi[3], xb.w, p);
                            const float s = somme_quad(p);
                            if (valide) acc[v] = fmaf(s, sc, acc[v]);
                        }
                    }
                }
            }
#pragma unroll
            for (uint32_t v = 0; v < PF_V; ++v) {
                if (v >= nv) break;
                const float P = arbre8(acc[v]);
                const float t = k == 0 ? P : total[v] + P;
                if (voie == 0) sortie[uint64_t(act[v]) * R + r] = t + biais[r];
            }
        }
    }
}

// Position b = blockIdx.y: residu[b] += ((w0 y0 + w1 y1) + w2 y2) + ... over its k routed slots
// in slot order, products and sums rounded separately (passe.cuh:611-622); an activation whose
// expert had no part is left out and counted. Block x = 0 also adds each distinct expert's
// decode counters to the controle of every activation routed to it. On an expert share, the
// activations of experts not held are left out (not counted), and with `partiel` residu[b] = the
// sum alone (0 when no activation of the position is held), as the fused layer's partial combine.
__global__ void __launch_bounds__(256) k_combiner_flux(ArgsParFlux a) {
    attendre_amont();
    liberer_aval();
    const Couche& c = a.c;
    const uint32_t b = blockIdx.y, d = c.lignes[2], i = blockIdx.x * 256u + threadIdx.x;
    const uint32_t* slot_de = zone<uint32_t>(a, a.p.slot_de);
    const uint32_t* ctl = zone<uint32_t>(a, a.p.ctl);
    if (blockIdx.x == 0 && threadIdx.x < 4u * c.k) {
        const uint32_t act = b * c.k + threadIdx.x / 4u, w = threadIdx.x % 4u;
        const uint32_t e = c.indices[act];
        const uint32_t u = e < c.experts ? slot_de[e] : NUL32;
        const bool ailleurs = e < c.experts && !tient(c, e);  // held by another device
        const uint32_t v = u != NUL32 ? ctl[4u * u + w] : (w == CTL_FORMAT && !ailleurs ? 1u : 0u);
        if (v != 0u) atomicAdd(&c.controle[4u * act + w], v);
    }
    if (i >= d) return;
    const float* y = zone<float>(a, a.p.y);
    float s = 0.0f;
    bool premier = true;
    for (uint32_t jj = 0; jj < c.k; ++jj) {
        const uint32_t act = b * c.k + jj;
        const uint32_t e = c.indices[act];
        if (e >= c.experts || slot_de[e] == NUL32 || ctl[4u * slot_de[e] + CTL_FORMAT] != 0u) continue;
        const float p = __fmul_rn(c.poids[act], y[uint64_t(act) * d + i]);
        s = premier ? p : __fadd_rn(s, p);
        premier = false;
    }
    float* res = c.residu + uint64_t(b) * d;
    res[i] = c.partiel ? s : __fadd_rn(res[i], s);
}

cudaError_t lancer_par_flux(const Couche& c, void* espace, cudaStream_t flux) {
    const uint32_t na = c.jetons * c.k;
    ArgsParFlux a{c, static_cast<uint8_t*>(espace), plan_par_flux(c.lignes, c.colonnes, c.experts, na), 0, 0, nullptr};
    cudaError_t e;
    if ((e = lancer_pdl(k_grouper, dim3(1), dim3(1024), 0, flux, a)) != cudaSuccess) return e;
    Dims dims;
    for (int j = 0; j < 3; ++j) {
        dims.lignes[j] = c.lignes[j];
        dims.colonnes[j] = c.colonnes[j];
    }
    if ((e = remplir_slots(a, dims, flux)) != cudaSuccess) return e;
    // About two blocks per SM over the (expert, matrix) planes: each warp walks many rows, and
    // each block stages its activations once.
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto grille = [&](uint32_t R, uint32_t plans) {
        const uint32_t vague = (uint32_t(sms) * 4u + plans - 1u) / plans;
        return std::max(1u, std::min((R + PF_WARPS - 1) / PF_WARPS, vague));
    };
    const uint32_t cmax = std::max(c.colonnes[0], c.colonnes[2]);
    const size_t smem = size_t(pf_vecteurs(cmax)) * x2_octets(cmax);
    if ((e = assurer_smem(reinterpret_cast<const void*>(k_gemv_flux), int(smem))) != cudaSuccess) return e;
    if ((e = lancer_pdl(k_gemv_flux, dim3(grille(c.lignes[0], 2u * a.p.U), 2, a.p.U), dim3(PF_WARPS * 32), smem, flux, a)) !=
        cudaSuccess)
        return e;
    if ((e = lancer_swiglu(reinterpret_cast<const float*>(a.espace + a.p.g), reinterpret_cast<const float*>(a.espace + a.p.u),
                           reinterpret_cast<float*>(a.espace + a.p.h), na * c.lignes[0], flux)) != cudaSuccess)
        return e;
    a.j0 = 2;
    if ((e = lancer_pdl(k_gemv_flux, dim3(grille(c.lignes[2], a.p.U), 1, a.p.U), dim3(PF_WARPS * 32), smem, flux, a)) !=
        cudaSuccess)
        return e;
    return lancer_pdl(k_combiner_flux, dim3((c.lignes[2] + 255) / 256, c.jetons), dim3(256), 0, flux, a);
}

// ------------------------------------------------------------------ with the tensor cores

// Descriptors of one GEMM per (big expert, group of up to 256 of its activations) and matrix.
constexpr uint32_t PF_MMA_N = 256;

// The GEMMs' descriptors (at most this many per matrix group) for na activations and a threshold.
static uint32_t pf_mma_max(uint32_t na, uint32_t seuil) { return na / seuil + na / PF_MMA_N + 1u; }

uint64_t par_flux_mma_octets(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t experts, uint32_t na,
                             uint32_t seuil) {
    const EspaceParFlux p = plan_par_flux(lignes, colonnes, experts, na);
    const uint32_t cmax = std::max(std::max(colonnes[0], colonnes[1]), colonnes[2]);
    return p.total + al256(4ull * p.U) + gemm_mxfp4_lot_espace(cmax, PF_MMA_N, 2u * pf_mma_max(na, seuil));
}

// The layer par flux with the experts that have at least `seuil` activations (>= 1) multiplied
// on the tensor cores: gate and up of their activations as GEMMs over the expert's decoded slot
// (x rows gathered through the expert's activation list: token = activation / k), SwiGLU for
// every activation, down as GEMMs (h rows of the activations), the outputs scattered to the
// activations' rows; the other experts through k_gemv_flux as in lancer_par_flux. The routing is
// read back on the host (one wait on the stream) to size the GEMMs. Not bit-identical to the
// GEMV (the GEMM quantizes x and h to MXFP8); `erreur` (device u32) is set when a bounded wait of
// the GEMM kernel gave up.
cudaError_t lancer_par_flux_mma(const Couche& c, void* espace, uint32_t seuil, uint32_t* erreur, cudaStream_t flux) {
    const uint32_t na = c.jetons * c.k;
    ArgsParFlux a{c, static_cast<uint8_t*>(espace), plan_par_flux(c.lignes, c.colonnes, c.experts, na), 0, seuil, nullptr};
    cudaError_t e;
    if ((e = lancer_pdl(k_grouper, dim3(1), dim3(1024), 0, flux, a)) != cudaSuccess) return e;
    Dims dims;
    for (int j = 0; j < 3; ++j) {
        dims.lignes[j] = c.lignes[j];
        dims.colonnes[j] = c.colonnes[j];
    }
    if ((e = remplir_slots(a, dims, flux)) != cudaSuccess) return e;
    // the groups, on the host
    const uint32_t U = a.p.U;
    uint32_t nu = 0;
    std::vector<uint32_t> debut(U + 1u);
    if ((e = cudaMemcpyAsync(&nu, a.espace + a.p.nu, 4, cudaMemcpyDeviceToHost, flux)) != cudaSuccess ||
        (e = cudaMemcpyAsync(debut.data(), a.espace + a.p.debut, 4ull * (U + 1u), cudaMemcpyDeviceToHost, flux)) !=
            cudaSuccess ||
        (e = cudaStreamSynchronize(flux)) != cudaSuccess)
        return e;
    nu = std::min(nu, U);
    std::vector<DescGemm> dg[2];
    std::vector<RenvoiGemm> rg[2];
    std::vector<uint32_t> petits;  // the experts below the threshold: the GEMV's grid covers them alone
    uint32_t n_max = 1;
    for (uint32_t u = 0; u < nu; ++u) {
        const uint32_t d0 = debut[u], n = debut[u + 1] - d0;
        if (n < seuil) {
            petits.push_back(u);
            continue;
        }
        const uint8_t* slot = a.espace + a.p.slots + a.p.taille_slot * u;
        for (uint32_t g0 = 0; g0 < n; g0 += PF_MMA_N) {
            const uint32_t ng = std::min(PF_MMA_N, n - g0);
            n_max = std::max(n_max, ng);
            const uint32_t* liste = reinterpret_cast<const uint32_t*>(a.espace + a.p.liste) + d0 + g0;
            for (uint32_t j = 0; j < 3; ++j) {
                const Disposition dp = disposition(dims, j);
                const uint8_t* mat = slot + dp.base;
                const uint64_t x = j < 2 ? reinterpret_cast<uint64_t>(c.x) : reinterpret_cast<uint64_t>(a.espace + a.p.h);
                const uint64_t y = reinterpret_cast<uint64_t>(a.espace + (j == 0 ? a.p.g : j == 1 ? a.p.u : a.p.y));
                DescGemm d{reinterpret_cast<uint64_t>(mat), reinterpret_cast<uint64_t>(mat + dp.echelles),
                           reinterpret_cast<uint64_t>(mat + dp.biais), x, y, c.lignes[j], c.colonnes[j], ng,
                           j < 2 ? c.x_bf16 : 0u};
                dg[j < 2 ? 0 : 1].push_back(d);
                rg[j < 2 ? 0 : 1].push_back(RenvoiGemm{liste, liste, j < 2 ? c.k : 1u});
            }
        }
    }
    uint32_t* petits_d = reinterpret_cast<uint32_t*>(a.espace + a.p.total);
    uint8_t* eg = a.espace + a.p.total + al256(4ull * U);  // the GEMMs' workspace (quantized activations)
    if (!petits.empty() && (e = cudaMemcpyAsync(petits_d, petits.data(), 4ull * petits.size(), cudaMemcpyHostToDevice,
                                                flux)) != cudaSuccess)
        return e;
    a.petits = petits_d;
    const uint32_t np = uint32_t(petits.size());
    const uint32_t rmax = std::max(c.lignes[0], c.lignes[2]), cmax = std::max(c.colonnes[0], c.colonnes[2]);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    auto grille = [&](uint32_t R, uint32_t plans) {
        const uint32_t vague = (uint32_t(sms) * 4u + plans - 1u) / plans;
        return std::max(1u, std::min((R + PF_WARPS - 1) / PF_WARPS, vague));
    };
    const size_t smem = size_t(pf_vecteurs(cmax)) * x2_octets(cmax);
    if ((e = assurer_smem(reinterpret_cast<const void*>(k_gemv_flux), int(smem))) != cudaSuccess) return e;
    if (np != 0 &&
        (e = lancer_pdl(k_gemv_flux, dim3(grille(c.lignes[0], 2u * np), 2, np), dim3(PF_WARPS * 32), smem, flux, a)) !=
            cudaSuccess)
        return e;
    if (!dg[0].empty() && (e = lancer_gemm_mxfp4_lot(dg[0].data(), uint32_t(dg[0].size()), rmax, cmax, n_max, eg, erreur,
                                                      flux, rg[0].data())) != cudaSuccess)
        return e;
    if ((e = lancer_swiglu(reinterpret_cast<const float*>(a.espace + a.p.g), reinterpret_cast<const float*>(a.espace + a.p.u),
                           reinterpret_cast<float*>(a.espace + a.p.h), na * c.lignes[0], flux)) != cudaSuccess)
        return e;
    a.j0 = 2;
    if (np != 0 &&
        (e = lancer_pdl(k_gemv_flux, dim3(grille(c.lignes[2], np), 1, np), dim3(PF_WARPS * 32), smem, flux, a)) != cudaSuccess)
        return e;
    if (!dg[1].empty() && (e = lancer_gemm_mxfp4_lot(dg[1].data(), uint32_t(dg[1].size()), rmax, cmax, n_max, eg, erreur,
                                                      flux, rg[1].data())) != cudaSuccess)
        return e;
    return lancer_pdl(k_combiner_flux, dim3((c.lignes[2] + 255) / 256, c.jetons), dim3(256), 0, flux, a);
}

}  // namespace tb
