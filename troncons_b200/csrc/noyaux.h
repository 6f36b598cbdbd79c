// troncons_b200 — internal declarations shared by the host entry points (abi.cpp) and the
// kernel launchers (*.cu). Not a public header: the boundary is include/troncons_b200.h.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

namespace tb {

struct Dims;

// Device twins of the C-ABI batch descriptors (32 bytes each; abi.rs:16-53 of the reference).
struct DescDecodage {
    uint64_t partie, emplacement, luts, controle;
};
struct DescGemv {
    uint64_t matrice, x, y;
    uint32_t lignes, colonnes;
};

// One expert of a GPU encode batch (mirror of trc_desc_codage, 72 bytes).
struct DescCodage {
    uint64_t blocs[3], biais[3], sortie, capacite;
    uint32_t expert, reserve;
};

// The combine's exchange across GPUs (mirror of trc_echange_pairs; monde < 2: none).
struct Echange {
    uint64_t tampons[8];
    uint32_t rang, monde;
};

// One rank's exchange buffer: slots [monde][jetons][R] f32 (rank q's share in slot q), flags
// [monde][blocs] u32 (rank q's flag for combine block b), the expected sequence per block.
struct DispositionEchange {
    uint64_t slots, flags, attendus, total;
    uint32_t blocs;
};
__host__ __device__ __forceinline__ DispositionEchange disposition_echange(uint32_t R, uint32_t jetons, uint32_t monde) {
    DispositionEchange d;
    d.blocs = ((R + 255u) / 256u) * jetons;
    d.slots = 0;
    d.flags = (uint64_t(monde) * jetons * R * 4u + 255u) & ~uint64_t(255);
    d.attendus = (d.flags + uint64_t(monde) * d.blocs * 4u + 255u) & ~uint64_t(255);
    d.total = (d.attendus + uint64_t(d.blocs) * 4u + 255u) & ~uint64_t(255);
    return d;
}

// The fused layer, as the kernels see it (mirror of trc_moe_couche).
struct Couche {
    const uint64_t* parties;
    const uint64_t* parties_octets;
    uint32_t experts, k;
    const uint32_t* luts;
    uint32_t lignes[3], colonnes[3];
    const uint32_t* indices;
    const float* poids;
    const void* x;
    uint32_t x_bf16, brut;
    float* residu;
    uint32_t* controle;
    uint32_t n_delta, n_codes;
    uint32_t jetons;                    // tokens (>= 1): activation i = token i / k, slot i % k
    uint32_t expert_debut, expert_fin;  // experts held here ([debut, fin); fin = 0: all)
    uint32_t partiel;                   // 1: the combine writes this call's sum, not residu +=
    Echange ech;                        // the combine's sum across GPUs over peer memory
    const uint8_t* deltas;              // every expert's delta bytes decoded ahead, or null
};

// Activations of a call: tokens x routed experts per token.
__host__ __device__ __forceinline__ uint32_t activations(const Couche& c) { return c.k * c.jetons; }

// Workspace of the fused layer (offsets in bytes from its 256-aligned base).
struct Espace {
    uint64_t ek[3];      // delta byte per block, per matrix, times the activations
    uint64_t parts[3];   // f32 per-segment row partials [activation][R][K] per matrix
    uint64_t h;          // f32 [activation][lignes[0]] SwiGLU output
    uint64_t total;      // the sequential schedule's workspace
    uint64_t cd;         // the overlapped schedule's decoded down codes (16 bytes per block and
    uint64_t total_recouvrant;  // activation), and its workspace
    uint64_t cdh[2];     // the decoded gate and up codes when all three are decoded first, and
    uint64_t total_tout;        // that schedule's workspace
    uint32_t K[3];       // partial slots per row
};
// Workspace of the layer "par flux" (par_flux.cu): decoded slots of the batch's distinct
// experts, the decode batch, the grouping, per-activation gate / up / h / down outputs.
struct EspaceParFlux {
    uint64_t slots, descs, nu, ordre, slot_de, debut, liste, ctl, g, u, h, y, total, taille_slot;
    uint32_t U;  // slots: min(activations, experts)
};
EspaceParFlux plan_par_flux(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t experts, uint32_t na);
cudaError_t lancer_par_flux(const Couche& c, void* espace, cudaStream_t flux);
// The same with the experts that have at least `seuil` activations multiplied on the tensor
// cores (mma_mxfp4.cu); waits for the routing on the host.
uint64_t par_flux_mma_octets(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t experts, uint32_t na,
                             uint32_t seuil);
cudaError_t lancer_par_flux_mma(const Couche& c, void* espace, uint32_t seuil, uint32_t* erreur, cudaStream_t flux);

// Activations up to which the down projection's decode may overlap gate/up (its codes then go
// through the workspace: 4.15 MB per activation for gpt-oss; measured faster than the
// sequential schedule at 4, 8, 16 and 32 activations on one GPU).
constexpr uint32_t RECOUVRE_MAX = 32;
Espace plan_espace(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t k);

cudaError_t lancer_decodage(const DescDecodage* descs, uint32_t n, const void* partie, uint64_t taille, void* emplacement,
                            const uint32_t* luts, const Dims& dims, uint32_t* controle, cudaStream_t flux);
cudaError_t lancer_copier_brut(const void* partie, uint64_t taille, void* emplacement, const Dims& dims, uint32_t* controle,
                               cudaStream_t flux);
cudaError_t lancer_gemv(const void* matrice, const float* x, float* y, uint32_t R, uint32_t C, cudaStream_t flux);
cudaError_t lancer_gemv_lot(const DescGemv* descs, uint32_t n, uint32_t lignes_max, cudaStream_t flux);
cudaError_t lancer_gemv_f32(const float* w, const void* x, uint32_t x_bf16, const float* biais, float* y, uint32_t R,
                            uint32_t C, cudaStream_t flux, uint32_t jetons = 1);
cudaError_t lancer_topk(const float* logits, uint32_t E, uint32_t k, uint32_t* indices, float* poids, uint32_t* boite,
                        uint32_t sequence, cudaStream_t flux, uint32_t jetons = 1);
cudaError_t lancer_swiglu(const float* g, const float* u, float* y, uint32_t n, cudaStream_t flux);
cudaError_t lancer_combiner(float* residu, const float* sorties, uint32_t pas, const float* poids, uint32_t n, uint32_t d,
                            cudaStream_t flux);
cudaError_t lancer_moe(const Couche& c, void* espace, uint64_t espace_octets, cudaStream_t flux, cudaEvent_t const* ev = nullptr);
uint64_t deltas_octets(const uint32_t lignes[3], const uint32_t colonnes[3], uint32_t experts);
// The MXFP4 expert GEMM on the tensor cores (mma_mxfp4.cu); DescGemm mirrors trc_desc_gemm.
struct DescGemm {
    uint64_t codes, echelles, biais, x, y;
    uint32_t lignes, colonnes, n, x_bf16;
};
uint64_t gemm_mxfp4_espace(uint32_t C, uint32_t N);
bool gemm_mxfp4_possible(uint32_t C, uint32_t N);  // the staged tiles and scales fit shared memory
uint64_t gemm_mxfp4_lot_espace(uint32_t colonnes_max, uint32_t n_max, uint32_t nb);
// Token n of a GEMM reads x row ix[n] / div_x and writes y row iy[n] (each list null: row n).
struct RenvoiGemm {
    const uint32_t* ix;
    const uint32_t* iy;
    uint32_t div_x;
};
cudaError_t lancer_gemm_mxfp4_lot(const DescGemm* descs, uint32_t nb, uint32_t lignes_max, uint32_t colonnes_max,
                                  uint32_t n_max, uint8_t* espace, uint32_t* erreur, cudaStream_t flux,
                                  const RenvoiGemm* renvois = nullptr);
cudaError_t lancer_gemm_mxfp4(const uint8_t* codes, const uint8_t* ech, const float* biais, const void* x, uint32_t x_bf16,
                              float* y, uint32_t R, uint32_t C, uint32_t N, uint8_t* espace, uint32_t* erreur,
                              cudaStream_t flux);
cudaError_t lancer_predecoder_deltas(const Couche& c, uint8_t* deltas, cudaStream_t flux);

// Attention side (mirrors of trc_params_rope, 48 bytes, and trc_params_attention, 32 bytes).
struct ParamsRope {
    double base, facteur, ctx_origine, beta_rapide, beta_lent;
    uint32_t dim_tete, variante;
};
struct ParamsAttention {
    uint32_t tetes, tetes_kv, dim_tete, debut, fin, anneau;
    float echelle;
    uint32_t reserve;
};
constexpr uint32_t Q8_LOT_MAX = 8;  // tokens per launch of the batched Q8_0 GEMV
cudaError_t lancer_gemv_q8_0_lot(const void* w, const float* x, const float* biais, float* y, uint32_t R, uint32_t C,
                                 uint32_t n, cudaStream_t flux);
cudaError_t lancer_gemv_q8_0(const void* w, const float* x, const float* biais, float* y, uint32_t R, uint32_t C,
                             cudaStream_t flux);
cudaError_t lancer_rmsnorm(const float* x, const float* w, float* y, uint32_t n, uint32_t lignes, float eps,
                           cudaStream_t flux);
// One launch of up to three Q8_0 GEMVs on the same input (the rows of matrix 0, then 1, then 2),
// each row in lancer_gemv_q8_0's order: with `norme`, the input is RMSNorm(x) (lancer_rmsnorm's
// order, recomputed by every block; block 0 also writes it to `h` when given); with `residu`
// (one matrix), residu[r] += y[r] after y[r] is written (lancer_combiner's single-term add).
// `jetons` tokens (x [jetons][C], y[m] [jetons][lignes[m]]; neither norme nor residu) in
// launches of up to Q8_LOT_MAX, as lancer_gemv_q8_0_lot.
struct DescQ8Couche {
    const void* w[3];
    const float* biais[3];
    float* y[3];
    uint32_t lignes[3];
    uint32_t n;  // matrices
    uint32_t C;
    const float* x;
    const float* norme;
    float eps;
    float* h;
    float* residu;
};
cudaError_t lancer_q8_0_couche(const DescQ8Couche& d, cudaStream_t flux, uint32_t jetons = 1);
cudaError_t lancer_rope_yarn(float* q, float* k, uint32_t tetes_q, uint32_t tetes_k, uint32_t position, const ParamsRope& p,
                             cudaStream_t flux);
// lancer_rope_yarn then lancer_ecrire_kv (dkv = tetes_k x dim_tete) in one launch, the same bits.
cudaError_t lancer_rope_kv(float* q, float* k, const float* v, uint16_t* ck, uint16_t* cv, uint32_t tetes_q,
                           uint32_t tetes_k, uint32_t position, uint32_t case_kv, const ParamsRope& p, cudaStream_t flux);
cudaError_t lancer_ecrire_kv(const float* k, const float* v, uint16_t* ck, uint16_t* cv, uint32_t dkv, uint32_t case_kv,
                             cudaStream_t flux);
cudaError_t lancer_attention(const float* q, const uint16_t* ck, const uint16_t* cv, const float* puits, float* sortie,
                             const ParamsAttention& p, cudaStream_t flux);

// GPU encoder of one geometry-1 stream (codeur_gpu.cu).
uint64_t coder_flux_espace(uint32_t P, uint32_t N);
cudaError_t lancer_coder_flux(const uint8_t* src, uint32_t P, uint32_t N, const uint8_t* kappa, uint32_t n_kappa,
                              const uint16_t* freqs, uint32_t n_tables, uint8_t* sortie, uint64_t capacite, uint64_t* octets,
                              uint8_t* espace, cudaStream_t flux);
// Level-0 parts of n experts on the GPU (codeur_gpu.cu), and the layer's symbol counts.
uint64_t coder_parties_espace(const Dims& dims, uint32_t n, uint32_t n_delta, uint32_t n_codes);
cudaError_t lancer_coder_parties(const DescCodage* descs, uint32_t n, const Dims& dims, const uint16_t* freqs,
                                 bool canonique, uint16_t couche, uint32_t n_delta, uint32_t n_codes, uint64_t* octets,
                                 uint8_t* espace, int sms, cudaStream_t flux);
cudaError_t lancer_comptes(const DescCodage* descs, uint32_t n, const Dims& dims, bool canonique, uint64_t* comptes,
                           int sms, cudaStream_t flux);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device).
cudaError_t assurer_smem(const void* noyau, int octets);

// For entry points outside abi.cu: set this thread's error message (usage error, or the CUDA
// error's text; cudaSuccess clears it) and return the status; make the caller's stream's device
// current in this library's runtime.
int erreur_usage(const char* message);
int erreur_cuda(cudaError_t e);
cudaError_t aligner_device(void* flux);

// Launch with programmatic dependent launch allowed: the kernel may start while the previous
// kernel on the stream finishes, and must call attendre_amont() before it reads what that kernel
// (or anything before it) wrote. Kernels call liberer_aval() once their own wait is done.
template <typename... P, typename... A>
cudaError_t lancer_pdl(void (*noyau)(P...), dim3 grille, dim3 bloc, size_t smem, cudaStream_t flux, A&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grille;
    cfg.blockDim = bloc;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = flux;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, noyau, static_cast<A&&>(args)...);
}

}  // namespace tb
